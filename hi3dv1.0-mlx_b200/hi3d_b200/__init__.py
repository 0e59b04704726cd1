"""hi3d_b200: the Hi3D v1.0 sparse-voxel refinement-transformer block on B200.

Operator surface mirrors ``hi3d_mac.mlx_backend`` of devin-lai/Hi3Dv1.0-mlx:

* :mod:`hi3d_b200.kernels`    ``layer_norm_modulate``, ``qkv_rope_rms``, ``qkv_rope_rms_simd``
* :mod:`hi3d_b200.attention`  ``flash_attention`` (+ varlen)
* :mod:`hi3d_b200.transformer` the block (``block_forward``), ``rope_tables``, the 24-block stack
* :mod:`hi3d_b200.torch_backend` ``flash_attn`` drop-in module for the upstream ``sparc3d`` code

All compute runs in ``libhi3d_b200.so`` (hand-written sm_100a CUDA behind a C ABI).
"""

__version__ = "0.1.0"
