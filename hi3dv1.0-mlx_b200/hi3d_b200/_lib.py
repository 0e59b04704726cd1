"""ctypes binding of ``libhi3d_b200.so`` (the C ABI in ``include/hi3d_b200.h``).

The library is loaded on first use.  There is no fallback: if it is missing or
fails to load, every operator raises ``ImportError`` naming the library, so a
GPU run can never silently take another code path.
"""

from __future__ import annotations

import ctypes
import os
import threading
from pathlib import Path

import torch

# HI3D_B200_LIB selects another build of the same library (e.g. a tuning variant).
LIB_PATH = Path(os.environ.get("HI3D_B200_LIB", Path(__file__).resolve().parent / "_lib" / "libhi3d_b200.so"))

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_UNSUPPORTED = 2
ERR_CUDA = 3
ERR_DEVICE_TIMEOUT = 4
ERR_CAPACITY = 5
ERR_NCCL = 6

F16, BF16, F32, I32 = 0, 1, 2, 3
EPI_STORE, EPI_GELU, EPI_RESIDUAL = 0, 1, 2

_c_void_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_f32 = ctypes.c_float


class AttnArgs(ctypes.Structure):
    """Mirror of ``hi3d_attn_args``."""

    _fields_ = [
        ("q", _c_void_p), ("k", _c_void_p), ("v", _c_void_p), ("out", _c_void_p),
        ("q_row", _i64), ("q_head", _i64), ("q_batch", _i64),
        ("k_row", _i64), ("k_head", _i64), ("k_batch", _i64),
        ("v_row", _i64), ("v_head", _i64), ("v_batch", _i64),
        ("o_row", _i64), ("o_head", _i64), ("o_batch", _i64),
        ("cu_seqlens_q", _c_void_p), ("cu_seqlens_k", _c_void_p),
        ("nq", _i64), ("nk", _i64), ("max_seqlen_q", _i64),
        ("num_seqs", _i32), ("heads", _i32), ("head_dim", _i32), ("dtype", _i32),
        ("scale", _f32),
    ]


# name -> (restype, argtypes); every entry of include/hi3d_b200.h
SIGNATURES: dict[str, tuple] = {
    "hi3d_version": (_i32, []),
    "hi3d_last_error_string": (ctypes.c_char_p, []),
    "hi3d_device_status": (_i32, [ctypes.POINTER(_i32)] * 4 + [_i32]),
    "hi3d_wait_timeout_selftest": (_i32, [_i64, _c_void_p]),
    "hi3d_layer_norm_modulate": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _f32, _c_void_p, _c_void_p, _c_void_p,
                                        _c_void_p, _i64, _i64, _i32, _c_void_p]),
    "hi3d_qkv_rope_rms": (_i32, [_c_void_p] * 8 + [_i64, _i64, _i32, _i32, _i32, _i32, _c_void_p]),
    "hi3d_flash_attn_fwd": (_i32, [ctypes.POINTER(AttnArgs), _c_void_p]),
    "hi3d_gate_residual": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _i64, _i64, _i32, _c_void_p]),
    "hi3d_gelu_tanh": (_i32, [_c_void_p, _c_void_p, _i64, _i32, _c_void_p]),
    "hi3d_gemm": (_i32, [_c_void_p] * 4 + [_i64] * 4 + [_i32, _c_void_p, _i64, _i64, _i32, _c_void_p]),
    "hi3d_gemm_w8a8": (_i32, [_c_void_p] * 6 + [_i64] * 4 + [_i32, _c_void_p, _i64, _i64, _i32, _c_void_p]),
    "hi3d_quantize_act_i8": (_i32, [_c_void_p] * 4 + [_i64, _i64, _i32, _i32, _c_void_p]),
    "hi3d_flash_attn_split_workspace_size": (_i32, [ctypes.POINTER(AttnArgs), _i32, ctypes.POINTER(_i64)]),
    "hi3d_flash_attn_fwd_split": (_i32, [ctypes.POINTER(AttnArgs), _i32, _c_void_p, _i64, _c_void_p]),
    "hi3d_flash_attn_fwd_partial": (_i32, [ctypes.POINTER(AttnArgs), _i32, _i32, _c_void_p, _c_void_p, _i64,
                                           _c_void_p]),
    "hi3d_flash_attn_fwd_partial_merge": (_i32, [ctypes.POINTER(AttnArgs), _i32, _c_void_p, _c_void_p, _i64,
                                                 _c_void_p]),
    "hi3d_flash_attn_merge": (_i32, [ctypes.POINTER(AttnArgs), _i32, _c_void_p, _c_void_p, _c_void_p]),
    "hi3d_nccl_unique_id": (_i32, [_c_void_p]),
    "hi3d_nccl_comm_init": (_i32, [_c_void_p, _i32, _i32, ctypes.POINTER(_c_void_p)]),
    "hi3d_nccl_comm_destroy": (_i32, [_c_void_p]),
    "hi3d_nccl_comm_check": (_i32, [_c_void_p]),
    "hi3d_nccl_comm_wait": (_i32, [_c_void_p, _c_void_p, _i64]),
    "hi3d_nccl_comm_abort": (_i32, [_c_void_p]),
    "hi3d_sharded_attn_workspace_size": (_i32, [_c_void_p, _i64, _i32, _i32, ctypes.POINTER(_i64)]),
    "hi3d_sharded_attn": (_i32, [_c_void_p] * 7 + [_i64, _i32, _i32, ctypes.c_float, _i32, _c_void_p, _i64,
                                                   _c_void_p]),
    "hi3d_gemm_qkv_rope": (_i32, [_c_void_p] * 10 + [_i64, _i64, _i32, _i32, _i64, _i32, _i32, _c_void_p]),
    "hi3d_gemm_w8a8_qkv_rope": (_i32, [_c_void_p] * 12 + [_i64, _i64, _i32, _i32, _i64, _i32, _i32, _c_void_p]),
    "hi3d_gemm_qkv_rope_peers": (_i32, [_c_void_p] * 10 + [_i64, _i64, _i32, _i32, _i64, _i32, _i32, _c_void_p,
                                                           _i32, _i64, _c_void_p]),
    "hi3d_gemm_w8a8_qkv_rope_peers": (_i32, [_c_void_p] * 12 + [_i64, _i64, _i32, _i32, _i64, _i32, _i32,
                                                                _c_void_p, _i32, _i64, _c_void_p]),
    "hi3d_peer_barrier": (_i32, [_c_void_p, _i32, _i32, ctypes.c_uint32, _i64, _c_void_p]),
    "hi3d_neighbour_map_workspace_size": (_i32, [_i64, ctypes.POINTER(_i64)]),
    "hi3d_neighbour_map_build": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _i32, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "hi3d_neighbour_map_build_noalloc": (_i32, [_c_void_p, _i64, _c_void_p, _i64, _i32, _c_void_p, _c_void_p]),
    "hi3d_downsample_workspace_size": (_i32, [_i64, ctypes.POINTER(_i64)]),
    "hi3d_downsample_structure": (_i32, [_c_void_p, _i64] + [_c_void_p] * 5 + [_i64, _c_void_p]),
    "hi3d_conv_tap_mask": (_i32, [_c_void_p, _i64, _i64, _c_void_p, _c_void_p]),
    "hi3d_sparse_conv": (_i32, [_c_void_p] * 6 + [_i64, _i64, _i32, _i32, _i32, _c_void_p]),
    "hi3d_layer_norm_act": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _f32, _c_void_p, _c_void_p, _c_void_p,
                                   _c_void_p, _i64, _i64, _i32, _i32, _c_void_p]),
    "hi3d_sparse_conv_act": (_i32, [_c_void_p] * 6 + [_i64, _i64, _i32, _i32, _i32, _i32, _c_void_p]),
    "hi3d_downsample_structure_children": (_i32, [_c_void_p, _i64] + [_c_void_p] * 7 + [_i64, _c_void_p]),
    "hi3d_downsample_mean": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _i32, _c_void_p]),
    "hi3d_upconv_gather_sum": (_i32, [_c_void_p, _c_void_p, _c_void_p, _i64, _i64, _c_void_p, _c_void_p, _i32,
                                      _c_void_p]),
    "hi3d_gather_rows": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _c_void_p, _i32, _c_void_p]),
    "hi3d_group_norm_stats_workspace_size": (_i32, [_i64, _i64, ctypes.POINTER(_i64)]),
    "hi3d_group_norm_stats": (_i32, [_c_void_p, _i64, _i64, _i32, _f32, _c_void_p, _c_void_p, _c_void_p, _i64, _i32,
                                     _c_void_p]),
    "hi3d_group_norm_swish": (_i32, [_c_void_p, _i64, _i64] + [_c_void_p] * 5 + [_i32, _i32, _c_void_p]),
    "hi3d_child_table_workspace_size": (_i32, [_i64, ctypes.POINTER(_i64)]),
    "hi3d_child_structure": (_i32, [_c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "hi3d_child_table": (_i32, [_c_void_p, _i64, _c_void_p, _c_void_p, _i64, _c_void_p, _c_void_p, _c_void_p]),
    "hi3d_layer_norm_quantize": (_i32, [_c_void_p] * 3 + [_i64, _i64, _f32] + [_c_void_p] * 4 + [_i64, _i64,
                                                                                          _c_void_p, _i32,
                                                                                          _c_void_p]),
    "hi3d_serialize_workspace_size": (_i32, [_i64, ctypes.POINTER(_i64)]),
    "hi3d_serialize": (_i32, [_c_void_p, _i64, _i32, _i32, _c_void_p, _c_void_p, _c_void_p, _i64, _c_void_p]),
    "hi3d_window_attention": (_i32, [_c_void_p, _c_void_p, _i64, _i64, _i32, _i32, _i32, _f32, _c_void_p, _i32,
                                     _c_void_p]),
}

_lib = None
_lock = threading.Lock()

# Kernel launches enqueued through this binding (every successful operator call is one
# launch of a library kernel); benchmarks read and reset it.
LAUNCHES = [0]


def load() -> ctypes.CDLL:
    """Load the library (once) and attach the declared signatures."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                raise ImportError(f"hi3d_b200 native library not built: {LIB_PATH} (run build.py)")
            lib = ctypes.CDLL(str(LIB_PATH))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def check(rc: int, what: str, launched: bool = True) -> None:
    """Raise the reference's exception type for a non-zero status."""
    if rc == OK:
        if launched:
            LAUNCHES[0] += 1
        return
    msg = (load().hi3d_last_error_string() or b"").decode(errors="replace")
    text = f"{what}: {msg}" if msg else what
    if rc == ERR_INVALID_ARGUMENT:
        raise ValueError(text)
    if rc == ERR_UNSUPPORTED:
        raise NotImplementedError(text)
    raise RuntimeError(f"{text} (status {rc})")


def device_status(reset: bool = False) -> dict:
    """The library's device status word (first device-side error); syncs the device."""
    vals = [_i32() for _ in range(4)]
    check(load().hi3d_device_status(*[ctypes.byref(v) for v in vals], int(reset)), "device_status", launched=False)
    return dict(zip(("code", "where", "block", "detail"), (v.value for v in vals)))


def dtype_code(t: torch.Tensor) -> int:
    if t.dtype == torch.float16:
        return F16
    if t.dtype == torch.bfloat16:
        return BF16
    if t.dtype == torch.float32:
        return F32
    raise ValueError(f"unsupported dtype {t.dtype}")


def ptr(t: torch.Tensor | None) -> int | None:
    return None if t is None else t.data_ptr()


def stream(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


def require_cuda(*ts: torch.Tensor | None) -> None:
    for t in ts:
        if t is not None and not t.is_cuda:
            raise ValueError("hi3d_b200 operators take CUDA tensors")
