"""Query-sharded execution of the block stack across the GPUs of one node.

Rank ``r`` of ``P`` owns a contiguous slice of the object's tokens (query rows).
Everything in the block is row-local except self-attention, which needs the
keys/values of every token: each block all-gathers K and V (token-major
``[T/P, H, D]`` shards -> ``[T, H, D]``) with NCCL over NVLink, then runs the
local queries against all keys.  Cross-attention K/V (the condition) are
replicated.  This is a plain context-parallel split; softmax rows never cross
ranks, so the result equals the single-GPU block up to GEMM shape effects.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import attention, kernels
from .peer import PeerKV
from .transformer import _modulation, linear, modulation_all, qkv_rope


def init_nccl(device, timeout_s: float = 300.0) -> None:
    """``torch.distributed`` over NCCL for one process per GPU (env:// rendezvous), with the
    NCCL streams at high priority: the K/V gather's copy kernels then take the next SMs that
    free up while the attention grid (one CTA per SM) occupies the GPU, instead of waiting
    behind the whole grid."""
    import datetime

    opts = dist.ProcessGroupNCCL.Options()
    opts.is_high_priority_stream = True
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=timeout_s), device_id=device,
                            pg_options=opts)


def shard_slice(total: int, rank: int, world: int) -> slice:
    """Contiguous query-row slice of ``rank``: the rows ``[rank * total / world, ...)``."""
    if total % world:
        raise ValueError(f"{total} rows do not split evenly over {world} ranks")
    per = total // world
    return slice(rank * per, (rank + 1) * per)


def gather_rows(local: torch.Tensor, group=None, out: torch.Tensor | None = None, async_op: bool = False):
    """All-gather equal row shards ``[rows, ...]`` of every rank into ``[world * rows, ...]`` in rank
    order (NCCL over NVLink for CUDA tensors, gloo for CPU tensors)."""
    world = dist.get_world_size(group)
    if out is None:
        out = torch.empty((world * local.shape[0], *local.shape[1:]), dtype=local.dtype, device=local.device)
    work = dist.all_gather_into_tensor(out, local.contiguous(), group=group, async_op=async_op)
    return (out, work) if async_op else out


class PhaseTimer:
    """CUDA events at the phase boundaries of the sharded block, on the compute stream: the
    time between consecutive marks is charged to the phase named by the later mark.  Used by
    the benchmark's per-phase breakdown; None (the default) records nothing."""

    def __init__(self):
        self.marks: list[tuple[str, torch.cuda.Event]] = []

    def mark(self, name: str) -> None:
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        self.marks.append((name, e))

    def totals(self) -> dict[str, float]:
        """Milliseconds per phase, summed over everything recorded (synchronises)."""
        torch.cuda.synchronize()
        out: dict[str, float] = {}
        for (_, e0), (name, e1) in zip(self.marks, self.marks[1:]):
            if name != "start":
                out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        return out


def sharded_self_attention(q: torch.Tensor, k_all: torch.Tensor, v_all: torch.Tensor, scale: float, group=None,
                           mark=None) -> torch.Tensor:
    """Self-attention of this rank's query rows over the keys of every rank of ``group``, which
    hold consecutive slices of one sequence.  ``q [1, S, H, D]`` (token-major); ``k_all, v_all
    [P * S, H, D]`` whose rows ``[r * S, (r + 1) * S)`` already hold this rank's keys / values
    (the QKV projection writes them there, ``qkv_rope(out=...)``).  The other ranks' rows are
    filled by one in-place all-gather each (NCCL over NVLink, on the high-priority NCCL stream,
    which the current stream then waits for), and the queries attend all keys in one pass;
    returns ``[1, S, H * D]``.  Softmax rows never cross ranks, so the result is the single-GPU
    attention of these rows.  Attending the own keys while the gather runs and merging partials
    was measured slower: the partial kernel and the merge cost more than the exposed gather.
    ``mark`` (a :class:`PhaseTimer` method) receives the phase boundaries."""
    mark = mark or (lambda name: None)
    gather_kv(k_all, v_all, group)
    mark("kv_gather_wait")
    out = attend_gathered(q, k_all, v_all, scale)
    mark("attention")
    return out


def attend_gathered(q: torch.Tensor, k_all: torch.Tensor, v_all: torch.Tensor, scale: float) -> torch.Tensor:
    """This rank's queries ``[1, S, H, D]`` over all gathered keys ``[P * S, H, D]`` in one pass
    (key-split only when the grid is short of waves); returns ``[1, S, H * D]``."""
    bhnd = lambda x: x.permute(1, 0, 2)[None]  # [rows, H, D] token-major -> [1, H, rows, D] view
    return attention.flash_attention(q, bhnd(k_all), bhnd(v_all), scale, q_layout="bnhd")


def gather_kv(k_all: torch.Tensor, v_all: torch.Tensor, group=None) -> None:
    """Fill the other ranks' rows of ``k_all, v_all [P * S, ...]`` from this rank's rows
    (:func:`own_rows`) in place: one all-gather each, both in one NCCL group for CUDA tensors
    (gloo for CPU ones)."""
    if dist.get_world_size(group) == 1:
        return
    if k_all.is_cuda:  # both gathers in one NCCL group (one launch)
        from torch.distributed.distributed_c10d import _coalescing_manager

        with _coalescing_manager(group):
            for buf in (k_all, v_all):
                dist.all_gather_into_tensor(buf, own_rows(buf, group)[0], group=group)
        return
    for buf in (k_all, v_all):
        dist.all_gather_into_tensor(buf, own_rows(buf, group)[0], group=group)


def kv_gather_buffers(t_local: int, heads: int, d: int, dtype, device, group=None):
    """``k_all, v_all [P * t_local, H, D]``: the gather buffers of :func:`sharded_self_attention`."""
    shape = (dist.get_world_size(group) * t_local, heads, d)
    return tuple(torch.empty(shape, dtype=dtype, device=device) for _ in range(2))


def own_rows(buf: torch.Tensor, group=None) -> torch.Tensor:
    """This rank's slice ``[1, S, H, D]`` of a gather buffer ``[P * S, H, D]`` (contiguous)."""
    world = dist.get_world_size(group)
    t = buf.shape[0] // world
    r = dist.get_rank(group)
    return buf[r * t:(r + 1) * t].view(1, t, *buf.shape[1:])


def object_group(objects: int, group=None):
    """For ``objects`` equal packed sequences split into contiguous slices over the ranks of
    ``group``: the subgroup of the ranks that share this rank's object when there are more ranks
    than objects (each object over ``world / objects`` ranks), or None when every rank holds
    whole objects and self-attention needs no exchange.  Every rank of ``group`` must call this
    (subgroup creation is collective)."""
    world = dist.get_world_size(group)
    rank = dist.get_rank(group)
    if world <= objects:
        if objects % world:
            raise ValueError(f"{objects} objects do not split evenly over {world} ranks")
        return None
    if world % objects:
        raise ValueError(f"{world} ranks do not split evenly over {objects} objects")
    per = world // objects
    ranks = dist.get_process_group_ranks(group) if group is not None else list(range(world))
    mine = None
    for o in range(objects):
        sub = dist.new_group(ranks[o * per:(o + 1) * per])
        if o == rank // per:
            mine = sub
    return mine


def block_forward_sharded(w: dict, x: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                          ck: torch.Tensor, cv: torch.Tensor, heads: int, group=None,
                          kv_buffers=None, timer: PhaseTimer | None = None,
                          mods: tuple | None = None) -> torch.Tensor:
    """One block on this rank's rows ``x [T/P, C]`` (updated in place) of a single object.
    ``kv_buffers``: the K/V gather buffers, either a pair from :func:`kv_gather_buffers` (filled
    by an NCCL all-gather after the projection; allocated when None) or a
    :class:`hi3d_b200.peer.PeerKV` (the projection stores the rows into every peer's buffer
    itself, then a cross-GPU barrier).  ``timer`` marks the phases: LN + QKV projection, K/V
    gather (or barrier), self-attention, its output projection, LN + cross-attention Q,
    cross-attention, its output projection, LN + MLP.
    ``mods``: this block's modulation vectors precomputed by
    :func:`hi3d_b200.transformer.modulation_all`."""
    mark = timer.mark if timer is not None else (lambda name: None)
    mark("start")
    t_local, c = x.shape
    d = c // heads
    scale = d ** -0.5
    dt = x.dtype
    shift_msa, scale_msa, gate_msa, shift_mlp, scale_mlp, gate_mlp = mods if mods is not None else \
        _modulation(w, mod, c, dt)

    if kv_buffers is None:
        kv_buffers = kv_gather_buffers(t_local, heads, d, dt, x.device, group)
    h = kernels.layer_norm_modulate(x, 1e-6, scale=scale_msa, shift=shift_msa)
    if isinstance(kv_buffers, PeerKV):
        k_all, v_all, store = kv_buffers.next()
        q, _, _ = qkv_rope(h, w, cos, sin, 1, heads, d, token_major=True,
                           out=(None, own_rows(k_all, group), own_rows(v_all, group)), **store)
        mark("qkv")
        kv_buffers.barrier(q)
        mark("kv_gather_wait")
        a = attend_gathered(q, k_all, v_all, scale)
        mark("attention")
    else:
        k_all, v_all = kv_buffers
        q, _, _ = qkv_rope(h, w, cos, sin, 1, heads, d, token_major=True,
                           out=(None, own_rows(k_all, group), own_rows(v_all, group)))
        mark("qkv")
        a = sharded_self_attention(q, k_all, v_all, scale, group, mark)
    linear(a[0], w, "self_attn.to_out", epilogue="residual", residual=x, gate=gate_msa)
    mark("to_out")

    h = kernels.layer_norm_modulate(x, 1e-6, weight=w["norm2.weight"], bias=w["norm2.bias"])
    qc = linear(h, w, "cross_attn.to_q").view(1, t_local, heads, d)
    mark("cross_q")
    o = attention.flash_attention(qc, ck, cv, scale, q_layout="bnhd")[0]
    mark("cross_attention")
    linear(o, w, "cross_attn.to_out", epilogue="residual", residual=x)
    mark("cross_out")

    h = kernels.layer_norm_modulate(x, 1e-6, scale=scale_mlp, shift=shift_mlp)
    h = linear(h, w, "mlp.mlp.0", epilogue="gelu")
    linear(h, w, "mlp.mlp.2", epilogue="residual", residual=x, gate=gate_mlp)
    mark("mlp")
    return x


def auto_transport(world: int, device=None) -> str:
    """The K/V transport measured fastest for the cfg1 stack at this rank count (ms per step):
    the peer stores at 2 ranks (88.6; NCCL 90.7), the multicast stores at 4 and 8 ranks (50.5
    and 29.8; NCCL 51.3 and 30.6, the peer stores 31.8 at 8), or the NCCL all-gather there when
    the GPUs offer no NVLink multicast (``device``: the CUDA device to ask; assumed to offer it
    when None)."""
    if world <= 2:
        return "peer"
    if device is not None:
        import torch.distributed._symmetric_memory as symm

        dev = torch.device(device)
        if dev.type != "cuda" or not symm._SymmetricMemory.has_multicast_support(
                torch._C._autograd.DeviceType.CUDA, dev.index if dev.index is not None else 0):
            return "nccl"
    return "multicast"


class ShardedBlockStack:
    """The block stack over ``P`` ranks, token-sharded; weights replicated on every rank.
    ``transport``: how each block's K/V reach the other ranks, ``"nccl"`` (in-place NCCL
    all-gather after the projection), ``"peer"`` (the projection's epilogue stores them into
    the peers' symmetric buffers over NVLink, then a cross-GPU barrier; :class:`PeerKV`) or
    ``"multicast"`` (the same with one multimem store per row through NVSwitch)."""

    def __init__(self, weights: list[dict], heads: int, group=None, transport: str = "auto"):
        if transport not in ("auto", "nccl", "peer", "multicast"):
            raise ValueError(f"unknown K/V transport {transport!r}")
        self.weights = weights
        self.heads = heads
        self.group = group
        self.transport = transport
        self._kv = None
        self._kv_key = None
        self._mod_w = None  # [blocks, 6C] stacked modulation parameters (built on first use)

    def close(self) -> None:
        """Release the K/V buffers; collective with the peer transports (:meth:`PeerKV.close`):
        every rank calls it at the same point before the buffers go away."""
        if isinstance(self._kv, PeerKV):
            self._kv.close()
        self._kv, self._kv_key = None, None

    def __call__(self, x_local: torch.Tensor, mod: torch.Tensor, cos: torch.Tensor, sin: torch.Tensor,
                 kvs: list[tuple[torch.Tensor, torch.Tensor]], timer: PhaseTimer | None = None) -> torch.Tensor:
        x = x_local.clone()
        t_local, c = x.shape
        world = dist.get_world_size(self.group)
        key = (t_local, c, x.dtype, x.device)
        if self._kv is None or self._kv_key != key:  # (re)built on every rank alike: PeerKV is collective
            self.close()
            d = c // self.heads
            if self.transport == "auto":
                self.transport = auto_transport(world, x.device)
            if self.transport in ("peer", "multicast") and world > 1:
                self._kv = PeerKV(t_local, self.heads, d, x.dtype, x.device, self.group,
                                  multicast=self.transport == "multicast")
            else:
                self._kv = kv_gather_buffers(t_local, self.heads, d, x.dtype, x.device, self.group)
            self._kv_key = key
        if self._mod_w is None:
            self._mod_w = torch.stack([w["modulation"].reshape(-1).float() for w in self.weights])
        mods = modulation_all(self._mod_w, mod, c, x.dtype)  # every block's vectors in a few launches
        for i, w in enumerate(self.weights):
            block_forward_sharded(w, x, mod, cos, sin, kvs[i][0], kvs[i][1], self.heads, self.group, self._kv,
                                  timer=timer, mods=mods[i])
        return x


class NcclComm:
    """The library's own NCCL communicator (``hi3d_nccl_comm_init``) over the ranks of a
    torch.distributed group: rank 0 creates the id, which is broadcast through the group."""

    def __init__(self, group=None):
        import ctypes

        from . import _lib

        lib = _lib.load()
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        buf = ctypes.create_string_buffer(128)
        if self.rank == 0:
            _lib.check(lib.hi3d_nccl_unique_id(buf), "nccl_unique_id", launched=False)
        obj = [buf.raw if self.rank == 0 else None]
        dist.broadcast_object_list(obj, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
        self._id = ctypes.create_string_buffer(obj[0], 128)
        handle = ctypes.c_void_p()
        _lib.check(lib.hi3d_nccl_comm_init(self._id, self.world, self.rank, ctypes.byref(handle)), "nccl_comm_init",
                   launched=False)
        self.handle = handle

    def check(self) -> None:
        """Raise ``RuntimeError`` if NCCL reports an asynchronous error on this communicator."""
        from . import _lib

        _lib.check(_lib.load().hi3d_nccl_comm_check(self.handle), "nccl_comm_check", launched=False)

    def wait(self, stream=None, timeout_s: float = 30.0) -> None:
        """Wait on the host for the work enqueued on ``stream`` (default: the current stream) and
        on the gather's side stream; on an asynchronous NCCL error or after ``timeout_s`` the
        communicator is aborted (which ends collectives still waiting for a peer) and
        ``RuntimeError`` is raised."""
        import torch

        from . import _lib

        st = (stream or torch.cuda.current_stream()).cuda_stream
        _lib.check(_lib.load().hi3d_nccl_comm_wait(self.handle, st, int(timeout_s * 1000)), "nccl_comm_wait",
                   launched=False)

    def abort(self) -> None:
        """Abort the communicator (a peer is known to be gone); it then refuses new work."""
        from . import _lib

        _lib.check(_lib.load().hi3d_nccl_comm_abort(self.handle), "nccl_comm_abort", launched=False)

    def close(self) -> None:
        from . import _lib

        if self.handle:
            _lib.check(_lib.load().hi3d_nccl_comm_destroy(self.handle), "nccl_comm_destroy", launched=False)
            self.handle = None


def sharded_attention(comm: NcclComm, q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                      kv_buffers: tuple[torch.Tensor, torch.Tensor] | None = None) -> torch.Tensor:
    """Self-attention of this rank's rows through the native ``hi3d_sharded_attn``: ``q, k, v
    [S, H, D]`` (token-major slices of one sequence, rank order); K/V gathered over the library's
    NCCL communicator, then all keys attended in one launch.  Returns ``[S, H * D]``."""
    import ctypes

    from . import _lib

    _lib.require_cuda(q, k, v)
    s_rows, heads, d = q.shape
    if k.shape != q.shape or v.shape != q.shape or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("q, k, v must be [S, H, D] slices of one dtype")
    q, k, v = q.contiguous(), k.contiguous(), v.contiguous()
    if kv_buffers is None:
        kv_buffers = tuple(torch.empty((comm.world * s_rows, heads, d), dtype=q.dtype, device=q.device)
                           for _ in range(2))
    k_all, v_all = kv_buffers
    lib = _lib.load()
    nbytes = ctypes.c_int64()
    _lib.check(lib.hi3d_sharded_attn_workspace_size(comm.handle, s_rows, heads, d, ctypes.byref(nbytes)),
               "sharded_attn workspace", launched=False)
    ws = torch.empty(nbytes.value, dtype=torch.uint8, device=q.device)
    out = torch.empty((s_rows, heads * d), dtype=q.dtype, device=q.device)
    rc = lib.hi3d_sharded_attn(comm.handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), k_all.data_ptr(),
                               v_all.data_ptr(), out.data_ptr(), s_rows, heads, d, float(scale), _lib.dtype_code(q),
                               ws.data_ptr(), ws.numel(), _lib.stream(q))
    _lib.check(rc, "sharded_attention")
    return out
