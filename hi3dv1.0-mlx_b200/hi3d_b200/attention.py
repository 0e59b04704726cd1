"""Flash attention on the B200 tensor cores (tcgen05 + TMEM, TMA-fed).

:func:`flash_attention` keeps the signature and output layout of
``hi3d_mac.mlx_backend.attention.flash_attention`` (src/hi3d_mac/mlx_backend/attention.py:238-277);
:func:`flash_attn_varlen` is the packed variable-length form the upstream
``flash_attn`` API needs (src/sparc3d/nn/sparse/attention/full_attn.py:56-76).

Arithmetic (as the reference kernel, attention.py:19-22): ``S = Q K^T`` in fp32,
online softmax in fp32 in the exp2 domain, ``P`` rounded to the input dtype for
``P V`` which accumulates in fp32, output ``O / l`` rounded once.
"""

from __future__ import annotations

import ctypes
import functools
import math

import torch

from . import _lib

SUPPORTED_HEAD_DIMS = (64, 96, 128)


def _strides3(t: torch.Tensor, layout: str) -> tuple[int, int, int]:
    """(row, head, batch) element strides of a 4-D tensor in ``bhnd`` / ``bnhd`` layout."""
    s = t.stride()
    if layout == "bhnd":
        return s[2], s[1], s[0]
    return s[1], s[2], s[0]


def _check_inner(t: torch.Tensor, name: str) -> None:
    if t.stride(-1) != 1:
        raise ValueError(f"{name} must have a contiguous head dimension")


class KernelTimer:
    """Optional CUDA-event timing of every attention launch on the launching stream.

    ``start()`` arms it, ``stop()`` synchronises and returns one record per launch
    (``nq``, ``nk`` rows; ``flops`` = 4 * Nq * Nk * H * D for dense launches, None for varlen
    ones; ``ms`` the event-timed duration).
    """

    def __init__(self):
        self.records = None

    def start(self) -> None:
        self.records = []

    def stop(self) -> list[dict]:
        recs, self.records = self.records or [], None
        torch.cuda.synchronize()
        return [dict(r, ms=r.pop("e0").elapsed_time(r.pop("e1"))) for r in recs]


TIMER = KernelTimer()


@functools.lru_cache(maxsize=None)
def _sm_count(device_index: int) -> int:
    return torch.cuda.get_device_properties(device_index).multi_processor_count


# Fixed time of one attention CTA (set-up, Q load and first scores, epilogue) in key blocks:
# ≈ 5670 cycles against ≈ 2525 per 128-key block (cfg1 clock traces).
CTA_OVERHEAD_BLOCKS = 2.25
PARTIAL_FACTOR = 1.2  # measured: the partial kernel + merge against the single pass, same keys


def auto_splits(ctas: int, key_blocks: int, sms: int, max_splits: int = 8) -> int:
    """Key splits per query block for ``ctas`` query-block CTAs over ``key_blocks`` key blocks on
    ``sms`` SMs (one CTA per SM): the s minimising the modelled launch time
    ceil(ctas * s / sms) * (overhead + key_blocks / s), a split launch (the partial kernel, its
    fp32 partials and the merge) charged :data:`PARTIAL_FACTOR` times the single pass, taken only
    when it beats no split by more than 3 %.  Short key ranges (cross-attention) and grids of
    about two waves or more stay unsplit."""
    cost = lambda s: (math.ceil(ctas * s / sms) * (CTA_OVERHEAD_BLOCKS + key_blocks / s)
                      * (PARTIAL_FACTOR if s > 1 else 1.0))
    best, best_t = 1, cost(1)
    for s in range(2, max_splits + 1):
        if key_blocks < 2 * s:
            break
        t = cost(s)
        if t < best_t * 0.97:
            best, best_t = s, t
    return best


def _resolve_splits(k_splits, args: _lib.AttnArgs, dev_tensor: torch.Tensor) -> int:
    if k_splits != "auto":
        return int(k_splits)
    tiles = math.ceil(args.max_seqlen_q / 256)
    bk = 128 if args.head_dim == 64 else 64
    longest_k = args.nk if not args.cu_seqlens_k else args.nk  # packed: bounded by the total
    return auto_splits(tiles * args.num_seqs * args.heads, math.ceil(longest_k / bk), _sm_count(dev_tensor.device.index))


def _launch(args: _lib.AttnArgs, dev_tensor: torch.Tensor, k_splits=1) -> None:
    stream = _lib.stream(dev_tensor)
    splits = _resolve_splits(k_splits, args, dev_tensor)
    rec = TIMER.records is not None
    if rec:
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
    lib = _lib.load()
    if splits > 1:
        nbytes = ctypes.c_int64()
        _lib.check(lib.hi3d_flash_attn_split_workspace_size(ctypes.byref(args), splits, ctypes.byref(nbytes)),
                   "flash_attention split workspace", launched=False)
        ws = torch.empty(nbytes.value, dtype=torch.uint8, device=dev_tensor.device)
        rc = lib.hi3d_flash_attn_fwd_split(ctypes.byref(args), splits, ws.data_ptr(), ws.numel(), stream)
    else:
        rc = lib.hi3d_flash_attn_fwd(ctypes.byref(args), stream)
    _lib.check(rc, "flash_attention")
    if rec:
        e1.record()
        dense = not args.cu_seqlens_q
        flops = 4.0 * args.nq * args.nk * args.heads * args.head_dim * args.num_seqs if dense else None
        TIMER.records.append({"nq": args.nq, "nk": args.nk, "flops": flops, "e0": e0, "e1": e1})


def flash_attention(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, scale: float,
                    q_layout: str = "bhnd", k_splits: int | str = "auto") -> torch.Tensor:
    """``softmax(q k^T * scale) v`` for fp16/bf16 inputs, returned as ``[B, Nq, H * D]``.

    Args:
        q: ``[B, H, Nq, D]`` (``q_layout="bhnd"``) or ``[B, Nq, H, D]`` (``"bnhd"``).
        k, v: ``[B, H, Nk, D]``, or ``[1, H, Nk, D]`` shared by every batch element.
        scale: softmax scale applied to ``q k^T``.
        k_splits: key ranges per query block computed by separate CTAs and merged
            (``hi3d_flash_attn_fwd_split``); ``"auto"`` splits only when the query blocks alone
            leave a partial last wave (e.g. one query shard per GPU).
    """
    _lib.require_cuda(q, k, v)
    if q_layout == "bhnd":
        batch, heads, nq, dim = q.shape
    elif q_layout == "bnhd":
        batch, nq, heads, dim = q.shape
    else:
        raise ValueError(f"unknown q layout {q_layout!r}")
    nk = k.shape[2]
    if (dim not in SUPPORTED_HEAD_DIMS or k.shape[1] != heads or k.shape[3] != dim or k.shape[0] not in (1, batch)
            or v.shape != k.shape):
        raise ValueError(f"unsupported shapes q {tuple(q.shape)} k {tuple(k.shape)}")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("flash_attention takes float16 (or bfloat16) inputs of one dtype")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check_inner(t, n)
    out = torch.empty((batch, nq, heads * dim), dtype=q.dtype, device=q.device)
    if nq == 0 or batch == 0:
        return out
    _launch(_dense_args(q, k, v, out, scale, q_layout), q, k_splits)
    return out


def _dense_args(q, k, v, out, scale: float, q_layout: str) -> _lib.AttnArgs:
    if q_layout == "bhnd":
        batch, heads, nq, dim = q.shape
    else:
        batch, nq, heads, dim = q.shape
    qr, qh, qb = _strides3(q, q_layout)
    kr, kh, kb = _strides3(k, "bhnd")
    vr, vh, vb = _strides3(v, "bhnd")
    if k.shape[0] == 1:
        kb = vb = 0
    return _lib.AttnArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
        q_row=qr, q_head=qh, q_batch=qb, k_row=kr, k_head=kh, k_batch=kb, v_row=vr, v_head=vh, v_batch=vb,
        o_row=heads * dim, o_head=dim, o_batch=nq * heads * dim,
        cu_seqlens_q=None, cu_seqlens_k=None, nq=nq, nk=k.shape[2], max_seqlen_q=nq,
        num_seqs=batch, heads=heads, head_dim=dim, dtype=_lib.dtype_code(q), scale=float(scale))


def auto_key_splits(q_rows: int, k_rows: int, heads: int, head_dim: int, batch: int = 1, device=None) -> int:
    """The key splits :func:`flash_attention` picks with ``k_splits="auto"`` for these sizes."""
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    bk = 128 if head_dim == 64 else 64
    return auto_splits(math.ceil(q_rows / 256) * batch * heads, math.ceil(k_rows / bk), _sm_count(dev.index))


class AttentionParts:
    """Attention of one set of queries over several disjoint key sets, combined exactly by their
    log-sum-exp weights: :meth:`add` one key set at a time (``hi3d_flash_attn_fwd_partial``), then
    :meth:`merge` (``hi3d_flash_attn_merge``), or finish with :meth:`add_final`, which merges in
    the last launch's epilogue.  For key sets that arrive at different times; the sharded block
    gathers all keys first and attends them in one pass, which measured faster.  Queries and keys as in
    :func:`flash_attention`; ``slots`` bounds the total key splits of all ``add`` calls."""

    def __init__(self, q: torch.Tensor, scale: float, slots: int, q_layout: str = "bhnd"):
        _lib.require_cuda(q)
        if q_layout not in ("bhnd", "bnhd"):
            raise ValueError(f"unknown q layout {q_layout!r}")
        _check_inner(q, "q")
        self.q, self.scale, self.layout = q, float(scale), q_layout
        if q_layout == "bhnd":
            self.batch, self.heads, self.nq, self.dim = q.shape
        else:
            self.batch, self.nq, self.heads, self.dim = q.shape
        rows = self.batch * self.nq
        self.part_o = torch.empty((slots, rows, self.heads, self.dim), dtype=torch.float32, device=q.device)
        self.part_lse = torch.empty((slots, rows, self.heads), dtype=torch.float32, device=q.device)
        self.slots, self.used = slots, 0

    def add(self, k: torch.Tensor, v: torch.Tensor, k_splits: int | str = "auto") -> None:
        _lib.require_cuda(k, v)
        if k.shape[1] != self.heads or k.shape[3] != self.dim or v.shape != k.shape or k.dtype != self.q.dtype:
            raise ValueError(f"keys {tuple(k.shape)} do not match the queries")
        for t, n in ((k, "k"), (v, "v")):
            _check_inner(t, n)
        if k.shape[2] == 0 or self.nq == 0 or self.batch == 0:
            return
        args = _dense_args(self.q, k, v, self.part_o, self.scale, self.layout)
        splits = _resolve_splits(k_splits, args, self.q)
        if self.used + splits > self.slots:
            raise ValueError(f"{self.used + splits} key splits exceed the {self.slots} partial slots")
        rec = TIMER.records is not None
        if rec:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        rc = _lib.load().hi3d_flash_attn_fwd_partial(ctypes.byref(args), splits, self.used, self.part_o.data_ptr(),
                                                     self.part_lse.data_ptr(), self.batch * self.nq,
                                                     _lib.stream(self.q))
        _lib.check(rc, "flash_attention partial")
        if rec:
            e1.record()
            flops = 4.0 * args.nq * args.nk * args.heads * args.head_dim * args.num_seqs
            TIMER.records.append({"nq": args.nq, "nk": args.nk, "flops": flops, "e0": e0, "e1": e1, "part": True})
        self.used += splits

    def add_final(self, k: torch.Tensor, v: torch.Tensor) -> torch.Tensor:
        """The last key set in one pass, merged with the partials added so far inside the
        attention kernel's epilogue (``hi3d_flash_attn_fwd_partial_merge``); returns the
        ``[B, Nq, H * D]`` output that :meth:`merge` would return after ``add(k, v, 1)``."""
        _lib.require_cuda(k, v)
        if k.shape[1] != self.heads or k.shape[3] != self.dim or v.shape != k.shape or k.dtype != self.q.dtype:
            raise ValueError(f"keys {tuple(k.shape)} do not match the queries")
        for t, n in ((k, "k"), (v, "v")):
            _check_inner(t, n)
        if k.shape[2] == 0:
            return self.merge()
        out = torch.empty((self.batch, self.nq, self.heads * self.dim), dtype=self.q.dtype, device=self.q.device)
        if self.nq == 0 or self.batch == 0:
            return out
        args = _dense_args(self.q, k, v, out, self.scale, self.layout)
        rec = TIMER.records is not None
        if rec:
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
        rc = _lib.load().hi3d_flash_attn_fwd_partial_merge(ctypes.byref(args), self.used, self.part_o.data_ptr(),
                                                           self.part_lse.data_ptr(), self.batch * self.nq,
                                                           _lib.stream(self.q))
        _lib.check(rc, "flash_attention partial merge")
        if rec:
            e1.record()
            flops = 4.0 * args.nq * args.nk * args.heads * args.head_dim * args.num_seqs
            TIMER.records.append({"nq": args.nq, "nk": args.nk, "flops": flops, "e0": e0, "e1": e1, "part": True})
        return out

    def merge(self) -> torch.Tensor:
        """``[B, Nq, H * D]`` from all key sets added so far."""
        out = torch.empty((self.batch, self.nq, self.heads * self.dim), dtype=self.q.dtype, device=self.q.device)
        if self.used == 0 or self.nq == 0 or self.batch == 0:
            return out
        args = _dense_args(self.q, self.q if self.layout == "bhnd" else self.q.transpose(1, 2),
                           self.q if self.layout == "bhnd" else self.q.transpose(1, 2), out, self.scale, self.layout)
        rc = _lib.load().hi3d_flash_attn_merge(ctypes.byref(args), self.used, self.part_o.data_ptr(),
                                               self.part_lse.data_ptr(), _lib.stream(self.q))
        _lib.check(rc, "flash_attention merge")
        return out


def flash_attn_varlen(q: torch.Tensor, k: torch.Tensor, v: torch.Tensor, cu_seqlens_q: torch.Tensor,
                      cu_seqlens_k: torch.Tensor | None, max_seqlen_q: int, scale: float,
                      out: torch.Tensor | None = None, k_splits: int | str = "auto") -> torch.Tensor:
    """Packed variable-length attention: ``q [Tq, H, D]``, ``k, v [Tk, H, D]`` (any row
    stride, contiguous head dim), ``cu_seqlens_*`` int32 ``[num_seqs + 1]`` on the device.
    ``cu_seqlens_k=None`` shares all ``Tk`` keys with every sequence.  Returns ``[Tq, H, D]``.
    ``k_splits`` as in :func:`flash_attention`.
    """
    _lib.require_cuda(q, k, v, cu_seqlens_q, cu_seqlens_k)
    tq, heads, dim = q.shape
    tk = k.shape[0]
    if dim not in SUPPORTED_HEAD_DIMS or k.shape[1:] != (heads, dim) or v.shape[1:] != (heads, dim):
        raise ValueError(f"unsupported shapes q {tuple(q.shape)} k {tuple(k.shape)} v {tuple(v.shape)}")
    if q.dtype not in (torch.float16, torch.bfloat16) or k.dtype != q.dtype or v.dtype != q.dtype:
        raise ValueError("flash attention takes float16 or bfloat16 inputs of one dtype")
    for t, n in ((q, "q"), (k, "k"), (v, "v")):
        _check_inner(t, n)
    cu_q = cu_seqlens_q.to(torch.int32).contiguous()
    cu_k = None if cu_seqlens_k is None else cu_seqlens_k.to(torch.int32).contiguous()
    num_seqs = cu_q.numel() - 1
    if cu_k is not None and cu_k.numel() != cu_q.numel():
        raise ValueError("cu_seqlens_q and cu_seqlens_k must have the same length")
    if out is None:
        out = torch.empty((tq, heads, dim), dtype=q.dtype, device=q.device)
    if tq == 0 or num_seqs <= 0:
        return out
    args = _lib.AttnArgs(
        q=q.data_ptr(), k=k.data_ptr(), v=v.data_ptr(), out=out.data_ptr(),
        q_row=q.stride(0), q_head=q.stride(1), q_batch=0, k_row=k.stride(0), k_head=k.stride(1), k_batch=0,
        v_row=v.stride(0), v_head=v.stride(1), v_batch=0,
        o_row=out.stride(0), o_head=out.stride(1), o_batch=0,
        cu_seqlens_q=cu_q.data_ptr(), cu_seqlens_k=None if cu_k is None else cu_k.data_ptr(),
        nq=tq, nk=tk, max_seqlen_q=int(max_seqlen_q), num_seqs=num_seqs, heads=heads, head_dim=dim,
        dtype=_lib.dtype_code(q), scale=float(scale))
    _launch(args, q, k_splits)
    return out
