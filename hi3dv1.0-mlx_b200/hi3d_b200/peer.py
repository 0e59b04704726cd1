"""K/V gather of the query-sharded block by peer stores over NVLink.

The gather buffers ``[2, P * S, H, D]`` (K then V, every rank's rows in rank
order) live in symmetric memory: each rank's buffer is mapped into every other
rank's process.  The QKV projection writes this rank's K/V rows into its own
buffer and, from the same epilogue, into the same rows of every peer's buffer
(``hi3d_gemm_qkv_rope_peers``: plain stores over NVLink, so the all-gather
overlaps the projection instead of following it).  ``hi3d_peer_barrier`` then
orders the peers' stores before this rank's attention reads.  Two buffer sets
alternate from block to block, which keeps a rank's stores for block i + 1 off
rows that a peer may still read in block i - 1 (see ``csrc/peer.cu``).

With ``multicast=True`` the projection instead stores each K/V row once to an
NVLink multicast mapping of the buffers (``multimem.st``): NVSwitch writes it
into every GPU's buffer, this one included, so the epilogue issues one store per
row instead of one per GPU.  Either way every load (the attention's TMA loads of
K/V) reads this GPU's own memory; there is no TMA or bulk load with multicast.
"""

from __future__ import annotations

import torch
import torch.distributed as dist

from . import _lib


class PeerKV:
    """Two sets of symmetric K/V gather buffers for ``S = t_local`` rows per rank, plus the
    barrier flags.  Construction is collective over ``group`` (every rank, same sizes).

    ``next()`` returns the next set's ``(k_all, v_all, store)``: ``k_all, v_all [P * S, H, D]``
    and the keyword arguments for ``qkv_rope(..., **store)``: the byte offsets from this rank's
    buffer to each peer's (``peer_offsets``), or to the buffer's multicast mapping
    (``multicast_offset``, with ``multicast=True``; ``RuntimeError`` at construction when the
    GPUs offer no multicast).  ``barrier()`` (after the projection, on the same stream) returns
    once every peer's rows of that set have arrived; a peer that does not arrive within
    ``limit_s`` leaves ``HI3D_ERR_DEVICE_TIMEOUT`` (where 950) in the device status word instead
    of hanging the GPU."""

    def __init__(self, t_local: int, heads: int, d: int, dtype, device, group=None, limit_s: float = 5.0,
                 multicast: bool = False):
        import torch.distributed._symmetric_memory as symm

        pg = group if group is not None else dist.group.WORLD
        self.group = group
        self.world, self.rank = dist.get_world_size(group), dist.get_rank(group)
        if not 1 < self.world <= 8:
            raise ValueError(f"peer stores need 2 to 8 ranks of one node, not {self.world}")
        self.shape = (2, self.world * t_local, heads, d)
        self.dtype, self.device = dtype, torch.device(device)
        self._sets = []
        for _ in range(2):
            buf = symm.empty(self.shape, dtype=dtype, device=self.device)
            handle = symm.rendezvous(buf, pg)
            ptrs = list(handle.buffer_ptrs)
            # the buffer must sit at the same place of every rank's mapping: peer address = own + delta
            place = [None] * self.world
            dist.all_gather_object(place, buf.data_ptr() - ptrs[self.rank], group=group)
            if len(set(place)) != 1:
                raise RuntimeError(f"symmetric buffers at different offsets on the ranks: {place}")
            if multicast:
                mc = int(handle.multicast_ptr)
                if not mc:
                    raise RuntimeError("symmetric memory has no multicast mapping on these GPUs")
                store = {"multicast_offset": mc - ptrs[self.rank]}
            else:
                store = {"peer_offsets": tuple(int(ptrs[p] - ptrs[self.rank])
                                               for p in range(self.world) if p != self.rank)}
            self._sets.append((buf, handle, store))
        flags = symm.empty((self.world,), dtype=torch.int32, device=self.device)
        flags.zero_()
        fh = symm.rendezvous(flags, pg)
        fptrs = list(fh.buffer_ptrs)
        delta = flags.data_ptr() - fptrs[self.rank]  # the flags' place inside each rank's mapping
        place = [None] * self.world
        dist.all_gather_object(place, delta, group=group)
        if len(set(place)) != 1:
            raise RuntimeError(f"symmetric flags at different offsets on the ranks: {place}")
        self._flag_ptrs = torch.tensor([p + delta for p in fptrs], dtype=torch.int64, device=self.device)
        self._flags = (flags, fh)
        torch.cuda.synchronize(self.device)
        dist.barrier(group=group)  # every rank's flags are zero before anyone signals
        self.epoch = 0
        self.limit_ns = int(limit_s * 1e9)
        self._next = 0

    def next(self) -> tuple[torch.Tensor, torch.Tensor, dict]:
        buf, _, store = self._sets[self._next % 2]
        self._next += 1
        return buf[0], buf[1], store

    def close(self) -> None:
        """Drop the buffers on every rank at the same point (collective): each rank first waits
        for its own kernels, then all ranks meet, so no GPU still stores into a buffer (or its
        multicast mapping) while a peer releases it; all ranks meet again afterwards."""
        import gc

        if not self._sets:
            return
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)
        self._sets, self._flags, self._flag_ptrs = [], None, None
        gc.collect()
        torch.cuda.synchronize(self.device)
        dist.barrier(group=self.group)

    def barrier(self, like: torch.Tensor) -> None:
        """The cross-rank barrier on the current stream of ``like``'s device."""
        self.epoch = (self.epoch + 1) & 0xFFFFFFFF or 1  # flags start at 0: never wait for 0
        rc = _lib.load().hi3d_peer_barrier(self._flag_ptrs.data_ptr(), self.rank, self.world, self.epoch,
                                           self.limit_ns, _lib.stream(like))
        _lib.check(rc, "peer_barrier")
