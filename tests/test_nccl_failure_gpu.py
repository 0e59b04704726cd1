"""Failure handling of the library's own NCCL communicator, made to happen without a GPU fault.

* One GPU: ``hi3d_nccl_comm_wait`` on a stream that is still busy (the library's bounded
  wait self-test keeps it busy for 200 ms) with a 20 ms limit must give up, abort the
  communicator and return HI3D_ERR_NCCL; the aborted communicator then refuses work.  A wait
  on finished work returns OK.
* Two GPUs: rank 1 runs one sharded-attention step, then leaves between steps (no kernel or
  collective in flight).  Rank 0 learns of it on the host through a TCP store before its next
  launch, aborts the communicator, and the next ``sharded_attention`` raises instead of
  launching a collective that would wait for the missing peer.

NVLS is off in every process (NCCL_NVLS_ENABLE=0) and the kernels use plain peer copies.
"""

from __future__ import annotations

import ctypes
import datetime
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _comm(lib, uid: bytes, world: int, rank: int):
    from hi3d_b200 import _lib

    handle = ctypes.c_void_p()
    _lib.check(lib.hi3d_nccl_comm_init(ctypes.create_string_buffer(uid, 128), world, rank, ctypes.byref(handle)),
               "nccl_comm_init", launched=False)
    return handle


def _native_attn(lib, handle, q, k, v, world):
    """hi3d_sharded_attn through the C ABI; returns (status, out)."""
    from hi3d_b200 import _lib

    s_rows, heads, d = q.shape
    need = ctypes.c_int64()
    assert lib.hi3d_sharded_attn_workspace_size(handle, s_rows, heads, d, ctypes.byref(need)) == _lib.OK
    ws = torch.empty(need.value, dtype=torch.uint8, device=q.device)
    k_all, v_all = (torch.empty((world * s_rows, heads, d), dtype=q.dtype, device=q.device) for _ in range(2))
    out = torch.empty((s_rows, heads * d), dtype=q.dtype, device=q.device)
    rc = lib.hi3d_sharded_attn(handle, q.data_ptr(), k.data_ptr(), v.data_ptr(), k_all.data_ptr(), v_all.data_ptr(),
                               out.data_ptr(), s_rows, heads, d, d ** -0.5, _lib.F16, ws.data_ptr(), ws.numel(),
                               torch.cuda.current_stream().cuda_stream)
    return rc, out


def test_wait_limit_aborts_the_communicator_on_one_gpu():
    os.environ.setdefault("NCCL_NVLS_ENABLE", "0")
    from hi3d_b200 import _lib, attention

    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    uid = ctypes.create_string_buffer(128)
    _lib.check(lib.hi3d_nccl_unique_id(uid), "nccl_unique_id", launched=False)

    # finished work: the wait returns OK and the single-rank result is the plain attention
    handle = _comm(lib, uid.raw, 1, 0)
    g = torch.Generator(device="cuda").manual_seed(1)
    q, k, v = (torch.randn((1024, 4, 64), generator=g, device="cuda").half() for _ in range(3))
    rc, out = _native_attn(lib, handle, q, k, v, 1)
    assert rc == _lib.OK, lib.hi3d_last_error_string()
    assert lib.hi3d_nccl_comm_wait(handle, stream, 10_000) == _lib.OK
    assert lib.hi3d_nccl_comm_check(handle) == _lib.OK
    bhnd = lambda z: z.permute(1, 0, 2)[None]
    ref = attention.flash_attention(bhnd(q), bhnd(k), bhnd(v), 64 ** -0.5, k_splits=1)[0]
    assert float((out.float() - ref.float()).abs().max()) <= 2 * 2 ** -10 * float(ref.float().abs().max())

    # unfinished work: the stream is held ~200 ms by a bounded wait; a 20 ms limit expires
    _lib.device_status(reset=True)
    assert lib.hi3d_wait_timeout_selftest(200_000_000, stream) == _lib.OK
    assert lib.hi3d_nccl_comm_wait(handle, stream, 20) == _lib.ERR_NCCL
    assert b"communicator aborted" in lib.hi3d_last_error_string()
    assert lib.hi3d_nccl_comm_check(handle) == _lib.ERR_NCCL
    rc, _ = _native_attn(lib, handle, q, k, v, 1)
    assert rc == _lib.ERR_NCCL and b"aborted" in lib.hi3d_last_error_string()
    torch.cuda.synchronize()
    assert _lib.device_status(reset=True)["code"] == _lib.ERR_DEVICE_TIMEOUT  # the self-test's own record
    assert lib.hi3d_nccl_comm_destroy(handle) == _lib.OK
    assert _lib.device_status()["code"] == 0


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _peer_leaves(rank, world, port, result_path):
    sys.path.insert(0, os.path.join(REPO, "hi3dv1.0-mlx_b200"))
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    from hi3d_b200 import _lib

    store = torch.distributed.TCPStore("127.0.0.1", port, world, rank == 0, timeout=datetime.timedelta(seconds=60))
    lib = _lib.load()
    if rank == 0:
        uid = ctypes.create_string_buffer(128)
        _lib.check(lib.hi3d_nccl_unique_id(uid), "nccl_unique_id", launched=False)
        store.set("uid", uid.raw)
    handle = _comm(lib, store.get("uid"), world, rank)
    g = torch.Generator(device="cuda").manual_seed(2 + rank)
    q, k, v = (torch.randn((1024, 4, 64), generator=g, device="cuda").half() for _ in range(3))
    stream = torch.cuda.current_stream().cuda_stream
    rc, _ = _native_attn(lib, handle, q, k, v, world)
    ok_step = rc == _lib.OK and lib.hi3d_nccl_comm_wait(handle, stream, 30_000) == _lib.OK
    torch.cuda.synchronize()
    if rank == 1:
        store.set("left", b"1")  # leaves between steps: nothing of it is in flight
        os._exit(0)
    store.wait(["left"], datetime.timedelta(seconds=60))  # learnt on the host, before the next launch
    assert lib.hi3d_nccl_comm_abort(handle) == _lib.OK
    rc, _ = _native_attn(lib, handle, q, k, v, world)
    refused = rc == _lib.ERR_NCCL and b"aborted" in lib.hi3d_last_error_string()
    np.save(result_path, np.array([ok_step, refused, lib.hi3d_nccl_comm_destroy(handle) == _lib.OK]))
    os._exit(0)


@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_that_leaves_between_steps_is_refused_not_waited_for(tmp_path):
    out = tmp_path / "r.npy"
    mp.spawn(_peer_leaves, args=(2, _free_port(), str(out)), nprocs=2, join=True)
    ok_step, refused, destroyed = np.load(out)
    assert ok_step and refused and destroyed
