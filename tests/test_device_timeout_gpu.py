"""The library's device-side time-out path, made to run out on purpose in the one sanctioned
form: a kernel waits on an mbarrier that nothing arrives at, through the same bounded wait
every kernel of the library uses, with a 1 ms limit instead of 2 s.  The wait must give up,
record HI3D_ERR_DEVICE_TIMEOUT in the status word (site 900) and return, and the context must
stay usable: a following attention launch gives the right answer with a clean status."""

from __future__ import annotations

import numpy as np
import pytest
import torch

from hi3d_b200 import _lib, attention


@pytest.mark.gpu
def test_bounded_wait_reports_timeout_and_the_context_stays_usable():
    lib = _lib.load()
    _lib.device_status(reset=True)
    stream = torch.cuda.current_stream().cuda_stream
    assert lib.hi3d_wait_timeout_selftest(999, stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.hi3d_wait_timeout_selftest(1_000_000, stream) == _lib.OK
    status = _lib.device_status(reset=True)
    assert status["code"] == _lib.ERR_DEVICE_TIMEOUT
    assert status["where"] == 900
    assert _lib.device_status()["code"] == 0

    # the context still runs library kernels correctly
    g = torch.Generator().manual_seed(5)
    q, k, v = (torch.randn(1, 2, 300, 64, generator=g).half().cuda() for _ in range(3))
    out = attention.flash_attention(q, k, v, 64 ** -0.5)
    qf, kf, vf = (t.double().cpu() for t in (q, k, v))
    ref = torch.softmax(qf @ kf.transpose(-1, -2) * 64 ** -0.5, -1) @ vf
    ref = ref.transpose(1, 2).reshape(1, 300, 128)
    err = float((out.double().cpu() - ref).norm() / ref.norm())
    assert err < 3e-4
    assert _lib.device_status()["code"] == 0


@pytest.mark.gpu
def test_peer_barrier_returns_on_arrival_and_reports_a_missing_peer():
    """The cross-GPU barrier of the peer-store gather on one GPU: both entries of the flag
    pointer array name this GPU's own flag words, so "peer" 1 is a word in local memory.  With
    that word already at the epoch the barrier returns at once with a clean status; with a word
    that nothing sets, the 2 ms wait runs out, the status word holds HI3D_ERR_DEVICE_TIMEOUT at
    site 950 naming the peer, and the context stays usable."""
    lib = _lib.load()
    _lib.device_status(reset=True)
    stream = torch.cuda.current_stream().cuda_stream
    flags = torch.zeros(2, dtype=torch.int32, device="cuda")
    ptrs = torch.tensor([flags.data_ptr(), flags.data_ptr()], dtype=torch.int64, device="cuda")
    assert lib.hi3d_peer_barrier(ptrs.data_ptr(), 0, 2, 1, 999, stream) == _lib.ERR_INVALID_ARGUMENT
    assert lib.hi3d_peer_barrier(ptrs.data_ptr(), 2, 2, 1, 2_000_000, stream) == _lib.ERR_INVALID_ARGUMENT

    flags[1] = 7  # the peer's word already at epoch 7
    assert lib.hi3d_peer_barrier(ptrs.data_ptr(), 0, 2, 7, 2_000_000, stream) == _lib.OK
    assert _lib.device_status()["code"] == 0
    assert int(flags[0]) == 7  # this rank's signal landed in the "peer's" word 0

    assert lib.hi3d_peer_barrier(ptrs.data_ptr(), 0, 2, 8, 2_000_000, stream) == _lib.OK  # word 1 stays 7
    status = _lib.device_status(reset=True)
    assert status["code"] == _lib.ERR_DEVICE_TIMEOUT
    assert status["where"] == 950 and status["detail"] == 1
    x = torch.ones(1024, device="cuda")
    assert float(x.sum()) == 1024.0 and _lib.device_status()["code"] == 0
