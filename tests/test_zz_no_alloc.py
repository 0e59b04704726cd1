"""The neighbour map built without any device allocation, checked against the workspace form.

``hi3d_neighbour_map_build_noalloc`` serves callers that cannot allocate device memory (a host
whose memory pool already owns the GPU's memory, a plain C host with no allocator, a caller
that cannot take cudaMalloc's device-wide synchronisation).  Its hash table lives in a fixed
array inside the library that every call reuses, so these tests make two calls in a row, the
second smaller than the first, and check that each gives exactly the table that
``hi3d_neighbour_map_build`` gives from a fresh workspace (index work: bit-exact).

This file sorts last so that a ``-x`` run has already run every other test if it fails.
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest
import torch

from hi3d_b200 import _lib, synthetic

MAX_VOXELS = 262144  # HI3D_NEIGHBOUR_MAP_NOALLOC_MAX_VOXELS in include/hi3d_b200.h


def _with_workspace(lib, coords, query, stride, stream):
    n = coords.shape[0]
    nq = n if query is None else query.shape[0]
    need = ctypes.c_int64()
    assert lib.hi3d_neighbour_map_workspace_size(n, ctypes.byref(need)) == _lib.OK
    ws = torch.empty(need.value, dtype=torch.uint8, device="cuda")
    table = torch.full((nq, 27), -7, dtype=torch.int32, device="cuda")
    rc = lib.hi3d_neighbour_map_build(coords.data_ptr(), n, _lib.ptr(query), nq, stride, table.data_ptr(),
                                      ws.data_ptr(), ws.numel(), stream)
    assert rc == _lib.OK, lib.hi3d_last_error_string()
    return table


def _no_alloc(lib, coords, query, stride, stream):
    n = coords.shape[0]
    nq = n if query is None else query.shape[0]
    table = torch.full((nq, 27), -7, dtype=torch.int32, device="cuda")
    rc = lib.hi3d_neighbour_map_build_noalloc(coords.data_ptr(), n, _lib.ptr(query), nq, stride,
                                              table.data_ptr(), stream)
    assert rc == _lib.OK, lib.hi3d_last_error_string()
    return table


@pytest.mark.gpu
def test_noalloc_neighbour_map_matches_workspace_form_on_consecutive_calls():
    lib = _lib.load()
    stream = torch.cuda.current_stream().cuda_stream
    # call 1: the full limit, submanifold (stride 1) self-query
    big = torch.from_numpy(synthetic.shell_coords(MAX_VOXELS, 160, 60, 6, seed=31)).cuda()
    # call 2: a smaller, different set with duplicate rows (last row wins), queried at stride 2
    # from its downsampled coordinates; stale entries of call 1 would show up as wrong rows
    small_np = synthetic.shell_coords(5000, 64, 24, 3, seed=32)
    small_np = np.concatenate([small_np, small_np[::97]])
    small = torch.from_numpy(small_np).cuda()
    low = torch.from_numpy(np.unique(small_np // 2, axis=0).astype(np.int32)).cuda()
    cases = [(big, None, 1), (small, low, 2)]

    got = [_no_alloc(lib, c, q, s, stream) for c, q, s in cases]
    want = [_with_workspace(lib, c, q, s, stream) for c, q, s in cases]
    torch.cuda.synchronize()
    for (c, _, _), g, w in zip(cases, got, want):
        assert torch.equal(g, w)
        n = c.shape[0]
        assert int((g < n).sum()) > g.shape[0]  # every voxel sees itself plus neighbours
    assert _lib.device_status()["code"] == 0


@pytest.mark.gpu
def test_noalloc_neighbour_map_rejects_more_voxels_than_its_scratch_holds():
    lib = _lib.load()
    coords = torch.zeros((MAX_VOXELS + 1, 3), dtype=torch.int32, device="cuda")
    table = torch.empty((1, 27), dtype=torch.int32, device="cuda")
    rc = lib.hi3d_neighbour_map_build_noalloc(coords.data_ptr(), MAX_VOXELS + 1, None, 0, 1, table.data_ptr(),
                                              torch.cuda.current_stream().cuda_stream)
    assert rc == _lib.ERR_CAPACITY
    assert b"scratch limit" in lib.hi3d_last_error_string()
