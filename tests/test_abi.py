"""C-ABI checks that need no GPU: the library loads, exports every declared entry
point, and rejects bad arguments with the documented status before touching CUDA."""

from __future__ import annotations

import ctypes
import re

import pytest
from conftest import REPO

from hi3d_b200 import _lib

HEADER = REPO / "include" / "hi3d_b200.h"


def declared_symbols() -> set[str]:
    text = HEADER.read_text()
    return set(re.findall(r"HI3D_API\s+[\w\s\*]+?\b(hi3d_\w+)\s*\(", text))


def test_library_exports_every_declared_symbol():
    lib = _lib.load()
    names = declared_symbols()
    assert len(names) >= 8
    for name in names:
        assert hasattr(lib, name), name


def test_python_binding_covers_every_declared_symbol():
    assert declared_symbols() == set(_lib.SIGNATURES)


def test_version():
    assert _lib.load().hi3d_version() >= 100


def test_invalid_arguments_are_rejected_without_a_gpu():
    lib = _lib.load()
    rc = lib.hi3d_layer_norm_modulate(None, None, 4, 256, 1e-6, None, None, None, None, 0, 0, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    assert b"layer_norm_modulate" in lib.hi3d_last_error_string()
    rc = lib.hi3d_qkv_rope_rms(*([None] * 8), 1, 4, 2, 63, 0, 0, None)
    assert rc == _lib.ERR_INVALID_ARGUMENT
    args = _lib.AttnArgs(head_dim=64, dtype=0)
    assert lib.hi3d_flash_attn_fwd(ctypes.byref(args), None) == _lib.ERR_INVALID_ARGUMENT
    args = _lib.AttnArgs(q=16, k=16, v=16, out=16, head_dim=80, dtype=0, heads=1, num_seqs=1, nq=1, nk=1)
    assert lib.hi3d_flash_attn_fwd(ctypes.byref(args), None) == _lib.ERR_UNSUPPORTED
    assert lib.hi3d_gelu_tanh(None, None, 7, 0, None) == _lib.ERR_INVALID_ARGUMENT


def test_check_maps_status_to_reference_exceptions():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_INVALID_ARGUMENT, "x")
    with pytest.raises(NotImplementedError):
        _lib.check(_lib.ERR_UNSUPPORTED, "x")
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA, "x")
