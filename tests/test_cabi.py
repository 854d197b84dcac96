"""The C-ABI library loads and exports every symbol include/polarflash_b200.h
declares; host-side validation answers without a GPU (no compute calls)."""
import ctypes
import os
import re

import pytest

from conftest import ROOT
from polarflash_b200 import _lib


def _header_functions():
    src = open(os.path.join(ROOT, "include", "polarflash_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(pf_[a-z0-9_]+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    L = _lib.load()
    declared = _header_functions()
    assert declared, "no functions parsed from the header"
    for name in declared:
        assert hasattr(L, name), f"{name} declared in the header but not exported"
    assert set(declared) == set(_lib.EXPORTS)


def test_version_and_status_strings():
    assert "sm_100a" in _lib.version()
    L = _lib.load()
    for st in range(8):
        assert L.pf_status_string(st)
    assert L.pf_status_string(_lib.OK) == b"ok"


def _desc(fmt=_lib.FMT_INT4_G128, M=64, K=256, codes=0x10000, scales=0x20000, mins=0x30000):
    d = _lib.PFQWeight()
    d.format, d.M, d.K = fmt, M, K
    d.codes, d.scales, d.mins = codes, scales, mins
    return d


def _check(d):
    return _lib.load().pf_qweight_check(ctypes.byref(d))


def test_descriptor_validation_without_gpu():
    assert _check(_desc()) == _lib.OK
    assert _check(_desc(K=200)) == _lib.ERR_SHAPE                    # K % 128
    assert _check(_desc(codes=0x10004)) == _lib.ERR_ALIGNMENT         # INT4 words need 16 B
    assert _check(_desc(mins=0)) == _lib.ERR_INVALID_ARGUMENT         # group format needs mins
    assert _check(_desc(fmt=99)) == _lib.ERR_INVALID_ARGUMENT
    assert _check(_desc(M=0)) == _lib.ERR_SHAPE
    d = _desc()
    d.had_block = 128
    assert _check(d) == _lib.ERR_INVALID_ARGUMENT                     # rotation without signs
    d.had_signs = 0x40000
    assert _check(d) == _lib.OK
    d.had_block = 96
    assert _check(d) == _lib.ERR_UNSUPPORTED                          # not a power of two
    # reference INT streams need K % 32
    assert _check(_desc(fmt=_lib.FMT_INT3, K=48, scales=0, mins=0)) == _lib.ERR_SHAPE
    assert _check(_desc(fmt=_lib.FMT_INT3, K=64, scales=0, mins=0)) == _lib.OK
    # polar: block size 8, 14-bit alloc, K rows must be whole bytes
    p = _desc(fmt=_lib.FMT_POLAR_RECURSIVE, K=4096, scales=0, mins=0)
    for i, v in enumerate([8, 3, 2, 2, 2, 2, 1, 1, 1]):
        p.params[i] = v
    assert _check(p) == _lib.OK
    p.K = 4104  # 513 blocks * 14 bits is not whole bytes
    assert _check(p) == _lib.ERR_SHAPE


def test_workspace_size_query():
    L = _lib.load()
    n = ctypes.c_size_t(0)
    d = _desc(M=4096, K=4096)
    assert L.pf_qlinear_workspace_size(ctypes.byref(d), 1, ctypes.byref(n)) == _lib.OK
    assert n.value >= 32 * 2048  # one n8 tile of B fragments per 128-column group
    assert L.pf_qlinear_workspace_size(ctypes.byref(d), -1, ctypes.byref(n)) == _lib.ERR_INVALID_ARGUMENT


def test_python_status_mapping():
    with pytest.raises(ValueError):
        _lib.check(_lib.ERR_SHAPE)
    with pytest.raises(RuntimeError):
        _lib.check(_lib.ERR_CUDA)
    _lib.check(_lib.OK)
