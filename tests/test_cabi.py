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


def test_kv_cache_entry_points_validate_without_gpu():
    """Compressed KV cache and decode attention: argument errors are answered
    on the host before any launch.  The addresses are fake, so every call here
    either fails validation or has no rows to process: none may launch."""
    L = _lib.load()
    P = ctypes.c_void_p
    A = P(0x100000)  # 256-byte aligned stand-in address
    INT8, TWO, ASYM = 1, 2, 3
    launches = L.pf_kernel_launches()
    assert [L.pf_kv_row_bytes(m, d) for m, d in ((1, 128), (2, 130), (3, 8), (0, 16), (4, 8), (1, 0))] == \
        [128, 33, 2, 64, 0, 0]
    q = L.pf_kv_quantize
    assert q(None, 4, 64, INT8, A, A, None, None) == _lib.ERR_INVALID_ARGUMENT
    assert q(A, 4, 64, 0, A, A, None, None) == _lib.ERR_INVALID_ARGUMENT        # fp32 is not a quantizer mode
    assert q(A, 4, 64, ASYM, A, A, None, None) == _lib.ERR_INVALID_ARGUMENT     # 2bit_asym needs zeros
    assert q(A, 4, 0, TWO, A, A, None, None) == _lib.ERR_SHAPE
    assert q(P(0x100001), 4, 64, INT8, A, A, None, None) == _lib.ERR_ALIGNMENT
    assert q(A, 0, 64, INT8, A, A, None, None) == _lib.OK                       # nothing to do, nothing launched
    dq = L.pf_kv_dequantize
    assert dq(A, A, None, 4, 64, ASYM, A, None) == _lib.ERR_INVALID_ARGUMENT
    assert dq(A, P(0x100002), None, 4, 64, INT8, A, None) == _lib.ERR_ALIGNMENT
    assert dq(A, A, None, 0, 64, TWO, A, None) == _lib.OK
    r = L.pf_rope_kv_compressed
    args = lambda hd, mode, pos=A: (A, A, A, A, A, A, A, A, A, pos, A, 8, 2, hd, 64, mode, None)  # noqa: E731
    assert r(*args(128, 9)) == _lib.ERR_INVALID_ARGUMENT
    assert r(*args(127, INT8)) == _lib.ERR_SHAPE                                # odd head_dim
    assert r(*args(4096, INT8)) == _lib.ERR_SHAPE
    assert r(*args(128, INT8, P(0x100004))) == _lib.ERR_ALIGNMENT               # pos is an int64
    ws = L.pf_decode_attention_workspace_size(8, 128, 64)
    assert ws == 8 * 1 * 130 * 4
    att = L.pf_decode_attention_compressed

    def run(nh=8, nkv=2, hd=128, ms=64, mode=INT8, kc=A, wsb=ws):
        return att(A, kc, A, A, A, A, A, A, A, nh, nkv, hd, ms, mode, 0.1, A, wsb, None)

    assert run(hd=126) == _lib.ERR_SHAPE                                        # head_dim % 4
    assert run(hd=132) == _lib.ERR_SHAPE                                        # head_dim > 128
    assert run(nh=9, nkv=1) == _lib.ERR_SHAPE                                   # > 8 query heads per KV head
    assert run(ms=40000) == _lib.ERR_SHAPE
    assert run(mode=0) == _lib.ERR_INVALID_ARGUMENT
    assert run(kc=P(0x100002)) == _lib.ERR_ALIGNMENT                            # int8 rows are read as words
    assert run(kc=P(0x100002), mode=TWO, wsb=ws - 4) == _lib.ERR_WORKSPACE      # 2-bit codes: byte reads
    assert run(wsb=ws - 4) == _lib.ERR_WORKSPACE
    fp = L.pf_decode_attention
    assert fp(A, P(0x100008), A, A, A, 8, 2, 128, 64, 0.1, A, ws, None) == _lib.ERR_ALIGNMENT  # float4 rows
    assert fp(A, A, A, A, A, 8, 2, 128, 64, 0.1, A, ws - 1, None) == _lib.ERR_WORKSPACE
    assert L.pf_kernel_launches() == launches


def test_status_entry_points_validate_on_the_host():
    """pf_wait_selftest and pf_workspace_status refuse bad arguments before
    touching the device."""
    L = _lib.load()
    st = ctypes.c_int(0)
    assert L.pf_workspace_status(None, 0, ctypes.byref(st), None, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_workspace_status(0x10000, 0, None, None, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_workspace_status(0x10010, 0, ctypes.byref(st), None, None) == _lib.ERR_ALIGNMENT
    assert L.pf_wait_selftest(None, 1000, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_wait_selftest(0x10000, 0, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_wait_selftest(0x10000, 3_000_000_000, None) == _lib.ERR_INVALID_ARGUMENT  # above the 2 s limit
    assert L.pf_wait_selftest(0x10010, 1000, None) == _lib.ERR_ALIGNMENT
    assert L.pf_qlinear_noalloc_status(0, None, None, None) == _lib.ERR_INVALID_ARGUMENT


def test_gather_entry_points_validate_on_the_host():
    """pf_qlinear_group_gather, pf_peers_wait and pf_allgather_rows refuse bad
    peer sets, sizes and alignments before touching the device."""
    L = _lib.load()
    peers = _lib.PFPeers()
    peers.world, peers.rank, peers.bytes = 2, 0, 1 << 20
    peers.bases[0], peers.bases[1] = 0x100000, 0x200000
    d = _desc(fmt=_lib.FMT_INT3_G128, M=128, K=512)
    arr = (ctypes.POINTER(_lib.PFQWeight) * 1)(ctypes.pointer(d))
    xs = (ctypes.c_void_p * 1)(0x300000)
    offs = (ctypes.c_size_t * 1)(256)
    mfull = (ctypes.c_int * 1)(256)
    call = lambda p, o=offs, m=mfull: L.pf_qlinear_group_gather(1, arr, xs, 1, 1, None, o, m, ctypes.byref(p),  # noqa: E731
                                                                  0x400000, 1 << 20, None)
    assert call(peers, m=(ctypes.c_int * 1)(200)) == _lib.ERR_SHAPE          # m_full != world * M
    assert call(peers, o=(ctypes.c_size_t * 1)(64)) == _lib.ERR_ALIGNMENT    # inside the header
    assert call(peers, o=(ctypes.c_size_t * 1)(1 << 20)) == _lib.ERR_SHAPE   # past the buffer
    bad = _lib.PFPeers()
    bad.world, bad.rank, bad.bytes = 9, 0, 1 << 20
    assert call(bad) == _lib.ERR_INVALID_ARGUMENT
    bad.world, bad.rank = 2, 2
    assert call(bad) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_peers_wait(ctypes.byref(bad), 0x400000, None) == _lib.ERR_INVALID_ARGUMENT
    assert L.pf_peers_wait(ctypes.byref(peers), None, None) == _lib.ERR_INVALID_ARGUMENT
    # pf_allgather_rows: the same peer-set checks, then sizes and alignments
    ag = lambda p, src=0x500000, nb=4096, off=256: L.pf_allgather_rows(ctypes.byref(p), src, nb, off,  # noqa: E731
                                                                       0x400000, None)
    assert ag(bad) == _lib.ERR_INVALID_ARGUMENT
    assert ag(peers, off=64) == _lib.ERR_SHAPE            # inside the header
    assert ag(peers, nb=1 << 20) == _lib.ERR_SHAPE        # world x bytes past the buffer
    assert ag(peers, nb=0) == _lib.ERR_SHAPE
    assert ag(peers, nb=4100) == _lib.ERR_ALIGNMENT       # not whole 16-byte words
    assert ag(peers, src=0x500004) == _lib.ERR_ALIGNMENT
    assert L.pf_allgather_rows(ctypes.byref(peers), None, 4096, 256, 0x400000, None) == _lib.ERR_INVALID_ARGUMENT
