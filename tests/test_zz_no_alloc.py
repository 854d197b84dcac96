"""pf_qlinear_noalloc: the fused linear for callers that cannot allocate.

Some hosts of the library (an engine plugin's enqueue step, a runtime that
owns a fixed memory pool, code that must not touch the caching allocator)
cannot provide a workspace.  This entry point runs the same kernels on a
fixed scratch array inside the library.  The test calls it through the C ABI
twice in a row with different inputs and checks each result against the
workspace-taking entry point (pf_qlinear) within the library's output
tolerance (1e-3 normwise), and checks that an oversized request is refused.
This file is collected last so a stop-at-first-failure run has already run
every other test; it also passes alone in a fresh process (the first call
does the per-device set-up).
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _lib():
    from polarflash_b200 import _lib

    L = _lib.load()
    L.pf_qlinear_noalloc.restype = ctypes.c_int
    L.pf_qlinear_noalloc.argtypes = [ctypes.POINTER(_lib.PFQWeight), ctypes.c_void_p, ctypes.c_int, ctypes.c_int,
                                     ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p]
    L.pf_qlinear_noalloc_status.restype = ctypes.c_int
    L.pf_qlinear_noalloc_status.argtypes = [ctypes.c_int, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_int),
                                            ctypes.c_void_p]
    return L


def _close(y, ref, rel=1e-3):
    err = float((y - ref).abs().max())
    scale = float(ref.abs().max())
    assert err <= rel * scale + 1e-7, f"max err {err} vs {rel} * {scale}"


# The last case is a 48-token batch: the tensor-core GEMM, which in the fixed
# scratch runs without the stream-K partial tiles pf_qlinear's workspace holds.
@pytest.mark.parametrize("fmt,M,K,N", [("int3_g128", 4096, 4096, 1), ("int2_g128", 14336, 4096, 5),
                                       ("int4_g128", 1024, 14336, 16), ("int3_g128", 2048, 4096, 48)])
def test_noalloc_matches_workspace_entry_point_twice(fmt, M, K, N):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from polarflash_b200 import UnifiedQuantizer, qlinear

    L = _lib()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(M + K + N)
    W = torch.randn(M, K, generator=g, device=dev) * 0.02
    qw, _ = UnifiedQuantizer(backend=fmt, hadamard_block_size=128).quantize_to_qweight(W)
    stream = torch.cuda.current_stream(dev)
    for call in range(2):
        x = torch.randn(N, K, generator=g, device=dev).half()
        bias = torch.randn(M, generator=g, device=dev)
        y = torch.empty(N, M, dtype=torch.float32, device=dev)
        st = L.pf_qlinear_noalloc(ctypes.byref(qw.descriptor()), ctypes.c_void_p(x.data_ptr()), 1, N,
                                  ctypes.c_void_p(bias.data_ptr()), ctypes.c_void_p(y.data_ptr()),
                                  ctypes.c_void_p(stream.cuda_stream))
        assert st == 0, L.pf_status_string(st)
        ref = qlinear(qw, x, bias)
        torch.cuda.synchronize()
        _close(y, ref)
    assert _noalloc_status() == (0, 0)  # status word clear, every arrival counter back at zero


def _noalloc_status():
    L = _lib()
    st, busy = ctypes.c_int(-1), ctypes.c_int(-1)
    rc = L.pf_qlinear_noalloc_status(0, ctypes.byref(st), ctypes.byref(busy),
                                     ctypes.c_void_p(torch.cuda.current_stream().cuda_stream))
    assert rc == 0, L.pf_status_string(rc)
    return st.value, busy.value


def _call(L, qw, x, N, bias, y):
    stream = torch.cuda.current_stream()
    return L.pf_qlinear_noalloc(ctypes.byref(qw.descriptor()), ctypes.c_void_p(x.data_ptr()), 1, N,
                                ctypes.c_void_p(bias.data_ptr()) if bias is not None else None,
                                ctypes.c_void_p(y.data_ptr()), ctypes.c_void_p(stream.cuda_stream))


# The paths whose scratch use differs from the INT streaming GEMV: the E8
# table GEMV (batch 1) and tensor-core GEMM (batch 3), the block-8 polar
# table GEMV, and an INT3 input only 2-byte aligned, which takes the
# register-prefetch GEMV and its split-K arrival counters.
@pytest.mark.parametrize("case", ["e8_n1", "e8_n3", "polar8_n1", "int3_misaligned"])
def test_noalloc_other_paths_twice_and_counters_clear(case):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from polarflash_b200 import encoders, qlinear
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.qweight import QWeight
    from polarflash_b200 import UnifiedQuantizer

    L = _lib()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(17)
    M, K = 1536, 2048
    W = torch.randn(M, K, generator=g, device=dev) * 0.02
    N = 3 if case == "e8_n3" else 1
    if case.startswith("e8"):
        idx, sc = encoders.e8_encode(BlockHadamardTransform(K, 128, device=dev).forward(W))
        qw = QWeight(7, M, K, idx.reshape(-1), sc, None, effective_block(128, K), column_signs(K, 128, dev))
    elif case == "polar8_n1":
        payload, meta = encoders.polar_encode(BlockHadamardTransform(K, 128, device=dev).forward(W), 8, 1.75)
        qw = QWeight(8, M, K, payload, None, None, effective_block(128, K), column_signs(K, 128, dev),
                     meta["r_scale"], [8] + meta["alloc"])
    else:
        qw, _ = UnifiedQuantizer(backend="int3_g128", hadamard_block_size=128).quantize_to_qweight(W)
    for call in range(2):
        x = torch.randn(N, K, generator=g, device=dev).half()
        if case == "int3_misaligned":
            buf = torch.zeros(N * K + 1, dtype=torch.float16, device=dev)
            xm = buf[1:].view(N, K)
            xm.copy_(x)
            assert xm.data_ptr() % 8 != 0
            x = xm
        bias = torch.randn(M, generator=g, device=dev)
        y = torch.empty(N, M, dtype=torch.float32, device=dev)
        st = _call(L, qw, x, N, bias, y)
        assert st == 0, L.pf_status_string(st)
        ref = qlinear(qw, x, bias)
        torch.cuda.synchronize()
        _close(y, ref)
        assert _noalloc_status() == (0, 0)


def test_noalloc_rejects_requests_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from polarflash_b200 import _lib as plib
    from polarflash_b200.qweight import QWeight

    L = _lib()
    dev = torch.device("cuda")
    # E8 scratch is N * K * 4 bytes of prepared activations: K = 262144 at
    # N = 16 needs 16 MiB, more than the 8 MiB array.
    M, K, N = 16, 262144, 16
    qw = QWeight(plib.FMT_E8_RVQ2_G128, M, K, torch.zeros(M * K // 4, dtype=torch.uint8, device=dev),
                 torch.zeros(M, K // 128, 2, dtype=torch.float16, device=dev))
    x = torch.zeros(N, K, dtype=torch.float16, device=dev)
    y = torch.empty(N, M, dtype=torch.float32, device=dev)
    st = L.pf_qlinear_noalloc(ctypes.byref(qw.descriptor()), ctypes.c_void_p(x.data_ptr()), 1, N, None,
                              ctypes.c_void_p(y.data_ptr()),
                              ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream))
    assert st == plib.ERR_WORKSPACE
