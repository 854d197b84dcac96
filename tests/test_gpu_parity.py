"""GPU parity: the CUDA library (through its C ABI) against the oracle and the
reference's own outputs.

Tolerances: codes and E8 indices bit-exact; decoded weights within 1e-5
absolute of the oracle's fp32 decode; outputs y within 1e-3 relative, measured
normwise:  max|y - y_ref| <= 1e-3 * max|y_ref|  (y_ref from the reference /
oracle fp32 path, accumulated in double by the oracle).
"""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN

pytestmark = pytest.mark.gpu

REL = 1e-3


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import polarflash_b200  # noqa: F401  (loads the library; fails loudly if not built)
    torch.cuda.init()


def assert_rel(y, ref, rel=REL):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    assert y.shape == ref.shape, (y.shape, ref.shape)
    err = np.max(np.abs(y - ref)) if y.size else 0.0
    scale = np.max(np.abs(ref)) if ref.size else 0.0
    assert err <= rel * scale + 1e-7, f"max err {err:.3e} vs {rel} * {scale:.3e}"


def _w(M, K, seed, std=0.02):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(M, K, generator=g) * std
    n = max(1, int(0.001 * M * K))
    pos = torch.randperm(M * K, generator=g)[:n]
    W.view(-1)[pos] = (torch.randint(0, 2, (n,), generator=g).float() * 2 - 1) * 20 * std
    return W


def _x(N, K, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    return torch.randn(N, K, generator=g).to(dtype)


FMT = {4: 1, 3: 2, 2: 3}


def _g128_qweight(W, bits, hb=128):
    """Oracle-encoded group-128 weight (rotated with block hb) as a device QWeight."""
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight
    from polarflash_b200.quantizer import rwht_cpu

    M, K = W.shape
    Wr = rwht_cpu(W, hb).numpy() if hb else W.numpy()
    q, s, m = oracle.quant_g128_asym(bits, Wr)
    words = oracle.pack_g128(bits, q)
    dev = torch.device("cuda")
    qw = QWeight(FMT[bits], M, K, torch.from_numpy(words.view(np.uint8).reshape(-1).copy()).to(dev),
                 torch.from_numpy(s.copy()).to(dev), torch.from_numpy(m.copy()).to(dev),
                 effective_block(hb, K) if hb else 0, column_signs(K, hb, dev) if hb else None)
    meta = {"hadamard_rotation": bool(hb), "hadamard_block_size": hb}
    payload = {"words": words, "s": s, "m": m}
    return qw, payload, meta


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("M,K,N,xdt", [
    (256, 1024, 1, torch.float16), (256, 1024, 4, torch.float32), (130, 512, 5, torch.bfloat16),
    (96, 256, 8, torch.float16), (64, 384, 13, torch.float16), (1024, 4096, 16, torch.float16),
    (33, 128, 20, torch.float32), (4096, 4096, 1, torch.float16),
])
def test_g128_gemv_matches_oracle(bits, M, K, N, xdt):
    from polarflash_b200 import qlinear

    W = _w(M, K, 100 * bits + M)
    qw, payload, meta = _g128_qweight(W, bits)
    x = _x(N, K, 7 + N, xdt)
    bias = torch.randn(M, generator=torch.Generator().manual_seed(3)) * 0.1
    y = qlinear(qw, x.cuda(), bias.cuda())
    ref = oracle.linear(f"int{bits}_g128", payload, M, K, meta, x.float().numpy(), bias.numpy())
    assert_rel(y.cpu().numpy(), ref)


@pytest.mark.parametrize("bits", [4, 3, 2])
def test_g128_unpack_and_dequant_bit_exact(bits):
    from polarflash_b200 import dequantize, unpack_codes

    W = _w(130, 512, bits)
    qw, payload, meta = _g128_qweight(W, bits)
    codes = unpack_codes(qw).cpu().numpy()
    assert np.array_equal(codes, oracle.unpack_g128(bits, payload["words"], 130, 512))
    Wr = dequantize(qw, inverse_rwht=False).cpu().numpy()
    assert np.array_equal(Wr, oracle.dequant_g128_asym(codes, payload["s"], payload["m"]))
    Wh = dequantize(qw, inverse_rwht=True).cpu().numpy()
    np.testing.assert_allclose(Wh, oracle.dequantize(f"int{bits}_g128", payload, 130, 512, meta), atol=1e-5)


def _unified_cases():
    with open(os.path.join(GOLDEN, "unified_meta.json")) as f:
        return sorted(json.load(f).items())


@pytest.mark.parametrize("key,meta", _unified_cases())
def test_reference_payloads_gemv_and_dequant(key, meta):
    """Payloads written by the reference UnifiedQuantizer (int4/int3/int2 per-tensor,
    2-D polar; RWHT 512 and 128): y against the reference's own y."""
    from polarflash_b200 import dequantize, qlinear, qweight_from_payload, unpack_codes

    g = np.load(os.path.join(GOLDEN, "unified.npz"))
    be, shape, _ = key.split("_")
    M, K = (int(v) for v in shape.split("x"))
    qw = qweight_from_payload(meta["dtype"], meta, g[f"payload_{key}"].tobytes(), M, K, "cuda")
    x = torch.from_numpy(g[f"x_{key}"])
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, g[f"y_{key}"])
    np.testing.assert_allclose(dequantize(qw).cpu().numpy(), g[f"deq_{key}"], atol=1e-5)
    if be in ("int4", "int3", "int2"):
        codes = unpack_codes(qw).cpu().numpy().ravel()
        n = M * K
        p = g[f"payload_{key}"].tobytes()
        ref = {"int4": lambda: oracle.unpack_int4(p, n).astype(np.int16) + 8,
               "int3": lambda: oracle.unpack_int3(p, n), "int2": lambda: oracle.unpack_int2(p, n)}[be]()
        assert np.array_equal(codes.astype(np.int16), np.asarray(ref, np.int16))


def _polar_cases():
    with open(os.path.join(GOLDEN, "polar_recursive_meta.json")) as f:
        meta = json.load(f)
    meta.pop("_allocs")
    return sorted(meta.items())


@pytest.mark.parametrize("key,meta", _polar_cases())
@pytest.mark.parametrize("N", [1, 3])
def test_polar_recursive_gemv(key, meta, N):
    from polarflash_b200 import dequantize, qlinear, qweight_from_payload

    g = np.load(os.path.join(GOLDEN, "polar_recursive.npz"))
    W = g[f"W_{key}"]
    M, K = W.shape
    qm = dict(meta)
    if meta["rotated"]:
        qm.update(hadamard_rotation=True, hadamard_block_size=128)
    qw = qweight_from_payload("polar_recursive", qm, g[f"packed_{key}"].tobytes(), M, K, "cuda")
    x = _x(N, K, 5).float()
    y = qlinear(qw, x.cuda()).cpu().numpy()
    Wh = oracle.dequantize("polar_recursive", g[f"packed_{key}"].tobytes(), M, K, qm)
    assert_rel(y, oracle.matvec(Wh, x.numpy()))
    dec = dequantize(qw, inverse_rwht=False).cpu().numpy()
    np.testing.assert_allclose(dec, g[f"dec_{key}"], atol=1e-6)


@pytest.mark.parametrize("M,K,N", [(256, 1024, 1), (130, 512, 8), (64, 256, 16)])
def test_e8_gemv_matches_oracle(M, K, N):
    from polarflash_b200 import dequantize, qlinear, unpack_codes
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight
    from polarflash_b200.quantizer import rwht_cpu

    W = _w(M, K, 31, std=0.015)
    Wr = rwht_cpu(W, 128).numpy()
    idx, sc = oracle.e8_encode(Wr)
    dev = torch.device("cuda")
    qw = QWeight(7, M, K, torch.from_numpy(idx.reshape(-1).copy()).to(dev),
                 torch.from_numpy(sc.copy()).to(dev), None, effective_block(128, K), column_signs(K, 128, dev))
    x = _x(N, K, 9)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    ref = oracle.linear("e8_rvq2_g128", {"idx": idx, "scales": sc}, M, K, meta, x.float().numpy())
    assert_rel(y, ref)
    assert np.array_equal(unpack_codes(qw).cpu().numpy(), idx)
    np.testing.assert_array_equal(dequantize(qw, inverse_rwht=False).cpu().numpy(), oracle.e8_decode(idx, sc, M, K))


def test_native_engine_matches_reference():
    """NativeLowBitCUDAEngine ops on the reference tests' own seeded shapes
    (test_native_cuda_kernels.py:15-92): max abs diff < 1e-4."""
    from polarflash_b200 import NativeLowBitCUDAEngine

    g = np.load(os.path.join(GOLDEN, "native.npz"))
    eng = NativeLowBitCUDAEngine.get_instance()
    assert eng.is_available
    c = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    y4 = eng.gemv_int4(c(g["i4_x"]), c(g["i4_packed"]), c(g["i4_scales"]), 64, 128)
    assert np.max(np.abs(y4.cpu().numpy() - g["i4_y"])) < 1e-4
    y2 = eng.gemv_int2(c(g["i2_x"]), c(g["i2_packed"]), c(g["i2_scales"]), 32, 64)
    assert np.max(np.abs(y2.cpu().numpy() - g["i2_y"])) < 1e-4
    Y = eng.gemm_int4(c(g["g4_X"]), c(g["g4_packed"]), c(g["g4_scales"]), 32, 64)
    assert np.max(np.abs(Y.cpu().numpy() - g["g4_Y"])) < 1e-4


@pytest.mark.parametrize("K,req", [(128, 128), (4096, 128), (500, 512), (11008, 512), (1000, 128), (129, 128)])
def test_device_rwht_matches_reference(K, req):
    from polarflash_b200 import BlockHadamardTransform

    g = np.load(os.path.join(GOLDEN, "hadamard.npz"))
    key = f"{K}_{req}"
    bht = BlockHadamardTransform(K, req)
    x = torch.from_numpy(g[f"x_{key}"]).cuda()
    np.testing.assert_allclose(bht.forward(x).cpu().numpy(), g[f"fwd_{key}"], atol=1e-5)
    np.testing.assert_allclose(bht.inverse(x).cpu().numpy(), g[f"inv_{key}"], atol=1e-5)


def test_engine_over_reference_pflash():
    """PFlashCUDAEngine.forward_layer over a .pflash written by the reference."""
    from polarflash_b200 import PFlashCUDAEngine

    io = np.load(os.path.join(GOLDEN, "small_pflash_io.npz"))
    x = torch.from_numpy(io["x"])
    with PFlashCUDAEngine(os.path.join(GOLDEN, "small.pflash")) as eng:
        yq = eng.forward_layer("model.layers.0.self_attn.q_proj.weight", x).cpu().numpy()
        yu = eng.forward_layer("model.layers.0.mlp.up_proj.weight", x).cpu().numpy()
        assert eng.get_layer("model.layers.0.self_attn.q_proj.weight").is_packed
        with pytest.raises(KeyError):
            eng.get_layer("missing")
    assert_rel(yq, oracle.matvec(io["W_q_hat"], io["x"]))
    assert_rel(yu, oracle.matvec(io["W_up_hat"], io["x"]))


@pytest.mark.parametrize("bits", [4, 3, 2])
def test_gpu_encoders_bit_exact(bits):
    """Product encoders on CUDA tensors reproduce the oracle's codes."""
    from polarflash_b200 import encoders

    W = _w(96, 512, 77 + bits)
    q, s, m = encoders.quant_g128_asym(W.cuda(), bits)
    oq, os_, om = oracle.quant_g128_asym(bits, W.numpy())
    assert np.array_equal(q.cpu().numpy(), oq)
    assert np.array_equal(s.cpu().numpy().view(np.uint16), os_.view(np.uint16))
    assert np.array_equal(m.cpu().numpy().view(np.uint16), om.view(np.uint16))
    words = encoders.pack_g128(q, bits)
    assert np.array_equal(words.cpu().numpy().view(np.uint32), oracle.pack_g128(bits, oq))
    if bits == 2:
        idx, sc = encoders.e8_encode(W.cuda() * 0.75)
        oidx, osc = oracle.e8_encode((W * 0.75).numpy())
        assert np.array_equal(idx.cpu().numpy(), oidx)
        assert np.array_equal(sc.cpu().numpy().view(np.uint16), osc.view(np.uint16))


def test_torch_custom_op_and_layer():
    from polarflash_b200 import PolarLinearLayer, UnifiedQuantizer
    from polarflash_b200.ops import qlinear as op_qlinear

    W = _w(512, 1024, 5)
    uq = UnifiedQuantizer(backend="int4_g128", hadamard_block_size=128)
    payload, meta, w_hat = uq.quantize(W.cuda())
    layer = PolarLinearLayer(1024, 512, meta["dtype"], meta, payload, device="cuda")
    x = _x(3, 1024, 1).cuda()
    y_layer = layer(x)
    y_op = op_qlinear(layer.qweight, x)
    torch.testing.assert_close(y_layer, y_op, rtol=0, atol=0)
    assert_rel(y_layer.cpu().numpy(), oracle.matvec(w_hat.numpy(), x.float().cpu().numpy()))


def test_errors_are_raised_not_fallen_back():
    from polarflash_b200 import UnifiedQuantizer, qlinear

    uq = UnifiedQuantizer(backend="int2_g128", hadamard_block_size=128)
    qw, _ = uq.quantize_to_qweight(_w(64, 256, 1).cuda())
    with pytest.raises(ValueError):
        qlinear(qw, torch.randn(2, 256))            # CPU input: no CPU path
    with pytest.raises(ValueError):
        qlinear(qw, torch.randn(2, 128).cuda())     # wrong K
    with pytest.raises(ValueError):
        uq.quantize_to_qweight(_w(64, 200, 1).cuda())  # K % 128 != 0
    assert qlinear(qw, torch.randn(0, 256).cuda()).shape == (0, 64)


@pytest.mark.parametrize("bits", [3, 2])
def test_full_size_llama8b_ffn_linear(bits):
    """gate/up projection 14336 x 4096 at the benchmark's settings (RWHT 128,
    fp16 x, N = 1 and 16) against the oracle's full decode + matvec; plus the
    size-independent linearity check y(a x1 + b x2) = a y(x1) + b y(x2)."""
    from polarflash_b200 import UnifiedQuantizer, qlinear

    M, K = 14336, 4096
    W = _w(M, K, 1234 + bits)
    uq = UnifiedQuantizer(backend=f"int{bits}_g128", hadamard_block_size=128)
    qw, _ = uq.quantize_to_qweight(W.cuda())
    # the oracle decodes exactly the payload the device holds
    payload = {"words": qw.codes.cpu().numpy().view(np.uint32).reshape(M, -1),
               "s": qw.scales.cpu().numpy(), "m": qw.mins.cpu().numpy()}
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    for N in (1, 16):
        x = _x(N, K, 40 + N)
        y = qlinear(qw, x.cuda()).cpu().numpy()
        assert_rel(y, oracle.linear(f"int{bits}_g128", payload, M, K, meta, x.float().numpy()))
    x1, x2 = _x(1, K, 1).cuda().float(), _x(1, K, 2).cuda().float()
    lhs = qlinear(qw, 0.5 * x1 + 2.0 * x2)
    rhs = 0.5 * qlinear(qw, x1) + 2.0 * qlinear(qw, x2)
    assert_rel(lhs.cpu().numpy(), rhs.cpu().numpy(), rel=1e-5)


def test_workspace_counters_return_to_zero():
    """After a batch of calls (split-K combines on both GEMV paths), every
    arrival counter is re-armed to zero and the device status word is clear."""
    from polarflash_b200 import UnifiedQuantizer, qlinear
    from polarflash_b200.qweight import workspace

    dev = torch.device("cuda")
    for fmt, K in (("int3_g128", 4096), ("int2_g128", 1024), ("int4_g128", 384)):
        qw, _ = UnifiedQuantizer(backend=fmt, hadamard_block_size=128).quantize_to_qweight(_w(2048, K, 3).to(dev))
        for N in (1, 6, 16):
            qlinear(qw, _x(N, K, N).to(dev))
    torch.cuda.synchronize()
    ws = workspace(dev, 1)
    head = ws[: 16384 * 4].view(torch.int32)
    assert int(head.abs().sum()) == 0
