"""GPU parity of the tensor-core dequant-GEMM (batches of more than 16 tokens,
group-128 INT4/INT3/INT2 and E8 RVQ2): y against the oracle's fp32 decode and
double-accumulated matmul, normwise within 1e-3 (the GEMM multiplies fp16
dequantised weights by fp16 x' scaled per token, accumulating in fp32).
Cases cover partial 128-row and 128-token tiles, several token chunks,
rotation blocks 128 and 512, every x dtype, and bias."""
import pytest
import torch

import oracle
from test_gpu_parity import _g128_qweight, _w, _x, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import polarflash_b200  # noqa: F401
    torch.cuda.init()


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("M,K,N,hb,xdt", [
    (256, 1024, 64, 128, torch.float16), (200, 512, 33, 128, torch.bfloat16), (384, 2048, 17, 512, torch.float32),
    (1024, 4096, 300, 128, torch.float16), (128, 1024, 600, 128, torch.float16),
])
def test_int_g128_gemm_matches_oracle(bits, M, K, N, hb, xdt):
    from polarflash_b200 import qlinear

    qw, pay, _ = _g128_qweight(_w(M, K, 3 * bits + N), bits, hb=hb)
    x = _x(N, K, 17 + N, xdt)
    bias = torch.randn(M, generator=torch.Generator().manual_seed(5)) * 0.1
    y = qlinear(qw, x.cuda(), bias.cuda()).cpu().numpy()
    meta = {"hadamard_rotation": True, "hadamard_block_size": hb}
    assert_rel(y, oracle.linear(f"int{bits}_g128", pay, M, K, meta, x.float().numpy(), bias.numpy()))


@pytest.mark.parametrize("M,K,N", [(256, 1024, 64), (130, 512, 100), (2048, 8192, 64)])
def test_e8_gemm_matches_oracle(M, K, N):
    from polarflash_b200 import qlinear
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight
    from polarflash_b200.quantizer import rwht_cpu

    W = _w(M, K, 41, std=0.015)
    Wr = rwht_cpu(W, 128).numpy()
    idx, sc = oracle.e8_encode(Wr)
    dev = torch.device("cuda")
    qw = QWeight(7, M, K, torch.from_numpy(idx.reshape(-1).copy()).to(dev), torch.from_numpy(sc.copy()).to(dev),
                 None, effective_block(128, K), column_signs(K, 128, dev))
    x = _x(N, K, 23)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    assert_rel(y, oracle.linear("e8_rvq2_g128", {"idx": idx, "scales": sc}, M, K, meta, x.float().numpy()))


def test_gemm_linearity_and_status_word():
    """Size-independent check at a gate-projection shape: y(a x1 + b x2) =
    a y(x1) + b y(x2), and the device status word stays clear."""
    from polarflash_b200 import UnifiedQuantizer, qlinear
    from polarflash_b200.qweight import workspace

    M, K, N = 14336, 4096, 128
    qw, _ = UnifiedQuantizer(backend="int3_g128", hadamard_block_size=128).quantize_to_qweight(_w(M, K, 9).cuda())
    x1, x2 = _x(N, K, 1).cuda().float(), _x(N, K, 2).cuda().float()
    lhs = qlinear(qw, 0.5 * x1 + 2.0 * x2)
    rhs = 0.5 * qlinear(qw, x1) + 2.0 * qlinear(qw, x2)
    assert_rel(lhs.cpu().numpy(), rhs.cpu().numpy(), rel=2e-3)
    torch.cuda.synchronize()
    head = workspace(torch.device("cuda"), 1)[: 16384 * 4].view(torch.int32)
    assert int(head.abs().sum()) == 0


@pytest.mark.parametrize("hb", [0, 64, 128, 256, 512])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16, torch.float32])
def test_prep_paths_bit_identical(hb, xdt):
    """The x' preparation with in-register butterflies (16-byte aligned x) and
    the shared-memory one (x one element off alignment) give the same y to
    the bit, for every rotation block the register kernel takes."""
    from polarflash_b200 import qlinear

    M, K, N = 300, 2048, 40
    qw, pay, _ = _g128_qweight(_w(M, K, 70 + hb), 3, hb=hb)
    x = _x(N, K, 71 + hb, xdt).cuda()
    buf = torch.zeros(N * K + 1, dtype=xdt, device="cuda")
    xm = buf[1:].view(N, K)
    xm.copy_(x)
    assert x.data_ptr() % 16 == 0 and xm.data_ptr() % 16 != 0
    y = qlinear(qw, x)
    assert torch.equal(y, qlinear(qw, xm))
    meta = {"hadamard_rotation": bool(hb), "hadamard_block_size": hb}
    assert_rel(y.cpu().numpy(), oracle.linear("int3_g128", pay, M, K, meta, x.float().cpu().numpy()))


def test_split_tiles_deterministic():
    """Stream-K: 3000 rows x 600 tokens over K = 2048 is 24 x 3 tiles of 16
    groups split across the CTAs; repeated calls give identical bits, and y
    matches the oracle on a slice of rows."""
    from polarflash_b200 import qlinear

    M, K, N = 3000, 2048, 600
    qw, pay, _ = _g128_qweight(_w(M, K, 81), 2, hb=128)
    x = _x(N, K, 82).cuda()
    y0 = qlinear(qw, x)
    for _ in range(3):
        assert torch.equal(qlinear(qw, x), y0)
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    ref = oracle.linear("int2_g128", pay, M, K, meta, x[:64].float().cpu().numpy())
    assert_rel(y0[:64].cpu().numpy(), ref)


@pytest.mark.parametrize("M,N", [(200, 129), (200, 257), (712, 300), (130, 600)])
def test_two_sm_pair_edges(M, N):
    """Batches above 128 tokens run on two-SM pairs (256-row tiles, each CTA
    holding 128 rows and half of the 256-token x' tile): a pair tile only
    partly inside M (the second CTA's rows partly or wholly past M), a token
    tile whose second half is nearly empty (N = 129) or a second token tile
    of one token (N = 257).  y matches the oracle and repeats bit for bit."""
    from polarflash_b200 import qlinear

    K = 2048
    qw, pay, _ = _g128_qweight(_w(M, K, 90 + M + N), 3, hb=128)
    x = _x(N, K, 91 + N).cuda()
    y = qlinear(qw, x)
    assert torch.equal(qlinear(qw, x), y)
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    assert_rel(y.cpu().numpy(), oracle.linear("int3_g128", pay, M, K, meta, x.float().cpu().numpy()))


def test_two_sm_pair_e8():
    """E8 RVQ2 on two-SM pairs: 300 rows x 2048 columns at 200 tokens."""
    from polarflash_b200 import qlinear
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight
    from polarflash_b200.quantizer import rwht_cpu

    M, K, N = 300, 2048, 200
    W = _w(M, K, 93, std=0.015)
    idx, sc = oracle.e8_encode(rwht_cpu(W, 128).numpy())
    dev = torch.device("cuda")
    qw = QWeight(7, M, K, torch.from_numpy(idx.reshape(-1).copy()).to(dev), torch.from_numpy(sc.copy()).to(dev),
                 None, effective_block(128, K), column_signs(K, 128, dev))
    x = _x(N, K, 94)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    assert_rel(y, oracle.linear("e8_rvq2_g128", {"idx": idx, "scales": sc}, M, K, meta, x.float().numpy()))
