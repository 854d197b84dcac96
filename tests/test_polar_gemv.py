"""GPU parity of recursive polar (block 8, 1.75 bpw: allocation
3 | 2 2 2 2 | 1 1 | 1) on its two fast paths.

* The lookup-table GEMV (batch 1): the kernel folds the radius scale and the
  psi / phi / theta cos-sin tree into two 64-entry tables per x'-vector, so
  these tests cover rotation blocks from none to 512 columns, the three
  activation dtypes, ragged row blocks, a full Llama-3-8B layer shape against
  the CUDA-core kernel, and the inputs and allocations the kernel does not
  take.
* The tcgen05 stream-K GEMM (batches of 2 and more, K a multiple of 512):
  every block decoded into the fp16 A tile from the same cos / sin tables,
  against the reference's own payload and decode_packed output
  (tests/golden/polar_recursive.npz, 128 x 1024) at N = 2 ... 2048, and a
  ragged 1000 x 4096 weight with and without learned angle codebooks.

Tolerance as in test_gpu_parity: y within 1e-3 normwise of the oracle's fp32
decode + double-accumulated matvec.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import oracle
from test_gpu_parity import _w, _x, assert_rel

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import polarflash_b200  # noqa: F401
    torch.cuda.init()


def _polar_qweight(M, K, seed, hb=128, bpw=1.75):
    """Device-encoded recursive-polar weight (rotated with block hb) and the
    metadata the oracle decodes it with."""
    from polarflash_b200 import encoders
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.quantizer import rwht_cpu
    from polarflash_b200.qweight import QWeight

    W = _w(M, K, seed)
    Wr = rwht_cpu(W, hb) if hb else W
    payload, meta = encoders.polar_encode(Wr.cuda(), 8, bpw)
    qw = QWeight(8, M, K, payload, None, None, effective_block(hb, K) if hb else 0,
                 column_signs(K, hb, torch.device("cuda")) if hb else None, meta["r_scale"], [8] + meta["alloc"])
    om = {"block_size": 8, "num_blocks": M * K // 8, "alloc": meta["alloc"], "r_scale": meta["r_scale"],
          "hadamard_rotation": bool(hb), "hadamard_block_size": hb}
    return qw, payload.cpu().numpy().tobytes(), om


def _ref(pay, M, K, meta, x, bias=None):
    return oracle.linear("polar_recursive", pay, M, K, meta, x, bias)


@pytest.mark.parametrize("hb", [0, 64, 128, 256, 512])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16, torch.float32])
def test_rotation_blocks_and_dtypes(hb, xdt):
    from polarflash_b200 import qlinear

    M, K = 1000, 2048
    qw, pay, meta = _polar_qweight(M, K, 13 + hb, hb)
    assert meta["alloc"] == [3, 2, 2, 2, 2, 1, 1, 1]
    x = _x(1, K, 7 + hb, xdt)
    b = torch.randn(M, generator=torch.Generator().manual_seed(hb)) * 0.1
    y = qlinear(qw, x.cuda(), b.cuda()).cpu().numpy()
    assert_rel(y, _ref(pay, M, K, meta, x.float().numpy(), b.numpy()))


@pytest.mark.parametrize("M,K", [(1, 512), (33, 512), (700, 1024), (4096, 14336), (64, 65536)])
def test_shapes(M, K):
    """One stage (no partial sums), one row, a ragged last row block, the down
    projection's K and a long K over one row block."""
    from polarflash_b200 import qlinear

    qw, pay, meta = _polar_qweight(M, K, M + 3)
    x = _x(1, K, 2)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, _ref(pay, M, K, meta, x.float().numpy()))


def test_repeated_calls_bit_identical():
    from polarflash_b200 import qlinear

    qw, _, _ = _polar_qweight(2048, 4096, 5)
    x = _x(1, 4096, 4).cuda()
    y0 = qlinear(qw, x)
    for _ in range(3):
        assert torch.equal(qlinear(qw, x), y0)


def test_other_inputs_take_other_kernels():
    """A 2-byte aligned fp16 x and the 2.0 bpw allocation (3 | 2 2 2 2 | 2 2 |
    1) are served by the CUDA-core kernel, batch 3 by the tensor-core GEMM;
    all agree."""
    from polarflash_b200 import qlinear

    M, K = 256, 1024
    qw, pay, meta = _polar_qweight(M, K, 21)
    x = _x(1, K, 8)
    buf = torch.zeros(K + 1, dtype=torch.float16, device="cuda")
    xm = buf[1:].view(1, K)
    xm.copy_(x.cuda())
    assert xm.data_ptr() % 8 != 0
    assert_rel(qlinear(qw, xm).cpu().numpy(), _ref(pay, M, K, meta, x.float().numpy()))
    x3 = _x(3, K, 9)
    assert_rel(qlinear(qw, x3.cuda()).cpu().numpy(), _ref(pay, M, K, meta, x3.float().numpy()))
    qw2, pay2, meta2 = _polar_qweight(M, K, 22, bpw=2.0)
    assert meta2["alloc"] == [3, 2, 2, 2, 2, 2, 2, 1]
    assert_rel(qlinear(qw2, x.cuda()).cpu().numpy(), _ref(pay2, M, K, meta2, x.float().numpy()))


_FULL_SCRIPT = r"""
import sys, numpy as np, torch
sys.path[:0] = sys.argv[2:]
from polarflash_b200 import encoders, qlinear
from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
from polarflash_b200.qweight import QWeight
M, K = 14336, 4096
dev = torch.device("cuda")
g = torch.Generator().manual_seed(0)
W = (torch.randn(M, K, generator=g) * 0.02).to(dev)
payload, meta = encoders.polar_encode(BlockHadamardTransform(K, 128, device=dev).forward(W), 8, 1.75)
qw = QWeight(8, M, K, payload, None, None, effective_block(128, K), column_signs(K, 128, dev), meta["r_scale"],
             [8] + meta["alloc"])
x = torch.randn(1, K, generator=torch.Generator().manual_seed(1)).half().to(dev)
rows = payload.view(M, -1)[:2048].contiguous().cpu().numpy()
np.savez(sys.argv[1], y=qlinear(qw, x).cpu().numpy(), rows=rows, x=x.float().cpu().numpy(),
         r_scale=np.float64(meta["r_scale"]), alloc=np.array(meta["alloc"]))
"""


def test_full_size_against_cuda_core_kernel(tmp_path):
    """A 14336 x 4096 gate projection at batch 1: the table GEMV (default) and
    the CUDA-core kernel (PF_POLAR_LUT=0) on the same weights, both against the
    oracle on the first 2048 rows, and against each other over all rows."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    paths = [root, os.path.join(root, "polar-flash_b200"), here]
    script = tmp_path / "run.py"
    script.write_text(_FULL_SCRIPT)
    res = {}
    for mode in ("1", "0"):
        out = tmp_path / f"y{mode}.npz"
        subprocess.run([sys.executable, str(script), str(out)] + paths, check=True,
                       env=dict(os.environ, PF_POLAR_LUT=mode), timeout=900)
        res[mode] = np.load(out)
    K, R = 4096, 2048
    meta = {"block_size": 8, "num_blocks": R * K // 8, "alloc": [int(v) for v in res["1"]["alloc"]],
            "r_scale": float(res["1"]["r_scale"]), "hadamard_rotation": True, "hadamard_block_size": 128}
    ref = _ref(res["1"]["rows"].tobytes(), R, K, meta, res["1"]["x"])
    assert_rel(res["1"]["y"][:, :R], ref)
    assert_rel(res["0"]["y"][:, :R], ref)
    assert_rel(res["1"]["y"], res["0"]["y"])


def test_group_launch_bit_identical_to_single():
    """gate|up-like members reading one x share the table-GEMV launches (each
    member's r_scale applied to its row sums) and give exactly the
    single-weight results."""
    from polarflash_b200 import qlinear
    from polarflash_b200.qweight import qlinear_group

    K = 4096
    qws, pays, metas = [], [], []
    for i, M in enumerate((1500, 512, 512, 2048, 100)):
        qw, pay, meta = _polar_qweight(M, K, 60 + i)
        qws.append(qw)
        pays.append(pay)
        metas.append(meta)
    x = _x(1, K, 12).cuda()
    ys = qlinear_group(qws, [x] * len(qws))
    for i, qw in enumerate(qws):
        assert torch.equal(ys[i], qlinear(qw, x)), f"weight {i}"
        assert_rel(ys[i].cpu().numpy(), _ref(pays[i], qw.M, K, metas[i], x.float().cpu().numpy()))


def _golden_polar(key):
    import json

    here = os.path.dirname(os.path.abspath(__file__))
    g = np.load(os.path.join(here, "golden", "polar_recursive.npz"))
    with open(os.path.join(here, "golden", "polar_recursive_meta.json")) as f:
        meta = dict(json.load(f)[key])
    meta.update(hadamard_rotation=True, hadamard_block_size=128)
    return g, meta


@pytest.mark.parametrize("N", [2, 17, 64, 300, 2048])
def test_tensor_core_gemm_reference_payload(N):
    """The reference's own 1.75 bpw payload (128 x 1024, RWHT-128): y on the
    tcgen05 GEMM against the reference's decode_packed output, rotated back
    (the oracle's inverse RWHT), times x."""
    from polarflash_b200 import dequantize, qlinear, qweight_from_payload
    from test_gpu_parity import _x

    key = "d8_b1.75_128x1024"
    g, meta = _golden_polar(key)
    M, K = 128, 1024
    qw = qweight_from_payload("polar_recursive", meta, g[f"packed_{key}"].tobytes(), M, K, "cuda")
    x = _x(N, K, 40 + N)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    signs, block = oracle.hadamard_signs(K, 128)
    W = oracle.rwht(np.ascontiguousarray(g[f"dec_{key}"], np.float32), block, signs, inverse=True)
    assert_rel(y, oracle.matvec(W, x.float().numpy()))
    np.testing.assert_allclose(dequantize(qw, inverse_rwht=False).cpu().numpy(), g[f"dec_{key}"], atol=1e-6)


@pytest.mark.parametrize("codebooks", [False, True])
@pytest.mark.parametrize("N", [5, 64, 512])
def test_tensor_core_gemm_ragged(N, codebooks):
    """1000 x 4096 (a ragged last row tile), RWHT-128, device-encoded, with
    the uniform angle grid or learned codebooks (fitted on the weight)."""
    from polarflash_b200 import encoders, qlinear
    from polarflash_b200.quantizer import rwht_cpu
    from polarflash_b200.qweight import qweight_from_payload

    M, K = 1000, 4096
    Wr = rwht_cpu(_w(M, K, 77), 128)
    books = encoders.fit_polar_codebooks(Wr[:64], 8, 4, 8) if codebooks else None
    payload, meta = encoders.polar_encode(Wr.cuda(), 8, 1.75, codebooks=books)
    meta.update(hadamard_rotation=True, hadamard_block_size=128)
    qw = qweight_from_payload("polar_recursive", meta, payload, M, K, "cuda")
    x = _x(N, K, 78)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, _ref(payload.cpu().numpy().tobytes(), M, K, meta, x.float().numpy()))
