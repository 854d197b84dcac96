"""GPU parity of the E8 RVQ2 lookup-table GEMV (batch 1): the kernel builds a
table of <root, x'-vector> products per 256-column stage and adds table
entries, so these tests cover rotation blocks from none to 512 columns, the
three activation dtypes, ragged row blocks, CTAs whose units span more stages
than stay resident, the full 28672 x 8192 shape against the tensor-core path,
and the fall back for inputs the kernel cannot take.

Tolerance as in test_gpu_parity: y within 1e-3 normwise of the oracle's fp32
decode + double-accumulated matvec.  Every sum is taken in a fixed order, so
repeated calls give identical bits.
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


def _e8_qweight(M, K, seed, hb=128, std=0.015):
    """Oracle-encoded E8 weight (rotated with block hb) as a device QWeight."""
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.quantizer import rwht_cpu
    from polarflash_b200.qweight import QWeight

    W = _w(M, K, seed, std=std)
    Wr = rwht_cpu(W, hb).numpy() if hb else W.numpy()
    idx, sc = oracle.e8_encode(Wr)
    dev = torch.device("cuda")
    qw = QWeight(7, M, K, torch.from_numpy(idx.reshape(-1).copy()).to(dev), torch.from_numpy(sc.copy()).to(dev),
                 None, effective_block(hb, K) if hb else 0, column_signs(K, hb, dev) if hb else None)
    meta = {"hadamard_rotation": bool(hb), "hadamard_block_size": hb}
    return qw, {"idx": idx, "scales": sc}, meta


@pytest.mark.parametrize("hb", [0, 64, 128, 256, 512])
@pytest.mark.parametrize("xdt", [torch.float16, torch.bfloat16, torch.float32])
def test_rotation_blocks_and_dtypes(hb, xdt):
    from polarflash_b200 import qlinear

    M, K = 1000, 2048
    qw, pay, meta = _e8_qweight(M, K, 11 + hb, hb)
    x = _x(1, K, 5 + hb, xdt)
    b = (torch.randn(M, generator=torch.Generator().manual_seed(hb)) * 0.1)
    y = qlinear(qw, x.cuda(), b.cuda()).cpu().numpy()
    assert_rel(y, oracle.linear("e8_rvq2_g128", pay, M, K, meta, x.float().numpy(), b.numpy()))


@pytest.mark.parametrize("M,K", [(1, 256), (33, 512), (512, 1024), (4100, 4096), (64, 65536)])
def test_shapes(M, K):
    """Single stage (no partial sums), ragged last row block, one row, and a
    long K with one row block (every CTA's units on few rows)."""
    from polarflash_b200 import qlinear

    qw, pay, meta = _e8_qweight(M, K, M + 7)
    x = _x(1, K, 3)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, oracle.linear("e8_rvq2_g128", pay, M, K, meta, x.float().numpy()))


def test_table_windows_rebuilt():
    """512 rows x 131072 columns: 512 units over the CTAs, each CTA's units
    span more stages than its resident tables, so tables are rebuilt mid-run."""
    from polarflash_b200 import qlinear

    M, K = 512, 131072
    qw, pay, meta = _e8_qweight(M, K, 77)
    x = _x(1, K, 9)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, oracle.linear("e8_rvq2_g128", pay, M, K, meta, x.float().numpy()))


def test_repeated_calls_bit_identical():
    from polarflash_b200 import qlinear

    qw, _, _ = _e8_qweight(2048, 8192, 3)
    x = _x(1, 8192, 4).cuda()
    y0 = qlinear(qw, x)
    for _ in range(3):
        assert torch.equal(qlinear(qw, x), y0)


def test_misaligned_input_takes_the_gemm():
    """An fp16 x that is only 2-byte aligned cannot feed the table build's
    vector loads; the call still succeeds (tensor-core path) and agrees."""
    from polarflash_b200 import qlinear

    M, K = 256, 1024
    qw, pay, meta = _e8_qweight(M, K, 21)
    x = _x(1, K, 8)
    buf = torch.zeros(K + 1, dtype=torch.float16, device="cuda")
    xm = buf[1:].view(1, K)
    xm.copy_(x.cuda())
    assert xm.data_ptr() % 8 != 0
    y = qlinear(qw, xm).cpu().numpy()
    assert_rel(y, oracle.linear("e8_rvq2_g128", pay, M, K, meta, x.float().numpy()))


_FULL_SCRIPT = r"""
import sys, numpy as np, torch
sys.path[:0] = sys.argv[2:]
from polarflash_b200 import encoders, qlinear
from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
from polarflash_b200.qweight import QWeight
M, K = 28672, 8192
dev = torch.device("cuda")
g = torch.Generator().manual_seed(0)
W = (torch.randn(M, K, generator=g) * 0.015).to(dev)
idx, sc = encoders.e8_encode(BlockHadamardTransform(K, 128, device=dev).forward(W))
qw = QWeight(7, M, K, idx.reshape(-1), sc, None, effective_block(128, K), column_signs(K, 128, dev))
x = torch.randn(1, K, generator=torch.Generator().manual_seed(1)).half().to(dev)
np.savez(sys.argv[1], y=qlinear(qw, x).cpu().numpy(), idx=idx[:4096].cpu().numpy(), sc=sc[:4096].cpu().numpy(),
         x=x.float().cpu().numpy())
"""


def test_full_size_against_tensor_core_path(tmp_path):
    """28672 x 8192 at batch 1: the table GEMV (default) and the tensor-core
    GEMM (PF_E8_LUT=0, which decodes roots x scales in fp16) on the same
    weights, both against the oracle on the first 4096 rows, and against each
    other over all rows."""
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    paths = [root, os.path.join(root, "polar-flash_b200"), here]
    script = tmp_path / "run.py"
    script.write_text(_FULL_SCRIPT)
    res = {}
    for mode in ("1", "0"):
        out = tmp_path / f"y{mode}.npz"
        subprocess.run([sys.executable, str(script), str(out)] + paths, check=True,
                       env=dict(os.environ, PF_E8_LUT=mode), timeout=900)
        res[mode] = np.load(out)
    K = 8192
    pay = {"idx": res["1"]["idx"], "scales": res["1"]["sc"]}
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    ref = oracle.linear("e8_rvq2_g128", pay, 4096, K, meta, res["1"]["x"])
    assert_rel(res["1"]["y"][:, :4096], ref)
    assert_rel(res["0"]["y"][:, :4096], ref)
    assert_rel(res["1"]["y"], res["0"]["y"])


def test_group_launch_bit_identical_to_single():
    """q|k|v-like members reading one x share the table-GEMV launches (four per
    launch, here 4 + 1) and give exactly the single-weight results."""
    from polarflash_b200 import qlinear
    from polarflash_b200.qweight import qlinear_group

    K = 2048
    qws, pays, metas, bs = [], [], [], []
    for i, M in enumerate((1000, 256, 256, 700, 512)):
        qw, pay, meta = _e8_qweight(M, K, 40 + i)
        qws.append(qw)
        pays.append(pay)
        metas.append(meta)
        bs.append((torch.randn(M, generator=torch.Generator().manual_seed(i)) * 0.1).cuda())
    x = _x(1, K, 6).cuda()
    ys = qlinear_group(qws, [x] * len(qws), bs)
    for i, qw in enumerate(qws):
        assert torch.equal(ys[i], qlinear(qw, x, bs[i])), f"weight {i}"
        assert_rel(ys[i].cpu().numpy(), oracle.linear("e8_rvq2_g128", pays[i], qw.M, K, metas[i],
                                                      x.float().cpu().numpy(), bs[i].cpu().numpy()))


@pytest.mark.parametrize("N", [1, 32, 2048])
def test_llama70b_down_projection(N):
    """The 70B stack's longest linear (down, 8192 x 28672, W ~ N(0, 0.01^2) with
    0.1 % outliers, RWHT-128) at decode batch 1 (table GEMV) and 32 and at a
    2048-token prefill (tensor-core GEMM), against the oracle on its first rows."""
    from polarflash_b200 import encoders, qlinear
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.qweight import QWeight

    M, K = 8192, 28672
    dev = torch.device("cuda")
    W = _w(M, K, 70, std=0.01).to(dev)
    idx, sc = encoders.e8_encode(BlockHadamardTransform(K, 128, device=dev).forward(W))
    del W
    qw = QWeight(7, M, K, idx.reshape(-1), sc, None, effective_block(128, K), column_signs(K, 128, dev))
    x = _x(N, K, 71)
    y = qlinear(qw, x.to(dev)).cpu().numpy()
    R = 256 if N <= 32 else 32
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    pay = {"idx": idx[:R].cpu().numpy(), "scales": sc[:R].cpu().numpy()}
    assert_rel(y[:, :R], oracle.linear("e8_rvq2_g128", pay, R, K, meta, x.float().numpy()))
