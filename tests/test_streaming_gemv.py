"""GPU parity of the streaming GEMV (the INT formats' decode path, K % 512 == 0):
grouped and mixed-format launches, rotation-block variants, row blocks split
over many CTAs, and the fall back for misaligned inputs.

Tolerance as in test_gpu_parity: y within 1e-3 normwise of the oracle's fp32
decode + double-accumulated matvec.
"""
import numpy as np
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


META = {"hadamard_rotation": True, "hadamard_block_size": 128}


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("N", [1, 3, 16])
def test_group_launch_matches_single(bits, N):
    """q/k/v-like group (three M, one K) plus two weights with other shapes,
    each with its own x and bias, in one launch.  The launch deals its units
    over the CTAs differently from a single-weight launch, so the order of the
    fp32 stage additions differs: agreement within 1e-5 normwise, and the
    same call twice gives the same bits."""
    from polarflash_b200 import qlinear
    from polarflash_b200.qweight import qlinear_group

    shapes = [(512, 1024), (128, 1024), (128, 1024), (640, 1024), (384, 2048)]
    qws, pays, xs, bs = [], [], [], []
    for i, (M, K) in enumerate(shapes):
        qw, pay, _ = _g128_qweight(_w(M, K, 10 * bits + i), bits)
        qws.append(qw)
        pays.append(pay)
        xs.append(_x(N, K, 50 + i).cuda())
        bs.append((torch.randn(M, generator=torch.Generator().manual_seed(i)) * 0.1).cuda())
    ys = qlinear_group(qws, xs, bs)
    ys2 = qlinear_group(qws, xs, bs)
    for i, (M, K) in enumerate(shapes):
        assert torch.equal(ys[i], ys2[i]), f"weight {i}: repeated call differs"
        y1 = qlinear(qws[i], xs[i], bs[i])
        assert_rel(ys[i].cpu().numpy(), y1.cpu().numpy(), rel=1e-5)
        ref = oracle.linear(f"int{bits}_g128", pays[i], M, K, META, xs[i].float().cpu().numpy(),
                            bs[i].cpu().numpy())
        assert_rel(ys[i].cpu().numpy(), ref)


@pytest.mark.parametrize("N", [1, 4])
def test_mixed_format_set_in_one_call(N):
    """A Llama-like linear set at INT3 and INT2 (and one INT4 weight) in ONE
    pf_qlinear_group call: one x' preparation launch, one GEMV launch for the
    INT3 and INT2 weights together and one for INT4; inputs shared by several
    weights are prepared once.  Every output against the oracle."""
    from polarflash_b200._lib import kernel_launches
    from polarflash_b200.qweight import qlinear_group

    shapes = [("q", 512, 1024), ("k", 128, 1024), ("v", 128, 1024), ("o", 512, 512), ("up", 1536, 1024),
              ("down", 1024, 1536)]
    xin = {K: _x(N, K, K).cuda() for K in (512, 1024, 1536)}
    qws, pays, fmts, xs = [], [], [], []
    for bits in (3, 2):
        for i, (_, M, K) in enumerate(shapes):
            qw, pay, _ = _g128_qweight(_w(M, K, 100 * bits + i), bits)
            qws.append(qw)
            pays.append(pay)
            fmts.append(f"int{bits}_g128")
            xs.append(xin[K])
    qw4, pay4, _ = _g128_qweight(_w(256, 1024, 77), 4)
    qws.append(qw4)
    pays.append(pay4)
    fmts.append("int4_g128")
    xs.append(xin[1024])
    qlinear_group(qws, xs)  # first call: one-time set-up
    torch.cuda.synchronize()
    n0 = kernel_launches()
    ys = qlinear_group(qws, xs)
    assert kernel_launches() - n0 == 3  # x' preparation, the INT3 + INT2 GEMV, the INT4 GEMV
    for y, qw, pay, fmt, x in zip(ys, qws, pays, fmts, xs):
        ref = oracle.linear(fmt, pay, qw.M, qw.K, META, x.float().cpu().numpy())
        assert_rel(y.cpu().numpy(), ref)


@pytest.mark.parametrize("bits", [4, 3, 2])
@pytest.mark.parametrize("hb", [0, 64, 256, 512])
@pytest.mark.parametrize("N,xdt", [(1, torch.float16), (5, torch.bfloat16), (2, torch.float32)])
def test_rotation_blocks(bits, hb, N, xdt):
    """In-kernel forward RWHT for blocks below, at and above one 128-column
    group (and no rotation)."""
    from polarflash_b200 import qlinear

    M, K = 384, 2048
    qw, pay, _ = _g128_qweight(_w(M, K, 7 * bits + hb), bits, hb=hb)
    x = _x(N, K, 3 + hb, xdt)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    meta = {"hadamard_rotation": bool(hb), "hadamard_block_size": hb}
    assert_rel(y, oracle.linear(f"int{bits}_g128", pay, M, K, meta, x.float().numpy()))


@pytest.mark.parametrize("bits,N", [(2, 1), (3, 1), (4, 1), (3, 4)])
def test_cta_spanning_many_stages(bits, N):
    """One 128-row block and a very long K: the row block is split over every
    CTA of the launch, each streaming many column stages through its x' ring,
    and the last warp to arrive adds all the parts."""
    from polarflash_b200 import qlinear

    M, K = 128, 512 * 640
    qw, pay, _ = _g128_qweight(_w(M, K, 99 + bits), bits)
    x = _x(N, K, 11)
    y = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y, oracle.linear(f"int{bits}_g128", pay, M, K, META, x.float().numpy()))


@pytest.mark.parametrize("bits", [3, 2])
def test_partial_row_block_and_single_stage(bits):
    """M not a multiple of 128 (zero-filled rows of the last block) and K of
    one column stage (outputs written without the partial-sum pass)."""
    from polarflash_b200 import qlinear

    for M, K in ((200, 512), (1000, 4096), (16, 1024)):
        qw, pay, _ = _g128_qweight(_w(M, K, M + bits), bits)
        x = _x(2, K, M)
        y = qlinear(qw, x.cuda()).cpu().numpy()
        assert_rel(y, oracle.linear(f"int{bits}_g128", pay, M, K, META, x.float().numpy()))


def test_misaligned_input_takes_the_other_path():
    """An fp16 x that is only 2-byte aligned cannot feed the streaming GEMV's
    vector loads; the call still succeeds (register-prefetch GEMV) and agrees."""
    from polarflash_b200 import qlinear

    M, K, N = 256, 1024, 3
    qw, pay, _ = _g128_qweight(_w(M, K, 5), 3)
    x = _x(N, K, 8)
    buf = torch.zeros(N * K + 1, dtype=torch.float16, device="cuda")
    xm = buf[1:].view(N, K)
    xm.copy_(x.cuda())
    assert xm.data_ptr() % 8 != 0
    y = qlinear(qw, xm).cpu().numpy()
    assert_rel(y, oracle.linear("int3_g128", pay, M, K, META, x.float().numpy()))
    y_al = qlinear(qw, x.cuda()).cpu().numpy()
    assert_rel(y_al, y, rel=1e-4)


def test_group_workspace_counters_return_to_zero():
    from polarflash_b200.qweight import qlinear_group, workspace

    dev = torch.device("cuda")
    qws = [_g128_qweight(_w(M, 4096, M), 2)[0] for M in (4096, 1024, 1024)]
    for N in (1, 4, 16):
        qlinear_group(qws, [_x(N, 4096, N).to(dev)] * 3)
    torch.cuda.synchronize()
    head = workspace(dev, 1)[: 16384 * 4].view(torch.int32)
    assert int(head.abs().sum()) == 0
    assert np.isfinite(qlinear_group(qws, [_x(1, 4096, 0).to(dev)] * 3)[0].cpu().numpy()).all()
