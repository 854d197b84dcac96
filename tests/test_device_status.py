"""Device timeouts reach the caller.

Every wait in the library's kernels is bounded; one that runs out records
PF_ERR_TIMEOUT in the workspace status word and the kernel ends early.
Here a wait is made to run out on purpose the only safe way: the library's
own wait loop on a barrier that no thread completes, with a 50 ms limit
(pf_wait_selftest).  No fault, trap or hang is involved; the context stays
usable, which the tests check by running a linear afterwards.
"""
import ctypes

import numpy as np
import pytest
import torch

import oracle
from test_gpu_parity import _g128_qweight, _w, _x, assert_rel

pytestmark = pytest.mark.gpu

META = {"hadamard_rotation": True, "hadamard_block_size": 128}


@pytest.fixture(scope="module", autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import polarflash_b200  # noqa: F401
    torch.cuda.init()


def test_timed_out_wait_is_reported_and_reset():
    from polarflash_b200 import _lib, qlinear
    from polarflash_b200.qweight import workspace_status

    dev = torch.device("cuda")
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    assert workspace_status(ws, counters=True) == (_lib.OK, 0)
    s = torch.cuda.current_stream(dev)
    _lib.check(_lib.load().pf_wait_selftest(ctypes.c_void_p(ws.data_ptr()), 50_000_000,
                                            ctypes.c_void_p(s.cuda_stream)), "pf_wait_selftest")
    st, busy = workspace_status(ws, counters=True)
    assert st == _lib.ERR_TIMEOUT and busy == 0
    assert workspace_status(ws, reset=True)[0] == _lib.ERR_TIMEOUT
    assert workspace_status(ws)[0] == _lib.OK
    # the context is still usable: a linear on the same workspace is correct
    qw, pay, _ = _g128_qweight(_w(512, 2048, 3), 3)
    x = _x(1, 2048, 4)
    y = qlinear(qw, x.cuda(), workspace=ws).cpu().numpy()
    assert_rel(y, oracle.linear("int3_g128", pay, 512, 2048, META, x.float().numpy()))
    assert workspace_status(ws, counters=True) == (_lib.OK, 0)


def test_engine_check_raises_runtime_error():
    """check_device_status (called by PFlashCUDAEngine.forward_layer after its
    per-layer synchronisation) turns a recorded timeout into RuntimeError, as
    the reference reports driver failures, and re-arms the workspace."""
    from polarflash_b200 import _lib, qlinear
    from polarflash_b200.qweight import check_device_status, workspace

    dev = torch.device("cuda")
    s = torch.cuda.Stream(device=dev)
    ws = workspace(dev, 1 << 20, s)
    _lib.check(_lib.load().pf_wait_selftest(ctypes.c_void_p(ws.data_ptr()), 20_000_000,
                                            ctypes.c_void_p(s.cuda_stream)), "pf_wait_selftest")
    with pytest.raises(RuntimeError, match="timed out"):
        check_device_status(dev, s)
    check_device_status(dev, s)  # reset: nothing left to report
    qw, pay, _ = _g128_qweight(_w(256, 1024, 9), 2)
    x = _x(2, 1024, 5)
    with torch.cuda.stream(s):
        y = qlinear(qw, x.cuda())
    s.synchronize()
    assert_rel(y.cpu().numpy(), oracle.linear("int2_g128", pay, 256, 1024, META, x.float().numpy()))
    check_device_status(dev, s)
    assert np.isfinite(y.cpu().numpy()).all()
