"""Column-parallel packed linear on two GPUs over NCCL: every rank runs the
fused kernel on its row shard, one all-gather assembles y, and the result
agrees with the unsharded product on one GPU and with the oracle.

Row shards of 128-row multiples keep every row block's contents, and the
streaming GEMV's stage partials are summed in a fixed order, so the sharded
y equals the unsharded one to within 1e-5 (normwise); the oracle bound is the
parity suite's 1e-3.  Needs two CUDA devices; the process group has a short
timeout so that a rank that fails ends the other's collective with an error.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

# (format, world, batch): batch 64 takes the tensor-core GEMM, the others the GEMV
CASES = [("int3_g128", 2, 1), ("int2_g128", 2, 4), ("int4_g128", 2, 64), ("e8", 2, 3)]


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import sys
    from datetime import timedelta

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "polar-flash_b200"), os.path.join(root, "tests")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import torch.distributed as dist

    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=dev, timeout=timedelta(seconds=60))
    try:
        import oracle
        from test_gpu_parity import _g128_qweight, _w, _x

        from polarflash_b200.hadamard import column_signs, effective_block
        from polarflash_b200.parallel import ColumnParallelQLinear
        from polarflash_b200.quantizer import rwht_cpu
        from polarflash_b200.qweight import QWeight, qlinear

        M, K = 1024, 2048
        res = {}
        for name, _, N in CASES:
            W = _w(M, K, 31 + N)
            if name == "e8":
                idx, sc = oracle.e8_encode(rwht_cpu(W, 128).numpy())
                qw = QWeight(7, M, K, torch.from_numpy(idx.reshape(-1).copy()).to(dev),
                             torch.from_numpy(sc.copy()).to(dev), None, effective_block(128, K),
                             column_signs(K, 128, dev))
                pay = {"idx": idx, "scales": sc}
            else:
                # built on the current device, cuda:rank
                qw, pay, _ = _g128_qweight(W, int(name[3]))
            bias = (torch.randn(M, generator=torch.Generator().manual_seed(N)) * 0.1).to(dev)
            x = _x(N, K, 17 + N).to(dev)
            layer = ColumnParallelQLinear(qw, bias=bias)
            y = layer(x)
            y_full = qlinear(qw, x, bias)
            torch.cuda.synchronize()
            if rank == 0:
                res[name] = (y.cpu().numpy(), y_full.cpu().numpy(), pay, x.float().cpu().numpy(),
                             bias.cpu().numpy())
        dist.barrier()
        if rank == 0:
            out_q.put(res)
    finally:
        dist.destroy_process_group()


def test_column_parallel_nccl_world2():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")
    import oracle
    from test_gpu_parity import assert_rel

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = q.get(timeout=300)
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    M, K = 1024, 2048
    for name, _, _ in CASES:
        y, y_full, pay, x, bias = res[name]
        assert_rel(y, y_full, rel=1e-5)
        fmt = "e8_rvq2_g128" if name == "e8" else name
        meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
        assert_rel(y, oracle.linear(fmt, pay, M, K, meta, x, bias))
