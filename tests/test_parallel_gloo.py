"""Column-parallel host logic with two gloo ranks on CPU: row shards of every
packed format slice without re-encoding, and the rank-major all-gather of the
shard outputs equals the unsharded product."""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

import oracle


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, out_q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "polar-flash_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from polarflash_b200 import encoders
        from polarflash_b200.parallel import gather_rows, shard_bounds
        from polarflash_b200.qweight import QWeight

        M, K, N = 256, 512, 3
        g = torch.Generator().manual_seed(0)
        W = torch.randn(M, K, generator=g) * 0.02
        x = torch.randn(N, K, generator=g)
        results = {}
        # group-128 INT3: full weight encoded once, then sharded by rows
        q, s, m = encoders.quant_g128_asym(W, 3)
        words = encoders.pack_g128(q, 3)
        full = QWeight(2, M, K, words.view(torch.uint8).flatten(), s, m)
        r0, r1 = shard_bounds(M, world, rank)
        sh = full.shard_rows(r0, r1)
        Wq = oracle.dequant_g128_asym(oracle.unpack_g128(3, sh.codes.numpy().view(np.uint32).reshape(r1 - r0, -1),
                                                         r1 - r0, K), sh.scales.numpy(), sh.mins.numpy())
        y_local = torch.from_numpy(oracle.matvec(Wq, x.numpy()))
        results["int3"] = gather_rows(y_local, world).numpy()
        # polar rows (byte-aligned rows of K/8 14-bit blocks)
        payload, meta = encoders.polar_encode(W, 8, 1.75)
        pw = QWeight(8, M, K, payload, None, None, 0, None, meta["r_scale"], [8] + meta["alloc"])
        ps = pw.shard_rows(r0, r1)
        dec = oracle.polar_decode(ps.codes.numpy().tobytes(), (r1 - r0) * K // 8, 8, meta["alloc"], meta["r_scale"])
        y_p = torch.from_numpy(oracle.matvec(dec.reshape(r1 - r0, K), x.numpy()))
        results["polar"] = gather_rows(y_p, world).numpy()
        if rank == 0:
            Wfull = oracle.dequant_g128_asym(q.numpy(), s.numpy(), m.numpy())
            results["int3_ref"] = oracle.matvec(Wfull, x.numpy())
            dfull = oracle.polar_decode(payload.numpy().tobytes(), M * K // 8, 8, meta["alloc"], meta["r_scale"])
            results["polar_ref"] = oracle.matvec(dfull.reshape(M, K), x.numpy())
            out_q.put(results)
    finally:
        dist.destroy_process_group()


def test_column_parallel_gloo_world2():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    res = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    np.testing.assert_allclose(res["int3"], res["int3_ref"], rtol=1e-6, atol=1e-7)
    np.testing.assert_allclose(res["polar"], res["polar_ref"], rtol=1e-6, atol=1e-7)


def test_shard_bounds_rejects_uneven():
    from polarflash_b200.parallel import shard_bounds

    assert shard_bounds(1024, 8, 7) == (896, 1024)
    with pytest.raises(ValueError):
        shard_bounds(1001, 8, 0)


def _group_worker(rank, world, port, out_q):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [root, os.path.join(root, "polar-flash_b200")]
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from polarflash_b200.parallel import GroupGather

        g = torch.Generator().manual_seed(1)
        S, Ms = 3, (96, 24, 24)  # q|k|v-like group, full widths
        full = [torch.randn(S, M, generator=g) for M in Ms]
        shards = [f[:, rank * (M // world):(rank + 1) * (M // world)].contiguous() for f, M in zip(full, Ms)]
        out = GroupGather().gather(shards)
        if rank == 0:
            out_q.put(([o.numpy() for o in out], [f.numpy() for f in full]))
    finally:
        dist.destroy_process_group()


def test_group_gather_one_collective_world2():
    """GroupGather packs a projection group's row-shard outputs, gathers them
    in one collective and hands back each full output (the tensor-parallel
    decode step's gather)."""
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_group_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    out, full = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for o, f in zip(out, full):
        np.testing.assert_array_equal(o, f)
