"""Column-parallel linears with the all-gather fused into the GEMV, on two
GPUs: each rank's kernel stores its output rows straight into both ranks'
peer buffers over NVLink, raises its flag and waits for the other rank's
(bounded waits; no collective library).

Checked: the gathered y on every rank equals the one-GPU product of the
whole weight within 1e-5 normwise (the shard's launch sums the same stage
partials in a different CTA grouping) and the oracle within 1e-3, over three
calls in a row (the epochs advance) and over replays of a CUDA graph of the
call; and pf_allgather_rows of already computed shards, interleaved with the
fused calls, puts each rank's shard rank-major in both buffers, bit for bit.
Needs two CUDA devices; the process group has a short timeout.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


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
    peer = None
    try:
        from test_gpu_parity import _g128_qweight, _w, _x

        from polarflash_b200.parallel import (PeerBuffer, allgather_rows, peers_wait, qlinear_group_gather,
                                              shard_bounds)
        from polarflash_b200.qweight import qlinear, workspace, workspace_status

        # a q|k|v-like group (INT3) and an o-like weight (INT2) on different inputs
        shapes = [(1024, 2048, 3), (256, 2048, 3), (512, 1024, 2)]
        full, pays, shards = [], [], []
        for i, (M, K, bits) in enumerate(shapes):
            qw, pay, _ = _g128_qweight(_w(M, K, 71 + i), bits)
            r0, r1 = shard_bounds(M, world, rank)
            full.append(qw)
            pays.append(pay)
            shards.append(qw.shard_rows(r0, r1))
        offs, off = [], 256
        for M, _, _ in shapes:
            offs.append(off)
            off += ((4 * M + 255) // 256) * 256
        gather_off = off  # pf_allgather_rows of a 3 x 1000 fp32 shard per rank
        peer = PeerBuffer(off + world * 3 * 1000 * 4, device=dev)
        ws = workspace(dev, 1)
        res = {"calls": [], "graph": None}
        for call in range(3):
            xs = [_x(1, K, 5 * call + i).to(dev) for i, (_, K, _) in enumerate(shapes)]
            qlinear_group_gather(shards, xs, peer, offs)
            if call == 2:  # the call's kernel waits for every rank's rows; pf_peers_wait repeats it
                peers_wait(peer, ws)
            ys = [peer.view(o, (1, M)).clone() for o, (M, _, _) in zip(offs, shapes)]
            refs = [qlinear(q, x) for q, x in zip(full, xs)]
            torch.cuda.synchronize()
            res["calls"].append([(y.cpu().numpy(), r.cpu().numpy(), x.float().cpu().numpy())
                                 for y, r, x in zip(ys, refs, xs)])
        # a CUDA graph of the call and its wait, replayed with new inputs
        s = torch.cuda.Stream(device=dev)
        xs = [_x(1, K, 40 + i).to(dev) for i, (_, K, _) in enumerate(shapes)]
        with torch.cuda.stream(s):
            qlinear_group_gather(shards, xs, peer, offs, stream=s)
            peers_wait(peer, ws, stream=s)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                qlinear_group_gather(shards, xs, peer, offs, stream=s)
                peers_wait(peer, ws, stream=s)
        s.synchronize()
        dist.barrier()
        for rep in range(3):
            for i, (_, K, _) in enumerate(shapes):
                xs[i].copy_(_x(1, K, 60 + 3 * rep + i).to(dev))
            with torch.cuda.stream(s):
                g.replay()
            s.synchronize()
        ys = [peer.view(o, (1, M)).clone() for o, (M, _, _) in zip(offs, shapes)]
        refs = [qlinear(q, x) for q, x in zip(full, xs)]
        torch.cuda.synchronize()
        res["graph"] = [(y.cpu().numpy(), r.cpu().numpy(), x.float().cpu().numpy()) for y, r, x in zip(ys, refs, xs)]
        # standalone all-gather of already computed shards, interleaved with the fused calls
        got = []
        for rep in range(2):
            shard = torch.randn(3, 1000, generator=torch.Generator().manual_seed(10 * rep + rank)).to(dev)
            out = allgather_rows(peer, shard, gather_off, ws).clone()
            got.append(out.cpu().numpy())
            qlinear_group_gather(shards, xs, peer, offs)
        torch.cuda.synchronize()
        res["allgather"] = got
        res["status"] = workspace_status(ws, counters=True)
        del g
        dist.barrier()
        out_q.put((rank, res, pays, shapes))
    finally:
        if peer is not None:
            torch.cuda.synchronize()
            dist.barrier()
            peer.close()
        dist.destroy_process_group()


def test_gathering_linears_world2():
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
        outs = [q.get(timeout=300) for _ in range(2)]
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    meta = {"hadamard_rotation": True, "hadamard_block_size": 128}
    for rank, res, pays, shapes in outs:
        assert res["status"] == (0, 0)
        for rep, got in enumerate(res["allgather"]):
            for r in range(2):  # rank-major: rank r's shard at [r]
                want = torch.randn(3, 1000, generator=torch.Generator().manual_seed(10 * rep + r)).numpy()
                np.testing.assert_array_equal(got[r], want)
        for triples in res["calls"] + [res["graph"]]:
            for (y, ref, x), pay, (M, K, bits) in zip(triples, pays, shapes):
                assert_rel(y, ref, rel=1e-5)
                assert_rel(y, oracle.linear(f"int{bits}_g128", pay, M, K, meta, x))
