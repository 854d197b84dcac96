"""Column-parallel decode step on two GPUs: PFlashDecoder(tp=GroupGather())
with every projection of the two-layer model of tests/decode_model.py row-
sharded over two NCCL ranks, one all-gather per projection group, the step
captured as a CUDA graph (NCCL calls inside).  Both ranks' logits match the
reference's golden logits (tests/golden/decode_step.npz) within 1e-3 and the
one-GPU decoder within 1e-4 (normwise).  The process group has a short
timeout, and the graph holding NCCL calls is released before the group is
destroyed.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_step.npz")


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
    dec = None
    try:
        import decode_model as dm
        from test_decode_step import _decoder

        from polarflash_b200.decode import DecoderLayer, PFlashDecoder
        from polarflash_b200.parallel import GroupGather, shard_bounds

        g = np.load(GOLD)
        w = dm.build()
        full = _decoder(w)  # the one-GPU decoder, as test_decode_step builds it
        layers = []
        for ly in full.layers:
            sh = {}
            for name in ("q", "k", "v", "o", "gate", "up", "down"):
                qw = getattr(ly, name)
                r0, r1 = shard_bounds(qw.M, world, rank)
                sh[name] = qw.shard_rows(r0, r1)
            layers.append(DecoderLayer(sh["q"], sh["k"], sh["v"], sh["o"], sh["gate"], sh["up"], sh["down"],
                                       ly.input_norm, ly.post_norm))
        dec = PFlashDecoder(dm.CFG, layers, full.embed, full.final_norm, full.lm_head, 32, tp=GroupGather())
        prompt = torch.tensor(g["prompt"], device=dev)
        pre = dec.forward(prompt).cpu().numpy()
        pre1 = full.forward(prompt).cpu().numpy()
        dec.capture()
        full.capture()
        steps, steps1 = [], []
        for tok in g["decode"].tolist():
            steps.append(dec.step(tok)[0].cpu().numpy().copy())
            steps1.append(full.step(tok)[0].cpu().numpy().copy())
        torch.cuda.synchronize()
        dist.barrier()
        out_q.put((rank, pre, pre1, steps, steps1))
    finally:
        if dec is not None:
            dec._graph = None  # the graph holds NCCL calls: release it before the group goes
        del dec
        import gc

        gc.collect()
        torch.cuda.synchronize()
        dist.destroy_process_group()


def test_column_parallel_decode_step_world2():
    if not torch.cuda.is_available() or torch.cuda.device_count() < 2:
        pytest.skip("needs two CUDA devices")

    def rel(a, b):
        a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
        return float(np.abs(a - b).max() / np.abs(b).max())

    g = np.load(GOLD)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = [q.get(timeout=300) for _ in range(2)]
    finally:
        for p in procs:
            p.join(timeout=120)
    for p in procs:
        assert p.exitcode == 0
    for rank, pre, pre1, steps, steps1 in res:
        assert rel(pre, g["prefill_logits"]) < 1e-3, rank
        assert rel(pre, pre1) < 1e-4, rank
        for i in range(len(steps)):
            assert rel(steps[i], g["step_logits"][i]) < 1e-3, (rank, i)
            assert rel(steps[i], steps1[i]) < 1e-4, (rank, i)
