#!/usr/bin/env python
"""Fused dequant-GEMV throughput on the Llama-3-8B linear set (INT3 and INT2,
group-128 asymmetric, block-128 RWHT), batch-1 decode.

One step = one pass over the 7-linear set (q/o 4096x4096, k/v 1024x4096,
gate/up 14336x4096, down 4096x14336) at INT3 and again at INT2: 14 fused
GEMVs over 156.7 MB of packed weights, computed by one pf_qlinear_group call
(one x' preparation launch for the set's inputs, then one streaming GEMV
launch per format over its 7 weights).  The same weights issued in layer
order (one call per shared input: q|k|v, o, gate|up, down) are timed too and
reported as "layer_order".  32 resident copies of the packed sets (one per
layer of the 8B model, 5.0 GB) are cycled so every step reads weights
untouched for the previous 31 steps (inputs >> the 126 MB L2).  The timed
region replays CUDA graphs of the steps; inputs are resident in HBM.

Metric: effective packed-weight GB/s (algorithmic bytes: packed codes +
fp16 scales/mins + x + y).  At N GPUs (torchrun) the same fixed set is
column-sharded: rank r holds rows [r M / N, (r + 1) M / N) of every linear
(strong scaling), and every step ends with one NCCL all-gather of the step's
outputs, captured in the CUDA graphs; the all-gather's time per step is
reported beside the kernel-only figure (`--scaling weak`: each rank a full
set of its own).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "polar-flash_b200"))
sys.path.insert(0, ROOT)

import numpy as np  # noqa: E402
import torch  # noqa: E402

LINEARS = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
           ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
FORMATS = ("int3_g128", "int2_g128")
# linears sharing one input (q/k/v and gate/up read the same x in a layer): one launch each
SHARED = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]
METRIC = "fused dequant-GEMV packed-weight HBM GB/s (Llama-3-8B linear set, INT3+INT2 g128, batch 1)"
# the GEMV design a recorded ncu traffic capture must be of
TRAFFIC_DESIGN = "stream-k row-major, in-kernel fixup, x' records from xprep_frag_kernel"
WORKLOAD = "llama3-8b linear set (q,k,v,o,gate,up,down) INT3 g128 + INT2 g128, RWHT-128, fp16 x, batch 1"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=2000)
    ap.add_argument("--warmup", type=int, default=50)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--copies", type=int, default=32)
    ap.add_argument("--graph-steps", type=int, default=32,
                    help="steps captured per CUDA graph (the 32 layers of an 8B decode graph)")
    ap.add_argument("--gather", default="nccl", choices=["peer", "nccl"],
                    help="at N GPUs: peer = the GEMV stores its rows into every rank's buffer over NVLink "
                         "(pf_qlinear_group_gather); nccl = an NCCL all-gather after the GEMV")
    ap.add_argument("--scaling", default="strong", choices=["strong", "weak"],
                    help="at N GPUs: strong = one fixed set, each rank a row shard of every linear; "
                         "weak = each rank a full set of its own")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-decode", action="store_true", help="skip the decode tokens/s figures")
    ap.add_argument("--tp-decode", action="store_true",
                    help="at N GPUs: also time the column-parallel config-4 decode step (4 all-gathers per layer)")
    return ap.parse_args()


def synth_weight(M, K, seed, device, std=0.02):
    """W ~ N(0, std^2) with 0.1% of entries at +-20 sigma (seeded positions)."""
    g = torch.Generator(device=device).manual_seed(seed)
    W = torch.randn(M, K, generator=g, device=device) * std
    n = max(1, int(0.001 * M * K))
    pos = torch.randint(0, M * K, (n,), generator=g, device=device)
    sg = torch.randint(0, 2, (n,), generator=g, device=device).float() * 2 - 1
    W.view(-1)[pos] = sg * (20.0 * std)
    return W


def upload_graphs(gl, stream):
    """Uploads instantiated CUDA graphs to the device (cuGraphUpload) without
    running them, so a graph's first replay inside a timed region does not
    also pay its one-time upload."""
    import ctypes

    try:
        cu = ctypes.CDLL("libcuda.so.1")
    except OSError:
        return
    cu.cuGraphUpload.argtypes = [ctypes.c_void_p, ctypes.c_void_p]
    cu.cuGraphUpload.restype = ctypes.c_int
    for g in gl:
        ex = g.raw_cuda_graph_exec()
        if not ex or cu.cuGraphUpload(ctypes.c_void_p(ex), ctypes.c_void_p(stream.cuda_stream)) != 0:
            print("bench: a CUDA graph was not uploaded ahead of its first replay", file=sys.stderr)
            return


def time_tokens(graphs, stream, tokens):
    """Device ms per token of a decode step that replays every graph once (one
    graph per layer), over `tokens` tokens after two untimed ones."""
    with torch.cuda.stream(stream):
        for _ in range(2):
            for gr in graphs:
                gr.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(tokens):
            for gr in graphs:
                gr.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    return e0.elapsed_time(e1) / tokens


def decode_rates(copies, xs, outs, ws, stream, dev, layers, tokens=20):
    """Tokens/s of the linears of one batch-1 decode token of the Llama-3-8B
    shape (`layers` layers of q|k|v, o, gate|up, down, each layer its own
    resident weight copy): INT3 g128 and INT2 g128 (the bench's weights), and
    recursive polar at 1.75 bpw (block 8, RWHT-128) encoded here."""
    from polarflash_b200 import encoders
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.qweight import QWeight, group_workspace_bytes, qlinear_multi

    res = {}
    for fmt in FORMATS:
        graphs = []
        with torch.cuda.stream(stream):
            for li in range(layers):
                cp = copies[li % len(copies)]
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for grp in SHARED:
                        qlinear_multi([cp[(fmt, n)] for n in grp], xs[grp], workspace=ws,
                                      outs=[outs[(fmt, n)] for n in grp])
                graphs.append(gr)
        ms = time_tokens(graphs, stream, tokens)
        nb = sum(alg_bytes(copies[0][(fmt, n)], 1) for n, _, _ in LINEARS) * layers
        res[fmt] = {"tok_s": round(1e3 / ms, 1), "ms_per_token": round(ms, 4), "GB_s": round(nb / ms / 1e6, 1)}
        del graphs
    # recursive polar 1.75 bpw: one encoded layer, `layers` resident copies
    base = {}
    for i, (name, M, K) in enumerate(LINEARS):
        W = synth_weight(M, K, 2000 + i, dev)
        payload, meta = encoders.polar_encode(BlockHadamardTransform(K, 128, device=dev).forward(W), 8, 1.75)
        base[name] = QWeight(8, M, K, payload, None, None, effective_block(128, K), column_signs(K, 128, dev),
                             meta["r_scale"], [8] + meta["alloc"])
        del W
    pc = [base] + [{n: QWeight(q.format, q.M, q.K, q.codes.clone(), None, None, q.had_block, q.had_signs,
                               q.tensor_scale, list(q.params)) for n, q in base.items()} for _ in range(layers - 1)]
    need = max(group_workspace_bytes([base[n] for n in grp], 1) for grp in SHARED)
    pws = torch.zeros(need, dtype=torch.uint8, device=dev)
    pout = {n: torch.empty(1, M, device=dev) for n, M, _ in LINEARS}
    graphs = []
    with torch.cuda.stream(stream):
        for cp in pc:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for grp in SHARED:  # one launch per shared input, as for the INT formats
                    qlinear_multi([cp[n] for n in grp], xs[grp], workspace=pws, outs=[pout[n] for n in grp])
            graphs.append(gr)
    ms = time_tokens(graphs, stream, tokens)
    nb = sum(q.nbytes() + q.K * 2 + q.M * 4 for q in base.values()) * layers
    res["polar_recursive_1.75"] = {"tok_s": round(1e3 / ms, 1), "ms_per_token": round(ms, 4),
                                   "GB_s": round(nb / ms / 1e6, 1)}
    del graphs
    # the whole step of the recursive-polar stack at a 2048-token context
    res.update(decode_full_step(pc, stream, dev, 2048, tokens, "llama3_8b_polar1.75_full_step_ctx2048", nb))
    del pc, base
    int3 = [{n: copies[li % len(copies)][("int3_g128", n)] for n, _, _ in LINEARS} for li in range(layers)]
    nb3 = sum(alg_bytes(copies[0][("int3_g128", n)], 1) for n, _, _ in LINEARS) * layers
    res.update(decode_full_step(int3, stream, dev, 512, tokens, "llama3_8b_int3_full_step_ctx512", nb3))
    res.update(decode_rates_70b_e8(stream, dev, tokens))
    res.update(kv_attention_rates(stream, dev, tokens=tokens))
    return res


def decode_full_step(layer_ws, stream, dev, ctx, tokens, name, lin_bytes):
    """Tokens/s of a whole batch-1 decode step of the Llama-3-8B shape
    (polarflash_b200.decode.PFlashDecoder, one CUDA graph per token): the
    packed linears of every layer (`layer_ws`: one dict q..down -> QWeight
    per layer, `lin_bytes` their algorithmic bytes), RMSNorms, RoPE, the fp32
    KV cache at `ctx` previous tokens, the library's attention kernels and a
    dense fp16 embedding and lm_head (128256 x 4096, 1.05 GB)."""
    from polarflash_b200.decode import DecoderLayer, PFlashDecoder

    H, V = 4096, 128256
    cfg = dict(hidden_size=H, num_attention_heads=32, num_key_value_heads=8, intermediate_size=14336, vocab_size=V,
               rope_theta=500000.0, rms_norm_eps=1e-5)
    g = torch.Generator(device=dev).manual_seed(5)
    ones = torch.ones(H, device=dev)
    layers = len(layer_ws)
    lys = [DecoderLayer(w["q"], w["k"], w["v"], w["o"], w["gate"], w["up"], w["down"], ones, ones) for w in layer_ws]
    embed = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    head = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    dec = PFlashDecoder(cfg, lys, embed, ones, head, max_seq=ctx + 1)
    with torch.cuda.stream(stream):
        dec.forward(torch.tensor([1], device=dev))  # one-time set-up of every launch path, outside the capture
        dec.length = ctx  # attend over `ctx` cached positions (contents are the cache's zeros)
        dec.capture(stream)
        for _ in range(2):
            dec._pos.fill_(ctx)
            dec._graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(tokens):
            dec._graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / tokens
    nb = lin_bytes + V * H * 2 + layers * 2 * (ctx + 1) * 8 * 128 * 4
    del dec, embed, head, lys
    return {name: {"tok_s": round(1e3 / ms, 1), "ms_per_token": round(ms, 4), "GB_s": round(nb / ms / 1e6, 1)}}


def decode_tp_step(stream, dev, world, layers=32, ctx=2048, tokens=20):
    """Config 4 column-parallel: the whole batch-1 decode step of the
    recursive-polar 1.75 bpw Llama-3-8B stack at a `ctx`-token context with
    every projection row-sharded over the `world` ranks
    (PFlashDecoder(tp=GroupGather()): one NCCL all-gather per projection
    group, four per layer, inside the step's CUDA graph); norms, RoPE,
    attention, the KV cache and the lm_head replicated.  Returns ms per token,
    max over ranks."""
    import torch.distributed as dist

    from polarflash_b200 import encoders
    from polarflash_b200.decode import DecoderLayer, PFlashDecoder
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.parallel import GroupGather, shard_bounds
    from polarflash_b200.qweight import QWeight

    rank = dist.get_rank()
    shards = {}
    for i, (name, M, K) in enumerate(LINEARS):
        W = synth_weight(M, K, 2000 + i, dev)
        payload, meta = encoders.polar_encode(BlockHadamardTransform(K, 128, device=dev).forward(W), 8, 1.75)
        full = QWeight(8, M, K, payload, None, None, effective_block(128, K), column_signs(K, 128, dev),
                       meta["r_scale"], [8] + meta["alloc"])
        shards[name] = full.shard_rows(*shard_bounds(M, world, rank))
        del W, full, payload
    H, V = 4096, 128256
    ones = torch.ones(H, device=dev)
    lys = []
    for li in range(layers):
        w = shards if li == 0 else {n: QWeight(q.format, q.M, q.K, q.codes.clone(), None, None, q.had_block,
                                               q.had_signs, q.tensor_scale, list(q.params))
                                    for n, q in shards.items()}
        lys.append(DecoderLayer(w["q"], w["k"], w["v"], w["o"], w["gate"], w["up"], w["down"], ones, ones))
    g = torch.Generator(device=dev).manual_seed(5)
    embed = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    head = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    cfg = dict(hidden_size=H, num_attention_heads=32, num_key_value_heads=8, intermediate_size=14336,
               vocab_size=V, rope_theta=500000.0, rms_norm_eps=1e-5)
    dec = PFlashDecoder(cfg, lys, embed, ones, head, max_seq=ctx + 1, tp=GroupGather())
    with torch.cuda.stream(stream):
        dec.forward(torch.tensor([1], device=dev))
        dec.length = ctx
        dec.capture(stream)
        for _ in range(2):
            dec._graph.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(tokens):
            dec._graph.replay()
        e1.record(stream)
        torch.cuda.synchronize()
    ms = torch.tensor([e0.elapsed_time(e1) / tokens], device=dev, dtype=torch.float64)
    dec._graph = None  # holds NCCL calls: released before the process group
    del dec, lys, shards, embed, head
    import gc

    gc.collect()
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms.item())


def kv_attention_rates(stream, dev, layers=32, ctx=16384, tokens=20):
    """Device time of the attention over the KV cache of one batch-1 decode
    token, Llama-3-8B attention shape (32 query / 8 KV heads of 128), one cache
    per layer at `ctx` cached positions (every layer's cache resident, the
    set larger than L2), for the fp32 cache (pf_decode_attention) and the
    compressed int8 / 2bit / 2bit_asym caches (pf_decode_attention_compressed,
    codes dequantized inside the kernel).  GB_s counts the cache bytes read
    (codes, scales, zeros of ctx positions x 8 KV heads, K and V)."""
    import ctypes
    import math

    from polarflash_b200 import _lib
    from polarflash_b200.kv_cache import KV_MODES, kv_row_bytes

    L = _lib.load()
    nh, nkv, hd, ms = 32, 8, 128, ctx
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    st = ctypes.c_void_p(stream.cuda_stream)
    q = torch.randn(nh * hd, device=dev)
    out = torch.empty(nh * hd, device=dev)
    pos = torch.tensor([ctx - 1], dtype=torch.long, device=dev)
    aws = torch.empty(int(L.pf_decode_attention_workspace_size(nh, hd, ms)), dtype=torch.uint8, device=dev)
    res = {}
    for mode in ("fp32", "int8", "2bit", "2bit_asym"):
        rb = 4 * hd if mode == "fp32" else kv_row_bytes(mode, hd)
        asym = mode == "2bit_asym"
        caches = []
        for _ in range(layers):
            kc = torch.zeros(ms, nkv, rb, dtype=torch.uint8, device=dev)
            vc = torch.zeros(ms, nkv, rb, dtype=torch.uint8, device=dev)
            sc = None if mode == "fp32" else torch.ones(2, ms, nkv, device=dev)
            zr = torch.zeros(2, ms, nkv, device=dev) if asym else None
            caches.append((kc, vc, sc, zr))

        def run():
            for kc, vc, sc, zr in caches:
                if mode == "fp32":
                    _lib.check(L.pf_decode_attention(p(q), p(kc), p(vc), p(pos), p(out), nh, nkv, hd, ms,
                                                     1.0 / math.sqrt(hd), p(aws), aws.numel(), st))
                else:
                    _lib.check(L.pf_decode_attention_compressed(
                        p(q), p(kc), p(sc[0]), p(zr[0] if asym else None), p(vc), p(sc[1]),
                        p(zr[1] if asym else None), p(pos), p(out), nh, nkv, hd, ms, KV_MODES[mode],
                        1.0 / math.sqrt(hd), p(aws), aws.numel(), st))

        gr = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            run()  # eager set-up outside the capture
            with torch.cuda.graph(gr, stream=stream):
                run()
        ms_tok = time_tokens([gr], stream, tokens)
        nb = layers * 2 * ctx * nkv * (rb + (0 if mode == "fp32" else 4) + (4 if asym else 0))
        res[mode] = {"us_per_layer": round(ms_tok * 1e3 / layers, 2), "GB_s": round(nb / ms_tok / 1e6, 1),
                     "cache_MB_per_layer": round(nb / layers / 1e6, 2)}
        del gr, caches
    return {"kv_attention_llama3_8b_ctx16k": res}


LINEARS_70B = [("q", 8192, 8192), ("k", 1024, 8192), ("v", 1024, 8192), ("o", 8192, 8192),
               ("gate", 28672, 8192), ("up", 28672, 8192), ("down", 8192, 28672)]


def decode_rates_70b_e8(stream, dev, tokens, layers=80):
    """Tokens/s of the linears of a Llama-3-70B-shaped decode step (80 layers of
    q|k|v, o, gate|up, down; W ~ N(0, 0.01^2) with 0.1 % outliers, RWHT-128,
    E8 RVQ2) at batch 1 (table GEMV) and batch 32 (tensor-core GEMM): one
    encoded layer, one resident copy per layer (19.3 GB)."""
    from polarflash_b200 import encoders
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.qweight import QWeight, group_workspace_bytes, qlinear_multi

    base = {}
    for i, (name, M, K) in enumerate(LINEARS_70B):
        W = synth_weight(M, K, 3000 + i, dev, std=0.01)
        idx, sc = encoders.e8_encode(BlockHadamardTransform(K, 128, device=dev).forward(W))
        base[name] = QWeight(7, M, K, idx.reshape(-1), sc, None, effective_block(128, K), column_signs(K, 128, dev))
        del W
    pc = [base] + [{n: QWeight(q.format, q.M, q.K, q.codes.clone(), q.scales.clone(), None, q.had_block,
                               q.had_signs) for n, q in base.items()} for _ in range(layers - 1)]
    kdim = {n: K for n, _, K in LINEARS_70B}
    layer_bytes = sum(q.nbytes() for q in base.values())
    res = {}
    for B in (1, 32):
        g = torch.Generator().manual_seed(B)
        xs = {grp: torch.randn(B, kdim[grp[0]], generator=g).half().to(dev) for grp in SHARED}
        outs = {n: torch.empty(B, M, device=dev) for n, M, _ in LINEARS_70B}
        need = max(group_workspace_bytes([base[n] for n in grp], B) for grp in SHARED)
        ws = torch.zeros(need, dtype=torch.uint8, device=dev)
        graphs = []
        with torch.cuda.stream(stream):
            for cp in pc:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for grp in SHARED:
                        qlinear_multi([cp[n] for n in grp], xs[grp], workspace=ws, outs=[outs[n] for n in grp])
                graphs.append(gr)
        ms = time_tokens(graphs, stream, max(4, tokens // (4 if B > 1 else 1)))
        res[f"e8_rvq2_70b_batch{B}"] = {"tok_s": round(B * 1e3 / ms, 1), "ms_per_step": round(ms, 4),
                                        "GB_s": round(layer_bytes * layers / ms / 1e6, 1)}
        del graphs
    # config 5's prefill: 2048 tokens through the linears of `pl` layers (each
    # layer's own copy), the tensor-core GEMM in 512-token chunks
    B, pl = 2048, 4
    g = torch.Generator().manual_seed(B)
    xs = {grp: torch.randn(B, kdim[grp[0]], generator=g).half().to(dev) for grp in SHARED}
    outs = {n: torch.empty(B, M, device=dev) for n, M, _ in LINEARS_70B}
    need = max(group_workspace_bytes([base[n] for n in grp], B) for grp in SHARED)
    ws = torch.zeros(need, dtype=torch.uint8, device=dev)
    graphs = []
    with torch.cuda.stream(stream):
        for cp in pc[:pl]:
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for grp in SHARED:
                    qlinear_multi([cp[n] for n in grp], xs[grp], workspace=ws, outs=[outs[n] for n in grp])
            graphs.append(gr)
    ms = time_tokens(graphs, stream, 2) / pl  # ms per layer
    flops = 2.0 * B * sum(M * K for _, M, K in LINEARS_70B)
    res["e8_rvq2_70b_prefill_2048"] = {"ms_per_layer": round(ms, 4), "TFLOP_s": round(flops / ms / 1e9, 1),
                                       "tok_s": round(B * 1e3 / (ms * layers), 1)}
    del graphs, xs, outs, ws
    del pc, base
    return res


def alg_bytes(qw, N):
    """Algorithmic bytes of one fused GEMV: packed payload + scales/mins + x
    (fp16) + y (fp32)."""
    return qw.nbytes() + N * qw.K * 2 + N * qw.M * 4


class Clocks:
    """nvidia-smi sampler (SM clock, max clock, throttle reasons) during a window."""

    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
         "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
         "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:  # noqa: BLE001
            self.proc = None

    def stop(self):
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        out, _ = self.proc.communicate(timeout=10)
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in out.strip().splitlines():
            f = [v.strip() for v in line.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for nm, v in zip(names, f[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def cpu_reference_leg(fmt_sets, samples, threads=None, outputs=None):
    """The reference's CPU path (decode -> inverse block RWHT -> fp32 matvec,
    polarflash_rt/cpu/engine.py:58-96 via unified_quantizer.py:242-324) as the
    oracle's C port, all host threads.  Returns (GB/s, seconds, cores); the
    y of every sample is appended to `outputs` when given."""
    import oracle

    if threads:
        oracle.set_num_threads(threads)
    cores = oracle.num_threads()
    t_total, b_total = 0.0, 0
    for (fmt, name, payload, M, K, x) in samples:
        t0 = time.perf_counter()
        W = oracle.dequantize(fmt, payload, M, K, {"hadamard_rotation": True, "hadamard_block_size": 128})
        y = oracle.matvec_f32(W, x)
        t_total += time.perf_counter() - t0
        b_total += payload["words"].nbytes + payload["s"].nbytes + payload["m"].nbytes + x.size * 2 + M * 4
        if outputs is not None:
            outputs.append(y)
    return b_total / t_total / 1e9, t_total, cores


def parity_stats(pairs):
    """Device y against the CPU reference y over (y, y_ref) pairs: the bound
    the tests apply is normwise per linear, max|y - y_ref| <= 1e-3 max|y_ref|;
    the elementwise relative error |y_i - y_ref_i| / |y_ref_i| is reported
    beside it (its max over elements with |y_ref_i| >= 1 % of max|y_ref|, and
    its 99th percentile over all elements)."""
    norm, emax, ep99 = 0.0, 0.0, []
    for y, r in pairs:
        y = np.asarray(y, np.float64).ravel()
        r = np.asarray(r, np.float64).ravel()
        d = np.abs(y - r)
        scale = np.abs(r).max()
        norm = max(norm, d.max() / scale)
        big = np.abs(r) >= 0.01 * scale
        emax = max(emax, float((d[big] / np.abs(r[big])).max()))
        nz = np.abs(r) > 0
        ep99.append(d[nz] / np.abs(r[nz]))
    return {"bound": "normwise per linear: max|y - y_ref| <= 1e-3 * max|y_ref| (the 1e-3 of the tests)",
            "normwise_max": float(f"{norm:.3e}"), "elementwise_max_rel_above_1pct": float(f"{emax:.3e}"),
            "elementwise_p99_rel": float(f"{np.percentile(np.concatenate(ep99), 99):.3e}"),
            "reference": "the oracle's fp32 decode + inverse RWHT + matvec (the CPU baseline leg's outputs)"}


def cpu_model():
    """The host CPU's model string (/proc/cpuinfo), for the CPU baseline records."""
    try:
        with open("/proc/cpuinfo") as f:
            for line in f:
                if line.startswith("model name"):
                    return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def host_payload(qw):
    return {"words": qw.codes.cpu().numpy().view(np.uint32).reshape(qw.M, -1),
            "s": qw.scales.cpu().numpy(), "m": qw.mins.cpu().numpy()}


def run_reference(args, rank, world):
    """--impl reference: the reference CPU path timed on the host cores; each
    step is one linear of the set (cycled), a bounded sample."""
    if rank != 0:
        return
    import oracle
    from polarflash_b200.quantizer import rwht_cpu
    from polarflash_b200 import encoders

    # every host core, whatever OMP_NUM_THREADS the launcher set (torchrun sets 1)
    oracle.set_num_threads(os.cpu_count() or 1)
    torch.set_num_threads(os.cpu_count() or 1)
    samples = []
    for fmt in FORMATS:
        bits = int(fmt[3])
        for i, (name, M, K) in enumerate(LINEARS):
            W = synth_weight(M, K, 1000 + i, "cpu")
            Wr = rwht_cpu(W, 128)
            q, s, m = encoders.quant_g128_asym(Wr, bits)
            words = encoders.pack_g128(q, bits).numpy().view(np.uint32)
            x = torch.randn(args.batch, K, generator=torch.Generator().manual_seed(7)).half().float().numpy()
            samples.append((fmt, name, {"words": words, "s": s.numpy(), "m": m.numpy()}, M, K, x))
    cores = oracle.num_threads()
    for w in range(args.warmup):
        cpu_reference_leg(None, [samples[w % len(samples)]])
    t, b = 0.0, 0
    for k in range(args.steps):
        gbs, tt, _ = cpu_reference_leg(None, [samples[k % len(samples)]])
        t += tt
        b += gbs * tt * 1e9
    value = b / t / 1e9
    # the reference engine's keep_cached=True steady state (cpu/engine.py:58-96):
    # the fp32 weight decoded once, then one torch.matmul per call
    tc, bc = 0.0, 0
    for fmt, name, payload, M, K, x in samples[:len(LINEARS)]:
        W = torch.from_numpy(oracle.dequantize(fmt, payload, M, K, {"hadamard_rotation": True,
                                                                     "hadamard_block_size": 128}))
        xt = torch.from_numpy(x)
        torch.matmul(xt, W.t())
        t0 = time.perf_counter()
        for _ in range(3):
            torch.matmul(xt, W.t())
        tc += (time.perf_counter() - t0) / 3
        bc += payload["words"].nbytes + payload["s"].nbytes + payload["m"].nbytes + x.size * 2 + M * 4
        del W
    line = {
        "impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": args.scaling, "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": {"workload": WORKLOAD, "batch": args.batch, "step": "one linear of the set, cycled"},
        "cpu_baseline": {"value": round(value, 4), "unit": "GB/s", "cores": cores, "kind": "port",
                         "cpu_model": cpu_model(),
                         "sample": f"{args.steps} linears of the set (cycled), decode + inverse RWHT + fp32 matvec",
                         "cached_steady": {"value": round(bc / tc / 1e9, 4), "unit": "GB/s",
                                           "sample": "the reference engine's keep_cached=True steady state: "
                                                     "fp32 weights decoded beforehand (4-byte weights held in "
                                                     "host memory), one torch.matmul per linear, "
                                                     f"{samples[0][0]} set"}},
        "e2e": {"value": round(value, 4), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def main():
    args = parse()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if args.impl == "reference":
        return run_reference(args, rank, world)

    import torch.distributed as dist

    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        from datetime import timedelta

        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        dist.init_process_group("nccl", device_id=dev, timeout=timedelta(seconds=120))

    from polarflash_b200 import encoders
    from polarflash_b200.hadamard import BlockHadamardTransform, column_signs, effective_block
    from polarflash_b200.qweight import QWeight, group_workspace_bytes, qlinear, qlinear_group, qlinear_multi, workspace
    from polarflash_b200._lib import kernel_launches

    N = args.batch
    from polarflash_b200.parallel import shard_bounds

    strong = world > 1 and args.scaling == "strong"
    # --- encode one set per format, then replicate the packed buffers into
    # `copies` resident copies.  Strong scaling: every rank encodes the same
    # set and keeps rows [r M / N, (r + 1) M / N) of every linear (column
    # parallel; row shards slice without re-encoding).  Weak: each rank
    # encodes a full set of its own.
    base = {}
    for fmt in FORMATS:
        bits = int(fmt[3])
        for i, (name, M, K) in enumerate(LINEARS):
            seed = 1000 + i if (strong or world == 1) else 1000 + 97 * rank + i
            W = synth_weight(M, K, seed, dev)
            Wr = BlockHadamardTransform(K, 128, device=dev).forward(W)
            q, s, m = encoders.quant_g128_asym(Wr, bits)
            words = encoders.pack_g128(q, bits)
            fmt_id = {3: 2, 2: 3}[bits]
            qw = QWeight(fmt_id, M, K, words.view(torch.uint8).flatten(), s, m, effective_block(128, K),
                         column_signs(K, 128, dev))
            if strong:
                r0, r1 = shard_bounds(M, world, rank)
                qw = qw.shard_rows(r0, r1)
            base[(fmt, name)] = qw
            del W, Wr, q
    copies = []
    for c in range(args.copies):
        cp = {}
        for key, qw in base.items():
            if c == 0:
                cp[key] = qw
            else:
                cp[key] = QWeight(qw.format, qw.M, qw.K, qw.codes.clone(), qw.scales.clone(), qw.mins.clone(),
                                  qw.had_block, qw.had_signs)
        copies.append(cp)
    torch.cuda.synchronize()

    g = torch.Generator().manual_seed(7)
    kdim = {name: K for name, _, K in LINEARS}
    # the step's inputs are views into one device buffer, so the end-to-end
    # path copies them in from pinned host memory with one copy per step
    x_sizes = [N * kdim[grp[0]] for grp in SHARED]
    x_flat = torch.empty(sum(x_sizes), dtype=torch.float16, device=dev)
    xs, off = {}, 0
    for grp, n in zip(SHARED, x_sizes):
        xs[grp] = x_flat[off:off + n].view(N, kdim[grp[0]])
        xs[grp].copy_(torch.randn(N, kdim[grp[0]], generator=g).half())
        off += n
    # every linear's y [N, M] is a contiguous block of one flat buffer, which is
    # also the all-gather buffer at N GPUs and the D2H source of the e2e leg
    y_total = sum(base[(fmt, name)].M for fmt in FORMATS for name, _, _ in LINEARS)
    y_all = torch.empty(N * y_total, dtype=torch.float32, device=dev)
    outs = {}
    off = 0
    for fmt in FORMATS:
        for name, _, _ in LINEARS:
            M = base[(fmt, name)].M  # this rank's rows
            outs[(fmt, name)] = y_all[off:off + N * M].view(N, M)
            off += N * M
    keys = [(fmt, n) for fmt in FORMATS for n, _, _ in LINEARS]
    grp_of = {n: grp for grp in SHARED for n in grp}
    set_xs = [xs[grp_of[n]] for _, n in keys]
    set_outs = [outs[k] for k in keys]
    ws_need = max([group_workspace_bytes([base[k] for k in keys], N)] +
                  [group_workspace_bytes([base[(fmt, n)] for n in grp], N) for fmt in FORMATS for grp in SHARED])
    ws = workspace(dev, ws_need)  # zero-filled once; every launch leaves its counters zero
    step_bytes = sum(alg_bytes(qw, N) for qw in base.values())
    packed_bytes = sum(qw.nbytes() for qw in base.values())

    def step(cp):
        """The whole set in one call: one x' preparation launch for the four
        inputs (per format), then one GEMV launch per format over its 7 weights."""
        qlinear_group([cp[k] for k in keys], set_xs, workspace=ws, outs=set_outs)

    def step_layer(cp):
        """As a decoder layer issues them: one call per shared input (q|k|v,
        o, gate|up, down) and format."""
        for fmt in FORMATS:
            for grp in SHARED:
                qlinear_multi([cp[(fmt, n)] for n in grp], xs[grp], workspace=ws, outs=[outs[(fmt, n)] for n in grp])

    # warm-up (also compiles lazily-loaded modules)
    for _ in range(3):
        step(copies[0])
    torch.cuda.synchronize()

    stream = torch.cuda.Stream(device=dev)
    # one CUDA graph per step (per resident copy), and graphs of G consecutive
    # steps on G different copies, as a decoder captures several layers in one
    # graph: consecutive launches then overlap through programmatic dependent
    # launch (a step's weights stream in while the previous step's last CTAs
    # finish).  The timed region replays K steps as K // G group graphs and
    # K % G single-step graphs.
    G = max(1, min(args.graph_steps, len(copies), args.steps))  # at most the timed steps: one group graph
    fused = world > 1 and strong and args.gather == "peer"
    peer = None
    if fused:
        # every rank's copy of every linear's whole y, written by all ranks'
        # GEMVs (peer stores over NVLink) in place of an all-gather
        from polarflash_b200.parallel import PeerBuffer, peers_wait, qlinear_group_gather

        y_offs, off = [], PeerBuffer.HEADER
        for k in keys:
            y_offs.append(off)
            off += (4 * N * world * base[k].M + 255) // 256 * 256
        peer = PeerBuffer(off, device=dev)
        gather_out = peer.local[PeerBuffer.HEADER:off]
        set_ws = [copies[0][k] for k in keys]
        with torch.cuda.stream(stream):  # set-up outside any capture
            qlinear_group_gather(set_ws, set_xs, peer, y_offs, ws=ws, stream=stream)
            peers_wait(peer, ws, stream=stream)
        torch.cuda.synchronize()
    elif world > 1:
        # the step's outputs of every rank, rank-major (at batch 1 each
        # linear's y is the concatenation of the ranks' row shards)
        gather_buf = torch.empty(world * y_all.numel(), dtype=torch.float32, device=dev)
        gather_out = gather_buf
        with torch.cuda.stream(stream):
            dist.all_gather_into_tensor(gather_buf, y_all)  # communicator set-up before any capture
        torch.cuda.synchronize()

    def gstep(cp, gather):
        if gather and fused:  # the GEMV's own last CTA waits for the other ranks' rows
            qlinear_group_gather([cp[k] for k in keys], set_xs, peer, y_offs, ws=ws, stream=stream)
            return
        step(cp)
        if gather:
            dist.all_gather_into_tensor(gather_buf, y_all)

    # graphs of the step with the NCCL all-gather captured in them (at N GPUs)
    # and without it (the kernel-only time; the same at one GPU)
    def build(gather):
        singles, groups = [], []
        with torch.cuda.stream(stream):
            for cp in copies:
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    gstep(cp, gather)
                singles.append(gr)
            for g0 in range(0, len(copies) - G + 1, G):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    for cp in copies[g0:g0 + G]:
                        gstep(cp, gather)
                groups.append(gr)
        torch.cuda.synchronize()
        return singles, groups

    def count_launches():
        """The library's own count of the kernels one step holds (one x'
        preparation and one GEMV launch), from a capture."""
        n0 = kernel_launches()
        with torch.cuda.stream(stream):
            g1 = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g1, stream=stream):
                step(copies[0])
        return kernel_launches() - n0

    launches_per_step = count_launches()
    graphs, ggraphs = build(world > 1)
    kgraphs, kggraphs = build(False) if world > 1 else (graphs, ggraphs)
    upload_graphs(graphs + ggraphs + (kgraphs + kggraphs if world > 1 else []), stream)

    def replay(k, gl):
        gl[k % len(gl)].replay()

    def replay_steps(n, gather=True):
        """n steps: n // G group graphs, then n % G single-step graphs; with
        `gather` (at N GPUs) the graphs that hold each step's all-gather."""
        sg, gg = (graphs, ggraphs) if gather else (kgraphs, kggraphs)
        for i in range(n // G):
            gg[i % len(gg)].replay()
        for i in range(n % G):
            sg[i % len(sg)].replay()

    with torch.cuda.stream(stream):
        for k in range(args.warmup):
            replay(k, graphs)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
        clocks = Clocks(vis[local].strip() if local < len(vis) else str(local))
        clocks.start()
        t_wall0 = time.perf_counter()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record(stream)
        replay_steps(args.steps)
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1)
        # keep sampling clocks for at least ~1.5 s of the same GEMV graphs when
        # the timed region is shorter than the sampling interval allows (local
        # replays only: ranks may stop at different counts, so no collective)
        extra = 0
        while time.perf_counter() - t_wall0 < 1.5 and extra < 200000:
            for k in range(200):
                kgraphs[k % len(kgraphs)].replay()  # no collectives: the ranks' counts may differ
            extra += 200
            torch.cuda.synchronize()
        clk = clocks.stop()
        if extra:
            clk["window"] = "timed region + same-graph replays to 1.5 s"

        # kernel-only time per step: at one GPU the step holds nothing but the
        # library's launches, so it is the timed region's; at N GPUs graphs of
        # the same steps without the all-gather are timed too
        if world > 1:
            for k in range(args.warmup):
                replay(k, kgraphs)
            torch.cuda.synchronize()
            r0, r1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            r0.record(stream)
            replay_steps(args.steps, gather=False)
            r1.record(stream)
            torch.cuda.synchronize()
            ms_run = r0.elapsed_time(r1) / args.steps
        else:
            ms_run = ms / args.steps

        # the same weights issued in layer order (8 calls per step), timed alike
        # (G steps per graph as above; the step count rounded up to whole graphs)
        layer_graphs = []
        n0 = kernel_launches()
        for g0 in range(0, len(copies) - G + 1, G):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                for cp in copies[g0:g0 + G]:
                    step_layer(cp)
            layer_graphs.append(gr)
        layer_launches = (kernel_launches() - n0) // (len(layer_graphs) * G)
        upload_graphs(layer_graphs, stream)
        for k in range(max(1, args.warmup // G)):
            layer_graphs[k % len(layer_graphs)].replay()
        torch.cuda.synchronize()
        n_lg = max(1, (args.steps + G - 1) // G)
        l0, l1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        l0.record(stream)
        for k in range(n_lg):
            layer_graphs[k % len(layer_graphs)].replay()
        l1.record(stream)
        torch.cuda.synchronize()
        ms_layer = l0.elapsed_time(l1) / (n_lg * G)
        del layer_graphs, gr

        # e2e through the public API with host buffers: pinned x in, y out,
        # copies inside the timed region (graph of H2D -> GEMVs -> D2H)
        x_host = torch.empty(x_flat.numel(), dtype=torch.float16, pin_memory=True)
        x_host.copy_(x_flat.cpu())
        # at N GPUs the step's result is the gathered y of every rank's shard
        y_src = gather_out if world > 1 else y_all
        y_host = torch.empty(y_src.numel() // (4 if y_src.dtype == torch.uint8 else 1),
                             dtype=torch.float32, pin_memory=True)

        def e2e_graph(cp):
            gr = torch.cuda.CUDAGraph()
            with torch.cuda.graph(gr, stream=stream):
                x_flat.copy_(x_host, non_blocking=True)  # every input of the step, one H2D copy
                gstep(cp, world > 1)
                y_host.copy_(y_src.view(torch.float32) if y_src.dtype == torch.uint8 else y_src, non_blocking=True)
            return gr

        e2e_graphs = [e2e_graph(cp) for cp in copies[:4]]
        upload_graphs(e2e_graphs, stream)

        def e2e_step(k):
            e2e_graphs[k % len(e2e_graphs)].replay()

        for k in range(5):
            e2e_step(k)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
        q0, q1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        n_e2e = max(50, min(args.steps, 2000))
        q0.record(stream)
        for k in range(n_e2e):
            e2e_step(k)
        q1.record(stream)
        torch.cuda.synchronize()
        ms_e2e_serial = q0.elapsed_time(q1) / n_e2e
        h2d = x_host.numel() * x_host.element_size()
        d2h = y_host.numel() * 4

        # The same end-to-end steps pipelined, as a server overlaps them: graphs
        # of GE steps over two device buffer sets (inputs, outputs, gather
        # buffer).  Step i's H2D (its own pinned input) runs on a copy stream
        # once step i-2 has finished with buffer set i % 2; step i's compute
        # waits for that copy and for the D2H of step i-2; its D2H (into its own
        # pinned output) runs on a second copy stream once it is computed.  So
        # every step still copies its inputs in and its result out inside the
        # timed region, while the copies overlap the neighbouring steps.
        pipe_note, pipes = None, []
        if fused:
            pipe_note = "not pipelined: the peer-store gather has one receive buffer"
        else:
            def rebase(t, old, new):
                o = t.storage_offset() - old.storage_offset()
                return new.view(-1)[o:o + t.numel()].view(t.shape)

            x_flat2 = x_flat.clone()
            y_all2 = torch.empty_like(y_all)
            bsets = [(x_flat, set_xs, set_outs, y_all, gather_buf if world > 1 else None),
                     (x_flat2, [rebase(t, x_flat, x_flat2) for t in set_xs],
                      [rebase(t, y_all, y_all2) for t in set_outs], y_all2,
                      torch.empty_like(gather_buf) if world > 1 else None)]
            GE = G
            x_hosts = [x_host, torch.empty_like(x_host).pin_memory()]
            x_hosts[1].copy_(x_host)
            y_hosts = [torch.empty_like(y_host).pin_memory() for _ in range(GE)]
            hs, ds = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

            def pipe_graph(cps):
                gr = torch.cuda.CUDAGraph()
                with torch.cuda.graph(gr, stream=stream):
                    hs.wait_stream(stream)
                    ds.wait_stream(stream)
                    done, read = [], []
                    for i, cp in enumerate(cps):
                        xb, sx, so, yb, gb = bsets[i % 2]
                        if i >= 2:
                            hs.wait_event(done[i - 2])
                        with torch.cuda.stream(hs):
                            xb.copy_(x_hosts[i % 2], non_blocking=True)
                        stream.wait_stream(hs)
                        if i >= 2:
                            stream.wait_event(read[i - 2])
                        qlinear_group([cp[k] for k in keys], sx, workspace=ws, outs=so)
                        if gb is not None:
                            dist.all_gather_into_tensor(gb, yb)
                        ev = torch.cuda.Event()
                        ev.record(stream)
                        done.append(ev)
                        ds.wait_event(ev)
                        with torch.cuda.stream(ds):
                            y_hosts[i].copy_(gb if gb is not None else yb, non_blocking=True)
                        ev = torch.cuda.Event()
                        ev.record(ds)
                        read.append(ev)
                    stream.wait_stream(hs)
                    stream.wait_stream(ds)
                return gr

            pipes += [pipe_graph(copies[g0:g0 + GE]) for g0 in list(range(0, len(copies) - GE + 1, GE))[:2]]
            upload_graphs(pipes, stream)
            for k in range(-(-5 // GE)):
                pipes[k % len(pipes)].replay()
            torch.cuda.synchronize()
            if world > 1:
                dist.barrier()
            n_pipe = -(-n_e2e // GE)
            q0.record(stream)
            for k in range(n_pipe):
                pipes[k % len(pipes)].replay()
            q1.record(stream)
            torch.cuda.synchronize()
            ms_e2e = q0.elapsed_time(q1) / (n_pipe * GE)
            # the last step's result reached its pinned output
            _, _, _, yb, gb = bsets[(GE - 1) % 2]
            if not torch.equal(y_hosts[GE - 1], (gb if gb is not None else yb).cpu()):
                pipe_note = "pipelined outputs differ from the device's"
        if pipe_note is not None:
            ms_e2e = ms_e2e_serial

    decode = None
    if world == 1 and not args.no_decode and N == 1:
        try:
            decode = decode_rates(copies, xs, outs, ws, stream, dev, layers=32)
        except Exception as e:  # the decode extras never cost the headline line
            decode = {"error": f"{type(e).__name__}: {e}"[:300]}
        decode["what"] = ("linears of one decode step: Llama-3-8B shape (32 layers x q|k|v, o, gate|up, down) at "
                          "batch 1 for INT3 / INT2 / polar 1.75, Llama-3-70B shape (80 layers, E8 RVQ2) at batch 1 "
                          "and 32 and its 2048-token prefill (e8_rvq2_70b_prefill_2048: the linears of one layer "
                          "per graph, tensor-core GEMM; tok_s scales the layer time to 80 layers); "
                          "one resident weight copy per layer, CUDA-graph replays; attention, norms and "
                          "lm_head not included, except llama3_8b_int3_full_step_ctx512 and "
                          "llama3_8b_polar1.75_full_step_ctx2048: the whole batch-1 step "
                          "through polarflash_b200.decode (the library's RMSNorm, RoPE + cache write, attention "
                          "and SiLU kernels, fp32 KV cache at 512 / 2048 tokens, fp16 embedding and lm_head), one CUDA "
                          "graph per token; kv_attention_llama3_8b_ctx16k: the attention alone over 32 layers' "
                          "caches at 16384 tokens, fp32 and compressed (int8, 2bit, 2bit_asym) caches")

    tp_step = None
    if world > 1 and args.tp_decode:
        ms_tok = decode_tp_step(stream, dev, world)
        tp_step = {"llama3_8b_polar1.75_full_step_ctx2048": {"tok_s": round(1e3 / ms_tok, 1),
                                                             "ms_per_token": round(ms_tok, 4)},
                   "what": f"config 4 column-parallel over {world} GPUs: every projection row-sharded, one NCCL "
                           "all-gather per projection group (4 per layer) in the step's CUDA graph, the rest "
                           "replicated; max over ranks"}

    # max over ranks
    t = torch.tensor([ms, ms_run, ms_e2e, ms_layer, ms_e2e_serial], device=dev, dtype=torch.float64)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms, ms_run, ms_e2e, ms_layer, ms_e2e_serial = (float(v) for v in t.tolist())
    ms_step = ms / args.steps
    value = world * step_bytes / (ms_step / 1e3) / 1e9

    peaks = {}
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            peaks = json.load(f)
    except Exception:  # noqa: BLE001
        pass
    hbm_peak = float(peaks.get("hbm_gbs", 6650.0))
    achieved = step_bytes / (ms_run / 1e3) / 1e9
    # DRAM bytes of one step's GEMV launches, from the ncu capture recorded in
    # profiles/gemv_tma_traffic.json (its "command" reproduces it); used only
    # while that capture is of the GEMV design this build launches
    traffic, traffic_src = None, None
    try:
        with open(os.path.join(ROOT, "profiles", "gemv_tma_traffic.json")) as f:
            tj = json.load(f)
        if tj.get("kernel_design") == TRAFFIC_DESIGN:
            traffic, traffic_src = tj.get("bytes_per_step"), tj.get("command")
    except Exception:  # noqa: BLE001
        pass

    cpu = None
    if world == 1 and not args.no_cpu_baseline:
        samples = []
        for fmt in FORMATS:
            for name, M, K in LINEARS:
                qw = base[(fmt, name)]
                grp = next(gp for gp in SHARED if name in gp)
                samples.append((fmt, name, host_payload(qw), M, K, xs[grp].float().cpu().numpy()))
        y_ref = []
        gbs, secs, cores = cpu_reference_leg(None, samples, outputs=y_ref)
        cpu = {"value": round(gbs, 4), "unit": "GB/s", "cores": cores, "kind": "port", "cpu_model": cpu_model(),
               "sample": f"one pass over the 14-linear set (decode + inverse RWHT + fp32 matvec), {secs:.1f} s"}
        pairs = []
        for (fmt, name, _, _, _, _), yr in zip(samples, y_ref):
            grp = next(gp for gp in SHARED if name in gp)
            pairs.append((qlinear(base[(fmt, name)], xs[grp]).cpu().numpy(), yr))
        cpu["parity"] = parity_stats(pairs)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_step, 5), "higher_is_better": True,
            "scaling": args.scaling,  # one GPU: the same set whichever way N would grow
            "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": {"workload": WORKLOAD, "batch": N, "copies": args.copies,
                       "packed_bytes_per_step": packed_bytes, "alg_bytes_per_step": step_bytes,
                       "l2": f"{args.copies} resident copies ({args.copies * packed_bytes / 1e9:.2f} GB) cycled; "
                             "inputs > 126 MB L2",
                       "parallelism": (f"column-shard x{world}: every linear's rows split over the ranks, "
                                       "NCCL all-gather of the step's outputs in the CUDA graph"
                                       if strong else f"x{world} ranks, each a full set of its own"
                                       if world > 1 else "one GPU"),
                       "graph_steps": G},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm_peak, "unit": "GB/s",
                         "frac": round(achieved / hbm_peak, 4), "traffic": traffic,
                         "traffic_unit": "DRAM bytes per step (the step's GEMV launches, one ncu capture)",
                         "traffic_source": traffic_src,
                         "kernel": "gemv_tma_kernel (one launch per format per step, 7 weights each, after one "
                                   "xprep_frag_kernel launch); achieved = algorithmic bytes / whole step time "
                                   "(CUDA events over the timed region, preparation launch included)",
                         "peak_source": "of measured (MEASURED_PEAKS.json hbm_gbs)" if peaks else "of fallback"},
            "cpu_baseline": cpu,
            "e2e": {"value": round(world * step_bytes / (ms_e2e / 1e3) / 1e9, 2), "unit": "GB/s",
                    "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
                    "how": "public-API calls, every step: pinned x H2D, one pf_qlinear_group call over the set"
                           + ((", the GEMV storing its rows into every rank's buffer (peer stores), peer wait"
                               if fused else ", NCCL all-gather of the column shards") if world > 1 else "")
                           + ", y D2H into the step's own pinned buffer; "
                           + (f"pipelined: CUDA graphs of {G} steps over two device buffer sets, H2D and D2H on "
                              "two copy streams overlapping the neighbouring steps' kernels"
                              if pipe_note is None else f"one CUDA graph per step ({pipe_note})"),
                    "serial": {"value": round(world * step_bytes / (ms_e2e_serial / 1e3) / 1e9, 2),
                               "how": "one CUDA graph per step: H2D, the call, D2H, each step after the last"}},
            "layer_order": {"ms_per_step": round(ms_layer, 5),
                            "GB_s": round(world * step_bytes / (ms_layer / 1e3) / 1e9, 2),
                            "frac": round(step_bytes / (ms_layer / 1e3) / 1e9 / hbm_peak, 4),
                            "launches_per_step": layer_launches,
                            "how": "the same weights as 8 calls per step, one per shared input (q|k|v, o, "
                                   "gate|up, down) and format, as a decoder layer issues them"},
            "allgather_us_per_step": (round((ms_step - ms_run) * 1e3, 2) if world > 1 else None),
            "gather": (("peer stores from the GEMV over NVLink + flag wait (pf_qlinear_group_gather)" if fused
                        else "NCCL all-gather captured in the graph") if world > 1 else None),
            "gpu_launches": launches_per_step * args.steps,
            "decode_tok_s": decode,
            "decode_tp": tp_step,
            "clocks": clk,
        }
        print(json.dumps(line), flush=True)
    # graphs that hold NCCL calls are released before the process group
    torch.cuda.synchronize()
    for gl in (graphs, ggraphs, kgraphs, kggraphs, e2e_graphs, pipes):
        gl.clear()
    import gc

    gc.collect()
    if world > 1:
        dist.barrier()
        if peer is not None:
            peer.close()
            dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
