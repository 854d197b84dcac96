"""One fused linear on synthetic weights, launched a few times: the small case
used for single-kernel ncu captures of the library's kernels.

    python polar-flash_b200/profile_case.py --fmt int3_g128 --M 14336 --K 4096 --N 1 --iters 3

With --set, the Llama-3-8B linear set (q/k/v/o/gate/up/down at INT3 and INT2
group-128, RWHT 128, batch --N) as ONE pf_qlinear_group call, as bench.py
issues it (--layer-order: one call per shared input and format instead),
cycling --copies resident copies of the set:

    python polar-flash_b200/profile_case.py --set --copies 4 --iters 6 --time

With --attention, the decode attention over a KV cache instead: one new
token, 32 query / 8 KV heads of 128 (Llama-3-8B), --ctx cached positions of
random rows, for each listed cache mode (fp32 through pf_decode_attention,
int8 / 2bit / 2bit_asym through pf_decode_attention_compressed):

    python polar-flash_b200/profile_case.py --attention fp32,int8,2bit --ctx 16384 --iters 1

With --decode-step, a whole batch-1 decode step of a Llama-3-8B-shaped stack
(PFlashDecoder, --layers layers, recursive polar 1.75 bpw or INT3 g128 linears
via --fmt, fp32 KV cache at --ctx positions, fp16 embedding and lm_head),
captured once as a CUDA graph and replayed --iters times:

    python polar-flash_b200/profile_case.py --decode-step --fmt polar_recursive --layers 32 --ctx 2048 --iters 3
"""
import argparse
import os
import sys

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))

import torch  # noqa: E402

from polarflash_b200 import UnifiedQuantizer, qlinear  # noqa: E402


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--fmt", default="int3_g128")
    ap.add_argument("--M", type=int, default=14336)
    ap.add_argument("--K", type=int, default=4096)
    ap.add_argument("--N", type=int, default=1)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--time", action="store_true", help="report device time per call (CUDA events)")
    ap.add_argument("--graph", action="store_true", help="with --time: replay the calls as one CUDA graph "
                                                         "(no host launch overhead between calls)")
    ap.add_argument("--copies", type=int, default=1,
                    help="resident copies of the weight cycled by the timed calls (more than L2 holds: 126 MB)")
    ap.add_argument("--attention", default=None, help="comma-separated KV cache modes: run decode attention")
    ap.add_argument("--ctx", type=int, default=16384, help="cached positions (--attention)")
    ap.add_argument("--set", action="store_true", help="the Llama-3-8B linear set at INT3 + INT2 in one call")
    ap.add_argument("--layer-order", action="store_true", help="with --set: one call per shared input")
    ap.add_argument("--decode-step", action="store_true", help="a whole batch-1 decode step (PFlashDecoder)")
    ap.add_argument("--layers", type=int, default=32, help="layers of the --decode-step stack")
    a = ap.parse_args()
    if a.attention:
        return attention_case(a)
    if a.set:
        return set_case(a)
    if a.decode_step:
        return decode_step_case(a)
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    W = torch.randn(a.M, a.K, generator=g, device=dev) * 0.02
    qw, _ = UnifiedQuantizer(backend=a.fmt, hadamard_block_size=128).quantize_to_qweight(W)
    del W
    x = torch.randn(a.N, a.K, generator=g, device=dev).half()
    for _ in range(a.iters):
        y = qlinear(qw, x)
    torch.cuda.synchronize()
    print(f"{a.fmt} {a.M}x{a.K} N={a.N}: packed {qw.nbytes()} B, y[0,:4] = {y[0, :4].tolist()}")
    if a.time:
        from polarflash_b200.qweight import QWeight

        qws = [qw] + [QWeight(qw.format, qw.M, qw.K, qw.codes.clone(),
                              qw.scales.clone() if qw.scales is not None else None,
                              qw.mins.clone() if qw.mins is not None else None, qw.had_block, qw.had_signs,
                              qw.tensor_scale, list(qw.params)) for _ in range(a.copies - 1)]
        out = torch.empty_like(y)
        for i in range(len(qws)):
            qlinear(qws[i], x, out=out)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(5, a.iters)
        if a.graph:
            st = torch.cuda.Stream()
            st.wait_stream(torch.cuda.current_stream())
            g = torch.cuda.CUDAGraph()
            with torch.cuda.stream(st):
                qlinear(qws[0], x, out=out)  # the workspace exists before the capture
                st.synchronize()
                with torch.cuda.graph(g, stream=st):
                    for i in range(reps):
                        qlinear(qws[i % len(qws)], x, out=out)
            g.replay()
            torch.cuda.synchronize()
            e0.record()
            g.replay()
            e1.record()
        else:
            e0.record()
            for i in range(reps):
                qlinear(qws[i % len(qws)], x, out=out)
            e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        flops = 2.0 * a.M * a.K * a.N
        print(f"time {us:.1f} us  {flops / us / 1e6:.1f} TFLOP/s  {qw.nbytes() / us / 1e3:.1f} GB/s packed")


LINEARS = [("q", 4096, 4096), ("k", 1024, 4096), ("v", 1024, 4096), ("o", 4096, 4096),
           ("gate", 14336, 4096), ("up", 14336, 4096), ("down", 4096, 14336)]
SHARED = [("q", "k", "v"), ("o",), ("gate", "up"), ("down",)]


def set_case(a):
    from polarflash_b200.qweight import QWeight, qlinear_group

    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    base = {}
    for fmt in ("int3_g128", "int2_g128"):
        for name, M, K in LINEARS:
            W = torch.randn(M, K, generator=g, device=dev) * 0.02
            base[(fmt, name)], _ = UnifiedQuantizer(backend=fmt, hadamard_block_size=128).quantize_to_qweight(W)
            del W
    copies = [base] + [{k: QWeight(q.format, q.M, q.K, q.codes.clone(), q.scales.clone(), q.mins.clone(),
                                   q.had_block, q.had_signs) for k, q in base.items()} for _ in range(a.copies - 1)]
    kdim = {n: K for n, _, K in LINEARS}
    xs = {grp: torch.randn(a.N, kdim[grp[0]], generator=g, device=dev).half() for grp in SHARED}
    keys = list(base.keys())
    xl = [xs[next(gp for gp in SHARED if n in gp)] for _, n in keys]
    outs = [torch.empty(a.N, base[k].M, device=dev) for k in keys]

    def call(i):
        cp = copies[i % len(copies)]
        if not a.layer_order:
            qlinear_group([cp[k] for k in keys], xl, outs=outs)
            return
        for fmt in ("int3_g128", "int2_g128"):
            for grp in SHARED:
                idx = [keys.index((fmt, n)) for n in grp]
                qlinear_group([cp[keys[i]] for i in idx], [xl[i] for i in idx], outs=[outs[i] for i in idx])

    for i in range(a.iters):
        call(i)
    torch.cuda.synchronize()
    nbytes = sum(q.nbytes() + a.N * q.K * 2 + a.N * q.M * 4 for q in base.values())
    print(f"linear set N={a.N}: {nbytes} algorithmic bytes per call, y[0][0,:4] = {outs[0][0, :4].tolist()}")
    if a.time:
        reps = max(5, a.iters)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for i in range(reps):
            call(i)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        print(f"time {us:.1f} us per set call  {nbytes / us / 1e3:.1f} GB/s")


def attention_case(a):
    import ctypes
    import math

    from polarflash_b200 import _lib
    from polarflash_b200.kv_cache import KV_MODES, kv_row_bytes

    L = _lib.load()
    dev = torch.device("cuda")
    g = torch.Generator(device=dev).manual_seed(0)
    nh, nkv, hd, ms = 32, 8, 128, a.ctx
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    st = ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
    q = torch.randn(nh * hd, generator=g, device=dev)
    out = torch.empty(nh * hd, device=dev)
    pos = torch.tensor([ms - 1], dtype=torch.long, device=dev)
    aws = torch.empty(int(L.pf_decode_attention_workspace_size(nh, hd, ms)), dtype=torch.uint8, device=dev)
    for mode in a.attention.split(","):
        rb = 4 * hd if mode == "fp32" else kv_row_bytes(mode, hd)

        def rows():
            if mode == "fp32":
                return torch.randn(ms, nkv, hd, generator=g, device=dev).view(torch.uint8)
            return torch.randint(0, 256, (ms, nkv, rb), generator=g, device=dev, dtype=torch.uint8)

        layers = [(rows(), rows(), torch.rand(2, ms, nkv, generator=g, device=dev) * 0.01,
                   torch.rand(2, ms, nkv, generator=g, device=dev) if mode == "2bit_asym" else None)
                  for _ in range(max(1, a.copies))]

        def call(i):
            kc, vc, sc, zr = layers[i % len(layers)]
            if mode == "fp32":
                _lib.check(L.pf_decode_attention(p(q), p(kc), p(vc), p(pos), p(out), nh, nkv, hd, ms,
                                                 1.0 / math.sqrt(hd), p(aws), aws.numel(), st))
            else:
                _lib.check(L.pf_decode_attention_compressed(
                    p(q), p(kc), p(sc[0]), p(zr[0] if zr is not None else None), p(vc), p(sc[1]),
                    p(zr[1] if zr is not None else None), p(pos), p(out), nh, nkv, hd, ms, KV_MODES[mode],
                    1.0 / math.sqrt(hd), p(aws), aws.numel(), st))

        for i in range(a.iters):
            call(i)
        torch.cuda.synchronize()
        print(f"attention {mode} ctx {ms}: out[:4] = {out[:4].tolist()}")
        if a.time:
            reps = max(20, a.iters)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for i in range(reps):
                call(i)
            e1.record()
            torch.cuda.synchronize()
            us = e0.elapsed_time(e1) * 1e3 / reps
            nb = 2 * ms * nkv * (rb + (0 if mode == "fp32" else 4) + (4 if mode == "2bit_asym" else 0))
            print(f"time {us:.1f} us  {nb / us / 1e3:.1f} GB/s of cache rows")


def decode_step_case(a):
    from polarflash_b200.decode import DecoderLayer, PFlashDecoder

    dev = torch.device("cuda")
    H, V, FF = 4096, 128256, 14336
    shapes = {"q": (4096, H), "k": (1024, H), "v": (1024, H), "o": (H, 4096), "gate": (FF, H), "up": (FF, H),
              "down": (H, FF)}
    g = torch.Generator(device=dev).manual_seed(0)
    base = {}
    for n, (M, K) in shapes.items():
        W = torch.randn(M, K, generator=g, device=dev) * 0.02
        base[n], _ = UnifiedQuantizer(backend=a.fmt, hadamard_block_size=128).quantize_to_qweight(W)
        del W
    from polarflash_b200.qweight import QWeight

    def copy(q):
        return QWeight(q.format, q.M, q.K, q.codes.clone(), q.scales.clone() if q.scales is not None else None,
                       q.mins.clone() if q.mins is not None else None, q.had_block, q.had_signs, q.tensor_scale,
                       list(q.params))
    ones = torch.ones(H, device=dev)
    layers = []
    for li in range(a.layers):
        w = base if li == 0 else {n: copy(q) for n, q in base.items()}
        layers.append(DecoderLayer(w["q"], w["k"], w["v"], w["o"], w["gate"], w["up"], w["down"], ones, ones))
    cfg = dict(hidden_size=H, num_attention_heads=32, num_key_value_heads=8, intermediate_size=FF, vocab_size=V,
               rope_theta=500000.0, rms_norm_eps=1e-5)
    embed = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    head = (torch.randn(V, H, generator=g, device=dev) * 0.02).half()
    dec = PFlashDecoder(cfg, layers, embed, ones, head, max_seq=a.ctx + 1)
    st = torch.cuda.Stream()
    with torch.cuda.stream(st):
        dec.forward(torch.tensor([1], device=dev))
        dec.length = a.ctx
        dec.capture(st)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        dec._graph.replay()
        e0.record(st)
        for _ in range(a.iters):
            dec._graph.replay()
        e1.record(st)
    torch.cuda.synchronize()
    print(f"decode step {a.fmt}, {a.layers} layers, ctx {a.ctx}: {e0.elapsed_time(e1) / a.iters:.3f} ms per token")


if __name__ == "__main__":
    main()
