"""One fused linear on synthetic weights, launched a few times: the small case
used for single-kernel ncu captures of the library's kernels.

    python polar-flash_b200/profile_case.py --fmt int3_g128 --M 14336 --K 4096 --N 1 --iters 3
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
    ap.add_argument("--copies", type=int, default=1,
                    help="resident copies of the weight cycled by the timed calls (more than L2 holds: 126 MB)")
    a = ap.parse_args()
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
        e0.record()
        for i in range(reps):
            qlinear(qws[i % len(qws)], x, out=out)
        e1.record()
        torch.cuda.synchronize()
        us = e0.elapsed_time(e1) * 1e3 / reps
        flops = 2.0 * a.M * a.K * a.N
        print(f"time {us:.1f} us  {flops / us / 1e6:.1f} TFLOP/s  {qw.nbytes() / us / 1e3:.1f} GB/s packed")


if __name__ == "__main__":
    main()
