"""Times the reference's own CPU engine beside the oracle port, on this host.

    POLARFLASH_REF=/path/to/POLAR-FLASH python oracle/time_reference_engine.py [--iters 5]

Measurement script, not part of the library: it imports the reference
package (read-only, from $POLARFLASH_REF) and runs
PFlashCPUEngine.forward_layer (polarflash_rt/cpu/engine.py:187-193) over a
.pflash archive written by the reference's own UnifiedQuantizer and
PFlashWriter, in both keep_cached modes:

  keep_cached=True   the first call decodes (unpack -> scale -> inverse RWHT,
                     unified_quantizer.py:242-324) and caches the fp32
                     weight; later calls are one torch.matmul
                     (cpu/engine.py:58-96);
  keep_cached=False  every call decodes again, then multiplies.

Beside it, the oracle port (oracle.linear: the C restatement of the same
decode + inverse RWHT + matvec) on the same payload.  Weights: two
Llama-3-8B linear shapes (q 4096 x 4096, down 4096 x 14336), ~N(0, 0.02^2)
with 0.1 % outliers at +-20 sigma, block-128 RWHT, the reference's per-tensor
INT3 and INT2 formats (its engine has no group-128 decoder); x is one fp16
~N(0, 1) row.  Rates are packed payload bytes per second of call time, with
every host core (torch and OpenMP threads = os.cpu_count()).  Prints one
JSON line per (format, shape, mode) and the CPU model string.
"""
import argparse
import json
import os
import sys
import tempfile
import time

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("POLARFLASH_REF")
if not REF or not os.path.isdir(REF):
    sys.exit("set POLARFLASH_REF to a checkout of the reference POLAR-FLASH sources")
sys.path[:0] = [os.path.dirname(HERE), REF]

import oracle  # noqa: E402
from polarflash_core.formats.pflash_format import PFlashWriter  # noqa: E402
from polarflash_quant.unified_quantizer import UnifiedQuantizer  # noqa: E402
from polarflash_rt.cpu.engine import PFlashCPUEngine  # noqa: E402

SHAPES = [("q_proj", 4096, 4096), ("down_proj", 4096, 14336)]
FORMATS = ["int3", "int2"]


def cpu_model():
    with open("/proc/cpuinfo") as f:
        for line in f:
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    return "unknown"


def weight(M, K, seed):
    g = torch.Generator().manual_seed(seed)
    w = torch.randn(M, K, generator=g) * 0.02
    n = max(1, (M * K) // 1000)
    pos = torch.randperm(M * K, generator=g)[:n]
    sign = torch.where(torch.rand(n, generator=g) < 0.5, -1.0, 1.0)
    w.view(-1)[pos] = sign * 0.4
    return w.half().float()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--iters", type=int, default=5)
    args = ap.parse_args()
    cores = os.cpu_count() or 1
    torch.set_num_threads(cores)
    oracle.set_num_threads(cores)
    model = cpu_model()
    with tempfile.TemporaryDirectory() as tmp:
        path = os.path.join(tmp, "sample.pflash")
        writer = PFlashWriter()
        payloads = {}
        for fmt in FORMATS:
            q = UnifiedQuantizer(backend=fmt, hadamard_block_size=128)
            for i, (name, M, K) in enumerate(SHAPES):
                payload, meta, _ = q.quantize(weight(M, K, 100 + i), name=f"{fmt}.{name}")
                writer.add_tensor(f"{fmt}.{name}", payload, [M, K], meta["dtype"], meta)
                payloads[(fmt, name)] = (payload, meta)
        writer.save(path)
        for fmt in FORMATS:
            for name, M, K in SHAPES:
                payload, meta = payloads[(fmt, name)]
                nbytes = len(payload)
                x = torch.randn(1, K, generator=torch.Generator().manual_seed(7)).half().float()
                rows = []
                for keep in (True, False):
                    eng = PFlashCPUEngine(path, keep_cached=keep)
                    t0 = time.perf_counter()
                    eng.forward_layer(f"{fmt}.{name}", x)
                    first = time.perf_counter() - t0
                    t0 = time.perf_counter()
                    for _ in range(args.iters):
                        eng.forward_layer(f"{fmt}.{name}", x)
                    steady = (time.perf_counter() - t0) / args.iters
                    eng.reclaim_memory()
                    rows.append((f"reference keep_cached={keep}", first, steady))
                oracle.linear(fmt, payload, M, K, meta, x.numpy())
                t0 = time.perf_counter()
                for _ in range(args.iters):
                    oracle.linear(fmt, payload, M, K, meta, x.numpy())
                port = (time.perf_counter() - t0) / args.iters
                rows.append(("oracle port", port, port))
                for impl, first, steady in rows:
                    print(json.dumps({"impl": impl, "format": fmt, "linear": name, "M": M, "K": K,
                                      "payload_bytes": nbytes, "first_call_ms": round(first * 1e3, 2),
                                      "steady_ms": round(steady * 1e3, 3),
                                      "steady_GBps": round(nbytes / steady / 1e9, 4),
                                      "cores": cores, "cpu_model": model}), flush=True)


if __name__ == "__main__":
    main()
