"""Generate the golden fixtures in this folder by running the reference itself.

Run in a checkout that has the reference POLAR-FLASH sources (read-only) at
``$POLARFLASH_REF`` (required):

    POLARFLASH_REF=/path/to/POLAR-FLASH python tests/golden/make_golden.py

Every array written here comes out of the reference's own Python functions on
seeded inputs; the tests compare the CPU oracle (and, on a GPU, the CUDA
library) against these files.  The GPU machines never read the reference.
"""
import json
import os
import sys

import numpy as np
import torch

REF = os.environ.get("POLARFLASH_REF")
if not REF or not os.path.isdir(REF):
    sys.exit("set POLARFLASH_REF to a checkout of the reference POLAR-FLASH sources")
OUT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, REF)

from polarflash_quant.bitpacking import (  # noqa: E402
    pack_int2, pack_int3, pack_int4, unpack_int2, unpack_int3, unpack_int4,
)
from polarflash_quant.transforms.hadamard import BlockHadamardTransform  # noqa: E402
from polarflash_quant.unified_quantizer import UnifiedQuantizer  # noqa: E402
from polarflash_quant.polar.polar_quant import RecursivePolarQuant  # noqa: E402
from polarflash_quant.lattice.e8_lattice import generate_e8_roots  # noqa: E402
from polarflash_core.formats.pflash_format import PFlashWriter  # noqa: E402
from polarflash_rt.cuda.native_kernels import NativeLowBitCUDAEngine  # noqa: E402


def _bytes_arr(b):
    return np.frombuffer(bytes(b), np.uint8).copy()


def bitpack():
    g = torch.Generator().manual_seed(7)
    out = {}
    for n in (240, 241, 1000):
        v4 = torch.randint(-8, 8, (n,), generator=g, dtype=torch.int8)
        v2 = torch.randint(0, 4, (n,), generator=g, dtype=torch.uint8)
        v3 = torch.randint(0, 8, (n,), generator=g, dtype=torch.uint8)
        p4, p2, p3 = pack_int4(v4), pack_int2(v2), pack_int3(v3)
        out[f"v4_{n}"] = v4.numpy()
        out[f"v2_{n}"] = v2.numpy()
        out[f"v3_{n}"] = v3.numpy()
        out[f"p4_{n}"] = _bytes_arr(p4)
        out[f"p2_{n}"] = _bytes_arr(p2)
        out[f"p3_{n}"] = _bytes_arr(p3)
        out[f"u4_{n}"] = unpack_int4(p4, n).numpy()
        out[f"u2_{n}"] = unpack_int2(p2, n).numpy()
        out[f"u3_{n}"] = unpack_int3(p3, n).numpy()
    np.savez_compressed(os.path.join(OUT, "bitpack.npz"), **out)


def hadamard():
    out = {}
    cases = [(128, 128), (4096, 128), (500, 512), (11008, 512), (1000, 128), (129, 128), (768, 512)]
    for K, req in cases:
        bht = BlockHadamardTransform(in_features=K, block_size=req, seed=42)
        signs = [bht.signs.numpy()] * bht.num_full_blocks + [s.numpy() for _, s in bht.rem_blocks]
        x = torch.randn(3, K, generator=torch.Generator().manual_seed(K + req))
        key = f"{K}_{req}"
        out[f"block_{key}"] = np.array(bht.block_size)
        out[f"signs_{key}"] = np.concatenate(signs).astype(np.float32)
        out[f"x_{key}"] = x.numpy()
        out[f"fwd_{key}"] = bht.forward(x).numpy()
        out[f"inv_{key}"] = bht.inverse(x).numpy()
    np.savez_compressed(os.path.join(OUT, "hadamard.npz"), **out)


def unified_int():
    out = {}
    meta_all = {}
    for (M, K, hb) in [(64, 128, 512), (96, 512, 128), (32, 1024, 512)]:
        g = torch.Generator().manual_seed(M * 1000 + K)
        W = torch.randn(M, K, generator=g) * 0.05
        x = torch.randn(2, K, generator=g)
        for be in ("int4", "int3", "int2", "polar"):
            uq = UnifiedQuantizer(backend=be, hadamard_block_size=hb, apply_hadamard=True)
            payload, meta, w_hat = uq.quantize(W, name=f"t_{be}")
            deq = UnifiedQuantizer.dequantize(payload, [M, K], meta["dtype"], meta)
            key = f"{be}_{M}x{K}_h{hb}"
            out[f"payload_{key}"] = _bytes_arr(payload)
            out[f"what_{key}"] = w_hat.numpy()
            out[f"deq_{key}"] = deq.numpy()
            out[f"x_{key}"] = x.numpy()
            out[f"y_{key}"] = torch.matmul(x, deq.t()).numpy()
            meta_all[key] = {k: v for k, v in meta.items() if isinstance(v, (int, float, str, bool, list))}
        out[f"W_{M}x{K}_h{hb}"] = W.numpy()
    np.savez_compressed(os.path.join(OUT, "unified.npz"), **out)
    with open(os.path.join(OUT, "unified_meta.json"), "w") as f:
        json.dump(meta_all, f, indent=1, sort_keys=True)


def polar_recursive():
    out = {}
    meta_all = {}
    cases = [(8, 1.75, 64, 256), (8, 2.0, 64, 256), (8, 4.0, 16, 128), (2, 2.0, 32, 64),
             (4, 2.0, 32, 64), (16, 2.0, 32, 64), (8, 1.75, 128, 1024)]
    for d, bpw, M, K in cases:
        g = torch.Generator().manual_seed(int(d * 100 + bpw * 10 + M))
        W = torch.randn(M, K, generator=g) * 0.02
        rpq = RecursivePolarQuant(block_size=d)
        if d == 8:
            bht = BlockHadamardTransform(in_features=K, block_size=128, seed=42)
            Wr = bht.forward(W)
        else:
            Wr = W
        packed, meta = rpq.encode_packed(Wr, target_bpw=bpw)
        dec = rpq.decode_packed(packed, meta)
        key = f"d{d}_b{bpw}_{M}x{K}"
        out[f"W_{key}"] = W.numpy()
        out[f"Wrot_{key}"] = Wr.numpy()
        out[f"packed_{key}"] = _bytes_arr(packed)
        out[f"dec_{key}"] = dec.numpy()
        meta_all[key] = {k: v for k, v in meta.items() if k != "orig_shape"}
        meta_all[key]["rotated"] = d == 8
    allocs = {}
    for d in (2, 4, 8, 16):
        for bpw in (1.75, 2.0, 2.5, 3.0, 4.0):
            allocs[f"{d}_{bpw}"] = RecursivePolarQuant(block_size=d).compute_adaptive_bit_allocation(bpw)
    meta_all["_allocs"] = allocs
    np.savez_compressed(os.path.join(OUT, "polar_recursive.npz"), **out)
    with open(os.path.join(OUT, "polar_recursive_meta.json"), "w") as f:
        json.dump(meta_all, f, indent=1, sort_keys=True)


def e8():
    np.savez_compressed(os.path.join(OUT, "e8_roots.npz"), roots=generate_e8_roots().numpy())


def native_fallback():
    """The reference's NativeLowBitCUDAEngine maths (native_kernels.py:415-576) on
    the reference tests' own seeded shapes; without a usable driver it runs the
    torch fallback, which is the definition of the op."""
    eng = NativeLowBitCUDAEngine()
    out = {}
    torch.manual_seed(42)
    M, K = 64, 128
    raw = torch.randint(-8, 8, (M, K), dtype=torch.int8)
    u4 = (raw + 8).to(torch.uint8)
    packed = (u4[:, 0::2] | (u4[:, 1::2] << 4)).contiguous()
    scales = (torch.rand(M) * 0.2 + 0.05).float()
    x = torch.randn(K, dtype=torch.float32)
    out.update(i4_packed=packed.numpy(), i4_scales=scales.numpy(), i4_x=x.numpy(),
               i4_y=eng.gemv_int4(x, packed, scales, M, K).numpy())
    torch.manual_seed(123)
    M, K = 32, 64
    raw2 = torch.randint(0, 4, (M, K), dtype=torch.uint8)
    packed2 = (raw2[:, 0::4] | (raw2[:, 1::4] << 2) | (raw2[:, 2::4] << 4) | (raw2[:, 3::4] << 6)).contiguous()
    scales2 = torch.ones(M, dtype=torch.float32) * 0.5
    x2 = torch.randn(K, dtype=torch.float32)
    out.update(i2_packed=packed2.numpy(), i2_scales=scales2.numpy(), i2_x=x2.numpy(),
               i2_y=eng.gemv_int2(x2, packed2, scales2, M, K).numpy())
    torch.manual_seed(777)
    B, M, K = 4, 32, 64
    raw3 = torch.randint(-8, 8, (M, K), dtype=torch.int8)
    u43 = (raw3 + 8).to(torch.uint8)
    packed3 = (u43[:, 0::2] | (u43[:, 1::2] << 4)).contiguous()
    scales3 = torch.ones(M, dtype=torch.float32) * 0.1
    X = torch.randn(B, K, dtype=torch.float32)
    out.update(g4_packed=packed3.numpy(), g4_scales=scales3.numpy(), g4_X=X.numpy(),
               g4_Y=eng.gemm_int4(X, packed3, scales3, M, K).numpy())
    np.savez_compressed(os.path.join(OUT, "native.npz"), **out)


def container():
    """A small .pflash written by the reference PFlashWriter
    (polarflash_core/formats/pflash_format.py:26-157)."""
    w = PFlashWriter()
    w.set_metadata({"hidden_size": 256, "num_layers": 1, "backend": "mixed"})
    g = torch.Generator().manual_seed(99)
    W1 = torch.randn(64, 256, generator=g) * 0.02
    payload, meta, _ = UnifiedQuantizer(backend="int4", hadamard_block_size=128).quantize(W1, "q")
    w.add_tensor("model.layers.0.self_attn.q_proj.weight", payload, [64, 256], meta["dtype"], meta)
    rpq = RecursivePolarQuant(block_size=8)
    W2 = torch.randn(32, 256, generator=g) * 0.02
    pb, pm = rpq.encode_packed(W2, target_bpw=1.75)
    w.add_tensor("model.layers.0.mlp.up_proj.weight", pb, [32, 256], "polar_recursive", pm)
    nb = torch.randn(256, generator=g)
    w.add_tensor("model.norm.weight", nb.half().numpy().tobytes(), [256], "fp16", {"dtype": "fp16"})
    w.save(os.path.join(OUT, "small.pflash"))
    x = torch.randn(3, 256, generator=g)
    np.savez_compressed(os.path.join(OUT, "small_pflash_io.npz"), x=x.numpy(),
                        W_q_hat=UnifiedQuantizer.dequantize(payload, [64, 256], meta["dtype"], meta).numpy(),
                        W_up_hat=rpq.decode_packed(pb, pm).numpy())


if __name__ == "__main__":
    torch.set_num_threads(4)
    bitpack()
    hadamard()
    unified_int()
    polar_recursive()
    e8()
    native_fallback()
    container()
    print("golden fixtures written to", OUT)
