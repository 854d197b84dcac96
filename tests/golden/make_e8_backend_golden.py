"""Golden vectors for UnifiedQuantizer's "e8" backend, from the reference's
own code (polarflash_quant/unified_quantizer.py:180-192 with
E8LatticeQuantizer and E8ResidualVectorQuantizer,
polarflash_quant/lattice/e8_lattice.py:52-232).

    POLARFLASH_REF=/path/to/POLAR-FLASH python tests/golden/make_e8_backend_golden.py

For e8_stages 1, 2 and 3, with and without the Hadamard pre-rotation, on
seeded weights (32 x 256, randn * 0.02, plus one 45 x 203 weight whose block
count needs a padded tail): the fp16 payload, the quant_meta and the
reference dequantize output.  Also quantize_e8 on seeded 8-vectors with hand
made ties (coordinates at +-0.5, odd-sum D8 roundings).  Needs the reference
sources at $POLARFLASH_REF (required); the GPU machines only read the .npz.
"""
import json
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("POLARFLASH_REF")
if not REF or not os.path.isdir(REF):
    sys.exit("set POLARFLASH_REF to a checkout of the reference POLAR-FLASH sources")
sys.path.insert(0, REF)

from polarflash_quant.lattice.e8_lattice import quantize_e8  # noqa: E402
from polarflash_quant.unified_quantizer import UnifiedQuantizer  # noqa: E402


def main():
    out, metas = {}, {}
    g = torch.Generator().manual_seed(3)
    weights = {"w32x256": torch.randn(32, 256, generator=g) * 0.02,
               "w45x203": torch.randn(45, 203, generator=g) * 0.05}
    for wname, w in weights.items():
        out[wname] = w.numpy()
        for stages in (1, 2, 3):
            for had in (True, False):
                q = UnifiedQuantizer(backend="e8", e8_stages=stages, apply_hadamard=had, hadamard_block_size=128)
                payload, meta, w_hat = q.quantize(w, name=wname)
                key = f"{wname}_s{stages}_h{int(had)}"
                out[key + "_payload"] = np.frombuffer(payload, np.uint8).copy()
                out[key + "_what"] = w_hat.numpy()
                out[key + "_deq"] = UnifiedQuantizer.dequantize(payload, list(w.shape), meta["dtype"], meta).numpy()
                metas[key] = meta
    x = torch.randn(4096, 8, generator=g) * 1.5
    x[:64] = torch.round(x[:64] * 2) / 2  # exact half-integers: rounding ties
    x[64:128] = torch.round(x[64:128]) + torch.tensor([0.5, 0, 0, 0, 0, 0, 0, 0])
    out["qe8_x"] = x.numpy()
    out["qe8_y"] = quantize_e8(x).numpy()
    np.savez_compressed(os.path.join(HERE, "e8_backend.npz"), **out)
    with open(os.path.join(HERE, "e8_backend_meta.json"), "w") as f:
        json.dump(metas, f, indent=1, sort_keys=True, default=float)
    print("wrote e8_backend.npz", len(metas), "cases")


if __name__ == "__main__":
    main()
