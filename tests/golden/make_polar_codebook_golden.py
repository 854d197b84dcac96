"""Golden vectors for recursive polar with learned angle codebooks, from the
reference's own RecursivePolarQuant (polarflash_quant/polar/polar_quant.py):
fit_codebooks (274-300), encode_packed with codebook codes (381-487) and
decode_packed with codebook angles (489-575).

    POLARFLASH_REF=/path/to/POLAR-FLASH python tests/golden/make_polar_codebook_golden.py

Cases (name: block size, angle_bits, target bpw, train / test shapes):
  ref_test  the reference's own test (seed 101, d 8, 2 angle bits, 2.0 bpw,
            train 128 x 128, test 64 x 64, 10 Lloyd iterations);
  d8_b4     d 8, 4 angle bits (16-entry codebooks, codes wider than the
            1-3 bit fields), 1.75 bpw (14-bit blocks, the bit-stream path);
  d4_b3     d 4, 3 angle bits, 2.0 bpw (one byte per block).
Stores the train / test weights, the codebooks, the payload, its meta and the
reference decode.  Needs the reference sources at $POLARFLASH_REF (required);
the GPU machines only read the .npz.
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

from polarflash_quant.polar.polar_quant import RecursivePolarQuant  # noqa: E402

CASES = {
    # name: (d, angle_bits, bpw, train shape, test shape, iters, seed)
    "ref_test": (8, 2, 2.0, (128, 128), (64, 64), 10, 101),
    "d8_b4": (8, 4, 1.75, (64, 256), (48, 256), 15, 7),
    "d4_b3": (4, 3, 2.0, (64, 64), (32, 64), 15, 11),
}


def main():
    out, metas = {}, {}
    for name, (d, ab, bpw, tr, te, iters, seed) in CASES.items():
        torch.manual_seed(seed)
        train = torch.randn(*tr)
        test = torch.randn(*te)
        rpq = RecursivePolarQuant(block_size=d, norm_bits=4, angle_bits=ab)
        rpq.fit_codebooks(train, iters=iters)
        packed, meta = rpq.encode_packed(test, target_bpw=bpw)
        recon = rpq.decode_packed(packed, meta)
        out[f"{name}_train"] = train.numpy()
        out[f"{name}_test"] = test.numpy()
        for lvl, cb in enumerate(rpq.learned_codebooks):
            out[f"{name}_cb{lvl}"] = cb.numpy().astype(np.float32)
        out[f"{name}_payload"] = np.frombuffer(packed, np.uint8).copy()
        out[f"{name}_recon"] = recon.numpy()
        metas[name] = {"block_size": d, "angle_bits": ab, "bpw": bpw, "iters": iters,
                       "levels": len(rpq.learned_codebooks),
                       **{k: meta[k] for k in ("alloc", "r_scale", "num_blocks", "pad_len", "orig_shape",
                                              "has_learned_codebooks")}}
    np.savez_compressed(os.path.join(HERE, "polar_codebooks.npz"), **out)
    with open(os.path.join(HERE, "polar_codebooks_meta.json"), "w") as f:
        json.dump(metas, f, indent=1, sort_keys=True)
    print("wrote polar_codebooks.npz", sorted(metas))


if __name__ == "__main__":
    main()
