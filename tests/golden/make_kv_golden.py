"""Golden vectors for the compressed KV cache, from the reference's own
CompressedKVCache (polarflash_rt/kv_cache/compressed_kv.py).

    POLARFLASH_REF=/path/to/POLAR-FLASH python tests/golden/make_kv_golden.py

For modes int8, 2bit and 2bit_asym: seeded randn keys/values [1, 4, 16, 64]
(the shape of the reference's own test) appended in two update() calls
(10 then 6 tokens), a ragged head dim of 62 (padded 2-bit bytes), and
hand-made rows that land on rounding ties, exact floor boundaries, a
constant row and an all-zero row (the 1e-8 scale clamp).  Stores the
reference's codes, scales, zeros and returned (dequantized) K/V, plus one
sliding-window call (window 12, 4 sinks).  Needs the reference sources at
$POLARFLASH_REF (required); the GPU machines only read the
.npz.
"""
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REF = os.environ.get("POLARFLASH_REF")
if not REF or not os.path.isdir(REF):
    sys.exit("set POLARFLASH_REF to a checkout of the reference POLAR-FLASH sources")
sys.path.insert(0, REF)

from polarflash_rt.kv_cache.compressed_kv import CompressedKVCache  # noqa: E402

EDGE = np.array([
    [0.0, 1.0, 2.0, 3.0, 1.5, 0.5, 2.5, 1.25],      # asym ties: 1.5 -> 2, 0.5 -> 0, 2.5 -> 2
    [1.75, -1.75, -1.0, 0.0, 1.0, -0.5, 0.5, 0.25],  # 2bit floor boundaries (delta = 1)
    [127.0, -127.0, 0.5, 1.5, 2.5, -0.5, -2.5, 63.5],  # int8 ties (s = 1)
    [0.7, 0.7, 0.7, 0.7, 0.7, 0.7, 0.7, 0.7],        # constant row
    [0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0, 0.0],        # all zero: the 1e-8 clamp
    [-3.0, -2.0, -1.0, -4.0, -2.5, -3.5, -1.5, -0.5],
], np.float32).reshape(1, 1, 6, 8)


def main():
    g = torch.Generator().manual_seed(1234)
    k = torch.randn(1, 4, 16, 64, generator=g)
    v = torch.randn(1, 4, 16, 64, generator=g)
    kr = torch.randn(1, 2, 5, 62, generator=g) * 3.0
    vr = torch.randn(1, 2, 5, 62, generator=g) * 0.1
    out = {"k": k.numpy(), "v": v.numpy(), "kr": kr.numpy(), "vr": vr.numpy(), "edge": EDGE}
    for mode in ("int8", "2bit", "2bit_asym"):
        c = CompressedKVCache(num_layers=1, num_kv_heads=4, head_dim=64, mode=mode)
        c.update(0, k[:, :, :10], v[:, :, :10])
        ko, vo = c.update(0, k[:, :, 10:], v[:, :, 10:])
        ly = c.layers[0]
        out[f"{mode}_k_codes"] = ly["k_data"].numpy()
        out[f"{mode}_k_scales"] = ly["k_scales"].numpy()
        out[f"{mode}_v_codes"] = ly["v_data"].numpy()
        out[f"{mode}_v_scales"] = ly["v_scales"].numpy()
        if mode == "2bit_asym":
            out[f"{mode}_k_zeros"] = ly["k_zeros"].numpy()
            out[f"{mode}_v_zeros"] = ly["v_zeros"].numpy()
        out[f"{mode}_k_out"] = ko.numpy()
        out[f"{mode}_v_out"] = vo.numpy()
        cr = CompressedKVCache(num_layers=1, num_kv_heads=2, head_dim=62, mode=mode)
        ko, vo = cr.update(0, kr, vr)
        out[f"{mode}_kr_codes"] = cr.layers[0]["k_data"].numpy()
        out[f"{mode}_kr_out"] = ko.numpy()
        out[f"{mode}_vr_out"] = vo.numpy()
        ce = CompressedKVCache(num_layers=1, num_kv_heads=1, head_dim=8, mode=mode)
        ko, _ = ce.update(0, torch.from_numpy(EDGE), torch.from_numpy(EDGE))
        out[f"{mode}_edge_codes"] = ce.layers[0]["k_data"].numpy()
        out[f"{mode}_edge_scales"] = ce.layers[0]["k_scales"].numpy()
        out[f"{mode}_edge_out"] = ko.numpy()
        cw = CompressedKVCache(num_layers=1, num_kv_heads=4, head_dim=64, mode=mode, window_size=12,
                               num_sink_tokens=4)
        ko, vo = cw.update(0, k, v)
        out[f"{mode}_window_k_out"] = ko.numpy()
        out[f"{mode}_window_v_out"] = vo.numpy()
    np.savez_compressed(os.path.join(HERE, "kv_cache.npz"), **out)
    print("wrote kv_cache.npz", {k_: v_.shape for k_, v_ in out.items() if k_.startswith("int8")})


if __name__ == "__main__":
    main()
