"""UnifiedQuantizer(backend="e8", e8_stages=k) against the reference's own
outputs (tests/golden/e8_backend.npz, made by make_e8_backend_golden.py from
unified_quantizer.py:180-192 and e8_lattice.py:52-232).

CPU: the E8 nearest-point search equals quantize_e8 bit for bit (random
vectors plus rounding ties); the quantizer's fp16 payloads are byte-identical
and its metadata (searched scales, per-stage errors) equal, for 1, 2 and 3
stages with and without the RWHT, on a weight whose size is a multiple of 8
and one that needs a padded tail.  GPU: the payloads decode on the device to
the reference's dequantize output (1e-6 absolute: the device RWHT sums in a
different order), and PolarLinearLayer runs them within the parity suite's
1e-3 of the oracle.
"""
import json
import os

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "e8_backend.npz"))
with open(os.path.join(HERE, "golden", "e8_backend_meta.json")) as f:
    META = json.load(f)
KEYS = sorted(META)


def test_nearest_point_matches_reference():
    from polarflash_b200.encoders import e8_nearest

    y = e8_nearest(torch.from_numpy(G["qe8_x"])).numpy()
    np.testing.assert_array_equal(y, G["qe8_y"])
    # every output is an E8 point: all integers or all half-integers, even sum
    twice = y * 2
    assert np.all(twice == np.round(twice))
    assert np.all((np.all(y == np.round(y), 1)) | (np.all(y - 0.5 == np.round(y - 0.5), 1)))
    assert np.all(np.round(y.sum(1)) % 2 == 0)


@pytest.mark.parametrize("key", KEYS)
def test_payload_and_meta_match_reference(key):
    from polarflash_b200.quantizer import UnifiedQuantizer

    wname, st, hh = key.split("_")
    ref = META[key]
    q = UnifiedQuantizer(backend="e8", e8_stages=int(st[1:]), apply_hadamard=hh == "h1", hadamard_block_size=128)
    w = torch.from_numpy(G[wname])
    payload, meta, w_hat = q.quantize(w, name=wname)  # e8's w_hat is the fp32 reconstruction: no device
    assert bytes(payload) == G[key + "_payload"].tobytes()
    for k in ("dtype", "bpw", "stages", "num_stages", "optimal_scale", "stage_scales", "padding_added",
              "hadamard_rotation", "hadamard_block_size", "shape", "num_elements", "payload_bytes",
              "effective_bpw"):
        assert meta.get(k) == ref.get(k), k
    for k in ("stage_mses", "total_mse", "mse_distortion"):
        if k in ref:
            np.testing.assert_allclose(meta[k], ref[k], rtol=1e-12)
    np.testing.assert_array_equal(w_hat.numpy(), G[key + "_what"])
    assert meta["mse"] == ref["mse"] and meta["snr_db"] == ref["snr_db"]


@pytest.mark.gpu
@pytest.mark.parametrize("key", KEYS)
def test_device_decode_and_layer(key):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import oracle
    from polarflash_b200.linear import PolarLinearLayer
    from polarflash_b200.quantizer import UnifiedQuantizer

    wname = key.split("_")[0]
    M, K = G[wname].shape
    meta = dict(META[key])
    payload = G[key + "_payload"].tobytes()
    deq = UnifiedQuantizer.dequantize(payload, [M, K], meta["dtype"], meta).cpu().numpy()
    np.testing.assert_allclose(deq, G[key + "_deq"], rtol=0, atol=1e-6)
    x = torch.randn(3, K, generator=torch.Generator().manual_seed(M)).half()
    layer = PolarLinearLayer(K, M, meta["dtype"], meta, payload, device="cuda")
    y = layer(x.cuda()).float().cpu().numpy()
    ref = oracle.linear(meta["dtype"], payload, M, K, meta, x.float().numpy())
    assert np.max(np.abs(y - ref)) <= 1e-3 * np.max(np.abs(ref))
