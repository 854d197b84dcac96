"""Product encoders (polarflash_b200.encoders / UnifiedQuantizer, torch on CPU)
against the oracle and the reference's own payloads.  Codes, indices and
payload bytes must match exactly."""
import json
import os

import numpy as np
import pytest
import torch

import oracle
from conftest import GOLDEN
from polarflash_b200 import encoders
from polarflash_b200.hadamard import column_signs_cpu, effective_block
from polarflash_b200.quantizer import UnifiedQuantizer, rwht_cpu


def _w(M, K, seed, std=0.02, outliers=True):
    g = torch.Generator().manual_seed(seed)
    W = torch.randn(M, K, generator=g) * std
    if outliers:
        n = max(1, int(0.001 * M * K))
        pos = torch.randperm(M * K, generator=g)[:n]
        sg = torch.randint(0, 2, (n,), generator=g).float() * 2 - 1
        W.view(-1)[pos] = sg * 0.4
    return W


@pytest.mark.parametrize("bits", [4, 3, 2])
def test_g128_asym_encoder_matches_oracle(bits):
    W = _w(96, 1024, bits)
    q, s, m = encoders.quant_g128_asym(W, bits)
    oq, os_, om = oracle.quant_g128_asym(bits, W.numpy())
    assert np.array_equal(q.numpy(), oq)
    assert np.array_equal(s.numpy().view(np.uint16), os_.view(np.uint16))
    assert np.array_equal(m.numpy().view(np.uint16), om.view(np.uint16))
    words = encoders.pack_g128(q, bits)
    assert np.array_equal(words.numpy().view(np.uint32), oracle.pack_g128(bits, oq))
    assert np.array_equal(oracle.unpack_g128(bits, words.numpy().view(np.uint32), 96, 1024), oq)


def test_g128_degenerate_groups():
    W = torch.zeros(4, 256)
    W[1] = 0.3            # constant group: range 0
    W[2, :128] = 1e-9     # tiny values: fp16 underflow of the step
    for bits in (4, 3, 2):
        q, s, m = encoders.quant_g128_asym(W, bits)
        oq, os_, om = oracle.quant_g128_asym(bits, W.numpy())
        assert np.array_equal(q.numpy(), oq)
        assert np.array_equal(s.numpy().view(np.uint16), os_.view(np.uint16))
        assert (s.float() > 0).all()


def test_e8_encoder_matches_oracle():
    W = _w(24, 512, 11, std=0.015)
    idx, sc = encoders.e8_encode(W, rows_per_chunk=7)
    oidx, osc = oracle.e8_encode(W.numpy())
    assert np.array_equal(idx.numpy(), oidx)
    assert np.array_equal(sc.numpy().view(np.uint16), osc.view(np.uint16))
    dec = encoders.e8_decode(idx, sc)
    np.testing.assert_array_equal(dec.numpy(), oracle.e8_decode(oidx, osc, 24, 512))
    # residual VQ: stage 2 lowers the error of stage 1 (test_milestone0:282-295)
    err = torch.mean((dec - W) ** 2).item()
    assert err < torch.mean(W ** 2).item() * 0.5


def test_e8_encoder_ties_take_lowest_index():
    e = torch.zeros(1, 128)  # all dot products tie at 0 -> root 0 everywhere
    idx, sc = encoders.e8_encode(e)
    assert int(idx.max()) == 0 and float(sc.float().abs().max()) == 0.0
    oidx, _ = oracle.e8_encode(e.numpy())
    assert np.array_equal(idx.numpy(), oidx)


def test_e8_roots_order():
    np.testing.assert_array_equal(encoders.e8_roots().numpy(), np.load(os.path.join(GOLDEN, "e8_roots.npz"))["roots"])


def _polar_cases():
    with open(os.path.join(GOLDEN, "polar_recursive_meta.json")) as f:
        meta = json.load(f)
    meta.pop("_allocs")
    return sorted(meta.items())


@pytest.mark.parametrize("key,meta", _polar_cases())
def test_polar_encoder_matches_reference_payload(key, meta):
    g = np.load(os.path.join(GOLDEN, "polar_recursive.npz"))
    Wr = torch.from_numpy(g[f"Wrot_{key}"])
    bpw = float(key.split("_")[1][1:])
    payload, pm = encoders.polar_encode(Wr, meta["block_size"], bpw, blocks_per_chunk=64)
    assert pm["alloc"] == meta["alloc"]
    assert pm["r_scale"] == meta["r_scale"]
    assert payload.numpy().tobytes() == g[f"packed_{key}"].tobytes()


def test_polar_alloc_matches_reference():
    with open(os.path.join(GOLDEN, "polar_recursive_meta.json")) as f:
        allocs = json.load(f)["_allocs"]
    for k, ref in allocs.items():
        d, bpw = k.split("_")
        assert encoders.polar_alloc(int(d), float(bpw)) == ref


@pytest.mark.parametrize("K,req", [(128, 128), (4096, 128), (500, 512), (11008, 512), (129, 128)])
def test_cpu_rwht_and_signs_match_reference(K, req):
    g = np.load(os.path.join(GOLDEN, "hadamard.npz"))
    key = f"{K}_{req}"
    assert effective_block(req, K) == int(g[f"block_{key}"])
    ref_signs = g[f"signs_{key}"]
    assert np.array_equal(column_signs_cpu(K, req).numpy()[: len(ref_signs)].astype(np.float32), ref_signs)
    x = torch.from_numpy(g[f"x_{key}"])
    np.testing.assert_allclose(rwht_cpu(x, req).numpy(), g[f"fwd_{key}"], atol=1e-6, rtol=0)
    np.testing.assert_allclose(rwht_cpu(x, req, inverse=True).numpy(), g[f"inv_{key}"], atol=1e-6, rtol=0)


def _unified_cases():
    with open(os.path.join(GOLDEN, "unified_meta.json")) as f:
        return sorted(json.load(f).items())


@pytest.mark.parametrize("key,meta", _unified_cases())
def test_unified_quantizer_reference_backends_give_reference_payloads(key, meta):
    g = np.load(os.path.join(GOLDEN, "unified.npz"))
    be, shape, hb = key.split("_")
    W = torch.from_numpy(g[f"W_{shape}_{hb}"])
    uq = UnifiedQuantizer(backend=be, hadamard_block_size=int(hb[1:]))
    payload, m, _ = uq.quantize(W, return_w_hat=False)
    assert payload == g[f"payload_{key}"].tobytes()
    for k in ("scale", "r_scale", "r_bits", "theta_bits", "padded"):
        if k in meta:
            assert m[k] == meta[k], k


@pytest.mark.parametrize("n", [240, 241, 1000])
def test_reference_packers(n):
    g = np.load(os.path.join(GOLDEN, "bitpack.npz"))
    assert encoders.pack_int4(torch.from_numpy(g[f"v4_{n}"])).numpy().tobytes() == g[f"p4_{n}"].tobytes()
    assert encoders.pack_int2(torch.from_numpy(g[f"v2_{n}"])).numpy().tobytes() == g[f"p2_{n}"].tobytes()
    assert encoders.pack_int3(torch.from_numpy(g[f"v3_{n}"])).numpy().tobytes() == g[f"p3_{n}"].tobytes()
