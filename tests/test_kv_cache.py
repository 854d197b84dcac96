"""Compressed KV cache (CompressedKVCache, polarflash_rt/kv_cache/
compressed_kv.py): modes int8, 2bit, 2bit_asym.

Pins: tests/golden/kv_cache.npz holds the reference's own codes, scales,
zeros and returned K/V (tests/golden/make_kv_golden.py): two appends of
[1, 4, 16, 64] rows, a ragged head dim of 62, hand-made rows on rounding
ties, floor boundaries, a constant and an all-zero row, and a sliding
window with sink tokens.

Bars: codes, scales, zeros and dequantized values bit-exact (integer codes,
and every fp32 step explicitly rounded as the reference's); attention over a
compressed cache within 1e-5 normwise of torch SDPA over the dequantized
cache; the decoder with an int8 cache within 1e-2 of the fp32 restatement
whose cache passes through the same quantizer (its linears compute with
fp16 x'), and its captured steps within 1e-4 of its eager steps.
"""
import ctypes
import math
import os

import numpy as np
import pytest
import torch

import decode_model as dm
from oracle import kv_cache as okv

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "kv_cache.npz")
MODES = ("int8", "2bit", "2bit_asym")


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))


# ---- CPU: oracle and host logic ----------------------------------------------
@pytest.mark.parametrize("mode", MODES)
def test_oracle_matches_reference_golden(mode):
    g = np.load(GOLD)
    for nm in ("k", "v"):
        c, s, z = okv.quantize(g[nm], mode)
        assert np.array_equal(c, g[f"{mode}_{nm}_codes"])
        assert np.array_equal(s, g[f"{mode}_{nm}_scales"])
        if mode == "2bit_asym":
            assert np.array_equal(z, g[f"{mode}_{nm}_zeros"])
        assert np.array_equal(okv.dequantize(c, s, z, 64, mode), g[f"{mode}_{nm}_out"])
    c, s, z = okv.quantize(g["kr"], mode)
    assert np.array_equal(c, g[f"{mode}_kr_codes"])
    assert np.array_equal(okv.dequantize(c, s, z, 62, mode), g[f"{mode}_kr_out"])
    c, s, z = okv.quantize(g["edge"], mode)
    assert np.array_equal(c, g[f"{mode}_edge_codes"]) and np.array_equal(s, g[f"{mode}_edge_scales"])
    assert np.array_equal(okv.dequantize(c, s, z, 8, mode), g[f"{mode}_edge_out"])
    c, s, z = okv.quantize(g["k"], mode)
    keep = okv.window_indices(16, 12, 4)
    assert np.array_equal(okv.dequantize(c, s, z, 64, mode)[:, :, keep], g[f"{mode}_window_k_out"])


def test_mirror_bookkeeping():
    """Memory accounting and code layout of the host mirror (no GPU)."""
    from polarflash_b200.kv_cache import CompressedKVCache, kv_row_bytes

    for mode, q in (("fp16", 2.0), ("int8", 1.0), ("2bit", 0.25), ("2bit_asym", 0.25), ("polar_qjl", 0.5),
                    ("dictionary", 0.25), ("other", 1.0)):
        c = CompressedKVCache(num_layers=3, num_kv_heads=8, head_dim=128, mode=mode.upper())
        assert c.q_bytes == q
        assert c.theoretical_memory_bytes(1000) == int(2 * 3 * 1000 * 8 * 128 * q)
        assert len(c.layers) == 3 and c.layers[0]["k_data"] is None
    assert [kv_row_bytes(m, 62) for m in MODES] == [62, 16, 16]
    assert okv.window_indices(10, None, 4) == list(range(10))
    assert okv.window_indices(20, 12, 4) == [0, 1, 2, 3] + list(range(12, 20))


def test_no_cpu_path():
    """The mirror refuses host tensors instead of quantizing on the CPU, and
    the decoder refuses an unknown cache mode before allocating anything."""
    from polarflash_b200.decode import PFlashDecoder
    from polarflash_b200.kv_cache import CompressedKVCache

    c = CompressedKVCache(num_layers=1, num_kv_heads=2, head_dim=8, mode="int8")
    with pytest.raises(RuntimeError, match="CUDA"):
        c.update(0, torch.zeros(1, 2, 3, 8), torch.zeros(1, 2, 3, 8))
    with pytest.raises(ValueError, match="kv_mode"):
        PFlashDecoder(dm.CFG, [], torch.zeros(4, 256), torch.ones(256), torch.zeros(4, 256), 8, kv_mode="int4")


def test_restatement_hook_is_identity_for_fp32():
    """decode_model.reference_forward with an identity KV hook reproduces its
    own uncompressed logits (the hook only touches the cached rows)."""
    w = dm.build()
    a = dm.reference_forward(w, dm.PROMPT[:6], [{} for _ in range(2)])
    b = dm.reference_forward(w, dm.PROMPT[:6], [{} for _ in range(2)], kv_quant=lambda x: x)
    assert torch.equal(a, b)


# ---- GPU --------------------------------------------------------------------
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    return torch.device("cuda")


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
def test_kernels_match_reference_golden(mode):
    from polarflash_b200.kv_cache import kv_dequantize, kv_quantize

    dev = _cuda()
    g = np.load(GOLD)
    for key, d in (("k", 64), ("v", 64), ("kr", 62), ("edge", 8)):
        x = torch.from_numpy(g[key]).to(dev)
        c, s, z = kv_quantize(x, mode)
        ref = {"k": f"{mode}_k", "v": f"{mode}_v", "kr": f"{mode}_kr", "edge": f"{mode}_edge"}[key]
        assert np.array_equal(c.cpu().numpy(), g[ref + "_codes"]), key
        if key in ("k", "v", "edge"):
            assert np.array_equal(s.cpu().numpy(), g[ref + "_scales"]), key
        if mode == "2bit_asym" and key in ("k", "v"):
            assert np.array_equal(z.cpu().numpy(), g[ref + "_zeros"]), key
        out = kv_dequantize(c, s, z, d, mode).cpu().numpy()
        exp = {"k": f"{mode}_k_out", "v": f"{mode}_v_out", "kr": f"{mode}_kr_out", "edge": f"{mode}_edge_out"}[key]
        assert np.array_equal(out, g[exp]), key


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES + ("fp16", "polar_qjl"))
def test_mirror_update_matches_reference(mode):
    """CompressedKVCache.update on the device, two appends and a window, as
    the reference returns them (fp16: a plain half cache; polar_qjl: the
    reference's int8 fallback)."""
    from polarflash_b200.kv_cache import CompressedKVCache

    dev = _cuda()
    g = np.load(GOLD)
    k, v = torch.from_numpy(g["k"]).to(dev), torch.from_numpy(g["v"]).to(dev)
    c = CompressedKVCache(num_layers=1, num_kv_heads=4, head_dim=64, mode=mode)
    c.update(0, k[:, :, :10], v[:, :, :10])
    ko, vo = c.update(0, k[:, :, 10:], v[:, :, 10:])
    assert c.layers[0]["seq_len"] == 16
    q = torch.randn(1, 4, 1, 64, generator=torch.Generator(device=dev).manual_seed(3), device=dev)
    err = c.compute_attention_error(q, k, ko)
    assert err["cosine_similarity"] > (0.85 if mode in ("2bit", "2bit_asym") else 0.95)
    ke, _ = c.update(0, k[:, :, :0], v[:, :, :0])  # an empty append returns the context unchanged
    assert torch.equal(ke, ko)
    if mode == "fp16":
        assert ko.dtype == torch.float16 and torch.equal(ko, k.half()) and torch.equal(vo, v.half())
        return
    gm = "int8" if mode == "polar_qjl" else mode
    assert np.array_equal(ko.cpu().numpy(), g[f"{gm}_k_out"])
    assert np.array_equal(vo.cpu().numpy(), g[f"{gm}_v_out"])
    assert np.array_equal(c.layers[0]["k_data"].cpu().numpy(), g[f"{gm}_k_codes"])
    cw = CompressedKVCache(num_layers=1, num_kv_heads=4, head_dim=64, mode=mode, window_size=12, num_sink_tokens=4)
    ko, vo = cw.update(0, k, v)
    assert np.array_equal(ko.cpu().numpy(), g[f"{gm}_window_k_out"])
    assert np.array_equal(vo.cpu().numpy(), g[f"{gm}_window_v_out"])


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
@pytest.mark.parametrize("ms,pos", [(64, 0), (64, 63), (300, 200), (300, 299)])
def test_rope_write_and_attention_over_compressed_cache(mode, ms, pos):
    """pf_rope_kv_compressed writes the codes pf_kv_quantize (and the
    oracle) give for the key pf_rope_kv rotates; pf_decode_attention_
    compressed matches SDPA over the dequantized cache (GQA 8/2 heads of 128)."""
    from polarflash_b200 import _lib
    from polarflash_b200.kv_cache import KV_MODES, kv_dequantize, kv_quantize

    import torch.nn.functional as F

    dev = _cuda()
    L = _lib.load()
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    m = KV_MODES[mode]
    g = torch.Generator(device=dev).manual_seed(1000 + pos)
    nh, nkv, hd = 8, 2, 128
    # a filled compressed cache: rows [ms, nkv, hd]
    kc, ks, kz = kv_quantize(torch.randn(ms, nkv, hd, generator=g, device=dev), mode)
    vc, vs, vz = kv_quantize(torch.randn(ms, nkv, hd, generator=g, device=dev) * 0.5, mode)
    q = torch.randn(nh * hd, generator=g, device=dev)
    k = torch.randn(nkv * hd, generator=g, device=dev)
    v = torch.randn(nkv * hd, generator=g, device=dev)
    inv = 1.0 / (500000.0 ** (torch.arange(0, hd // 2, dtype=torch.float32, device=dev) / (hd // 2)))
    pt = torch.tensor([pos], dtype=torch.long, device=dev)
    # fp32 kernel for the rotated k (same rotation arithmetic)
    q32, kc32, vc32 = q.clone(), torch.zeros(ms, nkv, hd, device=dev), torch.zeros(ms, nkv, hd, device=dev)
    _lib.check(L.pf_rope_kv(p(q32), p(k), p(v), p(kc32), p(vc32), p(pt), p(inv), nh, nkv, hd, ms, st))
    before = (kc.clone(), vc.clone())
    _lib.check(L.pf_rope_kv_compressed(p(q), p(k), p(v), p(kc), p(ks), p(kz), p(vc), p(vs), p(vz), p(pt), p(inv),
                                       nh, nkv, hd, ms, m, st))
    assert torch.equal(q, q32)
    ek, eks, ekz = kv_quantize(kc32[pos], mode)
    ev, evs, evz = kv_quantize(vc32[pos], mode)
    assert torch.equal(kc[pos], ek) and torch.equal(ks[pos], eks) and torch.equal(vc[pos], ev)
    assert torch.equal(vs[pos], evs)
    if mode == "2bit_asym":
        assert torch.equal(kz[pos], ekz) and torch.equal(vz[pos], evz)
    oc, os_, oz = okv.quantize(kc32[pos].cpu().numpy(), mode)
    assert np.array_equal(kc[pos].cpu().numpy(), oc) and np.array_equal(ks[pos].cpu().numpy(), os_)
    others = [i for i in range(ms) if i != pos]
    assert torch.equal(kc[others], before[0][others]) and torch.equal(vc[others], before[1][others])
    # attention over positions 0..pos of the compressed cache
    att = torch.empty(nh * hd, device=dev)
    aws = torch.empty(int(L.pf_decode_attention_workspace_size(nh, hd, ms)), dtype=torch.uint8, device=dev)
    _lib.check(L.pf_decode_attention_compressed(p(q), p(kc), p(ks), p(kz), p(vc), p(vs), p(vz), p(pt), p(att), nh,
                                                nkv, hd, ms, m, 1.0 / math.sqrt(hd), p(aws), aws.numel(), st))
    K = kv_dequantize(kc, ks, kz, hd, mode)[: pos + 1].permute(1, 0, 2)[None]
    V = kv_dequantize(vc, vs, vz, hd, mode)[: pos + 1].permute(1, 0, 2)[None]
    ref = F.scaled_dot_product_attention(q.view(1, nh, 1, hd), K, V, enable_gqa=True).reshape(-1)
    assert _rel(att.cpu().numpy(), ref.cpu().numpy()) < 1e-5


@pytest.mark.gpu
@pytest.mark.parametrize("mode", MODES)
def test_decoder_with_compressed_cache(mode):
    """PFlashDecoder(kv_mode=mode): prefill and captured steps.  int8 against
    the fp32 restatement whose cached rows pass through the oracle's int8
    quantizer; every mode: captured steps against eager steps."""
    from test_decode_step import _decoder

    _cuda()
    w = dm.build()
    a, b = _decoder(w, kv_mode=mode), _decoder(w, kv_mode=mode)
    prompt = torch.tensor(dm.PROMPT, device="cuda")
    pa = a.forward(prompt).cpu().numpy()
    b.forward(prompt)
    b.capture()
    steps = []
    for tok in dm.DECODE:
        ea = a.forward(torch.tensor([tok], device="cuda"))[0]
        eb = b.step(tok)[0]
        assert _rel(eb.cpu().numpy(), ea.cpu().numpy()) < 1e-4
        steps.append(eb.cpu().numpy())
    if mode != "int8":
        return

    def quant(x):
        c, s, z = okv.quantize(x.numpy(), "int8")
        return torch.from_numpy(okv.dequantize(c, s, z, x.shape[-1], "int8"))

    caches = [{} for _ in range(dm.CFG["num_hidden_layers"])]
    ref = dm.reference_forward(w, dm.PROMPT, caches, kv_quant=quant).numpy()
    assert _rel(pa, ref) < 1e-2
    for i, tok in enumerate(dm.DECODE):
        r = dm.reference_forward(w, [tok], caches, kv_quant=quant)[-1].numpy()
        assert _rel(steps[i], r) < 1e-2, f"step {i}"
