"""Decode-step integration (PFlashDecoder): a two-layer Llama-style model
(tests/decode_model.py: INT4 group-128 packed linears, GQA 4/2 heads, RoPE,
SwiGLU) against golden logits from the reference's own
PFlashModelForCausalLM (tests/golden/make_decode_golden.py): a 20-token
prefill (tensor-core GEMM for the linears, causal mask) and three cached
single-token steps (streaming GEMV, CUDA-graph replays).

Tolerances (normwise, max|a - b| / max|b|): the fp32 restatement reproduces
the reference's logits within 1e-5; the GPU decoder within 1e-3, both with
the default tensor-core prefill GEMM (fp16 weights and x' products; measured
on a B200: 4.9e-5 at the prefill, <= 1e-5 at the steps) and with
faithful_prefill (every packed linear on the streaming GEMV: fp32 group
scales, x' as an fp16 hi + lo pair; 2.3e-5 and <= 5e-7)."""
import os

import numpy as np
import pytest
import torch

import decode_model as dm

GOLD = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "decode_step.npz")


def _rel(a, b):
    a, b = np.asarray(a, np.float64), np.asarray(b, np.float64)
    return float(np.abs(a - b).max() / np.abs(b).max())


def test_restatement_matches_reference_logits():
    g = np.load(GOLD)
    w = dm.build()
    caches = [{} for _ in range(dm.CFG["num_hidden_layers"])]
    pre = dm.reference_forward(w, g["prompt"].tolist(), caches).numpy()
    assert _rel(pre, g["prefill_logits"]) < 1e-5
    for i, tok in enumerate(g["decode"].tolist()):
        lg = dm.reference_forward(w, [tok], caches)[-1].numpy()
        assert _rel(lg, g["step_logits"][i]) < 1e-5


def _decoder(w, max_seq=32, kv_mode="fp32", faithful_prefill=False):
    from polarflash_b200.decode import DecoderLayer, PFlashDecoder
    from polarflash_b200.hadamard import column_signs, effective_block
    from polarflash_b200.qweight import QWeight

    dev = torch.device("cuda")
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a, np.float32)).to(dev)  # noqa: E731
    layers = []
    for ly in w["layers"]:
        qw = {}
        for name, M, K in dm.LIN:
            p = ly[name]
            qw[name] = QWeight(1, M, K, torch.from_numpy(p["words"].view(np.uint8).reshape(-1).copy()).to(dev),
                               torch.from_numpy(p["s"].copy()).to(dev), torch.from_numpy(p["m"].copy()).to(dev),
                               effective_block(128, K), column_signs(K, 128, dev))
        layers.append(DecoderLayer(qw["q"], qw["k"], qw["v"], qw["o"], qw["gate"], qw["up"], qw["down"],
                                   t(ly["in_norm"]), t(ly["post_norm"])))
    return PFlashDecoder(dm.CFG, layers, t(w["embed"]), t(w["final_norm"]), t(w["lm_head"]), max_seq,
                         kv_mode=kv_mode, faithful_prefill=faithful_prefill)


@pytest.mark.gpu
@pytest.mark.parametrize("faithful,tol", [(True, 1e-3), (False, 1e-3)])
def test_prefill_and_graph_steps_match_reference(faithful, tol):
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = np.load(GOLD)
    dec = _decoder(dm.build(), faithful_prefill=faithful)
    pre = dec.forward(torch.tensor(g["prompt"], device="cuda")).cpu().numpy()
    errs = [_rel(pre, g["prefill_logits"])]
    dec.capture()
    for i, tok in enumerate(g["decode"].tolist()):
        errs.append(_rel(dec.step(tok)[0].cpu().numpy(), g["step_logits"][i]))
    print(f"faithful_prefill={faithful}: normwise logits error prefill {errs[0]:.2e}, steps "
          + ", ".join(f"{e:.2e}" for e in errs[1:]))
    assert max(errs) < tol, errs
    assert dec.length == len(g["prompt"]) + len(g["decode"])


@pytest.mark.gpu
def test_graph_steps_equal_eager_steps():
    """The captured step (the library's decode kernels: add + RMSNorm, RoPE
    with the cache write, attention over the cache, SiLU gate; token and
    position from device tensors) agrees with eager single-token calls (torch
    ops around the same packed linears)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    g = np.load(GOLD)
    w = dm.build()
    a, b = _decoder(w), _decoder(w)
    prompt = torch.tensor(g["prompt"], device="cuda")
    a.forward(prompt)
    b.forward(prompt)
    b.capture()
    for tok in g["decode"].tolist():
        ea = a.forward(torch.tensor([tok], device="cuda"))[0]
        eb = b.step(tok)[0]
        assert _rel(eb.cpu().numpy(), ea.cpu().numpy()) < 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("ms,pos", [(64, 0), (64, 37), (64, 63), (300, 64), (300, 200), (300, 299)])
def test_decode_kernels_match_torch(ms, pos):
    """pf_add_rmsnorm, pf_rope_kv, pf_decode_attention and pf_silu_mul against
    torch fp32 restatements of the reference blocks (1e-5 normwise), GQA
    8 query / 2 KV heads of 128, an `ms`-position cache at position `pos`
    (one or several 64-position attention chunks)."""
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    import ctypes
    import math

    import torch.nn.functional as F

    from polarflash_b200 import _lib

    L = _lib.load()
    dev = torch.device("cuda")
    st = ctypes.c_void_p(torch.cuda.current_stream(dev).cuda_stream)
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    g = torch.Generator(device=dev).manual_seed(pos)
    nh, nkv, hd, H = 8, 2, 128, 1024
    # add + RMSNorm
    h = torch.randn(3, H, generator=g, device=dev)
    d = torch.randn(3, H, generator=g, device=dev)
    w = torch.rand(H, generator=g, device=dev) + 0.5
    out = torch.empty_like(h)
    ref_h = h + d
    ref = ref_h * torch.rsqrt(ref_h.pow(2).mean(-1, keepdim=True) + 1e-6) * w
    _lib.check(L.pf_add_rmsnorm(p(h), p(d), p(w), p(out), 3, H, 1e-6, st))
    assert _rel(h.cpu().numpy(), ref_h.cpu().numpy()) < 1e-6
    assert _rel(out.cpu().numpy(), ref.cpu().numpy()) < 1e-5
    # RoPE + cache write
    q = torch.randn(nh * hd, generator=g, device=dev)
    k = torch.randn(nkv * hd, generator=g, device=dev)
    v = torch.randn(nkv * hd, generator=g, device=dev)
    kc = torch.randn(ms, nkv, hd, generator=g, device=dev)
    vc = torch.randn(ms, nkv, hd, generator=g, device=dev)
    kc0, vc0, q0 = kc.clone(), vc.clone(), q.clone()
    inv = 1.0 / (500000.0 ** (torch.arange(0, hd // 2, dtype=torch.float32, device=dev) / (hd // 2)))
    pt = torch.tensor([pos], dtype=torch.long, device=dev)
    _lib.check(L.pf_rope_kv(p(q), p(k), p(v), p(kc), p(vc), p(pt), p(inv), nh, nkv, hd, ms, st))
    f = pos * inv
    c, s = torch.cos(f), torch.sin(f)

    def rot(x):
        x1, x2 = x[..., : hd // 2], x[..., hd // 2:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], -1)

    assert _rel(q.view(nh, hd).cpu().numpy(), rot(q0.view(nh, hd)).cpu().numpy()) < 1e-5
    kc0[pos] = rot(k.view(nkv, hd))
    vc0[pos] = v.view(nkv, hd)
    assert torch.allclose(kc, kc0, rtol=1e-5, atol=1e-6) and torch.equal(vc, vc0)
    # attention over positions 0..pos
    att = torch.empty(nh * hd, device=dev)
    aws = torch.empty(int(L.pf_decode_attention_workspace_size(nh, hd, ms)), dtype=torch.uint8, device=dev)
    _lib.check(L.pf_decode_attention(p(q), p(kc), p(vc), p(pt), p(att), nh, nkv, hd, ms, 1.0 / math.sqrt(hd),
                                     p(aws), aws.numel(), st))
    K = kc[: pos + 1].permute(1, 0, 2)[None]
    V = vc[: pos + 1].permute(1, 0, 2)[None]
    ref_att = F.scaled_dot_product_attention(q.view(1, nh, 1, hd), K, V, enable_gqa=True).reshape(-1)
    assert _rel(att.cpu().numpy(), ref_att.cpu().numpy()) < 1e-5
    # SiLU gate
    a = torch.randn(5000, generator=g, device=dev)
    b = torch.randn(5000, generator=g, device=dev)
    o = torch.empty_like(a)
    _lib.check(L.pf_silu_mul(p(a), p(b), p(o), a.numel(), st))
    assert _rel(o.cpu().numpy(), (F.silu(a) * b).cpu().numpy()) < 1e-6
