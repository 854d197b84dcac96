"""Tiny Llama-style model for the decode-step tests (not a test module).

Every weight comes from a seeded generator; each linear is RWHT-128 rotated,
INT4 group-128 quantized and packed by the oracle, and decoded back by the
oracle (W_hat).  tests/golden/make_decode_golden.py runs the reference's
PFlashModelForCausalLM on the decoded weights; the GPU test runs
polarflash_b200.decode.PFlashDecoder on the packed ones.
"""
import numpy as np
import torch

import oracle

CFG = dict(hidden_size=256, num_attention_heads=4, num_key_value_heads=2, intermediate_size=512, vocab_size=384,
           num_hidden_layers=2, rope_theta=1000000.0, rms_norm_eps=1e-6)
LIN = [("q", 256, 256), ("k", 128, 256), ("v", 128, 256), ("o", 256, 256), ("gate", 512, 256), ("up", 512, 256),
       ("down", 256, 512)]
PROMPT = [5, 17, 42, 99, 7, 250, 3, 128, 64, 31, 200, 9, 77, 301, 12, 45, 88, 160, 2, 19]
DECODE = [11, 300, 64]
META = {"hadamard_rotation": True, "hadamard_block_size": 128}


def _randn(shape, seed, scale):
    return torch.randn(*shape, generator=torch.Generator().manual_seed(seed)) * scale


def build():
    """{"layers": [{name: dict(words, s, m, W_hat, M, K)}, ...] with "in_norm" /
    "post_norm" per layer, "embed", "final_norm", "lm_head"} (numpy fp32)."""
    from polarflash_b200.quantizer import rwht_cpu

    out = {"layers": []}
    seed = 100
    for li in range(CFG["num_hidden_layers"]):
        ly = {}
        for name, M, K in LIN:
            W = _randn((M, K), seed, 0.02)
            seed += 1
            q, s, m = oracle.quant_g128_asym(4, rwht_cpu(W, 128).numpy())
            words = oracle.pack_g128(4, q)
            pay = {"words": words, "s": s, "m": m}
            ly[name] = dict(words=words, s=s, m=m, M=M, K=K, W_hat=oracle.dequantize("int4_g128", pay, M, K, META))
        H = CFG["hidden_size"]
        ly["in_norm"] = (1.0 + _randn((H,), seed, 0.1)).numpy()
        ly["post_norm"] = (1.0 + _randn((H,), seed + 1, 0.1)).numpy()
        seed += 2
        out["layers"].append(ly)
    V, H = CFG["vocab_size"], CFG["hidden_size"]
    out["embed"] = _randn((V, H), 7, 1.0).numpy()
    out["final_norm"] = (1.0 + _randn((H,), 8, 0.1)).numpy()
    out["lm_head"] = _randn((V, H), 9, 0.02).numpy()
    return out


def reference_forward(w, ids, caches, cfg=CFG, kv_quant=None):
    """fp32 torch restatement of PFlashModelForCausalLM.forward
    (model_integration.py:240-254) on the decoded weights; `caches` is a list
    of per-layer dicts (k, v: [1, T, heads, hd]) updated in place.
    `kv_quant` (rows [..., hd] -> dequantized rows) stands for a compressed
    KV cache: the new keys (after RoPE) and values pass through it before
    they are cached, as CompressedKVCache.update quantizes each appended row
    and attends over the dequantized context."""
    import math

    import torch.nn.functional as F

    H, nh, nkv = cfg["hidden_size"], cfg["num_attention_heads"], cfg["num_key_value_heads"]
    hd, eps, theta = H // nh, cfg["rms_norm_eps"], cfg["rope_theta"]
    t = lambda a: torch.from_numpy(np.asarray(a, np.float32))  # noqa: E731

    def norm(x, g):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps) * g

    def rope(x, S, off):
        half = hd // 2
        fr = 1.0 / (theta ** (torch.arange(0, half, dtype=torch.float32) / half))
        f = torch.outer(torch.arange(off, off + S, dtype=torch.float32), fr)
        c, s = torch.cos(f)[None, :, None], torch.sin(f)[None, :, None]
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * c - x2 * s, x1 * s + x2 * c], dim=-1)

    ids = torch.as_tensor(ids)[None]
    S = ids.shape[1]
    h = t(w["embed"])[ids]
    for li, ly in enumerate(w["layers"]):
        n = norm(h, t(ly["in_norm"]))
        q = (n @ t(ly["q"]["W_hat"]).T).view(1, S, nh, hd)
        k = (n @ t(ly["k"]["W_hat"]).T).view(1, S, nkv, hd)
        v = (n @ t(ly["v"]["W_hat"]).T).view(1, S, nkv, hd)
        c = caches[li]
        off = c["k"].shape[1] if "k" in c else 0
        q, k = rope(q, S, off), rope(k, S, off)
        if kv_quant is not None:
            k, v = kv_quant(k), kv_quant(v)
        if "k" in c:
            k, v = torch.cat([c["k"], k], 1), torch.cat([c["v"], v], 1)
        c["k"], c["v"] = k, v
        T = k.shape[1]
        kk = torch.repeat_interleave(k, nh // nkv, dim=2).transpose(1, 2)
        vv = torch.repeat_interleave(v, nh // nkv, dim=2).transpose(1, 2)
        sc = q.transpose(1, 2) @ kk.transpose(-1, -2) / math.sqrt(hd)
        if S > 1:
            sc = sc + torch.triu(torch.full((S, T), float("-inf")), diagonal=T - S + 1)[None, None]
        o = (F.softmax(sc, -1) @ vv).transpose(1, 2).reshape(1, S, H)
        h = h + o @ t(ly["o"]["W_hat"]).T
        n2 = norm(h, t(ly["post_norm"]))
        a = F.silu(n2 @ t(ly["gate"]["W_hat"]).T) * (n2 @ t(ly["up"]["W_hat"]).T)
        h = h + a @ t(ly["down"]["W_hat"]).T
    return (norm(h, t(w["final_norm"])) @ t(w["lm_head"]).T)[0]
