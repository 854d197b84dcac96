"""Decode-step integration: a Llama-style causal LM whose linears run on the
packed-weight op.

Mirrors ``PFlashModelForCausalLM`` (polarflash_core/model_integration.py:
203-254) and its blocks: ``RMSNorm`` (:27-37), ``apply_rotary_pos_emb``
(:40-60, half-split rotation, theta = rope_theta), ``PFlashAttentionBlock``
(:63-147, GQA with a growing KV cache, causal mask for multi-token calls),
``PFlashMLPBlock`` (:150-163, SwiGLU) and ``PFlashTransformerLayer``
(:166-192).  The reference keeps every projection as a decoded dense weight
and runs ``F.linear``; here each projection is a packed ``QWeight`` run by
the library (q|k|v and gate|up as one grouped call each), the KV cache is
preallocated on the device, and a batch-1 decode step (embedding, 2·L norms,
RoPE, cache write, attention over the cache, linears, final norm, lm_head)
can be captured once as a CUDA graph and replayed per token with the token
id and position read from device tensors.

The captured step (fp32 cache) runs the library's decode kernels around the
packed linears: residual add + RMSNorm (pf_add_rmsnorm), RoPE with the cache
write (pf_rope_kv), GQA attention over the cache (pf_decode_attention) and
the SwiGLU gate (pf_silu_mul): about a dozen launches per layer.  The eager
forward (prompts, any batch of new tokens) uses torch ops for everything but
the linears (``scaled_dot_product_attention`` for the attention); the
embedding lookup and the dense lm_head are torch ops in both.  There is no
CPU path.
"""
import ctypes
import math
from typing import Dict, List, Optional

import torch
import torch.nn.functional as F

from . import _lib
from .kv_cache import KV_MODES, kv_row_bytes
from .qweight import QWeight, group_workspace_bytes, qlinear, qlinear_multi


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


class DecoderLayer:
    """Packed weights of one transformer layer (PFlashTransformerLayer):
    projections q, k, v, o, gate, up, down as QWeights, the two RMSNorm weights
    and the optional q/k/v biases (Qwen-style models have them)."""

    def __init__(self, q: QWeight, k: QWeight, v: QWeight, o: QWeight, gate: QWeight, up: QWeight,
                 down: QWeight, input_norm: torch.Tensor, post_norm: torch.Tensor,
                 q_bias: Optional[torch.Tensor] = None, k_bias: Optional[torch.Tensor] = None,
                 v_bias: Optional[torch.Tensor] = None):
        self.q, self.k, self.v, self.o = q, k, v, o
        self.gate, self.up, self.down = gate, up, down
        self.input_norm = input_norm
        self.post_norm = post_norm
        self.qkv_bias = None if q_bias is None else [q_bias, k_bias, v_bias]


class PFlashDecoder:
    """Causal LM forward over packed layers with a device KV cache.

    config keys as PFlashModelForCausalLM's: hidden_size, num_attention_heads,
    num_key_value_heads, intermediate_size, vocab_size, rope_theta
    (default 1e6), rms_norm_eps (default 1e-6); head_dim = hidden_size /
    num_attention_heads.  ``embed`` [vocab, hidden] and ``lm_head`` [vocab,
    hidden] are dense device tensors, ``final_norm`` [hidden].  ``max_seq``
    bounds the cache; ``kv_dtype`` is the uncompressed cache's dtype (fp32
    keeps the reference's arithmetic; other dtypes run the captured step's
    attention as torch ops).  ``kv_mode`` "int8", "2bit" or "2bit_asym"
    stores the cache compressed as CompressedKVCache quantizes it
    (polarflash_rt/kv_cache/compressed_kv.py:68-150): each (token, KV head)
    row as codes plus an fp32 scale (and zero), written by the RoPE kernel and
    dequantized inside the attention kernel; the eager forward attends over
    the dequantized rows.  ``faithful_prefill`` runs the packed linears of a
    multi-token forward in slices of at most 16 tokens, so they take the
    streaming GEMV (fp32 group scales, x' as an fp16 hi + lo pair: fp32-level
    products) instead of the tensor-core GEMM (fp16 weights and x'); it costs
    one weight pass per 16 tokens.

    ``tp`` runs the stack column-parallel (one process per GPU): every layer
    holds this rank's row shards of its seven projections (QWeight.shard_rows:
    rows [r M / P, (r + 1) M / P), q|k|v biases sliced alike), and after each
    projection group (q|k|v, o, gate|up, down) ``tp.gather`` assembles the full
    outputs (parallel.GroupGather: one all-gather per group); norms, RoPE,
    attention, the cache and the lm_head are replicated on every rank.
    """

    GEMV_TOKENS = 16  # the largest batch the streaming GEMV takes in one pass

    def __init__(self, config: Dict, layers: List[DecoderLayer], embed: torch.Tensor, final_norm: torch.Tensor,
                 lm_head: torch.Tensor, max_seq: int, kv_dtype: torch.dtype = torch.float32, kv_mode: str = "fp32",
                 faithful_prefill: bool = False, tp=None):
        self.hidden = int(config["hidden_size"])
        self.nh = int(config["num_attention_heads"])
        self.nkv = int(config["num_key_value_heads"])
        self.hd = self.hidden // self.nh
        self.theta = float(config.get("rope_theta", 1000000.0))
        self.eps = float(config.get("rms_norm_eps", 1e-6))
        self.layers = layers
        self.faithful_prefill = bool(faithful_prefill)
        self.tp = tp
        self.embed = embed
        self.final_norm = final_norm
        self.lm_head = lm_head
        self.max_seq = int(max_seq)
        self.device = embed.device
        dev = self.device
        L = len(layers)
        if kv_mode != "fp32" and kv_mode not in KV_MODES:
            raise ValueError(f"kv_mode {kv_mode!r}: one of fp32, {', '.join(KV_MODES)}")
        self.kv_mode = kv_mode
        if kv_mode == "fp32":
            self.k_cache = torch.zeros(L, self.max_seq, self.nkv, self.hd, dtype=kv_dtype, device=dev)
            self.v_cache = torch.zeros(L, self.max_seq, self.nkv, self.hd, dtype=kv_dtype, device=dev)
        else:
            # rows [L][max_seq][nkv]: codes, fp32 scales, fp32 zeros (2bit_asym)
            rb = kv_row_bytes(kv_mode, self.hd)
            shp = (L, self.max_seq, self.nkv)
            self.k_cache = torch.zeros(shp + (rb,), dtype=torch.uint8, device=dev)
            self.v_cache = torch.zeros(shp + (rb,), dtype=torch.uint8, device=dev)
            self.k_scales = torch.zeros(shp, dtype=torch.float32, device=dev)
            self.v_scales = torch.zeros(shp, dtype=torch.float32, device=dev)
            asym = kv_mode == "2bit_asym"
            self.k_zeros = torch.zeros(shp, dtype=torch.float32, device=dev) if asym else None
            self.v_zeros = torch.zeros(shp, dtype=torch.float32, device=dev) if asym else None
        half = self.hd // 2
        # reference: 1 / theta ** (arange(0, half) / half), fp32
        self.inv_freq = 1.0 / (self.theta ** (torch.arange(0, half, dtype=torch.float32, device=dev) / half))
        self.length = 0  # tokens in the cache
        # one workspace for every packed call of a batch-1 step
        need = 0
        for ly in layers:
            need = max(need, group_workspace_bytes([ly.q, ly.k, ly.v], 1), group_workspace_bytes([ly.gate, ly.up], 1),
                       ly.o.workspace_bytes(1), ly.down.workspace_bytes(1))
        self.ws1 = torch.zeros(need, dtype=torch.uint8, device=dev)
        self.attn_ws = torch.empty(int(_lib.load().pf_decode_attention_workspace_size(self.nh, self.hd, self.max_seq)),
                                   dtype=torch.uint8, device=dev)
        self._graph = None

    # ---- blocks (reference semantics) -------------------------------------
    def _rmsnorm(self, x: torch.Tensor, w: torch.Tensor) -> torch.Tensor:
        var = x.pow(2).mean(-1, keepdim=True)
        return x * torch.rsqrt(var + self.eps) * w

    def _rope_cs(self, pos: torch.Tensor):
        """cos / sin [S, 1, hd/2] of the positions pos [S] (fp32), shared by
        every layer's q and k."""
        f = pos[:, None] * self.inv_freq[None, :]
        return torch.cos(f)[:, None, :], torch.sin(f)[:, None, :]

    def _rope(self, x: torch.Tensor, cs) -> torch.Tensor:
        """x [S, heads, hd] rotated as apply_rotary_pos_emb does (halves)."""
        half = self.hd // 2
        cos, sin = cs
        x1, x2 = x[..., :half], x[..., half:]
        return torch.cat([x1 * cos - x2 * sin, x1 * sin + x2 * cos], dim=-1)

    def _sliced(self, fn, x: torch.Tensor):
        """fn(x), or, under faithful_prefill, fn over 16-token slices of x
        with the outputs concatenated (fn returns a tensor or a list)."""
        n = self.GEMV_TOKENS
        if not self.faithful_prefill or x.shape[0] <= n:
            return fn(x)
        parts = [fn(x[i:i + n]) for i in range(0, x.shape[0], n)]
        if isinstance(parts[0], torch.Tensor):
            return torch.cat(parts)
        return [torch.cat([p[j] for p in parts]) for j in range(len(parts[0]))]

    def _lin(self, ws: List[QWeight], x: torch.Tensor, biases=None, workspace=None) -> List[torch.Tensor]:
        """One projection group over input x (full outputs under tp)."""
        ys = qlinear_multi(ws, x, biases, workspace=workspace) if len(ws) > 1 else \
            [qlinear(ws[0], x, biases[0] if biases else None, workspace=workspace)]
        return self.tp.gather(ys) if self.tp is not None else ys

    def _layer(self, li: int, h: torch.Tensor, cs, attend, ws) -> torch.Tensor:
        ly = self.layers[li]
        S = h.shape[0]
        n = self._rmsnorm(h, ly.input_norm)
        q, k, v = self._sliced(lambda t: self._lin([ly.q, ly.k, ly.v], t, ly.qkv_bias, workspace=ws), n)
        q = self._rope(q.view(S, self.nh, self.hd), cs)
        k = self._rope(k.view(S, self.nkv, self.hd), cs)
        v = v.view(S, self.nkv, self.hd)
        attn = attend(li, q, k, v)  # [S, hidden]
        h = h + self._sliced(lambda t: self._lin([ly.o], t, workspace=ws)[0], attn)
        n2 = self._rmsnorm(h, ly.post_norm)
        g, u = self._sliced(lambda t: self._lin([ly.gate, ly.up], t, workspace=ws), n2)
        return h + self._sliced(lambda t: self._lin([ly.down], t, workspace=ws)[0], F.silu(g) * u)

    # ---- eager forward (prefill, or any number of new tokens) --------------
    def forward(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Logits [S, vocab] for the S new tokens `input_ids` (1-D, on the
        device), appended after the tokens already in the cache."""
        ids = input_ids.reshape(-1).to(self.device)
        S, start = ids.shape[0], self.length
        if start + S > self.max_seq:
            raise ValueError(f"cache holds {self.max_seq} tokens; {start} + {S} requested")
        pos = torch.arange(start, start + S, dtype=torch.float32, device=self.device)
        T = start + S
        # causal within the new tokens, everything before them visible
        mask = torch.arange(T, device=self.device)[None, :] <= (start + torch.arange(S, device=self.device))[:, None]

        def attend(li, q, k, v):
            if self.kv_mode == "fp32":
                self.k_cache[li, start:T] = k.to(self.k_cache.dtype)
                self.v_cache[li, start:T] = v.to(self.v_cache.dtype)
                K = self.k_cache[li, :T].float().permute(1, 0, 2)[None]  # [1, nkv, T, hd]
                V = self.v_cache[li, :T].float().permute(1, 0, 2)[None]
            else:
                K = self._kv_append(li, 0, k, start, T).permute(1, 0, 2)[None]
                V = self._kv_append(li, 1, v, start, T).permute(1, 0, 2)[None]
            o = F.scaled_dot_product_attention(q.permute(1, 0, 2)[None], K, V, attn_mask=mask[None, None],
                                               enable_gqa=True)
            return o[0].permute(1, 0, 2).reshape(S, self.hidden)

        h = self.embed[ids].float()
        ws = self.ws1 if S == 1 else None
        cs = self._rope_cs(pos)
        for li in range(len(self.layers)):
            h = self._layer(li, h, cs, attend, ws)
        self.length = T
        return self._head(self._rmsnorm(h, self.final_norm))

    def _kv_rows(self, li: int, which: int):
        if which == 0:
            return self.k_cache[li], self.k_scales[li], None if self.k_zeros is None else self.k_zeros[li]
        return self.v_cache[li], self.v_scales[li], None if self.v_zeros is None else self.v_zeros[li]

    def _kv_append(self, li: int, which: int, x: torch.Tensor, start: int, T: int) -> torch.Tensor:
        """Quantize rows x [S, nkv, hd] into cache positions start..T-1 and
        return the dequantized rows 0..T-1 [T, nkv, hd] (fp32)."""
        L = _lib.load()
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        m = KV_MODES[self.kv_mode]
        codes, sc, zr = self._kv_rows(li, which)
        x = x.float().contiguous()
        S = T - start
        _lib.check(L.pf_kv_quantize(_p(x), S * self.nkv, self.hd, m, _p(codes[start]), _p(sc[start]),
                                    _p(None if zr is None else zr[start]), st), "pf_kv_quantize")
        out = torch.empty(T, self.nkv, self.hd, dtype=torch.float32, device=self.device)
        _lib.check(L.pf_kv_dequantize(_p(codes), _p(sc), _p(zr), T * self.nkv, self.hd, m, _p(out), st),
                   "pf_kv_dequantize")
        return out

    def _head(self, hn: torch.Tensor) -> torch.Tensor:
        """Dense lm_head in its own dtype, fp32 logits."""
        if self.lm_head.dtype == torch.float32:
            return hn @ self.lm_head.t()
        return (hn.to(self.lm_head.dtype) @ self.lm_head.t()).float()

    # ---- batch-1 decode step as one CUDA graph -----------------------------
    def _step_body(self):
        if self.kv_mode == "fp32" and self.k_cache.dtype != torch.float32:
            return self._step_body_torch()
        L = _lib.load()
        st = ctypes.c_void_p(torch.cuda.current_stream(self.device).cuda_stream)
        H, nh, nkv, hd, ms = self.hidden, self.nh, self.nkv, self.hd, self.max_seq
        scale = 1.0 / math.sqrt(hd)
        h = self.embed.index_select(0, self._tok).float()  # [1, H]: the residual stream, updated in place
        n = torch.empty_like(h)
        delta = None
        for li, ly in enumerate(self.layers):
            _lib.check(L.pf_add_rmsnorm(_p(h), _p(delta), _p(ly.input_norm), _p(n), 1, H, self.eps, st),
                       "pf_add_rmsnorm")
            q, k, v = self._lin([ly.q, ly.k, ly.v], n, ly.qkv_bias, workspace=self.ws1)
            attn = torch.empty(1, H, dtype=torch.float32, device=self.device)
            if self.kv_mode == "fp32":
                _lib.check(L.pf_rope_kv(_p(q), _p(k), _p(v), _p(self.k_cache[li]), _p(self.v_cache[li]),
                                        _p(self._pos), _p(self.inv_freq), nh, nkv, hd, ms, st), "pf_rope_kv")
                _lib.check(L.pf_decode_attention(_p(q), _p(self.k_cache[li]), _p(self.v_cache[li]), _p(self._pos),
                                                 _p(attn), nh, nkv, hd, ms, scale, _p(self.attn_ws),
                                                 self.attn_ws.numel(), st), "pf_decode_attention")
            else:
                m = KV_MODES[self.kv_mode]
                kc, ks, kz = self._kv_rows(li, 0)
                vc, vs, vz = self._kv_rows(li, 1)
                _lib.check(L.pf_rope_kv_compressed(_p(q), _p(k), _p(v), _p(kc), _p(ks), _p(kz), _p(vc), _p(vs),
                                                   _p(vz), _p(self._pos), _p(self.inv_freq), nh, nkv, hd, ms, m, st),
                           "pf_rope_kv_compressed")
                _lib.check(L.pf_decode_attention_compressed(_p(q), _p(kc), _p(ks), _p(kz), _p(vc), _p(vs), _p(vz),
                                                            _p(self._pos), _p(attn), nh, nkv, hd, ms, m, scale,
                                                            _p(self.attn_ws), self.attn_ws.numel(), st),
                           "pf_decode_attention_compressed")
            o = self._lin([ly.o], attn, workspace=self.ws1)[0]
            n2 = torch.empty_like(h)
            _lib.check(L.pf_add_rmsnorm(_p(h), _p(o), _p(ly.post_norm), _p(n2), 1, H, self.eps, st),
                       "pf_add_rmsnorm")
            g, u = self._lin([ly.gate, ly.up], n2, workspace=self.ws1)
            a = torch.empty_like(g)
            _lib.check(L.pf_silu_mul(_p(g), _p(u), _p(a), g.numel(), st), "pf_silu_mul")
            delta = self._lin([ly.down], a, workspace=self.ws1)[0]
        hn = torch.empty_like(h)
        _lib.check(L.pf_add_rmsnorm(_p(h), _p(delta), _p(self.final_norm), _p(hn), 1, H, self.eps, st),
                   "pf_add_rmsnorm")
        self._logits.copy_(self._head(hn))

    def _step_body_torch(self):
        pos_f = self._pos.float()
        slots = torch.arange(self.max_seq, device=self.device)
        mask = (slots <= self._pos)[None, None, None, :]  # [1, 1, 1, max_seq]

        def attend(li, q, k, v):
            self.k_cache[li].index_copy_(0, self._pos, k.to(self.k_cache.dtype))
            self.v_cache[li].index_copy_(0, self._pos, v.to(self.v_cache.dtype))
            K = self.k_cache[li].float().permute(1, 0, 2)[None]  # [1, nkv, max_seq, hd]
            V = self.v_cache[li].float().permute(1, 0, 2)[None]
            o = F.scaled_dot_product_attention(q.permute(1, 0, 2)[None], K, V, attn_mask=mask, enable_gqa=True)
            return o[0].permute(1, 0, 2).reshape(1, self.hidden)

        h = self.embed.index_select(0, self._tok).float()
        cs = self._rope_cs(pos_f)
        for li in range(len(self.layers)):
            h = self._layer(li, h, cs, attend, self.ws1)
        self._logits.copy_(self._head(self._rmsnorm(h, self.final_norm)))

    def capture(self, stream: Optional[torch.cuda.Stream] = None):
        """Capture the batch-1 decode step once (after at least one eager call
        on this device, so the library's one-time set-up has run)."""
        dev = self.device
        self._tok = torch.zeros(1, dtype=torch.long, device=dev)
        self._pos = torch.zeros(1, dtype=torch.long, device=dev)
        self._logits = torch.zeros(1, self.embed.shape[0], dtype=torch.float32, device=dev)
        s = stream if stream is not None else torch.cuda.Stream(dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        saved = self.length
        with torch.cuda.stream(s):
            self._pos.fill_(min(saved, self.max_seq - 1))
            self._step_body()  # warm-up outside the graph (writes the slot the next step overwrites)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=s):
                self._step_body()
        torch.cuda.current_stream(dev).wait_stream(s)
        self._graph = g
        self.length = saved
        return g

    def step(self, token) -> torch.Tensor:
        """Logits [1, vocab] of one new token (int or 1-element device tensor)
        through the captured graph; appends it to the cache."""
        if self._graph is None:
            raise RuntimeError("PFlashDecoder.step: call capture() first")
        if self.length >= self.max_seq:
            raise ValueError(f"cache holds {self.max_seq} tokens")
        if isinstance(token, torch.Tensor):
            self._tok.copy_(token.reshape(1))
        else:
            self._tok.fill_(int(token))
        self._pos.fill_(self.length)
        self._graph.replay()
        self.length += 1
        return self._logits
