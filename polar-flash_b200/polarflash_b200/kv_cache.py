"""Compressed KV cache on the device.

Mirrors ``CompressedKVCache`` (polarflash_rt/kv_cache/compressed_kv.py:
22-282): the same constructor, ``theoretical_memory_bytes``, ``update`` and
``compute_attention_error``, the same per-layer dict of codes / scales /
zeros laid out as the reference lays them out ([batch, heads, seq, ...]),
and the same sliding-window eviction with sink tokens.  The row quantizers
and dequantizers are the library's kernels (pf_kv_quantize,
pf_kv_dequantize), bit-identical to the reference's fp32 arithmetic; inputs
are quantized from their fp32 values.  Modes "polar_qjl", "dictionary" and
unknown names store int8 rows, as the reference's fallback branch does
(:213-225), while ``q_bytes`` keeps the reference's table.

For a decode step, ``PFlashDecoder(kv_mode=...)`` keeps the codes in a
preallocated cache and dequantizes them inside the attention kernel instead
of materialising the context (pf_rope_kv_compressed,
pf_decode_attention_compressed).
"""
import ctypes
import math
from typing import Any, Dict, List, Optional, Tuple

import torch

from . import _lib

KV_MODES = {"int8": 1, "2bit": 2, "2bit_asym": 3}
Q_BYTES = {"fp16": 2.0, "int8": 1.0, "2bit": 0.25, "2bit_asym": 0.25, "polar_qjl": 0.50, "dictionary": 0.25}


def _p(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def kv_row_bytes(mode: str, dim: int) -> int:
    """Bytes of one row of codes: dim for int8, ceil(dim / 4) for the 2-bit modes."""
    return dim if mode == "int8" else (dim + 3) // 4


def kv_quantize(x: torch.Tensor, mode: str) -> Tuple[torch.Tensor, torch.Tensor, Optional[torch.Tensor]]:
    """Rows of x [..., d] (CUDA) -> (codes [..., row_bytes] int8/uint8,
    scales [..., 1] fp32, zeros [..., 1] fp32 for 2bit_asym else None)."""
    if not x.is_cuda:
        raise RuntimeError("kv_quantize: the compressed KV cache runs on a CUDA device only")
    m = KV_MODES[mode]
    xf = x.detach().float().contiguous()
    d = xf.shape[-1]
    rows = xf.numel() // d if d else 0
    lead = tuple(xf.shape[:-1])
    codes = torch.empty(lead + (kv_row_bytes(mode, d),), dtype=torch.int8 if mode == "int8" else torch.uint8,
                        device=x.device)
    scales = torch.empty(lead + (1,), dtype=torch.float32, device=x.device)
    zeros = torch.empty_like(scales) if mode == "2bit_asym" else None
    if rows == 0:
        return codes, scales, zeros
    L = _lib.load()
    st = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(L.pf_kv_quantize(_p(xf), rows, d, m, _p(codes), _p(scales), _p(zeros), st), "pf_kv_quantize")
    return codes, scales, zeros


def kv_dequantize(codes: torch.Tensor, scales: torch.Tensor, zeros: Optional[torch.Tensor], d: int,
                  mode: str) -> torch.Tensor:
    """fp32 rows [..., d] of kv_quantize's output."""
    m = KV_MODES[mode]
    codes = codes.contiguous()
    scales = scales.contiguous()
    zeros = zeros.contiguous() if zeros is not None else None
    lead = tuple(codes.shape[:-1])
    out = torch.empty(lead + (d,), dtype=torch.float32, device=codes.device)
    rows = out.numel() // d if d else 0
    if rows == 0:
        return out
    L = _lib.load()
    st = ctypes.c_void_p(torch.cuda.current_stream(codes.device).cuda_stream)
    _lib.check(L.pf_kv_dequantize(_p(codes), _p(scales), _p(zeros), rows, d, m, _p(out), st), "pf_kv_dequantize")
    return out


class CompressedKVCache:
    """Compressed KV cache with the reference's interface (compressed_kv.py:22-282)."""

    def __init__(self, num_layers: int, num_kv_heads: int, head_dim: int, max_context_len: int = 8192,
                 mode: str = "int8", window_size: Optional[int] = None, num_sink_tokens: int = 4):
        self.num_layers = num_layers
        self.num_kv_heads = num_kv_heads
        self.head_dim = head_dim
        self.max_context_len = max_context_len
        self.mode = mode.lower()
        self.window_size = window_size
        self.num_sink_tokens = num_sink_tokens
        self.q_bytes = Q_BYTES.get(self.mode, 1.0)
        self.layers: List[Dict[str, Any]] = [
            {"k_data": None, "v_data": None, "k_scales": None, "v_scales": None, "k_zeros": None, "v_zeros": None,
             "seq_len": 0}
            for _ in range(num_layers)
        ]

    def theoretical_memory_bytes(self, num_tokens: int) -> int:
        """M_KV = 2 * L * T * H_kv * D * q (compressed_kv.py:63-66)."""
        return int(2 * self.num_layers * num_tokens * self.num_kv_heads * self.head_dim * self.q_bytes)

    @property
    def _qmode(self) -> str:
        return self.mode if self.mode in KV_MODES else "int8"

    def update(self, layer_idx: int, key_states: torch.Tensor,
               value_states: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Append key/value states [batch, kv_heads, seq, head_dim] to layer
        `layer_idx` and return the whole (dequantized) context, windowed."""
        layer = self.layers[layer_idx]
        d = key_states.shape[-1]
        cat = (lambda a, b: b if a is None else torch.cat([a, b], dim=2))  # noqa: E731
        if self.mode == "fp16":
            layer["k_data"] = cat(layer["k_data"], key_states.half())
            layer["v_data"] = cat(layer["v_data"], value_states.half())
            k_out, v_out = layer["k_data"], layer["v_data"]
        else:
            mode = self._qmode
            kq, ks, kz = kv_quantize(key_states, mode)
            vq, vs, vz = kv_quantize(value_states, mode)
            layer["k_data"] = cat(layer["k_data"], kq)
            layer["v_data"] = cat(layer["v_data"], vq)
            layer["k_scales"] = cat(layer["k_scales"], ks)
            layer["v_scales"] = cat(layer["v_scales"], vs)
            if mode == "2bit_asym":
                layer["k_zeros"] = cat(layer["k_zeros"], kz)
                layer["v_zeros"] = cat(layer["v_zeros"], vz)
            k_out = kv_dequantize(layer["k_data"], layer["k_scales"], layer["k_zeros"], d, mode)
            v_out = kv_dequantize(layer["v_data"], layer["v_scales"], layer["v_zeros"], d, mode)
        total = k_out.shape[2]
        if self.window_size and total > self.window_size:
            keep = list(range(self.num_sink_tokens)) + list(
                range(total - self.window_size + self.num_sink_tokens, total))
            idx = torch.tensor(keep, device=k_out.device)
            k_out = k_out.index_select(2, idx)
            v_out = v_out.index_select(2, idx)
        layer["seq_len"] = k_out.shape[2]
        return k_out, v_out

    def compute_attention_error(self, query: torch.Tensor, fp_key: torch.Tensor,
                                quant_key: torch.Tensor) -> Dict[str, float]:
        """Logit MSE, logit cosine similarity and softmax KL between exact and
        quantized keys (compressed_kv.py:235-258); query [b, h, 1, d]."""
        scale = 1.0 / math.sqrt(self.head_dim)
        fp_key = fp_key.to(query.dtype)
        quant_key = quant_key.to(query.dtype)
        exact = torch.matmul(query, fp_key.transpose(-1, -2)) * scale
        quant = torch.matmul(query, quant_key.transpose(-1, -2)) * scale
        mse = float(torch.mean((exact - quant) ** 2).item())
        cos = float(torch.nn.functional.cosine_similarity(exact.flatten(), quant.flatten(), dim=0).item())
        pe, pq = torch.softmax(exact, dim=-1), torch.softmax(quant, dim=-1)
        kl = float(torch.sum(pe * (torch.log(pe + 1e-9) - torch.log(pq + 1e-9))).item())
        return {"logit_mse": mse, "cosine_similarity": cos, "kl_divergence": max(0.0, kl)}
