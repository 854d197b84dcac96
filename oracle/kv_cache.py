"""CPU oracle for the compressed KV cache -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU legs use
it, as the checker.  A numpy fp32 restatement of CompressedKVCache's row
quantizers (polarflash_rt/kv_cache/compressed_kv.py):

  int8       _quantize_int8 / _dequantize_int8           :68-77
  2bit       _quantize_2bit / _dequantize_2bit           :79-112
  2bit_asym  _quantize_2bit_asym / _dequantize_2bit_asym :114-150
  update     append + dequantize whole context, sliding window with sink
             tokens                                      :152-233

Every step is one fp32 operation as in the reference (numpy float32 with
Python-float operands stays float32), round is to nearest even.  Pinned by
tests/golden/kv_cache.npz, written by the reference itself
(tests/golden/make_kv_golden.py).
"""
import numpy as np

MODES = {"int8": 1, "2bit": 2, "2bit_asym": 3}


def _pack2(c):
    """uint8 codes [..., d] -> [..., ceil(d/4)], c0 << 6 | c1 << 4 | c2 << 2 | c3."""
    d = c.shape[-1]
    pad = (-d) % 4
    if pad:
        c = np.concatenate([c, np.zeros(c.shape[:-1] + (pad,), np.uint8)], -1)
    r = c.reshape(c.shape[:-1] + (-1, 4))
    return ((r[..., 0] << 6) | (r[..., 1] << 4) | (r[..., 2] << 2) | r[..., 3]).astype(np.uint8)


def _unpack2(p, d):
    v = np.stack([(p >> 6) & 3, (p >> 4) & 3, (p >> 2) & 3, p & 3], -1)
    return v.reshape(p.shape[:-1] + (-1,))[..., :d]


def quantize(x, mode):
    """Rows of x [..., d] (fp32) -> (codes, scales [..., 1], zeros [..., 1] or None)."""
    x = np.asarray(x, np.float32)
    if mode == "int8":
        s = np.maximum(np.abs(x).max(-1, keepdims=True) / np.float32(127.0), np.float32(1e-8))
        q = np.clip(np.rint(x / s), -128, 127).astype(np.int8)
        return q, s, None
    if mode == "2bit":
        delta = np.maximum(np.abs(x).max(-1, keepdims=True) / np.float32(1.75), np.float32(1e-8))
        idx = np.clip(np.floor(x / delta + np.float32(2.0)), 0, 3).astype(np.uint8)
        return _pack2(idx), delta, None
    if mode == "2bit_asym":
        mn = x.min(-1, keepdims=True)
        mx = x.max(-1, keepdims=True)
        s = np.maximum((mx - mn) / np.float32(3.0), np.float32(1e-8))
        q = np.clip(np.rint((x - mn) / s), 0, 3).astype(np.uint8)
        return _pack2(q), s, mn
    raise ValueError(mode)


def dequantize(codes, scales, zeros, d, mode):
    """fp32 rows [..., d] of quantize()'s output."""
    if mode == "int8":
        return codes.astype(np.float32) * scales
    c = _unpack2(codes, d).astype(np.float32)
    if mode == "2bit":
        return (c - np.float32(1.5)) * scales
    return c * scales + zeros


def window_indices(total, window, sinks):
    """Positions CompressedKVCache.update keeps (compressed_kv.py:227-231)."""
    if not window or total <= window:
        return list(range(total))
    return list(range(sinks)) + list(range(total - window + sinks, total))
