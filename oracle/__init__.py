"""CPU oracle for the compressed-linear path -- TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg
import this package, and only as the checker (never as the thing measured on
the GPU, never shipped in the product path).  It wraps ``pf_oracle.c`` (built
by ``oracle/build.py``) with numpy-facing helpers and composes the reference
pipeline ``UnifiedQuantizer.dequantize`` -> inverse RWHT -> matvec
(polarflash_quant/unified_quantizer.py:242-324, polarflash_rt/cpu/engine.py:58-96).

Parity pins: tests/golden holds fixtures produced by the reference itself.
"""
import ctypes
import os

import numpy as np

from . import build as _build

_LIB = None


def lib():
    global _LIB
    if _LIB is None:
        path = _build.OUT
        if not os.path.exists(path):
            path = _build.build()
        L = ctypes.CDLL(path)
        P = ctypes.c_void_p
        I64 = ctypes.c_int64
        I = ctypes.c_int
        sigs = {
            "pfo_unpack_int4": [P, I64, P], "pfo_pack_int4": [P, I64, P],
            "pfo_unpack_int2": [P, I64, P], "pfo_pack_int2": [P, I64, P],
            "pfo_unpack_int3": [P, I64, P], "pfo_pack_int3": [P, I64, P],
            "pfo_g128_words": [I],
            "pfo_pack_g128": [I, P, I64, I64, P], "pfo_unpack_g128": [I, P, I64, I64, P],
            "pfo_quant_g128_asym": [I, P, I64, I64, P, P, P],
            "pfo_dequant_g128_asym": [P, P, P, I64, I64, P],
            "pfo_hadamard_block": [I, I64],
            "pfo_hadamard_plan": [I, I64, P, P, I],
            "pfo_rwht": [P, I64, I64, I, P, I, P],
            "pfo_e8_roots": [P], "pfo_e8_encode": [P, I64, I64, P, P],
            "pfo_e8_decode": [P, P, I64, I64, P],
            "pfo_polar_alloc": [I, ctypes.c_double, P],
            "pfo_pack_bits_msb": [P, I64, I, P], "pfo_unpack_bits_msb": [P, I64, I, P],
            "pfo_polar_decode": [P, I64, I, P, ctypes.c_double, P],
            "pfo_polar_decode_cb": [P, I64, I, P, ctypes.c_double, P, P, I, P],
            "pfo_polar2d_decode": [P, I64, I, I, ctypes.c_double, P],
            "pfo_matvec": [P, I64, I64, P, I64, P],
            "pfo_matvec_f32": [P, I64, I64, P, I64, P],
            "pfo_num_threads": [], "pfo_set_num_threads": [I],
        }
        for name, argt in sigs.items():
            fn = getattr(L, name)
            fn.argtypes = argt
        L.pfo_g128_words.restype = I
        L.pfo_pack_g128.restype = I
        L.pfo_unpack_g128.restype = I
        L.pfo_quant_g128_asym.restype = I
        L.pfo_hadamard_block.restype = I
        L.pfo_hadamard_plan.restype = I
        L.pfo_e8_encode.restype = I
        L.pfo_polar_alloc.restype = I
        L.pfo_num_threads.restype = I
        _LIB = L
    return _LIB


def _p(a):
    return a.ctypes.data_as(ctypes.c_void_p)


def _c(a, dtype):
    return np.ascontiguousarray(a, dtype=dtype)


# ----------------------------------------------------------------- bit packing
def unpack_int4(packed, n):
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    out = np.empty(n, np.int8)
    lib().pfo_unpack_int4(_p(b), n, _p(out))
    return out


def pack_int4(v):
    v = _c(v, np.int8).ravel()
    out = np.empty((v.size + 1) // 2, np.uint8)
    lib().pfo_pack_int4(_p(v), v.size, _p(out))
    return out


def unpack_int2(packed, n):
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    out = np.empty(n, np.uint8)
    lib().pfo_unpack_int2(_p(b), n, _p(out))
    return out


def pack_int2(v):
    v = _c(v, np.uint8).ravel()
    out = np.empty((v.size + 3) // 4, np.uint8)
    lib().pfo_pack_int2(_p(v), v.size, _p(out))
    return out


def unpack_int3(packed, n):
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    out = np.empty(n, np.uint8)
    lib().pfo_unpack_int3(_p(b), n, _p(out))
    return out


def pack_int3(v):
    v = _c(v, np.uint8).ravel()
    out = np.empty(((v.size + 7) // 8) * 3, np.uint8)
    lib().pfo_pack_int3(_p(v), v.size, _p(out))
    return out


def g128_words(bits):
    return lib().pfo_g128_words(bits)


def pack_g128(bits, q):
    q = _c(q, np.uint8)
    M, K = q.shape
    out = np.empty((M, (K // 128) * g128_words(bits)), np.uint32)
    assert lib().pfo_pack_g128(bits, _p(q), M, K, _p(out)) == 0
    return out


def unpack_g128(bits, words, M, K):
    words = _c(words, np.uint32)
    out = np.empty((M, K), np.uint8)
    assert lib().pfo_unpack_g128(bits, _p(words), M, K, _p(out)) == 0
    return out


def quant_g128_asym(bits, w):
    w = _c(w, np.float32)
    M, K = w.shape
    q = np.empty((M, K), np.uint8)
    s = np.empty((M, K // 128), np.uint16)
    m = np.empty((M, K // 128), np.uint16)
    assert lib().pfo_quant_g128_asym(bits, _p(w), M, K, _p(q), _p(s), _p(m)) == 0
    return q, s.view(np.float16), m.view(np.float16)


def dequant_g128_asym(q, s, m):
    q = _c(q, np.uint8)
    M, K = q.shape
    s = _c(np.asarray(s).view(np.uint16) if np.asarray(s).dtype == np.float16 else s, np.uint16)
    m = _c(np.asarray(m).view(np.uint16) if np.asarray(m).dtype == np.float16 else m, np.uint16)
    out = np.empty((M, K), np.float32)
    lib().pfo_dequant_g128_asym(_p(q), _p(s), _p(m), M, K, _p(out))
    return out


# ----------------------------------------------------------------- Hadamard
def hadamard_block(req, K):
    return lib().pfo_hadamard_block(req, K)


def hadamard_signs(K, req_block, seed=42):
    """Per-column +-1 signs of BlockHadamardTransform(K, req_block, seed)
    (hadamard.py:93-116): the same torch generator calls, full-block signs
    repeated over the full blocks, then one draw per remainder block."""
    import torch

    block = hadamard_block(req_block, K)
    gen = torch.Generator().manual_seed(seed)
    full = (torch.randint(0, 2, (block,), generator=gen).float() * 2.0 - 1.0).numpy()
    nfull = K // block
    parts = [np.tile(full, nfull)]
    rem = K - nfull * block
    while rem > 1:
        p2 = 1
        while p2 * 2 <= rem:
            p2 *= 2
        parts.append((torch.randint(0, 2, (p2,), generator=gen).float() * 2.0 - 1.0).numpy())
        rem -= p2
    if rem == 1:
        parts.append(np.ones(1, np.float32))
    return np.concatenate(parts).astype(np.float32), block


def rwht(x, block, signs, inverse=False):
    x = _c(x, np.float32)
    shp = x.shape
    K = shp[-1]
    rows = int(np.prod(shp[:-1])) if len(shp) > 1 else 1
    signs = _c(signs, np.float32)
    out = np.empty_like(x)
    lib().pfo_rwht(_p(x), rows, K, block, _p(signs), 1 if inverse else 0, _p(out))
    return out


# ----------------------------------------------------------------- E8
def e8_roots():
    r = np.empty((240, 8), np.float32)
    lib().pfo_e8_roots(_p(r))
    return r


def e8_encode(w):
    w = _c(w, np.float32)
    M, K = w.shape
    idx = np.empty((M, K // 8, 2), np.uint8)
    sc = np.empty((M, K // 128, 2), np.uint16)
    assert lib().pfo_e8_encode(_p(w), M, K, _p(idx), _p(sc)) == 0
    return idx, sc.view(np.float16)


def e8_decode(idx, scales, M, K):
    idx = _c(idx, np.uint8)
    sc = _c(np.asarray(scales).view(np.uint16), np.uint16)
    out = np.empty((M, K), np.float32)
    lib().pfo_e8_decode(_p(idx), _p(sc), M, K, _p(out))
    return out


# ----------------------------------------------------------------- polar
def polar_alloc(d, bpw):
    a = np.empty(64, np.int32)
    n = lib().pfo_polar_alloc(d, float(bpw), _p(a))
    return [int(v) for v in a[:n]]


def _forward_recursive(blocks):
    """forward_recursive (polar_quant.py:219-250) with the same torch ops, so the
    radii and angles are the reference's to the last bit."""
    import torch

    eps = 1e-12
    curr = blocks.clone()
    angles = []
    d = curr.shape[-1]
    level = 0
    while d > 1:
        left = curr[..., 0::2]
        right = curr[..., 1::2]
        sum_sq = left ** 2 + right ** 2
        zero = sum_sq <= eps ** 2
        r = torch.sqrt(torch.clamp(sum_sq, min=0.0))
        r[zero] = 0.0
        if level == 0:
            th = torch.atan2(right, left)
        else:
            th = torch.atan2(torch.clamp(right, min=0.0), torch.clamp(left, min=0.0))
        th[zero] = 0.0
        angles.append(th)
        curr = r
        d = curr.shape[-1]
        level += 1
    return curr.squeeze(-1), angles


def polar_encode(w, d, alloc):
    """encode_packed (polar_quant.py:381-487) for uniform angle codes: torch for
    the float steps (as the reference), C for the MSB-first bit stream.
    Returns (payload bytes, r_scale)."""
    import math

    import torch

    flat = torch.from_numpy(np.ascontiguousarray(w, np.float32).ravel())
    rem = flat.numel() % d
    if rem:
        flat = torch.cat([flat, torch.zeros(d - rem)])
    nblk = flat.numel() // d
    top, angle_levels = _forward_recursive(flat.view(nblk, d))
    r_bits = alloc[0]
    r_max = float(torch.max(top).item()) + 1e-12
    r_scale = r_max / float((1 << r_bits) - 1)
    r_code = torch.clamp(torch.round(top / r_scale), 0, (1 << r_bits) - 1).long()
    codes = [r_code]
    col = 1
    for lvl, angles in enumerate(angle_levels):
        fa = angles.view(nblk, -1)
        for j in range(fa.shape[1]):
            th = fa[:, j]
            levels = 1 << alloc[col]
            if lvl == 0:
                nt = (th + math.pi) / (2.0 * math.pi)
            else:
                nt = th / (0.5 * math.pi)
            nt = torch.clamp(nt, 0.0, 1.0 - 1e-7)
            codes.append(torch.clamp(torch.floor(nt * levels), 0, levels - 1).long())
            col += 1
    acc = torch.zeros(nblk, dtype=torch.int64)
    shift = 0
    for i in range(len(alloc) - 1, -1, -1):
        acc |= codes[i] << shift
        shift += alloc[i]
    words = np.ascontiguousarray(acc.numpy().astype(np.uint64))
    tb = sum(alloc)
    out = np.zeros((nblk * tb + 7) // 8, np.uint8)
    lib().pfo_pack_bits_msb(_p(words), nblk, tb, _p(out))
    return out.tobytes(), r_scale


def unpack_bits_msb(packed, nblk, total_bits):
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    out = np.empty(nblk, np.uint64)
    lib().pfo_unpack_bits_msb(_p(b), nblk, total_bits, _p(out))
    return out


def polar_decode(packed, nblk, d, alloc, r_scale, codebooks=None):
    """decode_packed (polar_quant.py:489-575); `codebooks` is the list of
    learned per-level angle codebooks (fit_codebooks, polar_quant.py:274-300)
    when the payload was encoded with them."""
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    a = _c(alloc, np.int32)
    out = np.empty(nblk * d, np.float32)
    if codebooks:
        cb = _c(np.concatenate([np.asarray(c, np.float32).ravel() for c in codebooks]), np.float32)
        ln = _c([len(np.asarray(c).ravel()) for c in codebooks], np.int32)
        lib().pfo_polar_decode_cb(_p(b), nblk, d, _p(a), float(r_scale), _p(cb), _p(ln), len(codebooks), _p(out))
    else:
        lib().pfo_polar_decode(_p(b), nblk, d, _p(a), float(r_scale), _p(out))
    return out


def polar2d_decode(packed, npairs, r_bits, th_bits, r_scale):
    b = _c(np.frombuffer(bytes(packed), np.uint8), np.uint8)
    out = np.empty(npairs * 2, np.float32)
    lib().pfo_polar2d_decode(_p(b), npairs, r_bits, th_bits, float(r_scale), _p(out))
    return out


# ----------------------------------------------------------------- dense
def matvec(W, x):
    """y[n, m] = sum_k W[m, k] x[n, k] in double."""
    W = _c(W, np.float32)
    x = _c(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    M, K = W.shape
    N = x.shape[0]
    y = np.empty((N, M), np.float32)
    lib().pfo_matvec(_p(W), M, K, _p(x), N, _p(y))
    return y


def matvec_f32(W, x):
    W = _c(W, np.float32)
    x = _c(x, np.float32)
    if x.ndim == 1:
        x = x[None]
    M, K = W.shape
    N = x.shape[0]
    y = np.empty((N, M), np.float32)
    lib().pfo_matvec_f32(_p(W), M, K, _p(x), N, _p(y))
    return y


def num_threads():
    return lib().pfo_num_threads()


def set_num_threads(n):
    lib().pfo_set_num_threads(n)


# ----------------------------------------------------------------- pipelines
def dequantize(fmt, payload, M, K, meta):
    """W_hat for a payload, as UnifiedQuantizer.dequantize does it
    (unified_quantizer.py:242-324): decode, then inverse block RWHT when the
    metadata says the weight was rotated.

    fmt names: int4_g128 / int3_g128 / int2_g128 (payload = dict(words, s, m)),
    int4 / int3 / int2 (reference per-tensor streams), e8_rvq2_g128
    (dict(idx, scales)), polar_recursive (bytes, meta alloc/r_scale/block_size,
    learned_codebooks when has_learned_codebooks), polar (2-D pairs), fp16 and
    the e8 backends' fp16 reconstructions (e8_lattice, e8_rvq).
    """
    bits = {"int4": 4, "int3": 3, "int2": 2}
    if fmt.endswith("_g128") and fmt[:4] in bits:
        b = bits[fmt[:4]]
        q = unpack_g128(b, payload["words"], M, K)
        W = dequant_g128_asym(q, payload["s"], payload["m"])
    elif fmt in bits:
        n = M * K
        scale = np.float32(meta.get("scale", 1.0))
        if fmt == "int4":
            q = unpack_int4(payload, n).astype(np.float32)
        elif fmt == "int3":
            q = unpack_int3(payload, n).astype(np.float32) - np.float32(4)
        else:
            q = unpack_int2(payload, n).astype(np.float32) - np.float32(2)
        W = (q * scale).reshape(M, K).astype(np.float32)
    elif fmt == "e8_rvq2_g128":
        W = e8_decode(payload["idx"], payload["scales"], M, K)
    elif fmt == "polar_recursive":
        d = int(meta.get("block_size", 8))
        nblk = int(meta["num_blocks"])
        cbs = meta.get("learned_codebooks") if meta.get("has_learned_codebooks") else None
        flat = polar_decode(payload, nblk, d, meta["alloc"], meta["r_scale"], cbs)
        pad = int(meta.get("pad_len", 0))
        if pad:
            flat = flat[:-pad]
        W = flat.reshape(M, K)
    elif fmt == "polar":
        npairs = (M * K + int(meta.get("padded", 0))) // 2
        flat = polar2d_decode(payload, npairs, int(meta.get("r_bits", 4)),
                              int(meta.get("theta_bits", 4)), meta.get("r_scale", 1.0))
        W = flat[: M * K].reshape(M, K)
    elif fmt in ("fp16", "e8_lattice", "e8_rvq"):  # e8 backends store fp16 reconstructions (:304-306)
        W = np.frombuffer(bytes(payload), np.float16).astype(np.float32).reshape(M, K)
    else:
        raise ValueError(f"oracle: unknown format {fmt}")
    if meta.get("hadamard_rotation", False):
        signs, block = hadamard_signs(K, int(meta.get("hadamard_block_size", 512)))
        W = rwht(W, block, signs, inverse=True)
    return np.ascontiguousarray(W, np.float32)


def linear(fmt, payload, M, K, meta, x, bias=None):
    """Reference forward: W_hat = dequantize(...); y = x @ W_hat.T (+ bias)
    (polarflash_rt/cpu/engine.py:90-96)."""
    W = dequantize(fmt, payload, M, K, meta)
    y = matvec(W, np.asarray(x, np.float32).reshape(-1, K))
    if bias is not None:
        y = y + np.asarray(bias, np.float32)[None]
    return y
