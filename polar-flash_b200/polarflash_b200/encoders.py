"""Weight encoders (offline, torch; CPU or CUDA tensors).

Reference formats are restated from the reference encoders so payloads are
byte-identical; the extension formats (group-128 asymmetric INT, E8 root
residual VQ) are defined here in the reference's conventions, with every float
step written as separate elementwise torch ops in a fixed order so CPU and
CUDA produce the same codes.
"""
import math
from typing import Dict, List, Tuple

import torch

GROUP = 128


# ---------------------------------------------------------------- bit packing
def pack_int4(q: torch.Tensor) -> torch.Tensor:
    """pack_int4 (polarflash_quant/bitpacking.py:16-31): signed [-8, 7] -> bytes,
    even element in the low nibble, odd length padded with the value 0."""
    flat = q.flatten().to(torch.int16)
    if flat.numel() % 2:
        flat = torch.cat([flat, flat.new_zeros(1)])
    u = ((flat + 8) & 0xF).to(torch.uint8)
    return u[0::2] | (u[1::2] << 4)


def pack_int2(q: torch.Tensor) -> torch.Tensor:
    """pack_int2 (bitpacking.py:49-65): codes [0, 3], 4 per byte, LSB first."""
    flat = q.flatten().to(torch.uint8) & 3
    rem = flat.numel() % 4
    if rem:
        flat = torch.cat([flat, flat.new_zeros(4 - rem)])
    return flat[0::4] | (flat[1::4] << 2) | (flat[2::4] << 4) | (flat[3::4] << 6)


def pack_int3(q: torch.Tensor) -> torch.Tensor:
    """pack_int3 (bitpacking.py:88-123): codes [0, 7], 8 per 3 bytes, LSB-first
    24-bit chunks."""
    flat = q.flatten().to(torch.int32) & 7
    rem = flat.numel() % 8
    if rem:
        flat = torch.cat([flat, flat.new_zeros(8 - rem)])
    v = flat.view(-1, 8)
    chunk = torch.zeros(v.shape[0], dtype=torch.int32, device=v.device)
    for i in range(8):
        chunk |= v[:, i] << (3 * i)
    out = torch.stack([chunk & 0xFF, (chunk >> 8) & 0xFF, (chunk >> 16) & 0xFF], 1)
    return out.to(torch.uint8).flatten()


def g128_words_per_group(bits: int) -> int:
    return {4: 16, 3: 13, 2: 8}[bits]


def pack_g128(q: torch.Tensor, bits: int) -> torch.Tensor:
    """Group-128 word layout: per (row, 128-column group) INT4 16 words of 8
    codes, INT2 8 words of 16 codes (code i at bits bits*i, the reference
    order read as little-endian u32), INT3 13 words of 10 codes (bits 30-31 and
    the last 2 slots zero).  Returns int32 [M, (K/128) * words]."""
    M, K = q.shape
    if K % GROUP:
        raise ValueError(f"group-128 formats need K % 128 == 0, got K={K}")
    G = K // GROUP
    per = 10 if bits == 3 else 32 // bits
    v = q.to(torch.int64).view(M, G, GROUP)
    if bits == 3:
        v = torch.cat([v, v.new_zeros(M, G, 2)], -1)
    v = v.view(M, G, -1, per)
    w = torch.zeros(v.shape[:-1], dtype=torch.int64, device=q.device)
    for i in range(per):
        w |= v[..., i] << (bits * i)
    w = torch.where(w >= 2 ** 31, w - 2 ** 32, w)
    return w.to(torch.int32).reshape(M, -1).contiguous()


# ---------------------------------------------------------------- group asym INT
def quant_g128_asym(w: torch.Tensor, bits: int) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
    """Group-128 asymmetric quantizer in the reference's asymmetric convention
    (polarflash_rt/kv_cache/compressed_kv.py:115-146): s = clamp((max-min)/(2^b-1),
    1e-8), q = clamp(round((w - min)/s), 0, 2^b - 1), w_hat = q*s + min; s and min
    stored as fp16 and q computed against the stored values (an s that rounds
    to 0 in fp16 becomes 2^-24).  Returns (q uint8 [M,K], s fp16 [M,G], m fp16 [M,G])."""
    M, K = w.shape
    if K % GROUP:
        raise ValueError(f"group-128 formats need K % 128 == 0, got K={K}")
    G = K // GROUP
    g = w.float().reshape(M, G, GROUP)
    mn = g.amin(-1)
    mx = g.amax(-1)
    L = float((1 << bits) - 1)
    s = torch.clamp((mx - mn) / L, min=1e-8)
    sh = s.half()
    tiny = torch.tensor(2.0 ** -24, dtype=torch.float16, device=w.device)
    sh = torch.where(sh == 0, tiny, sh)
    mh = mn.half()
    q = torch.round((g - mh.float()[..., None]) / sh.float()[..., None])
    q = torch.clamp(q, 0.0, L).to(torch.uint8).reshape(M, K)
    return q, sh.contiguous(), mh.contiguous()


# ---------------------------------------------------------------- reference per-tensor INT
def quant_int_per_tensor(w: torch.Tensor, backend: str) -> Tuple[torch.Tensor, float]:
    """UnifiedQuantizer int4/int3/int2 branches (unified_quantizer.py:154-178):
    per-tensor symmetric scale, returns (packed bytes uint8, scale)."""
    w = w.float()
    max_val = torch.max(torch.abs(w)).item()
    if backend == "int4":
        scale = max_val / 7.0 if max_val > 1e-12 else 1.0
        q = torch.clamp(torch.round(w / scale), -8, 7).to(torch.int8)
        return pack_int4(q), float(scale)
    if backend == "int3":
        scale = max_val / 3.0 if max_val > 1e-12 else 1.0
        q = torch.clamp(torch.round(w / scale), -4, 3).to(torch.int8)
        return pack_int3((q + 4).to(torch.uint8)), float(scale)
    if backend == "int2":
        scale = max_val / 1.5 if max_val > 1e-12 else 1.0
        q = torch.clamp(torch.round(w / scale), -2, 1).to(torch.int8)
        return pack_int2((q + 2).to(torch.uint8)), float(scale)
    raise ValueError(f"not a per-tensor INT backend: {backend}")


# ---------------------------------------------------------------- E8 roots / RVQ
def e8_roots(device="cpu") -> torch.Tensor:
    """generate_e8_roots order (polarflash_quant/lattice/e8_lattice.py:21-50)."""
    roots = []
    for i in range(8):
        for j in range(i + 1, 8):
            for s1 in (-1.0, 1.0):
                for s2 in (-1.0, 1.0):
                    v = [0.0] * 8
                    v[i] = s1
                    v[j] = s2
                    roots.append(v)
    for mask in range(256):
        if bin(mask).count("1") % 2 == 0:
            roots.append([-0.5 if (mask >> b) & 1 else 0.5 for b in range(8)])
    return torch.tensor(roots, dtype=torch.float32, device=device)


def _e8_tables(device):
    roots = e8_roots(device)
    pairs = []
    for i in range(8):
        for j in range(i + 1, 8):
            for s1 in (-1.0, 1.0):
                for s2 in (-1.0, 1.0):
                    pairs.append((i, j, s1, s2))
    I = torch.tensor([p[0] for p in pairs], device=device)
    J = torch.tensor([p[1] for p in pairs], device=device)
    S1 = torch.tensor([p[2] for p in pairs], device=device)
    S2 = torch.tensor([p[3] for p in pairs], device=device)
    signs2 = torch.sign(roots[112:])  # +-1 per coordinate of the half-integer roots
    return roots, I, J, S1, S2, signs2


def _tree16(v: torch.Tensor) -> torch.Tensor:
    """Pairwise-tree sum over the last dim of size 16: (0+1)+(2+3) ... level by level."""
    while v.shape[-1] > 1:
        v = v[..., 0::2] + v[..., 1::2]
    return v[..., 0]


def e8_dots(e: torch.Tensor, tables) -> torch.Tensor:
    """<r_k, e> for all 240 roots in the fixed fp32 order of the format:
    (+-1,+-1) roots one add; half-integer roots ((t0+t1)+(t2+t3)) +
    ((t4+t5)+(t6+t7)) then * 0.5."""
    roots, I, J, S1, S2, signs2 = tables
    a = e[..., I] * S1
    b = e[..., J] * S2
    d1 = a + b
    t = e.unsqueeze(-2) * signs2  # [..., 128, 8]
    p0 = (t[..., 0] + t[..., 1]) + (t[..., 2] + t[..., 3])
    p1 = (t[..., 4] + t[..., 5]) + (t[..., 6] + t[..., 7])
    d2 = (p0 + p1) * 0.5
    return torch.cat([d1, d2], -1)


def e8_encode(w: torch.Tensor, rows_per_chunk: int = 64) -> Tuple[torch.Tensor, torch.Tensor]:
    """Extension "E8 2-stage root residual VQ, group 128".  For each 8-vector e
    of a (row, 128-column group) and stage t = 1, 2: idx = argmax_k <r_k, e>
    (lowest k on ties; the nearest root for any positive scale since every root
    has |r|^2 = 2, e8_lattice.py:46-49), s_t = fp16(tree16(<r_idx, e>) / 32) (least
    squares for the group), e <- e - s_t r_idx.  Returns idx uint8 [M, K/8, 2]
    and scales fp16 [M, K/128, 2]."""
    M, K = w.shape
    if K % GROUP:
        raise ValueError(f"E8 group-128 format needs K % 128 == 0, got K={K}")
    G = K // GROUP
    dev = w.device
    tables = _e8_tables(dev)
    roots = tables[0]
    idx_out = torch.empty(M, K // 8, 2, dtype=torch.uint8, device=dev)
    sc_out = torch.empty(M, G, 2, dtype=torch.float16, device=dev)
    for r0 in range(0, M, rows_per_chunk):
        r1 = min(M, r0 + rows_per_chunk)
        e = w[r0:r1].float().reshape(r1 - r0, G, 16, 8).clone()
        for t in range(2):
            d = e8_dots(e, tables)
            best = torch.argmax(d, dim=-1)
            bv = torch.gather(d, -1, best.unsqueeze(-1)).squeeze(-1)
            sh = (_tree16(bv) / 32.0).half()
            sc_out[r0:r1, :, t] = sh
            e = e - sh.float()[..., None, None] * roots[best]
            idx_out[r0:r1, :, t] = best.reshape(r1 - r0, K // 8).to(torch.uint8)
    return idx_out, sc_out


def e8_decode(idx: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """w8 = s1 r[i1] + s2 r[i2]."""
    M = idx.shape[0]
    roots = e8_roots(idx.device)
    G = scales.shape[1]
    i = idx.long().view(M, G, 16, 2)
    s = scales.float()
    a = s[:, :, None, 0, None] * roots[i[..., 0]]
    b = s[:, :, None, 1, None] * roots[i[..., 1]]
    return (a + b).reshape(M, -1)


# ---------------------------------------------------------------- E8 lattice (fp16 reconstructions)
def _d8_nearest(x: torch.Tensor) -> torch.Tensor:
    """Nearest point of D8 = {z in Z^8 : sum z even} to each 8-vector: round
    every coordinate; when the rounded sum is odd, move the coordinate with
    the largest rounding error one step toward x (the first such coordinate on
    a tie; an error of exactly 0 steps up).  quantize_d8, e8_lattice.py:53-84."""
    f = torch.round(x)
    err = x - f
    odd = torch.remainder(torch.sum(f, dim=-1, keepdim=True).long(), 2) != 0
    worst = torch.argmax(torch.abs(err), dim=-1, keepdim=True)
    step = torch.where(err >= 0, torch.ones_like(err), -torch.ones_like(err))
    fix = torch.zeros_like(x, dtype=torch.bool).scatter_(-1, worst, True) & odd
    return torch.where(fix, f + step, f)


def e8_nearest(x: torch.Tensor) -> torch.Tensor:
    """Nearest point of the E8 lattice, E8 = D8 u (D8 + 1/2), to each
    8-vector of x [..., 8] (Conway & Sloane, "Fast quantizing and decoding
    algorithms for lattice quantizers and codes", IEEE Trans. IT 28 (1982)):
    the nearer of the two cosets' nearest points, D8's on a tie (quantize_e8,
    e8_lattice.py:87-105)."""
    a = _d8_nearest(x)
    b = _d8_nearest(x - 0.5) + 0.5
    da = torch.sum((x - a) ** 2, dim=-1, keepdim=True)
    db = torch.sum((x - b) ** 2, dim=-1, keepdim=True)
    return torch.where(da <= db, a, b)


def _e8_best_scale(blocks: torch.Tensor, steps: int, eps: float = 1e-12) -> float:
    """Grid search of s in [0.2 rms, 2.5 rms] (`steps` points) minimising
    mean |x - s Q_E8(x / s)|^2, the first minimum kept (optimize_scale,
    e8_lattice.py:118-145)."""
    rms = float(torch.sqrt(torch.mean(blocks ** 2)).item())
    if rms <= eps:
        return 1.0
    best, best_loss = rms, float("inf")
    for s in torch.linspace(0.2 * rms, 2.5 * rms, steps=steps, device=blocks.device).tolist():
        if s <= eps:
            continue
        loss = float(torch.mean((blocks - e8_nearest(blocks / s) * s) ** 2).item())
        if loss < best_loss:
            best, best_loss = s, loss
    return best


def e8_lattice_quantize(x: torch.Tensor, search_steps: int = 16, scale: float = None,
                        eps: float = 1e-12) -> Tuple[torch.Tensor, Dict]:
    """x_hat = s Q_E8(x / s) over consecutive 8-element blocks of x (flattened,
    zero-padded to a multiple of 8), s from _e8_best_scale unless given.
    Returns x_hat (fp32, x's shape) and the reference's metadata keys
    (E8LatticeQuantizer.quantize, e8_lattice.py:147-190)."""
    flat = x.reshape(-1)
    pad = (-flat.numel()) % 8
    if pad:
        flat = torch.cat([flat, torch.zeros(pad, device=x.device, dtype=x.dtype)])
    blocks = flat.view(-1, 8).float()
    if scale is None:
        scale = _e8_best_scale(blocks, search_steps, eps)
    xh = (e8_nearest(blocks / max(scale, eps)) * scale).view(-1)
    if pad:
        xh = xh[:-pad]
    xh = xh.reshape(x.shape)
    mse = float(torch.mean((x - xh) ** 2).item())
    var = float(torch.var(x).item())
    return xh, {"optimal_scale": scale, "mse_distortion": mse,
                "snr_db": 10.0 * math.log10(max(var, 1e-15) / max(mse, 1e-15)), "dimension": 8,
                "sphere_packing_density_e8": math.pi ** 4 / 384.0, "padding_added": pad}


def e8_rvq_quantize(x: torch.Tensor, num_stages: int = 2, search_steps: int = 12) -> Tuple[torch.Tensor, Dict]:
    """Residual E8 lattice VQ: stage t quantizes x - (sum of earlier stages)
    with its own searched scale; x_hat is the sum of the stages
    (E8ResidualVectorQuantizer.quantize, e8_lattice.py:193-232)."""
    stages = max(1, num_stages)
    residual = x.clone()
    rec = torch.zeros_like(x)
    scales, mses = [], []
    for _ in range(stages):
        q, m = e8_lattice_quantize(residual, search_steps)
        rec += q
        residual = x - rec
        scales.append(m["optimal_scale"])
        mses.append(float(torch.mean(residual ** 2).item()))
    total = float(torch.mean((x - rec) ** 2).item())
    var = float(torch.var(x).item())
    return rec.reshape(x.shape), {"num_stages": stages, "stage_scales": scales, "stage_mses": mses,
                                  "total_mse": total,
                                  "snr_db": 10.0 * math.log10(max(var, 1e-15) / max(total, 1e-15))}


# ---------------------------------------------------------------- recursive polar
def polar_alloc(block_size: int, target_bpw: float) -> List[int]:
    """compute_adaptive_bit_allocation (polar_quant.py:352-379)."""
    d = block_size
    total = int(round(d * target_bpw))
    if d == 2:
        r_b = max(2, total // 2)
        return [r_b, max(1, total - r_b)]
    r_bits = max(2, min(4, int(round(target_bpw + 1))))
    remaining = max(d - 1, total - r_bits)
    alloc = [r_bits]
    na = d - 1
    base, rem = remaining // na, remaining % na
    for i in range(na):
        alloc.append(max(1, base + (1 if i < rem else 0)))
    while sum(alloc) < total:
        alloc[1] += 1
    while sum(alloc) > total and alloc[-1] > 1:
        alloc[-1] -= 1
    return alloc


def _forward_recursive(blocks: torch.Tensor):
    """forward_recursive (polar_quant.py:219-250)."""
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


def pack_bits_msb(words: torch.Tensor, total_bits: int) -> torch.Tensor:
    """Writes each int64 word's low `total_bits` bits as one MSB-first stream
    (polar_quant.py:463-473)."""
    n = words.numel()
    shifts = torch.arange(total_bits - 1, -1, -1, device=words.device)
    bits = ((words.view(-1, 1) >> shifts) & 1).to(torch.uint8).flatten()
    pad = (-bits.numel()) % 8
    if pad:
        bits = torch.cat([bits, bits.new_zeros(pad)])
    weights = torch.tensor([128, 64, 32, 16, 8, 4, 2, 1], dtype=torch.int32, device=words.device)
    out = (bits.view(-1, 8).to(torch.int32) * weights).sum(-1).to(torch.uint8)
    assert out.numel() == (n * total_bits + 7) // 8
    return out


def fit_polar_codebooks(sample: torch.Tensor, block_size: int, angle_bits: int = 4,
                        iters: int = 15) -> List[torch.Tensor]:
    """Per-level angle codebooks of 2^angle_bits entries by 1-D Lloyd-Max
    iterations (fit_codebooks, polar_quant.py:274-300): the sample's blocks
    are taken to polar form; each level's centroids start evenly spaced over
    the level's range ([-pi, pi] at level 0, [0, pi/2] above, 1e-3 in from
    each end), then `iters` times every angle is assigned to its nearest
    centroid (the lowest index on a tie) and each centroid that received
    angles moves to their mean; the result is sorted."""
    L = 1 << angle_bits
    _, levels = _forward_recursive(sample.detach().cpu().reshape(-1, block_size))
    books = []
    for lvl, angles in enumerate(levels):
        a = angles.flatten()
        c = (torch.linspace(-math.pi + 1e-3, math.pi - 1e-3, L) if lvl == 0
             else torch.linspace(1e-3, 0.5 * math.pi - 1e-3, L))
        for _ in range(iters):
            near = torch.argmin(torch.abs(a.unsqueeze(1) - c.unsqueeze(0)), dim=1)
            for k in range(L):
                members = a[near == k]
                if members.numel() > 0:
                    c[k] = members.mean()
        books.append(torch.sort(c)[0])
    return books


def polar_angle_table(block_size: int, alloc: List[int], codebooks, device="cpu") -> torch.Tensor:
    """The device decoders' learned angle table, fp32 [d-1][64]: entry 64 j + c
    is the angle of code c in angle column j (level 0 columns first), i.e.
    codebook[level(j)][min(c, len - 1)] (decode_packed, polar_quant.py:552-554);
    columns of levels without a codebook keep the uniform grid (:555-558)."""
    d = block_size
    tab = torch.zeros(d - 1, 64, dtype=torch.float32)
    col, width, lvl = 0, d // 2, 0
    while width >= 1:
        for j in range(width):
            levels = 1 << alloc[1 + col + j]
            c = torch.arange(levels)
            if lvl < len(codebooks):
                cb = torch.as_tensor(codebooks[lvl], dtype=torch.float32).flatten()
                tab[col + j, :levels] = cb[torch.clamp(c, 0, cb.numel() - 1)]
            elif lvl == 0:
                tab[col + j, :levels] = ((c.float() + 0.5) / float(levels)) * (2.0 * math.pi) - math.pi
            else:
                tab[col + j, :levels] = ((c.float() + 0.5) / float(levels)) * (0.5 * math.pi)
        col += width
        width //= 2
        lvl += 1
    return tab.flatten().to(device)


def polar_encode(w: torch.Tensor, block_size: int = 8, target_bpw: float = 1.75,
                 blocks_per_chunk: int = 1 << 22, codebooks=None) -> Tuple[torch.Tensor, Dict]:
    """RecursivePolarQuant.encode_packed (polar_quant.py:381-487); returns
    (payload uint8, meta) with the reference's meta keys.  The global max
    radius fixes r_scale, then blocks are coded chunk by chunk.  Angles are
    coded on the uniform grid, or, at the levels `codebooks` covers, as the
    index of the nearest codebook entry (lowest on a tie).  As in the
    reference, a codebook index wider than its column's bit field is OR-ed
    in unmasked (polar_quant.py:440-444), so its high bits land in the
    fields above; meta then also carries the codebooks (learned_codebooks),
    which the reference keeps on the quantizer object."""
    d = block_size
    flat = w.float().flatten()
    pad = (-flat.numel()) % d
    if pad:
        flat = torch.cat([flat, flat.new_zeros(pad)])
    nblk = flat.numel() // d
    blocks = flat.view(nblk, d)
    alloc = polar_alloc(d, target_bpw)
    tb = sum(alloc)
    if tb % 8 == 0 and tb // 8 not in (1, 2, 4, 8):
        raise ValueError(f"{tb}-bit polar blocks take the reference's truncating word path "
                         "(polar_quant.py:459-460), which does not round-trip")
    rmax = None
    for b0 in range(0, nblk, blocks_per_chunk):
        top, _ = _forward_recursive(blocks[b0:b0 + blocks_per_chunk])
        m = torch.max(top)
        rmax = m if rmax is None else torch.maximum(rmax, m)
    r_scale = (float(rmax.item()) + 1e-12) / float((1 << alloc[0]) - 1)
    out = []
    # chunks of whole bytes: a multiple of 8 blocks keeps every chunk byte aligned
    step = max(8, (blocks_per_chunk // 8) * 8)
    for b0 in range(0, nblk, step):
        top, angle_levels = _forward_recursive(blocks[b0:b0 + step])
        n = top.shape[0]
        r_code = torch.clamp(torch.round(top / r_scale), 0, (1 << alloc[0]) - 1).long()
        codes = [r_code]
        col = 1
        for lvl, angles in enumerate(angle_levels):
            fa = angles.view(n, -1)
            for j in range(fa.shape[1]):
                th = fa[:, j]
                levels = 1 << alloc[col]
                if codebooks and lvl < len(codebooks):
                    cb = torch.as_tensor(codebooks[lvl], dtype=torch.float32, device=th.device)
                    codes.append(torch.argmin(torch.abs(th.unsqueeze(1) - cb.unsqueeze(0)), dim=1).long())
                    col += 1
                    continue
                nt = (th + math.pi) / (2.0 * math.pi) if lvl == 0 else th / (0.5 * math.pi)
                nt = torch.clamp(nt, 0.0, 1.0 - 1e-7)
                codes.append(torch.clamp(torch.floor(nt * levels), 0, levels - 1).long())
                col += 1
        acc = torch.zeros(n, dtype=torch.int64, device=w.device)
        shift = 0
        for i in range(len(alloc) - 1, -1, -1):
            acc |= codes[i] << shift
            shift += alloc[i]
        out.append(pack_bits_msb(acc, tb))
    payload = torch.cat(out)
    meta = {
        "block_size": d, "orig_shape": list(w.shape), "pad_len": pad, "num_blocks": nblk,
        "alloc": alloc, "r_scale": r_scale,
        "exact_bpw": payload.numel() * 8.0 / float(w.numel()), "has_learned_codebooks": bool(codebooks),
    }
    if codebooks:
        meta["learned_codebooks"] = [[float(v) for v in torch.as_tensor(cb).flatten().tolist()] for cb in codebooks]
    return payload, meta
