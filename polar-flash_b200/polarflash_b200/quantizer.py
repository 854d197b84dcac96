"""UnifiedQuantizer mirror: quantize weights into packed payloads and decode them.

Same constructor and method signatures as the reference
(polarflash_quant/unified_quantizer.py:83-324).  Encoding runs where the weight
lives (a CPU weight follows the reference's CPU arithmetic step for step, so
reference backends give byte-identical payloads; a CUDA weight is rotated by
pf_rwht and encoded with torch CUDA ops).  ``dequantize`` decodes on the GPU.

Backends: the reference's fp16, bf16, int8, int4, int3, int2, e8 (E8
lattice / residual E8 lattice VQ, stored as an fp16 reconstruction) and (2-D)
polar, plus the packed formats of this library: int4_g128, int3_g128,
int2_g128 (group-128 asymmetric), e8_rvq2_g128 (E8 root residual VQ indices)
and polar_recursive (RecursivePolarQuant block codes).
"""
import math
from typing import Any, Dict, List, Tuple

import numpy as np
import torch

from . import _lib, encoders
from .hadamard import BlockHadamardTransform, column_signs_cpu, effective_block, plan
from .qweight import (QWeight, dequantize as _dequant_qw, extension_payload_bytes, qweight_from_payload,
                      resolve_format)


def _fwht_cpu(x: torch.Tensor) -> torch.Tensor:
    """Normalised Walsh-Hadamard over the last dim (power of two) with the
    butterfly order of the reference (distance 1, 2, 4, ...; (u+v, u-v)),
    then / sqrt(d)."""
    d = x.shape[-1]
    out = x.reshape(-1, d).clone()
    h = 1
    while h < d:
        v = out.view(-1, d // (2 * h), 2, h)
        a = v[:, :, 0, :].clone()
        b = v[:, :, 1, :].clone()
        v[:, :, 0, :] = a + b
        v[:, :, 1, :] = a - b
        h *= 2
    return (out / math.sqrt(d)).reshape(x.shape)


def rwht_cpu(w: torch.Tensor, block_size: int, seed: int = 42, inverse: bool = False) -> torch.Tensor:
    """Block RWHT on a CPU tensor (forward z = H D x / sqrt(b), inverse
    x = D H z / sqrt(b), per block; hadamard.py:119-169)."""
    K = w.shape[-1]
    block = effective_block(block_size, K)
    signs = column_signs_cpu(K, block_size, seed).float()
    nfull, casc = plan(K, block)
    flat = w.reshape(-1, K).float()
    out = flat.clone()
    if nfull:
        span = nfull * block
        blk = flat[:, :span].reshape(-1, nfull, block)
        sg = signs[:span].reshape(nfull, block)
        if inverse:
            out[:, :span] = (_fwht_cpu(blk) * sg).reshape(-1, span)
        else:
            out[:, :span] = _fwht_cpu(blk * sg).reshape(-1, span)
    for off, p2 in casc:
        chunk = flat[:, off:off + p2]
        sg = signs[off:off + p2]
        out[:, off:off + p2] = _fwht_cpu(chunk) * sg if inverse else _fwht_cpu(chunk * sg)
    return out.reshape(w.shape)


def rotate(w: torch.Tensor, block_size: int, seed: int = 42, inverse: bool = False) -> torch.Tensor:
    if w.device.type == "cuda":
        bht = BlockHadamardTransform(w.shape[-1], block_size, seed, w.device)
        return bht.inverse(w) if inverse else bht.forward(w)
    return rwht_cpu(w, block_size, seed, inverse)


def _bytes(t: torch.Tensor) -> bytes:
    return t.detach().contiguous().cpu().numpy().tobytes()


class UnifiedQuantizer:
    """Mirror of the reference UnifiedQuantizer (unified_quantizer.py:83-324)."""

    SUPPORTED_BACKENDS = ["fp16", "bf16", "int8", "int4", "int3", "int2", "e8", "polar",
                          "int4_g128", "int3_g128", "int2_g128", "e8_rvq2_g128", "polar_recursive"]

    def __init__(self, backend: str = "polar", hadamard_block_size: int = 512, apply_hadamard: bool = True,
                 polar_r_bits: int = 4, polar_theta_bits: int = 4, e8_stages: int = 1,
                 polar_target_bpw: float = 1.75, polar_block_size: int = 8):
        backend = backend.lower()
        if backend not in self.SUPPORTED_BACKENDS:
            raise ValueError(f"Unsupported backend '{backend}'. Choose from {self.SUPPORTED_BACKENDS}")
        self.backend = backend
        self.hadamard_block_size = hadamard_block_size
        self.apply_hadamard = apply_hadamard
        self.polar_r_bits = polar_r_bits
        self.polar_theta_bits = polar_theta_bits
        self.e8_stages = e8_stages
        self.polar_target_bpw = polar_target_bpw
        self.polar_block_size = polar_block_size

    # ------------------------------------------------------------------ quantize
    def quantize_to_qweight(self, weight: torch.Tensor) -> Tuple[QWeight, Dict[str, Any]]:
        """Encodes a 2-D weight straight into a device QWeight (packed formats)."""
        payload, meta, _ = self.quantize(weight, name="w", return_w_hat=False)
        M, K = weight.shape
        dev = weight.device if weight.device.type == "cuda" else torch.device("cuda")
        return qweight_from_payload(meta["dtype"], meta, payload, M, K, dev), meta

    def quantize(self, weight: torch.Tensor, name: str = "tensor", return_w_hat: bool = True):
        orig_shape = list(weight.shape)
        w = weight.detach().float()
        n = w.numel()
        rotated = False
        if self.apply_hadamard and w.ndim == 2:
            w = rotate(w, self.hadamard_block_size)
            rotated = True
        be = self.backend
        meta: Dict[str, Any]
        w_rec = None  # the e8 backend's fp32 reconstruction (the reference's w_hat before the cast)
        if be == "e8":
            # unified_quantizer.py:180-192: one lattice stage (8-point scale grid) or
            # e8_stages residual stages (12-point grids); the payload is fp16
            wc = w.cpu()
            if self.e8_stages > 1:
                w_rec, em = encoders.e8_rvq_quantize(wc, self.e8_stages)
                meta = {"dtype": "e8_rvq", "stages": self.e8_stages, "bpw": 8.0 / 8.0 + 1.0, **em}
            else:
                w_rec, em = encoders.e8_lattice_quantize(wc, search_steps=8)
                meta = {"dtype": "e8_lattice", "bpw": 2.0, **em}
            payload = _bytes(w_rec.half())
        elif be in ("fp16", "bf16", "int8", "int4", "int3", "int2", "polar"):
            wc = w.cpu()
            if be == "fp16":
                payload = _bytes(wc.half())
                meta = {"dtype": "fp16", "bpw": 16.0}
            elif be == "bf16":
                payload = _bytes(wc.bfloat16().view(torch.int16))
                meta = {"dtype": "bf16", "bpw": 16.0}
            elif be == "int8":
                mx = torch.max(torch.abs(wc)).item()
                scale = mx / 127.0 if mx > 1e-12 else 1.0
                payload = _bytes(torch.clamp(torch.round(wc / scale), -128, 127).to(torch.int8))
                meta = {"dtype": "int8", "scale": float(scale), "bpw": 8.0}
            elif be in ("int4", "int3", "int2"):
                packed, scale = encoders.quant_int_per_tensor(wc, be)
                payload = _bytes(packed)
                meta = {"dtype": be, "scale": scale, "bpw": float(be[-1]), "num_elements": n}
            else:  # 2-D polar
                payload, meta = self._polar2d(wc)
        elif be in ("int4_g128", "int3_g128", "int2_g128"):
            bits = int(be[3])
            q, s, m = encoders.quant_g128_asym(w, bits)
            words = encoders.pack_g128(q, bits)
            qw = QWeight({4: _lib.FMT_INT4_G128, 3: _lib.FMT_INT3_G128, 2: _lib.FMT_INT2_G128}[bits],
                         w.shape[0], w.shape[1], words.view(torch.uint8).flatten(), s, m)
            payload = extension_payload_bytes(qw)
            meta = {"dtype": be, "bpw": bits + 32.0 / 128, "group_size": 128}
        elif be == "e8_rvq2_g128":
            idx, sc = encoders.e8_encode(w)
            qw = QWeight(_lib.FMT_E8_RVQ2_G128, w.shape[0], w.shape[1], idx.flatten(), sc, None)
            payload = extension_payload_bytes(qw)
            meta = {"dtype": be, "bpw": 2.0 + 32.0 / 128, "stages": 2, "group_size": 128}
        else:  # polar_recursive
            packed, pm = encoders.polar_encode(w, self.polar_block_size, self.polar_target_bpw)
            payload = _bytes(packed)
            meta = dict(pm)
            meta["dtype"] = "polar_recursive"
        if rotated:
            meta["hadamard_rotation"] = True
            meta["hadamard_block_size"] = self.hadamard_block_size
        meta.update({"name": name, "shape": orig_shape, "num_elements": n, "payload_bytes": len(payload),
                     "effective_bpw": round(len(payload) * 8.0 / max(n, 1), 3)})
        w_hat = None
        if return_w_hat:
            if w_rec is not None:  # the reference reports the fp32 reconstruction, not the fp16 payload
                w_hat = (rotate(w_rec, self.hadamard_block_size, inverse=True) if rotated else w_rec).view(*orig_shape)
            else:
                w_hat = UnifiedQuantizer.dequantize(payload, orig_shape, meta["dtype"], meta).cpu()
            ref = weight.detach().float().cpu()
            mse = float(torch.mean((ref - w_hat) ** 2).item())
            var = float(torch.var(ref).item()) if ref.numel() > 1 else 0.0
            meta["mse"] = mse
            meta["snr_db"] = round(10.0 * np.log10(max(var, 1e-12) / max(mse, 1e-15)), 2)
        return payload, meta, w_hat

    def _polar2d(self, wc: torch.Tensor):
        """PolarQuant2D.quantize with packed bytes (polar_quant.py:76-191) for the
        'polar' backend (unified_quantizer.py:194-212)."""
        rb, tb = self.polar_r_bits, self.polar_theta_bits
        flat = wc.reshape(-1)
        padded = flat.numel() % 2
        if padded:
            flat = torch.cat([flat, torch.zeros(1)])
        x1, x2 = flat.view(-1, 2)[:, 0], flat.view(-1, 2)[:, 1]
        eps = 1e-12
        ss = x1 ** 2 + x2 ** 2
        zero = ss <= eps ** 2
        r = torch.sqrt(torch.clamp(ss, min=0.0))
        r[zero] = 0.0
        th = torch.atan2(x2, x1)
        th[zero] = 0.0
        r_levels, t_levels = 2 ** rb, 2 ** tb
        r_scale = max(float(torch.max(r).item()), eps) / float(r_levels - 1)
        rq = torch.clamp(torch.round(r / r_scale), 0, r_levels - 1).long()
        tn = torch.clamp((th + math.pi) / (2.0 * math.pi), 0.0, 1.0 - 1e-7)
        tq = torch.clamp(torch.floor(tn * t_levels), 0, t_levels - 1).long()
        words = ((rq & (r_levels - 1)) << tb) | (tq & (t_levels - 1))
        payload = _bytes(encoders.pack_bits_msb(words, rb + tb))
        meta = {"dtype": "polar", "r_bits": rb, "theta_bits": tb, "r_scale": r_scale,
                "num_elements": wc.numel(), "padded": padded, "bpw": (rb + tb) / 2.0}
        return payload, meta

    # ------------------------------------------------------------------ dequantize
    @staticmethod
    def dequantize(payload_bytes, shape: List[int], dtype: str, quant_meta: Dict[str, Any],
                   device="cuda") -> torch.Tensor:
        """Decoded fp32 weight on `device` (a CUDA device), inverse RWHT
        included when quant_meta says the weight was rotated."""
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("polarflash_b200 decodes on CUDA devices only")
        M, K = int(shape[0]), int(np.prod(shape[1:])) if len(shape) > 1 else 1
        fmt = resolve_format(dtype, quant_meta)
        if fmt is not None and len(shape) == 2:
            qw = qweight_from_payload(dtype, quant_meta, payload_bytes, M, K, dev)
            return _dequant_qw(qw, inverse_rwht=True).view(*shape)
        return dense_weight(payload_bytes, shape, dtype, quant_meta, dev)


def dense_weight(payload_bytes, shape, dtype: str, quant_meta: Dict[str, Any], device) -> torch.Tensor:
    """Dense payloads (fp16 / bf16 / int8 / fp16 E8 reconstructions / legacy
    'polar4'): cast on the device, then the inverse RWHT on the device."""
    raw = torch.frombuffer(bytearray(bytes(payload_bytes)), dtype=torch.uint8).to(device)
    d = dtype.lower()
    if d == "bf16":
        t = raw.view(torch.bfloat16).float()
    elif d == "int8":
        t = raw.view(torch.int8).float() * float(quant_meta.get("scale", 1.0))
    elif d == "int4" and "scale" not in quant_meta:
        t = raw.view(torch.int8).float()  # unpacked int8 stored as int4 (cpu/engine.py:70-73)
    else:
        t = raw.view(torch.float16).float()
    t = t.view(*shape)
    if quant_meta.get("hadamard_rotation", False) and t.ndim == 2:
        t = rotate(t.contiguous(), int(quant_meta.get("hadamard_block_size", 512)), inverse=True)
    return t
