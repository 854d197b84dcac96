"""RecursivePolarQuant mirror (polarflash_quant/polar/polar_quant.py:194-620).

Same constructor and method names as the reference class.  Encoding runs
where the weight lives (torch ops in the reference's order, so a CPU weight
gives the reference's bytes); decode_packed decodes on the GPU through the
library's polar decoder, with the learned angle codebooks when the payload
was encoded with them.  The codebooks travel in the metadata
(``learned_codebooks``) as well as on the object, so a payload decodes
without the quantizer that made it.
"""
import math
from typing import Any, Dict, List, Tuple

import torch

from . import _lib, encoders
from .qweight import QWeight, dequantize as _dequant_qw


class RecursivePolarQuant:
    """Mirror of the reference RecursivePolarQuant (polar_quant.py:194-620)."""

    def __init__(self, block_size: int = 4, norm_bits: int = 6, angle_bits: int = 4, epsilon: float = 1e-12):
        if (block_size & (block_size - 1)) != 0 or block_size < 2:
            raise ValueError(f"block_size must be a power of 2 >= 2, got {block_size}")
        self.block_size = block_size
        self.norm_bits = norm_bits
        self.angle_bits = angle_bits
        self.epsilon = epsilon
        self.norm_levels = 2 ** norm_bits
        self.angle_levels = 2 ** angle_bits
        self.learned_codebooks: List[torch.Tensor] = []

    def forward_recursive(self, x: torch.Tensor):
        """(top radius, per-level angles) of blocks x [..., d] (polar_quant.py:219-250)."""
        return encoders._forward_recursive(x.reshape(-1, self.block_size))

    def compute_adaptive_bit_allocation(self, target_bpw: float = 2.0) -> List[int]:
        return encoders.polar_alloc(self.block_size, target_bpw)

    def fit_codebooks(self, sample_weights: torch.Tensor, iters: int = 15) -> None:
        """Lloyd-Max angle codebooks per level (polar_quant.py:274-300)."""
        self.learned_codebooks = encoders.fit_polar_codebooks(sample_weights, self.block_size, self.angle_bits,
                                                              iters)

    def encode_packed(self, weights: torch.Tensor, target_bpw: float = 2.0) -> Tuple[bytes, Dict[str, Any]]:
        """Packed bit stream and metadata (polar_quant.py:381-487)."""
        packed, meta = encoders.polar_encode(weights, self.block_size, target_bpw,
                                             codebooks=self.learned_codebooks or None)
        return packed.cpu().numpy().tobytes(), meta

    def decode_packed(self, packed_bytes, meta: Dict[str, Any], device: str = "cuda") -> torch.Tensor:
        """Decoded weight (meta["orig_shape"], fp32) on a CUDA device
        (polar_quant.py:489-575)."""
        dev = torch.device(device)
        if dev.type != "cuda":
            raise ValueError("polarflash_b200 decodes on CUDA devices only")
        d, alloc = int(meta.get("block_size", self.block_size)), [int(a) for a in meta["alloc"]]
        nblk, tb = int(meta["num_blocks"]), sum(alloc)
        shape = list(meta["orig_shape"])
        M, K = (shape[0], math.prod(shape[1:])) if len(shape) > 1 else (1, shape[0])
        if M * K != nblk * d - int(meta.get("pad_len", 0)) or K % d or (K // d) * tb % 8:
            M, K = 1, nblk * d  # decode the stream as one row; the pad is cut below
        codebooks = None
        if meta.get("has_learned_codebooks"):
            codebooks = meta.get("learned_codebooks") or self.learned_codebooks or None
        angles = encoders.polar_angle_table(d, alloc, codebooks, dev) if codebooks else None
        raw = torch.frombuffer(bytearray(bytes(packed_bytes)), dtype=torch.uint8).to(dev)
        qw = QWeight(_lib.FMT_POLAR_RECURSIVE, M, K, raw, angles, None, 0, None, float(meta["r_scale"]),
                     [d] + alloc)
        flat = _dequant_qw(qw, inverse_rwht=False).reshape(-1)
        pad = int(meta.get("pad_len", 0))
        if pad:
            flat = flat[:-pad]
        return flat.reshape(shape)
