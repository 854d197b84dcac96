"""Block randomized Walsh-Hadamard transform: plan, signs and device transform.

Mirrors ``BlockHadamardTransform`` (polarflash_quant/transforms/hadamard.py:78-169):
the same block-size rule, the same torch generator draws for the Rademacher
signs (full-block signs, then one draw per remainder block), and forward /
inverse applied on the GPU by ``pf_rwht``.
"""
import ctypes
import functools
from typing import List, Tuple

import torch

from . import _lib


def effective_block(block_size: int, in_features: int) -> int:
    """_init_dims (hadamard.py:93-99): largest power of two <= min(request, K), >= 2."""
    bs = 1
    lim = min(block_size, in_features)
    while bs * 2 <= lim:
        bs *= 2
    return max(bs, 2)


def plan(in_features: int, block: int) -> Tuple[int, List[Tuple[int, int]]]:
    """(number of full blocks, remainder cascade [(offset, size)]), hadamard.py:100-116."""
    nfull = in_features // block
    off = nfull * block
    rem = in_features - off
    casc = []
    while rem > 1:
        p2 = 1
        while p2 * 2 <= rem:
            p2 *= 2
        casc.append((off, p2))
        off += p2
        rem -= p2
    return nfull, casc


@functools.lru_cache(maxsize=256)
def column_signs_cpu(in_features: int, block_size: int, seed: int = 42) -> torch.Tensor:
    """Per-column +-1 signs (int8, CPU) of BlockHadamardTransform(K, block_size, seed):
    torch.Generator().manual_seed(seed), randint(0, 2, (block,)) * 2 - 1 for the
    full blocks (hadamard.py:104-105), then one randint draw per cascade block
    (hadamard.py:110-116).  A trailing single column keeps sign +1 (it is not
    rotated)."""
    block = effective_block(block_size, in_features)
    gen = torch.Generator().manual_seed(seed)
    full = torch.randint(0, 2, (block,), generator=gen).to(torch.int8) * 2 - 1
    nfull, casc = plan(in_features, block)
    parts = [full.repeat(nfull)]
    for _, p2 in casc:
        parts.append(torch.randint(0, 2, (p2,), generator=gen).to(torch.int8) * 2 - 1)
    out = torch.cat(parts) if parts else torch.empty(0, dtype=torch.int8)
    if out.numel() < in_features:
        out = torch.cat([out, torch.ones(in_features - out.numel(), dtype=torch.int8)])
    return out.contiguous()


_device_cache = {}


def column_signs(in_features: int, block_size: int, device, seed: int = 42) -> torch.Tensor:
    key = (in_features, block_size, seed, str(torch.device(device)))
    t = _device_cache.get(key)
    if t is None:
        t = column_signs_cpu(in_features, block_size, seed).to(device)
        _device_cache[key] = t
    return t


class BlockHadamardTransform:
    """Drop-in for the reference class on CUDA tensors (fp32, last dim = K)."""

    def __init__(self, in_features: int, block_size: int = 256, seed: int = 42, device="cuda"):
        self.in_features = in_features
        self.block_size_req = block_size
        self.seed = seed
        self.device = torch.device(device)
        self.block_size = effective_block(block_size, in_features)
        self.num_full_blocks, cascade = plan(in_features, self.block_size)
        self.remainder = in_features % self.block_size
        self.rem_blocks = cascade

    def _apply(self, x: torch.Tensor, inverse: bool) -> torch.Tensor:
        if x.shape[-1] != self.in_features:
            raise ValueError(f"last dimension {x.shape[-1]} != in_features {self.in_features}")
        if x.device.type != "cuda":
            raise ValueError("BlockHadamardTransform (polarflash_b200) runs on CUDA tensors only")
        xf = x.reshape(-1, self.in_features).float().contiguous()
        out = torch.empty_like(xf)
        signs = column_signs(self.in_features, self.block_size_req, xf.device, self.seed)
        st = _lib.load().pf_rwht(
            ctypes.c_void_p(xf.data_ptr()), ctypes.c_void_p(out.data_ptr()), xf.shape[0],
            self.in_features, self.block_size, ctypes.c_void_p(signs.data_ptr()), 1 if inverse else 0,
            ctypes.c_void_p(torch.cuda.current_stream(xf.device).cuda_stream))
        _lib.check(st, "pf_rwht")
        return out.reshape(x.shape)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        return self._apply(x, inverse=False)

    def inverse(self, z: torch.Tensor) -> torch.Tensor:
        return self._apply(z, inverse=True)
