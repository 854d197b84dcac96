"""``torch.ops.polarflash.qlinear``: the fused forward as a torch custom op.

The op takes the packed weight's tensors plus its format fields, so it can be
called from any torch code (and traced) without the QWeight object; its
implementation is the same C-ABI call as ``qweight.qlinear``.
"""
from typing import List, Optional

import torch

from .qweight import QWeight, qlinear as _qlinear


@torch.library.custom_op("polarflash::qlinear", mutates_args=())
def qlinear_op(x: torch.Tensor, codes: torch.Tensor, scales: Optional[torch.Tensor], mins: Optional[torch.Tensor],
               had_signs: Optional[torch.Tensor], fmt: int, M: int, K: int, had_block: int, tensor_scale: float,
               params: List[int], bias: Optional[torch.Tensor]) -> torch.Tensor:
    qw = QWeight(fmt, M, K, codes, scales, mins, had_block, had_signs, tensor_scale, list(params))
    return _qlinear(qw, x, bias)


@qlinear_op.register_fake
def _(x, codes, scales, mins, had_signs, fmt, M, K, had_block, tensor_scale, params, bias):
    return x.new_empty((*x.shape[:-1], M), dtype=torch.float32)


def qlinear(qw: QWeight, x: torch.Tensor, bias: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Calls the registered op for a QWeight."""
    return torch.ops.polarflash.qlinear(x, qw.codes, qw.scales, qw.mins, qw.had_signs, qw.format, qw.M, qw.K,
                                        qw.had_block, float(qw.tensor_scale), list(qw.params), bias)
