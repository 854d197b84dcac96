"""Column-parallel packed linear over torch.distributed (NCCL on B200s).

Rank r of P owns output rows [r*M/P, (r+1)*M/P) of W: packed rows, per-row
group scales, E8 and polar row payloads all slice without re-encoding, and the
activations x are replicated (the RWHT runs along K, unaffected by the row
split).  Each rank runs the fused GEMV on its shard and one all-gather
assembles y.  The shard output is written M-major per rank so the rank-major
concatenation is the full [N, M] after one transpose of a tiny buffer.
"""
from typing import List, Optional

import torch
import torch.distributed as dist

from .qweight import QWeight, qlinear


def shard_bounds(M: int, world: int, rank: int):
    if M % world:
        raise ValueError(f"out_features {M} is not divisible by the world size {world}")
    per = M // world
    return rank * per, (rank + 1) * per


class ColumnParallelQLinear:
    def __init__(self, full: QWeight, group: Optional[dist.ProcessGroup] = None,
                 bias: Optional[torch.Tensor] = None):
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        self.M, self.K = full.M, full.K
        r0, r1 = shard_bounds(full.M, self.world, self.rank)
        self.local = full.shard_rows(r0, r1) if self.world > 1 else full
        self.bias = bias[r0:r1].contiguous() if bias is not None else None
        self._ws = None

    def local_forward(self, x: torch.Tensor) -> torch.Tensor:
        """This rank's [N, M/P] slice of y."""
        return qlinear(self.local, x, self.bias, workspace=self._ws)

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        lead = x.shape[:-1]
        y_local = self.local_forward(x).reshape(-1, self.local.M)
        if self.world == 1:
            return y_local.reshape(*lead, self.M)
        N = y_local.shape[0]
        # [P, N, M/P] gathered rank-major, then [N, M]
        gathered = torch.empty(self.world, N, self.local.M, dtype=y_local.dtype, device=y_local.device)
        dist.all_gather_into_tensor(gathered, y_local.contiguous(), group=self.group)
        return gathered.permute(1, 0, 2).reshape(*lead, self.M)

    __call__ = forward


def gather_rows(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather of [N, M/P] shards into [N, M] (host-side helper for tests)."""
    N, m = y_local.shape
    out: List[torch.Tensor] = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(out, y_local.contiguous(), group=group)
    return torch.cat(out, dim=1)
