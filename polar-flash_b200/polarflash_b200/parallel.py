"""Column-parallel packed linear over torch.distributed (NCCL on B200s).

Rank r of P owns output rows [r*M/P, (r+1)*M/P) of W: packed rows, per-row
group scales, E8 and polar row payloads all slice without re-encoding, and the
activations x are replicated (the RWHT runs along K, unaffected by the row
split).  Each rank runs the fused GEMV on its shard and one all-gather
assembles y.  The shard output is written M-major per rank so the rank-major
concatenation is the full [N, M] after one transpose of a tiny buffer.
"""
from typing import List, Optional

import ctypes

import torch
import torch.distributed as dist

from . import _lib
from .qweight import QWeight, _desc_array, _X_DTYPES, group_workspace_bytes, qlinear, workspace


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


class GroupGather:
    """Assembles the full outputs of one group of row-sharded linears that
    read one input (q|k|v, gate|up, or a single linear) with ONE all-gather:
    the group's shard outputs [S, M_i / P] are packed side by side, gathered
    rank-major into [P, S, sum M_i / P] and each output taken back out as the
    full [S, M_i] (rank r's rows at [r M_i / P, (r + 1) M_i / P)).  Used by
    PFlashDecoder(tp=...) for a column-parallel decode step; capturable in a
    CUDA graph."""

    def __init__(self, group: Optional[dist.ProcessGroup] = None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)

    def gather(self, ys: List[torch.Tensor]) -> List[torch.Tensor]:
        if self.world == 1:
            return ys
        S = ys[0].shape[0]
        packed = torch.cat([y.reshape(S, -1) for y in ys], dim=1).contiguous()
        out = torch.empty(self.world, S, packed.shape[1], dtype=packed.dtype, device=packed.device)
        dist.all_gather_into_tensor(out.view(-1), packed.view(-1), group=self.group)
        full, off = [], 0
        for y in ys:
            m = y.shape[-1]
            full.append(out[:, :, off:off + m].permute(1, 0, 2).reshape(S, self.world * m))
            off += m
        return full


def gather_rows(y_local: torch.Tensor, world: int, group=None) -> torch.Tensor:
    """All-gather of [N, M/P] shards into [N, M] (host-side helper for tests)."""
    N, m = y_local.shape
    out: List[torch.Tensor] = [torch.empty_like(y_local) for _ in range(world)]
    dist.all_gather(out, y_local.contiguous(), group=group)
    return torch.cat(out, dim=1)


class PeerBuffer:
    """A device buffer of the same size on every rank of `group`, each rank's
    mapped into every other rank's process (CUDA IPC; the handles travel
    through torch.distributed), for column-parallel linears that store their
    rows straight into every rank's copy of y (pf_qlinear_group_gather).

    The first 256 bytes are the header of the fused calls (an epoch and one
    flag per rank); `view(offset, shape)` gives fp32 views of the local buffer
    at byte offsets >= 256.  Every rank must create its PeerBuffers in the
    same order and make the same sequence of gathering calls."""

    HEADER = 256

    def __init__(self, nbytes: int, group: Optional[dist.ProcessGroup] = None, device=None):
        L = _lib.load()
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        if self.world > 8:
            raise ValueError("at most 8 ranks")
        dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        self.nbytes = (nbytes + 255) // 256 * 256
        # its own allocation (the IPC handle covers the whole allocation)
        self.local = torch.zeros(self.nbytes, dtype=torch.uint8, device=dev)
        handle = (ctypes.c_ubyte * 64)()
        off = ctypes.c_size_t(0)
        _lib.check(L.pf_peer_export(ctypes.c_void_p(self.local.data_ptr()), handle, ctypes.byref(off)),
                   "pf_peer_export")
        mine = (bytes(handle), int(off.value))
        allh = [None] * self.world
        dist.all_gather_object(allh, mine, group=group)
        self._mappings = []
        self.peers = _lib.PFPeers()
        self.peers.world, self.peers.rank, self.peers.bytes = self.world, self.rank, self.nbytes
        for r, (h, o) in enumerate(allh):
            if r == self.rank:
                self.peers.bases[r] = self.local.data_ptr()
                continue
            ptr, mp = ctypes.c_void_p(0), ctypes.c_void_p(0)
            hb = (ctypes.c_ubyte * 64).from_buffer_copy(h)
            _lib.check(L.pf_peer_open(hb, o, ctypes.byref(ptr), ctypes.byref(mp)), "pf_peer_open")
            self.peers.bases[r] = ptr.value
            self._mappings.append(mp.value)
        torch.cuda.synchronize(dev)
        dist.barrier(group=group)

    def view(self, offset: int, shape) -> torch.Tensor:
        n = 1
        for d in shape:
            n *= d
        if offset < self.HEADER or offset % 16 or offset + 4 * n > self.nbytes:
            raise ValueError("view outside the buffer's output area")
        return self.local[offset:offset + 4 * n].view(torch.float32).view(*shape)

    def close(self):
        """Unmaps the peers' buffers (after all work that uses them)."""
        L = _lib.load()
        for mp in self._mappings:
            _lib.check(L.pf_peer_close(ctypes.c_void_p(mp)), "pf_peer_close")
        self._mappings = []


def qlinear_group_gather(shards, xs, peer: PeerBuffer, y_offsets, biases=None, ws: Optional[torch.Tensor] = None,
                         stream=None):
    """Row shards `shards` (this rank's rows of each linear) times xs, each
    linear's whole y [N, world * M_i] written into every rank's peer buffer at
    y_offsets[i] (pf_qlinear_group_gather).  Call peers_wait before reading
    the outputs on this rank."""
    L = _lib.load()
    n = len(shards)
    N = xs[0].shape[0]
    dt = xs[0].dtype
    dev = xs[0].device
    s = stream if stream is not None else torch.cuda.current_stream(dev)
    need = group_workspace_bytes(shards, N)
    ws = ws if ws is not None else workspace(dev, need, s)
    VP = ctypes.c_void_p * n
    xa = VP(*[x.data_ptr() for x in xs])
    ba = VP(*[b.data_ptr() if b is not None else None for b in (biases or [None] * n)])
    offs = (ctypes.c_size_t * n)(*y_offsets)
    mfull = (ctypes.c_int * n)(*[peer.world * q.M for q in shards])
    _lib.check(L.pf_qlinear_group_gather(n, _desc_array(shards), xa, _X_DTYPES[dt], N, ba, offs, mfull,
                                         ctypes.byref(peer.peers), ctypes.c_void_p(ws.data_ptr()), ws.numel(),
                                         ctypes.c_void_p(s.cuda_stream)), "pf_qlinear_group_gather")


def peers_wait(peer: PeerBuffer, ws: torch.Tensor, stream=None):
    """Makes `stream` wait until every rank's rows of its latest gathering
    call are in this rank's buffer (bounded; a wait that gives up is recorded
    in the workspace status word)."""
    L = _lib.load()
    s = stream if stream is not None else torch.cuda.current_stream(ws.device)
    _lib.check(L.pf_peers_wait(ctypes.byref(peer.peers), ctypes.c_void_p(ws.data_ptr()),
                               ctypes.c_void_p(s.cuda_stream)), "pf_peers_wait")


def allgather_rows(peer: PeerBuffer, src: torch.Tensor, dst_offset: int, ws: torch.Tensor, stream=None):
    """pf_allgather_rows: this rank's contiguous `src` lands at byte
    dst_offset + rank * src.nbytes of every rank's peer buffer (rank-major);
    when the launch completes on this rank, every rank's part is in its
    buffer.  Returns the local gathered view [world, *src.shape]."""
    L = _lib.load()
    s = stream if stream is not None else torch.cuda.current_stream(src.device)
    nb = src.numel() * src.element_size()
    _lib.check(L.pf_allgather_rows(ctypes.byref(peer.peers), ctypes.c_void_p(src.data_ptr()), nb, dst_offset,
                                   ctypes.c_void_p(ws.data_ptr()), ctypes.c_void_p(s.cuda_stream)),
               "pf_allgather_rows")
    return peer.local[dst_offset:dst_offset + peer.world * nb].view(src.dtype).view(peer.world, *src.shape)

