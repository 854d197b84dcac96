"""Device-resident packed weights and the fused forward through the C ABI.

A ``QWeight`` owns one device copy of the packed payload, its scales and the
RWHT column signs (uploaded once, as the layer's only device state: no decoded
weight is ever kept).  ``qlinear`` computes ``y = x W^T (+ bias)`` with
``pf_qlinear`` on the current stream.
"""
import ctypes
from dataclasses import dataclass, field
from typing import Dict, List, Optional

import numpy as np
import torch

from . import _lib, encoders
from .hadamard import column_signs, effective_block

# quant_meta "dtype" -> pf_format for the packed formats
DTYPE_TO_FMT = {
    "int4_g128": _lib.FMT_INT4_G128,
    "int3_g128": _lib.FMT_INT3_G128,
    "int2_g128": _lib.FMT_INT2_G128,
    "int4": _lib.FMT_INT4,
    "int3": _lib.FMT_INT3,
    "int2": _lib.FMT_INT2,
    "e8_rvq2_g128": _lib.FMT_E8_RVQ2_G128,
    "polar_recursive": _lib.FMT_POLAR_RECURSIVE,
}

_X_DTYPES = {torch.float32: _lib.DTYPE_F32, torch.float16: _lib.DTYPE_F16, torch.bfloat16: _lib.DTYPE_BF16}


def resolve_format(dtype: str, quant_meta: Dict) -> Optional[int]:
    """pf_format for a (dtype, quant_meta) pair of the reference catalog, or
    None for the dense payloads (fp16/bf16/int8/e8 reconstructions).  The
    reference writes recursive-polar payloads as "polar" from
    RecursivePolarQuant.export_to_pflash (polar_quant.py:577-593) and as
    "polar_recursive" from ingestion (model_integration.py:421-429); the 2-D
    polar backend also uses "polar" (unified_quantizer.py:194-212)."""
    d = dtype.lower()
    if d == "polar":
        return _lib.FMT_POLAR_RECURSIVE if "alloc" in quant_meta else _lib.FMT_POLAR2D
    return DTYPE_TO_FMT.get(d)


def _as_u8(payload, device) -> torch.Tensor:
    if isinstance(payload, torch.Tensor):
        t = payload.detach().contiguous().view(torch.uint8).flatten()
    else:
        t = torch.frombuffer(bytearray(bytes(payload)), dtype=torch.uint8)
    # 256-byte aligned device copy
    return t.to(device, non_blocking=False)


@dataclass
class QWeight:
    format: int
    M: int
    K: int
    codes: torch.Tensor
    scales: Optional[torch.Tensor] = None
    mins: Optional[torch.Tensor] = None
    had_block: int = 0
    had_signs: Optional[torch.Tensor] = None
    tensor_scale: float = 1.0
    params: List[int] = field(default_factory=list)
    _desc: Optional[_lib.PFQWeight] = None

    @property
    def device(self) -> torch.device:
        return self.codes.device

    def descriptor(self) -> _lib.PFQWeight:
        if self._desc is None:
            d = _lib.PFQWeight()
            d.format = self.format
            d.M = self.M
            d.K = self.K
            d.had_block = self.had_block
            d.codes = self.codes.data_ptr()
            d.scales = self.scales.data_ptr() if self.scales is not None else None
            d.mins = self.mins.data_ptr() if self.mins is not None else None
            d.had_signs = self.had_signs.data_ptr() if self.had_signs is not None else None
            d.tensor_scale = float(self.tensor_scale)
            for i, p in enumerate(self.params[:20]):
                d.params[i] = int(p)
            _lib.check(_lib.load().pf_qweight_check(ctypes.byref(d)), "pf_qweight_check")
            self._desc = d
        return self._desc

    def nbytes(self) -> int:
        """Device bytes of the packed representation (codes + scales + mins)."""
        n = self.codes.numel() * self.codes.element_size()
        for t in (self.scales, self.mins):
            if t is not None:
                n += t.numel() * t.element_size()
        return n

    def workspace_bytes(self, N: int) -> int:
        out = ctypes.c_size_t(0)
        _lib.check(_lib.load().pf_qlinear_workspace_size(ctypes.byref(self.descriptor()), N, ctypes.byref(out)),
                   "pf_qlinear_workspace_size")
        return int(out.value)

    def shard_rows(self, r0: int, r1: int) -> "QWeight":
        """Rows [r0, r1) as a QWeight sharing no storage (column-parallel shard)."""
        if self.format in (_lib.FMT_POLAR_RECURSIVE, _lib.FMT_POLAR2D):
            d = self.params[0] if self.format == _lib.FMT_POLAR_RECURSIVE else 2
            tb = sum(self.params[1:1 + d]) if self.format == _lib.FMT_POLAR_RECURSIVE else sum(self.params[:2])
            rb = (self.K // d) * tb // 8
            codes = self.codes.view(self.M, rb)[r0:r1].contiguous()
        else:
            codes = self.codes.view(self.M, -1)[r0:r1].contiguous()
        sc = self.scales  # recursive polar: the learned angle table, shared by every row
        if sc is not None and sc.dim() > 0 and sc.shape[0] == self.M and self.format != _lib.FMT_POLAR_RECURSIVE:
            sc = sc[r0:r1].contiguous()
        mins = self.mins[r0:r1].contiguous() if self.mins is not None else None
        return QWeight(self.format, r1 - r0, self.K, codes, sc, mins, self.had_block, self.had_signs,
                       self.tensor_scale, list(self.params))


def _signs_for(quant_meta: Dict, K: int, device) -> (int, Optional[torch.Tensor]):
    if not quant_meta.get("hadamard_rotation", False):
        return 0, None
    req = int(quant_meta.get("hadamard_block_size", 512))
    return effective_block(req, K), column_signs(K, req, device)


def qweight_from_payload(dtype: str, quant_meta: Dict, payload, M: int, K: int, device="cuda") -> QWeight:
    """Uploads a reference payload (bytes / memoryview / uint8 tensor) plus its
    quant_meta, as stored in a .pflash catalog entry, to the device."""
    fmt = resolve_format(dtype, quant_meta)
    if fmt is None:
        raise ValueError(f"dtype '{dtype}' is a dense payload, not a packed low-bit format")
    device = torch.device(device)
    hb, signs = _signs_for(quant_meta, K, device)
    if fmt in (_lib.FMT_INT4, _lib.FMT_INT3, _lib.FMT_INT2):
        codes = _as_u8(payload, device)
        return QWeight(fmt, M, K, codes, None, None, hb, signs, float(quant_meta.get("scale", 1.0)))
    if fmt == _lib.FMT_POLAR_RECURSIVE:
        d = int(quant_meta.get("block_size", 8))
        alloc = [int(a) for a in quant_meta["alloc"]]
        codes = _as_u8(payload, device)
        angles = None
        if quant_meta.get("has_learned_codebooks") and quant_meta.get("learned_codebooks"):
            angles = encoders.polar_angle_table(d, alloc, quant_meta["learned_codebooks"], device)
        return QWeight(fmt, M, K, codes, angles, None, hb, signs, float(quant_meta["r_scale"]), [d] + alloc)
    if fmt == _lib.FMT_POLAR2D:
        codes = _as_u8(payload, device)
        return QWeight(fmt, M, K, codes, None, None, hb, signs, float(quant_meta.get("r_scale", 1.0)),
                       [int(quant_meta.get("r_bits", 4)), int(quant_meta.get("theta_bits", 4))])
    # extension formats: payload = codes followed by the scale arrays (layout below)
    raw = _as_u8(payload, device)
    return _split_extension_payload(fmt, raw, M, K, hb, signs)


def extension_payload_layout(fmt: int, M: int, K: int):
    """Byte layout of an extension payload as stored in a .pflash tensor:
    group INT: [codes u32 M*(K/128)*w][scales fp16 M*(K/128)][mins fp16 M*(K/128)];
    E8: [idx u8 M*(K/8)*2][scales fp16 M*(K/128)*2].  Each part padded to 256 B."""
    G = K // 128
    pad = lambda n: (n + 255) // 256 * 256  # noqa: E731
    if fmt in (_lib.FMT_INT4_G128, _lib.FMT_INT3_G128, _lib.FMT_INT2_G128):
        w = {_lib.FMT_INT4_G128: 16, _lib.FMT_INT3_G128: 13, _lib.FMT_INT2_G128: 8}[fmt]
        return [("codes", M * G * w * 4), ("scales", M * G * 2), ("mins", M * G * 2)], pad
    if fmt == _lib.FMT_E8_RVQ2_G128:
        return [("codes", M * (K // 8) * 2), ("scales", M * G * 2 * 2)], pad
    raise ValueError(fmt)


def _split_extension_payload(fmt, raw, M, K, hb, signs) -> QWeight:
    parts, pad = extension_payload_layout(fmt, M, K)
    off = 0
    views = {}
    for name, n in parts:
        views[name] = raw[off:off + n].clone()
        off += pad(n)
    G = K // 128
    if fmt == _lib.FMT_E8_RVQ2_G128:
        return QWeight(fmt, M, K, views["codes"], views["scales"].view(torch.float16).view(M, G, 2), None, hb, signs)
    return QWeight(fmt, M, K, views["codes"], views["scales"].view(torch.float16).view(M, G),
                   views["mins"].view(torch.float16).view(M, G), hb, signs)


def extension_payload_bytes(qw: QWeight) -> bytes:
    """Serialises an extension-format QWeight into its .pflash payload."""
    parts, pad = extension_payload_layout(qw.format, qw.M, qw.K)
    tensors = {"codes": qw.codes, "scales": qw.scales, "mins": qw.mins}
    out = bytearray()
    for name, n in parts:
        b = tensors[name].detach().contiguous().view(torch.uint8).flatten().cpu().numpy().tobytes()
        assert len(b) == n, (name, len(b), n)
        out += b + b"\x00" * (pad(n) - n)
    return bytes(out)


_ws_cache = {}


def workspace(device, nbytes: int, stream=None) -> torch.Tensor:
    """A zero-initialised workspace of at least `nbytes` for `device`, cached
    per (device, stream): calls on one stream run in order, which is what
    sharing a workspace needs."""
    device = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    key = (device.index, s.cuda_stream)
    ws = _ws_cache.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(max(nbytes, 1 << 20), dtype=torch.uint8, device=device)
        _ws_cache[key] = ws
    return ws


def workspace_status(ws: torch.Tensor, reset: bool = False, counters: bool = False, stream=None):
    """(status, busy_counters) of a workspace after the work queued on
    `stream`: status is OK or the pf_status a device wait recorded
    (ERR_TIMEOUT); busy_counters (when `counters`) the split-K arrival
    counters left non-zero.  `reset` zeroes both so the workspace is usable
    again.  Synchronises the stream."""
    s = stream if stream is not None else torch.cuda.current_stream(ws.device)
    st, busy = ctypes.c_int(0), ctypes.c_int(0)
    _lib.check(_lib.load().pf_workspace_status(_ptr(ws), 1 if reset else 0, ctypes.byref(st),
                                               ctypes.byref(busy) if counters else None,
                                               ctypes.c_void_p(s.cuda_stream)), "pf_workspace_status")
    return int(st.value), (int(busy.value) if counters else None)


def check_device_status(device, stream=None) -> None:
    """Raises RuntimeError (as the reference does for driver failures,
    native_kernels.py:396-410) when a kernel on `stream`'s cached workspace
    recorded a timed-out device wait; the workspace is reset first, so later
    calls can run."""
    device = torch.device(device)
    s = stream if stream is not None else torch.cuda.current_stream(device)
    ws = _ws_cache.get((device.index, s.cuda_stream))
    if ws is None:
        return
    st, _ = workspace_status(ws, stream=s)
    if st != _lib.OK:
        workspace_status(ws, reset=True, stream=s)
        _lib.check(st, "device kernel")


def _x2(qw: QWeight, x: torch.Tensor):
    if x.device.type != "cuda":
        raise ValueError("polarflash_b200.qlinear needs CUDA input tensors (no CPU path)")
    if x.shape[-1] != qw.K:
        raise ValueError(f"input feature dim {x.shape[-1]} != in_features {qw.K}")
    if x.dtype not in _X_DTYPES:
        x = x.float()
    x2 = x.reshape(-1, qw.K)
    if not x2.is_contiguous():
        x2 = x2.contiguous()
    return x2


def _ptr(t: Optional[torch.Tensor]):
    return ctypes.c_void_p(t.data_ptr()) if t is not None else None


def qlinear(qw: QWeight, x: torch.Tensor, bias: Optional[torch.Tensor] = None,
            workspace: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """y = x @ W_hat.T (+ bias), fp32, W_hat never materialised.  x: [..., K]
    CUDA tensor (fp32/fp16/bf16).  Launches on torch's current stream.  A
    caller-provided `workspace` must have been zero-filled once."""
    lead = x.shape[:-1]
    x2 = _x2(qw, x)
    N = x2.shape[0]
    y = out if out is not None else torch.empty(N, qw.M, dtype=torch.float32, device=x.device)
    if N == 0:
        return y.reshape(*lead, qw.M)
    need = qw.workspace_bytes(N)
    stream = torch.cuda.current_stream(x.device)
    ws = workspace if workspace is not None else globals()["workspace"](x.device, need, stream)
    if ws.numel() < need:
        raise ValueError(f"workspace of {ws.numel()} bytes < {need} needed")
    b = bias.to(device=x.device, dtype=torch.float32).contiguous() if bias is not None else None
    st = _lib.load().pf_qlinear(
        ctypes.byref(qw.descriptor()), _ptr(x2), _X_DTYPES[x2.dtype], N, _ptr(b), _ptr(y), _ptr(ws),
        ws.numel(), ctypes.c_void_p(stream.cuda_stream))
    _lib.check(st, "pf_qlinear")
    return y.reshape(*lead, qw.M)


def _desc_array(qws):
    n = len(qws)
    arr = (ctypes.POINTER(_lib.PFQWeight) * n)()
    for i, q in enumerate(qws):
        arr[i] = ctypes.pointer(q.descriptor())
    return arr


def group_workspace_bytes(qws, N: int) -> int:
    """Device workspace bytes of one qlinear_group call over `qws`."""
    out = ctypes.c_size_t(0)
    _lib.check(_lib.load().pf_qlinear_group_workspace_size(len(qws), _desc_array(qws), N, ctypes.byref(out)),
               "pf_qlinear_group_workspace_size")
    return int(out.value)


def qlinear_group(qws, xs, biases=None, workspace: Optional[torch.Tensor] = None, outs=None):
    """[x_i @ W_i^T (+ b_i)] through one pf_qlinear_group call: weights of one
    INT format that the streaming GEMV serves run as ONE launch per 16 tokens
    (up to four weights per launch); other weights run one after another.
    Every x_i has the same leading shape and dtype."""
    n = len(qws)
    if n == 0:
        return []
    lead = xs[0].shape[:-1]
    x2s = [_x2(q, x) for q, x in zip(qws, xs)]
    dt = x2s[0].dtype
    if any(x.dtype != dt for x in x2s):
        x2s = [x.float() for x in x2s]
        dt = torch.float32
    N = x2s[0].shape[0]
    if any(x.shape[0] != N for x in x2s):
        raise ValueError("qlinear_group inputs need the same number of rows")
    dev = x2s[0].device
    ys = [outs[i] if outs is not None else torch.empty(N, q.M, dtype=torch.float32, device=dev)
          for i, q in enumerate(qws)]
    if N == 0:
        return [y.reshape(*lead, q.M) for y, q in zip(ys, qws)]
    bs = []
    for i in range(n):
        b = None if biases is None else biases[i]
        bs.append(b.to(device=dev, dtype=torch.float32).contiguous() if b is not None else None)
    need = group_workspace_bytes(qws, N)
    stream = torch.cuda.current_stream(dev)
    ws = workspace if workspace is not None else globals()["workspace"](dev, need, stream)
    if ws.numel() < need:
        raise ValueError(f"workspace of {ws.numel()} bytes < {need} needed")
    VP = ctypes.c_void_p * n
    xa = VP(*[x.data_ptr() for x in x2s])
    ya = VP(*[y.data_ptr() for y in ys])
    ba = VP(*[b.data_ptr() if b is not None else None for b in bs])
    st = _lib.load().pf_qlinear_group(n, _desc_array(qws), xa, _X_DTYPES[dt], N, ba, ya, _ptr(ws), ws.numel(),
                                      ctypes.c_void_p(stream.cuda_stream))
    _lib.check(st, "pf_qlinear_group")
    return [y.reshape(*lead, q.M) for y, q in zip(ys, qws)]


def qlinear_multi(qws, x: torch.Tensor, biases=None, workspace: Optional[torch.Tensor] = None, outs=None):
    """[x @ W_i^T (+ b_i)] for weights sharing one input (q/k/v, gate/up):
    qlinear_group with the same x for every weight."""
    return qlinear_group(qws, [x] * len(qws), biases, workspace, outs)


def dequantize(qw: QWeight, inverse_rwht: bool = True) -> torch.Tensor:
    """W_hat fp32 [M, K] on the device (UnifiedQuantizer.dequantize semantics)."""
    W = torch.empty(qw.M, qw.K, dtype=torch.float32, device=qw.device)
    st = _lib.load().pf_dequant(ctypes.byref(qw.descriptor()), ctypes.c_void_p(W.data_ptr()),
                                1 if inverse_rwht else 0,
                                ctypes.c_void_p(torch.cuda.current_stream(qw.device).cuda_stream))
    _lib.check(st, "pf_dequant")
    return W


def unpack_codes(qw: QWeight) -> torch.Tensor:
    """Raw codes u8 [M, K] (INT formats) or E8 indices u8 [M, K/8, 2]."""
    if qw.format == _lib.FMT_E8_RVQ2_G128:
        out = torch.empty(qw.M, qw.K // 8, 2, dtype=torch.uint8, device=qw.device)
    else:
        out = torch.empty(qw.M, qw.K, dtype=torch.uint8, device=qw.device)
    st = _lib.load().pf_unpack_codes(ctypes.byref(qw.descriptor()), ctypes.c_void_p(out.data_ptr()),
                                     ctypes.c_void_p(torch.cuda.current_stream(qw.device).cuda_stream))
    _lib.check(st, "pf_unpack_codes")
    return out


def payload_nbytes(qw: QWeight) -> int:
    return qw.nbytes()


def numpy_f16_bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.float16)
