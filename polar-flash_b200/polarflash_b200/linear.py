"""PolarLinearLayer mirror: a quantized linear layer whose forward is the fused
dequant-GEMV/GEMM of this library.

Same constructor as the reference (polarflash_rt/cpu/engine.py:36-56).  The
packed payload is uploaded to the device once (the layer's only device state);
``forward`` never materialises W.  Dense payloads (fp16 / bf16 / int8 /
fp16 E8 reconstructions) keep one decoded device copy and use torch.matmul,
as the reference's cached path does.
"""
from typing import Any, Dict, Optional, Union

import torch
import torch.nn as nn

from .qweight import QWeight, dequantize as _dequant, qlinear, qweight_from_payload, resolve_format
from .quantizer import dense_weight


class PolarLinearLayer(nn.Module):
    def __init__(self, in_features: int, out_features: int, dtype: str, quant_meta: Dict[str, Any],
                 raw_bytes: Union[bytes, memoryview, torch.Tensor], bias: Optional[torch.Tensor] = None,
                 keep_cached: bool = True, device: Union[str, torch.device, None] = None):
        super().__init__()
        self.in_features = in_features
        self.out_features = out_features
        self.dtype = dtype.lower()
        self.quant_meta = quant_meta
        self.bias = bias
        self.keep_cached = keep_cached
        self.cached_weight: Optional[torch.Tensor] = None
        self._raw_bytes = raw_bytes
        self.fmt = resolve_format(self.dtype, quant_meta)
        self.qweight: Optional[QWeight] = None
        self._device = torch.device(device) if device is not None else None
        self._bias_dev: Optional[torch.Tensor] = None
        if self._device is not None and self._device.type == "cuda":
            self._materialise(self._device)

    @property
    def is_packed(self) -> bool:
        return self.fmt is not None

    def _materialise(self, device: torch.device) -> None:
        if self.is_packed:
            if self.qweight is None or self.qweight.device != device:
                self.qweight = qweight_from_payload(self.dtype, self.quant_meta, self._raw_bytes,
                                                    self.out_features, self.in_features, device)
        elif self.cached_weight is None or self.cached_weight.device != device:
            self.cached_weight = dense_weight(self._raw_bytes, [self.out_features, self.in_features],
                                              self.dtype, self.quant_meta, device)
        if self.bias is not None:
            self._bias_dev = self.bias.to(device=device, dtype=torch.float32)
        self._device = device

    def dequantize(self, device: str = "cuda") -> torch.Tensor:
        """Decoded fp32 weight (inverse RWHT applied) on `device`."""
        dev = torch.device(device)
        if dev.type != "cuda":
            dev = torch.device("cuda")
        self._materialise(dev)
        if self.is_packed:
            return _dequant(self.qweight, inverse_rwht=True)
        return self.cached_weight

    def clear_cache(self) -> None:
        """Drops the decoded dense copy (packed layers hold none)."""
        if not self.is_packed:
            self.cached_weight = None

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        """Y = X @ W.T + bias, fp32 output (cpu/engine.py:90-96)."""
        if x.device.type != "cuda":
            raise ValueError("PolarLinearLayer (polarflash_b200) runs on CUDA inputs; move x to the GPU")
        if self._device != x.device or (self.is_packed and self.qweight is None) or \
                (not self.is_packed and self.cached_weight is None):
            self._materialise(x.device)
        if self.is_packed:
            return qlinear(self.qweight, x, self._bias_dev)
        out = torch.matmul(x.float(), self.cached_weight.t())
        if self._bias_dev is not None:
            out = out + self._bias_dev
        if not self.keep_cached:
            self.cached_weight = None
        return out

    @classmethod
    def from_qweight(cls, qw: QWeight, dtype: str = "packed", bias: Optional[torch.Tensor] = None):
        layer = cls.__new__(cls)
        nn.Module.__init__(layer)
        layer.in_features, layer.out_features = qw.K, qw.M
        layer.dtype, layer.quant_meta, layer.bias = dtype, {}, bias
        layer.keep_cached, layer.cached_weight, layer._raw_bytes = True, None, None
        layer.fmt, layer.qweight, layer._device = qw.format, qw, qw.device
        layer._bias_dev = bias.to(device=qw.device, dtype=torch.float32) if bias is not None else None
        return layer
