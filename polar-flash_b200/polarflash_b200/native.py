"""NativeLowBitCUDAEngine mirror (polarflash_rt/cuda/native_kernels.py:336-655).

The reference's three hand-written kernels (int4/int2 GEMV, int4 GEMM; per-row
fp32 scales, codes nibble-8 / code-2, no rotation) map onto the library's
tensor-core GEMV through pf_native_*.  Unlike the reference there is no PyTorch
fallback: ``is_available`` is True only when a CUDA device and the built
library are present, and the ops raise otherwise.
"""
import ctypes
import time
from typing import Any, Dict, Optional

import torch

from . import _lib
from .qweight import workspace as _workspace


class NativeLowBitCUDAEngine:
    _instance: Optional["NativeLowBitCUDAEngine"] = None

    def __init__(self, arch: str = "sm_100a"):
        self.arch = arch
        self.is_available = False
        self.init_error = ""
        if not torch.cuda.is_available():
            self.init_error = "no CUDA device"
            return
        try:
            _lib.load()
            self.is_available = True
        except Exception as e:  # noqa: BLE001
            self.init_error = str(e)

    @classmethod
    def get_instance(cls) -> "NativeLowBitCUDAEngine":
        if cls._instance is None:
            cls._instance = NativeLowBitCUDAEngine()
        return cls._instance

    def _require(self):
        if not self.is_available:
            raise RuntimeError(f"NativeLowBitCUDAEngine unavailable: {self.init_error}")

    def _call(self, fn, x, packed, scales, M, K, N=None):
        self._require()
        x = x.contiguous().float()
        packed = packed.contiguous()
        scales = scales.contiguous().float()
        y_shape = (M,) if N is None else (N, M)
        y = torch.empty(y_shape, dtype=torch.float32, device=x.device)
        qw = _lib.PFQWeight()
        qw.format = _lib.FMT_INT4 if fn != "pf_native_gemv_int2" else _lib.FMT_INT2
        qw.M, qw.K = M, K
        qw.codes, qw.scales = packed.data_ptr(), scales.data_ptr()
        need = ctypes.c_size_t(0)
        _lib.check(_lib.load().pf_qlinear_workspace_size(ctypes.byref(qw), N or 1, ctypes.byref(need)), fn)
        ws = _workspace(x.device, int(need.value))
        stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
        P = ctypes.c_void_p
        L = _lib.load()
        if N is None:
            st = getattr(L, fn)(P(x.data_ptr()), P(packed.data_ptr()), P(scales.data_ptr()), M, K, P(y.data_ptr()),
                                P(ws.data_ptr()), ws.numel(), stream)
        else:
            st = L.pf_native_gemm_int4(P(x.data_ptr()), P(packed.data_ptr()), P(scales.data_ptr()), N, M, K,
                                       P(y.data_ptr()), P(ws.data_ptr()), ws.numel(), stream)
        _lib.check(st, fn)
        return y

    def gemv_int4(self, x, packed_weights, scales, out_features, in_features):
        """y = W x, W[m, k] = (nibble - 8) * scales[m]; packed [M, K/2] uint8."""
        return self._call("pf_native_gemv_int4", x, packed_weights, scales, out_features, in_features)

    def gemv_int2(self, x, packed_weights, scales, out_features, in_features):
        """y = W x, W[m, k] = (code - 2) * scales[m]; packed [M, K/4] uint8."""
        return self._call("pf_native_gemv_int2", x, packed_weights, scales, out_features, in_features)

    def gemm_int4(self, X, packed_weights, scales, out_features, in_features):
        """Y = X W^T for X [N, K]."""
        return self._call("pf_native_gemm_int4", X, packed_weights, scales, out_features, in_features,
                          N=X.shape[0])

    def benchmark_comparison(self, out_features: int = 2048, in_features: int = 2048,
                             iterations: int = 50) -> Dict[str, Any]:
        """Side-by-side timing (CUDA events) of fp16 torch.matmul, the reference's
        unpack-then-GEMM path, and the fused kernel (native_kernels.py:578-655)."""
        self._require()
        dev = "cuda"
        torch.manual_seed(42)
        raw = torch.randint(-8, 8, (out_features, in_features), dtype=torch.int8, device=dev)
        u4 = (raw + 8).to(torch.uint8)
        packed = (u4[:, 0::2] | (u4[:, 1::2] << 4)).contiguous()
        scales = (torch.rand(out_features, device=dev) * 0.1 + 0.01).float()
        x = torch.randn(in_features, device=dev)
        w16 = (raw.float() * scales[:, None]).half()
        x16 = x.half()

        def unpack_gemm():
            lo = (packed & 0x0F).to(torch.int8) - 8
            hi = ((packed >> 4) & 0x0F).to(torch.int8) - 8
            w = torch.empty(out_features, in_features, dtype=torch.int8, device=dev)
            w[:, 0::2] = lo
            w[:, 1::2] = hi
            return torch.matmul(w.float() * scales[:, None], x)

        def timed(fn):
            for _ in range(5):
                fn()
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            for _ in range(iterations):
                fn()
            e.record()
            e.synchronize()
            return s.elapsed_time(e) / iterations

        fp16 = timed(lambda: torch.matmul(w16, x16))
        deq = timed(unpack_gemm)
        fused = timed(lambda: self.gemv_int4(x, packed, scales, out_features, in_features))
        return {
            "device": torch.cuda.get_device_name(0), "architecture": self.arch,
            "kernel_execution_path": "NATIVE_FUSED_CUDA_KERNEL",
            "dimensions": f"{out_features}x{in_features}",
            "fp16_latency_ms": round(fp16, 4), "dequantize_plus_gemm_latency_ms": round(deq, 4),
            "native_fused_int4_latency_ms": round(fused, 4),
            "speedup_vs_dequantize_plus_gemm": round(deq / max(fused, 1e-6), 2),
            "vram_savings_ratio": round(out_features * in_features * 4 / packed.numel(), 2),
            "packed_weight_vram_kb": packed.numel() / 1024.0,
            "materialized_fp32_vram_kb": out_features * in_features * 4 / 1024.0,
            "timestamp": time.time(),
        }
