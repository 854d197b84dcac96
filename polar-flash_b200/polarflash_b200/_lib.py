"""ctypes binding of libpolarflash_b200.so (the C ABI in include/polarflash_b200.h).

The library is required: there is no CPU or PyTorch fallback for the compute
path.  If the shared object is missing the import of the compute entry points
raises immediately with the build command to run.
"""
import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "lib", "libpolarflash_b200.so")

# pf_format
FMT_INT4_G128 = 1
FMT_INT3_G128 = 2
FMT_INT2_G128 = 3
FMT_INT4 = 4
FMT_INT3 = 5
FMT_INT2 = 6
FMT_E8_RVQ2_G128 = 7
FMT_POLAR_RECURSIVE = 8
FMT_POLAR2D = 9

# pf_dtype
DTYPE_F32 = 0
DTYPE_F16 = 1
DTYPE_BF16 = 2

# pf_status
OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_SHAPE = 2
ERR_ALIGNMENT = 3
ERR_UNSUPPORTED = 4
ERR_WORKSPACE = 5
ERR_CUDA = 6
ERR_TIMEOUT = 7

# Every symbol include/polarflash_b200.h declares.
EXPORTS = (
    "pf_version", "pf_status_string", "pf_last_cuda_error", "pf_kernel_launches", "pf_qweight_check",
    "pf_qlinear_workspace_size", "pf_qlinear", "pf_qlinear_group_workspace_size", "pf_qlinear_group",
    "pf_dequant", "pf_unpack_codes", "pf_rwht",
    "pf_native_gemv_int4", "pf_native_gemv_int2", "pf_native_gemm_int4", "pf_qlinear_noalloc",
    "pf_add_rmsnorm", "pf_rope_kv", "pf_decode_attention_workspace_size", "pf_decode_attention", "pf_silu_mul",
    "pf_kv_row_bytes", "pf_kv_quantize", "pf_kv_dequantize", "pf_rope_kv_compressed",
    "pf_decode_attention_compressed", "pf_workspace_status", "pf_qlinear_noalloc_status", "pf_wait_selftest",
    "pf_peer_export", "pf_peer_open", "pf_peer_close", "pf_qlinear_group_gather", "pf_peers_wait",
    "pf_allgather_rows",
)


class PFQWeight(ctypes.Structure):
    """Mirror of ``struct pf_qweight``."""

    _fields_ = [
        ("format", ctypes.c_int32),
        ("M", ctypes.c_int32),
        ("K", ctypes.c_int32),
        ("had_block", ctypes.c_int32),
        ("codes", ctypes.c_void_p),
        ("scales", ctypes.c_void_p),
        ("mins", ctypes.c_void_p),
        ("had_signs", ctypes.c_void_p),
        ("tensor_scale", ctypes.c_double),
        ("params", ctypes.c_int32 * 20),
    ]


class PFPeers(ctypes.Structure):
    """Mirror of ``struct pf_peers``."""

    _fields_ = [
        ("world", ctypes.c_int32),
        ("rank", ctypes.c_int32),
        ("bases", ctypes.c_void_p * 8),
        ("bytes", ctypes.c_size_t),
    ]


class PolarFlashError(RuntimeError):
    pass


_lib = None


def load():
    """Loads the CUDA library (once).  Raises if it has not been built."""
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build the CUDA library with "
            "`python polar-flash_b200/build.py` (there is no CPU fallback)")
    L = ctypes.CDLL(LIB_PATH)
    P, I, SZ = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    QW = ctypes.POINTER(PFQWeight)
    L.pf_version.restype = ctypes.c_char_p
    L.pf_version.argtypes = []
    L.pf_status_string.restype = ctypes.c_char_p
    L.pf_status_string.argtypes = [I]
    L.pf_last_cuda_error.restype = I
    L.pf_last_cuda_error.argtypes = []
    L.pf_kernel_launches.restype = ctypes.c_ulonglong
    L.pf_kernel_launches.argtypes = []
    L.pf_qweight_check.restype = I
    L.pf_qweight_check.argtypes = [QW]
    L.pf_qlinear_workspace_size.restype = I
    L.pf_qlinear_workspace_size.argtypes = [QW, I, ctypes.POINTER(SZ)]
    L.pf_qlinear.restype = I
    L.pf_qlinear.argtypes = [QW, P, I, I, P, P, P, SZ, P]
    PP = ctypes.POINTER(ctypes.c_void_p)
    QWP = ctypes.POINTER(QW)
    L.pf_qlinear_group_workspace_size.restype = I
    L.pf_qlinear_group_workspace_size.argtypes = [I, QWP, I, ctypes.POINTER(SZ)]
    L.pf_qlinear_group.restype = I
    L.pf_qlinear_group.argtypes = [I, QWP, PP, I, I, PP, PP, P, SZ, P]
    L.pf_dequant.restype = I
    L.pf_dequant.argtypes = [QW, P, I, P]
    L.pf_unpack_codes.restype = I
    L.pf_unpack_codes.argtypes = [QW, P, P]
    L.pf_rwht.restype = I
    L.pf_rwht.argtypes = [P, P, I, I, I, P, I, P]
    for name in ("pf_native_gemv_int4", "pf_native_gemv_int2"):
        fn = getattr(L, name)
        fn.restype = I
        fn.argtypes = [P, P, P, I, I, P, P, SZ, P]
    L.pf_native_gemm_int4.restype = I
    L.pf_native_gemm_int4.argtypes = [P, P, P, I, I, I, P, P, SZ, P]
    F = ctypes.c_float
    L.pf_add_rmsnorm.restype = I
    L.pf_add_rmsnorm.argtypes = [P, P, P, P, I, I, F, P]
    L.pf_rope_kv.restype = I
    L.pf_rope_kv.argtypes = [P, P, P, P, P, P, P, I, I, I, I, P]
    L.pf_decode_attention.restype = I
    L.pf_decode_attention.argtypes = [P, P, P, P, P, I, I, I, I, F, P, SZ, P]
    L.pf_decode_attention_workspace_size.restype = SZ
    L.pf_decode_attention_workspace_size.argtypes = [I, I, I]
    L.pf_silu_mul.restype = I
    L.pf_silu_mul.argtypes = [P, P, P, ctypes.c_longlong, P]
    LL = ctypes.c_longlong
    L.pf_kv_row_bytes.restype = SZ
    L.pf_kv_row_bytes.argtypes = [I, I]
    L.pf_kv_quantize.restype = I
    L.pf_kv_quantize.argtypes = [P, LL, I, I, P, P, P, P]
    L.pf_kv_dequantize.restype = I
    L.pf_kv_dequantize.argtypes = [P, P, P, LL, I, I, P, P]
    L.pf_rope_kv_compressed.restype = I
    L.pf_rope_kv_compressed.argtypes = [P, P, P, P, P, P, P, P, P, P, P, I, I, I, I, I, P]
    L.pf_decode_attention_compressed.restype = I
    L.pf_decode_attention_compressed.argtypes = [P, P, P, P, P, P, P, P, P, I, I, I, I, I, F, P, SZ, P]
    IP = ctypes.POINTER(I)
    L.pf_workspace_status.restype = I
    L.pf_workspace_status.argtypes = [P, I, IP, IP, P]
    L.pf_qlinear_noalloc_status.restype = I
    L.pf_qlinear_noalloc_status.argtypes = [I, IP, IP, P]
    L.pf_wait_selftest.restype = I
    L.pf_wait_selftest.argtypes = [P, ctypes.c_ulonglong, P]
    U8P = ctypes.POINTER(ctypes.c_ubyte)
    L.pf_peer_export.restype = I
    L.pf_peer_export.argtypes = [P, U8P, ctypes.POINTER(SZ)]
    L.pf_peer_open.restype = I
    L.pf_peer_open.argtypes = [U8P, SZ, ctypes.POINTER(P), ctypes.POINTER(P)]
    L.pf_peer_close.restype = I
    L.pf_peer_close.argtypes = [P]
    PEERS = ctypes.POINTER(PFPeers)
    L.pf_qlinear_group_gather.restype = I
    L.pf_qlinear_group_gather.argtypes = [I, QWP, PP, I, I, PP, ctypes.POINTER(SZ), ctypes.POINTER(I), PEERS, P, SZ, P]
    L.pf_peers_wait.restype = I
    L.pf_peers_wait.argtypes = [PEERS, P, P]
    L.pf_allgather_rows.restype = I
    L.pf_allgather_rows.argtypes = [PEERS, P, ctypes.c_size_t, ctypes.c_size_t, P, P]
    _lib = L
    return L


def check(status: int, what: str = "polarflash_b200") -> None:
    """Raises the reference's exception classes for a non-zero pf_status:
    ValueError for argument problems (unified_quantizer.py:100-101,
    cuda/engine.py:91-92), RuntimeError for CUDA failures
    (native_kernels.py:396-410, 465-466)."""
    if status == OK:
        return
    L = load()
    msg = L.pf_status_string(status).decode()
    if status in (ERR_CUDA, ERR_TIMEOUT):
        raise PolarFlashError(f"{what}: {msg} (cuda error {L.pf_last_cuda_error()})")
    raise ValueError(f"{what}: {msg}")


def version() -> str:
    return load().pf_version().decode()


def kernel_launches() -> int:
    """Kernel launches the library has issued in this process (graph captures
    count once; replays add nothing)."""
    return int(load().pf_kernel_launches())
