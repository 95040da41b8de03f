"""ctypes binding of libb200fo.so (declared in include/b200fo.h).

The library is the only compute path of this package: there is no CPU or PyTorch
fallback.  If the shared object is missing, `lib()` builds it with nvcc when a CUDA
toolkit is present and otherwise raises.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

_PKG = Path(__file__).resolve().parent
LIB_PATH = _PKG / "libb200fo.so"

FO_OK = 0
FO_EINVAL = -1
FO_ECUDA = -2
FO_EUNSUPPORTED = -3
FO_ENODEVICE = -4
FO_ETIMEOUT = -5

FO_DT_F16, FO_DT_BF16, FO_DT_F32 = 0, 1, 2
FO_B_KN, FO_B_NK = 0, 1
(FO_EPI_NONE, FO_EPI_BIAS, FO_EPI_BIAS_RELU, FO_EPI_BIAS_GELU_TANH, FO_EPI_BIAS_GELU_ERF,
 FO_EPI_BIAS_LN, FO_EPI_RELU, FO_EPI_BIAS_RESIDUAL_LN, FO_EPI_BN, FO_EPI_BN_RELU, FO_EPI_BN_ADD_RELU) = range(11)
FO_NOALLOC_LN_SCRATCH_BYTES = 8 << 20

# Every symbol include/b200fo.h declares; tests check the library exports all of them.
EXPORTED = (
    "fo_gemm", "fo_gemm_workspace_size", "fo_conv2d", "fo_query_config_legal",
    "fo_config_smem_bytes", "fo_device_status", "fo_set_wait_timeout_ns",
    "fo_selftest_wait_timeout", "fo_last_error", "fo_version", "fo_launch_count",
    "fo_gemm_bias_layernorm_noalloc", "fo_conv2d_workspace_size",
)


class FoTileCfg(ctypes.Structure):
    _fields_ = [("block_m", ctypes.c_int32), ("block_n", ctypes.c_int32),
                ("block_k", ctypes.c_int32), ("stages", ctypes.c_int32),
                ("group_m", ctypes.c_int32), ("max_ctas", ctypes.c_int32), ("swap_ab", ctypes.c_int32),
                ("split_k", ctypes.c_int32), ("split_mode", ctypes.c_int32), ("ln_mode", ctypes.c_int32)]


class FoGemmDesc(ctypes.Structure):
    _fields_ = [("M", ctypes.c_int64), ("N", ctypes.c_int64), ("K", ctypes.c_int64),
                ("a", ctypes.c_void_p), ("b", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("gamma", ctypes.c_void_p), ("beta", ctypes.c_void_p), ("out", ctypes.c_void_p),
                ("lda", ctypes.c_int64), ("ldb", ctypes.c_int64), ("ldo", ctypes.c_int64),
                ("in_dtype", ctypes.c_int32), ("vec_dtype", ctypes.c_int32),
                ("out_dtype", ctypes.c_int32), ("b_layout", ctypes.c_int32),
                ("epilogue", ctypes.c_int32), ("eps", ctypes.c_float),
                ("workspace", ctypes.c_void_p), ("workspace_bytes", ctypes.c_size_t),
                ("residual", ctypes.c_void_p), ("ldr", ctypes.c_int64)]


class FoConvDesc(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("n", "h", "w", "c", "f", "kh", "kw", "stride", "pad", "dil")] + [
                ("x", ctypes.c_void_p), ("wgt", ctypes.c_void_p), ("bias", ctypes.c_void_p),
                ("out", ctypes.c_void_p), ("in_dtype", ctypes.c_int32),
                ("vec_dtype", ctypes.c_int32), ("out_dtype", ctypes.c_int32),
                ("epilogue", ctypes.c_int32), ("workspace", ctypes.c_void_p),
                ("workspace_bytes", ctypes.c_size_t), ("bn_gamma", ctypes.c_void_p),
                ("bn_beta", ctypes.c_void_p), ("bn_mean", ctypes.c_void_p), ("bn_var", ctypes.c_void_p),
                ("bn_eps", ctypes.c_float), ("residual", ctypes.c_void_p)]


class FoError(RuntimeError):
    """A libb200fo call returned a non-zero code; `code` is the FO_E* value."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"[b200fo {code}] {msg}")
        self.code = code


_lock = threading.Lock()
_lib: ctypes.CDLL | None = None


def _declare(l: ctypes.CDLL) -> None:
    P = ctypes.POINTER
    l.fo_gemm.argtypes = [P(FoGemmDesc), P(FoTileCfg), ctypes.c_void_p]
    l.fo_gemm.restype = ctypes.c_int
    l.fo_gemm_bias_layernorm_noalloc.argtypes = [P(FoGemmDesc), P(FoTileCfg), ctypes.c_void_p]
    l.fo_gemm_bias_layernorm_noalloc.restype = ctypes.c_int
    l.fo_gemm_workspace_size.argtypes = [P(FoGemmDesc), P(FoTileCfg)]
    l.fo_gemm_workspace_size.restype = ctypes.c_size_t
    l.fo_conv2d.argtypes = [P(FoConvDesc), P(FoTileCfg), ctypes.c_void_p]
    l.fo_conv2d.restype = ctypes.c_int
    l.fo_conv2d_workspace_size.argtypes = [P(FoConvDesc), P(FoTileCfg)]
    l.fo_conv2d_workspace_size.restype = ctypes.c_size_t
    l.fo_query_config_legal.argtypes = [ctypes.c_int32, ctypes.c_int32, P(FoTileCfg),
                                        ctypes.c_char_p, ctypes.c_size_t]
    l.fo_query_config_legal.restype = ctypes.c_int
    l.fo_config_smem_bytes.argtypes = [ctypes.c_int32, ctypes.c_int32, P(FoTileCfg)]
    l.fo_config_smem_bytes.restype = ctypes.c_size_t
    l.fo_device_status.argtypes = [ctypes.c_int32, ctypes.c_int32, P(ctypes.c_int32)]
    l.fo_device_status.restype = ctypes.c_int
    l.fo_set_wait_timeout_ns.argtypes = [ctypes.c_uint64]
    l.fo_set_wait_timeout_ns.restype = ctypes.c_int
    l.fo_selftest_wait_timeout.argtypes = [ctypes.c_uint64, ctypes.c_void_p]
    l.fo_selftest_wait_timeout.restype = ctypes.c_int
    l.fo_last_error.argtypes = [ctypes.c_char_p, ctypes.c_size_t]
    l.fo_last_error.restype = ctypes.c_int
    l.fo_version.argtypes = []
    l.fo_version.restype = ctypes.c_char_p
    l.fo_launch_count.argtypes = []
    l.fo_launch_count.restype = ctypes.c_uint64


def lib() -> ctypes.CDLL:
    """Loads libb200fo.so (building it first if it is absent and nvcc is available)."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not LIB_PATH.exists():
                from . import build as _build
                _build.build()
            l = ctypes.CDLL(str(LIB_PATH))
            _declare(l)
            _lib = l
    return _lib


def last_error() -> str:
    buf = ctypes.create_string_buffer(1024)
    lib().fo_last_error(buf, len(buf))
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != FO_OK:
        raise FoError(rc, last_error())


def version() -> str:
    return lib().fo_version().decode()


def launch_count() -> int:
    return int(lib().fo_launch_count())


SPLIT_AUTO, SPLIT_WORKSPACE, SPLIT_CLUSTER = 0, 1, 2
LN_AUTO, LN_TWO_KERNELS, LN_ONE_KERNEL, LN_HELD = 0, 1, 2, 3


def tile_cfg(block_n: int = 256, stages: int = 4, group_m: int = 8, max_ctas: int = 0,
             block_m: int = 128, block_k: int = 64, swap_ab: int = 0, split_k: int = 0,
             split_mode: int = 0, ln_mode: int = 0) -> FoTileCfg:
    return FoTileCfg(block_m, block_n, block_k, stages, group_m, max_ctas, swap_ab, split_k, split_mode, ln_mode)


def config_legal(op: int, out_dtype: int, cfg: FoTileCfg) -> tuple[bool, str]:
    why = ctypes.create_string_buffer(256)
    rc = lib().fo_query_config_legal(op, out_dtype, ctypes.byref(cfg), why, len(why))
    return rc == FO_OK, why.value.decode()


def config_smem_bytes(op: int, out_dtype: int, cfg: FoTileCfg) -> int:
    return int(lib().fo_config_smem_bytes(op, out_dtype, ctypes.byref(cfg)))


def device_status(device: int, clear: bool = True) -> tuple[int, int]:
    where = ctypes.c_int32(0)
    rc = lib().fo_device_status(device, 1 if clear else 0, ctypes.byref(where))
    return rc, int(where.value)


def set_wait_timeout_ns(ns: int) -> None:
    check(lib().fo_set_wait_timeout_ns(ns))
