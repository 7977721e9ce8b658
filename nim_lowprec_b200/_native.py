"""ctypes binding of liblowprec_cuda.so (the C ABI in include/lowprec_cuda.h).

Loading fails loudly: there is no CPU fallback anywhere in this package.
"""
from __future__ import annotations

import ctypes
import os
import re

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "liblowprec_cuda.so")
HEADER = os.path.join(os.path.dirname(HERE), "include", "lowprec_cuda.h")

LP_OK = 0
LP_ERR_SHAPE = 1
LP_ERR_ARG = 2
LP_ERR_CUDA = 3
LP_ERR_NCCL = 4
LP_ERR_TIMEOUT = 5
LP_ERR_UNSUPPORTED = 6
LP_ERR_NO_DEVICE = 7

LP_FP32_FAST = 0
LP_FP32_EXACT = 1

_i64 = ctypes.c_int64
_i32 = ctypes.c_int32
_vp = ctypes.c_void_p
_f32 = ctypes.c_float

# argument kinds by C type, for the prototype table below
_CT = {"p": _vp, "n": _i64, "f": _f32, "i": _i32}

# name -> argument signature (p = pointer, n = int64, f = float, i = int32)
SIGNATURES = {
    "lp_dequant_gemv": "pnpnnpnpnp",
    "lp_dequant_gemv_i4": "pnpnnpnpnp",
    "lp_dequant_gemv_f4": "pnpnnpnpnp",
    "lp_dequant_gemv_q8_0": "pnnpnpnp",
    "lp_dequant_gemv_q4_0": "pnnpnpnp",
    "lp_dequant_gemv_q8": "pnpnnpnpnpnp",
    "lp_dequant_gemv_i4q8": "pnpnnpnpnpnp",
    "lp_dequant_gemv_q8_0q8": "pnnpnpnp",
    "lp_dequant_gemv_q4_0q8": "pnnpnpnp",
    "lp_dequant_gemm_q8": "pnpnnpnpnnpnp",
    "lp_dequant_gemm_i4q8": "pnpnnpnpnnpnp",
    "lp_quantize_q8_0_batch": "pnpnp",
    "lp_quantize_q4_0_batch": "pnpnp",
    "lp_quantize_q8_0_split": "pnpnpnp",
    "lp_quantize_batch": "pnpnpnnpnp",
    "lp_host_device_pointer": "pp",
    "lp_quantize_dequant_gemv_q8": "pnpnnpnpnp",
    "lp_quantize_dequant_gemv_i4q8": "pnpnnpnpnp",
    "lp_copy_in": "ppnp",
    "lp_dequantize_batch": "pnpnpnnpnp",
    "lp_calibrate_symmetric": "pnnfpnp",
    "lp_calibrate_mx": "pnnipnp",
    "lp_quantize_i4_packed": "pnpnnpnp",
    "lp_quantize_f4_packed": "pnpnnpnp",
    "lp_dequantize_q8_0_batch": "pnpnp",
    "lp_dequantize_q4_0_batch": "pnpnp",
    "lp_dequantize_q4_k": "pnpnp",
    "lp_dequantize_q6_k": "pnpnp",
    "lp_quantize_nvfp4": "pnpnpnpp",
    "lp_dequantize_nvfp4": "pnpnfpnp",
    "lph_dequant_gemv": "pnpnnpnpn",
    "lph_dequant_gemv_i4": "pnpnnpnpn",
    "lph_dequant_gemv_f4": "pnpnnpnpn",
    "lph_dequant_gemv_q8_0": "pnnpnpn",
    "lph_dequant_gemv_q4_0": "pnnpnpn",
    "lph_dequant_gemv_q4_0_static": "pnnpnpn",
    "lph_dequant_gemv_q8": "pnpnnpnpnpn",
    "lph_dequant_gemv_i4q8": "pnpnnpnpnpn",
    "lph_dequant_gemv_q8_0q8": "pnnpnpn",
    "lph_dequant_gemv_q4_0q8": "pnnpnpn",
    "lph_dequant_gemm_q8": "pnpnnpnpnnpn",
    "lph_dequant_gemm_i4q8": "pnpnnpnpnnpn",
    "lph_quantize_q8_0_batch": "pnpn",
    "lph_quantize_q4_0_batch": "pnpn",
    "lph_quantize_batch": "pnpnpnnpn",
    "lph_dequantize_batch": "pnpnpnnpn",
    "lp_set_fp32_mode": "i",
    "lp_get_fp32_mode": "",
    "lp_pool_rows": "niipp",
    "lp_pool_unique_id": "p",
    "lp_pool_init": "ppiii",
    "lp_batch_begin": "p",
    "lp_batch_end": "p",
    "lp_pool_destroy": "p",
    "lp_pool_size": "ppp",
    "lp_pool_gather_rows": "ppnnp",
    "lp_pool_group_begin": "ppn",
    "lp_pool_group_end": "pp",
    "lp_pool_set_p2p": "pi",
    "lp_pool_get_p2p": "pp",
    "lp_pool_dequant_gemv": "ppnpnnpnpnp",
    "lp_pool_dequant_gemv_i4": "ppnpnnpnpnp",
    "lp_pool_dequant_gemv_f4": "ppnpnnpnpnp",
    "lp_pool_dequant_gemv_q8_0": "ppnnpnpnp",
    "lp_pool_dequant_gemv_q4_0": "ppnnpnpnp",
    "lp_pool_dequant_gemv_q8": "ppnpnnpnpnpnp",
    "lp_pool_dequant_gemv_i4q8": "ppnpnnpnpnpnp",
    "lp_pool_dequant_gemm_q8": "ppnpnnpnpnnpnp",
    "lp_pool_dequant_gemm_i4q8": "ppnpnnpnpnnpnp",
    "lp_pool_quantize_dequant_gemv_q8": "ppnpnnpnpnp",
    "lp_pool_quantize_dequant_gemv_i4q8": "ppnpnnpnpnp",
    "lp_dequant_gemm_f4": "pnpnnpnpnnpnp",
    "lp_dequant_gemv_q4_k": "pnnpnpnp",
    "lp_dequant_gemv_q6_k": "pnnpnpnp",
    "lp_gemm_nvfp4": "pnpnppnpnpnpnp",
    "lph_pool_init": "pi",
    "lph_pool_shutdown": "p",
    "lph_pool_thread_count": "p",
    "lph_pool_dequant_gemv_q8": "ppnpnnpnpnpn",
    "lph_pool_dequant_gemv_i4q8": "ppnpnnpnpnpn",
    "lph_pool_dequant_gemm_q8": "ppnpnnpnpnnpn",
    "lph_pool_dequant_gemm_i4q8": "ppnpnnpnpnnpn",
    "lph_par_dequant_gemv": "pnpnnpnpni",
    "lph_par_dequant_gemv_i4": "pnpnnpnpni",
    "lph_par_dequant_gemv_f4": "pnpnnpnpni",
    "lph_par_dequant_gemv_q8_0": "pnnpnpni",
    "lph_par_dequant_gemv_q4_0": "pnnpnpni",
    "lph_par_dequant_gemv_q8": "pnpnnpnpnpni",
    "lph_par_dequant_gemv_i4q8": "pnpnnpnpnpni",
}


def header_symbols(path: str = HEADER):
    """Every function the public header declares (for export checks)."""
    text = open(path).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(lph?_[a-z0-9_]+)\s*\(", text)))


class NativeError(RuntimeError):
    def __init__(self, status: int, where: str):
        detail = ""
        if status == LP_ERR_CUDA:
            try:
                detail = " [" + lib().lp_last_error_detail().decode() + "]"
            except Exception:  # pragma: no cover
                pass
        super().__init__(f"{where}: {status_string(status)} (status {status}){detail}")
        self.status = status


_lib = None


def lib():
    """Load liblowprec_cuda.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(
                f"{LIB_PATH} is missing: build it with `python nim_lowprec_b200/build.py` "
                "(this package has no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, sig in SIGNATURES.items():
            fn = getattr(L, name)
            fn.restype = ctypes.c_int
            fn.argtypes = [_CT[c] for c in sig]
        L.lp_version.restype = ctypes.c_int
        L.lp_version.argtypes = []
        L.lp_status_string.restype = ctypes.c_char_p
        L.lp_status_string.argtypes = [ctypes.c_int]
        L.lp_last_error_detail.restype = ctypes.c_char_p
        L.lp_last_error_detail.argtypes = []
        L.lp_device_error.restype = ctypes.c_int
        L.lp_device_error.argtypes = []
        _lib = L
    return _lib


def status_string(status: int) -> str:
    try:
        return lib().lp_status_string(int(status)).decode()
    except Exception:  # pragma: no cover
        return f"status {status}"


def check(status: int, where: str) -> None:
    if status == LP_OK:
        return
    if status == LP_ERR_SHAPE:
        # the reference asserts its shape preconditions (AssertionDefect)
        raise AssertionError(f"{where}: {status_string(status)}")
    raise NativeError(status, where)


def host_device_pointer(host_addr: int) -> int:
    """Device address of page-locked host memory (e.g. a pinned torch CPU
    tensor's data_ptr()), for passing activations or outputs that live in
    host memory straight to a device form; raises NativeError otherwise."""
    d = ctypes.c_void_p()
    check(lib().lp_host_device_pointer(ctypes.c_void_p(host_addr), ctypes.byref(d)),
          "host_device_pointer")
    return int(d.value)


def device_error() -> int:
    """Synchronise, then return and clear the first device-side error code."""
    return int(lib().lp_device_error())
