"""CPU checks of the C ABI: the library loads without a GPU, exports every
symbol the public header declares, and rejects bad shapes with LP_ERR_SHAPE
before touching the device (the reference's entry asserts)."""
import ctypes

import numpy as np
import pytest

from nim_lowprec_b200 import _native as N


def test_library_exports_every_header_symbol():
    L = N.lib()
    syms = N.header_symbols()
    assert len(syms) >= 38
    missing = [s for s in syms if not hasattr(L, s)]
    assert missing == []


def test_every_header_symbol_has_a_prototype():
    syms = set(N.header_symbols())
    bound = set(N.SIGNATURES) | {"lp_version", "lp_status_string", "lp_device_error",
                                  "lp_last_error_detail"}
    assert syms <= bound


def test_version_and_status_strings():
    L = N.lib()
    assert L.lp_version() == 100
    assert N.status_string(N.LP_ERR_SHAPE) == "shape precondition failed"
    assert N.status_string(N.LP_ERR_TIMEOUT) == "device-side wait timed out"


NULL = None


@pytest.mark.parametrize("args", [
    # wq_len != m*k
    (NULL, 10, NULL, 2, 32, NULL, 64, NULL, 2, NULL, 1, NULL),
    # k not a multiple of groupSize
    (NULL, 40, NULL, 2, 32, NULL, 40, NULL, 2, NULL, 1, NULL),
    # groupSize 0 (the reference divides by it)
    (NULL, 64, NULL, 2, 0, NULL, 64, NULL, 2, NULL, 1, NULL),
    # xScales.len != gpr
    (NULL, 64, NULL, 2, 32, NULL, 64, NULL, 3, NULL, 1, NULL),
])
def test_gemv_q8_shape_rules(args):
    assert N.lib().lp_dequant_gemv_q8(*args) == N.LP_ERR_SHAPE


def test_i4_requires_even_k_and_packed_length():
    L = N.lib()
    # k = 3 odd, gs 3
    assert L.lp_dequant_gemv_i4q8(NULL, 1, NULL, 1, 3, NULL, 3, NULL, 1, NULL, 1, NULL) == N.LP_ERR_SHAPE
    # packed length must be m*k/2
    assert L.lp_dequant_gemv_i4q8(NULL, 64, NULL, 2, 32, NULL, 64, NULL, 2, NULL, 1, NULL) == N.LP_ERR_SHAPE


def test_ggml_shape_rules():
    L = N.lib()
    # x.len must be blocksPerRow * 32
    assert L.lp_dequant_gemv_q4_0(NULL, 4, 4, NULL, 100, NULL, 1, NULL) == N.LP_ERR_SHAPE
    # w.len must be m * blocksPerRow
    assert L.lp_dequant_gemv_q8_0q8(NULL, 5, 4, NULL, 4, NULL, 1, NULL) == N.LP_ERR_SHAPE
    # quantize: src.len == blocks.len * 32
    assert L.lp_quantize_q8_0_batch(NULL, 33, NULL, 1, NULL) == N.LP_ERR_SHAPE


def test_gemm_shape_rules():
    L = N.lib()
    # n = 0 (the reference divides by n)
    assert L.lp_dequant_gemm_q8(NULL, 0, NULL, 0, 32, NULL, 0, NULL, 0, 0, NULL, 0, NULL) == N.LP_ERR_SHAPE
    # y.len not m*n
    assert L.lp_dequant_gemm_q8(NULL, 64, NULL, 2, 32, NULL, 128, NULL, 4, 2, NULL, 3, NULL) == N.LP_ERR_SHAPE


def test_null_pointer_with_valid_shape_is_an_argument_error():
    L = N.lib()
    assert L.lp_dequant_gemv_q8(NULL, 64, NULL, 2, 32, NULL, 64, NULL, 2, NULL, 1, NULL) == N.LP_ERR_ARG


def test_python_api_maps_shape_errors_to_assertion():
    import nim_lowprec_b200 as L
    with pytest.raises(AssertionError):
        L.dequantGemvQ8(np.zeros(10, np.int8), np.zeros(2, np.float32), 32,
                        np.zeros(64, np.int8), np.zeros(2, np.float32), np.zeros(1, np.float32))


def test_python_api_rejects_wrong_dtypes_and_mixed_arrays():
    import nim_lowprec_b200 as L
    with pytest.raises(TypeError):
        L.dequantGemvQ8(np.zeros(64, np.int16), np.zeros(2, np.float32), 32,
                        np.zeros(64, np.int8), np.zeros(2, np.float32), np.zeros(1, np.float32))


def test_host_buffer_entries_check_their_arguments_before_the_device():
    """lp_copy_in and lp_host_device_pointer refuse null pointers and negative
    sizes, and an empty copy is a no-op, all without a CUDA call."""
    L = N.lib()
    out = ctypes.c_void_p()
    assert L.lp_host_device_pointer(NULL, ctypes.byref(out)) == N.LP_ERR_ARG
    assert L.lp_host_device_pointer(ctypes.c_void_p(16), NULL) == N.LP_ERR_ARG
    assert L.lp_copy_in(NULL, NULL, 0, NULL) == N.LP_OK
    assert L.lp_copy_in(NULL, ctypes.c_void_p(16), 64, NULL) == N.LP_ERR_ARG
    assert L.lp_copy_in(ctypes.c_void_p(16), NULL, 64, NULL) == N.LP_ERR_ARG
    assert L.lp_copy_in(ctypes.c_void_p(16), ctypes.c_void_p(16), -1, NULL) == N.LP_ERR_ARG
    with pytest.raises(N.NativeError):
        N.host_device_pointer(0)


def test_dequantize_batch_shape_rules():
    """dequantizeBatch asserts q.len == dst.len; scales and zero points must
    cover every group."""
    L = N.lib()
    assert L.lp_dequantize_batch(NULL, 64, NULL, 2, NULL, 0, 32, NULL, 63, NULL) == N.LP_ERR_SHAPE
    assert L.lp_dequantize_batch(NULL, 64, NULL, 1, NULL, 0, 32, NULL, 64, NULL) == N.LP_ERR_SHAPE
    assert L.lp_dequantize_batch(NULL, 64, NULL, 2, NULL, 1, 32, NULL, 64, NULL) == N.LP_ERR_SHAPE
    assert L.lp_dequantize_batch(NULL, 0, NULL, 0, NULL, 0, 32, NULL, 0, NULL) == N.LP_OK


def test_quantize_dequant_gemv_shape_rules():
    """The fused quantizeQ8_0 + GEMV entries need Q8_0-sized groups (32),
    whole blocks of x, and the weight/scale lengths of the GEMV they fuse."""
    L = N.lib()
    for fn, rb in ((L.lp_quantize_dequant_gemv_q8, 64), (L.lp_quantize_dequant_gemv_i4q8, 32)):
        assert fn(NULL, 2 * rb, NULL, 4, 64, NULL, 64, NULL, 2, NULL) == N.LP_ERR_SHAPE   # gs 64
        assert fn(NULL, 2 * rb, NULL, 4, 32, NULL, 48, NULL, 2, NULL) == N.LP_ERR_SHAPE   # x 48
        assert fn(NULL, 2 * rb - 1, NULL, 4, 32, NULL, 64, NULL, 2, NULL) == N.LP_ERR_SHAPE
        assert fn(NULL, 2 * rb, NULL, 3, 32, NULL, 64, NULL, 2, NULL) == N.LP_ERR_SHAPE
        assert fn(NULL, 2 * rb, NULL, 4, 32, NULL, 64, NULL, 2, NULL) == N.LP_ERR_ARG     # nulls


def test_nim_shim_binds_only_exported_symbols():
    """Every C symbol the Nim shim imports (importc, dynlib) is exported by the
    library with the header's name -- the shim cannot be compiled here."""
    import os
    import re
    shim = os.path.join(os.path.dirname(N.LIB_PATH), "nim", "nim_lowprec_cuda.nim")
    src = open(shim).read()
    names = re.findall(r"^proc\s+(lph?_\w+)\s*\(", src, flags=re.M)
    assert len(names) >= 15
    L = N.lib()
    header = open(N.HEADER).read()
    for name in names:
        assert hasattr(L, name), name
        assert re.search(r"\b" + name + r"\s*\(", header), name


def test_local_pool_handles_without_a_gpu():
    """initPool / shutdown / threadCount (parallel.nim:134-171) at the C ABI:
    shutdown of a null pool is a no-op (idempotent), threadCount of it is 0,
    and without a GPU initPool reports LP_ERR_NO_DEVICE instead of failing
    later.  The per-call forms check shapes before looking for a device."""
    import ctypes
    import torch
    lib = N.lib()
    h = ctypes.c_void_p()
    assert lib.lph_pool_shutdown(ctypes.byref(h)) == N.LP_OK
    assert lib.lph_pool_shutdown(None) == N.LP_OK
    assert lib.lph_pool_thread_count(None) == 0
    y = (ctypes.c_float * 3)()
    x = (ctypes.c_float * 64)()
    w = (ctypes.c_int8 * (3 * 64))()
    s = (ctypes.c_float * 6)()
    # 3 rows of 64 int8 weights need 3 * 2 scales at group 32: 5 is a shape error
    assert lib.lph_par_dequant_gemv(w, 3 * 64, s, 5, 32, x, 64, y, 3, 0) == N.LP_ERR_SHAPE
    if not torch.cuda.is_available():
        assert lib.lph_pool_init(ctypes.byref(h), 2) == N.LP_ERR_NO_DEVICE
        assert lib.lph_par_dequant_gemv(w, 3 * 64, s, 6, 32, x, 64, y, 3, 0) == N.LP_ERR_NO_DEVICE


def test_batch_bracket_without_queued_calls():
    """lp_batch_begin / lp_batch_end with nothing queued launch nothing (no
    device needed); a nested begin ends the open batch; argument errors of a
    call made inside a batch return at once, as outside one."""
    L = N.lib()
    assert L.lp_batch_begin(NULL) == N.LP_OK
    assert L.lp_batch_begin(NULL) == N.LP_OK      # ends the open one
    assert L.lp_quantize_dequant_gemv_i4q8(NULL, 63, NULL, 4, 32, NULL, 64, NULL, 2,
                                           NULL) == N.LP_ERR_SHAPE
    assert L.lp_batch_end(NULL) == N.LP_OK
    assert L.lp_batch_end(NULL) == N.LP_OK        # no open batch: nothing to do
