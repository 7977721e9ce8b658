"""lph_dequant_gemv_q4_0_static: the host form of dequantGemvQ4_0 that stages
through a static device array instead of allocating.  It must give the bits of
the existing host form, call after call, and reject calls larger than its
array.  (This file is collected last, so it also runs after every other GPU
test in the same process.)"""
import ctypes

import numpy as np
import pytest

from gpu_util import F, acts, bits_equal, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402


def static_form(blk, bpr, x, y):
    return N.lib().lph_dequant_gemv_q4_0_static(
        blk.ctypes.data_as(ctypes.c_void_p), blk.size // 18, bpr,
        x.ctypes.data_as(ctypes.c_void_p), x.size, y.ctypes.data_as(ctypes.c_void_p), y.size)


@pytest.mark.parametrize("M,K", [(11008, 4096), (37, 512)])
def test_static_stage_matches_the_host_form_twice(M, K):
    blk = O.quantizeQ4_0(weights(70, M * K)).reshape(-1)
    for call in range(2):  # two calls in a row, different activations
        x = acts(71 + call, K)
        want = np.zeros(M, F)
        L.dequantGemvQ4_0(blk, K // 32, x, want)
        got = np.full(M, np.nan, F)
        assert static_form(blk, K // 32, x, got) == N.LP_OK
        assert bits_equal(got, want)
    assert N.device_error() == 0


@pytest.mark.parametrize("mode", ["exact", "fast"])
def test_static_stage_matches_the_oracle(mode):
    """The same calls checked against the CPU oracle of the reference's
    dequantGemvQ4_0: bit for bit in the exact fp32 mode, and in the fast mode
    within 1e-6 of sum|w||x| per row (the bound of the fast-mode tests)."""
    M, K = 37, 512
    blk = O.quantizeQ4_0(weights(72, M * K)).reshape(-1)
    absw = np.abs(O.dequantizeQ4_0(blk).reshape(M, K).astype(np.float64))
    with L.fp32_mode(mode):
        for call in range(2):
            x = acts(73 + call, K)
            want = O.dequantGemvQ4_0(blk, K // 32, x)
            got = np.full(M, np.nan, F)
            assert static_form(blk, K // 32, x, got) == N.LP_OK
            if mode == "exact":
                assert bits_equal(got, want)
            else:
                bound = 1e-6 * (absw @ np.abs(x.astype(np.float64)))
                assert np.all(np.abs(got.astype(np.float64) - want) <= bound)
    assert N.device_error() == 0


def test_static_stage_rejects_calls_beyond_its_array():
    M, K = 16384, 4096  # 37.7 MB of blocks > 32 MiB
    blk = np.zeros(M * (K // 32) * 18, np.uint8)
    x = np.zeros(K, F)
    y = np.zeros(M, F)
    assert static_form(blk, K // 32, x, y) == N.LP_ERR_UNSUPPORTED


def test_static_stage_reports_shape_errors():
    blk = np.zeros(10 * 18, np.uint8)
    x = np.zeros(64, F)
    y = np.zeros(3, F)  # 10 blocks are not 3 rows of 2 blocks
    assert static_form(blk, 2, x, y) == N.LP_ERR_SHAPE
    # a bad shape beyond the array's size is a shape error, found before any copy
    big = np.zeros(40 << 20, np.uint8)
    assert static_form(big, 2, x, y) == N.LP_ERR_SHAPE
