"""The default (block-float) fp32-activation GEMVs against the CPU oracle.

The fast path represents each activation group as 22-bit block-float
integers and computes exact integer group dots, so it is not bit-identical to
the reference's sequential fp32 order; the north-star bound is 1e-5 relative
to the fp32 reference.  Checked here, per output row r:

  |y_r - ref_r| <= 1e-6 * sum_k |w_rk x_k|      (condition-aware, 10x margin)
  max_r |y_r - ref_r| <= 1e-5 * max_r |ref_r|   (the stated tolerance, M >= 64)

with ref the oracle (the reference's scalar order).  Non-finite activations
must give the same inf/NaN pattern as the reference; group sizes that are not
multiples of 8 fall back to the exact kernels and must match bit for bit.
"""
import numpy as np
import pytest

from gpu_util import F, acts, bits_equal, mismatch_report, to_dev, to_host, weights
from numpy_refs import LUT2X, _unpack_nibbles
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402

REL_ROW = 1e-6
REL_NORM = 1e-5


@pytest.fixture(autouse=True)
def _fast_mode_and_no_device_error():
    with L.fp32_mode("fast"):
        yield
    assert N.device_error() == 0


def dev_y(m):
    return torch.full((m,), float("nan"), dtype=torch.float32, device="cuda")


# ---- dequantized weight values (fp64) for the |w| |x| error scale ----

def vals_i8(q8, s, gs, k):
    m = q8.size // k
    return q8.reshape(m, k).astype(np.float64) * np.repeat(s.reshape(m, k // gs), gs, 1)


def vals_i4(p4, s, gs, k):
    m = p4.size // (k // 2)
    n = _unpack_nibbles(p4, m, k).astype(np.int16)
    v = np.where(n >= 8, n - 16, n).astype(np.float64)
    return v * np.repeat(s.reshape(m, k // gs), gs, 1)


def vals_f4(pf, s, gs, k):
    m = pf.size // (k // 2)
    v = LUT2X[_unpack_nibbles(pf, m, k)].astype(np.float64) * 0.5
    return v * np.repeat(s.reshape(m, k // gs), gs, 1)


def vals_blocks(blk, k, q4):
    deq = (O.dequantizeQ4_0 if q4 else O.dequantizeQ8_0)(blk)
    return deq.reshape(-1, k).astype(np.float64)


def assert_close(y, ref, wvals, x):
    y = np.asarray(y, np.float64)
    ref = np.asarray(ref, np.float64)
    # rows the reference overflows (or NaNs) must come out the same
    assert np.array_equal(np.isnan(y), np.isnan(ref))
    inf = np.isinf(ref)
    assert np.array_equal(y[inf], ref[inf])
    fin = np.isfinite(ref)
    y, ref, wvals = y[fin], ref[fin], wvals[fin]
    absdot = np.abs(wvals) @ np.abs(x.astype(np.float64))
    err = np.abs(y - ref)
    bad = np.nonzero(err > REL_ROW * absdot + 1e-37)[0]
    assert bad.size == 0, (f"{bad.size} rows off; first {bad[:5].tolist()}: got {y[bad[:5]]} "
                           f"want {ref[bad[:5]]} scale {absdot[bad[:5]]}")
    if y.size >= 64:  # a vector norm; one or two rows only measure the reference's own rounding
        assert err.max(initial=0.0) <= REL_NORM * max(np.abs(ref).max(initial=0.0), 1e-30)


def run_group_formats(M, K, gs, x, seed):
    """I8 / I4 / F4 with fp32 scales: kernel vs oracle, fast tolerance."""
    w = weights(seed, M * K)
    (xd,) = to_dev(x)
    y = dev_y(M)
    out = []
    s8 = O.calibrateSymmetric(w, gs, 127.0)
    q8 = O.quantize(w, s8, gs, "i8")
    a, b = to_dev(q8, s8)
    L.dequantGemv(a, b, gs, xd, y)
    out.append((to_host(y).copy(), O.dequantGemv(q8, s8, gs, x), vals_i8(q8, s8, gs, K)))
    s4 = O.calibrateSymmetric(w, gs, 7.0)
    p4 = O.packInt4(O.quantize(w, s4, gs, "i4"))
    a, b = to_dev(p4, s4)
    L.dequantGemvI4(a, b, gs, xd, y)
    out.append((to_host(y).copy(), O.dequantGemvI4(p4, s4, gs, x), vals_i4(p4, s4, gs, K)))
    sm = O.calibrateMX(w, gs, 2)
    pf = O.packF4(O.quantize(w, sm, gs, "f4"))
    a, b = to_dev(pf, sm)
    L.dequantGemvF4(a, b, gs, xd, y)
    out.append((to_host(y).copy(), O.dequantGemvF4(pf, sm, gs, x), vals_f4(pf, sm, gs, K)))
    return out


def run_block_formats(M, K, x, seed):
    w = weights(seed, M * K)
    (xd,) = to_dev(x)
    y = dev_y(M)
    out = []
    for q4, enc, fn, ofn in ((False, O.quantizeQ8_0, L.dequantGemvQ8_0, O.dequantGemvQ8_0),
                             (True, O.quantizeQ4_0, L.dequantGemvQ4_0, O.dequantGemvQ4_0)):
        blk = enc(w).reshape(-1)
        (bd,) = to_dev(blk)
        fn(bd, K // 32, xd, y)
        out.append((to_host(y).copy(), ofn(blk, K // 32, x), vals_blocks(blk, K, q4)))
    return out


@pytest.mark.parametrize("M,K", [(1, 64), (7, 96), (5, 384), (37, 4096), (300, 512),
                                 (1024, 4096), (2960, 4096), (333, 11008)])
def test_fast_fp32_within_tolerance(M, K):
    x = acts(3 + M, K)
    for y, ref, wv in run_group_formats(M, K, 32, x, 3 + M) + run_block_formats(M, K, x, 3 + M):
        assert_close(y, ref, wv, x)


@pytest.mark.parametrize("gs", [8, 16, 40, 48, 64, 96, 128, 256])
def test_fast_fp32_group_sizes(gs):
    M, K = 29, gs * 8
    x = acts(gs, K)
    for y, ref, wv in run_group_formats(M, K, gs, x, gs):
        assert_close(y, ref, wv, x)


@pytest.mark.parametrize("gs", [20, 36, 100])
def test_group_sizes_off_the_8_grid_take_the_exact_kernels(gs):
    M, K = 17, gs * 4
    x = acts(gs, K)
    for y, ref, _ in run_group_formats(M, K, gs, x, gs):
        assert bits_equal(y, ref), mismatch_report(y, ref)


def test_fast_fp32_wide_dynamic_range():
    """Groups of tiny, huge, subnormal and mixed-magnitude activations."""
    M, K = 64, 1024
    rng = np.random.default_rng(9)
    x = acts(9, K)
    x[0:32] *= F(1e-30)
    x[32:64] *= F(1e30)
    x[64:96] = (rng.standard_normal(32) * 1e-40).astype(F)   # subnormal
    x[96:128] = 0.0
    x[128:160] *= np.where(np.arange(32) % 2 == 0, F(1e20), F(1e-20)).astype(F)
    x[160] = F(3.4e38)
    for y, ref, wv in run_group_formats(M, K, 32, x, 9) + run_block_formats(M, K, x, 9):
        assert_close(y, ref, wv, x)


def test_fast_fp32_non_finite_activations_match_reference_pattern():
    M, K = 40, 512
    x = acts(11, K)
    x[5] = np.inf
    x[100] = -np.inf
    x[300] = np.nan
    for y, ref, _ in run_group_formats(M, K, 32, x, 11) + run_block_formats(M, K, x, 11):
        assert np.array_equal(np.isnan(y), np.isnan(ref))
        fin = np.isfinite(ref)
        assert np.array_equal(y[~fin & ~np.isnan(ref)], ref[~fin & ~np.isnan(ref)])
    # one non-finite group among finite ones: the other rows stay close
    x2 = acts(12, K)
    x2[33] = np.inf
    for y, ref, _ in run_group_formats(M, K, 32, x2, 12):
        assert np.array_equal(np.isinf(y), np.isinf(ref))


def test_fast_fp32_zero_activations_give_zero():
    M, K = 16, 256
    x = np.zeros(K, F)
    for y, ref, _ in run_group_formats(M, K, 32, x, 13) + run_block_formats(M, K, x, 13):
        assert np.all(y == 0.0) and np.all(ref == 0.0)


def test_fast_fp32_config1_and_config2_full():
    M, K = 11008, 4096
    x = acts(1, K)
    (y, ref, wv), = run_block_formats(M, K, x, 1)[1:]
    assert_close(y, ref, wv, x)
    M, K = 14336, 4096
    x = acts(2, K)
    w = weights(2, M * K)
    sm = O.calibrateMX(w, 32, 2)
    pf = O.packF4(O.quantize(w, sm, 32, "f4"))
    a, b, xd = to_dev(pf, sm, x)
    y = dev_y(M)
    L.dequantGemvF4(a, b, 32, xd, y)
    assert_close(to_host(y), O.dequantGemvF4(pf, sm, 32, x), vals_f4(pf, sm, 32, K), x)


def test_mode_switch_and_host_forms():
    assert L.fp32Mode() == "fast"
    with L.fp32_mode("exact"):
        assert L.fp32Mode() == "exact"
    assert L.fp32Mode() == "fast"
    with pytest.raises(ValueError):
        L.setFp32Mode("approximate")
    # host (numpy) form runs the same kernels
    M, K = 50, 256
    x = acts(14, K)
    w = weights(14, M * K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    y = np.zeros(M, F)
    L.dequantGemvQ4_0(blk, K // 32, x, y)
    assert_close(y, O.dequantGemvQ4_0(blk, K // 32, x), vals_blocks(blk, K, True), x)


@pytest.mark.parametrize("M,K", [(8, 256), (149, 1024), (1500, 2048), (18944, 256),
                                 (20000, 4096)])
def test_fast_q4_0_row_tile_shapes(M, K):
    """Row counts from a few rows per CTA to full tiles with a ragged last
    tile, and 8..128 blocks per row; results are identical run to run."""
    x = acts(40 + M, K)
    w = weights(40 + M, M * K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    bd, xd = to_dev(blk, x)
    y = dev_y(M)
    L.dequantGemvQ4_0(bd, K // 32, xd, y)
    first = to_host(y).copy()
    assert_close(first, O.dequantGemvQ4_0(blk, K // 32, x), vals_blocks(blk, K, True), x)
    L.dequantGemvQ4_0(bd, K // 32, xd, y)
    assert bits_equal(to_host(y), first)  # run to run identical


def test_fast_q4_0_several_sequential_groups_in_a_row():
    """Finite groups at or above 2^100 take the sequential path; several of
    them in one row, spread over the row's K-chunks, add up deterministically."""
    M, K = 300, 4096
    x = acts(15, K)
    for j in (1, 9, 10, 63, 64, 127):
        x[32 * j + 3] = F(3e30 * (1 if j % 2 else -1))
    w = weights(15, M * K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    bd, xd = to_dev(blk, x)
    y = dev_y(M)
    L.dequantGemvQ4_0(bd, K // 32, xd, y)
    first = to_host(y).copy()
    assert_close(first, O.dequantGemvQ4_0(blk, K // 32, x), vals_blocks(blk, K, True), x)
    L.dequantGemvQ4_0(bd, K // 32, xd, y)
    assert bits_equal(to_host(y), first)


@pytest.mark.parametrize("xoff,woff", [(1, 0), (0, 2), (3, 18)])
def test_fast_q4_0_unaligned_pointers(xoff, woff):
    """Activations off the 16-byte grid (staged with scalar loads) and block
    arrays only 2-byte aligned (the reference's blocks need no more; their
    rows are staged with plain loads instead of bulk copies) stay within the
    fast-mode tolerance."""
    M, K = 333, 4096
    x = acts(70 + xoff, K)
    w = weights(70 + woff, M * K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    xb = torch.zeros(K + xoff, dtype=torch.float32, device="cuda")
    xb[xoff:] = torch.from_numpy(x).cuda()
    bb = torch.zeros(blk.size + woff, dtype=torch.uint8, device="cuda")
    bb[woff:] = torch.from_numpy(blk).cuda()
    y = dev_y(M)
    L.dequantGemvQ4_0(bb[woff:], K // 32, xb[xoff:], y)
    assert_close(to_host(y), O.dequantGemvQ4_0(blk, K // 32, x), vals_blocks(blk, K, True), x)


def test_fast_fp32_long_rows_fit_two_stages():
    """K = 14336: the longest tiles the tile cap allows leave shared memory
    for fewer than two weight stages next to the staged activations and the
    term ring, so the planner shortens them; Q4_0 and MXFP4 rows of that
    length still run and stay within tolerance."""
    M, K = 300, 14336
    x = acts(80, K)
    (y, ref, wv), = run_block_formats(M, K, x, 80)[1:]
    assert_close(y, ref, wv, x)
    w = weights(81, M * K)
    sm = O.calibrateMX(w, 32, 2)
    pf = O.packF4(O.quantize(w, sm, 32, "f4"))
    a, b, xd = to_dev(pf, sm, x)
    yd = dev_y(M)
    L.dequantGemvF4(a, b, 32, xd, yd)
    assert_close(to_host(yd), O.dequantGemvF4(pf, sm, 32, x), vals_f4(pf, sm, 32, K), x)
