"""CUDA kernels vs the CPU oracle, through the C ABI (device and host forms).

Bit-exact for every path (integer, encoder and fp32-activation GEMVs alike:
every test here runs the fp32 kernels in their exact mode, which reproduces
the reference's scalar summation order), on
  * the reference tests' own inputs (test_sdot.nim, test_parallel.nim,
    test_quant_simd.nim, test_scheme_conformance.nim goldens),
  * edge shapes (M = 1, odd M, block tails bpr = 3 mod 4, group tails),
  * the BASELINE configurations at full size (configs 0-2 and the GEMM).
"""
import os

import numpy as np
import pytest

import refcases as C
from gpu_util import F, acts, bits_equal, mismatch_report, to_dev, to_host, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def dev_y(m):
    return torch.full((m,), float("nan"), dtype=torch.float32, device="cuda")


def assert_bits(got, want):
    assert bits_equal(got, want), mismatch_report(got, want)


@pytest.fixture(autouse=True)
def _exact_fp32_and_no_device_error():
    with L.fp32_mode("exact"):
        yield
    assert N.device_error() == 0


# ------------------------------------------------------------ encoders --

def test_quantize_q8_0_matches_gguf_golden():
    x = np.fromfile(os.path.join(G, "ref_scheme_input.bin"), np.float32)
    want = np.fromfile(os.path.join(G, "ref_ggml_q8_0_bytes.bin"), np.uint8)
    (xd,) = to_dev(x)
    blocks = torch.empty(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    L.quantizeQ8_0Batch(xd, blocks)
    assert np.array_equal(to_host(blocks), want)


def test_quantize_q4_0_matches_gguf_golden():
    x = np.fromfile(os.path.join(G, "ref_scheme_input.bin"), np.float32)
    want = np.fromfile(os.path.join(G, "ref_ggml_q4_0_bytes.bin"), np.uint8)
    (xd,) = to_dev(x)
    blocks = torch.empty(x.size // 32 * 18, dtype=torch.uint8, device="cuda")
    L.quantizeQ4_0Batch(xd, blocks)
    assert np.array_equal(to_host(blocks), want)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_dequantize_blocks_match_gguf_golden(fmt):
    raw = np.fromfile(os.path.join(G, f"ref_ggml_{fmt}_bytes.bin"), np.uint8)
    want = np.fromfile(os.path.join(G, f"ref_ggml_{fmt}_dq.bin"), np.uint32)
    (rd,) = to_dev(raw)
    out = torch.empty(want.size, dtype=torch.float32, device="cuda")
    (L.dequantizeQ8_0Batch if fmt == "q8_0" else L.dequantizeQ4_0Batch)(rd, out)
    assert np.array_equal(to_host(out).view(np.uint32), want)


@pytest.mark.parametrize("fmt", ["q4_k", "q6_k"])
def test_dequantize_kquants_match_gguf_golden_and_oracle(fmt):
    """The k-quant super-blocks: gguf-py's goldens, then 4099 random
    super-blocks (every byte random except finite f16 d / dmin) vs the oracle."""
    bb, fn, ofn = ((144, L.dequantizeQ4_K, O.dequantizeQ4_K) if fmt == "q4_k"
                   else (210, L.dequantizeQ6_K, O.dequantizeQ6_K))
    raw = np.fromfile(os.path.join(G, f"ref_ggml_{fmt}_bytes.bin"), np.uint8)
    want = np.fromfile(os.path.join(G, f"ref_ggml_{fmt}_dq.bin"), np.uint32)
    (rd,) = to_dev(raw)
    out = torch.empty(want.size, dtype=torch.float32, device="cuda")
    fn(rd, out)
    assert np.array_equal(to_host(out).view(np.uint32), want)
    rng = np.random.default_rng(17)
    nb = 4099
    blk = rng.integers(0, 256, size=(nb, bb), dtype=np.uint16).astype(np.uint8)
    dpos = [0, 2] if fmt == "q4_k" else [208]
    for p_ in dpos:
        blk[:, p_:p_ + 2] = (rng.standard_normal(nb) * 0.1).astype(np.float16).view(np.uint8).reshape(nb, 2)
    raw = blk.reshape(-1)
    (rd,) = to_dev(raw)
    out = torch.empty(nb * 256, dtype=torch.float32, device="cuda")
    fn(rd, out)
    want = ofn(raw)
    assert bits_equal(to_host(out), want)
    # unaligned blocks and output (element-wise loads and stores)
    rd2 = torch.zeros(raw.size + 1, dtype=torch.uint8, device="cuda")
    rd2[1:].copy_(rd)
    out2 = torch.full((nb * 256 + 1,), float("nan"), dtype=torch.float32, device="cuda")
    fn(rd2[1:], out2[1:])
    assert bits_equal(to_host(out2[1:]), want)


def _nvfp4_on_device(x):
    (xd,) = to_dev(x)
    codes = torch.empty(x.size, dtype=torch.uint8, device="cuda")
    scales = torch.empty(x.size // 16, dtype=torch.uint8, device="cuda")
    gds = torch.empty(1, dtype=torch.float32, device="cuda")
    L.quantizeNVFP4(xd, codes, scales, gds)
    return codes, scales, gds


def test_nvfp4_matches_the_te_golden_and_oracle():
    """quantizeNVFP4 / dequantizeNVFP4 (nvfp4.nim:39-92) on the device: the TE
    golden, then random tensors with zero, huge-range, inf and NaN entries vs
    the oracle."""
    x = np.fromfile(os.path.join(G, "ref_nvfp4_input.bin"), np.float32)
    raw = np.fromfile(os.path.join(G, "ref_nvfp4_out.bin"), np.uint8)
    nb = x.size // 16
    codes, scales, gds = _nvfp4_on_device(x)
    assert to_host(gds)[0] == raw[:4].view("<f4")[0]
    assert np.array_equal(to_host(scales), raw[4:4 + nb])
    assert np.array_equal(to_host(codes), raw[4 + nb:])
    rng = np.random.default_rng(23)
    for case in range(4):
        x = (rng.standard_normal(16 * 4099) * 3).astype(F)
        x = (x.reshape(-1, 16) * (F(2.0) ** rng.integers(-30, 30, size=(4099, 1)).astype(F))).reshape(-1)
        if case >= 1:
            x[16 * 3:16 * 4] = 0.0
            x[100] = -0.0
        if case >= 2:
            x[5000] = np.nan
        if case == 3:
            x[777] = np.inf
        codes, scales, gds = _nvfp4_on_device(x)
        oc, os_, og = O.quantizeNVFP4(x)
        assert bits_equal(to_host(gds), np.array([og], F))
        assert np.array_equal(to_host(scales), os_)
        assert np.array_equal(to_host(codes), oc)
        out = torch.empty(x.size, dtype=torch.float32, device="cuda")
        L.dequantizeNVFP4(codes, scales, float(og), out)
        assert bits_equal(to_host(out), O.dequantizeNVFP4(oc, os_, og))


def test_quantize_q8_0_random_and_edges_vs_oracle():
    rng = np.random.default_rng(3)
    x = (rng.standard_normal(32 * 4099) * 3).astype(F)
    x[32 * 5:32 * 6] = 0.0                # all-zero block: d = 0 path
    x[32 * 7:32 * 8] = np.float32(1e-30)  # tiny block, d underflows fp16
    x[32 * 9 + 3] = np.float32(-7.0)      # ties and sign
    (xd,) = to_dev(x)
    blocks = torch.empty(x.size // 32 * 34, dtype=torch.uint8, device="cuda")
    L.quantizeQ8_0Batch(xd, blocks)
    assert np.array_equal(to_host(blocks), O.quantizeQ8_0(x).reshape(-1))
    qs = torch.empty(x.size, dtype=torch.int8, device="cuda")
    d = torch.empty(x.size // 32, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(xd, qs, d)
    oq, od = O.quantizeQ8_0Split(x)
    assert np.array_equal(to_host(qs), oq) and bits_equal(to_host(d), od)


def test_quantize_q4_0_sign_keeping_max_ties():
    x = np.zeros(32 * 3, F)
    x[3], x[10] = -2.0, 2.0      # equal magnitude: the first (negative) wins
    x[32 + 1], x[32 + 5] = 1.5, -1.5
    x[64:96] = np.linspace(-1, 1, 32, dtype=F)
    (xd,) = to_dev(x)
    blocks = torch.empty(3 * 18, dtype=torch.uint8, device="cuda")
    L.quantizeQ4_0Batch(xd, blocks)
    assert np.array_equal(to_host(blocks), O.quantizeQ4_0(x).reshape(-1))


@pytest.mark.parametrize("gs", [4, 8, 16, 32, 64, 128])
@pytest.mark.parametrize("n", [4096 * 37, 4100, 4])
def test_calibrate_vector_path_vs_oracle(n, gs):
    """The float4 form of calibrateSymmetric / calibrateMX (16-byte aligned x,
    n % 4 == 0, gs / 4 a power of two <= 32): every group size it takes, a
    ragged last group, all-zero groups, a NaN (dropped by the max, as by the
    reference's scan) and an infinity."""
    x = acts(77 + gs, n) * F(3.0)
    x[: min(n, gs)] = 0.0                      # an all-zero group
    if n > 3 * gs:
        x[2 * gs + 1] = np.float32("nan")
        x[3 * gs] = np.float32("inf")
    (xd,) = to_dev(x)
    for qmax in (127.0, 7.0):
        sc_o = O.calibrateSymmetric(x, gs, qmax)
        sc = torch.empty(sc_o.size, dtype=torch.float32, device="cuda")
        L.calibrateSymmetric(xd, gs, qmax, sc)
        assert_bits(to_host(sc), sc_o)
    mx_o = O.calibrateMX(x, gs, 2)
    mx = torch.empty(mx_o.size, dtype=torch.float32, device="cuda")
    L.calibrateMX(xd, gs, 2, mx)
    assert_bits(to_host(mx), mx_o)


@pytest.mark.parametrize("n,gs", [(4096, 128), (4099, 64), (1000, 0), (4096, 32)])
def test_quantize_batch_and_calibrate_vs_oracle(n, gs):
    """test_quant_simd.nim:330-355 shapes (per-group, ragged, per-tensor)."""
    u = 55555
    x = np.empty(n, F)
    for i in range(n):
        u = (u * 1664525 + 1013904223) & 0xFFFFFFFF
        x[i] = (F(u >> 8) / F(1 << 24) - F(0.5)) * F(30.0)
    sc_o = O.calibrateSymmetric(x, gs, 127.0)
    (xd,) = to_dev(x)
    sc = torch.empty(sc_o.size, dtype=torch.float32, device="cuda")
    L.calibrateSymmetric(xd, gs, 127.0, sc)
    assert bits_equal(to_host(sc), sc_o)
    q = torch.empty(n, dtype=torch.int8, device="cuda")
    L.quantizeBatch(xd, sc, gs, q)
    assert np.array_equal(to_host(q), O.quantizeBatch(x, sc_o, gs))
    # host drop-in form of the same entry point
    qh = np.empty(n, np.int8)
    L.quantizeBatch(x, sc_o, gs, qh)
    assert np.array_equal(qh, O.quantizeBatch(x, sc_o, gs))
    # QParams with zero points: the reference's scalar quantize fall-through,
    # toI8(x / scale + zeroPoint), clamped (quant.nim:48-60)
    zp = ((np.arange(sc_o.size, dtype=F) % 7) * F(9.5) - F(30.0)).astype(F)
    want = O.quantizeBatch(x, sc_o, gs, zp)
    assert want.min() == -128 or want.max() == 127  # a clamp is reached
    (zd,) = to_dev(zp)
    L.quantizeBatch(xd, sc, gs, q, zd)
    assert np.array_equal(to_host(q), want)
    L.quantizeBatch(x, sc_o, gs, qh, zp)
    assert np.array_equal(qh, want)


@pytest.mark.parametrize("n,gs,asym,off", [
    (1000, 0, False, 0), (1000, 64, False, 0), (512, 32, False, 0),  # test_quant_simd.nim:33-64
    (4_000_003, 128, False, 0), (4_000_003, 128, True, 0), (16_000_000, 128, False, 0),
    (333, 7, True, 0), (97, 1, False, 0), (1001, 64, True, 3), (1001, 24, False, 1), (0, 32, False, 0)])
def test_dequantize_batch_vs_oracle(n, gs, asym, off):
    """dequantizeBatch (simd/dequant.nim:159-206): device and host forms equal
    the oracle bit for bit -- symmetric and zero-point, per tensor and per
    group (groups shorter than a thread's 16-value run included), ragged
    tails, and pointers off the 16-byte vector alignment."""
    rng = np.random.default_rng(n + gs)
    q = rng.integers(-128, 128, n, dtype=np.int8)
    ng = (n + gs - 1) // gs if gs > 0 else 1
    sc = (rng.random(ng, dtype=np.float32) * F(0.1) + F(1e-3)).astype(F)
    sc[::5] = -sc[::5]
    zp = (rng.random(ng, dtype=np.float32) * F(40.0) - F(20.0)).astype(F) if asym else None
    want = O.dequantizeBatch(q, sc, gs, zp)
    qb = torch.zeros(n + off, dtype=torch.int8, device="cuda")
    qb[off:] = torch.from_numpy(q).cuda()
    out = torch.full((n + off,), float("nan"), dtype=torch.float32, device="cuda")
    sc_d = to_dev(sc)[0]
    zp_d = to_dev(zp)[0] if asym else None
    L.dequantizeBatch(qb[off:], sc_d, gs, out[off:], zp_d)
    assert_bits(to_host(out[off:]), want)
    if n <= 5000:
        host = np.full(n, np.nan, F)
        L.dequantizeBatch(q, sc, gs, host, zp)
        assert_bits(host, want)


def test_dequantize_batch_rejects_short_scales():
    q = torch.zeros(100, dtype=torch.int8, device="cuda")
    y = torch.empty(100, dtype=torch.float32, device="cuda")
    sc = torch.ones(3, dtype=torch.float32, device="cuda")  # 4 groups of 32 needed
    # shape preconditions raise AssertionError, as the reference's asserts do
    with pytest.raises(AssertionError):
        L.dequantizeBatch(q, sc, 32, y)
    with pytest.raises(AssertionError):
        L.dequantizeBatch(q, torch.ones(4, dtype=torch.float32, device="cuda"), 32, y, sc)


def test_calibrate_mx_and_f4_pack_vs_golden_input():
    x = np.fromfile(os.path.join(G, "ref_mx_input.bin"), np.float32)
    sc_o = O.calibrateMX(x, 32, 2)
    (xd,) = to_dev(x)
    sc = torch.empty(sc_o.size, dtype=torch.float32, device="cuda")
    L.calibrateMX(xd, 32, 2, sc)
    assert bits_equal(to_host(sc), sc_o)
    pk = torch.empty(x.size // 2, dtype=torch.uint8, device="cuda")
    L.quantizeF4Packed(xd, sc, 32, pk)
    assert np.array_equal(to_host(pk), O.packF4(O.quantize(x, sc_o, 32, "f4")))


def test_i4_weight_prep_vs_oracle():
    w = weights(11, 4096 * 8)
    sc_o = O.calibrateSymmetric(w, 32, 7.0)
    (wd,) = to_dev(w)
    sc = torch.empty(sc_o.size, dtype=torch.float32, device="cuda")
    L.calibrateSymmetric(wd, 32, 7.0, sc)
    assert bits_equal(to_host(sc), sc_o)
    pk = torch.empty(w.size // 2, dtype=torch.uint8, device="cuda")
    L.quantizeI4Packed(wd, sc, 32, pk)
    assert np.array_equal(to_host(pk), O.packInt4(O.quantize(w, sc_o, 32, "i4")))


# ------------------------------------------- int8-activation GEMVs ------

@pytest.mark.parametrize("M,K,gs", C.SDOT_INT8_SHAPES)
def test_gemv_q8_sdot_cases(M, K, gs):
    wq, ws, xq, xs = C.sdot_int8_case(M, K, gs)
    want = O.dequantGemvQ8(wq, ws, gs, xq, xs)
    d = to_dev(wq, ws, xq, xs)
    y = dev_y(M)
    L.dequantGemvQ8(*d[:2], gs, *d[2:], y)
    assert_bits(to_host(y), want)
    yh = np.empty(M, F)
    L.dequantGemvQ8(wq, ws, gs, xq, xs, yh)   # host drop-in
    assert_bits(yh, want)


@pytest.mark.parametrize("M,K,gs", C.SDOT_INT4_SHAPES)
def test_gemv_i4q8_sdot_cases(M, K, gs):
    vals, ws, xq, xs = C.sdot_int4_case(M, K, gs)
    wp = C.pack_i4_values(vals)
    want = O.dequantGemvI4Q8(wp, ws, gs, xq, xs)
    d = to_dev(wp, ws, xq, xs)
    y = dev_y(M)
    L.dequantGemvI4Q8(*d[:2], gs, *d[2:], y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("M,bpr", C.GGML_SHAPES)
def test_gemv_ggml_q8_sdot_cases(M, bpr):
    w8, w4, x = C.ggml_q8_w_blocks(M, bpr), C.ggml_q4_w_blocks(M, bpr), C.ggml_x_blocks(bpr)
    for fn, ofn, w in ((L.dequantGemvQ8_0Q8, O.dequantGemvQ8_0Q8, w8),
                       (L.dequantGemvQ4_0Q8, O.dequantGemvQ4_0Q8, w4)):
        want = ofn(w, bpr, x)
        wd, xd = to_dev(w.reshape(-1), x.reshape(-1))
        y = dev_y(M)
        fn(wd, bpr, xd, y)
        assert_bits(to_host(y), want)
        yh = np.empty(M, F)
        fn(w, bpr, x, yh)
        assert_bits(yh, want)


@pytest.mark.parametrize("M", [1, 7, 300, 4096])
@pytest.mark.parametrize("K", [4096, 11008])
def test_gemv_q8_i4q8_q8_0_split_random(M, K):
    """Config 0 / config 4 arithmetic: weights and activations Q8_0-encoded
    (split form), gs 32."""
    w = weights(100 + M, M * K)
    x = acts(100 + M, K)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    d = to_dev(wq, wd, xq, xd)
    y = dev_y(M)
    L.dequantGemvQ8(*d[:2], 32, *d[2:], y)
    assert_bits(to_host(y), O.dequantGemvQ8(wq, wd, 32, xq, xd))
    # int4 weights (config 4 weight prep: symmetric qmax 7)
    s4 = O.calibrateSymmetric(w, 32, 7.0)
    wp = O.packInt4(O.quantize(w, s4, 32, "i4"))
    d4 = to_dev(wp, s4)
    L.dequantGemvI4Q8(d4[0], d4[1], 32, d[2], d[3], y)
    assert_bits(to_host(y), O.dequantGemvI4Q8(wp, s4, 32, xq, xd))


# ------------------------------------------- fp32-activation GEMVs ------

def _fp32_cases():
    # 2960 rows = 20 per CTA: several row pairs per consumer thread per tile
    return [(1, 64), (7, 96), (5, 384), (37, 4096), (300, 512), (1024, 4096), (2960, 4096)]


@pytest.mark.parametrize("M,K", _fp32_cases())
def test_fp32_gemvs_bit_exact_vs_scalar_order(M, K):
    w = weights(7 + M, M * K)
    x = acts(7 + M, K)
    y = dev_y(M)
    (xd,) = to_dev(x)
    # int8 per-group
    s8 = O.calibrateSymmetric(w, 32, 127.0)
    q8 = O.quantize(w, s8, 32, "i8")
    a, b = to_dev(q8, s8)
    L.dequantGemv(a, b, 32, xd, y)
    assert_bits(to_host(y), O.dequantGemv(q8, s8, 32, x))
    # int4 packed
    s4 = O.calibrateSymmetric(w, 32, 7.0)
    p4 = O.packInt4(O.quantize(w, s4, 32, "i4"))
    a, b = to_dev(p4, s4)
    L.dequantGemvI4(a, b, 32, xd, y)
    assert_bits(to_host(y), O.dequantGemvI4(p4, s4, 32, x))
    # MXFP4
    sm = O.calibrateMX(w, 32, 2)
    pf = O.packF4(O.quantize(w, sm, 32, "f4"))
    a, b = to_dev(pf, sm)
    L.dequantGemvF4(a, b, 32, xd, y)
    assert_bits(to_host(y), O.dequantGemvF4(pf, sm, 32, x))
    # ggml blocks
    bpr = K // 32
    for enc, fn, ofn in ((O.quantizeQ8_0, L.dequantGemvQ8_0, O.dequantGemvQ8_0),
                         (O.quantizeQ4_0, L.dequantGemvQ4_0, O.dequantGemvQ4_0)):
        blk = enc(w).reshape(-1)
        (bd,) = to_dev(blk)
        fn(bd, bpr, xd, y)
        assert_bits(to_host(y), ofn(blk, bpr, x))


@pytest.mark.parametrize("gs", [20, 40, 48, 64, 96, 128])
def test_fp32_gemvs_generic_group_sizes(gs):
    """Group tails that are not 32 (test_quant_simd.nim uses 40 and 48)."""
    M, K = 23, gs * 6
    w = weights(gs, M * K)
    x = acts(gs, K)
    (xd,) = to_dev(x)
    y = dev_y(M)
    s8 = O.calibrateSymmetric(w, gs, 127.0)
    q8 = O.quantize(w, s8, gs, "i8")
    a, b = to_dev(q8, s8)
    L.dequantGemv(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemv(q8, s8, gs, x))
    s4 = O.calibrateSymmetric(w, gs, 7.0)
    p4 = O.packInt4(O.quantize(w, s4, gs, "i4"))
    a, b = to_dev(p4, s4)
    L.dequantGemvI4(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemvI4(p4, s4, gs, x))
    sm = O.calibrateMX(w, gs, 2)
    pf = O.packF4(O.quantize(w, sm, gs, "f4"))
    a, b = to_dev(pf, sm)
    L.dequantGemvF4(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemvF4(pf, sm, gs, x))
    xs = O.calibrateSymmetric(x, gs, 127.0)
    xq = O.quantizeBatch(x, xs, gs)
    a, b, c, d = to_dev(q8, s8, xq, xs)
    L.dequantGemvQ8(a, b, gs, c, d, y)
    assert_bits(to_host(y), O.dequantGemvQ8(q8, s8, gs, xq, xs))


@pytest.mark.parametrize("M", C.PAR_ROWS)
def test_parallel_test_inputs(M):
    """The inputs of test_parallel.nim through every fp32 kernel."""
    x = C.par_x()
    (xd,) = to_dev(x)
    y = dev_y(M)
    gs = C.PAR_GS
    wq, sc = C.par_int8(M)
    a, b = to_dev(wq, sc)
    L.dequantGemv(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemv(wq, sc, gs, x))
    w4, sc4 = C.par_int4(M)
    a, b = to_dev(w4, sc4)
    L.dequantGemvI4(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemvI4(w4, sc4, gs, x))
    wf, scf = C.par_f4(M)
    a, b = to_dev(wf, scf)
    L.dequantGemvF4(a, b, gs, xd, y)
    assert_bits(to_host(y), O.dequantGemvF4(wf, scf, gs, x))
    for blocks_fn, fn, ofn in ((C.par_q8_0, L.dequantGemvQ8_0, O.dequantGemvQ8_0),
                               (C.par_q4_0, L.dequantGemvQ4_0, O.dequantGemvQ4_0)):
        blk, bpr = blocks_fn(M)
        (bd,) = to_dev(blk.reshape(-1))
        fn(bd, bpr, xd, y)
        assert_bits(to_host(y), ofn(blk, bpr, x))


# ----------------------------------------------------------------- GEMM --

@pytest.mark.parametrize("M,K,gs,n", C.GEMM_I8_SHAPES)
def test_gemm_q8_sdot_cases(M, K, gs, n):
    wq, ws, xq, xs = C.gemm_int8_case(M, K, gs, n)
    want = O.dequantGemmQ8(wq, ws, gs, xq, xs, n)
    d = to_dev(wq, ws, xq, xs)
    y = dev_y(M * n)
    L.dequantGemmQ8(*d[:2], gs, *d[2:], n, y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("M,K,gs,n", C.GEMM_I4_SHAPES)
def test_gemm_i4q8_sdot_cases(M, K, gs, n):
    wp, ws, xq, xs = C.gemm_int4_case(M, K, gs, n)
    want = O.dequantGemmI4Q8(wp, ws, gs, xq, xs, n)
    d = to_dev(wp, ws, xq, xs)
    y = dev_y(M * n)
    L.dequantGemmI4Q8(*d[:2], gs, *d[2:], n, y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("n", [8, 64])
def test_gemm_config3_full(n):
    """Config 3: Q8_0 weight 4096x4096 times n Q8_0-quantized columns."""
    M = K = 4096
    w = weights(3, M * K)
    x = acts(3, K * n)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)   # column c = x[c*K:(c+1)*K]
    pool = O.Pool(0)
    try:
        want = O.dequantGemmQ8(wq, wd, 32, xq, xd, n, pool=pool)
    finally:
        pool.shutdown()
    d = to_dev(wq, wd, xq, xd)
    y = dev_y(M * n)
    L.dequantGemmQ8(*d[:2], 32, *d[2:], n, y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("M,K,n", [(128, 128, 16), (128, 128, 8), (129, 512, 5), (300, 256, 64),
                                   (256, 512, 100), (128, 4096, 512), (1, 128, 1), (257, 384, 65)])
def test_gemm_q8_tensor_core_shapes(M, K, n):
    """32-wide groups with K a multiple of 128 run on tcgen05 (ragged M and n
    tiles included); bit-exact like every other path."""
    w = weights(M + K + n, M * K)
    x = acts(M + K + n, K * n)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    want = O.dequantGemmQ8(wq, wd, 32, xq, xd, n)
    d = to_dev(wq, wd, xq, xd)
    y = dev_y(M * n)
    L.dequantGemmQ8(*d[:2], 32, *d[2:], n, y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("M,K,n", [(128, 128, 17), (129, 512, 64), (300, 256, 64),
                                   (256, 512, 100), (128, 4096, 512), (257, 384, 65)])
def test_gemm_i4q8_tensor_core_shapes(M, K, n):
    """dequantGemmI4Q8 (simd/dequant.nim:1460-1583) past 16 columns runs on
    tcgen05 kind::i8: the packed int4 tile is widened to int8 in shared memory
    before the MMA; bit-exact like every other path."""
    w = weights(M + K + n + 1, M * K)
    x = acts(M + K + n + 1, K * n)
    ws = O.calibrateSymmetric(w, 32, 7.0)
    wp = O.packInt4(O.quantize(w, ws, 32, "i4"))
    xq, xd = O.quantizeQ8_0Split(x)
    want = O.dequantGemmI4Q8(wp, ws, 32, xq, xd, n)
    d = to_dev(wp, ws, xq, xd)
    y = dev_y(M * n)
    L.dequantGemmI4Q8(*d[:2], 32, *d[2:], n, y)
    assert_bits(to_host(y), want)


@pytest.mark.parametrize("M,K,n", [(1, 32, 1), (37, 512, 2), (300, 256, 3), (149, 4096, 7),
                                   (4100, 1024, 8), (333, 512, 9), (150, 2048, 16),
                                   (64, 512, 17), (97, 11008, 8)])
def test_gemm_few_columns_q8_and_i4q8(M, K, n):
    """Up to 16 columns with 32-wide groups run as the GEMV skeleton's column
    formats (ragged row tiles, one to sixteen columns, K = 11008 as in the
    Llama down projection); 17 columns take the wide-GEMM kernels."""
    w = weights(M + n, M * K)
    x = acts(M + n, K * n)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    d = to_dev(wq, wd, xq, xd)
    y = dev_y(M * n)
    L.dequantGemmQ8(*d[:2], 32, *d[2:], n, y)
    assert_bits(to_host(y), O.dequantGemmQ8(wq, wd, 32, xq, xd, n))
    s4 = O.calibrateSymmetric(w, 32, 7.0)
    p4 = O.packInt4(O.quantize(w, s4, 32, "i4"))
    d4 = to_dev(p4, s4)
    y4 = dev_y(M * n)
    L.dequantGemmI4Q8(*d4, 32, *d[2:], n, y4)
    assert_bits(to_host(y4), O.dequantGemmI4Q8(p4, s4, 32, xq, xd, n))


def test_gemm_column_equals_gemv_on_device():
    """test_sdot.nim:243-282 on the device: every GEMM column is the GEMV."""
    M, K, n = 129, 512, 5
    w = weights(9, M * K)
    x = acts(9, K * n)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    d = to_dev(wq, wd, xq, xd)
    y = dev_y(M * n)
    L.dequantGemmQ8(*d[:2], 32, *d[2:], n, y)
    Y = to_host(y).reshape(M, n)
    for c in range(n):
        yc = dev_y(M)
        L.dequantGemvQ8(d[0], d[1], 32, d[2][c * K:(c + 1) * K], d[3][c * 16:(c + 1) * 16], yc)
        assert_bits(Y[:, c], to_host(yc))


# ------------------------------------------ configs at full size -------

def test_config0_full_q8_gemv():
    M = K = 4096
    w = weights(0, M * K)
    x = acts(0, K)
    wq, wd = O.quantizeQ8_0Split(w)
    xq, xd = O.quantizeQ8_0Split(x)
    d = to_dev(wq, wd, x)
    # activations quantized on the GPU, as a caller does
    xq_d = torch.empty(K, dtype=torch.int8, device="cuda")
    xd_d = torch.empty(K // 32, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(d[2], xq_d, xd_d)
    assert np.array_equal(to_host(xq_d), xq)
    y = dev_y(M)
    L.dequantGemvQ8(d[0], d[1], 32, xq_d, xd_d, y)
    assert_bits(to_host(y), O.dequantGemvQ8(wq, wd, 32, xq, xd))


def test_config1_full_q4_0_gemv():
    M, K = 11008, 4096
    w = weights(1, M * K)
    x = acts(1, K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    wd_, xd_ = to_dev(w, x)
    bd = torch.empty(blk.size, dtype=torch.uint8, device="cuda")
    L.quantizeQ4_0Batch(wd_, bd)                 # GPU weight prep == oracle
    assert np.array_equal(to_host(bd), blk)
    y = dev_y(M)
    L.dequantGemvQ4_0(bd, K // 32, xd_, y)
    assert_bits(to_host(y), O.dequantGemvQ4_0(blk, K // 32, x))


def test_config2_full_mxfp4_gemv():
    M, K = 14336, 4096
    w = weights(2, M * K)
    x = acts(2, K)
    sm = O.calibrateMX(w, 32, 2)
    pf = O.packF4(O.quantize(w, sm, 32, "f4"))
    a, b, xd = to_dev(pf, sm, x)
    y = dev_y(M)
    L.dequantGemvF4(a, b, 32, xd, y)
    assert_bits(to_host(y), O.dequantGemvF4(pf, sm, 32, x))


# ------------------------------------------------------- errors, edges --

def test_shape_errors_raise_like_reference_asserts():
    wq, ws, xq, xs = to_dev(np.zeros(64, np.int8), np.zeros(2, F), np.zeros(32, np.int8),
                            np.zeros(1, F))
    with pytest.raises(AssertionError):
        L.dequantGemvQ8(wq, ws, 32, xq, xs, dev_y(3))       # wq.len != m*k
    with pytest.raises(AssertionError):
        L.dequantGemvQ8(wq, ws, 0, xq, xs, dev_y(2))        # groupSize 0
    with pytest.raises(AssertionError):
        L.dequantGemvQ8(wq, ws, 32, xq, torch.zeros(2, device="cuda"), dev_y(2))


def test_empty_shapes():
    # m = 0: nothing to do; k = 0: every row is the empty fold 0.0
    e8 = torch.empty(0, dtype=torch.int8, device="cuda")
    ef = torch.empty(0, dtype=torch.float32, device="cuda")
    L.dequantGemvQ8(e8, ef, 32, e8, ef, ef)
    y = dev_y(4)
    L.dequantGemv(e8, ef, 32, ef, y)
    assert np.array_equal(to_host(y), np.zeros(4, F))


def test_unaligned_device_pointers_take_plain_staging():
    """A weight view starting 1 byte into an allocation cannot use bulk
    copies; the plain-load staging must give the same bits."""
    M, K = 65, 512
    w = weights(5, M * K)
    x = acts(5, K)
    s8 = O.calibrateSymmetric(w, 32, 127.0)
    q8 = O.quantize(w, s8, 32, "i8")
    big = torch.zeros(q8.size + 1, dtype=torch.int8, device="cuda")
    big[1:] = torch.from_numpy(q8).cuda()
    sd, xd = to_dev(s8, x)
    y = dev_y(M)
    L.dequantGemv(big[1:], sd, 32, xd, y)
    assert_bits(to_host(y), O.dequantGemv(q8, s8, 32, x))


def test_page_locked_host_buffers_through_the_device_forms():
    """lp_host_device_pointer: a device form given page-locked host memory for
    its activations and output reads and writes it in place, with the bits of
    the device-buffer call (fp32 Q4_0 in both modes, int8 Q8); pageable
    memory is refused before anything is launched."""
    M, K = 1000, 4096
    bpr, gpr = K // 32, K // 32
    w = weights(90, M * K)
    x = acts(91, K)
    blk = O.quantizeQ4_0(w).reshape(-1)
    (bd,) = to_dev(blk)
    xd = torch.from_numpy(x).cuda()
    xh = torch.from_numpy(x).pin_memory()
    yh = torch.full((M,), float("nan"), dtype=torch.float32).pin_memory()
    xp, yp = N.host_device_pointer(xh.data_ptr()), N.host_device_pointer(yh.data_ptr())
    st = torch.cuda.current_stream().cuda_stream
    for mode in ("fast", "exact"):
        with L.fp32_mode(mode):
            yd = dev_y(M)
            L.dequantGemvQ4_0(bd, bpr, xd, yd)
            N.check(N.lib().lp_dequant_gemv_q4_0(bd.data_ptr(), M * bpr, bpr, xp, K, yp, M, st), "q4_0")
            torch.cuda.synchronize()
            assert_bits(yh.numpy(), to_host(yd))
    wq, ws = O.quantizeQ8_0Split(w)
    xq, xs = O.quantizeQ8_0Split(x)
    wqd, wsd, xqd, xsd = to_dev(wq, ws, xq, xs)
    yd = dev_y(M)
    L.dequantGemvQ8(wqd, wsd, 32, xqd, xsd, yd)
    xqh, xsh = torch.from_numpy(xq).pin_memory(), torch.from_numpy(xs).pin_memory()
    yh.fill_(float("nan"))
    N.check(N.lib().lp_dequant_gemv_q8(wqd.data_ptr(), M * K, wsd.data_ptr(), M * gpr, 32,
                                       N.host_device_pointer(xqh.data_ptr()), K,
                                       N.host_device_pointer(xsh.data_ptr()), gpr, yp, M, st), "q8")
    torch.cuda.synchronize()
    assert_bits(yh.numpy(), to_host(yd))
    pageable = np.zeros(16, np.float32)
    with pytest.raises(N.NativeError):
        N.host_device_pointer(pageable.ctypes.data)



@pytest.mark.parametrize("nbytes,soff,doff", [(16384, 0, 0), (44032, 0, 0), (4097, 0, 0),
                                              (1000, 3, 5), (0, 0, 0)])
def test_copy_in_from_page_locked_memory(nbytes, soff, doff):
    """lp_copy_in moves bytes from page-locked host memory into device memory
    in stream order (16-byte units when both ends and the size allow)."""
    rng = np.random.default_rng(nbytes)
    src = torch.from_numpy(rng.integers(0, 256, nbytes + soff, dtype=np.uint8)).pin_memory()
    dst = torch.zeros(nbytes + doff + 7, dtype=torch.uint8, device="cuda")
    st = torch.cuda.current_stream().cuda_stream
    # (an empty pinned tensor has no storage: zero bytes take a null source)
    sp = N.host_device_pointer(src.data_ptr()) + soff if nbytes else None
    N.check(N.lib().lp_copy_in(dst.data_ptr() + doff, sp, nbytes, st), "copy_in")
    torch.cuda.synchronize()
    got = dst.cpu().numpy()
    assert np.array_equal(got[doff:doff + nbytes], src.numpy()[soff:])
    assert not got[:doff].any() and not got[doff + nbytes:].any()


@pytest.mark.parametrize("M,K,xoff", [(1, 32, 0), (333, 4096, 0), (4096, 11008, 0),
                                      (300, 4096, 1), (4800, 4096, 0)])
def test_quantize_dequant_gemv_is_the_two_calls(M, K, xoff):
    """quantizeQ8_0 + dequantGemvQ8 / dequantGemvI4Q8 fused into one launch give
    the bits of the two separate calls and of the oracle -- an all-zero
    block, a block of large values, ragged row counts and activations off the
    16-byte grid included."""
    w = weights(100 + M, M * K)
    x = acts(101 + M, K)
    x[:32] = 0.0
    if K >= 96:
        x[64:96] *= F(1e4)  # large, with the block's f16 scale still finite
    gpr = K // 32
    xq_o, xs_o = O.quantizeQ8_0Split(x)
    xb = torch.zeros(K + xoff, dtype=torch.float32, device="cuda")
    xb[xoff:] = torch.from_numpy(x).cuda()
    xd = xb[xoff:]
    xq = torch.empty(K, dtype=torch.int8, device="cuda")
    xs = torch.empty(gpr, dtype=torch.float32, device="cuda")
    L.quantizeQ8_0Split(xd, xq, xs)
    wq, ws = O.quantizeQ8_0Split(w)
    s4 = O.calibrateSymmetric(w, 32, 7.0)
    p4 = O.packInt4(O.quantize(w, s4, 32, "i4"))
    for fused, two, ofn, wt, st in (
            (L.quantizeDequantGemvQ8, L.dequantGemvQ8, O.dequantGemvQ8, wq, ws),
            (L.quantizeDequantGemvI4Q8, L.dequantGemvI4Q8, O.dequantGemvI4Q8, p4, s4)):
        wd, sd = to_dev(wt, st)
        y1, y2 = dev_y(M), dev_y(M)
        fused(wd, sd, 32, xd, y1)
        two(wd, sd, 32, xq, xs, y2)
        assert_bits(to_host(y1), to_host(y2))
        assert_bits(to_host(y1), ofn(wt, st, 32, xq_o, xs_o))
    with pytest.raises(AssertionError):
        L.quantizeDequantGemvQ8(*to_dev(wq, ws), 64, xd, dev_y(M))
