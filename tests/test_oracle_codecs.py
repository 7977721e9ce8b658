"""Pin the oracle's encoders and element codecs to external golden vectors.

Fixtures in tests/golden/ come from the reference's own generator
(gen_reference.py, via tests/golden/make_golden.py): gguf-py for ggml Q8_0/Q4_0
and the OCP-MX scheme with ml_dtypes elements.  These are the checks of
test_scheme_conformance.nim:46-86,117-140, test_mx_conformance.nim and
test_f16_conformance.nim, run against the oracle.
"""
import os

import numpy as np
import pytest

from oracle import oracle as O

G = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def rd(name, dtype):
    return np.fromfile(os.path.join(G, name), dtype=dtype)


def test_q8_0_quantize_bytes_match_gguf():
    x = rd("ref_scheme_input.bin", np.float32)
    want = rd("ref_ggml_q8_0_bytes.bin", np.uint8)
    got = O.quantizeQ8_0(x).reshape(-1)
    assert got.size == want.size
    assert np.array_equal(got, want)


def test_q4_0_quantize_bytes_match_gguf():
    x = rd("ref_scheme_input.bin", np.float32)
    want = rd("ref_ggml_q4_0_bytes.bin", np.uint8)
    got = O.quantizeQ4_0(x).reshape(-1)
    assert np.array_equal(got, want)


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_ggml_dequant_of_gguf_bytes_bit_exact(fmt):
    raw = rd(f"ref_ggml_{fmt}_bytes.bin", np.uint8)
    want = rd(f"ref_ggml_{fmt}_dq.bin", np.uint32)
    dq = O.dequantizeQ8_0(raw) if fmt == "q8_0" else O.dequantizeQ4_0(raw)
    assert np.array_equal(dq.view(np.uint32), want)


@pytest.mark.parametrize("fmt", ["q4_k", "q6_k"])
def test_kquant_dequant_of_gguf_bytes_bit_exact(fmt):
    """dequantizeQ4_K / Q6_K (ggml.nim:136-213) against gguf-py's dequantization
    of valid random super-blocks with finite d / dmin (gen_reference.py:175-195;
    test_scheme_conformance.nim's k-quant checks)."""
    raw = rd(f"ref_ggml_{fmt}_bytes.bin", np.uint8)
    want = rd(f"ref_ggml_{fmt}_dq.bin", np.uint32)
    dq = O.dequantizeQ4_K(raw) if fmt == "q4_k" else O.dequantizeQ6_K(raw)
    assert dq.size == want.size == raw.size // (144 if fmt == "q4_k" else 210) * 256
    assert np.array_equal(dq.view(np.uint32), want)


def test_nvfp4_scheme_matches_the_te_golden():
    """quantizeNVFP4 (nvfp4.nim:39-78) against the numpy transcription of
    TransformerEngine's NVFP4QuantizerRef (gen_reference.py:237-294): global
    decode scale, e4m3 block scales and e2m1 codes, bit for bit."""
    x = rd("ref_nvfp4_input.bin", np.float32)
    raw = rd("ref_nvfp4_out.bin", np.uint8)
    nb = x.size // 16
    codes, scales, gds = O.quantizeNVFP4(x)
    assert gds == raw[:4].view("<f4")[0]
    assert np.array_equal(scales, raw[4:4 + nb])
    assert np.array_equal(codes, raw[4 + nb:])
    dq = O.dequantizeNVFP4(codes, scales, gds)
    lut = np.array([O.lib().lpo_f4e2m1_to_f32(c) for c in range(16)], np.float32)
    e4 = np.array([O.lib().lpo_f8e4m3_to_f32(c) for c in range(256)], np.float32)
    want = (lut[codes] * np.repeat(e4[scales], 16)).astype(np.float32) * np.float32(gds)
    assert np.array_equal(dq.view(np.uint32), want.astype(np.float32).view(np.uint32))


def test_e4m3_codec_round_trip_and_rounding():
    """e4m3fn (float8.nim:28-112): every finite code decodes and re-encodes to
    itself; midpoints between neighbours round to the even code."""
    for c in range(256):
        if (c & 0x7F) == 0x7F:
            continue  # NaN
        v = O.lib().lpo_f8e4m3_to_f32(c)
        assert O.lib().lpo_to_f8e4m3(v) == (c if v != 0 or c == 0 else c)
    for c in range(0, 0x7E):
        a, b = O.lib().lpo_f8e4m3_to_f32(c), O.lib().lpo_f8e4m3_to_f32(c + 1)
        mid = np.float32((np.float64(a) + np.float64(b)) / 2)
        if np.float64(mid) == (np.float64(a) + np.float64(b)) / 2:
            assert O.lib().lpo_to_f8e4m3(float(mid)) == (c if c % 2 == 0 else c + 1)
    assert O.lib().lpo_to_f8e4m3(460.0) == 0x7E and O.lib().lpo_to_f8e4m3(465.0) == 0x7F


def test_golden_input_has_the_edge_blocks():
    x = rd("ref_scheme_input.bin", np.float32)
    assert np.all(x[100:132] == 0)                       # the all-zero block
    assert np.all(x[4096:4104] == np.float32(1e-30))     # the tiny-scale block


def test_mx_fp4_scheme_end_to_end():
    """calibrateMX(x, 32, 2) + quantize + dequantize vs the OCP-MX golden
    (test_scheme_conformance.nim:117-140)."""
    x = rd("ref_mx_input.bin", np.float32)
    want = rd("ref_mx_f4e2m1_dq.bin", np.uint32)
    sc = O.calibrateMX(x, 32, 2)
    codes = O.quantize(x, sc, 32, "f4")
    lut = np.array([O.lib().lpo_f4e2m1_to_f32(c) for c in range(16)], np.float32)
    dq = (lut[codes] * np.repeat(sc, 32)).astype(np.float32)   # dequantize: decode * scale
    assert np.array_equal(dq.view(np.uint32), want)


def test_mx_scales_are_exact_e8m0():
    x = rd("ref_mx_input.bin", np.float32)
    sc = O.calibrateMX(x, 32, 2)
    for s in sc:
        assert O.e8m0_to_f32(O.to_e8m0(float(s))) == s


def test_e2m1_encode_matches_ml_dtypes():
    z = np.load(os.path.join(G, "e2m1_encode.npz"))
    ins, outs = z["ins"], z["outs"]
    f = ins.view(np.float32)
    L = O.lib()
    got = np.array([L.lpo_to_f4e2m1(float(v)) for v in f], np.uint8)
    assert np.array_equal(got, outs)


def test_e2m1_decode_round_trips_every_code():
    """test_mx_conformance.nim:24-28 (code 8 is -0 and encodes back to 8)."""
    for c in range(16):
        assert O.to_f4e2m1(O.lib().lpo_f4e2m1_to_f32(c)) == c


def test_e8m0_encode_matches_ml_dtypes():
    z = np.load(os.path.join(G, "e8m0_encode.npz"))
    f = z["ins"].view(np.float32)
    L = O.lib()
    got = np.array([L.lpo_to_e8m0(float(v)) for v in f], np.uint8)
    assert np.array_equal(got, z["outs"])


def test_f16_encode_matches_numpy():
    z = np.load(os.path.join(G, "f16_encode.npz"))
    f = z["ins"].view(np.float32)
    L = O.lib()
    got = np.array([L.lpo_f32_to_f16(float(v)) for v in f], np.uint16)
    want = z["outs"]
    nan = np.isnan(f)
    assert np.array_equal(got[~nan], want[~nan])
    # NaN stays NaN (payload rules differ between ports; only NaN-ness matters)
    assert np.all((got[nan] & 0x7C00) == 0x7C00) and np.all((got[nan] & 0x03FF) != 0)


def test_f16_decode_exhaustive():
    codes = np.arange(65536, dtype=np.uint16)
    want = codes.view(np.float16).astype(np.float32).view(np.uint32)
    L = O.lib()
    got = np.array([L.lpo_f16_to_f32(int(c)) for c in codes], np.float32).view(np.uint32)
    nan = np.isnan(codes.view(np.float16))
    assert np.array_equal(got[~nan], want[~nan])


def test_int4_pack_layout():
    """test_intx_conformance.nim:32-36: low = 3, high = -2 -> 0xE3."""
    assert O.packInt4(np.array([3, -2], np.int8))[0] == 0xE3
    # odd tail keeps only the low nibble (test_intx_conformance.nim:49-52)
    assert O.packInt4(np.array([5], np.int8))[0] & 0x0F == 5


def test_i8_i4_encoders():
    """test_intx_conformance.nim:8-30: rounding and clamps."""
    one = np.ones(1, np.float32)
    for v, q in [(2.6, 3), (-2.6, -3), (200.0, 127), (-200.0, -128), (2.5, 3), (-2.5, -3)]:
        assert O.quantize(np.array([v], np.float32), one, 1, "i8")[0] == q
    for v, q in [(100.0, 7), (-100.0, -8), (2.6, 3)]:
        assert O.quantize(np.array([v], np.float32), one, 1, "i4")[0] == q


def test_calibrate_symmetric_zero_group_and_ragged_tail():
    """quant.nim:84-110: a zero group gets scale 1.0; the last group may be short."""
    assert O.calibrateSymmetric(np.zeros(8, np.float32), 0, 127.0)[0] == 1.0
    x = np.arange(100, dtype=np.float32) - 50
    sc = O.calibrateSymmetric(x, 64, 127.0)
    assert sc.size == 2
    assert sc[0] == np.float32(50.0) / np.float32(127.0)
    assert sc[1] == np.float32(49.0) / np.float32(127.0)


def _affine(x, gs, qmin, qmax):
    """calibrateAsymmetric's (scale, zeroPoint) per group (quant.nim:139-177)."""
    n = x.size
    gs = gs if gs > 0 else n
    sc, zp = [], []
    for lo in range(0, n, gs):
        mn, mx = np.float32(x[lo:lo + gs].min()), np.float32(x[lo:lo + gs].max())
        span = np.float32(mx - mn)
        s = np.float32(span / np.float32(qmax - qmin)) if span > 0 else np.float32(1.0)
        sc.append(s)
        zp.append(np.float32(np.float32(qmin) - np.float32(mn / s)))
    return np.array(sc, np.float32), np.array(zp, np.float32)


@pytest.mark.parametrize("kind,n,gs,qmax", [("i8", 1000, 0, 127.0), ("i8", 1000, 64, 127.0),
                                            ("i4", 512, 32, 7.0), ("i8", 333, 7, 127.0)])
def test_dequantize_batch_is_the_scalar_formula(kind, n, gs, qmax):
    """test_quant_simd.nim:33-64: dequantizeBatch of calibrateSymmetric +
    quantize output equals the scalar dequantize, f32(q) * scale[i div gs],
    bit for bit; the asymmetric form is (f32(q) - zeroPoint) * scale."""
    i = np.arange(n, dtype=np.float32)
    x = (np.sin(i * np.float32(0.1)) * np.float32(5.0)).astype(np.float32)
    sc = O.calibrateSymmetric(x, gs, qmax)
    q = O.quantize(x, sc, gs, kind)
    g = np.arange(n) // (gs if gs > 0 else max(n, 1))
    want = (q.astype(np.float32) * sc[g]).astype(np.float32)
    assert np.array_equal(O.dequantizeBatch(q, sc, gs).view(np.uint32), want.view(np.uint32))
    sa, za = _affine(x, gs, -128.0, 127.0)
    qa = np.clip(np.round(x / sa[g] + za[g]), -128, 127).astype(np.int8)
    want = ((qa.astype(np.float32) - za[g]) * sa[g]).astype(np.float32)
    got = O.dequantizeBatch(qa, sa, gs, za)
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))
    assert np.max(np.abs(got - x)) <= np.max(sa) * 0.5 + 1e-6


def test_q8_0_split_matches_blocks():
    rng = np.random.default_rng(0)
    x = rng.standard_normal(4096).astype(np.float32)
    blocks = O.quantizeQ8_0(x)
    qs, d = O.quantizeQ8_0Split(x)
    assert np.array_equal(blocks[:, 2:].reshape(-1).view(np.int8), qs)
    dh = blocks[:, :2].copy().view(np.uint16).reshape(-1)
    assert np.array_equal(dh.view(np.float16).astype(np.float32), d)


@pytest.mark.parametrize("n,gs", [(1000, 0), (1000, 64), (333, 7)])
def test_quantize_batch_with_zero_points_is_the_scalar_formula(n, gs):
    """quantizeBatch with QParams carrying zero points falls through to the
    scalar quantize (simd/dequant.nim:1717-1750 -> quant.nim:48-60):
    toI8(fl(fl(x / scale) + zeroPoint)), ties away from zero, clamped to
    [-128, 127]; the symmetric form adds 0.0."""
    i = np.arange(n, dtype=np.float32)
    x = (np.sin(i * np.float32(0.1)) * np.float32(5.0)).astype(np.float32)
    sa, za = _affine(x, gs, -128.0, 127.0)
    za = (za + np.float32(100.0) * (np.arange(za.size) % 2)).astype(np.float32)  # reach the clamp
    g = np.arange(n) // (gs if gs > 0 else max(n, 1))
    v = ((x / sa[g]).astype(np.float32) + za[g]).astype(np.float32).astype(np.float64)
    want = np.clip(np.sign(v) * np.floor(np.abs(v) + 0.5), -128, 127).astype(np.int8)
    assert np.array_equal(O.quantizeBatch(x, sa, gs, za), want)
    v0 = ((x / sa[g]).astype(np.float32) + np.float32(0.0)).astype(np.float64)
    want0 = np.clip(np.sign(v0) * np.floor(np.abs(v0) + 0.5), -128, 127).astype(np.int8)
    assert np.array_equal(O.quantizeBatch(x, sa, gs), want0)
