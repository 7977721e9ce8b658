"""Pin the oracle's kernels to the reference tests' own references.

Bit-exact cases restate test_sdot.nim (intRef / refQ8 / refQ4 and GEMM column
== GEMV) and test_parallel.nim (pooled/sharded == serial for thread counts
0,1,2,3,64).  Tolerance cases restate test_quant_simd.nim:85-245 (fp64,
maxRel < 1e-3), and a numpy restatement of the scalar fp32 order must agree
with the C oracle bit for bit.
"""
import numpy as np
import pytest

import numpy_refs as R
import refcases as C
from oracle import oracle as O

F = np.float32


def bits_equal(a, b):
    return np.array_equal(np.asarray(a, F).view(np.uint32), np.asarray(b, F).view(np.uint32))


@pytest.mark.parametrize("M,K,gs", C.SDOT_INT8_SHAPES)
def test_gemv_q8_equals_int_ref(M, K, gs):
    wq, ws, xq, xs = C.sdot_int8_case(M, K, gs)
    assert bits_equal(O.dequantGemvQ8(wq, ws, gs, xq, xs), R.int_ref(wq, ws, gs, xq, xs))


@pytest.mark.parametrize("M,K,gs", C.SDOT_INT4_SHAPES)
def test_gemv_i4q8_equals_int_ref(M, K, gs):
    vals, ws, xq, xs = C.sdot_int4_case(M, K, gs)
    want = R.int_ref(vals, ws, gs, xq, xs)
    got = O.dequantGemvI4Q8(C.pack_i4_values(vals), ws, gs, xq, xs)
    assert bits_equal(got, want)


def test_packed_and_unpacked_agree():
    """test_sdot.nim:129-157."""
    M, K, gs = 8, 128, 64
    vals = np.array([(i % 15) - 7 for i in range(M * K)], np.int8)
    xq = np.array([(i % 200) - 100 for i in range(K)], np.int8)
    ws = np.full(M * (K // gs), F(0.02), F)
    xs = np.full(K // gs, F(0.03), F)
    a = O.dequantGemvQ8(vals, ws, gs, xq, xs)
    b = O.dequantGemvI4Q8(C.pack_i4_values(vals), ws, gs, xq, xs)
    assert bits_equal(a, b)


@pytest.mark.parametrize("M,bpr", C.GGML_SHAPES)
def test_gemv_q8_0q8_equals_ref(M, bpr):
    w = C.ggml_q8_w_blocks(M, bpr)
    x = C.ggml_x_blocks(bpr)
    assert bits_equal(O.dequantGemvQ8_0Q8(w, bpr, x), R.ref_q8(w, bpr, x))


@pytest.mark.parametrize("M,bpr", C.GGML_SHAPES)
def test_gemv_q4_0q8_equals_ref(M, bpr):
    w = C.ggml_q4_w_blocks(M, bpr)
    x = C.ggml_x_blocks(bpr)
    assert bits_equal(O.dequantGemvQ4_0Q8(w, bpr, x), R.ref_q4(w, bpr, x))


@pytest.mark.parametrize("M,K,gs,n", C.GEMM_I8_SHAPES)
def test_gemm_q8_column_equals_gemv(M, K, gs, n):
    wq, ws, xq, xs = C.gemm_int8_case(M, K, gs, n)
    gpr = K // gs
    y = O.dequantGemmQ8(wq, ws, gs, xq, xs, n).reshape(M, n)
    for c in range(n):
        yc = O.dequantGemvQ8(wq, ws, gs, xq[c * K:(c + 1) * K], xs[c * gpr:(c + 1) * gpr])
        assert bits_equal(y[:, c], yc)
        assert bits_equal(yc, R.int_ref(wq, ws, gs, xq[c * K:(c + 1) * K], xs[c * gpr:(c + 1) * gpr]))


@pytest.mark.parametrize("M,K,gs,n", C.GEMM_I4_SHAPES)
def test_gemm_i4q8_column_equals_gemv(M, K, gs, n):
    wp, ws, xq, xs = C.gemm_int4_case(M, K, gs, n)
    gpr = K // gs
    y = O.dequantGemmI4Q8(wp, ws, gs, xq, xs, n).reshape(M, n)
    for c in range(n):
        yc = O.dequantGemvI4Q8(wp, ws, gs, xq[c * K:(c + 1) * K], xs[c * gpr:(c + 1) * gpr])
        assert bits_equal(y[:, c], yc)


# ---------------------------------------------- fp32-activation kernels

def test_fp32_gemv_i8_tolerance_and_order():
    """test_quant_simd.nim:85-107 (M=37, K=200, gs=40)."""
    M, K, gs = 37, 200, 40
    u = 2463534242
    wq = np.empty(M * K, np.int8)
    for i in range(wq.size):
        u, r = C.next_rnd(u)
        wq[i] = O.quantize(np.array([r * F(110.0)], F), np.ones(1, F), 1, "i8")[0]
    sc = np.empty(M * (K // gs), F)
    for i in range(sc.size):
        u, r = C.next_rnd(u)
        sc[i] = F(0.005) + abs(r) * F(0.02)
    x = np.empty(K, F)
    for i in range(K):
        u, r = C.next_rnd(u)
        x[i] = r * F(3.0)
    y = O.dequantGemv(wq, sc, gs, x)
    assert R.max_rel(y, R.fp64_gemv(wq.reshape(M, K), sc, gs, x)) < 1e-3
    assert bits_equal(y, R.seq_gemv_i8(wq, sc, gs, x))


def test_fp32_gemv_i4_tolerance_and_order():
    """test_quant_simd.nim:109-144 (M=17, K=192, gs=48)."""
    M, K, gs = 17, 192, 48
    u = 88172645
    vals = np.empty(M * K, np.int8)
    for i in range(vals.size):
        u, r = C.next_rnd(u)
        vals[i] = int(r * F(7.9))        # Nim int(float) truncates
    sc = np.empty(M * (K // gs), F)
    for i in range(sc.size):
        u, r = C.next_rnd(u)
        sc[i] = F(0.01) + abs(r) * F(0.03)
    x = np.empty(K, F)
    for i in range(K):
        u, r = C.next_rnd(u)
        x[i] = r * F(2.0)
    wp = C.pack_i4_values(vals)
    y = O.dequantGemvI4(wp, sc, gs, x)
    assert R.max_rel(y, R.fp64_gemv(vals.reshape(M, K), sc, gs, x)) < 1e-3
    assert bits_equal(y, R.seq_gemv_i4(wp, sc, gs, x))


def test_fp32_gemv_f4_tolerance_and_order():
    """test_quant_simd.nim:146-182: calibrateMX per row, e2m1 codes, packF4."""
    M, K, gs = 17, 192, 48
    u = 20260728
    x = np.empty(K, F)
    for i in range(K):
        u, r = C.next_rnd(u)
        x[i] = r * F(2.0)
    wp = np.empty(M * K // 2, np.uint8)
    sc = np.empty(M * (K // gs), F)
    ref = np.empty(M)
    lut = np.array([O.lib().lpo_f4e2m1_to_f32(c) for c in range(16)], F)
    for r_ in range(M):
        row = np.empty(K, F)
        for c in range(K):
            u, r = C.next_rnd(u)
            row[c] = r * F(4.5)
        s = O.calibrateMX(row, gs, 2)
        codes = O.quantize(row, s, gs, "f4")
        sc[r_ * (K // gs):(r_ + 1) * (K // gs)] = s
        wp[r_ * K // 2:(r_ + 1) * K // 2] = O.packF4(codes)
        ref[r_] = np.sum(lut[codes].astype(np.float64) * np.repeat(s, gs).astype(np.float64) * x)
    y = O.dequantGemvF4(wp, sc, gs, x)
    assert R.max_rel(y, ref) < 1e-3
    assert bits_equal(y, R.seq_gemv_f4(wp, sc, gs, x))


@pytest.mark.parametrize("fmt", ["q8_0", "q4_0"])
def test_fp32_gemv_ggml_tolerance_and_order(fmt):
    """test_quant_simd.nim:184-245."""
    M, BPR, seed, amp = (11, 3, 55555, 4.0) if fmt == "q8_0" else (9, 4, 24680, 3.0)
    K = BPR * 32
    u = seed
    x = np.empty(K, F)
    for i in range(K):
        u, r = C.next_rnd(u)
        x[i] = r * F(2.0)
    blocks = []
    ref = np.empty(M)
    for r_ in range(M):
        row = np.empty(K, F)
        for c in range(K):
            u, r = C.next_rnd(u)
            row[c] = r * F(amp)
        b = O.quantizeQ8_0(row) if fmt == "q8_0" else O.quantizeQ4_0(row)
        deq = O.dequantizeQ8_0(b) if fmt == "q8_0" else O.dequantizeQ4_0(b)
        ref[r_] = np.sum(deq.astype(np.float64) * x.astype(np.float64))
        blocks.append(b)
    w = np.concatenate(blocks)
    if fmt == "q8_0":
        y = O.dequantGemvQ8_0(w, BPR, x)
        assert bits_equal(y, R.seq_gemv_q8_0(w, BPR, x))
    else:
        y = O.dequantGemvQ4_0(w, BPR, x)
        assert bits_equal(y, R.seq_gemv_q4_0(w, BPR, x))
    assert R.max_rel(y, ref) < 1e-3


# ------------------------------------------------------- pool (LpPool)

@pytest.mark.parametrize("M", C.PAR_ROWS)
def test_sharded_fp32_forms_equal_serial(M):
    """test_parallel.nim:46-100 over every thread count."""
    x = C.par_x()
    gs = C.PAR_GS
    cases = []
    wq, sc = C.par_int8(M); cases.append((O.dequantGemv, (wq, sc, gs, x)))
    w4, sc4 = C.par_int4(M); cases.append((O.dequantGemvI4, (w4, sc4, gs, x)))
    wf, scf = C.par_f4(M); cases.append((O.dequantGemvF4, (wf, scf, gs, x)))
    q8, bpr = C.par_q8_0(M); cases.append((O.dequantGemvQ8_0, (q8, bpr, x)))
    q4, bpr = C.par_q4_0(M); cases.append((O.dequantGemvQ4_0, (q4, bpr, x)))
    for fn, args in cases:
        want = fn(*args)
        for nt in C.PAR_THREADS:
            pool = O.Pool(O.shardCount(M, nt))
            try:
                assert bits_equal(fn(*args, pool=pool), want)
            finally:
                pool.shutdown()


def test_pooled_int8_act_reused_across_calls():
    """test_parallel.nim:109-160: one pool, repeated dispatches."""
    pool = O.Pool(4)
    try:
        for M in (300, 129, 64):
            wq, w4, ws, xq, xs = C.pooled_case(M)
            for fn, w in ((O.dequantGemvQ8, wq), (O.dequantGemvI4Q8, w4)):
                want = fn(w, ws, C.PAR_GS, xq, xs)
                for _ in range(3):
                    assert bits_equal(fn(w, ws, C.PAR_GS, xq, xs, pool=pool), want)
    finally:
        pool.shutdown()
    pool.shutdown()                     # idempotent (test_parallel.nim:162-169)
    assert pool.threadCount() == 0


def test_pooled_gemm_reused():
    """test_parallel.nim:171-220 (n = 3)."""
    n = 3
    pool = O.Pool(4)
    try:
        for M in (300, 128):
            wq, w4, ws, xq, xs = C.pooled_case(M, n)
            for fn, w in ((O.dequantGemmQ8, wq), (O.dequantGemmI4Q8, w4)):
                want = fn(w, ws, C.PAR_GS, xq, xs, n)
                for _ in range(2):
                    assert bits_equal(fn(w, ws, C.PAR_GS, xq, xs, n, pool=pool), want)
    finally:
        pool.shutdown()


def test_shard_count_rules():
    """parallel.nim:45-53: at most rows div 64 shards, at least 1."""
    assert O.shardCount(1, 64) == 1
    assert O.shardCount(300, 64) == 4
    assert O.shardCount(300, 3) == 3
    assert O.shardCount(64, 2) == 1


def test_fp4_gemm_oracle_is_the_exact_gemm_of_the_decoded_operands():
    """lpo_gemm_fp4 against numpy: e2m1 table (simd/dequant.nim:57-58,
    halved) times the per-block scales, fp64 GEMM; MXFP4 and NVFP4."""
    rng = np.random.default_rng(5)
    m, k, n = 7, 96, 5
    wp = rng.integers(0, 256, m * k // 2, dtype=np.uint8)
    xp = rng.integers(0, 256, n * k // 2, dtype=np.uint8)
    tab = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6])

    def dec(p, rows):
        v = np.empty((rows, k))
        q = p.reshape(rows, k // 2)
        v[:, 0::2], v[:, 1::2] = tab[q & 15], tab[q >> 4]
        return v
    ws = np.ldexp(1.0, rng.integers(-8, 3, m * k // 32)).astype(np.float32)
    xs = np.ldexp(1.0, rng.integers(-8, 3, n * k // 32)).astype(np.float32)
    W = dec(wp, m) * np.repeat(ws.reshape(m, -1).astype(np.float64), 32, 1)
    X = dec(xp, n) * np.repeat(xs.reshape(n, -1).astype(np.float64), 32, 1)
    got = O.gemmFp4(wp, ws, xp, xs, n)
    assert np.allclose(got, (W @ X.T).reshape(-1), rtol=1e-12, atol=1e-300)
    # NVFP4: e4m3 block scales per 16, global factor
    wb = rng.integers(0x20, 0x50, m * k // 16, dtype=np.uint8)
    xb = rng.integers(0x20, 0x50, n * k // 16, dtype=np.uint8)
    e4 = np.array([O.lib().lpo_f8e4m3_to_f32(int(c)) for c in range(256)], np.float64)
    W = dec(wp, m) * np.repeat(e4[wb].reshape(m, -1), 16, 1)
    X = dec(xp, n) * np.repeat(e4[xb].reshape(n, -1), 16, 1)
    got = O.gemmFp4(wp, wb, xp, xb, n, nvfp4=True, globalScale=0.75)
    assert np.allclose(got, 0.75 * (W @ X.T).reshape(-1), rtol=1e-12, atol=1e-300)
