"""LocalPool -- the reference's in-process LpPool shape over this box's GPUs
(lph_pool_* / lph_par_*, one worker thread per GPU, host arrays).

The reference's test_parallel.nim:12-220 restated: every per-call par* form
over thread counts 0 / 1 / 2 / 3 / 64 and 300 / 64 / 1 rows, and the pooled
int8-activation GEMV / GEMM forms reused across calls, must equal the serial
call bit for bit; shutdown is idempotent and a fresh pool still works.  The
serial results are also pinned to the CPU oracle (bit for bit in the exact
fp32 mode).  With one GPU visible the pool has one worker and exercises the
serial fall-back; with more, the rows really are split across GPUs.
"""
import numpy as np
import pytest

from gpu_util import F
import refcases as R
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import parallel as P  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402


def bits(a):
    return np.asarray(a, F).view(np.uint32)


def _fp32_cases(M):
    x = R.par_x()
    wq, sc8 = R.par_int8(M)
    w4, sc4 = R.par_int4(M)
    wf4, scf = R.par_f4(M)
    q80, bpr = R.par_q8_0(M)
    q40, _ = R.par_q4_0(M)
    return [
        ("int8", lambda y: L.dequantGemv(wq, sc8, R.PAR_GS, x, y),
         lambda y, t: P.parDequantGemvThreads(wq, sc8, R.PAR_GS, x, y, t),
         lambda: O.dequantGemv(wq, sc8, R.PAR_GS, x)),
        ("int4", lambda y: L.dequantGemvI4(w4, sc4, R.PAR_GS, x, y),
         lambda y, t: P.parDequantGemvI4Threads(w4, sc4, R.PAR_GS, x, y, t),
         lambda: O.dequantGemvI4(w4, sc4, R.PAR_GS, x)),
        ("mxfp4", lambda y: L.dequantGemvF4(wf4, scf, R.PAR_GS, x, y),
         lambda y, t: P.parDequantGemvF4Threads(wf4, scf, R.PAR_GS, x, y, t),
         lambda: O.dequantGemvF4(wf4, scf, R.PAR_GS, x)),
        ("q8_0", lambda y: L.dequantGemvQ8_0(q80.reshape(-1), bpr, x, y),
         lambda y, t: P.parDequantGemvQ8_0Threads(q80, bpr, x, y, t),
         lambda: O.dequantGemvQ8_0(q80.reshape(-1), bpr, x)),
        ("q4_0", lambda y: L.dequantGemvQ4_0(q40.reshape(-1), bpr, x, y),
         lambda y, t: P.parDequantGemvQ4_0Threads(q40, bpr, x, y, t),
         lambda: O.dequantGemvQ4_0(q40.reshape(-1), bpr, x)),
    ]


@pytest.mark.parametrize("mode", ["exact", "fast"])
@pytest.mark.parametrize("M", R.PAR_ROWS)
def test_per_call_par_forms_equal_serial_bits(M, mode):
    """test_parallel.nim:48-100: par*(..., threads) == serial, bit for bit."""
    with L.fp32_mode(mode):
        for name, serial, par, oracle in _fp32_cases(M):
            want = np.full(M, np.nan, F)
            serial(want)
            if mode == "exact":
                assert np.array_equal(bits(want), bits(oracle())), name
            for t in R.PAR_THREADS:
                got = np.full(M, np.nan, F)
                par(got, t)
                assert np.array_equal(bits(got), bits(want)), (name, t)


@pytest.mark.parametrize("M", R.PAR_ROWS)
def test_per_call_int8_activation_forms_equal_serial_bits(M):
    """The per-call parDequantGemvQ8 / parDequantGemvI4Q8 overloads."""
    wq, w4, ws, xq, xs = R.pooled_case(M)
    for serial, par, oracle in (
            (L.dequantGemvQ8, P.parDequantGemvQ8Threads, O.dequantGemvQ8),
            (L.dequantGemvI4Q8, P.parDequantGemvI4Q8Threads, O.dequantGemvI4Q8)):
        w = wq if serial is L.dequantGemvQ8 else w4
        want = np.full(M, np.nan, F)
        serial(w, ws, R.PAR_GS, xq, xs, want)
        assert np.array_equal(bits(want), bits(oracle(w, ws, R.PAR_GS, xq, xs)))
        for t in R.PAR_THREADS:
            got = np.full(M, np.nan, F)
            par(w, ws, R.PAR_GS, xq, xs, got, t)
            assert np.array_equal(bits(got), bits(want)), t


def test_pooled_forms_reused_across_calls():
    """test_parallel.nim:114-160 and :171-220: one pool, repeated dispatches,
    GEMV rows 300 / 129 / 64 and GEMM (n = 3) rows 300 / 128."""
    pool = P.LocalPool(4)
    try:
        assert pool.threadCount() == min(4, torch.cuda.device_count())
        for M in (300, 129, 64):
            wq, w4, ws, xq, xs = R.pooled_case(M)
            for w, serial, par in ((wq, L.dequantGemvQ8, P.parDequantGemvQ8),
                                   (w4, L.dequantGemvI4Q8, P.parDequantGemvI4Q8)):
                want = np.full(M, np.nan, F)
                serial(w, ws, R.PAR_GS, xq, xs, want)
                for _ in range(3):
                    got = np.full(M, np.nan, F)
                    par(pool, w, ws, R.PAR_GS, xq, xs, got)
                    assert np.array_equal(bits(got), bits(want))
        n = 3
        for M in (300, 128):
            wq, w4, ws, xq, xs = R.pooled_case(M, n)
            for w, serial, par, oracle in (
                    (wq, L.dequantGemmQ8, P.parDequantGemmQ8, O.dequantGemmQ8),
                    (w4, L.dequantGemmI4Q8, P.parDequantGemmI4Q8, O.dequantGemmI4Q8)):
                want = np.full(M * n, np.nan, F)
                serial(w, ws, R.PAR_GS, xq, xs, n, want)
                assert np.array_equal(bits(want), bits(oracle(w, ws, R.PAR_GS, xq, xs, n)))
                for _ in range(2):
                    got = np.full(M * n, np.nan, F)
                    par(pool, w, ws, R.PAR_GS, xq, xs, n, got)
                    assert np.array_equal(bits(got), bits(want))
    finally:
        pool.shutdown()
    assert N.device_error() == 0


def test_shutdown_is_idempotent_and_a_fresh_pool_works():
    """test_parallel.nim:162-169."""
    p = P.LocalPool(2)
    p.shutdown()
    p.shutdown()
    assert p.threadCount() == 0
    q = P.LocalPool(2)
    assert q.threadCount() == min(2, torch.cuda.device_count())
    q.shutdown()


def test_pool_reports_shape_errors_before_any_work():
    pool = P.LocalPool(0)
    try:
        wq, w4, ws, xq, xs = R.pooled_case(300)
        with pytest.raises(AssertionError):
            P.parDequantGemvQ8(pool, wq, ws, R.PAR_GS, xq, xs, np.zeros(299, F))
    finally:
        pool.shutdown()
