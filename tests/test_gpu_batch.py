"""Batched GEMV launches (lp_batch_begin / lp_batch_end, ``L.batch()``).

Every call queued in a batch must give the bits of the same call made on its
own, and the oracle's: across jobs of different shapes in one launch (rows
fewer than the SMs, one row, K = 4096 and 11008, group tails), for every
format that batches, when a later call reads an earlier call's output (the
queue launches first), when another library call comes in between, past the
64-call limit, and replayed from a CUDA graph.
"""
import numpy as np
import pytest

from gpu_util import acts, bits_equal, mismatch_report, to_dev, to_host, weights
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402

# (rows, K): fewer rows than SMs, one row, the config-4 shapes, a row of
# one group, and K = 96 (three groups)
SHAPES = [(1, 32), (7, 4096), (148, 4096), (300, 11008), (4800, 4096), (512, 11008),
          (4096, 4096), (149, 64), (2, 96), (1000, 2048)]


def dev_y(m):
    return torch.full((m,), float("nan"), dtype=torch.float32, device="cuda")


def assert_bits(got, want):
    assert bits_equal(got, want), mismatch_report(got, want)


@pytest.fixture(autouse=True)
def _no_device_error():
    yield
    assert N.device_error() == 0


def i4_case(seed, m, k):
    w = weights(seed, m * k)
    s4 = O.calibrateSymmetric(w, 32, 7.0)
    return O.packInt4(O.quantize(w, s4, 32, "i4")), s4


def q8_case(seed, m, k):
    return O.quantizeQ8_0Split(weights(seed, m * k))


def cases(make, shapes=SHAPES, seed=0):
    out = []
    for i, (m, k) in enumerate(shapes):
        wt, st = make(seed + 200 + i, m, k)
        x = acts(seed + 300 + i, k)
        out.append((m, k, wt, st, x, *to_dev(wt, st, x)))
    return out


@pytest.mark.parametrize("fmt", ["i4q8", "q8"])
def test_batch_fused_quantize_gemv_equals_lone_calls(fmt):
    fused = L.quantizeDequantGemvI4Q8 if fmt == "i4q8" else L.quantizeDequantGemvQ8
    ofn = O.dequantGemvI4Q8 if fmt == "i4q8" else O.dequantGemvQ8
    cs = cases(i4_case if fmt == "i4q8" else q8_case)
    lone = []
    for m, k, _, _, _, wd, sd, xd in cs:
        y = dev_y(m)
        fused(wd, sd, 32, xd, y)
        lone.append(to_host(y))
    ys = [dev_y(c[0]) for c in cs]
    with L.batch():
        for c, y in zip(cs, ys):
            fused(c[5], c[6], 32, c[7], y)
    for (m, k, wt, st, x, *_), y, yl in zip(cs, ys, lone):
        got = to_host(y)
        assert_bits(got, yl)
        xq, xs = O.quantizeQ8_0Split(x)
        assert_bits(got, ofn(wt, st, 32, xq, xs))


@pytest.mark.parametrize("fmt", ["i4q8", "q8"])
def test_batch_prequantized_gemv_equals_lone_calls(fmt):
    fn = L.dequantGemvI4Q8 if fmt == "i4q8" else L.dequantGemvQ8
    ofn = O.dequantGemvI4Q8 if fmt == "i4q8" else O.dequantGemvQ8
    cs = cases(i4_case if fmt == "i4q8" else q8_case, seed=50)
    acts_q = []
    for m, k, wt, st, x, *_ in cs:
        xq, xs = O.quantizeQ8_0Split(x)
        acts_q.append((xq, xs, *to_dev(xq, xs)))
    ys = [dev_y(c[0]) for c in cs]
    with L.batch():
        for c, a, y in zip(cs, acts_q, ys):
            fn(c[5], c[6], 32, a[2], a[3], y)
    for (m, k, wt, st, x, wd, sd, _), a, y in zip(cs, acts_q, ys):
        yl = dev_y(m)
        fn(wd, sd, 32, a[2], a[3], yl)
        assert_bits(to_host(y), to_host(yl))
        assert_bits(to_host(y), ofn(wt, st, 32, a[0], a[1]))


def test_batch_ggml_q8_0q8_and_q4_0q8_mixed_formats():
    """Calls alternating between the two ggml formats (each switch launches
    the queue) and runs of one format."""
    shapes = [(1, 1), (9, 3), (300, 128), (4096, 128), (150, 5)]  # (rows, blocks per row)
    jobs = []
    for i, (m, bpr) in enumerate(shapes):
        x = O.quantizeQ8_0(acts(400 + i, 32 * bpr))
        for j, (fn, ofn, enc) in enumerate(((L.dequantGemvQ8_0Q8, O.dequantGemvQ8_0Q8,
                                             O.quantizeQ8_0),
                                            (L.dequantGemvQ4_0Q8, O.dequantGemvQ4_0Q8,
                                             O.quantizeQ4_0))):
            w = enc(weights(500 + 10 * i + j, m * 32 * bpr))
            jobs.append((fn, ofn, w, x, bpr, m, *to_dev(w.reshape(-1), x.reshape(-1))))
    order = jobs + sorted(jobs, key=lambda j: j[0].__name__)  # alternating, then runs
    ys = [dev_y(j[5]) for j in order]
    with L.batch():
        for j, y in zip(order, ys):
            j[0](j[6], j[4], j[7], y)
    for j, y in zip(order, ys):
        assert_bits(to_host(y), j[1](j[2], j[4], j[3]))


def test_batch_chained_calls_read_earlier_outputs():
    """y of one call is x of the next (a layer chain), and a quantize of an
    earlier output comes in between: each read sees the finished output."""
    dims = [4096, 11008, 4096, 4096]
    ws = [i4_case(600 + i, dims[i + 1], dims[i]) for i in range(3)]
    wd = [to_dev(w, s) for w, s in ws]
    x0 = acts(601, dims[0])
    (x0d,) = to_dev(x0)
    ys = [dev_y(dims[i + 1]) for i in range(3)]
    xq = torch.empty(dims[2], dtype=torch.int8, device="cuda")
    xs = torch.empty(dims[2] // 32, dtype=torch.float32, device="cuda")
    with L.batch():
        L.quantizeDequantGemvI4Q8(*wd[0], 32, x0d, ys[0])
        L.quantizeDequantGemvI4Q8(*wd[1], 32, ys[0], ys[1])
        L.quantizeQ8_0Split(ys[1], xq, xs)
        L.dequantGemvI4Q8(*wd[2], 32, xq, xs, ys[2])
    x = x0
    for i in range(3):
        q, s = O.quantizeQ8_0Split(x)
        want = O.dequantGemvI4Q8(ws[i][0], ws[i][1], 32, q, s)
        assert_bits(to_host(ys[i]), want)
        x = want


def test_batch_past_64_calls_and_empty_calls():
    m, k = 64, 256
    w, s = i4_case(700, m, k)
    wd, sd = to_dev(w, s)
    xs = [acts(800 + i, k) for i in range(150)]
    xds = [to_dev(x)[0] for x in xs]
    ys = [dev_y(m) for _ in xs]
    empty = torch.empty(0, dtype=torch.float32, device="cuda")
    with L.batch():
        for i, (xd, y) in enumerate(zip(xds, ys)):
            L.quantizeDequantGemvI4Q8(wd, sd, 32, xd, y)
            if i == 70:  # no rows: nothing to queue
                L.quantizeDequantGemvI4Q8(wd[:0], sd[:0], 32, xd, empty)
    for x, y in zip(xs, ys):
        q, sc = O.quantizeQ8_0Split(x)
        assert_bits(to_host(y), O.dequantGemvI4Q8(w, s, 32, q, sc))


def test_batch_replayed_from_cuda_graph():
    """The decode-loop form: a batch captured once (after an eager batch of
    the same calls), replayed with new activations copied in."""
    shapes = [(4800, 4096), (512, 11008), (4800, 4096), (512, 11008)]
    cs = cases(i4_case, shapes, seed=900)
    ys = [dev_y(c[0]) for c in cs]

    def step():
        with L.batch():
            for c, y in zip(cs, ys):
                L.quantizeDequantGemvI4Q8(c[5], c[6], 32, c[7], y)

    step()
    torch.cuda.synchronize()
    s = torch.cuda.Stream()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        with torch.cuda.graph(g, stream=s):
            step()
    new_x = [acts(950 + i, c[1]) for i, c in enumerate(cs)]
    for c, x in zip(cs, new_x):
        c[7].copy_(torch.from_numpy(x))
    for y in ys:
        y.fill_(float("nan"))
    g.replay()
    torch.cuda.synchronize()
    for c, x, y in zip(cs, new_x, ys):
        q, sc = O.quantizeQ8_0Split(x)
        assert_bits(to_host(y), O.dequantGemvI4Q8(c[2], c[3], 32, q, sc))
    del g


def test_batch_on_page_locked_host_buffers():
    """The decode-loop form: activations and outputs in page-locked host
    memory, passed by their device addresses (lp_host_device_pointer) to
    queued calls -- the images kernel reads x over the host link and the
    folds write y there -- give the device-buffer bits."""
    shapes = [(4800, 4096), (512, 11008), (300, 4096)]
    cs = cases(i4_case, shapes, seed=1200)
    xh = [torch.from_numpy(c[4]).pin_memory() for c in cs]
    yh = [torch.full((c[0],), float("nan"), dtype=torch.float32).pin_memory() for c in cs]
    xdev = [N.host_device_pointer(t.data_ptr()) for t in xh]
    ydev = [N.host_device_pointer(t.data_ptr()) for t in yh]
    lib = N.lib()
    st = torch.cuda.current_stream().cuda_stream
    with L.batch():
        for c, xa, ya in zip(cs, xdev, ydev):
            m, k, wd, sd = c[0], c[1], c[5], c[6]
            N.check(lib.lp_quantize_dequant_gemv_i4q8(wd.data_ptr(), wd.numel(), sd.data_ptr(),
                                                      sd.numel(), 32, xa, k, ya, m, st), "gemv")
    torch.cuda.synchronize()
    for c, y in zip(cs, yh):
        yd = dev_y(c[0])
        L.quantizeDequantGemvI4Q8(c[5], c[6], 32, c[7], yd)
        assert_bits(y.numpy(), to_host(yd))


# ---- fp32-activation formats: exact mode bit for bit, fast mode in tolerance

FP32_SHAPES = [(7, 4096), (300, 11008), (4800, 4096), (149, 64), (2, 96), (1000, 2048)]


def fp32_jobs(seed, shapes=FP32_SHAPES):
    """One call per (shape, format): the three group formats (gs 32) and the
    two ggml block formats, each with its oracle and dequantized values."""
    from test_gpu_fast_fp32 import vals_blocks, vals_f4, vals_i4, vals_i8
    jobs = []
    for i, (m, k) in enumerate(shapes):
        w = weights(seed + i, m * k)
        x = acts(seed + 100 + i, k)
        s8 = O.calibrateSymmetric(w, 32, 127.0)
        q8 = O.quantize(w, s8, 32, "i8")
        s4 = O.calibrateSymmetric(w, 32, 7.0)
        p4 = O.packInt4(O.quantize(w, s4, 32, "i4"))
        sm = O.calibrateMX(w, 32, 2)
        pf = O.packF4(O.quantize(w, sm, 32, "f4"))
        b8 = O.quantizeQ8_0(w).reshape(-1)
        b4 = O.quantizeQ4_0(w).reshape(-1)
        xd = to_dev(x)[0]
        for fn, args, ofn, vals in (
                (L.dequantGemv, (q8, s8), lambda a=q8, b=s8, x=x: O.dequantGemv(a, b, 32, x),
                 lambda a=q8, b=s8, k=k: vals_i8(a, b, 32, k)),
                (L.dequantGemvI4, (p4, s4), lambda a=p4, b=s4, x=x: O.dequantGemvI4(a, b, 32, x),
                 lambda a=p4, b=s4, k=k: vals_i4(a, b, 32, k)),
                (L.dequantGemvF4, (pf, sm), lambda a=pf, b=sm, x=x: O.dequantGemvF4(a, b, 32, x),
                 lambda a=pf, b=sm, k=k: vals_f4(a, b, 32, k)),
                (L.dequantGemvQ8_0, (b8,), lambda a=b8, x=x, k=k: O.dequantGemvQ8_0(a, k // 32, x),
                 lambda a=b8, k=k: vals_blocks(a, k, False)),
                (L.dequantGemvQ4_0, (b4,), lambda a=b4, x=x, k=k: O.dequantGemvQ4_0(a, k // 32, x),
                 lambda a=b4, k=k: vals_blocks(a, k, True))):
            dev = to_dev(*args)
            call = ((lambda y, fn=fn, d=dev, xd=xd: fn(d[0], d[1], 32, xd, y)) if len(dev) == 2
                    else (lambda y, fn=fn, d=dev, xd=xd, k=k: fn(d[0], k // 32, xd, y)))
            jobs.append((m, x, call, ofn, vals))
    return jobs


def run_batched(jobs):
    """Each job's lone result, then all jobs in one batch (formats
    interleaved, then grouped: every format switch launches the queue)."""
    lone = []
    for m, _, call, _, _ in jobs:
        y = dev_y(m)
        call(y)
        lone.append(to_host(y))
    order = list(range(len(jobs)))
    order = order + sorted(order, key=lambda i: i % 5)
    ys = [dev_y(jobs[i][0]) for i in order]
    with L.batch():
        for i, y in zip(order, ys):
            jobs[i][2](y)
    return lone, [(i, to_host(y)) for i, y in zip(order, ys)]


def test_batch_fp32_exact_formats_equal_lone_calls_and_oracle():
    jobs = fp32_jobs(1500)
    with L.fp32_mode("exact"):
        lone, got = run_batched(jobs)
    for i, y in got:
        assert_bits(y, lone[i])
        assert_bits(y, jobs[i][3]())


def test_batch_fp32_fast_formats_within_tolerance():
    """The block-float fold is unordered, and its order follows the launch's
    tiles, so a batched call may differ from the lone call in the last bits:
    both are held to the fast-mode bound against the oracle."""
    from test_gpu_fast_fp32 import assert_close
    jobs = fp32_jobs(1600)
    with L.fp32_mode("fast"):
        lone, got = run_batched(jobs)
    for i, y in got:
        m, x, _, ofn, vals = jobs[i]
        ref, wv = ofn(), vals()
        assert_close(lone[i], ref, wv, x)
        assert_close(y, ref, wv, x)


@pytest.mark.parametrize("kind", ["q4_k", "q6_k"])
def test_batch_kquant_gemvs_within_tolerance(kind):
    from test_gpu_kquant_gemv import q4k_min_magnitude, rand_blocks
    rng = np.random.default_rng(1700 + (7 if kind == "q6_k" else 0))
    bb, dpos = (144, (0, 2)) if kind == "q4_k" else (210, (208,))
    fn = L.dequantGemvQ4_K if kind == "q4_k" else L.dequantGemvQ6_K
    cs = []
    for M, sbpr in ((37, 16), (4096, 16), (300, 43), (11008, 16)):
        raw = rand_blocks(rng, M * sbpr, bb, dpos)
        K = 256 * sbpr
        x = rng.standard_normal(K).astype(np.float32)
        deq = (O.dequantizeQ4_K if kind == "q4_k" else O.dequantizeQ6_K)(raw.reshape(-1))
        W = deq.reshape(M, K).astype(np.float64)
        bound = np.abs(W) @ np.abs(x.astype(np.float64))
        if kind == "q4_k":
            xg = np.abs(x.astype(np.float64)).reshape(-1, 32).sum(1)
            bound = bound + q4k_min_magnitude(raw, M, sbpr) @ xg
        cs.append((M, sbpr, W @ x.astype(np.float64), bound,
                   torch.from_numpy(raw.reshape(-1)).cuda(), torch.from_numpy(x).cuda()))
    ys = [dev_y(c[0]) for c in cs]
    with L.batch():
        for c, y in zip(cs, ys):
            fn(c[4], c[1], c[5], y)
    for c, y in zip(cs, ys):
        got = to_host(y).astype(np.float64)
        assert np.all(np.abs(got - c[2]) <= 2e-6 * c[3]), np.max(np.abs(got - c[2]) / c[3])
