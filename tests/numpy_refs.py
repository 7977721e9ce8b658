"""Independent numpy restatements of the reference tests' exact references.

These mirror the reference's *test-side* references (not its kernels):
``intRef`` (test_sdot.nim:21-39), ``refQ8``/``refQ4`` (test_sdot.nim:164-199)
and the fp64 references of test_quant_simd.nim:63-245.  float32 arrays keep one
rounding per numpy operation, so the op order below is the exact fp32 order.
A second set restates the scalar fp32-activation kernels' sequential order,
vectorised across rows, as an independent check of the C oracle.
"""
import numpy as np

F = np.float32


def int_ref(wq, ws, gs, xq, xs):
    """test_sdot.nim:21-39: int64 isum -> f32(int32(isum)) * ws * xs, serial."""
    k = xq.size
    m = wq.size // k
    gpr = k // gs
    w = wq.reshape(m, k).astype(np.int64)
    x = xq.astype(np.int64)
    ws = ws.reshape(m, gpr)
    total = np.zeros(m, F)
    for g in range(gpr):
        isum = (w[:, g * gs:(g + 1) * gs] * x[g * gs:(g + 1) * gs]).sum(1)
        term = isum.astype(np.int32).astype(F) * ws[:, g]
        term = term * xs[g]
        total = total + term
    return total


def _blk_d(blocks):
    return blocks[:, 0:2].copy().view(np.uint16).reshape(-1).view(np.float16).astype(F)


def ref_q8(wblocks, bpr, xblocks):
    """test_sdot.nim:164-180 refQ8 (lane discipline)."""
    wb = wblocks.reshape(-1, 34)
    m = wb.shape[0] // bpr
    xb = xblocks.reshape(-1, 34)
    wq = wb[:, 2:].view(np.int8).astype(np.int64).reshape(m, bpr, 32)
    xq = xb[:, 2:].view(np.int8).astype(np.int64)
    wd = _blk_d(wb).reshape(m, bpr)
    xd = _blk_d(xb)
    lanes = np.zeros((m, 4), F)
    for bi in range(bpr):
        isum = (wq[:, bi, :] * xq[bi]).sum(1).astype(np.int32).astype(F)
        dd = wd[:, bi] * xd[bi]
        lanes[:, bi & 3] = lanes[:, bi & 3] + isum * dd
    return (lanes[:, 0] + lanes[:, 1]) + (lanes[:, 2] + lanes[:, 3])


def ref_q4(wblocks, bpr, xblocks):
    """test_sdot.nim:182-199 refQ4."""
    wb = wblocks.reshape(-1, 18)
    m = wb.shape[0] // bpr
    xb = xblocks.reshape(-1, 34)
    qs = wb[:, 2:].astype(np.int64).reshape(m, bpr, 16)
    lo = (qs & 0x0F) - 8
    hi = (qs >> 4) - 8
    xq = xb[:, 2:].view(np.int8).astype(np.int64)
    wd = _blk_d(wb).reshape(m, bpr)
    xd = _blk_d(xb)
    lanes = np.zeros((m, 4), F)
    for bi in range(bpr):
        isum = (lo[:, bi, :] * xq[bi, :16]).sum(1) + (hi[:, bi, :] * xq[bi, 16:]).sum(1)
        dd = wd[:, bi] * xd[bi]
        lanes[:, bi & 3] = lanes[:, bi & 3] + isum.astype(np.int32).astype(F) * dd
    return (lanes[:, 0] + lanes[:, 1]) + (lanes[:, 2] + lanes[:, 3])


# ------------------------------------------------ fp32-activation kernels

def _unpack_nibbles(wp, m, k):
    b = wp.reshape(m, k // 2)
    out = np.empty((m, k), np.uint8)
    out[:, 0::2] = b & 0x0F
    out[:, 1::2] = b >> 4
    return out


def seq_gemv(wvals_f32, scales, gs, x, scale_mul=None):
    """Scalar fp32-activation order: partial = sequential sum of w*x inside a
    group, total += partial*s (simd/dequant.nim:253-256 and kin)."""
    m, k = wvals_f32.shape
    gpr = k // gs
    sc = scales.reshape(m, gpr)
    total = np.zeros(m, F)
    for g in range(gpr):
        partial = np.zeros(m, F)
        for kk in range(g * gs, (g + 1) * gs):
            partial = partial + wvals_f32[:, kk] * x[kk]
        s = sc[:, g] if scale_mul is None else sc[:, g] * F(scale_mul)
        total = total + partial * s
    return total


def seq_gemv_i8(wq, scales, gs, x):
    k = x.size
    return seq_gemv(wq.reshape(-1, k).astype(F), scales, gs, x)


def seq_gemv_i4(wp, scales, gs, x):
    k = x.size
    m = wp.size // (k // 2)
    nib = _unpack_nibbles(wp, m, k).astype(np.int16)
    vals = np.where(nib >= 8, nib - 16, nib).astype(F)
    return seq_gemv(vals, scales, gs, x)


LUT2X = np.array([0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12], F)


def seq_gemv_f4(wp, scales, gs, x):
    k = x.size
    m = wp.size // (k // 2)
    vals = LUT2X[_unpack_nibbles(wp, m, k)]
    return seq_gemv(vals, scales, gs, x, scale_mul=0.5)


def seq_gemv_q8_0(blocks, bpr, x):
    wb = blocks.reshape(-1, 34)
    m = wb.shape[0] // bpr
    vals = wb[:, 2:].view(np.int8).astype(F).reshape(m, bpr * 32)
    d = _blk_d(wb)
    return seq_gemv(vals, d, 32, x)


def seq_gemv_q4_0(blocks, bpr, x):
    """Interleaved order of simd/dequant.nim:616-620: (lo_i, x[i]), (hi_i, x[i+16])."""
    wb = blocks.reshape(-1, 18)
    m = wb.shape[0] // bpr
    qs = wb[:, 2:].astype(np.int16).reshape(m, bpr, 16)
    lo = ((qs & 0x0F) - 8).astype(F)
    hi = ((qs >> 4) - 8).astype(F)
    d = _blk_d(wb).reshape(m, bpr)
    total = np.zeros(m, F)
    for bi in range(bpr):
        partial = np.zeros(m, F)
        xb = x[bi * 32:(bi + 1) * 32]
        for i in range(16):
            partial = partial + lo[:, bi, i] * xb[i]
            partial = partial + hi[:, bi, i] * xb[i + 16]
        total = total + partial * d[:, bi]
    return total


def fp64_gemv(wvals, scales, gs, x):
    """fp64 reference of test_quant_simd.nim:63-80."""
    m, k = wvals.shape
    gpr = k // gs
    sc = np.repeat(scales.reshape(m, gpr).astype(np.float64), gs, axis=1)
    return (wvals.astype(np.float64) * sc) @ x.astype(np.float64)


def max_rel(y, ref):
    return float(np.max(np.abs(y.astype(np.float64) - ref) / (np.abs(ref) + 1e-4)))
