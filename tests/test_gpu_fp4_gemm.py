"""FP4 x FP4 GEMMs on the block-scaled tensor cores (gemm_fp4.cu) against the
fp64 oracle (oracle/lowprec_oracle.c: lpo_gemm_fp4).

MXFP4 (tcgen05 kind::mxf4): weights and activations both encoded on the GPU by
calibrateMX + packF4 (quant.nim:112-137, mxfloat.nim:52-66, 138-149; bit-exact
encoders checked elsewhere).  NVFP4 (kind::mxf4nvf4): both operands encoded by
quantizeNVFP4 (nvfp4.nim:39-78), codes packed two per byte.

Tolerance: the products of e2m1 values and power-of-two (or e4m3) scales are
exact in the tensor core; only the fp32 sums round, so every output must be
within 1e-6 * sum_i |w_i x_i| of the exact (fp64) value -- the bound the
block-float GEMV tests use.  Shapes cover a ragged row tile (m % 128 != 0), a
ragged column tile (n % 64 != 0), K not a multiple of the 256-element stage,
and both column tiles (64 and 128)."""
import numpy as np
import pytest

from gpu_util import F
from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402

E2M1 = np.array([0, .5, 1, 1.5, 2, 3, 4, 6, 0, -.5, -1, -1.5, -2, -3, -4, -6], np.float64)


def decode_packed(packed, rows, k):
    p = packed.reshape(rows, k // 2)
    v = np.empty((rows, k), np.float64)
    v[:, 0::2] = E2M1[p & 15]
    v[:, 1::2] = E2M1[p >> 4]
    return v


def mx_encode(t, rows, k):
    """calibrateMX + packF4 on the GPU: (packed codes, fp32 scales)."""
    sc = torch.empty(rows * k // 32, dtype=torch.float32, device="cuda")
    L.calibrateMX(t, 32, 2, sc)
    pk = torch.empty(rows * k // 2, dtype=torch.uint8, device="cuda")
    L.quantizeF4Packed(t, sc, 32, pk)
    return pk, sc


@pytest.mark.parametrize("m,k,n", [(128, 256, 8), (256, 512, 64), (300, 1024, 70),
                                   (200, 288, 130), (4096, 4096, 64), (1024, 2048, 512)])
def test_mxfp4_gemm_vs_fp64_oracle(m, k, n):
    g = torch.Generator(device="cuda").manual_seed(m + 7 * n + k)
    w = torch.randn(m * k, generator=g, device="cuda") * 0.02
    x = torch.randn(n * k, generator=g, device="cuda")
    wp, ws = mx_encode(w, m, k)
    xp, xs = mx_encode(x, n, k)
    y = torch.full((m * n,), float("nan"), device="cuda")
    L.dequantGemmF4(wp, ws, 32, xp, xs, n, y)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    wph, wsh, xph, xsh = (t.cpu().numpy() for t in (wp, ws, xp, xs))
    if m * n * k <= 300 * 70 * 1024:
        want = O.gemmFp4(wph, wsh, xph, xsh, n)
    else:  # same exact arithmetic, vectorised
        W = decode_packed(wph, m, k) * np.repeat(wsh.reshape(m, -1).astype(np.float64), 32, 1)
        X = decode_packed(xph, n, k) * np.repeat(xsh.reshape(n, -1).astype(np.float64), 32, 1)
        want = (W @ X.T).reshape(-1)
    W = decode_packed(wph, m, k) * np.repeat(wsh.reshape(m, -1).astype(np.float64), 32, 1)
    X = decode_packed(xph, n, k) * np.repeat(xsh.reshape(n, -1).astype(np.float64), 32, 1)
    absdot = (np.abs(W) @ np.abs(X).T).reshape(-1)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - want) <= 1e-6 * absdot + 1e-30)
    assert N.device_error() == 0


def test_mxfp4_gemm_one_column_is_dequant_gemv_f4_of_the_decoded_activations():
    """n = 1: the GEMM equals dequantGemvF4 (the reference proc, exact fp32
    mode here) applied to the MXFP4-decoded activation vector, within the
    rounding of the two summation orders."""
    m, k = 512, 4096
    g = torch.Generator(device="cuda").manual_seed(3)
    w = torch.randn(m * k, generator=g, device="cuda") * 0.02
    x = torch.randn(k, generator=g, device="cuda")
    wp, ws = mx_encode(w, m, k)
    xp, xs = mx_encode(x, 1, k)
    xdec = torch.from_numpy((decode_packed(xp.cpu().numpy(), 1, k).reshape(-1)
                             * np.repeat(xs.cpu().numpy().astype(np.float64), 32)).astype(F)).cuda()
    y = torch.empty(m, device="cuda")
    L.dequantGemmF4(wp, ws, 32, xp, xs, 1, y)
    yv = torch.empty(m, device="cuda")
    with L.fp32_mode("exact"):
        L.dequantGemvF4(wp, ws, 32, xdec, yv)
    want = O.dequantGemvF4(wp.cpu().numpy(), ws.cpu().numpy(), 32, xdec.cpu().numpy())
    assert np.array_equal(yv.cpu().numpy().view(np.uint32), want.view(np.uint32))
    W = decode_packed(wp.cpu().numpy(), m, k) * np.repeat(ws.cpu().numpy().reshape(m, -1).astype(np.float64), 32, 1)
    absdot = np.abs(W) @ np.abs(xdec.cpu().numpy().astype(np.float64))
    assert np.all(np.abs(y.cpu().numpy().astype(np.float64) - want) <= 2e-6 * absdot)


def nv_encode(t):
    """quantizeNVFP4 on the GPU, codes packed two per byte."""
    n = t.numel()
    codes = torch.empty(n, dtype=torch.uint8, device="cuda")
    bs = torch.empty(n // 16, dtype=torch.uint8, device="cuda")
    gds = torch.empty(1, dtype=torch.float32, device="cuda")
    L.quantizeNVFP4(t, codes, bs, gds)
    packed = (codes[0::2] | (codes[1::2] << 4)).contiguous()
    return packed, bs, gds, codes


@pytest.mark.parametrize("m,k,n", [(128, 256, 8), (300, 1024, 70), (200, 288, 130),
                                   (2048, 2048, 64)])
def test_nvfp4_gemm_vs_fp64_oracle(m, k, n):
    g = torch.Generator(device="cuda").manual_seed(11 * m + n + k)
    w = torch.randn(m * k, generator=g, device="cuda") * 0.02
    x = torch.randn(n * k, generator=g, device="cuda")
    wp, wbs, wg, wcodes = nv_encode(w)
    xp, xbs, xg, xcodes = nv_encode(x)
    y = torch.full((m * n,), float("nan"), device="cuda")
    L.gemmNVFP4(wp, wbs, wg, xp, xbs, xg, n, y)
    torch.cuda.synchronize()
    got = y.cpu().numpy().astype(np.float64)
    G = float(wg.item()) * float(xg.item())
    wph, wbh, xph, xbh = (t.cpu().numpy() for t in (wp, wbs, xp, xbs))
    want = O.gemmFp4(wph, wbh, xph, xbh, n, nvfp4=True, globalScale=G)
    # the reference's own decode of each operand (nvfp4.nim:80-92), in fp64
    Wd = O.dequantizeNVFP4(wcodes.cpu().numpy(), wbh, float(wg.item())).astype(np.float64)
    Xd = O.dequantizeNVFP4(xcodes.cpu().numpy(), xbh, float(xg.item())).astype(np.float64)
    absdot = (np.abs(Wd.reshape(m, k)) @ np.abs(Xd.reshape(n, k)).T).reshape(-1)
    assert np.all(np.isfinite(got))
    assert np.all(np.abs(got - want) <= 1e-6 * absdot + 1e-30)
    # and the exact GEMM of the decoded operands agrees with the oracle
    assert np.all(np.abs((Wd.reshape(m, k) @ Xd.reshape(n, k).T).reshape(-1) - want)
                  <= 1e-6 * absdot + 1e-30)
    assert N.device_error() == 0


def test_fp4_gemms_check_shapes():
    z8 = torch.zeros(64, dtype=torch.uint8, device="cuda")
    zf = torch.zeros(8, dtype=torch.float32, device="cuda")
    y = torch.zeros(4, device="cuda")
    with pytest.raises(AssertionError):  # group size must be the MX block, 32
        L.dequantGemmF4(z8, zf, 16, z8, zf, 1, y)
    with pytest.raises(AssertionError):  # 64 bytes of x are not 3 columns
        L.dequantGemmF4(z8, zf, 32, z8, zf, 3, torch.zeros(3, device="cuda"))
