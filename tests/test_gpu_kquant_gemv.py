"""Fused GEMVs over GGUF k-quant super-blocks (Q4_K, Q6_K) against the
reference's own element values: the oracle's dequantizeQ4_K / dequantizeQ6_K
(ggml.nim:136-161, 163-213, pinned to gguf-py goldens elsewhere), then an fp64
product.  The reference has no fused k-quant GEMV, so the bar is tolerance:
each row within 1e-6 of sum_i (|d*sc*q_i| + |dmin*m|) |x_i| (the block-float
bound of the fp32 GEMVs; the Q4_K minimum term is carried separately, so its
magnitude enters the bound)."""
import numpy as np
import pytest

from oracle import oracle as O

pytestmark = pytest.mark.gpu

torch = pytest.importorskip("torch")
if not torch.cuda.is_available():  # pragma: no cover
    pytest.skip("no CUDA device", allow_module_level=True)

import nim_lowprec_b200 as L  # noqa: E402
from nim_lowprec_b200 import _native as N  # noqa: E402


def rand_blocks(rng, nb, bb, dpos):
    raw = rng.integers(0, 256, (nb, bb), dtype=np.uint8)
    for p in dpos:  # finite f16 super-block scales
        raw[:, p:p + 2] = (rng.standard_normal(nb).astype(np.float32) * 0.01).astype(
            np.float16).view(np.uint8).reshape(nb, 2)
    return raw


def q4k_min_magnitude(raw, M, sbpr):
    """|dmin * m| per 32-element group (get_scale_min_k4, ggml.nim:118-128)."""
    dmin = raw[:, 2:4].copy().view(np.float16).astype(np.float64).reshape(-1)
    q = raw[:, 4:16].astype(np.int64)
    m = np.empty((raw.shape[0], 8), np.int64)
    for j in range(8):
        m[:, j] = (q[:, j + 4] & 63) if j < 4 else ((q[:, j + 4] >> 4) | ((q[:, j] >> 6) << 4))
    return np.abs(dmin[:, None] * m).reshape(M, sbpr * 8)


@pytest.mark.parametrize("kind,M,sbpr", [("q4_k", 37, 4), ("q4_k", 4096, 16), ("q6_k", 37, 4),
                                         ("q6_k", 4096, 16), ("q4_k", 300, 43), ("q6_k", 300, 43)])
def test_kquant_gemv_vs_dequantized_oracle(kind, M, sbpr):
    rng = np.random.default_rng(M + sbpr + (7 if kind == "q6_k" else 0))
    bb, dpos = (144, (0, 2)) if kind == "q4_k" else (210, (208,))
    raw = rand_blocks(rng, M * sbpr, bb, dpos)
    K = 256 * sbpr
    x = rng.standard_normal(K).astype(np.float32)
    x[:32] *= np.float32(2.0 ** 100)  # one group takes the sequential path
    deq = (O.dequantizeQ4_K if kind == "q4_k" else O.dequantizeQ6_K)(raw.reshape(-1))
    W = deq.reshape(M, K).astype(np.float64)
    want = W @ x.astype(np.float64)
    bound = np.abs(W) @ np.abs(x.astype(np.float64))
    if kind == "q4_k":
        mm = q4k_min_magnitude(raw, M, sbpr)
        xg = np.abs(x.astype(np.float64)).reshape(-1, 32).sum(1)
        bound = bound + mm @ xg
    wd = torch.from_numpy(raw.reshape(-1)).cuda()
    xd = torch.from_numpy(x).cuda()
    y = torch.full((M,), float("nan"), device="cuda")
    fn = L.dequantGemvQ4_K if kind == "q4_k" else L.dequantGemvQ6_K
    for mode in ("fast", "exact"):  # the same arithmetic in both fp32 modes
        with L.fp32_mode(mode):
            fn(wd, sbpr, xd, y)
        got = y.cpu().numpy().astype(np.float64)
        assert np.all(np.isfinite(got))
        assert np.all(np.abs(got - want) <= 2e-6 * bound), (mode, np.max(np.abs(got - want) / bound))
    assert N.device_error() == 0


def test_kquant_gemv_shape_checks():
    w = torch.zeros(144 * 6, dtype=torch.uint8, device="cuda")
    x = torch.zeros(512, device="cuda")
    with pytest.raises(AssertionError):  # 6 super-blocks are not 4 rows of 2
        L.dequantGemvQ4_K(w, 2, x, torch.zeros(4, device="cuda"))
