"""Inputs of nim-lowprec's own hot-path tests, regenerated exactly.

Each generator restates the inline data recipe of a reference test
(file:line cited) so the same inputs can be fed to the oracle and to the CUDA
kernels.  float32 arithmetic is done with numpy float32 scalars (one rounding
per operation, like the reference compiled with -ffp-contract=off).
"""
import numpy as np

F = np.float32
M32 = 0xFFFFFFFF
M64 = 0xFFFFFFFFFFFFFFFF


def xorshift32_bytes(seed, count):
    """test_sdot.nim:66-71: xorshift32 (13,17,5), byte = (u & 0xff) - 128."""
    u = seed
    out = np.empty(count, np.int64)
    for i in range(count):
        u ^= (u << 13) & M32
        u ^= u >> 17
        u ^= (u << 5) & M32
        out[i] = (u & 0xFF) - 128
    return out, u


def sdot_int8_case(M, K, gs):
    """test_sdot.nim:59-90 (dequantGemvQ8 vs intRef)."""
    seq, _ = xorshift32_bytes(2463534242, M * K + K)
    wq = np.maximum(seq[:M * K], -127).astype(np.int8)
    xq = np.maximum(seq[M * K:], -127).astype(np.int8)
    gpr = K // gs
    ws = np.array([F(0.011) + F(i % 5) * F(0.0013) for i in range(M * gpr)], F)
    xs = np.array([F(0.023) + F(i % 3) * F(0.0007) for i in range(gpr)], F)
    return wq, ws, xq, xs


SDOT_INT8_SHAPES = [(7, 96, 32), (4, 96, 96), (1, 96, 32), (9, 40, 20)]
SDOT_INT4_SHAPES = [(7, 128, 64), (4, 128, 128), (1, 128, 64), (5, 96, 48)]


def sdot_int4_case(M, K, gs):
    """test_sdot.nim:92-127 (dequantGemvI4Q8 vs intRef over unpacked int4)."""
    u = 88172645463325252

    def step(u):
        u ^= (u << 13) & M64
        u ^= u >> 7
        u ^= (u << 17) & M64
        return u

    vals = np.empty(M * K, np.int8)
    for i in range(M * K):
        u = step(u)
        vals[i] = (u & 0x0F) - 8
    xq = np.empty(K, np.int8)
    for i in range(K):
        u = step(u)
        xq[i] = max((u & 0xFF) - 128, -127)
    gpr = K // gs
    ws = np.array([F(0.017) + F(i % 4) * F(0.0011) for i in range(M * gpr)], F)
    xs = np.array([F(0.031) + F(i % 3) * F(0.0005) for i in range(gpr)], F)
    return vals, ws, xq, xs


def pack_i4_values(vals):
    """test_sdot.nim:41-48 packI4: low nibble = even column."""
    v = (vals.astype(np.int16) & 0x0F).astype(np.uint8)
    return (v[0::2] | (v[1::2] << 4)).astype(np.uint8)


def f16_bits(x):
    return np.array([x], F).astype(np.float16).view(np.uint16)[0]


def ggml_x_blocks(bpr):
    """test_sdot.nim:201-206 mkX: activation Q8_0 blocks."""
    out = np.zeros((bpr, 34), np.uint8)
    for b in range(bpr):
        d = f16_bits(F(0.031) + F(b % 5) * F(0.0017))
        out[b, 0:2] = np.array([d], np.uint16).view(np.uint8)
        out[b, 2:] = np.array([((b * 29 + i * 13) % 255) - 127 for i in range(32)], np.int8).view(np.uint8)
    return out


def ggml_q8_w_blocks(M, bpr):
    """test_sdot.nim:208-215."""
    out = np.zeros((M * bpr, 34), np.uint8)
    for b in range(M * bpr):
        d = f16_bits(F((b % 9) - 4) * F(0.011) + F(0.003))
        out[b, 0:2] = np.array([d], np.uint16).view(np.uint8)
        out[b, 2:] = np.array([((b * 17 + i * 11) % 255) - 127 for i in range(32)], np.int8).view(np.uint8)
    return out


def ggml_q4_w_blocks(M, bpr):
    """test_sdot.nim:227-233."""
    out = np.zeros((M * bpr, 18), np.uint8)
    for b in range(M * bpr):
        d = f16_bits(F((b % 7) - 3) * F(0.013) + F(0.002))
        out[b, 0:2] = np.array([d], np.uint16).view(np.uint8)
        out[b, 2:] = np.array([(b * 23 + i * 19) & 0xFF for i in range(16)], np.uint8)
    return out


GGML_SHAPES = [(5, 12), (4, 7), (1, 4), (3, 3)]

GEMM_I8_SHAPES = [(9, 128, 64, 3), (4, 256, 128, 2), (5, 96, 48, 1), (6, 80, 40, 4)]
GEMM_I4_SHAPES = [(9, 128, 64, 3), (4, 256, 128, 2), (5, 192, 96, 1), (6, 160, 80, 4)]


def gemm_int8_case(M, K, gs, n):
    """test_sdot.nim:249-266."""
    gpr = K // gs
    wq = np.array([((i * 37) % 251) - 125 for i in range(M * K)], np.int8)
    xq = np.array([((i * 41) % 241) - 120 for i in range(n * K)], np.int8)
    ws = np.array([F(0.012) + F(i % 6) * F(0.0009) for i in range(M * gpr)], F)
    xs = np.array([F(0.021) + F(i % 4) * F(0.0013) for i in range(n * gpr)], F)
    return wq, ws, xq, xs


def gemm_int4_case(M, K, gs, n):
    """test_sdot.nim:286-302."""
    gpr = K // gs
    wp = np.array([(i * 29 + 5) & 0xFF for i in range(M * (K // 2))], np.uint8)
    xq = np.array([((i * 43) % 239) - 119 for i in range(n * K)], np.int8)
    ws = np.array([F(0.014) + F(i % 5) * F(0.0011) for i in range(M * gpr)], F)
    xs = np.array([F(0.019) + F(i % 3) * F(0.0017) for i in range(n * gpr)], F)
    return wp, ws, xq, xs


# ---------------------------------------------------- test_parallel.nim --

PAR_K = 512
PAR_GS = 64
PAR_ROWS = [300, 64, 1]
PAR_THREADS = [0, 1, 2, 3, 64]


def par_x():
    """test_parallel.nim:22-27: LCG x in [-1, 1)."""
    u = 7919
    x = np.empty(PAR_K, F)
    for i in range(PAR_K):
        u = (u * 1664525 + 1013904223) & M32
        x[i] = F(u >> 16) / F(32768.0) - F(1.0)
    return x


def par_int8(M):
    """test_parallel.nim:48-56."""
    gpr = PAR_K // PAR_GS
    wq = np.array([(i % 15) - 7 for i in range(M * PAR_K)], np.int8)
    sc = np.array([F(0.02) + F(i % 3) * F(0.001) for i in range(M * gpr)], F)
    return wq, sc


def par_int4(M):
    """test_parallel.nim:58-67."""
    gpr = PAR_K // PAR_GS
    w4 = np.array([(i * 7 + 3) & 0xFF for i in range(M * PAR_K // 2)], np.uint8)
    sc = np.array([F(0.02) + F(i % 3) * F(0.001) for i in range(M * gpr)], F)
    return w4, sc


def par_f4(M):
    """test_parallel.nim:69-80 (scales = toFloat32(toE8M0(0.03125)) = 0.03125)."""
    gpr = PAR_K // PAR_GS
    wf4 = np.array([(i * 11 + 5) & 0xFF for i in range(M * PAR_K // 2)], np.uint8)
    sc = np.full(M * gpr, F(0.03125), F)
    return wf4, sc


def par_q8_0(M):
    """test_parallel.nim:82-90."""
    bpr = PAR_K // 32
    out = np.zeros((M * bpr, 34), np.uint8)
    for b in range(M * bpr):
        d = f16_bits(F(0.0125) + F(b % 3) * F(0.001))
        out[b, 0:2] = np.array([d], np.uint16).view(np.uint8)
        out[b, 2:] = np.array([((b + i) % 255) - 127 for i in range(32)], np.int8).view(np.uint8)
    return out, bpr


def par_q4_0(M):
    """test_parallel.nim:92-100."""
    bpr = PAR_K // 32
    out = np.zeros((M * bpr, 18), np.uint8)
    for b in range(M * bpr):
        d = f16_bits(F(0.0125) + F(b % 3) * F(0.001))
        out[b, 0:2] = np.array([d], np.uint16).view(np.uint8)
        out[b, 2:] = np.array([(b * 7 + i * 11) & 0xFF for i in range(16)], np.uint8)
    return out, bpr


def pooled_case(M, n=1):
    """test_parallel.nim:114-131 and :176-194 (gs 64, pooled int8-act forms)."""
    gpr = PAR_K // PAR_GS
    wq = np.array([(i % 200) - 100 for i in range(M * PAR_K)], np.int8)
    w4 = np.array([(i * 13 + 7) & 0xFF for i in range(M * PAR_K // 2)], np.uint8)
    ws = np.array([F(0.019) + F(i % 4) * F(0.0007) for i in range(M * gpr)], F)
    xq = np.array([(i % 150) - 75 for i in range(n * PAR_K)], np.int8)
    xs = np.array([F(0.027) + F(i % 3) * F(0.0011) for i in range(n * gpr)], F)
    return wq, w4, ws, xq, xs


# ----------------------------------------------- test_quant_simd.nim -----

def next_rnd(u):
    """test_quant_simd.nim:21-25: xorshift32 -> float32 in [-1, 1)."""
    u ^= (u << 13) & M32
    u ^= u >> 17
    u ^= (u << 5) & M32
    return u, F(u >> 8) / F(1 << 24) * F(2.0) - F(1.0)
