// gemm.cu -- dequantGemmQ8 / dequantGemmI4Q8 (simd/dequant.nim:1382-1583),
// CUDA-core form.
//
// y[row*n + c] = fold_g (f32(isum_{row,c,g}) * ws[row,g]) * xs[c,g], serial
// over g from 0.0 (scalar path :1449-1458) -- each output column is the
// dequantGemvQ8 arithmetic on that column, bit for bit.  Here every thread
// owns a 4 x 2 tile of outputs and walks K in order, so the fold is
// sequential inside the thread; weights and activations of a K chunk are
// staged in shared memory and shared by the CTA's 64 rows x 32 columns.
// Packed int4 weights are widened to int8 while staging.
#include <algorithm>

#include "lp_device.cuh"
#include "lp_internal.h"

namespace lp {
namespace {

constexpr int TM = 64, TN = 32, kThreads = 256;
constexpr int RPT = 4, CPT = 2;  // rows / columns per thread

struct GemmArgs {
  const uint8_t* w;
  int packed;
  const float* ws;
  const int8_t* xq;
  const float* xs;
  float* y;
  int m, k, n, gs, gpr, kc, gpc;  // kc: K chunk (multiple of gs), gpc = kc / gs
};

__global__ void __launch_bounds__(kThreads) k_gemm_dp4a(const GemmArgs a) {
  extern __shared__ __align__(16) uint8_t sm[];
  const int ldk = a.kc + 4;  // row pitch in bytes (word pad: conflict-free)
  int8_t* Ws = reinterpret_cast<int8_t*>(sm);
  int8_t* Xs = Ws + TM * ldk;
  float* WSs = reinterpret_cast<float*>(Xs + TN * ldk);
  float* XSs = WSs + TM * a.gpc;

  const int tid = threadIdx.x;
  const int ty = tid / 16, tx = tid % 16;
  const int row0 = blockIdx.y * TM, col0 = blockIdx.x * TN;
  float tot[RPT][CPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i)
#pragma unroll
    for (int j = 0; j < CPT; ++j) tot[i][j] = 0.0f;

  const int row_bytes = a.packed ? a.k / 2 : a.k;
  for (int k0 = 0; k0 < a.k; k0 += a.kc) {
    const int kc = min(a.kc, a.k - k0);
    const int gc = kc / a.gs;
    // stage weights (widen int4), activations and scales
    for (int idx = tid; idx < TM * kc; idx += kThreads) {
      const int r = idx / kc, e = idx - r * kc;
      const int row = row0 + r;
      int8_t v = 0;
      if (row < a.m) {
        const int kk = k0 + e;
        if (a.packed) {
          const uint32_t b = a.w[static_cast<int64_t>(row) * row_bytes + (kk >> 1)];
          const int nb = static_cast<int>((kk & 1) ? (b >> 4) : (b & 15u));
          v = static_cast<int8_t>(nb >= 8 ? nb - 16 : nb);
        } else {
          v = static_cast<int8_t>(a.w[static_cast<int64_t>(row) * row_bytes + kk]);
        }
      }
      Ws[r * ldk + e] = v;
    }
    for (int idx = tid; idx < TN * kc; idx += kThreads) {
      const int c = idx / kc, e = idx - c * kc;
      const int col = col0 + c;
      Xs[c * ldk + e] = col < a.n ? a.xq[static_cast<int64_t>(col) * a.k + k0 + e] : 0;
    }
    for (int idx = tid; idx < TM * gc; idx += kThreads) {
      const int r = idx / gc, g = idx - r * gc;
      const int row = row0 + r;
      WSs[r * a.gpc + g] = row < a.m ? a.ws[static_cast<int64_t>(row) * a.gpr + k0 / a.gs + g] : 0.0f;
    }
    for (int idx = tid; idx < TN * gc; idx += kThreads) {
      const int c = idx / gc, g = idx - c * gc;
      const int col = col0 + c;
      XSs[c * a.gpc + g] = col < a.n ? a.xs[static_cast<int64_t>(col) * a.gpr + k0 / a.gs + g] : 0.0f;
    }
    __syncthreads();
    for (int g = 0; g < gc; ++g) {
      int isum[RPT][CPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i)
#pragma unroll
        for (int j = 0; j < CPT; ++j) isum[i][j] = 0;
      const int e0 = g * a.gs;
      if ((a.gs & 3) == 0) {
        for (int e = e0; e < e0 + a.gs; e += 4) {
          uint32_t wv[RPT], xv[CPT];
#pragma unroll
          for (int i = 0; i < RPT; ++i)
            wv[i] = *reinterpret_cast<const uint32_t*>(Ws + (ty * RPT + i) * ldk + e);
#pragma unroll
          for (int j = 0; j < CPT; ++j)
            xv[j] = *reinterpret_cast<const uint32_t*>(Xs + (tx * CPT + j) * ldk + e);
#pragma unroll
          for (int i = 0; i < RPT; ++i)
#pragma unroll
            for (int j = 0; j < CPT; ++j) isum[i][j] = dp4a_ss(wv[i], xv[j], isum[i][j]);
        }
      } else {
        for (int e = e0; e < e0 + a.gs; ++e)
#pragma unroll
          for (int i = 0; i < RPT; ++i)
#pragma unroll
            for (int j = 0; j < CPT; ++j)
              isum[i][j] += static_cast<int>(Ws[(ty * RPT + i) * ldk + e]) *
                            static_cast<int>(Xs[(tx * CPT + j) * ldk + e]);
      }
#pragma unroll
      for (int i = 0; i < RPT; ++i) {
        const float wsv = WSs[(ty * RPT + i) * a.gpc + g];
#pragma unroll
        for (int j = 0; j < CPT; ++j) {
          const float t = fmul(fmul(i2f_rn(isum[i][j]), wsv), XSs[(tx * CPT + j) * a.gpc + g]);
          tot[i][j] = fadd(tot[i][j], t);
        }
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    const int row = row0 + ty * RPT + i;
    if (row >= a.m) continue;
#pragma unroll
    for (int j = 0; j < CPT; ++j) {
      const int col = col0 + tx * CPT + j;
      if (col < a.n) a.y[static_cast<int64_t>(row) * a.n + col] = tot[i][j];
    }
  }
}

}  // namespace

int launch_gemm(const uint8_t* w, int packed_i4, const float* ws, int64_t gs, const int8_t* xq,
                const float* xs, int64_t n, float* y, int64_t m, int64_t k, cudaStream_t st) {
  if (m == 0 || n == 0) return LP_OK;
  GemmArgs a;
  a.w = w;
  a.packed = packed_i4;
  a.ws = ws;
  a.xq = xq;
  a.xs = xs;
  a.y = y;
  a.m = static_cast<int>(m);
  a.k = static_cast<int>(k);
  a.n = static_cast<int>(n);
  a.gs = static_cast<int>(gs);
  a.gpr = static_cast<int>(k / gs);
  a.gpc = std::max(1, 128 / a.gs);
  a.kc = a.gpc * a.gs;
  if (a.kc > 1024) return LP_ERR_UNSUPPORTED;
  const int ldk = a.kc + 4;
  const size_t smem = static_cast<size_t>(TM + TN) * ldk + static_cast<size_t>(TM + TN) * a.gpc * 4;
  static bool attr_set[kMaxDevices] = {};
  const DeviceInfo& di = device_info();
  if (!attr_set[di.ordinal % kMaxDevices]) {
    cudaFuncAttributes fa;
    int lim = di.max_smem_optin;
    if (cudaFuncGetAttributes(&fa, k_gemm_dp4a) == cudaSuccess) lim -= static_cast<int>(fa.sharedSizeBytes);
    cudaFuncSetAttribute(k_gemm_dp4a, cudaFuncAttributeMaxDynamicSharedMemorySize, lim);
    attr_set[di.ordinal % kMaxDevices] = true;
  }
  if (a.k == 0) {
    // no groups: every output is the empty fold, 0.0
    return cuda_status(cudaMemsetAsync(y, 0, static_cast<size_t>(m * n) * 4, st));
  }
  dim3 grid(static_cast<unsigned>((n + TN - 1) / TN), static_cast<unsigned>((m + TM - 1) / TM));
  k_gemm_dp4a<<<grid, kThreads, smem, st>>>(a);
  return cuda_status(cudaGetLastError());
}

}  // namespace lp
