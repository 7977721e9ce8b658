// gemm_tc.cu -- dequantGemmQ8 (simd/dequant.nim:1382-1458) on the
// 5th-generation tensor cores: tcgen05.mma kind::i8 fed by TMA, accumulators
// in tensor memory, bit-exact.
//
// y[row*n + c] = fold_g fl(fl(f32(isum) * ws[row,g]) * xs[c,g]), serial over
// the groups g from 0.0 (scalar path :1449-1458); isum is the exact int32 dot
// of a 32-element group, which is what one K = 32 kind::i8 MMA produces.
// Every group needs its own scaling before the in-order fp32 fold, so each
// group's MMA writes its own accumulator slot in TMEM (nothing accumulates
// across groups) and the epilogue folds the slots in group order.
//
// CTA = one 128-row x NT-column output tile over all of K (32-wide groups).
//   warp 0     producer: per K-stage of 4 groups, two TMA tile loads with
//              128-byte swizzle -- weights [128 rows x 128 B] and activations
//              [NT columns x 128 B] (xq is K x n column-major, so both are
//              K-major) -- into a kStages-deep ring.
//   warps 2-3  (dequantGemmI4Q8 only) widen the stage's packed int4 weight
//              tile, loaded by TMA as [128 rows x 64 B], to the int8 A tile
//              in the 128-byte-swizzled layout the MMA reads (two rows per
//              thread), then release it to the MMA issuer.
//   warp 1     owns the TMEM allocation; one lane issues the stage's four
//              MMAs (one per group, M=128, N=NT, K=32) into the four
//              accumulators of TMEM stage slot kb mod ER and commits once to
//              that slot's mbarrier and once to release the smem stage.
//   warps 4-19 epilogue: warp w reads TMEM lanes 32*(w%4).. (its 32 rows) and
//              a quarter of the NT columns, four groups per wait, converts,
//              scales and folds them in order in fp32 registers, releases
//              the slot, and finally writes y.
// Every wait is bounded (lp_device.cuh) and TMEM is freed on every exit path.
#include <cuda.h>

#include <algorithm>
#include <mutex>

#include "lp_internal.h"
#include "tc_ptx.cuh"

namespace lp {
namespace {

constexpr int kKStage = 128;  // K bytes per stage = 4 groups of 32
constexpr int kEpiWarps = 16;  // four per TMEM lane quarter
constexpr int kThreads = 32 * (4 + kEpiWarps);

// Stages: narrow tiles are few (one per 128 rows) and must keep more bytes in
// flight per SM.
template <int NT>
constexpr int stages_for() { return NT <= 16 ? 10 : 8; }

// Tensor-memory columns per CTA: 16-column tiles take half of TMEM, so two
// CTAs can share an SM; wider tiles take all of it.
template <int NT>
constexpr uint32_t tmem_cols() { return NT <= 16 ? 256u : 512u; }

struct TcArgs {
  const float* ws;  // M x gpr
  const float* xs;  // n x gpr
  float* y;         // M x n
  int m, k, n, gpr;
  float neg_zero;   // -0.0f at run time (see mul2_rn)
};

using namespace tc;

// Instruction descriptor: D s32, A s8, B s8, both K-major, N = NT, M = 128.
template <int NT>
constexpr uint32_t idesc_i8() {
  return (2u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(NT >> 3) << 17) |
         (static_cast<uint32_t>(128 >> 4) << 24);
}

// Two's-complement nibbles (low = even column) of a packed word -> the eight
// int8 values in column order: out[0] = columns 0-3, out[1] = columns 4-7.
__device__ __forceinline__ void widen_i4(uint32_t w, uint32_t& o0, uint32_t& o1) {
  uint32_t lo = w & 0x0F0F0F0Fu, hi = (w >> 4) & 0x0F0F0F0Fu;
  lo |= (lo & 0x08080808u) * 0x1Eu;  // sign-extend each byte: n >= 8 -> n - 16
  hi |= (hi & 0x08080808u) * 0x1Eu;
  o0 = prmt(lo, hi, 0x5140u);
  o1 = prmt(lo, hi, 0x7362u);
}

template <int NT, bool I4>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
              const TcArgs a) {
  constexpr int kStages = stages_for<NT>();
  constexpr int COLS = NT / (kEpiWarps / 4);  // columns per epilogue warp
  constexpr uint32_t kTmemCols = tmem_cols<NT>();
  constexpr int ER = static_cast<int>(kTmemCols) / (4 * NT);  // TMEM stage slots
  constexpr int A_BYTES = 128 * kKStage;
  constexpr int B_BYTES = NT * kKStage;
  constexpr int RAW_BYTES = I4 ? 128 * kKStage / 2 : 0;  // packed int4 tile
  constexpr int STAGE = A_BYTES + B_BYTES + RAW_BYTES;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], empty[kStages], cvt[kStages], tfull[ER], tempty[ER], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int s_abort;

  uint8_t* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  float* xsT = reinterpret_cast<float*>(smem + kStages * STAGE);  // [gpr][NT]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * NT, m0 = blockIdx.y * 128;
  const int nkb = a.k / kKStage;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&cvt[s], 2);
    }
    for (int e = 0; e < ER; ++e) {
      mbar_init(&tfull[e], 1);
      mbar_init(&tempty[e], kEpiWarps);
    }
    mbar_init(&mma_done, 1);
    s_abort = 0;
    mbar_fence_init();
  }
  if (warp == 1) tmem_alloc(&tmem_base, kTmemCols);
  fence_before();
  __syncthreads();
  fence_after();
  const uint32_t tbase = tmem_base;

  if (warp == 0) {
    // ------------------------------------------------------ producer
    int kb = 0;
    if (lane == 0) {
      for (; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, &s_abort)) break;
        if (s_abort) break;
        uint8_t* st = smem + s * STAGE;
        mbar_arrive_expect_tx(&full[s], (I4 ? RAW_BYTES : A_BYTES) + B_BYTES);
        if (I4) tma_load_2d(st + A_BYTES + B_BYTES, &tmA, kb * (kKStage / 2), m0, &full[s]);
        else tma_load_2d(st, &tmA, kb * kKStage, m0, &full[s]);
        tma_load_2d(st + A_BYTES, &tmB, kb * kKStage, n0, &full[s]);
      }
      // never leave with a tile still landing in shared memory
      for (int u = max(0, kb - kStages); u < kb; ++u)
        mbar_wait(&full[u % kStages], (u / kStages) & 1);
    }
  } else if (warp == 1) {
    // --------------------------------------------------- MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_i8<NT>();
      for (int kb = 0; kb < nkb && !s_abort; ++kb) {
        const int s = kb % kStages;
        const int e = kb % ER;
        if (!mbar_wait(&full[s], (kb / kStages) & 1, &s_abort)) break;
        if (I4 && !mbar_wait(&cvt[s], (kb / kStages) & 1, &s_abort)) break;
        if (kb >= ER && !mbar_wait(&tempty[e], ((kb / ER) - 1) & 1, &s_abort)) break;
        fence_after();
        const uint8_t* st = smem + s * STAGE;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          mma_i8(tbase + static_cast<uint32_t>((4 * e + j) * NT), sw128_desc(st + 32 * j),
                 sw128_desc(st + A_BYTES + 32 * j), idesc);
        mma_commit(&tfull[e]);
        mma_commit(&empty[s]);
      }
      // every MMA issued must be finished before the accumulators are freed
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0);
    }
  } else if (warp < 4) {
    // ------------------------------------------- int4 -> int8 converters
    if constexpr (I4) {
      const int t = threadIdx.x - 64;  // 0..63
      for (int kb = 0; kb < nkb; ++kb) {
        const int s = kb % kStages;
        // the producer reloaded this stage only after its previous MMAs
        // completed, so the A tile is free once the new data has landed
        if (!mbar_wait(&full[s], (kb / kStages) & 1, &s_abort)) break;
        uint8_t* st = smem + s * STAGE;
        const uint8_t* raw = st + A_BYTES + B_BYTES;
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int r = t + 64 * h;
          const uint4 u0 = reinterpret_cast<const uint4*>(raw + r * (kKStage / 2))[0];
          const uint4 u1 = reinterpret_cast<const uint4*>(raw + r * (kKStage / 2))[1];
          const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
#pragma unroll
          for (int c = 0; c < 8; ++c) {  // 16-byte chunk c = packed words 2c, 2c+1
            uint32_t o[4];
            widen_i4(w[2 * c], o[0], o[1]);
            widen_i4(w[2 * c + 1], o[2], o[3]);
            // 128-byte swizzle: chunk c of row r at chunk c ^ (r & 7)
            *reinterpret_cast<uint4*>(st + r * kKStage + ((c ^ (r & 7)) << 4)) =
                make_uint4(o[0], o[1], o[2], o[3]);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if ((threadIdx.x & 31) == 0) mbar_arrive(&cvt[s]);
      }
    }
  } else {
    // ------------------------------------------------------ epilogue
    const int q = warp & 3;                 // TMEM lane quarter = 32 rows
    const int h = (warp - 4) >> 2;          // column slice
    const int et = threadIdx.x - 128;
    // activation scales of this column tile, transposed: xsT[g][c]
    // (consecutive threads take consecutive columns: conflict-free stores)
    for (int idx = et; idx < NT * a.gpr; idx += kEpiWarps * 32) {
      const int g = idx / NT, c = idx - g * NT;
      xsT[g * NT + c] = (n0 + c < a.n) ? a.xs[static_cast<int64_t>(n0 + c) * a.gpr + g] : 0.0f;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(kEpiWarps * 32) : "memory");

    const int row = m0 + 32 * q + lane;
    const int c0 = h * COLS;
    const bool active = n0 + c0 < a.n;  // a slice wholly past n only releases slots
    const float* wsr = a.ws + static_cast<int64_t>(min(row, a.m - 1)) * a.gpr;
    uint64_t tot[COLS / 2];
#pragma unroll
    for (int c = 0; c < COLS / 2; ++c) tot[c] = 0ull;  // (+0.0f, +0.0f)
    const uint64_t nz = pk(a.neg_zero, a.neg_zero);
    const uint64_t nbias = pk(-12582912.0f, -12582912.0f);
    const uint32_t lane_addr = tbase + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0);
    float4 w4 = *reinterpret_cast<const float4*>(wsr);
    for (int kb = 0; kb < nkb; ++kb) {
      const int e = kb % ER;
      // next stage's weight scales go out now
      const float4 w4n = kb + 1 < nkb ? *reinterpret_cast<const float4*>(wsr + 4 * (kb + 1)) : w4;
      if (!mbar_wait(&tfull[e], (kb / ER) & 1, &s_abort)) break;
      fence_after();
      uint32_t v[4][COLS];
      if (active) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int c4 = 0; c4 < COLS; c4 += 4)
            tmem_ld4(lane_addr + static_cast<uint32_t>((4 * e + j) * NT + c4), v[j] + c4);
        tmem_wait_ld();
        // the registers the loads wrote are defined only after the wait: tie
        // them to it so no use is scheduled above it
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int i = 0; i < COLS; ++i) asm volatile("" : "+r"(v[j][i]));
      }
      fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&tempty[e]);
      if (active) {
        const float wsv[4] = {w4.x, w4.y, w4.z, w4.w};
        // isum (|isum| <= 32*128*128 < 2^22) is exact as M - C, M the float
        // with bits 0x4B400000 + isum, C = 1.5 * 2^23.  When C * ws is itself
        // exact (ws has two trailing zero significand bits, e.g. every
        // fp16-derived scale) fl(isum * ws) = fma(M, ws, -C * ws) in one
        // rounding; otherwise M - C is formed first.  Then fl(. * xs) and the
        // in-order add.
        bool ok4 = true;
#pragma unroll
        for (int j = 0; j < 4; ++j)
          ok4 = ok4 && (__float_as_uint(wsv[j]) & 3u) == 0u && fabsf(wsv[j]) < 1e30f &&
                fabsf(wsv[j]) > 1e-30f;
        const bool fused = __all_sync(0xffffffffu, ok4);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int g = 4 * kb + j;
          const uint64_t ws2 = pk(wsv[j], wsv[j]);
          const uint64_t ncw2 = pk(-12582912.0f * wsv[j], -12582912.0f * wsv[j]);
          const float4* xg4 = reinterpret_cast<const float4*>(xsT + g * NT + c0);
#pragma unroll
          for (int c4 = 0; c4 < COLS / 4; ++c4) {
            const float4 x4 = xg4[c4];
            const uint64_t xa = pk(x4.x, x4.y), xb = pk(x4.z, x4.w);
            const uint64_t ma = pk(__int_as_float(static_cast<int>(v[j][4 * c4]) + 0x4B400000),
                                   __int_as_float(static_cast<int>(v[j][4 * c4 + 1]) + 0x4B400000));
            const uint64_t mb = pk(__int_as_float(static_cast<int>(v[j][4 * c4 + 2]) + 0x4B400000),
                                   __int_as_float(static_cast<int>(v[j][4 * c4 + 3]) + 0x4B400000));
            uint64_t pa, pb;
            if (fused) {
              pa = fma2(ma, ws2, ncw2);
              pb = fma2(mb, ws2, ncw2);
            } else {
              pa = mul2(add2(ma, nbias), ws2);
              pb = mul2(add2(mb, nbias), ws2);
            }
            tot[2 * c4] = add2(tot[2 * c4], mul2_rn(pa, xa, nz));
            tot[2 * c4 + 1] = add2(tot[2 * c4 + 1], mul2_rn(pb, xb, nz));
          }
        }
      }
      w4 = w4n;
    }
    if (row < a.m && active) {
      float* yr = a.y + static_cast<int64_t>(row) * a.n + n0 + c0;
#pragma unroll
      for (int c = 0; c < COLS / 2; ++c) {
        float t0, t1;
        upk(tot[c], t0, t1);
        if (n0 + c0 + 2 * c < a.n) yr[2 * c] = t0;
        if (n0 + c0 + 2 * c + 1 < a.n) yr[2 * c + 1] = t1;
      }
    }
  }
  fence_before();
  __syncthreads();
  if (warp == 1) {
    fence_after();
    tmem_dealloc(tbase, kTmemCols);
  }
}

// A K-major int8 matrix of `rows` rows x k bytes, boxes of box_rows x 128 B,
// 128-byte swizzle.
bool encode_rows(CUtensorMap* tm, const void* base, int64_t k, int64_t rows, int box_rows) {
  return encode_u8(tm, base, k, rows, kKStage, box_rows, true);
}

template <int NT, bool I4>
int launch_nt(const void* wq, const float* ws, const int8_t* xq, const float* xs, int n,
              float* y, int m, int k, cudaStream_t st) {
  const int gpr = k / 32;
  CUtensorMap tmA, tmB;
  const bool aok = I4 ? encode_u8(&tmA, wq, k / 2, m, kKStage / 2, 128, false)
                      : encode_rows(&tmA, wq, k, m, 128);
  if (!aok || !encode_rows(&tmB, xq, k, n, NT)) return LP_ERR_UNSUPPORTED;
  constexpr int STAGE = (128 + NT) * kKStage + (I4 ? 128 * kKStage / 2 : 0);
  const int smem = 1024 + stages_for<NT>() * STAGE + gpr * NT * 4;
  const DeviceInfo& di = device_info();
  if (smem > di.max_smem_optin - 2048) return LP_ERR_UNSUPPORTED;  // (static smem: 1 KB)
  auto kern = k_gemm_tc<NT, I4>;
  static int attr_set[kMaxDevices];
  const int slot = di.ordinal % kMaxDevices;
  if (attr_set[slot] < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      cudaGetLastError();  // not sticky: clear it, the caller falls back
      return LP_ERR_UNSUPPORTED;
    }
    attr_set[slot] = smem;
  }
  TcArgs a{ws, xs, y, m, k, n, gpr, -0.0f};
  const dim3 grid((n + NT - 1) / NT, (m + 127) / 128);
  kern<<<grid, kThreads, smem, st>>>(tmA, tmB, a);
  return cuda_status(cudaGetLastError());
}

}  // namespace

// Tensor-core dequantGemmQ8 for 32-wide groups, K a multiple of 128 and
// 16-byte aligned operands; LP_ERR_UNSUPPORTED otherwise (the caller then
// runs the CUDA-core kernel).
int launch_gemm_tc(const void* wq, int packed_i4, const float* ws, int64_t gs, const int8_t* xq,
                   const float* xs, int64_t n, float* y, int64_t m, int64_t k,
                   cudaStream_t st) {
  if (gs != 32 || k % kKStage != 0 || k <= 0 || m <= 0 || n <= 0) return LP_ERR_UNSUPPORTED;
  if (m > (1 << 30) || n > (1 << 30) || k > (1 << 30)) return LP_ERR_UNSUPPORTED;
  const uintptr_t al = reinterpret_cast<uintptr_t>(wq) | reinterpret_cast<uintptr_t>(xq) |
                       reinterpret_cast<uintptr_t>(ws);
  if (al & 15) return LP_ERR_UNSUPPORTED;
  const int ni = static_cast<int>(n), mi = static_cast<int>(m), ki = static_cast<int>(k);
  if (packed_i4)
    return n <= 64 ? launch_nt<16, true>(wq, ws, xq, xs, ni, y, mi, ki, st)
                   : launch_nt<32, true>(wq, ws, xq, xs, ni, y, mi, ki, st);
  return n <= 64 ? launch_nt<16, false>(wq, ws, xq, xs, ni, y, mi, ki, st)
                 : launch_nt<32, false>(wq, ws, xq, xs, ni, y, mi, ki, st);
}

unsigned int take_error_gemm_tc() {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return LP_ERR_CUDA;
  if (v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace lp
