// gemm_fp4.cu -- FP4 x FP4 GEMMs on the block-scaled 5th-generation tensor
// cores: MXFP4 (e2m1 codes, one E8M0 scale per 32 elements; tcgen05.mma
// kind::mxf4) and NVFP4 (e2m1 codes, one e4m3 scale per 16 elements plus one
// fp32 global decode scale per operand; kind::mxf4nvf4).
//
//   y[row*n + c] = G * sum_b sw[row,b] * sx[c,b] * sum_{k in b} e2m1(w[row,k]) * e2m1(x[c,k])
//
// with b the scale blocks along K and G = 1 (MXFP4) or the product of the two
// global decode scales (NVFP4).  The e2m1 element values are those of
// dequantGemvF4's table (simd/dequant.nim:57-58, 341-420; mxfloat.nim:52-66),
// the MXFP4 scales those of calibrateMX (quant.nim:112-137), the NVFP4 scheme
// that of nvfp4.nim:39-92.  The reference computes these in its scalar fp32
// order; here the products are exact in the tensor core and the sums are fp32
// accumulations, so the result is compared within a tolerance.
//
// Layout in HBM (nothing is repacked): weights M x K/2 bytes, activations
// n x K/2 bytes (K x n column-major, as dequantGemmQ8 takes xq), two codes
// per byte, low nibble = even element.  MXFP4 scales are fp32 values that
// are powers of two (the form calibrateMX writes), M x K/32 and n x K/32;
// their E8M0 code is the fp32 exponent field.  NVFP4 block scales are e4m3
// bytes, M x K/16 and n x K/16.
//
// CTA = one 128-row x NT-column output tile over all of K, in stages of 256
// elements (128 bytes of codes per row):
//   warp 0     producer: per stage two TMA tile loads with 128-byte swizzle
//              (weights [128 rows x 128 B], activations [NT rows x 128 B]).
//   warp 1     owns TMEM; one lane copies the stage's scale factors from
//              shared memory into TMEM (tcgen05.cp) and issues its four
//              K = 64 block-scaled MMAs into one fp32 accumulator, then
//              commits to release the stage.
//   warps 2-5  write each stage's scale factors into shared memory in the
//              tensor core's scale-factor layout (128 rows x 4 blocks per
//              512-byte atom), then run the epilogue: tcgen05.ld of their 32
//              accumulator rows, times G, stored to y.
// Every wait is bounded and TMEM is freed on every path.
#include <cuda.h>

#include <algorithm>

#include "lp_internal.h"
#include "tc_ptx.cuh"

namespace lp {
namespace {

using namespace tc;

constexpr int kStageK = 256;     // elements of K per stage
constexpr int kStageBytes = 128; // code bytes of K per stage and row
constexpr int kThreads = 192;    // 6 warps
constexpr int kStages = 4;

// Scale-factor atom of the tensor core: 128 rows x 4 consecutive scale
// blocks, 512 bytes; row r = 32 m1 + m0, block j at byte 16 m0 + 4 m1 + j.
// One tcgen05.cp (32x128b.warpx4) moves an atom into four TMEM columns.
__device__ __forceinline__ int sf_off(int r, int j) {
  return 16 * (r & 31) + 4 * (r >> 5) + j;
}

// Shared-memory descriptor of a 32 x 16-byte block (no swizzle): 8-row core
// matrices 128 bytes apart.
__device__ __forceinline__ uint64_t sf_desc(const void* p) {
  uint64_t d = static_cast<uint64_t>((saddr(p) & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>(128 >> 4) << 16;   // leading byte offset (one core matrix wide)
  d |= static_cast<uint64_t>(128 >> 4) << 32;   // stride byte offset
  d |= static_cast<uint64_t>(1) << 46;          // descriptor version
  return d;                                     // layout type 0: no swizzle
}

__device__ __forceinline__ void sf_copy(uint32_t taddr, const void* atom) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sf_desc(atom))
               : "memory");
}

template <bool NV>
__device__ __forceinline__ void mma_fp4(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                        uint32_t idesc, uint32_t sfa, uint32_t sfb, int accum) {
  if constexpr (NV) {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::mxf4nvf4.block_scale.block16 [%0], %1, %2, %3, [%5], [%6], p; }"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
        : "memory");
  } else {
    asm volatile(
        "{ .reg .pred p; setp.ne.b32 p, %4, 0; "
        "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%5], [%6], p; }"
        ::"r"(d_tmem), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa), "r"(sfb)
        : "memory");
  }
}

// Block-scaled instruction descriptor: A, B e2m1 (format 1), K-major, M =
// 128, N = NT, scale format E8M0 (MXFP4) or e4m3 (NVFP4), scale-factor ids.
template <bool NV, int NT>
__host__ __device__ constexpr uint32_t idesc_fp4(int a_sf_id, int b_sf_id) {
  return (static_cast<uint32_t>(b_sf_id) << 4) | (1u << 7) | (1u << 10) |
         (static_cast<uint32_t>(NT >> 3) << 17) | ((NV ? 0u : 1u) << 23) |
         (static_cast<uint32_t>(128 >> 4) << 24) | (static_cast<uint32_t>(a_sf_id) << 29);
}

// 32 lanes x 16 consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, "
      "%12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

struct Fp4Args {
  const void* ws;   // MXFP4: float M x K/32; NVFP4: e4m3 bytes M x K/16
  const void* xs;   // same for the n activation columns
  float* y;         // M x n row-major
  int m, k, n;
  int nblk;         // scale blocks per row: K/32 or K/16
  const float* gw;  // NVFP4: the operands' global decode scales (device); else null
  const float* gx;
};

// E8M0 code of a power-of-two fp32 scale: its exponent field (2^-127, the
// smallest E8M0 value, is the fp32 subnormal 0x00400000 and has code 0).
__device__ __forceinline__ uint32_t e8m0_code(float s) {
  return (__float_as_uint(s) >> 23) & 0xFFu;
}

// The scale-factor bytes of row `r` (of `rows` valid) for the stage's blocks
// [b0, b0 + NB) into the stage's atoms.
template <bool NV>
__device__ __forceinline__ void stage_scales(uint8_t* atoms, const void* src, int row, int rows,
                                             int nblk, int b0, int r) {
  constexpr int NB = NV ? 16 : 8;  // scale blocks per 256-element stage
#pragma unroll
  for (int a = 0; a < NB / 4; ++a) {
    uint32_t word = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int b = b0 + 4 * a + j;
      uint32_t code = 0;
      if (row < rows && b < nblk) {
        const int64_t idx = static_cast<int64_t>(row) * nblk + b;
        code = NV ? static_cast<uint32_t>(static_cast<const uint8_t*>(src)[idx])
                  : e8m0_code(static_cast<const float*>(src)[idx]);
      }
      word |= code << (8 * j);
    }
    *reinterpret_cast<uint32_t*>(atoms + 512 * a + sf_off(r, 0)) = word;
  }
}

// The same from a stage's raw scale tile in shared memory (row r at r * SB
// bytes: MXFP4 8 fp32 scales, NVFP4 16 e4m3 bytes), as TMA left it.
template <bool NV>
__device__ __forceinline__ void stage_scales_smem(uint8_t* atoms, const uint8_t* raw, int r,
                                                  bool valid) {
  constexpr int NB = NV ? 16 : 8;
#pragma unroll
  for (int a = 0; a < NB / 4; ++a) {
    uint32_t word = 0;
    if (valid) {
      if (NV) {
        word = reinterpret_cast<const uint32_t*>(raw + 16 * r)[a];
      } else {
        const float4 f = reinterpret_cast<const float4*>(raw + 32 * r)[a];
        word = e8m0_code(f.x) | (e8m0_code(f.y) << 8) | (e8m0_code(f.z) << 16) |
               (e8m0_code(f.w) << 24);
      }
    }
    *reinterpret_cast<uint32_t*>(atoms + 512 * a + sf_off(r, 0)) = word;
  }
}

// TS: the stage's scale tiles come in by TMA with the codes (row strides of
// the scale arrays a multiple of 16 bytes: K % 256 == 0); otherwise the
// scale warps read them from global memory.
template <bool NV, int NT, bool TS>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemm_fp4(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
               const __grid_constant__ CUtensorMap tmSA, const __grid_constant__ CUtensorMap tmSB,
               const Fp4Args a) {
  constexpr int NB = NV ? 16 : 8;          // scale blocks per stage
  constexpr int NATOM = NB / 4;            // atoms per operand per stage
  constexpr int SB = NV ? 16 : 32;         // raw scale bytes per row and stage
  constexpr int A_BYTES = 128 * kStageBytes;
  constexpr int B_BYTES = NT * kStageBytes;
  constexpr int RAW_A = TS ? 128 * SB : 0, RAW_B = TS ? NT * SB : 0;
  constexpr int SF_BYTES = 2 * NATOM * 512;
  constexpr int SF_OFF = A_BYTES + B_BYTES + RAW_A + RAW_B;
  constexpr int STAGE = SF_OFF + SF_BYTES;
  constexpr uint32_t kTmemCols = 256;
  constexpr uint32_t kSfaCol = 128, kSfbCol = 128 + 4 * NATOM;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  __shared__ uint64_t full[kStages], sfull[kStages], empty[kStages], mma_done;
  __shared__ uint32_t tmem_base;
  __shared__ volatile int s_abort;

  uint8_t* smem = smem_raw + ((1024u - (saddr(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n0 = blockIdx.x * NT, m0 = blockIdx.y * 128;
  const int nkb = (a.k + kStageK - 1) / kStageK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&sfull[s], 4);
      mbar_init(&empty[s], 1);
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
    if (lane == 0) {
      int kb = 0;
      for (; kb < nkb; ++kb) {
        const int s = kb % kStages;
        if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, &s_abort)) break;
        if (s_abort) break;
        uint8_t* st = smem + s * STAGE;
        mbar_arrive_expect_tx(&full[s], A_BYTES + B_BYTES + RAW_A + RAW_B);
        tma_load_2d(st, &tmA, kb * kStageBytes, m0, &full[s]);
        tma_load_2d(st + A_BYTES, &tmB, kb * kStageBytes, n0, &full[s]);
        if constexpr (TS) {
          tma_load_2d(st + A_BYTES + B_BYTES, &tmSA, kb * SB, m0, &full[s]);
          tma_load_2d(st + A_BYTES + B_BYTES + RAW_A, &tmSB, kb * SB, n0, &full[s]);
        }
      }
      for (int u = max(0, kb - kStages); u < kb; ++u)
        mbar_wait(&full[u % kStages], (u / kStages) & 1);
    }
  } else if (warp == 1) {
    // --------------------------------------------------- MMA issuer
    if (lane == 0) {
      for (int kb = 0; kb < nkb && !s_abort; ++kb) {
        const int s = kb % kStages;
        if (!mbar_wait(&full[s], (kb / kStages) & 1, &s_abort)) break;
        if (!mbar_wait(&sfull[s], (kb / kStages) & 1, &s_abort)) break;
        fence_after();
        const uint8_t* st = smem + s * STAGE;
        const uint8_t* sfa = st + SF_OFF;
        const uint8_t* sfb = sfa + NATOM * 512;
#pragma unroll
        for (int t = 0; t < NATOM; ++t) {
          sf_copy(tbase + kSfaCol + 4 * t, sfa + 512 * t);
          sf_copy(tbase + kSfbCol + 4 * t, sfb + 512 * t);
        }
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          // MXFP4: MMA j reads blocks 2j, 2j+1 = bytes (2j) % 4.. of atom j/2;
          // NVFP4: blocks 4j..4j+3 = atom j
          const int atom = NV ? j : (j >> 1);
          const int id = NV ? 0 : ((2 * j) & 3);
          const uint32_t sa = (tbase + kSfaCol + 4 * atom) | (static_cast<uint32_t>(id) << 30);
          const uint32_t sb = (tbase + kSfbCol + 4 * atom) | (static_cast<uint32_t>(id) << 30);
          mma_fp4<NV>(tbase, sw128_desc(st + 32 * j), sw128_desc(st + A_BYTES + 32 * j),
                      idesc_fp4<NV, NT>(id, id), sa, sb, (kb > 0 || j > 0) ? 1 : 0);
        }
        mma_commit(&empty[s]);
      }
      // every MMA issued must be finished before TMEM is freed
      mma_commit(&mma_done);
      mbar_wait(&mma_done, 0);
    }
  } else {
    // ------------------------------------- scale factors, then epilogue
    const int r = threadIdx.x - 64;  // 0..127: one A row and one B row each
    for (int kb = 0; kb < nkb; ++kb) {
      const int s = kb % kStages;
      uint8_t* st = smem + s * STAGE;
      uint8_t* sfa = st + SF_OFF;
      if constexpr (TS) {
        // the producer reissued this stage only after its previous MMAs
        // (and scale copies) completed, so the atoms are free once it lands
        if (!mbar_wait(&full[s], (kb / kStages) & 1, &s_abort)) break;
        if (s_abort) break;
        stage_scales_smem<NV>(sfa, st + A_BYTES + B_BYTES, r, true);
        // rows past the column tile (NT = 64) hold zeros; their raw rows do not exist
        stage_scales_smem<NV>(sfa + NATOM * 512, st + A_BYTES + B_BYTES + RAW_A, r, r < NT);
      } else {
        if (kb >= kStages && !mbar_wait(&empty[s], ((kb / kStages) - 1) & 1, &s_abort)) break;
        if (s_abort) break;
        stage_scales<NV>(sfa, a.ws, m0 + r, a.m, a.nblk, kb * NB, r);
        stage_scales<NV>(sfa + NATOM * 512, a.xs, n0 + r, min(a.n, n0 + NT), a.nblk, kb * NB, r);
      }
      // generic-proxy writes, read by tcgen05.cp (async proxy)
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&sfull[s]);
    }
    // one decision per warp: the TMEM loads below are warp-collective
    const bool ok = __all_sync(0xffffffffu, mbar_wait(&mma_done, 0, &s_abort) && !s_abort);
    fence_after();
    const float g = a.gw ? __fmul_rn(*a.gw, *a.gx) : 1.0f;
    const int q = warp & 3;  // TMEM lane quarter of this warp (warps 2..5 -> 2,3,0,1)
    const int row = m0 + 32 * q + lane;
    if (ok) {
#pragma unroll 1
      for (int c0 = 0; c0 < NT; c0 += 16) {
        uint32_t v[16];
        tmem_ld16(tbase + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), v);
        tmem_wait_ld();
#pragma unroll
        for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(v[i]));
        if (row < a.m) {
          float* yr = a.y + static_cast<int64_t>(row) * a.n;
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = n0 + c0 + i;
            if (c < a.n) yr[c] = __fmul_rn(__uint_as_float(v[i]), g);
          }
        }
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

template <bool NV, int NT, bool TS>
int launch_nt(const uint8_t* w, const void* ws, const uint8_t* x, const void* xs, int n, float* y,
              int m, int k, const float* gw, const float* gx, cudaStream_t st) {
  constexpr int SB = NV ? 16 : 32;  // raw scale bytes per row and stage
  const int64_t srow = static_cast<int64_t>(k) / (NV ? 16 : 32) * (NV ? 1 : 4);  // scale row bytes
  CUtensorMap tmA, tmB, tmSA, tmSB;
  if (!encode_u8(&tmA, w, k / 2, m, kStageBytes, 128, true) ||
      !encode_u8(&tmB, x, k / 2, n, kStageBytes, NT, true))
    return LP_ERR_UNSUPPORTED;
  if (TS) {
    if (!encode_u8(&tmSA, ws, srow, m, SB, 128, false) ||
        !encode_u8(&tmSB, xs, srow, n, SB, NT, false))
      return LP_ERR_UNSUPPORTED;
  } else {
    tmSA = tmA;  // unused
    tmSB = tmB;
  }
  constexpr int NATOM = (NV ? 16 : 8) / 4;
  constexpr int STAGE = (128 + NT) * kStageBytes + (TS ? (128 + NT) * SB : 0) + 2 * NATOM * 512;
  const int smem = 1024 + kStages * STAGE;
  const DeviceInfo& di = device_info();
  if (smem > di.max_smem_optin - 2048) return LP_ERR_UNSUPPORTED;
  auto kern = k_gemm_fp4<NV, NT, TS>;
  static int attr_set[kMaxDevices];
  const int slot = di.ordinal % kMaxDevices;
  if (attr_set[slot] < smem) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem) != cudaSuccess) {
      cudaGetLastError();
      return LP_ERR_UNSUPPORTED;
    }
    attr_set[slot] = smem;
  }
  Fp4Args args{ws, xs, y, m, k, n, k / (NV ? 16 : 32), gw, gx};
  const dim3 grid((n + NT - 1) / NT, (m + 127) / 128);
  kern<<<grid, kThreads, smem, st>>>(tmA, tmB, tmSA, tmSB, args);
  return cuda_status(cudaGetLastError());
}

template <bool NV, bool TS>
int launch_tiles(const uint8_t* w, const void* ws, const uint8_t* x, const void* xs, int64_t n,
                 float* y, int64_t m, int64_t k, const float* gw, const float* gx, cudaStream_t st) {
  if (n <= 64)
    return launch_nt<NV, 64, TS>(w, ws, x, xs, static_cast<int>(n), y, static_cast<int>(m),
                                 static_cast<int>(k), gw, gx, st);
  return launch_nt<NV, 128, TS>(w, ws, x, xs, static_cast<int>(n), y, static_cast<int>(m),
                                static_cast<int>(k), gw, gx, st);
}

template <bool NV>
int launch_fp4(const uint8_t* w, const void* ws, const uint8_t* x, const void* xs, int64_t n,
               float* y, int64_t m, int64_t k, const float* gw, const float* gx, cudaStream_t st) {
  if (m <= 0 || n <= 0 || k <= 0) return LP_OK;
  if (k % 32 != 0 || m > (1 << 30) || n > (1 << 30) || k > (1 << 30)) return LP_ERR_UNSUPPORTED;
  // TMA: 16-byte aligned bases and row strides (k/2 bytes)
  if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) return LP_ERR_UNSUPPORTED;
  // scale tiles by TMA when the scale rows are 16-byte multiples and aligned
  const bool ts = k % 256 == 0 &&
                  ((reinterpret_cast<uintptr_t>(ws) | reinterpret_cast<uintptr_t>(xs)) & 15) == 0;
  return ts ? launch_tiles<NV, true>(w, ws, x, xs, n, y, m, k, gw, gx, st)
            : launch_tiles<NV, false>(w, ws, x, xs, n, y, m, k, gw, gx, st);
}

}  // namespace

int launch_gemm_mxf4(const uint8_t* w, const float* ws, const uint8_t* x, const float* xs,
                     int64_t n, float* y, int64_t m, int64_t k, cudaStream_t st) {
  return launch_fp4<false>(w, ws, x, xs, n, y, m, k, nullptr, nullptr, st);
}

int launch_gemm_nvf4(const uint8_t* w, const uint8_t* ws, const float* gw, const uint8_t* x,
                     const uint8_t* xs, const float* gx, int64_t n, float* y, int64_t m, int64_t k,
                     cudaStream_t st) {
  return launch_fp4<true>(w, ws, x, xs, n, y, m, k, gw, gx, st);
}

unsigned int take_error_gemm_fp4() {
  unsigned int v = 0;
  if (cudaMemcpyFromSymbol(&v, g_device_error, sizeof(v)) != cudaSuccess) return LP_ERR_CUDA;
  if (v) {
    const unsigned int z = 0;
    cudaMemcpyToSymbol(g_device_error, &z, sizeof(z));
  }
  return v;
}

}  // namespace lp
