// quant.cu -- the encoders of the hot path, bit-exact against the reference:
//   quantizeQ8_0 / quantizeQ8_0Batch   one warp per 32-element block: warp
//                                      abs-max (order-free), d = amax/127,
//                                      q = clamp(round(x * (1/d)), +-127)
//   quantizeQ4_0                        sign-keeping max, first index wins
//   quantizeBatch                       q = toI8(x / scale)
//   calibrateSymmetric / calibrateMX    per-group abs-max -> scale
//   quantize[I4]+packInt4, quantize[F4E2M1]+packF4   weight preparation
//   dequantizeQ8_0 / Q4_0               blocks -> fp32
// Division, reciprocal and the fp16 conversion are the IEEE round-to-nearest
// operations (__fdiv_rn, __float2half_rn); roundf rounds half away from zero
// like Nim's round (simd/dequant.nim:1589-1591).  These kernels stream
// activation-sized data (or run once at weight load), so they are simple
// coalesced grid-stride kernels.
#include <algorithm>

#include "lp_device.cuh"
#include "lp_internal.h"

namespace lp {
namespace {

constexpr int kThreads = 256;

inline int grid_for(int64_t work, int per_block) {
  const DeviceInfo& di = device_info();
  const int64_t need = (work + per_block - 1) / per_block;
  return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(need, di.sm_count * 16)));
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// ggml.nim:60-75.  Writes packed blocks and/or the split (qs, f32(f16(d))).
__global__ void k_quantize_q8_0(const float* __restrict__ src, int64_t nblocks,
                                uint8_t* __restrict__ blocks, int8_t* __restrict__ qs,
                                float* __restrict__ dsplit) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t b = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       b < nblocks; b += warps) {
    const float v = src[b * 32 + lane];
    const float amax = warp_max(fabsf(v));  // NaN never wins, as with the strict > scan
    const float d = __fdiv_rn(amax, 127.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    float r = roundf(__fmul_rn(v, id));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    const int8_t q = static_cast<int8_t>(static_cast<int>(r));
    const unsigned short dh = __half_as_ushort(__float2half_rn(d));
    if (blocks) {
      uint8_t* blk = blocks + b * 34;
      blk[2 + lane] = static_cast<uint8_t>(q);
      if (lane == 0) {
        blk[0] = static_cast<uint8_t>(dh & 0xFF);
        blk[1] = static_cast<uint8_t>(dh >> 8);
      }
    }
    if (qs) qs[b * 32 + lane] = q;
    if (dsplit && lane == 0) dsplit[b] = h2f(dh);
  }
}

// The same encoder, bandwidth-shaped: 8 lanes per block, a float4 per lane,
// two blocks per thread per pass (two loads in flight); the block max meets
// by three shuffles inside the 8-lane group.  fmaxf ignores NaN like the
// reference's strict `>` scan.  It waits for the previous kernel in the
// stream before reading or writing anything (it is launched with
// programmatic stream serialization, so its launch overlaps that kernel's
// tail) and does not release its own dependents early: its output may be the
// next GEMV's weights.
__device__ __forceinline__ void q8_block4(const float4 v, int sub, int lane, int64_t b, bool valid,
                                          uint8_t* blocks, int8_t* qs, float* dsplit) {
  const unsigned gm = 0xFFu << (lane & 24);  // this block's 8 lanes
  float a = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
  a = fmaxf(a, __shfl_xor_sync(gm, a, 1, 8));
  a = fmaxf(a, __shfl_xor_sync(gm, a, 2, 8));
  a = fmaxf(a, __shfl_xor_sync(gm, a, 4, 8));
  if (!valid) return;
  const float d = __fdiv_rn(a, 127.0f);
  const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
  const float e[4] = {v.x, v.y, v.z, v.w};
  uint32_t word = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    float r = roundf(__fmul_rn(e[i], id));
    r = fminf(fmaxf(r, -127.0f), 127.0f);
    word |= (static_cast<uint32_t>(static_cast<int>(r)) & 0xFFu) << (8 * i);
  }
  const unsigned short dh = __half_as_ushort(__float2half_rn(d));
  if (blocks) {
    unsigned short* blk = reinterpret_cast<unsigned short*>(blocks + b * 34);
    blk[1 + 2 * sub] = static_cast<unsigned short>(word & 0xFFFFu);
    blk[2 + 2 * sub] = static_cast<unsigned short>(word >> 16);
    if (sub == 0) blk[0] = dh;
  }
  if (qs) reinterpret_cast<uint32_t*>(qs + b * 32)[sub] = word;
  if (dsplit && sub == 0) dsplit[b] = h2f(dh);
}

__global__ void __launch_bounds__(128) k_quantize_q8_0_v4(const float* __restrict__ src,
                                                          int64_t nblocks, uint8_t* blocks,
                                                          int8_t* qs, float* dsplit) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int lane = threadIdx.x & 31, sub = lane & 7;
  const int64_t groups = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 3);
  const int64_t first = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 3;
  const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
  // the loop bound is uniform over the warp (whole passes), so the 8-lane
  // shuffles always see all of their lanes
  const int64_t warp0 = first - (lane >> 3);
  for (int64_t p = 0; warp0 + p * 2 * groups < nblocks; ++p) {
    const int64_t b1 = first + p * 2 * groups, b2 = b1 + groups;
    const bool v1 = b1 < nblocks, v2 = b2 < nblocks;
    const float4 x1 = v1 ? __ldg(reinterpret_cast<const float4*>(src + b1 * 32) + sub) : z;
    const float4 x2 = v2 ? __ldg(reinterpret_cast<const float4*>(src + b2 * 32) + sub) : z;
    q8_block4(x1, sub, lane, b1, v1, blocks, qs, dsplit);
    q8_block4(x2, sub, lane, b2, v2, blocks, qs, dsplit);
  }
}

// ggml.nim:77-97: vmax = the first element of largest magnitude (strict >
// scan from 0), d = vmax / -8, q = clamp(int(round(x*id)) + 8, 0, 15).
__global__ void k_quantize_q4_0(const float* __restrict__ src, int64_t nblocks,
                                uint8_t* __restrict__ blocks) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t b = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
       b < nblocks; b += warps) {
    const float v = src[b * 32 + lane];
    const float a = fabsf(v);
    // key: magnitude bits (NaN excluded), ties to the lowest index
    const uint64_t mag = (a == a) ? __float_as_uint(a) : 0u;
    uint64_t key = (mag << 32) | static_cast<uint32_t>(31 - lane);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const uint64_t other = __shfl_xor_sync(0xffffffffu, key, o);
      key = other > key ? other : key;
    }
    const int win = 31 - static_cast<int>(key & 31u);
    const float vw = __shfl_sync(0xffffffffu, v, win);
    const float vmax = (key >> 32) != 0 ? vw : 0.0f;
    const float d = __fdiv_rn(vmax, -8.0f);
    const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
    int q = static_cast<int>(roundf(__fmul_rn(v, id))) + 8;
    q = min(max(q, 0), 15);
    // byte i (i < 16) = q[i] | q[i+16] << 4; the 18-byte block is written as
    // nine 2-byte-aligned halfwords: d, then qs byte pairs.
    const int qhi = __shfl_down_sync(0xffffffffu, q, 16);
    const uint32_t byte = static_cast<uint32_t>(q | (qhi << 4)) & 0xFFu;
    const uint32_t lo = __shfl_sync(0xffffffffu, byte, (2 * lane - 2) & 31);
    const uint32_t hi = __shfl_sync(0xffffffffu, byte, (2 * lane - 1) & 31);
    const unsigned short dh = __half_as_ushort(__float2half_rn(d));
    unsigned short* blk = reinterpret_cast<unsigned short*>(blocks + b * 18);
    if (lane == 0) blk[0] = dh;
    else if (lane < 9) blk[lane] = static_cast<unsigned short>(lo | (hi << 8));
  }
}

// quant.nim:48-60 (quantizeBatch, simd/dequant.nim:1717-1750, whose
// zero-point case falls through to this scalar quantize):
// toI8(x / scale + zeroPoint): round half away, clamp [-128, 127]; the
// symmetric case adds 0.0 (zp null).
__global__ void k_quantize_batch(const float* __restrict__ x, int64_t n,
                                 const float* __restrict__ scales,
                                 const float* __restrict__ zp, int64_t gs,
                                 int8_t* __restrict__ dst) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t g = gs > 0 ? i / gs : 0;
    const float s = scales[g];
    const float z = zp ? zp[g] : 0.0f;
    float r = roundf(__fadd_rn(__fdiv_rn(x[i], s), z));
    r = fminf(fmaxf(r, -128.0f), 127.0f);
    dst[i] = static_cast<int8_t>(static_cast<int>(r));
  }
}

// floor(log2(a)) the way frexp reports it (a > 0 finite); glibc's frexp
// gives exponent 0 for an infinity, which the reference then uses as is.
__device__ __forceinline__ int floor_log2(float a) {
  const uint32_t u = __float_as_uint(a);
  if (u >= 0x7F800000u) return -1;              // +inf: frexp exp 0 -> 0 - 1
  if (u >= 0x00800000u) return static_cast<int>(u >> 23) - 127;
  return (31 - __clz(static_cast<int>(u))) - 149;  // subnormal
}

__device__ __forceinline__ float pow2i(int k) {  // exact 2^k, k in [-127, 127]
  return k >= -126 ? __uint_as_float(static_cast<uint32_t>(k + 127) << 23)
                   : __uint_as_float(0x00400000u);
}

// The scale of a group from its max |x| (quant.nim:95-110 symmetric, 125-137 MX).
__device__ __forceinline__ float group_scale(float v, float qmax, int emax, int mx) {
  if (mx) {
    if (v == 0.0f) return 1.0f;
    int k = floor_log2(v) - emax;
    k = max(-127, min(127, k));
    return pow2i(k);
  }
  return v == 0.0f ? 1.0f : __fdiv_rn(v, qmax);
}

// calibrateSymmetric / calibrateMX for groups of 4 * L values, L a power of
// two <= 32: each thread loads one float4 and L lanes reduce a group with
// shuffles (max is order-free, fmaxf drops NaN as the scalar scan does).
// x 16-byte aligned and n % 4 == 0; a ragged last group reads zeros past n.
template <int L>
__global__ void __launch_bounds__(256) k_calibrate_vec(const float4* __restrict__ x, int64_t n4,
                                                       float qmax, int emax, int mx,
                                                       float* __restrict__ scales, int64_t nscales) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  // every lane runs the same number of rounds, so the shuffles stay converged
  const int64_t total = nscales * L;
  for (int64_t t0 = static_cast<int64_t>(blockIdx.x) * blockDim.x; t0 < total; t0 += stride) {
    const int64_t t = t0 + threadIdx.x;
    float m = 0.0f;
    if (t < total && t < n4) {
      const float4 v = __ldg(x + t);
      m = fmaxf(fmaxf(fabsf(v.x), fabsf(v.y)), fmaxf(fabsf(v.z), fabsf(v.w)));
    }
#pragma unroll
    for (int o = L / 2; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if ((threadIdx.x & (L - 1)) == 0 && t < total) scales[t / L] = group_scale(m, qmax, emax, mx);
  }
}

// calibrateSymmetric (quant.nim:84-110) and calibrateMX (quant.nim:112-137),
// any group size: one CTA per group.
__global__ void k_calibrate(const float* __restrict__ x, int64_t n, int64_t gs, float qmax,
                            int emax, int mx, float* __restrict__ scales, int64_t nscales) {
  __shared__ float red[kThreads / 32];
  for (int64_t g = blockIdx.x; g < nscales; g += gridDim.x) {
    const int64_t lo = g * gs;
    const int64_t hi = min(lo + gs, n);
    float m = 0.0f;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) m = fmaxf(m, fabsf(x[i]));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    if (threadIdx.x < 32) {
      float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
      v = warp_max(v);
      if (threadIdx.x == 0) scales[g] = group_scale(v, qmax, emax, mx);
    }
    __syncthreads();
  }
}

// toF4E2M1 (mxfloat.nim:52-66, nearestCode tinyfloat.nim:24-46).
__device__ __forceinline__ uint32_t to_e2m1(float f) {
  const uint32_t sign = (__float_as_uint(f) >> 31) ? 8u : 0u;
  const float a = fabsf(f);
  if (a != a) return 0u;
  if (a >= 6.0f) return sign | 7u;
  const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  int lo = 0, hi = 7;
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (mag[mid] >= a) hi = mid;
    else lo = mid + 1;
  }
  int code = 0;
  if (hi != 0) {
    const int clo = hi - 1;
    const float midv = (mag[clo] + mag[hi]) * 0.5f;  // exact on this grid
    if (a < midv) code = clo;
    else if (a > midv) code = hi;
    else code = (clo & 1) == 0 ? clo : hi;
  }
  return code == 0 ? sign : (sign | static_cast<uint32_t>(code));
}

// ------------------------------------------------------------ NVFP4 ---
// nvfp4.nim:39-92 (TransformerEngine NVFP4QuantizerRef, 1D path): e2m1
// codes in 16-element blocks, one e4m3 decode scale per block, one fp32
// global decode scale per tensor.

// e4m3fn code of a finite a in [0, 448] (float8.nim:78-112): round to
// nearest even on the e4m3 grid, subnormal step 2^-9.  (The scheme clamps
// its block scales into this range before encoding.)
__device__ __forceinline__ uint32_t e4m3_code(float a) {
  if (a < 0.015625f) return static_cast<uint32_t>(__float2int_rn(a * 512.0f));  // exact scaling
  const uint32_t bits = __float_as_uint(a);
  int ex = static_cast<int>((bits >> 23) & 255u) - 127;
  const uint32_t f = bits & 0x7FFFFFu;
  uint32_t q = f >> 20;
  const uint32_t rem = f & 0xFFFFFu;
  if (rem > 0x80000u || (rem == 0x80000u && (q & 1u))) ++q;
  if (q == 8u) {
    q = 0;
    ++ex;
  }
  const uint32_t code = (static_cast<uint32_t>(ex + 7) << 3) | q;
  return code > 0x7Eu ? 0x7Eu : code;
}
__device__ __forceinline__ float e4m3_value(uint32_t u) {
  const uint32_t ef = (u >> 3) & 15u, mf = u & 7u;
  const float mag = ef ? __uint_as_float(((ef + 120u) << 23) | (mf << 20))
                       : static_cast<float>(mf) * 0.001953125f;
  return (u & 0x80u) ? -mag : mag;
}

// Pass 1: the tensor's largest |x| (NaN never wins, like the strict > scan)
// as non-negative float bits, max-combined into *amax (zeroed beforehand).
__global__ void k_nvfp4_amax(const float* __restrict__ x, int64_t n, uint32_t* amax) {
  uint32_t m = 0;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const float a = fabsf(x[i]);
    if (a == a) m = max(m, __float_as_uint(a));
  }
  for (int o = 16; o > 0; o >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, o));
  if ((threadIdx.x & 31) == 0 && m) atomicMax(amax, m);
}

__device__ __forceinline__ void nvfp4_globals(float gamax, float& ges, float& gds) {
  const float F32MAX = 3.4028234663852886e38f;
  ges = fminf(__fdiv_rn(2688.0f, gamax), F32MAX);  // 448 * 6
  if (ges == 0.0f) ges = 1.0f;
  gds = __fdiv_rn(1.0f, ges);
}

// Pass 2: one thread per 16-element block.
__global__ void k_nvfp4_encode(const float* __restrict__ x, int64_t nblocks,
                               const uint32_t* amax, uint8_t* __restrict__ codes,
                               uint8_t* __restrict__ scales) {
  const float F32MAX = 3.4028234663852886e38f;
  float ges, gds;
  nvfp4_globals(__uint_as_float(*amax), ges, gds);
  const float mult = __fmul_rn(ges, __fdiv_rn(1.0f, 6.0f));
  for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < nblocks;
       b += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    float v[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = x[b * 16 + i];
    float vmax = 0.0f;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const float a = fabsf(v[i]);
      if (a > vmax) vmax = a;
    }
    float ds = fminf(__fmul_rn(vmax, mult), F32MAX);
    ds = fminf(fmaxf(ds, -448.0f), 448.0f);
    const uint32_t ds8 = e4m3_code(ds);
    scales[b] = static_cast<uint8_t>(ds8);
    const float es = fminf(__fdiv_rn(1.0f, __fmul_rn(e4m3_value(ds8), gds)), F32MAX);
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      float sc = __fmul_rn(v[i], es);
      if (sc < -6.0f) sc = -6.0f;  // NaN passes through, as in the reference's clamp
      if (sc > 6.0f) sc = 6.0f;
      codes[b * 16 + i] = static_cast<uint8_t>(sc == 0.0f ? 0u : to_e2m1(sc));
    }
  }
}

// Pass 3: the global decode scale replaces the amax in place.
__global__ void k_nvfp4_finish(float* gds_out) {
  float ges, gds;
  nvfp4_globals(*gds_out, ges, gds);
  *gds_out = gds;
}

// dequantizeNVFP4 (nvfp4.nim:80-92): (value(code) * value(scale)) * gds.
__global__ void k_nvfp4_dequant(const uint8_t* __restrict__ codes,
                                const uint8_t* __restrict__ scales, float gds, int64_t n,
                                float* __restrict__ dst) {
  const float lut[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint32_t c = codes[i];
    const float q = (c & 8u) ? -lut[c & 7u] : lut[c & 7u];
    dst[i] = __fmul_rn(__fmul_rn(q, e4m3_value(scales[i >> 4])), gds);
  }
}

// quantize[T] (quant.nim:48-60, value = x/scale + 0.0) + pack two per byte,
// low nibble = even index (intx.nim:83-94, mxfloat.nim:138-149).
__global__ void k_quantize_packed(const float* __restrict__ x, int64_t n,
                                  const float* __restrict__ scales, int64_t gs, int f4,
                                  uint8_t* __restrict__ packed) {
  const int64_t nbytes = (n + 1) / 2;
  for (int64_t j = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; j < nbytes;
       j += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    uint32_t nib[2] = {0u, 0u};
    for (int h = 0; h < 2; ++h) {
      const int64_t i = 2 * j + h;
      if (i >= n) break;
      const float s = scales[gs > 0 ? i / gs : 0];
      const float v = __fadd_rn(__fdiv_rn(x[i], s), 0.0f);
      if (f4) {
        nib[h] = to_e2m1(v);
      } else {
        float r = roundf(v);
        r = fminf(fmaxf(r, -8.0f), 7.0f);
        nib[h] = static_cast<uint32_t>(static_cast<int>(r)) & 15u;
      }
    }
    packed[j] = static_cast<uint8_t>(nib[0] | (nib[1] << 4));
  }
}

// dequantizeQ8_0 / dequantizeQ4_0 (ggml.nim:36-56): value = d * q.
__global__ void k_dequantize_blocks(const uint8_t* __restrict__ blocks, int64_t nblocks, int q4,
                                    float* __restrict__ dst) {
  const int64_t n = nblocks * 32;
  const int bs = q4 ? 18 : 34;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* blk = blocks + (i >> 5) * bs;
    const int e = static_cast<int>(i & 31);
    const float d = h2f(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
    int q;
    if (q4) {
      const uint32_t b = blk[2 + (e & 15)];
      q = static_cast<int>(e < 16 ? (b & 15u) : (b >> 4)) - 8;
    } else {
      q = static_cast<int8_t>(blk[2 + e]);
    }
    dst[i] = __fmul_rn(d, i2f_rn(q));
  }
}

// ggml.nim:136-161 (dequantizeQ4_K).  256-element super-block: d, dmin,
// 12 bytes of 6-bit sub-scales/mins, 128 bytes of nibbles; element
// 64c + 32h + l is nibble h of qs byte 32c + l with sub-block 2c + h:
// fl(fl(d * sc) * q) - fl(dmin * m).  A thread takes 8 consecutive elements
// (one sub-block, one 8-byte load of codes, two float4 stores).
template <bool kVec>
__device__ __forceinline__ void store8(float* o, const float (&v)[8]) {
  if (kVec) {
    reinterpret_cast<float4*>(o)[0] = make_float4(v[0], v[1], v[2], v[3]);
    reinterpret_cast<float4*>(o)[1] = make_float4(v[4], v[5], v[6], v[7]);
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) o[i] = v[i];
  }
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

// kVec: blocks and dst 16-byte aligned (vector code loads and stores)
template <bool kVec>
__global__ void k_dequantize_q4_k(const uint8_t* __restrict__ blocks, int64_t nblocks,
                                  float* __restrict__ dst) {
  const int64_t n8 = nblocks * 32;  // 8-element pieces
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n8;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* blk = blocks + (t >> 5) * 144;
    const int e0 = static_cast<int>(t & 31) * 8, c = e0 >> 6, h = (e0 >> 5) & 1, l0 = e0 & 31;
    const float d = h2f(static_cast<uint32_t>(blk[0]) | (static_cast<uint32_t>(blk[1]) << 8));
    const float dmin = h2f(static_cast<uint32_t>(blk[2]) | (static_cast<uint32_t>(blk[3]) << 8));
    int sc, m;
    scale_min_k4(2 * c + h, blk + 4, sc, m);
    const float d1 = __fmul_rn(d, i2f_rn(sc)), mm = __fmul_rn(dmin, i2f_rn(m));
    uint32_t wv[2];
    if (kVec) {
      const uint2 w = *reinterpret_cast<const uint2*>(blk + 16 + 32 * c + l0);  // 8-byte aligned
      wv[0] = w.x;
      wv[1] = w.y;
    } else {
      const uint8_t* qb = blk + 16 + 32 * c + l0;
      wv[0] = qb[0] | (qb[1] << 8) | (qb[2] << 16) | (static_cast<uint32_t>(qb[3]) << 24);
      wv[1] = qb[4] | (qb[5] << 8) | (qb[6] << 16) | (static_cast<uint32_t>(qb[7]) << 24);
    }
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t b = (wv[i >> 2] >> (8 * (i & 3))) & 0xFFu;
      const int q = static_cast<int>(h ? (b >> 4) : (b & 15u));
      v[i] = __fsub_rn(__fmul_rn(d1, i2f_rn(q)), mm);
    }
    store8<kVec>(dst + t * 8, v);
  }
}

// ggml.nim:163-213 (dequantizeQ6_K): ql[128] low four bits, qh[64] high two
// bits, int8 scales[16], d (f16) last.  Element 128h + 32k + l takes
// fl(fl(d * scale[8h + l/16 + 2k]) * (q - 32)); a thread takes 8 consecutive
// elements (one scale; the 210-byte blocks are only 2-byte aligned, so the
// codes come as bytes).
template <bool kVec>
__global__ void k_dequantize_q6_k(const uint8_t* __restrict__ blocks, int64_t nblocks,
                                  float* __restrict__ dst) {
  const int64_t n8 = nblocks * 32;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n8;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const uint8_t* blk = blocks + (t >> 5) * 210;
    const int e0 = static_cast<int>(t & 31) * 8, h = e0 >> 7, k = (e0 >> 5) & 3, l0 = e0 & 31;
    const uint8_t* ql = blk + 64 * h + l0 + ((k & 1) ? 32 : 0);
    const uint8_t* qh = blk + 128 + 32 * h + l0;
    const int scale = static_cast<int8_t>(blk[192 + 8 * h + (l0 >> 4) + 2 * k]);
    const float d = h2f(static_cast<uint32_t>(blk[208]) | (static_cast<uint32_t>(blk[209]) << 8));
    const float ds = __fmul_rn(d, i2f_rn(scale));
    float v[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t lo = ql[i], hi = qh[i];
      const int q =
          static_cast<int>(((k & 2) ? (lo >> 4) : (lo & 15u)) | (((hi >> (2 * k)) & 3u) << 4)) - 32;
      v[i] = __fmul_rn(ds, i2f_rn(q));
    }
    store8<kVec>(dst + t * 8, v);
  }
}

// dequantizeBatch (simd/dequant.nim:159-206; scalar quant.nim:62-74):
// dst = fl(fl(f32(q) - zp[g]) * scale[g]), g = i div gs, zp = 0 when absent
// (f32(q) - 0 == f32(q), so the symmetric form is the same arithmetic).  A
// thread takes 16 consecutive values: one 16-byte load, four 16-byte stores
// when kVec (q and dst 16-byte aligned), and walks the group boundaries
// inside its run.  gs > 0 here (per tensor: gs = n).
template <bool kVec>
__global__ void k_dequantize_batch(const int8_t* __restrict__ q, int64_t n,
                                   const float* __restrict__ scales,
                                   const float* __restrict__ zp, int64_t gs,
                                   float* __restrict__ dst) {
  const int64_t n16 = (n + 15) / 16;
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; t < n16;
       t += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t i0 = t * 16;
    const int cnt = n - i0 < 16 ? static_cast<int>(n - i0) : 16;
    int8_t v[16];
    if (kVec && cnt == 16) {
      const int4 w = *reinterpret_cast<const int4*>(q + i0);
      memcpy(v, &w, 16);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j) v[j] = j < cnt ? q[i0 + j] : 0;
    }
    int64_t g = i0 / gs, r = i0 - g * gs;
    float sc = scales[g], z = zp ? zp[g] : 0.0f;
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      if (r == gs && i0 + j < n) {
        ++g;
        r = 0;
        sc = scales[g];
        z = zp ? zp[g] : 0.0f;
      }
      o[j] = __fmul_rn(__fsub_rn(static_cast<float>(v[j]), z), sc);
      ++r;
    }
    float* out = dst + i0;
    if (kVec && cnt == 16) {
#pragma unroll
      for (int j = 0; j < 16; j += 4)
        *reinterpret_cast<float4*>(out + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
    } else {
#pragma unroll
      for (int j = 0; j < 16; ++j)
        if (j < cnt) out[j] = o[j];
    }
  }
}

}  // namespace

int launch_quantize_nvfp4(const float* x, int64_t n, uint8_t* codes, uint8_t* scales,
                          float* gds_out, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(gds_out, 0, sizeof(float), st);
  if (e != cudaSuccess) return cuda_status(e);
  if (n > 0) {
    k_nvfp4_amax<<<grid_for(n, kThreads), kThreads, 0, st>>>(x, n, reinterpret_cast<uint32_t*>(gds_out));
    k_nvfp4_encode<<<grid_for(n / 16, kThreads), kThreads, 0, st>>>(
        x, n / 16, reinterpret_cast<const uint32_t*>(gds_out), codes, scales);
  }
  k_nvfp4_finish<<<1, 1, 0, st>>>(gds_out);
  return cuda_status(cudaGetLastError());
}

int launch_dequantize_batch(const int8_t* q, int64_t n, const float* scales, const float* zp,
                            int64_t gs, float* dst, cudaStream_t st) {
  if (n == 0) return LP_OK;
  if (gs <= 0 || gs > n) gs = n;
  const int grid = grid_for((n + 15) / 16, kThreads);
  if (((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(dst)) & 15) == 0)
    k_dequantize_batch<true><<<grid, kThreads, 0, st>>>(q, n, scales, zp, gs, dst);
  else
    k_dequantize_batch<false><<<grid, kThreads, 0, st>>>(q, n, scales, zp, gs, dst);
  return cuda_status(cudaGetLastError());
}

int launch_dequantize_nvfp4(const uint8_t* codes, const uint8_t* scales, float gds, int64_t n,
                            float* dst, cudaStream_t st) {
  if (n == 0) return LP_OK;
  k_nvfp4_dequant<<<grid_for(n, kThreads), kThreads, 0, st>>>(codes, scales, gds, n, dst);
  return cuda_status(cudaGetLastError());
}

int launch_dequantize_kquant(const uint8_t* blocks, int64_t nblocks, int q6, float* dst,
                             cudaStream_t st) {
  if (nblocks == 0) return LP_OK;
  // vector stores (and Q4_K's 8-byte code loads) need 16-byte alignment
  const bool vec = ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(blocks)) & 15) == 0;
  const int grid = grid_for(nblocks * 32, kThreads);
  if (q6) {
    if (vec) k_dequantize_q6_k<true><<<grid, kThreads, 0, st>>>(blocks, nblocks, dst);
    else k_dequantize_q6_k<false><<<grid, kThreads, 0, st>>>(blocks, nblocks, dst);
  } else {
    if (vec) k_dequantize_q4_k<true><<<grid, kThreads, 0, st>>>(blocks, nblocks, dst);
    else k_dequantize_q4_k<false><<<grid, kThreads, 0, st>>>(blocks, nblocks, dst);
  }
  return cuda_status(cudaGetLastError());
}

int launch_quantize_q8_0(const float* src, int64_t n, uint8_t* blocks, int8_t* qs, float* d,
                         cudaStream_t st) {
  const int64_t nb = n / 32;
  if (nb == 0) return LP_OK;
  const bool aligned = (reinterpret_cast<uintptr_t>(src) & 15) == 0 &&
                       (reinterpret_cast<uintptr_t>(qs) & 3) == 0 &&
                       (reinterpret_cast<uintptr_t>(blocks) & 1) == 0;
  if (!aligned) {
    k_quantize_q8_0<<<grid_for(nb * 32, kThreads), kThreads, 0, st>>>(src, nb, blocks, qs, d);
    return cuda_status(cudaGetLastError());
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid_for(nb * 4, 128)));
  cfg.blockDim = dim3(128);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cuda_status(cudaLaunchKernelEx(&cfg, k_quantize_q8_0_v4, src, nb, blocks, qs, d));
}

int launch_quantize_q4_0(const float* src, int64_t n, uint8_t* blocks, cudaStream_t st) {
  const int64_t nb = n / 32;
  if (nb == 0) return LP_OK;
  k_quantize_q4_0<<<grid_for(nb * 32, kThreads), kThreads, 0, st>>>(src, nb, blocks);
  return cuda_status(cudaGetLastError());
}

int launch_quantize_batch(const float* x, int64_t n, const float* scales, const float* zp,
                          int64_t gs, int8_t* dst, cudaStream_t st) {
  if (n == 0) return LP_OK;
  k_quantize_batch<<<grid_for(n, kThreads), kThreads, 0, st>>>(x, n, scales, zp, gs, dst);
  return cuda_status(cudaGetLastError());
}

int launch_calibrate(const float* x, int64_t n, int64_t gs, float qmax, int mx_emax, int mx,
                     float* scales, int64_t nscales, cudaStream_t st) {
  if (nscales == 0) return LP_OK;
  const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0 && n % 4 == 0 && gs % 4 == 0 &&
                   gs <= 128 && ((gs / 4) & (gs / 4 - 1)) == 0;
  if (vec) {
    const int64_t threads = nscales * (gs / 4);
    const int grid = static_cast<int>(std::min<int64_t>((threads + kThreads - 1) / kThreads,
                                                        int64_t{device_info().sm_count} * 16));
    const float4* x4 = reinterpret_cast<const float4*>(x);
    const int64_t n4 = n / 4;
    switch (gs / 4) {
      case 1: k_calibrate_vec<1><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
      case 2: k_calibrate_vec<2><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
      case 4: k_calibrate_vec<4><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
      case 8: k_calibrate_vec<8><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
      case 16: k_calibrate_vec<16><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
      default: k_calibrate_vec<32><<<grid, kThreads, 0, st>>>(x4, n4, qmax, mx_emax, mx, scales, nscales); break;
    }
    return cuda_status(cudaGetLastError());
  }
  const int grid = static_cast<int>(std::min<int64_t>(nscales, device_info().sm_count * 8));
  k_calibrate<<<grid, kThreads, 0, st>>>(x, n, gs, qmax, mx_emax, mx, scales, nscales);
  return cuda_status(cudaGetLastError());
}

int launch_quantize_packed(const float* x, int64_t n, const float* scales, int64_t gs, int f4,
                           uint8_t* packed, cudaStream_t st) {
  if (n == 0) return LP_OK;
  k_quantize_packed<<<grid_for((n + 1) / 2, kThreads), kThreads, 0, st>>>(x, n, scales, gs, f4,
                                                                           packed);
  return cuda_status(cudaGetLastError());
}

int launch_dequantize_blocks(const uint8_t* blocks, int64_t nblocks, int q4, float* dst,
                             cudaStream_t st) {
  if (nblocks == 0) return LP_OK;
  k_dequantize_blocks<<<grid_for(nblocks * 32, kThreads), kThreads, 0, st>>>(blocks, nblocks, q4,
                                                                             dst);
  return cuda_status(cudaGetLastError());
}

}  // namespace lp
