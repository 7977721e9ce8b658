// gemv_formats.cuh -- one policy per weight/activation format for the GEMV
// skeleton in gemv.cuh.  A policy supplies:
//   kScales      the format has a separate per-row scale array (streamed with
//                the weights) rather than scales inline in ggml blocks;
//   kFold        Serial (from 0.0, group order) or Lanes4 (ggml int8 forms);
//   stage_x      copies the activations into shared memory once per CTA;
//   prepare      loads what a thread keeps of group g's activations into
//                registers (called before term2 whenever g changes);
//   term2        the terms of two rows that share the prepared group g --
//                straight-line code, so two calls back to back interleave;
//   kFix / fix2  formats whose term2 can meet a group it does not handle
//                (block-float groups with a non-finite activation) redo those
//                terms in fix2.
//
// Exactness notes.  fp32 chains use mul.rn then add.rn (two roundings, no
// FMA), in the reference's scalar element order.  Small integers become
// floats exactly through the "magic" form: the float with bit pattern
// 0x4B000000 | u is 2^23 + u for u < 2^23, so subtracting 2^23 + bias yields
// u - bias exactly; a byte permute (prmt) builds that bit pattern from a
// packed byte in one instruction.  Two rows of the same group share the
// activations, so their chains run together as one packed f32x2 chain
// (add.rn.f32x2 / mul.rn.f32x2 round each lane exactly like the scalar op).
#pragma once
#include "gemv.cuh"

namespace lp {

// ------------------------------------------------------------- helpers
__device__ __forceinline__ float magic_byte(uint32_t word, int b) {
  // float(2^23 + byte b of word)
  return __uint_as_float(prmt(word, 0x4B000000u, 0x7440u | static_cast<uint32_t>(b)));
}
__device__ __forceinline__ uint64_t magic_pair(uint32_t wa, uint32_t wb, int b) {
  return pk(magic_byte(wa, b), magic_byte(wb, b));
}

// 32-bit loads of a 2-byte-aligned record in shared memory: word-aligned
// window of `NW` words starting at or before p; returns the byte offset (0/2).
template <int NW>
__device__ __forceinline__ int load_window(const uint8_t* p, uint32_t (&w)[NW]) {
  // (pointer arithmetic, not an integer round trip, so the compiler keeps
  // the shared-memory address space and emits shared loads)
  const int off = static_cast<int>(reinterpret_cast<uintptr_t>(p) & 3);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(p - off);
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = base[i];
  return off;
}

// ggml Q4_0 block (d:2, qs:16) at a 2-byte-aligned shared address.
__device__ __forceinline__ void load_q4_0(const uint8_t* p, uint32_t& d, uint32_t (&q)[4]) {
  uint32_t w[5];
  const int off = load_window<5>(p, w);
  const uint32_t sel = off ? 0x7654u : 0x5432u;
  d = (w[0] >> (off * 8)) & 0xFFFFu;
#pragma unroll
  for (int j = 0; j < 4; ++j) q[j] = prmt(w[j], w[j + 1], sel);
}
// ggml Q8_0 block (d:2, qs:32) at a 2-byte-aligned shared address.
__device__ __forceinline__ void load_q8_0(const uint8_t* p, uint32_t& d, uint32_t (&q)[8]) {
  uint32_t w[9];
  const int off = load_window<9>(p, w);
  const uint32_t sel = off ? 0x7654u : 0x5432u;
  d = (w[0] >> (off * 8)) & 0xFFFFu;
#pragma unroll
  for (int j = 0; j < 8; ++j) q[j] = prmt(w[j], w[j + 1], sel);
}

__device__ __forceinline__ int nib_at(const uint8_t* row, int kk) {
  const uint32_t b = row[kk >> 1];
  return static_cast<int>((kk & 1) ? (b >> 4) : (b & 15u));
}

// Staged fp32 activations use a swizzled layout: the 16-byte unit i (0..7) of
// 32-float block b lives at unit 8 b + (i ^ (b & 7)).  Consumer lanes load
// whole blocks of consecutive b, so without it the eight lanes of each
// shared-memory wavefront would all hit one bank group.
__device__ __forceinline__ int xsw(int kk) {
  const int b = kk >> 5;
  return (((b << 3) | (((kk >> 2) & 7) ^ (b & 7))) << 2) | (kk & 3);
}

// The fp32 activations of one group of 32, each duplicated into an f32x2.
struct XPairs {
  int g = -1;
  uint64_t x2[32];
  __device__ __forceinline__ void load(const float* x, int grp) {
    if (grp == g) return;
    g = grp;
    const float4* v = reinterpret_cast<const float4*>(x) + (grp << 3);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float4 f = v[i ^ (grp & 7)];
      x2[4 * i + 0] = pk(f.x, f.x);
      x2[4 * i + 1] = pk(f.y, f.y);
      x2[4 * i + 2] = pk(f.z, f.z);
      x2[4 * i + 3] = pk(f.w, f.w);
    }
  }
};

// fp32 activation staging shared by the fp32 formats (swizzled, see xsw).
struct StageXF32 {
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    const float* src = static_cast<const float*>(p.x);
    float* dst = reinterpret_cast<float*>(xsm);
    if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (p.k & 3) == 0) {
      const int n4 = p.k >> 2;
      for (int q = tid; q < n4; q += nthr) {
        const int b = q >> 3;
        reinterpret_cast<float4*>(dst)[(b << 3) | ((q & 7) ^ (b & 7))] =
            __ldg(reinterpret_cast<const float4*>(src) + q);
      }
    } else {
      for (int i = tid; i < p.k; i += nthr) dst[xsw(i)] = src[i];
    }
  }
};

// ============================================= fp32-activation formats

// dequantGemv (simd/dequant.nim:210-257; scalar order :253-256):
// int8 weights, partial = sum f32(w)*x in column order, term = partial*s.
struct FmtI8 : StageXF32 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;  // 64 registers of duplicated activations
  XPairs xp;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs == 32) xp.load(reinterpret_cast<const float*>(xsm), g);
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* x = reinterpret_cast<const float*>(xsm);
    if (p.gs == 32) {
      const uint4* pa = reinterpret_cast<const uint4*>(wA + g * 32);
      const uint4* pb = reinterpret_cast<const uint4*>(wB + g * 32);
      const uint4 a0 = pa[0], a1 = pa[1], b0 = pb[0], b1 = pb[1];
      const uint32_t A[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
      const uint32_t B[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
      const uint64_t bias = pk(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
      uint64_t acc = pk(0.0f, 0.0f);
      const uint64_t nz = pk(p.neg_zero, p.neg_zero);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint32_t ua = A[j] ^ 0x80808080u, ub = B[j] ^ 0x80808080u;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const uint64_t wv = add2(magic_pair(ua, ub, b), bias);
          acc = add2(acc, mul2_rn(wv, xp.x2[4 * j + b], nz));
        }
      }
      float pa_, pb_;
      upk(acc, pa_, pb_);
      tA = fmul(pa_, sA[g]);
      tB = fmul(pb_, sB[g]);
      return;
    }
    tA = generic(p, x, wA, sA, g);
    tB = generic(p, x, wB, sB, g);
  }
  static __device__ float generic(const GemvParams& p, const float* x, const uint8_t* w,
                                  const float* s, int g) {
    float partial = 0.0f;
    for (int kk = g * p.gs; kk < (g + 1) * p.gs; ++kk)
      partial = fadd(partial, fmul(i2f_rn(static_cast<int8_t>(w[kk])), x[xsw(kk)]));
    return fmul(partial, s[g]);
  }
};

// dequantGemvI4 (simd/dequant.nim:259-339; scalar :329-338): packed
// two's-complement nibbles, low nibble = even column.
struct FmtI4 : StageXF32 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;  // 64 registers of duplicated activations
  XPairs xp;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs == 32) xp.load(reinterpret_cast<const float*>(xsm), g);
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* x = reinterpret_cast<const float*>(xsm);
    if (p.gs == 32) {
      const uint4 a = *reinterpret_cast<const uint4*>(wA + g * 16);
      const uint4 bq = *reinterpret_cast<const uint4*>(wB + g * 16);
      const uint32_t A[4] = {a.x, a.y, a.z, a.w};
      const uint32_t B[4] = {bq.x, bq.y, bq.z, bq.w};
      const uint64_t bias = pk(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
      uint64_t acc = pk(0.0f, 0.0f);
      const uint64_t nz = pk(p.neg_zero, p.neg_zero);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        // n ^ 8 = value + 8 for a two's-complement nibble n
        const uint32_t loA = (A[j] & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t hiA = ((A[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t loB = (B[j] & 0x0F0F0F0Fu) ^ 0x08080808u;
        const uint32_t hiB = ((B[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int c = 8 * j + 2 * b;  // even column: low nibble of byte 4j+b
          const uint64_t we = add2(magic_pair(loA, loB, b), bias);
          acc = add2(acc, mul2_rn(we, xp.x2[c], nz));
          const uint64_t wo = add2(magic_pair(hiA, hiB, b), bias);
          acc = add2(acc, mul2_rn(wo, xp.x2[c + 1], nz));
        }
      }
      float pa_, pb_;
      upk(acc, pa_, pb_);
      tA = fmul(pa_, sA[g]);
      tB = fmul(pb_, sB[g]);
      return;
    }
    tA = generic(p, x, wA, sA, g);
    tB = generic(p, x, wB, sB, g);
  }
  static __device__ float generic(const GemvParams& p, const float* x, const uint8_t* w,
                                  const float* s, int g) {
    float partial = 0.0f;
    for (int kk = g * p.gs; kk < (g + 1) * p.gs; ++kk) {
      const int n = nib_at(w, kk);
      partial = fadd(partial, fmul(i2f_rn(n >= 8 ? n - 16 : n), x[xsw(kk)]));
    }
    return fmul(partial, s[g]);
  }
};

// dequantGemvF4 (simd/dequant.nim:341-420; scalar :375, :410-419):
// e2m1 codes decoded to 2x value (mxfp4Lut2x, :57-58), s = scale*0.5.
// Decode: a byte permute indexed by the raw 4-bit codes maps 4 codes to 4
// bytes u = lut2x + 12 at once.  Codes 0..7 index the positive table; codes
// 8..15 hit prmt's sign-replicate mode on it and read 0x00 (every table
// byte is < 0x80), and the mirrored lookup with bit 3 flipped fills them.
struct FmtF4 : StageXF32 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;  // 64 registers of duplicated activations
  XPairs xp;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs == 32) xp.load(reinterpret_cast<const float*>(xsm), g);
  }
  static __device__ __forceinline__ uint32_t lut4(uint32_t codes16) {
    // positive codes 0..7: 2v + 12 = 12,13,14,15,16,18,20,24
    // negative codes 8..15 (index c ^ 8): 12,11,10,9,8,6,4,0
    return prmt(0x0F0E0D0Cu, 0x18141210u, codes16) |
           prmt(0x090A0B0Cu, 0x00040608u, codes16 ^ 0x8888u);
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* x = reinterpret_cast<const float*>(xsm);
    if (p.gs == 32) {
      const uint4 a = *reinterpret_cast<const uint4*>(wA + g * 16);
      const uint4 bq = *reinterpret_cast<const uint4*>(wB + g * 16);
      const uint32_t A[4] = {a.x, a.y, a.z, a.w};
      const uint32_t B[4] = {bq.x, bq.y, bq.z, bq.w};
      const uint64_t bias = pk(-8388620.0f, -8388620.0f);  // -(2^23 + 12)
      uint64_t acc = pk(0.0f, 0.0f);
      const uint64_t nz = pk(p.neg_zero, p.neg_zero);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {  // 16-bit half = 4 codes = 4 columns
          const uint32_t ua = lut4(A[j] >> (16 * h));
          const uint32_t ub = lut4(B[j] >> (16 * h));
#pragma unroll
          for (int b = 0; b < 4; ++b) {
            const uint64_t wv = add2(magic_pair(ua, ub, b), bias);
            acc = add2(acc, mul2_rn(wv, xp.x2[8 * j + 4 * h + b], nz));
          }
        }
      }
      float pa_, pb_;
      upk(acc, pa_, pb_);
      tA = fmul(pa_, fmul(sA[g], 0.5f));
      tB = fmul(pb_, fmul(sB[g], 0.5f));
      return;
    }
    tA = generic(p, x, wA, sA, g);
    tB = generic(p, x, wB, sB, g);
  }
  static __device__ float generic(const GemvParams& p, const float* x, const uint8_t* w,
                                  const float* s, int g) {
    const int lut[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
    const float sc = fmul(s[g], 0.5f);
    float partial = 0.0f;
    for (int kk = g * p.gs; kk < (g + 1) * p.gs; ++kk)
      partial = fadd(partial, fmul(i2f_rn(lut[nib_at(w, kk)]), x[xsw(kk)]));
    return fmul(partial, sc);
  }
};

// dequantGemvQ8_0 (simd/dequant.nim:530-568; scalar :564-567).
struct FmtQ8_0 : StageXF32 {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;  // 64 registers of duplicated activations
  XPairs xp;
  __device__ __forceinline__ void prepare(const GemvParams&, const uint8_t* xsm, int g) {
    xp.load(reinterpret_cast<const float*>(xsm), g);
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[8], B[8];
    load_q8_0(wA + g * 34, dA, A);
    load_q8_0(wB + g * 34, dB, B);
    const uint64_t bias = pk(-8388736.0f, -8388736.0f);
    uint64_t acc = pk(0.0f, 0.0f);
      const uint64_t nz = pk(p.neg_zero, p.neg_zero);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const uint32_t ua = A[j] ^ 0x80808080u, ub = B[j] ^ 0x80808080u;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const uint64_t wv = add2(magic_pair(ua, ub, b), bias);
        acc = add2(acc, mul2_rn(wv, xp.x2[4 * j + b], nz));
      }
    }
    float pa_, pb_;
    upk(acc, pa_, pb_);
    tA = fmul(pa_, h2f(dA));
    tB = fmul(pb_, h2f(dB));
  }
};

// dequantGemvQ4_0 (simd/dequant.nim:570-622): the scalar order interleaves
// the halves: for i in 0..15, (lo_i - 8)*x[i] then (hi_i - 8)*x[i+16]
// (:616-620).
struct FmtQ4_0 : StageXF32 {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;  // 64 registers of duplicated activations
  XPairs xp;
  __device__ __forceinline__ void prepare(const GemvParams&, const uint8_t* xsm, int g) {
    xp.load(reinterpret_cast<const float*>(xsm), g);
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[4], B[4];
    load_q4_0(wA + g * 18, dA, A);
    load_q4_0(wB + g * 18, dB, B);
    const uint64_t bias = pk(-8388616.0f, -8388616.0f);  // -(2^23 + 8)
    uint64_t acc = pk(0.0f, 0.0f);
      const uint64_t nz = pk(p.neg_zero, p.neg_zero);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t loA = A[j] & 0x0F0F0F0Fu, hiA = (A[j] >> 4) & 0x0F0F0F0Fu;
      const uint32_t loB = B[j] & 0x0F0F0F0Fu, hiB = (B[j] >> 4) & 0x0F0F0F0Fu;
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        const int i = 4 * j + b;
        const uint64_t wl = add2(magic_pair(loA, loB, b), bias);
        acc = add2(acc, mul2_rn(wl, xp.x2[i], nz));
        const uint64_t wh = add2(magic_pair(hiA, hiB, b), bias);
        acc = add2(acc, mul2_rn(wh, xp.x2[i + 16], nz));
      }
    }
    float pa_, pb_;
    upk(acc, pa_, pb_);
    tA = fmul(pa_, h2f(dA));
    tB = fmul(pb_, h2f(dB));
  }
};

// ================================= fp32 activations, block-float path
//
// The fast fp32 path (the default; the scalar-order formats above are the
// bit-exact mode).  Each activation group j (the weight group) is written as
// integers X = rint(x * 2^(22 - E_j)) with 2^E_j > max|x| over the group, so
// |X| <= 2^22 and the representation error is at most 2^-23 of the group's
// largest magnitude.  X's two's-complement bytes are the digits:
// X = d0 + 256 d1 + 65536 d2 with d0, d1 unsigned and d2 = X >> 16 signed
// (planes P0..P2), and every group dot becomes three exact int32 dp4a sums
// of the integer weight codes against the planes.  Formats whose codes carry
// an offset (Q4_0: u = w + 8; I4: u = w + 8; F4: u = 2w + 12) start each
// plane sum at -offset * sum(d_p).  The group value is
// (65536 D2 + 256 D1 + D0) * 2^(E_j - 22); its only roundings are the final
// int->float conversions and the scaling, so it is within a few ulp of the
// exact dot -- well inside the reference's fp32 tolerance (1e-5 relative),
// not bit-identical to its sequential order.
// Groups holding a non-finite activation, or one of magnitude 2^100 or more
// (where the reference's fp32 partial sums can overflow), are marked (scale
// NaN) and take the scalar sequential path from global memory, so inf, NaN
// and overflow come out as in the reference.

struct GInfo {
  float s;       // 2^(E - 22); 0 for an all-zero group; NaN: sequential path
  int sx[3];     // sum of the group's digits in each plane (groups other than
                 // 32 wide; 32-wide groups leave them to PlaneCache)
};

constexpr uint32_t kBigBits = (100u + 127u) << 23;  // |x| >= 2^100

__device__ __forceinline__ int planes_stride(const GemvParams& p) { return (p.k + 15) & ~15; }

// Smallest E with m < 2^E for the bit pattern mb of a finite m > 0.
__device__ __forceinline__ int exp_above_bits(uint32_t mb) {
  const int e = static_cast<int>(mb >> 23);
  if (e) return e - 126;
  return 32 - __clz(static_cast<int>(mb)) - 149;  // subnormal: mb * 2^-149
}

// 2^e as float for e in [-149, 127]; 0 below.
__device__ __forceinline__ float pow2f(int e) {
  if (e >= -126) return __uint_as_float(static_cast<uint32_t>(e + 127) << 23);
  if (e >= -149) return __uint_as_float(1u << (e + 149));
  return 0.0f;
}

// rint(x * 2^sh) for |x * 2^sh| < 2^22 and sh in [-106, 171], in fp32 only:
// two exact power-of-two scalings (the first may only lose bits of values far
// below one half, which round to 0 either way), then round-to-nearest-even by
// adding 1.5 * 2^23, whose bit pattern then holds the integer.
__device__ __forceinline__ int scaled_rint(float x, float sa, float sb) {
  const float f = (x * sa) * sb;
  return __float_as_int(f + 12582912.0f) - 0x4B400000;
}
__device__ __forceinline__ void scale_pair(int sh, float& sa, float& sb) {
  const int a = min(sh, 127);
  sa = pow2f(a);
  sb = pow2f(sh - a);
}

// Group header from the largest |x| bit pattern of the group.
__device__ __forceinline__ GInfo group_info(uint32_t mb, const int (&sum)[3], bool special) {
  GInfo g;
  g.s = special ? __uint_as_float(0x7FC00000u)
                : (mb ? pow2f(exp_above_bits(mb) - 22) : 0.0f);
  g.sx[0] = sum[0];
  g.sx[1] = sum[1];
  g.sx[2] = sum[2];
  return g;
}

// kEvenOdd: within each 8-element chunk the planes hold the even columns
// then the odd ones (the order of low and high nibbles of packed int4).
template <bool kEvenOdd>
struct StageXPlanes {
  static __device__ __forceinline__ int pos(int k) {
    if (!kEvenOdd) return k;
    const int c = k & 7;
    return (k & ~7) | ((c & 1) << 2) | (c >> 1);
  }
  // Four lanes per 32-element group, eight activations each: the two 16-byte
  // loads of every lane go out together (under the weight stream an
  // activation load waits on the order of a microsecond) and only the group
  // maximum crosses lanes (two shuffles).  The digit sums are left to the
  // consumer threads (PlaneCache), which need them once per group.
  static __device__ __noinline__ void stage_g32(const float* x, int gpr, int8_t* P, int Kp,
                                                GInfo* gi, int tid, int nthr) {
    const int ntask = gpr * 4;
    for (int q0 = tid & ~31; q0 < ntask; q0 += nthr) {
      const int q = q0 + (tid & 31);
      const bool valid = q < ntask;
      const float4* xv4 = reinterpret_cast<const float4*>(x) + 2 * q;
      const float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
      const float4 f0 = valid ? __ldg(xv4) : z, f1 = valid ? __ldg(xv4 + 1) : z;
      const float v[8] = {f0.x, f0.y, f0.z, f0.w, f1.x, f1.y, f1.z, f1.w};
      uint32_t mb = 0;
#pragma unroll
      for (int i = 0; i < 8; ++i) mb = max(mb, __float_as_uint(v[i]) & 0x7FFFFFFFu);
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 1));
      mb = max(mb, __shfl_xor_sync(0xffffffffu, mb, 2));
      const bool special = mb >= kBigBits;  // also inf / NaN
      float sa, sb;
      scale_pair(22 - (mb ? exp_above_bits(mb) : 0), sa, sb);
      uint32_t word[3][2];
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        int X[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) X[i] = special ? 0 : scaled_rint(v[4 * c + i], sa, sb);
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
          const uint32_t sel = 0x0040u + 0x11u * pl;
          word[pl][c] = prmt(prmt(X[0], X[1], sel), prmt(X[2], X[3], sel), 0x5410u);
        }
      }
      if (valid) {
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) {
          uint32_t a = word[pl][0], b = word[pl][1];
          if (kEvenOdd) {  // the 8-element chunk: even columns, then odd
            const uint32_t e = prmt(a, b, 0x6420u), o = prmt(a, b, 0x7531u);
            a = e;
            b = o;
          }
          reinterpret_cast<uint2*>(P + pl * Kp)[q] = make_uint2(a, b);
        }
        if ((q & 3) == 0) {
          GInfo g;
          g.s = special ? __uint_as_float(0x7FC00000u) : (mb ? pow2f(exp_above_bits(mb) - 22) : 0.0f);
          g.sx[0] = g.sx[1] = g.sx[2] = 0;
          gi[q >> 2] = g;
        }
      }
    }
  }

  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    const float* x = static_cast<const float*>(p.x);
    const int Kp = planes_stride(p);
    int8_t* P = reinterpret_cast<int8_t*>(xsm);
    GInfo* gi = reinterpret_cast<GInfo*>(xsm + 3 * Kp);
    const int gs = p.gs;
    if (gs == 32 && (reinterpret_cast<uintptr_t>(x) & 15) == 0) {
      stage_g32(x, p.gpr, P, Kp, gi, tid, nthr);
    } else {
      for (int j = tid; j < p.gpr; j += nthr) {
        const float* xg = x + j * gs;
        uint32_t mb = 0;
        for (int i = 0; i < gs; ++i) mb = max(mb, __float_as_uint(xg[i]) & 0x7FFFFFFFu);
        const bool special = mb >= kBigBits;
        float sa, sb;
        scale_pair(22 - (mb ? exp_above_bits(mb) : 0), sa, sb);
        int sum[3] = {0, 0, 0};
        for (int i = 0; i < gs; ++i) {
          const int X = special ? 0 : scaled_rint(xg[i], sa, sb);
          const int d[3] = {X & 255, (X >> 8) & 255, X >> 16};
          const int at = pos(j * gs + i);
#pragma unroll
          for (int pl = 0; pl < 3; ++pl) {
            P[pl * Kp + at] = static_cast<int8_t>(d[pl]);
            sum[pl] += d[pl];
          }
        }
        gi[j] = group_info(mb, sum, special);
      }
    }
  }
};

// The planes and group data of one group, cached across the rows a thread
// visits (a thread keeps one group when the consumer count is a multiple of
// the groups per row).  Only used for 32-element groups.
template <int kOff>
struct PlaneCache {
  int g = -1;
  uint32_t P[3][8];
  int b[3];  // -kOff * sum(d_p)
  float s;
  __device__ __forceinline__ void load(const GemvParams& p, const uint8_t* xsm, int grp) {
    if (grp == g) return;
    g = grp;
    const int Kp = planes_stride(p);
#pragma unroll
    for (int pl = 0; pl < 3; ++pl) {
      const uint4 u0 = reinterpret_cast<const uint4*>(xsm + pl * Kp + grp * 32)[0];
      const uint4 u1 = reinterpret_cast<const uint4*>(xsm + pl * Kp + grp * 32)[1];
      P[pl][0] = u0.x; P[pl][1] = u0.y; P[pl][2] = u0.z; P[pl][3] = u0.w;
      P[pl][4] = u1.x; P[pl][5] = u1.y; P[pl][6] = u1.z; P[pl][7] = u1.w;
    }
    s = reinterpret_cast<const GInfo*>(xsm + 3 * Kp)[grp].s;
    if (kOff) {
      int sum[3] = {0, 0, 0};
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        sum[0] = dp4a_uu(0x01010101u, P[0][j], sum[0]);
        sum[1] = dp4a_uu(0x01010101u, P[1][j], sum[1]);
        sum[2] = dp4a_us(0x01010101u, P[2][j], sum[2]);
      }
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) b[pl] = -kOff * sum[pl];
    } else {
      b[0] = b[1] = b[2] = 0;
    }
  }
};

// (65536 D2 + 256 D1 + D0) as float.  kSmall: 32-element groups, where
// |D1| <= 32 * 255 * 255 < 2^21 so 256 D1 + D0 stays in int32.
template <bool kSmall>
__device__ __forceinline__ float bf_value(int a0, int a1, int a2) {
  if (kSmall)
    return fmaf(__int2float_rn(a2), 65536.0f, __int2float_rn(a1 * 256 + a0));
  return fmaf(__int2float_rn(a2), 65536.0f, fmaf(__int2float_rn(a1), 256.0f, __int2float_rn(a0)));
}

// Three plane sums of 4 codes against plane words w0..w2 (planes 0 and 1
// hold unsigned digits, plane 2 signed ones); codes unsigned (US) or signed (SS).
#define LP_DP3_US(acc, codes, w0, w1, w2)      \
  do {                                         \
    acc[0] = dp4a_uu(codes, w0, acc[0]);       \
    acc[1] = dp4a_uu(codes, w1, acc[1]);       \
    acc[2] = dp4a_us(codes, w2, acc[2]);       \
  } while (0)
#define LP_DP3_SS(acc, codes, w0, w1, w2)      \
  do {                                         \
    acc[0] = dp4a_su(codes, w0, acc[0]);       \
    acc[1] = dp4a_su(codes, w1, acc[1]);       \
    acc[2] = dp4a_ss(codes, w2, acc[2]);       \
  } while (0)

// Scalar sequential group sums from the unstaged fp32 activations (the
// non-finite-group path of the block-float formats).
__device__ __forceinline__ float seq_q4_0(const uint8_t* blk, const float* xg) {
  float partial = 0.0f;
  for (int i = 0; i < 16; ++i) {
    const int b = blk[2 + i];
    partial = fadd(partial, fmul(static_cast<float>((b & 15) - 8), xg[i]));
    partial = fadd(partial, fmul(static_cast<float>((b >> 4) - 8), xg[i + 16]));
  }
  return fmul(partial, h2f(blk[0] | (blk[1] << 8)));
}
__device__ __forceinline__ float seq_q8_0(const uint8_t* blk, const float* xg) {
  float partial = 0.0f;
  for (int i = 0; i < 32; ++i)
    partial = fadd(partial, fmul(static_cast<float>(static_cast<int8_t>(blk[2 + i])), xg[i]));
  return fmul(partial, h2f(blk[0] | (blk[1] << 8)));
}

// dequantGemvQ4_0, block-float path: u = nibble (w = u - 8), low nibbles
// against elements 0..15, high against 16..31.
struct FmtQ4_0F : StageXPlanes<false> {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Tree;
  static constexpr bool kFix = true;
  static constexpr bool kTwoPairs = true;
  PlaneCache<8> pc;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    pc.load(p, xsm, g);
  }
  __device__ __forceinline__ void fix2(const GemvParams& p, const uint8_t* wA, const uint8_t* wB,
                                       const float*, const float*, int g, float& tA, float& tB) {
    if (isnan(pc.s)) {
      const float* xg = static_cast<const float*>(p.x) + g * 32;
      tA = seq_q4_0(wA + g * 18, xg);
      tB = seq_q4_0(wB + g * 18, xg);
    }
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[4], B[4];
    load_q4_0(wA + g * 18, dA, A);
    load_q4_0(wB + g * 18, dB, B);
    int a[3] = {pc.b[0], pc.b[1], pc.b[2]};
    int c[3] = {pc.b[0], pc.b[1], pc.b[2]};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const uint32_t la = A[j] & 0x0F0F0F0Fu, ha = (A[j] >> 4) & 0x0F0F0F0Fu;
      const uint32_t lb = B[j] & 0x0F0F0F0Fu, hb = (B[j] >> 4) & 0x0F0F0F0Fu;
      LP_DP3_US(a, la, pc.P[0][j], pc.P[1][j], pc.P[2][j]);
      LP_DP3_US(c, lb, pc.P[0][j], pc.P[1][j], pc.P[2][j]);
      LP_DP3_US(a, ha, pc.P[0][j + 4], pc.P[1][j + 4], pc.P[2][j + 4]);
      LP_DP3_US(c, hb, pc.P[0][j + 4], pc.P[1][j + 4], pc.P[2][j + 4]);
    }
    tA = bf_value<true>(a[0], a[1], a[2]) * (h2f(dA) * pc.s);
    tB = bf_value<true>(c[0], c[1], c[2]) * (h2f(dB) * pc.s);
  }
};

// dequantGemvQ8_0, block-float path: signed codes, natural order.
struct FmtQ8_0F : StageXPlanes<false> {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Tree;
  static constexpr bool kFix = true;
  static constexpr bool kTwoPairs = true;
  PlaneCache<0> pc;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    pc.load(p, xsm, g);
  }
  __device__ __forceinline__ void fix2(const GemvParams& p, const uint8_t* wA, const uint8_t* wB,
                                       const float*, const float*, int g, float& tA, float& tB) {
    if (isnan(pc.s)) {
      const float* xg = static_cast<const float*>(p.x) + g * 32;
      tA = seq_q8_0(wA + g * 34, xg);
      tB = seq_q8_0(wB + g * 34, xg);
    }
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[8], B[8];
    load_q8_0(wA + g * 34, dA, A);
    load_q8_0(wB + g * 34, dB, B);
    int a[3] = {0, 0, 0};
    int c[3] = {0, 0, 0};
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      LP_DP3_SS(a, A[j], pc.P[0][j], pc.P[1][j], pc.P[2][j]);
      LP_DP3_SS(c, B[j], pc.P[0][j], pc.P[1][j], pc.P[2][j]);
    }
    tA = bf_value<true>(a[0], a[1], a[2]) * (h2f(dA) * pc.s);
    tB = bf_value<true>(c[0], c[1], c[2]) * (h2f(dB) * pc.s);
  }
};

// Group-scale formats (I8, I4, F4) on the block-float path: any group size
// that is a multiple of 8.  Codes per 8-element chunk c of group g come from
// Codes::get (two words of byte codes in plane order); planes from the cache
// (32-element groups) or shared memory.
template <class Codes>
struct FmtGroupF : StageXPlanes<Codes::kEvenOdd> {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Tree;
  static constexpr bool kFix = true;
  static constexpr bool kTwoPairs = true;
  PlaneCache<Codes::kOff> pc;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs == 32) pc.load(p, xsm, g);
  }
  __device__ __forceinline__ void fix2(const GemvParams& p, const uint8_t* wA, const uint8_t* wB,
                                       const float* sA, const float* sB, int g, float& tA,
                                       float& tB) {
    if (p.gs == 32 && isnan(pc.s)) {
      const float* xg = static_cast<const float*>(p.x) + g * 32;
      tA = Codes::seq(wA, g, 32, xg, sA[g]);
      tB = Codes::seq(wB, g, 32, xg, sB[g]);
    }
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const int Kp = planes_stride(p);
    float s;
    int a[3], c[3];
    if (p.gs == 32) {
      s = pc.s;
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) a[pl] = c[pl] = pc.b[pl];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t ua[2], ub[2];
        Codes::get(wA, g * 32 + 8 * ch, ua);
        Codes::get(wB, g * 32 + 8 * ch, ub);
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          Codes::dp3(a, ua[h], pc.P[0][2 * ch + h], pc.P[1][2 * ch + h], pc.P[2][2 * ch + h]);
          Codes::dp3(c, ub[h], pc.P[0][2 * ch + h], pc.P[1][2 * ch + h], pc.P[2][2 * ch + h]);
        }
      }
      tA = bf_value<true>(a[0], a[1], a[2]) * (Codes::scale(sA[g]) * s);
      tB = bf_value<true>(c[0], c[1], c[2]) * (Codes::scale(sB[g]) * s);
      return;
    } else {
      const GInfo gi = reinterpret_cast<const GInfo*>(xsm + 3 * Kp)[g];
      s = gi.s;
      if (!isnan(s)) {
#pragma unroll
        for (int pl = 0; pl < 3; ++pl) a[pl] = c[pl] = -Codes::kOff * gi.sx[pl];
        for (int e = g * p.gs; e < (g + 1) * p.gs; e += 8) {
          uint32_t ua[2], ub[2];
          Codes::get(wA, e, ua);
          Codes::get(wB, e, ub);
          uint2 w[3];
#pragma unroll
          for (int pl = 0; pl < 3; ++pl) w[pl] = *reinterpret_cast<const uint2*>(xsm + pl * Kp + e);
          Codes::dp3(a, ua[0], w[0].x, w[1].x, w[2].x);
          Codes::dp3(a, ua[1], w[0].y, w[1].y, w[2].y);
          Codes::dp3(c, ub[0], w[0].x, w[1].x, w[2].x);
          Codes::dp3(c, ub[1], w[0].y, w[1].y, w[2].y);
        }
      }
    }
    if (isnan(s)) {
      const float* xg = static_cast<const float*>(p.x) + g * p.gs;
      tA = Codes::seq(wA, g, p.gs, xg, sA[g]);
      tB = Codes::seq(wB, g, p.gs, xg, sB[g]);
      return;
    }
    tA = bf_value<false>(a[0], a[1], a[2]) * (Codes::scale(sA[g]) * s);
    tB = bf_value<false>(c[0], c[1], c[2]) * (Codes::scale(sB[g]) * s);
  }
};

// int8 codes, natural order.
struct CodesI8 {
  static constexpr bool kEvenOdd = false;
  static constexpr int kOff = 0;
  static __device__ __forceinline__ void get(const uint8_t* row, int e, uint32_t (&u)[2]) {
    const uint2 v = *reinterpret_cast<const uint2*>(row + e);
    u[0] = v.x;
    u[1] = v.y;
  }
  static __device__ __forceinline__ void dp3(int (&acc)[3], uint32_t u, uint32_t w0, uint32_t w1,
                                             uint32_t w2) {
    LP_DP3_SS(acc, u, w0, w1, w2);
  }
  static __device__ __forceinline__ float scale(float s) { return s; }
  static __device__ float seq(const uint8_t* row, int g, int gs, const float* xg, float s) {
    float partial = 0.0f;
    for (int i = 0; i < gs; ++i)
      partial = fadd(partial, fmul(static_cast<float>(static_cast<int8_t>(row[g * gs + i])), xg[i]));
    return fmul(partial, s);
  }
};

// packed two's-complement int4 (low nibble = even column): u = n ^ 8,
// low nibbles are the even columns, high the odd (planes in even/odd order).
struct CodesI4 {
  static constexpr bool kEvenOdd = true;
  static constexpr int kOff = 8;
  static __device__ __forceinline__ void get(const uint8_t* row, int e, uint32_t (&u)[2]) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(row + (e >> 1));
    u[0] = (v & 0x0F0F0F0Fu) ^ 0x08080808u;
    u[1] = ((v >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
  }
  static __device__ __forceinline__ void dp3(int (&acc)[3], uint32_t u, uint32_t w0, uint32_t w1,
                                             uint32_t w2) {
    LP_DP3_US(acc, u, w0, w1, w2);
  }
  static __device__ __forceinline__ float scale(float s) { return s; }
  static __device__ float seq(const uint8_t* row, int g, int gs, const float* xg, float s) {
    float partial = 0.0f;
    for (int i = 0; i < gs; ++i) {
      const int n = nib_at(row, g * gs + i);
      partial = fadd(partial, fmul(static_cast<float>(n >= 8 ? n - 16 : n), xg[i]));
    }
    return fmul(partial, s);
  }
};

// packed MXFP4 e2m1 codes: u = 2v + 12 via FmtF4::lut4, natural order.
struct CodesF4 {
  static constexpr bool kEvenOdd = false;
  static constexpr int kOff = 12;
  static __device__ __forceinline__ uint32_t lut4(uint32_t codes16) {
    return prmt(0x0F0E0D0Cu, 0x18141210u, codes16) |
           prmt(0x090A0B0Cu, 0x00040608u, codes16 ^ 0x8888u);
  }
  static __device__ __forceinline__ void get(const uint8_t* row, int e, uint32_t (&u)[2]) {
    const uint32_t v = *reinterpret_cast<const uint32_t*>(row + (e >> 1));
    u[0] = lut4(v);
    u[1] = lut4(v >> 16);
  }
  static __device__ __forceinline__ void dp3(int (&acc)[3], uint32_t u, uint32_t w0, uint32_t w1,
                                             uint32_t w2) {
    LP_DP3_US(acc, u, w0, w1, w2);
  }
  static __device__ __forceinline__ float scale(float s) { return s * 0.5f; }
  static __device__ float seq(const uint8_t* row, int g, int gs, const float* xg, float s) {
    const int lut[16] = {0, 1, 2, 3, 4, 6, 8, 12, 0, -1, -2, -3, -4, -6, -8, -12};
    float partial = 0.0f;
    for (int i = 0; i < gs; ++i)
      partial = fadd(partial, fmul(static_cast<float>(lut[nib_at(row, g * gs + i)]), xg[i]));
    return fmul(partial, fmul(s, 0.5f));
  }
};

struct FmtI8F : FmtGroupF<CodesI8> {};
struct FmtI4F : FmtGroupF<CodesI4> {};
struct FmtF4F : FmtGroupF<CodesF4> {};

// ------------------------------------------- k-quant fused GEMVs (GGUF)
// The reference dequantizes k-quant super-blocks (ggml.nim:108-213) but has
// no fused GEMV over them; these compute y = W x over the super-blocks
// directly, on the block-float path, with one 32-element group of a 256-
// element super-block as the skeleton's group.  Element values are the
// reference's: Q4_K fl(d*sc)*q - fl(dmin*m) (q 0..15, 6-bit sc/m per 32),
// Q6_K fl(d*sc)*(q - 32) (q 0..63, int8 sc per 16).  A group's integer dot
// sum(q * X) against the activation digit planes is exact, so a term is the
// block-float group value times fl(d*sc), minus (Q4_K) fl(dmin*m) times the
// group's activation sum -- within a few ulp of the exact term, not the
// reference's element order (none exists for a fused form).

// get_scale_min_k4 of ggml.nim:118-128: 6-bit scale and min of sub-block j.
__device__ __forceinline__ void kq_scale_min(int j, const uint8_t* q, int& sc, int& m) {
  if (j < 4) {
    sc = q[j] & 63;
    m = q[j + 4] & 63;
  } else {
    sc = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
    m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
  }
}

__device__ __forceinline__ uint32_t h16_at(const uint8_t* p) {
  return static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
}

// Sequential fp32 group sums from the unstaged activations (groups holding a
// non-finite or huge activation), over the reference's dequantized values.
__device__ __forceinline__ float seq_q4_k(const uint8_t* blk, int j, const float* xg) {
  int sc, m;
  kq_scale_min(j, blk + 4, sc, m);
  const float d1 = fmul(h2f(h16_at(blk)), i2f_rn(sc)), mm = fmul(h2f(h16_at(blk + 2)), i2f_rn(m));
  const uint8_t* qs = blk + 16 + 32 * (j >> 1);
  float partial = 0.0f;
  for (int l = 0; l < 32; ++l) {
    const int q = (j & 1) ? (qs[l] >> 4) : (qs[l] & 15);
    partial = fadd(partial, fmul(__fsub_rn(fmul(d1, i2f_rn(q)), mm), xg[l]));
  }
  return partial;
}
__device__ __forceinline__ int q6_code(const uint8_t* blk, int hh, int k, int l) {
  const uint32_t lo = blk[64 * hh + 32 * (k & 1) + l], hi = blk[128 + 32 * hh + l];
  return static_cast<int>(((k & 2) ? (lo >> 4) : (lo & 15u)) | (((hi >> (2 * k)) & 3u) << 4));
}
__device__ __forceinline__ float seq_q6_k(const uint8_t* blk, int gi, const float* xg) {
  const int hh = gi >> 2, k = gi & 3;
  const float d = h2f(h16_at(blk + 208));
  float partial = 0.0f;
  for (int l = 0; l < 32; ++l) {
    const int sc = static_cast<int8_t>(blk[192 + 8 * hh + (l >> 4) + 2 * k]);
    const float v = fmul(fmul(d, i2f_rn(sc)), i2f_rn(q6_code(blk, hh, k, l) - 32));
    partial = fadd(partial, fmul(v, xg[l]));
  }
  return partial;
}

// dequantizeQ4_K's values (ggml.nim:136-161) in a fused GEMV: 144-byte
// super-blocks (d, dmin, 12 bytes of 6-bit scales/mins, 128 bytes of
// nibbles); group j of a super-block is nibble j & 1 of qs bytes 32 (j >> 1)..
struct FmtQ4_KF : StageXPlanes<false> {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Tree;
  static constexpr bool kFix = true;
  static constexpr bool kTwoPairs = true;
  PlaneCache<1> pc;  // kOff = 1: b[p] = -(digit sum of plane p) -- the group's activation sum
  float xsum = 0.0f;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    pc.load(p, xsm, g);
    xsum = bf_value<true>(-pc.b[0], -pc.b[1], -pc.b[2]) * pc.s;
  }
  __device__ __forceinline__ void fix2(const GemvParams& p, const uint8_t* wA, const uint8_t* wB,
                                       const float*, const float*, int g, float& tA, float& tB) {
    if (isnan(pc.s)) {
      const float* xg = static_cast<const float*>(p.x) + g * 32;
      tA = seq_q4_k(wA + (g >> 3) * 144, g & 7, xg);
      tB = seq_q4_k(wB + (g >> 3) * 144, g & 7, xg);
    }
  }
  __device__ __forceinline__ float one(const uint8_t* blk, int j) const {
    const uint4* q = reinterpret_cast<const uint4*>(blk + 16 + 32 * (j >> 1));
    const uint4 u0 = q[0], u1 = q[1];
    const uint32_t w[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    const int sh = 4 * (j & 1);
    int a[3] = {0, 0, 0};
#pragma unroll
    for (int i = 0; i < 8; ++i) LP_DP3_US(a, (w[i] >> sh) & 0x0F0F0F0Fu, pc.P[0][i], pc.P[1][i], pc.P[2][i]);
    int sc, m;
    kq_scale_min(j, blk + 4, sc, m);
    const float d1 = h2f(h16_at(blk)) * static_cast<float>(sc);
    const float mm = h2f(h16_at(blk + 2)) * static_cast<float>(m);
    return d1 * (bf_value<true>(a[0], a[1], a[2]) * pc.s) - mm * xsum;
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*, const uint8_t* wA,
                                        const uint8_t* wB, const float*, const float*, int g,
                                        float& tA, float& tB) {
    tA = one(wA + (g >> 3) * 144, g & 7);
    tB = one(wB + (g >> 3) * 144, g & 7);
  }
};

// dequantizeQ6_K's values (ggml.nim:163-213) in a fused GEMV: 210-byte
// super-blocks (ql[128], qh[64], int8 scales[16], d); group gi = 4 hh + k of a
// super-block holds elements 128 hh + 32 k + l, two scales (l < 16, l >= 16).
struct FmtQ6_KF : StageXPlanes<false> {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Tree;
  static constexpr bool kFix = true;
  static constexpr bool kTwoPairs = true;
  PlaneCache<0> pc;
  int off32[2][3];  // -32 * digit sums of each half of the group, per plane
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    pc.load(p, xsm, g);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      int s[3] = {0, 0, 0};
#pragma unroll
      for (int i = 4 * h; i < 4 * h + 4; ++i) {
        s[0] = dp4a_uu(0x01010101u, pc.P[0][i], s[0]);
        s[1] = dp4a_uu(0x01010101u, pc.P[1][i], s[1]);
        s[2] = dp4a_us(0x01010101u, pc.P[2][i], s[2]);
      }
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) off32[h][pl] = -32 * s[pl];
    }
  }
  __device__ __forceinline__ void fix2(const GemvParams& p, const uint8_t* wA, const uint8_t* wB,
                                       const float*, const float*, int g, float& tA, float& tB) {
    if (isnan(pc.s)) {
      const float* xg = static_cast<const float*>(p.x) + g * 32;
      tA = seq_q6_k(wA + (g >> 3) * 210, g & 7, xg);
      tB = seq_q6_k(wB + (g >> 3) * 210, g & 7, xg);
    }
  }
  __device__ __forceinline__ float one(const uint8_t* blk, int gi) const {
    const int hh = gi >> 2, k = gi & 3;
    uint32_t lo[8], hi[8], w[9];
    // 32 bytes at a 2-byte-aligned address: a word window and byte permutes
    int off = load_window<9>(blk + 64 * hh + 32 * (k & 1), w);
    uint32_t sel = off ? 0x5432u : 0x3210u;
#pragma unroll
    for (int i = 0; i < 8; ++i) lo[i] = prmt(w[i], w[i + 1], sel);
    off = load_window<9>(blk + 128 + 32 * hh, w);
    sel = off ? 0x5432u : 0x3210u;
#pragma unroll
    for (int i = 0; i < 8; ++i) hi[i] = prmt(w[i], w[i + 1], sel);
    const int lsh = (k & 2) ? 4 : 0, hsh = 2 * k;
    int a[2][3];
#pragma unroll
    for (int h = 0; h < 2; ++h)
#pragma unroll
      for (int pl = 0; pl < 3; ++pl) a[h][pl] = off32[h][pl];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const uint32_t code = ((lo[i] >> lsh) & 0x0F0F0F0Fu) | (((hi[i] >> hsh) & 0x03030303u) << 4);
      LP_DP3_US(a[i >> 2], code, pc.P[0][i], pc.P[1][i], pc.P[2][i]);
    }
    const float d = h2f(h16_at(blk + 208));
    const float s0 = d * static_cast<float>(static_cast<int8_t>(blk[192 + 8 * hh + 2 * k]));
    const float s1 = d * static_cast<float>(static_cast<int8_t>(blk[192 + 8 * hh + 2 * k + 1]));
    return (s0 * bf_value<true>(a[0][0], a[0][1], a[0][2]) +
            s1 * bf_value<true>(a[1][0], a[1][1], a[1][2])) * pc.s;
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*, const uint8_t* wA,
                                        const uint8_t* wB, const float*, const float*, int g,
                                        float& tA, float& tB) {
    tA = one(wA + (g >> 3) * 210, g & 7);
    tB = one(wB + (g >> 3) * 210, g & 7);
  }
};

// ============================================= int8-activation formats

// Group-scale int8 activations: xq (k bytes) then xScales (gpr floats).
struct StageXQ8 {
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    copy_bytes(xsm, static_cast<const uint8_t*>(p.x), p.k, tid, nthr);
    const int xoff = (p.k + 15) & ~15;
    copy_bytes(xsm + xoff, reinterpret_cast<const uint8_t*>(p.xs), p.gpr * 4, tid, nthr);
  }
  static __device__ __forceinline__ const float* xscales(const GemvParams& p,
                                                         const uint8_t* xsm) {
    return reinterpret_cast<const float*>(xsm + ((p.k + 15) & ~15));
  }
};

// fp32 activations quantized to Q8_0 while they are staged -- the same
// arithmetic as quantizeQ8_0 (ggml.nim:60-75, k_quantize_q8_0): amax of the
// 32-value block, d = fl(amax / 127), id = d ? fl(1 / d) : 0, q =
// clamp(roundf(fl(x * id)), +-127), scale = f32(f16(d)) -- into StageXQ8's
// layout, so quantizeQ8_0 followed by a Q8-activation GEMV becomes one launch
// with the two-launch bits.  Eight threads per block, four values each.
struct StageXQ8FromF32 {
  static __device__ __noinline__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid,
                                              int nthr) {
    const float* x = static_cast<const float*>(p.x);
    uint32_t* q = reinterpret_cast<uint32_t*>(xsm);
    float* xs = reinterpret_cast<float*>(xsm + ((p.k + 15) & ~15));
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    const int ntask = p.gpr * 8;
    // Under the weight stream an activation load waits on the order of a
    // microsecond, so each thread issues the loads of up to kR rounds before
    // it uses any (one wait instead of one per round).
    constexpr int kR = 8;
    for (int b0 = tid & ~31; b0 < ntask; b0 += kR * nthr) {
      float4 v[kR];
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        const int t = b0 + r * nthr + (tid & 31);
        v[r] = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < ntask)
          v[r] = vec ? __ldg(reinterpret_cast<const float4*>(x) + t)
                     : make_float4(__ldg(x + 4 * t), __ldg(x + 4 * t + 1), __ldg(x + 4 * t + 2),
                                   __ldg(x + 4 * t + 3));
      }
#pragma unroll
      for (int r = 0; r < kR; ++r) {
        const int t = b0 + r * nthr + (tid & 31);
        if (b0 + r * nthr >= ntask) break;  // warp-uniform
        float a = fmaxf(fmaxf(fabsf(v[r].x), fabsf(v[r].y)), fmaxf(fabsf(v[r].z), fabsf(v[r].w)));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 1));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 2));
        a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, 4));
        // d and 1/d once per 32-element block (lane 0 of its 8), then shared
        float d = 0.0f, id = 0.0f;
        if ((tid & 7) == 0) {
          d = __fdiv_rn(a, 127.0f);
          id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        }
        d = __shfl_sync(0xffffffffu, d, (tid & 31) & ~7);
        id = __shfl_sync(0xffffffffu, id, (tid & 31) & ~7);
        if (t >= ntask) continue;
        const float e[4] = {v[r].x, v[r].y, v[r].z, v[r].w};
        uint32_t word = 0;
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          float rr = roundf(__fmul_rn(e[i], id));
          rr = fminf(fmaxf(rr, -127.0f), 127.0f);
          word |= (static_cast<uint32_t>(static_cast<int>(rr)) & 0xFFu) << (8 * i);
        }
        q[t] = word;
        if ((t & 7) == 0) xs[t >> 3] = h2f(__half_as_ushort(__float2half_rn(d)));
      }
    }
  }
};

// dequantGemvQ8 (simd/dequant.nim:753-878; scalar :868-878).
struct FmtQ8 : StageXQ8 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = true;
  int cg = -1;
  uint32_t X[8];
  float xsg;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs != 32 || g == cg) return;
    cg = g;
    const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
    X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
    X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
    xsg = xscales(p, xsm)[g];
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* xs = xscales(p, xsm);
    if (p.gs == 32) {
      const uint4* pa = reinterpret_cast<const uint4*>(wA + g * 32);
      const uint4* pb = reinterpret_cast<const uint4*>(wB + g * 32);
      const uint4 a0 = pa[0], a1 = pa[1], b0 = pb[0], b1 = pb[1];
      int ia = 0, ib = 0;
      ia = dp4a_ss(a0.x, X[0], ia); ib = dp4a_ss(b0.x, X[0], ib);
      ia = dp4a_ss(a0.y, X[1], ia); ib = dp4a_ss(b0.y, X[1], ib);
      ia = dp4a_ss(a0.z, X[2], ia); ib = dp4a_ss(b0.z, X[2], ib);
      ia = dp4a_ss(a0.w, X[3], ia); ib = dp4a_ss(b0.w, X[3], ib);
      ia = dp4a_ss(a1.x, X[4], ia); ib = dp4a_ss(b1.x, X[4], ib);
      ia = dp4a_ss(a1.y, X[5], ia); ib = dp4a_ss(b1.y, X[5], ib);
      ia = dp4a_ss(a1.z, X[6], ia); ib = dp4a_ss(b1.z, X[6], ib);
      ia = dp4a_ss(a1.w, X[7], ia); ib = dp4a_ss(b1.w, X[7], ib);
      tA = fmul(fmul(i2f_rn(ia), sA[g]), xsg);
      tB = fmul(fmul(i2f_rn(ib), sB[g]), xsg);
      return;
    }
    tA = generic(p, xsm, wA, sA[g], xs[g], g);
    tB = generic(p, xsm, wB, sB[g], xs[g], g);
  }
  static __device__ float generic(const GemvParams& p, const uint8_t* xq, const uint8_t* w,
                                  float ws, float xs, int g) {
    int isum = 0;
    for (int kk = g * p.gs; kk < (g + 1) * p.gs; ++kk)
      isum += static_cast<int>(static_cast<int8_t>(w[kk])) * static_cast<int8_t>(xq[kk]);
    return fmul(fmul(i2f_rn(isum), ws), xs);
  }
};

// dequantGemvI4Q8 (simd/dequant.nim:968-1145; scalar :1134-1145).  With
// t = nibble ^ 8 (0..15) the weight is t - 8, so the exact group dot is
// dp4a(t, x) - 8 * sum(x) with unsigned-by-signed byte dots; the activations
// are split into even/odd columns once per group to line up with the low and
// high nibbles.
struct FmtI4Q8 : StageXQ8 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = true;
  int cg = -1;
  uint32_t XE[4], XO[4];
  int sumx8;
  float xsg;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (p.gs != 32 || g == cg) return;
    cg = g;
    const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
    const uint32_t X[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
    int sx = 0;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      XE[j] = prmt(X[2 * j], X[2 * j + 1], 0x6420u);
      XO[j] = prmt(X[2 * j], X[2 * j + 1], 0x7531u);
      sx = dp4a_us(0x01010101u, X[2 * j], sx);
      sx = dp4a_us(0x01010101u, X[2 * j + 1], sx);
    }
    sumx8 = 8 * sx;
    xsg = xscales(p, xsm)[g];
  }
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* xs = xscales(p, xsm);
    if (p.gs == 32) {
      const uint4 a = *reinterpret_cast<const uint4*>(wA + g * 16);
      const uint4 bq = *reinterpret_cast<const uint4*>(wB + g * 16);
      const uint32_t A[4] = {a.x, a.y, a.z, a.w};
      const uint32_t B[4] = {bq.x, bq.y, bq.z, bq.w};
      int ia = -sumx8, ib = -sumx8;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        ia = dp4a_us((A[j] & 0x0F0F0F0Fu) ^ 0x08080808u, XE[j], ia);
        ia = dp4a_us(((A[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, XO[j], ia);
        ib = dp4a_us((B[j] & 0x0F0F0F0Fu) ^ 0x08080808u, XE[j], ib);
        ib = dp4a_us(((B[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u, XO[j], ib);
      }
      tA = fmul(fmul(i2f_rn(ia), sA[g]), xsg);
      tB = fmul(fmul(i2f_rn(ib), sB[g]), xsg);
      return;
    }
    tA = generic(p, xsm, wA, sA[g], xs[g], g);
    tB = generic(p, xsm, wB, sB[g], xs[g], g);
  }
  static __device__ float generic(const GemvParams& p, const uint8_t* xq, const uint8_t* w,
                                  float ws, float xs, int g) {
    int isum = 0;
    for (int kk = g * p.gs; kk < (g + 1) * p.gs; ++kk) {
      const int n = nib_at(w, kk);
      isum += (n >= 8 ? n - 16 : n) * static_cast<int8_t>(xq[kk]);
    }
    return fmul(fmul(i2f_rn(isum), ws), xs);
  }
};

// quantizeQ8_0 of fp32 x, then dequantGemvQ8 / dequantGemvI4Q8, in one launch.
struct FmtQ8FromF32 : FmtQ8 {
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    StageXQ8FromF32::stage_x(xsm, p, tid, nthr);
  }
};
struct FmtI4Q8FromF32 : FmtI4Q8 {
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    StageXQ8FromF32::stage_x(xsm, p, tid, nthr);
  }
};

// ----------------------------------------------- small-n GEMM (columns)
// dequantGemmQ8 / dequantGemmI4Q8 for a few activation columns
// (simd/dequant.nim:1382-1583; scalar :1449-1458):
//   y[row * n + c] = fold_g fl(fl(f32(isum) * ws[row, g]) * xs[c * gpr + g]),
// serial over g from 0.0 -- the GEMV term of each column.  Staged once per
// CTA: the n columns of xq (K x n, column-major: column c is K bytes) and
// xs (n x gpr).  Group size 32 only; the weight group is loaded once and
// dotted with every column.
struct StageXCols {
  static __device__ __forceinline__ int xs_off(const GemvParams& p) {
    return (p.k * p.ncol + 15) & ~15;
  }
  static __device__ __forceinline__ const float* xscales(const GemvParams& p,
                                                         const uint8_t* xsm) {
    return reinterpret_cast<const float*>(xsm + xs_off(p));
  }
};

struct FmtQ8Cols : StageXCols {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;
  static constexpr bool kCols = true;
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    copy_bytes(xsm, static_cast<const uint8_t*>(p.x), p.k * p.ncol, tid, nthr);
    copy_bytes(xsm + xs_off(p), reinterpret_cast<const uint8_t*>(p.xs), p.gpr * p.ncol * 4, tid,
               nthr);
  }
  // Rows A and B (TB == nullptr: row B is a duplicate of A and not stored).
  __device__ __forceinline__ void termcols2(const GemvParams& p, const uint8_t* xsm,
                                            const uint8_t* wA, const uint8_t* wB, const float* sA,
                                            const float* sB, int g, float* TA, float* TB,
                                            int tstride) {
    // Consecutive lanes take consecutive groups, 32 bytes apart: lanes g
    // and g + 4 would meet in the same banks, so lanes with bit 2 of g set
    // read the second 16 bytes first (weights and activations alike; the
    // integer dot does not depend on the order of its words).
    const int sw = (g >> 2) & 1;
    const uint4* pa = reinterpret_cast<const uint4*>(wA + g * 32);
    const uint4* pb = reinterpret_cast<const uint4*>(wB + g * 32);
    const uint4 a0 = pa[sw], a1 = pa[sw ^ 1], b0 = pb[sw], b1 = pb[sw ^ 1];
    const float ga = sA[g], gb = sB[g];
    const float* xs = xscales(p, xsm);
#pragma unroll 2
    for (int c = 0; c < p.ncol; ++c) {
      const uint4* px = reinterpret_cast<const uint4*>(xsm + c * p.k + g * 32);
      const uint4 x0 = px[sw], x1 = px[sw ^ 1];
      int ia = 0, ib = 0;
      ia = dp4a_ss(a0.x, x0.x, ia); ib = dp4a_ss(b0.x, x0.x, ib);
      ia = dp4a_ss(a0.y, x0.y, ia); ib = dp4a_ss(b0.y, x0.y, ib);
      ia = dp4a_ss(a0.z, x0.z, ia); ib = dp4a_ss(b0.z, x0.z, ib);
      ia = dp4a_ss(a0.w, x0.w, ia); ib = dp4a_ss(b0.w, x0.w, ib);
      ia = dp4a_ss(a1.x, x1.x, ia); ib = dp4a_ss(b1.x, x1.x, ib);
      ia = dp4a_ss(a1.y, x1.y, ia); ib = dp4a_ss(b1.y, x1.y, ib);
      ia = dp4a_ss(a1.z, x1.z, ia); ib = dp4a_ss(b1.z, x1.z, ib);
      ia = dp4a_ss(a1.w, x1.w, ia); ib = dp4a_ss(b1.w, x1.w, ib);
      const float xsc = xs[c * p.gpr + g];
      TA[c * tstride + g] = fmul(fmul(i2f_rn(ia), ga), xsc);
      if (TB) TB[c * tstride + g] = fmul(fmul(i2f_rn(ib), gb), xsc);
    }
  }
};

// The int4 weights as in FmtI4Q8 (t = nibble ^ 8, weight t - 8; low nibble =
// even column): the staging splits each column's group into its even and odd
// bytes (16 + 16) and keeps 8 * sum(x) per (column, group), after xs.
struct FmtI4Q8Cols : StageXCols {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = false;
  static constexpr bool kCols = true;
  static __device__ __forceinline__ const int* sums8(const GemvParams& p, const uint8_t* xsm) {
    return reinterpret_cast<const int*>(xsm + xs_off(p) + p.gpr * p.ncol * 4);
  }
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    copy_bytes(xsm + xs_off(p), reinterpret_cast<const uint8_t*>(p.xs), p.gpr * p.ncol * 4, tid,
               nthr);
    int* s8 = const_cast<int*>(sums8(p, xsm));
    const uint8_t* xq = static_cast<const uint8_t*>(p.x);
    for (int u = tid; u < p.gpr * p.ncol; u += nthr) {  // u = c * gpr + g
      const uint4* src = reinterpret_cast<const uint4*>(xq + u * 32);
      const uint4 u0 = __ldg(src), u1 = __ldg(src + 1);
      const uint32_t X[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
      uint32_t E[4], O[4];
      int sx = 0;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        E[j] = prmt(X[2 * j], X[2 * j + 1], 0x6420u);
        O[j] = prmt(X[2 * j], X[2 * j + 1], 0x7531u);
        sx = dp4a_us(0x01010101u, X[2 * j], sx);
        sx = dp4a_us(0x01010101u, X[2 * j + 1], sx);
      }
      uint4* dst = reinterpret_cast<uint4*>(xsm + u * 32);
      dst[0] = make_uint4(E[0], E[1], E[2], E[3]);
      dst[1] = make_uint4(O[0], O[1], O[2], O[3]);
      s8[u] = 8 * sx;
    }
  }
  __device__ __forceinline__ void termcols2(const GemvParams& p, const uint8_t* xsm,
                                            const uint8_t* wA, const uint8_t* wB, const float* sA,
                                            const float* sB, int g, float* TA, float* TB,
                                            int tstride) {
    const uint4 a = *reinterpret_cast<const uint4*>(wA + g * 16);
    const uint4 b = *reinterpret_cast<const uint4*>(wB + g * 16);
    const uint32_t A[4] = {a.x, a.y, a.z, a.w}, B[4] = {b.x, b.y, b.z, b.w};
    uint32_t alo[4], ahi[4], blo[4], bhi[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      alo[j] = (A[j] & 0x0F0F0F0Fu) ^ 0x08080808u;
      ahi[j] = ((A[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
      blo[j] = (B[j] & 0x0F0F0F0Fu) ^ 0x08080808u;
      bhi[j] = ((B[j] >> 4) & 0x0F0F0F0Fu) ^ 0x08080808u;
    }
    const float ga = sA[g], gb = sB[g];
    const float* xs = xscales(p, xsm);
    const int* s8 = sums8(p, xsm);
    // As in FmtQ8Cols: lanes with bit 2 of g set read the odd half (16
    // bytes) of their 32 first, paired with the odd-column weights.
    const int sw = (g >> 2) & 1;
    uint32_t a1[4], a2[4], b1[4], b2[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      a1[j] = sw ? ahi[j] : alo[j];
      a2[j] = sw ? alo[j] : ahi[j];
      b1[j] = sw ? bhi[j] : blo[j];
      b2[j] = sw ? blo[j] : bhi[j];
    }
#pragma unroll 2
    for (int c = 0; c < p.ncol; ++c) {
      const int u = c * p.gpr + g;
      const uint4* px = reinterpret_cast<const uint4*>(xsm + u * 32);
      const uint4 h1 = px[sw], h2 = px[sw ^ 1];  // paired with a1/b1, a2/b2
      int ia = -s8[u], ib = ia;
      ia = dp4a_us(a1[0], h1.x, ia); ib = dp4a_us(b1[0], h1.x, ib);
      ia = dp4a_us(a2[0], h2.x, ia); ib = dp4a_us(b2[0], h2.x, ib);
      ia = dp4a_us(a1[1], h1.y, ia); ib = dp4a_us(b1[1], h1.y, ib);
      ia = dp4a_us(a2[1], h2.y, ia); ib = dp4a_us(b2[1], h2.y, ib);
      ia = dp4a_us(a1[2], h1.z, ia); ib = dp4a_us(b1[2], h1.z, ib);
      ia = dp4a_us(a2[2], h2.z, ia); ib = dp4a_us(b2[2], h2.z, ib);
      ia = dp4a_us(a1[3], h1.w, ia); ib = dp4a_us(b1[3], h1.w, ib);
      ia = dp4a_us(a2[3], h2.w, ia); ib = dp4a_us(b2[3], h2.w, ib);
      const float xsc = xs[u];
      TA[c * tstride + g] = fmul(fmul(i2f_rn(ia), ga), xsc);
      if (TB) TB[c * tstride + g] = fmul(fmul(i2f_rn(ib), gb), xsc);
    }
  }
};

// ggml Q8_0 activation blocks staged as qs (k bytes) + decoded d (bpr floats),
// the once-per-call decode of simd/dequant.nim:1171-1175.
struct StageXBlocks {
  static __device__ void stage_x(uint8_t* xsm, const GemvParams& p, int tid, int nthr) {
    const uint8_t* xb = static_cast<const uint8_t*>(p.x);
    float* xd = reinterpret_cast<float*>(xsm + ((p.k + 15) & ~15));
    for (int i = tid; i < p.k; i += nthr) xsm[(i >> 5) * 32 + (i & 31)] = xb[(i >> 5) * 34 + 2 + (i & 31)];
    for (int b = tid; b < p.gpr; b += nthr) {
      const uint32_t h = static_cast<uint32_t>(xb[b * 34]) | (static_cast<uint32_t>(xb[b * 34 + 1]) << 8);
      xd[b] = h2f(h);
    }
  }
  static __device__ __forceinline__ const float* xd(const GemvParams& p, const uint8_t* xsm) {
    return reinterpret_cast<const float*>(xsm + ((p.k + 15) & ~15));
  }
};

// dequantGemvQ8_0Q8 (simd/dequant.nim:1187-1286): term = f32(isum)*(wd*xd),
// 4-lane fold.
struct FmtQ8_0Q8 : StageXBlocks {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Lanes4;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = true;
  int cg = -1;
  uint32_t X[8];
  float xdg;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (g == cg) return;
    cg = g;
    const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
    X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
    X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
    xdg = xd(p, xsm)[g];
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[8], B[8];
    load_q8_0(wA + g * 34, dA, A);
    load_q8_0(wB + g * 34, dB, B);
    int ia = 0, ib = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      ia = dp4a_ss(A[j], X[j], ia);
      ib = dp4a_ss(B[j], X[j], ib);
    }
    tA = fmul(i2f_rn(ia), fmul(h2f(dA), xdg));
    tB = fmul(i2f_rn(ib), fmul(h2f(dB), xdg));
  }
};

// dequantGemvQ4_0Q8 (simd/dequant.nim:1288-1365): q = nibble - 8, low
// nibbles against activation lanes 0..15, high against 16..31.
struct FmtQ4_0Q8 : StageXBlocks {
  static constexpr bool kScales = false;
  static constexpr Fold kFold = Fold::Lanes4;
  static constexpr bool kFix = false;
  static constexpr bool kTwoPairs = true;
  int cg = -1;
  uint32_t X[8];
  int sumx8;
  float xdg;
  __device__ __forceinline__ void prepare(const GemvParams& p, const uint8_t* xsm, int g) {
    if (g == cg) return;
    cg = g;
    const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
    const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
    X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
    X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
    int sx = 0;
#pragma unroll
    for (int j = 0; j < 8; ++j) sx = dp4a_us(0x01010101u, X[j], sx);
    sumx8 = 8 * sx;
    xdg = xd(p, xsm)[g];
  }
  __device__ __forceinline__ void term2(const GemvParams&, const uint8_t*,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    uint32_t dA, dB, A[4], B[4];
    load_q4_0(wA + g * 18, dA, A);
    load_q4_0(wB + g * 18, dB, B);
    int ia = -sumx8, ib = -sumx8;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      ia = dp4a_us(A[j] & 0x0F0F0F0Fu, X[j], ia);
      ia = dp4a_us((A[j] >> 4) & 0x0F0F0F0Fu, X[j + 4], ia);
      ib = dp4a_us(B[j] & 0x0F0F0F0Fu, X[j], ib);
      ib = dp4a_us((B[j] >> 4) & 0x0F0F0F0Fu, X[j + 4], ib);
    }
    tA = fmul(i2f_rn(ia), fmul(h2f(dA), xdg));
    tB = fmul(i2f_rn(ib), fmul(h2f(dB), xdg));
  }
};

}  // namespace lp
