// gemv_formats.cuh -- one policy per weight/activation format for the GEMV
// skeleton in gemv.cuh.  A policy supplies:
//   kScales      the format has a separate per-row scale array (streamed with
//                the weights) rather than scales inline in ggml blocks;
//   kFold        Serial (from 0.0, group order) or Lanes4 (ggml int8 forms);
//   stage_x      copies the activations into shared memory once per CTA;
//   term2        the terms of two rows that share group g.
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
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  const uint32_t* base = reinterpret_cast<const uint32_t*>(a & ~uintptr_t(3));
#pragma unroll
  for (int i = 0; i < NW; ++i) w[i] = base[i];
  return static_cast<int>(a & 3);
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
  XPairs xp;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* x = reinterpret_cast<const float*>(xsm);
    if (p.gs == 32) {
      xp.load(x, g);
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
  XPairs xp;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* x = reinterpret_cast<const float*>(xsm);
    if (p.gs == 32) {
      xp.load(x, g);
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
  XPairs xp;
  __device__ void init(const GemvParams&, const uint8_t*) {}
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
      xp.load(x, g);
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
  XPairs xp;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    xp.load(reinterpret_cast<const float*>(xsm), g);
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
  XPairs xp;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    xp.load(reinterpret_cast<const float*>(xsm), g);
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

// dequantGemvQ8 (simd/dequant.nim:753-878; scalar :868-878).
struct FmtQ8 : StageXQ8 {
  static constexpr bool kScales = true;
  static constexpr Fold kFold = Fold::Serial;
  int cg = -1;
  uint32_t X[8];
  float xsg;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* xs = xscales(p, xsm);
    if (p.gs == 32) {
      if (g != cg) {
        cg = g;
        const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
        const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
        X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
        X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
        xsg = xs[g];
      }
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
  int cg = -1;
  uint32_t XE[4], XO[4];
  int sumx8;
  float xsg;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float* sA,
                                        const float* sB, int g, float& tA, float& tB) {
    const float* xs = xscales(p, xsm);
    if (p.gs == 32) {
      if (g != cg) {
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
        xsg = xs[g];
      }
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
  int cg = -1;
  uint32_t X[8];
  float xdg;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    if (g != cg) {
      cg = g;
      const uint4 u0 = reinterpret_cast<const uint4*>(xsm + g * 32)[0];
      const uint4 u1 = reinterpret_cast<const uint4*>(xsm + g * 32)[1];
      X[0] = u0.x; X[1] = u0.y; X[2] = u0.z; X[3] = u0.w;
      X[4] = u1.x; X[5] = u1.y; X[6] = u1.z; X[7] = u1.w;
      xdg = xd(p, xsm)[g];
    }
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
  int cg = -1;
  uint32_t X[8];
  int sumx8;
  float xdg;
  __device__ void init(const GemvParams&, const uint8_t*) {}
  __device__ __forceinline__ void term2(const GemvParams& p, const uint8_t* xsm,
                                        const uint8_t* wA, const uint8_t* wB, const float*,
                                        const float*, int g, float& tA, float& tB) {
    if (g != cg) {
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
