// fp4_codec.h -- E2M1 / E4M3 / E8M0 codecs shared by device kernels and the
// host-side packers. Every rounding step is spelled out with explicit
// round-to-nearest FP32 operations so device and host produce the same bits
// as the reference's torch encoders:
//   NVFP4: reference/glm5x_ref/nvfp4.py:101-177 (_quantize_payload)
//   MXFP4: reference/k3x_ref/mxfp4.py:31-107   (encode_mxfp4)
#pragma once
#include <cstdint>
#include <cstring>
#include <cmath>

#if defined(__CUDACC__)
#define G5_HD __host__ __device__ __forceinline__
#else
#define G5_HD inline
#endif

namespace glm5x {

constexpr float kE4M3Tiny = 0.015625f;  // 2^-6, torch.finfo(float8_e4m3fn).tiny
constexpr float kE4M3Max = 448.0f;
constexpr float kFp4Max = 6.0f;

G5_HD float f_mul(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fmul_rn(a, b);
#else
  volatile float r = a * b;
  return r;
#endif
}
G5_HD float f_div(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fdiv_rn(a, b);
#else
  volatile float r = a / b;
  return r;
#endif
}
G5_HD float f_add(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fadd_rn(a, b);
#else
  volatile float r = a + b;
  return r;
#endif
}
G5_HD float f_sub(float a, float b) {
#if defined(__CUDA_ARCH__)
  return __fsub_rn(a, b);
#else
  volatile float r = a - b;
  return r;
#endif
}

G5_HD uint32_t f_bits(float x) {
#if defined(__CUDA_ARCH__)
  return __float_as_uint(x);
#else
  uint32_t b;
  std::memcpy(&b, &x, 4);
  return b;
#endif
}
G5_HD float bits_f(uint32_t b) {
#if defined(__CUDA_ARCH__)
  return __uint_as_float(b);
#else
  float x;
  std::memcpy(&x, &b, 4);
  return x;
#endif
}

// E2M1 value of a code in the reference's code order (codes 8..15 negate):
// magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6 = half of the 4-bit table
// 0, 1, 2, 3, 4, 6, 8, 12 held in one register (no indexed local array).
G5_HD float e2m1_value(uint32_t code) {
  const uint32_t twice = (0xC8643210u >> (4u * (code & 7u))) & 0xFu;
  const float m = static_cast<float>(twice) * 0.5f;
  return (code & 8u) ? -m : m;
}

// The reference picks argmin_i |v - codebook[i]| with the first index
// winning ties. For |v| < 16 (every normalized value the encoders produce)
// every candidate difference near a midpoint is exact in FP32, so the argmin
// is: magnitude rounded to the nearest E2M1 value with ties toward the smaller
// magnitude, and code 0 (+0) for anything rounding to 0. The seven decision
// thresholds (0.25 0.75 1.25 1.75 2.5 3.5 5) have zero low 21 mantissa bits,
// so the magnitude code is a table lookup on bits(|v| - 1 ulp) >> 21. Checked
// against the reference's argmin for all 2.2e9 floats with |v| <= 16.
G5_HD uint32_t e2m1_encode(float v) {
  const uint32_t b = f_bits(v) & 0x7fffffffu;
  if (b == 0) return 0;
  int k = static_cast<int>((b - 1u) >> 21) - 500;  // 500 = bits(0.25) >> 21
  if (k < 0) return 0;
  if (k > 17) k = 17;
  // magnitude code for k = 0..17: 1 x6, 2 x3, 3 x2, 4 x2, 5 x2, 6 x2, 7
  constexpr uint64_t kLut = 0x3ed6c8da489249ull;
  const uint32_t m = static_cast<uint32_t>((kLut >> (3 * k)) & 7u);
  return (f_bits(v) >> 31) ? (m | 8u) : m;
}

// x / d for the encoders: RN(x * RN(1/d)) is within 2 ulps of the IEEE
// quotient; the E2M1 code can differ only when the quotient sits within 2
// ulps of a value with a 2-bit mantissa (all thresholds are such values), in
// which case the IEEE quotient is computed. rcp = RN(1/d).
G5_HD float ratio_for_code(float x, float d, float rcp) {
  float q = f_mul(x, rcp);
  const uint32_t qb = f_bits(q) & 0x7fffffffu;
  if (qb != 0 && ((qb + 2u) & 0x1fffffu) <= 4u) q = f_div(x, d);
  return q;
}

G5_HD float f_rcp(float d) {
#if defined(__CUDA_ARCH__)
  return __frcp_rn(d);
#else
  volatile float r = 1.0f / d;
  return r;
#endif
}

// float -> float8_e4m3fn, round to nearest even, saturating at 448.
G5_HD uint32_t e4m3_encode(float x) {
  uint32_t b = f_bits(x);
  const uint32_t sign = (b >> 24) & 0x80u;
  b &= 0x7fffffffu;
  if (b == 0) return sign;
  if (b >= 0x7f800000u) return sign | 0x7eu;
  const int exp = static_cast<int>(b >> 23) - 127;
  if (exp < -6) {
    // subnormal: m * 2^-9 with m = rne(|x| * 512), m == 8 is the min normal
    const float q = f_mul(bits_f(b), 512.0f);
#if defined(__CUDA_ARCH__)
    const float m = rintf(q);
#else
    const float m = nearbyintf(q);
#endif
    return sign | static_cast<uint32_t>(m);
  }
  const uint32_t rounded = (b + 0x7ffffu + ((b >> 20) & 1u)) & ~0xfffffu;
  const int e = static_cast<int>(rounded >> 23) - 127;
  const uint32_t mant = (rounded >> 20) & 7u;
  if (e > 8 || (e == 8 && mant == 7u)) return sign | 0x7eu;
  return sign | (static_cast<uint32_t>(e + 7) << 3) | mant;
}

G5_HD float e4m3_decode(uint32_t c) {
  const uint32_t e = (c >> 3) & 15u;
  const uint32_t m = c & 7u;
  float v;
  if (e == 0)
    v = static_cast<float>(m) * 0.001953125f;  // m * 2^-9, exact
  else
    v = bits_f(((e + 120u) << 23) | (m << 20));  // (1 + m/8) * 2^(e-7)
  if (e == 15u && m == 7u) v = bits_f(0x7fc00000u);
  return (c & 0x80u) ? -v : v;
}

// 2^e as FP32 for e in [-127, 127] (2^-127 is an FP32 subnormal).
G5_HD float pow2f(int e) {
  if (e >= -126) return bits_f(static_cast<uint32_t>(e + 127) << 23);
  return bits_f(0x00400000u);  // 2^-127
}

// NVFP4 global scale: max(amax / (448 * 6), 1e-12) (nvfp4.py:127-130).
G5_HD float nvfp4_global_scale(float amax) {
  float g = f_div(amax, 2688.0f);
  if (!(g >= 1e-12f)) g = 1e-12f;
  return g;
}

// max_abs block scale byte for one 16-element block (nvfp4.py:131-134,
// 164-166): E4M3(clamp(bmax / (6 * g), 2^-6, 448)).
G5_HD uint32_t nvfp4_block_scale_maxabs(float bmax, float g) {
  float base = f_div(bmax, f_mul(kFp4Max, g));
  if (base < kE4M3Tiny) base = kE4M3Tiny;
  if (base > kE4M3Max) base = kE4M3Max;
  return e4m3_encode(base);
}

// Quantizes one 16-element block against global scale g. mse selects the
// reference's 9-candidate search (nvfp4.py:139-163), else max_abs. Writes 8
// packed bytes (low nibble first, nvfp4.py:173) and returns the scale byte.
G5_HD uint32_t nvfp4_quantize_block(const float* x, float g, bool mse, uint8_t* packed) {
  float bmax = 0.0f;
  for (int i = 0; i < 16; ++i) {
    const float a = fabsf(x[i]);
    bmax = a > bmax ? a : bmax;
  }
  float base = f_div(bmax, f_mul(kFp4Max, g));
  if (base < kE4M3Tiny) base = kE4M3Tiny;
  if (base > kE4M3Max) base = kE4M3Max;
  uint32_t codes[16];
  uint32_t sel;
  if (!mse) {
    sel = e4m3_encode(base);
    const float denom = f_mul(e4m3_decode(sel), g);
    const float rcp = f_rcp(denom);
    for (int i = 0; i < 16; ++i) codes[i] = e2m1_encode(ratio_for_code(x[i], denom, rcp));
  } else {
    const float factors[9] = {0.5f, 0.625f, 0.75f, 0.875f, 1.0f, 1.125f, 1.25f, 1.5f, 2.0f};
    float best_err = 0.0f;
    sel = 0;
    for (int c = 0; c < 9; ++c) {
      float cand = f_mul(base, factors[c]);
      if (cand < kE4M3Tiny) cand = kE4M3Tiny;
      if (cand > kE4M3Max) cand = kE4M3Max;
      const uint32_t cb = e4m3_encode(cand);
      const float denom = f_mul(e4m3_decode(cb), g);
      const float rcp = f_rcp(denom);
      uint32_t cc[16];
      float lane[8];
      for (int i = 0; i < 16; ++i) {
        cc[i] = e2m1_encode(ratio_for_code(x[i], denom, rcp));
        const float d = f_sub(f_mul(e2m1_value(cc[i]), denom), x[i]);
        const float sq = f_mul(d, d);
        if (i < 8)
          lane[i] = sq;
        else
          lane[i - 8] = f_add(lane[i - 8], sq);
      }
      // torch's CPU mean over a contiguous 16-wide row: 8 lanes folded in order
      float s = lane[0];
      for (int j = 1; j < 8; ++j) s = f_add(s, lane[j]);
      const float err = f_mul(s, 0.0625f);
      if (c == 0 || err < best_err) {
        best_err = err;
        sel = cb;
        for (int i = 0; i < 16; ++i) codes[i] = cc[i];
      }
    }
  }
  for (int i = 0; i < 8; ++i)
    packed[i] = static_cast<uint8_t>(codes[2 * i] | (codes[2 * i + 1] << 4));
  return sel;
}

// MXFP4 shared exponent: ceil(log2(max / 6)) rounded the way torch's FP32
// log2 rounds (the FP32 rounding of an accurate log2, then ceil; this differs
// from the exact ceil only for maxima within a few ulps above 6 * 2^k).
// Returns -127 for an all-zero group; *overflow set when e > 126
// (mxfp4.py:57-66).
G5_HD int mxfp4_exponent(float gmax, bool* overflow) {
  if (!(gmax > 0.0f)) return -127;
  const float q = f_div(gmax, 6.0f);
  const float l = static_cast<float>(log2(static_cast<double>(q)));
  const float c = ceilf(l);
  if (c > 126.0f) {
    *overflow = true;
    return 126;
  }
  int e = static_cast<int>(c);
  return e < -127 ? -127 : e;
}

// Byte offset of scale (row r, scale column c) inside the 128x4 blocked
// layout of a [rows, cols] scale matrix (nvfp4.py:23-40, _to_blocked): the
// tcgen05 block-scaled MMA's scale-factor tile.
G5_HD uint64_t blocked_sf_offset(uint64_t r, uint64_t c, uint64_t sf_cols) {
  const uint64_t cb = (sf_cols + 3) / 4;
  const uint64_t chunk = (r / 128) * cb + c / 4;
  const uint64_t rr = r % 128;
  return chunk * 512 + (rr % 32) * 16 + (rr / 32) * 4 + (c % 4);
}

}  // namespace glm5x
