// quant.cu -- FP4 packing / unpacking kernels.
//
//  * nvfp4_quantize_matrix: the converter's NVFP4 packing of one matrix with
//    one global scale (reference/glm5x_ref/nvfp4.py:180-198, both scale modes),
//    writing scales straight into the 128x4 blocked layout (nvfp4.py:23-40).
//  * nvfp4_quantize_segments: the runtime activation quantizer. Rows are
//    gathered into expert-major segments and every segment gets its own global
//    scale, as the reference quantizes each expert's token slab separately
//    (reference/glm5x_ref/layer10_moe.py:729 -> nvfp4.py:236-252, max_abs).
//  * nvfp4_dequantize / mxfp4_decode: bit-exact decoders (nvfp4.py:201-217,
//    reference/k3x_ref/mxfp4.py:110-144, runtime/src/ops.cpp:40-63).
//  * mxfp4_encode: encode_mxfp4 (mxfp4.py:31-107, both scale modes).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cstdint>

#include "fp4_codec.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {

__device__ __forceinline__ float bf16_bits_to_float(uint16_t b) {
  return __uint_as_float(static_cast<uint32_t>(b) << 16);
}

__device__ __forceinline__ void atomic_max_nonneg(float* addr, float v) {
  // valid for v >= 0: the IEEE bit pattern of non-negative floats orders like
  // unsigned integers
  atomicMax(reinterpret_cast<unsigned int*>(addr), __float_as_uint(v));
}

// ------------------------------------------------------------------ amax
// Max |x| over the whole matrix (row-major, `n` elements) into *out (which the
// caller zeroes). Records kErrNonFinite on NaN/Inf.
template <typename T>
__global__ void amax_kernel(const T* __restrict__ src, int64_t n, float* out, uint32_t* err) {
  float m = 0.0f;
  bool bad = false;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x) {
    float v;
    if constexpr (sizeof(T) == 2)
      v = bf16_bits_to_float(reinterpret_cast<const uint16_t*>(src)[i]);
    else
      v = static_cast<float>(src[i]);
    bad |= !isfinite(v);
    m = fmaxf(m, fabsf(v));
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (bad) atomicOr(err, kErrNonFinite);
  if (lane_id() == 0) atomic_max_nonneg(out, m);
}

// Per-row max |x| of a BF16 [rows, cols] matrix, one warp per row.
__global__ void row_amax_bf16_kernel(const uint16_t* __restrict__ src, int64_t rows, int cols,
                                     float* __restrict__ out, uint32_t* err) {
  const int64_t row = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
  if (row >= rows) return;
  const uint4* p = reinterpret_cast<const uint4*>(src + row * cols);
  float m = 0.0f;
  bool bad = false;
  for (int i = lane_id(); i < cols / 8; i += 32) {
    const uint4 v = __ldg(p + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float a = __uint_as_float(w[j] << 16), b = __uint_as_float(w[j] & 0xffff0000u);
      bad |= !isfinite(a) || !isfinite(b);
      m = fmaxf(m, fmaxf(fabsf(a), fabsf(b)));
    }
  }
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  if (lane_id() == 0) {
    out[row] = m;
    if (bad) atomicOr(err, kErrNonFinite);
  }
}

// ------------------------------------------------------------------ NVFP4 matrix
// One thread per 16-element block. `amax` holds max|x| over the matrix.
template <typename T>
__global__ void nvfp4_quantize_matrix_kernel(const T* __restrict__ src, int64_t rows, int64_t cols,
                                             int mse, const float* __restrict__ amax,
                                             uint8_t* __restrict__ packed,
                                             uint8_t* __restrict__ scales_blocked,
                                             float* __restrict__ global_out) {
  const int64_t nb = cols / 16;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  const float g = nvfp4_global_scale(*amax);
  if (idx == 0) *global_out = g;
  if (idx >= rows * nb) return;
  const int64_t r = idx / nb, b = idx % nb;
  float x[16];
  const T* s = src + r * cols + b * 16;
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    if constexpr (sizeof(T) == 2)
      x[i] = bf16_bits_to_float(reinterpret_cast<const uint16_t*>(s)[i]);
    else
      x[i] = static_cast<float>(s[i]);
  }
  uint8_t p[8];
  const uint32_t sb = nvfp4_quantize_block(x, g, mse != 0, p);
  uint2 pk;
  pk.x = p[0] | (p[1] << 8) | (p[2] << 16) | ((uint32_t)p[3] << 24);
  pk.y = p[4] | (p[5] << 8) | (p[6] << 16) | ((uint32_t)p[7] << 24);
  *reinterpret_cast<uint2*>(packed + r * (cols / 2) + b * 8) = pk;
  scales_blocked[blocked_sf_offset(r, b, nb)] = static_cast<uint8_t>(sb);
}

// ------------------------------------------------------------------ NVFP4 segments
// Expert-major activation quantization (max_abs). Flat row f in
// [0, qprefix[nseg]) maps to segment s (qprefix is the prefix sum of each
// segment's row count rounded up to 8) and row seg_start[s] + (f - qprefix[s])
// of the output. Rows past count[s] are zero-filled so the MMA's N padding
// reads zeros. Source rows are gathered by row_token (a token index into src).
// seg_amax[s] = max |x| over the segment's gathered rows; seg_global[s] is
// written here. One warp per row; K must be a multiple of 512.
// E2M1 codes of eight values (already divided by the block's scale), packed
// two per byte with the first value in the low nibble, by the hardware
// converter (round to nearest even, saturating at 6).
__device__ __forceinline__ uint32_t e2m1x8_rn(const float* q) {
  uint32_t r;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b0, %2, %1;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b1, %4, %3;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b2, %6, %5;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b3, %8, %7;\n\t"
      "mov.b32 %0, {b0, b1, b2, b3};\n\t}"
      : "=r"(r)
      : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]), "f"(q[7]));
  return r;
}

// Nibbles equal to 0x8 (negative zero) become 0x0 (the reference's argmin
// picks +0, code 0, for anything that rounds to zero).
__device__ __forceinline__ uint32_t clear_negative_zero(uint32_t w) {
  const uint32_t t = w ^ 0x88888888u;                              // 0 where w == 8
  const uint32_t nz = ((t & 0x77777777u) + 0x77777777u) | t;       // bit 3: t != 0
  return w & ~(~nz & 0x88888888u);
}

// max that returns NaN when either input is NaN (fmaxf drops NaNs)
__device__ __forceinline__ float fmax_nan(float a, float b) {
  float r;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(r) : "f"(a), "f"(b));
  return r;
}

__device__ __forceinline__ float rcp_approx(float d) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(d));
  return r;
}

// float -> E4M3 byte by the hardware converter (round to nearest even,
// saturating), for values already clamped to [2^-6, 448]: the same bits as
// e4m3_encode on that range.
__device__ __forceinline__ uint32_t e4m3_rn_hw(float v) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(0.0f), "f"(v));
  return r & 0xffu;
}

// E2M1 code of x / d (d > 0) when RN(x / d) is known to round to magnitude k
// or k + 1 (k <= 6): decides which side of the threshold t_k between them the
// quotient falls. RN(x / d) lands above t_k exactly when |x| / d > t_k +
// ulp(t_k) / 2 (every threshold has an even significand, so the midpoint
// itself rounds down to t_k), and (t_k + ulp(t_k) / 2) * d has at most
// 25 + 24 significant bits, so the comparison is exact in double precision.
// The code is the argmin's: ties toward the smaller magnitude, the sign from
// x, and +0 for a zero magnitude.
__device__ __forceinline__ uint32_t e2m1_code_across(float x, double d, uint32_t k) {
  // t_k = (v_k + v_(k+1)) / 2 for the E2M1 magnitudes v = 0, 0.5, 1, ..., 6
  // (their doubles 0, 1, 2, 3, 4, 6, 8, 12 one nibble each)
  const uint32_t twice = 0xC8643210u;
  const float t = (float)(((twice >> (4 * k)) & 0xfu) + ((twice >> (4 * k + 4)) & 0xfu)) * 0.25f;
  const uint32_t tb = f_bits(t);
  const double t_mid = (double)t + (double)__uint_as_float((tb & 0x7f800000u) - (24u << 23));
  const uint32_t mag = k + (fabs((double)x) > t_mid * d ? 1u : 0u);
  return mag == 0u ? 0u : (mag | (x < 0.0f ? 8u : 0u));
}

// E2M1 codes of eight BF16 values (four packed pairs w[0..3], low half
// first) times r_lo and times r_hi: two code words from the hardware
// converter (nearest, saturating at 6), the products as packed f32x2.
__device__ __forceinline__ void e2m1x8_bracket(const uint32_t* w, float r_lo, float r_hi,
                                               uint32_t& ca, uint32_t& cb) {
  asm("{\n\t.reg .b32 x0, x1;\n\t.reg .b64 ra, rb, xx, qa, qb;\n\t"
      ".reg .f32 a0, a1, b0, b1;\n\t.reg .b8 p0, p1, p2, p3, q0, q1, q2, q3;\n\t"
      "mov.b64 ra, {%6, %6};\n\tmov.b64 rb, {%7, %7};\n\t"
#define G5_BRACKET_PAIR(W, P, Q)                                              \
      "shl.b32 x0, " W ", 16;\n\tand.b32 x1, " W ", 0xffff0000;\n\t"            \
      "mov.b64 xx, {x0, x1};\n\t"                                             \
      "mul.rn.f32x2 qa, xx, ra;\n\tmul.rn.f32x2 qb, xx, rb;\n\t"               \
      "mov.b64 {a0, a1}, qa;\n\tmov.b64 {b0, b1}, qb;\n\t"                     \
      "cvt.rn.satfinite.e2m1x2.f32 " P ", a1, a0;\n\t"                          \
      "cvt.rn.satfinite.e2m1x2.f32 " Q ", b1, b0;\n\t"
      G5_BRACKET_PAIR("%2", "p0", "q0")
      G5_BRACKET_PAIR("%3", "p1", "q1")
      G5_BRACKET_PAIR("%4", "p2", "q2")
      G5_BRACKET_PAIR("%5", "p3", "q3")
#undef G5_BRACKET_PAIR
      "mov.b32 %0, {p0, p1, p2, p3};\n\tmov.b32 %1, {q0, q1, q2, q3};\n\t}"
      : "=r"(ca), "=r"(cb)
      : "r"(w[0]), "r"(w[1]), "r"(w[2]), "r"(w[3]), "f"(r_lo), "f"(r_hi));
}

// max of two BF16 pairs, NaN-propagating
__device__ __forceinline__ uint32_t bf16x2_max_nan(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("max.NaN.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Bit 4j of the result is set when nibble j of v is nonzero.
__device__ __forceinline__ uint64_t nibbles_nonzero(uint64_t v) {
  v |= v >> 2;
  v |= v >> 1;
  return v & 0x1111111111111111ull;
}

// One 16-element NVFP4 block of BF16 values (w = the block's eight packed
// pairs, xb = the same 16 values in memory) with max_abs scaling against
// global scale g (six_g = 6 * g, rcp_six_g = rcp.approx(six_g)): writes the 8
// packed bytes as two words and returns the E4M3 scale byte. Bit-identical to
// nvfp4_quantize_block(..., mse = false), i.e. to the reference's
// scale = E4M3(clamp(bmax / (6 g))), code = argmin |RN(x / (scale * g)) - c|.
//
// The scale's quotient is taken as RN(bmax * rcp.approx(6 g)), within 3 ulps
// of the IEEE quotient; when that lies within 8 bit steps of an E4M3 rounding
// midpoint (low 20 bits 0x80000) the IEEE quotient is computed instead.
// Codes: with r = rcp.approx(d) (relative error below 2^-22 together with the
// products' roundings), x * r * (1 - 2^-19) and x * r * (1 + 2^-19) bracket
// the exact quotient x / d strictly, so when the hardware converter (nearest,
// saturating at 6, its -0 mapped to +0 like the argmin) gives both the same
// code, no decision threshold lies between them and that code is the
// argmin's. Otherwise the two codes are neighbours around one threshold and
// e2m1_code_across decides exactly; BF16 data sends a fraction of a percent
// of the codes there (exact ties are common). Blocks with a non-finite value
// take IEEE division for every code.
__device__ __forceinline__ uint32_t quantize_block16_bf16(const uint32_t (&w)[8],
                                                          const uint16_t* __restrict__ xb,
                                                          float g, float six_g, float rcp_six_g,
                                                          uint32_t& lo32, uint32_t& hi32) {
  uint32_t m = w[0] & 0x7fff7fffu;
#pragma unroll
  for (int j = 1; j < 8; ++j) m = bf16x2_max_nan(m, w[j] & 0x7fff7fffu);
  const float bmax = fmax_nan(__uint_as_float(m << 16), __uint_as_float(m & 0xffff0000u));
  float base = __fmul_rn(bmax, rcp_six_g);
  if (((f_bits(base) + 8u - 0x80000u) & 0xfffffu) <= 16u || !(base <= 3.0e38f))
    base = f_div(bmax, six_g);
  base = fminf(fmaxf(base, kE4M3Tiny), kE4M3Max);
  const uint32_t sb = e4m3_rn_hw(base);
  const float denom = f_mul(e4m3_decode(sb), g);
  if (!(bmax <= 3.0e38f)) {
    // NaN / Inf in the block: every code by IEEE division and the argmin
    lo32 = hi32 = 0u;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const uint32_t xw = w[i >> 1];
      const float xi = __uint_as_float((i & 1) ? (xw & 0xffff0000u) : (xw << 16));
      const uint32_t code = e2m1_encode(f_div(xi, denom));
      if (i < 8) lo32 |= code << (4 * i); else hi32 |= code << (4 * (i - 8));
    }
    return sb;
  }
  const float ra = rcp_approx(denom);
  const float ra_lo = __fmul_rn(ra, 1.0f - 0x1p-19f);
  const float ra_hi = __fmul_rn(ra, 1.0f + 0x1p-19f);
  uint32_t ca[2], cb[2];
  e2m1x8_bracket(w, ra_lo, ra_hi, ca[0], cb[0]);
  e2m1x8_bracket(w + 4, ra_lo, ra_hi, ca[1], cb[1]);
  // -0 (code 8) only comes with magnitude 0 on both sides, so comparing the
  // raw words finds exactly the codes whose magnitudes differ
  lo32 = clear_negative_zero(ca[0]);
  hi32 = clear_negative_zero(ca[1]);
  if (((ca[0] ^ cb[0]) | (ca[1] ^ cb[1])) == 0u) return sb;
  uint64_t codes = ((uint64_t)hi32 << 32) | lo32;
  const uint64_t other = ((uint64_t)cb[1] << 32) | cb[0];
  const uint64_t raw = ((uint64_t)ca[1] << 32) | ca[0];
  uint64_t todo = nibbles_nonzero(raw ^ other);
  const double dd = (double)denom;
  while (todo) {
    const int bit = __ffsll((long long)todo) - 1;
    todo &= todo - 1;
    const float xi = __uint_as_float((uint32_t)__ldg(xb + (bit >> 2)) << 16);
    const uint32_t k = min((uint32_t)(codes >> bit) & 7u, (uint32_t)(other >> bit) & 7u);
    codes = (codes & ~(0xfull << bit)) | ((uint64_t)e2m1_code_across(xi, dd, k) << bit);
  }
  lo32 = (uint32_t)codes;
  hi32 = (uint32_t)(codes >> 32);
  return sb;
}

// 32 bytes (16 BF16 values) from global memory with an L2 cache policy
__device__ __forceinline__ void ld32_policy(const void* p, uint64_t pol, uint32_t (&w)[8]) {
  asm volatile("ld.global.nc.L2::cache_hint.v8.b32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8], %9;"
               : "=r"(w[0]), "=r"(w[1]), "=r"(w[2]), "=r"(w[3]), "=r"(w[4]), "=r"(w[5]),
                 "=r"(w[6]), "=r"(w[7])
               : "l"(p), "l"(pol));
}

// Expert-major rows gathered from token rows (GATHER) read each source row
// once per routed slot: the loads ask the L2 to keep the source rows (evict
// last) and the packed output, written once and read by the next GEMM, to go
// first. Without a gather the source is read once and goes first. WIDE: the
// source is 32-byte aligned and each lane's block is one 256-bit load.
template <bool GATHER, bool WIDE>
__global__ void nvfp4_quantize_segments_kernel(
    const uint16_t* __restrict__ src, int K, const int32_t* __restrict__ row_token,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ seg_count,
    const int32_t* __restrict__ qprefix, int nseg, int bn, const float* __restrict__ seg_amax,
    uint8_t* __restrict__ packed, uint8_t* __restrict__ scales_blocked,
    float* __restrict__ seg_global, int first_seg) {
  const int warps = blockDim.x / 32;
  const int64_t f = blockIdx.x * (int64_t)warps + threadIdx.x / 32;
  const int total = qprefix[nseg];
  if (f >= total || f < qprefix[first_seg]) return;  // segments before first_seg are filled elsewhere
  // upper_bound over qprefix[0..nseg]
  int lo = 0, hi = nseg;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (qprefix[mid] <= f) lo = mid; else hi = mid;
  }
  const int s = lo;
  const int r = static_cast<int>(f - qprefix[s]);
  const int64_t row = seg_start[s] + segment_row(r, bn);
  const float g = nvfp4_global_scale(seg_amax[s]);
  if (r == 0 && lane_id() == 0) seg_global[s] = g;
  const int nb = K / 16;  // a multiple of 32: every lane runs every iteration
  const int lane = lane_id();
  uint8_t* prow = packed + row * (K / 2) + lane * 8;
  // blocked scale layout: block b = lane + 32 i sits 4096 i bytes after b = lane
  uint8_t* psf = scales_blocked + blocked_sf_offset(row, lane, nb);
  if (r >= seg_count[s]) {
    for (int b = lane; b < nb; b += 32, prow += 256, psf += 4096) {
      *reinterpret_cast<uint2*>(prow) = make_uint2(0, 0);
      *psf = 0;
    }
    return;
  }
  const int64_t t = GATHER ? row_token[row] : row;
  const uint16_t* xrow = src + t * (int64_t)K + lane * 16;
  const float six_g = f_mul(kFp4Max, g);
  const float rcp_six_g = rcp_approx(six_g);
  uint64_t pol_src, pol_out;
  if (GATHER) {
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol_src));
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_out));
  } else {
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol_src));
  }
  for (int b = lane; b < nb; b += 32, xrow += 512, prow += 256, psf += 4096) {
    uint32_t w[8];
    if (WIDE) {
      ld32_policy(xrow, pol_src, w);
    } else {
      const uint4* q = reinterpret_cast<const uint4*>(xrow);
      const uint4 v0 = __ldg(q), v1 = __ldg(q + 1);
      w[0] = v0.x; w[1] = v0.y; w[2] = v0.z; w[3] = v0.w;
      w[4] = v1.x; w[5] = v1.y; w[6] = v1.z; w[7] = v1.w;
    }
    uint32_t lo32, hi32;
    const uint32_t sb = quantize_block16_bf16(w, xrow, g, six_g, rcp_six_g, lo32, hi32);
    if (GATHER)
      asm volatile("st.global.L2::cache_hint.v2.u32 [%0], {%1, %2}, %3;" ::"l"(prow), "r"(lo32),
                   "r"(hi32), "l"(pol_out)
                   : "memory");
    else
      *reinterpret_cast<uint2*>(prow) = make_uint2(lo32, hi32);
    *psf = static_cast<uint8_t>(sb);
  }
}

// ------------------------------------------------------------------ NVFP4 rows for dispatch
// Expert-parallel FP4 dispatch. The sender quantizes each (token, expert)
// row it sends with the expert's slab global scale, taken from the slab
// amax reduced over all ranks, so every row's codes and block scales are the
// ones the single-GPU segment quantizer gives the same row in that expert's
// slab. Rows: row r is token row_token[r] of src for expert row_expert[r];
// packed [n, K/2], scales [n, K/16] row-major E4M3. One warp per row.
__global__ void nvfp4_quantize_rows_kernel(const uint16_t* __restrict__ src, int K,
                                           const int32_t* __restrict__ row_token,
                                           const int32_t* __restrict__ row_expert, int64_t n,
                                           const float* __restrict__ amax,
                                           uint8_t* __restrict__ packed,
                                           uint8_t* __restrict__ scales) {
  const int64_t r = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
  if (r >= n) return;
  const int lane = lane_id();
  const int nb = K / 16;
  const float g = nvfp4_global_scale(amax[row_expert[r]]);
  const float six_g = f_mul(kFp4Max, g);
  const float rcp_six_g = rcp_approx(six_g);
  const uint16_t* xrow = src + (int64_t)row_token[r] * K;
  for (int b = lane; b < nb; b += 32) {
    const uint16_t* xb = xrow + b * 16;
    const uint4* q = reinterpret_cast<const uint4*>(xb);
    const uint4 v0 = __ldg(q), v1 = __ldg(q + 1);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t lo32, hi32;
    const uint32_t sb = quantize_block16_bf16(w, xb, g, six_g, rcp_six_g, lo32, hi32);
    *reinterpret_cast<uint2*>(packed + r * (K / 2) + b * 8) = make_uint2(lo32, hi32);
    scales[r * nb + b] = static_cast<uint8_t>(sb);
  }
}

// The receiver's side: rows quantized by their senders go into the routed
// segments [0, nseg_routed) of the expert-major layout (codes copied, scales
// into the blocked layout, rows past a segment's count zero-filled as the
// segment quantizer does); segment s's global scale comes from the reduced
// slab amax of global expert expert_begin + s. row_token[row] - row_base is
// the received row index.
__global__ void place_nvfp4_rows_kernel(const uint8_t* __restrict__ packed_in,
                                        const uint8_t* __restrict__ scales_in, int K,
                                        const int32_t* __restrict__ row_token, int row_base,
                                        const int32_t* __restrict__ seg_start,
                                        const int32_t* __restrict__ seg_count,
                                        const int32_t* __restrict__ qprefix, int nseg_routed,
                                        int bn, const float* __restrict__ amax, int expert_begin,
                                        uint8_t* __restrict__ packed,
                                        uint8_t* __restrict__ scales_blocked,
                                        float* __restrict__ seg_global) {
  const int64_t f = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
  if (f >= qprefix[nseg_routed]) return;
  int lo = 0, hi = nseg_routed;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (qprefix[mid] <= f) lo = mid; else hi = mid;
  }
  const int s = lo;
  const int r = static_cast<int>(f - qprefix[s]);
  const int64_t row = seg_start[s] + segment_row(r, bn);
  const int lane = lane_id();
  if (r == 0 && lane == 0) seg_global[s] = nvfp4_global_scale(amax[expert_begin + s]);
  const int nb = K / 16;
  uint4* prow = reinterpret_cast<uint4*>(packed + row * (K / 2));
  if (r >= seg_count[s]) {
    for (int v = lane; v < K / 32; v += 32) prow[v] = make_uint4(0, 0, 0, 0);
    for (int b = lane; b < nb; b += 32) scales_blocked[blocked_sf_offset(row, b, nb)] = 0;
    return;
  }
  const int64_t i = row_token[row] - row_base;
  const uint4* src = reinterpret_cast<const uint4*>(packed_in + i * (K / 2));
  for (int v = lane; v < K / 32; v += 32) prow[v] = __ldg(src + v);
  for (int b = lane; b < nb; b += 32)
    scales_blocked[blocked_sf_offset(row, b, nb)] = scales_in[i * nb + b];
}

cudaError_t launch_nvfp4_quantize_rows(const uint16_t* src, int K, const int32_t* row_token,
                                       const int32_t* row_expert, int64_t n, const float* amax,
                                       uint8_t* packed, uint8_t* scales, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  if (K % 512 || (reinterpret_cast<uintptr_t>(src) & 15)) return cudaErrorInvalidValue;
  const int warps = 8;
  nvfp4_quantize_rows_kernel<<<(unsigned)((n + warps - 1) / warps), warps * 32, 0, st>>>(
      src, K, row_token, row_expert, n, amax, packed, scales);
  return cudaGetLastError();
}

cudaError_t launch_place_nvfp4_rows(const uint8_t* packed_in, const uint8_t* scales_in, int K,
                                    const int32_t* row_token, int row_base,
                                    const int32_t* seg_start, const int32_t* seg_count,
                                    const int32_t* qprefix, int nseg_routed, int bn,
                                    const float* amax, int expert_begin, int64_t max_rows,
                                    uint8_t* packed, uint8_t* scales_blocked, float* seg_global,
                                    cudaStream_t st) {
  if (max_rows <= 0) return cudaSuccess;
  if (K % 512) return cudaErrorInvalidValue;
  const int warps = 8;
  place_nvfp4_rows_kernel<<<(unsigned)((max_rows + warps - 1) / warps), warps * 32, 0, st>>>(
      packed_in, scales_in, K, row_token, row_base, seg_start, seg_count, qprefix, nseg_routed,
      bn, amax, expert_begin, packed, scales_blocked, seg_global);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ MXFP4 terms
// Four-term MXFP4 expansion of expert-major rows for the MXFP4 expert path.
// The reference runs MXFP4 experts on decoded weights with BF16/FP32
// activations (reference/glm5x_ref/layer10_moe.py:572-593, runtime/src/
// backend_cpu.cpp:197-270); the FP4 tensor cores need FP4 on both sides, so
// every activation row x becomes four MXFP4 rows q_0..q_3 with
// q_j = MXFP4(x - q_0 - ... - q_{j-1}) (E2M1 codes, one E8M0 scale per 32,
// scale = the smallest power of two with max|residual| <= 6 * scale).
// sum_j q_j matches x to about 4e-5 relative, so the GEMM reproduces the
// reference's FP32-activation products within its tolerance.
// Segments hold 4 rows per token (row 4q + j of the segment is term j of its
// q-th token, placed with segment_row); token slot f of qprefix maps to one
// token, slots past the segment's tokens are zero-filled. Source rows are
// row_token[term-0 row], or the term-0 row itself when row_token is null.
// One warp per token; K must be a multiple of 1024.
__global__ void mxfp4_terms_segments_kernel(
    const uint16_t* __restrict__ src, int K, const int32_t* __restrict__ row_token,
    const int32_t* __restrict__ seg_start, const int32_t* __restrict__ seg_count,
    const int32_t* __restrict__ qprefix, int nseg, int bn, uint8_t* __restrict__ packed,
    uint8_t* __restrict__ scales_blocked, uint32_t* __restrict__ err) {
  // one warp per (token slot, 1024-element chunk of the row); lane = group
  const int warps = blockDim.x / 32;
  const int ng = K / 32;
  const int nchunk = (ng + 31) / 32;
  const int64_t wid = blockIdx.x * (int64_t)warps + threadIdx.x / 32;
  const int64_t f = wid / nchunk;
  const int g = static_cast<int>(wid % nchunk) * 32 + lane_id();
  if (f >= qprefix[nseg]) return;
  int lo = 0, hi = nseg;
  while (hi - lo > 1) {
    const int mid = (lo + hi) >> 1;
    if (qprefix[mid] <= f) lo = mid; else hi = mid;
  }
  const int s = lo;
  const int r = static_cast<int>(f - qprefix[s]);  // token slot in the segment
  int64_t rows[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) rows[j] = seg_start[s] + segment_row(4 * r + j, bn);
  if (g >= ng) return;
  if (4 * r >= seg_count[s]) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      *reinterpret_cast<uint4*>(packed + rows[j] * (K / 2) + g * 16) = make_uint4(0, 0, 0, 0);
      scales_blocked[blocked_sf_offset(rows[j], g, ng)] = 0;
    }
    return;
  }
  const int64_t t = row_token ? row_token[rows[0]] : rows[0];
  const uint4* qv = reinterpret_cast<const uint4*>(src + t * (int64_t)K + g * 32);
  float res[32];
  bool bad = false;
#pragma unroll
  for (int u = 0; u < 4; ++u) {
    const uint4 v = __ldg(qv + u);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      res[8 * u + 2 * i] = __uint_as_float(w[i] << 16);
      res[8 * u + 2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
      // BF16 Inf / NaN: all exponent bits set in either half
      bad |= (w[i] & 0x7f80u) == 0x7f80u || (w[i] & 0x7f800000u) == 0x7f800000u;
    }
  }
  if (bad) atomicOr(err, kErrNonFinite);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < 32; ++i) m = fmaxf(m, fabsf(res[i]));
    // smallest e with m <= 6 * 2^e: e = ceil(log2(m / 6)) from the bits
    int e = -127;
    if (m > 0.0f) {
      const uint32_t qb = __float_as_uint(m / 6.0f);
      const int ex = (int)(qb >> 23) - 127;
      e = ex + ((qb & 0x7fffffu) != 0u ? 1 : 0);
      if (ex == -127) e = -126;  // subnormal quotient
      e = e < -127 ? -127 : (e > 127 ? 127 : e);
    }
    const float scale = pow2f(e);
    const float inv = e == -127 ? 0.0f : pow2f(-e);
    // Any rounding of the codes is valid here (the residual is taken from the
    // codes actually chosen): the hardware converter encodes 8 values and
    // decodes them back to FP16 pairs for the residual update.
    uint32_t word[4];
#pragma unroll
    for (int w8 = 0; w8 < 4; ++w8) {
      float q[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) q[i] = __fmul_rn(res[8 * w8 + i], inv);
      uint32_t h[4];
      asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b0, %6, %5;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b1, %8, %7;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b2, %10, %9;\n\t"
          "cvt.rn.satfinite.e2m1x2.f32 b3, %12, %11;\n\t"
          "mov.b32 %0, {b0, b1, b2, b3};\n\t"
          "cvt.rn.f16x2.e2m1x2 %1, b0;\n\t"
          "cvt.rn.f16x2.e2m1x2 %2, b1;\n\t"
          "cvt.rn.f16x2.e2m1x2 %3, b2;\n\t"
          "cvt.rn.f16x2.e2m1x2 %4, b3;\n\t}"
          : "=r"(word[w8]), "=r"(h[0]), "=r"(h[1]), "=r"(h[2]), "=r"(h[3])
          : "f"(q[0]), "f"(q[1]), "f"(q[2]), "f"(q[3]), "f"(q[4]), "f"(q[5]), "f"(q[6]),
            "f"(q[7]));
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        // low half = the low nibble's value (element 2i), high half element 2i + 1
        const float2 v = __half22float2(*reinterpret_cast<const __half2*>(&h[i]));
        res[8 * w8 + 2 * i] = fmaf(-v.x, scale, res[8 * w8 + 2 * i]);
        res[8 * w8 + 2 * i + 1] = fmaf(-v.y, scale, res[8 * w8 + 2 * i + 1]);
      }
    }
    *reinterpret_cast<uint4*>(packed + rows[j] * (K / 2) + g * 16) =
        make_uint4(word[0], word[1], word[2], word[3]);
    scales_blocked[blocked_sf_offset(rows[j], g, ng)] = static_cast<uint8_t>(e + 127);
  }
}

// ------------------------------------------------------------------ decoders
__global__ void nvfp4_dequantize_kernel(const uint8_t* __restrict__ packed,
                                        const uint8_t* __restrict__ scales_blocked, float g,
                                        int64_t rows, int64_t cols, float* __restrict__ out) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;  // one byte (2 values)
  if (idx >= rows * cols / 2) return;
  const int64_t r = idx / (cols / 2), c = (idx % (cols / 2)) * 2;
  const uint8_t byte = packed[idx];
  const float s = f_mul(e4m3_decode(scales_blocked[blocked_sf_offset(r, c / 16, cols / 16)]), g);
  out[r * cols + c] = f_mul(e2m1_value(byte & 15u), s);
  out[r * cols + c + 1] = f_mul(e2m1_value(byte >> 4), s);
}

__global__ void mxfp4_decode_kernel(const uint8_t* __restrict__ packed,
                                    const uint8_t* __restrict__ scales, int64_t n, int group,
                                    float* __restrict__ out, uint32_t* err) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= n / 2) return;
  const uint8_t byte = packed[idx];
  const int64_t e0 = idx * 2;
  const uint8_t sc = scales[e0 / group];
  if (sc == 0xff) atomicOr(err, kErrBadScale);
  const float s = pow2f(static_cast<int>(sc) - 127);
  out[e0] = f_mul(e2m1_value(byte & 15u), s);
  out[e0 + 1] = f_mul(e2m1_value(byte >> 4), s);
}

// One thread per group of `group` (<= 64) elements.
template <typename T>
__global__ void mxfp4_encode_kernel(const T* __restrict__ src, int64_t ngroups, int group,
                                    int mse, uint8_t* __restrict__ packed,
                                    uint8_t* __restrict__ scales, uint32_t* err) {
  const int64_t gi = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (gi >= ngroups) return;
  float x[64];
  float m = 0.0f;
  for (int i = 0; i < group; ++i) {
    float v;
    if constexpr (sizeof(T) == 2)
      v = bf16_bits_to_float(reinterpret_cast<const uint16_t*>(src)[gi * group + i]);
    else
      v = static_cast<float>(src[gi * group + i]);
    if (!isfinite(v)) atomicOr(err, kErrNonFinite);
    x[i] = v;
    m = fmaxf(m, fabsf(v));
  }
  bool overflow = false;
  const int e = mxfp4_exponent(m, &overflow);
  if (overflow) atomicOr(err, kErrBadScale);
  int sel = e;
  uint32_t codes[64];
  if (!mse) {
    const float sc = pow2f(e);
    for (int i = 0; i < group; ++i) codes[i] = e2m1_encode(f_div(x[i], sc));
  } else {
    float best = 0.0f;
    for (int c = 0; c < 7; ++c) {
      int ce = e - 4 + c;
      ce = ce < -127 ? -127 : (ce > 126 ? 126 : ce);
      const float sc = pow2f(ce);
      uint32_t cc[64];
      float sum = 0.0f;
      for (int i = 0; i < group; ++i) {
        cc[i] = e2m1_encode(f_div(x[i], sc));
        const float d = f_sub(f_mul(e2m1_value(cc[i]), sc), x[i]);
        sum = f_add(sum, f_mul(d, d));
      }
      const float err_c = f_div(sum, static_cast<float>(group));
      if (c == 0 || err_c < best) {
        best = err_c;
        sel = ce;
        for (int i = 0; i < group; ++i) codes[i] = cc[i];
      }
    }
  }
  scales[gi] = static_cast<uint8_t>(sel + 127);
  for (int i = 0; i < group / 2; ++i)
    packed[gi * (group / 2) + i] = static_cast<uint8_t>(codes[2 * i] | (codes[2 * i + 1] << 4));
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_row_amax_bf16(const uint16_t* src, int64_t rows, int cols, float* out,
                                 uint32_t* err, cudaStream_t st) {
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  row_amax_bf16_kernel<<<(unsigned)((rows + warps - 1) / warps), warps * 32, 0, st>>>(
      src, rows, cols, out, err);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_nvfp4_quantize_matrix(const T* src, int64_t rows, int64_t cols, int mse,
                                         float* amax_scratch, uint8_t* packed,
                                         uint8_t* scales_blocked, float* global_out,
                                         uint32_t* err, cudaStream_t st) {
  cudaMemsetAsync(amax_scratch, 0, sizeof(float), st);
  const int64_t n = rows * cols;
  const int amax_blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, 148 * 8));
  amax_kernel<T><<<amax_blocks, 256, 0, st>>>(src, n, amax_scratch, err);
  // padded scale entries of the blocked layout stay zero, as in _to_blocked
  cudaMemsetAsync(scales_blocked, 0,
                  ((rows + 127) / 128) * ((cols / 16 + 3) / 4) * 512, st);
  const int64_t blocks = rows * (cols / 16);
  nvfp4_quantize_matrix_kernel<T><<<(unsigned)((blocks + 127) / 128), 128, 0, st>>>(
      src, rows, cols, mse, amax_scratch, packed, scales_blocked, global_out);
  return cudaGetLastError();
}
template cudaError_t launch_nvfp4_quantize_matrix<float>(const float*, int64_t, int64_t, int,
                                                         float*, uint8_t*, uint8_t*, float*,
                                                         uint32_t*, cudaStream_t);
template cudaError_t launch_nvfp4_quantize_matrix<__nv_bfloat16>(const __nv_bfloat16*, int64_t,
                                                                 int64_t, int, float*, uint8_t*,
                                                                 uint8_t*, float*, uint32_t*,
                                                                 cudaStream_t);

cudaError_t launch_nvfp4_quantize_segments(const uint16_t* src, int K, const int32_t* row_token,
                                           const int32_t* seg_start, const int32_t* seg_count,
                                           const int32_t* qprefix, int nseg, int bn,
                                           const float* seg_amax, int64_t max_rows,
                                           uint8_t* packed, uint8_t* scales_blocked,
                                           float* seg_global, cudaStream_t st, int first_seg) {
  if (max_rows <= 0) return cudaSuccess;
  if (K % 512) return cudaErrorInvalidValue;
  const int warps = 8;
  const bool wide = (reinterpret_cast<uintptr_t>(src) & 31) == 0;
  const dim3 grid((unsigned)((max_rows + warps - 1) / warps)), block(warps * 32);
  auto kernel = row_token ? (wide ? nvfp4_quantize_segments_kernel<true, true>
                                  : nvfp4_quantize_segments_kernel<true, false>)
                          : (wide ? nvfp4_quantize_segments_kernel<false, true>
                                  : nvfp4_quantize_segments_kernel<false, false>);
  kernel<<<grid, block, 0, st>>>(src, K, row_token, seg_start, seg_count, qprefix, nseg, bn,
                                 seg_amax, packed, scales_blocked, seg_global, first_seg);
  return cudaGetLastError();
}

cudaError_t launch_mxfp4_terms_segments(const uint16_t* src, int K, const int32_t* row_token,
                                        const int32_t* seg_start, const int32_t* seg_count,
                                        const int32_t* qprefix, int nseg, int bn,
                                        int64_t max_slots, uint8_t* packed,
                                        uint8_t* scales_blocked, uint32_t* err, cudaStream_t st) {
  if (max_slots <= 0) return cudaSuccess;
  if (K % 32) return cudaErrorInvalidValue;
  const int warps = 8;
  const int64_t nwarps = max_slots * ((K / 32 + 31) / 32);
  mxfp4_terms_segments_kernel<<<(unsigned)((nwarps + warps - 1) / warps), warps * 32, 0, st>>>(
      src, K, row_token, seg_start, seg_count, qprefix, nseg, bn, packed, scales_blocked, err);
  return cudaGetLastError();
}

cudaError_t launch_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales_blocked,
                                    float g, int64_t rows, int64_t cols, float* out,
                                    cudaStream_t st) {
  const int64_t n = rows * cols / 2;
  if (n == 0) return cudaSuccess;
  nvfp4_dequantize_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(packed, scales_blocked,
                                                                       g, rows, cols, out);
  return cudaGetLastError();
}

cudaError_t launch_mxfp4_decode(const uint8_t* packed, const uint8_t* scales, int64_t n,
                                int group, float* out, uint32_t* err, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  mxfp4_decode_kernel<<<(unsigned)((n / 2 + 255) / 256), 256, 0, st>>>(packed, scales, n, group,
                                                                       out, err);
  return cudaGetLastError();
}

template <typename T>
cudaError_t launch_mxfp4_encode(const T* src, int64_t n, int group, int mse, uint8_t* packed,
                                uint8_t* scales, uint32_t* err, cudaStream_t st) {
  const int64_t ng = n / group;
  if (ng == 0) return cudaSuccess;
  mxfp4_encode_kernel<T><<<(unsigned)((ng + 127) / 128), 128, 0, st>>>(src, ng, group, mse,
                                                                       packed, scales, err);
  return cudaGetLastError();
}
template cudaError_t launch_mxfp4_encode<float>(const float*, int64_t, int, int, uint8_t*,
                                                uint8_t*, uint32_t*, cudaStream_t);
template cudaError_t launch_mxfp4_encode<__nv_bfloat16>(const __nv_bfloat16*, int64_t, int, int,
                                                        uint8_t*, uint8_t*, uint32_t*,
                                                        cudaStream_t);

}  // namespace glm5x
