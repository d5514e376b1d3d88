// router_tc.cu -- fused router: BF16 logits on tcgen05 tensor cores with the
// sigmoid / correction-bias / top-k / renormalization epilogue in TMEM order.
//
// Replaces the router of the reference (reference/glm5x_ref/layer10_moe.py:
// 760-789: FP32 logits, sigmoid, + correction bias, top-k, renormalize,
// x routed_scaling_factor; C++ runtime/src/cuda_glm5x_real_expert_bench.cpp:
// 287-328 + runtime/src/routing_policy.cpp:31-159 natural mode). Selection
// follows std::stable_sort's order: descending choice score, ties to the
// lower expert id; the denominator sums the selected scores in slot order.
//
// One CTA per 128-token tile: the 128 x 256 FP32 logit tile lives in TMEM
// (kind::f16, BF16 inputs, K = 16 per MMA); each epilogue thread owns one
// token (one TMEM lane) and reads its 256 logits 32 columns at a time.
// Split mode (gridDim.y > 1, small batches): CTA (tile, y) contracts K-steps
// [y * ks_per, (y + 1) * ks_per) and writes its partial logits to plane y of
// `partials`; topk_kernel sums the planes in order and selects.
#include <cuda.h>
#include <algorithm>
#include <cstdint>

#include "fp4_codec.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {
namespace {

constexpr int kTok = 128;        // tokens per tile (MMA M)
constexpr int kMaxExp = 256;     // experts (MMA N = E, a multiple of 16)
constexpr int kKStage = 64;      // BF16 elements per stage (128 bytes per row)
constexpr int kStages = 4;
constexpr int kABytes = kTok * 128;
constexpr int kBBytes = kMaxExp * 128;
constexpr int kStageBytes = kABytes + kBBytes;
constexpr size_t kSmem = (size_t)kStages * kStageBytes + 1024 + 256;

// KL = length of the running top list (>= k).
template <int KL>
__global__ void __launch_bounds__(192, 1)
    router_tc_kernel(const __grid_constant__ CUtensorMap tmap_x,
                     const __grid_constant__ CUtensorMap tmap_w, const float* __restrict__ bias,
                     int T, int H, int E, int k, uint32_t tmem_cols, float routed_scale,
                     float* __restrict__ logits, int32_t* __restrict__ ids,
                     float* __restrict__ weights, uint32_t* err, int ks_per,
                     float* __restrict__ partials, float* __restrict__ row_amax) {
  constexpr int kMaxK = KL;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kStages * kStageBytes);
  uint64_t* empty = full + kStages;
  uint64_t* done = empty + kStages;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(done + 1);
  __shared__ float s_bias[kMaxExp];

  const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
  const int t0 = blockIdx.x * kTok;
  const bool split = gridDim.y > 1;
  const int ks_begin = split ? (int)blockIdx.y * ks_per : 0;
  const int ks_end = split ? min(H / kKStage, ks_begin + ks_per) : H / kKStage;
  for (int i = threadIdx.x; i < kMaxExp; i += blockDim.x) s_bias[i] = i < E ? bias[i] : 0.0f;
  const uint32_t b_bytes = (uint32_t)E * 128;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      // the MMA commit, and with row_amax the four epilogue warps' reads
      mbar_init(&empty[s], row_amax ? 5 : 1);
    }
    mbar_init(done, 1);
    fence_barrier_init();
    fence_proxy_async_smem();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, tmem_cols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      tma_prefetch_desc(&tmap_x);
      tma_prefetch_desc(&tmap_w);
      uint32_t phase = 0;
      for (int ks = ks_begin, stage = 0; ks < ks_end; ++ks) {
        if (!mbar_wait(&empty[stage], phase ^ 1u, err)) break;
        uint8_t* sa = smem + stage * kStageBytes;
        mbar_arrive_expect_tx(&full[stage], kABytes + b_bytes);
        tma_load_2d(sa, &tmap_x, &full[stage], ks * kKStage, t0);
        tma_load_2d(sa + kABytes, &tmap_w, &full[stage], ks * kKStage, 0);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
    }
    __syncwarp();
  } else if (warp == 1) {
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(kTok, (uint32_t)E);
      uint32_t phase = 0;
      bool ok = true;
      for (int ks = ks_begin, stage = 0; ks < ks_end; ++ks) {
        if (!mbar_wait(&full[stage], phase, err)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t a = smem_u32(smem + stage * kStageBytes);
        const uint32_t b = a + kABytes;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          mma_bf16(tmem, desc_kmajor_sw128(a + 32 * c), desc_kmajor_sw128(b + 32 * c), idesc,
                   (ks != ks_begin || c != 0) ? 1u : 0u);
        tc_commit(&empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      tc_commit(done);
      if (!ok) mbar_wait(done, 0, err);
    }
    __syncwarp();
  } else {
    const int q = warp & 3;
    const int t = t0 + 32 * q + lane;
    if (row_amax) {
      // Per-token max |x| (the NVFP4 slab scales' input) from the token
      // tiles the MMAs read: lane = token row 32q + lane of the tile, its
      // 128-byte row read as eight 16-byte pieces in a lane-rotated order (the
      // 128-byte swizzle only permutes pieces within a row, and the rotation
      // spreads a warp's reads over all banks). NaN is skipped by the max and
      // flagged, as the stand-alone row amax kernel does; rows past T are
      // TMA zero fill.
      const int r = 32 * q + lane;
      uint32_t mx = 0u, mn = 0u;
      uint32_t phase = 0;
      bool ok = true;
      for (int ks = ks_begin, stage = 0; ks < ks_end; ++ks) {
        if (!mbar_wait(&full[stage], phase, err)) {
          ok = false;
          break;
        }
        const uint32_t row = smem_u32(smem + stage * kStageBytes) + r * 128;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          uint32_t w0, w1, w2, w3;
          asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];"
                       : "=r"(w0), "=r"(w1), "=r"(w2), "=r"(w3)
                       : "r"(row + 16 * ((i + r) & 7)));
          const uint32_t wd[4] = {w0, w1, w2, w3};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const uint32_t a = wd[j] & 0x7fff7fffu;
            asm("max.bf16x2 %0, %0, %1;" : "+r"(mx) : "r"(a));
            asm("max.NaN.bf16x2 %0, %0, %1;" : "+r"(mn) : "r"(a));
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[stage]);
        if (++stage == kStages) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (ok && t < T) {
        const float m = fmaxf(__uint_as_float(mx << 16), __uint_as_float(mx & 0xffff0000u));
        // an Inf or NaN half of the NaN-propagating max: a non-finite input
        if ((mn & 0x7f80u) == 0x7f80u || (mn & 0x7f800000u) == 0x7f800000u)
          atomicOr(err, kErrNonFinite);
        if (split)
          atomicMax(reinterpret_cast<unsigned int*>(row_amax + t), __float_as_uint(m));
        else
          row_amax[t] = m;
      }
    }
    if (split) {
      if (mbar_wait(done, 0, err)) {
        tc_fence_after();
        float* dst = partials + (int64_t)blockIdx.y * T * E + (int64_t)t * E;
        for (int c0 = 0; c0 < E; c0 += 32) {
          uint32_t v[32];
          tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
          tmem_ld_wait(v);
          if (t < T) {
#pragma unroll
            for (int i = 0; i < 32; i += 4)
              if (c0 + i < E)
                *reinterpret_cast<float4*>(dst + c0 + i) =
                    make_float4(__uint_as_float(v[i]), __uint_as_float(v[i + 1]),
                                __uint_as_float(v[i + 2]), __uint_as_float(v[i + 3]));
          }
        }
      }
    } else if (mbar_wait(done, 0, err)) {
      tc_fence_after();
      float top_v[kMaxK], top_s[kMaxK];
      int top_i[kMaxK];
#pragma unroll
      for (int j = 0; j < kMaxK; ++j) {
        top_v[j] = -INFINITY;
        top_s[j] = 0.0f;
        top_i[j] = 0x7fffffff;
      }
      bool bad = false;
      for (int c0 = 0; c0 < E; c0 += 32) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(tmem + ((uint32_t)(32 * q) << 16) + c0, v);
        tmem_ld_wait(v);
        if (t < T) {
          if (logits) {
            float* dst = logits + (int64_t)t * E + c0;
#pragma unroll
            for (int i = 0; i < 32; ++i)
              if (c0 + i < E) dst[i] = __uint_as_float(v[i]);
          }
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const float l = __uint_as_float(v[i]);
            const float s = f_div(1.0f, f_add(1.0f, expf(-l)));
            const float ch = f_add(s, s_bias[c0 + i]);
            bad |= !isfinite(ch) && c0 + i < E;
            if (c0 + i < E && ch > top_v[kMaxK - 1]) {
              top_v[kMaxK - 1] = ch;
              top_s[kMaxK - 1] = s;
              top_i[kMaxK - 1] = c0 + i;
#pragma unroll
              for (int j = kMaxK - 1; j > 0; --j) {
                if (top_v[j] > top_v[j - 1]) {
                  const float tv = top_v[j], ts = top_s[j];
                  const int ti = top_i[j];
                  top_v[j] = top_v[j - 1];
                  top_s[j] = top_s[j - 1];
                  top_i[j] = top_i[j - 1];
                  top_v[j - 1] = tv;
                  top_s[j - 1] = ts;
                  top_i[j - 1] = ti;
                }
              }
            }
          }
        }
      }
      if (t < T) {
        if (bad) atomicOr(err, kErrNonFinite);
        float denom = 0.0f;
#pragma unroll
        for (int j = 0; j < kMaxK; ++j)
          if (j < k) denom = f_add(denom, top_s[j]);
#pragma unroll
        for (int j = 0; j < kMaxK; ++j)
          if (j < k) {
            ids[(int64_t)t * k + j] = top_i[j];
            weights[(int64_t)t * k + j] = f_mul(f_div(top_s[j], denom), routed_scale);
          }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

template <int KL>
cudaError_t launch_kl(const CUtensorMap* tx, const CUtensorMap* tw, const float* bias, int T,
                      int H, int E, int k, float scale, float* logits, int32_t* ids,
                      float* weights, uint32_t* err, cudaStream_t st, int nsplit, int ks_per,
                      float* partials, float* row_amax) {
  uint32_t cols = 32;
  while (cols < (uint32_t)E) cols <<= 1;
  cudaError_t e = cudaFuncSetAttribute(router_tc_kernel<KL>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem);
  if (e != cudaSuccess) return e;
  router_tc_kernel<KL><<<dim3((T + kTok - 1) / kTok, nsplit), 192, kSmem, st>>>(
      *tx, *tw, bias, T, H, E, k, cols, scale, logits, ids, weights, err, ks_per, partials,
      row_amax);
  return cudaGetLastError();
}

}  // namespace

bool router_tc_supported(int E, int H, int k) {
  return E >= 16 && E <= kMaxExp && E % 16 == 0 && H % kKStage == 0 && k > 0 && k <= 16 &&
         k <= E;
}

// logits[i] = sum of the nsplit partial planes at i, added in plane order.
__global__ void sum_partials_kernel(const float* __restrict__ partials, int nsplit, int64_t n,
                                    float* __restrict__ logits) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  float v = partials[i];
#pragma unroll 8
  for (int p = 1; p < nsplit; ++p) v = f_add(v, partials[(int64_t)p * n + i]);
  logits[i] = v;
}

// K-split plane counts up to this are summed inside the selection kernel
constexpr int kFusedPlanes = 4;

size_t router_partials_floats(int num_sms, int E) {
  // nsplit * T <= (num_sms / tiles) * tiles * 128
  return (size_t)(num_sms + 1) * kTok * E;
}

cudaError_t launch_router_tc(const CUtensorMap* tmap_x, const CUtensorMap* tmap_w,
                             const float* bias, int T, int H, int E, int k, float routed_scale,
                             float* logits, int32_t* ids, float* weights, uint32_t* err,
                             cudaStream_t st, float* partials, int num_sms, int* launches,
                             const RoutingPolicy& policy, int32_t* sel, float* diag,
                             float* row_amax) {
  if (!router_tc_supported(E, H, k)) return cudaErrorInvalidValue;
  if (launches) *launches = 0;
  if (T == 0) return cudaSuccess;
  const int tiles = (T + kTok - 1) / kTok;
  const int ksteps = H / kKStage;
  // K-split count: fill the SMs, at least 4 K-steps per CTA
  int nsplit = partials && num_sms > 0 ? num_sms / tiles : 1;
  nsplit = std::max(1, std::min(nsplit, ksteps / 4));
  const int ks_per = (ksteps + nsplit - 1) / nsplit;
  nsplit = (ksteps + ks_per - 1) / ks_per;
  cudaError_t e = cudaSuccess;
  if (row_amax && nsplit > 1) {
    // the K planes' partial maxima meet in atomicMax (non-negative floats
    // order as their bit patterns)
    e = cudaMemsetAsync(row_amax, 0, sizeof(float) * (size_t)T, st);
    if (e != cudaSuccess) return e;
  }
  e = k <= 8 ? launch_kl<8>(tmap_x, tmap_w, bias, T, H, E, k, routed_scale, logits, ids, weights,
                            err, st, nsplit, ks_per, partials, row_amax)
             : launch_kl<16>(tmap_x, tmap_w, bias, T, H, E, k, routed_scale, logits, ids,
                             weights, err, st, nsplit, ks_per, partials, row_amax);
  if (e != cudaSuccess) return e;
  const bool policy_pass = policy.mode != 0 || sel || diag;
  if (launches) *launches = 1;
  if (nsplit == 1) {
    if (!policy_pass) return cudaSuccess;
    if (!logits) return cudaErrorInvalidValue;
    if (launches) *launches = 2;
    return launch_topk(logits, 0, bias, T, E, k, routed_scale, ids, weights, err, st, policy,
                       sel, diag);
  }
  if (!logits) return cudaErrorInvalidValue;
  if (nsplit <= kFusedPlanes) {
    // few planes (large batches): the selection kernel sums them in plane
    // order as it reads them (and stores the logits), one launch and one
    // pass over the planes
    if (launches) *launches = 2;
    return launch_topk_planes(partials, nsplit, logits, 0, bias, T, E, k, routed_scale, ids,
                              weights, err, st, policy, sel, diag);
  }
  // many planes (small batches): one warp per token would add them up in a
  // long chain of dependent loads, so a thread per logit sums them first
  if (launches) *launches = 3;
  const int64_t n = (int64_t)T * E;
  sum_partials_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(partials, nsplit, n, logits);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  return launch_topk(logits, 0, bias, T, E, k, routed_scale, ids, weights, err, st, policy, sel,
                     diag);
}

}  // namespace glm5x
