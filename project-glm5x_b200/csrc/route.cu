// route.cu -- router top-k and the expert-major token permutation.
//
// Routing follows the reference's C++ policy (natural, fixed and adaptive
// Top-K of runtime/src/routing_policy.cpp:31-159, natural mode called from
// runtime/src/cuda_glm5x_real_expert_bench.cpp:287-328) and the Python router
// (reference/glm5x_ref/layer10_moe.py:760-789): score = sigmoid(logit),
// choice = score + bias, top-k by choice with ties to the lower expert index
// (std::stable_sort order), weight = score / sum(selected scores, summed in
// slot order) * routed_scaling.
//
// The permutation replaces build_expert_major_plan / packed plan
// (runtime/src/expert_major.cpp:12-98) with a device counting sort: segments
// in ascending expert order, each segment's tokens in ascending token order,
// every segment starting on a 128-row boundary (one 128-row block of the
// block-scaled operand never spans two experts). The shared expert is segment
// `num_experts` holding every token in order.
#include <cstdint>

#include "fp4_codec.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {

// ------------------------------------------------------------------ top-k
// One warp per token. Lane l owns experts l, l+32, ... (E <= 32 * 16).
// `values_are_scores` = 1 means `in` already holds sigmoid scores (the
// select_routing parity entry point), else logits.
// select_routing's K ladder (routing_policy.cpp:13)
__device__ __forceinline__ bool k_in_ladder(int k) {
  return k == 4 || k == 6 || k == 8 || k == 12 || k == 16;
}

// boundary_confidence (routing_policy.cpp:21-29): the probability gap at the
// selected K relative to the largest natural probability, 1 at K = k.
__device__ float boundary_confidence(const float* p, int k, int selected) {
  if (selected >= k) return 1.0f;
  const float gap = fmaxf(0.0f, f_sub(p[selected - 1], p[selected]));
  return f_div(gap, fmaxf(p[0], 1.17549435e-38f));
}

// choose_adaptive (routing_policy.cpp:115-133): the first ladder K >= floor
// whose cumulative natural probability reaches mass_target, that covers the
// entropy's effective support and whose boundary gap reaches
// minimum_boundary_gap, each test with the 1e-5 slack; k when none does.
__device__ int choose_adaptive(const float* p, int k, int floor_k, float support,
                               const RoutingPolicy& pol) {
  constexpr float kEps = 1.0e-5f;
  float cumulative = 0.0f;
  for (int slot = 0; slot < k; ++slot) {
    cumulative = f_add(cumulative, p[slot]);
    const int candidate = slot + 1;
    if (!k_in_ladder(candidate) || candidate < floor_k) continue;
    const float confidence = boundary_confidence(p, k, candidate);
    if (f_add(cumulative, kEps) >= pol.mass_target &&
        f_add(static_cast<float>(candidate), kEps) >= support &&
        f_add(confidence, kEps) >= pol.minimum_boundary_gap)
      return candidate;
  }
  return k;
}

// in: nplanes planes of [T, E] (plane p at in + p * T * E) whose sum, taken
// in plane order, is the value (the K-split router's partial logits; one
// plane otherwise); logits_out, when given, receives that sum.
template <int kMaxPer>
__global__ void topk_kernel(const float* __restrict__ in, int nplanes,
                            float* __restrict__ logits_out, int values_are_scores,
                            const float* __restrict__ bias, int T, int E, int k,
                            float routed_scale, int32_t* __restrict__ ids,
                            float* __restrict__ weights, uint32_t* err, RoutingPolicy pol,
                            int32_t* __restrict__ sel_out, float* __restrict__ diag) {
  const int warps = blockDim.x / 32;
  const int t = blockIdx.x * warps + threadIdx.x / 32;
  if (t >= T) return;
  const int lane = lane_id();
  float score[kMaxPer], choice[kMaxPer];
  const int per = (E + 31) / 32;
  const int64_t plane = (int64_t)T * E;
  bool bad = false;
#pragma unroll
  for (int j = 0; j < kMaxPer; ++j) {
    const int e = lane + 32 * j;
    if (j < per && e < E) {
      const int64_t i = (int64_t)t * E + e;
      float v = in[i];
#pragma unroll 4
      for (int q = 1; q < nplanes; ++q) v = f_add(v, in[q * plane + i]);
      if (logits_out) logits_out[i] = v;
      float s;
      if (values_are_scores) {
        s = v;
        bad |= !(s >= 0.0f && s <= 1.0f);
      } else {
        s = f_div(1.0f, f_add(1.0f, expf(-v)));
      }
      score[j] = s;
      choice[j] = f_add(s, bias[e]);
      bad |= !isfinite(choice[j]);
    } else {
      score[j] = 0.0f;
      choice[j] = -INFINITY;
    }
  }
  if (bad) atomicOr(err, kErrNonFinite);
  uint32_t taken = 0;
  float denom = 0.0f;
  float sel_score[16];
  int sel_id[16];
  for (int s = 0; s < k; ++s) {
    // local best: max choice, lowest expert id on ties
    float best = -INFINITY;
    int best_e = 0x7fffffff;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j) {
      const int e = lane + 32 * j;
      if (j < per && e < E && !((taken >> j) & 1u)) {
        if (choice[j] > best || (choice[j] == best && e < best_e)) {
          best = choice[j];
          best_e = e;
        }
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oe = __shfl_xor_sync(0xffffffffu, best_e, o);
      if (ob > best || (ob == best && oe < best_e)) {
        best = ob;
        best_e = oe;
      }
    }
    const int owner = best_e % 32, slot = best_e / 32;
    float sc = 0.0f;
#pragma unroll
    for (int j = 0; j < kMaxPer; ++j)
      if (lane == owner && j == slot) {
        taken |= 1u << j;
        sc = score[j];
      }
    sc = __shfl_sync(0xffffffffu, sc, owner);
    sel_score[s] = sc;
    sel_id[s] = best_e;
    denom = f_add(denom, sc);
  }
  if (lane != 0) return;
  // natural probabilities, entropy and the policy's K (routing_policy.cpp:
  // 89-134), in the reference's FP32 operation order
  if (!(denom > 0.0f) || !isfinite(denom)) atomicOr(err, kErrRoutingMass);
  int selected = k;
  if (pol.mode != 0 || sel_out || diag) {
    float p[16];
    float entropy = 0.0f;
    for (int s = 0; s < k; ++s) {
      p[s] = f_div(sel_score[s], denom);
      if (p[s] > 0.0f) entropy = f_sub(entropy, f_mul(p[s], logf(p[s])));
    }
    const float support = expf(entropy);
    int unfloored = k;
    if (pol.mode == 1) {
      unfloored = pol.fixed_k;
      selected = max(pol.fixed_k, pol.quality_floor_k);
    } else if (pol.mode == 2) {
      unfloored = choose_adaptive(p, k, 0, support, pol);
      selected = choose_adaptive(p, k, pol.quality_floor_k, support, pol);
    }
    if (sel_out) {
      sel_out[2 * (int64_t)t] = selected;
      sel_out[2 * (int64_t)t + 1] = selected > unfloored ? 1 : 0;
    }
    if (diag) {
      float mass = 0.0f;
      for (int s = 0; s < selected; ++s) mass = f_add(mass, p[s]);
      float4 d;
      d.x = k == 1 ? 0.0f : f_div(entropy, logf(static_cast<float>(k)));
      d.y = support;
      d.z = mass;
      d.w = boundary_confidence(p, k, selected);
      reinterpret_cast<float4*>(diag)[t] = d;
    }
  }
  float sdenom = denom;
  if (selected < k) {
    sdenom = 0.0f;
    for (int s = 0; s < selected; ++s) sdenom = f_add(sdenom, sel_score[s]);
    if (!(sdenom > 0.0f) || !isfinite(sdenom)) atomicOr(err, kErrRoutingMass);
  }
  for (int s = 0; s < k; ++s) {
    const bool on = s < selected;
    ids[(int64_t)t * k + s] = on ? sel_id[s] : -1;
    weights[(int64_t)t * k + s] = on ? f_mul(f_div(sel_score[s], sdenom), routed_scale) : 0.0f;
  }
}

// ------------------------------------------------------------------ permutation
constexpr int kChunk = 256;  // tokens per counting chunk

// Per 256-token chunk: per-expert counts and each (token, slot)'s rank among
// the chunk's tokens routed to the same expert (stable). E <= 256.
// skip_invalid = 1: an id outside [0, E) marks a slot with no expert here (the
// expert-parallel engines receive rows whose other slots live on other
// ranks); 2: only -1 does (a slot a fixed / adaptive routing policy left
// empty); 0, and other ids under 2: an error.
__global__ void __launch_bounds__(kChunk) permute_count_kernel(
    const int32_t* __restrict__ ids, int T, int k, int E, int skip_invalid,
    int32_t* __restrict__ chunk_count, int32_t* __restrict__ rank, uint32_t* err) {
  __shared__ uint32_t bits[256][kChunk / 32];
  const int c = blockIdx.x;
  for (int i = threadIdx.x; i < 256 * (kChunk / 32); i += blockDim.x) (&bits[0][0])[i] = 0;
  __syncthreads();
  const int t = c * kChunk + threadIdx.x;
  const int word = threadIdx.x / 32, bit = threadIdx.x % 32;
  int my[16];
  if (t < T) {
    for (int s = 0; s < k; ++s) {
      int e = ids[(int64_t)t * k + s];
      if (e < 0 || e >= E) {
        if (skip_invalid == 1 || (skip_invalid == 2 && e == -1)) {
          my[s] = -1;
          continue;
        }
        atomicOr(err, kErrBounds);
        e = 0;
      }
      my[s] = e;
      const uint32_t prev = atomicOr(&bits[e][word], 1u << bit);
      if (prev & (1u << bit)) atomicOr(err, kErrBounds);  // duplicate expert in one token
    }
  }
  __syncthreads();
  if (threadIdx.x < E) {
    int n = 0;
    for (int w = 0; w < kChunk / 32; ++w) n += __popc(bits[threadIdx.x][w]);
    chunk_count[(int64_t)c * E + threadIdx.x] = n;
  }
  if (t < T) {
    for (int s = 0; s < k; ++s) {
      const int e = my[s];
      if (e < 0) {
        rank[(int64_t)t * k + s] = -1;
        continue;
      }
      int r = __popc(bits[e][word] & ((1u << bit) - 1u));
      for (int w = 0; w < word; ++w) r += __popc(bits[e][w]);
      rank[(int64_t)t * k + s] = r;
    }
  }
}

// Block-wide exclusive scan over n <= blockDim.x values (Hillis-Steele).
__device__ int block_exclusive_scan(int v, int* buf, int* total) {
  const int i = threadIdx.x;
  buf[i] = v;
  __syncthreads();
  for (int off = 1; off < (int)blockDim.x; off <<= 1) {
    const int add = i >= off ? buf[i - off] : 0;
    __syncthreads();
    buf[i] += add;
    __syncthreads();
  }
  const int incl = buf[i];
  if (total) *total = buf[blockDim.x - 1];
  __syncthreads();
  return incl - v;
}

// Single block, blockDim >= nseg = E + has_shared (<= 1024). Turns chunk
// counts into per-chunk bases, builds segment starts (128-aligned), the
// quantizer row prefix (counts rounded up to 8) and the GEMM N-tile prefix,
// and clears the per-segment amax accumulators.
__global__ void permute_scan_kernel(int32_t* __restrict__ chunk_count, int nchunks, int T, int E,
                                    int has_shared, int shared_rows, int bn, int rows_per,
                                    int32_t* __restrict__ seg_count,
                                    int32_t* __restrict__ seg_start,
                                    int32_t* __restrict__ qprefix,
                                    int32_t* __restrict__ ntile_prefix,
                                    float* __restrict__ seg_amax, float* __restrict__ h_amax) {
  extern __shared__ int scan_buf[];
  const int e = threadIdx.x;
  const int nseg = E + has_shared;
  int count = 0;
  if (e < E) {
    for (int c = 0; c < nchunks; ++c) {
      const int v = chunk_count[(int64_t)c * E + e];
      chunk_count[(int64_t)c * E + e] = count;
      count += v;
    }
  } else if (e == E && has_shared) {
    count = shared_rows;  // tokens 0 .. shared_rows - 1 take the shared expert
  }
  const bool valid = e < nseg;
  // every (token, slot) takes rows_per operand rows (4 for the MXFP4 term
  // expansion); segment counts, starts and tiles are in rows, the quantizer
  // prefix in groups of rows_per rows (the rows rounded up to 8)
  const int rows = count * rows_per;
  int tot;
  const int start = block_exclusive_scan(valid ? segment_rows(rows, bn) : 0, scan_buf, &tot);
  const int q = block_exclusive_scan(valid ? (rows + 7) / 8 * 8 / rows_per : 0, scan_buf, &tot);
  const int qt = tot;
  // N tiles of at most bn rows
  const int nt = valid ? (rows + bn - 1) / bn : 0;
  const int tp = block_exclusive_scan(nt, scan_buf, &tot);
  if (valid) {
    seg_count[e] = rows;
    seg_start[e] = start;
    qprefix[e] = q;
    ntile_prefix[e] = tp;
    seg_amax[e] = 0.0f;
    h_amax[e] = 0.0f;
  }
  if (e == 0) {
    qprefix[nseg] = qt;
    ntile_prefix[nseg] = tot;
  }
  __syncthreads();
  if (e == nseg - 1) seg_start[nseg] = start + segment_rows(rows, bn);
}

// One thread per (token, slot) pair, plus one per token for the shared expert.
// Slots without an expert here (rank -1) and shared slots of tokens past
// shared_rows get pos = -1.
__global__ void permute_scatter_kernel(const int32_t* __restrict__ ids,
                                       const float* __restrict__ weights, int T, int k, int E,
                                       int has_shared, int shared_rows, int bn, int rows_per,
                                       const int32_t* __restrict__ chunk_base,
                                       const int32_t* __restrict__ rank,
                                       const int32_t* __restrict__ seg_start,
                                       const float* __restrict__ token_amax,
                                       int32_t* __restrict__ pos, int32_t* __restrict__ row_token,
                                       float* __restrict__ row_weight,
                                       float* __restrict__ seg_amax) {
  const int kk = k + has_shared;
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)T * kk) return;
  const int t = static_cast<int>(idx / kk), s = static_cast<int>(idx % kk);
  int p, e;
  float w;
  if (s < k) {
    const int r = rank[(int64_t)t * k + s];
    if (r < 0) {
      pos[idx] = -1;
      return;
    }
    e = ids[(int64_t)t * k + s];
    e = e < 0 || e >= E ? 0 : e;
    p = seg_start[e] + segment_row(rows_per * (chunk_base[(int64_t)(t / kChunk) * E + e] + r),
                                   bn);
    w = weights[(int64_t)t * k + s];
  } else {
    if (t >= shared_rows) {
      pos[idx] = -1;
      return;
    }
    e = E;
    p = seg_start[E] + segment_row(rows_per * t, bn);
    w = 1.0f;
  }
  pos[idx] = p;
  row_token[p] = t;
  row_weight[p] = w;
  atomicMax(reinterpret_cast<unsigned int*>(seg_amax + e), __float_as_uint(token_amax[t]));
}

// Global expert ids -> this engine's local ids (begin .. begin + count - 1
// -> 0 .. count - 1), -1 for experts held elsewhere.
__global__ void map_local_ids_kernel(const int32_t* __restrict__ ids, int64_t n, int begin,
                                     int count, int32_t* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int e = ids[i];
  out[i] = (e >= begin && e < begin + count) ? e - begin : -1;
}

cudaError_t launch_map_local_ids(const int32_t* ids, int64_t n, int begin, int count,
                                 int32_t* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  map_local_ids_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ids, n, begin, count, out);
  return cudaGetLastError();
}

// Batches of at most one 256-token chunk (decode): the count, scan and
// scatter above in one block, so the three dependent launches become one.
// Same outputs as the three kernels (chunk bases are 0 with one chunk; the
// per-(token, slot) ranks are recomputed from the shared bitmaps).
// blockDim = a power of two >= max(256, E + has_shared + 1).
__global__ void permute_small_kernel(const int32_t* __restrict__ ids,
                                     const float* __restrict__ weights,
                                     const float* __restrict__ token_amax, int T, int k, int E,
                                     int has_shared, int shared_rows, int bn, int rows_per,
                                     int skip_invalid, PermuteBuffers b, uint32_t* err) {
  __shared__ uint32_t bits[256][kChunk / 32];
  extern __shared__ int scan_buf[];
  for (int i = threadIdx.x; i < 256 * (kChunk / 32); i += blockDim.x) (&bits[0][0])[i] = 0;
  __syncthreads();
  auto skipped = [&](int e) {
    return (e < 0 || e >= E) && (skip_invalid == 1 || (skip_invalid == 2 && e == -1));
  };
  {
    const int t = threadIdx.x;
    const int word = t / 32, bit = t % 32;
    if (t < T) {
      for (int s = 0; s < k; ++s) {
        int e = ids[(int64_t)t * k + s];
        if (skipped(e)) continue;
        if (e < 0 || e >= E) {
          atomicOr(err, kErrBounds);
          e = 0;
        }
        const uint32_t prev = atomicOr(&bits[e][word], 1u << bit);
        if (prev & (1u << bit)) atomicOr(err, kErrBounds);  // duplicate expert in one token
      }
    }
  }
  __syncthreads();
  // segment counts, starts, quantizer prefix, tile prefix (permute_scan_kernel)
  const int e = threadIdx.x;
  const int nseg = E + has_shared;
  int count = 0;
  if (e < E) {
    for (int w = 0; w < kChunk / 32; ++w) count += __popc(bits[e][w]);
  } else if (e == E && has_shared) {
    count = shared_rows;
  }
  const bool valid = e < nseg;
  const int rows = count * rows_per;
  int tot;
  const int start = block_exclusive_scan(valid ? segment_rows(rows, bn) : 0, scan_buf, &tot);
  const int q = block_exclusive_scan(valid ? (rows + 7) / 8 * 8 / rows_per : 0, scan_buf, &tot);
  const int qt = tot;
  const int nt = valid ? (rows + bn - 1) / bn : 0;
  const int tp = block_exclusive_scan(nt, scan_buf, &tot);
  if (valid) {
    b.seg_count[e] = rows;
    b.seg_start[e] = start;
    b.qprefix[e] = q;
    b.ntile_prefix[e] = tp;
    b.seg_amax[e] = 0.0f;
    b.h_amax[e] = 0.0f;
  }
  if (e == 0) {
    b.qprefix[nseg] = qt;
    b.ntile_prefix[nseg] = tot;
  }
  if (e == nseg - 1) b.seg_start[nseg] = start + segment_rows(rows, bn);
  __syncthreads();
  // scatter (permute_scatter_kernel with chunk base 0)
  const int kk = k + has_shared;
  for (int idx = threadIdx.x; idx < T * kk; idx += blockDim.x) {
    const int t = idx / kk, s = idx % kk;
    int p, ex;
    float w;
    if (s < k) {
      ex = ids[(int64_t)t * k + s];
      if (skipped(ex)) {
        b.pos[idx] = -1;
        continue;
      }
      ex = ex < 0 || ex >= E ? 0 : ex;
      const int word = t / 32, bit = t % 32;
      int r = __popc(bits[ex][word] & ((1u << bit) - 1u));
      for (int wd = 0; wd < word; ++wd) r += __popc(bits[ex][wd]);
      p = b.seg_start[ex] + segment_row(rows_per * r, bn);
      w = weights[(int64_t)t * k + s];
    } else {
      if (t >= shared_rows) {
        b.pos[idx] = -1;
        continue;
      }
      ex = E;
      p = b.seg_start[E] + segment_row(rows_per * t, bn);
      w = 1.0f;
    }
    b.pos[idx] = p;
    b.row_token[p] = t;
    b.row_weight[p] = w;
    atomicMax(reinterpret_cast<unsigned int*>(b.seg_amax + ex), __float_as_uint(token_amax[t]));
  }
}

// Expert-parallel FP4 dispatch helpers. slab amax: amax[e] = max over the
// (token, slot) pairs routed to e of the token's max |x| (the slab amax the
// permutation scatter accumulates per segment), amax zeroed by the caller.
// group positions: out[i] = the expert-major row of received row
// group_rows[i] (its only routed slot, slot 0 of row row_base + g), -1 kept.
__global__ void slab_amax_kernel(const float* __restrict__ token_amax,
                                 const int32_t* __restrict__ ids, int64_t n, int k, int E,
                                 float* __restrict__ amax) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int e = ids[i];
  if (e >= 0 && e < E)
    atomicMax(reinterpret_cast<unsigned int*>(amax + e), __float_as_uint(token_amax[i / k]));
}

__global__ void map_group_pos_kernel(const int32_t* __restrict__ group_rows, int64_t n,
                                     const int32_t* __restrict__ pos, int kk, int row_base,
                                     int32_t* __restrict__ out) {
  const int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  const int g = group_rows[i];
  out[i] = g < 0 ? -1 : pos[(int64_t)(row_base + g) * kk];
}

cudaError_t launch_slab_amax(const float* token_amax, const int32_t* ids, int T, int k, int E,
                             float* amax, cudaStream_t st) {
  cudaError_t e = cudaMemsetAsync(amax, 0, sizeof(float) * E, st);
  if (e != cudaSuccess || T <= 0) return e;
  const int64_t n = (int64_t)T * k;
  slab_amax_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(token_amax, ids, n, k, E, amax);
  return cudaGetLastError();
}

cudaError_t launch_map_group_pos(const int32_t* group_rows, int64_t n, const int32_t* pos,
                                 int kk, int row_base, int32_t* out, cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  map_group_pos_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(group_rows, n, pos, kk,
                                                                    row_base, out);
  return cudaGetLastError();
}

// ------------------------------------------------------------------ launchers
cudaError_t launch_topk(const float* in, int values_are_scores, const float* bias, int T, int E,
                        int k, float routed_scale, int32_t* ids, float* weights, uint32_t* err,
                        cudaStream_t st, const RoutingPolicy& policy, int32_t* sel,
                        float* diag) {
  return launch_topk_planes(in, 1, nullptr, values_are_scores, bias, T, E, k, routed_scale, ids,
                            weights, err, st, policy, sel, diag);
}

cudaError_t launch_topk_planes(const float* in, int nplanes, float* logits_out,
                               int values_are_scores, const float* bias, int T, int E, int k,
                               float routed_scale, int32_t* ids, float* weights, uint32_t* err,
                               cudaStream_t st, const RoutingPolicy& policy, int32_t* sel,
                               float* diag) {
  if (T == 0) return cudaSuccess;
  if (E > 512 || nplanes < 1) return cudaErrorInvalidValue;
  const int warps = 8;
  const dim3 grid((T + warps - 1) / warps), block(warps * 32);
  if (E <= 256)
    topk_kernel<8><<<grid, block, 0, st>>>(in, nplanes, logits_out, values_are_scores, bias, T,
                                           E, k, routed_scale, ids, weights, err, policy, sel,
                                           diag);
  else
    topk_kernel<16><<<grid, block, 0, st>>>(in, nplanes, logits_out, values_are_scores, bias, T,
                                            E, k, routed_scale, ids, weights, err, policy, sel,
                                            diag);
  return cudaGetLastError();
}

cudaError_t launch_permute(const int32_t* ids, const float* weights, const float* token_amax,
                           int T, int k, int E, int has_shared, int bn, PermuteBuffers b,
                           uint32_t* err, cudaStream_t st, int rows_per, int skip_invalid,
                           int shared_rows, int* launches) {
  const int nchunks = (T + kChunk - 1) / kChunk;
  if (shared_rows < 0 || shared_rows > T) shared_rows = T;
  if (nchunks == 1 && E <= 256) {
    int threads = 256;
    while (threads < E + has_shared + 1) threads <<= 1;
    permute_small_kernel<<<1, threads, threads * sizeof(int), st>>>(
        ids, weights, token_amax, T, k, E, has_shared, shared_rows, bn, rows_per, skip_invalid,
        b, err);
    if (launches) *launches = 1;
    return cudaGetLastError();
  }
  if (launches) *launches = 3;
  if (T > 0) {
    permute_count_kernel<<<nchunks, kChunk, 0, st>>>(ids, T, k, E, skip_invalid, b.chunk_count,
                                                     b.rank, err);
  }
  const int nseg = E + has_shared;
  int threads = 32;
  while (threads < nseg + 1) threads <<= 1;
  permute_scan_kernel<<<1, threads, threads * sizeof(int), st>>>(
      b.chunk_count, nchunks, T, E, has_shared, shared_rows, bn, rows_per, b.seg_count,
      b.seg_start, b.qprefix, b.ntile_prefix, b.seg_amax, b.h_amax);
  const int64_t n = (int64_t)T * (k + has_shared);
  if (n > 0) {
    permute_scatter_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(
        ids, weights, T, k, E, has_shared, shared_rows, bn, rows_per, b.chunk_count, b.rank,
        b.seg_start,
        token_amax, b.pos,
        b.row_token, b.row_weight, b.seg_amax);
  }
  return cudaGetLastError();
}

}  // namespace glm5x
