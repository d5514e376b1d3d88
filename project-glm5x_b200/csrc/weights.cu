// weights.cu -- admission-time weight layout kernels and the combine kernel.
//
// Weight admission keeps the reference's NVFP4 sidecar layout (packed
// [rows, K/2], low nibble first, scales in the 128x4 blocked layout of
// reference/glm5x_ref/nvfp4.py:23-40 as stored by packed_cache.py:277-309);
// the only change is the gate/up interleave that lets one 128-row MMA tile
// hold 64 gate rows and the 64 matching up rows. MXFP4 row-major E8M0 scales
// (reference/k3x_ref/mxfp4.py:98-101) are reordered into the same blocked
// layout.
//
// combine replaces the reference's weighted scatter (index_add_,
// reference/glm5x_ref/layer10_moe.py:843-846; ragged_expert_mix_kernel,
// runtime/cuda/moe_layer.cu:25-44; shared add moe_layer.cu:64-70): every
// token gathers its k routed rows plus its shared-expert row (already
// weighted in the down-projection epilogue) in FP32.
#include <algorithm>
#include <cstdint>

#include "fp4_codec.h"
#include "glm5x_kernels.cuh"

namespace glm5x {

// Interleaved row R of the stacked gate/up matrix: group q = R / 32, rows
// 0-15 of the group are gate rows 16q..16q+15 and rows 16-31 the same up rows.
__device__ __forceinline__ void interleave_source(int R, int* which, int* j) {
  *which = (R & 16) ? 1 : 0;
  *j = (R >> 5) * 16 + (R & 15);
}

__global__ void interleave_rows_kernel(const uint8_t* __restrict__ gate,
                                       const uint8_t* __restrict__ up, int I, int row_bytes,
                                       uint8_t* __restrict__ dst) {
  const int R = blockIdx.x;
  int which, j;
  interleave_source(R, &which, &j);
  const uint4* s = reinterpret_cast<const uint4*>((which ? up : gate) + (size_t)j * row_bytes);
  uint4* d = reinterpret_cast<uint4*>(dst + (size_t)R * row_bytes);
  for (int i = threadIdx.x; i < row_bytes / 16; i += blockDim.x) d[i] = s[i];
}

__global__ void interleave_scales_kernel(const uint8_t* __restrict__ gate_sf,
                                         const uint8_t* __restrict__ up_sf, int I, int sf_cols,
                                         uint8_t* __restrict__ dst_sf) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= (int64_t)2 * I * sf_cols) return;
  const int R = static_cast<int>(idx / sf_cols), c = static_cast<int>(idx % sf_cols);
  int which, j;
  interleave_source(R, &which, &j);
  dst_sf[blocked_sf_offset(R, c, sf_cols)] =
      (which ? up_sf : gate_sf)[blocked_sf_offset(j, c, sf_cols)];
}

__global__ void scales_to_blocked_kernel(const uint8_t* __restrict__ rm, int64_t rows,
                                         int64_t sf_cols, uint8_t* __restrict__ blocked) {
  const int64_t idx = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (idx >= rows * sf_cols) return;
  const int64_t r = idx / sf_cols, c = idx % sf_cols;
  blocked[blocked_sf_offset(r, c, sf_cols)] = rm[idx];
}

// acc[0..7] += the 8 values of piece v (16 bytes) of y rows rows[0..KK), in
// slot order, empty slots (-1) skipped; every slot's load is issued before
// the first sum, so a thread has all of them in flight at once.
template <int KK>
__device__ __forceinline__ void sum_slot_pieces(const uint16_t* __restrict__ y,
                                                const int32_t* rows, int v, int H,
                                                float (&acc)[8]) {
  uint4 q[KK];
#pragma unroll
  for (int s = 0; s < KK; ++s)
    q[s] = rows[s] >= 0 ? __ldg(reinterpret_cast<const uint4*>(y + (int64_t)rows[s] * H) + v)
                        : make_uint4(0u, 0u, 0u, 0u);
#pragma unroll
  for (int s = 0; s < KK; ++s) {
    if (rows[s] < 0) continue;
    const uint32_t w[4] = {q[s].x, q[s].y, q[s].z, q[s].w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] += __uint_as_float(w[i] << 16);
      acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

// The same for any slot count, one slot's load at a time.
__device__ __forceinline__ void sum_slot_pieces_any(const uint16_t* __restrict__ y,
                                                    const int32_t* rows, int kk, int v, int H,
                                                    float (&acc)[8]) {
  for (int s = 0; s < kk; ++s) {
    if (rows[s] < 0) continue;
    const uint4 q = __ldg(reinterpret_cast<const uint4*>(y + (int64_t)rows[s] * H) + v);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      acc[2 * i] += __uint_as_float(w[i] << 16);
      acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
    }
  }
}

// One block per token; 8 BF16 (16 bytes) per vector. accumulate: add the
// sum to out instead of storing it.
__global__ void combine_kernel(const uint16_t* __restrict__ y, const int32_t* __restrict__ pos,
                               int kk, int H, float* __restrict__ out, int accumulate) {
  // block (t, y) sums 8-element groups y * per .. (y + 1) * per - 1 of token t
  const int t = blockIdx.x;
  const int per = (H / 8 + gridDim.y - 1) / gridDim.y;
  const int v_end = min(H / 8, ((int)blockIdx.y + 1) * per);
  __shared__ int32_t rows[32];
  if (threadIdx.x < kk) rows[threadIdx.x] = pos[(int64_t)t * kk + threadIdx.x];
  __syncthreads();
  for (int v = blockIdx.y * per + threadIdx.x; v < v_end; v += blockDim.x) {
    float acc[8] = {};
    sum_slot_pieces_any(y, rows, kk, v, H, acc);  // empty slots: no expert on this engine
    float4* o = reinterpret_cast<float4*>(out + (int64_t)t * H) + 2 * v;
    if (accumulate) {
      const float4 a = o[0], b = o[1];
      o[0] = make_float4(a.x + acc[0], a.y + acc[1], a.z + acc[2], a.w + acc[3]);
      o[1] = make_float4(b.x + acc[4], b.y + acc[5], b.z + acc[6], b.w + acc[7]);
    } else {
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// combine_kernel for a fixed slot count (the layer's top-8 + shared expert),
// all slot loads of a piece in flight at once; the sums still run in slot
// order, skipping empty slots, so the result is combine_kernel's bit for bit.
template <int KK>
__global__ void combine_fixed_kernel(const uint16_t* __restrict__ y,
                                     const int32_t* __restrict__ pos, int H,
                                     float* __restrict__ out, int accumulate) {
  const int t = blockIdx.x;
  const int per = (H / 8 + gridDim.y - 1) / gridDim.y;
  const int v_end = min(H / 8, ((int)blockIdx.y + 1) * per);
  __shared__ int32_t rows[KK];
  if (threadIdx.x < KK) rows[threadIdx.x] = pos[(int64_t)t * KK + threadIdx.x];
  __syncthreads();
  for (int v = blockIdx.y * per + threadIdx.x; v < v_end; v += blockDim.x) {
    float acc[8] = {};
    sum_slot_pieces<KK>(y, rows, v, H, acc);
    float4* o = reinterpret_cast<float4*>(out + (int64_t)t * H) + 2 * v;
    if (accumulate) {
      const float4 a = o[0], b = o[1];
      o[0] = make_float4(a.x + acc[0], a.y + acc[1], a.z + acc[2], a.w + acc[3]);
      o[1] = make_float4(b.x + acc[4], b.y + acc[5], b.z + acc[6], b.w + acc[7]);
    } else {
      o[0] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

// Received rows of an expert-parallel engine: partial[r] = BF16(sum over the
// row's slots of y[pos[r, s]]) for r < *count (a device value), FP32 sums in
// slot order then one round to nearest even. Grid-stride over rows, so the
// launch is sized by the capacity and the count is read on the device.
__global__ void combine_rows_bf16_kernel(const uint16_t* __restrict__ y,
                                         const int32_t* __restrict__ pos, int64_t cap,
                                         const int32_t* __restrict__ count, int kk, int H,
                                         uint16_t* __restrict__ out) {
  const int64_t n = cap < (int64_t)*count ? cap : (int64_t)*count;
  __shared__ int32_t rows[32];
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    __syncthreads();
    if (threadIdx.x < kk) rows[threadIdx.x] = pos[r * kk + threadIdx.x];
    __syncthreads();
    for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
      float acc[8] = {};
      if (kk == 9)
        sum_slot_pieces<9>(y, rows, v, H, acc);
      else
        sum_slot_pieces_any(y, rows, kk, v, H, acc);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i]));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i + 1]));
        o[i] = lo | (hi << 16);
      }
      reinterpret_cast<uint4*>(out + r * H)[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
}

cudaError_t launch_combine_rows_bf16(const uint16_t* y, const int32_t* pos, int64_t cap,
                                     const int32_t* count, int kk, int H, uint16_t* out,
                                     cudaStream_t st) {
  if (cap <= 0) return cudaSuccess;
  if (kk > 32 || H % 8) return cudaErrorInvalidValue;
  const unsigned blocks = (unsigned)std::min<int64_t>(cap, 148 * 8);
  combine_rows_bf16_kernel<<<blocks, 256, 0, st>>>(y, pos, cap, count, kk, H, out);
  return cudaGetLastError();
}

__global__ void combine_rows_return_kernel(const uint16_t* __restrict__ y,
                                           const int32_t* __restrict__ pos, int64_t cap,
                                           const int32_t* __restrict__ count, int kk, int H,
                                           RowReturn ret) {
  const int64_t n = cap < (int64_t)*count ? cap : (int64_t)*count;
  __shared__ int32_t rows[32];
  __shared__ int32_t off[kMaxReturnRanks];
  if ((int)threadIdx.x < ret.W) off[threadIdx.x] = ret.recv_off[threadIdx.x];
  for (int64_t r = blockIdx.x; r < n; r += gridDim.x) {
    __syncthreads();
    if (threadIdx.x < kk) rows[threadIdx.x] = pos[r * kk + threadIdx.x];
    __syncthreads();
    int s = 0;
    for (int i = 1; i < ret.W; ++i)
      if (off[i] <= r) s = i;
    const int64_t p = r - off[s];
    if (p < 0 || p >= ret.limit) {
      if (threadIdx.x == 0) atomicOr(ret.err, 1u << 3);  // kErrBounds
      continue;
    }
    uint4* dst = reinterpret_cast<uint4*>(ret.base[s] + p * H);
    for (int v = threadIdx.x; v < H / 8; v += blockDim.x) {
      float acc[8] = {};
      if (kk == 9)
        sum_slot_pieces<9>(y, rows, v, H, acc);
      else
        sum_slot_pieces_any(y, rows, kk, v, H, acc);
      uint32_t o[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i]));
        const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(acc[2 * i + 1]));
        o[i] = lo | (hi << 16);
      }
      dst[v] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  // every store visible system-wide, then the grid's last block raises the
  // sources' flags
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(ret.done, 1ull) + 1ull == ret.done_target;
  __syncthreads();
  if (last && (int)threadIdx.x < ret.W) {
    __threadfence_system();
    asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(ret.flag[threadIdx.x]),
                 "l"(ret.epoch)
                 : "memory");
  }
}

cudaError_t launch_combine_rows_return(const uint16_t* y, const int32_t* pos, int64_t cap,
                                       const int32_t* count, int kk, int H,
                                       const RowReturn& ret, cudaStream_t st) {
  if (kk > 32 || H % 8 || ret.W > kMaxReturnRanks || ret.grid <= 0)
    return cudaErrorInvalidValue;
  combine_rows_return_kernel<<<ret.grid, 256, 0, st>>>(y, pos, cap, count, kk, H, ret);
  return cudaGetLastError();
}

cudaError_t launch_interleave_gate_up(const uint8_t* gate_packed, const uint8_t* gate_sf,
                                      const uint8_t* up_packed, const uint8_t* up_sf, int I,
                                      int K, int group, uint8_t* dst_packed, uint8_t* dst_sf,
                                      cudaStream_t st) {
  interleave_rows_kernel<<<2 * I, 128, 0, st>>>(gate_packed, up_packed, I, K / 2, dst_packed);
  const int sf_cols = K / group;
  const int64_t n = (int64_t)2 * I * sf_cols;
  interleave_scales_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(gate_sf, up_sf, I,
                                                                        sf_cols, dst_sf);
  return cudaGetLastError();
}

cudaError_t launch_scales_to_blocked(const uint8_t* rm, int64_t rows, int64_t sf_cols,
                                     uint8_t* blocked, cudaStream_t st) {
  const int64_t n = rows * sf_cols;
  if (n == 0) return cudaSuccess;
  scales_to_blocked_kernel<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(rm, rows, sf_cols,
                                                                        blocked);
  return cudaGetLastError();
}

__global__ void find_byte_kernel(const uint8_t* __restrict__ p, int64_t n, uint32_t value,
                                 uint32_t* __restrict__ found) {
  bool hit = false;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    hit |= p[i] == value;
  if (__any_sync(0xffffffffu, hit) && (threadIdx.x & 31) == 0) atomicOr(found, 1u);
}

cudaError_t launch_find_byte(const uint8_t* p, int64_t n, uint32_t value, uint32_t* found,
                             cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = std::min<int64_t>((n + 255) / 256, 1184);
  find_byte_kernel<<<(unsigned)blocks, 256, 0, st>>>(p, n, value, found);
  return cudaGetLastError();
}

cudaError_t launch_combine(const uint16_t* y, const int32_t* pos, int T, int kk, int H,
                           float* out, cudaStream_t st, int accumulate) {
  if (T == 0) return cudaSuccess;
  if (kk > 32 || H % 8) return cudaErrorInvalidValue;
  // small batches split each token's row over several blocks to fill the SMs
  const int split = std::max(1, std::min(H / 8 / 256, 296 / T));
  if (kk == 9)
    combine_fixed_kernel<9><<<dim3(T, split), 256, 0, st>>>(y, pos, H, out, accumulate);
  else
    combine_kernel<<<dim3(T, split), 256, 0, st>>>(y, pos, kk, H, out, accumulate);
  return cudaGetLastError();
}

// Moves the engine's error word into a per-forward slot and clears it, in
// stream order after the forward's kernels.
__global__ void error_snapshot_kernel(uint32_t* err, uint32_t* snap) {
  *snap = *err;
  *err = 0u;
}

// Stores device words into mapped page-locked host memory from the SMs, so a
// small read-back needs no copy engine (and does not queue behind a large
// download another stream has on one).
__global__ void store_ints_to_host_kernel(const int64_t* __restrict__ src, int64_t n,
                                          volatile int64_t* dst) {
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) dst[i] = src[i];
  __threadfence_system();
}

cudaError_t launch_store_ints_to_host(const int64_t* src, int64_t n, int64_t* dst_mapped,
                                      cudaStream_t st) {
  if (n <= 0) return cudaSuccess;
  store_ints_to_host_kernel<<<1, 256, 0, st>>>(src, n, dst_mapped);
  return cudaGetLastError();
}

cudaError_t launch_error_snapshot(uint32_t* err, uint32_t* snap, cudaStream_t st) {
  error_snapshot_kernel<<<1, 1, 0, st>>>(err, snap);
  return cudaGetLastError();
}

}  // namespace glm5x
