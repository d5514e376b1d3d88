// ep_peer.cu -- expert parallelism with the token exchange in the library's
// own kernels over NVLink peer memory.
//
// The reference runs every expert in one process (layer10_moe.py:791-847 +
// 954-961); this is the multi-GPU form of the same computation, one process
// per GPU, rank r of W holding experts [r * E/W, (r + 1) * E/W) plus a
// replica of the shared expert and the router. Every rank allocates one
// block of device memory with the same layout (below) and maps every peer's
// block through CUDA IPC; a forward on rank r then runs, in stream order:
//
//   route      the engine's router over the T local tokens;
//   plan       per destination d: which tokens have an expert on d and each
//              such token's place among them (prefix sum), the send counts;
//   exchange   each rank writes its row of send counts into every peer's
//              count matrix and raises a flag there; after all W flags, the
//              received-row count and this rank's offset in each
//              destination's receive area follow from the matrix;
//   dispatch   each token's BF16 row, its top-k ids masked to d's experts,
//              its weights and its max |x| are stored straight into d's
//              receive area (NVLink stores), one warp per token reading the
//              row once for all destinations; the grid's last block to
//              finish then adds one to each destination's arrival counter;
//   experts    after all arrivals: the engine over [local tokens | received
//              rows] in one call; local tokens take the shared expert (FP32
//              out), received rows their held experts, and the engine's last
//              kernel stores each received row's weighted sum as BF16 straight
//              into its source's return area (NVLink stores), then raises a
//              ready flag in every source;
//   combine    after all W ready flags: each local token's partial sums are
//              read from this rank's own return area and added in
//              destination order onto its shared-expert row.
//
// The received rows and their sums match ep.py's NCCL all-to-all path bit
// for bit (same rows, same order, same BF16 rounding, same FP32 order).
// Buffers are double-buffered by forward parity; every flag holds the
// forward's epoch, so nothing is reset between forwards. A rank reuses a
// parity's areas two forwards later, after every peer has finished the
// combine that read them (each combine waits for every destination, and the
// next dispatch follows it in stream order). Every wait is bounded
// (kWaitBudgetNs): on expiry the kernel records kErrWaitTimeout and goes on,
// and the host reports GLM5X_WAIT_TIMEOUT. No TMA and no multicast here:
// plain 16-byte loads and stores to peer memory.
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <string>
#include <vector>

#include "../../include/glm5x_moe.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {
glm5x_status engine_forward_peer_rows(glm5x_moe* m, const uint16_t* rows, int64_t local_cap,
                                      int64_t local_tokens, int64_t recv_cap,
                                      const int32_t* ids, const float* weights,
                                      const float* row_amax, const int32_t* recv_count,
                                      float* out_local, const RowReturn* ret, cudaStream_t st);
int engine_device(const glm5x_moe* m);

namespace {

constexpr int kMaxWorld = 16;
// Most blocks of the dispatch / combine kernels: four 256-thread blocks per
// SM keep more NVLink stores in flight than two (N = 2, C5: dispatch 0.182 ->
// 0.174 ms, combine 0.135 -> 0.104 ms, step 2.669 -> 2.629 ms; at N = 8 the
// two measured within 1 % of each other).
#ifndef G5_EP_GRID
#define G5_EP_GRID 592
#endif
constexpr int kGrid = G5_EP_GRID;
constexpr int kThreads = 256;

// Byte offsets inside one rank's block; identical on every rank.
struct Layout {
  size_t rows[2];     // [local_cap + recv_cap, H] BF16: local tokens, then received rows
  size_t ids[2];      // [local_cap + recv_cap, k] int32 (global ids, -1 = none)
  size_t wts[2];      // [local_cap + recv_cap, k] FP32
  size_t amax[2];     // [local_cap + recv_cap] FP32
  size_t ret[2];      // [W, local_cap, H] BF16: the sums destination d returns for this
                      // rank's rows sent to d, at row d * local_cap + position
  size_t counts[2];   // [W, W] int32: counts[s][d] = rows s sends to d
  size_t cnt_flag[2]; // [W] uint64: epoch when source s's count row arrived
  size_t ready[2];    // [W] uint64: epoch when destination d's partial sums are ready
  size_t arrive;      // uint64: dispatch blocks arrived (monotonic)
  size_t total;
};

struct Peers {
  uint8_t* base[kMaxWorld];
};

__device__ __forceinline__ uint64_t ld_acquire_sys(const uint64_t* p) {
  uint64_t v;
  asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ void red_add_release_sys(uint64_t* p, uint64_t v) {
  asm volatile("red.release.sys.global.add.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// Spins until *p >= target, for at most kWaitBudgetNs; records a timeout.
__device__ bool wait_at_least(const uint64_t* p, uint64_t target, uint32_t* err) {
  if (ld_acquire_sys(p) >= target) return true;
  const uint64_t t0 = globaltimer_ns();
  for (uint32_t n = 1;; ++n) {
    if (ld_acquire_sys(p) >= target) return true;
    if ((n & 63u) == 0 && globaltimer_ns() - t0 > kWaitBudgetNs) {
      atomicOr(err, kErrWaitTimeout);
      return false;
    }
  }
}

template <typename T>
__host__ __device__ __forceinline__ T* at(uint8_t* base, size_t off) {
  return reinterpret_cast<T*>(base + off);
}

// ------------------------------------------------------------------ plan
// Block d: mask[t] = token t has an expert on rank d; pos[t, d] = its place
// among those tokens (ascending t), -1 if none; send_count[d].
__global__ void ep_plan_kernel(const int32_t* __restrict__ ids, int T, int k, int per, int W,
                               int32_t* __restrict__ pos, int32_t* __restrict__ send_count) {
  const int d = blockIdx.x;
  __shared__ int warp_tot[32];
  __shared__ int base;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  if (threadIdx.x == 0) base = 0;
  __syncthreads();
  for (int t0 = 0; t0 < T; t0 += blockDim.x) {
    const int t = t0 + threadIdx.x;
    int m = 0;
    if (t < T)
      for (int s = 0; s < k; ++s) {
        const int e = ids[(int64_t)t * k + s];
        m |= (e >= 0 && e / per == d) ? 1 : 0;
      }
    int incl = m;
    for (int o = 1; o < 32; o <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += v;
    }
    if (lane == 31) warp_tot[warp] = incl;
    __syncthreads();
    int before = 0, chunk = 0;
    for (int w = 0; w < nwarps; ++w) {
      if (w < warp) before += warp_tot[w];
      chunk += warp_tot[w];
    }
    if (t < T) pos[(int64_t)t * W + d] = m ? base + before + incl - m : -1;
    __syncthreads();
    if (threadIdx.x == 0) base += chunk;
    __syncthreads();
  }
  if (threadIdx.x == 0) send_count[d] = base;
}

// ------------------------------------------------------------------ exchange
struct ExchangeArgs {
  Peers peers;
  size_t counts_off, flag_off;
  int rank, W;
  uint64_t epoch;
  int64_t recv_cap;
  const int32_t* send_count;  // [W] local
  int32_t* recv_count;        // out: rows received this forward
  int32_t* send_off;          // out [W]: first row of this rank's rows in d's receive area
  int32_t* recv_off;          // out [W]: first received row from each source
  uint32_t* err;
};

__global__ void ep_exchange_kernel(ExchangeArgs a) {
  const int tid = threadIdx.x;
  if (tid < a.W) {
    const int d = tid;
    int32_t* row = at<int32_t>(a.peers.base[d], a.counts_off) + (int64_t)a.rank * a.W;
    for (int j = 0; j < a.W; ++j) row[j] = a.send_count[j];
    __threadfence_system();
    st_release_sys(at<uint64_t>(a.peers.base[d], a.flag_off) + a.rank, a.epoch);
  }
  __syncthreads();
  if (tid < a.W)
    wait_at_least(at<uint64_t>(a.peers.base[a.rank], a.flag_off) + tid, a.epoch, a.err);
  __syncthreads();
  if (tid == 0) {
    const volatile int32_t* c = at<int32_t>(a.peers.base[a.rank], a.counts_off);
    int64_t R = 0;
    for (int s = 0; s < a.W; ++s) R += c[s * a.W + a.rank];
    if (R > a.recv_cap) {
      atomicOr(a.err, kErrBounds);
      R = a.recv_cap;
    }
    *a.recv_count = (int32_t)R;
    int64_t off_s = 0;
    for (int s = 0; s < a.W; ++s) {
      a.recv_off[s] = (int32_t)off_s;
      off_s += c[s * a.W + a.rank];
    }
    for (int d = 0; d < a.W; ++d) {
      int64_t off = 0;
      for (int s = 0; s < a.rank; ++s) off += c[s * a.W + d];
      if (off + c[a.rank * a.W + d] > a.recv_cap) atomicOr(a.err, kErrBounds);
      a.send_off[d] = (int32_t)off;
    }
  }
}

// ids / weights of received rows past the count: -1 / 0, so the engine's
// capacity-sized permutation skips them.
__global__ void ep_clear_tail_kernel(int32_t* __restrict__ ids, float* __restrict__ wts,
                                     int64_t local_cap, int64_t recv_cap, int k,
                                     const int32_t* __restrict__ recv_count) {
  const int64_t first = (local_cap + *recv_count) * k, end = (local_cap + recv_cap) * k;
  for (int64_t i = first + blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < end;
       i += (int64_t)gridDim.x * blockDim.x) {
    ids[i] = -1;
    wts[i] = 0.0f;
  }
}

// ------------------------------------------------------------------ dispatch
struct DispatchArgs {
  Peers peers;
  size_t rows_off, ids_off, wts_off, amax_off, arrive_off;
  unsigned long long* done;       // local count of finished dispatch blocks (monotonic)
  unsigned long long done_target; // its value once this forward's blocks have all finished
  const uint16_t* x;      // [T, H] local tokens
  const int32_t* ids;     // [T, k] global ids
  const float* w;         // [T, k]
  const int32_t* pos;     // [T, W]
  const int32_t* send_off;
  int T, H, k, W, per, rank;
  int64_t local_cap, recv_cap;
  uint32_t* err;
};

__global__ void __launch_bounds__(kThreads) ep_dispatch_kernel(DispatchArgs a) {
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int vec = a.H / 8;  // 16-byte vectors per row
  uint8_t* own = a.peers.base[a.rank];
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.T; t += warps) {
    // destination rows of this token (lane d computes destination d's)
    int64_t my_row = -1;
    if (lane < a.W) {
      const int p = a.pos[(int64_t)t * a.W + lane];
      if (p >= 0) {
        my_row = a.local_cap + a.send_off[lane] + p;
        if (my_row >= a.local_cap + a.recv_cap) {
          atomicOr(a.err, kErrBounds);
          my_row = -1;
        }
      }
    }
    // every lane gets every destination's row (fixed-trip loop: registers)
    uint4* dst[kMaxWorld];
#pragma unroll
    for (int d = 0; d < kMaxWorld; ++d) {
      const int64_t row = __shfl_sync(0xffffffffu, my_row, d & 31);
      dst[d] = (d < a.W && row >= 0) ? at<uint4>(a.peers.base[d], a.rows_off) + row * vec
                                     : nullptr;
      if (d < a.W && row >= 0 && lane < a.k) {
        // this token's ids masked to d's experts, and their weights
        const int e = a.ids[(int64_t)t * a.k + lane];
        const bool held = e >= 0 && e / a.per == d;
        at<int32_t>(a.peers.base[d], a.ids_off)[row * a.k + lane] = held ? e : -1;
        at<float>(a.peers.base[d], a.wts_off)[row * a.k + lane] =
            held ? a.w[(int64_t)t * a.k + lane] : 0.0f;
      }
    }
    // the row: read once, stored locally (shared expert) and to every destination
    const uint4* src = reinterpret_cast<const uint4*>(a.x + (int64_t)t * a.H);
    uint4* local = at<uint4>(own, a.rows_off) + (int64_t)t * vec;
    float amax = 0.0f;
    for (int v = lane; v < vec; v += 32) {
      const uint4 q = __ldg(src + v);
      const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
      for (int i = 0; i < 4; ++i)
        amax = fmaxf(amax, fmaxf(fabsf(__uint_as_float(wd[i] << 16)),
                                 fabsf(__uint_as_float(wd[i] & 0xffff0000u))));
      local[v] = q;
#pragma unroll
      for (int d = 0; d < kMaxWorld; ++d)
        if (dst[d]) dst[d][v] = q;
    }
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) at<float>(own, a.amax_off)[t] = amax;
    if (my_row >= 0) at<float>(a.peers.base[lane], a.amax_off)[my_row] = amax;
  }
  // Every thread's stores become visible system-wide, then the block counts
  // itself done; the last block of the grid adds one arrival at every
  // destination (one per source rank and forward).
  __threadfence_system();
  __syncthreads();
  __shared__ bool last;
  if (threadIdx.x == 0) last = atomicAdd(a.done, 1ull) + 1ull == a.done_target;
  __syncthreads();
  if (last && (int)threadIdx.x < a.W) {
    __threadfence_system();
    red_add_release_sys(at<uint64_t>(a.peers.base[threadIdx.x], a.arrive_off), 1);
  }
}

__global__ void ep_wait_arrivals_kernel(const uint64_t* arrive, uint64_t target, uint32_t* err) {
  if (threadIdx.x == 0) wait_at_least(arrive, target, err);
}

// ------------------------------------------------------------------ ready / combine
// ------------------------------------------------------------------ combine
struct CombineArgs {
  Peers peers;
  size_t ret_off, ready_off;
  int64_t local_cap;
  float* out;           // [T, H] FP32 holding the shared-expert rows
  const int32_t* pos;   // [T, W]
  int T, H, W, rank;
  uint64_t epoch;
  uint32_t* err;
};

__global__ void __launch_bounds__(kThreads) ep_combine_kernel(CombineArgs a) {
  if ((int)threadIdx.x < a.W)
    wait_at_least(at<uint64_t>(a.peers.base[a.rank], a.ready_off) + threadIdx.x, a.epoch, a.err);
  __syncthreads();
  const int lane = threadIdx.x & 31;
  const int warps = gridDim.x * (blockDim.x >> 5);
  const int vec = a.H / 8;
  const uint4* ret = at<const uint4>(a.peers.base[a.rank], a.ret_off);
  for (int t = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); t < a.T; t += warps) {
    int64_t my_row = -1;
    if (lane < a.W) {
      const int p = a.pos[(int64_t)t * a.W + lane];
      if (p >= 0) {
        if (p < a.local_cap) my_row = (int64_t)lane * a.local_cap + p;
        else atomicOr(a.err, kErrBounds);
      }
    }
    const uint4* src[kMaxWorld];
#pragma unroll
    for (int d = 0; d < kMaxWorld; ++d) {
      const int64_t row = __shfl_sync(0xffffffffu, my_row, d & 31);
      src[d] = (d < a.W && row >= 0) ? ret + row * vec : nullptr;
    }
    float4* o = reinterpret_cast<float4*>(a.out + (int64_t)t * a.H);
    for (int v = lane; v < vec; v += 32) {
      const float4 lo = o[2 * v], hi = o[2 * v + 1];
      float acc[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
#pragma unroll
      for (int d = 0; d < kMaxWorld; ++d) {
        if (!src[d]) continue;
        // stored by another GPU this forward: read past the L1
        const uint4 q = __ldcg(src[d] + v);
        const uint32_t wd[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          acc[2 * i] += __uint_as_float(wd[i] << 16);
          acc[2 * i + 1] += __uint_as_float(wd[i] & 0xffff0000u);
        }
      }
      o[2 * v] = make_float4(acc[0], acc[1], acc[2], acc[3]);
      o[2 * v + 1] = make_float4(acc[4], acc[5], acc[6], acc[7]);
    }
  }
}

__global__ void ep_fill_kernel(int32_t* p, int64_t n, int32_t v) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n;
       i += (int64_t)gridDim.x * blockDim.x)
    p[i] = v;
}

// ------------------------------------------------------------------ NCCL (handle exchange)
// The few NCCL entry points glm5x_moe_create_ep uses, resolved at run time
// from the NCCL the process already loaded (the one that made the
// communicator), else libnccl.so.2. ncclResult_t 0 = ncclSuccess; data type
// 0 = ncclInt8.
using NcclAllGather = int (*)(const void*, void*, size_t, int, void*, cudaStream_t);
using NcclCommCount = int (*)(const void*, int*);
using NcclCommUserRank = int (*)(const void*, int*);

void* nccl_symbol(const char* name) {
  if (void* f = dlsym(RTLD_DEFAULT, name)) return f;
  static void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
  return h ? dlsym(h, name) : nullptr;
}

}  // namespace
}  // namespace glm5x

using namespace glm5x;

struct glm5x_moe_ep {
  glm5x_moe* engine = nullptr;
  int device = 0, rank = 0, world = 1, k = 8, H = 0, per = 0, mx = 0;
  int64_t local_cap = 0, recv_cap = 0;
  Layout L{};
  uint8_t* block = nullptr;  // this rank's exported block
  Peers peers{};
  bool connected = false;
  uint64_t epoch = 0;
  // local (not exported) buffers
  int32_t* ids = nullptr;     // [local_cap, k] routes of the local tokens
  float* wts = nullptr;
  int32_t* pos = nullptr;     // [local_cap, W]
  int32_t* small = nullptr;   // send_count [W], send_off [W], recv_count [1], recv_off [W]
  unsigned long long* done = nullptr;  // finished dispatch blocks, all forwards
  unsigned long long done_total = 0;
  unsigned long long* rdone = nullptr;  // finished return blocks, all forwards
  unsigned long long rdone_total = 0;
  uint32_t* err = nullptr;
  cudaStream_t stream = nullptr;
  std::string error;
  // stage timing (glm5x_moe_ep_set_profiling): one set of events per profiled
  // forward, read and released by glm5x_moe_ep_stage_times
  bool profiling = false;
  std::vector<std::vector<cudaEvent_t>> pending;
  double stage_ms[GLM5X_EP_STAGES]{};
  int profiled = 0;
};

namespace {

glm5x_status ep_fail(glm5x_moe_ep* ep, glm5x_status st, const std::string& msg) {
  if (ep) ep->error = msg;
  set_last_error(msg.c_str());
  return st;
}

size_t align_up(size_t v) { return (v + 255) / 256 * 256; }

Layout make_layout(int64_t local_cap, int64_t recv_cap, int H, int k, int W) {
  Layout L{};
  size_t off = 0;
  const int64_t rows = local_cap + recv_cap;
  for (int p = 0; p < 2; ++p) {
    L.rows[p] = off; off = align_up(off + (size_t)rows * H * 2);
    L.ids[p] = off; off = align_up(off + (size_t)rows * k * 4);
    L.wts[p] = off; off = align_up(off + (size_t)rows * k * 4);
    L.amax[p] = off; off = align_up(off + (size_t)rows * 4);
    L.ret[p] = off; off = align_up(off + (size_t)W * local_cap * H * 2);
    L.counts[p] = off; off = align_up(off + (size_t)W * W * 4);
    L.cnt_flag[p] = off; off = align_up(off + (size_t)W * 8);
    L.ready[p] = off; off = align_up(off + (size_t)W * 8);
  }
  L.arrive = off; off = align_up(off + 8);
  L.total = off;
  return L;
}

}  // namespace

extern "C" {

glm5x_status glm5x_moe_ep_create(const glm5x_moe_config* cfg, int device, int32_t rank,
                                 int32_t world, int64_t max_local_tokens, glm5x_moe_ep** out) {
  if (!cfg || !out) return ep_fail(nullptr, GLM5X_INVALID_STATE, "ep create: null argument");
  *out = nullptr;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world)
    return ep_fail(nullptr, GLM5X_INVALID_EXTENT, "ep create: need 0 <= rank < world <= 16");
  if (cfg->num_experts <= 0 || cfg->num_experts % world)
    return ep_fail(nullptr, GLM5X_INVALID_EXTENT, "ep create: num_experts not divisible by world");
  if (max_local_tokens <= 0 || max_local_tokens * (world + 1) > (1 << 20))
    return ep_fail(nullptr, GLM5X_INVALID_EXTENT, "ep create: max_local_tokens out of range");
  if (!cfg->has_shared)
    return ep_fail(nullptr, GLM5X_INVALID_STATE, "ep create: the layer needs its shared expert");
  if (cfg->hidden % 8 || cfg->top_k > 32)
    return ep_fail(nullptr, GLM5X_INVALID_EXTENT, "ep create: hidden % 8 or top_k > 32");
  auto* ep = new glm5x_moe_ep();
  ep->device = device;
  ep->rank = rank;
  ep->world = world;
  ep->k = cfg->top_k;
  ep->H = cfg->hidden;
  ep->per = cfg->num_experts / world;
  ep->mx = cfg->precision == GLM5X_PRECISION_MXFP4;
  ep->local_cap = max_local_tokens;
  ep->recv_cap = max_local_tokens * world;  // each source sends a token at most once
  glm5x_moe_config c = *cfg;
  c.expert_begin = rank * ep->per;
  c.expert_count = ep->per;
  c.max_tokens = (int32_t)(ep->local_cap + ep->recv_cap);
  glm5x_status st = glm5x_moe_create(&c, device, &ep->engine);
  if (st != GLM5X_OK) {
    const std::string msg = glm5x_last_error_message();
    delete ep;
    return ep_fail(nullptr, st, "ep create: " + msg);
  }
  cudaSetDevice(device);
  ep->L = make_layout(ep->local_cap, ep->recv_cap, ep->H, ep->k, world);
  const size_t W = world;
  bool ok = cudaMalloc(&ep->block, ep->L.total) == cudaSuccess &&
            cudaMalloc(&ep->ids, (size_t)ep->local_cap * ep->k * 4) == cudaSuccess &&
            cudaMalloc(&ep->wts, (size_t)ep->local_cap * ep->k * 4) == cudaSuccess &&
            cudaMalloc(&ep->pos, (size_t)ep->local_cap * W * 4) == cudaSuccess &&
            cudaMalloc(&ep->small, (3 * W + 1) * 4) == cudaSuccess &&
            cudaMalloc(&ep->rdone, 8) == cudaSuccess &&
            cudaMalloc(&ep->err, 4) == cudaSuccess &&
            cudaMalloc(&ep->done, 8) == cudaSuccess &&
            cudaStreamCreateWithFlags(&ep->stream, cudaStreamNonBlocking) == cudaSuccess;
  if (ok)
    ok = cudaMemsetAsync(ep->block, 0, ep->L.total, ep->stream) == cudaSuccess &&
         cudaMemsetAsync(ep->err, 0, 4, ep->stream) == cudaSuccess &&
         cudaMemsetAsync(ep->done, 0, 8, ep->stream) == cudaSuccess &&
         cudaMemsetAsync(ep->rdone, 0, 8, ep->stream) == cudaSuccess;
  if (ok) {
    // every id slot starts as -1: local rows never carry routed slots, and
    // received rows get theirs from their senders
    const int64_t n = (ep->local_cap + ep->recv_cap) * ep->k;
    for (int p = 0; p < 2; ++p)
      ep_fill_kernel<<<1184, 256, 0, ep->stream>>>(at<int32_t>(ep->block, ep->L.ids[p]), n, -1);
    ok = cudaGetLastError() == cudaSuccess && cudaStreamSynchronize(ep->stream) == cudaSuccess;
  }
  if (!ok) {
    glm5x_moe_ep_destroy(ep);
    return ep_fail(nullptr, GLM5X_OUT_OF_MEMORY, "ep create: device allocation failed");
  }
  ep->peers.base[rank] = ep->block;
  *out = ep;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_handle(glm5x_moe_ep* ep, void* handle) {
  if (!ep || !handle) return ep_fail(ep, GLM5X_INVALID_STATE, "ep handle: null argument");
  cudaSetDevice(ep->device);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, ep->block);
  if (e != cudaSuccess)
    return ep_fail(ep, GLM5X_DEVICE_ERROR, std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  static_assert(sizeof(h) == GLM5X_EP_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof h);
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_connect(glm5x_moe_ep* ep, const void* handles) {
  if (!ep || !handles) return ep_fail(ep, GLM5X_INVALID_STATE, "ep connect: null argument");
  if (ep->connected) return ep_fail(ep, GLM5X_INVALID_STATE, "ep connect: already connected");
  cudaSetDevice(ep->device);
  for (int s = 0; s < ep->world; ++s) {
    if (s == ep->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, static_cast<const uint8_t*>(handles) + (size_t)s * GLM5X_EP_HANDLE_BYTES,
                sizeof h);
    void* p = nullptr;
    const cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int q = 0; q < s; ++q)
        if (q != ep->rank && ep->peers.base[q]) {
          cudaIpcCloseMemHandle(ep->peers.base[q]);
          ep->peers.base[q] = nullptr;
        }
      return ep_fail(ep, GLM5X_BACKEND_UNAVAILABLE,
                     std::string("cudaIpcOpenMemHandle (peer ") + std::to_string(s) +
                         "): " + cudaGetErrorString(e));
    }
    ep->peers.base[s] = static_cast<uint8_t*>(p);
  }
  ep->connected = true;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_create_ep(const glm5x_moe_config* cfg, int device, void* nccl_comm,
                                 int32_t rank, int32_t world, int64_t max_local_tokens,
                                 glm5x_moe_ep** out) {
  if (!nccl_comm || !out) return ep_fail(nullptr, GLM5X_INVALID_STATE, "create_ep: null argument");
  auto all_gather = reinterpret_cast<NcclAllGather>(nccl_symbol("ncclAllGather"));
  auto comm_count = reinterpret_cast<NcclCommCount>(nccl_symbol("ncclCommCount"));
  auto user_rank = reinterpret_cast<NcclCommUserRank>(nccl_symbol("ncclCommUserRank"));
  if (!all_gather || !comm_count || !user_rank)
    return ep_fail(nullptr, GLM5X_BACKEND_UNAVAILABLE, "create_ep: NCCL is not loaded");
  int n = 0, r = -1;
  if (comm_count(nccl_comm, &n) != 0 || user_rank(nccl_comm, &r) != 0 || n != world || r != rank)
    return ep_fail(nullptr, GLM5X_INVALID_STATE, "create_ep: rank / world differ from the communicator's");
  glm5x_status st = glm5x_moe_ep_create(cfg, device, rank, world, max_local_tokens, out);
  if (st != GLM5X_OK) return st;
  glm5x_moe_ep* ep = *out;
  uint8_t* dev = nullptr;
  std::vector<uint8_t> all((size_t)world * GLM5X_EP_HANDLE_BYTES);
  st = glm5x_moe_ep_handle(ep, all.data() + (size_t)rank * GLM5X_EP_HANDLE_BYTES);
  bool ok = st == GLM5X_OK &&
            cudaMalloc(&dev, all.size()) == cudaSuccess &&
            cudaMemcpy(dev + (size_t)rank * GLM5X_EP_HANDLE_BYTES,
                       all.data() + (size_t)rank * GLM5X_EP_HANDLE_BYTES, GLM5X_EP_HANDLE_BYTES,
                       cudaMemcpyHostToDevice) == cudaSuccess &&
            all_gather(dev + (size_t)rank * GLM5X_EP_HANDLE_BYTES, dev, GLM5X_EP_HANDLE_BYTES,
                       /*ncclInt8*/ 0, nccl_comm, ep->stream) == 0 &&
            cudaStreamSynchronize(ep->stream) == cudaSuccess &&
            cudaMemcpy(all.data(), dev, all.size(), cudaMemcpyDeviceToHost) == cudaSuccess;
  if (dev) cudaFree(dev);
  if (ok) st = glm5x_moe_ep_connect(ep, all.data());
  if (!ok || st != GLM5X_OK) {
    const std::string msg = ok ? ep->error : std::string("create_ep: IPC handle exchange failed");
    glm5x_moe_ep_destroy(ep);
    *out = nullptr;
    return ep_fail(nullptr, ok ? st : GLM5X_BACKEND_UNAVAILABLE, msg);
  }
  return GLM5X_OK;
}

glm5x_moe* glm5x_moe_ep_engine(glm5x_moe_ep* ep) { return ep ? ep->engine : nullptr; }

const char* glm5x_moe_ep_error_message(const glm5x_moe_ep* ep) {
  return ep ? ep->error.c_str() : "";
}

glm5x_status glm5x_moe_ep_forward(glm5x_moe_ep* ep, const void* hidden_bf16, int64_t tokens,
                                  float* out, void* stream) {
  if (!ep || (tokens > 0 && (!hidden_bf16 || !out)))
    return ep_fail(ep, GLM5X_INVALID_STATE, "ep forward: null argument");
  if (!ep->connected) return ep_fail(ep, GLM5X_INVALID_STATE, "ep forward: not connected");
  if (tokens < 0 || tokens > ep->local_cap)
    return ep_fail(ep, GLM5X_INVALID_EXTENT, "ep forward: tokens outside [0, max_local_tokens]");
  if (tokens > 0 && reinterpret_cast<uintptr_t>(hidden_bf16) % 16)
    return ep_fail(ep, GLM5X_INVALID_EXTENT, "ep forward: hidden must be 16-byte aligned");
  cudaSetDevice(ep->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ep->stream;
  const int T = static_cast<int>(tokens), W = ep->world, p = static_cast<int>(++ep->epoch & 1);
  const uint64_t epoch = ep->epoch;
  int32_t* send_count = ep->small;
  int32_t* send_off = ep->small + W;
  int32_t* recv_count = ep->small + 2 * W;
  int32_t* recv_off = ep->small + 2 * W + 1;
  auto cuda_fail = [&](const char* what) {
    return ep_fail(ep, GLM5X_DEVICE_ERROR, std::string("ep forward: ") + what + ": " +
                                               cudaGetErrorString(cudaGetLastError()));
  };
  std::vector<cudaEvent_t> evs;
  auto mark = [&]() {
    if (!ep->profiling) return;
    cudaEvent_t e;
    if (cudaEventCreate(&e) == cudaSuccess) {
      cudaEventRecord(e, st);
      evs.push_back(e);
    }
  };
  mark();
  // route
  if (T > 0) {
    const glm5x_status rs = glm5x_moe_route(ep->engine, hidden_bf16, T, ep->ids, ep->wts, nullptr, st);
    if (rs != GLM5X_OK) return ep_fail(ep, rs, glm5x_moe_error_message(ep->engine));
  }
  mark();
  // plan
  ep_plan_kernel<<<W, 1024, 0, st>>>(ep->ids, T, ep->k, ep->per, W, ep->pos, send_count);
  if (cudaGetLastError() != cudaSuccess) return cuda_fail("plan");
  // exchange counts
  ExchangeArgs xa{};
  xa.peers = ep->peers;
  xa.counts_off = ep->L.counts[p];
  xa.flag_off = ep->L.cnt_flag[p];
  xa.rank = ep->rank;
  xa.W = W;
  xa.epoch = epoch;
  xa.recv_cap = ep->recv_cap;
  xa.send_count = send_count;
  xa.recv_count = recv_count;
  xa.send_off = send_off;
  xa.recv_off = recv_off;
  xa.err = ep->err;
  ep_exchange_kernel<<<1, 64, 0, st>>>(xa);
  ep_clear_tail_kernel<<<592, 256, 0, st>>>(at<int32_t>(ep->block, ep->L.ids[p]),
                                            at<float>(ep->block, ep->L.wts[p]), ep->local_cap,
                                            ep->recv_cap, ep->k, recv_count);
  if (cudaGetLastError() != cudaSuccess) return cuda_fail("exchange");
  mark();
  // dispatch
  DispatchArgs da{};
  da.peers = ep->peers;
  da.rows_off = ep->L.rows[p];
  da.ids_off = ep->L.ids[p];
  da.wts_off = ep->L.wts[p];
  da.amax_off = ep->L.amax[p];
  da.arrive_off = ep->L.arrive;
  da.x = static_cast<const uint16_t*>(hidden_bf16);
  da.ids = ep->ids;
  da.w = ep->wts;
  da.pos = ep->pos;
  da.send_off = send_off;
  da.T = T;
  da.H = ep->H;
  da.k = ep->k;
  da.W = W;
  da.per = ep->per;
  da.rank = ep->rank;
  da.local_cap = ep->local_cap;
  da.recv_cap = ep->recv_cap;
  da.err = ep->err;
  // one warp per token: as many blocks as the tokens need, at most kGrid
  const int grid = std::max(1, std::min(kGrid, (T + kThreads / 32 - 1) / (kThreads / 32)));
  ep->done_total += (unsigned long long)grid;
  da.done = ep->done;
  da.done_target = ep->done_total;
  ep_dispatch_kernel<<<grid, kThreads, 0, st>>>(da);
  // one arrival per source rank and forward
  ep_wait_arrivals_kernel<<<1, 32, 0, st>>>(at<uint64_t>(ep->block, ep->L.arrive),
                                            epoch * (uint64_t)W, ep->err);
  if (cudaGetLastError() != cudaSuccess) return cuda_fail("dispatch");
  mark();
  // experts over [local tokens | received rows]; each received row's sum goes
  // back into its source's return area, and the sources' ready flags rise
  RowReturn rr{};
  for (int s = 0; s < W; ++s) {
    rr.base[s] = at<uint16_t>(ep->peers.base[s], ep->L.ret[p]) +
                 (size_t)ep->rank * ep->local_cap * ep->H;
    rr.flag[s] = at<uint64_t>(ep->peers.base[s], ep->L.ready[p]) + ep->rank;
  }
  rr.recv_off = recv_off;
  rr.W = W;
  rr.limit = ep->local_cap;
  rr.epoch = epoch;
  rr.grid = (int)std::max<int64_t>(1, std::min<int64_t>(592, ep->recv_cap));
  ep->rdone_total += (unsigned long long)rr.grid;
  rr.done = ep->rdone;
  rr.done_target = ep->rdone_total;
  rr.err = ep->err;
  const glm5x_status es = engine_forward_peer_rows(
      ep->engine, at<uint16_t>(ep->block, ep->L.rows[p]), ep->local_cap, T, ep->recv_cap,
      at<int32_t>(ep->block, ep->L.ids[p]), at<float>(ep->block, ep->L.wts[p]),
      ep->mx ? nullptr : at<float>(ep->block, ep->L.amax[p]), recv_count, out, &rr, st);
  if (es != GLM5X_OK) return ep_fail(ep, es, glm5x_moe_error_message(ep->engine));
  mark();
  // the partial sums, returned into this rank's memory
  CombineArgs ca{};
  ca.peers = ep->peers;
  ca.ret_off = ep->L.ret[p];
  ca.local_cap = ep->local_cap;
  ca.ready_off = ep->L.ready[p];
  ca.out = out;
  ca.pos = ep->pos;
  ca.T = T;
  ca.H = ep->H;
  ca.W = W;
  ca.rank = ep->rank;
  ca.epoch = epoch;
  ca.err = ep->err;
  ep_combine_kernel<<<grid, kThreads, 0, st>>>(ca);
  if (cudaGetLastError() != cudaSuccess) return cuda_fail("combine");
  mark();
  if (ep->profiling && evs.size() == GLM5X_EP_STAGES + 1) ep->pending.push_back(std::move(evs));
  else
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_set_profiling(glm5x_moe_ep* ep, int32_t enable) {
  if (!ep) return ep_fail(nullptr, GLM5X_INVALID_STATE, "ep profiling: null argument");
  ep->profiling = enable != 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_stage_times(glm5x_moe_ep* ep, float* ms, int32_t* forwards) {
  if (!ep || !ms || !forwards)
    return ep_fail(ep, GLM5X_INVALID_STATE, "ep stage times: null argument");
  cudaSetDevice(ep->device);
  for (auto& evs : ep->pending) {
    cudaEventSynchronize(evs.back());
    for (int i = 0; i < GLM5X_EP_STAGES; ++i) {
      float t = 0.0f;
      if (cudaEventElapsedTime(&t, evs[i], evs[i + 1]) == cudaSuccess) ep->stage_ms[i] += t;
    }
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
    ep->profiled++;
  }
  ep->pending.clear();
  for (int i = 0; i < GLM5X_EP_STAGES; ++i) {
    ms[i] = static_cast<float>(ep->stage_ms[i]);
    ep->stage_ms[i] = 0.0;
  }
  *forwards = ep->profiled;
  ep->profiled = 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_last_counts(glm5x_moe_ep* ep, int64_t* sent, int64_t* received) {
  if (!ep || !sent || !received)
    return ep_fail(ep, GLM5X_INVALID_STATE, "ep counts: null argument");
  cudaSetDevice(ep->device);
  std::vector<int32_t> h(2 * ep->world + 1);
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(h.data(), ep->small, h.size() * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return ep_fail(ep, GLM5X_DEVICE_ERROR, "ep counts: device error");
  for (int d = 0; d < ep->world; ++d) sent[d] = h[d];
  *received = h[2 * ep->world];
  return GLM5X_OK;
}

glm5x_status glm5x_moe_ep_check(glm5x_moe_ep* ep) {
  if (!ep) return ep_fail(nullptr, GLM5X_INVALID_STATE, "ep check: null argument");
  cudaSetDevice(ep->device);
  const glm5x_status es = glm5x_moe_check(ep->engine);
  if (es != GLM5X_OK) return ep_fail(ep, es, glm5x_moe_error_message(ep->engine));
  uint32_t w = 0;
  if (cudaDeviceSynchronize() != cudaSuccess ||
      cudaMemcpy(&w, ep->err, 4, cudaMemcpyDeviceToHost) != cudaSuccess)
    return ep_fail(ep, GLM5X_DEVICE_ERROR, "ep check: device error");
  cudaMemset(ep->err, 0, 4);
  if (w & kErrWaitTimeout)
    return ep_fail(ep, GLM5X_WAIT_TIMEOUT, "ep: a peer did not answer within the wait budget");
  if (w) return ep_fail(ep, GLM5X_INVALID_EXTENT, "ep: receive area overflow (0x" + std::to_string(w) + ")");
  return GLM5X_OK;
}

void glm5x_moe_ep_destroy(glm5x_moe_ep* ep) {
  if (!ep) return;
  cudaSetDevice(ep->device);
  cudaDeviceSynchronize();
  for (int s = 0; s < ep->world; ++s)
    if (s != ep->rank && ep->peers.base[s]) cudaIpcCloseMemHandle(ep->peers.base[s]);
  for (void* q : {static_cast<void*>(ep->block), static_cast<void*>(ep->ids),
                  static_cast<void*>(ep->wts), static_cast<void*>(ep->pos),
                  static_cast<void*>(ep->small), static_cast<void*>(ep->err),
                  static_cast<void*>(ep->done), static_cast<void*>(ep->rdone)})
    if (q) cudaFree(q);
  for (auto& evs : ep->pending)
    for (cudaEvent_t e : evs) cudaEventDestroy(e);
  if (ep->stream) cudaStreamDestroy(ep->stream);
  if (ep->engine) glm5x_moe_destroy(ep->engine);
  delete ep;
}

}  // extern "C"
