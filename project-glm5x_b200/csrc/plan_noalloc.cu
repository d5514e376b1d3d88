// plan_noalloc.cu -- the expert-major plan without any device allocation.
//
// glm5x_expert_major_plan() allocates its scratch (per-chunk counts, ranks,
// prefix sums) with cudaMalloc and releases it with cudaFree on every call.
// Some callers cannot do that: a host framework whose caching allocator owns
// all device memory and forbids raw allocations, a process running close to
// its memory cap, or a serving loop that cannot afford cudaFree's implicit
// device-wide synchronization (it stalls every other stream on the GPU).
// glm5x_expert_major_plan_noalloc() computes the same plan with its scratch
// in a file-scope __device__ array of fixed size instead.
//
// Limits: tokens <= kNoAllocMaxTokens, tokens * top_k <= kNoAllocMaxSlots,
// num_experts <= 256. The array (about 1 MB) is resident on every GPU that
// loads this library until the process exits.
//
// Sharing: every call on a device uses the same array and leaves its
// contents behind. Counts, ranks and prefix sums are written earlier in the
// same call before they are read; the device error word and the routing
// weight / token amax inputs the permutation kernels also read are cleared at
// the start of every call. Calls whose GPU work overlaps (on two
// streams, or from two host threads) race on the array and must be
// serialized by the caller.
//
// Set-up: the first call on each device looks up the array's device address
// with cudaGetSymbolAddress while that device is current; host code must
// never hand the array's name itself to a kernel (on the host it names a
// host-side stand-in, not device memory). Make that first call on a device
// before capturing any stream on it.
#include <cuda_runtime.h>

#include <cstdint>
#include <cstdio>
#include <mutex>

#include "../../include/glm5x_moe.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"

namespace glm5x {
namespace {

constexpr int kNoAllocMaxTokens = 8192;
constexpr int kNoAllocMaxSlots = 65536;  // tokens * top_k
constexpr int kNoAllocMaxExperts = 256;
constexpr int kChunkTokens = 256;        // tokens per counting chunk (route.cu)

// scratch layout in 4-byte words
constexpr size_t kChunkCountWords =
    (size_t)(kNoAllocMaxTokens / kChunkTokens) * kNoAllocMaxExperts;  // 32 x 256
constexpr size_t kRankWords = kNoAllocMaxSlots;
constexpr size_t kPrefixWords = kNoAllocMaxExperts + 1;
constexpr size_t kOffChunk = 0;
constexpr size_t kOffRank = kOffChunk + kChunkCountWords;
constexpr size_t kOffQPrefix = kOffRank + kRankWords;
constexpr size_t kOffNtPrefix = kOffQPrefix + kPrefixWords;
constexpr size_t kOffSegAmax = kOffNtPrefix + kPrefixWords;
constexpr size_t kOffHAmax = kOffSegAmax + kNoAllocMaxExperts;
// inputs and outputs the shared permutation kernels use that a plan does not
// need: routing weights [slots], token amax [tokens], row weights [rows]
constexpr size_t kOffWeights = kOffHAmax + kNoAllocMaxExperts;
constexpr size_t kOffTokAmax = kOffWeights + kNoAllocMaxSlots;
constexpr size_t kOffRowWeight = kOffTokAmax + kNoAllocMaxTokens;
constexpr size_t kRowWeightWords = kNoAllocMaxSlots + (size_t)kNoAllocMaxExperts * 128;
constexpr size_t kOffErr = kOffRowWeight + kRowWeightWords;
constexpr size_t kScratchWords = kOffErr + 64;

__device__ __align__(256) uint32_t g_plan_scratch[kScratchWords];

constexpr int kMaxDevices = 64;
uint32_t* g_scratch_ptr[kMaxDevices] = {};
std::mutex g_scratch_mutex;

// Device address of g_plan_scratch on the current device (looked up once).
cudaError_t scratch_for_current_device(uint32_t** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(g_scratch_mutex);
  if (!g_scratch_ptr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_plan_scratch);
    if (e != cudaSuccess) return e;
    g_scratch_ptr[dev] = static_cast<uint32_t*>(p);
  }
  *out = g_scratch_ptr[dev];
  return cudaSuccess;
}

}  // namespace
}  // namespace glm5x

using namespace glm5x;

extern "C" glm5x_status glm5x_expert_major_plan_noalloc(const int32_t* ids, int64_t T, int32_t k,
                                                        int32_t E, int32_t* seg_count,
                                                        int32_t* seg_start, int32_t* pos,
                                                        int32_t* row_token, void* stream) {
  if (!ids || !seg_count || !seg_start || !pos || !row_token || T <= 0 || k <= 0 || k > 16 ||
      E <= 0 || E > kNoAllocMaxExperts) {
    set_last_error("expert_major_plan_noalloc: invalid plan dimensions or null pointer");
    return GLM5X_INVALID_EXTENT;
  }
  if (T > kNoAllocMaxTokens || T * k > kNoAllocMaxSlots) {
    set_last_error("expert_major_plan_noalloc: plan exceeds the fixed scratch (tokens <= 8192, "
                   "tokens * top_k <= 65536); use glm5x_expert_major_plan");
    return GLM5X_INVALID_EXTENT;
  }
  uint32_t* scratch = nullptr;
  if (scratch_for_current_device(&scratch) != cudaSuccess) {
    set_last_error("expert_major_plan_noalloc: cudaGetSymbolAddress failed");
    return GLM5X_DEVICE_ERROR;
  }
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  PermuteBuffers b{};
  b.chunk_count = reinterpret_cast<int32_t*>(scratch + kOffChunk);
  b.rank = reinterpret_cast<int32_t*>(scratch + kOffRank);
  b.qprefix = reinterpret_cast<int32_t*>(scratch + kOffQPrefix);
  b.ntile_prefix = reinterpret_cast<int32_t*>(scratch + kOffNtPrefix);
  b.seg_amax = reinterpret_cast<float*>(scratch + kOffSegAmax);
  b.h_amax = reinterpret_cast<float*>(scratch + kOffHAmax);
  b.seg_count = seg_count;
  b.seg_start = seg_start;
  b.pos = pos;
  b.row_token = row_token;
  b.row_weight = reinterpret_cast<float*>(scratch + kOffRowWeight);
  const float* weights = reinterpret_cast<const float*>(scratch + kOffWeights);
  const float* tok_amax = reinterpret_cast<const float*>(scratch + kOffTokAmax);
  uint32_t* err = scratch + kOffErr;
  // weights and token amax are read but do not affect the plan; clear them
  // (with the error word) so no call reads what an earlier call left behind
  auto device_fail = [](const char* step, cudaError_t e) {
    char buf[256];
    std::snprintf(buf, sizeof buf, "expert_major_plan_noalloc: %s: %s", step,
                  cudaGetErrorString(e));
    set_last_error(buf);
    return GLM5X_DEVICE_ERROR;
  };
  cudaError_t e = cudaMemsetAsync(scratch + kOffWeights, 0, sizeof(uint32_t) * (size_t)T * k, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(scratch + kOffTokAmax, 0, sizeof(uint32_t) * (size_t)T, st);
  if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, sizeof(uint32_t), st);
  if (e != cudaSuccess) return device_fail("clearing the scratch", e);
  e = launch_permute(ids, weights, tok_amax, (int)T, k, E, 0, 256, b, err, st);
  if (e != cudaSuccess) return device_fail("permutation launch", e);
  uint32_t word = 0;
  e = cudaMemcpyAsync(&word, err, sizeof word, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return device_fail("reading the error word", e);
  if (word) {
    set_last_error("expert_major_plan_noalloc: expert id out of range or repeated in a token");
    return GLM5X_INVALID_EXTENT;
  }
  return GLM5X_OK;
}
