// speculative.cu -- greedy verification of speculative draft blocks for many
// sequences at once: the caller side of the expert-major MTP pattern, where
// each sequence's [anchor, draft_1 .. draft_n] block runs through the target
// as one expert-major batch and the target's argmax tokens decide how much of
// the draft is committed (verify_greedy_target_block,
// runtime/src/speculative.cpp:75-113, called from runtime/src/model.cpp:
// 1640-1690). One thread per sequence; the per-sequence result and status are
// the reference's (INVALID_EXTENT for a bad proposal, INVALID_STATE for a
// target token outside the vocabulary).
#include <cstdint>

#include "glm5x_kernels.cuh"

namespace glm5x {

__global__ void verify_greedy_blocks_kernel(const uint32_t* __restrict__ anchors,
                                            const uint32_t* __restrict__ candidates,
                                            const int32_t* __restrict__ draft_counts,
                                            const uint32_t* __restrict__ targets, int64_t S,
                                            int max_draft, uint32_t vocab,
                                            int32_t* __restrict__ accepted,
                                            uint32_t* __restrict__ committed,
                                            int32_t* __restrict__ status) {
  const int64_t s = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (s >= S) return;
  const int n = draft_counts[s];
  const uint32_t* cand = candidates + s * max_draft;
  const uint32_t* tgt = targets + s * (int64_t)(max_draft + 1);
  uint32_t* out = committed + s * (int64_t)(max_draft + 1);
  accepted[s] = 0;
  // validate_proposal (speculative.cpp:8-21), then the target block's tokens
  bool bad_extent = anchors[s] >= vocab || n < 0 || n > max_draft;
  for (int i = 0; i < n && !bad_extent; ++i) bad_extent = cand[i] >= vocab;
  if (bad_extent) {
    status[s] = 9;  // INVALID_EXTENT
    return;
  }
  for (int i = 0; i <= n; ++i)
    if (tgt[i] >= vocab) {
      status[s] = 16;  // INVALID_STATE
      return;
    }
  int a = 0;
  while (a < n && cand[a] == tgt[a]) {
    out[a] = cand[a];
    ++a;
  }
  out[a] = tgt[a];  // the first mismatching target token, or the bonus token
  accepted[s] = a;
  status[s] = 0;
}

cudaError_t launch_verify_greedy_blocks(const uint32_t* anchors, const uint32_t* candidates,
                                        const int32_t* draft_counts, const uint32_t* targets,
                                        int64_t S, int max_draft, uint32_t vocab,
                                        int32_t* accepted, uint32_t* committed, int32_t* status,
                                        cudaStream_t st) {
  if (S <= 0) return cudaSuccess;
  verify_greedy_blocks_kernel<<<(unsigned)((S + 255) / 256), 256, 0, st>>>(
      anchors, candidates, draft_counts, targets, S, max_draft, vocab, accepted, committed,
      status);
  return cudaGetLastError();
}

}  // namespace glm5x
