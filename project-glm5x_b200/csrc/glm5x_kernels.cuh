// glm5x_kernels.cuh -- launcher declarations shared by the kernels and the
// host engine.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace glm5x {

// Sets the message glm5x_last_error_message() returns on this thread.
void set_last_error(const char* msg);

// ------------------------------------------------------------ segment layout
// Expert segments start on 128-row boundaries. With a token tile bn >= 128,
// logical row q of a segment is physical row q. With bn < 128 every bn-row
// tile owns a whole 128-row block (rows past bn unused), so that each tile's
// activation scales start a 128-row scale block, which is where the
// block-scaled MMA reads them (its scale-factor TMEM address must stay
// 4-column aligned, so a tile cannot start inside a block).
__host__ __device__ __forceinline__ int segment_row(int q, int bn) {
  return bn < 128 ? (q / bn) * 128 + q % bn : q;
}
__host__ __device__ __forceinline__ int segment_rows(int count, int bn) {
  return bn < 128 ? (count + bn - 1) / bn * 128 : (count + 127) / 128 * 128;
}

// ------------------------------------------------------------ quant.cu
cudaError_t launch_row_amax_bf16(const uint16_t* src, int64_t rows, int cols, float* out,
                                 uint32_t* err, cudaStream_t st);
template <typename T>
cudaError_t launch_nvfp4_quantize_matrix(const T* src, int64_t rows, int64_t cols, int mse,
                                         float* amax_scratch, uint8_t* packed,
                                         uint8_t* scales_blocked, float* global_out,
                                         uint32_t* err, cudaStream_t st);
cudaError_t launch_nvfp4_quantize_segments(const uint16_t* src, int K, const int32_t* row_token,
                                           const int32_t* seg_start, const int32_t* seg_count,
                                           const int32_t* qprefix, int nseg, int bn,
                                           const float* seg_amax, int64_t max_rows,
                                           uint8_t* packed, uint8_t* scales_blocked,
                                           float* seg_global, cudaStream_t st,
                                           int first_seg = 0);
// Expert-parallel FP4 dispatch: the sender's quantization of (token, expert)
// rows with the reduced slab scale of each row's expert (row-major E4M3
// scales), and the receiver's placement of such rows into the routed
// segments [0, nseg_routed) (blocked scales, padded rows zeroed, each
// segment's global scale from amax[expert_begin + s]).
cudaError_t launch_nvfp4_quantize_rows(const uint16_t* src, int K, const int32_t* row_token,
                                       const int32_t* row_expert, int64_t n, const float* amax,
                                       uint8_t* packed, uint8_t* scales, cudaStream_t st);
cudaError_t launch_place_nvfp4_rows(const uint8_t* packed_in, const uint8_t* scales_in, int K,
                                    const int32_t* row_token, int row_base,
                                    const int32_t* seg_start, const int32_t* seg_count,
                                    const int32_t* qprefix, int nseg_routed, int bn,
                                    const float* amax, int expert_begin, int64_t max_rows,
                                    uint8_t* packed, uint8_t* scales_blocked, float* seg_global,
                                    cudaStream_t st);
// Four-term MXFP4 expansion of expert-major rows (4 operand rows per token);
// records kErrNonFinite in *err for Inf / NaN inputs.
cudaError_t launch_mxfp4_terms_segments(const uint16_t* src, int K, const int32_t* row_token,
                                        const int32_t* seg_start, const int32_t* seg_count,
                                        const int32_t* qprefix, int nseg, int bn,
                                        int64_t max_slots, uint8_t* packed,
                                        uint8_t* scales_blocked, uint32_t* err, cudaStream_t st);
cudaError_t launch_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales_blocked,
                                    float g, int64_t rows, int64_t cols, float* out,
                                    cudaStream_t st);
cudaError_t launch_mxfp4_decode(const uint8_t* packed, const uint8_t* scales, int64_t n,
                                int group, float* out, uint32_t* err, cudaStream_t st);
template <typename T>
cudaError_t launch_mxfp4_encode(const T* src, int64_t n, int group, int mse, uint8_t* packed,
                                uint8_t* scales, uint32_t* err, cudaStream_t st);

// ------------------------------------------------------------ route.cu
struct PermuteBuffers {
  int32_t* chunk_count;   // [ceil(T/256), E]
  int32_t* rank;          // [T, k]
  int32_t* seg_count;     // [nseg]
  int32_t* seg_start;     // [nseg + 1], 128-aligned starts
  int32_t* qprefix;       // [nseg + 1], prefix of counts rounded up to 8
  int32_t* ntile_prefix;  // [nseg + 1], prefix of N-tile counts
  float* seg_amax;        // [nseg], max |x| of each segment's input rows
  float* h_amax;          // [nseg], max |h| of each segment's SwiGLU output
  int32_t* pos;           // [T, k + has_shared], row of each (token, slot)
  int32_t* row_token;     // [rows], token of each segment row
  float* row_weight;      // [rows], routing weight of each segment row
};

// Expert-parallel FP4 dispatch: per-expert slab amax from token amax and
// global ids [T, k] (amax [E] zeroed here), and the expert-major rows of
// received rows listed per group (see route.cu).
cudaError_t launch_slab_amax(const float* token_amax, const int32_t* ids, int T, int k, int E,
                             float* amax, cudaStream_t st);
cudaError_t launch_map_group_pos(const int32_t* group_rows, int64_t n, const int32_t* pos,
                                 int kk, int row_base, int32_t* out, cudaStream_t st);

// Top-K policy of k3x::select_routing (runtime/include/k3x/routing_policy.hpp:
// 11-19): mode 0 natural, 1 fixed (fixed_k of the ladder 4/6/8/12/16), 2
// adaptive (natural Top-16; the smallest ladder K meeting the mass, entropy
// support and boundary-gap tests), quality_floor_k raising fixed/adaptive K.
struct RoutingPolicy {
  int32_t mode = 0;
  int32_t fixed_k = 0;
  float mass_target = 0.9f;
  float minimum_boundary_gap = 0.0f;
  int32_t quality_floor_k = 0;
};

// One warp per token: sigmoid scores (or given scores), natural top-k by
// score + bias, the policy's selected K <= k. Slots past the selected K get id
// -1 and weight 0; the selected weights are score / sum(selected scores) *
// routed_scale. Optional per-token outputs: sel [T, 2] = (selected K,
// quality-floor escalated) and diag [T, 4] = (normalized entropy, entropy
// effective support, selected cumulative mass, boundary confidence).
cudaError_t launch_topk(const float* in, int values_are_scores, const float* bias, int T, int E,
                        int k, float routed_scale, int32_t* ids, float* weights, uint32_t* err,
                        cudaStream_t st, const RoutingPolicy& policy = RoutingPolicy(),
                        int32_t* sel = nullptr, float* diag = nullptr);
// The same over the sum of nplanes planes of [T, E] values (plane p at
// in + p * T * E, added in plane order: the K-split router's partial
// logits), writing the sums to logits_out when it is given.
cudaError_t launch_topk_planes(const float* in, int nplanes, float* logits_out,
                               int values_are_scores, const float* bias, int T, int E, int k,
                               float routed_scale, int32_t* ids, float* weights, uint32_t* err,
                               cudaStream_t st, const RoutingPolicy& policy, int32_t* sel,
                               float* diag);
// rows_per: operand rows per (token, slot) -- 1 for NVFP4, 4 for the MXFP4
// four-term activation expansion (pos and row_token refer to the first).
// ids in [begin, begin + count) -> id - begin, others -> -1.
cudaError_t launch_map_local_ids(const int32_t* ids, int64_t n, int begin, int count,
                                 int32_t* out, cudaStream_t st);
cudaError_t launch_permute(const int32_t* ids, const float* weights, const float* token_amax,
                           int T, int k, int E, int has_shared, int bn, PermuteBuffers b,
                           uint32_t* err, cudaStream_t st, int rows_per = 1,
                           int skip_invalid = 0, int shared_rows = -1, int* launches = nullptr);

// ------------------------------------------------------------ speculative.cu
// verify_greedy_target_block for S sequences (one thread each): status[s] 0,
// 9 (invalid extent) or 16 (invalid state); committed[s, 0 .. accepted[s]].
cudaError_t launch_verify_greedy_blocks(const uint32_t* anchors, const uint32_t* candidates,
                                        const int32_t* draft_counts, const uint32_t* targets,
                                        int64_t S, int max_draft, uint32_t vocab,
                                        int32_t* accepted, uint32_t* committed, int32_t* status,
                                        cudaStream_t st);

// ------------------------------------------------------------ router_tc.cu
// BF16 router logits on tcgen05 + sigmoid/bias/top-k epilogue. tmap_x: hidden
// [T, H] BF16, box {64, 128}; tmap_w: router weight [E, H] BF16, box {64, E}.
// When the 128-token tiles would leave SMs idle and `partials` is given
// (router_partials_floats() floats), the contraction is split along K over
// several CTAs per tile and the partial logits are summed in a fixed order
// before the top-k (by the top-k kernel itself for up to four planes, else
// by a separate kernel first). A non-natural policy or requested sel/diag
// outputs re-run the top-k over the logits with that policy (logits must be
// given). Returns the launches issued in *launches.
bool router_tc_supported(int E, int H, int k);
size_t router_partials_floats(int num_sms, int E);
cudaError_t launch_router_tc(const CUtensorMap* tmap_x, const CUtensorMap* tmap_w,
                             const float* bias, int T, int H, int E, int k, float routed_scale,
                             float* logits, int32_t* ids, float* weights, uint32_t* err,
                             cudaStream_t st, float* partials = nullptr, int num_sms = 0,
                             int* launches = nullptr,
                             const RoutingPolicy& policy = RoutingPolicy(),
                             int32_t* sel = nullptr, float* diag = nullptr,
                             float* row_amax = nullptr);
// row_amax (optional, [T]): each token's max |x| over its row, NaN skipped
// and any Inf / NaN flagged in err (launch_row_amax_bf16's values), taken
// from the token tiles the router streams anyway.

// ------------------------------------------------------------ gemm_nvfp4.cu
// Grouped block-scaled FP4 GEMM over expert segments, weights as the M side:
//   D[m, n] = sum_k W_e[m, k] * X[row_start + n, k]  (NVFP4: E4M3 per 16)
// Epilogue 0 (gate/up): W rows interleave 16 gate and 16 up rows per 32, and
//   h = silu(gate) * up is stored as BF16 into h_out[row, M_per / 2].
// Epilogue 1 (down): y * row_weight[row] stored as BF16 into y_out[row, M_per].
struct GemmParams {
  const uint8_t* a_packed;      // stacked weights (for L2 prefetch)
  const uint8_t* b_packed;      // activation rows (for L2 prefetch)
  const uint8_t* sfa;           // blocked scales of the stacked weights
  const uint8_t* sfb;           // blocked scales of the activation rows
  const int32_t* seg_count;     // [nseg]
  const int32_t* seg_start;     // [nseg + 1]
  const int32_t* ntile_prefix;  // [nseg + 1]
  const float* a_global;        // epi 0: [2 * nseg] (gate, up); epi 1: [nseg]
  const float* b_global;        // [nseg]
  const float* row_weight;      // epi 1
  uint16_t* out;                // epi 0: h [rows, M_per/2]; epi 1: y [rows, M_per]
  float* h_amax;                // epi 0: [nseg]
  uint32_t* err;
  int K;                        // contraction length (elements)
  int M_per;                    // weight rows per expert
  int nseg;
  int tile_group;               // CTA-pair GEMM tile order: 0 = segment-major, else
                                // token tiles per weight-tile-major group
};

// tmap_b[i]: the activation rows with a box of (32 << i) rows, i = 0..2
// (32, 64, 128); a tile loads its rows in pieces of at most 128.
// mxfp4 = 1: MXFP4 operands (E8M0 scale per 32 in the blocked layout) and
// four B rows per token (residual terms), summed in the epilogue; outputs and
// routing weights live on each token's term-0 row.
// epi = 2: token-major down projection (NVFP4, segments in 128-row tiles):
// tmap_a / p.a_packed / p.sfa are the token rows (box 128), tmap_b[2] /
// p.b_packed / p.sfb the weights; output and weighting as epi 1.
// weight_rows = 256 (token tiles of 32 or 64 rows only): each tile covers
// 256 weight rows as two 128-row halves with their own MMAs and accumulators,
// so one stage hand-off moves twice the weight bytes (M_per % 256 == 0).
cudaError_t launch_nvfp4_grouped_gemm(int bn, int epi, const CUtensorMap* tmap_a,
                                      const CUtensorMap* tmap_b, const GemmParams& p,
                                      int num_sms, cudaStream_t st, int mxfp4 = 0,
                                      int weight_rows = 128);
size_t nvfp4_gemm_smem_bytes(int bn);

// ------------------------------------------------------------ gemm_nvfp4_pair.cu
// Same GEMM on CTA pairs (cta_group::2, M = 256) for token tiles of up to 256
// rows. tmap_sfa / tmap_sfb: the blocked scale arrays as [bytes/256, 256]
// uint8 tensors with a {256, 8} box (four 512-byte chunks). grid = an even
// CTA count, at most nvfp4_pair_gemm_grid().
int nvfp4_pair_gemm_grid(int num_sms);
// wide = 1: stages of 512 K (three 64 KB operand stages, the block scales
// on their own two-slot ring and two TMEM scale slots), one barrier wait and
// one commit per eight MMAs; wide = 0: stages of 256 K (five 38 KB stages
// holding operands and scales).
cudaError_t launch_nvfp4_pair_gemm(int epi, const CUtensorMap* tmap_a, const CUtensorMap* tmap_b,
                                   const CUtensorMap* tmap_sfa, const CUtensorMap* tmap_sfb,
                                   const GemmParams& p, int grid, cudaStream_t st, int wide = 0);

// ------------------------------------------------------------ combine.cu
// out[t, :] (+)= sum_{s < kk} y[pos[t, s], :] in slot order (FP32
// accumulation of BF16 rows); pos < 0 marks an absent slot. kk <= 32.
cudaError_t launch_error_snapshot(uint32_t* err, uint32_t* snap, cudaStream_t st);
cudaError_t launch_store_ints_to_host(const int64_t* src, int64_t n, int64_t* dst_mapped,
                                      cudaStream_t st);
cudaError_t launch_combine(const uint16_t* y, const int32_t* pos, int T, int kk, int H,
                           float* out, cudaStream_t st, int accumulate = 0);

// Expert-parallel received rows: out[r] = BF16 of the slot sum (as
// launch_combine) for r < *count (device), r < cap; grid-stride.
cudaError_t launch_combine_rows_bf16(const uint16_t* y, const int32_t* pos, int64_t cap,
                                     const int32_t* count, int kk, int H, uint16_t* out,
                                     cudaStream_t st);

// The same sums stored straight into their sources' memory (expert
// parallelism over peer memory): received row r (r < *count) came from source
// s, the last s with recv_off[s] <= r, as that source's row p = r -
// recv_off[s]; its BF16 sum goes to base[s] + p * H (p < limit). Every thread
// then fences its stores at system scope and the grid's last block stores
// `epoch` into flag[s] of every source with release semantics.
constexpr int kMaxReturnRanks = 16;
struct RowReturn {
  uint16_t* base[kMaxReturnRanks];
  uint64_t* flag[kMaxReturnRanks];
  const int32_t* recv_off;  // [W] device
  int W;
  int64_t limit;            // rows each source's area holds
  uint64_t epoch;
  unsigned long long* done;        // finished blocks, all launches (monotonic)
  unsigned long long done_target;  // its value after this launch
  int grid;                        // blocks of this launch
  uint32_t* err;
};
cudaError_t launch_combine_rows_return(const uint16_t* y, const int32_t* pos, int64_t cap,
                                       const int32_t* count, int kk, int H,
                                       const RowReturn& ret, cudaStream_t st);

// ------------------------------------------------------------ weights.cu
// Interleave gate [I, K] and up [I, K] (packed NVFP4 + blocked scales) into
// the stacked gate/up weight slot: 16 gate rows then 16 up rows per 32.
cudaError_t launch_interleave_gate_up(const uint8_t* gate_packed, const uint8_t* gate_sf,
                                      const uint8_t* up_packed, const uint8_t* up_sf, int I,
                                      int K, int group, uint8_t* dst_packed, uint8_t* dst_sf,
                                      cudaStream_t st);
// Row-major scale bytes [rows, K/group] -> blocked layout (zero padding).
// Sets *found to 1 if any of the n bytes equals value (*found not cleared).
cudaError_t launch_find_byte(const uint8_t* p, int64_t n, uint32_t value, uint32_t* found,
                             cudaStream_t st);
cudaError_t launch_scales_to_blocked(const uint8_t* rm, int64_t rows, int64_t sf_cols,
                                     uint8_t* blocked, cudaStream_t st);

}  // namespace glm5x
