// moe_engine.cu -- host engine behind the C ABI in include/glm5x_moe.h.
//
// Owns the resident expert weights (the role of ResidentWeightTable,
// runtime/cuda/resident_weights.cuh:36-57, without eviction: every local
// expert stays in HBM), the forward workspace, the TMA descriptors, and the
// launch sequence of one MoE sublayer forward:
//   row amax -> router logits -> top-k -> expert-major permutation ->
//   activation NVFP4 slabs -> gate/up GEMM (+SwiGLU) -> h NVFP4 slabs ->
//   down GEMM (+routing weight) -> combine.
// Nothing in the forward synchronizes with the host; there is no CPU path.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/glm5x_moe.h"
#include "fp4_codec.h"
#include "glm5x_kernels.cuh"
#include "glm5x_ptx.cuh"
#include "activation_file.h"
#include "k3x_reader.h"
#include "sidecar.h"

using namespace glm5x;

namespace {

thread_local std::string g_last_error;

glm5x_status fail_global(glm5x_status st, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  std::vsnprintf(buf, sizeof buf, fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return st;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point, so the
// library does not link libcuda directly.
using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                   const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                   const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                   CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// 2-D BF16 tensor [rows, cols], box {64 elements, box_rows}, 128B swizzle.
bool make_tmap_bf16(CUtensorMap* m, const void* base, uint64_t cols, uint64_t rows,
                    uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {cols, rows};
  cuuint64_t strides[1] = {cols * 2};
  cuuint32_t box[2] = {64, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// A blocked scale array as a [bytes/256, 256] byte tensor, box {256, 8}: one
// TMA copy moves four consecutive 512-byte scale chunks.
bool make_tmap_sf(CUtensorMap* m, void* base, uint64_t bytes) {
  EncodeTiledFn fn = encode_fn();
  if (!fn || bytes % 256) return false;
  cuuint64_t dims[2] = {256, bytes / 256};
  cuuint64_t strides[1] = {256};
  cuuint32_t box[2] = {256, 8};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

// 2-D byte tensor [rows, row_bytes], box {128 bytes, box_rows}, 128B swizzle.
bool make_tmap_u8(CUtensorMap* m, void* base, uint64_t row_bytes, uint64_t rows,
                  uint32_t box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {128, box_rows};
  cuuint32_t estr[2] = {1, 1};
  return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, base, dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <typename T>
struct DevBuf {
  T* p = nullptr;
  size_t n = 0;
};

}  // namespace

namespace glm5x {
// Records the per-thread message returned by glm5x_last_error_message().
void set_last_error(const char* msg) { g_last_error = msg; }
}  // namespace glm5x

// select_routing's configuration checks (routing_policy.cpp:50-70), message
// for message.
static const char* routing_policy_error(const glm5x_routing_policy& p, int natural_k) {
  auto ladder = [](int k) { return k == 4 || k == 6 || k == 8 || k == 12 || k == 16; };
  if (p.mode < GLM5X_ROUTING_NATURAL || p.mode > GLM5X_ROUTING_ADAPTIVE)
    return "invalid routing mode";
  if (!std::isfinite(p.mass_target) || p.mass_target <= 0.0f || p.mass_target > 1.0f ||
      !std::isfinite(p.minimum_boundary_gap) || p.minimum_boundary_gap < 0.0f ||
      p.minimum_boundary_gap > 1.0f)
    return "invalid adaptive routing threshold";
  if (p.quality_floor_k != 0 &&
      (!ladder(p.quality_floor_k) ||
       (p.mode != GLM5X_ROUTING_NATURAL && p.quality_floor_k > natural_k)))
    return "invalid routing quality floor";
  if (p.mode == GLM5X_ROUTING_FIXED && (!ladder(p.fixed_k) || p.fixed_k > natural_k))
    return "invalid fixed routing K";
  if (p.mode == GLM5X_ROUTING_ADAPTIVE && natural_k != 16)
    return "adaptive routing requires natural Top-16";
  return nullptr;
}

static RoutingPolicy to_device_policy(const glm5x_routing_policy& p) {
  RoutingPolicy d;
  d.mode = p.mode;
  d.fixed_k = p.fixed_k;
  d.mass_target = p.mass_target;
  d.minimum_boundary_gap = p.minimum_boundary_gap;
  d.quality_floor_k = p.quality_floor_k;
  return d;
}

struct glm5x_moe {
  glm5x_moe_config cfg{};
  int device = 0;
  int num_sms = 148;
  cudaStream_t stream = nullptr;
  std::string error;
  glm5x_moe_stats stats{};
  std::vector<void*> allocations;
  int nseg = 0;      // local experts + shared
  int E_loc = 0;
  int64_t rows_cap = 0;
  int last_T = 0;
  int last_bn = 0;
  bool routed_last = false;

  // weights
  uint8_t *w13_packed = nullptr, *w13_sf = nullptr, *w2_packed = nullptr, *w2_sf = nullptr;
  float *w13_global = nullptr, *w2_global = nullptr;
  std::vector<uint8_t> loaded;  // per slot
  uint16_t* router_w = nullptr;
  float* router_bias = nullptr;
  bool router_set = false;

  // workspace
  uint32_t* err = nullptr;
  float *token_amax = nullptr, *logits = nullptr, *topk_w = nullptr;
  int32_t* topk_ids = nullptr;
  int32_t* ids_local = nullptr;  // expert-parallel rows: global -> local expert ids
  RoutingPolicy policy{};        // select_routing mode of the router
  bool routing_diag = false;     // keep per-token routing diagnostics
  int32_t* route_sel = nullptr;  // [max_tokens, 2] selected K, escalated
  float* route_diag = nullptr;   // [max_tokens, 4] entropy, support, mass, confidence
  int64_t route_T = 0;           // tokens of the last router pass with diagnostics
  PermuteBuffers pb{};
  uint8_t *act_packed = nullptr, *act_sf = nullptr, *h_packed = nullptr, *h_sf = nullptr;
  float *act_global = nullptr, *h_global = nullptr;
  float* ones = nullptr;  // unit global scales (MXFP4 has none)
  float* router_partials = nullptr;  // split-K router partial logits
  uint16_t *h_bf16 = nullptr, *y_bf16 = nullptr;
  uint16_t* stage_in = nullptr;  // host-API staging
  float* stage_out = nullptr;
  // Pipelined host API (glm5x_moe_submit_host / glm5x_moe_wait_host): two
  // staging slots, an upload and a download stream beside the compute
  // stream, and per-ticket events and error words in a ring.
  static constexpr int kTicketRing = 64;
  bool pipe_ready = false;
  cudaStream_t up_stream = nullptr, down_stream = nullptr;
  uint16_t* pipe_in[2]{};
  float* pipe_out[2]{};
  cudaEvent_t up_done[kTicketRing]{}, comp_done[kTicketRing]{}, down_done[kTicketRing]{};
  uint32_t* err_snap = nullptr;  // device: error word of each ticket's forward
  uint32_t* err_host = nullptr;  // page-locked copy of err_snap
  int64_t ticket_of[kTicketRing]{};
  int64_t next_ticket = 0;
  // glm5x_moe_read_ints: page-locked words the device writes with stores
  static constexpr int64_t kHostInts = 4096;
  int64_t* host_ints = nullptr;
  int64_t* host_ints_dev = nullptr;  // device address of host_ints
  uint8_t* stage_w = nullptr;    // weight admission staging
  size_t stage_w_bytes = 0;
  float* scratch_f = nullptr;

  int force_bn = 0;  // 0 = choose the token tile from the batch
  bool profiling = false;
  int profiled = 0;
  // Phase events of the last kProfRing forwards: accumulated lazily (when a
  // slot is reused or phase times are read), so profiled forwards do not wait
  // on the device.
  static constexpr int kProfRing = 64;
  cudaEvent_t ev[kProfRing][GLM5X_NUM_PHASES + 1]{};
  bool prof_pending[kProfRing]{};
  int prof_slot = 0;
  double phase_ms[GLM5X_NUM_PHASES]{};
  void accumulate_slot(int slot) {
    if (!prof_pending[slot]) return;
    cudaEventSynchronize(ev[slot][GLM5X_NUM_PHASES]);
    for (int i = 0; i < GLM5X_NUM_PHASES; ++i) {
      float ms = 0.0f;
      if (cudaEventElapsedTime(&ms, ev[slot][i], ev[slot][i + 1]) == cudaSuccess)
        phase_ms[i] += ms;
    }
    prof_pending[slot] = false;
    profiled++;
  }

  CUtensorMap tm_w13{}, tm_w2{};
  CUtensorMap tm_router{};
  CUtensorMap tm_w13_sf{}, tm_w2_sf{}, tm_act_sf{}, tm_h_sf{};
  int pair_grid = 0;       // CTAs for the pair GEMM (0 = unavailable)
  bool use_pair = true;    // 256-row token tiles on CTA pairs (cta_group::2)
  bool token_major_down = false;  // token-major down projection (opt-in: not faster here)
  int down_bn = 0;                // weight-major down projection tile width (0 = same)
  // weight rows per tile of the single-CTA GEMMs for 32- and 64-row token
  // tiles: 256 as two halves per stage (the default: config-4 decode 0.544 ->
  // 0.467 ms, 0.67 -> 0.78 of HBM), or 128 (glm5x_moe_set_weight_tile_rows)
  int weight_rows = 256;
  // CTA-pair GEMMs with 512-K stages (glm5x_moe_set_pair_wide_stages): one
  // barrier wait and one commit of the MMA thread per eight MMAs. Config 5:
  // gate/up GEMM 1.18 -> 1.10 ms, down 0.76 -> 0.75 ms.
  int pair_wide = 1;
  // CTA-pair GEMM tile order, token tiles per group for the gate/up and the
  // down GEMM (0 = segment-major; glm5x_moe_set_pair_tile_order). With the
  // wide stages, config 5: gate/up 1.10 -> 1.06-1.07 ms, down 0.75 -> 0.71 ms
  // (segment-major order runs light and heavy experts in separate phases).
  int tile_group_up = 8, tile_group_down = 16;
  CUtensorMap tm_act[4]{}, tm_h[4]{};  // box rows 32, 64, 128, 256

  glm5x_status fail(glm5x_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    std::vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    error = buf;
    g_last_error = buf;
    return st;
  }

  template <typename T>
  bool alloc(T** p, size_t count) {
    void* q = nullptr;
    if (cudaMalloc(&q, std::max<size_t>(count, 1) * sizeof(T)) != cudaSuccess) return false;
    allocations.push_back(q);
    stats.workspace_bytes += count * sizeof(T);
    *p = static_cast<T*>(q);
    return true;
  }

  int H() const { return cfg.hidden; }
  int I() const { return cfg.intermediate; }
  int K() const { return cfg.top_k; }
  int kk() const { return cfg.top_k + (cfg.has_shared ? 1 : 0); }

  bool mx() const { return cfg.precision == GLM5X_PRECISION_MXFP4; }
  int grp() const { return mx() ? 32 : 16; }   // values per scale
  int terms() const { return mx() ? 4 : 1; }   // B rows per token (MXFP4 residual terms)
  // bytes of blocked scales for `rows` rows of length K (128-row x 4-scale chunks of 512 B)
  size_t sf_bytes(int64_t rows, int64_t K) const { return (size_t)(rows / 128) * (K / grp() / 4) * 512; }
  size_t w13_packed_bytes() const { return (size_t)2 * I() * H() / 2; }
  size_t w13_sf_bytes() const { return sf_bytes(2 * I(), H()); }
  size_t w2_packed_bytes() const { return (size_t)H() * I() / 2; }
  size_t w2_sf_bytes() const { return sf_bytes(H(), I()); }
};

namespace {

glm5x_status cuda_fail(glm5x_moe* m, cudaError_t e, const char* what) {
  return m->fail(GLM5X_DEVICE_ERROR, "%s: %s", what, cudaGetErrorString(e));
}

#define G5_CHECK(m, expr, what)                  \
  do {                                           \
    cudaError_t e_ = (expr);                     \
    if (e_ != cudaSuccess) return cuda_fail(m, e_, what); \
  } while (0)

int bn_index(int bn) { return bn == 32 ? 0 : bn == 64 ? 1 : bn == 128 ? 2 : 3; }

int pick_bn(const glm5x_moe* m, int64_t T) {
  if (m->force_bn) return m->force_bn;
  // B rows per expert (4 per token for MXFP4 terms)
  const double per_expert = (double)T * m->K() * m->terms() / std::max(1, m->cfg.num_experts);
  if (per_expert <= 24) return 32;
  if (per_expert <= 48) return 64;
  if (per_expert <= 96) return 128;
  return 256;
}

int slot_of(const glm5x_moe* m, int32_t expert) {
  if (expert < 0) return m->cfg.has_shared ? m->E_loc : -1;
  const int s = expert - m->cfg.expert_begin;
  return (s >= 0 && s < m->E_loc) ? s : -1;
}

glm5x_status validate_nvfp4(glm5x_moe* m, const glm5x_nvfp4_matrix* w, int64_t rows,
                            int64_t cols, const char* role) {
  if (!w || !w->packed || !w->scales) return m->fail(GLM5X_INVALID_EXTENT, "%s: null matrix", role);
  if (w->rows != rows || w->cols != cols)
    return m->fail(GLM5X_INVALID_EXTENT, "%s: shape [%lld, %lld], expected [%lld, %lld]", role,
                   (long long)w->rows, (long long)w->cols, (long long)rows, (long long)cols);
  if (!(w->global_scale > 0.0f) || !std::isfinite(w->global_scale))
    return m->fail(GLM5X_INVALID_EXTENT, "%s: global scale must be finite and positive", role);
  return GLM5X_OK;
}

}  // namespace

// ============================================================== engine API
extern "C" {

const char* glm5x_last_error_message(void) { return g_last_error.c_str(); }

const char* glm5x_moe_error_message(const glm5x_moe* moe) {
  return moe ? moe->error.c_str() : g_last_error.c_str();
}

glm5x_status glm5x_moe_create(const glm5x_moe_config* cfg, int device, glm5x_moe** out) {
  if (!cfg || !out) return fail_global(GLM5X_INVALID_EXTENT, "null config or output");
  *out = nullptr;
  const glm5x_moe_config& c = *cfg;
  if (c.hidden <= 0 || c.intermediate <= 0 || c.hidden % 512 || c.intermediate % 512 ||
      c.intermediate % 64)
    return fail_global(GLM5X_INVALID_EXTENT, "hidden and intermediate must be multiples of 512");
  if (c.num_experts <= 0 || c.num_experts > 256 || c.top_k <= 0 || c.top_k > 16 ||
      c.top_k > c.num_experts)
    return fail_global(GLM5X_INVALID_EXTENT, "need 0 < top_k <= 16, top_k <= num_experts <= 256");
  if (!router_tc_supported(c.num_experts, c.hidden, c.top_k) && c.num_experts % 16 != 0 &&
      c.num_experts > 16)
    return fail_global(GLM5X_INVALID_EXTENT, "num_experts must be a multiple of 16");
  if (c.max_tokens <= 0 || c.max_tokens > (1 << 20))
    return fail_global(GLM5X_INVALID_EXTENT, "max_tokens out of range");
  if (!(c.routed_scaling > 0.0f)) return fail_global(GLM5X_INVALID_EXTENT, "routed_scaling <= 0");
  if (c.precision != GLM5X_PRECISION_NVFP4 && c.precision != GLM5X_PRECISION_MXFP4)
    return fail_global(GLM5X_INVALID_EXTENT, "unknown precision");
  const int ecount = c.expert_count > 0 ? c.expert_count : c.num_experts;
  if (c.expert_begin < 0 || c.expert_begin + ecount > c.num_experts)
    return fail_global(GLM5X_INVALID_EXTENT, "expert range outside [0, num_experts)");

  int ndev = 0;
  if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0)
    return fail_global(GLM5X_BACKEND_UNAVAILABLE, "no CUDA device");
  if (device < 0 || device >= ndev) return fail_global(GLM5X_BACKEND_UNAVAILABLE, "bad device");
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) != cudaSuccess)
    return fail_global(GLM5X_BACKEND_UNAVAILABLE, "cannot query device");
  if (prop.major != 10 || prop.minor != 0)
    return fail_global(GLM5X_UNSUPPORTED_ARCHITECTURE,
                       "device compute capability %d.%d; this build needs sm_100 (B200)",
                       prop.major, prop.minor);
  if (!encode_fn()) return fail_global(GLM5X_BACKEND_UNAVAILABLE, "cuTensorMapEncodeTiled missing");

  auto* m = new glm5x_moe();
  m->cfg = c;
  m->cfg.expert_count = ecount;
  m->device = device;
  m->num_sms = prop.multiProcessorCount;
  m->E_loc = ecount;
  m->nseg = ecount + (c.has_shared ? 1 : 0);
  cudaSetDevice(device);
  if (cudaStreamCreateWithFlags(&m->stream, cudaStreamNonBlocking) != cudaSuccess) {
    delete m;
    return fail_global(GLM5X_BACKEND_UNAVAILABLE, "stream creation failed");
  }
  const int64_t T = c.max_tokens;
  const int H = c.hidden, I = c.intermediate, E = c.num_experts, k = c.top_k;
  const int nseg = m->nseg;
  // segment rows for the widest layout the automatic tile choice can use:
  // 32-row tiles (4 x rows) up to 24 rows per expert, 64-row tiles (2 x) up
  // to 48, dense beyond; MXFP4 has 4 rows (terms) per token
  const int tr = m->terms();
  const int64_t per32 = std::min<int64_t>(T, 24LL * E / (k * tr)),
                per64 = std::min<int64_t>(T, 48LL * E / (k * tr));
  const int64_t logical =
      tr * std::max({T * (int64_t)m->kk(), 4 * per32 * m->kk(), 2 * per64 * m->kk()});
  m->rows_cap = logical + (int64_t)nseg * 128 + 256;
  const int64_t R = m->rows_cap;
  const int64_t rb = R / 128 + 2;
  bool ok = true;
  ok &= m->alloc(&m->w13_packed, (size_t)nseg * m->w13_packed_bytes());
  ok &= m->alloc(&m->w13_sf, (size_t)nseg * m->w13_sf_bytes());
  ok &= m->alloc(&m->w2_packed, (size_t)nseg * m->w2_packed_bytes());
  ok &= m->alloc(&m->w2_sf, (size_t)nseg * m->w2_sf_bytes());
  ok &= m->alloc(&m->w13_global, (size_t)2 * nseg);
  ok &= m->alloc(&m->w2_global, (size_t)nseg);
  ok &= m->alloc(&m->router_w, (size_t)E * H);
  ok &= m->alloc(&m->router_bias, (size_t)E);
  ok &= m->alloc(&m->err, 1);
  ok &= m->alloc(&m->token_amax, (size_t)T);
  ok &= m->alloc(&m->logits, (size_t)T * E);
  ok &= m->alloc(&m->topk_w, (size_t)T * k);
  ok &= m->alloc(&m->topk_ids, (size_t)T * k);
  ok &= m->alloc(&m->ids_local, (size_t)T * k);
  ok &= m->alloc(&m->route_sel, (size_t)T * 2);
  ok &= m->alloc(&m->route_diag, (size_t)T * 4);
  ok &= m->alloc(&m->pb.chunk_count, (size_t)((T + 255) / 256) * E);
  ok &= m->alloc(&m->pb.rank, (size_t)T * k);
  ok &= m->alloc(&m->pb.seg_count, (size_t)nseg + 1);
  ok &= m->alloc(&m->pb.seg_start, (size_t)nseg + 1);
  ok &= m->alloc(&m->pb.qprefix, (size_t)nseg + 1);
  ok &= m->alloc(&m->pb.ntile_prefix, (size_t)nseg + 1);
  ok &= m->alloc(&m->pb.seg_amax, (size_t)nseg);
  ok &= m->alloc(&m->pb.h_amax, (size_t)nseg);
  ok &= m->alloc(&m->pb.pos, (size_t)T * m->kk());
  ok &= m->alloc(&m->pb.row_token, (size_t)R);
  ok &= m->alloc(&m->pb.row_weight, (size_t)R);
  ok &= m->alloc(&m->act_packed, (size_t)R * H / 2);
  ok &= m->alloc(&m->act_sf, m->sf_bytes(rb * 128, H));
  ok &= m->alloc(&m->act_global, (size_t)nseg);
  ok &= m->alloc(&m->h_bf16, (size_t)R * I);
  ok &= m->alloc(&m->h_packed, (size_t)R * I / 2);
  ok &= m->alloc(&m->h_sf, m->sf_bytes(rb * 128, I));
  ok &= m->alloc(&m->ones, (size_t)2 * nseg);
  ok &= m->alloc(&m->router_partials, router_partials_floats(m->num_sms, E));
  ok &= m->alloc(&m->h_global, (size_t)nseg);
  ok &= m->alloc(&m->y_bf16, (size_t)R * H);
  ok &= m->alloc(&m->stage_in, (size_t)T * H);
  ok &= m->alloc(&m->stage_out, (size_t)T * H);
  ok &= m->alloc(&m->scratch_f, 16);
  if (!ok) {
    glm5x_moe_destroy(m);
    return fail_global(GLM5X_OUT_OF_MEMORY, "device allocation failed (max_tokens=%lld)",
                       (long long)T);
  }
  cudaMemset(m->err, 0, sizeof(uint32_t));
  cudaMemset(m->w13_global, 0, sizeof(float) * 2 * nseg);
  cudaMemset(m->w2_global, 0, sizeof(float) * nseg);
  cudaMemset(m->act_packed, 0, (size_t)R * H / 2);
  cudaMemset(m->h_packed, 0, (size_t)R * I / 2);
  cudaMemset(m->act_sf, 0, m->sf_bytes(rb * 128, H));
  cudaMemset(m->h_sf, 0, m->sf_bytes(rb * 128, I));
  if (m->ones) {
    std::vector<float> one(2 * nseg, 1.0f);
    cudaMemcpy(m->ones, one.data(), sizeof(float) * one.size(), cudaMemcpyHostToDevice);
  }
  m->loaded.assign(nseg, 0);
  ok = make_tmap_u8(&m->tm_w13, m->w13_packed, H / 2, (uint64_t)nseg * 2 * I, 128) &&
       make_tmap_u8(&m->tm_w2, m->w2_packed, I / 2, (uint64_t)nseg * H, 128);
  const int boxes[4] = {32, 64, 128, 256};
  for (int i = 0; i < 4 && ok; ++i) {
    ok = make_tmap_u8(&m->tm_act[i], m->act_packed, H / 2, R, boxes[i]) &&
         make_tmap_u8(&m->tm_h[i], m->h_packed, I / 2, R, boxes[i]);
  }
  ok = ok && make_tmap_sf(&m->tm_w13_sf, m->w13_sf, (uint64_t)nseg * m->w13_sf_bytes()) &&
       make_tmap_sf(&m->tm_w2_sf, m->w2_sf, (uint64_t)nseg * m->w2_sf_bytes()) &&
       make_tmap_sf(&m->tm_act_sf, m->act_sf, m->sf_bytes(rb * 128, H)) &&
       make_tmap_sf(&m->tm_h_sf, m->h_sf, m->sf_bytes(rb * 128, I));
  if (!ok) {
    glm5x_moe_destroy(m);
    return fail_global(GLM5X_BACKEND_UNAVAILABLE, "tensor map encoding failed");
  }
  m->pair_grid = nvfp4_pair_gemm_grid(m->num_sms);
  cudaGetLastError();
  if (cudaDeviceSynchronize() != cudaSuccess) {
    glm5x_moe_destroy(m);
    return fail_global(GLM5X_DEVICE_ERROR, "device initialization failed");
  }
  *out = m;
  return GLM5X_OK;
}

void glm5x_moe_destroy(glm5x_moe* m) {
  if (!m) return;
  cudaSetDevice(m->device);
  for (cudaStream_t s : {m->stream, m->up_stream, m->down_stream})
    if (s) cudaStreamSynchronize(s);
  for (void* p : m->allocations) cudaFree(p);
  if (m->stage_w) cudaFree(m->stage_w);
  for (cudaStream_t s : {m->stream, m->up_stream, m->down_stream})
    if (s) cudaStreamDestroy(s);
  for (int i = 0; i < glm5x_moe::kTicketRing; ++i)
    for (cudaEvent_t e : {m->up_done[i], m->comp_done[i], m->down_done[i]})
      if (e) cudaEventDestroy(e);
  if (m->err_host) cudaFreeHost(m->err_host);
  if (m->host_ints) cudaFreeHost(m->host_ints);
  for (auto& row : m->ev)
    for (auto& e : row)
      if (e) cudaEventDestroy(e);
  delete m;
}

glm5x_status glm5x_moe_set_router(glm5x_moe* m, const uint16_t* w, const float* bias) {
  if (!m || !w || !bias) return fail_global(GLM5X_INVALID_EXTENT, "null router argument");
  const int E = m->cfg.num_experts, H = m->H();
  for (int e = 0; e < E; ++e)
    if (!std::isfinite(bias[e])) return m->fail(GLM5X_INVALID_STATE, "router bias not finite");
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaMemcpyAsync(m->router_w, w, sizeof(uint16_t) * E * H, cudaMemcpyHostToDevice,
                              m->stream), "router upload");
  G5_CHECK(m, cudaMemcpyAsync(m->router_bias, bias, sizeof(float) * E, cudaMemcpyHostToDevice,
                              m->stream), "bias upload");
  G5_CHECK(m, cudaStreamSynchronize(m->stream), "router upload");
  if (!router_tc_supported(E, H, m->K()))
    return m->fail(GLM5X_INVALID_EXTENT, "router needs num_experts in [16, 256], a multiple of 16");
  if (!make_tmap_bf16(&m->tm_router, m->router_w, H, E, E))
    return m->fail(GLM5X_BACKEND_UNAVAILABLE, "router tensor map");
  m->router_set = true;
  return GLM5X_OK;
}

static glm5x_status admit_nvfp4(glm5x_moe* m, int slot, const glm5x_nvfp4_matrix* gate,
                                const glm5x_nvfp4_matrix* up, const glm5x_nvfp4_matrix* down,
                                bool device_ptrs) {
  const int H = m->H(), I = m->I();
  const size_t g_pb = (size_t)I * H / 2, g_sb = (size_t)(I / 128) * (H / 64) * 512;
  const size_t d_pb = m->w2_packed_bytes(), d_sb = m->w2_sf_bytes();
  const uint8_t *gp = gate->packed, *gs = gate->scales, *up_p = up->packed, *us = up->scales;
  const uint8_t *dp = down->packed, *ds = down->scales;
  cudaStream_t st = m->stream;
  if (!device_ptrs) {
    const size_t need = 2 * (g_pb + g_sb);
    if (m->stage_w_bytes < need) {
      if (m->stage_w) cudaFree(m->stage_w);
      m->stage_w = nullptr;
      m->stage_w_bytes = 0;
      G5_CHECK(m, cudaMalloc(&m->stage_w, need), "weight staging");
      m->stage_w_bytes = need;
    }
    uint8_t* s = m->stage_w;
    G5_CHECK(m, cudaMemcpyAsync(s, gp, g_pb, cudaMemcpyHostToDevice, st), "gate upload");
    G5_CHECK(m, cudaMemcpyAsync(s + g_pb, gs, g_sb, cudaMemcpyHostToDevice, st), "gate upload");
    G5_CHECK(m, cudaMemcpyAsync(s + g_pb + g_sb, up_p, g_pb, cudaMemcpyHostToDevice, st), "up");
    G5_CHECK(m, cudaMemcpyAsync(s + 2 * g_pb + g_sb, us, g_sb, cudaMemcpyHostToDevice, st), "up");
    gp = s;
    gs = s + g_pb;
    up_p = s + g_pb + g_sb;
    us = s + 2 * g_pb + g_sb;
  }
  G5_CHECK(m, launch_interleave_gate_up(gp, gs, up_p, us, I, H, 16,
                                        m->w13_packed + (size_t)slot * m->w13_packed_bytes(),
                                        m->w13_sf + (size_t)slot * m->w13_sf_bytes(), st),
           "gate/up interleave");
  const cudaMemcpyKind kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  G5_CHECK(m, cudaMemcpyAsync(m->w2_packed + (size_t)slot * d_pb, dp, d_pb, kind, st), "down");
  G5_CHECK(m, cudaMemcpyAsync(m->w2_sf + (size_t)slot * d_sb, ds, d_sb, kind, st), "down scales");
  const float g13[2] = {gate->global_scale, up->global_scale};
  G5_CHECK(m, cudaMemcpyAsync(m->w13_global + 2 * slot, g13, sizeof g13, cudaMemcpyHostToDevice, st),
           "globals");
  G5_CHECK(m, cudaMemcpyAsync(m->w2_global + slot, &down->global_scale, sizeof(float),
                              cudaMemcpyHostToDevice, st), "globals");
  G5_CHECK(m, cudaStreamSynchronize(st), "expert admission");
  if (!m->loaded[slot]) {
    m->loaded[slot] = 1;
    m->stats.loaded_experts++;
    m->stats.resident_weight_bytes += m->w13_packed_bytes() + m->w13_sf_bytes() + d_pb + d_sb;
  }
  return GLM5X_OK;
}

static glm5x_status load_nvfp4_common(glm5x_moe* m, int32_t expert,
                                      const glm5x_nvfp4_matrix* gate,
                                      const glm5x_nvfp4_matrix* up,
                                      const glm5x_nvfp4_matrix* down, bool dev) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (m->cfg.precision != GLM5X_PRECISION_NVFP4)
    return m->fail(GLM5X_INVALID_STATE, "engine precision is not NVFP4");
  const int slot = slot_of(m, expert);
  if (slot < 0) return m->fail(GLM5X_INVALID_EXTENT, "expert %d is not held by this engine", expert);
  glm5x_status s;
  if ((s = validate_nvfp4(m, gate, m->I(), m->H(), "gate")) != GLM5X_OK) return s;
  if ((s = validate_nvfp4(m, up, m->I(), m->H(), "up")) != GLM5X_OK) return s;
  if ((s = validate_nvfp4(m, down, m->H(), m->I(), "down")) != GLM5X_OK) return s;
  cudaSetDevice(m->device);
  return admit_nvfp4(m, slot, gate, up, down, dev);
}

glm5x_status glm5x_moe_load_expert_nvfp4(glm5x_moe* m, int32_t expert,
                                         const glm5x_nvfp4_matrix* gate,
                                         const glm5x_nvfp4_matrix* up,
                                         const glm5x_nvfp4_matrix* down) {
  return load_nvfp4_common(m, expert, gate, up, down, false);
}

glm5x_status glm5x_moe_load_expert_nvfp4_device(glm5x_moe* m, int32_t expert,
                                                const glm5x_nvfp4_matrix* gate,
                                                const glm5x_nvfp4_matrix* up,
                                                const glm5x_nvfp4_matrix* down) {
  return load_nvfp4_common(m, expert, gate, up, down, true);
}

// MXFP4 expert admission (GLM5XMXFP4 sidecars / .k3x MXFP4 records,
// reference/k3x_ref/mxfp4.py:31-107 layout): packed [rows, cols/2] and
// row-major E8M0 scales [rows, cols/32]. Scales go to the 128x4 blocked
// layout the block-scaled MMA reads; gate/up rows are interleaved like the
// NVFP4 path. A 0xFF scale byte (NaN in E8M0) is rejected, as the reference's
// decode_mxfp4 does (runtime/src/ops.cpp:40-63, mxfp4.py:110-144).
static glm5x_status admit_mxfp4(glm5x_moe* m, int slot, const glm5x_mxfp4_matrix* gate,
                                const glm5x_mxfp4_matrix* up, const glm5x_mxfp4_matrix* down,
                                bool device_ptrs) {
  const int H = m->H(), I = m->I();
  const size_t g_pb = (size_t)I * H / 2, g_rm = (size_t)I * H / 32, g_sb = m->sf_bytes(I, H);
  const size_t d_pb = m->w2_packed_bytes(), d_rm = (size_t)H * I / 32;
  cudaStream_t st = m->stream;
  const size_t need = 2 * (g_pb + g_rm + g_sb) + d_rm + 16;
  if (m->stage_w_bytes < need) {
    if (m->stage_w) cudaFree(m->stage_w);
    m->stage_w = nullptr;
    m->stage_w_bytes = 0;
    G5_CHECK(m, cudaMalloc(&m->stage_w, need), "weight staging");
    m->stage_w_bytes = need;
  }
  uint8_t* s = m->stage_w;
  uint8_t *gp = s, *grm = gp + g_pb, *gsb = grm + g_rm;
  uint8_t *upk = gsb + g_sb, *urm = upk + g_pb, *usb = urm + g_rm;
  uint8_t* drm = usb + g_sb;
  uint32_t* bad = reinterpret_cast<uint32_t*>(drm + d_rm);
  const cudaMemcpyKind kind = device_ptrs ? cudaMemcpyDeviceToDevice : cudaMemcpyHostToDevice;
  G5_CHECK(m, cudaMemcpyAsync(gp, gate->packed, g_pb, kind, st), "gate upload");
  G5_CHECK(m, cudaMemcpyAsync(grm, gate->scales, g_rm, kind, st), "gate scales");
  G5_CHECK(m, cudaMemcpyAsync(upk, up->packed, g_pb, kind, st), "up upload");
  G5_CHECK(m, cudaMemcpyAsync(urm, up->scales, g_rm, kind, st), "up scales");
  G5_CHECK(m, cudaMemcpyAsync(drm, down->scales, d_rm, kind, st), "down scales");
  G5_CHECK(m, cudaMemsetAsync(bad, 0, sizeof(uint32_t), st), "scale check");
  G5_CHECK(m, launch_find_byte(grm, g_rm, 0xFF, bad, st), "scale check");
  G5_CHECK(m, launch_find_byte(urm, g_rm, 0xFF, bad, st), "scale check");
  G5_CHECK(m, launch_find_byte(drm, d_rm, 0xFF, bad, st), "scale check");
  uint32_t found = 0;
  G5_CHECK(m, cudaMemcpyAsync(&found, bad, sizeof found, cudaMemcpyDeviceToHost, st), "scale check");
  G5_CHECK(m, cudaStreamSynchronize(st), "scale check");
  if (found) return m->fail(GLM5X_INVALID_MXFP4, "E8M0 scale 0xff is reserved");
  G5_CHECK(m, cudaMemsetAsync(gsb, 0, g_sb, st), "scales");
  G5_CHECK(m, cudaMemsetAsync(usb, 0, g_sb, st), "scales");
  G5_CHECK(m, launch_scales_to_blocked(grm, I, H / 32, gsb, st), "gate scales");
  G5_CHECK(m, launch_scales_to_blocked(urm, I, H / 32, usb, st), "up scales");
  G5_CHECK(m, launch_interleave_gate_up(gp, gsb, upk, usb, I, H, 32,
                                        m->w13_packed + (size_t)slot * m->w13_packed_bytes(),
                                        m->w13_sf + (size_t)slot * m->w13_sf_bytes(), st),
           "gate/up interleave");
  G5_CHECK(m, cudaMemcpyAsync(m->w2_packed + (size_t)slot * d_pb, down->packed, d_pb, kind, st),
           "down");
  G5_CHECK(m, launch_scales_to_blocked(drm, H, I / 32,
                                       m->w2_sf + (size_t)slot * m->w2_sf_bytes(), st),
           "down scales");
  G5_CHECK(m, cudaStreamSynchronize(st), "expert admission");
  if (!m->loaded[slot]) {
    m->loaded[slot] = 1;
    m->stats.loaded_experts++;
    m->stats.resident_weight_bytes +=
        m->w13_packed_bytes() + m->w13_sf_bytes() + d_pb + m->w2_sf_bytes();
  }
  return GLM5X_OK;
}

static glm5x_status load_mxfp4_common(glm5x_moe* m, int32_t expert,
                                      const glm5x_mxfp4_matrix* gate,
                                      const glm5x_mxfp4_matrix* up,
                                      const glm5x_mxfp4_matrix* down, bool dev) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (!m->mx()) return m->fail(GLM5X_INVALID_STATE, "engine precision is not MXFP4");
  const int slot = slot_of(m, expert);
  if (slot < 0) return m->fail(GLM5X_INVALID_EXTENT, "expert %d is not held by this engine", expert);
  const glm5x_mxfp4_matrix* mats[3] = {gate, up, down};
  const int64_t shape[3][2] = {{m->I(), m->H()}, {m->I(), m->H()}, {m->H(), m->I()}};
  const char* role[3] = {"gate", "up", "down"};
  for (int r = 0; r < 3; ++r) {
    const glm5x_mxfp4_matrix* w = mats[r];
    if (!w || !w->packed || !w->scales)
      return m->fail(GLM5X_INVALID_EXTENT, "%s: null matrix", role[r]);
    if (w->rows != shape[r][0] || w->cols != shape[r][1])
      return m->fail(GLM5X_INVALID_EXTENT, "%s: shape [%lld, %lld], expected [%lld, %lld]",
                     role[r], (long long)w->rows, (long long)w->cols, (long long)shape[r][0],
                     (long long)shape[r][1]);
    if (w->group_size != 32)
      return m->fail(GLM5X_INVALID_EXTENT, "%s: MXFP4 group size must be 32", role[r]);
  }
  cudaSetDevice(m->device);
  return admit_mxfp4(m, slot, gate, up, down, dev);
}

glm5x_status glm5x_moe_load_expert_mxfp4(glm5x_moe* m, int32_t expert,
                                         const glm5x_mxfp4_matrix* gate,
                                         const glm5x_mxfp4_matrix* up,
                                         const glm5x_mxfp4_matrix* down) {
  return load_mxfp4_common(m, expert, gate, up, down, false);
}

glm5x_status glm5x_moe_load_expert_mxfp4_device(glm5x_moe* m, int32_t expert,
                                                const glm5x_mxfp4_matrix* gate,
                                                const glm5x_mxfp4_matrix* up,
                                                const glm5x_mxfp4_matrix* down) {
  return load_mxfp4_common(m, expert, gate, up, down, true);
}

// BF16 experts packed on the device at admission. NVFP4 engines: each
// projection through quantize_nvfp4_weight (the reference's NVFP4 mode packs
// float experts when it loads them, _quantize_expert_nvfp4,
// reference/glm5x_ref/layer10_moe.py:603-619; scale_mode "mse" is its
// default, nvfp4.py:180-198). MXFP4 engines: encode_mxfp4 with group 32, as
// GLM5XPackedExpertCache.put encodes .pm4 sidecars (packed_cache.py:256-266,
// max_abs there). The packed bytes then take the NVFP4 / MXFP4 admission
// path, so the resident weights are those of loading the packed expert.
static glm5x_status load_bf16_common(glm5x_moe* m, int32_t expert, const uint16_t* gate,
                                     const uint16_t* up, const uint16_t* down, int32_t scale_mode,
                                     bool dev) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (!gate || !up || !down) return m->fail(GLM5X_INVALID_STATE, "null projection");
  if (scale_mode != GLM5X_SCALE_MAX_ABS && scale_mode != GLM5X_SCALE_MSE)
    return m->fail(GLM5X_INVALID_STATE, "scale_mode must be GLM5X_SCALE_MAX_ABS or _MSE");
  const int slot = slot_of(m, expert);
  if (slot < 0) return m->fail(GLM5X_INVALID_EXTENT, "expert %d is not held by this engine", expert);
  cudaSetDevice(m->device);
  const int64_t H = m->H(), I = m->I();
  const int64_t n = I * H;  // elements of each projection
  const uint16_t* src[3] = {gate, up, down};
  const int64_t rows[3] = {I, I, H}, cols[3] = {H, H, I};
  const bool mx = m->mx();
  size_t sb[3];
  for (int r = 0; r < 3; ++r)
    sb[r] = mx ? (size_t)(n / 32) : (size_t)((rows[r] + 127) / 128) * ((cols[r] / 16 + 3) / 4) * 512;
  // one scratch block: BF16 sources (host input only), packed, scales, FP32
  // amax / globals and the error word
  const size_t in_bytes = dev ? 0 : (size_t)3 * n * 2;
  const size_t total = in_bytes + (size_t)3 * n / 2 + sb[0] + sb[1] + sb[2] + 256;
  uint8_t* buf = nullptr;
  G5_CHECK(m, cudaMalloc(&buf, total), "BF16 admission scratch");
  struct Free {
    uint8_t* p;
    ~Free() { cudaFree(p); }
  } free_buf{buf};
  cudaStream_t st = m->stream;
  uint8_t* cur = buf;
  const __nv_bfloat16* d_src[3];
  for (int r = 0; r < 3; ++r) {
    if (dev) {
      d_src[r] = reinterpret_cast<const __nv_bfloat16*>(src[r]);
    } else {
      G5_CHECK(m, cudaMemcpyAsync(cur, src[r], (size_t)n * 2, cudaMemcpyHostToDevice, st),
               "BF16 upload");
      d_src[r] = reinterpret_cast<const __nv_bfloat16*>(cur);
      cur += (size_t)n * 2;
    }
  }
  uint8_t* packed[3];
  uint8_t* scales[3];
  for (int r = 0; r < 3; ++r) {
    packed[r] = cur;
    cur += n / 2;
  }
  for (int r = 0; r < 3; ++r) {
    scales[r] = cur;
    cur += sb[r];
  }
  cur = buf + (total - 256);
  float* amax = reinterpret_cast<float*>(cur);
  float* globals = amax + 4;
  uint32_t* err = reinterpret_cast<uint32_t*>(globals + 4);
  G5_CHECK(m, cudaMemsetAsync(err, 0, 4, st), "BF16 admission");
  for (int r = 0; r < 3; ++r) {
    if (mx)
      G5_CHECK(m, launch_mxfp4_encode<__nv_bfloat16>(d_src[r], n, 32, scale_mode, packed[r],
                                                     scales[r], err, st),
               "MXFP4 encode");
    else
      G5_CHECK(m, launch_nvfp4_quantize_matrix<__nv_bfloat16>(d_src[r], rows[r], cols[r],
                                                              scale_mode, amax + r, packed[r],
                                                              scales[r], globals + r, err, st),
               "NVFP4 quantize");
  }
  float g[3] = {1.0f, 1.0f, 1.0f};
  uint32_t word = 0;
  G5_CHECK(m, cudaMemcpyAsync(g, globals, sizeof g, cudaMemcpyDeviceToHost, st), "globals");
  G5_CHECK(m, cudaMemcpyAsync(&word, err, 4, cudaMemcpyDeviceToHost, st), "error word");
  G5_CHECK(m, cudaStreamSynchronize(st), "BF16 admission");
  if (word & (kErrBadScale | kErrNonFinite))
    return m->fail(mx ? GLM5X_INVALID_MXFP4 : GLM5X_INVALID_STATE,
                   "BF16 expert: non-finite weights or a scale out of range (0x%x)", word);
  if (word) return m->fail(GLM5X_DEVICE_ERROR, "BF16 expert: device error 0x%x", word);
  if (mx) {
    glm5x_mxfp4_matrix mats[3];
    for (int r = 0; r < 3; ++r) mats[r] = glm5x_mxfp4_matrix{packed[r], scales[r], rows[r], cols[r], 32};
    return admit_mxfp4(m, slot, &mats[0], &mats[1], &mats[2], true);
  }
  glm5x_nvfp4_matrix mats[3];
  for (int r = 0; r < 3; ++r) mats[r] = glm5x_nvfp4_matrix{packed[r], scales[r], g[r], rows[r], cols[r]};
  return admit_nvfp4(m, slot, &mats[0], &mats[1], &mats[2], true);
}

glm5x_status glm5x_moe_load_expert_bf16(glm5x_moe* m, int32_t expert, const uint16_t* gate,
                                        const uint16_t* up, const uint16_t* down,
                                        int32_t scale_mode) {
  return load_bf16_common(m, expert, gate, up, down, scale_mode, false);
}

glm5x_status glm5x_moe_load_expert_bf16_device(glm5x_moe* m, int32_t expert, const uint16_t* gate,
                                               const uint16_t* up, const uint16_t* down,
                                               int32_t scale_mode) {
  return load_bf16_common(m, expert, gate, up, down, scale_mode, true);
}

struct glm5x_k3x {
  K3xFile file;
};

glm5x_status glm5x_k3x_open(const char* path, int32_t verify, glm5x_k3x** out) {
  if (!path || !out) return fail_global(GLM5X_INVALID_STATE, "null argument");
  *out = nullptr;
  auto* h = new glm5x_k3x;
  std::string msg;
  const int rc = k3x_open(path, verify != 0, &h->file, &msg);
  if (rc != 0) {
    delete h;
    return fail_global(static_cast<glm5x_status>(rc), "%s: %s", path, msg.c_str());
  }
  *out = h;
  return GLM5X_OK;
}

void glm5x_k3x_close(glm5x_k3x* h) { delete h; }

static const K3xTensor* k3x_lookup(const glm5x_k3x* h, const char* name) {
  return (h && name) ? k3x_find(h->file, fnv1a64(name)) : nullptr;
}

glm5x_status glm5x_k3x_tensor(const glm5x_k3x* h, const char* name, glm5x_k3x_tensor_info* info) {
  if (!h || !name || !info) return fail_global(GLM5X_INVALID_STATE, "null argument");
  const K3xTensor* t = k3x_lookup(h, name);
  if (!t) return fail_global(GLM5X_TENSOR_NOT_FOUND, "%s", name);
  glm5x_k3x_tensor_info r{};
  r.tensor_id = t->tensor_id;
  r.dtype = t->dtype;
  r.quantization = t->quantization;
  r.rank = t->rank;
  r.layer_id = t->layer_id;
  r.expert_id = t->expert_id;
  for (int d = 0; d < 4; ++d) r.dimensions[d] = t->dims[d];
  r.data_length = t->data_length;
  r.logical_length = t->logical_length;
  r.auxiliary_length = t->auxiliary_length;
  *info = r;
  return GLM5X_OK;
}

glm5x_status glm5x_k3x_read(const glm5x_k3x* h, const char* name, void* data, uint64_t data_cap,
                            void* aux, uint64_t aux_cap) {
  if (!h || !name || !data) return fail_global(GLM5X_INVALID_STATE, "null argument");
  const K3xTensor* t = k3x_lookup(h, name);
  if (!t) return fail_global(GLM5X_TENSOR_NOT_FOUND, "%s", name);
  if (data_cap < t->data_length || (aux && t->auxiliary_length && aux_cap < t->auxiliary_length))
    return fail_global(GLM5X_INVALID_EXTENT, "%s: buffer smaller than the extent", name);
  std::string msg;
  int rc = k3x_read_extent(h->file, t->data_offset, t->data_length,
                           static_cast<uint8_t*>(data), &msg);
  if (rc == 0 && aux && t->auxiliary_length)
    rc = k3x_read_extent(h->file, t->auxiliary_offset, t->auxiliary_length,
                         static_cast<uint8_t*>(aux), &msg);
  if (rc != 0) return fail_global(static_cast<glm5x_status>(rc), "%s: %s", name, msg.c_str());
  return GLM5X_OK;
}

glm5x_status glm5x_moe_load_expert_k3x(glm5x_moe* m, int32_t expert, const glm5x_k3x* h,
                                       const char* prefix) {
  if (!m || !h || !prefix) return fail_global(GLM5X_INVALID_STATE, "null argument");
  static const char* roles[3] = {"gate", "up", "down"};
  std::vector<uint8_t> packed[3], scales[3];
  glm5x_mxfp4_matrix mats[3];
  for (int r = 0; r < 3; ++r) {
    const std::string name = std::string(prefix) + "." + roles[r];
    const K3xTensor* t = k3x_lookup(h, name.c_str());
    if (!t) return m->fail(GLM5X_TENSOR_NOT_FOUND, "%s", name.c_str());
    if (t->dtype != 2 || t->quantization != 1 || t->rank != 2)
      return m->fail(GLM5X_INVALID_MXFP4, "%s is not a rank-2 MXFP4 record", name.c_str());
    const uint64_t rows = t->dims[0], cols = t->dims[1];
    if (cols % 32 || t->data_length != rows * cols / 2 || t->auxiliary_length != rows * cols / 32)
      return m->fail(GLM5X_INVALID_EXTENT, "%s: extents do not match [%llu, %llu]", name.c_str(),
                     (unsigned long long)rows, (unsigned long long)cols);
    packed[r].resize(t->data_length);
    scales[r].resize(t->auxiliary_length);
    std::string msg;
    int rc = k3x_read_extent(h->file, t->data_offset, t->data_length, packed[r].data(), &msg);
    if (rc == 0)
      rc = k3x_read_extent(h->file, t->auxiliary_offset, t->auxiliary_length, scales[r].data(),
                           &msg);
    if (rc != 0) return m->fail(static_cast<glm5x_status>(rc), "%s: %s", name.c_str(), msg.c_str());
    mats[r] = glm5x_mxfp4_matrix{packed[r].data(), scales[r].data(), (int64_t)rows,
                                 (int64_t)cols, 32};
  }
  return glm5x_moe_load_expert_mxfp4(m, expert, &mats[0], &mats[1], &mats[2]);
}

glm5x_status glm5x_moe_load_expert_sidecar(glm5x_moe* m, int32_t expert,
                                           const glm5x_sidecar* sc) {
  if (!m || !sc) return fail_global(GLM5X_INVALID_STATE, "null argument");
  glm5x_sidecar_role ro[3];
  for (int r = 0; r < 3; ++r)
    if (glm5x_sidecar_get_role(sc, r, &ro[r]) != GLM5X_OK)
      return m->fail(GLM5X_INVALID_STATE, "sidecar role %d unreadable", r);
  if (ro[0].precision != m->cfg.precision)
    return m->fail(GLM5X_INVALID_STATE, "GLM5X_PACKED_CACHE_FORMAT: sidecar is %s, engine is %s",
                   ro[0].precision == 0 ? "NVFP4" : "MXFP4", m->mx() ? "MXFP4" : "NVFP4");
  if (ro[0].precision == GLM5X_PRECISION_NVFP4) {
    glm5x_nvfp4_matrix mats[3];
    for (int r = 0; r < 3; ++r) {
      if (ro[r].group_size != 16) return m->fail(GLM5X_INVALID_EXTENT, "NVFP4 group size must be 16");
      const int64_t expect = ((ro[r].rows + 127) / 128) * ((ro[r].cols / 16 + 3) / 4) * 512;
      if (ro[r].scale_bytes != expect)
        return m->fail(GLM5X_INVALID_EXTENT, "NVFP4 blocked scale size mismatch");
      mats[r] = glm5x_nvfp4_matrix{ro[r].packed, ro[r].scales, ro[r].global_scale, ro[r].rows,
                                   ro[r].cols};
    }
    return glm5x_moe_load_expert_nvfp4(m, expert, &mats[0], &mats[1], &mats[2]);
  }
  glm5x_mxfp4_matrix mats[3];
  for (int r = 0; r < 3; ++r) {
    if (ro[r].group_size <= 0 || ro[r].scale_bytes != ro[r].rows * ro[r].cols / ro[r].group_size)
      return m->fail(GLM5X_INVALID_EXTENT, "MXFP4 scale size mismatch");
    mats[r] = glm5x_mxfp4_matrix{ro[r].packed, ro[r].scales, ro[r].rows, ro[r].cols,
                                 ro[r].group_size};
  }
  return glm5x_moe_load_expert_mxfp4(m, expert, &mats[0], &mats[1], &mats[2]);
}

glm5x_status glm5x_moe_load_sidecar(glm5x_moe* m, int32_t expert, const char* path) {
  if (!m || !path) return fail_global(GLM5X_INVALID_STATE, "null argument");
  glm5x_sidecar* sc = nullptr;
  const glm5x_status rc = glm5x_sidecar_open(path, m->cfg.precision, nullptr, &sc);
  if (rc != GLM5X_OK) return m->fail(rc, "%s", glm5x_last_error_message());
  const glm5x_status st = glm5x_moe_load_expert_sidecar(m, expert, sc);
  glm5x_sidecar_close(sc);
  return st;
}

// ep_rows: the rows are tokens dispatched to this engine by expert-parallel
// ranks; ids_in holds global expert ids, slots of experts held elsewhere are
// skipped, and only rows < shared_rows take the shared expert.
// Rows quantized by their senders (expert-parallel FP4 dispatch): R rows of
// one held expert each, placed after the T local tokens (which take only the
// shared expert); outputs the local tokens' shared-expert rows and, per
// group of received rows (one source token), the sum of their weighted
// expert rows.
// Rows written into this engine's input by expert-parallel peers
// (glm5x_moe_ep_forward): the input holds local_cap local-token rows (the
// first local_tokens of them valid; they take the shared expert) and then
// the received rows, whose count the device knows (recv_count) but the host
// does not; ids of rows past it are -1. Outputs: the local tokens' rows
// (FP32, `out`) and each received row's weighted expert sum as BF16, stored
// into its source's memory as `ret` describes (the last block then raises the
// sources' flags); rows' max |x| come from their senders.
struct PeerRows {
  int64_t local_cap;
  int64_t local_tokens;
  const float* row_amax;      // [rows] (NVFP4 engines)
  const int32_t* recv_count;  // device: received rows
  const RowReturn* ret;
};

struct PrequantRows {
  const uint8_t* packed;      // [R, H/2] E2M1 codes
  const uint8_t* scales;      // [R, H/16] E4M3, row-major
  const int32_t* row_expert;  // [R] global expert ids (held by this engine)
  const float* row_weight;    // [R]
  int64_t R;
  const float* amax;          // [num_experts] slab amax reduced over all ranks
  const int32_t* group_rows;  // [groups, slots] received row indices, -1 = none
  int64_t groups;
  int slots;
  float* out_groups;          // [groups, H]
};

static glm5x_status run_forward(glm5x_moe* m, const uint16_t* x, int64_t T64,
                                const int32_t* ids_in, const float* w_in, float* out,
                                cudaStream_t st, bool ep_rows = false, int64_t shared_rows = -1,
                                const PrequantRows* pq = nullptr,
                                const PeerRows* peer = nullptr) {
  if (pq && (pq->R < 0 || T64 + pq->R > m->cfg.max_tokens || m->mx()))
    return m->fail(GLM5X_INVALID_EXTENT, "local tokens + received rows exceed max_tokens (or MXFP4)");
  // an expert-parallel rank without local tokens still runs the rows it received
  const bool rows_only = pq && T64 == 0 && pq->R > 0;
  if ((T64 <= 0 && !rows_only) || T64 > m->cfg.max_tokens)
    return m->fail(GLM5X_INVALID_EXTENT, "tokens %lld outside [1, %d]", (long long)T64,
                   m->cfg.max_tokens);
  if (!ep_rows && m->E_loc != m->cfg.num_experts)
    return m->fail(GLM5X_INVALID_STATE,
                   "expert-parallel engines run glm5x_moe_forward_expert_rows");
  if (ep_rows && !ids_in && !pq) return m->fail(GLM5X_INVALID_STATE, "expert rows need ids");
  for (int s = 0; s < m->nseg; ++s)
    if (!m->loaded[s]) return m->fail(GLM5X_INVALID_STATE, "expert slot %d not loaded", s);
  if (!ids_in && !pq && !m->router_set) return m->fail(GLM5X_INVALID_STATE, "router not set");
  const int T = static_cast<int>(T64);
  const int H = m->H(), I = m->I(), E = m->cfg.num_experts;
  // with sender-quantized rows: T + R one-slot rows (local tokens' slot empty)
  const int k = pq ? 1 : m->K();
  const int N = pq ? T + static_cast<int>(pq->R) : T;
  const int E_perm = ep_rows ? m->E_loc : E;  // segments the permutation builds
  const int hs = m->cfg.has_shared ? 1 : 0;
  int bn = pick_bn(m, N);
  // tiles narrower than 128 rows each take a 128-row block: make sure the
  // worst case still fits the workspace, else use 128-row tiles
  const bool mx = m->mx();
  if (bn < 128 && (int64_t)(128 / bn) * N * m->kk() * m->terms() + (int64_t)m->nseg * 128 >
                      m->rows_cap) {
    if (m->force_bn) return m->fail(GLM5X_INVALID_EXTENT, "token tile %d too narrow for %d tokens", bn, T);
    bn = 128;
  }
  uint64_t launches = 0;
  const int pslot = m->prof_slot;
  if (m->profiling) m->accumulate_slot(pslot);  // the ring wrapped onto an unread slot
  auto mark = [&](int phase) {
    if (m->profiling) cudaEventRecord(m->ev[pslot][phase], st);
  };
  mark(0);
  const float* row_amax = m->token_amax;
  // the tensor-core router reads every token row anyway: it takes the
  // per-token amax on the way (no separate pass over the batch)
  const bool router_runs = !ids_in && !pq;
  const bool amax_in_router = !mx && !(peer && peer->row_amax) && router_runs;
  if (!mx && peer && peer->row_amax) {
    row_amax = peer->row_amax;  // computed by the senders while they sent the rows
  } else if (!mx && !amax_in_router) {
    // per-token amax for the NVFP4 slab global scales (MXFP4 has none; its
    // term kernel checks for non-finite inputs itself)
    G5_CHECK(m, launch_row_amax_bf16(x, T, H, m->token_amax, m->err, st), "row amax");
    ++launches;
    if (pq && pq->R > 0)  // received rows carry no amax here: their slabs' scales are given
      G5_CHECK(m, cudaMemsetAsync(m->token_amax + T, 0, sizeof(float) * pq->R, st), "row amax");
  }
  mark(1);
  const int32_t* ids = ids_in;
  const float* wts = w_in;
  if (router_runs) {
    if (reinterpret_cast<uintptr_t>(x) % 16)
      return m->fail(GLM5X_INVALID_EXTENT, "hidden must be 16-byte aligned");
    CUtensorMap tm_x;
    if (!make_tmap_bf16(&tm_x, x, H, T, 128))
      return m->fail(GLM5X_BACKEND_UNAVAILABLE, "hidden tensor map");
    int rl = 0;
    const bool diag = m->policy.mode != 0 || m->routing_diag;
    G5_CHECK(m, launch_router_tc(&tm_x, &m->tm_router, m->router_bias, T, H, E, k,
                                 m->cfg.routed_scaling, m->logits, m->topk_ids, m->topk_w, m->err,
                                 st, m->router_partials, m->num_sms, &rl, m->policy,
                                 diag ? m->route_sel : nullptr, diag ? m->route_diag : nullptr,
                                 amax_in_router ? m->token_amax : nullptr),
             "router");
    m->route_T = diag ? T : 0;
    launches += rl;
    ids = m->topk_ids;
    wts = m->topk_w;
  }
  mark(2);
  mark(3);
  if (pq) {
    // rows [0, T): local tokens, no routed slot; rows [T, N): one held expert
    G5_CHECK(m, cudaMemsetAsync(m->ids_local, 0xFF, sizeof(int32_t) * T, st), "local ids");
    G5_CHECK(m, launch_map_local_ids(pq->row_expert, pq->R, m->cfg.expert_begin, m->E_loc,
                                     m->ids_local + T, st),
             "local ids");
    G5_CHECK(m, cudaMemsetAsync(m->topk_w, 0, sizeof(float) * T, st), "row weights");
    if (pq->R > 0)
      G5_CHECK(m, cudaMemcpyAsync(m->topk_w + T, pq->row_weight, sizeof(float) * pq->R,
                                  cudaMemcpyDeviceToDevice, st),
               "row weights");
    ids = m->ids_local;
    wts = m->topk_w;
    ++launches;
  } else if (ep_rows) {
    G5_CHECK(m, launch_map_local_ids(ids_in, (int64_t)T * k, m->cfg.expert_begin, m->E_loc,
                                     m->ids_local, st),
             "local ids");
    ids = m->ids_local;
    ++launches;
  }
  int pl = 0;
  G5_CHECK(m, launch_permute(ids, wts, row_amax, N, k, E_perm, hs, bn, m->pb, m->err, st,
                             m->terms(), ep_rows ? 1 : 2,
                             pq ? T : (shared_rows < 0 ? -1 : (int)std::min<int64_t>(shared_rows, T)),
                             &pl),
           "permute");
  launches += pl;
  const int64_t max_rows = (int64_t)N * m->kk() + (int64_t)m->nseg * 8;
  mark(4);
  if (mx) {
    // MXFP4 experts take full-precision activations in the reference; the
    // tensor cores get four MXFP4 residual terms per activation row
    G5_CHECK(m, launch_mxfp4_terms_segments(x, H, m->pb.row_token, m->pb.seg_start,
                                            m->pb.seg_count, m->pb.qprefix, m->nseg, bn, max_rows,
                                            m->act_packed, m->act_sf, m->err, st),
             "activation terms");
  } else if (pq) {
    // the shared expert's slab from the local tokens, the routed slabs from
    // the senders' rows
    G5_CHECK(m, launch_nvfp4_quantize_segments(x, H, m->pb.row_token, m->pb.seg_start,
                                               m->pb.seg_count, m->pb.qprefix, m->nseg, bn,
                                               m->pb.seg_amax, max_rows, m->act_packed,
                                               m->act_sf, m->act_global, st, m->E_loc),
             "activation quantize");
    G5_CHECK(m, launch_place_nvfp4_rows(pq->packed, pq->scales, H, m->pb.row_token, T,
                                        m->pb.seg_start, m->pb.seg_count, m->pb.qprefix,
                                        m->E_loc, bn, pq->amax, m->cfg.expert_begin, max_rows,
                                        m->act_packed, m->act_sf, m->act_global, st),
             "received rows");
    ++launches;
  } else {
    G5_CHECK(m, launch_nvfp4_quantize_segments(x, H, m->pb.row_token, m->pb.seg_start,
                                               m->pb.seg_count, m->pb.qprefix, m->nseg, bn,
                                               m->pb.seg_amax, max_rows, m->act_packed,
                                               m->act_sf, m->act_global, st),
             "activation quantize");
  }
  GemmParams g1{};
  g1.a_packed = m->w13_packed;
  g1.b_packed = m->act_packed;
  g1.sfa = m->w13_sf;
  g1.sfb = m->act_sf;
  g1.seg_count = m->pb.seg_count;
  g1.seg_start = m->pb.seg_start;
  g1.ntile_prefix = m->pb.ntile_prefix;
  g1.a_global = mx ? m->ones : m->w13_global;
  g1.b_global = mx ? m->ones : m->act_global;
  g1.out = m->h_bf16;
  g1.h_amax = m->pb.h_amax;
  g1.err = m->err;
  g1.K = H;
  g1.M_per = 2 * I;
  g1.nseg = m->nseg;
  g1.tile_group = m->tile_group_up;
  mark(5);
  const bool pair = !mx && bn == 256 && m->use_pair && m->pair_grid >= 2;
  G5_CHECK(m,
           pair ? launch_nvfp4_pair_gemm(0, &m->tm_w13, m->tm_act, &m->tm_w13_sf, &m->tm_act_sf,
                                         g1, m->pair_grid, st, m->pair_wide)
                : launch_nvfp4_grouped_gemm(bn, 0, &m->tm_w13, m->tm_act, g1, m->num_sms, st,
                                            mx ? 1 : 0, m->weight_rows),
           "gate/up GEMM");
  mark(6);
  if (mx) {
    G5_CHECK(m, launch_mxfp4_terms_segments(m->h_bf16, I, nullptr, m->pb.seg_start,
                                            m->pb.seg_count, m->pb.qprefix, m->nseg, bn, max_rows,
                                            m->h_packed, m->h_sf, m->err, st),
             "h terms");
  } else {
    G5_CHECK(m, launch_nvfp4_quantize_segments(m->h_bf16, I, nullptr, m->pb.seg_start,
                                               m->pb.seg_count, m->pb.qprefix, m->nseg, bn,
                                               m->pb.h_amax, max_rows, m->h_packed, m->h_sf,
                                               m->h_global, st),
             "h quantize");
  }
  GemmParams g2 = g1;
  g2.a_packed = m->w2_packed;
  g2.b_packed = m->h_packed;
  g2.sfa = m->w2_sf;
  g2.sfb = m->h_sf;
  g2.a_global = mx ? m->ones : m->w2_global;
  g2.b_global = mx ? m->ones : m->h_global;
  g2.row_weight = m->pb.row_weight;
  g2.out = m->y_bf16;
  g2.h_amax = nullptr;
  g2.K = I;
  g2.M_per = H;
  g2.tile_group = m->tile_group_down;
  mark(7);
  // Large batches (token tiles >= 128 rows): token-major down projection,
  // whose epilogue stores each token's output features contiguously.
  const bool token_major = !mx && !pair && bn >= 128 && m->token_major_down && H % 256 == 0;
  if (token_major) {
    GemmParams g2t = g2;
    g2t.a_packed = m->h_packed;
    g2t.b_packed = m->w2_packed;
    g2t.sfa = m->h_sf;
    g2t.sfb = m->w2_sf;
    const CUtensorMap tw[3] = {m->tm_w2, m->tm_w2, m->tm_w2};
    G5_CHECK(m, launch_nvfp4_grouped_gemm(256, 2, &m->tm_h[2], tw, g2t, m->num_sms, st),
             "down GEMM");
  } else if (!mx && !pair && bn >= 128 && m->down_bn >= 128 && m->down_bn != bn) {
    // another tile width >= 128 for the down projection (its own tile prefix)
    GemmParams g2w = g2;
    g2w.ntile_prefix = nullptr;
    G5_CHECK(m, launch_nvfp4_grouped_gemm(m->down_bn, 1, &m->tm_w2, m->tm_h, g2w, m->num_sms, st),
             "down GEMM");
  } else {
    G5_CHECK(m,
             pair ? launch_nvfp4_pair_gemm(1, &m->tm_w2, m->tm_h, &m->tm_w2_sf, &m->tm_h_sf, g2,
                                           m->pair_grid, st, m->pair_wide)
                  : launch_nvfp4_grouped_gemm(bn, 1, &m->tm_w2, m->tm_h, g2, m->num_sms, st,
                                              mx ? 1 : 0, m->weight_rows),
             "down GEMM");
  }
  mark(8);
  if (peer) {
    // local tokens: their shared-expert rows (FP32); received rows: their
    // weighted expert sums, BF16, for the senders to pull back
    G5_CHECK(m, launch_combine(m->y_bf16, m->pb.pos, (int)peer->local_tokens, m->kk(), H, out, st),
             "combine");
    G5_CHECK(m, launch_combine_rows_return(m->y_bf16, m->pb.pos + peer->local_cap * m->kk(),
                                           N - peer->local_cap, peer->recv_count, m->kk(), H,
                                           *peer->ret, st),
             "partial sums");
    ++launches;
  } else if (pq) {
    // local tokens: their shared-expert rows; received rows: per group
    G5_CHECK(m, launch_combine(m->y_bf16, m->pb.pos, T, 1 + hs, H, out, st), "combine");
    const int64_t n = pq->groups * pq->slots;
    G5_CHECK(m, launch_map_group_pos(pq->group_rows, n, m->pb.pos, 1 + hs, T, m->ids_local, st),
             "group rows");
    if (pq->groups > 0)
      G5_CHECK(m, launch_combine(m->y_bf16, m->ids_local, (int)pq->groups, pq->slots, H,
                                 pq->out_groups, st),
               "group combine");
    launches += 2;
  } else {
    G5_CHECK(m, launch_combine(m->y_bf16, m->pb.pos, T, m->kk(), H, out, st), "combine");
  }
  mark(9);
  if (m->profiling) {
    m->prof_pending[pslot] = true;
    m->prof_slot = (pslot + 1) % glm5x_moe::kProfRing;
  }
  launches += 5;
  m->stats.forward_calls++;
  m->stats.kernel_launches += launches;
  m->last_T = T;
  m->last_bn = bn;
  m->routed_last = ids_in == nullptr && !pq;
  return GLM5X_OK;
}


extern "C++" {
namespace glm5x {
// Expert forward over rows peers wrote into this engine's input (see
// PeerRows); used by the expert-parallel engine in ep_peer.cu.
glm5x_status engine_forward_peer_rows(glm5x_moe* m, const uint16_t* rows, int64_t local_cap,
                                      int64_t local_tokens, int64_t recv_cap,
                                      const int32_t* ids, const float* weights,
                                      const float* row_amax, const int32_t* recv_count,
                                      float* out_local, const RowReturn* ret, cudaStream_t st) {
  if (local_tokens < 0 || local_tokens > local_cap || recv_cap < 0)
    return m->fail(GLM5X_INVALID_EXTENT, "peer rows: bad extents");
  cudaSetDevice(m->device);
  PeerRows pr{local_cap, local_tokens, row_amax, recv_count, ret};
  return run_forward(m, rows, local_cap + recv_cap, ids, weights, out_local, st, true,
                     local_tokens, nullptr, &pr);
}

glm5x_status engine_fail(glm5x_moe* m, glm5x_status st, const char* msg) {
  return m->fail(st, "%s", msg);
}

int engine_device(const glm5x_moe* m) { return m->device; }
int engine_num_sms(const glm5x_moe* m) { return m->num_sms; }
}  // namespace glm5x
}  // extern "C++"

glm5x_status glm5x_moe_forward(glm5x_moe* m, const void* hidden, int64_t T, float* out,
                               void* stream) {
  if (!m || !hidden || !out) return fail_global(GLM5X_INVALID_STATE, "null argument");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  return run_forward(m, static_cast<const uint16_t*>(hidden), T, nullptr, nullptr, out, st);
}

glm5x_status glm5x_moe_forward_routed(glm5x_moe* m, const void* hidden, int64_t T,
                                      const int32_t* ids, const float* weights, float* out,
                                      void* stream) {
  if (!m || !hidden || !out || !ids || !weights)
    return fail_global(GLM5X_INVALID_STATE, "null argument");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  return run_forward(m, static_cast<const uint16_t*>(hidden), T, ids, weights, out, st);
}

glm5x_status glm5x_moe_forward_expert_rows(glm5x_moe* m, const void* rows, int64_t R,
                                           const int32_t* ids, const float* weights,
                                           int64_t shared_rows, float* out, void* stream) {
  if (!m || !rows || !out || !ids || !weights)
    return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (shared_rows < 0 || shared_rows > R)
    return m->fail(GLM5X_INVALID_EXTENT, "shared_rows outside [0, rows]");
  if (shared_rows > 0 && !m->cfg.has_shared)
    return m->fail(GLM5X_INVALID_STATE, "engine has no shared expert");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  return run_forward(m, static_cast<const uint16_t*>(rows), R, ids, weights, out, st, true,
                     shared_rows);
}

glm5x_status glm5x_moe_slab_amax(glm5x_moe* m, const void* hidden, int64_t T, const int32_t* ids,
                                 float* amax, void* stream) {
  if (!m || !hidden || !ids || !amax) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (m->mx()) return m->fail(GLM5X_INVALID_STATE, "slab amax: NVFP4 engines only");
  if (reinterpret_cast<uintptr_t>(hidden) % 16)
    return m->fail(GLM5X_INVALID_EXTENT, "hidden must be 16-byte aligned");
  if (T <= 0 || T > m->cfg.max_tokens)
    return m->fail(GLM5X_INVALID_EXTENT, "tokens %lld outside [1, %d]", (long long)T,
                   m->cfg.max_tokens);
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  G5_CHECK(m, launch_row_amax_bf16(static_cast<const uint16_t*>(hidden), T, m->H(), m->token_amax,
                                   m->err, st),
           "row amax");
  G5_CHECK(m, launch_slab_amax(m->token_amax, ids, (int)T, m->K(), m->cfg.num_experts, amax, st),
           "slab amax");
  m->stats.kernel_launches += 2;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_quantize_rows(glm5x_moe* m, const void* hidden, int64_t T,
                                     const int32_t* row_token, const int32_t* row_expert,
                                     int64_t n, const float* amax, void* packed, void* scales,
                                     void* stream) {
  if (!m || !hidden || !amax || (n > 0 && (!row_token || !row_expert || !packed || !scales)))
    return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (m->mx()) return m->fail(GLM5X_INVALID_STATE, "row quantization: NVFP4 engines only");
  if (T <= 0 || n < 0 || reinterpret_cast<uintptr_t>(hidden) % 16)
    return m->fail(GLM5X_INVALID_EXTENT, "bad row quantization extents");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  G5_CHECK(m, launch_nvfp4_quantize_rows(static_cast<const uint16_t*>(hidden), m->H(), row_token,
                                         row_expert, n, amax, static_cast<uint8_t*>(packed),
                                         static_cast<uint8_t*>(scales), st),
           "row quantize");
  m->stats.kernel_launches += n > 0 ? 1 : 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_forward_quantized_rows(
    glm5x_moe* m, const void* hidden, int64_t T, const void* packed, const void* scales,
    const int32_t* row_expert, const float* row_weight, int64_t R, const float* amax,
    float* out_local, const int32_t* group_rows, int64_t groups, int32_t slots,
    float* out_groups, void* stream) {
  if (!m || (T > 0 && (!hidden || !out_local)) || !amax ||
      (R > 0 && (!packed || !scales || !row_expert || !row_weight)) ||
      (groups > 0 && (!group_rows || !out_groups)))
    return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (R < 0 || groups < 0 || groups > R || slots <= 0 || slots > 32)
    return m->fail(GLM5X_INVALID_EXTENT, "bad received-row extents");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  PrequantRows pq{static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scales),
                  row_expert, row_weight, R, amax, group_rows, groups, slots, out_groups};
  return run_forward(m, static_cast<const uint16_t*>(hidden), T, nullptr, nullptr, out_local, st,
                     true, T, &pq);
}

glm5x_status glm5x_moe_route(glm5x_moe* m, const void* hidden, int64_t T, int32_t* ids,
                             float* weights, float* logits, void* stream) {
  if (!m || !hidden || !ids || !weights) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (!m->router_set) return m->fail(GLM5X_INVALID_STATE, "router not set");
  if (T <= 0 || T > m->cfg.max_tokens)
    return m->fail(GLM5X_INVALID_EXTENT, "tokens %lld outside [1, %d]", (long long)T,
                   m->cfg.max_tokens);
  if (reinterpret_cast<uintptr_t>(hidden) % 16)
    return m->fail(GLM5X_INVALID_EXTENT, "hidden must be 16-byte aligned");
  cudaSetDevice(m->device);
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  CUtensorMap tm_x;
  if (!make_tmap_bf16(&tm_x, hidden, m->H(), T, 128))
    return m->fail(GLM5X_BACKEND_UNAVAILABLE, "hidden tensor map");
  int rl = 0;
  const bool diag = m->policy.mode != 0 || m->routing_diag;
  G5_CHECK(m, launch_router_tc(&tm_x, &m->tm_router, m->router_bias, (int)T, m->H(),
                               m->cfg.num_experts, m->K(), m->cfg.routed_scaling,
                               logits ? logits : m->logits, ids, weights, m->err, st,
                               m->router_partials, m->num_sms, &rl, m->policy,
                               diag ? m->route_sel : nullptr, diag ? m->route_diag : nullptr),
           "router");
  m->route_T = diag ? T : 0;
  m->stats.kernel_launches += rl;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_forward_host(glm5x_moe* m, const uint16_t* hidden, int64_t T,
                                    float* out) {
  if (!m || !hidden || !out) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (T <= 0 || T > m->cfg.max_tokens)
    return m->fail(GLM5X_INVALID_EXTENT, "tokens outside [1, max_tokens]");
  cudaSetDevice(m->device);
  const size_t in_bytes = sizeof(uint16_t) * T * m->H(), out_bytes = sizeof(float) * T * m->H();
  G5_CHECK(m, cudaMemcpyAsync(m->stage_in, hidden, in_bytes, cudaMemcpyHostToDevice, m->stream),
           "hidden upload");
  glm5x_status s = run_forward(m, m->stage_in, T, nullptr, nullptr, m->stage_out, m->stream);
  if (s != GLM5X_OK) return s;
  G5_CHECK(m, cudaMemcpyAsync(out, m->stage_out, out_bytes, cudaMemcpyDeviceToHost, m->stream),
           "output download");
  G5_CHECK(m, cudaStreamSynchronize(m->stream), "forward");
  m->stats.activation_h2d_bytes += in_bytes;
  m->stats.device_to_host_bytes += out_bytes;
  m->stats.stream_synchronization_count++;
  return glm5x_moe_check(m);
}

static glm5x_status error_word_status(glm5x_moe* m, uint32_t e) {
  if (!e) return GLM5X_OK;
  if (e & kErrWaitTimeout) return m->fail(GLM5X_WAIT_TIMEOUT, "device wait timed out (0x%x)", e);
  if (e & kErrNonFinite) return m->fail(GLM5X_INVALID_STATE, "non-finite input (0x%x)", e);
  if (e & kErrBounds) return m->fail(GLM5X_INVALID_EXTENT, "routing ids invalid (0x%x)", e);
  if (e & kErrRoutingMass) return m->fail(GLM5X_INVALID_STATE, "zero routing mass (0x%x)", e);
  return m->fail(GLM5X_DEVICE_ERROR, "device error word 0x%x", e);
}

glm5x_status glm5x_moe_check(glm5x_moe* m) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaDeviceSynchronize(), "device synchronize");
  uint32_t e = 0;
  G5_CHECK(m, cudaMemcpy(&e, m->err, sizeof e, cudaMemcpyDeviceToHost), "error word");
  if (e) cudaMemset(m->err, 0, sizeof(uint32_t));
  return error_word_status(m, e);
}

// Staging slots, streams and events of the pipelined host API, made on its
// first use so engines that never call it hold none of them.
static glm5x_status pipe_init(glm5x_moe* m) {
  if (m->pipe_ready) return GLM5X_OK;
  const size_t n = (size_t)m->cfg.max_tokens * m->H();
  bool ok = true;
  for (int b = 0; b < 2; ++b) {
    if (!m->pipe_in[b]) ok = ok && m->alloc(&m->pipe_in[b], n);
    if (!m->pipe_out[b]) ok = ok && m->alloc(&m->pipe_out[b], n);
  }
  if (!m->err_snap) ok = ok && m->alloc(&m->err_snap, glm5x_moe::kTicketRing);
  if (!ok) return m->fail(GLM5X_OUT_OF_MEMORY, "pipelined staging buffers");
  if (!m->err_host)
    G5_CHECK(m, cudaHostAlloc(&m->err_host, sizeof(uint32_t) * glm5x_moe::kTicketRing,
                              cudaHostAllocDefault),
             "page-locked error words");
  for (cudaStream_t* s : {&m->up_stream, &m->down_stream})
    if (!*s) G5_CHECK(m, cudaStreamCreateWithFlags(s, cudaStreamNonBlocking), "copy stream");
  for (int i = 0; i < glm5x_moe::kTicketRing; ++i) {
    for (cudaEvent_t* e : {&m->up_done[i], &m->comp_done[i], &m->down_done[i]})
      if (!*e) G5_CHECK(m, cudaEventCreateWithFlags(e, cudaEventDisableTiming), "event create");
    m->ticket_of[i] = -1;
  }
  m->pipe_ready = true;
  return GLM5X_OK;
}

// Ticket t uses staging slot t % 2 and ring entry t % kTicketRing. Its upload
// waits until the forward of ticket t - 2 has read the slot's input, its
// forward until the download of ticket t - 2 has read the slot's output, and
// its download until its own forward is done, so the upload of one batch, the
// forward of the previous one and the download of the one before can run at
// the same time. The error word is copied and cleared after each forward so
// every ticket reports the device errors of its own kernels.
glm5x_status glm5x_moe_submit_host(glm5x_moe* m, const uint16_t* hidden, int64_t T, float* out,
                                   int64_t* ticket) {
  if (!m || !hidden || !out || !ticket) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (T <= 0 || T > m->cfg.max_tokens)
    return m->fail(GLM5X_INVALID_EXTENT, "tokens outside [1, max_tokens]");
  cudaSetDevice(m->device);
  glm5x_status s = pipe_init(m);
  if (s != GLM5X_OK) return s;
  const int64_t t = m->next_ticket;
  const int b = (int)(t & 1), r = (int)(t % glm5x_moe::kTicketRing);
  const int rp = (int)((t + glm5x_moe::kTicketRing - 2) % glm5x_moe::kTicketRing);
  const size_t in_bytes = sizeof(uint16_t) * T * m->H(), out_bytes = sizeof(float) * T * m->H();
  if (t >= 2) G5_CHECK(m, cudaStreamWaitEvent(m->up_stream, m->comp_done[rp], 0), "upload order");
  G5_CHECK(m, cudaMemcpyAsync(m->pipe_in[b], hidden, in_bytes, cudaMemcpyHostToDevice,
                              m->up_stream),
           "hidden upload");
  G5_CHECK(m, cudaEventRecord(m->up_done[r], m->up_stream), "event record");
  G5_CHECK(m, cudaStreamWaitEvent(m->stream, m->up_done[r], 0), "forward order");
  if (t >= 2) G5_CHECK(m, cudaStreamWaitEvent(m->stream, m->down_done[rp], 0), "forward order");
  s = run_forward(m, m->pipe_in[b], T, nullptr, nullptr, m->pipe_out[b], m->stream);
  if (s == GLM5X_OK) {
    const cudaError_t ce = launch_error_snapshot(m->err, m->err_snap + r, m->stream);
    if (ce != cudaSuccess) s = cuda_fail(m, ce, "error word snapshot");
    m->stats.kernel_launches += 1;
  }
  // the events are recorded on failure too, so the next submission of this
  // ticket number orders itself after whatever this one launched
  G5_CHECK(m, cudaEventRecord(m->comp_done[r], m->stream), "event record");
  G5_CHECK(m, cudaStreamWaitEvent(m->down_stream, m->comp_done[r], 0), "download order");
  if (s == GLM5X_OK) {
    G5_CHECK(m, cudaMemcpyAsync(out, m->pipe_out[b], out_bytes, cudaMemcpyDeviceToHost,
                                m->down_stream),
             "output download");
    G5_CHECK(m, cudaMemcpyAsync(m->err_host + r, m->err_snap + r, sizeof(uint32_t),
                                cudaMemcpyDeviceToHost, m->down_stream),
             "error word download");
  }
  G5_CHECK(m, cudaEventRecord(m->down_done[r], m->down_stream), "event record");
  if (s != GLM5X_OK) return s;
  m->ticket_of[r] = t;
  m->next_ticket = t + 1;
  m->stats.activation_h2d_bytes += in_bytes;
  m->stats.device_to_host_bytes += out_bytes;
  *ticket = t;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_read_ints(glm5x_moe* m, const int64_t* src, int64_t n, int64_t* dst,
                                 void* stream) {
  if (!m || (n > 0 && (!src || !dst))) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (n < 0 || n > glm5x_moe::kHostInts)
    return m->fail(GLM5X_INVALID_EXTENT, "read_ints: n outside [0, %lld]",
                   (long long)glm5x_moe::kHostInts);
  if (n == 0) return GLM5X_OK;
  cudaSetDevice(m->device);
  if (!m->host_ints) {
    G5_CHECK(m, cudaHostAlloc(&m->host_ints, sizeof(int64_t) * glm5x_moe::kHostInts,
                              cudaHostAllocMapped),
             "mapped host words");
    void* d = nullptr;
    G5_CHECK(m, cudaHostGetDevicePointer(&d, m->host_ints, 0), "mapped host words");
    m->host_ints_dev = static_cast<int64_t*>(d);
  }
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : m->stream;
  G5_CHECK(m, launch_store_ints_to_host(src, n, m->host_ints_dev, st), "read_ints");
  m->stats.kernel_launches += 1;
  G5_CHECK(m, cudaStreamSynchronize(st), "read_ints");
  m->stats.stream_synchronization_count++;
  std::memcpy(dst, m->host_ints, sizeof(int64_t) * n);
  return GLM5X_OK;
}

glm5x_status glm5x_moe_wait_host(glm5x_moe* m, int64_t t) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (!m->pipe_ready || t < 0 || t >= m->next_ticket)
    return m->fail(GLM5X_INVALID_STATE, "ticket %lld was not submitted", (long long)t);
  const int r = (int)(t % glm5x_moe::kTicketRing);
  if (m->ticket_of[r] != t)
    return m->fail(GLM5X_INVALID_STATE, "ticket %lld is older than the last %d submissions",
                   (long long)t, glm5x_moe::kTicketRing);
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaEventSynchronize(m->down_done[r]), "pipelined forward");
  m->stats.stream_synchronization_count++;
  return error_word_status(m, m->err_host[r]);
}

glm5x_status glm5x_moe_last_routing(glm5x_moe* m, int32_t* ids, float* weights, float* logits,
                                    int64_t T) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (!m->routed_last || T != m->last_T)
    return m->fail(GLM5X_INVALID_STATE, "no routed forward with %lld tokens", (long long)T);
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaStreamSynchronize(m->stream), "sync");
  const int k = m->K();
  if (ids) G5_CHECK(m, cudaMemcpy(ids, m->topk_ids, sizeof(int32_t) * T * k, cudaMemcpyDeviceToHost), "ids");
  if (weights) G5_CHECK(m, cudaMemcpy(weights, m->topk_w, sizeof(float) * T * k, cudaMemcpyDeviceToHost), "w");
  if (logits)
    G5_CHECK(m, cudaMemcpy(logits, m->logits, sizeof(float) * T * m->cfg.num_experts,
                           cudaMemcpyDeviceToHost), "logits");
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_routing_policy(glm5x_moe* m, const glm5x_routing_policy* p) {
  if (!m || !p) return fail_global(GLM5X_INVALID_STATE, "null argument");
  if (const char* why = routing_policy_error(*p, m->K())) return m->fail(GLM5X_INVALID_STATE, "%s", why);
  m->policy = to_device_policy(*p);
  m->routing_diag = p->collect_diagnostics != 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_routing_decisions(glm5x_moe* m, int64_t T, int32_t* sel, float* diag) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (m->route_T <= 0 || T != m->route_T)
    return m->fail(GLM5X_INVALID_STATE, "no router pass with diagnostics over %lld tokens",
                   (long long)T);
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaDeviceSynchronize(), "sync");
  if (sel)
    G5_CHECK(m, cudaMemcpy(sel, m->route_sel, sizeof(int32_t) * 2 * T, cudaMemcpyDeviceToHost),
             "routing decisions");
  if (diag)
    G5_CHECK(m, cudaMemcpy(diag, m->route_diag, sizeof(float) * 4 * T, cudaMemcpyDeviceToHost),
             "routing diagnostics");
  return GLM5X_OK;
}

glm5x_status glm5x_moe_routing_stats(glm5x_moe* m, glm5x_routing_stats* out) {
  if (!m || !out) return fail_global(GLM5X_INVALID_STATE, "null argument");
  const int64_t T = m->route_T;
  if (T <= 0) return m->fail(GLM5X_INVALID_STATE, "no router pass with diagnostics");
  std::vector<int32_t> sel(2 * T);
  std::vector<float> diag(4 * T);
  glm5x_status st = glm5x_moe_routing_decisions(m, T, sel.data(), diag.data());
  if (st != GLM5X_OK) return st;
  glm5x_routing_stats r{};
  r.decisions = (uint64_t)T;
  for (int64_t t = 0; t < T; ++t) {
    r.selected_experts += (uint64_t)sel[2 * t];
    r.quality_escalated_decisions += sel[2 * t + 1] ? 1u : 0u;
    r.normalized_entropy_sum += diag[4 * t];
    r.selected_mass_sum += diag[4 * t + 2];
    r.boundary_confidence_sum += diag[4 * t + 3];
  }
  *out = r;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_get_stats(const glm5x_moe* m, glm5x_moe_stats* out) {
  if (!m || !out) return fail_global(GLM5X_INVALID_STATE, "null argument");
  *out = m->stats;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_debug_buffer(glm5x_moe* m, int32_t which, void** ptr, size_t* bytes) {
  if (!m || !ptr || !bytes) return fail_global(GLM5X_INVALID_STATE, "null argument");
  const int64_t R = m->rows_cap, H = m->H(), I = m->I();
  const int64_t rb = R / 128 + 2;
  switch (which) {
    case 0: *ptr = m->act_packed; *bytes = R * H / 2; break;
    case 1: *ptr = m->act_sf; *bytes = rb * (H / 64) * 512; break;
    case 2: *ptr = m->act_global; *bytes = sizeof(float) * m->nseg; break;
    case 3: *ptr = m->h_bf16; *bytes = R * I * 2; break;
    case 4: *ptr = m->h_packed; *bytes = R * I / 2; break;
    case 5: *ptr = m->h_sf; *bytes = rb * (I / 64) * 512; break;
    case 6: *ptr = m->h_global; *bytes = sizeof(float) * m->nseg; break;
    case 7: *ptr = m->y_bf16; *bytes = R * H * 2; break;
    case 8: *ptr = m->pb.seg_start; *bytes = sizeof(int32_t) * (m->nseg + 1); break;
    case 9: *ptr = m->pb.seg_count; *bytes = sizeof(int32_t) * m->nseg; break;
    case 10: *ptr = m->pb.row_token; *bytes = sizeof(int32_t) * R; break;
    case 11: *ptr = m->pb.pos; *bytes = sizeof(int32_t) * m->cfg.max_tokens * m->kk(); break;
    case 12: *ptr = m->pb.row_weight; *bytes = sizeof(float) * R; break;
    default: return m->fail(GLM5X_INVALID_EXTENT, "unknown debug buffer %d", which);
  }
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_profiling(glm5x_moe* m, int32_t enable) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  cudaSetDevice(m->device);
  if (enable && !m->ev[0][0]) {
    for (auto& row : m->ev)
      for (auto& e : row) G5_CHECK(m, cudaEventCreate(&e), "event create");
  }
  m->profiling = enable != 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_phase_times(glm5x_moe* m, float* ms, int32_t* forwards) {
  if (!m || !ms) return fail_global(GLM5X_INVALID_STATE, "null argument");
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaDeviceSynchronize(), "sync");
  for (int k = 0; k < glm5x_moe::kProfRing; ++k) m->accumulate_slot((m->prof_slot + k) % glm5x_moe::kProfRing);
  for (int i = 0; i < GLM5X_NUM_PHASES; ++i) {
    ms[i] = static_cast<float>(m->phase_ms[i]);
    m->phase_ms[i] = 0.0;
  }
  if (forwards) *forwards = m->profiled;
  m->profiled = 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_tile_n(glm5x_moe* m, int32_t bn) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (bn != 0 && bn != 32 && bn != 64 && bn != 128 && bn != 256)
    return m->fail(GLM5X_INVALID_EXTENT, "token tile must be 0, 32, 64, 128 or 256");
  m->force_bn = bn;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_pair_mma(glm5x_moe* m, int32_t enable) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  m->use_pair = enable != 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_token_major_down(glm5x_moe* m, int32_t enable) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  m->token_major_down = enable != 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_pair_wide_stages(glm5x_moe* m, int32_t enable) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  m->pair_wide = enable ? 1 : 0;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_pair_tile_order(glm5x_moe* m, int32_t up_group, int32_t down_group) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (up_group < 0 || down_group < 0)
    return m->fail(GLM5X_INVALID_EXTENT, "tile group sizes must be >= 0");
  m->tile_group_up = up_group;
  m->tile_group_down = down_group;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_weight_tile_rows(glm5x_moe* m, int32_t rows) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (rows != 128 && rows != 256)
    return m->fail(GLM5X_INVALID_EXTENT, "weight tile rows must be 128 or 256");
  if (rows == 256 && (m->H() % 256 || (2 * m->I()) % 256))
    return m->fail(GLM5X_INVALID_EXTENT, "256-row weight tiles need hidden and 2 x intermediate "
                                         "multiples of 256");
  m->weight_rows = rows;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_set_down_tile_n(glm5x_moe* m, int32_t bn) {
  if (!m) return fail_global(GLM5X_INVALID_STATE, "null engine");
  if (bn != 0 && bn != 128 && bn != 256)
    return m->fail(GLM5X_INVALID_EXTENT, "down tile must be 0, 128 or 256");
  m->down_bn = bn;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_get_stream(glm5x_moe* m, void** stream) {
  if (!m || !stream) return fail_global(GLM5X_INVALID_STATE, "null argument");
  *stream = m->stream;
  return GLM5X_OK;
}

glm5x_status glm5x_moe_debug_copy(glm5x_moe* m, int32_t which, void* dst, size_t bytes) {
  void* src = nullptr;
  size_t size = 0;
  glm5x_status st = glm5x_moe_debug_buffer(m, which, &src, &size);
  if (st != GLM5X_OK) return st;
  if (!dst || bytes > size) return m->fail(GLM5X_INVALID_EXTENT, "debug copy larger than buffer");
  cudaSetDevice(m->device);
  G5_CHECK(m, cudaStreamSynchronize(m->stream), "sync");
  G5_CHECK(m, cudaMemcpy(dst, src, bytes, cudaMemcpyDeviceToDevice), "debug copy");
  return GLM5X_OK;
}

// ============================================================== kernel API
}  // extern "C"

static cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }


static glm5x_status sync_error(cudaStream_t st, uint32_t* err_dev, uint32_t mask_invalid,
                               const char* what) {
  cudaError_t e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail_global(GLM5X_DEVICE_ERROR, "%s: %s", what, cudaGetErrorString(e));
  uint32_t w = 0;
  cudaMemcpy(&w, err_dev, sizeof w, cudaMemcpyDeviceToHost);
  cudaFree(err_dev);
  if (w & mask_invalid) return fail_global(GLM5X_INVALID_MXFP4, "%s: invalid input (0x%x)", what, w);
  if (w) return fail_global(GLM5X_INVALID_STATE, "%s: device error 0x%x", what, w);
  return GLM5X_OK;
}

template <typename T>
static glm5x_status nvfp4_quantize_any(const T* src, int64_t rows, int64_t cols, int32_t mode,
                                       uint8_t* packed, uint8_t* scales, float* g, void* stream) {
  if (!src || !packed || !scales || !g) return fail_global(GLM5X_INVALID_EXTENT, "null pointer");
  if (rows <= 0 || cols <= 0 || cols % 16)
    return fail_global(GLM5X_INVALID_EXTENT, "NVFP4 needs cols to be a positive multiple of 16");
  uint32_t* err = nullptr;
  float* amax = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess || cudaMalloc(&amax, 4) != cudaSuccess)
    return fail_global(GLM5X_OUT_OF_MEMORY, "scratch allocation");
  cudaStream_t st = as_stream(stream);
  cudaMemsetAsync(err, 0, 4, st);
  cudaError_t e = launch_nvfp4_quantize_matrix<T>(src, rows, cols, mode, amax, packed, scales, g,
                                                  err, st);
  if (e != cudaSuccess) return fail_global(GLM5X_DEVICE_ERROR, "quantize: %s", cudaGetErrorString(e));
  glm5x_status s = sync_error(st, err, 0, "nvfp4 quantize");
  cudaFree(amax);
  return s;
}

extern "C" {
glm5x_status glm5x_nvfp4_quantize_f32(const float* src, int64_t rows, int64_t cols,
                                      int32_t mode, uint8_t* packed, uint8_t* scales,
                                      float* g, void* stream) {
  return nvfp4_quantize_any<float>(src, rows, cols, mode, packed, scales, g, stream);
}

glm5x_status glm5x_nvfp4_quantize_bf16(const uint16_t* src, int64_t rows, int64_t cols,
                                       int32_t mode, uint8_t* packed, uint8_t* scales,
                                       float* g, void* stream) {
  return nvfp4_quantize_any<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(src), rows,
                                           cols, mode, packed, scales, g, stream);
}

glm5x_status glm5x_nvfp4_quantize_slabs_bf16(const uint16_t* src, int64_t cols,
                                             const int32_t* row_token, const int32_t* seg_start,
                                             const int32_t* seg_count, int32_t nseg,
                                             int64_t out_rows, uint8_t* packed,
                                             uint8_t* scales, float* seg_global, void* stream) {
  if (!src || !row_token || !seg_start || !seg_count || !packed || !scales || !seg_global)
    return fail_global(GLM5X_INVALID_EXTENT, "null pointer");
  if (cols <= 0 || cols % 512 || nseg <= 0 || nseg > 1024 || out_rows <= 0)
    return fail_global(GLM5X_INVALID_EXTENT, "slab quantize: bad extents");
  cudaStream_t st = as_stream(stream);
  // segment bookkeeping on the host: counts rounded to 8, amax per segment
  std::vector<int32_t> cnt(nseg), start(nseg + 1);
  cudaMemcpy(cnt.data(), seg_count, sizeof(int32_t) * nseg, cudaMemcpyDeviceToHost);
  cudaMemcpy(start.data(), seg_start, sizeof(int32_t) * (nseg + 1), cudaMemcpyDeviceToHost);
  std::vector<int32_t> q(nseg + 1, 0);
  for (int s = 0; s < nseg; ++s) {
    if (cnt[s] < 0 || start[s] % 128 || start[s] + (cnt[s] + 7) / 8 * 8 > out_rows)
      return fail_global(GLM5X_INVALID_EXTENT, "segment %d out of range", s);
    q[s + 1] = q[s] + (cnt[s] + 7) / 8 * 8;
  }
  std::vector<int32_t> tok(out_rows);
  cudaMemcpy(tok.data(), row_token, sizeof(int32_t) * out_rows, cudaMemcpyDeviceToHost);
  int32_t max_tok = 0;
  for (int s = 0; s < nseg; ++s)
    for (int r = 0; r < cnt[s]; ++r) max_tok = std::max(max_tok, tok[start[s] + r]);
  // per-token amax, then per-segment max
  float *tok_amax = nullptr, *seg_amax = nullptr;
  int32_t* qp = nullptr;
  uint32_t* err = nullptr;
  cudaMalloc(&tok_amax, sizeof(float) * (max_tok + 1));
  cudaMalloc(&seg_amax, sizeof(float) * nseg);
  cudaMalloc(&qp, sizeof(int32_t) * (nseg + 1));
  cudaMalloc(&err, 4);
  cudaMemsetAsync(err, 0, 4, st);
  launch_row_amax_bf16(src, max_tok + 1, (int)cols, tok_amax, err, st);
  std::vector<float> ta(max_tok + 1), sa(nseg, 0.0f);
  cudaMemcpyAsync(ta.data(), tok_amax, sizeof(float) * (max_tok + 1), cudaMemcpyDeviceToHost, st);
  cudaStreamSynchronize(st);
  for (int s = 0; s < nseg; ++s)
    for (int r = 0; r < cnt[s]; ++r) sa[s] = std::max(sa[s], ta[tok[start[s] + r]]);
  cudaMemcpyAsync(seg_amax, sa.data(), sizeof(float) * nseg, cudaMemcpyHostToDevice, st);
  cudaMemcpyAsync(qp, q.data(), sizeof(int32_t) * (nseg + 1), cudaMemcpyHostToDevice, st);
  cudaError_t e = launch_nvfp4_quantize_segments(src, (int)cols, row_token, seg_start, seg_count,
                                                 qp, nseg, 256, seg_amax, q[nseg], packed, scales,
                                                 seg_global, st);
  glm5x_status s = e == cudaSuccess ? sync_error(st, err, 0, "slab quantize")
                                    : fail_global(GLM5X_DEVICE_ERROR, "slab quantize launch");
  cudaFree(tok_amax);
  cudaFree(seg_amax);
  cudaFree(qp);
  cudaFree(err);
  return s;
}

glm5x_status glm5x_nvfp4_dequantize(const uint8_t* packed, const uint8_t* scales, float g,
                                    int64_t rows, int64_t cols, float* out, void* stream) {
  if (!packed || !scales || !out || rows <= 0 || cols <= 0 || cols % 16)
    return fail_global(GLM5X_INVALID_EXTENT, "dequantize: bad arguments");
  cudaError_t e = launch_nvfp4_dequantize(packed, scales, g, rows, cols, out, as_stream(stream));
  return e == cudaSuccess ? GLM5X_OK : fail_global(GLM5X_DEVICE_ERROR, "dequantize launch");
}

glm5x_status glm5x_mxfp4_encode_f32(const float* src, int64_t rows, int64_t cols,
                                    int64_t group, int32_t mode, uint8_t* packed,
                                    uint8_t* scales, void* stream) {
  if (!src || !packed || !scales || rows <= 0 || cols <= 0 || group <= 0 || group > 64 ||
      cols % group || cols % 2)
    return fail_global(GLM5X_INVALID_MXFP4, "cols must align to group_size and nibble pairs");
  uint32_t* err = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess) return fail_global(GLM5X_OUT_OF_MEMORY, "scratch");
  cudaStream_t st = as_stream(stream);
  cudaMemsetAsync(err, 0, 4, st);
  launch_mxfp4_encode<float>(src, rows * cols, (int)group, mode, packed, scales, err, st);
  return sync_error(st, err, kErrBadScale | kErrNonFinite, "mxfp4 encode");
}

glm5x_status glm5x_mxfp4_decode(const uint8_t* packed, const uint8_t* scales, int64_t rows,
                                int64_t cols, int64_t group, float* out, void* stream) {
  if (!packed || !scales || !out || rows <= 0 || cols <= 0 || group <= 0 || cols % group ||
      cols % 2)
    return fail_global(GLM5X_INVALID_MXFP4, "cols must align to group_size and nibble pairs");
  uint32_t* err = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess) return fail_global(GLM5X_OUT_OF_MEMORY, "scratch");
  cudaStream_t st = as_stream(stream);
  cudaMemsetAsync(err, 0, 4, st);
  launch_mxfp4_decode(packed, scales, rows * cols, (int)group, out, err, st);
  return sync_error(st, err, kErrBadScale, "mxfp4 decode");
}

glm5x_status glm5x_select_routing(const float* scores, const float* bias, int64_t T, int32_t E,
                                  int32_t k, float scale, int32_t* ids, float* weights,
                                  void* stream) {
  if (!scores || !bias || !ids || !weights || T <= 0 || E <= 0 || E > 512 || k <= 0 || k > 16 ||
      k > E)
    return fail_global(GLM5X_INVALID_STATE, "invalid routing dimensions");
  uint32_t* err = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess) return fail_global(GLM5X_OUT_OF_MEMORY, "scratch");
  cudaStream_t st = as_stream(stream);
  cudaMemsetAsync(err, 0, 4, st);
  launch_topk(scores, 1, bias, (int)T, E, k, scale, ids, weights, err, st);
  return sync_error(st, err, 0, "select routing");
}

glm5x_status glm5x_read_bf16_activation(const char* path, uint32_t expected_tokens,
                                        uint32_t expected_hidden, uint32_t* tokens,
                                        uint32_t* hidden, uint16_t* out, uint64_t out_elems) {
  if (!path) return fail_global(GLM5X_INVALID_STATE, "null path");
  ActivationHeader hdr;
  std::string msg;
  const int rc = out ? read_activation(path, expected_tokens, expected_hidden, &hdr, out,
                                       out_elems, &msg)
                     : read_activation_header(path, expected_tokens, expected_hidden, &hdr, &msg);
  if (rc != 0) return fail_global(static_cast<glm5x_status>(rc), "%s", msg.c_str());
  if (tokens) *tokens = hdr.tokens;
  if (hidden) *hidden = hdr.hidden;
  return GLM5X_OK;
}

glm5x_status glm5x_write_bf16_activation(const char* path, const uint16_t* data,
                                         uint32_t tokens, uint32_t hidden) {
  if (!path || !data) return fail_global(GLM5X_INVALID_STATE, "null argument");
  std::string msg;
  const int rc = write_activation(path, data, tokens, hidden, &msg);
  if (rc != 0) return fail_global(static_cast<glm5x_status>(rc), "%s", msg.c_str());
  return GLM5X_OK;
}

glm5x_status glm5x_select_routing_policy(const float* scores, const float* bias, int64_t T,
                                         int32_t E, int32_t k, const glm5x_routing_policy* p,
                                         float scale, int32_t* ids, float* weights,
                                         int32_t* sel, float* diag, void* stream) {
  if (!scores || !bias || !ids || !weights || !p || T <= 0 || E <= 0 || E > 512 || k <= 0 ||
      k > 16 || k > E)
    return fail_global(GLM5X_INVALID_STATE, "invalid routing dimensions");
  if (const char* why = routing_policy_error(*p, k)) return fail_global(GLM5X_INVALID_STATE, "%s", why);
  uint32_t* err = nullptr;
  if (cudaMalloc(&err, 4) != cudaSuccess) return fail_global(GLM5X_OUT_OF_MEMORY, "scratch");
  cudaStream_t st = as_stream(stream);
  cudaMemsetAsync(err, 0, 4, st);
  launch_topk(scores, 1, bias, (int)T, E, k, scale, ids, weights, err, st, to_device_policy(*p),
              sel, diag);
  return sync_error(st, err, 0, "select routing");
}

glm5x_status glm5x_verify_greedy_target_blocks(const uint32_t* anchors, const uint32_t* candidates,
                                               const int32_t* draft_counts,
                                               const uint32_t* targets, int64_t S,
                                               int32_t max_draft, uint32_t vocab,
                                               int32_t* accepted, uint32_t* committed,
                                               int32_t* status, void* stream) {
  if (!anchors || !draft_counts || !targets || !accepted || !committed || !status || S <= 0 ||
      max_draft < 0 || (max_draft > 0 && !candidates))
    return fail_global(GLM5X_INVALID_STATE, "verify: null buffer or bad sizes");
  if (vocab == 0) return fail_global(GLM5X_INVALID_EXTENT, "verify: empty vocabulary");
  if (launch_verify_greedy_blocks(anchors, candidates, draft_counts, targets, S, max_draft, vocab,
                                  accepted, committed, status, as_stream(stream)) != cudaSuccess)
    return fail_global(GLM5X_DEVICE_ERROR, "verify launch");
  return GLM5X_OK;
}

glm5x_status glm5x_combine_rows(const void* rows_bf16, const int32_t* pos, int64_t T,
                                int32_t slots, int64_t hidden, float* out, int32_t accumulate,
                                void* stream) {
  if (!rows_bf16 || !pos || !out || T <= 0 || slots <= 0 || slots > 32 || hidden <= 0 ||
      hidden % 8)
    return fail_global(GLM5X_INVALID_EXTENT, "combine_rows: bad extents or null pointer");
  if (launch_combine(static_cast<const uint16_t*>(rows_bf16), pos, (int)T, slots, (int)hidden,
                     out, as_stream(stream), accumulate ? 1 : 0) != cudaSuccess)
    return fail_global(GLM5X_DEVICE_ERROR, "combine_rows launch");
  return GLM5X_OK;
}

glm5x_status glm5x_expert_major_plan(const int32_t* ids, int64_t T, int32_t k, int32_t E,
                                     int32_t* seg_count, int32_t* seg_start, int32_t* pos,
                                     int32_t* row_token, void* stream) {
  if (!ids || !seg_count || !seg_start || !pos || !row_token || T <= 0 || k <= 0 || k > 16 ||
      E <= 0 || E > 256)
    return fail_global(GLM5X_INVALID_EXTENT, "invalid plan dimensions");
  cudaStream_t st = as_stream(stream);
  PermuteBuffers b{};
  const int nchunks = (int)((T + 255) / 256);
  float* wts = nullptr;
  float* amax = nullptr;
  uint32_t* err = nullptr;
  bool ok = cudaMalloc(&b.chunk_count, sizeof(int32_t) * nchunks * E) == cudaSuccess &&
            cudaMalloc(&b.rank, sizeof(int32_t) * T * k) == cudaSuccess &&
            cudaMalloc(&b.qprefix, sizeof(int32_t) * (E + 1)) == cudaSuccess &&
            cudaMalloc(&b.ntile_prefix, sizeof(int32_t) * (E + 1)) == cudaSuccess &&
            cudaMalloc(&b.seg_amax, sizeof(float) * E) == cudaSuccess &&
            cudaMalloc(&b.h_amax, sizeof(float) * E) == cudaSuccess &&
            cudaMalloc(&b.row_weight, sizeof(float) * (T * k + E * 128)) == cudaSuccess &&
            cudaMalloc(&wts, sizeof(float) * T * k) == cudaSuccess &&
            cudaMalloc(&amax, sizeof(float) * T) == cudaSuccess &&
            cudaMalloc(&err, 4) == cudaSuccess;
  glm5x_status s = GLM5X_OK;
  if (!ok) {
    s = fail_global(GLM5X_OUT_OF_MEMORY, "plan scratch");
  } else {
    b.seg_count = seg_count;
    b.seg_start = seg_start;
    b.pos = pos;
    b.row_token = row_token;
    cudaMemsetAsync(wts, 0, sizeof(float) * T * k, st);
    cudaMemsetAsync(amax, 0, sizeof(float) * T, st);
    cudaMemsetAsync(err, 0, 4, st);
    launch_permute(ids, wts, amax, (int)T, k, E, 0, 256, b, err, st);
    s = sync_error(st, err, 0, "expert-major plan");
    err = nullptr;
  }
  cudaFree(b.chunk_count);
  cudaFree(b.rank);
  cudaFree(b.qprefix);
  cudaFree(b.ntile_prefix);
  cudaFree(b.seg_amax);
  cudaFree(b.h_amax);
  cudaFree(b.row_weight);
  cudaFree(wts);
  cudaFree(amax);
  if (err) cudaFree(err);
  return s;
}

}  // extern "C"
