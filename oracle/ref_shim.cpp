// ref_shim.cpp -- TEST INFRASTRUCTURE ONLY.
//
// A C-ABI shim over the reference's own C++ CPU implementation of the MoE
// expert path. oracle/Makefile compiles this file together with the
// reference's sources where they lie (runtime/src/{routing_policy,
// expert_major,ops,backend_cpu,profile}.cpp) into oracle/_ref/libk3x_ref.so.
// Used by tests (to pin the C restatement in glm5x_oracle.c) and by bench.py's
// `--impl reference` / cpu_baseline legs (the reference's CPU expert path).
#include "k3x/backend.hpp"
#include "k3x/expert_major.hpp"
#include "k3x/ops.hpp"
#include "k3x/routing_policy.hpp"
#include "k3x/reader.hpp"
#include "k3x/speculative.hpp"

#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <span>
#include <vector>

namespace {
std::unique_ptr<k3x::ComputeBackend>& cpu() {
  static thread_local std::unique_ptr<k3x::ComputeBackend> backend = k3x::make_cpu_backend();
  return backend;
}
}  // namespace

extern "C" {

// k3x::select_routing natural mode (runtime/src/routing_policy.cpp:31-159).
int ref_select_routing(const float* scores, const float* bias, int n, int k, int32_t* ids,
                       float* weights) {
  auto r = k3x::select_routing(std::span<const float>(scores, n), std::span<const float>(bias, n),
                               static_cast<std::size_t>(k),
                               k3x::RoutingPolicyConfig{.mode = k3x::RoutingMode::natural});
  if (!r) return -1;
  for (int s = 0; s < k; ++s) {
    ids[s] = static_cast<int32_t>(r.value().expert_ids[s]);
    weights[s] = r.value().normalized_weights[s];
  }
  return 0;
}

// k3x::select_routing with a policy (runtime/src/routing_policy.cpp:31-159):
// ids / weights [k] (-1 / 0 past the selected K), sel [2], diag [4] as
// orc_select_routing_policy.
int ref_select_routing_policy(const float* scores, const float* bias, int n, int k, int mode,
                              int fixed_k, float mass_target, float min_gap, int floor_k,
                              int32_t* ids, float* weights, int32_t* sel, float* diag) {
  k3x::RoutingPolicyConfig cfg{};
  cfg.mode = mode == 1 ? k3x::RoutingMode::fixed
                       : (mode == 2 ? k3x::RoutingMode::adaptive : k3x::RoutingMode::natural);
  cfg.fixed_k = static_cast<std::size_t>(fixed_k);
  cfg.mass_target = mass_target;
  cfg.minimum_boundary_gap = min_gap;
  cfg.quality_floor_k = static_cast<std::size_t>(floor_k);
  auto r = k3x::select_routing(std::span<const float>(scores, n), std::span<const float>(bias, n),
                               static_cast<std::size_t>(k), cfg);
  if (!r) return -1;
  const auto& d = r.value();
  for (int s = 0; s < k; ++s) {
    const bool on = static_cast<std::size_t>(s) < d.selected_k;
    ids[s] = on ? static_cast<int32_t>(d.expert_ids[s]) : -1;
    weights[s] = on ? d.normalized_weights[s] : 0.0f;
  }
  sel[0] = static_cast<int32_t>(d.selected_k);
  sel[1] = d.quality_floor_escalated ? 1 : 0;
  diag[0] = d.normalized_entropy;
  diag[1] = d.entropy_effective_support;
  diag[2] = d.selected_cumulative_mass;
  diag[3] = d.boundary_confidence;
  return 0;
}

// k3x::Reader::open (runtime/src/reader.cpp:420-702): the ErrorCode value,
// verify = the checksums mode.
int ref_k3x_open(const char* path, int verify) {
  auto r = k3x::Reader::open(path, verify ? k3x::VerifyMode::checksums
                                          : k3x::VerifyMode::metadata_only);
  return r ? 0 : static_cast<int>(r.error());
}

// Reader::read_tensor / read_auxiliary (runtime/src/reader.cpp:749-778) of the
// tensor with the given id, metadata-only open; lengths in *data_len / *aux_len.
int ref_k3x_read(const char* path, uint64_t tensor_id, uint8_t* data, uint64_t data_cap,
                 uint8_t* aux, uint64_t aux_cap, uint64_t* data_len, uint64_t* aux_len) {
  auto r = k3x::Reader::open(path, k3x::VerifyMode::metadata_only);
  if (!r) return static_cast<int>(r.error());
  auto d = r.value().read_tensor(tensor_id);
  if (!d) return static_cast<int>(d.error());
  *data_len = d.value().size();
  if (*data_len > data_cap) return -1;
  std::memcpy(data, d.value().data(), *data_len);
  *aux_len = 0;
  for (const auto& t : r.value().tensors()) {
    if (t.tensor_id != tensor_id || !t.auxiliary_length) continue;
    auto a = r.value().read_auxiliary(tensor_id);
    if (!a) return static_cast<int>(a.error());
    *aux_len = a.value().size();
    if (*aux_len > aux_cap) return -1;
    std::memcpy(aux, a.value().data(), *aux_len);
  }
  return 0;
}

// k3x::verify_greedy_target_block (runtime/src/speculative.cpp:75-113):
// 0 (committed / accepted filled) or the ErrorCode value.
int ref_verify_greedy_target_block(uint32_t anchor, const uint32_t* candidates, int n,
                                   int max_draft, uint32_t vocab, const uint32_t* targets,
                                   int n_targets, int* accepted, uint32_t* committed) {
  k3x::DraftProposal p;
  p.anchor_token = anchor;
  p.candidate_tokens.assign(candidates, candidates + n);
  auto r = k3x::verify_greedy_target_block(
      p, static_cast<std::size_t>(max_draft), vocab,
      std::span<const std::uint32_t>(targets, static_cast<std::size_t>(n_targets)));
  if (!r) return static_cast<int>(r.error());
  *accepted = static_cast<int>(r.value().accepted_draft_tokens);
  for (std::size_t i = 0; i < r.value().committed_tokens.size(); ++i)
    committed[i] = r.value().committed_tokens[i];
  return 0;
}

// k3x::decode_mxfp4 (runtime/src/ops.cpp:40-63).
int ref_decode_mxfp4(const uint8_t* packed, const uint8_t* scales, int64_t rows, int64_t cols,
                     int64_t group, float* out) {
  auto r = k3x::decode_mxfp4(
      std::span<const std::byte>(reinterpret_cast<const std::byte*>(packed), rows * cols / 2),
      std::span<const std::byte>(reinterpret_cast<const std::byte*>(scales), rows * cols / group),
      rows, cols, group);
  if (!r) return -1;
  std::memcpy(out, r.value().data(), sizeof(float) * r.value().size());
  return 0;
}

// CpuBackend::dense_situ_mlp(..., MlpActivation::silu) (runtime/src/backend_cpu.cpp:107-128).
int ref_dense_silu_mlp(const float* x, const float* gate, const float* up, const float* down,
                       int64_t H, int64_t I, float* out) {
  k3x::DenseMlpView view{
      {1, std::span<const float>(gate, H * I), static_cast<std::size_t>(I), static_cast<std::size_t>(H)},
      {2, std::span<const float>(up, H * I), static_cast<std::size_t>(I), static_cast<std::size_t>(H)},
      {3, std::span<const float>(down, H * I), static_cast<std::size_t>(H), static_cast<std::size_t>(I)}};
  auto r = cpu()->dense_situ_mlp(std::span<const float>(x, H), view, 1.0F, std::nullopt, 0,
                                 k3x::ProfilePhase::decode, k3x::MlpActivation::silu);
  if (!r) return -1;
  std::memcpy(out, r.value().data(), sizeof(float) * H);
  return 0;
}

// k3x::build_expert_major_plan (runtime/src/expert_major.cpp:12-56). Writes
// groups in first-use order: group_expert[g], group_size[g]; and per
// assignment (group-major) token, slot and contribution. Returns the number
// of groups, or -1.
int ref_expert_major_plan(const int32_t* ids, const float* contributions, int T, int k,
                          int32_t* group_expert, int32_t* group_size, int32_t* a_token,
                          int32_t* a_slot, float* a_contrib) {
  std::vector<k3x::ExpertMajorTokenRoute> routes(T);
  for (int t = 0; t < T; ++t)
    for (int s = 0; s < k; ++s) {
      routes[t].expert_ids.push_back(static_cast<uint32_t>(ids[t * k + s]));
      routes[t].contributions.push_back(contributions[t * k + s]);
    }
  auto r = k3x::build_expert_major_plan(routes);
  if (!r) return -1;
  int a = 0;
  const auto& groups = r.value().groups;
  for (std::size_t g = 0; g < groups.size(); ++g) {
    group_expert[g] = static_cast<int32_t>(groups[g].expert_id);
    group_size[g] = static_cast<int32_t>(groups[g].assignments.size());
    for (const auto& as : groups[g].assignments) {
      a_token[a] = static_cast<int32_t>(as.token_index);
      a_slot[a] = static_cast<int32_t>(as.router_slot);
      a_contrib[a] = as.contribution;
      ++a;
    }
  }
  return static_cast<int>(groups.size());
}
}
