// k3x_b200_backend.hpp -- a k3x::ComputeBackend over the B200 MoE engine.
//
// Drop-in for the reference runtime's CUDA backend on its expert-major hot
// path (runtime/include/k3x/backend.hpp:170-294, make_cuda_backend :296-298):
// a maintainer adds this file to the reference build and returns
// make_b200_backend(...) where make_cuda_backend is used today. The routed
// expert MLPs of raw_bf16_situ_mlp_expert_major_with_shared (:228-236) with
// MlpActivation::silu run on libglm5x_moe.so (tcgen05 NVFP4 grouped GEMMs);
// every other virtual answers ErrorCode::backend_unavailable, as the
// reference's own base-class defaults do for what a backend does not offer.
//
// Residency follows the reference's ResidentWeightTable (keyed by tensor id,
// runtime/cuda/resident_weights.cuh:36-57): the first call that names an
// expert's gate tensor id packs its BF16 views to NVFP4 on the device
// (glm5x_moe_load_expert_bf16, the reference's NVFP4 packing) into the next
// free engine slot; later calls reuse it. Not thread-safe, like CudaBackend.
#pragma once

#include <cstdint>
#include <memory>
#include <string>
#include <unordered_map>

#include "k3x/backend.hpp"

struct glm5x_moe;

namespace glm5x_b200 {

struct B200BackendConfig {
    int device = 0;
    std::uint32_t hidden_size = 6144;
    std::uint32_t intermediate_size = 2048;
    std::uint32_t expert_slots = 256;   // routed experts resident at once
    std::uint32_t max_router_slots = 8; // largest router_slot + 1 in a plan
    std::uint32_t max_tokens = 8192;    // largest token_count per call
    bool mse_packing = true;            // quantize_nvfp4_weight's default scale_mode
};

class B200ComputeBackend final : public k3x::ComputeBackend {
public:
    static k3x::Result<std::unique_ptr<k3x::ComputeBackend>> create(
        const k3x::BackendOptions& options, const B200BackendConfig& config);
    ~B200ComputeBackend() override;

    k3x::BackendKind kind() const noexcept override { return k3x::BackendKind::cuda_custom; }
    const k3x::BackendOptions& options() const noexcept override { return options_; }
    k3x::BackendRuntimeStats runtime_stats() const noexcept override { return stats_; }
    k3x::BackendMemoryStats memory_stats() const noexcept override;
    std::string_view device_name() const noexcept override { return "NVIDIA B200 (sm_100a)"; }

    // hot path
    k3x::Result<std::vector<float>> raw_bf16_situ_mlp_expert_major_with_shared(
        std::span<const float> token_hidden, std::size_t token_count,
        const k3x::ExpertMajorPackedPlan& plan,
        std::span<const k3x::RawBf16MlpView> expert_views, k3x::RawBf16MlpView shared_view,
        float situ_beta, std::optional<float> situ_linear, std::uint32_t layer,
        k3x::ProfilePhase phase, k3x::MlpActivation activation) override;

    // not on this backend (backend_unavailable)
    k3x::Result<std::vector<float>> dense_matvec(std::span<const float>, k3x::DenseWeightView,
                                                 std::uint32_t, k3x::ProfilePhase) override;
    k3x::Result<std::vector<float>> mxfp4_matvec(std::span<const float>, k3x::Mxfp4WeightView,
                                                 std::uint32_t, k3x::ProfilePhase) override;
    k3x::Result<std::vector<std::vector<float>>> dense_matvec_group(
        std::span<const float>, std::span<const k3x::DenseWeightView>, std::uint32_t,
        k3x::ProfilePhase) override;
    k3x::Result<std::vector<std::vector<float>>> mxfp4_matvec_group(
        std::span<const float>, std::span<const k3x::Mxfp4WeightView>, std::uint32_t,
        k3x::ProfilePhase) override;
    k3x::Result<std::vector<float>> dense_situ_mlp(std::span<const float>, k3x::DenseMlpView,
                                                   float, std::optional<float>, std::uint32_t,
                                                   k3x::ProfilePhase,
                                                   k3x::MlpActivation) override;
    k3x::Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_group(
        std::span<const float>, std::span<const k3x::Mxfp4MlpView>, float, std::optional<float>,
        std::uint32_t, k3x::ProfilePhase) override;
    k3x::Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_batch(
        std::span<const float>, std::size_t, k3x::Mxfp4MlpView, float, std::optional<float>,
        std::uint32_t, k3x::ProfilePhase) override;
    k3x::Result<std::vector<float>> mxfp4_situ_moe(std::span<const float>,
                                                   std::span<const k3x::Mxfp4MlpView>,
                                                   std::span<const float>, float,
                                                   std::optional<float>, std::uint32_t,
                                                   k3x::ProfilePhase) override;
    k3x::Result<k3x::Mxfp4PrefetchToken> prefetch_mxfp4_situ_mlp_group(
        std::span<const k3x::Mxfp4MlpView>, std::uint64_t, std::uint32_t,
        k3x::ProfilePhase) override;
    k3x::Result<std::vector<std::vector<float>>> mxfp4_situ_mlp_group_prepared(
        std::span<const float>, k3x::Mxfp4PrefetchToken, float, std::optional<float>,
        std::uint32_t, k3x::ProfilePhase) override;
    k3x::Result<std::vector<float>> mxfp4_situ_moe_prepared(std::span<const float>,
                                                            k3x::Mxfp4PrefetchToken,
                                                            std::span<const float>, float,
                                                            std::optional<float>, std::uint32_t,
                                                            k3x::ProfilePhase) override;

private:
    B200ComputeBackend(const k3x::BackendOptions& options, const B200BackendConfig& config);
    // engine slot of an expert view (admitted on first use); -1 = the shared slot
    k3x::Result<int> resident_slot(const k3x::RawBf16MlpView& view, bool shared);

    k3x::BackendOptions options_;
    B200BackendConfig config_;
    glm5x_moe* engine_ = nullptr;
    std::unordered_map<std::uint64_t, int> slot_of_gate_id_;
    std::uint64_t shared_gate_id_ = 0;
    int next_slot_ = 0;
    // device buffers of one call (sized for max_tokens)
    void* d_hidden_ = nullptr;
    void* d_ids_ = nullptr;
    void* d_weights_ = nullptr;
    void* d_out_ = nullptr;
    k3x::BackendRuntimeStats stats_{};
};

// make_cuda_backend's counterpart (backend.hpp:296-298).
k3x::Result<std::unique_ptr<k3x::ComputeBackend>> make_b200_backend(
    const k3x::BackendOptions& options, const B200BackendConfig& config = {});

}  // namespace glm5x_b200
