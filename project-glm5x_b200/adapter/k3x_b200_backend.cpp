// k3x_b200_backend.cpp -- k3x::ComputeBackend over libglm5x_moe.so (see the
// header). Compiled against the reference runtime's headers.
#include "k3x_b200_backend.hpp"

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <limits>
#include <unordered_set>
#include <utility>

#include "glm5x_moe.h"

namespace glm5x_b200 {
namespace {

using k3x::ErrorCode;

template <typename T>
k3x::Result<T> unavailable(const char* what) {
    return k3x::Result<T>::failure(ErrorCode::backend_unavailable,
                                   std::string(what) + " is not offered by the B200 backend");
}

// glm5x_status keeps k3x::ErrorCode's numbering for 0..19; device-side
// failures (100+) surface as backend_unavailable.
ErrorCode to_error(glm5x_status st) {
    const int v = static_cast<int>(st);
    return v >= 0 && v <= 19 ? static_cast<ErrorCode>(v) : ErrorCode::backend_unavailable;
}

// FP32 -> BF16, round to nearest even (finite inputs; NaN stays NaN).
std::uint16_t to_bf16(float x) {
    std::uint32_t u;
    std::memcpy(&u, &x, 4);
    if ((u & 0x7F800000u) == 0x7F800000u) return static_cast<std::uint16_t>((u >> 16) | ((u & 0xFFFF) ? 0x40 : 0));
    u += 0x7FFFu + ((u >> 16) & 1u);
    return static_cast<std::uint16_t>(u >> 16);
}

bool view_ok(const k3x::RawBf16WeightView& v, std::size_t rows, std::size_t cols) {
    return v.tensor_id != 0 && v.rows == rows && v.cols == cols &&
           v.values.size() == rows * cols * 2;
}

}  // namespace

B200ComputeBackend::B200ComputeBackend(const k3x::BackendOptions& options,
                                       const B200BackendConfig& config)
    : options_(options), config_(config) {}

B200ComputeBackend::~B200ComputeBackend() {
    if (engine_) glm5x_moe_destroy(engine_);
    for (void* p : {d_hidden_, d_ids_, d_weights_, d_out_})
        if (p) cudaFree(p);
}

k3x::Result<std::unique_ptr<k3x::ComputeBackend>> B200ComputeBackend::create(
    const k3x::BackendOptions& options, const B200BackendConfig& config) {
    using R = k3x::Result<std::unique_ptr<k3x::ComputeBackend>>;
    std::unique_ptr<B200ComputeBackend> b(new B200ComputeBackend(options, config));
    glm5x_moe_config cfg{};
    cfg.hidden = static_cast<int32_t>(config.hidden_size);
    cfg.intermediate = static_cast<int32_t>(config.intermediate_size);
    cfg.num_experts = static_cast<int32_t>(config.expert_slots);
    cfg.top_k = static_cast<int32_t>(config.max_router_slots);
    cfg.has_shared = 1;
    cfg.routed_scaling = 1.0f;  // the plan carries final contributions
    cfg.precision = GLM5X_PRECISION_NVFP4;
    cfg.max_tokens = static_cast<int32_t>(config.max_tokens);
    cfg.expert_begin = 0;
    cfg.expert_count = cfg.num_experts;
    const glm5x_status st = glm5x_moe_create(&cfg, config.device, &b->engine_);
    if (st != GLM5X_OK) return R::failure(to_error(st), glm5x_last_error_message());
    const std::size_t T = config.max_tokens, H = config.hidden_size, K = config.max_router_slots;
    if (cudaSetDevice(config.device) != cudaSuccess ||
        cudaMalloc(&b->d_hidden_, T * H * 2) != cudaSuccess ||
        cudaMalloc(&b->d_ids_, T * K * 4) != cudaSuccess ||
        cudaMalloc(&b->d_weights_, T * K * 4) != cudaSuccess ||
        cudaMalloc(&b->d_out_, T * H * 4) != cudaSuccess)
        return R::failure(ErrorCode::backend_unavailable, "B200 backend buffers");
    b->stats_.device_allocation_count += 4;
    return R::success(std::unique_ptr<k3x::ComputeBackend>(b.release()));
}

k3x::BackendMemoryStats B200ComputeBackend::memory_stats() const noexcept {
    glm5x_moe_stats s{};
    glm5x_moe_get_stats(engine_, &s);
    k3x::BackendMemoryStats m{};
    m.current_device_bytes = s.workspace_bytes;
    m.peak_device_bytes = s.workspace_bytes;
    return m;
}

k3x::Result<int> B200ComputeBackend::resident_slot(const k3x::RawBf16MlpView& view,
                                                   bool shared) {
    using R = k3x::Result<int>;
    const std::size_t H = config_.hidden_size, I = config_.intermediate_size;
    if (!view_ok(view.gate, I, H) || !view_ok(view.up, I, H) || !view_ok(view.down, H, I))
        return R::failure(ErrorCode::invalid_extent, "expert view is not [I, H] / [H, I] BF16");
    const std::uint64_t id = view.gate.tensor_id;
    if (shared) {
        if (shared_gate_id_ == id) {
            stats_.weight_cache_hits++;
            return R::success(-1);
        }
    } else if (auto it = slot_of_gate_id_.find(id); it != slot_of_gate_id_.end()) {
        stats_.weight_cache_hits++;
        return R::success(it->second);
    }
    int slot = -1;
    if (!shared) {
        if (next_slot_ >= static_cast<int>(config_.expert_slots))
            return R::failure(ErrorCode::invalid_state, "all B200 expert slots are resident");
        slot = next_slot_;
    }
    const glm5x_status st = glm5x_moe_load_expert_bf16(
        engine_, slot, reinterpret_cast<const uint16_t*>(view.gate.values.data()),
        reinterpret_cast<const uint16_t*>(view.up.values.data()),
        reinterpret_cast<const uint16_t*>(view.down.values.data()),
        config_.mse_packing ? GLM5X_SCALE_MSE : GLM5X_SCALE_MAX_ABS);
    if (st != GLM5X_OK) return R::failure(to_error(st), glm5x_moe_error_message(engine_));
    stats_.weight_cache_misses++;
    stats_.stream_synchronization_count++;
    if (shared) {
        shared_gate_id_ = id;
    } else {
        slot_of_gate_id_.emplace(id, slot);
        ++next_slot_;
    }
    return R::success(slot);
}

k3x::Result<std::vector<float>> B200ComputeBackend::raw_bf16_situ_mlp_expert_major_with_shared(
    std::span<const float> token_hidden, std::size_t token_count,
    const k3x::ExpertMajorPackedPlan& plan, std::span<const k3x::RawBf16MlpView> expert_views,
    k3x::RawBf16MlpView shared_view, float, std::optional<float>, std::uint32_t,
    k3x::ProfilePhase, k3x::MlpActivation activation) {
    using R = k3x::Result<std::vector<float>>;
    if (activation != k3x::MlpActivation::silu)
        return unavailable<std::vector<float>>("the SiTU activation");
    const std::size_t H = config_.hidden_size, K = config_.max_router_slots;
    // the reference's checks of the same call (backend_cuda.cu:1566-1640)
    if (token_count == 0 || plan.hidden_size != H || token_hidden.size() != token_count * H ||
        plan.groups.empty() || plan.groups.size() != expert_views.size() ||
        plan.assignment_count == 0)
        return R::failure(ErrorCode::invalid_extent);
    if (token_count > config_.max_tokens)
        return R::failure(ErrorCode::invalid_extent, "token_count above the backend's max_tokens");
    std::unordered_set<std::uint64_t> routed_ids;
    for (const auto& v : expert_views)
        routed_ids.insert({v.gate.tensor_id, v.up.tensor_id, v.down.tensor_id});
    if (routed_ids.contains(shared_view.gate.tensor_id) ||
        routed_ids.contains(shared_view.up.tensor_id) ||
        routed_ids.contains(shared_view.down.tensor_id))
        return R::failure(ErrorCode::invalid_extent,
                          "shared GLM expert tensor id collides with routed expert");
    auto shared = resident_slot(shared_view, true);
    if (!shared) return R::failure(shared.error(), shared.message());
    // routes in the engine's form: ids / weights [T, K], the router slot as column
    std::vector<int32_t> ids(token_count * K, -1);
    std::vector<float> weights(token_count * K, 0.0f);
    std::size_t assignments = 0;
    for (std::size_t g = 0; g < plan.groups.size(); ++g) {
        auto slot = resident_slot(expert_views[g], false);
        if (!slot) return R::failure(slot.error(), slot.message());
        for (const auto& a : plan.groups[g].assignments) {
            if (a.token_index >= token_count || a.router_slot >= K ||
                !std::isfinite(a.contribution) || ids[a.token_index * K + a.router_slot] != -1)
                return R::failure(ErrorCode::invalid_extent, "assignment outside the plan");
            ids[a.token_index * K + a.router_slot] = slot.value();
            weights[a.token_index * K + a.router_slot] = a.contribution;
            ++assignments;
        }
    }
    if (assignments != plan.assignment_count) return R::failure(ErrorCode::invalid_extent);
    std::vector<std::uint16_t> x(token_count * H);
    for (std::size_t i = 0; i < x.size(); ++i) x[i] = to_bf16(token_hidden[i]);
    void* stream = nullptr;
    glm5x_moe_get_stream(engine_, &stream);
    auto st_ = static_cast<cudaStream_t>(stream);
    if (cudaMemcpyAsync(d_hidden_, x.data(), x.size() * 2, cudaMemcpyHostToDevice, st_) ||
        cudaMemcpyAsync(d_ids_, ids.data(), ids.size() * 4, cudaMemcpyHostToDevice, st_) ||
        cudaMemcpyAsync(d_weights_, weights.data(), weights.size() * 4, cudaMemcpyHostToDevice,
                        st_))
        return R::failure(ErrorCode::backend_unavailable, "B200 backend upload");
    const glm5x_status st = glm5x_moe_forward_routed(
        engine_, d_hidden_, static_cast<int64_t>(token_count), static_cast<int32_t*>(d_ids_),
        static_cast<float*>(d_weights_), static_cast<float*>(d_out_), stream);
    if (st != GLM5X_OK) return R::failure(to_error(st), glm5x_moe_error_message(engine_));
    std::vector<float> out(token_count * H);
    if (cudaMemcpyAsync(out.data(), d_out_, out.size() * 4, cudaMemcpyDeviceToHost, st_) ||
        cudaStreamSynchronize(st_))
        return R::failure(ErrorCode::backend_unavailable, "B200 backend download");
    stats_.stream_synchronization_count++;
    const glm5x_status chk = glm5x_moe_check(engine_);
    if (chk != GLM5X_OK) return R::failure(to_error(chk), glm5x_moe_error_message(engine_));
    return R::success(std::move(out));
}

// ---------------------------------------------------------------- not offered
k3x::Result<std::vector<float>> B200ComputeBackend::dense_matvec(std::span<const float>,
                                                                 k3x::DenseWeightView,
                                                                 std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<float>>("dense_matvec");
}
k3x::Result<std::vector<float>> B200ComputeBackend::mxfp4_matvec(std::span<const float>,
                                                                 k3x::Mxfp4WeightView,
                                                                 std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<float>>("mxfp4_matvec");
}
k3x::Result<std::vector<std::vector<float>>> B200ComputeBackend::dense_matvec_group(
    std::span<const float>, std::span<const k3x::DenseWeightView>, std::uint32_t,
    k3x::ProfilePhase) {
    return unavailable<std::vector<std::vector<float>>>("dense_matvec_group");
}
k3x::Result<std::vector<std::vector<float>>> B200ComputeBackend::mxfp4_matvec_group(
    std::span<const float>, std::span<const k3x::Mxfp4WeightView>, std::uint32_t,
    k3x::ProfilePhase) {
    return unavailable<std::vector<std::vector<float>>>("mxfp4_matvec_group");
}
k3x::Result<std::vector<float>> B200ComputeBackend::dense_situ_mlp(
    std::span<const float>, k3x::DenseMlpView, float, std::optional<float>, std::uint32_t,
    k3x::ProfilePhase, k3x::MlpActivation) {
    return unavailable<std::vector<float>>("dense_situ_mlp");
}
k3x::Result<std::vector<std::vector<float>>> B200ComputeBackend::mxfp4_situ_mlp_group(
    std::span<const float>, std::span<const k3x::Mxfp4MlpView>, float, std::optional<float>,
    std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<std::vector<float>>>("mxfp4_situ_mlp_group (SiTU)");
}
k3x::Result<std::vector<std::vector<float>>> B200ComputeBackend::mxfp4_situ_mlp_batch(
    std::span<const float>, std::size_t, k3x::Mxfp4MlpView, float, std::optional<float>,
    std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<std::vector<float>>>("mxfp4_situ_mlp_batch (SiTU)");
}
k3x::Result<std::vector<float>> B200ComputeBackend::mxfp4_situ_moe(
    std::span<const float>, std::span<const k3x::Mxfp4MlpView>, std::span<const float>, float,
    std::optional<float>, std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<float>>("mxfp4_situ_moe (SiTU)");
}
k3x::Result<k3x::Mxfp4PrefetchToken> B200ComputeBackend::prefetch_mxfp4_situ_mlp_group(
    std::span<const k3x::Mxfp4MlpView>, std::uint64_t, std::uint32_t, k3x::ProfilePhase) {
    return unavailable<k3x::Mxfp4PrefetchToken>("prefetch_mxfp4_situ_mlp_group");
}
k3x::Result<std::vector<std::vector<float>>> B200ComputeBackend::mxfp4_situ_mlp_group_prepared(
    std::span<const float>, k3x::Mxfp4PrefetchToken, float, std::optional<float>, std::uint32_t,
    k3x::ProfilePhase) {
    return unavailable<std::vector<std::vector<float>>>("mxfp4_situ_mlp_group_prepared");
}
k3x::Result<std::vector<float>> B200ComputeBackend::mxfp4_situ_moe_prepared(
    std::span<const float>, k3x::Mxfp4PrefetchToken, std::span<const float>, float,
    std::optional<float>, std::uint32_t, k3x::ProfilePhase) {
    return unavailable<std::vector<float>>("mxfp4_situ_moe_prepared");
}

k3x::Result<std::unique_ptr<k3x::ComputeBackend>> make_b200_backend(
    const k3x::BackendOptions& options, const B200BackendConfig& config) {
    return B200ComputeBackend::create(options, config);
}

}  // namespace glm5x_b200
