// adapter_check.cpp -- test harness (not product code): drives the B200
// k3x::ComputeBackend adapter the way the reference runtime would. The
// expert-major plan comes from the reference's own
// k3x::build_expert_major_packed_plan (runtime/src/expert_major.cpp, compiled
// into oracle/_ref/libk3x_ref.so), and the call goes through a
// k3x::ComputeBackend& to the virtual
// raw_bf16_situ_mlp_expert_major_with_shared (backend.hpp:228-236). Used by
// tests/test_gpu_adapter.py through ctypes.
#include <cstdio>
#include <cstring>
#include <memory>
#include <span>
#include <vector>

#include "k3x/backend.hpp"
#include "k3x/expert_major.hpp"
#include "../project-glm5x_b200/adapter/k3x_b200_backend.hpp"

extern "C" int adapter_expert_major(int device, int H, int I, int E, int K, int T,
                                    const float* hidden, const unsigned* route_ids,
                                    const float* contributions, const unsigned short* experts,
                                    const unsigned short* shared, int calls, float* out,
                                    unsigned long long* cache_hits, char* msg, int msg_cap) {
    std::vector<k3x::ExpertMajorTokenRoute> routes(T);
    for (int t = 0; t < T; ++t) {
        routes[t].expert_ids.assign(route_ids + (size_t)t * K, route_ids + (size_t)(t + 1) * K);
        routes[t].contributions.assign(contributions + (size_t)t * K,
                                       contributions + (size_t)(t + 1) * K);
    }
    auto plan = k3x::build_expert_major_packed_plan(
        std::span<const float>(hidden, (size_t)T * H), T, H, routes);
    if (!plan) {
        std::snprintf(msg, msg_cap, "plan: %s", plan.message().c_str());
        return static_cast<int>(plan.error());
    }
    const size_t per = (size_t)3 * I * H;  // gate, up, down BF16 values of one expert
    auto view_of = [&](const unsigned short* base, std::uint64_t id0) {
        auto bytes = [&](size_t off, size_t n) {
            return std::span<const std::byte>(reinterpret_cast<const std::byte*>(base + off), n * 2);
        };
        k3x::RawBf16MlpView v{};
        v.gate = {id0, bytes(0, (size_t)I * H), (size_t)I, (size_t)H};
        v.up = {id0 + 1, bytes((size_t)I * H, (size_t)I * H), (size_t)I, (size_t)H};
        v.down = {id0 + 2, bytes((size_t)2 * I * H, (size_t)H * I), (size_t)H, (size_t)I};
        return v;
    };
    std::vector<k3x::RawBf16MlpView> views;
    for (const auto& g : plan.value().groups) {
        if (g.expert_id >= (unsigned)E) return static_cast<int>(k3x::ErrorCode::invalid_extent);
        views.push_back(view_of(experts + g.expert_id * per, 1000 + 3 * (std::uint64_t)g.expert_id));
    }
    const k3x::RawBf16MlpView shared_view = view_of(shared, 1);
    k3x::BackendOptions options;
    options.kind = k3x::BackendKind::cuda_custom;
    options.cuda_expert_major_device_accumulate = true;
    glm5x_b200::B200BackendConfig cfg;
    cfg.device = device;
    cfg.hidden_size = H;
    cfg.intermediate_size = I;
    cfg.expert_slots = E;
    cfg.max_router_slots = K;
    cfg.max_tokens = T;
    auto made = glm5x_b200::make_b200_backend(options, cfg);
    if (!made) {
        std::snprintf(msg, msg_cap, "create: %s", made.message().c_str());
        return static_cast<int>(made.error());
    }
    k3x::ComputeBackend& backend = *made.value();
    for (int c = 0; c < calls; ++c) {
        auto r = backend.raw_bf16_situ_mlp_expert_major_with_shared(
            std::span<const float>(hidden, (size_t)T * H), T, plan.value(), views, shared_view,
            1.0f, std::nullopt, 0, k3x::ProfilePhase::prefill, k3x::MlpActivation::silu);
        if (!r) {
            std::snprintf(msg, msg_cap, "call %d: %s", c, r.message().c_str());
            return static_cast<int>(r.error());
        }
        std::memcpy(out + (size_t)c * T * H, r.value().data(), sizeof(float) * T * H);
    }
    // the SiTU activation is not offered: backend_unavailable, as the
    // reference's base-class defaults answer
    auto situ = backend.raw_bf16_situ_mlp_expert_major_with_shared(
        std::span<const float>(hidden, (size_t)T * H), T, plan.value(), views, shared_view, 1.0f,
        std::nullopt, 0, k3x::ProfilePhase::prefill, k3x::MlpActivation::situ);
    if (situ || situ.error() != k3x::ErrorCode::backend_unavailable) {
        std::snprintf(msg, msg_cap, "SiTU call was not refused");
        return -1;
    }
    *cache_hits = backend.runtime_stats().weight_cache_hits;
    return 0;
}
