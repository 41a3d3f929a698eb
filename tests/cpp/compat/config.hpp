// Test stand-in for the reference project's include/config.hpp: only the
// ModelConfig fields the MoE layer reads (reference config.hpp:12, 33-36).
// In the reference project its own config.hpp is used instead.
#pragma once
#include <cstdint>
namespace qwen {
struct ModelConfig {
    int32_t d_model = 0;
    int32_t num_experts = 0;
    int32_t num_experts_per_tok = 0;
    int32_t moe_intermediate_dim = 0;
    int32_t shared_expert_dim = 0;
};
}  // namespace qwen
