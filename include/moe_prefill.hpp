// Batched (multi-token) MoE half of the decoder-layer loop.  The reference
// runs its model one token per call (src/main.cpp:391-393 feeds the prompt to
// QwenModel::decode_logits token by token; src/model.cpp:193-212 loops over
// the layers for that one token), so a prompt never reaches a grouped expert
// product.  MoePrefill runs the MoE half of every layer for a batch of T
// tokens at once -- model.cpp:208-211 (rmsnorm, MoeLayer::forward,
// residual_add) with the norm and the residual add fused into the block's
// kernels -- and takes the token mixing between the MoE halves (attention or
// GDN, outside this library) as a callback, so the layer order of model.cpp
// is kept.  T > 8 tokens take the tensor-core prefill path of
// qmoe_block_forward.  Definitions: qwen-3.5-cuda_b200/cpp/moe_prefill_shim.cpp.
#ifndef QWEN_MOE_PREFILL_HPP
#define QWEN_MOE_PREFILL_HPP

#include <cstddef>
#include <functional>
#include <vector>

#include "config.hpp"
#include "cuda_utils.hpp"
#include "qmoe.h"
#include "quantized.hpp"

namespace qwen {

// One layer's MoE tensors as QwenModel holds them (src/model.cpp:141-147) and
// the post-attention norm weight it applies before the MoE block (:208).
struct MoeLayerTensors {
    const QuantTensor* router = nullptr;
    const QuantTensor* eg = nullptr;
    const QuantTensor* eu = nullptr;
    const QuantTensor* ed = nullptr;
    const QuantTensor* sgate = nullptr;
    const QuantTensor* sg = nullptr;
    const QuantTensor* su = nullptr;
    const QuantTensor* sd = nullptr;
    const float* post_norm = nullptr;  // device F32 [d_model]
};

class MoePrefill {
public:
    ~MoePrefill();

    // Allocates the device workspace for batches of up to max_tokens tokens
    // and a second residual-stream buffer (may throw).
    void init(const ModelConfig& cfg, int max_tokens);

    // Releases the buffers; safe to call more than once.
    void free_buffers();

    // resid: device F32 [T][d_model], the residual stream of T tokens, updated
    // in place.  For each layer l in order: mix(l, stream, T) when given (the
    // caller's token mixing, in place on the current stream buffer), then
    // stream <- stream + MoE_l(rmsnorm(stream, eps) * post_norm_l).  Enqueued
    // on ctx.stream() without synchronising; routing errors are recorded on
    // the device (check_routing).
    void forward(float* resid, int T, const std::vector<MoeLayerTensors>& layers, float eps, const CudaContext& ctx,
                 const std::function<void(int, float*, int)>& mix = nullptr);

    // Synchronises ctx.stream() and throws std::runtime_error with the
    // reference's messages (src/layer_moe.cpp:117, :123) if a routing check of
    // an earlier forward() failed.
    void check_routing(const CudaContext& ctx);

private:
    ModelConfig cfg_{};
    int max_tokens_ = 0;
    qmoe_dims dims_{};
    void* ws_ = nullptr;
    size_t ws_bytes_ = 0;
    float* tmp_ = nullptr;
};

}  // namespace qwen

#endif  // QWEN_MOE_PREFILL_HPP
