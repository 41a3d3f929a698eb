// The MoE layer of one decoder block.  Drop-in for the reference's
// include/layer_moe.hpp:10-56: the public interface is unchanged; the
// private per-token scratch buffers are replaced by one device workspace of
// the qmoe library (include/qmoe.h).  Definitions:
// qwen-3.5-cuda_b200/cpp/layer_moe_shim.cpp.
#ifndef QWEN_LAYER_MOE_HPP
#define QWEN_LAYER_MOE_HPP

#include <cstddef>
#include "config.hpp"
#include "cuda_utils.hpp"
#include "qmoe.h"
#include "quantized.hpp"

namespace qwen {

class MoeLayer {
public:
    ~MoeLayer();

    // Sizes and allocates the layer's device workspace (may throw).
    void init(const ModelConfig& cfg, int layer_idx);

    // Releases the workspace; safe to call more than once.
    void free_buffers();

    // out[d_model] = MoE(x[d_model]) for one token (device pointers), enqueued on
    // ctx.stream() without synchronising.  Errors of a call are recorded on the
    // device and in a host-mapped word; the next forward() throws them
    // (std::runtime_error, the reference's messages for routing errors) after
    // re-initialising the workspace, and check_routing() reports them at once.
    void forward(const float* x, float* out, const QuantTensor& router, const QuantTensor& eg,
                 const QuantTensor& eu, const QuantTensor& ed, const QuantTensor& sgate,
                 const QuantTensor& sg, const QuantTensor& su, const QuantTensor& sd, const CudaContext& ctx);

    // Synchronises ctx.stream() and throws std::runtime_error with the
    // reference's messages (src/layer_moe.cpp:117, :123) if a routing check failed.
    void check_routing(const CudaContext& ctx);

private:
    ModelConfig cfg_{};
    int layer_idx_ = -1;
    qmoe_dims dims_{};
    void* ws_ = nullptr;
    size_t ws_bytes_ = 0;
    uint32_t* err_host_ = nullptr;  // host-mapped error word of the kernels (qmoe_workspace_set_error_sink)
    uint32_t* err_dev_ = nullptr;   // its device address

    void throw_flags(uint32_t flags, const CudaContext* ctx);
};

}  // namespace qwen

#endif  // QWEN_LAYER_MOE_HPP
