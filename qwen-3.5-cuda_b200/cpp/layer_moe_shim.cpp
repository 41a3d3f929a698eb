// Definitions of include/layer_moe.hpp over the C-ABI (include/qmoe.h).
// One qmoe_block_forward call replaces the reference's host loop over the
// eight selected experts (src/layer_moe.cpp:82-155); the routing checks that
// the reference runs on the host after a synchronisation (:102-124) run on
// the device and are reported by check_routing().
#include "layer_moe.hpp"

#include <stdexcept>
#include <string>

namespace qwen {
namespace {

qmoe_tensor view(const QuantTensor& t) {
    qmoe_tensor v{};
    v.data = t.device_ptr;
    v.ggml_type = static_cast<uint32_t>(t.type);
    v.num_elements = t.num_elements;
    return v;
}

}  // namespace

MoeLayer::~MoeLayer() { free_buffers(); }

void MoeLayer::init(const ModelConfig& cfg, int layer_idx) {
    free_buffers();
    cfg_ = cfg;
    layer_idx_ = layer_idx;
    dims_.d_model = cfg.d_model;
    dims_.num_experts = cfg.num_experts;
    dims_.top_k = cfg.num_experts_per_tok;
    dims_.expert_dim = cfg.moe_intermediate_dim;
    dims_.shared_dim = cfg.shared_expert_dim;
    const size_t n = qmoe_workspace_size(&dims_, 1);
    if (n == 0) throw std::runtime_error("MoE dimensions not supported by the qmoe kernels");
    CUDA_CHECK(cudaMalloc(&ws_, n));
    ws_bytes_ = n;
    const int st = qmoe_workspace_init(ws_, ws_bytes_, nullptr);
    if (st != QMOE_OK) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
    CUDA_CHECK(cudaDeviceSynchronize());
}

void MoeLayer::free_buffers() {
    if (ws_) cudaFree(ws_);
    ws_ = nullptr;
    ws_bytes_ = 0;
}

void MoeLayer::forward(const float* x, float* out, const QuantTensor& router, const QuantTensor& eg,
                       const QuantTensor& eu, const QuantTensor& ed, const QuantTensor& sgate,
                       const QuantTensor& sg, const QuantTensor& su, const QuantTensor& sd, const CudaContext& ctx) {
    if (!ws_) throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + " used before init");
    qmoe_block b{};
    b.router = view(router);
    b.gate_exps = view(eg);
    b.up_exps = view(eu);
    b.down_exps = view(ed);
    b.shared_gate_inp = view(sgate);
    b.shared_gate = view(sg);
    b.shared_up = view(su);
    b.shared_down = view(sd);
    b.expert_bias = nullptr;
    const int st = qmoe_block_forward(&b, &dims_, x, out, nullptr, 1, ws_, ws_bytes_, ctx.stream());
    if (st == QMOE_ERR_CUDA) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
    if (st != QMOE_OK)
        throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + ": " + qmoe_status_string(st));
}

void MoeLayer::check_routing(const CudaContext& ctx) {
    uint32_t err[2] = {0, 0};
    const int st = qmoe_check_errors(ws_, &dims_, err, ctx.stream());
    if (st == QMOE_ERR_ROUTING)
        throw std::runtime_error("invalid/non-finite MoE routing result in layer " + std::to_string(layer_idx_));
    if (st == QMOE_ERR_NOT_NORMALIZED)
        throw std::runtime_error("MoE routing weights are not normalized in layer " + std::to_string(layer_idx_));
    if (st != QMOE_OK)
        throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + ": " + qmoe_status_string(st));
}

}  // namespace qwen
