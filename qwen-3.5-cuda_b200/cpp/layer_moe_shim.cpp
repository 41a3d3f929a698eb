// Definitions of include/layer_moe.hpp over the C-ABI (include/qmoe.h).
// One qmoe_block_forward call replaces the reference's host loop over the
// eight selected experts (src/layer_moe.cpp:82-155); the routing checks that
// the reference runs on the host after a synchronisation (:102-124) run on
// the device and are reported by the next forward() (through a host-mapped
// error word, without a synchronisation) or by check_routing().
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
    CUDA_CHECK(cudaHostAlloc(reinterpret_cast<void**>(&err_host_), sizeof(uint32_t), cudaHostAllocMapped));
    *err_host_ = 0;
    CUDA_CHECK(cudaHostGetDevicePointer(reinterpret_cast<void**>(&err_dev_), err_host_, 0));
    int st = qmoe_workspace_init(ws_, ws_bytes_, nullptr);
    if (st == QMOE_OK) st = qmoe_workspace_set_error_sink(ws_, err_dev_, nullptr);
    if (st != QMOE_OK) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
    CUDA_CHECK(cudaDeviceSynchronize());
}

void MoeLayer::free_buffers() {
    if (ws_) cudaFree(ws_);
    if (err_host_) cudaFreeHost(err_host_);
    ws_ = nullptr;
    ws_bytes_ = 0;
    err_host_ = nullptr;
    err_dev_ = nullptr;
}

// Throws the exception of error flags from an earlier call.  With a context,
// the workspace is re-initialised first (stream-ordered), so that the layer
// works again once the caller has handled the error.
void MoeLayer::throw_flags(uint32_t flags, const CudaContext* ctx) {
    if (ctx) {
        cudaStream_t s = ctx->stream();
        if (qmoe_workspace_init(ws_, ws_bytes_, s) != QMOE_OK || qmoe_workspace_set_error_sink(ws_, err_dev_, s) != QMOE_OK)
            throw std::runtime_error("CUDA Error: workspace re-initialisation failed");
    }
    if (flags & 1u)
        throw std::runtime_error("invalid/non-finite MoE routing result in layer " + std::to_string(layer_idx_));
    if (flags & 2u)
        throw std::runtime_error("MoE routing weights are not normalized in layer " + std::to_string(layer_idx_));
    throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + ": " + qmoe_status_string(QMOE_ERR_TIMEOUT));
}

void MoeLayer::forward(const float* x, float* out, const QuantTensor& router, const QuantTensor& eg,
                       const QuantTensor& eu, const QuantTensor& ed, const QuantTensor& sgate,
                       const QuantTensor& sg, const QuantTensor& su, const QuantTensor& sd, const CudaContext& ctx) {
    if (!ws_) throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + " used before init");
    // errors of earlier calls that have run by now (the kernels OR their flags
    // into the host-mapped word; no synchronisation here)
    const uint32_t flags = *reinterpret_cast<volatile uint32_t*>(err_host_);
    if (flags) {
        *reinterpret_cast<volatile uint32_t*>(err_host_) = 0;
        throw_flags(flags, &ctx);
    }
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
    if (err_host_) *reinterpret_cast<volatile uint32_t*>(err_host_) = 0;  // reported here, not again by forward()
    if (st == QMOE_ERR_TIMEOUT) throw_flags(err[0], &ctx);
    if (st == QMOE_ERR_ROUTING)
        throw std::runtime_error("invalid/non-finite MoE routing result in layer " + std::to_string(layer_idx_));
    if (st == QMOE_ERR_NOT_NORMALIZED)
        throw std::runtime_error("MoE routing weights are not normalized in layer " + std::to_string(layer_idx_));
    if (st != QMOE_OK)
        throw std::runtime_error("MoE layer " + std::to_string(layer_idx_) + ": " + qmoe_status_string(st));
}

}  // namespace qwen
