// Definitions of include/moe_prefill.hpp over the C-ABI (include/qmoe.h):
// one qmoe_block_forward_prenorm per layer, the residual stream alternating
// between the caller's buffer and an internal one.
#include "moe_prefill.hpp"

#include <stdexcept>
#include <string>

namespace qwen {
namespace {

qmoe_tensor view(const QuantTensor* t) {
    qmoe_tensor v{};
    if (!t) return v;
    v.data = t->device_ptr;
    v.ggml_type = static_cast<uint32_t>(t->type);
    v.num_elements = t->num_elements;
    return v;
}

}  // namespace

MoePrefill::~MoePrefill() { free_buffers(); }

void MoePrefill::init(const ModelConfig& cfg, int max_tokens) {
    free_buffers();
    if (max_tokens <= 0) throw std::runtime_error("MoePrefill: max_tokens must be positive");
    cfg_ = cfg;
    max_tokens_ = max_tokens;
    dims_.d_model = cfg.d_model;
    dims_.num_experts = cfg.num_experts;
    dims_.top_k = cfg.num_experts_per_tok;
    dims_.expert_dim = cfg.moe_intermediate_dim;
    dims_.shared_dim = cfg.shared_expert_dim;
    const size_t n = qmoe_workspace_size(&dims_, max_tokens);
    if (n == 0) throw std::runtime_error("MoE dimensions not supported by the qmoe kernels");
    CUDA_CHECK(cudaMalloc(&ws_, n));
    ws_bytes_ = n;
    CUDA_CHECK(cudaMalloc(reinterpret_cast<void**>(&tmp_), sizeof(float) * static_cast<size_t>(max_tokens) * cfg.d_model));
    const int st = qmoe_workspace_init(ws_, ws_bytes_, nullptr);
    if (st != QMOE_OK) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
    CUDA_CHECK(cudaDeviceSynchronize());
}

void MoePrefill::free_buffers() {
    if (ws_) cudaFree(ws_);
    if (tmp_) cudaFree(tmp_);
    ws_ = nullptr;
    tmp_ = nullptr;
    ws_bytes_ = 0;
}

void MoePrefill::forward(float* resid, int T, const std::vector<MoeLayerTensors>& layers, float eps,
                         const CudaContext& ctx, const std::function<void(int, float*, int)>& mix) {
    if (!ws_) throw std::runtime_error("MoePrefill used before init");
    if (T <= 0 || T > max_tokens_)
        throw std::runtime_error("MoePrefill: batch of " + std::to_string(T) + " tokens exceeds max_tokens " +
                                 std::to_string(max_tokens_));
    float* cur = resid;
    for (size_t l = 0; l < layers.size(); ++l) {
        const MoeLayerTensors& z = layers[l];
        if (mix) mix(static_cast<int>(l), cur, T);
        if (!z.post_norm) throw std::runtime_error("MoePrefill: layer " + std::to_string(l) + " has no post_norm weight");
        qmoe_block b{};
        b.router = view(z.router);
        b.gate_exps = view(z.eg);
        b.up_exps = view(z.eu);
        b.down_exps = view(z.ed);
        b.shared_gate_inp = view(z.sgate);
        b.shared_gate = view(z.sg);
        b.shared_up = view(z.su);
        b.shared_down = view(z.sd);
        b.expert_bias = nullptr;
        float* next = cur == resid ? tmp_ : resid;
        const int st = qmoe_block_forward_prenorm(&b, &dims_, cur, z.post_norm, eps, next, T, ws_, ws_bytes_, ctx.stream());
        if (st == QMOE_ERR_CUDA) throw std::runtime_error(std::string("CUDA Error: ") + qmoe_status_string(st));
        if (st != QMOE_OK)
            throw std::runtime_error("MoE layer " + std::to_string(l) + ": " + qmoe_status_string(st));
        cur = next;
    }
    if (cur != resid)
        CUDA_CHECK(cudaMemcpyAsync(resid, cur, sizeof(float) * static_cast<size_t>(T) * cfg_.d_model,
                                   cudaMemcpyDeviceToDevice, ctx.stream()));
}

void MoePrefill::check_routing(const CudaContext& ctx) {
    uint32_t err[2] = {0, 0};
    const int st = qmoe_check_errors(ws_, &dims_, err, ctx.stream());
    if (st == QMOE_ERR_ROUTING) throw std::runtime_error("invalid/non-finite MoE routing result");
    if (st == QMOE_ERR_NOT_NORMALIZED) throw std::runtime_error("MoE routing weights are not normalized");
    if (st != QMOE_OK) throw std::runtime_error(std::string("MoE prefill: ") + qmoe_status_string(st));
}

}  // namespace qwen
