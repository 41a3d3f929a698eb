// C entry points over the reference's own MoE path (layer_moe.cpp,
// matmul_q4.cu, moe.cu compiled unmodified from the reference tree), so the
// parity tests can run the reference on the GPU box with the same device
// buffers as the product.  TEST INFRASTRUCTURE ONLY.
#include "layer_moe.hpp"
#include "matmul_q4.hpp"
#include "ops.hpp"
#include <cstring>
#include <stdexcept>
#include <vector>
#include <exception>
#include <string>

namespace qwen {
void moe_topk(const float* router, int* top_idx, float* top_weight, int experts, int k, cudaStream_t stream);
}

namespace {
thread_local std::string g_last_error;

qwen::QuantTensor make_tensor(const char* name, const void* p, int type, unsigned long long n) {
    qwen::QuantTensor t;
    t.name = name;
    t.type = static_cast<qwen::GgmlType>(type);
    t.shape = {static_cast<int64_t>(n)};
    t.num_elements = n;
    t.size_bytes = qwen::calculate_tensor_bytes(t.type, n);
    t.offset = 0;
    t.device_ptr = const_cast<void*>(p);
    return t;
}
}  // namespace

extern "C" {

const char* ref_last_error(void) { return g_last_error.c_str(); }

// matmul_dispatch (matmul_q4.cu:185-207); returns 0 or 1 (exception text in ref_last_error).
int ref_gemv(const void* w, int type, unsigned long long n, const float* x, float* y, int M, int K,
             unsigned long long off, void* stream) {
    try {
        qwen::QuantTensor t = make_tensor("w", w, type, n);
        qwen::matmul_dispatch(t, x, y, M, K, static_cast<cudaStream_t>(stream), off);
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

int ref_dequantize_row(const void* w, int type, unsigned long long n, float* out, int row, int cols, void* stream) {
    try {
        qwen::QuantTensor t = make_tensor("w", w, type, n);
        qwen::dequantize_row(t, out, row, cols, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

// rmsnorm_forward (ops.cu:143-154): out = x * rsqrt(mean(x^2) + eps) * weight.
int ref_rmsnorm(const float* x, const float* weight, float* out, int n, float eps, void* stream) {
    try {
        qwen::rmsnorm_forward(x, weight, out, n, eps, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

int ref_topk(const float* logits, int* idx, float* w, int n, int k, void* stream) {
    try {
        qwen::moe_topk(logits, idx, w, n, k, static_cast<cudaStream_t>(stream));
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

// T tokens through MoeLayer::forward, one call per token, as model.cpp:209
// does.  Tensor arguments: pointer, GGML type, element count, 8 tensors in
// the order router, gate_exps, up_exps, down_exps, shared_gate_inp,
// shared_gate, shared_up, shared_down.
int ref_moe_forward(int d, int E, int k, int F, int Fs, int T, const float* x, float* out,
                    const void* const* ptrs, const int* types, const unsigned long long* nelem, void* stream) {
    try {
        qwen::ModelConfig c;
        c.d_model = d;
        c.num_experts = E;
        c.num_experts_per_tok = k;
        c.moe_intermediate_dim = F;
        c.shared_expert_dim = Fs;
        static const char* names[8] = {"ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps",
                                       "ffn_gate_inp_shexp", "ffn_gate_shexp", "ffn_up_shexp", "ffn_down_shexp"};
        qwen::QuantTensor t[8];
        for (int i = 0; i < 8; ++i) t[i] = make_tensor(names[i], ptrs[i], types[i], nelem[i]);
        qwen::CudaContext ctx(static_cast<cudaStream_t>(stream));
        qwen::MoeLayer layer;
        layer.init(c, 0);
        for (int i = 0; i < T; ++i)
            layer.forward(x + (size_t)i * d, out + (size_t)i * d, t[0], t[1], t[2], t[3], t[4], t[5], t[6], t[7], ctx);
        ctx.synchronize();
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

// A stack of L MoE layers run the way model.cpp:207-211 runs the MoE half of
// each decoder layer (rmsnorm_forward -> MoeLayer::forward -> residual_add),
// for timing the reference's own GPU path.  The layers are created once
// (MoeLayer::init allocates its buffers); tensors: 8 per layer as in
// ref_moe_forward, layer-major.
struct RefStack {
    int L = 0, d = 0;
    qwen::ModelConfig cfg;
    std::vector<qwen::QuantTensor> t;
    std::vector<qwen::MoeLayer*> layers;
    float *normed = nullptr, *moe_out = nullptr;
};

void* ref_stack_create(int L, int d, int E, int k, int F, int Fs, const void* const* ptrs, const int* types,
                       const unsigned long long* nelem) {
    try {
        RefStack* s = new RefStack();
        s->L = L;
        s->d = d;
        s->cfg.d_model = d;
        s->cfg.num_experts = E;
        s->cfg.num_experts_per_tok = k;
        s->cfg.moe_intermediate_dim = F;
        s->cfg.shared_expert_dim = Fs;
        static const char* names[8] = {"ffn_gate_inp", "ffn_gate_exps", "ffn_up_exps", "ffn_down_exps",
                                       "ffn_gate_inp_shexp", "ffn_gate_shexp", "ffn_up_shexp", "ffn_down_shexp"};
        for (int l = 0; l < L; ++l) {
            for (int i = 0; i < 8; ++i) s->t.push_back(make_tensor(names[i], ptrs[8 * l + i], types[8 * l + i], nelem[8 * l + i]));
            s->layers.push_back(new qwen::MoeLayer());
            s->layers.back()->init(s->cfg, l);
        }
        if (cudaMalloc(&s->normed, sizeof(float) * d) != cudaSuccess ||
            cudaMalloc(&s->moe_out, sizeof(float) * d) != cudaSuccess)
            throw std::runtime_error("ref_stack_create: cudaMalloc failed");
        return s;
    } catch (const std::exception& e) { g_last_error = e.what(); return nullptr; }
}

// One token through the stack: x (device F32[d], the residual stream) is
// updated in place; norm_w = the post-attention norm weight (F32[d]).
int ref_stack_forward(void* handle, float* x, const float* norm_w, float eps, void* stream) {
    try {
        RefStack* s = static_cast<RefStack*>(handle);
        cudaStream_t st = static_cast<cudaStream_t>(stream);
        qwen::CudaContext ctx(st);
        for (int l = 0; l < s->L; ++l) {
            const qwen::QuantTensor* t = &s->t[8 * l];
            qwen::rmsnorm_forward(x, norm_w, s->normed, s->d, eps, st);
            s->layers[l]->forward(s->normed, s->moe_out, t[0], t[1], t[2], t[3], t[4], t[5], t[6], t[7], ctx);
            qwen::residual_add(x, s->moe_out, x, s->d, st);
        }
        return 0;
    } catch (const std::exception& e) { g_last_error = e.what(); return 1; }
}

void ref_stack_destroy(void* handle) {
    RefStack* s = static_cast<RefStack*>(handle);
    if (!s) return;
    for (auto* l : s->layers) delete l;
    cudaFree(s->normed);
    cudaFree(s->moe_out);
    delete s;
}

}  // extern "C"
