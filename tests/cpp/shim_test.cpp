// C++ parity driver for the drop-in headers (include/quantized.hpp,
// matmul_q4.hpp, layer_moe.hpp over libqmoe): the reference's interfaces
// called the way src/model.cpp and src/layer_gdn.cpp call them, checked
// against the CPU oracle (oracle/qmoe_oracle.c, linked as test
// infrastructure) on the same seeded bytes, plus the reference's error
// messages.  Exit status 0 = all checks passed.
#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "layer_moe.hpp"
#include "matmul_q4.hpp"
#include "moe_prefill.hpp"
#include "qmoe.h"
#include "quantized.hpp"

extern "C" {
typedef struct { const uint8_t* data; int type; uint64_t num_elements; } or_tensor;
typedef struct {
    or_tensor router, gate_exps, up_exps, down_exps, shared_gate_inp, shared_gate, shared_up, shared_down;
    const float* expert_bias;
} or_block;
int or_gemv(const uint8_t* w, int type, uint64_t n, const float* x, float* y, int M, int K, uint64_t off);
int or_dequantize_row(const uint8_t* w, int type, uint64_t n, float* out, int row, int cols);
int or_moe_forward_batch(const or_block* W, int d, int E, int k, int F, int Fs, int T, const float* x, float* out,
                         int* idx, float* wts, int* status, float* logits, float* h, float* hs, float* sg);
}

using namespace qwen;

static int g_fail = 0;
#define CHECK(cond, ...)                              \
    do {                                              \
        if (!(cond)) {                                \
            std::printf("FAIL %s:%d ", __FILE__, __LINE__); \
            std::printf(__VA_ARGS__);                 \
            std::printf("\n");                        \
            ++g_fail;                                 \
        }                                             \
    } while (0)

struct Tensor {
    QuantTensor q;
    std::vector<uint8_t> host;
};

static Tensor make(const char* name, GgmlType t, std::vector<int64_t> shape, uint64_t seed, uint64_t sid, float sigma) {
    Tensor r;
    uint64_t n = 1;
    for (int64_t s : shape) n *= static_cast<uint64_t>(s);
    r.q.name = name;
    r.q.type = t;
    r.q.shape = shape;
    r.q.num_elements = n;
    r.q.size_bytes = calculate_tensor_bytes(t, n);
    r.q.offset = 0;
    CUDA_CHECK(cudaMalloc(&r.q.device_ptr, r.q.size_bytes));
    if (qmoe_synth_fill(r.q.device_ptr, static_cast<uint32_t>(t), n, seed, sid, sigma, nullptr) != QMOE_OK)
        throw std::runtime_error("synth fill");
    r.host.resize(r.q.size_bytes);
    if (qmoe_synth_fill_host(r.host.data(), static_cast<uint32_t>(t), n, seed, sid, sigma) != QMOE_OK)
        throw std::runtime_error("synth fill host");
    return r;
}

template <typename F>
static void expect_throw(F f, const std::string& msg) {
    try {
        f();
        CHECK(false, "no exception, wanted '%s'", msg.c_str());
    } catch (const std::runtime_error& e) {
        CHECK(msg == e.what(), "message '%s', wanted '%s'", e.what(), msg.c_str());
    }
}

static bool close(float a, float b) { return std::fabs(a - b) <= 1e-3f + 1e-2f * std::fabs(b); }

int main() {
    ModelConfig cfg;
    cfg.d_model = 1024;
    cfg.num_experts = 64;
    cfg.num_experts_per_tok = 4;
    cfg.moe_intermediate_dim = 256;
    cfg.shared_expert_dim = 512;
    const int d = cfg.d_model, E = cfg.num_experts, k = cfg.num_experts_per_tok, F = cfg.moe_intermediate_dim,
              Fs = cfg.shared_expert_dim;
    const uint64_t seed = 2024;
    Tensor router = make("blk.3.ffn_gate_inp.weight", GgmlType::F32, {d, E}, seed, 1, 0.02f);
    Tensor eg = make("blk.3.ffn_gate_exps.weight", GgmlType::Q4_K, {d, F, E}, seed, 2, 0.02f);
    Tensor eu = make("blk.3.ffn_up_exps.weight", GgmlType::Q4_K, {d, F, E}, seed, 3, 0.02f);
    Tensor ed = make("blk.3.ffn_down_exps.weight", GgmlType::Q6_K, {F, d, E}, seed, 4, 0.02f);
    Tensor sgate = make("blk.3.ffn_gate_inp_shexp.weight", GgmlType::F32, {d}, seed, 5, 0.02f);
    Tensor sg = make("blk.3.ffn_gate_shexp.weight", GgmlType::Q8_0, {d, Fs}, seed, 6, 0.02f);
    Tensor su = make("blk.3.ffn_up_shexp.weight", GgmlType::Q8_0, {d, Fs}, seed, 7, 0.02f);
    Tensor sd = make("blk.3.ffn_down_shexp.weight", GgmlType::Q8_0, {Fs, d}, seed, 8, 0.02f);
    Tensor xt = make("x", GgmlType::F32, {d}, seed, 9, 1.0f);
    const float* hx = reinterpret_cast<const float*>(xt.host.data());
    const float* dx = static_cast<const float*>(xt.q.device_ptr);
    CUDA_CHECK(cudaDeviceSynchronize());

    CudaContext ctx;
    float* dy = nullptr;
    CUDA_CHECK(cudaMalloc(&dy, sizeof(float) * d));
    std::vector<float> y(d), want(d);

    // quantized.hpp helpers (reference quantized.hpp:49-105)
    CHECK(ggml_type_block_size(GgmlType::Q4_K) == 256 && ggml_type_size(GgmlType::Q4_K) == 144, "Q4_K geometry");
    CHECK(calculate_tensor_bytes(GgmlType::Q8_0, 64) == 68 && calculate_tensor_bytes(GgmlType::Q8_0, 65) == 0,
          "tensor bytes");

    // matmul_dispatch: the router GEMV is bit-identical to the reference order
    matmul_dispatch(router.q, dx, dy, E, d, ctx.stream());
    ctx.synchronize();
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * E, cudaMemcpyDeviceToHost));
    or_gemv(router.host.data(), 0, router.q.num_elements, hx, want.data(), E, d, 0);
    CHECK(std::memcmp(y.data(), want.data(), sizeof(float) * E) == 0, "router GEMV not bit-identical");
    // a quantised GEMV at an element offset (expert 5's gate rows)
    const uint64_t off = 5ull * F * d;
    matmul_dispatch(eg.q, dx, dy, F, d, ctx.stream(), off);
    ctx.synchronize();
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * F, cudaMemcpyDeviceToHost));
    or_gemv(eg.host.data(), 12, eg.q.num_elements, hx, want.data(), F, d, off);
    for (int i = 0; i < F; ++i) CHECK(close(y[i], want[i]), "gate row %d: %g vs %g", i, y[i], want[i]);
    // dequantize_row
    dequantize_row(ed.q, dy, 77, F, ctx.stream());
    ctx.synchronize();
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * F, cudaMemcpyDeviceToHost));
    or_dequantize_row(ed.host.data(), 14, ed.q.num_elements, want.data(), 77, F);
    CHECK(std::memcmp(y.data(), want.data(), sizeof(float) * F) == 0, "Q6_K row not identical");

    // error behaviour of src/cuda/matmul_q4.cu:187-217
    QuantTensor unloaded = eg.q;
    unloaded.device_ptr = nullptr;
    expect_throw([&] { matmul_dispatch(unloaded, dx, dy, F, d, ctx.stream()); },
                 "tensor 'blk.3.ffn_gate_exps.weight' is not loaded");
    QuantTensor q2k = eg.q;
    q2k.type = GgmlType::Q2_K;
    expect_throw([&] { matmul_dispatch(q2k, dx, dy, F, d, ctx.stream()); },
                 "unsupported GGML type for tensor 'blk.3.ffn_gate_exps.weight'");
    expect_throw([&] { matmul_dispatch(eg.q, dx, dy, F, d, ctx.stream(), static_cast<uint64_t>(E) * F * d); },
                 "GEMV shape exceeds tensor 'blk.3.ffn_gate_exps.weight'");
    expect_throw([&] { dequantize_row(ed.q, dy, d * E, F, ctx.stream()); },
                 "row is outside tensor 'blk.3.ffn_down_exps.weight'");
    expect_throw([&] { dequantize_row(q2k, dy, 0, d, ctx.stream()); },
                 "cannot dequantize tensor 'blk.3.ffn_gate_exps.weight'");
    CHECK(matmul_type_supported(GgmlType::Q6_K) && !matmul_type_supported(GgmlType::Q3_K), "type support");

    // MoeLayer: init / forward / check_routing, against the oracle's MoE block
    MoeLayer layer;
    layer.init(cfg, 3);
    layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    layer.check_routing(ctx);
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * d, cudaMemcpyDeviceToHost));
    auto ot = [](const Tensor& t) { return or_tensor{t.host.data(), static_cast<int>(t.q.type), t.q.num_elements}; };
    or_block W{ot(router), ot(eg), ot(eu), ot(ed), ot(sgate), ot(sg), ot(su), ot(sd), nullptr};
    std::vector<int> idx(k), status(1);
    std::vector<float> wts(k), logits(E), h(static_cast<size_t>(k) * F), hs(Fs), sgo(1);
    or_moe_forward_batch(&W, d, E, k, F, Fs, 1, hx, want.data(), idx.data(), wts.data(), status.data(),
                         logits.data(), h.data(), hs.data(), sgo.data());
    CHECK(status[0] == 0, "oracle status %d", status[0]);
    int bad = 0;
    for (int i = 0; i < d; ++i) bad += close(y[i], want[i]) ? 0 : 1;
    CHECK(bad == 0, "%d of %d MoE outputs outside max-abs 1e-3 / rel 1e-2", bad, d);
    // a second layer object on the same stream, then free_buffers twice (idempotent)
    MoeLayer other;
    other.init(cfg, 4);
    other.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    other.check_routing(ctx);
    other.free_buffers();
    other.free_buffers();

    // non-finite input: the reference throws from its host checks
    // (src/layer_moe.cpp:117); here forward records it and check_routing throws
    std::vector<float> nanx(hx, hx + d);
    nanx[17] = NAN;
    float* dnan = nullptr;
    CUDA_CHECK(cudaMalloc(&dnan, sizeof(float) * d));
    CUDA_CHECK(cudaMemcpy(dnan, nanx.data(), sizeof(float) * d, cudaMemcpyHostToDevice));
    layer.forward(dnan, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    expect_throw([&] { layer.check_routing(ctx); }, "invalid/non-finite MoE routing result in layer 3");
    // the error word is cleared by the report: the next clean token passes
    layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    layer.check_routing(ctx);

    // without check_routing: the next forward() throws the earlier call's error
    // (host-mapped error word, no synchronisation inside forward), and the one
    // after it works again
    layer.forward(dnan, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    CUDA_CHECK(cudaStreamSynchronize(ctx.stream()));  // the kernels have run
    expect_throw([&] { layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx); },
                 "invalid/non-finite MoE routing result in layer 3");
    layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    layer.check_routing(ctx);
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * d, cudaMemcpyDeviceToHost));
    bad = 0;
    for (int i = 0; i < d; ++i) bad += close(y[i], want[i]) ? 0 : 1;
    CHECK(bad == 0, "after a reported error: %d of %d MoE outputs outside tolerance", bad, d);

    // a grid-barrier wait that runs out (the test hook makes the fused decode
    // kernel wait for one CTA that never arrives, for 1 ms): the kernel
    // returns, the next forward() reports the timeout, and after it the layer
    // computes correctly again
    CHECK(qmoe_debug_grid_barrier(1000000ull, 1) == QMOE_OK, "debug hook");
    layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    CUDA_CHECK(cudaStreamSynchronize(ctx.stream()));
    CHECK(qmoe_debug_grid_barrier(0, 0) == QMOE_OK, "debug hook reset");
    expect_throw([&] { layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx); },
                 "MoE layer 3: device-side wait timed out");
    layer.forward(dx, dy, router.q, eg.q, eu.q, ed.q, sgate.q, sg.q, su.q, sd.q, ctx);
    layer.check_routing(ctx);
    CUDA_CHECK(cudaMemcpy(y.data(), dy, sizeof(float) * d, cudaMemcpyDeviceToHost));
    bad = 0;
    for (int i = 0; i < d; ++i) bad += close(y[i], want[i]) ? 0 : 1;
    CHECK(bad == 0, "after a barrier timeout: %d of %d MoE outputs outside tolerance", bad, d);

    // repack_tensor: a Q6_K tensor read by matmul_dispatch moves to the
    // 16-byte-aligned layout; the products are bit-identical, and a Q4_K
    // tensor is left alone
    {
        const int rows = 300;
        Tensor head = make("output.weight", GgmlType::Q6_K, {d, rows}, seed, 30, 0.02f);
        std::vector<float> a(rows), b(rows);
        matmul_dispatch(head.q, dx, dy, rows, d, ctx.stream());
        ctx.synchronize();
        CUDA_CHECK(cudaMemcpy(a.data(), dy, sizeof(float) * rows, cudaMemcpyDeviceToHost));
        const uint64_t before = head.q.size_bytes;
        CHECK(repack_tensor(head.q, ctx.stream()), "Q6_K tensor not repacked");
        CHECK(head.q.layout == QMOE_LAYOUT_Q6K_A16 && head.q.size_bytes == before / 210 * 224, "repacked layout/size");
        matmul_dispatch(head.q, dx, dy, rows, d, ctx.stream());
        ctx.synchronize();
        CUDA_CHECK(cudaMemcpy(b.data(), dy, sizeof(float) * rows, cudaMemcpyDeviceToHost));
        CHECK(std::memcmp(a.data(), b.data(), sizeof(float) * rows) == 0, "GEMV on the repacked tensor differs");
        CHECK(!repack_tensor(eg.q, ctx.stream()) && eg.q.layout == 0, "Q4_K tensor must stay as uploaded");
        cudaFree(head.q.device_ptr);
    }

    // MoePrefill: the MoE halves of two layers for a batch of T = 20 tokens
    // (tensor-core path) with a token mixer between them, against the same
    // layer loop written out with the C-ABI (bit-identical: same kernels)
    {
        const int T = 20, L = 2;
        const float eps = 1e-6f;
        Tensor xs = make("xs", GgmlType::F32, {d, T}, seed, 20, 1.0f);
        Tensor nw0 = make("post_norm0", GgmlType::F32, {d}, seed, 21, 0.1f);
        Tensor nw1 = make("post_norm1", GgmlType::F32, {d}, seed, 22, 0.1f);
        std::vector<MoeLayerTensors> layers(L);
        for (int l = 0; l < L; ++l)
            layers[l] = MoeLayerTensors{&router.q, &eg.q, &eu.q, &ed.q, &sgate.q, &sg.q, &su.q, &sd.q,
                                        static_cast<const float*>((l ? nw1 : nw0).q.device_ptr)};
        float *stream_buf = nullptr, *a = nullptr, *b = nullptr;
        const size_t nb = sizeof(float) * static_cast<size_t>(T) * d;
        CUDA_CHECK(cudaMalloc(&stream_buf, nb));
        CUDA_CHECK(cudaMalloc(&a, nb));
        CUDA_CHECK(cudaMalloc(&b, nb));
        CUDA_CHECK(cudaMemcpy(stream_buf, xs.q.device_ptr, nb, cudaMemcpyDeviceToDevice));
        CUDA_CHECK(cudaMemcpy(a, xs.q.device_ptr, nb, cudaMemcpyDeviceToDevice));
        std::vector<int> mixed;
        // the mixer stands in for attention/GDN + residual add: here it halves the stream
        auto mix = [&](int l, float* buf, int n) {
            mixed.push_back(l);
            CHECK(n == T, "mixer got %d tokens", n);
            std::vector<float> h(static_cast<size_t>(n) * d);
            CUDA_CHECK(cudaMemcpyAsync(h.data(), buf, sizeof(float) * h.size(), cudaMemcpyDeviceToHost, ctx.stream()));
            CUDA_CHECK(cudaStreamSynchronize(ctx.stream()));
            for (float& v : h) v *= 0.5f;
            CUDA_CHECK(cudaMemcpyAsync(buf, h.data(), sizeof(float) * h.size(), cudaMemcpyHostToDevice, ctx.stream()));
        };
        MoePrefill pre;
        pre.init(cfg, 64);
        pre.forward(stream_buf, T, layers, eps, ctx, mix);
        pre.check_routing(ctx);
        CHECK(mixed.size() == 2 && mixed[0] == 0 && mixed[1] == 1, "mixer calls");
        // the same loop by hand
        qmoe_dims dm{d, E, k, F, Fs};
        const size_t wsb = qmoe_workspace_size(&dm, T);
        void* ws2 = nullptr;
        CUDA_CHECK(cudaMalloc(&ws2, wsb));
        CHECK(qmoe_workspace_init(ws2, wsb, nullptr) == QMOE_OK, "ws init");
        auto qt = [](const Tensor& t) {
            qmoe_tensor v{};
            v.data = t.q.device_ptr;
            v.ggml_type = static_cast<uint32_t>(t.q.type);
            v.num_elements = t.q.num_elements;
            return v;
        };
        qmoe_block blk{qt(router), qt(eg), qt(eu), qt(ed), qt(sgate), qt(sg), qt(su), qt(sd), nullptr};
        float* cur = a;
        for (int l = 0; l < L; ++l) {
            mix(l, cur, T);
            float* nxt = cur == a ? b : a;
            CHECK(qmoe_block_forward_prenorm(&blk, &dm, cur, layers[l].post_norm, eps, nxt, T, ws2, wsb, ctx.stream()) ==
                      QMOE_OK,
                  "block_forward_prenorm");
            cur = nxt;
        }
        ctx.synchronize();
        std::vector<float> got(static_cast<size_t>(T) * d), ref(static_cast<size_t>(T) * d);
        CUDA_CHECK(cudaMemcpy(got.data(), stream_buf, nb, cudaMemcpyDeviceToHost));
        CUDA_CHECK(cudaMemcpy(ref.data(), cur, nb, cudaMemcpyDeviceToHost));
        CHECK(std::memcmp(got.data(), ref.data(), nb) == 0, "MoePrefill differs from the layer loop over the C-ABI");
        bool finite = true;
        for (float v : got) finite = finite && std::isfinite(v);
        CHECK(finite, "MoePrefill output not finite");
        expect_throw([&] { pre.forward(stream_buf, 65, layers, eps, ctx); },
                     "MoePrefill: batch of 65 tokens exceeds max_tokens 64");
        pre.free_buffers();
        pre.free_buffers();
        cudaFree(ws2);
        cudaFree(stream_buf);
        cudaFree(a);
        cudaFree(b);
    }

    std::printf(g_fail ? "shim_test: %d failures\n" : "shim_test: all checks passed\n", g_fail);
    return g_fail ? 1 : 0;
}
