// extern "C" entry points of include/qmoe.h: argument checks (the reference's
// host-side exceptions become status codes), workspace layout, launches.
#include <algorithm>
#include <cstring>
#include "qmoe_dev.cuh"
#include "qmoe_internal.h"
#include "qmoe_units.cuh"
#include "qmoe_tgemm.h"

namespace qmoe {
cudaError_t launch_router(const DecodeParams& P, cudaStream_t s);
cudaError_t launch_gateup(const DecodeParams& P, cudaStream_t s);
cudaError_t launch_down(const DecodeParams& P, cudaStream_t s);
bool decode_supported(const DecodeParams& P);
bool fused_supported(const DecodeParams& P);
bool prefill_supported(const DecodeParams& P);
cudaError_t launch_prefill(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s);
int prefill_kernel_count(const DecodeParams& P);
cudaError_t launch_ep_route(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s);
cudaError_t launch_ep_experts(const DecodeParams& P, const PrefillBufs& B, const __half* x16, const int32_t* meta,
                              const int32_t* qmap, int32_t* out_pos, __half* y, int y_rows, const TgScatter* sc,
                              __half* xp, cudaStream_t s);
cudaError_t launch_ep_combine(const DecodeParams& P, const PrefillBufs& B, const __half* y_pairs,
                              const int32_t* pair_pos, cudaStream_t s);
cudaError_t launch_ep_shared(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s);
cudaError_t launch_ep_combine_routed(const DecodeParams& P, const PrefillBufs& B, const __half* y_pairs,
                                     const int32_t* pair_pos, cudaStream_t s);
size_t ep_dispatch_scratch_bytes(int T, int G);
bool ep_dispatch_supported(int k, int G);
cudaError_t launch_ep_dispatch(const int32_t* idx, const int32_t* placement, int T, int k, int E, int G,
                               const __half* x16, int d, __half* send_rows, int32_t* send_meta, int32_t* counts,
                               int32_t* pair_pos, void* scratch, cudaStream_t s);
cudaError_t launch_ep_qmap(const int32_t* meta, int n, int k, int32_t* qblk, int32_t* qmap, cudaStream_t s);
cudaError_t launch_experts(const DecodeParams& P, cudaStream_t s);
void set_grid_barrier_limits(uint64_t wait_ns, int phantom);
int decode_num_sms();
cudaError_t launch_gemv(const uint8_t* w, int type, const float* x, float* y, int M, int K, uint64_t off,
                        cudaStream_t s);
cudaError_t launch_dequant_row(const uint8_t* w, int type, float* out, uint64_t start, int cols, cudaStream_t s);
bool gemv_stream_supported(const uint8_t* w, int type, int K, uint64_t off);
cudaError_t launch_gemv_stream(const uint8_t* w, int type, uint64_t w_bytes, const float* x, float* y, int M, int K,
                               uint64_t off, cudaStream_t s);
cudaError_t launch_repack_q6k_a16(const uint8_t* src, void* dst, uint64_t nblocks, cudaStream_t s);
cudaError_t launch_synth(void* dst, int type, uint64_t nblocks, uint64_t seed, uint64_t stream_id, float sigma,
                         cudaStream_t s);
cudaError_t launch_dispatch(const int32_t* idx, int NP, int E, int32_t* offsets, int32_t* perm, int32_t* inv_perm,
                            int32_t* table, cudaStream_t s);
size_t dispatch_scratch_bytes(int E);
cudaError_t dispatch_noalloc_scratch(int32_t** p);

// The fused expert kernel serves calls of up to kFusedMaxT tokens; larger
// decode batches run gate/up and down as two kernels, which measured faster
// at 8 tokens (at one CTA per SM the fused kernel's shared memory then holds
// one gate/up slot and few down slots, so its items and down rounds
// serialise) and slower at 4 (the fused kernel also saves the router's
// routing step); outputs are bit-identical either way.
constexpr int kFusedMaxT = 4;
static bool use_fused(const DecodeParams& P) { return P.T <= kFusedMaxT && fused_supported(P); }

__global__ void k_set_sink(uint32_t* ctrl, unsigned long long sink) {
    *reinterpret_cast<unsigned long long*>(ctrl + CTRL_SINK) = sink;
}

__global__ void k_ws_init(uint32_t* ctrl) {
    const int i = threadIdx.x;
    if (i < CTRL_WORDS) ctrl[i] = (i == CTRL_ERR_TOKEN) ? 0xFFFFFFFFu : 0u;
}
}  // namespace qmoe

using namespace qmoe;

namespace {

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

inline int cuda_status(cudaError_t e) { return e == cudaSuccess ? QMOE_OK : QMOE_ERR_CUDA; }

bool gemv_type(uint32_t t) {
    return t == 0 || t == 1 || t == 30 || t == 2 || t == 6 || t == 8 || t == 12 || t == 13 || t == 14;
}
bool expert_type(uint32_t t) { return t == 8 || t == 12 || t == 13 || t == 14; }
bool router_type(uint32_t t) { return t == 0 || t == 1 || t == 30; }

bool pow2_in(int v, int lo, int hi) { return v >= lo && v <= hi && (v & (v - 1)) == 0; }

int check_dims(const qmoe_dims* D) {
    if (!D) return QMOE_ERR_ARG;
    if (D->d_model <= 0 || D->num_experts <= 0 || D->top_k <= 0 || D->expert_dim <= 0 || D->shared_dim <= 0)
        return QMOE_ERR_ARG;
    if (D->top_k > D->num_experts) return QMOE_ERR_ARG;
    // decode kernels: one 64-element unit per lane, up to 32 units per row;
    // K-quant rows need multiples of 256
    if (!pow2_in(D->d_model, 256, 2048) || !pow2_in(D->expert_dim, 256, 2048) || !pow2_in(D->shared_dim, 256, 2048))
        return QMOE_ERR_UNSUPPORTED;
    if (D->num_experts > kMaxExperts || D->top_k > kMaxTopK) return QMOE_ERR_UNSUPPORTED;
    return QMOE_OK;
}

int check_tensor(const qmoe_tensor& t, uint64_t need, bool (*typeok)(uint32_t)) {
    if (!t.data) return QMOE_ERR_ARG;
    if (t.layout != QMOE_LAYOUT_GGUF) return QMOE_ERR_UNSUPPORTED;  // the block kernels read GGUF blocks
    if (!typeok(t.ggml_type)) return QMOE_ERR_TYPE;
    if (t.num_elements < need) return QMOE_ERR_SHAPE;
    const int be = blk_elems(static_cast<int>(t.ggml_type));
    if (be == 0 || t.num_elements % be) return QMOE_ERR_SHAPE;
    if (!aligned16(t.data)) return QMOE_ERR_ALIGN;
    return QMOE_OK;
}

int check_block(const qmoe_block* B, const qmoe_dims* D) {
    if (!B) return QMOE_ERR_ARG;
    const uint64_t d = D->d_model, E = D->num_experts, F = D->expert_dim, Fs = D->shared_dim;
    int st;
    if ((st = check_tensor(B->router, E * d, router_type))) return st;
    if ((st = check_tensor(B->gate_exps, E * F * d, expert_type))) return st;
    if ((st = check_tensor(B->up_exps, E * F * d, expert_type))) return st;
    if ((st = check_tensor(B->down_exps, E * d * F, expert_type))) return st;
    if (B->up_exps.ggml_type != B->gate_exps.ggml_type) return QMOE_ERR_TYPE;
    if ((st = check_tensor(B->shared_gate_inp, d, router_type))) return st;
    if ((st = check_tensor(B->shared_gate, Fs * d, expert_type))) return st;
    if ((st = check_tensor(B->shared_up, Fs * d, expert_type))) return st;
    if ((st = check_tensor(B->shared_down, d * Fs, expert_type))) return st;
    if (B->shared_up.ggml_type != B->shared_gate.ggml_type) return QMOE_ERR_TYPE;
    if (B->expert_bias && (reinterpret_cast<uintptr_t>(B->expert_bias) & 3u)) return QMOE_ERR_ALIGN;
    return QMOE_OK;
}

WArg warg(const qmoe_tensor& t) {
    WArg a;
    a.p = static_cast<const uint8_t*>(t.data);
    a.end = a.p + qmoe_tensor_bytes(t.ggml_type, t.num_elements);
    a.type = static_cast<int>(t.ggml_type);
    a.pad = 0;
    return a;
}

uint64_t* g_trace = nullptr;  // qmoe_trace_enable

// DecodeParams for tokens [0, T) of x/out at the given workspace.
DecodeParams make_params(const qmoe_block* B, const qmoe_dims* D, const float* x, float* out, const float* residual,
                         int T, void* ws) {
    DecodeParams P;
    std::memset(&P, 0, sizeof(P));
    P.d = D->d_model; P.E = D->num_experts; P.k = D->top_k; P.F = D->expert_dim; P.Fs = D->shared_dim; P.T = T;
    P.has_shared = 1;
    P.num_sms = decode_num_sms();
    P.router = static_cast<const uint8_t*>(B->router.data);
    P.router_type = static_cast<int>(B->router.ggml_type);
    P.sgate_inp = static_cast<const uint8_t*>(B->shared_gate_inp.data);
    P.sgate_type = static_cast<int>(B->shared_gate_inp.ggml_type);
    P.bias = B->expert_bias;
    P.gate = warg(B->gate_exps); P.up = warg(B->up_exps); P.down = warg(B->down_exps);
    P.sgate = warg(B->shared_gate); P.sup = warg(B->shared_up); P.sdown = warg(B->shared_down);
    P.x = x; P.out = out; P.residual = residual;
    const WsLayout L = ws_layout(*D, T);
    uint8_t* w = static_cast<uint8_t*>(ws);
    P.ctrl = reinterpret_cast<uint32_t*>(w + L.ctrl);
    P.logits = reinterpret_cast<float*>(w + L.logits);
    P.topk_idx = reinterpret_cast<int32_t*>(w + L.topk_idx);
    P.topk_w = reinterpret_cast<float*>(w + L.topk_w);
    P.offsets = reinterpret_cast<int32_t*>(w + L.offsets);
    P.perm = reinterpret_cast<int32_t*>(w + L.perm);
    P.inv_perm = reinterpret_cast<int32_t*>(w + L.inv_perm);
    P.active = reinterpret_cast<int32_t*>(w + L.active);
    P.sched = reinterpret_cast<int32_t*>(w + L.sched);
    P.xnorm = reinterpret_cast<float*>(w + L.xnorm);
    P.norm_w = nullptr;
    P.eps = 0.0f;
    P.prenorm = 0;
    P.route_in_router = 1;
    P.xq_stride = L.xq_stride;
    P.hidden = reinterpret_cast<float*>(w + L.hidden);
    P.hq = w + L.hq; P.hq_stride = L.hq_stride; P.H = L.H;
    P.trace = g_trace;
    return P;
}

PrefillBufs prefill_bufs(const qmoe_dims& D, int T, void* ws) {
    const WsLayout L = ws_layout(D, T);
    uint8_t* w = static_cast<uint8_t*>(ws);
    PrefillBufs pb;
    pb.tok_of_pos = reinterpret_cast<int32_t*>(w + L.tok_of_pos);
    pb.tile_start = reinterpret_cast<int32_t*>(w + L.tile_start);
    pb.sh_grp = reinterpret_cast<int32_t*>(w + L.sh_grp);
    pb.sh_tiles = pb.sh_grp + 2;
    pb.disp = reinterpret_cast<int32_t*>(w + L.disp);
    pb.X16 = reinterpret_cast<__half*>(w + L.X16);
    pb.H = reinterpret_cast<__half*>(w + L.Hpf);
    pb.Hs = reinterpret_cast<__half*>(w + L.Hs);
    pb.Y = reinterpret_cast<__half*>(w + L.Y);
    pb.Ys = reinterpret_cast<__half*>(w + L.Ys);
    pb.xperm = reinterpret_cast<float*>(w + L.xperm);
    pb.wperm = reinterpret_cast<float*>(w + L.wperm);
    return pb;
}

int check_common(const qmoe_block* B, const qmoe_dims* D, int T, void* ws, size_t ws_bytes, int maxT) {
    int st;
    if ((st = check_dims(D))) return st;
    if ((st = check_block(B, D))) return st;
    if (T <= 0) return QMOE_ERR_ARG;
    if (T > maxT) return QMOE_ERR_UNSUPPORTED;
    if (!ws || !aligned16(ws)) return QMOE_ERR_WORKSPACE;
    if (ws_layout(*D, std::min(T, kDecodeMaxT)).total > ws_bytes) return QMOE_ERR_WORKSPACE;
    return QMOE_OK;
}

}  // namespace

extern "C" {

int qmoe_abi_version(void) { return 1; }

const char* qmoe_status_string(int s) {
    switch (s) {
        case QMOE_OK: return "ok";
        case QMOE_ERR_ARG: return "invalid argument (null or not-loaded tensor)";
        case QMOE_ERR_TYPE: return "unsupported GGML type";
        case QMOE_ERR_SHAPE: return "shape exceeds tensor";
        case QMOE_ERR_ALIGN: return "pointer not 16-byte aligned";
        case QMOE_ERR_WORKSPACE: return "workspace missing or too small";
        case QMOE_ERR_UNSUPPORTED: return "dimensions not supported by the kernels";
        case QMOE_ERR_CUDA: return "CUDA error";
        case QMOE_ERR_ROUTING: return "invalid/non-finite MoE routing result";
        case QMOE_ERR_NOT_NORMALIZED: return "MoE routing weights are not normalized";
        case QMOE_ERR_TIMEOUT: return "device-side wait timed out";
        case QMOE_ERR_COMM: return "collective communication error";
        default: return "unknown status";
    }
}

int qmoe_type_supported(uint32_t t) { return gemv_type(t) ? 1 : 0; }

uint64_t qmoe_tensor_bytes(uint32_t t, uint64_t n) {
    const int be = blk_elems(static_cast<int>(t)), bb = blk_bytes(static_cast<int>(t));
    if (be == 0 || bb == 0 || n % static_cast<uint64_t>(be)) return 0;
    return n / be * static_cast<uint64_t>(bb);
}

int qmoe_gemv(const qmoe_tensor* w, const float* x, float* y, int M, int K, uint64_t off, qmoe_stream_t stream) {
    if (!w || !w->data || !x || !y) return QMOE_ERR_ARG;
    if (!gemv_type(w->ggml_type)) return QMOE_ERR_TYPE;
    if (M <= 0 || K <= 0 || off + static_cast<uint64_t>(M) * K > w->num_elements) return QMOE_ERR_SHAPE;
    const uint8_t* wp = static_cast<const uint8_t*>(w->data);
    int type = static_cast<int>(w->ggml_type);
    uint64_t wbytes = qmoe_tensor_bytes(w->ggml_type, w->num_elements);
    if (w->layout == QMOE_LAYOUT_Q6K_A16) {
        if (type != T_Q6_K) return QMOE_ERR_UNSUPPORTED;
        type = T_Q6_K_A16;
        wbytes = qmoe_repack_bytes(w->ggml_type, w->num_elements, w->layout);
        // the repacked layout has only the streaming kernel
        if (!gemv_stream_supported(wp, type, K, off) || reinterpret_cast<uintptr_t>(x) % 16)
            return QMOE_ERR_UNSUPPORTED;
    } else if (w->layout != QMOE_LAYOUT_GGUF) {
        return QMOE_ERR_UNSUPPORTED;
    }
    if (gemv_stream_supported(wp, type, K, off) && reinterpret_cast<uintptr_t>(x) % 16 == 0)
        return cuda_status(launch_gemv_stream(wp, type, wbytes, x, y, M, K, off, reinterpret_cast<cudaStream_t>(stream)));
    return cuda_status(launch_gemv(wp, type, x, y, M, K, off, reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_gemv_exact(const qmoe_tensor* w, const float* x, float* y, int M, int K, uint64_t off,
                    qmoe_stream_t stream) {
    if (!w || !w->data || !x || !y) return QMOE_ERR_ARG;
    if (!gemv_type(w->ggml_type)) return QMOE_ERR_TYPE;
    if (w->layout != QMOE_LAYOUT_GGUF) return QMOE_ERR_UNSUPPORTED;
    if (M <= 0 || K <= 0 || off + static_cast<uint64_t>(M) * K > w->num_elements) return QMOE_ERR_SHAPE;
    return cuda_status(launch_gemv(static_cast<const uint8_t*>(w->data), static_cast<int>(w->ggml_type), x, y, M, K,
                                   off, reinterpret_cast<cudaStream_t>(stream)));
}

uint64_t qmoe_repack_bytes(uint32_t t, uint64_t n, uint32_t layout) {
    if (layout == QMOE_LAYOUT_GGUF) return qmoe_tensor_bytes(t, n);
    if (layout == QMOE_LAYOUT_Q6K_A16 && static_cast<int>(t) == T_Q6_K && n % 256 == 0) return n / 256 * 224;
    return 0;
}

int qmoe_repack(const qmoe_tensor* src, uint32_t layout, void* dst, size_t dst_bytes, qmoe_stream_t stream) {
    if (!src || !src->data || !dst) return QMOE_ERR_ARG;
    if (src->layout != QMOE_LAYOUT_GGUF) return QMOE_ERR_UNSUPPORTED;
    const uint64_t need = qmoe_repack_bytes(src->ggml_type, src->num_elements, layout);
    if (need == 0) return layout == QMOE_LAYOUT_Q6K_A16 ? QMOE_ERR_TYPE : QMOE_ERR_UNSUPPORTED;
    if (dst_bytes < need) return QMOE_ERR_SHAPE;
    if (!aligned16(dst)) return QMOE_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (layout == QMOE_LAYOUT_GGUF)
        return cuda_status(cudaMemcpyAsync(dst, src->data, need, cudaMemcpyDeviceToDevice, s));
    if (reinterpret_cast<uintptr_t>(src->data) % 2) return QMOE_ERR_ALIGN;
    return cuda_status(launch_repack_q6k_a16(static_cast<const uint8_t*>(src->data), dst, src->num_elements / 256, s));
}

int qmoe_dequant_row(const qmoe_tensor* w, float* out, int row, int cols, qmoe_stream_t stream) {
    if (!w || !w->data || !out || !gemv_type(w->ggml_type)) return QMOE_ERR_TYPE;
    if (w->layout != QMOE_LAYOUT_GGUF) return QMOE_ERR_UNSUPPORTED;
    const uint64_t start = static_cast<uint64_t>(row) * cols;
    if (row < 0 || cols <= 0 || start + cols > w->num_elements) return QMOE_ERR_SHAPE;
    return cuda_status(launch_dequant_row(static_cast<const uint8_t*>(w->data), static_cast<int>(w->ggml_type), out,
                                          start, cols, reinterpret_cast<cudaStream_t>(stream)));
}

size_t qmoe_workspace_size(const qmoe_dims* D, int max_tokens) {
    if (check_dims(D) || max_tokens <= 0) return 0;
    const size_t a = ws_layout(*D, std::min(max_tokens, kDecodeMaxT)).total;
    const size_t b = dispatch_scratch_bytes(D->num_experts) + 256;
    const size_t c = max_tokens > kDecodeMaxT ? ws_layout(*D, max_tokens).total : 0;  // prefill path
    return std::max(std::max(a, b), c);
}

void* qmoe_ws_view(void* ws, const qmoe_dims* D, int T, int which) {
    if (!ws || check_dims(D) || T <= 0) return nullptr;
    const WsLayout L = ws_layout(*D, T);
    uint8_t* w = static_cast<uint8_t*>(ws);
    switch (which) {
        case QMOE_WS_LOGITS: return w + L.logits;
        case QMOE_WS_TOPK_IDX: return w + L.topk_idx;
        case QMOE_WS_TOPK_W: return w + L.topk_w;
        case QMOE_WS_OFFSETS: return w + L.offsets;
        case QMOE_WS_PERM: return w + L.perm;
        case QMOE_WS_INV_PERM: return w + L.inv_perm;
        case QMOE_WS_HIDDEN: return w + L.hidden;
        case QMOE_WS_ERROR: return w + L.ctrl + CTRL_ERROR * 4;
        case QMOE_WS_INPUT: return w + L.xnorm;
        case QMOE_WS_INPUT16: return T > kDecodeMaxT ? w + L.X16 : nullptr;
        default: return nullptr;
    }
}

int qmoe_workspace_init(void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    if (!ws || ws_bytes < 256) return QMOE_ERR_WORKSPACE;
    k_ws_init<<<1, CTRL_WORDS, 0, reinterpret_cast<cudaStream_t>(stream)>>>(static_cast<uint32_t*>(ws));
    return cuda_status(cudaGetLastError());
}

int qmoe_workspace_set_error_sink(void* ws, uint32_t* sink, qmoe_stream_t stream) {
    if (!ws) return QMOE_ERR_WORKSPACE;
    k_set_sink<<<1, 1, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t*>(ws), static_cast<unsigned long long>(reinterpret_cast<uintptr_t>(sink)));
    return cuda_status(cudaGetLastError());
}

int qmoe_debug_grid_barrier(uint64_t wait_ns, int phantom_arrivals) {
    if (phantom_arrivals < 0) return QMOE_ERR_ARG;
    set_grid_barrier_limits(wait_ns, phantom_arrivals);
    return QMOE_OK;
}

int qmoe_router_topk(const qmoe_block* B, const qmoe_dims* D, const float* x, int T, int32_t* topk_idx,
                     float* topk_w, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, kDecodeMaxT);
    if (st) return st;
    if (!x || !aligned16(x)) return x ? QMOE_ERR_ALIGN : QMOE_ERR_ARG;
    DecodeParams P = make_params(B, D, x, nullptr, nullptr, T, ws);
    P.out_idx = topk_idx;
    P.out_w = topk_w;
    return cuda_status(launch_router(P, reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_dispatch(const int32_t* idx, int T, int k, int E, int32_t* offsets, int32_t* perm, int32_t* inv_perm,
                  void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    if (!idx || !offsets || !perm || T <= 0 || k <= 0 || E <= 0) return QMOE_ERR_ARG;
    if (static_cast<int64_t>(T) * k > (1ll << 30)) return QMOE_ERR_UNSUPPORTED;
    if (!ws || ws_bytes < dispatch_scratch_bytes(E)) return QMOE_ERR_WORKSPACE;
    return cuda_status(launch_dispatch(idx, T * k, E, offsets, perm, inv_perm, static_cast<int32_t*>(ws),
                                       reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_dispatch_noalloc(const int32_t* idx, int T, int k, int E, int32_t* offsets, int32_t* perm,
                          int32_t* inv_perm, qmoe_stream_t stream) {
    if (!idx || !offsets || !perm || T <= 0 || k <= 0 || E <= 0) return QMOE_ERR_ARG;
    if (E > kNoAllocMaxExperts) return QMOE_ERR_UNSUPPORTED;  // the fixed scratch holds E <= 256
    if (static_cast<int64_t>(T) * k > (1ll << 30)) return QMOE_ERR_UNSUPPORTED;
    // the scratch array's device address in the current context, looked up on
    // every call (a host-side query, no allocation): a cached address would
    // be stale after cudaDeviceReset or in another context of the device
    int32_t* table = nullptr;
    if (dispatch_noalloc_scratch(&table) != cudaSuccess || !table) return QMOE_ERR_CUDA;
    return cuda_status(launch_dispatch(idx, T * k, E, offsets, perm, inv_perm, table,
                                       reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_expert_gateup(const qmoe_block* B, const qmoe_dims* D, const float* x, int T, void* ws, size_t ws_bytes,
                       qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, kDecodeMaxT);
    if (st) return st;
    (void)x;  // the block input x_in (workspace) was written by qmoe_router_topk
    DecodeParams P = make_params(B, D, x, nullptr, nullptr, T, ws);
    if (!decode_supported(P)) return QMOE_ERR_UNSUPPORTED;
    return cuda_status(launch_gateup(P, reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_down_combine(const qmoe_block* B, const qmoe_dims* D, int T, float* out, const float* residual, void* ws,
                      size_t ws_bytes, qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, kDecodeMaxT);
    if (st) return st;
    if (!out) return QMOE_ERR_ARG;
    DecodeParams P = make_params(B, D, nullptr, out, residual, T, ws);
    if (!decode_supported(P)) return QMOE_ERR_UNSUPPORTED;
    return cuda_status(launch_down(P, reinterpret_cast<cudaStream_t>(stream)));
}

int qmoe_expert_block(const qmoe_block* B, const qmoe_dims* D, int T, float* out, const float* residual, void* ws,
                      size_t ws_bytes, qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, kDecodeMaxT);
    if (st) return st;
    if (!out) return QMOE_ERR_ARG;
    DecodeParams P = make_params(B, D, nullptr, out, residual, T, ws);
    if (!decode_supported(P)) return QMOE_ERR_UNSUPPORTED;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (use_fused(P)) return cuda_status(launch_experts(P, s));
    cudaError_t e = launch_gateup(P, s);
    if (e == cudaSuccess) e = launch_down(P, s);
    return cuda_status(e);
}

// ---- expert parallelism ----
int qmoe_ep_route(const qmoe_block* B, const qmoe_dims* D, const float* x, const float* norm_w, float eps, int T,
                  void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, 1 << 30);
    if (st) return st;
    if (T <= kDecodeMaxT) return QMOE_ERR_UNSUPPORTED;
    if (!x) return QMOE_ERR_ARG;
    if (!aligned16(x) || (norm_w && !aligned16(norm_w))) return QMOE_ERR_ALIGN;
    if (norm_w && !(eps > 0.0f)) return QMOE_ERR_ARG;
    if (ws_layout(*D, T).total > ws_bytes) return QMOE_ERR_WORKSPACE;
    DecodeParams P = make_params(B, D, x, nullptr, nullptr, T, ws);
    if (!prefill_supported(P)) return QMOE_ERR_UNSUPPORTED;
    if (norm_w) {
        P.prenorm = 1;
        P.norm_w = norm_w;
        P.eps = eps;
    }
    return cuda_status(launch_ep_route(P, prefill_bufs(*D, T, ws), reinterpret_cast<cudaStream_t>(stream)));
}

size_t qmoe_ep_dispatch_scratch_size(int T, int G) {
    if (T <= 0 || G <= 0 || G > 32) return 0;
    return ep_dispatch_scratch_bytes(T, G);
}

int qmoe_ep_dispatch(const qmoe_dims* D, int T, int G, const int32_t* placement, void* ws, size_t ws_bytes,
                     void* send_rows, int32_t* send_meta, int32_t* counts, int32_t* pair_pos, void* scratch,
                     size_t scratch_bytes, qmoe_stream_t stream) {
    int st;
    if ((st = check_dims(D))) return st;
    if (T <= kDecodeMaxT) return QMOE_ERR_UNSUPPORTED;
    if (G <= 0 || D->num_experts % G) return QMOE_ERR_ARG;
    if (!ep_dispatch_supported(D->top_k, G)) return QMOE_ERR_UNSUPPORTED;
    if (!ws || !send_rows || !send_meta || !counts || !pair_pos || !scratch) return QMOE_ERR_ARG;
    if (!aligned16(ws) || !aligned16(send_rows)) return QMOE_ERR_ALIGN;
    if (ws_layout(*D, T).total > ws_bytes || ep_dispatch_scratch_bytes(T, G) > scratch_bytes)
        return QMOE_ERR_WORKSPACE;
    const WsLayout L = ws_layout(*D, T);
    uint8_t* w = static_cast<uint8_t*>(ws);
    return cuda_status(launch_ep_dispatch(reinterpret_cast<const int32_t*>(w + L.topk_idx), placement, T, D->top_k,
                                          D->num_experts, G, reinterpret_cast<const __half*>(w + L.X16), D->d_model,
                                          static_cast<__half*>(send_rows), send_meta, counts, pair_pos, scratch,
                                          reinterpret_cast<cudaStream_t>(stream)));
}

size_t qmoe_ep_rows_workspace_size(const qmoe_dims* D, int max_rows) {
    if (check_dims(D) || max_rows <= 0) return 0;
    return ep_rows_layout(*D, max_rows).total;
}

static int ep_experts_impl(const qmoe_block* B, const qmoe_dims* D, const void* x16, const int32_t* meta, int n,
                           int n_pairs, void* y, const TgScatter* sc, void* ws, size_t ws_bytes,
                           qmoe_stream_t stream) {
    int st;
    if (!B || (st = check_dims(D))) return B ? st : QMOE_ERR_ARG;
    if (n < 0 || n_pairs < 0 || static_cast<int64_t>(n_pairs) > static_cast<int64_t>(n) * D->top_k) return QMOE_ERR_ARG;
    if (n == 0 || n_pairs == 0) return QMOE_OK;
    if (!x16 || !meta || (!y && !sc) || !ws) return QMOE_ERR_ARG;
    if (!aligned16(x16) || (y && !aligned16(y)) || !aligned16(ws)) return QMOE_ERR_ALIGN;
    if (D->top_k > 8) return QMOE_ERR_UNSUPPORTED;
    const uint64_t d = D->d_model, E = D->num_experts, F = D->expert_dim;
    if ((st = check_tensor(B->gate_exps, E * F * d, expert_type))) return st;
    if ((st = check_tensor(B->up_exps, E * F * d, expert_type))) return st;
    if ((st = check_tensor(B->down_exps, E * d * F, expert_type))) return st;
    if (B->up_exps.ggml_type != B->gate_exps.ggml_type) return QMOE_ERR_TYPE;
    const EpRowsLayout L = ep_rows_layout(*D, n);
    if (L.total > ws_bytes) return QMOE_ERR_WORKSPACE;
    qmoe_block lb = *B;  // the router and shared tensors are not read
    lb.router = lb.shared_gate_inp = B->gate_exps;
    lb.shared_gate = lb.shared_up = B->gate_exps;
    lb.shared_down = B->down_exps;
    DecodeParams P = make_params(&lb, D, nullptr, nullptr, nullptr, kDecodeMaxT, ws);
    uint8_t* w = static_cast<uint8_t*>(ws);
    P.T = n;
    P.has_shared = 0;
    P.ctrl = reinterpret_cast<uint32_t*>(w + L.ctrl);
    P.offsets = reinterpret_cast<int32_t*>(w + L.offsets);
    P.perm = reinterpret_cast<int32_t*>(w + L.perm);
    P.inv_perm = reinterpret_cast<int32_t*>(w + L.inv_perm);
    if (!prefill_supported(P)) return QMOE_ERR_UNSUPPORTED;
    if (sc && !(P.gate.type == P.up.type && tgemm_supported(P.gate.type, 0, P.F, P.d) &&
                tgemm_supported(P.down.type, 1, P.d, P.F)))
        return QMOE_ERR_UNSUPPORTED;
    PrefillBufs pb{};
    pb.tok_of_pos = reinterpret_cast<int32_t*>(w + L.tok_of_pos);
    pb.tile_start = reinterpret_cast<int32_t*>(w + L.tile_start);
    pb.disp = reinterpret_cast<int32_t*>(w + L.disp);
    pb.H = reinterpret_cast<__half*>(w + L.H);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    int32_t* qmap = reinterpret_cast<int32_t*>(w + L.qmap);
    cudaError_t e = launch_ep_qmap(meta, n, D->top_k, reinterpret_cast<int32_t*>(w + L.qblk), qmap, s);
    if (e == cudaSuccess)
        e = launch_ep_experts(P, pb, static_cast<const __half*>(x16), meta, qmap,
                              reinterpret_cast<int32_t*>(w + L.out_pos), static_cast<__half*>(y), n_pairs, sc,
                              reinterpret_cast<__half*>(w + L.Xp), s);
    return cuda_status(e);
}

int qmoe_ep_experts(const qmoe_block* B, const qmoe_dims* D, const void* x16, const int32_t* meta, int n,
                    int n_pairs, void* y, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    return ep_experts_impl(B, D, x16, meta, n, n_pairs, y, nullptr, ws, ws_bytes, stream);
}

int qmoe_ep_experts_return(const qmoe_block* B, const qmoe_dims* D, const void* x16, const int32_t* meta, int n,
                           const qmoe_ep_return* ret, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    if (!ret || ret->n_ranks < 1 || ret->n_ranks > 32) return QMOE_ERR_ARG;
    TgScatter sc{};
    sc.n_src = ret->n_ranks;
    for (int r = 0; r <= ret->n_ranks; ++r) {
        sc.start[r] = ret->pair_start[r];
        if (r > 0 && ret->pair_start[r] < ret->pair_start[r - 1]) return QMOE_ERR_ARG;
    }
    if (ret->pair_start[0] != 0) return QMOE_ERR_ARG;
    for (int r = 0; r < ret->n_ranks; ++r) {
        const bool has = ret->pair_start[r + 1] > ret->pair_start[r];
        if (has && (!ret->dst[r] || !aligned16(ret->dst[r]) || ret->dst_row[r] < 0)) return QMOE_ERR_ARG;
        sc.dst[r] = static_cast<__half*>(ret->dst[r]);
        sc.dst_row[r] = ret->dst_row[r];
    }
    return ep_experts_impl(B, D, x16, meta, n, ret->pair_start[ret->n_ranks], nullptr, &sc, ws, ws_bytes, stream);
}

int qmoe_peer_alloc(size_t bytes, void** ptr, void* handle) {
    if (!ptr || !handle || bytes == 0) return QMOE_ERR_ARG;
    *ptr = nullptr;
    cudaError_t e = cudaMalloc(ptr, bytes);
    if (e == cudaSuccess) e = cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(handle), *ptr);
    if (e != cudaSuccess && *ptr) {
        cudaFree(*ptr);
        *ptr = nullptr;
    }
    return cuda_status(e);
}

int qmoe_peer_open(const void* handle, void** ptr) {
    if (!ptr || !handle) return QMOE_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int qmoe_peer_close(void* ptr) { return ptr ? cuda_status(cudaIpcCloseMemHandle(ptr)) : QMOE_ERR_ARG; }

int qmoe_peer_free(void* ptr) { return ptr ? cuda_status(cudaFree(ptr)) : QMOE_ERR_ARG; }

int qmoe_copy_async(void* dst, const void* src, size_t bytes, qmoe_stream_t stream) {
    if (bytes == 0) return QMOE_OK;
    if (!dst || !src) return QMOE_ERR_ARG;
    return cuda_status(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)));
}

static int ep_combine_impl(const qmoe_block* B, const qmoe_dims* D, const void* y_pairs, const int32_t* pair_pos,
                           int T, const float* residual, float* out, void* ws, size_t ws_bytes, qmoe_stream_t stream,
                           int part) {
    int st = check_common(B, D, T, ws, ws_bytes, 1 << 30);
    if (st) return st;
    if (T <= kDecodeMaxT) return QMOE_ERR_UNSUPPORTED;
    if (part != 1 && (!y_pairs || !pair_pos || !out)) return QMOE_ERR_ARG;
    if (part != 1 && !aligned16(y_pairs)) return QMOE_ERR_ALIGN;
    if (ws_layout(*D, T).total > ws_bytes) return QMOE_ERR_WORKSPACE;
    DecodeParams P = make_params(B, D, nullptr, out, residual, T, ws);
    if (!prefill_supported(P)) return QMOE_ERR_UNSUPPORTED;
    const PrefillBufs pb = prefill_bufs(*D, T, ws);
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const __half* y = static_cast<const __half*>(y_pairs);
    switch (part) {
        case 1: return cuda_status(launch_ep_shared(P, pb, s));
        case 2: return cuda_status(launch_ep_combine_routed(P, pb, y, pair_pos, s));
        default: return cuda_status(launch_ep_combine(P, pb, y, pair_pos, s));
    }
}

int qmoe_ep_combine(const qmoe_block* B, const qmoe_dims* D, const void* y_pairs, const int32_t* pair_pos, int T,
                    const float* residual, float* out, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    return ep_combine_impl(B, D, y_pairs, pair_pos, T, residual, out, ws, ws_bytes, stream, 0);
}

int qmoe_ep_shared(const qmoe_block* B, const qmoe_dims* D, int T, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    return ep_combine_impl(B, D, nullptr, nullptr, T, nullptr, nullptr, ws, ws_bytes, stream, 1);
}

int qmoe_ep_combine_routed(const qmoe_block* B, const qmoe_dims* D, const void* y_pairs, const int32_t* pair_pos,
                           int T, const float* residual, float* out, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    return ep_combine_impl(B, D, y_pairs, pair_pos, T, residual, out, ws, ws_bytes, stream, 2);
}

int qmoe_block_kernel_count(const qmoe_block* B, const qmoe_dims* D, int T) {
    int st;
    if (T <= 0) return -QMOE_ERR_ARG;
    if ((st = check_dims(D)) || (st = check_block(B, D))) return -st;
    if (T > kDecodeMaxT) {  // the prefill path (with a workspace sized for T)
        DecodeParams P = make_params(B, D, nullptr, nullptr, nullptr, T, nullptr);
        if (prefill_supported(P)) return prefill_kernel_count(P);
    }
    int n = 0;
    for (int t0 = 0; t0 < T; t0 += kDecodeMaxT) {
        const int nt = std::min(kDecodeMaxT, T - t0);
        DecodeParams P = make_params(B, D, nullptr, nullptr, nullptr, nt, nullptr);
        n += use_fused(P) ? 2 : 3;
    }
    return n;
}

static int block_forward_impl(const qmoe_block* B, const qmoe_dims* D, const float* x, float* out,
                              const float* residual, const float* norm_w, float eps, int T, void* ws,
                              size_t ws_bytes, qmoe_stream_t stream) {
    int st = check_common(B, D, T, ws, ws_bytes, 1 << 30);
    if (st) return st;
    if (!x || !out) return QMOE_ERR_ARG;
    if (!aligned16(x) || (norm_w && !aligned16(norm_w))) return QMOE_ERR_ALIGN;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (T > kDecodeMaxT && ws_layout(*D, T).total <= ws_bytes) {
        // prefill: one pass over all tokens, expert products on the tensor cores
        DecodeParams P = make_params(B, D, x, out, residual, T, ws);
        if (norm_w) {
            P.prenorm = 1;
            P.norm_w = norm_w;
            P.eps = eps;
        }
        if (prefill_supported(P)) {
            return cuda_status(launch_prefill(P, prefill_bufs(*D, T, ws), s));
        }
    }
    for (int t0 = 0; t0 < T; t0 += kDecodeMaxT) {
        const int n = std::min(kDecodeMaxT, T - t0);
        const size_t o = static_cast<size_t>(t0) * D->d_model;
        DecodeParams P = make_params(B, D, x + o, out + o, residual ? residual + o : nullptr, n, ws);
        if (norm_w) {
            P.prenorm = 1;
            P.norm_w = norm_w;
            P.eps = eps;
        }
        if (!decode_supported(P)) return QMOE_ERR_UNSUPPORTED;
        const bool fused = use_fused(P);
        P.route_in_router = fused ? 0 : 1;
        cudaError_t e = launch_router(P, s);
        if (fused) {
            if (e == cudaSuccess) e = launch_experts(P, s);
        } else {
            if (e == cudaSuccess) e = launch_gateup(P, s);
            if (e == cudaSuccess) e = launch_down(P, s);
        }
        if (e != cudaSuccess) return QMOE_ERR_CUDA;
    }
    return QMOE_OK;
}

int qmoe_block_forward(const qmoe_block* B, const qmoe_dims* D, const float* x, float* out, const float* residual,
                       int T, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    return block_forward_impl(B, D, x, out, residual, nullptr, 0.0f, T, ws, ws_bytes, stream);
}

int qmoe_block_forward_prenorm(const qmoe_block* B, const qmoe_dims* D, const float* resid, const float* norm_weight,
                               float eps, float* out, int T, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    if (!norm_weight) return QMOE_ERR_ARG;
    if (!(eps > 0.0f)) return QMOE_ERR_ARG;
    return block_forward_impl(B, D, resid, out, resid, norm_weight, eps, T, ws, ws_bytes, stream);
}

int qmoe_stack_forward(const qmoe_block* blocks, const float* const* norm_weights, int n_layers, const qmoe_dims* D,
                       float eps, float* resid, float* tmp, int T, void* ws, size_t ws_bytes, qmoe_stream_t stream) {
    if (!blocks || !norm_weights || n_layers <= 0 || !resid || !tmp || resid == tmp) return QMOE_ERR_ARG;
    // layers alternate between the two buffers; an odd count ends in tmp and is copied back
    const float* x = resid;
    for (int l = 0; l < n_layers; ++l) {
        float* out = (l & 1) ? resid : tmp;
        const int st = qmoe_block_forward_prenorm(blocks + l, D, x, norm_weights[l], eps, out, T, ws, ws_bytes, stream);
        if (st != QMOE_OK) return st;
        x = out;
    }
    if (n_layers & 1)
        return cuda_status(cudaMemcpyAsync(resid, tmp, sizeof(float) * static_cast<size_t>(T) * D->d_model,
                                           cudaMemcpyDeviceToDevice, reinterpret_cast<cudaStream_t>(stream)));
    return QMOE_OK;
}

int qmoe_trace_enable(uint64_t* buf, size_t bytes) {
    if (buf && bytes < qmoe_trace_bytes()) return QMOE_ERR_ARG;
    g_trace = buf;
    return QMOE_OK;
}

size_t qmoe_trace_bytes(void) { return sizeof(uint64_t) * kTraceKinds * kTraceCtas * kTraceEvents; }

int qmoe_check_errors(void* ws, const qmoe_dims* D, uint32_t* err, qmoe_stream_t stream) {
    (void)D;
    if (!ws) return QMOE_ERR_WORKSPACE;
    cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    if (cudaStreamSynchronize(s) != cudaSuccess) return QMOE_ERR_CUDA;
    uint32_t w[2] = {0, 0xFFFFFFFFu};
    uint32_t* ctrl = static_cast<uint32_t*>(ws);
    if (cudaMemcpy(w, ctrl + CTRL_ERROR, sizeof(w), cudaMemcpyDeviceToHost) != cudaSuccess) return QMOE_ERR_CUDA;
    const uint32_t clear[2] = {0u, 0xFFFFFFFFu};
    if (cudaMemcpy(ctrl + CTRL_ERROR, clear, sizeof(clear), cudaMemcpyHostToDevice) != cudaSuccess)
        return QMOE_ERR_CUDA;
    if (err) { err[0] = w[0]; err[1] = w[1]; }
    if (w[0] & EF_ROUTING) return QMOE_ERR_ROUTING;
    if (w[0] & EF_NOT_NORMALIZED) return QMOE_ERR_NOT_NORMALIZED;
    if (w[0] & (EF_TIMEOUT | EF_ALIGN)) return QMOE_ERR_TIMEOUT;
    return QMOE_OK;
}

int qmoe_synth_fill(void* dst, uint32_t type, uint64_t n, uint64_t seed, uint64_t stream_id, float sigma,
                    qmoe_stream_t stream) {
    const int be = blk_elems(static_cast<int>(type));
    if (!dst || be == 0 || n % be) return QMOE_ERR_ARG;
    return cuda_status(
        launch_synth(dst, static_cast<int>(type), n / be, seed, stream_id, sigma, reinterpret_cast<cudaStream_t>(stream)));
}

}  // extern "C"
