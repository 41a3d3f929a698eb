// Internal host/device structures of the qmoe library (not part of the C-ABI).
#pragma once
#include <cstddef>
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include "../../include/qmoe.h"

namespace qmoe {

constexpr int kDecodeMaxT = 8;   // tokens per decode-path launch (larger T is sliced)
constexpr int kMaxNormDim = 2048;  // largest d_model (the argument checks enforce it)
constexpr int kMaxExperts = 256; // experts supported by the routing kernels
constexpr int kMaxTopK = 32;
constexpr int kNoAllocMaxExperts = 256;  // largest E of qmoe_dispatch_noalloc (fixed scratch)

__host__ __device__ inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// GGML block geometry (reference include/quantized.hpp:49-96).
__host__ __device__ inline int blk_elems(int t) {
    switch (t) {
        case 0: case 1: case 30: return 1;
        case 2: case 6: case 8: return 32;
        case 12: case 13: case 14: return 256;
        default: return 0;
    }
}
__host__ __device__ inline int blk_bytes(int t) {
    switch (t) {
        case 0: return 4;
        case 1: case 30: return 2;
        case 2: return 18;
        case 6: return 22;
        case 8: return 34;
        case 12: return 144;
        case 13: return 176;
        case 14: return 210;
        default: return 0;
    }
}
__host__ __device__ inline uint64_t row_bytes(int t, int K) {
    int be = blk_elems(t);
    return be ? static_cast<uint64_t>(K / be) * static_cast<uint64_t>(blk_bytes(t)) : 0;
}

// Packed routing schedule written by the router's last CTA and read once by
// the expert kernels: [0] n_active, [1] n_pairs, [2..3] spare, then per
// active expert s: {expert, first permuted position, pair count}, then the
// permutation (pair ids in (expert, token, slot) order), then the token of
// each permuted pair.
constexpr int SCHED_HDR = 4;
__host__ __device__ inline int sched_max_src(int T, int k, int E) { return T * k < E ? T * k : E; }
__host__ __device__ inline int sched_perm_off(int T, int k, int E) { return SCHED_HDR + 3 * sched_max_src(T, k, E); }
__host__ __device__ inline int sched_tok_off(int T, int k, int E) { return sched_perm_off(T, k, E) + T * k; }
__host__ __device__ inline int sched_words(int T, int k, int E) { return sched_tok_off(T, k, E) + T * k; }

// Workspace layout for a call with T tokens (all offsets 256-byte aligned).
struct WsLayout {
    size_t ctrl, logits, topk_idx, topk_w, offsets, perm, inv_perm, active, sched, xnorm, hidden, hq, total;
    // prefill regions (T > kDecodeMaxT): source token per permuted pair, tile
    // prefix per expert, the shared expert's group, dispatch scratch, fp16
    // hidden vectors and expert outputs
    size_t tok_of_pos, tile_start, sh_grp, disp, X16, Hpf, Hs, Y, Ys, xperm, wperm;
    size_t xq_stride;  // bytes per token of x planes in shared memory: 3*d + (d/16)*8
    size_t hq_stride;  // bytes per hidden vector of planes: 3*H + (H/16)*8
    int H;             // max(F, Fs)
};

// Workspace layout for a call with T tokens.  Regions used only by the
// decode kernels (schedule, F32 hidden vectors and their planes) are sized
// for at most kDecodeMaxT tokens; for T > kDecodeMaxT the prefill regions
// follow.
inline WsLayout ws_layout(const qmoe_dims& D, int T) {
    WsLayout L{};
    const int E = D.num_experts, k = D.top_k, d = D.d_model;
    const int H = D.expert_dim > D.shared_dim ? D.expert_dim : D.shared_dim;
    const int P = T * k;
    const int Td = T < kDecodeMaxT ? T : kDecodeMaxT;
    const int nvec = Td * k + Td;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o = align_up(o + bytes, 256); return r; };
    L.ctrl = take(64 * 4);
    L.logits = take(sizeof(float) * static_cast<size_t>(T) * (E + 1));
    L.topk_idx = take(sizeof(int32_t) * P);
    L.topk_w = take(sizeof(float) * P);
    L.offsets = take(sizeof(int32_t) * (E + 1));
    L.perm = take(sizeof(int32_t) * P);
    L.inv_perm = take(sizeof(int32_t) * P);
    L.active = take(sizeof(int32_t) * (Td * k < E ? Td * k : E));
    L.sched = take(sizeof(int32_t) * sched_words(Td, k, E));
    L.xnorm = take(sizeof(float) * static_cast<size_t>(T) * d);
    L.xq_stride = align_up(3 * static_cast<size_t>(d) + static_cast<size_t>(d / 16) * 8, 16);
    L.H = H;
    L.hidden = take(sizeof(float) * static_cast<size_t>(nvec) * H);
    L.hq_stride = align_up(3 * static_cast<size_t>(H) + static_cast<size_t>(H / 16) * 8, 16);
    L.hq = take(L.hq_stride * nvec);
    if (T > kDecodeMaxT) {
        const int F = D.expert_dim, Fs = D.shared_dim;
        L.tok_of_pos = take(sizeof(int32_t) * P);
        L.tile_start = take(sizeof(int32_t) * (E + 1));
        L.sh_grp = take(sizeof(int32_t) * 4);  // {0, T} and the shared expert's tile prefix {0, tiles}
        L.disp = take(sizeof(int32_t) * static_cast<size_t>(E) * ((T + 63) / 64));  // per-64-token-block counts
        L.X16 = take(2 * static_cast<size_t>(T) * d);
        L.Hpf = take(2 * static_cast<size_t>(P) * F);
        L.Hs = take(2 * static_cast<size_t>(T) * Fs);
        L.Y = take(2 * static_cast<size_t>(P) * d);
        L.Ys = take(2 * static_cast<size_t>(T) * d);
        // x_in and the expert router rows in the router's leaf order (F32)
        L.xperm = take(sizeof(float) * static_cast<size_t>(T) * d);
        L.wperm = take(sizeof(float) * static_cast<size_t>(E) * d);
    }
    L.total = o;
    return L;
}

// Workspace of qmoe_ep_experts for up to n received rows of k slots (the
// expert-parallel receiver): dispatch of the (row, slot) pairs over the local
// experts, the GEMM tile plan, the rows gathered in pair order and the hidden
// vectors of the pairs.
struct EpRowsLayout {
    size_t ctrl, offsets, perm, inv_perm, tok_of_pos, out_pos, qmap, qblk, tile_start, disp, H, Xp, total;
};
inline EpRowsLayout ep_rows_layout(const qmoe_dims& D, int n) {
    EpRowsLayout L{};
    const size_t P = static_cast<size_t>(n) * D.top_k, E = D.num_experts;
    size_t o = 0;
    auto take = [&](size_t bytes) { size_t r = o; o = align_up(o + bytes, 256); return r; };
    L.ctrl = take(64 * 4);
    L.offsets = take(sizeof(int32_t) * (E + 1));
    L.perm = take(sizeof(int32_t) * P);
    L.inv_perm = take(sizeof(int32_t) * P);
    L.tok_of_pos = take(sizeof(int32_t) * P);
    L.out_pos = take(sizeof(int32_t) * P);
    L.qmap = take(sizeof(int32_t) * P);
    L.qblk = take(sizeof(int32_t) * ((static_cast<size_t>(n) + 255) / 256 + 1));
    L.tile_start = take(sizeof(int32_t) * (E + 1));
    L.disp = take(sizeof(int32_t) * E * ((static_cast<size_t>(n) + 63) / 64));
    L.H = take(2 * P * static_cast<size_t>(D.expert_dim));
    L.Xp = take(2 * P * static_cast<size_t>(D.d_model));  // received rows gathered in pair order
    L.total = o;
    return L;
}

// Prefill buffers of a workspace (fp16 data as raw 16-bit words).
struct PrefillBufs {
    int32_t* tok_of_pos;
    int32_t* tile_start;
    int32_t* sh_grp;    // [2] {0, T}
    int32_t* sh_tiles;  // [2] {0, ceil(T / 128)}
    int32_t* disp;
    __half* X16;  // fp16 block input, chunk element order
    __half* H;
    __half* Hs;
    __half* Y;
    __half* Ys;
    float* xperm;  // [T][d] x_in in the router leaf order
    float* wperm;  // [E][d] router rows in that order
};

// Phase tracer: kernel kinds x CTAs x events of %globaltimer (ns).
constexpr int kTraceKinds = 3, kTraceCtas = 160, kTraceEvents = 8;

// One weight tensor as seen by the kernels.
struct WArg {
    const uint8_t* p;    // payload
    const uint8_t* end;  // one past the last payload byte
    int type;
    int pad;
};

// Everything the decode kernels need (passed by value).
struct DecodeParams {
    int d, E, k, F, Fs, T;
    int has_shared;
    int num_sms;
    // router (F32/F16/BF16) and the shared-expert gate vector
    const uint8_t* router;
    int router_type;
    const uint8_t* sgate_inp;
    int sgate_type;
    const float* bias;
    WArg gate, up, down, sgate, sup, sdown;
    const float* x;  // [T][d]
    float* out;      // [T][d]
    const float* residual;
    uint64_t* trace;   // optional phase timestamps (qmoe_trace_enable), else null
    int32_t* out_idx;  // optional copies of the routing result
    float* out_w;
    // workspace
    uint32_t* ctrl;
    float* logits;
    int32_t* topk_idx;
    float* topk_w;
    int32_t* offsets;
    int32_t* perm;
    int32_t* inv_perm;
    int32_t* active;
    int32_t* sched;
    float* xnorm;       // [T][d] the block's input after the optional fused RMSNorm
    const float* norm_w;  // optional fused pre-MoE RMSNorm weight [d] (prenorm != 0)
    float eps;
    int prenorm;
    int route_in_router;  // 1: the router's last CTA selects experts; 0: the fused expert kernel does
    size_t xq_stride;
    float* hidden;
    uint8_t* hq;        // [T*k + T] 24-bit planes of silu(g)*u (written by the gate/up kernel)
    size_t hq_stride;
    int H;
};

}  // namespace qmoe
