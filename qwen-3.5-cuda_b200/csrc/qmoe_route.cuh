// Per-token expert selection shared by the decode and prefill paths:
// top-k over the router logits (moe.cu:7-52 semantics) and the softmax over
// the selected logits, one warp per token.
#pragma once
#include <cstdint>
#include "qmoe_dev.cuh"
#include "qmoe_internal.h"

namespace qmoe {

// Order-preserving key of a finite float (-0 and +0 map to the same key).
__device__ __forceinline__ uint32_t fkey(float v) {
    const uint32_t u = __float_as_uint(v + 0.0f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__device__ __forceinline__ float fkey_inv(uint32_t key) {
    return __uint_as_float((key & 0x80000000u) ? (key & 0x7FFFFFFFu) : ~key);
}

// 64-bit sort key of a lane's candidate i: logit key, then lower i first
__device__ __forceinline__ uint64_t cand_key(uint32_t key, int i) {
    return (static_cast<uint64_t>(key) << 8) | static_cast<uint32_t>(7 - i);
}
__device__ __forceinline__ void cex(uint64_t& a, uint64_t& b) {  // a <- max, b <- min
    const uint64_t hi = a > b ? a : b, lo = a > b ? b : a;
    a = hi;
    b = lo;
}

// Softmax over the k selected logits held by lanes 0..k-1 (moe.cu:41-51):
// max, then exp(v - max) summed sequentially over j = 0..k-1, then one
// division per weight.  `rs` is the sequential sum of the weights, checked by
// the caller as layer_moe.cpp:114-124 does on the host.  KM >= k bounds the
// unrolled chains.
template <int KM>
__device__ __forceinline__ void softmax_selected(float my_v, int k, int lane, float& wj, float& rs) {
    float sel[KM];
#pragma unroll
    for (int j = 0; j < KM; ++j) sel[j] = __shfl_sync(0xffffffffu, my_v, j);
    float mx = sel[0];
#pragma unroll
    for (int j = 1; j < KM; ++j) if (j < k) mx = fmaxf(mx, sel[j]);
    const float ex = (lane < k) ? expf(my_v - mx) : 0.0f;
#pragma unroll
    for (int j = 0; j < KM; ++j) sel[j] = __shfl_sync(0xffffffffu, ex, j);
    float sum = 0.0f;
#pragma unroll
    for (int j = 0; j < KM; ++j) if (j < k) sum += sel[j];
    wj = ex / sum;
#pragma unroll
    for (int j = 0; j < KM; ++j) sel[j] = __shfl_sync(0xffffffffu, wj, j);
    rs = 0.0f;
#pragma unroll
    for (int j = 0; j < KM; ++j) if (j < k) rs += sel[j];
}

// Top-k selection and softmax of one token by one warp (moe.cu:7-52 and the
// checks of layer_moe.cpp:114-124): lane j < k returns the j-th selected
// expert and its weight; `flag` is EF_ROUTING / EF_NOT_NORMALIZED / 0 on
// every lane.  Each lane holds the logits of experts lane + 32 i, sorted once
// (descending key, ascending i) by an 8-input Batcher network; a round is one
// redux for the largest head key and one for the lowest expert id among the
// lanes whose head holds it, after which the winning lane pops its head.
__device__ __forceinline__ void select_token(const float* logits, int E, int k, int lane, int& my_idx, float& wj,
                                             uint32_t& flag) {
    uint64_t c[8];
    uint32_t amax = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        const float v = e < E ? __ldcg(logits + e) : 0.0f;
        c[i] = cand_key(e < E ? fkey(v) : 0u, i);
        amax = max(amax, e < E ? (__float_as_uint(v) & 0x7FFFFFFFu) : 0u);
    }
    const bool finite = __reduce_max_sync(0xffffffffu, amax) < 0x7F800000u;
    // Batcher odd-even merge sort of 8 (19 comparators)
    cex(c[0], c[1]); cex(c[2], c[3]); cex(c[4], c[5]); cex(c[6], c[7]);
    cex(c[0], c[2]); cex(c[1], c[3]); cex(c[4], c[6]); cex(c[5], c[7]);
    cex(c[1], c[2]); cex(c[5], c[6]);
    cex(c[0], c[4]); cex(c[1], c[5]); cex(c[2], c[6]); cex(c[3], c[7]);
    cex(c[2], c[4]); cex(c[3], c[5]);
    cex(c[1], c[2]); cex(c[3], c[4]); cex(c[5], c[6]);
    my_idx = -1;
    float my_v = 0.0f;
    if (finite) {
        for (int j = 0; j < k; ++j) {
            const uint32_t hk = static_cast<uint32_t>(c[0] >> 8);
            const int he = lane + 32 * (7 - static_cast<int>(c[0] & 7u));
            const uint32_t mk = __reduce_max_sync(0xffffffffu, hk);
            const int win = static_cast<int>(__reduce_min_sync(0xffffffffu, hk == mk ? static_cast<uint32_t>(he) : 0xFFFFFFFFu));
            if (he == win) {
#pragma unroll
                for (int i = 0; i < 7; ++i) c[i] = c[i + 1];
                c[7] = 0;
            }
            if (lane == j) { my_idx = win; my_v = fkey_inv(mk); }
        }
    }
    // softmax over the selected logits (moe.cu:41-51)
    float rs;
    if (k <= 8) softmax_selected<8>(my_v, k, lane, wj, rs);
    else softmax_selected<kMaxTopK>(my_v, k, lane, wj, rs);
    const bool lane_ok = lane >= k || (my_idx >= 0 && my_idx < E && isfinite(wj) && wj >= 0.0f);
    const bool ok = finite && __all_sync(0xffffffffu, lane_ok);
    flag = 0;
    if (!ok) flag = EF_ROUTING;
    else if (!isfinite(rs) || fabsf(rs - 1.0f) > 1e-4f) flag = EF_NOT_NORMALIZED;
}

}  // namespace qmoe
