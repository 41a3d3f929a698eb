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

// Sum of lanes 0..k-1's v in lane order (one rounding per add, as a
// sequential loop): the first eight values are gathered with independent
// shuffles, then added in order.
__device__ __forceinline__ float ordered_sum(float v, int k) {
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = __shfl_sync(0xffffffffu, v, j);
    float s = 0.0f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s = j < k ? s + g[j] : s;
#pragma unroll 1
    for (int j = 8; j < k; ++j) s += __shfl_sync(0xffffffffu, v, j);
    return s;
}

// Top-k selection and softmax of one token by one warp (moe.cu:7-52 and the
// checks of layer_moe.cpp:114-124): lane j < k returns the j-th selected
// expert and its weight; `flag` is EF_ROUTING / EF_NOT_NORMALIZED / 0 on
// every lane.
//
// Lane L holds the order-preserving keys of experts L + 32 i (i = 0..7).  A
// round takes each lane's largest key not yet taken (strict >, so the lowest
// i wins a tie inside the lane), one redux for the largest key over the warp
// and one for the lowest expert id among the lanes that hold it -- the
// reference's "largest logit, lowest index on ties" (moe.cu:20-33) -- and the
// owning lane marks its candidate taken.  Softmax over the selected logits
// (moe.cu:41-51): max, exp(v - max), the sum in selection order j = 0..k-1,
// one division per weight.
//
// Every loop is rolled: this runs once per launch, so its code is fetched
// cold each time, and short code is what keeps it fast.
__device__ __forceinline__ void select_token(const float* logits, int E, int k, int lane, int& my_idx, float& wj,
                                             uint32_t& flag) {
    uint32_t key[8];
    uint32_t amax = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int e = lane + 32 * i;
        const float v = e < E ? __ldcg(logits + e) : 0.0f;
        key[i] = e < E ? fkey(v) : 0u;  // finite logits have keys >= 0x00800000
        amax = max(amax, e < E ? (__float_as_uint(v) & 0x7FFFFFFFu) : 0u);
    }
    const bool finite = __reduce_max_sync(0xffffffffu, amax) < 0x7F800000u;
    uint32_t taken = 0;
    my_idx = -1;
    float my_v = 0.0f;
#pragma unroll 1
    for (int j = 0; j < (finite ? k : 0); ++j) {
        uint32_t best = 0;
        int bi = 8;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const bool ok = !((taken >> i) & 1u) && key[i] > best;
            best = ok ? key[i] : best;
            bi = ok ? i : bi;
        }
        const uint32_t mk = __reduce_max_sync(0xffffffffu, best);
        const uint32_t win = __reduce_min_sync(0xffffffffu, (bi < 8 && best == mk) ? static_cast<uint32_t>(lane + 32 * bi)
                                                                                  : 0xFFFFFFFFu);
        if (static_cast<int>(win) == lane + 32 * bi) taken |= 1u << bi;
        if (lane == j) {
            my_idx = static_cast<int>(win);
            my_v = fkey_inv(mk);
        }
    }
    // the selection is in descending order, so the largest selected logit
    // (moe.cu:41-44) is lane 0's
    const float mx = __shfl_sync(0xffffffffu, my_v, 0);
    const float ex = (lane < k) ? expf(my_v - mx) : 0.0f;
    const float sum = ordered_sum(ex, k);
    wj = ex / sum;
    const float rs = ordered_sum(wj, k);
    const bool lane_ok = lane >= k || (my_idx >= 0 && my_idx < E && isfinite(wj) && wj >= 0.0f);
    const bool ok = finite && __all_sync(0xffffffffu, lane_ok);
    flag = 0;
    if (!ok) flag = EF_ROUTING;
    else if (!isfinite(rs) || fabsf(rs - 1.0f) > 1e-4f) flag = EF_NOT_NORMALIZED;
}

}  // namespace qmoe
