// Stable token->expert permutation for any number of tokens (no counterpart
// in the reference, which routes one token at a time on the host,
// src/layer_moe.cpp:127).  Pairs p = t*k + j are ordered by (expert, t, j).
//
// One CTA of DW warps.  Warp w owns the contiguous pair segment
// [w*seg, (w+1)*seg): pass 1 counts its experts, an exclusive scan over the
// (expert, warp) table gives every warp its first slot per expert, and pass 2
// walks the segment again in order, ranking equal experts inside each batch
// of 32 pairs with __match_any_sync, so the order within an expert is the
// pair order (a stable counting sort).
#include "qmoe_dev.cuh"
#include "qmoe_internal.h"

namespace qmoe {

constexpr int DW = 32;

__global__ void __launch_bounds__(DW * 32) k_dispatch(const int32_t* __restrict__ idx, int NP, int E,
                                                      int32_t* __restrict__ offsets, int32_t* __restrict__ perm,
                                                      int32_t* __restrict__ inv_perm, int32_t* __restrict__ table) {
    // table: [E][DW] counts -> bases (global scratch, E*DW ints)
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const unsigned FULLM = 0xffffffffu, lt = (1u << lane) - 1u;
    const int seg = (NP + DW - 1) / DW;
    const int p_lo = warp * seg, p_hi = min(NP, p_lo + seg);
    for (int i = threadIdx.x; i < E * DW; i += blockDim.x) table[i] = 0;
    __syncthreads();
    // pass 1: per-warp counts (only the group leader writes, so no races)
    for (int base = p_lo; base < p_hi; base += 32) {
        const int p = base + lane;
        const int e = p < p_hi ? idx[p] : -1;
        const bool valid = e >= 0 && e < E;
        const unsigned peers = __match_any_sync(FULLM, valid ? e : -1);
        if (valid && (peers >> lane) == 1u) table[e * DW + warp] += __popc(peers);
        __syncwarp();
    }
    __syncthreads();
    // exclusive scan over the table in (expert, warp) order, by warp 0
    __shared__ int s_total;
    if (warp == 0) {
        const int n = E * DW;
        const int per = (n + 31) / 32;
        const int lo = lane * per, hi = min(n, lo + per);
        int loc = 0;
        for (int i = lo; i < hi; ++i) loc += table[i];
        int inc = loc;
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(FULLM, inc, o);
            if (lane >= o) inc += a;
        }
        int run = inc - loc;
        for (int i = lo; i < hi; ++i) {
            const int c = table[i];
            table[i] = run;
            if ((i % DW) == 0) offsets[i / DW] = run;
            run += c;
        }
        if (lane == 31) s_total = inc;
    }
    __syncthreads();
    if (threadIdx.x == 0) offsets[E] = s_total;
    // pass 2: stable placement
    for (int base = p_lo; base < p_hi; base += 32) {
        const int p = base + lane;
        const int e = p < p_hi ? idx[p] : -1;
        const bool valid = e >= 0 && e < E;
        const unsigned peers = __match_any_sync(FULLM, valid ? e : -1);
        const int rank = __popc(peers & lt);
        const int pos = valid ? table[e * DW + warp] + rank : -1;
        __syncwarp();
        if (valid && (peers >> lane) == 1u) table[e * DW + warp] += __popc(peers);
        __syncwarp();
        if (p < p_hi) {
            if (valid) perm[pos] = p;
            if (inv_perm) inv_perm[p] = pos;
        }
    }
}

size_t dispatch_scratch_bytes(int E) { return sizeof(int32_t) * static_cast<size_t>(E) * DW; }

// Scratch of qmoe_dispatch_noalloc: a fixed per-device array of E * DW
// counters for E <= kNoAllocMaxExperts (32 KiB).  k_dispatch clears the part
// it uses at the start of every launch, so it needs no initialisation.
static __device__ __align__(256) int32_t g_dispatch_scratch[kNoAllocMaxExperts * DW];

cudaError_t dispatch_noalloc_scratch(int32_t** p) {
    return cudaGetSymbolAddress(reinterpret_cast<void**>(p), g_dispatch_scratch);
}

cudaError_t launch_dispatch(const int32_t* idx, int NP, int E, int32_t* offsets, int32_t* perm, int32_t* inv_perm,
                            int32_t* table, cudaStream_t s) {
    k_dispatch<<<1, DW * 32, 0, s>>>(idx, NP, E, offsets, perm, inv_perm, table);
    return cudaGetLastError();
}

}  // namespace qmoe
