// Expert-parallel exchange layout (no counterpart in the reference, which
// runs the MoE block on one GPU, src/layer_moe.cpp:98-154).
//
// Sending rank, from the top-k of its T tokens (Eloc = E / G experts per
// rank: contiguous shards, or any placement permutation):
//   k_ep_hcount  per 256-token block and rank: rows (tokens with at least one
//                expert on the rank) and pairs (token, slot) going there
//   k_ep_hscan   exclusive scan of those over the blocks, per rank; totals and
//                the rank offsets of the send rows and of the returned pairs
//   k_ep_hplace  positions: send row of (t, r) = rank offset + earlier blocks +
//                earlier tokens of the block; the meta row (slot j -> local
//                expert id or -1); pair_pos[t*k + j] = place of the pair in the
//                returned outputs; the source token of every send row
//   k_ep_copy    the fp16 rows into the send buffer, all SMs
// Receiving rank, from the meta rows of n received rows:
//   k_ep_qcount / k_ep_qscan / k_ep_qmap
//                the (row, slot) order number of every valid slot (-1 for the
//                others): the order the outputs go back in, the same numbering
//                the sender's pair_pos uses for its chunk.
#include <cuda_fp16.h>

#include "qmoe_dev.cuh"
#include "qmoe_internal.h"

namespace qmoe {

constexpr int EPB = 256;  // tokens (rows) per block
constexpr int kEpMaxRanks = 32;
constexpr int kEpMaxK = 8;  // top-k slots per token on this path

__device__ __forceinline__ int ep_rank_of(int e, int eloc) { return e >= 0 ? e / eloc : -1; }

// Expert id as placed on the ranks: slot p = r*Eloc + local id on rank r
// (placement: a permutation of the experts; null = contiguous shards).
__device__ __forceinline__ int ep_placed(const int32_t* __restrict__ idx, const int32_t* __restrict__ placement,
                                         int i) {
    const int e = __ldg(idx + i);
    return (placement && e >= 0) ? __ldg(placement + e) : e;
}

__global__ void __launch_bounds__(EPB) k_ep_hcount(const int32_t* __restrict__ idx, const int32_t* __restrict__ placement,
                                                   int T, int k, int eloc, int G, int32_t* __restrict__ blk) {
    __shared__ int s_cnt[2 * kEpMaxRanks];
    if (threadIdx.x < 2 * G) s_cnt[threadIdx.x] = 0;
    __syncthreads();
    const int t = blockIdx.x * EPB + threadIdx.x;
    if (t < T) {
        uint32_t mask = 0;
        for (int j = 0; j < k; ++j) {
            const int r = ep_rank_of(ep_placed(idx, placement, t * k + j), eloc);
            if (r >= 0 && r < G) {
                mask |= 1u << r;
                atomicAdd(s_cnt + G + r, 1);
            }
        }
        while (mask) {
            const int r = __ffs(mask) - 1;
            mask &= mask - 1;
            atomicAdd(s_cnt + r, 1);
        }
    }
    __syncthreads();
    if (threadIdx.x < 2 * G) blk[blockIdx.x * 2 * G + threadIdx.x] = s_cnt[threadIdx.x];
}

// One CTA of 64 threads: column c < 2G of blk[nb][2G] scanned over the blocks (in place),
// counts[c] = column total; rank_off[c] = prefix of the totals over the
// ranks (rows: c < G, pairs: c >= G).
__global__ void k_ep_hscan(int32_t* __restrict__ blk, int nb, int G, int32_t* __restrict__ counts,
                           int32_t* __restrict__ rank_off) {
    const int c = threadIdx.x;
    int run = 0;
    if (c < 2 * G)
        for (int b = 0; b < nb; ++b) {
            const int v = blk[b * 2 * G + c];
            blk[b * 2 * G + c] = run;
            run += v;
        }
    __shared__ int s_tot[2 * kEpMaxRanks];
    if (c < 2 * G) {
        s_tot[c] = run;
        counts[c] = run;
    }
    __syncthreads();
    if (c < 2 * G) {
        const int r0 = c < G ? 0 : G;
        int off = 0;
        for (int r = r0; r < c; ++r) off += s_tot[r];
        rank_off[c] = off;
    }
}

__global__ void __launch_bounds__(EPB) k_ep_hplace(const int32_t* __restrict__ idx, const int32_t* __restrict__ placement,
                                                   int T, int k, int eloc, int G,
                                                   const int32_t* __restrict__ blk, const int32_t* __restrict__ rank_off,
                                                   int32_t* __restrict__ row_src, int32_t* __restrict__ send_meta,
                                                   int32_t* __restrict__ pair_pos) {
    __shared__ int s_wrows[EPB / 32][kEpMaxRanks], s_wpairs[EPB / 32][kEpMaxRanks];
    __shared__ int2 s_copy[EPB * kEpMaxK];  // (source token, send row) of the block's rows
    __shared__ int s_ncopy;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int t = blockIdx.x * EPB + threadIdx.x;
    const bool live = t < T;
    const unsigned lt = (1u << lane) - 1u;
    if (threadIdx.x == 0) s_ncopy = 0;
    int ids[kEpMaxK];  // this token's experts (k <= kEpMaxK; unused slots -1)
    uint32_t mask = 0;
#pragma unroll
    for (int j = 0; j < kEpMaxK; ++j) {
        ids[j] = (live && j < k) ? ep_placed(idx, placement, t * k + j) : -1;
        const int r = ep_rank_of(ids[j], eloc);
        if (r >= 0 && r < G) mask |= 1u << r;
    }
    auto npairs = [&](int r) {
        int n = 0;
#pragma unroll
        for (int j = 0; j < kEpMaxK; ++j) n += ep_rank_of(ids[j], eloc) == r ? 1 : 0;
        return n;
    };
    // per-warp totals for every rank
    for (int r = 0; r < G; ++r) {
        const unsigned b = __ballot_sync(0xffffffffu, (mask >> r) & 1u);
        int np = npairs(r);
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) np += __shfl_xor_sync(0xffffffffu, np, o);
        if (lane == 0) {
            s_wrows[warp][r] = __popc(b);
            s_wpairs[warp][r] = np;
        }
    }
    __syncthreads();
    int2* copies = s_copy;
    for (int r = 0; r < G; ++r) {
        const bool has = (mask >> r) & 1u;
        const unsigned b = __ballot_sync(0xffffffffu, has);
        const int np = npairs(r);
        int incl = np;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, incl, o);
            if (lane >= o) incl += y;
        }
        int wrow = 0, wpair = 0;
        for (int w = 0; w < warp; ++w) {
            wrow += s_wrows[w][r];
            wpair += s_wpairs[w][r];
        }
        if (!has) continue;
        const int row = rank_off[r] + blk[blockIdx.x * 2 * G + r] + wrow + __popc(b & lt);
        const int pbase = rank_off[G + r] + blk[blockIdx.x * 2 * G + G + r] + wpair + incl - np;
        int q = 0;
#pragma unroll
        for (int j = 0; j < kEpMaxK; ++j) {
            if (j >= k) break;
            const bool mine = ep_rank_of(ids[j], eloc) == r;
            send_meta[static_cast<size_t>(row) * k + j] = mine ? ids[j] - r * eloc : -1;
            if (mine) pair_pos[t * k + j] = pbase + q++;
        }
        const int slot = atomicAdd(&s_ncopy, 1);
        copies[slot] = make_int2(t, row);
    }
    if (live) {
#pragma unroll
        for (int j = 0; j < kEpMaxK; ++j)
            if (j < k && (ids[j] < 0 || ep_rank_of(ids[j], eloc) >= G)) pair_pos[t * k + j] = -1;
    }
    __syncthreads();
    // the source token of every send row, for k_ep_copy
    for (int i = threadIdx.x; i < s_ncopy; i += EPB) row_src[copies[i].y] = copies[i].x;
}

// send_rows[i] = x16[row_src[i]] for the n = counts[0..G) rows: one warp per
// row, 16 bytes per lane and step, grid-stride over all SMs.
__global__ void __launch_bounds__(256) k_ep_copy(const __half* __restrict__ x16, int d, const int32_t* __restrict__ row_src,
                                                 const int32_t* __restrict__ counts, int G, __half* __restrict__ send_rows) {
    int n = 0;
    for (int r = 0; r < G; ++r) n += __ldg(counts + r);
    const int lane = threadIdx.x & 31, chunks = d / 8;
    for (int i = blockIdx.x * 8 + (threadIdx.x >> 5); i < n; i += gridDim.x * 8) {
        const uint4* src = reinterpret_cast<const uint4*>(x16 + static_cast<size_t>(__ldg(row_src + i)) * d);
        uint4* dst = reinterpret_cast<uint4*>(send_rows + static_cast<size_t>(i) * d);
        for (int c = lane; c < chunks; c += 32) dst[c] = __ldg(src + c);
    }
}

// Receiver: valid slots per 256-row block.
__global__ void __launch_bounds__(EPB) k_ep_qcount(const int32_t* __restrict__ meta, int n, int k,
                                                   int32_t* __restrict__ qblk) {
    __shared__ int s_w[EPB / 32];
    const int row = blockIdx.x * EPB + threadIdx.x;
    int c = 0;
    if (row < n)
        for (int j = 0; j < k; ++j) c += __ldg(meta + static_cast<size_t>(row) * k + j) >= 0 ? 1 : 0;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
    if ((threadIdx.x & 31) == 0) s_w[threadIdx.x >> 5] = c;
    __syncthreads();
    if (threadIdx.x == 0) {
        int s = 0;
        for (int w = 0; w < EPB / 32; ++w) s += s_w[w];
        qblk[blockIdx.x] = s;
    }
}

// One CTA: exclusive scan of qblk[nb] in place, qblk[nb] = total.
__global__ void __launch_bounds__(1024) k_ep_qscan(int32_t* __restrict__ qblk, int nb) {
    __shared__ int s_w[32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int per = (nb + blockDim.x - 1) / blockDim.x;
    const int lo = threadIdx.x * per, hi = min(nb, lo + per);
    int loc = 0;
    for (int i = lo; i < hi; ++i) loc += qblk[i];
    int inc = loc;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s_w[warp] = inc;
    __syncthreads();
    int base = 0, total = 0;
    for (int w = 0; w < static_cast<int>(blockDim.x >> 5); ++w) {
        base += w < warp ? s_w[w] : 0;
        total += s_w[w];
    }
    int run = base + inc - loc;
    for (int i = lo; i < hi; ++i) {
        const int v = qblk[i];
        qblk[i] = run;
        run += v;
    }
    if (threadIdx.x == 0) qblk[nb] = total;
}

__global__ void __launch_bounds__(EPB) k_ep_qmap(const int32_t* __restrict__ meta, int n, int k,
                                                 const int32_t* __restrict__ qblk, int32_t* __restrict__ qmap) {
    __shared__ int s_w[EPB / 32];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int row = blockIdx.x * EPB + threadIdx.x;
    int c = 0;
    if (row < n)
        for (int j = 0; j < k; ++j) c += __ldg(meta + static_cast<size_t>(row) * k + j) >= 0 ? 1 : 0;
    int inc = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s_w[warp] = inc;
    __syncthreads();
    int q = __ldg(qblk + blockIdx.x) + inc - c;
    for (int w = 0; w < warp; ++w) q += s_w[w];
    if (row < n)
        for (int j = 0; j < k; ++j) {
            const bool v = __ldg(meta + static_cast<size_t>(row) * k + j) >= 0;
            qmap[static_cast<size_t>(row) * k + j] = v ? q++ : -1;
        }
}

size_t ep_dispatch_scratch_bytes(int T, int G) {
    const size_t nb = (static_cast<size_t>(T) + EPB - 1) / EPB;
    const size_t rows = static_cast<size_t>(T) * (G < kEpMaxK ? G : kEpMaxK);
    return align_up(nb * 2 * G * sizeof(int32_t), 256) + align_up(2 * G * sizeof(int32_t), 256) +
           align_up(rows * sizeof(int32_t), 256);
}

bool ep_dispatch_supported(int k, int G) { return G >= 1 && G <= kEpMaxRanks && k >= 1 && k <= kEpMaxK; }

cudaError_t launch_ep_dispatch(const int32_t* idx, const int32_t* placement, int T, int k, int E, int G,
                               const __half* x16, int d, __half* send_rows, int32_t* send_meta, int32_t* counts,
                               int32_t* pair_pos, void* scratch, cudaStream_t s) {
    const int nb = (T + EPB - 1) / EPB, eloc = E / G;
    int32_t* blk = static_cast<int32_t*>(scratch);
    const size_t o1 = align_up(static_cast<size_t>(nb) * 2 * G * sizeof(int32_t), 256);
    int32_t* rank_off = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + o1);
    int32_t* row_src = reinterpret_cast<int32_t*>(static_cast<uint8_t*>(scratch) + o1 +
                                                  align_up(2 * G * sizeof(int32_t), 256));
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    k_ep_hcount<<<nb, EPB, 0, s>>>(idx, placement, T, k, eloc, G, blk);
    k_ep_hscan<<<1, 64, 0, s>>>(blk, nb, G, counts, rank_off);
    k_ep_hplace<<<nb, EPB, 0, s>>>(idx, placement, T, k, eloc, G, blk, rank_off, row_src, send_meta, pair_pos);
    k_ep_copy<<<4 * sms, 256, 0, s>>>(x16, d, row_src, counts, G, send_rows);
    return cudaGetLastError();
}

cudaError_t launch_ep_qmap(const int32_t* meta, int n, int k, int32_t* qblk, int32_t* qmap, cudaStream_t s) {
    const int nb = (n + EPB - 1) / EPB;
    k_ep_qcount<<<nb, EPB, 0, s>>>(meta, n, k, qblk);
    k_ep_qscan<<<1, 1024, 0, s>>>(qblk, nb);
    k_ep_qmap<<<nb, EPB, 0, s>>>(meta, n, k, qblk, qmap);
    return cudaGetLastError();
}

}  // namespace qmoe
