// Prefill path of the MoE block (many tokens per call): the expert products
// become real contractions (on average T*k/E tokens per expert), so they run
// as grouped GEMMs on the tcgen05 tensor cores with the accumulators in TMEM.
//
//   k_norm_many     RMSNorm of every token, the reference's exact reduction
//                   structure (ops.cu:25-65), x_in [T][d] F32
//   k_route_many    router logits for every token in the reference GEMV order
//                   (matmul_q4.cu:140-167): bit-identical logits, so the same
//                   experts as the reference for every token
//   k_topk_many     one warp per token: top-k, softmax, checks (moe.cu:7-57,
//                   layer_moe.cpp:102-124)
//   k_dispatch      stable (expert, token, slot) permutation (k_dispatch.cu)
//   k_pf_plan       source token of every permuted pair, tile prefix per expert
//   k_pgemm<W,0>    gate/up: H[pair] = silu(x Wg^T) * (x Wu^T), fp16 (routed
//                   experts: rows gathered by token; shared expert: all tokens)
//   k_pgemm<W,1>    down: Y[pair] = H Wd^T, fp16
//   k_pf_combine    out[t] = residual + sum_j w_j Y[pair(t,j)] in slot order j,
//                   then + sigmoid(shared gate) * Y_shared[t] (layer_moe.cpp:127-154)
//
// tcgen05 GEMM: C[128 x 256] (F32, TMEM) += A[128 x 16] * B[256 x 16]^T per
// instruction, kind::f16 (A and B both fp16), both operands K-major in shared
// memory with the 128-byte swizzle: a row of a 64-wide K block is 128 bytes,
// eight rows form a 1024-byte swizzle atom, 16-byte chunk c of row r sits at
// chunk c ^ (r % 8).  Producer warps dequantise the GGUF weight blocks to fp16
// straight into that layout and convert the activations; one thread issues
// the MMAs; four epilogue warps read TMEM.  Inside every 8-element chunk both
// operands use the same element order (0,2,1,3,4,6,5,7), which lets the Q4_K
// nibble pairs become half2 values with one logic op each; the product sums
// over K, so a common permutation of K leaves it unchanged.
#include <cuda_fp16.h>

#include "qmoe_dev.cuh"
#include "qmoe_dq1.cuh"
#include "qmoe_internal.h"
#include "qmoe_route.cuh"

namespace qmoe {

__device__ __forceinline__ __half2 bits_to_half2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

namespace pf {

constexpr int BM = 128;                // tile rows (tokens or pairs) = MMA M
constexpr int BN = 256;                // tile columns = MMA N
constexpr int BK = 64;                 // K per pipeline stage (128 bytes of fp16 per row)
constexpr int PROD_WARPS = 8;          // weight dequantisation + activation staging
constexpr int EPI_WARP0 = 8;           // warps 8..11: TMEM epilogue (lane quarter = warp % 4)
constexpr int MMA_WARP = 12;           // one thread issues the MMAs
constexpr int THREADS = 13 * 32;
constexpr uint32_t A_BYTES = BM * 128;  // 16 KB per stage
constexpr uint32_t B_BYTES = BN * 128;  // 32 KB per weight matrix per stage
// instruction descriptor: D F32, A/B fp16, both K-major, N = 256, M = 128
constexpr uint32_t IDESC = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);

// byte offset of 16-byte chunk c (0..7) of row r in a swizzled K-major tile
__device__ __forceinline__ uint32_t sw_off(uint32_t r, uint32_t c) { return r * 128u + ((c ^ (r & 7u)) << 4); }

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (the tile base is 1024-byte aligned)
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;           // leading byte offset (16 B; unused with this swizzle)
    d |= static_cast<uint64_t>(1024u >> 4) << 32;   // stride byte offset between 8-row groups
    d |= static_cast<uint64_t>(1u) << 46;           // descriptor version for sm_100
    d |= static_cast<uint64_t>(2u) << 61;           // 128-byte swizzle
    return d;
}

__device__ __forceinline__ void mma_f16(uint32_t tmem_d, uint64_t a, uint64_t b, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(tmem_d),
        "l"(a), "l"(b), "r"(IDESC), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 32 consecutive TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// 8 consecutive values v[0..7] -> one 16-byte chunk in the operand element
// order (0,2,1,3,4,6,5,7)
__device__ __forceinline__ uint4 pack_chunk(const float (&v)[8]) {
    uint4 o;
    o.x = h2_bits(__floats2half2_rn(v[0], v[2]));
    o.y = h2_bits(__floats2half2_rn(v[1], v[3]));
    o.z = h2_bits(__floats2half2_rn(v[4], v[6]));
    o.w = h2_bits(__floats2half2_rn(v[5], v[7]));
    return o;
}
// the same reordering of a chunk of 8 fp16 values in natural order
__device__ __forceinline__ uint4 reorder_chunk(uint4 n) {
    uint4 o;
    o.x = __byte_perm(n.x, n.y, 0x5410);
    o.y = __byte_perm(n.x, n.y, 0x7632);
    o.z = __byte_perm(n.z, n.w, 0x5410);
    o.w = __byte_perm(n.z, n.w, 0x7632);
    return o;
}

// Q4_K: 16 values of one row -- elements k0+8cp .. +7 (low nibbles of qs
// bytes 8cp..8cp+7 of the 64-element group, sub-block 2g) and k0+32+8cp .. +7
// (high nibbles, sub-block 2g+1) -- as two chunks.  value = d*sc*q - dmin*m
// (matmul_q4.cu:76-96), evaluated in fp16 as q*(d*sc) - dmin*m.
__device__ __forceinline__ void dq_q4k(const uint8_t* row, int k0, int cp, uint4& lo, uint4& hi) {
    const uint8_t* blk = row + (k0 >> 8) * 144;
    const int g = (k0 >> 6) & 3;
    const uint4 hd = __ldg(reinterpret_cast<const uint4*>(blk));
    const uint2 q = __ldg(reinterpret_cast<const uint2*>(blk + 16 + 32 * g + 8 * cp));
    float sc0, m0, sc1, m1;
    kscale(hd.y, hd.z, hd.w, 2 * g, sc0, m0);
    kscale(hd.y, hd.z, hd.w, 2 * g + 1, sc1, m1);
    const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
    const __half2 a0 = __float2half2_rn(d * sc0), b0 = __float2half2_rn(dmin * m0);
    const __half2 a1 = __float2half2_rn(d * sc1), b1 = __float2half2_rn(dmin * m1);
    const __half2 k1024 = __float2half2_rn(1024.0f);
    // half2(1024 + n(byte e), 1024 + n(byte e+2)) from one word: nibble in the mantissa
    auto cvt = [&](uint32_t w, uint32_t mask, __half2 a, __half2 b) {
        const __half2 raw = bits_h2((w & mask) | 0x64006400u);
        return h2_bits(__hfma2(__hsub2(raw, k1024), a, __hneg2(b)));
    };
    // low nibbles: words (bytes 0..3) and (4..7) -> element order 0,2,1,3 / 4,6,5,7
    lo.x = cvt(q.x, 0x000F000Fu, a0, b0);
    lo.y = cvt(q.x >> 8, 0x000F000Fu, a0, b0);
    lo.z = cvt(q.y, 0x000F000Fu, a0, b0);
    lo.w = cvt(q.y >> 8, 0x000F000Fu, a0, b0);
    // high nibbles, shifted down to bits 0..3 first
    hi.x = cvt(q.x >> 4, 0x000F000Fu, a1, b1);
    hi.y = cvt(q.x >> 12, 0x000F000Fu, a1, b1);
    hi.z = cvt(q.y >> 4, 0x000F000Fu, a1, b1);
    hi.w = cvt(q.y >> 12, 0x000F000Fu, a1, b1);
}

// any other type: the reference's per-element formulas (dq1), same chunks
__device__ __forceinline__ void dq_generic(const uint8_t* row, int type, int k0, int cp, uint4& lo, uint4& hi) {
    float a[8], b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        a[e] = dq1(row, type, static_cast<uint64_t>(k0 + 8 * cp + e));
        b[e] = dq1(row, type, static_cast<uint64_t>(k0 + 32 + 8 * cp + e));
    }
    lo = pack_chunk(a);
    hi = pack_chunk(b);
}

struct GemmParams {
    // A operand
    const float* x;           // MODE 0: F32 rows, row length K
    const int32_t* a_rows;    // MODE 0: source row of each output row (null: the output row itself)
    const __half* a16;        // MODE 1: fp16 rows [rows][K]
    // B operand: groups of N rows x K, GGUF rows
    const uint8_t* w0;        // gate (MODE 0) or down (MODE 1)
    const uint8_t* w1;        // up (MODE 0)
    uint64_t w_group_bytes;
    uint32_t w_row_bytes;
    int wtype;
    int N, K;
    int groups;
    const int32_t* grp_start;   // [groups + 1] first output row of each group
    const int32_t* tile_start;  // [groups + 1] prefix of 128-row tiles per group
    __half* out;                // [rows][N]
    uint32_t* ctrl;             // error word
};

template <int WT, int MODE>
__global__ void __launch_bounds__(THREADS, 1) k_pgemm(GemmParams p) {
    constexpr int NB = MODE == 0 ? 2 : 1;
    constexpr uint32_t STAGE = A_BYTES + NB * B_BYTES;
    constexpr int NST = MODE == 0 ? 2 : 4;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * STAGE);
    uint64_t* empty = full + NST;
    uint64_t* accf = empty + NST;
    uint64_t* accfree = accf + 1;
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accfree + 1);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nN = p.N / BN, nK = p.K / BK;
    const int total = __ldg(p.tile_start + p.groups) * nN;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(full + s, PROD_WARPS);
            mbar_init(empty + s, 1);
        }
        mbar_init(accf, 1);
        mbar_init(accfree, 4);
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(NB * BN));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    // tile index -> (group, m tile, n tile)
    auto decode = [&](int t, int& g, int& mt, int& nt) {
        const int mi = t / nN;
        nt = t - mi * nN;
        int lo = 0, hi = p.groups;  // largest g with tile_start[g] <= mi
        while (hi - lo > 1) {
            const int mid = (lo + hi) >> 1;
            if (__ldg(p.tile_start + mid) <= mi) lo = mid; else hi = mid;
        }
        g = lo;
        mt = mi - __ldg(p.tile_start + g);
    };

    if (warp < PROD_WARPS) {
        // ---------------- producers ----------------
        int stage = 0, use = 0;  // use = how many times the ring wrapped
        for (int t = blockIdx.x; t < total; t += gridDim.x) {
            int g, mt, nt;
            decode(t, g, mt, nt);
            const int r0 = __ldg(p.grp_start + g) + mt * BM;
            const int r1 = min(r0 + BM, __ldg(p.grp_start + g + 1));
            const uint8_t* wg0 = p.w0 + g * p.w_group_bytes + static_cast<uint64_t>(nt) * BN * p.w_row_bytes;
            const uint8_t* wg1 = MODE == 0 ? p.w1 + g * p.w_group_bytes + static_cast<uint64_t>(nt) * BN * p.w_row_bytes
                                           : nullptr;
            for (int kb = 0; kb < nK; ++kb) {
                if (use > 0) mbar_wait(empty + stage, (use - 1) & 1, p.ctrl);
                uint8_t* sa = smem + stage * STAGE;
                const int k0 = kb * BK;
                // A: 128 rows x 8 chunks
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    const int q = tid + j * (PROD_WARPS * 32);
                    const int r = q >> 3, c = q & 7;
                    const int row = r0 + r;
                    uint4 v = make_uint4(0u, 0u, 0u, 0u);
                    if (row < r1) {
                        if (MODE == 0) {
                            const int src = p.a_rows ? __ldg(p.a_rows + row) : row;
                            const float4* xp = reinterpret_cast<const float4*>(p.x + static_cast<size_t>(src) * p.K + k0 + 8 * c);
                            const float4 u0 = __ldg(xp), u1 = __ldg(xp + 1);
                            const float f[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                            v = pack_chunk(f);
                        } else {
                            v = reorder_chunk(__ldg(reinterpret_cast<const uint4*>(p.a16 + static_cast<size_t>(row) * p.K + k0 + 8 * c)));
                        }
                    }
                    *reinterpret_cast<uint4*>(sa + sw_off(r, c)) = v;
                }
                // B: NB matrices x 256 rows x 4 chunk pairs
#pragma unroll
                for (int m = 0; m < NB; ++m) {
                    const uint8_t* wb = m == 0 ? wg0 : wg1;
                    uint8_t* sb = sa + A_BYTES + m * B_BYTES;
#pragma unroll 2
                    for (int j = 0; j < 4; ++j) {
                        const int q = tid + j * (PROD_WARPS * 32);
                        const int n = q >> 2, cp = q & 3;
                        const uint8_t* row = wb + static_cast<uint64_t>(n) * p.w_row_bytes;
                        uint4 lo, hi;
                        if (WT == T_Q4_K) dq_q4k(row, k0, cp, lo, hi);
                        else dq_generic(row, WT, k0, cp, lo, hi);
                        *reinterpret_cast<uint4*>(sb + sw_off(n, cp)) = lo;
                        *reinterpret_cast<uint4*>(sb + sw_off(n, cp + 4)) = hi;
                    }
                }
                fence_async_smem();  // generic-proxy stores -> visible to the tensor core
                __syncwarp();
                if (lane == 0) mbar_arrive(full + stage);
                if (++stage == NST) { stage = 0; ++use; }
            }
        }
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue ----------------
        int stage = 0, use = 0, ti = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
            if (ti > 0) mbar_wait(accfree, (ti - 1) & 1, p.ctrl);
            tc_fence_after();
            for (int kb = 0; kb < nK; ++kb) {
                mbar_wait(full + stage, use & 1, p.ctrl);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = smem_u32(smem + stage * STAGE);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const uint64_t ad = sdesc(sa + kk * 32);
                        const uint32_t acc = (kb | kk) != 0;
                        mma_f16(tmem, ad, sdesc(sa + A_BYTES + kk * 32), acc);
                        if (MODE == 0) mma_f16(tmem + BN, ad, sdesc(sa + A_BYTES + B_BYTES + kk * 32), acc);
                    }
                    mma_commit(empty + stage);  // the stage is free once these MMAs have read it
                }
                __syncwarp();
                if (++stage == NST) { stage = 0; ++use; }
            }
            if (lane == 0) mma_commit(accf);  // accumulators complete
            __syncwarp();
        }
    } else {
        // ---------------- epilogue: TMEM -> global ----------------
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = tile rows
        int ti = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
            int g, mt, nt;
            decode(t, g, mt, nt);
            const int r0 = __ldg(p.grp_start + g) + mt * BM;
            const int r1 = min(r0 + BM, __ldg(p.grp_start + g + 1));
            mbar_wait(accf, ti & 1, p.ctrl);
            tc_fence_after();
            const int row = r0 + 32 * quarter + lane;
            const uint32_t tl = tmem + (static_cast<uint32_t>(32 * quarter) << 16);
            __half* orow = p.out + static_cast<size_t>(row) * p.N + nt * BN;
            for (int c0 = 0; c0 < BN; c0 += 32) {
                uint32_t a[32];
                tmem_ld32(tl + c0, a);
                uint32_t o[16];
                if (MODE == 0) {
                    uint32_t u[32];
                    tmem_ld32(tl + BN + c0, u);
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float g0 = __uint_as_float(a[2 * i]), g1 = __uint_as_float(a[2 * i + 1]);
                        const float h0 = g0 / (1.0f + expf(-g0)) * __uint_as_float(u[2 * i]);  // moe.cu:64
                        const float h1 = g1 / (1.0f + expf(-g1)) * __uint_as_float(u[2 * i + 1]);
                        o[i] = h2_bits(__floats2half2_rn(h0, h1));
                    }
                } else {
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 16; ++i)
                        o[i] = h2_bits(__floats2half2_rn(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1])));
                }
                if (row < r1) {
                    uint4* dst = reinterpret_cast<uint4*>(orow + c0);
#pragma unroll
                    for (int i = 0; i < 4; ++i) dst[i] = make_uint4(o[4 * i], o[4 * i + 1], o[4 * i + 2], o[4 * i + 3]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accfree);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(NB * BN));
    }
}

template <int MODE>
size_t gemm_smem_bytes() {
    constexpr int NB = MODE == 0 ? 2 : 1;
    constexpr int NST = MODE == 0 ? 2 : 4;
    return 1024 + static_cast<size_t>(NST) * (A_BYTES + NB * B_BYTES) + 256;
}

}  // namespace pf

// ---------------------------------------------------------------------------
// RMSNorm of every token (ops.cu:25-65 structure): one warp per token, the sum
// of squares with the reference GEMV's thread/shuffle structure (as in the
// decode router), then (x * scale) * weight.  Without a norm weight it copies.
// ---------------------------------------------------------------------------
__device__ __forceinline__ float pf_tree8(float (&acc)[2][4]);

template <int CH>
__global__ void __launch_bounds__(256) k_norm_many(const float* __restrict__ x, const float* __restrict__ w,
                                                   float eps, float* __restrict__ out, int T, int d) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    const float* xr = x + static_cast<size_t>(t) * d;
    float4 v[CH][2];
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) v[i][hh] = __ldg(reinterpret_cast<const float4*>(xr + 256 * i + 128 * hh + 4 * lane));
    float* orow = out + static_cast<size_t>(t) * d;
    if (w) {
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                acc[hh][0] = __fmaf_rn(v[i][hh].x, v[i][hh].x, acc[hh][0]);
                acc[hh][1] = __fmaf_rn(v[i][hh].y, v[i][hh].y, acc[hh][1]);
                acc[hh][2] = __fmaf_rn(v[i][hh].z, v[i][hh].z, acc[hh][2]);
                acc[hh][3] = __fmaf_rn(v[i][hh].w, v[i][hh].w, acc[hh][3]);
            }
        const float ss = pf_tree8(acc);
        const float sc = rsqrtf(ss / static_cast<float>(d) + eps);
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const float4 nv = __ldg(reinterpret_cast<const float4*>(w + 256 * i + 128 * hh + 4 * lane));
                v[i][hh].x = __fmul_rn(__fmul_rn(v[i][hh].x, sc), nv.x);
                v[i][hh].y = __fmul_rn(__fmul_rn(v[i][hh].y, sc), nv.y);
                v[i][hh].z = __fmul_rn(__fmul_rn(v[i][hh].z, sc), nv.z);
                v[i][hh].w = __fmul_rn(__fmul_rn(v[i][hh].w, sc), nv.w);
            }
    }
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) *reinterpret_cast<float4*>(orow + 256 * i + 128 * hh + 4 * lane) = v[i][hh];
}

// The reference GEMV's reduction of the 8 per-lane chains (lane L plays
// threads 4L+c+128h): shuffle-down tree 4,2,1 inside groups of 8 lanes, the
// two halves, then the 8 warp partials ((q0+q4)+(q2+q6))+((q1+q5)+(q3+q7)).
__device__ __forceinline__ float pf_tree8(float (&acc)[2][4]) {
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float a = acc[hh][c];
            a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 4));
            a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 2));
            a = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 1));
            acc[hh][c] = a;
        }
    const float s0 = __fadd_rn(__fadd_rn(acc[0][0], acc[0][2]), __fadd_rn(acc[0][1], acc[0][3]));
    const float s1 = __fadd_rn(__fadd_rn(acc[1][0], acc[1][2]), __fadd_rn(acc[1][1], acc[1][3]));
    float q[8];
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
        q[w4] = __shfl_sync(0xffffffffu, s0, 8 * w4);
        q[4 + w4] = __shfl_sync(0xffffffffu, s1, 8 * w4);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __fadd_rn(__fadd_rn(q[i], 0.0f), 0.0f);
    return __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                     __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
}

// ---------------------------------------------------------------------------
// Router logits of many tokens, reference GEMV order.  Each warp holds two
// router rows in registers (rows 2*gw and 2*gw+1 of the E+1 rows: the E
// expert rows, then the shared-expert gate vector) and walks a chunk of
// tokens; each x_in value it loads serves both rows.
// ---------------------------------------------------------------------------
template <int CH>
__device__ __forceinline__ void pf_load_row(float4 (&w)[CH][2], const uint8_t* row, int type, int lane) {
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int e = 256 * i + 128 * hh + 4 * lane;
            if (type == T_F32) {
                w[i][hh] = __ldg(reinterpret_cast<const float4*>(row) + e / 4);
            } else {
                const uint2 u = __ldg(reinterpret_cast<const uint2*>(row + 2 * e));
                if (type == T_F16) {
                    const float2 a = __half22float2(bits_to_half2(u.x)), b = __half22float2(bits_to_half2(u.y));
                    w[i][hh] = make_float4(a.x, a.y, b.x, b.y);
                } else {
                    w[i][hh] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u),
                                           __uint_as_float(u.y << 16), __uint_as_float(u.y & 0xFFFF0000u));
                }
            }
        }
}

template <int CH>
__global__ void __launch_bounds__(256) k_route_many(const uint8_t* __restrict__ router, int router_type,
                                                    const uint8_t* __restrict__ sgate, int sgate_type,
                                                    const float* __restrict__ bias, const float* __restrict__ xin,
                                                    float* __restrict__ logits, int T, int d, int E, int has_shared,
                                                    int tchunk) {
    const int lane = threadIdx.x & 31;
    const int gw = blockIdx.x * 8 + (threadIdx.x >> 5);
    const int nrows = E + (has_shared ? 1 : 0);
    const int ra = 2 * gw, rb = 2 * gw + 1;
    if (ra >= nrows) return;
    const bool has_b = rb < nrows;
    float4 wa[CH][2], wb[CH][2];
    auto row_ptr = [&](int r, int& type) {
        type = r < E ? router_type : sgate_type;
        return r < E ? router + static_cast<size_t>(r) * d * (type == T_F32 ? 4 : 2) : sgate;
    };
    int ta, tb = 0;
    pf_load_row<CH>(wa, row_ptr(ra, ta), ta, lane);
    if (has_b) {
        pf_load_row<CH>(wb, row_ptr(rb, tb), tb, lane);
    } else {
#pragma unroll
        for (int i = 0; i < CH; ++i) wb[i][0] = wb[i][1] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    const float bias_a = (ra < E && bias) ? __ldg(bias + ra) : 0.0f;
    const float bias_b = (has_b && rb < E && bias) ? __ldg(bias + rb) : 0.0f;
    const int LS = E + 1;
    const int t0 = blockIdx.y * tchunk, t1 = min(T, t0 + tchunk);
    for (int t = t0; t < t1; ++t) {
        const float* xr = xin + static_cast<size_t>(t) * d;
        float aa[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
        float ab[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const float4 xv = __ldg(reinterpret_cast<const float4*>(xr + 256 * i + 128 * hh + 4 * lane));
                aa[hh][0] = __fmaf_rn(wa[i][hh].x, xv.x, aa[hh][0]);
                aa[hh][1] = __fmaf_rn(wa[i][hh].y, xv.y, aa[hh][1]);
                aa[hh][2] = __fmaf_rn(wa[i][hh].z, xv.z, aa[hh][2]);
                aa[hh][3] = __fmaf_rn(wa[i][hh].w, xv.w, aa[hh][3]);
                ab[hh][0] = __fmaf_rn(wb[i][hh].x, xv.x, ab[hh][0]);
                ab[hh][1] = __fmaf_rn(wb[i][hh].y, xv.y, ab[hh][1]);
                ab[hh][2] = __fmaf_rn(wb[i][hh].z, xv.z, ab[hh][2]);
                ab[hh][3] = __fmaf_rn(wb[i][hh].w, xv.w, ab[hh][3]);
            }
        float va = pf_tree8(aa);
        float vb = pf_tree8(ab);
        if (lane == 0) {
            if (ra < E && bias) va = __fadd_rn(va, bias_a);
            logits[static_cast<size_t>(t) * LS + ra] = va;
            if (has_b) {
                if (rb < E && bias) vb = __fadd_rn(vb, bias_b);
                logits[static_cast<size_t>(t) * LS + rb] = vb;
            }
        }
    }
}

// ---------------------------------------------------------------------------
// One warp per token: top-k, softmax, checks; the failing tokens get id -1
// and NaN weights, and the error word records the first of them.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_topk_many(const float* __restrict__ logits, int T, int E, int k,
                                                   int32_t* __restrict__ idx, float* __restrict__ wts,
                                                   int32_t* __restrict__ out_idx, float* __restrict__ out_w,
                                                   uint32_t* ctrl) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t >= T) return;
    int my_idx;
    float wj;
    uint32_t flag;
    select_token(logits + static_cast<size_t>(t) * (E + 1), E, k, lane, my_idx, wj, flag);
    if (flag && lane == 0) {
        atomicOr(ctrl + CTRL_ERROR, flag);
        atomicMin(ctrl + CTRL_ERR_TOKEN, static_cast<uint32_t>(t));
    }
    if (lane < k) {
        const int oi = flag ? -1 : my_idx;
        const float ow = flag ? __uint_as_float(0x7FC00000u) : wj;
        idx[t * k + lane] = oi;
        wts[t * k + lane] = ow;
        if (out_idx) out_idx[t * k + lane] = oi;
        if (out_w) out_w[t * k + lane] = ow;
    }
}

// ---------------------------------------------------------------------------
// Source token of every permuted pair and the 128-row tile prefix per expert
// (routed experts) plus the shared expert's single group [0, T).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_plan(const int32_t* __restrict__ offsets, const int32_t* __restrict__ perm,
                                                 int E, int k, int T, int32_t* __restrict__ tok_of_pos,
                                                 int32_t* __restrict__ tile_start, int32_t* __restrict__ sh_grp,
                                                 int32_t* __restrict__ sh_tiles) {
    const int npairs = __ldg(offsets + E);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npairs; i += gridDim.x * blockDim.x)
        tok_of_pos[i] = __ldg(perm + i) / k;
    if (blockIdx.x == 0 && threadIdx.x < 32) {
        // warp 0: exclusive scan of ceil(count / 128) over the experts
        const int lane = threadIdx.x;
        int run = 0;
        for (int e0 = 0; e0 < E; e0 += 32) {
            const int e = e0 + lane;
            const int cnt = e < E ? __ldg(offsets + e + 1) - __ldg(offsets + e) : 0;
            const int v = (cnt + pf::BM - 1) / pf::BM;
            int inc = v;
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const int y = __shfl_up_sync(0xffffffffu, inc, o);
                if (lane >= o) inc += y;
            }
            if (e < E) tile_start[e] = run + inc - v;
            run += __shfl_sync(0xffffffffu, inc, 31);
        }
        if (lane == 0) {
            tile_start[E] = run;
            sh_grp[0] = 0;
            sh_grp[1] = T;
            sh_tiles[0] = 0;
            sh_tiles[1] = (T + pf::BM - 1) / pf::BM;
        }
    }
}

// ---------------------------------------------------------------------------
// Combine (moe.cu:76-81, 90-96; order of layer_moe.cpp:127-154): one CTA of
// 256 threads per token, 8 columns per thread.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_combine(const __half* __restrict__ Y, const __half* __restrict__ Ys,
                                                    const int32_t* __restrict__ inv_perm, const float* __restrict__ wts,
                                                    const float* __restrict__ logits, const float* __restrict__ residual,
                                                    float* __restrict__ out, int d, int E, int k, int has_shared) {
    const int t = blockIdx.x;
    __shared__ int s_pos[kMaxTopK];
    __shared__ float s_w[kMaxTopK];
    __shared__ float s_sg;
    if (threadIdx.x < k) {
        s_pos[threadIdx.x] = __ldg(inv_perm + t * k + threadIdx.x);
        s_w[threadIdx.x] = __ldg(wts + t * k + threadIdx.x);
    }
    if (threadIdx.x == 0) s_sg = has_shared ? 1.0f / (1.0f + expf(-__ldg(logits + static_cast<size_t>(t) * (E + 1) + E))) : 0.0f;
    __syncthreads();
    const bool bad = !(s_w[0] == s_w[0]);
    for (int c0 = threadIdx.x * 8; c0 < d; c0 += blockDim.x * 8) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int j = 0; j < k; ++j) {
            const int pos = s_pos[j];
            if (pos < 0) continue;
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(Y + static_cast<size_t>(pos) * d + c0));
            const float2 a = __half22float2(bits_to_half2(u.x)), b = __half22float2(bits_to_half2(u.y));
            const float2 c = __half22float2(bits_to_half2(u.z)), e = __half22float2(bits_to_half2(u.w));
            const float y[8] = {a.x, a.y, b.x, b.y, c.x, c.y, e.x, e.y};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(s_w[j], y[i], acc[i]);
        }
        if (has_shared) {
            const uint4 u = __ldg(reinterpret_cast<const uint4*>(Ys + static_cast<size_t>(t) * d + c0));
            const float2 a = __half22float2(bits_to_half2(u.x)), b = __half22float2(bits_to_half2(u.y));
            const float2 c = __half22float2(bits_to_half2(u.z)), e = __half22float2(bits_to_half2(u.w));
            const float y[8] = {a.x, a.y, b.x, b.y, c.x, c.y, e.x, e.y};
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[i] = fmaf(y[i], s_sg, acc[i]);
        }
        float* o = out + static_cast<size_t>(t) * d + c0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float v = bad ? __uint_as_float(0x7FC00000u) : acc[i];
            if (residual) v = __ldg(residual + static_cast<size_t>(t) * d + c0 + i) + v;
            o[i] = v;
        }
    }
}

}  // namespace qmoe

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace qmoe {

cudaError_t launch_dispatch(const int32_t* idx, int NP, int E, int32_t* offsets, int32_t* perm, int32_t* inv_perm,
                            int32_t* table, cudaStream_t s);

namespace {

template <typename K>
cudaError_t pf_set_smem(K kern, size_t smem) {
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
}

template <int MODE>
using GemmKern = void (*)(pf::GemmParams);

template <int MODE>
GemmKern<MODE> pick_gemm(int type) {
    switch (type) {
        case T_Q4_K: return pf::k_pgemm<T_Q4_K, MODE>;
        case T_Q5_K: return pf::k_pgemm<T_Q5_K, MODE>;
        case T_Q6_K: return pf::k_pgemm<T_Q6_K, MODE>;
        case T_Q8_0: return pf::k_pgemm<T_Q8_0, MODE>;
        default: return nullptr;
    }
}

int pf_num_sms() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

template <int MODE>
cudaError_t launch_pgemm(const pf::GemmParams& p, cudaStream_t s) {
    GemmKern<MODE> kern = pick_gemm<MODE>(p.wtype);
    if (!kern) return cudaErrorInvalidValue;
    const size_t smem = pf::gemm_smem_bytes<MODE>();
    cudaError_t e = pf_set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    kern<<<pf_num_sms(), pf::THREADS, smem, s>>>(p);
    return cudaGetLastError();
}

}  // namespace

bool prefill_supported(const DecodeParams& P) {
    auto ok_type = [](int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_Q8_0; };
    if (!ok_type(P.gate.type) || P.up.type != P.gate.type || !ok_type(P.down.type)) return false;
    if (P.has_shared && (!ok_type(P.sgate.type) || P.sup.type != P.sgate.type || !ok_type(P.sdown.type))) return false;
    if (P.d % pf::BN || P.F % pf::BN || P.Fs % pf::BN || P.d % pf::BK || P.F % pf::BK || P.Fs % pf::BK) return false;
    if (P.d > kMaxNormDim || P.d % 256) return false;
    return pf_num_sms() > 0;
}

// The whole block for T tokens through the prefill kernels.  `xin` is the
// block input after the optional norm, `pf` the prefill workspace regions.
cudaError_t launch_prefill(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) {
    const int T = P.T, d = P.d, E = P.E, k = P.k;
    const int CH = d / 256;
    cudaError_t e = cudaSuccess;
    // 1. x_in
    {
        const dim3 grid((T + 7) / 8);
        switch (CH) {
            case 1: k_norm_many<1><<<grid, 256, 0, s>>>(P.x, P.prenorm ? P.norm_w : nullptr, P.eps, P.xnorm, T, d); break;
            case 2: k_norm_many<2><<<grid, 256, 0, s>>>(P.x, P.prenorm ? P.norm_w : nullptr, P.eps, P.xnorm, T, d); break;
            case 4: k_norm_many<4><<<grid, 256, 0, s>>>(P.x, P.prenorm ? P.norm_w : nullptr, P.eps, P.xnorm, T, d); break;
            case 8: k_norm_many<8><<<grid, 256, 0, s>>>(P.x, P.prenorm ? P.norm_w : nullptr, P.eps, P.xnorm, T, d); break;
            default: return cudaErrorInvalidValue;
        }
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // 2. router logits
    {
        const int nrows = E + (P.has_shared ? 1 : 0);
        const int tchunk = 64;
        const dim3 grid((((nrows + 1) / 2) + 7) / 8, (T + tchunk - 1) / tchunk);
#define QMOE_RM(C)                                                                                               \
    k_route_many<C><<<grid, 256, 0, s>>>(P.router, P.router_type, P.sgate_inp, P.sgate_type, P.bias, P.xnorm, \
                                         P.logits, T, d, E, P.has_shared, tchunk)
        switch (CH) {
            case 1: QMOE_RM(1); break;
            case 2: QMOE_RM(2); break;
            case 4: QMOE_RM(4); break;
            case 8: QMOE_RM(8); break;
            default: return cudaErrorInvalidValue;
        }
#undef QMOE_RM
        if ((e = cudaGetLastError()) != cudaSuccess) return e;
    }
    // 3. top-k per token
    k_topk_many<<<(T + 7) / 8, 256, 0, s>>>(P.logits, T, E, k, P.topk_idx, P.topk_w, P.out_idx, P.out_w, P.ctrl);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // 4. permutation
    if ((e = launch_dispatch(P.topk_idx, T * k, E, P.offsets, P.perm, P.inv_perm, B.disp, s)) != cudaSuccess) return e;
    // 5. plan
    k_pf_plan<<<64, 256, 0, s>>>(P.offsets, P.perm, E, k, T, B.tok_of_pos, B.tile_start, B.sh_grp, B.sh_tiles);
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    // 6. gate/up: routed, then shared
    pf::GemmParams g{};
    g.x = P.xnorm;
    g.a_rows = B.tok_of_pos;
    g.w0 = P.gate.p;
    g.w1 = P.up.p;
    g.w_row_bytes = static_cast<uint32_t>(row_bytes(P.gate.type, d));
    g.w_group_bytes = static_cast<uint64_t>(P.F) * g.w_row_bytes;
    g.wtype = P.gate.type;
    g.N = P.F;
    g.K = d;
    g.groups = E;
    g.grp_start = P.offsets;
    g.tile_start = B.tile_start;
    g.out = B.H;
    g.ctrl = P.ctrl;
    if ((e = launch_pgemm<0>(g, s)) != cudaSuccess) return e;
    if (P.has_shared) {
        pf::GemmParams gs = g;
        gs.a_rows = nullptr;
        gs.w0 = P.sgate.p;
        gs.w1 = P.sup.p;
        gs.w_row_bytes = static_cast<uint32_t>(row_bytes(P.sgate.type, d));
        gs.w_group_bytes = static_cast<uint64_t>(P.Fs) * gs.w_row_bytes;
        gs.wtype = P.sgate.type;
        gs.N = P.Fs;
        gs.groups = 1;
        gs.grp_start = B.sh_grp;
        gs.tile_start = B.sh_tiles;
        gs.out = B.Hs;
        if ((e = launch_pgemm<0>(gs, s)) != cudaSuccess) return e;
    }
    // 7. down: routed, then shared
    pf::GemmParams dn{};
    dn.a16 = B.H;
    dn.w0 = P.down.p;
    dn.w_row_bytes = static_cast<uint32_t>(row_bytes(P.down.type, P.F));
    dn.w_group_bytes = static_cast<uint64_t>(d) * dn.w_row_bytes;
    dn.wtype = P.down.type;
    dn.N = d;
    dn.K = P.F;
    dn.groups = E;
    dn.grp_start = P.offsets;
    dn.tile_start = B.tile_start;
    dn.out = B.Y;
    dn.ctrl = P.ctrl;
    if ((e = launch_pgemm<1>(dn, s)) != cudaSuccess) return e;
    if (P.has_shared) {
        pf::GemmParams ds = dn;
        ds.a16 = B.Hs;
        ds.w0 = P.sdown.p;
        ds.w_row_bytes = static_cast<uint32_t>(row_bytes(P.sdown.type, P.Fs));
        ds.w_group_bytes = static_cast<uint64_t>(d) * ds.w_row_bytes;
        ds.wtype = P.sdown.type;
        ds.K = P.Fs;
        ds.groups = 1;
        ds.grp_start = B.sh_grp;
        ds.tile_start = B.sh_tiles;
        ds.out = B.Ys;
        if ((e = launch_pgemm<1>(ds, s)) != cudaSuccess) return e;
    }
    // 8. combine
    k_pf_combine<<<T, 256, 0, s>>>(B.Y, B.Ys, P.inv_perm, P.topk_w, P.logits, P.residual, P.out, d, E, k,
                                   P.has_shared);
    return cudaGetLastError();
}

}  // namespace qmoe
