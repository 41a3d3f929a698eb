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
//   k_pf_count/scan/place  stable (expert, token, slot) permutation
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

#include <algorithm>

#include "qmoe_dev.cuh"
#include "qmoe_dq1.cuh"
#include "qmoe_internal.h"
#include "qmoe_route.cuh"
#include "qmoe_tgemm.h"

namespace qmoe {

__device__ __forceinline__ __half2 bits_to_half2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

namespace pf {

constexpr int BM = 128;                // tile rows (tokens or pairs) = MMA M
constexpr int BN = 256;                // tile columns = MMA N (gate/up: 128 of each)
constexpr int BK = 32;                 // K per pipeline stage (64 bytes of fp16 per row)
constexpr int NST = 5;                 // pipeline stages
constexpr int LA = 3;                  // stages whose copies are in flight ahead of the dequantisation
constexpr int PROD_WARPS = 16;         // copies + weight dequantisation (half a B row per thread)
constexpr int PROD_THREADS = PROD_WARPS * 32;
constexpr int EPI_WARP0 = 16;          // warps 16..19: TMEM epilogue (lane quarter = warp % 4)
constexpr int MMA_WARP = 20;           // one thread issues the MMAs
constexpr int THREADS = 21 * 32;
static_assert(EPI_WARP0 == PROD_WARPS && MMA_WARP == EPI_WARP0 + 4 && THREADS == (MMA_WARP + 1) * 32, "warp roles");
constexpr uint32_t A_BYTES = BM * 64;    // 8 KB: fp16 activations of one stage
constexpr uint32_t B_BYTES = BN * 64;    // 16 KB: fp16 weights of one stage
constexpr uint32_t RAW_SLOT = 32;        // Q4_K bytes per producer thread and stage: block header + 16 qs bytes
constexpr uint32_t RAW_BYTES = PROD_THREADS * RAW_SLOT;  // 16 KB
constexpr uint32_t STAGE = A_BYTES + B_BYTES + RAW_BYTES;  // 40 KB (every part 1024-byte aligned)
constexpr uint32_t TMEM_COLS = 2 * BN;   // two accumulator buffers
// instruction descriptor: D F32, A/B fp16, both K-major, N = 256, M = 128
constexpr uint32_t IDESC = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);

// byte offset of 16-byte chunk c (0..3) of row r in a K-major tile with the
// 64-byte swizzle (rows of 64 bytes, 8-row groups of 512 bytes; chunk c of
// row r sits at chunk c ^ ((r / 2) % 4))
__device__ __forceinline__ uint32_t sw_off(uint32_t r, uint32_t c) { return r * 64u + ((c ^ ((r >> 1) & 3u)) << 4); }

// shared-memory matrix descriptor: K-major, 64-byte swizzle, 8-row groups
// 512 bytes apart (the tile base is 1024-byte aligned)
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;          // leading byte offset (16 B; unused with this swizzle)
    d |= static_cast<uint64_t>(512u >> 4) << 32;   // stride byte offset between 8-row groups
    d |= static_cast<uint64_t>(1u) << 46;          // descriptor version for sm_100
    d |= static_cast<uint64_t>(4u) << 61;          // 64-byte swizzle
    return d;
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

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
// 16 consecutive TMEM columns of this warp's 32 lanes
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
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
// Two chunks (16 values) of one sub-block of a Q4_K row from a producer
// thread's staged raw bytes: the block header (d, dmin, 12 scale bytes) and
// 16 qs bytes of the 64-element group; sub-block j uses the low (j even) or
// high nibbles.  value = d*sc*q - dmin*m (matmul_q4.cu:76-96), rounded to
// fp16 once as ((q - 8) * sc) * d + (8*d*sc - dmin*m): the first product is an
// exact fp16 integer, d the block's own fp16 scale, one fused half2
// multiply-add rounds the sum (the same evaluation as the TMA GEMM's).
__device__ __forceinline__ void dq_q4k_raw(uint32_t raw, int j, uint4 (&out)[2]) {
    const uint4 hd = lds128(raw);
    const uint4 q = lds128(raw + 16);
    float sc, m;
    kscale(hd.y, hd.z, hd.w, j, sc, m);
    const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
    const __half2 d2 = bits_h2((hd.x & 0xFFFFu) * 0x00010001u);
    const __half2 sc2 = __float2half2_rn(sc);
    const __half2 c2 = __float2half2_rn(fmaf(8.0f * d, sc, -(dmin * m)));
    const __half2 k1032 = __float2half2_rn(1032.0f);
    const int sh = (j & 1) * 4;
    // half2(1024 + n(byte e), 1024 + n(byte e+2)) from one word: element order 0,2 / 1,3
    auto cvt = [&](uint32_t w) {
        const __half2 raw2 = bits_h2(((w >> sh) & 0x000F000Fu) | 0x64006400u);
        return h2_bits(__hfma2(__hmul2(__hsub2(raw2, k1032), sc2), d2, c2));
    };
    out[0] = make_uint4(cvt(q.x), cvt(q.x >> 8), cvt(q.y), cvt(q.y >> 8));
    out[1] = make_uint4(cvt(q.z), cvt(q.z >> 8), cvt(q.w), cvt(q.w >> 8));
}

// any other type: 16 values (chunks c0, c0+1) of one row with the
// reference's per-element formulas (dq1), read from global memory
__device__ __forceinline__ void dq_generic(const uint8_t* row, int type, int k0, int c0, uint4 (&out)[2]) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = dq1(row, type, static_cast<uint64_t>(k0 + 8 * (c0 + c) + e));
        out[c] = pack_chunk(v);
    }
}

struct GemmParams {
    const __half* a16;        // fp16 A rows [*, K] in the chunk element order
    const int32_t* a_rows;    // source A row of each output row (null: the output row itself)
    // B operand: groups of weight rows, GGUF rows of K elements
    const uint8_t* w0;        // gate (MODE 0) or down (MODE 1)
    const uint8_t* w1;        // up (MODE 0)
    uint64_t w_group_bytes;
    uint32_t w_row_bytes;
    int wtype;
    int N, K;                 // output columns (F or d), reduction length
    int groups;
    const int32_t* grp_start;   // [groups + 1] first output row of each group
    const int32_t* tile_start;  // [groups + 1] prefix of 128-row tiles per group
    __half* out;                // [rows][N]; MODE 0 in the chunk element order
    const int32_t* out_rows;    // MODE 1: output row of each tile row (null: the tile row itself)
    int out_cap;                // rows of `out` (rows mapped past it are not written)
    uint32_t* ctrl;             // error word
};

// Tile iterator: tile t -> (group, m tile, n tile, row range)
struct PfTile {
    int g, mt, nt, r0, r1;
};
__device__ __forceinline__ PfTile pf_tile(const GemmParams& p, int t, int nN) {
    PfTile T;
    const int mi = t / nN;
    T.nt = t - mi * nN;
    int lo = 0, hi = p.groups;  // largest g with tile_start[g] <= mi
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (__ldg(p.tile_start + mid) <= mi) lo = mid; else hi = mid;
    }
    T.g = lo;
    T.mt = mi - __ldg(p.tile_start + lo);
    T.r0 = __ldg(p.grp_start + lo) + T.mt * BM;
    T.r1 = min(T.r0 + BM, __ldg(p.grp_start + lo + 1));
    return T;
}

// MODE 0 (gate/up): D[:, 0..127] = gate rows nt*128.., D[:, 128..255] = up rows;
// out = silu(gate) * up, 128 columns per tile.  MODE 1 (down): 256 columns.
template <int WT, int MODE>
__global__ void __launch_bounds__(THREADS, 1) k_pgemm(GemmParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + NST * STAGE);
    uint64_t* empty = full + NST;
    uint64_t* accf = empty + NST;     // [2]
    uint64_t* accfree = accf + 2;     // [2]
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(accfree + 2);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ncol = MODE == 0 ? BN / 2 : BN;  // output columns per tile
    const int nN = p.N / ncol, nK = p.K / BK;
    const int total = __ldg(p.tile_start + p.groups) * nN;

    if (tid == 0) {
        for (int s = 0; s < NST; ++s) {
            mbar_init(full + s, PROD_WARPS);
            mbar_init(empty + s, 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(accf + b, 1);
            mbar_init(accfree + b, 4);
        }
        fence_mbar_init();
    }
    if (warp == MMA_WARP) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp < PROD_WARPS) {
        // ---------------- producers ----------------
        // issue pointer (copies LA steps ahead) and consume pointer (dequantisation)
        int it = blockIdx.x, ikb = 0, istep = 0;
        int ct = blockIdx.x, ckb = 0, cstep = 0;
        PfTile iT = it < total ? pf_tile(p, it, nN) : PfTile{};
        PfTile cT = iT;
        const int row = tid >> 1, half = tid & 1;  // chunks 2*half, 2*half+1 of B row `row`; A chunk tid
        // source row of this thread's A chunk, looked up once per tile
        int a_src = -1;
        auto a_rows_of = [&](const PfTile& T) {
            const int orow = T.r0 + (tid >> 2);
            a_src = orow < T.r1 ? (p.a_rows ? __ldg(p.a_rows + orow) : orow) : -1;
        };
        if (it < total) a_rows_of(iT);
        auto wrow = [&](const PfTile& T) -> const uint8_t* {
            const uint8_t* base = (MODE == 0 && row >= BN / 2) ? p.w1 : p.w0;
            const int n = MODE == 0 ? T.nt * (BN / 2) + (row & (BN / 2 - 1)) : T.nt * BN + row;
            return base + T.g * p.w_group_bytes + static_cast<uint64_t>(n) * p.w_row_bytes;
        };
        auto issue = [&]() {
            const int stage = istep % NST;
            if (istep >= NST) mbar_wait(empty + stage, (istep / NST - 1) & 1, p.ctrl);
            const uint32_t sa = smem_u32(smem + stage * STAGE);
            const int k0 = ikb * BK;
            {  // A: 128 rows x 4 chunks (rows past the group are zero-filled)
                const int r = tid >> 2, c = tid & 3;
                const bool ok = a_src >= 0;
                cp_async16(sa + sw_off(r, c), p.a16 + static_cast<size_t>(ok ? a_src : 0) * p.K + k0 + 8 * c,
                           ok ? 16u : 0u);
            }
            if (WT == T_Q4_K) {  // raw bytes: block header + this half's 16 qs bytes of the group
                const uint8_t* blk = wrow(iT) + (k0 >> 8) * 144;
                const uint32_t rd = sa + A_BYTES + B_BYTES + tid * RAW_SLOT;
                cp_async16(rd, blk, 16u);
                cp_async16(rd + 16, blk + 16 + 32 * ((k0 >> 6) & 3) + 16 * half, 16u);
            }
            cp_async_commit();
            ++istep;
            if (++ikb == nK) {
                ikb = 0;
                it += gridDim.x;
                if (it < total) {
                    iT = pf_tile(p, it, nN);
                    a_rows_of(iT);
                }
            }
        };
        const int nsteps = ((total - blockIdx.x + gridDim.x - 1) / gridDim.x) * nK;
        for (int i = 0; i < LA && i < nsteps; ++i) issue();
        for (; cstep < nsteps; ++cstep) {
            if (cstep + LA < nsteps) issue(); else cp_async_commit();  // keep one group per step
            cp_async_wait<LA>();  // this thread's copies for step cstep have landed
            const int stage = cstep % NST;
            uint8_t* sb = smem + stage * STAGE + A_BYTES;
            uint4 v[2];
            if (WT == T_Q4_K) dq_q4k_raw(smem_u32(sb + B_BYTES + tid * RAW_SLOT), (ckb * BK / 32) & 7, v);
            else dq_generic(wrow(cT), WT, ckb * BK, 2 * half, v);
            *reinterpret_cast<uint4*>(sb + sw_off(row, 2 * half)) = v[0];
            *reinterpret_cast<uint4*>(sb + sw_off(row, 2 * half + 1)) = v[1];
            fence_async_smem();  // generic and cp.async stores -> visible to the tensor core
            __syncwarp();
            if (lane == 0) mbar_arrive(full + stage);
            if (++ckb == nK) {
                ckb = 0;
                ct += gridDim.x;
                if (ct < total) cT = pf_tile(p, ct, nN);
            }
        }
        cp_async_wait<0>();
    } else if (warp == MMA_WARP) {
        // ---------------- MMA issue ----------------
        int step = 0, ti = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
            const int buf = ti & 1;
            if (ti >= 2) mbar_wait(accfree + buf, ((ti >> 1) - 1) & 1, p.ctrl);
            tc_fence_after();
            for (int kb = 0; kb < nK; ++kb, ++step) {
                const int stage = step % NST;
                mbar_wait(full + stage, (step / NST) & 1, p.ctrl);
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = smem_u32(smem + stage * STAGE);
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk)
                        mma_f16(tmem + buf * BN, sdesc(sa + kk * 32), sdesc(sa + A_BYTES + kk * 32), (kb | kk) != 0);
                    mma_commit(empty + stage);  // the stage is free once these MMAs have read it
                }
                __syncwarp();
            }
            if (lane == 0) mma_commit(accf + buf);  // accumulators complete
            __syncwarp();
        }
    } else {
        // ---------------- epilogue: TMEM -> global ----------------
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = tile rows
        int ti = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
            const PfTile T = pf_tile(p, t, nN);
            const int buf = ti & 1;
            mbar_wait(accf + buf, (ti >> 1) & 1, p.ctrl);
            tc_fence_after();
            const int orow = T.r0 + 32 * quarter + lane;
            const uint32_t tl = tmem + buf * BN + (static_cast<uint32_t>(32 * quarter) << 16);
            const int drow = (MODE == 1 && p.out_rows && orow < T.r1) ? __ldg(p.out_rows + orow) : orow;
            __half* dst = p.out + static_cast<size_t>(drow) * p.N + T.nt * ncol;
            for (int c0 = 0; c0 < ncol; c0 += 16) {
                uint32_t a[16];
                tmem_ld16(tl + c0, a);
                uint32_t o[8];
                if (MODE == 0) {
                    uint32_t u[16];
                    tmem_ld16(tl + BN / 2 + c0, u);
                    tmem_wait_ld();
                    float h[16];
#pragma unroll
                    for (int i = 0; i < 16; ++i) {
                        const float g = __uint_as_float(a[i]);
                        // moe.cu:64 (fast exp/divide: the result is rounded to fp16 next)
                        h[i] = __fdividef(g, 1.0f + __expf(-g)) * __uint_as_float(u[i]);
                    }
#pragma unroll
                    for (int c = 0; c < 2; ++c) {  // chunk element order for the down GEMM
                        o[4 * c] = h2_bits(__floats2half2_rn(h[8 * c], h[8 * c + 2]));
                        o[4 * c + 1] = h2_bits(__floats2half2_rn(h[8 * c + 1], h[8 * c + 3]));
                        o[4 * c + 2] = h2_bits(__floats2half2_rn(h[8 * c + 4], h[8 * c + 6]));
                        o[4 * c + 3] = h2_bits(__floats2half2_rn(h[8 * c + 5], h[8 * c + 7]));
                    }
                } else {
                    tmem_wait_ld();
#pragma unroll
                    for (int i = 0; i < 8; ++i)
                        o[i] = h2_bits(__floats2half2_rn(__uint_as_float(a[2 * i]), __uint_as_float(a[2 * i + 1])));
                }
                if (orow < T.r1 && drow < p.out_cap) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
                    d4[0] = make_uint4(o[0], o[1], o[2], o[3]);
                    d4[1] = make_uint4(o[4], o[5], o[6], o[7]);
                }
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(accfree + buf);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

inline size_t gemm_smem_bytes() { return 1024 + static_cast<size_t>(NST) * STAGE + 256; }

}  // namespace pf

// ---------------------------------------------------------------------------
// RMSNorm of every token (ops.cu:25-65 structure): one warp per token, the sum
// of squares with the reference GEMV's thread/shuffle structure (as in the
// decode router), then (x * scale) * weight.  Without a norm weight it copies.
// Besides x_in (F32) it writes the fp16 copy for the tensor cores, the copy in
// the router's leaf order (pf_perm_pos) for k_route_tile, and the shared-expert
// gate logit x_in . w_sg in the reference GEMV order (logits[t][E]).
// ---------------------------------------------------------------------------
__device__ __forceinline__ float pf_tree8(float (&acc)[2][4]);

// Position of element k = 256i + 128hh + 32g + 4l + c of a row in the router
// leaf order: the reference GEMV's 256 FMA chains (thread 4(8g+l)+c+128hh,
// elements i = 0..CH-1) grouped by the first level of its reduction tree
// (eight chains l = 0..7 of one (hh, g, c)), each chain's elements contiguous.
template <int CH>
__device__ __forceinline__ int pf_perm_pos(int i, int hh, int g, int l, int c) {
    return ((((hh * 4 + g) * 4 + c) * 8 + l) * CH) + i;
}

// Lane L of a warp holds v[i][hh] = elements 256i + 128hh + 4L + (0..3) of a
// row; write them in the leaf order (CH consecutive floats per chain).
template <int CH>
__device__ __forceinline__ void pf_store_perm(float* __restrict__ dst, const float4 (&v)[CH][2], int lane) {
    const int g = lane >> 3, l = lane & 7;
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float e[CH];
#pragma unroll
            for (int i = 0; i < CH; ++i) e[i] = c == 0 ? v[i][hh].x : c == 1 ? v[i][hh].y : c == 2 ? v[i][hh].z : v[i][hh].w;
            float* o = dst + pf_perm_pos<CH>(0, hh, g, l, c);
            if (CH % 4 == 0) {
#pragma unroll
                for (int i = 0; i < CH; i += 4) *reinterpret_cast<float4*>(o + i) = make_float4(e[i], e[i + 1], e[i + 2], e[i + 3]);
            } else {
#pragma unroll
                for (int i = 0; i < CH; ++i) o[i] = e[i];
            }
        }
}

template <int CH>
__device__ __forceinline__ void pf_load_row(float4 (&w)[CH][2], const uint8_t* row, int type, int lane);

template <int CH>
__global__ void __launch_bounds__(256) k_norm_many(const float* __restrict__ x, const float* __restrict__ w,
                                                   float eps, float* __restrict__ out, __half* __restrict__ x16,
                                                   float* __restrict__ xperm, const uint8_t* __restrict__ sgate,
                                                   int sgate_type, float* __restrict__ logits, int E, int T, int d) {
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
    __half* hrow = x16 + static_cast<size_t>(t) * d;
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int e0 = 256 * i + 128 * hh + 4 * lane;
            *reinterpret_cast<float4*>(orow + e0) = v[i][hh];
            // fp16 copy for the tensor cores, in the chunk element order
            // (0,2,1,3,4,6,5,7): this lane holds half of an 8-element chunk
            const uint2 hv = make_uint2(pf::h2_bits(__floats2half2_rn(v[i][hh].x, v[i][hh].z)),
                                        pf::h2_bits(__floats2half2_rn(v[i][hh].y, v[i][hh].w)));
            *reinterpret_cast<uint2*>(hrow + (e0 & ~7) + 4 * (lane & 1)) = hv;
        }
    pf_store_perm<CH>(xperm + static_cast<size_t>(t) * d, v, lane);
    if (sgate) {  // shared-expert gate logit, row E of the router output (layer_moe.cpp:140-144)
        float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
#pragma unroll
        for (int i = 0; i < CH; ++i) {
            float4 sg[1][2];  // the gate elements of this lane at step i
            pf_load_row<1>(sg, sgate + (sgate_type == T_F32 ? 4 : 2) * 256 * i, sgate_type, lane);
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                acc[hh][0] = __fmaf_rn(sg[0][hh].x, v[i][hh].x, acc[hh][0]);
                acc[hh][1] = __fmaf_rn(sg[0][hh].y, v[i][hh].y, acc[hh][1]);
                acc[hh][2] = __fmaf_rn(sg[0][hh].z, v[i][hh].z, acc[hh][2]);
                acc[hh][3] = __fmaf_rn(sg[0][hh].w, v[i][hh].w, acc[hh][3]);
            }
        }
        const float lg = pf_tree8(acc);
        if (lane == 0) logits[static_cast<size_t>(t) * (E + 1) + E] = lg;
    }
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
// Router logits of many tokens in the reference GEMV order (matmul_q4.cu:
// 140-167: 256 threads, thread j accumulates elements j*4+c+... with one FMA
// chain per (thread, component), then a fixed shuffle/partial-sum tree).
// Every logit is that fixed arithmetic DAG: 256 chains of CH FMAs, grouped by
// the tree into 32 first-level groups G(hh, g, c) of eight chains,
//   G = ((v0 + v4) + (v2 + v6)) + ((v1 + v5) + (v3 + v7))   (v_l: chain 8g+l),
//   s(hh, g) = (G(c=0) + G(c=2)) + (G(c=1) + G(c=3)),
//   logit = ((z00 + z10) + (z02 + z12)) + ((z01 + z11) + (z03 + z13)),
//   z_hg = (s(h, g) + 0) + 0.
// k_route_tile evaluates it for a 64-token x 32-expert tile per CTA: the
// inputs come in the leaf order (pf_perm_pos), one first-level group (96 rows
// x 8*CH floats) per pipeline stage, and every lane computes 4 tokens x 2
// experts with the whole tree in registers -- no shuffles, each shared-memory
// value feeding 2 or 4 FMAs.
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

// Router rows (expert rows, any supported row type) -> F32 in the leaf order.
template <int CH>
__global__ void __launch_bounds__(256) k_perm_rows(const uint8_t* __restrict__ router, int type, int E, int d,
                                                   float* __restrict__ wp) {
    const int lane = threadIdx.x & 31;
    const int e = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (e >= E) return;
    float4 w[CH][2];
    pf_load_row<CH>(w, router + static_cast<size_t>(e) * d * (type == T_F32 ? 4 : 2), type, lane);
    pf_store_perm<CH>(wp + static_cast<size_t>(e) * d, w, lane);
}

namespace rt {
constexpr int TT = 64, TE = 32, ROWS = TT + TE, NSTG = 4;
template <int CH>
__host__ __device__ constexpr int rs() { return 8 * CH + 4; }  // padded row stride in floats (rows land on distinct bank groups)
template <int CH>
constexpr size_t smem_bytes() { return static_cast<size_t>(NSTG) * ROWS * rs<CH>() * sizeof(float); }

// Chain l of the current group for this lane's 8 (token, expert) pairs:
// pair p = (token p/2, expert p%2), acc = fma(w_i, x_i, acc) over i = 0..CH-1.
template <int CH>
__device__ __forceinline__ void chains(const float* xr, const float* wr, float (&v)[8]) {
    constexpr int RS = rs<CH>();
    float xv[4][CH], wv[2][CH];
#pragma unroll
    for (int tt = 0; tt < 4; ++tt) {
        const float* src = xr + tt * 4 * RS;
        if (CH % 4 == 0) {
#pragma unroll
            for (int i = 0; i < CH; i += 4) {
                const float4 q = *reinterpret_cast<const float4*>(src + i);
                xv[tt][i] = q.x; xv[tt][i + 1] = q.y; xv[tt][i + 2] = q.z; xv[tt][i + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) xv[tt][i] = src[i];
        }
    }
#pragma unroll
    for (int ee = 0; ee < 2; ++ee) {
        const float* src = wr + ee * 8 * RS;
        if (CH % 4 == 0) {
#pragma unroll
            for (int i = 0; i < CH; i += 4) {
                const float4 q = *reinterpret_cast<const float4*>(src + i);
                wv[ee][i] = q.x; wv[ee][i + 1] = q.y; wv[ee][i + 2] = q.z; wv[ee][i + 3] = q.w;
            }
        } else {
#pragma unroll
            for (int i = 0; i < CH; ++i) wv[ee][i] = src[i];
        }
    }
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        float acc = 0.0f;
#pragma unroll
        for (int i = 0; i < CH; ++i) acc = __fmaf_rn(wv[p & 1][i], xv[p >> 1][i], acc);
        v[p] = acc;
    }
}
}  // namespace rt

template <int CH>
__global__ void __launch_bounds__(256, 2) k_route_tile(const float* __restrict__ xp, const float* __restrict__ wp,
                                                       const float* __restrict__ bias, float* __restrict__ logits,
                                                       int T, int E, int d) {
    constexpr int GS = 8 * CH, RS = rt::rs<CH>();
    extern __shared__ __align__(16) float rt_smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int t0 = blockIdx.x * rt::TT, e0 = blockIdx.y * rt::TE;
    // warp: 16 tokens x 16 experts; lane: tokens wt*16 + tt*4 + tg, experts we*16 + ee*8 + eg
    const int wt = warp & 3, we = warp >> 2, tg = lane >> 3, eg = lane & 7;
    // group q = 4u + ci in tree order: unit u -> (g, hh), ci -> c
    auto stage = [&](int q) {
        const int u = q >> 2, ci = q & 3;
        const int g = (0x3120 >> (4 * (u >> 1))) & 0xF;   // units pair g = 0, 2, 1, 3
        const int hh = u & 1;
        const int c = (0x3120 >> (4 * ci)) & 0xF;          // c = 0, 2, 1, 3
        const int off = ((hh * 4 + g) * 4 + c) * GS;
        float* buf = rt_smem + (q % rt::NSTG) * rt::ROWS * RS;
        for (int ch = tid; ch < rt::ROWS * (GS / 4); ch += 256) {
            const int row = ch / (GS / 4), col = (ch % (GS / 4)) * 4;
            const float* src;
            bool ok;
            if (row < rt::TT) {
                const int t = t0 + row;
                ok = t < T;
                src = xp + static_cast<size_t>(ok ? t : 0) * d + off + col;
            } else {
                const int e = e0 + row - rt::TT;
                ok = e < E;
                src = wp + static_cast<size_t>(ok ? e : 0) * d + off + col;
            }
            pf::cp_async16(smem_u32(buf + row * RS + col), src, ok ? 16u : 0u);
        }
        pf::cp_async_commit();
    };
    float r0[8], r1[8], r2[8];  // pending partial sums of the last tree level
#pragma unroll
    for (int p = 0; p < 8; ++p) r0[p] = r1[p] = r2[p] = 0.0f;
    for (int q = 0; q < rt::NSTG - 1; ++q) stage(q);
    for (int u = 0; u < 8; ++u) {
        float sp[8], s1[8], sv[8];
#pragma unroll
        for (int ci = 0; ci < 4; ++ci) {
            const int q = 4 * u + ci;
            pf::cp_async_wait<rt::NSTG - 2>();  // group q has landed (this thread's copies)
            __syncthreads();                    // everyone's copies; everyone is done with group q-1
            if (q + rt::NSTG - 1 < 32) stage(q + rt::NSTG - 1); else pf::cp_async_commit();
            const float* buf = rt_smem + ci * rt::ROWS * RS;  // q % NSTG == ci
            const float* xr = buf + (wt * 16 + tg) * RS;
            const float* wr = buf + (rt::TT + we * 16 + eg) * RS;
            float G[8], A[8], C[8], tmp[8], v[8];
#pragma unroll
            for (int li = 0; li < 8; ++li) {
                const int l = (0x73516240 >> (4 * li)) & 0xF;  // 0, 4, 2, 6, 1, 5, 3, 7
                rt::chains<CH>(xr + l * CH, wr + l * CH, v);
#pragma unroll
                for (int p = 0; p < 8; ++p) {
                    if (li == 0 || li == 2 || li == 4 || li == 6) tmp[p] = v[p];
                    else if (li == 1) A[p] = __fadd_rn(tmp[p], v[p]);
                    else if (li == 3) A[p] = __fadd_rn(A[p], __fadd_rn(tmp[p], v[p]));
                    else if (li == 5) C[p] = __fadd_rn(tmp[p], v[p]);
                    else G[p] = __fadd_rn(A[p], __fadd_rn(C[p], __fadd_rn(tmp[p], v[p])));
                }
            }
#pragma unroll
            for (int p = 0; p < 8; ++p) {
                if (ci == 0) sp[p] = G[p];
                else if (ci == 1) sp[p] = __fadd_rn(sp[p], G[p]);
                else if (ci == 2) s1[p] = G[p];
                else sv[p] = __fadd_rn(sp[p], __fadd_rn(s1[p], G[p]));
            }
        }
#pragma unroll
        for (int p = 0; p < 8; ++p) {
            const float z = __fadd_rn(__fadd_rn(sv[p], 0.0f), 0.0f);
            switch (u) {
                case 0: r0[p] = z; break;
                case 1: r0[p] = __fadd_rn(r0[p], z); break;
                case 2: r1[p] = z; break;
                case 3: r0[p] = __fadd_rn(r0[p], __fadd_rn(r1[p], z)); break;
                case 4: r1[p] = z; break;
                case 5: r1[p] = __fadd_rn(r1[p], z); break;
                case 6: r2[p] = z; break;
                default: r0[p] = __fadd_rn(r0[p], __fadd_rn(r1[p], __fadd_rn(r2[p], z))); break;
            }
        }
    }
    pf::cp_async_wait<0>();
#pragma unroll
    for (int p = 0; p < 8; ++p) {
        const int t = t0 + wt * 16 + (p >> 1) * 4 + tg;
        const int e = e0 + we * 16 + (p & 1) * 8 + eg;
        if (t < T && e < E)
            logits[static_cast<size_t>(t) * (E + 1) + e] = bias ? __fadd_rn(r0[p], __ldg(bias + e)) : r0[p];
    }
}

// ---------------------------------------------------------------------------
// One warp per token: top-k, softmax, checks; the failing tokens get id -1
// and NaN weights, and the error word records the first of them.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_topk_many(const float* __restrict__ logits, int T, int E, int k,
                                                   int32_t* __restrict__ idx, float* __restrict__ wts,
                                                   int32_t* __restrict__ out_idx, float* __restrict__ out_w,
                                                   int32_t* __restrict__ sh_grp, uint32_t* ctrl) {
    const int lane = threadIdx.x & 31;
    const int t = blockIdx.x * 8 + (threadIdx.x >> 5);
    if (t == 0 && lane == 0) {
        // the shared expert's one-group GEMM plan: all T tokens, ceil(T / 128) tiles
        sh_grp[0] = 0;
        sh_grp[1] = T;
        sh_grp[2] = 0;
        sh_grp[3] = (T + pf::BM - 1) / pf::BM;
    }
    if (t >= T) return;
    int my_idx;
    float wj;
    uint32_t flag;
    select_token(logits + static_cast<size_t>(t) * (E + 1), E, k, lane, my_idx, wj, flag);
    if (flag && lane == 0) {
        raise_error(ctrl, flag);
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
// Stable (expert, token, slot) permutation of the top-k result for many
// tokens.  A token selects an expert at most once, so within a block of 64
// tokens the pairs of expert e are described by a 64-bit token mask; a pair's
// position is its expert's offset, plus the pairs of e in earlier blocks,
// plus the earlier tokens of its own block in the mask.  Three small
// kernels: masks -> per-block counts, one scan, placement.
// ---------------------------------------------------------------------------
constexpr int DB = 64;  // tokens per dispatch block

__device__ __forceinline__ void pf_block_masks(const int32_t* idx, int T, int k, int E, int b,
                                               unsigned long long* mask) {
    for (int e = threadIdx.x; e < E; e += blockDim.x) mask[e] = 0ull;
    __syncthreads();
    const int t0 = b * DB;
    for (int q = threadIdx.x; q < DB * k; q += blockDim.x) {
        const int tl = q / k, t = t0 + tl;
        if (t >= T) continue;
        const int e = __ldg(idx + t * k + (q - tl * k));
        if (e >= 0 && e < E) atomicOr(mask + e, 1ull << tl);
    }
    __syncthreads();
}

__global__ void __launch_bounds__(256) k_pf_count(const int32_t* __restrict__ idx, int T, int k, int E,
                                                  int32_t* __restrict__ counts) {
    __shared__ unsigned long long mask[kMaxExperts];
    pf_block_masks(idx, T, k, E, blockIdx.x, mask);
    for (int e = threadIdx.x; e < E; e += blockDim.x) counts[blockIdx.x * E + e] = __popcll(mask[e]);
}

// counts[b][e] -> first position of block b's pairs of expert e; offsets[E+1].
// One CTA of SCAN_SEG x 256 threads: thread (seg, e) owns expert e's counts
// in the seg-th quarter of the token blocks, so the dependent global
// round trips per thread are a quarter of the blocks: segment sums, then
// each segment's start (expert base from the scan over experts + the
// earlier segments of the same expert), then the running sum written back.
constexpr int SCAN_SEG = 4;
__global__ void __launch_bounds__(SCAN_SEG * 256) k_pf_scan(int32_t* __restrict__ counts, int nb, int E,
                                                            int32_t* __restrict__ offsets) {
    static_assert(kMaxExperts <= 256, "one thread per expert and segment");
    __shared__ int s_seg[SCAN_SEG][256];
    __shared__ int s_base[256];
    __shared__ int s_wsum[8];
    const int e = threadIdx.x & 255, seg = threadIdx.x >> 8, lane = e & 31, warp = e >> 5;
    const int per = (nb + SCAN_SEG - 1) / SCAN_SEG;
    const int b_lo = min(nb, seg * per), b_hi = min(nb, b_lo + per);
    constexpr int U = 8;  // loads issued ahead of the dependent adds / stores (64 registers)
    int sum = 0;
    if (e < E)
        for (int b0 = b_lo; b0 < b_hi; b0 += U) {
            int c[U];
#pragma unroll
            for (int j = 0; j < U; ++j) c[j] = b0 + j < b_hi ? counts[(b0 + j) * E + e] : 0;
#pragma unroll
            for (int j = 0; j < U; ++j) sum += c[j];
        }
    s_seg[seg][e] = e < E ? sum : 0;
    __syncthreads();
    if (seg == 0) {
        // exclusive scan of the experts' totals (threads 0..255)
        int tot = 0;
        for (int q = 0; q < SCAN_SEG; ++q) tot += s_seg[q][e];
        int inc = tot;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, inc, o);
            if (lane >= o) inc += y;
        }
        if (lane == 31) s_wsum[warp] = inc;
        asm volatile("bar.sync 1, 256;" ::: "memory");  // the first 256 threads only
        int base = 0, total = 0;
        for (int w = 0; w < 8; ++w) {
            base += w < warp ? s_wsum[w] : 0;
            total += s_wsum[w];
        }
        const int off = base + inc - tot;
        s_base[e] = off;
        if (e < E) offsets[e] = off;
        if (e == 0) offsets[E] = total;
    }
    __syncthreads();
    if (e < E) {
        int run = s_base[e];  // + expert e's pairs in the earlier segments
        for (int q = 0; q < seg; ++q) run += s_seg[q][e];
        for (int b0 = b_lo; b0 < b_hi; b0 += U) {
            int c[U];
#pragma unroll
            for (int j = 0; j < U; ++j) c[j] = b0 + j < b_hi ? counts[(b0 + j) * E + e] : 0;
#pragma unroll
            for (int j = 0; j < U; ++j)
                if (b0 + j < b_hi) {
                    counts[(b0 + j) * E + e] = run;
                    run += c[j];
                }
        }
    }
}

__global__ void __launch_bounds__(256) k_pf_place(const int32_t* __restrict__ idx, int T, int k, int E,
                                                  const int32_t* __restrict__ counts, int32_t* __restrict__ perm,
                                                  int32_t* __restrict__ inv_perm) {
    __shared__ unsigned long long mask[kMaxExperts];
    pf_block_masks(idx, T, k, E, blockIdx.x, mask);
    const int t0 = blockIdx.x * DB;
    for (int q = threadIdx.x; q < DB * k; q += blockDim.x) {
        const int tl = q / k, t = t0 + tl;
        if (t >= T) continue;
        const int p = t * k + (q - tl * k);
        const int e = __ldg(idx + p);
        int rank = -1;
        if (e >= 0 && e < E) {
            rank = counts[blockIdx.x * E + e] + __popcll(mask[e] & ((1ull << tl) - 1ull));
            perm[rank] = p;
        }
        inv_perm[p] = rank;
    }
}

// ---------------------------------------------------------------------------
// Source token of every permuted pair and the 128-row tile prefix per expert
// (routed experts) plus the shared expert's single group [0, T).
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) k_pf_plan(const int32_t* __restrict__ offsets, const int32_t* __restrict__ perm,
                                                 int E, int k, int32_t* __restrict__ tok_of_pos,
                                                 int32_t* __restrict__ tile_start, const int32_t* __restrict__ qmap,
                                                 int32_t* __restrict__ out_pos) {
    const int npairs = __ldg(offsets + E);
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < npairs; i += gridDim.x * blockDim.x) {
        const int p = __ldg(perm + i);
        tok_of_pos[i] = p / k;
        if (qmap) out_pos[i] = __ldg(qmap + p);  // output row of the pair (expert-parallel path)
    }
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
        if (lane == 0) tile_start[E] = run;
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
        // pair (t, j) sits at its permuted position, or at t*k + j when the
        // expert outputs come back in pair order (expert-parallel path)
        s_pos[threadIdx.x] = inv_perm ? __ldg(inv_perm + t * k + threadIdx.x) : t * k + threadIdx.x;
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
    const size_t smem = pf::gemm_smem_bytes();
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
    if (P.d % pf::BN || P.F % (pf::BN / 2) || P.Fs % (pf::BN / 2) || P.F % pf::BK || P.Fs % pf::BK) return false;
    if (P.d > kMaxNormDim || P.d % 256) return false;
    return pf_num_sms() > 0;
}

// Steps of the prefill path, also used by the expert-parallel entry points.
// x_in / X16 and the routing of T tokens.
cudaError_t pf_route(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) {
    const int T = P.T, d = P.d, E = P.E, k = P.k;
    const int CH = d / 256;
    cudaError_t e = cudaSuccess;
    const float* nw = P.prenorm ? P.norm_w : nullptr;
    const uint8_t* sg = P.has_shared ? P.sgate_inp : nullptr;
    const dim3 ngrid((T + 7) / 8), pgrid((E + 7) / 8), rgrid((T + rt::TT - 1) / rt::TT, (E + rt::TE - 1) / rt::TE);
#define QMOE_ROUTE(C)                                                                                               \
    do {                                                                                                            \
        k_norm_many<C><<<ngrid, 256, 0, s>>>(P.x, nw, P.eps, P.xnorm, B.X16, B.xperm, sg, P.sgate_type, P.logits, E, \
                                             T, d);                                                                 \
        k_perm_rows<C><<<pgrid, 256, 0, s>>>(P.router, P.router_type, E, d, B.wperm);                                \
        if ((e = pf_set_smem(k_route_tile<C>, rt::smem_bytes<C>())) != cudaSuccess) return e;                       \
        k_route_tile<C><<<rgrid, 256, rt::smem_bytes<C>(), s>>>(B.xperm, B.wperm, P.bias, P.logits, T, E, d);       \
    } while (0)
    switch (CH) {
        case 1: QMOE_ROUTE(1); break;
        case 2: QMOE_ROUTE(2); break;
        case 4: QMOE_ROUTE(4); break;
        case 8: QMOE_ROUTE(8); break;
        default: return cudaErrorInvalidValue;
    }
#undef QMOE_ROUTE
    if ((e = cudaGetLastError()) != cudaSuccess) return e;
    k_topk_many<<<(T + 7) / 8, 256, 0, s>>>(P.logits, T, E, k, P.topk_idx, P.topk_w, P.out_idx, P.out_w, B.sh_grp,
                                            P.ctrl);
    return cudaGetLastError();
}

// Permutation of the (row, slot) pairs of `idx` [T][k] by expert, and the
// GEMM tile plan.
static cudaError_t pf_dispatch(const int32_t* idx, int T, int k, int E, int32_t* offsets, int32_t* perm,
                               int32_t* inv_perm, const PrefillBufs& B, cudaStream_t s,
                               const int32_t* qmap = nullptr, int32_t* out_pos = nullptr) {
    const int nb = (T + DB - 1) / DB;
    k_pf_count<<<nb, 256, 0, s>>>(idx, T, k, E, B.disp);
    k_pf_scan<<<1, SCAN_SEG * 256, 0, s>>>(B.disp, nb, E, offsets);
    k_pf_place<<<nb, 256, 0, s>>>(idx, T, k, E, B.disp, perm, inv_perm);
    k_pf_plan<<<64, 256, 0, s>>>(offsets, perm, E, k, B.tok_of_pos, B.tile_start, qmap, out_pos);
    return cudaGetLastError();
}

// Routed experts: rows A (fp16, chunk order) gathered through tok_of_pos,
// hidden H, outputs Y (y_rows rows: at the permuted positions, or in
// `out_rows` order).  Q4_K experts take the TMA-fed GEMM (k_tgemm.cu), whose
// activation tiles must be contiguous: the rows are first gathered in
// position order into Y itself, which the down GEMM overwrites afterwards.
static cudaError_t pf_routed(const DecodeParams& P, const PrefillBufs& B, const __half* a16, __half* y, int y_rows,
                             const int32_t* out_rows, cudaStream_t s, const TgScatter* sc = nullptr,
                             __half* xp = nullptr) {
    const int d = P.d;
    const int h_rows = P.T * P.k;  // capacity of H (one row per pair)
    cudaError_t e;
    if (P.gate.type == P.up.type && tgemm_supported(P.gate.type, 0, P.F, d) &&
        tgemm_supported(P.down.type, 1, d, P.F)) {
        if (!xp) xp = y;  // the gathered rows live in Y until the down GEMM overwrites it
        if ((e = launch_gather_rows(a16, B.tok_of_pos, P.offsets + P.E, y_rows, d, xp, s)) != cudaSuccess) return e;
        TgArgs g{};
        g.mode = 0;
        g.a16 = xp;
        g.a_rows = static_cast<uint64_t>(y_rows);
        g.w0 = P.gate.p;
        g.w1 = P.up.p;
        g.K = d;
        g.p = TgParams{P.F, d, P.E, P.F, P.offsets, B.tile_start, B.H, nullptr, h_rows, P.ctrl, {}};
        if ((e = launch_tgemm(g, s)) != cudaSuccess) return e;
        TgArgs dn{};
        dn.mode = 1;
        dn.a16 = B.H;
        dn.a_rows = static_cast<uint64_t>(h_rows);
        dn.w0 = P.down.p;
        dn.K = P.F;
        dn.p = TgParams{d, P.F, P.E, d, P.offsets, B.tile_start, y, out_rows, y_rows, P.ctrl, {}};
        if (sc) dn.p.sc = *sc;
        return launch_tgemm(dn, s);
    }
    if (sc) return cudaErrorNotSupported;  // direct return needs the Q4_K GEMM
    pf::GemmParams g{};
    g.a16 = a16;
    g.a_rows = B.tok_of_pos;
    g.w0 = P.gate.p;
    g.w1 = P.up.p;
    g.w_row_bytes = static_cast<uint32_t>(row_bytes(P.gate.type, d));
    g.w_group_bytes = static_cast<uint64_t>(P.F) * g.w_row_bytes;
    g.wtype = P.gate.type;
    g.N = P.F;
    g.K = d;
    g.groups = P.E;
    g.grp_start = P.offsets;
    g.tile_start = B.tile_start;
    g.out = B.H;
    g.out_cap = h_rows;
    g.ctrl = P.ctrl;
    if ((e = launch_pgemm<0>(g, s)) != cudaSuccess) return e;
    pf::GemmParams dn{};
    dn.a16 = B.H;
    dn.w0 = P.down.p;
    dn.w_row_bytes = static_cast<uint32_t>(row_bytes(P.down.type, P.F));
    dn.w_group_bytes = static_cast<uint64_t>(d) * dn.w_row_bytes;
    dn.wtype = P.down.type;
    dn.N = d;
    dn.K = P.F;
    dn.groups = P.E;
    dn.grp_start = P.offsets;
    dn.tile_start = B.tile_start;
    dn.out = y;
    dn.out_rows = out_rows;
    dn.out_cap = y_rows;
    dn.ctrl = P.ctrl;
    return launch_pgemm<1>(dn, s);
}

// Shared expert over all T tokens (rows of X16), then the combine of the
// routed outputs Y (at inv_perm positions, or in pair order when null).
static cudaError_t pf_shared(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) {
    const int d = P.d;
    cudaError_t e;
    if (P.has_shared && P.sgate.type == P.sup.type && tgemm_supported(P.sgate.type, 0, P.Fs, d) &&
        tgemm_supported(P.sdown.type, 1, d, P.Fs)) {
        TgArgs g{};
        g.mode = 0;
        g.a16 = B.X16;
        g.a_rows = static_cast<uint64_t>(P.T);
        g.w0 = P.sgate.p;
        g.w1 = P.sup.p;
        g.K = d;
        g.p = TgParams{P.Fs, d, 1, P.Fs, B.sh_grp, B.sh_tiles, B.Hs, nullptr, P.T, P.ctrl, {}};
        if ((e = launch_tgemm(g, s)) != cudaSuccess) return e;
        TgArgs dn{};
        dn.mode = 1;
        dn.a16 = B.Hs;
        dn.a_rows = static_cast<uint64_t>(P.T);
        dn.w0 = P.sdown.p;
        dn.K = P.Fs;
        dn.p = TgParams{d, P.Fs, 1, d, B.sh_grp, B.sh_tiles, B.Ys, nullptr, P.T, P.ctrl, {}};
        if ((e = launch_tgemm(dn, s)) != cudaSuccess) return e;
    } else if (P.has_shared) {
        pf::GemmParams gs{};
        gs.a16 = B.X16;
        gs.w0 = P.sgate.p;
        gs.w1 = P.sup.p;
        gs.w_row_bytes = static_cast<uint32_t>(row_bytes(P.sgate.type, d));
        gs.w_group_bytes = static_cast<uint64_t>(P.Fs) * gs.w_row_bytes;
        gs.wtype = P.sgate.type;
        gs.N = P.Fs;
        gs.K = d;
        gs.groups = 1;
        gs.grp_start = B.sh_grp;
        gs.tile_start = B.sh_tiles;
        gs.out = B.Hs;
        gs.out_cap = P.T;
        gs.ctrl = P.ctrl;
        if ((e = launch_pgemm<0>(gs, s)) != cudaSuccess) return e;
        pf::GemmParams ds{};
        ds.a16 = B.Hs;
        ds.w0 = P.sdown.p;
        ds.w_row_bytes = static_cast<uint32_t>(row_bytes(P.sdown.type, P.Fs));
        ds.w_group_bytes = static_cast<uint64_t>(d) * ds.w_row_bytes;
        ds.wtype = P.sdown.type;
        ds.N = d;
        ds.K = P.Fs;
        ds.groups = 1;
        ds.grp_start = B.sh_grp;
        ds.tile_start = B.sh_tiles;
        ds.out = B.Ys;
        ds.out_cap = P.T;
        ds.ctrl = P.ctrl;
        if ((e = launch_pgemm<1>(ds, s)) != cudaSuccess) return e;
    }
    return cudaSuccess;
}

static cudaError_t pf_combine(const DecodeParams& P, const PrefillBufs& B, const __half* Y, const int32_t* inv_perm,
                              cudaStream_t s) {
    k_pf_combine<<<P.T, 256, 0, s>>>(Y, B.Ys, inv_perm, P.topk_w, P.logits, P.residual, P.out, P.d, P.E, P.k,
                                     P.has_shared);
    return cudaGetLastError();
}

static cudaError_t pf_shared_combine(const DecodeParams& P, const PrefillBufs& B, const __half* Y,
                                     const int32_t* inv_perm, cudaStream_t s) {
    cudaError_t e = pf_shared(P, B, s);
    return e != cudaSuccess ? e : pf_combine(P, B, Y, inv_perm, s);
}

// The whole block for T tokens through the prefill kernels.
cudaError_t launch_prefill(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) {
    cudaError_t e;
    if ((e = pf_route(P, B, s)) != cudaSuccess) return e;
    if ((e = pf_dispatch(P.topk_idx, P.T, P.k, P.E, P.offsets, P.perm, P.inv_perm, B, s)) != cudaSuccess) return e;
    if ((e = pf_routed(P, B, B.X16, B.Y, P.T * P.k, nullptr, s)) != cudaSuccess) return e;
    return pf_shared_combine(P, B, B.Y, P.inv_perm, s);
}

// Kernels one launch_prefill call issues: routing (norm, router rows, router
// tile, top-k), dispatch (count, scan, place, plan), the routed products
// (row gather + TMA gate/up + TMA down, or the two cp.async GEMMs), the
// shared expert's two GEMMs when there is one, and the combine.
int prefill_kernel_count(const DecodeParams& P) {
    const bool tma_routed = P.gate.type == P.up.type && tgemm_supported(P.gate.type, 0, P.F, P.d) &&
                            tgemm_supported(P.down.type, 1, P.d, P.F);
    return 4 + 4 + (tma_routed ? 3 : 2) + (P.has_shared ? 2 : 0) + 1;
}

// Expert-parallel pieces.  Route: x_in, X16 and top-k of T local tokens.
cudaError_t launch_ep_route(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) { return pf_route(P, B, s); }

// This rank's experts on n received rows: rows x16 [n][d] (chunk order) and
// meta [n][k] (local expert id per slot or -1; P.k = k, P.E = local experts);
// qmap [n*k] numbers the valid slots in (row, slot) order, out_pos receives
// that number for every expert-sorted pair; outputs y [pairs][d] fp16 in that
// order, or (sc) straight into the owning ranks' return buffers; xp holds the
// rows gathered in pair order.
cudaError_t launch_ep_experts(const DecodeParams& P, const PrefillBufs& B, const __half* x16, const int32_t* meta,
                              const int32_t* qmap, int32_t* out_pos, __half* y, int y_rows, const TgScatter* sc,
                              __half* xp, cudaStream_t s) {
    cudaError_t e;
    if ((e = pf_dispatch(meta, P.T, P.k, P.E, P.offsets, P.perm, P.inv_perm, B, s, qmap, out_pos)) != cudaSuccess)
        return e;
    return pf_routed(P, B, x16, y, y_rows, out_pos, s, sc, xp);
}

// Shared expert and combine of T local tokens; the routed outputs of pair
// (t, j) are row pair_pos[t*k + j] of y_pairs (-1: none).  The two halves
// separately: the shared expert (needs only the routing call's workspace), the
// combine (after the shared half).
cudaError_t launch_ep_combine(const DecodeParams& P, const PrefillBufs& B, const __half* y_pairs,
                              const int32_t* pair_pos, cudaStream_t s) {
    return pf_shared_combine(P, B, y_pairs, pair_pos, s);
}
cudaError_t launch_ep_shared(const DecodeParams& P, const PrefillBufs& B, cudaStream_t s) { return pf_shared(P, B, s); }
cudaError_t launch_ep_combine_routed(const DecodeParams& P, const PrefillBufs& B, const __half* y_pairs,
                                     const int32_t* pair_pos, cudaStream_t s) {
    return pf_combine(P, B, y_pairs, pair_pos, s);
}

}  // namespace qmoe
