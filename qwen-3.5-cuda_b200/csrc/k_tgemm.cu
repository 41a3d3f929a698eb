// Grouped Q4_K expert GEMM fed by TMA (the prefill path's weight type in the
// benchmark configurations; src/layer_moe.cpp:127-154 computes the same
// products one token at a time with matmul_q4.cu's GEMV).
//
// One persistent CTA per SM walks output tiles of 128 rows (pairs or tokens)
// x 256 columns (MODE 0: 128 gate + 128 up rows of the expert, epilogue
// silu(gate) * up -> 128 hidden columns; MODE 1: 256 rows of down), K in
// slices of 64:
//   warp 0        TMA of the activation slice [128 rows x 64 fp16], tensor
//                 map with the 128-byte swizzle, i.e. straight into the UMMA
//                 K-major operand layout (rows past the group are discarded)
//   warp 1        TMA of the weight super-blocks: [256 rows x 144 bytes] of
//                 raw Q4_K per 256 K (no swizzle), double-buffered
//   warps 2..17   dequantisation: thread (row, half) turns the 32 nibbles of
//                 one sub-block into fp16 (exact nibble -> half conversion,
//                 one hfma2 per pair with d*sc and -dmin*m, as the reference's
//                 d*sc*q - dmin*m rounded once to fp16) and stores them in the
//                 same 128-byte-swizzled K-major layout
//   warp 18       one thread issues tcgen05.mma kind::f16 (M 128, N 256,
//                 K 16) into one of two TMEM accumulators; commits free the
//                 operand slots and publish a finished accumulator
//   warps 19..22  epilogue: TMEM -> registers -> fp16 rows in global memory
// Inside each 8-element chunk both operands use the element order
// (0,2,1,3,4,6,5,7) (the activations are stored that way), which turns Q4_K
// nibble pairs into half2 values with one logic op; a common permutation of K
// leaves the products unchanged.
//
// Every wait is bounded: on expiry the role records EF_TIMEOUT and leaves its
// loop; the TMA issuers then wait (bounded) for their own copies in flight
// before the CTA frees its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_fp16.h>

#include "qmoe_dev.cuh"
#include "qmoe_internal.h"
#include "qmoe_units.cuh"
#include "qmoe_tgemm.h"

namespace qmoe {
namespace tg {

constexpr int BM = 128, BN = 256, KS = 64;  // tile rows, tile columns, K per slice
constexpr int SB_K = 256, SB_BYTES = 144;   // Q4_K super-block
constexpr int NA = 3, NB = 3, NR = 2;       // activation / dequantised-weight / raw-weight slots
constexpr uint32_t A_BYTES = BM * 128;      // 16 KB
constexpr uint32_t B_BYTES = BN * 128;      // 32 KB
constexpr uint32_t R_BYTES = BN * SB_BYTES;  // 36 KB
constexpr uint32_t OFF_A = 0, OFF_B = OFF_A + NA * A_BYTES, OFF_R = OFF_B + NB * B_BYTES;
constexpr uint32_t OFF_BAR = OFF_R + NR * R_BYTES;
constexpr int DQ_WARPS = 16;
constexpr int WARP_TA = 0, WARP_TR = 1, WARP_DQ = 2, WARP_MMA = WARP_DQ + DQ_WARPS, WARP_EPI = WARP_MMA + 1;
constexpr int THREADS = (WARP_EPI + 4) * 32;
constexpr uint32_t TMEM_COLS = 2 * BN;
constexpr uint32_t IDESC = (1u << 4) | (static_cast<uint32_t>(BN >> 3) << 17) | (static_cast<uint32_t>(BM >> 4) << 24);

constexpr int MAX_GROUPS = kMaxExperts;     // group tables staged in shared memory
constexpr uint32_t OFF_TAB = OFF_BAR + 256;  // tile_start[groups + 1], grp_start[groups + 1]
constexpr size_t smem_bytes() { return 1024 + OFF_TAB + 2 * (MAX_GROUPS + 1) * sizeof(int32_t); }

// shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row groups
// 1024 bytes apart (tile bases are 1024-byte aligned)
__device__ __forceinline__ uint64_t sdesc(uint32_t saddr) {
    uint64_t d = static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
    d |= static_cast<uint64_t>(1u) << 16;
    d |= static_cast<uint64_t>(1024u >> 4) << 32;
    d |= static_cast<uint64_t>(1u) << 46;
    d |= static_cast<uint64_t>(2u) << 61;
    return d;
}

__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
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
__device__ __forceinline__ void sts128(uint32_t a, uint32_t x, uint32_t y, uint32_t z, uint32_t w) {
    asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(a), "r"(x), "r"(y), "r"(z), "r"(w) : "memory");
}

// Sub-block H (0: low nibbles, 1: high) of group g of one Q4_K super-block
// (raw row in shared memory) -> 32 fp16 values = chunks 4H..4H+3 of row r of
// the operand slot (128-byte rows, chunk c stored at c ^ (r % 8)).
//
// The value d*sc*q - dmin*m (matmul_q4.cu:76-96) is rounded to fp16 once:
// written as ((q - 8) * sc) * d + (8*d*sc - dmin*m), the first product is an
// integer of at most 504 in magnitude (exact in fp16), d is the block's own
// fp16 scale, and one fused half2 multiply-add rounds the sum.  The constant
// c = 8*d*sc - dmin*m (computed in F32) is about half a quantisation step, so
// its own fp16 rounding is small.  (Rounding d*sc and dmin*m to fp16 first
// and applying them to q doubles the error of the products, and the error is
// shared by the sub-block's 32 weights and every token.)
template <int H>
__device__ __forceinline__ void dq_sub(uint32_t raw, int g, uint32_t brow, int r) {
    const uint4 hd = lds128(raw);
    const uint4 q0 = lds128(raw + 16 + 32 * g);
    const uint4 q1 = lds128(raw + 32 + 32 * g);
    float sc, m;
    kscale(hd.y, hd.z, hd.w, 2 * g + H, sc, m);
    const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
    const __half2 d2 = bits_h2((hd.x & 0xFFFFu) * 0x00010001u);  // the fp16 d, both halves
    const __half2 sc2 = __float2half2_rn(sc);                     // integer 0..63: exact
    const __half2 c2 = __float2half2_rn(fmaf(8.0f * d, sc, -(dmin * m)));
    const __half2 k1032 = __float2half2_rn(1032.0f);
    const int sh = 4 * H;
    // half2(1024 + n(byte e), 1024 + n(byte e+2)): element order 0,2 / 1,3
    auto cvt = [&](uint32_t w) {
        const __half2 raw2 = bits_h2(((w >> sh) & 0x000F000Fu) | 0x64006400u);
        return h2_bits(__hfma2(__hmul2(__hsub2(raw2, k1032), sc2), d2, c2));
    };
    const uint32_t x7 = static_cast<uint32_t>(r & 7);
    sts128(brow + (((4 * H + 0) ^ x7) << 4), cvt(q0.x), cvt(q0.x >> 8), cvt(q0.y), cvt(q0.y >> 8));
    sts128(brow + (((4 * H + 1) ^ x7) << 4), cvt(q0.z), cvt(q0.z >> 8), cvt(q0.w), cvt(q0.w >> 8));
    sts128(brow + (((4 * H + 2) ^ x7) << 4), cvt(q1.x), cvt(q1.x >> 8), cvt(q1.y), cvt(q1.y >> 8));
    sts128(brow + (((4 * H + 3) ^ x7) << 4), cvt(q1.z), cvt(q1.z >> 8), cvt(q1.w), cvt(q1.w >> 8));
}

struct Tile {
    int g, mt, nt, r0, r1;
};
// tile t -> (group, m tile, n tile, rows); ts / gs: the group tables in shared memory
__device__ __forceinline__ Tile tile_of(const int32_t* ts, const int32_t* gs, int groups, int t, int nN) {
    Tile T;
    const int mi = t / nN;
    T.nt = t - mi * nN;
    int lo = 0, hi = groups;  // largest g with tile_start[g] <= mi
    while (hi - lo > 1) {
        const int mid = (lo + hi) >> 1;
        if (ts[mid] <= mi) lo = mid; else hi = mid;
    }
    T.g = lo;
    T.mt = mi - ts[lo];
    T.r0 = gs[lo] + T.mt * BM;
    T.r1 = min(T.r0 + BM, gs[lo + 1]);
    return T;
}

template <int MODE>
__global__ void __launch_bounds__(THREADS, 1) k_tgemm(const __grid_constant__ CUtensorMap tmA,
                                                      const __grid_constant__ CUtensorMap tmW0,
                                                      const __grid_constant__ CUtensorMap tmW1, const TgParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~static_cast<uintptr_t>(1023));
    uint64_t* a_full = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* a_empty = a_full + NA;
    uint64_t* b_full = a_empty + NA;
    uint64_t* b_empty = b_full + NB;
    uint64_t* r_full = b_empty + NB;
    uint64_t* r_empty = r_full + NR;
    uint64_t* acc_full = r_empty + NR;    // [2]
    uint64_t* acc_free = acc_full + 2;    // [2]
    uint32_t* s_tmem = reinterpret_cast<uint32_t*>(acc_free + 2);
    int32_t* s_ts = reinterpret_cast<int32_t*>(smem + OFF_TAB);
    int32_t* s_gs = s_ts + MAX_GROUPS + 1;
    const uint32_t sbase = smem_u32(smem);
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int ncol = MODE == 0 ? BN / 2 : BN;  // output columns per tile
    const int nN = p.N / ncol, nKS = p.K / KS, nSB = p.K / SB_K;
    const int total = __ldg(p.tile_start + p.groups) * nN;
    for (int i = tid; i <= p.groups; i += THREADS) {
        s_ts[i] = __ldg(p.tile_start + i);
        s_gs[i] = __ldg(p.grp_start + i);
    }

    if (tid == 0) {
        for (int s = 0; s < NA; ++s) {
            mbar_init(a_full + s, 1);
            mbar_init(a_empty + s, 1);
        }
        for (int s = 0; s < NB; ++s) {
            mbar_init(b_full + s, DQ_WARPS);
            mbar_init(b_empty + s, 1);
        }
        for (int s = 0; s < NR; ++s) {
            mbar_init(r_full + s, 1);
            mbar_init(r_empty + s, DQ_WARPS);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(acc_full + b, 1);
            mbar_init(acc_free + b, 4);
        }
        fence_mbar_init();
    }
    if (warp == WARP_MMA) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(s_tmem)),
                     "r"(TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *s_tmem;

    if (warp == WARP_TA) {
        // ---------------- activations ----------------
        if (lane == 0) {
            int step = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
                const Tile T = tile_of(s_ts, s_gs, p.groups, t, nN);
                for (int ks = 0; ks < nKS; ++ks, ++step) {
                    const int s = step % NA;
                    if (step >= NA && !(ok = mbar_wait(a_empty + s, ((step / NA) - 1) & 1, p.ctrl))) break;
                    mbar_arrive_expect_tx(a_full + s, A_BYTES);
                    tma_2d(sbase + OFF_A + s * A_BYTES, &tmA, ks * KS, T.r0, a_full + s);
                }
            }
            // copies still in flight (none unless a wait expired): let them land
            for (int i = max(0, step - NA); i < step; ++i) mbar_wait(a_full + i % NA, (i / NA) & 1, nullptr);
        }
    } else if (warp == WARP_TR) {
        // ---------------- raw weight super-blocks ----------------
        if (lane == 0) {
            int step = 0;
            bool ok = true;
            for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
                const Tile T = tile_of(s_ts, s_gs, p.groups, t, nN);
                for (int sb = 0; sb < nSB; ++sb, ++step) {
                    const int s = step % NR;
                    if (step >= NR && !(ok = mbar_wait(r_empty + s, ((step / NR) - 1) & 1, p.ctrl))) break;
                    const uint32_t dst = sbase + OFF_R + s * R_BYTES;
                    mbar_arrive_expect_tx(r_full + s, R_BYTES);
                    if (MODE == 0) {
                        const int row = T.g * p.group_rows + T.nt * (BN / 2);
                        tma_2d(dst, &tmW0, sb * SB_BYTES, row, r_full + s);
                        tma_2d(dst + (BN / 2) * SB_BYTES, &tmW1, sb * SB_BYTES, row, r_full + s);
                    } else {
                        tma_2d(dst, &tmW0, sb * SB_BYTES, T.g * p.group_rows + T.nt * BN, r_full + s);
                    }
                }
            }
            for (int i = max(0, step - NR); i < step; ++i) mbar_wait(r_full + i % NR, (i / NR) & 1, nullptr);
        }
    } else if (warp < WARP_MMA) {
        // ---------------- dequantisation ----------------
        const int i = tid - WARP_DQ * 32;  // 0..511
        const int r = i & 255, h = i >> 8;  // weight row of the tile, sub-block of the slice (warp-uniform)
        int rstep = 0, bstep = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < total; t += gridDim.x) {
            for (int sb = 0; ok && sb < nSB; ++sb, ++rstep) {
                const int rs = rstep % NR;
                if (!(ok = mbar_wait(r_full + rs, (rstep / NR) & 1, p.ctrl))) break;
                const uint32_t raw = sbase + OFF_R + rs * R_BYTES + r * SB_BYTES;
                for (int g = 0; g < SB_K / KS; ++g, ++bstep) {
                    const int bs = bstep % NB;
                    if (bstep >= NB && !(ok = mbar_wait(b_empty + bs, ((bstep / NB) - 1) & 1, p.ctrl))) break;
                    if (h == 0) dq_sub<0>(raw, g, sbase + OFF_B + bs * B_BYTES + r * 128, r);
                    else dq_sub<1>(raw, g, sbase + OFF_B + bs * B_BYTES + r * 128, r);
                    fence_async_smem();  // generic stores -> visible to the tensor core
                    __syncwarp();
                    if (lane == 0) mbar_arrive(b_full + bs);
                }
                __syncwarp();
                if (lane == 0) mbar_arrive(r_empty + rs);
            }
        }
    } else if (warp == WARP_MMA) {
        // ---------------- MMA issue ----------------
        int step = 0, ti = 0;
        bool ok = true;
        for (int t = blockIdx.x; ok && t < total; t += gridDim.x, ++ti) {
            const int buf = ti & 1;
            if (ti >= 2 && !(ok = mbar_wait(acc_free + buf, ((ti >> 1) - 1) & 1, p.ctrl))) break;
            tc_fence_after();
            for (int ks = 0; ks < nKS; ++ks, ++step) {
                const int as = step % NA, bs = step % NB;
                if (!(ok = mbar_wait(a_full + as, (step / NA) & 1, p.ctrl))) break;
                if (!(ok = mbar_wait(b_full + bs, (step / NB) & 1, p.ctrl))) break;
                tc_fence_after();
                if (lane == 0) {
                    const uint32_t sa = sbase + OFF_A + as * A_BYTES, sbb = sbase + OFF_B + bs * B_BYTES;
#pragma unroll
                    for (int kk = 0; kk < KS / 16; ++kk)
                        mma_f16(tmem + buf * BN, sdesc(sa + kk * 32), sdesc(sbb + kk * 32), (ks | kk) != 0);
                    mma_commit(a_empty + as);  // the slots are free once these MMAs have read them
                    mma_commit(b_empty + bs);
                }
                __syncwarp();
            }
            if (!ok) break;
            if (lane == 0) mma_commit(acc_full + buf);  // accumulators complete
            __syncwarp();
        }
        // the MMAs issued last must be done before TMEM is freed
        if (lane == 0 && step > 0) mbar_wait(a_empty + (step - 1) % NA, ((step - 1) / NA) & 1, nullptr);
        __syncwarp();
    } else {
        // ---------------- epilogue: TMEM -> global ----------------
        const int quarter = warp & 3;  // TMEM lanes 32*quarter .. +31 = tile rows
        int ti = 0;
        for (int t = blockIdx.x; t < total; t += gridDim.x, ++ti) {
            const Tile T = tile_of(s_ts, s_gs, p.groups, t, nN);
            const int buf = ti & 1;
            if (!mbar_wait(acc_full + buf, (ti >> 1) & 1, p.ctrl)) break;
            tc_fence_after();
            const int orow = T.r0 + 32 * quarter + lane;
            const uint32_t tl = tmem + buf * BN + (static_cast<uint32_t>(32 * quarter) << 16);
            const int drow = (p.out_rows && orow < T.r1) ? __ldg(p.out_rows + orow) : orow;
            __half* dst = p.out + static_cast<size_t>(drow) * p.N + T.nt * ncol;
            bool to_peer = false;
            if (MODE == 1 && p.sc.n_src > 0) {  // the rank the row came from, and its row there
                int src = 0;
                while (src + 1 < p.sc.n_src && drow >= p.sc.start[src + 1]) ++src;
                to_peer = drow >= p.sc.start[src] && drow < p.sc.start[p.sc.n_src];
                dst = p.sc.dst[src] + (static_cast<size_t>(p.sc.dst_row[src]) + (drow - p.sc.start[src])) * p.N +
                      T.nt * ncol;
            }
            for (int c0 = 0; c0 < ncol; c0 += 16) {
                uint32_t a[16];
                tmem_ld16(tl + c0, a);
                uint32_t o[8];
                if (MODE == 0) {
                    uint32_t u[16];
                    tmem_ld16(tl + BN / 2 + c0, u);
                    tmem_wait_ld();
                    float hv[16];
#pragma unroll
                    for (int k = 0; k < 16; ++k) {
                        const float g = __uint_as_float(a[k]);
                        // moe.cu:64 (fast exp/divide: the result is rounded to fp16 next)
                        hv[k] = __fdividef(g, 1.0f + __expf(-g)) * __uint_as_float(u[k]);
                    }
#pragma unroll
                    for (int c = 0; c < 2; ++c) {  // chunk element order for the down GEMM
                        o[4 * c] = h2_bits(__floats2half2_rn(hv[8 * c], hv[8 * c + 2]));
                        o[4 * c + 1] = h2_bits(__floats2half2_rn(hv[8 * c + 1], hv[8 * c + 3]));
                        o[4 * c + 2] = h2_bits(__floats2half2_rn(hv[8 * c + 4], hv[8 * c + 6]));
                        o[4 * c + 3] = h2_bits(__floats2half2_rn(hv[8 * c + 5], hv[8 * c + 7]));
                    }
                } else {
                    tmem_wait_ld();
#pragma unroll
                    for (int k = 0; k < 8; ++k)
                        o[k] = h2_bits(__floats2half2_rn(__uint_as_float(a[2 * k]), __uint_as_float(a[2 * k + 1])));
                }
                if (orow < T.r1 && (MODE == 1 && p.sc.n_src > 0 ? to_peer : drow < p.out_cap)) {
                    uint4* d4 = reinterpret_cast<uint4*>(dst + c0);
                    d4[0] = make_uint4(o[0], o[1], o[2], o[3]);
                    d4[1] = make_uint4(o[4], o[5], o[6], o[7]);
                }
            }
            if (MODE == 1 && p.sc.n_src > 0) __threadfence_system();  // peer stores performed before completion
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive(acc_free + buf);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == WARP_MMA) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(TMEM_COLS));
    }
}

}  // namespace tg

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
namespace {

PFN_cuTensorMapEncodeTiled_v12000 tmap_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            f = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 2-D tensor map of a row-major matrix: `inner` elements per row, `rows`
// rows, `stride` bytes between rows; boxes of box_inner x box_rows.
bool map_2d(CUtensorMap* m, const void* base, CUtensorMapDataType dt, uint64_t inner, uint64_t rows, uint64_t stride,
            uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle sw) {
    auto enc = tmap_encoder();
    if (!enc || (reinterpret_cast<uintptr_t>(base) & 15u) || (stride & 15u)) return false;
    const cuuint64_t dims[2] = {inner, rows};
    const cuuint64_t strides[1] = {stride};
    const cuuint32_t box[2] = {box_inner, box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, dt, 2, const_cast<void*>(base), dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, sw,
               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int tg_num_sms() {
    int dev = 0, sms = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    return sms;
}

}  // namespace

bool tgemm_supported(int wtype, int mode, int N, int K) {
    return wtype == T_Q4_K && K % tg::SB_K == 0 && N % (mode == 0 ? tg::BN / 2 : tg::BN) == 0 &&
           tmap_encoder() != nullptr;
}
static_assert(tg::smem_bytes() <= 227 * 1024, "k_tgemm shared memory");

cudaError_t launch_tgemm(const TgArgs& a, cudaStream_t s) {
    if (a.p.groups < 1 || a.p.groups > tg::MAX_GROUPS) return cudaErrorInvalidValue;
    CUtensorMap mA, mW0, mW1;
    const uint64_t wrow = static_cast<uint64_t>(a.K / tg::SB_K) * tg::SB_BYTES;
    const uint32_t wbox = a.mode == 0 ? tg::BN / 2 : tg::BN;
    if (!map_2d(&mA, a.a16, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, a.K, a.a_rows, 2ull * a.K, tg::KS, tg::BM,
                CU_TENSOR_MAP_SWIZZLE_128B) ||
        !map_2d(&mW0, a.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, wrow, static_cast<uint64_t>(a.p.groups) * a.p.group_rows,
                wrow, tg::SB_BYTES, wbox, CU_TENSOR_MAP_SWIZZLE_NONE) ||
        !map_2d(&mW1, a.mode == 0 ? a.w1 : a.w0, CU_TENSOR_MAP_DATA_TYPE_UINT8, wrow,
                static_cast<uint64_t>(a.p.groups) * a.p.group_rows, wrow, tg::SB_BYTES, wbox,
                CU_TENSOR_MAP_SWIZZLE_NONE))
        return cudaErrorInvalidValue;
    auto kern = a.mode == 0 ? tg::k_tgemm<0> : tg::k_tgemm<1>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         static_cast<int>(tg::smem_bytes()));
    if (e != cudaSuccess) return e;
    kern<<<tg_num_sms(), tg::THREADS, tg::smem_bytes(), s>>>(mA, mW0, mW1, a.p);
    return cudaGetLastError();
}

// Rows of `src` gathered into `dst` in position order: dst[i] = src[idx[i]],
// i < n_rows[0] (a device count); one warp per row, 16 bytes per lane.
__global__ void __launch_bounds__(256) k_gather_rows(const __half* __restrict__ src, const int32_t* __restrict__ idx,
                                                     const int32_t* __restrict__ n_rows, int cap, int d,
                                                     __half* __restrict__ dst) {
    const int n = min(__ldg(n_rows), cap);
    const int chunks = d / 8;
    for (int row = blockIdx.x * 8 + (threadIdx.x >> 5); row < n; row += gridDim.x * 8) {
        const uint4* s4 = reinterpret_cast<const uint4*>(src + static_cast<size_t>(__ldg(idx + row)) * d);
        uint4* d4 = reinterpret_cast<uint4*>(dst + static_cast<size_t>(row) * d);
        for (int c = threadIdx.x & 31; c < chunks; c += 32) d4[c] = __ldg(s4 + c);
    }
}

cudaError_t launch_gather_rows(const __half* src, const int32_t* idx, const int32_t* n_rows, int cap, int d,
                               __half* dst, cudaStream_t s) {
    k_gather_rows<<<4 * tg_num_sms(), 256, 0, s>>>(src, idx, n_rows, cap, d, dst);
    return cudaGetLastError();
}

}  // namespace qmoe
