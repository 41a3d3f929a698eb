// Decode-path kernels of the MoE block (T <= kDecodeMaxT tokens per launch),
// three launches per block chained with programmatic dependent launch (PDL):
// every kernel fetches the weights that do not depend on the previous
// kernel's output before it waits for that output.
//
//   k_router   [prologue: router rows into registers]  optional fused
//              pre-MoE RMSNorm (src/cuda/ops.cu:25-65, same arithmetic),
//              router logits in the reference's exact F32 reduction order
//              (src/cuda/matmul_q4.cu:140-167), the shared-expert gate logit,
//              the block input and its 24-bit planes; the last CTA selects
//              the experts (src/cuda/moe.cu:7-52), checks the result on the
//              device (src/layer_moe.cpp:114-124) and writes the stable
//              token->expert permutation as a packed schedule.
//   k_gateup   [prologue: shared-expert gate/up rows -> shared memory (TMA)]
//              routed gate/up rows of every active expert, staged with 1-D
//              bulk copies straight from the GGUF payload, dp4a dot products
//              against 24-bit planes of the block input (written once by the
//              router), silu(g)*u (moe.cu:61-67), and the 24-bit planes of
//              each 32-row block of silu(g)*u for the down kernel.
//   k_down     [prologue: shared-expert and routed down rows -> shared memory]
//              planes of silu(g)*u (one bulk copy), down products, then the
//              combine in selection order j = 0..k-1 (moe.cu:76-81) and the
//              sigmoid-gated shared expert (moe.cu:90-96), optional residual.
#include <algorithm>
#include "qmoe_dev.cuh"
#include "qmoe_units.cuh"
#include "qmoe_route.cuh"
#include "qmoe_internal.h"

namespace qmoe {

constexpr unsigned FULL = 0xffffffffu;

// Phase timestamp (one thread per CTA) when a trace buffer is registered:
// %globaltimer ns, or with QMOE_TRACE_CLOCK the SM's cycle counter (exact
// durations inside one CTA; not comparable across SMs).
#ifdef QMOE_TRACE_CLOCK
#define QMOE_TRACE_NOW() static_cast<uint64_t>(clock64())
#else
#define QMOE_TRACE_NOW() gtimer()
#endif
#define QMOE_TRACE(P, kind, ev)                                                                          \
    do {                                                                                                 \
        if ((P).trace && blockIdx.x < kTraceCtas)                                                        \
            (P).trace[((kind) * kTraceCtas + blockIdx.x) * kTraceEvents + (ev)] = QMOE_TRACE_NOW();     \
    } while (0)

// Reads every 16-byte word of a kernel parameter block once, from warp 0 of
// the CTA, at the start of the kernel: later reads of any field then hit the
// SM's constant cache instead of missing on the critical path.  The loads are
// kept by an empty asm that consumes their combination.
template <typename T>
__device__ __forceinline__ void touch_params(const T& p) {
    static_assert(sizeof(T) % 4 == 0, "parameter block size");
    constexpr int W = static_cast<int>(sizeof(T) / 4);
    const uint32_t* w = reinterpret_cast<const uint32_t*>(&p);
    uint32_t acc = 0;
    for (int i = static_cast<int>(threadIdx.x) * 16; i < W; i += 32 * 16) acc ^= w[i];
    asm volatile("" ::"r"(acc));
}

// ---------------------------------------------------------------------------
// Router
// ---------------------------------------------------------------------------
constexpr int RT_WARPS = 4;

template <int CH>
__device__ __forceinline__ void load_router_row(float4 (&w)[CH][2], const uint8_t* row, int type, int lane) {
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int k0 = 256 * i + 128 * hh + 4 * lane;
            if (type == T_F32) {
                w[i][hh] = __ldg(reinterpret_cast<const float4*>(row) + (k0 >> 2));
            } else {
                uint2 v = __ldg(reinterpret_cast<const uint2*>(row + 2 * k0));
                if (type == T_F16) {
                    w[i][hh] = make_float4(h2f_bits(v.x), h2f_bits(v.x >> 16), h2f_bits(v.y), h2f_bits(v.y >> 16));
                } else {  // BF16
                    w[i][hh] = make_float4(__uint_as_float(v.x << 16), __uint_as_float(v.x & 0xFFFF0000u),
                                           __uint_as_float(v.y << 16), __uint_as_float(v.y & 0xFFFF0000u));
                }
            }
        }
}

// Activations produced by the previous kernel: read through L2 (ld.global.cg).
__device__ __forceinline__ float4 ld_act4(const float* p) { return __ldcg(reinterpret_cast<const float4*>(p)); }

// Dot product of two register-resident vectors in the router lane layout
// (lane L holds elements 256i + 128h + 4L + c) with the reference's order.
template <int CH>
__device__ __forceinline__ float reg_dot(const float4 (&w)[CH][2], const float4 (&x)[CH][2]) {
    float acc[2][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[hh][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            acc[hh][0] = __fmaf_rn(w[i][hh].x, x[i][hh].x, acc[hh][0]);
            acc[hh][1] = __fmaf_rn(w[i][hh].y, x[i][hh].y, acc[hh][1]);
            acc[hh][2] = __fmaf_rn(w[i][hh].z, x[i][hh].z, acc[hh][2]);
            acc[hh][3] = __fmaf_rn(w[i][hh].w, x[i][hh].w, acc[hh][3]);
        }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float a = acc[hh][c];
            a = __fadd_rn(a, __shfl_down_sync(FULL, a, 4));
            a = __fadd_rn(a, __shfl_down_sync(FULL, a, 2));
            a = __fadd_rn(a, __shfl_down_sync(FULL, a, 1));
            acc[hh][c] = a;
        }
    const float s0 = __fadd_rn(__fadd_rn(acc[0][0], acc[0][2]), __fadd_rn(acc[0][1], acc[0][3]));
    const float s1 = __fadd_rn(__fadd_rn(acc[1][0], acc[1][2]), __fadd_rn(acc[1][1], acc[1][3]));
    float q[8];
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
        q[w4] = __shfl_sync(FULL, s0, 8 * w4);
        q[4 + w4] = __shfl_sync(FULL, s1, 8 * w4);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __fadd_rn(__fadd_rn(q[i], 0.0f), 0.0f);
    return __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                     __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
}

// The block input of one token in registers: x, or with the fused norm
// (ops.cu:33-64) (x * rsqrt(mean(x^2) + eps)) * weight -- the sum of squares
// has exactly the GEMV's thread/shuffle structure, so reg_dot(x, x) is it.
template <int CH>
__device__ __forceinline__ void load_input(float4 (&xr)[CH][2], const DecodeParams& P, const float* x,
                                           const float* s_nw, int lane) {
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) xr[i][hh] = ld_act4(x + 256 * i + 128 * hh + 4 * lane);
    if (P.prenorm) {
        const float ss = reg_dot<CH>(xr, xr);
        const float sc = rsqrtf(ss / static_cast<float>(P.d) + P.eps);
#pragma unroll
        for (int i = 0; i < CH; ++i)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
                const float4 nv = *reinterpret_cast<const float4*>(s_nw + 256 * i + 128 * hh + 4 * lane);
                xr[i][hh].x = __fmul_rn(__fmul_rn(xr[i][hh].x, sc), nv.x);
                xr[i][hh].y = __fmul_rn(__fmul_rn(xr[i][hh].y, sc), nv.y);
                xr[i][hh].z = __fmul_rn(__fmul_rn(xr[i][hh].z, sc), nv.z);
                xr[i][hh].w = __fmul_rn(__fmul_rn(xr[i][hh].w, sc), nv.w);
            }
    }
}

__device__ __forceinline__ int router_esize(int type) { return type == T_F32 ? 4 : 2; }

// Top-k + softmax + validation for every token (select_token, one warp per
// token), then the permutation and the packed schedule.  Runs in the router's
// last CTA, or in every CTA of the fused expert kernel.
//
// Dispatch: a token picks an expert at most once, so each expert's pairs are
// described by a token bitmask (T <= 32).  One block-wide exclusive scan of
// (pair count, active flag) per expert gives the expert offsets and the
// source index of every active expert; a pair's permuted position is its
// expert's offset plus the number of earlier tokens in the mask -- the stable
// (expert, pair) order of a counting sort.
//
// Threads 0 .. 32*RT_WARPS-1 of the calling CTA take part; `bar_id` names the
// barrier they use among themselves.  The schedule goes to `sched` (global
// workspace or shared memory), the routing weights also to `w_out` when given.
// With `publish`, the workspace outputs (top-k ids and weights, offsets,
// permutation, active list, counters) and the error flags are written too.
__device__ void topk_and_schedule(const DecodeParams& P, int* sched, float* w_out, bool publish, int bar_id) {
    constexpr int MP = kDecodeMaxT * kMaxTopK;
    static_assert(kDecodeMaxT <= 32, "token masks are 32-bit");
    static_assert(RT_WARPS * 32 * 2 >= kMaxExperts, "two experts per thread in the scan");
    __shared__ uint32_t s_mask[kMaxExperts];
    __shared__ int s_off[kMaxExperts];
    __shared__ int s_idx[MP];
    __shared__ uint32_t s_wsum[RT_WARPS];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int E = P.E, k = P.k, LS = E + 1;
    const int NP = P.T * k;
    auto bar = [&]() { asm volatile("bar.sync %0, %1;" ::"r"(bar_id), "r"(RT_WARPS * 32) : "memory"); };
    for (int e = threadIdx.x; e < kMaxExperts; e += RT_WARPS * 32) s_mask[e] = 0u;
    bar();

    for (int t = warp; t < P.T; t += RT_WARPS) {
        int my_idx;
        float wj;
        uint32_t flag;
        select_token(P.logits + t * LS, E, k, lane, my_idx, wj, flag);
        if (publish && flag && lane == 0) {
            raise_error(P.ctrl, flag);
            atomicMin(P.ctrl + CTRL_ERR_TOKEN, static_cast<uint32_t>(t));
        }
        if (lane < k) {
            const int oi = flag ? -1 : my_idx;
            const float ow = flag ? __uint_as_float(0x7FC00000u) : wj;
            s_idx[t * k + lane] = oi;
            if (oi >= 0) atomicOr(s_mask + oi, 1u << t);
            if (w_out) w_out[t * k + lane] = ow;
            if (publish) {
                P.topk_idx[t * k + lane] = oi;
                P.topk_w[t * k + lane] = ow;
                if (P.out_idx) P.out_idx[t * k + lane] = oi;
                if (P.out_w) P.out_w[t * k + lane] = ow;
            }
        }
    }
    bar();

    // exclusive scan over experts of (pairs << 16 | active), two experts per thread
    const int e0 = 2 * threadIdx.x;
    const uint32_t m0 = e0 < E ? s_mask[e0] : 0u, m1 = e0 + 1 < E ? s_mask[e0 + 1] : 0u;
    const uint32_t v0 = (static_cast<uint32_t>(__popc(m0)) << 16) | (m0 ? 1u : 0u);
    const uint32_t v1 = (static_cast<uint32_t>(__popc(m1)) << 16) | (m1 ? 1u : 0u);
    uint32_t inc = v0 + v1;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t y = __shfl_up_sync(FULL, inc, o);
        if (lane >= o) inc += y;
    }
    if (lane == 31) s_wsum[warp] = inc;
    bar();
    uint32_t base = 0, total = 0;
    for (int w = 0; w < RT_WARPS; ++w) {
        const uint32_t ws = s_wsum[w];
        base += w < warp ? ws : 0u;
        total += ws;
    }
    const uint32_t ex0 = base + inc - v0 - v1, ex1 = ex0 + v0;
    const int npairs = static_cast<int>(total >> 16), nact = static_cast<int>(total & 0xFFFFu);
    const int poff = sched_perm_off(P.T, k, E), toff = sched_tok_off(P.T, k, E);
#pragma unroll
    for (int h = 0; h < 2; ++h) {
        const int e = e0 + h;
        const uint32_t ex = h ? ex1 : ex0, m = h ? m1 : m0;
        if (e < E) {
            s_off[e] = static_cast<int>(ex >> 16);
            if (publish) P.offsets[e] = static_cast<int>(ex >> 16);
            if (m) {
                const int s2 = static_cast<int>(ex & 0xFFFFu);
                if (publish) P.active[s2] = e;
                sched[SCHED_HDR + 3 * s2] = e;
                sched[SCHED_HDR + 3 * s2 + 1] = static_cast<int>(ex >> 16);
                sched[SCHED_HDR + 3 * s2 + 2] = __popc(m);
            }
        }
    }
    if (threadIdx.x == 0) {
        sched[0] = nact;
        sched[1] = npairs;
        if (publish) {
            P.offsets[E] = npairs;
            P.ctrl[CTRL_N_ACTIVE] = static_cast<uint32_t>(nact);
            P.ctrl[CTRL_N_PAIRS] = static_cast<uint32_t>(npairs);
        }
    }
    bar();
    for (int p = threadIdx.x; p < NP; p += RT_WARPS * 32) {
        const int e = s_idx[p];
        int rank = -1;
        if (e >= 0) {
            const int t = p / k;
            rank = s_off[e] + __popc(s_mask[e] & ((1u << t) - 1u));
            if (publish) P.perm[rank] = p;
            sched[poff + rank] = p;
            sched[toff + rank] = t;
        }
        if (publish) P.inv_perm[p] = rank;
    }
}

template <int CH>
__global__ void __launch_bounds__(RT_WARPS * 32) k_router(const __grid_constant__ DecodeParams P) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp == 0) touch_params(P);
    const int gw = blockIdx.x * RT_WARPS + warp;
    const int nrows = P.E + (P.has_shared ? 1 : 0);
    const int LS = P.E + 1;

    if (threadIdx.x == 0) QMOE_TRACE(P, 0, 0);
    // prologue: this warp's router row does not depend on the previous kernel
    float4 w[CH][2];
    const bool has_row = gw < nrows;
    const bool writer = gw < P.T * CH;  // publishes 256 elements of the block input
    if (has_row) {
        const int type = gw < P.E ? P.router_type : P.sgate_type;
        const uint8_t* row = gw < P.E ? P.router + static_cast<size_t>(gw) * P.d * router_esize(type) : P.sgate_inp;
        load_router_row<CH>(w, row, type, lane);
    }
    // the norm weights (shared memory) and this row's bias are weights too
    __shared__ __align__(16) float s_nw[kMaxNormDim];
    if (P.prenorm)
        for (int i = threadIdx.x; i < P.d / 4; i += blockDim.x)
            reinterpret_cast<float4*>(s_nw)[i] = __ldg(reinterpret_cast<const float4*>(P.norm_w) + i);
    const float bias_v = (has_row && gw < P.E && P.bias) ? __ldg(P.bias + gw) : 0.0f;
    pdl_trigger();
    if (threadIdx.x == 0) pdl_wait();  // one waiter; the CTA barrier releases the rest
    __syncthreads();
    if (threadIdx.x == 0) QMOE_TRACE(P, 0, 1);

    if (has_row || writer) {
        for (int t = 0; t < P.T; ++t) {
            float4 xr[CH][2];
            load_input<CH>(xr, P, P.x + static_cast<size_t>(t) * P.d, s_nw, lane);
            if (has_row) {
                float v = reg_dot<CH>(w, xr);
                if (lane == 0) {
                    if (gw < P.E && P.bias) v = __fadd_rn(v, bias_v);
                    P.logits[t * LS + gw] = v;
                }
            }
            if (writer && gw / CH == t) {
                const int i = gw % CH;
#pragma unroll
                for (int ii = 0; ii < CH; ++ii)
                    if (ii == i)
#pragma unroll
                        for (int hh = 0; hh < 2; ++hh) {
                            const int e0 = 256 * ii + 128 * hh + 4 * lane;
                            *reinterpret_cast<float4*>(P.xnorm + static_cast<size_t>(t) * P.d + e0) = xr[ii][hh];
                        }
            }
        }
    }

    if (!P.route_in_router) {  // the fused expert kernel selects the experts itself
        if (threadIdx.x == 0) QMOE_TRACE(P, 0, 2);
        return;
    }
    // last CTA to arrive selects the experts.  The CTA barrier orders every
    // thread's logit writes before thread 0's release; the acquire side of the
    // same atomic makes all CTAs' logits visible to the last one.
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        QMOE_TRACE(P, 0, 2);
        unsigned old;
        asm volatile("atom.add.acq_rel.gpu.u32 %0, [%1], %2;" : "=r"(old) : "l"(P.ctrl + CTRL_ARRIVE), "r"(1u)
                     : "memory");
        s_last = (old == gridDim.x - 1);
        QMOE_TRACE(P, 0, 3);
    }
    __syncthreads();
    if (!s_last) return;
    topk_and_schedule(P, P.sched, nullptr, true, 0);
    if (threadIdx.x == 0) {
        P.ctrl[CTRL_ARRIVE] = 0;
        QMOE_TRACE(P, 0, 4);
    }
}

// ---------------------------------------------------------------------------
// Expert kernels: shared pieces
// ---------------------------------------------------------------------------
constexpr int NCW = 8;                      // consumer warps
constexpr int XK_THREADS = (NCW + 1) * 32;  // + one producer warp
constexpr int SCHED_SMEM_WORDS = SCHED_HDR + 3 * kDecodeMaxT * kMaxTopK + 2 * kDecodeMaxT * kMaxTopK;

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float s = g / (1.0f + expf(-g));  // moe.cu:64
    return s * u;
}

__device__ __forceinline__ XPlanesView planes_view(uint32_t base, int K) {
    XPlanesView v;
    v.p0 = base;
    v.p1 = base + static_cast<uint32_t>(K);
    v.p2 = base + 2u * static_cast<uint32_t>(K);
    v.meta = base + 3u * static_cast<uint32_t>(K);
    return v;
}

struct StagePlan {
    const uint8_t* lo;
    uint32_t tx;
};

// Plans a copy of [src, src+bytes) into dst: the 16-byte aligned superset is
// bulk-copied (clipped to `limit`, the end of the source allocation); the
// few bytes past the last full chunk, if any, are copied here with plain
// loads.  The row data then starts at dst + (src & 15).
__device__ __forceinline__ StagePlan plan_stage(uint8_t* dst, const uint8_t* src, uint64_t bytes, const uint8_t* limit) {
    StagePlan sp;
    const uintptr_t s = reinterpret_cast<uintptr_t>(src);
    const uintptr_t lo = s & ~static_cast<uintptr_t>(15);
    const uintptr_t hi = (s + bytes + 15) & ~static_cast<uintptr_t>(15);
    const uintptr_t lim = reinterpret_cast<uintptr_t>(limit);
    const uintptr_t hi_full = hi <= lim ? hi : (lim & ~static_cast<uintptr_t>(15));
    sp.lo = reinterpret_cast<const uint8_t*>(lo);
    sp.tx = hi_full > lo ? static_cast<uint32_t>(hi_full - lo) : 0u;
    for (uintptr_t a = (hi_full > lo ? hi_full : lo); a < s + bytes; ++a)
        dst[a - lo] = *reinterpret_cast<const uint8_t*>(a);
    return sp;
}

__device__ __forceinline__ void load_sched(int* s_sched, const DecodeParams& P) {
    const int words = sched_words(P.T, P.k, P.E);
    for (int i = threadIdx.x; i < words; i += blockDim.x) s_sched[i] = __ldcg(P.sched + i);
}

// The same quantisation of one 32-block, written to global memory.
__device__ __forceinline__ void xq_block32_global(float v, uint8_t* base, int K, int e0, int lane) {
    const uint32_t ab = __reduce_max_sync(FULL, __float_as_uint(v) & 0x7FFFFFFFu);
    float s16 = v;
#pragma unroll
    for (int o = 8; o; o >>= 1) s16 += __shfl_xor_sync(FULL, s16, o);
    const bool bad = ab >= 0x7F800000u;
    const uint32_t eb = ab >> 23;
    int sh = eb == 0 ? 126 : 21 - (static_cast<int>(eb) - 127);
    sh = sh > 126 ? 126 : sh;
    const float mul = __uint_as_float(static_cast<uint32_t>(sh + 127) << 23);
    float scale = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
    const int X = bad ? 0 : __float2int_rn(v * mul);
    if (bad) scale = __uint_as_float(0x7FC00000u);
    const uint32_t o = pswz(static_cast<uint32_t>(e0 + lane));
    base[o] = static_cast<uint8_t>(X & 255);
    base[K + o] = static_cast<uint8_t>((X >> 8) & 255);
    base[2 * K + o] = static_cast<uint8_t>((X >> 16) & 255);
    if ((lane & 15) == 0) reinterpret_cast<float2*>(base + 3 * K)[(e0 >> 4) + (lane >> 4)] = make_float2(scale, s16);
}

__device__ __forceinline__ int ilog2(int v) { return 31 - __clz(v); }

// Block input x_in (F32, written by the router) of every token -> 24-bit
// planes in shared memory (token stride xq_stride).  Each warp quantises
// 128-element chunks (lanes 8m..8m+7 hold one 32-block); every load is issued
// before the first plane is written.  NTHREADS is a multiple of 32 and
// T * d / 4 a multiple of 32, so each chunk test is warp-uniform.  Two chunks
// per thread are unrolled (all of them for one token at d = 2048): this code
// runs cold while the routing warps run, and every further inlined copy of
// the plane writer takes instruction fetches from the routing.
template <int NTHREADS>
__device__ __forceinline__ void x_planes_smem(uint8_t* xs, const DecodeParams& P, int tid) {
    const int lq = ilog2(P.d) - 2;  // float4s per token = 2^lq
    const int nv = P.T << lq;
    const int lane = tid & 31;
    constexpr int J = 2;
    float4 v[J];
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int g = tid + j * NTHREADS;
        if (g < nv) v[j] = __ldcg(reinterpret_cast<const float4*>(P.xnorm) + g);
    }
#pragma unroll
    for (int j = 0; j < J; ++j) {
        const int g = tid + j * NTHREADS;
        if (g < nv) {
            const int t = g >> lq;
            write_planes4(v[j], xs + static_cast<size_t>(t) * P.xq_stride, P.d, (g - (t << lq)) * 4, lane);
        }
    }
    for (int g = tid + J * NTHREADS; g < nv; g += NTHREADS) {
        const int t = g >> lq;
        write_planes4(__ldcg(reinterpret_cast<const float4*>(P.xnorm) + g), xs + static_cast<size_t>(t) * P.xq_stride,
                      P.d, (g - (t << lq)) * 4, lane);
    }
}

// ---------------------------------------------------------------------------
// Expert gate/up
//
// Work is cut into items of 32 consecutive rows of one source (the shared
// expert's Fs/32 items first, then F/32 items per active expert): CTA c takes
// items c, c + grid, ...  At T = 1 with Qwen3.5-35B shapes that is 16 + 128
// items, one per SM.  An item's 32 results per token form one 32-block of
// silu(g)*u, which the CTA quantises into the 24-bit planes the down kernel
// reads -- each block exactly once.  All index arithmetic in the loops is
// shifts and running counters (row, unit and item counts are powers of two).
// ---------------------------------------------------------------------------
constexpr int GU_NCW = 16;
constexpr int GU_THREADS = (GU_NCW + 1) * 32;
constexpr int ITEM_ROWS = 32;


template <int TR, int TS>
__global__ void __launch_bounds__(GU_THREADS, 1) k_gateup(DecodeParams P, int nst, uint32_t half_bytes, int dn_rows) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = P.d;
    const int lgU = ilog2(d >> 6), U = 1 << lgU;   // units (64 elements) per row
    const int lgR = 5 - lgU;                        // rows per warp step = 32 / U
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + 8;
    int* s_sched = reinterpret_cast<int*>(smem + 256);
    uint8_t* xs = reinterpret_cast<uint8_t*>(s_sched) + align_up(SCHED_SMEM_WORDS * 4, 128);
    const uint32_t xs_bytes = static_cast<uint32_t>(P.xq_stride) * static_cast<uint32_t>(P.T);
    float* hb = reinterpret_cast<float*>(xs + align_up(xs_bytes, 128));
    uint8_t* stages = reinterpret_cast<uint8_t*>(hb) + align_up(static_cast<size_t>(ITEM_ROWS) * P.T * 4, 128);
    const uint64_t rbg = row_bytes(TR, d), rbs = row_bytes(TS, d);
    const int nb_sh = P.has_shared ? P.Fs / ITEM_ROWS : 0;
    const int lgF = ilog2(P.F / ITEM_ROWS);         // items per routed expert = 2^lgF
    const int G = gridDim.x, c = blockIdx.x;

    if (threadIdx.x == 0) {
        QMOE_TRACE(P, 1, 0);
        for (int i = 0; i < nst; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, GU_NCW); }
        fence_mbar_init();
    }
    __syncthreads();
    auto issue = [&](int slot, bool shared_src, int expert, int r0) {
        const uint64_t rb = shared_src ? rbs : rbg;
        const uint8_t* gsrc = shared_src ? P.sgate.p + r0 * rbs : P.gate.p + (static_cast<uint64_t>(expert) * P.F + r0) * rbg;
        const uint8_t* usrc = shared_src ? P.sup.p + r0 * rbs : P.up.p + (static_cast<uint64_t>(expert) * P.F + r0) * rbg;
        uint8_t* dg = stages + static_cast<size_t>(slot) * 2 * half_bytes;
        uint8_t* du = dg + half_bytes;
        const StagePlan pg = plan_stage(dg, gsrc, ITEM_ROWS * rb, shared_src ? P.sgate.end : P.gate.end);
        const StagePlan pu = plan_stage(du, usrc, ITEM_ROWS * rb, shared_src ? P.sup.end : P.up.end);
        mbar_arrive_expect_tx(full + slot, pg.tx + pu.tx);
        if (pg.tx) bulk_g2s(dg, pg.lo, pg.tx, full + slot, P.ctrl);
        if (pu.tx) bulk_g2s(du, pu.lo, pu.tx, full + slot, P.ctrl);
    };
    // prologue: a shared-expert item does not depend on the routing
    if (warp == GU_NCW && lane == 0 && c < nb_sh) issue(0, true, -1, c * ITEM_ROWS);
    if (threadIdx.x == 0) pdl_wait();  // the router has finished: schedule and block input are valid
    __syncthreads();
    if (threadIdx.x == 0) QMOE_TRACE(P, 1, 1);
    load_sched(s_sched, P);
    x_planes_smem<GU_THREADS>(xs, P, threadIdx.x);
    __syncthreads();
    const int nact = s_sched[0];
    const int* s_perm = s_sched + sched_perm_off(P.T, P.k, P.E);
    const int* s_tok = s_sched + sched_tok_off(P.T, P.k, P.E);
    const int nitems = nb_sh + (nact << lgF);
    const int ni = c < nitems ? (nitems - 1 - c) / G + 1 : 0;
    if (threadIdx.x == 0) QMOE_TRACE(P, 1, 2);
    pdl_trigger();  // the down kernel may start its prologue (routing is final)

    if (warp == GU_NCW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            // the down kernel's CTA c reads rows [c*dn_rows, ...) of every
            // active expert's down matrix: warm L2 with them now
            const int r0 = c * dn_rows, nr = min(dn_rows, P.d - r0);
            if (nr > 0) {
                const uint64_t rbd = row_bytes(P.down.type, P.F), rbsd = row_bytes(P.sdown.type, P.Fs);
                for (int s2 = 0; s2 <= nact; ++s2) {
                    const uint8_t* src = s2 < nact ? P.down.p + (static_cast<uint64_t>(s_sched[SCHED_HDR + 3 * s2]) * P.d + r0) * rbd
                                                   : P.sdown.p + static_cast<uint64_t>(r0) * rbsd;
                    if (s2 == nact && !P.has_shared) break;
                    const uint64_t nb = s2 < nact ? nr * rbd : nr * rbsd;
                    const uintptr_t lo = reinterpret_cast<uintptr_t>(src) & ~static_cast<uintptr_t>(15);
                    const uintptr_t hi = (reinterpret_cast<uintptr_t>(src) + nb) & ~static_cast<uintptr_t>(15);
                    if (hi > lo) prefetch_l2(reinterpret_cast<const void*>(lo), static_cast<uint32_t>(hi - lo));
                }
            }
            int i = c, slot = 0, round = 0;
            for (int kk = 0; kk < ni; ++kk, i += G) {
                if (kk > 0 || i >= nb_sh) {  // item 0 of a shared-expert CTA was issued in the prologue
                    if (round > 0) mbar_wait(empty + slot, (round - 1) & 1, P.ctrl);
                    if (i < nb_sh) {
                        issue(slot, true, -1, i * ITEM_ROWS);
                    } else {
                        const int j = i - nb_sh;
                        issue(slot, false, s_sched[SCHED_HDR + 3 * (j >> lgF)], (j & ((1 << lgF) - 1)) * ITEM_ROWS);
                    }
                }
                if (++slot == nst) { slot = 0; ++round; }
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    if (threadIdx.x == 0) QMOE_TRACE(P, 1, 3);
    const int ul = lane & (U - 1), rsub = lane >> lgU;
    const int u_r = unit_of_lane<TR>(ul, lgU), u_s = unit_of_lane<TS>(ul, lgU);
    const int lgS = 5 - lgR;  // steps per item = 32 / rows-per-step
    XU xr;
    int cur_key = -1;
    int i = c, slot = 0, round = 0;
    for (int kk = 0; kk < ni; ++kk, i += G) {
        const bool routed = i >= nb_sh;
        int bb, expert = -1, pair0 = 0, ntok = P.T;
        if (routed) {
            const int j = i - nb_sh, s2 = j >> lgF;
            bb = j & ((1 << lgF) - 1);
            expert = s_sched[SCHED_HDR + 3 * s2];
            pair0 = s_sched[SCHED_HDR + 3 * s2 + 1];
            ntok = s_sched[SCHED_HDR + 3 * s2 + 2];
        } else {
            bb = i;
        }
        const int r0 = bb * ITEM_ROWS;
        mbar_wait(full + slot, round & 1, P.ctrl);
        if (threadIdx.x == 0 && kk == 0) QMOE_TRACE(P, 1, 4);
        uint32_t dg = smem_u32(stages) + static_cast<uint32_t>(slot) * 2u * half_bytes;
        uint32_t du = dg + half_bytes;
        {
            const uintptr_t gsrc = routed ? reinterpret_cast<uintptr_t>(P.gate.p) + (static_cast<uint64_t>(expert) * P.F + r0) * rbg
                                          : reinterpret_cast<uintptr_t>(P.sgate.p) + static_cast<uint64_t>(r0) * rbs;
            const uintptr_t usrc = routed ? reinterpret_cast<uintptr_t>(P.up.p) + (static_cast<uint64_t>(expert) * P.F + r0) * rbg
                                          : reinterpret_cast<uintptr_t>(P.sup.p) + static_cast<uint64_t>(r0) * rbs;
            dg += static_cast<uint32_t>(gsrc & 15u);
            du += static_cast<uint32_t>(usrc & 15u);
        }
        const uint32_t rb = static_cast<uint32_t>(routed ? rbg : rbs);
        const int ntask = ntok << lgS;
        for (int tau = warp; tau < ntask; tau += GU_NCW) {
            const int ti = tau >> lgS, st = tau & ((1 << lgS) - 1);
            const int tok = routed ? s_tok[pair0 + ti] : ti;
            const int key = (tok << 1) | (routed ? 1 : 0);
            if (key != cur_key) {
                const XPlanesView xv = planes_view(smem_u32(xs) + static_cast<uint32_t>(tok) * static_cast<uint32_t>(P.xq_stride), d);
                if (routed) load_xu<TR>(xr, xv, u_r); else load_xu<TS>(xr, xv, u_s);
                cur_key = key;
            }
            const int rl = (st << lgR) + rsub;
            float g, up;
            if (routed) {
                g = unit_dot_t<TR>(dg + static_cast<uint32_t>(rl) * rb, u_r, xr);
                up = unit_dot_t<TR>(du + static_cast<uint32_t>(rl) * rb, u_r, xr);
            } else {
                g = unit_dot_t<TS>(dg + static_cast<uint32_t>(rl) * rb, u_s, xr);
                up = unit_dot_t<TS>(du + static_cast<uint32_t>(rl) * rb, u_s, xr);
            }
            for (int o = U >> 1; o; o >>= 1) {
                g += __shfl_xor_sync(FULL, g, o);
                up += __shfl_xor_sync(FULL, up, o);
            }
            if (ul == 0) stsf(smem_u32(hb) + 4u * static_cast<uint32_t>(rl * P.T + ti), silu_mul(g, up));
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GU_NCW * 32) : "memory");
        if (threadIdx.x == 0 && kk == 0) QMOE_TRACE(P, 1, 5);
        // the item's 32-blocks of silu(g)*u: F32 copy and 24-bit planes
        for (int ti = warp; ti < ntok; ti += GU_NCW) {
            const int vid = routed ? s_perm[pair0 + ti] : P.T * P.k + ti;
            const float v = ldsf(smem_u32(hb) + 4u * static_cast<uint32_t>(lane * P.T + ti));
            P.hidden[static_cast<size_t>(vid) * P.H + r0 + lane] = v;
            xq_block32_global(v, P.hq + static_cast<size_t>(vid) * P.hq_stride, P.H, r0, lane);
        }
        asm volatile("bar.sync 1, %0;" ::"r"(GU_NCW * 32) : "memory");
        if (lane == 0) mbar_arrive(empty + slot);
        if (++slot == nst) { slot = 0; ++round; }
    }
    if (threadIdx.x == 0) QMOE_TRACE(P, 1, 6);
}

// ---------------------------------------------------------------------------
// Expert down + combine
//
// CTA c owns output rows [c*Rd, c*Rd + Rd).  Its sources are the shared
// expert (chunk 0) and the active experts (chunks 1..); all of them must fit
// in shared memory at once (host plan).  The hidden vectors are visited in
// source order -- shared vectors first, then the permuted pairs -- so a
// contiguous range of (vector, row step) tasks per warp keeps one vector's
// planes in registers.
// ---------------------------------------------------------------------------
template <int TR, int TS>
__global__ void __launch_bounds__(XK_THREADS, 2)
    k_down(DecodeParams P, int nst, int Rd, uint32_t stage_bytes, int nvec) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    int* s_sched = reinterpret_cast<int*>(smem + 1280);
    uint8_t* hs = reinterpret_cast<uint8_t*>(s_sched) + align_up(SCHED_SMEM_WORDS * 4, 128);
    const uint32_t hs_bytes = static_cast<uint32_t>(P.hq_stride) * static_cast<uint32_t>(nvec);
    float* ybuf = reinterpret_cast<float*>(hs + align_up(hs_bytes, 128));
    // every region starts 128-byte aligned (the stages are bulk-copy targets)
    float* s_w = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(ybuf) +
                                          align_up(static_cast<size_t>(nvec) * Rd * 4, 128));  // [T*k] weights
    float* s_sg = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s_w) +
                                           align_up(static_cast<size_t>(P.T) * P.k * 4, 128));  // [T] shared gate
    float* s_res = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(s_sg) +
                                            align_up(static_cast<size_t>(P.T) * 4, 128));       // [T][Rd] residual
    uint8_t* stages = reinterpret_cast<uint8_t*>(s_res) + align_up(static_cast<size_t>(P.T) * Rd * 4, 128);
    const uint64_t rbd = row_bytes(TR, P.F), rbs = row_bytes(TS, P.Fs);

    const int r0 = blockIdx.x * Rd;
    const int nrow = min(Rd, P.d - r0);
    if (threadIdx.x == 0) {
        QMOE_TRACE(P, 2, 0);
        for (int i = 0; i <= nst; ++i) mbar_init(full + i, 1);  // full[nst] doubles as the planes barrier
        fence_mbar_init();
    }
    __syncthreads();
    const int sh = P.has_shared ? 1 : 0;
    // prologue 1: shared-expert down rows (chunk 0)
    if (warp == NCW && lane == 0 && sh) {
        const StagePlan sp = plan_stage(stages, P.sdown.p + static_cast<uint64_t>(r0) * rbs, nrow * rbs, P.sdown.end);
        mbar_arrive_expect_tx(full, sp.tx);
        if (sp.tx) bulk_g2s(stages, sp.lo, sp.tx, full, P.ctrl);
    }
    // prologue 2: the routing and the block's residual input are final (the
    // gate/up kernel lets this kernel start only after the router completed)
    load_sched(s_sched, P);
    const int LS = P.E + 1;
    for (int i = threadIdx.x; i < P.T * P.k; i += blockDim.x) s_w[i] = __ldcg(P.topk_w + i);
    for (int t = threadIdx.x; t < P.T; t += blockDim.x)
        s_sg[t] = sh ? 1.0f / (1.0f + expf(-__ldcg(P.logits + t * LS + P.E))) : 0.0f;
    if (P.residual)
        for (int t = 0; t < P.T; ++t)
            for (int r = threadIdx.x; r < nrow; r += blockDim.x)
                s_res[t * Rd + r] = __ldcg(P.residual + static_cast<size_t>(t) * P.d + r0 + r);
    __syncthreads();
    if (threadIdx.x == 0) QMOE_TRACE(P, 2, 1);
    const int nact = s_sched[0];
    const int npairs = s_sched[1];
    const int* s_perm = s_sched + sched_perm_off(P.T, P.k, P.E);
    const int nsrc = nact + sh;  // chunk 0 = shared (if any), then routed sources
    // chunk cc occupies slot cc - round*nst during round cc / nst
    auto issue = [&](int cc, int slot) {
        const int e = s_sched[SCHED_HDR + 3 * (cc - sh)];
        uint8_t* dst = stages + static_cast<size_t>(slot) * stage_bytes;
        const StagePlan sp = plan_stage(dst, P.down.p + (static_cast<uint64_t>(e) * P.d + r0) * rbd, nrow * rbd,
                                        P.down.end);
        mbar_arrive_expect_tx(full + slot, sp.tx);
        if (sp.tx) bulk_g2s(dst, sp.lo, sp.tx, full + slot, P.ctrl);
    };
    if (warp == NCW) {
        // ---------------- producer ----------------
        if (lane == 0)
            for (int cc = sh; cc < min(nsrc, nst); ++cc) issue(cc, cc);
        if (lane == 0) {
            pdl_wait();  // the planes of silu(g)*u are written
            mbar_arrive_expect_tx(full + nst, hs_bytes);
            bulk_g2s(hs, P.hq, hs_bytes, full + nst, P.ctrl);
        }
        pdl_trigger();
        for (int rb0 = nst; rb0 < nsrc; rb0 += nst) {
            asm volatile("bar.sync 2, %0;" ::"r"((NCW + 1) * 32) : "memory");  // previous round consumed
            if (lane == 0)
                for (int cc = rb0; cc < min(nsrc, rb0 + nst); ++cc) issue(cc, cc - rb0);
        }
        if (lane == 0) mbar_wait(full + nst, 0, P.ctrl);
        return;
    }
    // the consumers read the planes only through the producer's copy, which
    // it issues after its own dependency wait
    mbar_wait(full + nst, 0, P.ctrl);
    pdl_trigger();  // the next block's router may start loading its weights
    if (threadIdx.x == 0) QMOE_TRACE(P, 2, 2);
    if (threadIdx.x == 0) QMOE_TRACE(P, 2, 3);

    // Tasks are (vector, row step) in source order: the T shared vectors
    // (ids T*k ..) of chunk 0 first, then the permuted pairs, whose chunk is
    // their expert's source index + sh.  Round r covers chunks
    // [r*nst, r*nst + nst) -- a contiguous task range, split evenly over the
    // consumer warps so that each warp keeps one vector's planes in registers
    // across consecutive tasks.
    const int Ur = P.F >> 6, Us = P.Fs >> 6;
    const int lgUr = ilog2(Ur), lgUs = ilog2(Us);
    const int steps_r = (nrow + (32 >> lgUr) - 1) >> (5 - lgUr);
    const int steps_s = (nrow + (32 >> lgUs) - 1) >> (5 - lgUs);
    const int Tsh = sh ? P.T : 0;
    const int nt_sh = Tsh * steps_s;
    // first task of chunk cc (cc == nsrc gives the total)
    auto chunk_task = [&](int cc) {
        if (cc < sh) return 0;
        const int q = cc - sh < nact ? s_sched[SCHED_HDR + 3 * (cc - sh) + 1] : npairs;
        return nt_sh + q * steps_r;
    };
    XU xr;
    for (int rb0 = 0, round = 0; rb0 < nsrc; rb0 += nst, ++round) {
        const int rend = min(nsrc, rb0 + nst);
        const int A = chunk_task(rb0), B = chunk_task(rend);
        const int t_lo = A + ((warp * (B - A)) >> 3), t_hi = A + (((warp + 1) * (B - A)) >> 3);
        static_assert(NCW == 8, "task split assumes 8 consumer warps");
        if (t_lo < t_hi) {
            // cursor of task t_lo: vector index vi (source order), row step st, chunk cc
            int vi, st, cc;
            if (t_lo < nt_sh) {
                vi = t_lo / steps_s;
                st = t_lo - vi * steps_s;
                cc = 0;
            } else {
                const int q = t_lo - nt_sh;
                const int pv = q / steps_r;
                st = q - pv * steps_r;
                vi = Tsh + pv;
                cc = max(rb0, sh);
                while (cc + 1 < rend && s_sched[SCHED_HDR + 3 * (cc + 1 - sh) + 1] <= pv) ++cc;
            }
            int cend = cc < sh ? Tsh : Tsh + s_sched[SCHED_HDR + 3 * (cc - sh) + 1] + s_sched[SCHED_HDR + 3 * (cc - sh) + 2];
            int cur_cc = -1, cur_vi = -1;
            uint32_t wbase = 0;
            for (int tau = t_lo; tau < t_hi; ++tau) {
                const bool shv = cc < sh;
                if (cc != cur_cc) {
                    const int slot = cc - rb0;
                    mbar_wait(full + slot, round & 1, P.ctrl);
                    const uint64_t srcaddr =
                        shv ? reinterpret_cast<uintptr_t>(P.sdown.p) + static_cast<uint64_t>(r0) * rbs
                            : reinterpret_cast<uintptr_t>(P.down.p) +
                                  (static_cast<uint64_t>(s_sched[SCHED_HDR + 3 * (cc - sh)]) * P.d + r0) * rbd;
                    wbase = smem_u32(stages) + static_cast<uint32_t>(slot) * stage_bytes + static_cast<uint32_t>(srcaddr & 15u);
                    cur_cc = cc;
                }
                const int vid = shv ? P.T * P.k + vi : s_perm[vi - Tsh];
                const int lgU = shv ? lgUs : lgUr;
                if (vi != cur_vi) {
                    const XPlanesView hv =
                        planes_view(smem_u32(hs) + static_cast<uint32_t>(vid) * static_cast<uint32_t>(P.hq_stride), P.H);
                    if (shv) load_xu<TS>(xr, hv, unit_of_lane<TS>(lane & (Us - 1), lgUs));
                    else load_xu<TR>(xr, hv, unit_of_lane<TR>(lane & (Ur - 1), lgUr));
                    cur_vi = vi;
                }
                const int ul = lane & ((1 << lgU) - 1), rsub = lane >> lgU;
                const int rl = (st << (5 - lgU)) + rsub;
                const bool valid = rl < nrow;
                float y = 0.0f;
                if (valid)
                    y = shv ? unit_dot_t<TS>(wbase + static_cast<uint32_t>(rl) * static_cast<uint32_t>(rbs),
                                             unit_of_lane<TS>(ul, lgUs), xr)
                            : unit_dot_t<TR>(wbase + static_cast<uint32_t>(rl) * static_cast<uint32_t>(rbd),
                                             unit_of_lane<TR>(ul, lgUr), xr);
                for (int o = (1 << lgU) >> 1; o; o >>= 1) y += __shfl_xor_sync(FULL, y, o);
                if (valid && ul == 0) stsf(smem_u32(ybuf) + 4u * static_cast<uint32_t>(vid * Rd + rl), y);
                // advance the cursor
                if (++st == (shv ? steps_s : steps_r)) {
                    st = 0;
                    if (++vi == cend && cc + 1 < nsrc) {
                        ++cc;
                        cend = Tsh + s_sched[SCHED_HDR + 3 * (cc - sh) + 1] + s_sched[SCHED_HDR + 3 * (cc - sh) + 2];
                    }
                }
            }
        }
        if (rend < nsrc) asm volatile("bar.sync 2, %0;" ::"r"((NCW + 1) * 32) : "memory");  // slots may be refilled
    }
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");
    if (threadIdx.x == 0) QMOE_TRACE(P, 2, 5);

    // combine (moe.cu:76-81 and :90-96, accumulation order of layer_moe.cpp:127-153)
    for (int idx = threadIdx.x; idx < P.T * nrow; idx += NCW * 32) {
        const int t = idx / nrow, r = idx - (idx / nrow) * nrow;
        float acc = 0.0f;
        for (int j = 0; j < P.k; ++j)
            acc = fmaf(s_w[t * P.k + j], ldsf(smem_u32(ybuf) + 4u * static_cast<uint32_t>((t * P.k + j) * Rd + r)), acc);
        if (sh) acc = fmaf(ldsf(smem_u32(ybuf) + 4u * static_cast<uint32_t>((P.T * P.k + t) * Rd + r)), s_sg[t], acc);
        if (!(s_w[t * P.k] == s_w[t * P.k])) acc = __uint_as_float(0x7FC00000u);  // routing error: NaN weights
        const size_t o = static_cast<size_t>(t) * P.d + r0 + r;
        P.out[o] = P.residual ? s_res[t * Rd + r] + acc : acc;
    }
    if (threadIdx.x == 0) QMOE_TRACE(P, 2, 6);
}

// ---------------------------------------------------------------------------
// Fused expert kernel: gate/up items, one grid-wide barrier, down + combine
//
// One CTA per SM.  Before the barrier a CTA does what k_gateup does for its
// items and, at the same time, pulls its own down rows (rows [c*Rd, c*Rd+Rd)
// of the shared expert and of every active expert) into shared memory; after
// the barrier it reads the planes of every hidden vector and does what
// k_down does.  The down rows therefore stream from HBM while the gate/up
// items are still being computed, and no kernel boundary separates the two
// halves.
//
// The barrier is a 64-bit arrival count in the workspace control words that
// only grows: every CTA adds one (acq_rel) and waits (acquire polls) until
// the count reaches the next multiple of the grid size.  A CTA that waits
// longer than kGridWaitNs raises EF_TIMEOUT and goes on; the results of that
// call are then invalid, and the count is no longer a multiple of the grid
// size, so the workspace must be initialised again (qmoe_workspace_init).  All CTAs must be resident at
// once: the grid is one CTA per SM and the launch asks for the whole SM's
// worth of shared memory at most; the dependent launch is released only
// after the barrier, so a later kernel cannot take an SM that a CTA of this
// grid still needs.
// ---------------------------------------------------------------------------
constexpr int FX_NCW = 16;
constexpr int FX_THREADS = (FX_NCW + 1) * 32;
constexpr uint64_t kGridWaitNs = 200ull * 1000ull * 1000ull;

struct FxLayout {
    int gnst, gsub, dnst, Rd, nvec;
    uint32_t half_bytes, dstage;
    uint32_t off_sched, off_xs, off_hb, off_w, off_sg, off_res, off_yb, off_gu, off_dn;
    uint64_t wait_ns;  // bound of the grid barrier's wait
    int phantom;       // extra arrivals the barrier waits for (0; > 0 only to test the bounded wait)
};

__device__ __forceinline__ uint64_t ld_acquire_u64(const unsigned long long* p) {
    uint64_t v;
    asm volatile("ld.acquire.gpu.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}

// n bytes (a multiple of 16; both ends 16-byte aligned) global -> shared with
// plain L2 loads, threads [0, nth) taking 16 bytes each per pass
__device__ __forceinline__ void copy_g2s16(uint8_t* dst, const uint8_t* src, uint32_t n, int tid, int nth) {
    for (uint32_t o = 16u * static_cast<uint32_t>(tid); o < n; o += 16u * static_cast<uint32_t>(nth))
        *reinterpret_cast<uint4*>(dst + o) = __ldcg(reinterpret_cast<const uint4*>(src + o));
}

template <int TR, int TS, int DR, int DS>
__global__ void __launch_bounds__(FX_THREADS, 1) k_experts(const __grid_constant__ DecodeParams P,
                                                          const __grid_constant__ FxLayout L) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    if (warp == 0) {
        touch_params(P);
        touch_params(L);
    }
    uint64_t* gfull = reinterpret_cast<uint64_t*>(smem);  // [8 slots][4 sub-chunks]
    uint64_t* gempty = gfull + 32;
    uint64_t* dfull = gempty + 8;  // [72]
    int* s_sched = reinterpret_cast<int*>(smem + L.off_sched);
    uint8_t* xs = smem + L.off_xs;
    float* hb = reinterpret_cast<float*>(smem + L.off_hb);
    float* s_w = reinterpret_cast<float*>(smem + L.off_w);
    float* s_sg = reinterpret_cast<float*>(smem + L.off_sg);
    float* s_res = reinterpret_cast<float*>(smem + L.off_res);
    uint8_t* gst = smem + L.off_gu;
    uint8_t* hs = smem + L.off_gu;  // the gate/up stages are free once every item is done
    uint8_t* dst = smem + L.off_dn;

    const int d = P.d, G = gridDim.x, c = blockIdx.x;
    const int lgU = ilog2(d >> 6), U = 1 << lgU, lgR = 5 - lgU;
    const uint64_t rbg = row_bytes(TR, d), rbs = row_bytes(TS, d);
    const uint64_t rbd = row_bytes(DR, P.F), rbsd = row_bytes(DS, P.Fs);
    const int sh = P.has_shared ? 1 : 0;
    const int nb_sh = sh ? P.Fs / ITEM_ROWS : 0;
    const int lgF = ilog2(P.F / ITEM_ROWS);
    const int Rd = L.Rd, r0d = c * Rd;
    const int nrow = max(0, min(Rd, d - r0d));
    const int dnst = L.dnst;
    const uint32_t half_bytes = L.half_bytes;

    if (tid == 0) {
        QMOE_TRACE(P, 1, 0);
        for (int i = 0; i < L.gnst; ++i) {
            for (int j = 0; j < L.gsub; ++j) mbar_init(gfull + 4 * i + j, 1);
            mbar_init(gempty + i, FX_NCW);
        }
        for (int i = 0; i < L.dnst; ++i) mbar_init(dfull + i, 1);
        fence_mbar_init();
    }
    __syncthreads();

    auto issue_gu = [&](int slot, bool shared_src, int expert, int r0) {
        const uint64_t rb = shared_src ? rbs : rbg;
        const uint8_t* gsrc = shared_src ? P.sgate.p + r0 * rbs : P.gate.p + (static_cast<uint64_t>(expert) * P.F + r0) * rbg;
        const uint8_t* usrc = shared_src ? P.sup.p + r0 * rbs : P.up.p + (static_cast<uint64_t>(expert) * P.F + r0) * rbg;
        uint8_t* dg = gst + static_cast<size_t>(slot) * 2 * half_bytes;
        uint8_t* du = dg + half_bytes;
        // gsub sub-chunks of 32/gsub rows, each with its own barrier, so the
        // consumers start on the first rows while the rest stream in (the host
        // picks gsub > 1 only when every sub-chunk starts 16-byte aligned)
        const uint64_t cb = (ITEM_ROWS / L.gsub) * rb;
        for (int j = 0; j < L.gsub; ++j) {
            const StagePlan pg = plan_stage(dg + j * cb, gsrc + j * cb, cb, shared_src ? P.sgate.end : P.gate.end);
            const StagePlan pu = plan_stage(du + j * cb, usrc + j * cb, cb, shared_src ? P.sup.end : P.up.end);
            uint64_t* bar = gfull + 4 * slot + j;
            mbar_arrive_expect_tx(bar, pg.tx + pu.tx);
            if (pg.tx) bulk_g2s(dg + j * cb, pg.lo, pg.tx, bar, P.ctrl);
            if (pu.tx) bulk_g2s(du + j * cb, pu.lo, pu.tx, bar, P.ctrl);
        }
    };
    // chunk cc = 0: shared expert (when present); cc >= sh: routed source cc - sh
    auto dn_src = [&](int cc) -> const uint8_t* {
        return cc < sh ? P.sdown.p + static_cast<uint64_t>(r0d) * rbsd
                       : P.down.p + (static_cast<uint64_t>(s_sched[SCHED_HDR + 3 * (cc - sh)]) * d + r0d) * rbd;
    };
    auto issue_dn = [&](int cc, int slot) {
        uint8_t* dd = dst + static_cast<size_t>(slot) * L.dstage;
        const bool shc = cc < sh;
        const StagePlan sp = plan_stage(dd, dn_src(cc), nrow * (shc ? rbsd : rbd), shc ? P.sdown.end : P.down.end);
        mbar_arrive_expect_tx(dfull + slot, sp.tx);
        if (sp.tx) bulk_g2s(dd, sp.lo, sp.tx, dfull + slot, P.ctrl);
    };

    // The producer lane issues every copy of the first round through one
    // loop body: the prologue's routing-independent copies (the shared
    // expert's down rows in every CTA, a shared gate/up item in the first
    // CTAs) run it before the routing is known, so the instructions that
    // issue the routed copies right after the routing are already fetched
    // (code that runs for the first time in a launch stalls on instruction
    // fetches, and those stalls would also slow the consumers' first pass).
    // Job q < ngu: gate/up sub-chunk (item kk = kb + q / gsub, slot kk,
    // sub-chunk q % gsub, gate and up rows); otherwise down rows of source
    // cc = ccb + q - ngu into down slot cc.  Every field is a select, so both
    // kinds run the same instructions.
    if (warp == FX_NCW) {
        // ---------------- producer ----------------
        const int lgsub = L.gsub == 4 ? 2 : 0;
        int ni = 0, nsrc = sh;
#pragma unroll 1
        for (int phase = 0; phase < 2; ++phase) {
            if (phase) {
                // the routing warps have written the schedule
                asm volatile("bar.sync 5, %0;" ::"r"((RT_WARPS + 1) * 32) : "memory");
                const int nact = s_sched[0];
                const int nitems = nb_sh + (nact << lgF);
                ni = c < nitems ? (nitems - 1 - c) / G + 1 : 0;
                nsrc = nact + sh;
            }
            if (lane == 0) {
                const int kb = (phase && c < nb_sh) ? 1 : 0;  // a shared item 0 went out in the prologue
                const int ke = phase ? min(ni, L.gnst) : (c < nb_sh ? 1 : 0);
                const int ccb = phase ? sh : 0;
                const int cce = nrow > 0 ? (phase ? min(nsrc, dnst) : sh) : 0;
                const int ngu = max(ke - kb, 0) << lgsub;
                const int nj = ngu + max(cce - ccb, 0);
#pragma unroll 1
                for (int q = 0; q < nj; ++q) {
                    const bool gu = q < ngu;
                    const int kk = kb + (q >> lgsub);
                    const int jsub = q & (L.gsub - 1);
                    const int cc = ccb + (q - ngu);
                    const int it = c + kk * G;
                    const int jr = max(it - nb_sh, 0);
                    const bool shj = gu ? it < nb_sh : cc < sh;
                    const int si = gu ? (jr >> lgF) : max(cc - sh, 0);
                    const int expert = shj ? 0 : s_sched[SCHED_HDR + 3 * si];
                    const uint64_t rbj = gu ? (shj ? rbs : rbg) : (shj ? rbsd : rbd);
                    const int rsub = ITEM_ROWS >> lgsub;
                    const int r0 = (shj ? it : (jr & ((1 << lgF) - 1))) * ITEM_ROWS + jsub * rsub;
                    const uint64_t row = gu ? (shj ? static_cast<uint64_t>(r0) : static_cast<uint64_t>(expert) * P.F + r0)
                                            : (shj ? static_cast<uint64_t>(r0d) : static_cast<uint64_t>(expert) * d + r0d);
                    const uint8_t* b0 = gu ? (shj ? P.sgate.p : P.gate.p) : (shj ? P.sdown.p : P.down.p);
                    const uint8_t* e0 = gu ? (shj ? P.sgate.end : P.gate.end) : (shj ? P.sdown.end : P.down.end);
                    const uint8_t* b1 = shj ? P.sup.p : P.up.p;
                    const uint8_t* e1 = shj ? P.sup.end : P.up.end;
                    const uint32_t n0 = static_cast<uint32_t>((gu ? rsub : nrow) * rbj);
                    const uint32_t n1 = gu ? n0 : 0u;
                    uint8_t* d0 = gu ? gst + static_cast<size_t>(kk) * 2 * half_bytes + static_cast<size_t>(jsub) * n0
                                     : dst + static_cast<size_t>(cc) * L.dstage;
                    uint8_t* d1 = d0 + half_bytes;
                    uint64_t* bar = gu ? gfull + 4 * kk + jsub : dfull + cc;
                    const uint8_t *lo0 = nullptr, *lo1 = nullptr;
                    uint32_t tx0 = 0, tx1 = 0;
#pragma unroll 1
                    for (int h = 0; h < (n1 ? 2 : 1); ++h) {
                        const StagePlan sp = plan_stage(h ? d1 : d0, (h ? b1 : b0) + row * rbj, h ? n1 : n0, h ? e1 : e0);
                        if (h) { lo1 = sp.lo; tx1 = sp.tx; } else { lo0 = sp.lo; tx0 = sp.tx; }
                    }
                    mbar_arrive_expect_tx(bar, tx0 + tx1);
#pragma unroll 1
                    for (int h = 0; h < 2; ++h) {
                        const uint32_t tx = h ? tx1 : tx0;
                        if (tx) bulk_g2s(h ? d1 : d0, h ? lo1 : lo0, tx, bar, P.ctrl);
                    }
                }
            }
        }
        if (lane == 0) {  // later items of this CTA, as ring slots are released
            int kk = min(ni, L.gnst), it = c + kk * G, slot = kk % L.gnst, round = kk / L.gnst;
            for (; kk < ni; ++kk, it += G) {
                mbar_wait(gempty + slot, (round - 1) & 1, P.ctrl);
                if (it < nb_sh) {
                    issue_gu(slot, true, -1, it * ITEM_ROWS);
                } else {
                    const int jr = it - nb_sh;
                    issue_gu(slot, false, s_sched[SCHED_HDR + 3 * (jr >> lgF)], (jr & ((1 << lgF) - 1)) * ITEM_ROWS);
                }
                if (++slot == L.gnst) { slot = 0; ++round; }
            }
        }
        for (int rb0 = dnst; rb0 < nsrc; rb0 += dnst) {  // later down rounds, if the sources do not all fit
            asm volatile("bar.sync 2, %0;" ::"r"((FX_NCW + 1) * 32) : "memory");
            if (lane == 0 && nrow > 0)
                for (int cc = rb0; cc < min(nsrc, rb0 + dnst); ++cc) issue_dn(cc, cc - rb0);
        }
        return;
    }

    // ---------------- consumers ----------------
    if (tid == 0) pdl_wait();  // the router has finished: logits and block input are valid
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
    if (tid == 0) QMOE_TRACE(P, 1, 1);
    if (warp < RT_WARPS) {
        // every CTA selects the experts itself from the router logits (CTA 0
        // also publishes the routing to the workspace): no cross-CTA step
        // between the router's logits and this CTA's weight loads
        topk_and_schedule(P, s_sched, s_w, c == 0, 3);
        if (tid == 0) QMOE_TRACE(P, 1, 6);
        asm volatile("bar.arrive 5, %0;" ::"r"((RT_WARPS + 1) * 32) : "memory");  // to the producer
    } else {
        // the other warps: input planes, shared-expert gate, residual rows
        constexpr int NTH = (FX_NCW - RT_WARPS) * 32;
        const int t2 = tid - RT_WARPS * 32;
        const int nres = (P.residual && nrow > 0) ? P.T * nrow : 0;
        const int n32 = P.T + nres;
        const int LS = P.E + 1;
        auto load32 = [&](int q) -> float {
            if (q < P.T) return __ldcg(P.logits + q * LS + P.E);
            q -= P.T;
            const int t = q / nrow, r = q - t * nrow;
            return __ldcg(P.residual + static_cast<size_t>(t) * d + r0d + r);
        };
        auto store32 = [&](int q, float v) {
            if (q < P.T) { s_sg[q] = sh ? 1.0f / (1.0f + expf(-v)) : 0.0f; return; }
            q -= P.T;
            const int t = q / nrow, r = q - t * nrow;
            s_res[t * Rd + r] = v;
        };
        const float v0 = t2 < n32 ? load32(t2) : 0.0f;
        x_planes_smem<NTH>(xs, P, t2);  // its loads go out before the store below
        if (t2 < n32) store32(t2, v0);
        for (int q = t2 + NTH; q < n32; q += NTH) store32(q, load32(q));
        if (t2 == 0) QMOE_TRACE(P, 1, 7);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");  // schedule, planes and gates are written
    if (tid == 0) QMOE_TRACE(P, 1, 2);
    const int nact = s_sched[0];
    const int npairs = s_sched[1];
    const int* s_perm = s_sched + sched_perm_off(P.T, P.k, P.E);
    const int* s_tok = s_sched + sched_tok_off(P.T, P.k, P.E);
    const int nitems = nb_sh + (nact << lgF);
    const int ni = c < nitems ? (nitems - 1 - c) / G + 1 : 0;
    const int nsrc = nact + sh;

    // ---------------- consumers: gate/up items ----------------
    {
        const int ul = lane & (U - 1), rsub = lane >> lgU;
        const int u_r = unit_of_lane<TR>(ul, lgU), u_s = unit_of_lane<TS>(ul, lgU);
        const int lgS = lgU;  // steps per item = 32 / rows per step
        XU xr;
        int cur_key = -1;
        int i = c, slot = 0, round = 0;
        for (int kk = 0; kk < ni; ++kk, i += G) {
            const bool routed = i >= nb_sh;
            int bb, expert = -1, pair0 = 0, ntok = P.T;
            if (routed) {
                const int j = i - nb_sh, s2 = j >> lgF;
                bb = j & ((1 << lgF) - 1);
                expert = s_sched[SCHED_HDR + 3 * s2];
                pair0 = s_sched[SCHED_HDR + 3 * s2 + 1];
                ntok = s_sched[SCHED_HDR + 3 * s2 + 2];
            } else {
                bb = i;
            }
            const int r0 = bb * ITEM_ROWS;
            uint32_t waited = 0;  // sub-chunks of this item this warp has waited for
            uint32_t dg = smem_u32(gst) + static_cast<uint32_t>(slot) * 2u * half_bytes;
            uint32_t du = dg + half_bytes;
            {
                const uintptr_t gsrc = routed ? reinterpret_cast<uintptr_t>(P.gate.p) + (static_cast<uint64_t>(expert) * P.F + r0) * rbg
                                              : reinterpret_cast<uintptr_t>(P.sgate.p) + static_cast<uint64_t>(r0) * rbs;
                const uintptr_t usrc = routed ? reinterpret_cast<uintptr_t>(P.up.p) + (static_cast<uint64_t>(expert) * P.F + r0) * rbg
                                              : reinterpret_cast<uintptr_t>(P.sup.p) + static_cast<uint64_t>(r0) * rbs;
                dg += static_cast<uint32_t>(gsrc & 15u);
                du += static_cast<uint32_t>(usrc & 15u);
            }
            const uint32_t rb = static_cast<uint32_t>(routed ? rbg : rbs);
            const int ntask = ntok << lgS;
            for (int tau = warp; tau < ntask; tau += FX_NCW) {
                const int ti = tau >> lgS, st = tau & ((1 << lgS) - 1);
                const int tok = routed ? s_tok[pair0 + ti] : ti;
                const int key = (tok << 1) | (routed ? 1 : 0);
                if (key != cur_key) {
                    const XPlanesView xv = planes_view(smem_u32(xs) + static_cast<uint32_t>(tok) * static_cast<uint32_t>(P.xq_stride), d);
                    if (TR == TS || routed) load_xu<TR>(xr, xv, u_r); else load_xu<TS>(xr, xv, u_s);
                    cur_key = key;
                }
                const int rl = (st << lgR) + rsub;
                const int sub = (rl * L.gsub) >> 5;  // the warp's rows lie in one sub-chunk
                if (!((waited >> sub) & 1u)) {
                    mbar_wait(gfull + 4 * slot + sub, round & 1, P.ctrl);
                    waited |= 1u << sub;
                    if (tid == 0 && kk == 0) QMOE_TRACE(P, 1, 3);
                }
                float g, up;
                if (TR == TS || routed) {  // one copy of the dot code when the types agree
                    g = unit_dot_t<TR>(dg + static_cast<uint32_t>(rl) * rb, u_r, xr);
                    up = unit_dot_t<TR>(du + static_cast<uint32_t>(rl) * rb, u_r, xr);
                } else {
                    g = unit_dot_t<TS>(dg + static_cast<uint32_t>(rl) * rb, u_s, xr);
                    up = unit_dot_t<TS>(du + static_cast<uint32_t>(rl) * rb, u_s, xr);
                }
                for (int o = U >> 1; o; o >>= 1) {
                    g += __shfl_xor_sync(FULL, g, o);
                    up += __shfl_xor_sync(FULL, up, o);
                }
                if (ul == 0) stsf(smem_u32(hb) + 4u * static_cast<uint32_t>(rl * P.T + ti), silu_mul(g, up));
            }
            asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
            // the item's 32-blocks of silu(g)*u: F32 copy and 24-bit planes
            for (int ti = warp; ti < ntok; ti += FX_NCW) {
                const int vid = routed ? s_perm[pair0 + ti] : P.T * P.k + ti;
                const float v = ldsf(smem_u32(hb) + 4u * static_cast<uint32_t>(lane * P.T + ti));
                P.hidden[static_cast<size_t>(vid) * P.H + r0 + lane] = v;
                xq_block32_global(v, P.hq + static_cast<size_t>(vid) * P.hq_stride, P.H, r0, lane);
            }
            asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
            if (lane == 0) mbar_arrive(gempty + slot);
            if (++slot == L.gnst) { slot = 0; ++round; }
        }
    }

    // ---------------- grid-wide barrier: every hidden vector is written ----------------
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
    if (tid == 0) {
        QMOE_TRACE(P, 1, 4);
        // the CTA barrier above orders every consumer's stores before this
        // release (cumulativity); the acquire polls make all CTAs' stores
        // visible to this CTA's threads after the CTA barrier below
        unsigned long long* ctr = reinterpret_cast<unsigned long long*>(P.ctrl + CTRL_GRID_CTR);
        uint64_t old;
        asm volatile("atom.add.acq_rel.gpu.u64 %0, [%1], %2;" : "=l"(old) : "l"(ctr), "l"(1ull) : "memory");
        const uint64_t target = (old / static_cast<uint64_t>(G) + 1u) * static_cast<uint64_t>(G) +
                                static_cast<uint64_t>(L.phantom);
        if (old + 1u != target) {
            const uint64_t t0 = gtimer();
            while (ld_acquire_u64(ctr) < target) {
                if (gtimer() - t0 > L.wait_ns) {
                    raise_error(P.ctrl, EF_TIMEOUT);
                    break;
                }
                __nanosleep(32);
            }
        }
        QMOE_TRACE(P, 1, 5);
    }
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
    pdl_trigger();  // the next block's router may start loading its weights

    // ---------------- consumers: down + combine ----------------
    copy_g2s16(hs, P.hq, static_cast<uint32_t>(P.hq_stride) * static_cast<uint32_t>(L.nvec), tid, FX_NCW * 32);
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
    if (tid == 0) QMOE_TRACE(P, 2, 3);
    const int Ur = P.F >> 6, Us = P.Fs >> 6;
    const int lgUr = ilog2(Ur), lgUs = ilog2(Us);
    const int steps_r = (nrow + (32 >> lgUr) - 1) >> (5 - lgUr);
    const int steps_s = (nrow + (32 >> lgUs) - 1) >> (5 - lgUs);
    const int Tsh = sh ? P.T : 0;
    const int nt_sh = Tsh * steps_s;
    auto chunk_task = [&](int cc) {
        if (cc < sh) return 0;
        const int q = cc - sh < nact ? s_sched[SCHED_HDR + 3 * (cc - sh) + 1] : npairs;
        return nt_sh + q * steps_r;
    };
    XU xr;
    static_assert(FX_NCW == 16, "task split assumes 16 consumer warps");
    for (int rb0 = 0, round = 0; rb0 < nsrc; rb0 += dnst, ++round) {
        const int rend = min(nsrc, rb0 + dnst);
        const int A = chunk_task(rb0), B = chunk_task(rend);
        const int t_lo = A + ((warp * (B - A)) >> 4), t_hi = A + (((warp + 1) * (B - A)) >> 4);
        if (t_lo < t_hi) {
            int vi, st, cc;
            if (t_lo < nt_sh) {
                vi = t_lo / steps_s;
                st = t_lo - vi * steps_s;
                cc = 0;
            } else {
                const int q = t_lo - nt_sh;
                const int pv = q / steps_r;
                st = q - pv * steps_r;
                vi = Tsh + pv;
                cc = max(rb0, sh);
                while (cc + 1 < rend && s_sched[SCHED_HDR + 3 * (cc + 1 - sh) + 1] <= pv) ++cc;
            }
            int cend = cc < sh ? Tsh : Tsh + s_sched[SCHED_HDR + 3 * (cc - sh) + 1] + s_sched[SCHED_HDR + 3 * (cc - sh) + 2];
            int cur_cc = -1, cur_vi = -1;
            uint32_t wbase = 0;
            for (int tau = t_lo; tau < t_hi; ++tau) {
                const bool shv = cc < sh;
                if (cc != cur_cc) {
                    const int slot = cc - rb0;
                    mbar_wait(dfull + slot, round & 1, P.ctrl);
                    wbase = smem_u32(dst) + static_cast<uint32_t>(slot) * L.dstage +
                            static_cast<uint32_t>(reinterpret_cast<uintptr_t>(dn_src(cc)) & 15u);
                    cur_cc = cc;
                }
                const int vid = shv ? P.T * P.k + vi : s_perm[vi - Tsh];
                const int lgUv = shv ? lgUs : lgUr;
                if (vi != cur_vi) {
                    const XPlanesView hv =
                        planes_view(smem_u32(hs) + static_cast<uint32_t>(vid) * static_cast<uint32_t>(P.hq_stride), P.H);
                    if (DS == DR) load_xu<DR>(xr, hv, unit_of_lane<DR>(lane & ((1 << lgUv) - 1), lgUv));
                    else if (shv) load_xu<DS>(xr, hv, unit_of_lane<DS>(lane & (Us - 1), lgUs));
                    else load_xu<DR>(xr, hv, unit_of_lane<DR>(lane & (Ur - 1), lgUr));
                    cur_vi = vi;
                }
                const int ul = lane & ((1 << lgUv) - 1), rsub = lane >> lgUv;
                const int rl = (st << (5 - lgUv)) + rsub;
                const bool valid = rl < nrow;
                float y = 0.0f;
                // one copy of the dot code when the shared and routed down types agree
                if (valid && DS == DR)
                    y = unit_dot_t<DR>(wbase + static_cast<uint32_t>(rl) * static_cast<uint32_t>(shv ? rbsd : rbd),
                                       unit_of_lane<DR>(ul, lgUv), xr);
                else if (valid)
                    y = shv ? unit_dot_t<DS>(wbase + static_cast<uint32_t>(rl) * static_cast<uint32_t>(rbsd),
                                             unit_of_lane<DS>(ul, lgUs), xr)
                            : unit_dot_t<DR>(wbase + static_cast<uint32_t>(rl) * static_cast<uint32_t>(rbd),
                                             unit_of_lane<DR>(ul, lgUr), xr);
                for (int o = (1 << lgUv) >> 1; o; o >>= 1) y += __shfl_xor_sync(FULL, y, o);
                if (valid && ul == 0) stsf(smem_u32(smem + L.off_yb) + 4u * static_cast<uint32_t>(vid * Rd + rl), y);
                if (++st == (shv ? steps_s : steps_r)) {
                    st = 0;
                    if (++vi == cend && cc + 1 < nsrc) {
                        ++cc;
                        cend = Tsh + s_sched[SCHED_HDR + 3 * (cc - sh) + 1] + s_sched[SCHED_HDR + 3 * (cc - sh) + 2];
                    }
                }
            }
        }
        if (rend < nsrc) asm volatile("bar.sync 2, %0;" ::"r"((FX_NCW + 1) * 32) : "memory");  // slots may be refilled
    }
    if (tid == 0) QMOE_TRACE(P, 2, 4);
    asm volatile("bar.sync 1, %0;" ::"r"(FX_NCW * 32) : "memory");
    if (tid == 0) QMOE_TRACE(P, 2, 5);

    // combine (moe.cu:76-81 and :90-96, accumulation order of layer_moe.cpp:127-153)
    const uint32_t ybuf = smem_u32(smem + L.off_yb);
    for (int idx = tid; idx < P.T * nrow; idx += FX_NCW * 32) {
        const int t = idx / nrow, r = idx - t * nrow;
        float acc = 0.0f;
        for (int j = 0; j < P.k; ++j)
            acc = fmaf(s_w[t * P.k + j], ldsf(ybuf + 4u * static_cast<uint32_t>((t * P.k + j) * Rd + r)), acc);
        if (sh) acc = fmaf(ldsf(ybuf + 4u * static_cast<uint32_t>((P.T * P.k + t) * Rd + r)), s_sg[t], acc);
        if (!(s_w[t * P.k] == s_w[t * P.k])) acc = __uint_as_float(0x7FC00000u);  // routing error: NaN weights
        const size_t o = static_cast<size_t>(t) * d + r0d + r;
        P.out[o] = P.residual ? s_res[t * Rd + r] + acc : acc;
    }
    if (tid == 0) QMOE_TRACE(P, 2, 6);
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace {
struct DevCache {
    int sms = 0;
    int smem_optin = 0;
    bool pdl = true;
};
DevCache g_dev[64];

DevCache& dev_cache() {
    int dev = 0;
    cudaGetDevice(&dev);
    DevCache& c = g_dev[dev & 63];
    if (!c.sms) {
        cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&c.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
        const char* e = getenv("QMOE_PDL");
        c.pdl = !(e && e[0] == '0');
    }
    return c;
}

template <typename... Args>
cudaError_t launch(void (*kern)(Args...), int grid, int block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(block);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dev_cache().pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename K>
cudaError_t set_smem(K kern, size_t smem) {
    if (smem <= 48 * 1024) return cudaSuccess;
    return cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
}
}  // namespace

int decode_num_sms() { return dev_cache().sms; }

cudaError_t launch_router(const DecodeParams& P, cudaStream_t s) {
    const int nrows = P.E + (P.has_shared ? 1 : 0);
    const int grid = (nrows + RT_WARPS - 1) / RT_WARPS;
    switch (P.d / 256) {
        case 1: return launch(k_router<1>, grid, RT_WARPS * 32, 0, s, P);
        case 2: return launch(k_router<2>, grid, RT_WARPS * 32, 0, s, P);
        case 4: return launch(k_router<4>, grid, RT_WARPS * 32, 0, s, P);
        case 8: return launch(k_router<8>, grid, RT_WARPS * 32, 0, s, P);
        case 16: return launch(k_router<16>, grid, RT_WARPS * 32, 0, s, P);
        default: return cudaErrorInvalidValue;
    }
}

struct GuPlan { int grid, nst, dn_rows; uint32_t half_bytes; size_t smem; };

static bool plan_gateup(const DecodeParams& P, GuPlan& g) {
    DevCache& dc = dev_cache();
    if (dc.sms <= 0 || dc.smem_optin <= 0) return false;  // no usable device
    g.grid = dc.sms;
    g.dn_rows = (P.d + dc.sms - 1) / dc.sms;  // rows per down-kernel CTA (see plan_down)
    if (P.F % ITEM_ROWS || P.Fs % ITEM_ROWS) return false;
    const uint64_t rb = std::max(row_bytes(P.gate.type, P.d), row_bytes(P.sgate.type, P.d));
    g.half_bytes = static_cast<uint32_t>(align_up(ITEM_ROWS * rb + 32, 128));
    const int umax = sched_max_src(P.T, P.k, P.E);
    const int items_max = (P.has_shared ? P.Fs / ITEM_ROWS : 0) + umax * (P.F / ITEM_ROWS);
    const int per_cta = (items_max + g.grid - 1) / g.grid;
    const size_t fixed = 256 + align_up(SCHED_SMEM_WORDS * 4, 128) + align_up(P.xq_stride * P.T, 128) +
                         align_up(static_cast<size_t>(ITEM_ROWS) * P.T * 4, 128);
    const size_t stage = 2 * static_cast<size_t>(g.half_bytes);
    const size_t budget = static_cast<size_t>(dc.smem_optin) - 1024;
    if (fixed + stage > budget) return false;
    g.nst = static_cast<int>(std::min<size_t>(std::min<size_t>(per_cta, 8), (budget - fixed) / stage));
    g.nst = std::max(g.nst, 1);
    g.smem = fixed + static_cast<size_t>(g.nst) * stage;
    return true;
}

struct DnPlan { int grid, nst, Rd, nvec; uint32_t stage_bytes; size_t smem; };

static bool plan_down(const DecodeParams& P, DnPlan& p) {
    DevCache& dc = dev_cache();
    if (dc.sms <= 0 || dc.smem_optin <= 0) return false;  // no usable device
    p.Rd = (P.d + dc.sms - 1) / dc.sms;
    p.grid = (P.d + p.Rd - 1) / p.Rd;
    p.nvec = P.T * P.k + P.T;
    const uint64_t rb = std::max(row_bytes(P.down.type, P.F), row_bytes(P.sdown.type, P.Fs));
    p.stage_bytes = static_cast<uint32_t>(align_up(p.Rd * rb + 32, 128));
    const size_t fixed = 1280 + align_up(SCHED_SMEM_WORDS * 4, 128) + align_up(P.hq_stride * p.nvec, 128) +
                         align_up(static_cast<size_t>(p.nvec) * p.Rd * 4, 128) +
                         align_up(4 * static_cast<size_t>(P.T) * P.k, 128) + align_up(4 * static_cast<size_t>(P.T), 128) +
                         align_up(static_cast<size_t>(P.T) * p.Rd * 4, 128);
    const size_t optin = static_cast<size_t>(dc.smem_optin) - 1024;
    // as many sources resident at once as fit (shared + one per active
    // expert when possible); the rest follow in rounds
    if (fixed + p.stage_bytes > optin) return false;
    const int want = sched_max_src(P.T, P.k, P.E) + (P.has_shared ? 1 : 0);
    p.nst = static_cast<int>(std::min<size_t>({static_cast<size_t>(want), 71, (optin - fixed) / p.stage_bytes}));
    p.smem = fixed + static_cast<size_t>(p.nst) * p.stage_bytes;
    if (P.hq_stride * p.nvec >= (1u << 20)) return false;  // one bulk copy (transaction-count limit)
    return true;
}

bool decode_supported(const DecodeParams& P) {
    GuPlan g;
    DnPlan dn;
    return plan_gateup(P, g) && plan_down(P, dn);
}

// (routed type, shared type) -> kernel instantiation
template <template <int, int> class KS>
static typename KS<12, 12>::type pick(int tr, int ts) {  // NOLINT
#define QMOE_TS(TRV)                                         \
    switch (ts) {                                            \
        case 12: return KS<TRV, 12>::get();                  \
        case 13: return KS<TRV, 13>::get();                  \
        case 14: return KS<TRV, 14>::get();                  \
        case 8: return KS<TRV, 8>::get();                    \
        default: return nullptr;                             \
    }
    switch (tr) {
        case 12: QMOE_TS(12)
        case 13: QMOE_TS(13)
        case 14: QMOE_TS(14)
        case 8: QMOE_TS(8)
        default: return nullptr;
    }
#undef QMOE_TS
}

template <int A, int B>
struct GuSel {
    typedef void (*type)(DecodeParams, int, uint32_t, int);
    static type get() { return k_gateup<A, B>; }
};
template <int A, int B>
struct DnSel {
    typedef void (*type)(DecodeParams, int, int, uint32_t, int);
    static type get() { return k_down<A, B>; }
};

cudaError_t launch_gateup(const DecodeParams& P, cudaStream_t s) {
    GuPlan g;
    if (!plan_gateup(P, g)) return cudaErrorInvalidValue;
    auto kern = pick<GuSel>(P.gate.type, P.sgate.type);
    if (!kern) return cudaErrorInvalidValue;
    cudaError_t e = set_smem(kern, g.smem);
    if (e != cudaSuccess) return e;
    return launch(kern, g.grid, GU_THREADS, g.smem, s, P, g.nst, g.half_bytes, g.dn_rows);
}

// ---- fused expert kernel ----
// Bound of the fused kernel's grid-barrier wait and extra arrivals it waits
// for (qmoe_debug_grid_barrier; defaults kGridWaitNs and 0).
static uint64_t g_grid_wait_ns = kGridWaitNs;
static int g_grid_phantom = 0;

void set_grid_barrier_limits(uint64_t wait_ns, int phantom) {
    g_grid_wait_ns = wait_ns ? wait_ns : kGridWaitNs;
    g_grid_phantom = phantom > 0 ? phantom : 0;
}

static bool plan_fused(const DecodeParams& P, FxLayout& L, size_t& smem, int& grid) {
    DevCache& dc = dev_cache();
    L.wait_ns = g_grid_wait_ns;
    L.phantom = g_grid_phantom;
    if (dc.sms <= 0 || dc.smem_optin <= 0) return false;  // no usable device
    if (P.F % ITEM_ROWS || P.Fs % ITEM_ROWS) return false;
    grid = dc.sms;
    L.Rd = (P.d + grid - 1) / grid;
    L.nvec = P.T * P.k + P.T;
    const uint64_t rbg = std::max(row_bytes(P.gate.type, P.d), row_bytes(P.sgate.type, P.d));
    const uint64_t rbd = std::max(row_bytes(P.down.type, P.F), row_bytes(P.sdown.type, P.Fs));
    L.half_bytes = static_cast<uint32_t>(align_up(ITEM_ROWS * rbg + 32, 128));
    // four 8-row sub-chunks per item when 8 rows of every gate/up type are a
    // whole number of 16-byte chunks (item starts are then 16-byte aligned)
    L.gsub = ((8 * row_bytes(P.gate.type, P.d)) % 16 == 0 && (8 * row_bytes(P.sgate.type, P.d)) % 16 == 0) ? 4 : 1;
    L.dstage = static_cast<uint32_t>(align_up(L.Rd * rbd + 32, 128));
    size_t off = 1024;
    auto take = [&](size_t bytes) {
        const size_t o = off;
        off += align_up(bytes, 128);
        return static_cast<uint32_t>(o);
    };
    L.off_sched = take(SCHED_SMEM_WORDS * 4);
    L.off_xs = take(static_cast<size_t>(P.xq_stride) * P.T);
    L.off_hb = take(static_cast<size_t>(ITEM_ROWS) * P.T * 4);
    L.off_w = take(static_cast<size_t>(P.T) * P.k * 4);
    L.off_sg = take(static_cast<size_t>(P.T) * 4);
    L.off_res = take(static_cast<size_t>(P.T) * L.Rd * 4);
    L.off_yb = take(static_cast<size_t>(L.nvec) * L.Rd * 4);
    const size_t fixed = off;
    const size_t hs_bytes = static_cast<size_t>(P.hq_stride) * L.nvec;
    const size_t budget = static_cast<size_t>(dc.smem_optin) - 5120;  // static shared memory of the routing step
    const int nb_sh = P.has_shared ? P.Fs / ITEM_ROWS : 0;
    const int srcs = sched_max_src(P.T, P.k, P.E);
    const int per_cta = (nb_sh + srcs * (P.F / ITEM_ROWS) + grid - 1) / grid;
    const int want_d = srcs + (P.has_shared ? 1 : 0);
    auto gu_region = [&](int g) { return std::max(static_cast<size_t>(g) * 2 * L.half_bytes, hs_bytes); };
    L.gnst = 1;
    if (fixed + gu_region(1) + L.dstage > budget) return false;
    L.dnst = static_cast<int>(std::min<size_t>({static_cast<size_t>(want_d), 71,
                                                (budget - fixed - gu_region(1)) / L.dstage}));
    while (L.gnst < std::min(per_cta, 8) &&
           fixed + gu_region(L.gnst + 1) + static_cast<size_t>(L.dnst) * L.dstage <= budget)
        ++L.gnst;
    L.off_gu = static_cast<uint32_t>(fixed);
    L.off_dn = static_cast<uint32_t>(fixed + align_up(gu_region(L.gnst), 128));
    smem = L.off_dn + static_cast<size_t>(L.dnst) * L.dstage;
    return smem <= budget;
}

typedef void (*FxKern)(DecodeParams, FxLayout);

// (gate/up, shared gate/up, down, shared down) type combinations with a fused
// instance; other combinations run the two-kernel path
static FxKern pick_fused(int tr, int ts, int dr, int ds) {
#define QMOE_FX(A, B, C, D) \
    if (tr == A && ts == B && dr == C && ds == D) return k_experts<A, B, C, D>;
    QMOE_FX(12, 12, 12, 12)
    QMOE_FX(13, 13, 13, 13)
    QMOE_FX(14, 14, 14, 14)
    QMOE_FX(8, 8, 8, 8)
    QMOE_FX(12, 8, 14, 8)
    QMOE_FX(12, 8, 12, 8)
    QMOE_FX(13, 8, 14, 8)
    QMOE_FX(12, 12, 14, 14)
    QMOE_FX(12, 12, 14, 12)
#undef QMOE_FX
    return nullptr;
}

// The fused kernel's grid barrier needs every CTA resident at once: it is
// used only when the device supports cooperative launches and its occupancy
// holds the whole grid (it is then launched cooperatively, so the driver
// refuses rather than runs it when the SMs are not available).
static bool fused_fits(FxKern kern, size_t smem, int grid) {
    int dev = 0, coop = 0, per_sm = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return false;
    if (cudaDeviceGetAttribute(&coop, cudaDevAttrCooperativeLaunch, dev) != cudaSuccess || !coop) return false;
    if (set_smem(kern, smem) != cudaSuccess) return false;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, FX_THREADS, smem) != cudaSuccess) return false;
    return per_sm * dev_cache().sms >= grid;
}

bool fused_supported(const DecodeParams& P) {
    FxLayout L;
    size_t smem;
    int grid;
    FxKern kern = pick_fused(P.gate.type, P.sgate.type, P.down.type, P.sdown.type);
    return kern && plan_fused(P, L, smem, grid) && fused_fits(kern, smem, grid);
}

cudaError_t launch_experts(const DecodeParams& P, cudaStream_t s) {
    FxLayout L;
    size_t smem;
    int grid;
    FxKern kern = pick_fused(P.gate.type, P.sgate.type, P.down.type, P.sdown.type);
    if (!kern || !plan_fused(P, L, smem, grid)) return cudaErrorInvalidValue;
    cudaError_t e = set_smem(kern, smem);
    if (e != cudaSuccess) return e;
    // cooperative: all CTAs are resident together (the grid barrier's
    // requirement) or the launch is refused
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(FX_THREADS);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = dev_cache().pdl ? 2 : 1;
    return cudaLaunchKernelEx(&cfg, kern, P, L);
}

cudaError_t launch_down(const DecodeParams& P, cudaStream_t s) {
    DnPlan p;
    if (!plan_down(P, p)) return cudaErrorInvalidValue;
    auto kern = pick<DnSel>(P.down.type, P.sdown.type);
    if (!kern) return cudaErrorInvalidValue;
    cudaError_t e = set_smem(kern, p.smem);
    if (e != cudaSuccess) return e;
    return launch(kern, p.grid, XK_THREADS, p.smem, s, P, p.nst, p.Rd, p.stage_bytes, p.nvec);
}

}  // namespace qmoe
