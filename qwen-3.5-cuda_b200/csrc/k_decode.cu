// Decode-path kernels of the MoE block (T <= kDecodeMaxT tokens per launch).
//
//   k_router   router logits in the reference's exact F32 reduction order
//              (src/cuda/matmul_q4.cu:140-167), the shared-expert gate logit,
//              24-bit activation planes of x, then -- in the last CTA to
//              finish -- top-k + softmax over the selected logits
//              (src/cuda/moe.cu:7-52), the host checks of
//              src/layer_moe.cpp:114-124 as a device error word, and the
//              stable token->expert permutation.
//   k_gateup   gate and up rows of every active expert and of the shared
//              expert, staged into shared memory with 1-D bulk copies (TMA)
//              from the GGUF payload in place, dp4a dot products against the
//              activation planes, silu(g)*u (src/cuda/moe.cu:61-67), and the
//              24-bit planes of the result.
//   k_down     down rows of every active expert and the shared expert for a
//              slice of output rows, then the combine in selection order
//              j = 0..k-1 (src/cuda/moe.cu:76-81) and the sigmoid-gated
//              shared expert (src/cuda/moe.cu:90-96), optional residual.
#include "qmoe_dev.cuh"
#include "qmoe_units.cuh"
#include "qmoe_internal.h"

namespace qmoe {

constexpr unsigned FULL = 0xffffffffu;

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

// One logit with the reference's order.  Lane L plays the 8 "threads"
// t = 4L + c + 128h (c = 0..3, h = 0..1) of the reference's 256-thread block:
// each keeps the fmaf chain over k = t, t+256, ...  The reference's warp
// w' = L/8 + 4h holds these values at positions 4*(L%8) + c, so its shuffle
// tree (offsets 16, 8, 4, 2, 1) is shuffles by 4, 2, 1 lanes followed by the
// in-lane pairs (c, c+2), (c, c+1).  Warp 0's final tree over the 8 warp
// sums p0..p7 (lanes 8..31 zero) is ((q0+q4)+(q2+q6))+((q1+q5)+(q3+q7)) with
// q = (p + 0) + 0.  Valid in lane 0.
template <int CH>
__device__ __forceinline__ float router_dot(const float4 (&w)[CH][2], const float* x, int lane) {
    float acc[2][4];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) acc[hh][c] = 0.0f;
#pragma unroll
    for (int i = 0; i < CH; ++i)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const float4 xv = __ldg(reinterpret_cast<const float4*>(x + 256 * i + 128 * hh + 4 * lane));
            acc[hh][0] = __fmaf_rn(w[i][hh].x, xv.x, acc[hh][0]);
            acc[hh][1] = __fmaf_rn(w[i][hh].y, xv.y, acc[hh][1]);
            acc[hh][2] = __fmaf_rn(w[i][hh].z, xv.z, acc[hh][2]);
            acc[hh][3] = __fmaf_rn(w[i][hh].w, xv.w, acc[hh][3]);
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

__device__ __forceinline__ int router_esize(int type) { return type == T_F32 ? 4 : 2; }

// Top-k + softmax + validation for every token, then the permutation.
// Runs in the single CTA that finished the router last (RT_WARPS warps).
__device__ void topk_and_dispatch(const DecodeParams& P) {
    __shared__ int s_cnt[kMaxExperts];
    __shared__ int s_cur[kMaxExperts];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int E = P.E, k = P.k, LS = E + 1;

    for (int t = warp; t < P.T; t += RT_WARPS) {
        float v[8];
        bool finite = true;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = lane + 32 * i;
            v[i] = e < E ? __ldcg(P.logits + t * LS + e) : -INFINITY;
            if (e < E && !isfinite(v[i])) finite = false;
        }
        finite = __all_sync(FULL, finite);
        uint32_t used = 0;
        int my_idx = -1;
        float my_v = 0.0f;
        if (finite) {
            for (int j = 0; j < k; ++j) {
                float bv = -INFINITY;
                int bi = 0x7fffffff;
#pragma unroll
                for (int i = 0; i < 8; ++i) {
                    const int e = lane + 32 * i;
                    if (e < E && !((used >> i) & 1u) && v[i] > bv) { bv = v[i]; bi = e; }
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) {
                    const float ov = __shfl_xor_sync(FULL, bv, o);
                    const int oi = __shfl_xor_sync(FULL, bi, o);
                    if (ov > bv || (ov == bv && oi < bi)) { bv = ov; bi = oi; }
                }
                if ((bi & 31) == lane) used |= 1u << (bi >> 5);
                if (lane == j) { my_idx = bi; my_v = bv; }
            }
        }
        // softmax over the selected logits (moe.cu:41-51): max, then a
        // sequential sum j = 0..k-1, then division
        float mx = __shfl_sync(FULL, my_v, 0);
        for (int j = 1; j < k; ++j) mx = fmaxf(mx, __shfl_sync(FULL, my_v, j));
        const float ex = (lane < k) ? expf(my_v - mx) : 0.0f;
        float sum = 0.0f;
        for (int j = 0; j < k; ++j) sum += __shfl_sync(FULL, ex, j);
        const float wj = ex / sum;
        // host-side checks of layer_moe.cpp:114-124, on the device
        bool ok = finite;
        float rs = 0.0f;
        for (int j = 0; j < k; ++j) {
            const float w = __shfl_sync(FULL, wj, j);
            const int id = __shfl_sync(FULL, my_idx, j);
            ok = ok && id >= 0 && id < E && isfinite(w) && w >= 0.0f;
            rs += w;
        }
        uint32_t flag = 0;
        if (!ok) flag = EF_ROUTING;
        else if (!isfinite(rs) || fabsf(rs - 1.0f) > 1e-4f) flag = EF_NOT_NORMALIZED;
        if (flag && lane == 0) {
            atomicOr(P.ctrl + CTRL_ERROR, flag);
            atomicMin(P.ctrl + CTRL_ERR_TOKEN, static_cast<uint32_t>(t));
        }
        if (lane < k) {
            const int oi = flag ? -1 : my_idx;
            const float ow = flag ? __uint_as_float(0x7FC00000u) : wj;
            P.topk_idx[t * k + lane] = oi;
            P.topk_w[t * k + lane] = ow;
            if (P.out_idx) P.out_idx[t * k + lane] = oi;
            if (P.out_w) P.out_w[t * k + lane] = ow;
        }
    }
    __syncthreads();

    // ---- stable permutation: pairs p = t*k + j sorted by (expert, t, j) ----
    const int NP = P.T * k;
    for (int e = threadIdx.x; e < E; e += blockDim.x) s_cnt[e] = 0;
    __syncthreads();
    for (int p = threadIdx.x; p < NP; p += blockDim.x) {
        const int e = P.topk_idx[p];
        if (e >= 0 && e < E) atomicAdd(&s_cnt[e], 1);
    }
    __syncthreads();
    if (warp == 0) {
        // experts [8*lane, 8*lane+8): exclusive scan of counts and of "active"
        int c[8], loc = 0, nz = 0;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = 8 * lane + i;
            c[i] = e < E ? s_cnt[e] : 0;
            loc += c[i];
            nz += c[i] > 0;
        }
        int inc = loc, incz = nz;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int a = __shfl_up_sync(FULL, inc, o), b = __shfl_up_sync(FULL, incz, o);
            if (lane >= o) { inc += a; incz += b; }
        }
        int off = inc - loc, pos = incz - nz;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const int e = 8 * lane + i;
            if (e < E) {
                P.offsets[e] = off;
                s_cur[e] = off;
                if (c[i] > 0) P.active[pos++] = e;
            }
            off += c[i];
        }
        if (lane == 31) {
            P.offsets[E] = inc;
            P.ctrl[CTRL_N_PAIRS] = static_cast<uint32_t>(inc);
            P.ctrl[CTRL_N_ACTIVE] = static_cast<uint32_t>(incz);
        }
    }
    __syncthreads();
    if (warp == 0) {
        const unsigned lt = (1u << lane) - 1u;
        for (int base = 0; base < NP; base += 32) {
            const int p = base + lane;
            const int e = p < NP ? P.topk_idx[p] : -1;
            const bool valid = e >= 0 && e < E;
            const unsigned peers = __match_any_sync(FULL, valid ? e : -1);
            const int rank = __popc(peers & lt);
            const int pos = valid ? s_cur[e] + rank : -1;
            __syncwarp();
            const bool top = (peers >> lane) == 1u;
            if (valid && top) s_cur[e] += __popc(peers);
            __syncwarp();
            if (p < NP) {
                if (valid) P.perm[pos] = p;
                P.inv_perm[p] = pos;
            }
        }
    }
}

template <int CH>
__global__ void __launch_bounds__(RT_WARPS * 32) k_router(DecodeParams P) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int gw = blockIdx.x * RT_WARPS + warp, nw = gridDim.x * RT_WARPS;
    const int nrows = P.E + (P.has_shared ? 1 : 0);
    const int LS = P.E + 1;

    for (int r = gw; r < nrows; r += nw) {
        const uint8_t* row;
        int type;
        if (r < P.E) {
            type = P.router_type;
            row = P.router + static_cast<size_t>(r) * P.d * router_esize(type);
        } else {
            type = P.sgate_type;
            row = P.sgate_inp;
        }
        float4 w[CH][2];
        load_router_row<CH>(w, row, type, lane);
        for (int t = 0; t < P.T; ++t) {
            float v = router_dot<CH>(w, P.x + static_cast<size_t>(t) * P.d, lane);
            if (lane == 0) {
                if (r < P.E && P.bias) v = __fadd_rn(v, P.bias[r]);
                P.logits[t * LS + r] = v;
            }
        }
    }

    // 24-bit planes of x for the expert kernels
    const int nb = P.d / 32;
    for (int task = gw; task < P.T * nb; task += nw) {
        const int t = task / nb, b = task % nb;
        const float v = P.x[static_cast<size_t>(t) * P.d + 32 * b + lane];
        uint8_t* base = P.xq + static_cast<size_t>(t) * P.xq_stride;
        xq_block32(v, base + 32 * b + lane, base + P.d + 32 * b + lane, base + 2 * P.d + 32 * b + lane,
                   reinterpret_cast<float2*>(base + 3 * P.d) + 2 * b, lane);
    }

    // last CTA to arrive selects the experts (threadfence reduction pattern)
    __shared__ int s_last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        const unsigned old = atomicAdd(P.ctrl + CTRL_ARRIVE, 1u);
        s_last = (old == gridDim.x - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    topk_and_dispatch(P);
    if (threadIdx.x == 0) P.ctrl[CTRL_ARRIVE] = 0;
}

// ---------------------------------------------------------------------------
// Expert gate/up
// ---------------------------------------------------------------------------
constexpr int NCW = 8;                    // consumer warps
constexpr int XK_THREADS = (NCW + 1) * 32; // + one producer warp
constexpr int MAXCH = 128;

struct Chunk {
    int src;    // source index (== n_active: shared expert)
    int r0;     // first row inside the source
    int n;      // rows
    int task0;  // first task index
    int rflat;  // flattened row index of r0
    int ntok;
    int steps;
    int pad;
};

struct SrcInfo {
    int expert;   // -1 for the shared expert
    int ntok;
    int pair0;    // first permuted position (routed)
};

__device__ __forceinline__ SrcInfo src_info(const DecodeParams& P, int s, int n_active) {
    SrcInfo si;
    if (s < n_active) {
        si.expert = P.active[s];
        si.pair0 = P.offsets[si.expert];
        si.ntok = P.offsets[si.expert + 1] - si.pair0;
    } else {
        si.expert = -1;
        si.pair0 = 0;
        si.ntok = P.T;
    }
    return si;
}

__device__ __forceinline__ float silu_mul(float g, float u) {
    const float s = g / (1.0f + expf(-g));  // moe.cu:64
    return s * u;
}

__device__ __forceinline__ XPlanesView planes_view(const uint8_t* base, int K) {
    XPlanesView v;
    v.p0 = base;
    v.p1 = base + K;
    v.p2 = base + 2 * K;
    v.meta = reinterpret_cast<const float2*>(base + 3 * K);
    return v;
}

struct StagePlan {
    const uint8_t* lo;
    uint32_t tx;
    uint32_t skew;
};

// Plans (and performs the unaligned tail of) a copy of [src, src+bytes) into dst.
__device__ __forceinline__ StagePlan plan_stage(uint8_t* dst, const uint8_t* src, uint64_t bytes, const uint8_t* limit) {
    StagePlan sp;
    const uintptr_t s = reinterpret_cast<uintptr_t>(src);
    const uintptr_t lo = s & ~static_cast<uintptr_t>(15);
    const uintptr_t hi = (s + bytes + 15) & ~static_cast<uintptr_t>(15);
    const uintptr_t lim = reinterpret_cast<uintptr_t>(limit);
    const uintptr_t hi_full = hi <= lim ? hi : (lim & ~static_cast<uintptr_t>(15));
    sp.lo = reinterpret_cast<const uint8_t*>(lo);
    sp.skew = static_cast<uint32_t>(s - lo);
    sp.tx = hi_full > lo ? static_cast<uint32_t>(hi_full - lo) : 0u;
    for (uintptr_t a = (hi_full > lo ? hi_full : lo); a < s + bytes; ++a)
        dst[a - lo] = *reinterpret_cast<const uint8_t*>(a);
    return sp;
}

struct GateUpSmem {
    uint64_t* full;
    uint64_t* empty;
    uint64_t* xbar;
    Chunk* chunks;
    int* misc;  // [0] nch, [1] ntask, [2] R0, [3] R1, [4] n_active
    uint8_t* xs;
    float* hbuf;
    uint8_t* stages;
};

__global__ void __launch_bounds__(XK_THREADS, 1)
    k_gateup(DecodeParams P, int nst, int ch_rows, uint32_t half_bytes, int hbuf_rows) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int d = P.d, U = d / 64, RPS = 32 / U;
    GateUpSmem S;
    S.full = reinterpret_cast<uint64_t*>(smem);
    S.empty = S.full + 32;
    S.xbar = S.empty + 32;
    S.misc = reinterpret_cast<int*>(smem + 528);
    S.chunks = reinterpret_cast<Chunk*>(smem + 576);
    S.xs = smem + 576 + MAXCH * sizeof(Chunk);
    const size_t xs_bytes = P.xq_stride * P.T;
    S.hbuf = reinterpret_cast<float*>(S.xs + xs_bytes);
    S.stages = reinterpret_cast<uint8_t*>(S.hbuf) + align_up(static_cast<size_t>(hbuf_rows) * P.T * 4, 128);

    if (threadIdx.x == 0) {
        const int n_active = static_cast<int>(P.ctrl[CTRL_N_ACTIVE]);
        const int rows_tot = n_active * P.F + (P.has_shared ? P.Fs : 0);
        const int per = 32 * ((rows_tot + 32 * gridDim.x - 1) / (32 * gridDim.x));
        const int R0 = blockIdx.x * per;
        const int R1 = min(R0 + per, rows_tot);
        int nch = 0, ntask = 0;
        for (int r = R0; r < R1 && nch < MAXCH;) {
            int s, rr, rows;
            if (r < n_active * P.F) { s = r / P.F; rr = r % P.F; rows = P.F; }
            else { s = n_active; rr = r - n_active * P.F; rows = P.Fs; }
            const int n = min(min(ch_rows, R1 - r), rows - rr);
            const SrcInfo si = src_info(P, s, n_active);
            Chunk c;
            c.src = s; c.r0 = rr; c.n = n; c.task0 = ntask; c.rflat = r;
            c.ntok = si.ntok; c.steps = (n + RPS - 1) / RPS; c.pad = 0;
            S.chunks[nch++] = c;
            ntask += c.ntok * c.steps;
            r += n;
        }
        S.misc[0] = nch; S.misc[1] = ntask; S.misc[2] = R0; S.misc[3] = R1; S.misc[4] = n_active;
        for (int i = 0; i < nst; ++i) { mbar_init(S.full + i, 1); mbar_init(S.empty + i, NCW); }
        mbar_init(S.xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int nch = S.misc[0], ntask = S.misc[1], R0 = S.misc[2], R1 = S.misc[3], n_active = S.misc[4];
    if (R0 >= R1) return;

    const uint64_t rbg = row_bytes(P.gate.type, d), rbs = row_bytes(P.sgate.type, d);

    if (warp == NCW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            mbar_arrive_expect_tx(S.xbar, static_cast<uint32_t>(xs_bytes));
            bulk_g2s(S.xs, P.xq, static_cast<uint32_t>(xs_bytes), S.xbar);
            for (int c = 0; c < nch; ++c) {
                const int slot = c % nst;
                if (c >= nst) mbar_wait(S.empty + slot, ((c / nst) - 1) & 1, P.ctrl);
                const Chunk ck = S.chunks[c];
                const uint8_t *gsrc, *usrc, *gend, *uend;
                uint64_t rb;
                if (ck.src < n_active) {
                    const int e = P.active[ck.src];
                    rb = rbg;
                    gsrc = P.gate.p + (static_cast<uint64_t>(e) * P.F + ck.r0) * rbg;
                    usrc = P.up.p + (static_cast<uint64_t>(e) * P.F + ck.r0) * rbg;
                    gend = P.gate.end; uend = P.up.end;
                } else {
                    rb = rbs;
                    gsrc = P.sgate.p + static_cast<uint64_t>(ck.r0) * rbs;
                    usrc = P.sup.p + static_cast<uint64_t>(ck.r0) * rbs;
                    gend = P.sgate.end; uend = P.sup.end;
                }
                uint8_t* dg = S.stages + static_cast<size_t>(slot) * 2 * half_bytes;
                uint8_t* du = dg + half_bytes;
                const StagePlan pg = plan_stage(dg, gsrc, ck.n * rb, gend);
                const StagePlan pu = plan_stage(du, usrc, ck.n * rb, uend);
                mbar_arrive_expect_tx(S.full + slot, pg.tx + pu.tx);
                if (pg.tx) bulk_g2s(dg, pg.lo, pg.tx, S.full + slot);
                if (pu.tx) bulk_g2s(du, pu.lo, pu.tx, S.full + slot);
            }
        }
        return;
    }

    // ---------------- consumers ----------------
    mbar_wait(S.xbar, 0, P.ctrl);
    const int t_lo = (warp * ntask) / NCW, t_hi = ((warp + 1) * ntask) / NCW;
    const int u = lane % U, rsub = lane / U;
    XU xr;
    int cur_key = -1;
    for (int c = 0; c < nch; ++c) {
        const int slot = c % nst;
        mbar_wait(S.full + slot, (c / nst) & 1, P.ctrl);
        const Chunk ck = S.chunks[c];
        const int c_lo = max(t_lo, ck.task0), c_hi = min(t_hi, ck.task0 + ck.ntok * ck.steps);
        if (c_lo < c_hi) {
            const bool routed = ck.src < n_active;
            const int type = routed ? P.gate.type : P.sgate.type;
            const uint64_t rb = routed ? rbg : rbs;
            const SrcInfo si = src_info(P, ck.src, n_active);
            const uint8_t* dg = S.stages + static_cast<size_t>(slot) * 2 * half_bytes;
            const uint8_t* du = dg + half_bytes;
            const uint32_t skg = static_cast<uint32_t>(
                reinterpret_cast<uintptr_t>(routed ? P.gate.p + (static_cast<uint64_t>(si.expert) * P.F + ck.r0) * rbg
                                                   : P.sgate.p + static_cast<uint64_t>(ck.r0) * rbs) & 15u);
            const uint32_t sku = static_cast<uint32_t>(
                reinterpret_cast<uintptr_t>(routed ? P.up.p + (static_cast<uint64_t>(si.expert) * P.F + ck.r0) * rbg
                                                   : P.sup.p + static_cast<uint64_t>(ck.r0) * rbs) & 15u);
            for (int tau = c_lo; tau < c_hi; ++tau) {
                const int tl = tau - ck.task0;
                const int ti = tl / ck.steps, st = tl % ck.steps;
                const int tok = routed ? P.perm[si.pair0 + ti] / P.k : ti;
                const int key = tok * 64 + type;
                if (key != cur_key) {
                    load_xu(xr, planes_view(S.xs + static_cast<size_t>(tok) * P.xq_stride, d), type, u);
                    cur_key = key;
                }
                const int rl = st * RPS + rsub;  // row inside the chunk
                const bool valid = rl < ck.n;
                float g = 0.0f, up = 0.0f;
                if (valid) {
                    g = unit_dot(type, dg + skg + rl * rb, u, xr);
                    up = unit_dot(type, du + sku + rl * rb, u, xr);
                }
                for (int o = U / 2; o; o >>= 1) {
                    g += __shfl_xor_sync(FULL, g, o);
                    up += __shfl_xor_sync(FULL, up, o);
                }
                if (valid && u == 0)
                    S.hbuf[static_cast<size_t>(ck.rflat - R0 + rl) * P.T + ti] = silu_mul(g, up);
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(S.empty + slot);
    }
    // all consumer warps done with hbuf
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");

    // planes of silu(g)*u per 32-row block, and the F32 values
    const int nblk = (R1 - R0) / 32;
    for (int task = warp; task < nblk * P.T; task += NCW) {
        const int blk = task / P.T, ti = task % P.T;
        const int rf = R0 + 32 * blk;
        int s, rr;
        if (rf < n_active * P.F) { s = rf / P.F; rr = rf % P.F; }
        else { s = n_active; rr = rf - n_active * P.F; }
        const SrcInfo si = src_info(P, s, n_active);
        if (ti >= si.ntok) continue;
        const int vid = s < n_active ? P.perm[si.pair0 + ti] : P.T * P.k + ti;
        const float v = S.hbuf[static_cast<size_t>(32 * blk + lane) * P.T + ti];
        P.hidden[static_cast<size_t>(vid) * P.H + rr + lane] = v;
        uint8_t* base = P.hq + static_cast<size_t>(vid) * P.hq_stride;
        xq_block32(v, base + rr + lane, base + P.H + rr + lane, base + 2 * P.H + rr + lane,
                   reinterpret_cast<float2*>(base + 3 * P.H) + rr / 16, lane);
    }
}

// ---------------------------------------------------------------------------
// Expert down + combine
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(XK_THREADS, 1)
    k_down(DecodeParams P, int nst, int Rd, uint32_t stage_bytes, int nvec) {
    extern __shared__ __align__(128) uint8_t smem[];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + 64;
    uint64_t* hbar = empty + 64;
    int* misc = reinterpret_cast<int*>(smem + 1040);
    uint8_t* hs = smem + 1088;
    const size_t hs_bytes = P.hq_stride * static_cast<size_t>(nvec);
    float* ybuf = reinterpret_cast<float*>(hs + hs_bytes);
    uint8_t* stages = reinterpret_cast<uint8_t*>(ybuf) + align_up(static_cast<size_t>(nvec) * Rd * 4, 128);

    const int r0 = blockIdx.x * Rd;
    const int nrow = min(Rd, P.d - r0);
    if (threadIdx.x == 0) {
        misc[0] = static_cast<int>(P.ctrl[CTRL_N_ACTIVE]);
        for (int i = 0; i < nst; ++i) { mbar_init(full + i, 1); mbar_init(empty + i, NCW); }
        mbar_init(hbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const int n_active = misc[0];
    const int nsrc = n_active + (P.has_shared ? 1 : 0);
    if (nrow <= 0) return;
    const uint64_t rbd = row_bytes(P.down.type, P.F), rbs = row_bytes(P.sdown.type, P.Fs);

    if (warp == NCW) {
        if (lane == 0) {
            mbar_arrive_expect_tx(hbar, static_cast<uint32_t>(hs_bytes));
            bulk_g2s(hs, P.hq, static_cast<uint32_t>(hs_bytes), hbar);
            for (int c = 0; c < nsrc; ++c) {
                const int slot = c % nst;
                if (c >= nst) mbar_wait(empty + slot, ((c / nst) - 1) & 1, P.ctrl);
                const uint8_t *src, *end;
                uint64_t rb;
                if (c < n_active) {
                    const int e = P.active[c];
                    rb = rbd;
                    src = P.down.p + (static_cast<uint64_t>(e) * P.d + r0) * rbd;
                    end = P.down.end;
                } else {
                    rb = rbs;
                    src = P.sdown.p + static_cast<uint64_t>(r0) * rbs;
                    end = P.sdown.end;
                }
                uint8_t* dst = stages + static_cast<size_t>(slot) * stage_bytes;
                const StagePlan sp = plan_stage(dst, src, nrow * rb, end);
                mbar_arrive_expect_tx(full + slot, sp.tx);
                if (sp.tx) bulk_g2s(dst, sp.lo, sp.tx, full + slot);
            }
        }
        return;
    }

    mbar_wait(hbar, 0, P.ctrl);
    // tasks: (source, token, step), enumerated source-major; contiguous per warp
    int ntask = 0;
    for (int c = 0; c < nsrc; ++c) {
        const bool routed = c < n_active;
        const int K = routed ? P.F : P.Fs;
        const int rps = 32 / (K / 64);
        const SrcInfo si = src_info(P, c, n_active);
        ntask += si.ntok * ((nrow + rps - 1) / rps);
    }
    const int t_lo = (warp * ntask) / NCW, t_hi = ((warp + 1) * ntask) / NCW;
    XU xr;
    int cur_vid = -1;
    int task0 = 0;
    for (int c = 0; c < nsrc; ++c) {
        const int slot = c % nst;
        const bool routed = c < n_active;
        const int K = routed ? P.F : P.Fs;
        const int U = K / 64, rps = 32 / U;
        const int steps = (nrow + rps - 1) / rps;
        const SrcInfo si = src_info(P, c, n_active);
        const int nt = si.ntok * steps;
        mbar_wait(full + slot, (c / nst) & 1, P.ctrl);
        const int c_lo = max(t_lo, task0), c_hi = min(t_hi, task0 + nt);
        if (c_lo < c_hi) {
            const int type = routed ? P.down.type : P.sdown.type;
            const uint64_t rb = routed ? rbd : rbs;
            const uint8_t* src = routed ? P.down.p + (static_cast<uint64_t>(si.expert) * P.d + r0) * rbd
                                        : P.sdown.p + static_cast<uint64_t>(r0) * rbs;
            const uint8_t* wbase = stages + static_cast<size_t>(slot) * stage_bytes +
                                   (reinterpret_cast<uintptr_t>(src) & 15u);
            const int u = lane % U, rsub = lane / U;
            for (int tau = c_lo; tau < c_hi; ++tau) {
                const int tl = tau - task0;
                const int ti = tl / steps, st = tl % steps;
                const int vid = routed ? P.perm[si.pair0 + ti] : P.T * P.k + ti;
                if (vid != cur_vid) {
                    load_xu(xr, planes_view(hs + static_cast<size_t>(vid) * P.hq_stride, P.H), type, u);
                    cur_vid = vid;
                }
                const int rl = st * rps + rsub;
                const bool valid = rl < nrow;
                float y = valid ? unit_dot(type, wbase + rl * rb, u, xr) : 0.0f;
                for (int o = U / 2; o; o >>= 1) y += __shfl_xor_sync(FULL, y, o);
                if (valid && u == 0) ybuf[static_cast<size_t>(vid) * Rd + rl] = y;
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        task0 += nt;
    }
    asm volatile("bar.sync 1, %0;" ::"r"(NCW * 32) : "memory");

    // combine (moe.cu:76-81 and :90-96, accumulation order of layer_moe.cpp:127-153)
    const int LS = P.E + 1;
    for (int idx = threadIdx.x; idx < P.T * nrow; idx += NCW * 32) {
        const int t = idx / nrow, r = idx % nrow;
        float acc = 0.0f;
        const bool bad = P.topk_idx[t * P.k] < 0;
        for (int j = 0; j < P.k; ++j) acc = fmaf(P.topk_w[t * P.k + j], ybuf[static_cast<size_t>(t * P.k + j) * Rd + r], acc);
        if (P.has_shared) {
            const float sg = 1.0f / (1.0f + expf(-P.logits[t * LS + P.E]));
            acc = fmaf(ybuf[static_cast<size_t>(P.T * P.k + t) * Rd + r], sg, acc);
        }
        if (bad) acc = __uint_as_float(0x7FC00000u);
        const size_t o = static_cast<size_t>(t) * P.d + r0 + r;
        P.out[o] = P.residual ? P.residual[o] + acc : acc;
    }
}

// ---------------------------------------------------------------------------
// Host launchers
// ---------------------------------------------------------------------------
namespace {
struct DevCache {
    int sms = 0;
    int smem_optin = 0;
    bool attr_gu = false, attr_dn = false;
};
DevCache g_dev[64];

DevCache& dev_cache() {
    int dev = 0;
    cudaGetDevice(&dev);
    DevCache& c = g_dev[dev & 63];
    if (!c.sms) {
        cudaDeviceGetAttribute(&c.sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&c.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    }
    return c;
}
}  // namespace

int decode_num_sms() { return dev_cache().sms; }

cudaError_t launch_router(const DecodeParams& P, cudaStream_t s) {
    const int nrows = P.E + (P.has_shared ? 1 : 0);
    const int grid = (nrows + RT_WARPS - 1) / RT_WARPS;
    switch (P.d / 256) {
        case 1: k_router<1><<<grid, RT_WARPS * 32, 0, s>>>(P); break;
        case 2: k_router<2><<<grid, RT_WARPS * 32, 0, s>>>(P); break;
        case 4: k_router<4><<<grid, RT_WARPS * 32, 0, s>>>(P); break;
        case 8: k_router<8><<<grid, RT_WARPS * 32, 0, s>>>(P); break;
        case 16: k_router<16><<<grid, RT_WARPS * 32, 0, s>>>(P); break;
        default: return cudaErrorInvalidValue;
    }
    return cudaGetLastError();
}

// Shared-memory plan of k_gateup for this launch.
struct GuPlan { int grid, nst, ch_rows, hbuf_rows; uint32_t half_bytes; size_t smem; };

static bool plan_gateup(const DecodeParams& P, GuPlan& g) {
    DevCache& dc = dev_cache();
    const int U = P.d / 64;
    g.grid = dc.sms;
    g.ch_rows = (32 / U) * NCW;
    const uint64_t rb = std::max(row_bytes(P.gate.type, P.d), row_bytes(P.sgate.type, P.d));
    g.half_bytes = static_cast<uint32_t>(align_up(g.ch_rows * rb + 32, 128));
    const int umax = std::min(P.T * P.k, P.E);
    const int rows_tot = umax * P.F + (P.has_shared ? P.Fs : 0);
    g.hbuf_rows = 32 * ((rows_tot + 32 * g.grid - 1) / (32 * g.grid));
    const int nch_max = g.hbuf_rows / g.ch_rows + 2 + g.hbuf_rows / std::min(P.F, P.has_shared ? P.Fs : P.F) + 2;
    if (nch_max > MAXCH) return false;
    const size_t fixed = 576 + MAXCH * sizeof(Chunk) + P.xq_stride * P.T +
                         align_up(static_cast<size_t>(g.hbuf_rows) * P.T * 4, 128);
    const size_t budget = static_cast<size_t>(dc.smem_optin) - 1024;
    if (fixed + 2 * 2 * g.half_bytes > budget) return false;
    g.nst = static_cast<int>(std::min<size_t>(std::min<size_t>(nch_max, 32), (budget - fixed) / (2 * g.half_bytes)));
    if (g.nst < 2) g.nst = 2;
    g.smem = fixed + static_cast<size_t>(g.nst) * 2 * g.half_bytes;
    return true;
}

struct DnPlan { int grid, nst, Rd, nvec; uint32_t stage_bytes; size_t smem; };

static bool plan_down(const DecodeParams& P, DnPlan& p) {
    DevCache& dc = dev_cache();
    p.Rd = (P.d + dc.sms - 1) / dc.sms;
    p.grid = (P.d + p.Rd - 1) / p.Rd;
    p.nvec = P.T * P.k + P.T;
    const uint64_t rb = std::max(row_bytes(P.down.type, P.F), row_bytes(P.sdown.type, P.Fs));
    p.stage_bytes = static_cast<uint32_t>(align_up(p.Rd * rb + 32, 128));
    const size_t fixed = 1088 + P.hq_stride * p.nvec + align_up(static_cast<size_t>(p.nvec) * p.Rd * 4, 128);
    const size_t budget = static_cast<size_t>(dc.smem_optin) - 1024;
    if (fixed + 2 * p.stage_bytes > budget) return false;
    const int nsrc_max = std::min(P.T * P.k, P.E) + 1;
    p.nst = static_cast<int>(std::min<size_t>(std::min<size_t>(nsrc_max, 64), (budget - fixed) / p.stage_bytes));
    if (p.nst < 2) p.nst = 2;
    p.smem = fixed + static_cast<size_t>(p.nst) * p.stage_bytes;
    return true;
}

bool decode_supported(const DecodeParams& P) {
    GuPlan g;
    DnPlan dn;
    return plan_gateup(P, g) && plan_down(P, dn);
}

cudaError_t launch_gateup(const DecodeParams& P, cudaStream_t s) {
    GuPlan g;
    if (!plan_gateup(P, g)) return cudaErrorInvalidValue;
    DevCache& dc = dev_cache();
    if (!dc.attr_gu) {
        cudaError_t e = cudaFuncSetAttribute(k_gateup, cudaFuncAttributeMaxDynamicSharedMemorySize, dc.smem_optin);
        if (e != cudaSuccess) return e;
        dc.attr_gu = true;
    }
    k_gateup<<<g.grid, XK_THREADS, g.smem, s>>>(P, g.nst, g.ch_rows, g.half_bytes, g.hbuf_rows);
    return cudaGetLastError();
}

cudaError_t launch_down(const DecodeParams& P, cudaStream_t s) {
    DnPlan p;
    if (!plan_down(P, p)) return cudaErrorInvalidValue;
    DevCache& dc = dev_cache();
    if (!dc.attr_dn) {
        cudaError_t e = cudaFuncSetAttribute(k_down, cudaFuncAttributeMaxDynamicSharedMemorySize, dc.smem_optin);
        if (e != cudaSuccess) return e;
        dc.attr_dn = true;
    }
    k_down<<<p.grid, XK_THREADS, p.smem, s>>>(P, p.nst, p.Rd, p.stage_bytes, p.nvec);
    return cudaGetLastError();
}

}  // namespace qmoe
