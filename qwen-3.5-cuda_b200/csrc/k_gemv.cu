// General quantised GEMV and row dequantisation: the replacement of the
// reference's matmul_dispatch / dequantize_row (src/cuda/matmul_q4.cu:140-227)
// for its non-MoE callers (attention, GDN, LM head, embedding).
//
// One warp per output row.  Lane L plays the reference's threads
// t = 4L + c + 128h of its 256-thread block (c = 0..3, h = 0..1): it decodes
// the 4 consecutive elements k0 = 256i + 128h + 4L .. k0+3 of each 256-wide
// chunk i, keeps one fmaf chain per thread over i in ascending order, and the
// warp then evaluates the reference's shuffle trees exactly (see k_router).
// Element values use the reference's dequantisation formulas per type.
#include "qmoe_dev.cuh"
#include "qmoe_units.cuh"
#include "qmoe_internal.h"
#include "qmoe_dq1.cuh"

#include <algorithm>

namespace qmoe {

constexpr unsigned GFULL = 0xffffffffu;

constexpr int GV_WARPS = 4;

__global__ void __launch_bounds__(GV_WARPS * 32)
    k_gemv(const uint8_t* __restrict__ w, int type, const float* __restrict__ x, float* __restrict__ y, int M, int K,
           uint64_t element_offset) {
    const int lane = threadIdx.x & 31;
    const int row = blockIdx.x * GV_WARPS + (threadIdx.x >> 5);
    if (row >= M) return;  // whole warp leaves together
    const uint64_t base = element_offset + static_cast<uint64_t>(row) * K;
    float acc[2][4] = {{0.f, 0.f, 0.f, 0.f}, {0.f, 0.f, 0.f, 0.f}};
    const int nchunk = (K + 255) / 256;
    for (int i = 0; i < nchunk; ++i) {
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
            const int k0 = 256 * i + 128 * hh + 4 * lane;
#pragma unroll
            for (int c = 0; c < 4; ++c) {
                const int k = k0 + c;
                if (k < K) acc[hh][c] = __fmaf_rn(dq1(w, type, base + k), __ldg(x + k), acc[hh][c]);
            }
        }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
            float a = acc[hh][c];
            a = __fadd_rn(a, __shfl_down_sync(GFULL, a, 4));
            a = __fadd_rn(a, __shfl_down_sync(GFULL, a, 2));
            a = __fadd_rn(a, __shfl_down_sync(GFULL, a, 1));
            acc[hh][c] = a;
        }
    const float s0 = __fadd_rn(__fadd_rn(acc[0][0], acc[0][2]), __fadd_rn(acc[0][1], acc[0][3]));
    const float s1 = __fadd_rn(__fadd_rn(acc[1][0], acc[1][2]), __fadd_rn(acc[1][1], acc[1][3]));
    float q[8];
#pragma unroll
    for (int w4 = 0; w4 < 4; ++w4) {
        q[w4] = __shfl_sync(GFULL, s0, 8 * w4);
        q[4 + w4] = __shfl_sync(GFULL, s1, 8 * w4);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) q[i] = __fadd_rn(__fadd_rn(q[i], 0.0f), 0.0f);
    const float r = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[4]), __fadd_rn(q[2], q[6])),
                              __fadd_rn(__fadd_rn(q[1], q[5]), __fadd_rn(q[3], q[7])));
    if (lane == 0) y[row] = r;
}

// ---------------------------------------------------------------------------
// Streaming GEMV for the block-quantised types Q4_K / Q5_K / Q6_K / Q8_0
// (K a multiple of 256, at most 4096): the matmul_dispatch path for large
// matrices (LM head, attention and GDN projections).
//
// One CTA per SM, persistent: a producer lane streams chunks of RS
// consecutive weight rows into a shared-memory ring with 1-D bulk copies
// (TMA, cp.async.bulk + mbarrier transaction counts), straight from the GGUF
// payload; 8 consumer warps dot them against the 24-bit planes of x
// (qmoe_dev.cuh), built once per CTA.  A lane decodes whole 64-element units
// (qmoe_units.cuh: scales once per unit, dp4a over the nibble/byte words) and
// keeps its unit's activation planes in registers for the whole launch, so
// neither x nor the per-element type switch is re-read per row.  Results
// match an F32 dot product to ~2^-22 relative; the reduction order differs
// from the reference's, so outputs are not bit-identical (k_gemv is).
// ---------------------------------------------------------------------------
constexpr int GS_NCW = 16;                     // consumer warps
constexpr int GS_THREADS = (GS_NCW + 1) * 32;  // + one producer warp
constexpr int GS_MAX_STAGES = 12;

struct GemvStream {
    const uint8_t* w;     // first byte of row 0
    const uint8_t* wend;  // one past the tensor's last payload byte
    const float* x;
    float* y;
    int M, K;
    uint32_t rb;     // bytes per row
    int rs;          // rows per ring stage
    int nst;         // ring stages
    uint32_t stage;  // bytes per stage (16-byte multiple)
    uint32_t off_x, off_ring;
};

template <int TYPE, int UPL>  // UPL: units per lane (K/64 = 32 * UPL when UPL > 0; UPL == 0: K < 2048)
__global__ void __launch_bounds__(GS_THREADS, 1) k_gemv_stream(GemvStream p) {
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* full = reinterpret_cast<uint64_t*>(smem);
    uint64_t* empty = full + GS_MAX_STAGES;
    uint8_t* xs = smem + p.off_x;
    uint8_t* ring = smem + p.off_ring;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int G = gridDim.x, c = blockIdx.x;
    const int nchunk = (p.M + p.rs - 1) / p.rs;
    const int nmine = c < nchunk ? (nchunk - 1 - c) / G + 1 : 0;

    if (tid == 0) {
        for (int i = 0; i < p.nst; ++i) {
            mbar_init(full + i, 1);
            mbar_init(empty + i, GS_NCW);
        }
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == GS_NCW) {
        // ---------------- producer ----------------
        if (lane == 0) {
            for (int kk = 0, ch = c, slot = 0, round = 0; kk < nmine; ++kk, ch += G) {
                if (kk >= p.nst) mbar_wait(empty + slot, (round - 1) & 1, nullptr);
                const int r0 = ch * p.rs, nr = min(p.rs, p.M - r0);
                const uint8_t* src = p.w + static_cast<uint64_t>(r0) * p.rb;
                uint8_t* dst = ring + static_cast<size_t>(slot) * p.stage;
                const uint64_t bytes = static_cast<uint64_t>(nr) * p.rb;
                // the 16-byte aligned superset of the rows (plain loads for a ragged tail)
                const uintptr_t s = reinterpret_cast<uintptr_t>(src), lo = s & ~uintptr_t(15);
                const uintptr_t hi = (s + bytes + 15) & ~uintptr_t(15), lim = reinterpret_cast<uintptr_t>(p.wend);
                const uintptr_t hf = hi <= lim ? hi : (lim & ~uintptr_t(15));
                const uint32_t tx = hf > lo ? static_cast<uint32_t>(hf - lo) : 0u;
                for (uintptr_t a = (hf > lo ? hf : lo); a < s + bytes; ++a)
                    dst[a - lo] = *reinterpret_cast<const uint8_t*>(a);
                mbar_arrive_expect_tx(full + slot, tx);
                if (tx) bulk_g2s(dst, reinterpret_cast<const void*>(lo), tx, full + slot, nullptr);
                if (++slot == p.nst) { slot = 0; ++round; }
            }
        }
        return;
    }
    // ---------------- consumers ----------------
    // x -> 24-bit planes (each warp quantises 128-element chunks)
    for (int g = tid; g < p.K / 4; g += GS_NCW * 32)
        write_planes4(__ldg(reinterpret_cast<const float4*>(p.x) + g), xs, p.K, 4 * g, lane);
    asm volatile("bar.sync 1, %0;" ::"r"(GS_NCW * 32) : "memory");
    const XPlanesView xv{smem_u32(xs), smem_u32(xs) + static_cast<uint32_t>(p.K),
                         smem_u32(xs) + 2u * static_cast<uint32_t>(p.K), smem_u32(xs) + 3u * static_cast<uint32_t>(p.K)};
    constexpr int NU = UPL > 0 ? UPL : 1;
    const int U = p.K >> 6;
    const int lgU = 31 - __clz(U);
    const int lgG = UPL > 0 ? 5 : lgU;         // lanes per row: 32, or U when U < 32
    const int rpw = UPL > 0 ? 1 : 32 >> lgU;   // rows per warp step
    const int ul = lane & ((1 << lgG) - 1), rsub = lane >> lgG;
    int unit[NU];
    XU xr[NU];
#pragma unroll
    for (int m = 0; m < NU; ++m) {
        unit[m] = UPL > 0 ? 32 * m + unit_of_lane<TYPE>(lane, 5) : unit_of_lane<TYPE>(ul, lgU);
        load_xu<TYPE>(xr[m], xv, unit[m]);
    }
    for (int kk = 0, ch = c, slot = 0, round = 0; kk < nmine; ++kk, ch += G) {
        const int r0 = ch * p.rs, nr = min(p.rs, p.M - r0);
        mbar_wait(full + slot, round & 1, nullptr);
        const uint32_t base = smem_u32(ring) + static_cast<uint32_t>(slot) * p.stage +
                              static_cast<uint32_t>(reinterpret_cast<uintptr_t>(p.w + static_cast<uint64_t>(r0) * p.rb) & 15u);
        // two rows per warp step, as independent dependency chains (a row
        // past the chunk's end is computed on the last row and dropped)
        for (int rr = warp * rpw; rr < nr; rr += 2 * GS_NCW * rpw) {
            const int ra = rr + rsub, rb = rr + GS_NCW * rpw + rsub;
            const uint32_t pa = base + static_cast<uint32_t>(min(ra, nr - 1)) * p.rb;
            const uint32_t pb = base + static_cast<uint32_t>(min(rb, nr - 1)) * p.rb;
            float va = 0.0f, vb = 0.0f;
#pragma unroll
            for (int m = 0; m < NU; ++m) {
                va += unit_dot_t<TYPE>(pa, unit[m], xr[m]);
                vb += unit_dot_t<TYPE>(pb, unit[m], xr[m]);
            }
            for (int o = (1 << lgG) >> 1; o; o >>= 1) {
                va += __shfl_xor_sync(GFULL, va, o);
                vb += __shfl_xor_sync(GFULL, vb, o);
            }
            if (ul == 0 && ra < nr) p.y[r0 + ra] = va;
            if (ul == 0 && rb < nr) p.y[r0 + rb] = vb;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(empty + slot);
        if (++slot == p.nst) { slot = 0; ++round; }
    }
}

// Q6_K -> the 16-byte-aligned layout: super-block b's 210 bytes at 224*b,
// then 14 zero bytes.  One thread per 16-byte output chunk; the source is
// read in 2-byte words (GGUF Q6_K blocks are 2-byte aligned).
__global__ void k_repack_q6k_a16(const uint8_t* __restrict__ src, uint4* __restrict__ dst, uint64_t nblocks) {
    const uint64_t nchunks = nblocks * 14;
    for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < nchunks;
         i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
        const uint64_t b = i / 14;
        const int j = static_cast<int>(i - b * 14);
        const uint16_t* s16 = reinterpret_cast<const uint16_t*>(src + b * 210 + 16 * j);
        const int nw = j < 13 ? 8 : 1;  // the last chunk holds bytes 208..209, then padding
        uint32_t w[4] = {0u, 0u, 0u, 0u};
        for (int k = 0; k < nw; ++k) w[k >> 1] |= static_cast<uint32_t>(__ldg(s16 + k)) << (16 * (k & 1));
        dst[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
}

cudaError_t launch_repack_q6k_a16(const uint8_t* src, void* dst, uint64_t nblocks, cudaStream_t s) {
    const uint64_t nchunks = nblocks * 14;
    const int grid = static_cast<int>(std::min<uint64_t>((nchunks + 255) / 256, 148ull * 16));
    k_repack_q6k_a16<<<grid, 256, 0, s>>>(src, static_cast<uint4*>(dst), nblocks);
    return cudaGetLastError();
}

__global__ void k_dequant_row(const uint8_t* __restrict__ w, int type, float* __restrict__ out, uint64_t start, int cols) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < cols; i += blockDim.x * gridDim.x)
        out[i] = dq1(w, type, start + i);
}

cudaError_t launch_gemv(const uint8_t* w, int type, const float* x, float* y, int M, int K, uint64_t off,
                        cudaStream_t s) {
    const int grid = (M + GV_WARPS - 1) / GV_WARPS;
    k_gemv<<<grid, GV_WARPS * 32, 0, s>>>(w, type, x, y, M, K, off);
    return cudaGetLastError();
}

namespace {
typedef void (*GsKern)(GemvStream);
template <int TYPE>
GsKern pick_stream(int upl) {
    switch (upl) {
        case 0: return k_gemv_stream<TYPE, 0>;
        case 1: return k_gemv_stream<TYPE, 1>;
        case 2: return k_gemv_stream<TYPE, 2>;
        default: return nullptr;
    }
}
int g_sms[64], g_optin[64];
}  // namespace

// The streaming kernel applies to Q4_K / Q5_K / Q6_K / Q8_0 rows of K = 256 *
// 2^j elements (K <= 4096) whose first row starts on a boundary the unit
// decoders can read (16 bytes for the K-quants with 16-byte blocks, 4 for
// Q8_0, 2 for Q6_K).
// Block bytes of the types the streaming kernel reads (T_Q6_K_A16: the
// repacked Q6_K layout of qmoe_repack).
static int stream_block_bytes(int type) {
    return type == T_Q4_K ? 144 : type == T_Q5_K ? 176 : type == T_Q6_K ? 210 : type == T_Q6_K_A16 ? 224 : 34;
}

bool gemv_stream_supported(const uint8_t* w, int type, int K, uint64_t off) {
    if (type != T_Q4_K && type != T_Q5_K && type != T_Q6_K && type != T_Q6_K_A16 && type != T_Q8_0) return false;
    if (K < 256 || K > 4096 || (K & (K - 1))) return false;
    const int be = type == T_Q8_0 ? 32 : 256, bb = stream_block_bytes(type);
    if (off % be) return false;
    const uintptr_t a = reinterpret_cast<uintptr_t>(w) + off / be * bb;
    const uintptr_t need = (type == T_Q4_K || type == T_Q5_K || type == T_Q6_K_A16) ? 16 : type == T_Q8_0 ? 4 : 2;
    return a % need == 0;
}

cudaError_t launch_gemv_stream(const uint8_t* w, int type, uint64_t w_bytes, const float* x, float* y, int M, int K,
                               uint64_t off, cudaStream_t s) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    int& sms = g_sms[dev & 63];
    int& optin = g_optin[dev & 63];
    if (!sms) {
        if ((e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev)) != cudaSuccess) return e;
        if ((e = cudaDeviceGetAttribute(&optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev)) != cudaSuccess) return e;
    }
    const int be = type == T_Q8_0 ? 32 : 256, bb = stream_block_bytes(type);
    GemvStream p;
    p.w = w + off / be * bb;
    p.wend = w + w_bytes;
    p.x = x;
    p.y = y;
    p.M = M;
    p.K = K;
    p.rb = static_cast<uint32_t>(K / be * bb);
    const int U = K / 64;
    const int upl = U >= 32 ? U / 32 : 0;
    const int rpw = U >= 32 ? 1 : 32 / U;
    // stages of up to ~32 KB (whole double warp steps), as many as fit beside the planes
    int steps = 2;
    while (2 * steps * GS_NCW * rpw * p.rb <= 32768u && steps < 8) steps *= 2;
    p.rs = steps * GS_NCW * rpw;
    p.stage = (static_cast<uint32_t>(p.rs) * p.rb + 32u + 127u) & ~127u;
    p.off_x = 256;
    p.off_ring = (p.off_x + static_cast<uint32_t>(K) * 4u + 127u) & ~127u;  // planes: 3K bytes + K/2 meta
    const size_t budget = static_cast<size_t>(optin) - 1024;
    if (p.off_ring + p.stage > budget) return cudaErrorInvalidValue;
    p.nst = static_cast<int>(std::min<size_t>(GS_MAX_STAGES, (budget - p.off_ring) / p.stage));
    const size_t smem = p.off_ring + static_cast<size_t>(p.nst) * p.stage;
    GsKern kern = nullptr;
    switch (type) {
        case T_Q4_K: kern = pick_stream<T_Q4_K>(upl); break;
        case T_Q5_K: kern = pick_stream<T_Q5_K>(upl); break;
        case T_Q6_K: kern = pick_stream<T_Q6_K>(upl); break;
        case T_Q6_K_A16: kern = pick_stream<T_Q6_K_A16>(upl); break;
        case T_Q8_0: kern = pick_stream<T_Q8_0>(upl); break;
        default: break;
    }
    if (!kern) return cudaErrorInvalidValue;
    if ((e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem))) !=
        cudaSuccess)
        return e;
    const int nchunk = (M + p.rs - 1) / p.rs;
    kern<<<std::min(nchunk, sms), GS_THREADS, smem, s>>>(p);
    return cudaGetLastError();
}

cudaError_t launch_dequant_row(const uint8_t* w, int type, float* out, uint64_t start, int cols, cudaStream_t s) {
    const int grid = (cols + 255) / 256;
    k_dequant_row<<<grid, 256, 0, s>>>(w, type, out, start, cols);
    return cudaGetLastError();
}

}  // namespace qmoe
