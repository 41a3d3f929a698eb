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

namespace qmoe {

constexpr unsigned GFULL = 0xffffffffu;

__device__ __forceinline__ float g_h2f(const uint8_t* p) {
    const uint32_t bits = static_cast<uint32_t>(p[0]) | (static_cast<uint32_t>(p[1]) << 8);
    return h2f_bits(bits);
}

__device__ __forceinline__ void g_scale_min_k4(int j, const uint8_t* q, uint32_t& d, uint32_t& m) {
    if (j < 4) {
        d = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        d = (q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Value of element `index` of a GGML tensor (formulas of matmul_q4.cu:30-129).
__device__ __forceinline__ float dq1(const uint8_t* data, int type, uint64_t index) {
    switch (type) {
        case T_F32: return reinterpret_cast<const float*>(data)[index];
        case T_F16: return __half2float(reinterpret_cast<const __half*>(data)[index]);
        case T_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(data)[index]);
        case T_Q8_0: {
            const uint8_t* b = data + (index / 32) * 34;
            return g_h2f(b) * static_cast<float>(static_cast<int8_t>(b[2 + index % 32]));
        }
        case T_Q4_0: {
            const uint8_t* b = data + (index / 32) * 18;
            const int i = static_cast<int>(index % 32);
            const int q = (i < 16) ? (b[2 + i] & 15) : (b[2 + i - 16] >> 4);
            return g_h2f(b) * (q - 8);
        }
        case T_Q5_0: {
            const uint8_t* b = data + (index / 32) * 22;
            const int i = static_cast<int>(index % 32);
            const uint32_t qh = static_cast<uint32_t>(b[2]) | (static_cast<uint32_t>(b[3]) << 8) |
                                (static_cast<uint32_t>(b[4]) << 16) | (static_cast<uint32_t>(b[5]) << 24);
            const int j = i & 15;
            const int high = (i < 16) ? ((qh >> j) & 1) : ((qh >> (j + 16)) & 1);
            const int low = (i < 16) ? (b[6 + j] & 15) : (b[6 + j] >> 4);
            return g_h2f(b) * ((low | (high << 4)) - 16);
        }
        case T_Q4_K:
        case T_Q5_K: {
            const int bb = (type == T_Q4_K) ? 144 : 176;
            const uint8_t* b = data + (index / 256) * bb;
            const int i = static_cast<int>(index % 256);
            const float d = g_h2f(b), dmin = g_h2f(b + 2);
            uint32_t sc, mn;
            g_scale_min_k4(i / 32, b + 4, sc, mn);
            const int group64 = i / 64, in64 = i % 64, lane = in64 & 31;
            if (type == T_Q4_K) {
                const uint8_t q = b[16 + group64 * 32 + lane];
                return d * sc * ((in64 < 32) ? (q & 15) : (q >> 4)) - dmin * mn;
            }
            const uint8_t q = b[48 + group64 * 32 + lane];
            const uint8_t mask = static_cast<uint8_t>(1u << (2 * group64 + (in64 >= 32)));
            const int value = ((in64 < 32) ? (q & 15) : (q >> 4)) + ((b[16 + lane] & mask) ? 16 : 0);
            return d * sc * value - dmin * mn;
        }
        case T_Q6_K: {
            const uint8_t* b = data + (index / 256) * 210;
            const int i = static_cast<int>(index % 256);
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            const int8_t* scales = reinterpret_cast<const int8_t*>(b + 192);
            const int half = i / 128, r = i % 128, lane = r & 31, quarter = r / 32;
            const uint8_t lo = (quarter == 0) ? (ql[half * 64 + lane] & 15)
                             : (quarter == 1) ? (ql[half * 64 + 32 + lane] & 15)
                             : (quarter == 2) ? (ql[half * 64 + lane] >> 4)
                                              : (ql[half * 64 + 32 + lane] >> 4);
            const uint8_t hi = (qh[half * 32 + lane] >> (2 * quarter)) & 3;
            const int si = half * 8 + (lane / 16) + 2 * quarter;
            return g_h2f(b + 208) * scales[si] * (static_cast<int>(lo | (hi << 4)) - 32);
        }
        default: return 0.0f;
    }
}

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

cudaError_t launch_dequant_row(const uint8_t* w, int type, float* out, uint64_t start, int cols, cudaStream_t s) {
    const int grid = (cols + 255) / 256;
    k_dequant_row<<<grid, 256, 0, s>>>(w, type, out, start, cols);
    return cudaGetLastError();
}

}  // namespace qmoe
