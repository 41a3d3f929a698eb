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
