// Per-element dequantisation of GGML tensors with the reference's formulas
// (src/cuda/matmul_q4.cu:13-129): used by the general GEMV and by the
// prefill path's generic (non-Q4_K) weight staging.
#pragma once
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include "qmoe_dev.cuh"
#include "qmoe_units.cuh"

namespace qmoe {

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

}  // namespace qmoe
