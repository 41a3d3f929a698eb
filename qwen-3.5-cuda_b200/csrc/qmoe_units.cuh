// Per-type dot products of one 64-element "unit" of a GGUF weight row (in
// shared memory, read in place -- no repacking) against the 24-bit activation
// planes of qmoe_dev.cuh.
//
// Activation planes are stored with the chunk swizzle pswz() of
// qmoe_dev.cuh; weight rows are read as they are.
//
// Block layouts are the GGML ones the reference decodes per element in
// src/cuda/matmul_q4.cu:30-129; here a lane decodes a whole unit at once:
//   Q4_K (144 B / 256): unit u -> super-block u/4, 32 qs bytes at 16+32*(u%4);
//        low nibbles = sub-block 2*(u%4), high nibbles = 2*(u%4)+1
//        (matmul_q4.cu:76-96); value = d*sc*q - dmin*m.
//   Q5_K (176 B / 256): as Q4_K with qs at 48, fifth bit from qh[32] at 16,
//        bit 2g (+1 for the high half) (matmul_q4.cu:97-101).
//   Q6_K (210 B / 256): unit u -> super-block u/4, half (u/2)%2, lane range
//        16*(u%2)..+15 of that half: four 16-element runs (quarters 0..3)
//        with scales[half*8 + 2*quarter + u%2] (matmul_q4.cu:105-126);
//        value = d*scale*(q-32).
//   Q8_0 (34 B / 32): unit u -> blocks 2u, 2u+1 (matmul_q4.cu:47-50).
#pragma once
#include "qmoe_dev.cuh"

namespace qmoe {

enum : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q5_0 = 6, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14,
             T_BF16 = 30,
             // not a GGML id: Q6_K super-blocks repacked into 224-byte slots
             // (210 payload bytes + 14 zero bytes), every block 16-byte aligned
             T_Q6_K_A16 = 0x100 | T_Q6_K };

__host__ __device__ constexpr bool is_q6k(int type) { return type == T_Q6_K || type == T_Q6_K_A16; }

// Activation planes + meta of one unit, in registers.
struct XU {
    uint32_t x0[16], x1[16], x2[16];
    float sc[4];   // 2^-sh of the 32-block containing each 16-run
    float sum[4];  // sum of the original values of each 16-run
};

// Element index of run q (0..3) of unit u for a weight type.
__device__ __forceinline__ int unit_run_start(int type, int u, int q) {
    if (is_q6k(type)) return 256 * (u >> 2) + 128 * ((u >> 1) & 1) + 32 * q + 16 * (u & 1);
    return 64 * u + 16 * q;
}

// Unit handled by lane index i (0..U-1, U = 2^lgU units per row).  Identity
// except for Q6_K rows of at least 16 units, where the runs of unit u start
// at chunk 8(u/2) + 2q + u%2 of the plane: lanes are spread so that every
// quarter-warp reads eight distinct bank groups of the swizzled planes.
template <int TYPE>
__device__ __forceinline__ int unit_of_lane(int i, int lgU) {
    if (!is_q6k(TYPE) || lgU < 4) return i;
    const int m = 2 * ((i >> 1) & 3) + ((i >> 3) & 1) + 8 * (i >> 4);
    return 2 * m + (i & 1);
}

template <int TYPE>
__device__ __forceinline__ void load_xu(XU& x, const XPlanesView& xv, int u) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        const uint32_t o = pswz(static_cast<uint32_t>(unit_run_start(TYPE, u, q)));
        const uint4 a = lds128(xv.p0 + o);
        const uint4 b = lds128(xv.p1 + o);
        const uint4 c = lds128(xv.p2 + o);
        x.x0[4 * q] = a.x; x.x0[4 * q + 1] = a.y; x.x0[4 * q + 2] = a.z; x.x0[4 * q + 3] = a.w;
        x.x1[4 * q] = b.x; x.x1[4 * q + 1] = b.y; x.x1[4 * q + 2] = b.z; x.x1[4 * q + 3] = b.w;
        x.x2[4 * q] = c.x; x.x2[4 * q + 1] = c.y; x.x2[4 * q + 2] = c.z; x.x2[4 * q + 3] = c.w;
    }
    if (is_q6k(TYPE)) {
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            const float2 m = ldsf2(xv.meta + 8u * static_cast<uint32_t>(unit_run_start(TYPE, u, q) >> 4));
            x.sc[q] = m.x;
            x.sum[q] = m.y;
        }
    } else {  // the four runs' meta entries are contiguous: 32 bytes at 32u
        const uint4 m0 = lds128(xv.meta + 32u * static_cast<uint32_t>(u));
        const uint4 m1 = lds128(xv.meta + 32u * static_cast<uint32_t>(u) + 16u);
        x.sc[0] = __uint_as_float(m0.x); x.sum[0] = __uint_as_float(m0.y);
        x.sc[1] = __uint_as_float(m0.z); x.sum[1] = __uint_as_float(m0.w);
        x.sc[2] = __uint_as_float(m1.x); x.sum[2] = __uint_as_float(m1.y);
        x.sc[3] = __uint_as_float(m1.z); x.sum[3] = __uint_as_float(m1.w);
    }
}

// 6-bit scale/min of sub-block j from the 12 packed bytes (matmul_q4.cu:18-26).
// W0 = bytes 0..3, W1 = 4..7, W2 = 8..11.
__device__ __forceinline__ void kscale(uint32_t W0, uint32_t W1, uint32_t W2, int j, float& sc, float& mn) {
    uint32_t sh = 8u * static_cast<uint32_t>(j & 3);
    uint32_t b0 = (W0 >> sh) & 255u, b1 = (W1 >> sh) & 255u, b2 = (W2 >> sh) & 255u;
    uint32_t s_lo = b0 & 63u, m_lo = b1 & 63u;
    uint32_t s_hi = (b2 & 15u) | ((b0 >> 6) << 4), m_hi = (b2 >> 4) | ((b1 >> 6) << 4);
    bool hi = j >= 4;
    sc = static_cast<float>(hi ? s_hi : s_lo);
    mn = static_cast<float>(hi ? m_hi : m_lo);
}

// Q4_K / Q5_K unit dot.  `row` is the row start in shared memory (16-byte aligned).
template <bool Q5>
__device__ __forceinline__ float dot_qk45(uint32_t row, int u, const XU& x) {
    constexpr int BB = Q5 ? 176 : 144;
    constexpr int QS = Q5 ? 48 : 16;
    const uint32_t blk = row + static_cast<uint32_t>((u >> 2) * BB);
    const int g = u & 3;
    uint4 hd = lds128(blk);
    uint4 qa = lds128(blk + QS + 32 * g);
    uint4 qb = lds128(blk + QS + 16 + 32 * g);
    uint32_t q[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
    uint32_t hb[8];
    if (Q5) {
        uint4 ha = lds128(blk + 16);
        uint4 hc = lds128(blk + 32);
        hb[0] = ha.x; hb[1] = ha.y; hb[2] = ha.z; hb[3] = ha.w;
        hb[4] = hc.x; hb[5] = hc.y; hb[6] = hc.z; hb[7] = hc.w;
    }
    const float d = h2f_bits(hd.x), dmin = h2f_bits(hd.x >> 16);
    float sc0, m0, sc1, m1;
    kscale(hd.y, hd.z, hd.w, 2 * g, sc0, m0);
    kscale(hd.y, hd.z, hd.w, 2 * g + 1, sc1, m1);
    int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        uint32_t lo = q[w] & 0x0F0F0F0Fu;
        uint32_t hi = (q[w] >> 4) & 0x0F0F0F0Fu;
        if (Q5) {
            lo |= ((hb[w] >> (2 * g)) & 0x01010101u) << 4;
            hi |= ((hb[w] >> (2 * g + 1)) & 0x01010101u) << 4;
        }
        a0 = dp4a_uu(lo, x.x0[w], a0);
        a1 = dp4a_uu(lo, x.x1[w], a1);
        a2 = dp4a_us(lo, x.x2[w], a2);
        b0 = dp4a_uu(hi, x.x0[8 + w], b0);
        b1 = dp4a_uu(hi, x.x1[8 + w], b1);
        b2 = dp4a_us(hi, x.x2[8 + w], b2);
    }
    const float Sa = planes_combine(a0, a1, a2);
    const float Sb = planes_combine(b0, b1, b2);
    float r = (d * sc0) * (x.sc[0] * Sa) - (dmin * m0) * (x.sum[0] + x.sum[1]);
    r += (d * sc1) * (x.sc[2] * Sb) - (dmin * m1) * (x.sum[2] + x.sum[3]);
    return r;
}

// Q8_0 unit dot (two 34-byte blocks at byte 68*u of the row; 4-byte aligned).
__device__ __forceinline__ float dot_q8_0(uint32_t row, int u, const XU& x) {
    const uint32_t b = row + 68u * static_cast<uint32_t>(u);
    uint32_t w0 = lds32(b);        // d0 | q0[0..1]
    uint32_t w8 = lds32(b + 32);   // q0[30..31] | d1
    const float d0 = h2f_bits(w0), d1 = h2f_bits(w8 >> 16);
    uint4 qa = lds128_any(b + 2), qb = lds128_any(b + 18);
    uint4 qc = lds128_any(b + 36), qd = lds128_any(b + 52);
    uint32_t q[16] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w,
                      qc.x, qc.y, qc.z, qc.w, qd.x, qd.y, qd.z, qd.w};
    int a0 = 0, a1 = 0, a2 = 0, b0 = 0, b1 = 0, b2 = 0;
#pragma unroll
    for (int w = 0; w < 8; ++w) {
        a0 = dp4a_su(q[w], x.x0[w], a0);
        a1 = dp4a_su(q[w], x.x1[w], a1);
        a2 = dp4a_ss(q[w], x.x2[w], a2);
        b0 = dp4a_su(q[8 + w], x.x0[8 + w], b0);
        b1 = dp4a_su(q[8 + w], x.x1[8 + w], b1);
        b2 = dp4a_ss(q[8 + w], x.x2[8 + w], b2);
    }
    return d0 * (x.sc[0] * planes_combine(a0, a1, a2)) + d1 * (x.sc[2] * planes_combine(b0, b1, b2));
}

// Q6_K unit dot.  BB = 210: GGUF blocks, 2-byte aligned in general (each
// 16-byte read is two aligned reads and a funnel shift); BB = 224: the
// repacked layout, every block 16-byte aligned (plain 16-byte reads).
template <int BB = 210>
__device__ __forceinline__ float dot_q6_k(uint32_t row, int u, const XU& x) {
    const uint32_t blk = row + static_cast<uint32_t>(BB) * static_cast<uint32_t>(u >> 2);
    const int h = (u >> 1) & 1, a = u & 1;
    uint4 l0, l1, qh;
    uint32_t s0, s1;
    if (BB % 16 == 0) {
        l0 = lds128(blk + 64 * h + 16 * a);
        l1 = lds128(blk + 64 * h + 32 + 16 * a);
        qh = lds128(blk + 128 + 32 * h + 16 * a);
        s0 = lds32(blk + 192 + 8 * h);
        s1 = lds32(blk + 196 + 8 * h);
    } else {
        l0 = lds128_any(blk + 64 * h + 16 * a);
        l1 = lds128_any(blk + 64 * h + 32 + 16 * a);
        qh = lds128_any(blk + 128 + 32 * h + 16 * a);
        s0 = lds32_any(blk + 192 + 8 * h);
        s1 = lds32_any(blk + 196 + 8 * h);
    }
    const float d = h2f_bits(lds16(blk + 208));
    // scales[8h + 2q + a], q = 0..3 -> bytes a, a+2 of s0 and a, a+2 of s1
    const uint32_t sa = 8u * static_cast<uint32_t>(a);
    const float sc[4] = {static_cast<float>(static_cast<int8_t>((s0 >> sa) & 255u)),
                         static_cast<float>(static_cast<int8_t>((s0 >> (sa + 16)) & 255u)),
                         static_cast<float>(static_cast<int8_t>((s1 >> sa) & 255u)),
                         static_cast<float>(static_cast<int8_t>((s1 >> (sa + 16)) & 255u))};
    const uint32_t L0[4] = {l0.x, l0.y, l0.z, l0.w}, L1[4] = {l1.x, l1.y, l1.z, l1.w},
                   H[4] = {qh.x, qh.y, qh.z, qh.w};
    int P[4][3];
#pragma unroll
    for (int q = 0; q < 4; ++q) P[q][0] = P[q][1] = P[q][2] = 0;
#pragma unroll
    for (int w = 0; w < 4; ++w) {
        uint32_t q0 = (L0[w] & 0x0F0F0F0Fu) | ((H[w] & 0x03030303u) << 4);
        uint32_t q1 = (L1[w] & 0x0F0F0F0Fu) | (((H[w] >> 2) & 0x03030303u) << 4);
        uint32_t q2 = ((L0[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 4) & 0x03030303u) << 4);
        uint32_t q3 = ((L1[w] >> 4) & 0x0F0F0F0Fu) | (((H[w] >> 6) & 0x03030303u) << 4);
        const uint32_t qq[4] = {q0, q1, q2, q3};
#pragma unroll
        for (int q = 0; q < 4; ++q) {
            P[q][0] = dp4a_uu(qq[q], x.x0[4 * q + w], P[q][0]);
            P[q][1] = dp4a_uu(qq[q], x.x1[4 * q + w], P[q][1]);
            P[q][2] = dp4a_us(qq[q], x.x2[4 * q + w], P[q][2]);
        }
    }
    float r = 0.0f;
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        float S = planes_combine(P[q][0], P[q][1], P[q][2]);
        r += (d * sc[q]) * (x.sc[q] * S - 32.0f * x.sum[q]);
    }
    return r;
}

__device__ __forceinline__ float unit_dot(int type, uint32_t row, int u, const XU& x) {
    switch (type) {
        case T_Q4_K: return dot_qk45<false>(row, u, x);
        case T_Q5_K: return dot_qk45<true>(row, u, x);
        case T_Q6_K: return dot_q6_k(row, u, x);
        case T_Q8_0: return dot_q8_0(row, u, x);
        default: return __uint_as_float(0x7FC00000u);
    }
}

// The unit dot of a weight type known at compile time.
template <int TYPE>
__device__ __forceinline__ float unit_dot_t(uint32_t row, int u, const XU& x) {
    if (TYPE == T_Q4_K) return dot_qk45<false>(row, u, x);
    if (TYPE == T_Q5_K) return dot_qk45<true>(row, u, x);
    if (TYPE == T_Q6_K) return dot_q6_k<210>(row, u, x);
    if (TYPE == T_Q6_K_A16) return dot_q6_k<224>(row, u, x);
    return dot_q8_0(row, u, x);
}

// Sum over the U lanes (aligned group) that share one row.
template <int U>
__device__ __forceinline__ float group_sum(float v) {
#pragma unroll
    for (int o = U / 2; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace qmoe
