/*
 * Deterministic synthetic GGUF tensors for tests and benchmarks.
 *
 * The same source compiles as host C/C++ and as CUDA device code and yields
 * byte-identical tensors on both sides, so a tensor generated on the GPU can
 * be regenerated on the CPU (for the oracle) and vice versa.  To keep the two
 * sides bit-identical only integer arithmetic and correctly rounded IEEE
 * float operations (+ - * /, rint, comparisons) are used, each written
 * through the QS_* macros so that no multiply-add is ever contracted.
 *
 * Normal variates: Irwin-Hall sum of twelve 16-bit uniforms (mean 0,
 * variance 1, support [-6, 6]) from a splitmix64 counter hash.  The sum is
 * formed in integers and converted once, which is exact.
 *
 * Block encoders: one simple, valid encoder per GGML block type.  They only
 * need to produce legal blocks; the decoders under test and the oracle read
 * the same bytes.  Field layouts are the GGML ones that the reference decodes
 * in src/cuda/matmul_q4.cu:30-129 (Q8_0 :47-50, Q4_0 :53-58, Q5_0 :61-73,
 * Q4_K/Q5_K :76-102, Q6_K :105-126).
 */
#ifndef QMOE_SYNTH_H
#define QMOE_SYNTH_H

#include <stdint.h>
#include <math.h>

#ifdef __CUDACC__
#define QS_HD __host__ __device__ __forceinline__
#else
#define QS_HD static inline
#endif

#if defined(__CUDA_ARCH__)
#define QS_MUL(a, b) __fmul_rn((a), (b))
#define QS_ADD(a, b) __fadd_rn((a), (b))
#define QS_SUB(a, b) __fsub_rn((a), (b))
#define QS_DIV(a, b) __fdiv_rn((a), (b))
#define QS_RINT(a) rintf(a)
#else
/* Host: the including translation unit is compiled with -ffp-contract=off. */
#define QS_MUL(a, b) ((a) * (b))
#define QS_ADD(a, b) ((a) + (b))
#define QS_SUB(a, b) ((a) - (b))
#define QS_DIV(a, b) ((a) / (b))
#define QS_RINT(a) rintf(a)
#endif

/* GGML type ids (include/quantized.hpp:12-36 of the reference). */
enum {
    QS_F32 = 0, QS_F16 = 1, QS_Q4_0 = 2, QS_Q5_0 = 6, QS_Q8_0 = 8,
    QS_Q4_K = 12, QS_Q5_K = 13, QS_Q6_K = 14, QS_BF16 = 30
};

QS_HD uint64_t qs_mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

/* Stream key for (seed, stream id): every tensor gets its own stream. */
QS_HD uint64_t qs_stream_key(uint64_t seed, uint64_t stream) {
    return qs_mix64(seed ^ qs_mix64(stream ^ 0x5851F42D4C957F2Dull));
}

/* Standard normal (Irwin-Hall(12)) for element `index` of a stream. */
QS_HD float qs_normal(uint64_t key, uint64_t index) {
    uint64_t s = 0;
    for (int h = 0; h < 3; ++h) {
        uint64_t r = qs_mix64(key + index * 3ull + (uint64_t)h);
        s += (r & 0xFFFFull) + ((r >> 16) & 0xFFFFull) + ((r >> 32) & 0xFFFFull) + (r >> 48);
    }
    /* sum_i (k_i + 0.5)/65536 - 6 = (S + 6 - 393216) / 65536, exact in float */
    int32_t n = (int32_t)((int64_t)s + 6 - 393216);
    return QS_MUL((float)n, 1.0f / 65536.0f);
}

/* ---- IEEE half / bfloat16 conversions written in integer arithmetic ---- */

QS_HD uint32_t qs_f2u(float f) { union { float f; uint32_t u; } v; v.f = f; return v.u; }
QS_HD float qs_u2f(uint32_t u) { union { float f; uint32_t u; } v; v.u = u; return v.f; }

/* float -> IEEE binary16, round to nearest even, with subnormals. */
QS_HD uint16_t qs_f2h(float f) {
    uint32_t x = qs_f2u(f);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7FFFFFFFu;
    if (ax >= 0x7F800000u) return (uint16_t)(sign | (ax > 0x7F800000u ? 0x7E00u : 0x7C00u));
    if (ax >= 0x477FF000u) return (uint16_t)(sign | 0x7C00u); /* rounds to inf */
    if (ax < 0x38800000u) {                                  /* half subnormal or zero */
        if (ax < 0x33000000u) return (uint16_t)sign;          /* < 2^-25: rounds to 0 */
        uint32_t e = ax >> 23;
        uint32_t m = (ax & 0x7FFFFFu) | 0x800000u;
        uint32_t shift = 126u - e;                            /* 14..24 */
        uint32_t q = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t half = 1u << (shift - 1u);
        if (rem > half || (rem == half && (q & 1u))) q++;
        return (uint16_t)(sign | q);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7FFFFFu;
    uint32_t q = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1FFFu;
    if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
    return (uint16_t)(sign | q);
}

QS_HD float qs_h2f(uint16_t h) {
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = ((uint32_t)h >> 10) & 0x1Fu;
    uint32_t m = (uint32_t)h & 0x3FFu;
    if (e == 0x1Fu) return qs_u2f(sign | 0x7F800000u | (m << 13));
    if (e == 0) {
        if (m == 0) return qs_u2f(sign);
        /* subnormal: m * 2^-24 */
        float v = QS_MUL((float)m, 1.0f / 16777216.0f);
        return sign ? -v : v;
    }
    return qs_u2f(sign | ((e + 112u) << 23) | (m << 13));
}

QS_HD uint16_t qs_f2bf(float f) {
    uint32_t x = qs_f2u(f);
    if ((x & 0x7FFFFFFFu) > 0x7F800000u) return (uint16_t)((x >> 16) | 0x40u);
    uint32_t lsb = (x >> 16) & 1u;
    x += 0x7FFFu + lsb;
    return (uint16_t)(x >> 16);
}

QS_HD float qs_fabs(float a) { return qs_u2f(qs_f2u(a) & 0x7FFFFFFFu); }
QS_HD float qs_max(float a, float b) { return a > b ? a : b; }
QS_HD float qs_min(float a, float b) { return a < b ? a : b; }
QS_HD int qs_clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }

/* ---------------------------- block encoders ---------------------------- */

/* Q8_0: fp16 d + 32 x int8, value = d * q. */
QS_HD void qs_encode_q8_0(const float* x, uint8_t* b) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = qs_max(amax, qs_fabs(x[i]));
    uint16_t dh = qs_f2h(QS_DIV(amax, 127.0f));
    float d = qs_h2f(dh);
    b[0] = (uint8_t)(dh & 0xFF); b[1] = (uint8_t)(dh >> 8);
    for (int i = 0; i < 32; ++i) {
        int q = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[i], d)), -127, 127) : 0;
        b[2 + i] = (uint8_t)(int8_t)q;
    }
}

/* Q4_0: fp16 d + 16 bytes, value = d * (q - 8); element j low nibble, j+16 high. */
QS_HD void qs_encode_q4_0(const float* x, uint8_t* b) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = qs_max(amax, qs_fabs(x[i]));
    uint16_t dh = qs_f2h(QS_DIV(amax, 7.0f));
    float d = qs_h2f(dh);
    b[0] = (uint8_t)(dh & 0xFF); b[1] = (uint8_t)(dh >> 8);
    for (int j = 0; j < 16; ++j) {
        int q0 = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[j], d)) + 8, 0, 15) : 8;
        int q1 = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[j + 16], d)) + 8, 0, 15) : 8;
        b[2 + j] = (uint8_t)(q0 | (q1 << 4));
    }
}

/* Q5_0: fp16 d + 32-bit qh + 16 bytes, value = d * (q - 16). */
QS_HD void qs_encode_q5_0(const float* x, uint8_t* b) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = qs_max(amax, qs_fabs(x[i]));
    uint16_t dh = qs_f2h(QS_DIV(amax, 15.0f));
    float d = qs_h2f(dh);
    b[0] = (uint8_t)(dh & 0xFF); b[1] = (uint8_t)(dh >> 8);
    uint32_t qh = 0;
    for (int j = 0; j < 16; ++j) {
        int q0 = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[j], d)) + 16, 0, 31) : 16;
        int q1 = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[j + 16], d)) + 16, 0, 31) : 16;
        b[6 + j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
        qh |= (uint32_t)(q0 >> 4) << j;
        qh |= (uint32_t)(q1 >> 4) << (j + 16);
    }
    b[2] = (uint8_t)qh; b[3] = (uint8_t)(qh >> 8); b[4] = (uint8_t)(qh >> 16); b[5] = (uint8_t)(qh >> 24);
}

/* Q4_K / Q5_K share the 6-bit scale/min packing (decoded by scale_min_k4,
 * matmul_q4.cu:18-26). nlev = 15 (Q4_K) or 31 (Q5_K). Returns per-element q. */
QS_HD void qs_kquant_scales(const float* x, int nlev, uint8_t* hdr, int* q) {
    float s[8], m[8];
    float smax = 0.0f, mmax = 0.0f;
    for (int j = 0; j < 8; ++j) {
        float lo = 0.0f, hi = -1e30f;
        for (int i = 0; i < 32; ++i) { lo = qs_min(lo, x[32 * j + i]); hi = qs_max(hi, x[32 * j + i]); }
        hi = qs_max(hi, lo);
        s[j] = QS_DIV(QS_SUB(hi, lo), (float)nlev);
        m[j] = -lo;
        smax = qs_max(smax, s[j]);
        mmax = qs_max(mmax, m[j]);
    }
    uint16_t dh = qs_f2h(QS_DIV(smax, 63.0f));
    uint16_t mh = qs_f2h(QS_DIV(mmax, 63.0f));
    float d = qs_h2f(dh), dmin = qs_h2f(mh);
    int sc[8], mn[8];
    for (int j = 0; j < 8; ++j) {
        sc[j] = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(s[j], d)), 0, 63) : 0;
        mn[j] = dmin > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(m[j], dmin)), 0, 63) : 0;
    }
    hdr[0] = (uint8_t)(dh & 0xFF); hdr[1] = (uint8_t)(dh >> 8);
    hdr[2] = (uint8_t)(mh & 0xFF); hdr[3] = (uint8_t)(mh >> 8);
    uint8_t* p = hdr + 4;
    for (int j = 0; j < 4; ++j) {
        p[j]     = (uint8_t)((sc[j] & 63) | ((sc[j + 4] >> 4) << 6));
        p[j + 4] = (uint8_t)((mn[j] & 63) | ((mn[j + 4] >> 4) << 6));
        p[j + 8] = (uint8_t)((sc[j + 4] & 15) | ((mn[j + 4] & 15) << 4));
    }
    for (int j = 0; j < 8; ++j) {
        float es = QS_MUL(d, (float)sc[j]);
        float em = QS_MUL(dmin, (float)mn[j]);
        for (int i = 0; i < 32; ++i) {
            int v = es > 0.0f ? (int)QS_RINT(QS_DIV(QS_ADD(x[32 * j + i], em), es)) : 0;
            q[32 * j + i] = qs_clampi(v, 0, nlev);
        }
    }
}

/* Q4_K: 144 B = d, dmin, scales[12], qs[128]; element i -> byte
 * 16 + 32*(i/64) + i%32, low nibble for i%64 < 32 (matmul_q4.cu:89-96). */
QS_HD void qs_encode_q4_k(const float* x, uint8_t* b) {
    int q[256];
    qs_kquant_scales(x, 15, b, q);
    for (int g = 0; g < 4; ++g)
        for (int l = 0; l < 32; ++l)
            b[16 + 32 * g + l] = (uint8_t)(q[64 * g + l] | (q[64 * g + 32 + l] << 4));
}

/* Q5_K: 176 B = d, dmin, scales[12], qh[32], qs[128] (matmul_q4.cu:97-101). */
QS_HD void qs_encode_q5_k(const float* x, uint8_t* b) {
    int q[256];
    qs_kquant_scales(x, 31, b, q);
    for (int l = 0; l < 32; ++l) b[16 + l] = 0;
    for (int g = 0; g < 4; ++g)
        for (int l = 0; l < 32; ++l) {
            int lo = q[64 * g + l], hi = q[64 * g + 32 + l];
            b[48 + 32 * g + l] = (uint8_t)((lo & 15) | ((hi & 15) << 4));
            b[16 + l] |= (uint8_t)(((lo >> 4) << (2 * g)) | ((hi >> 4) << (2 * g + 1)));
        }
}

/* Q6_K: 210 B = ql[128], qh[64], scales[16] (int8), d (matmul_q4.cu:105-126).
 * value = d * scales[half*8 + lane/16 + 2*quarter] * (q - 32). */
QS_HD void qs_encode_q6_k(const float* x, uint8_t* b) {
    float s[16], smax = 0.0f;
    for (int j = 0; j < 16; ++j) {
        float amax = 0.0f;
        for (int i = 0; i < 16; ++i) amax = qs_max(amax, qs_fabs(x[16 * j + i]));
        s[j] = QS_DIV(amax, 31.0f);
        smax = qs_max(smax, s[j]);
    }
    uint16_t dh = qs_f2h(QS_DIV(smax, 127.0f));
    float d = qs_h2f(dh);
    int sc[16];
    for (int j = 0; j < 16; ++j) sc[j] = d > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(s[j], d)), 0, 127) : 0;
    for (int i = 0; i < 192; ++i) b[i] = 0;
    for (int i = 0; i < 256; ++i) {
        int half = i / 128, r = i % 128, quarter = r / 32, lane = r % 32;
        int si = half * 8 + lane / 16 + 2 * quarter;
        float es = QS_MUL(d, (float)sc[si]);
        int v = es > 0.0f ? qs_clampi((int)QS_RINT(QS_DIV(x[i], es)), -32, 31) : 0;
        int qv = v + 32;
        int lo = qv & 15, hi = qv >> 4;
        int qlb = half * 64 + (quarter & 1) * 32 + lane;
        b[qlb] |= (uint8_t)(quarter < 2 ? lo : (lo << 4));
        b[128 + half * 32 + lane] |= (uint8_t)(hi << (2 * quarter));
    }
    for (int j = 0; j < 16; ++j) b[192 + j] = (uint8_t)(int8_t)sc[j];
    b[208] = (uint8_t)(dh & 0xFF); b[209] = (uint8_t)(dh >> 8);
}

/* Elements and bytes per block for the generated types. */
QS_HD int qs_block_elems(int type) {
    switch (type) {
        case QS_F32: case QS_F16: case QS_BF16: return 1;
        case QS_Q4_0: case QS_Q5_0: case QS_Q8_0: return 32;
        case QS_Q4_K: case QS_Q5_K: case QS_Q6_K: return 256;
        default: return 0;
    }
}
QS_HD int qs_block_bytes(int type) {
    switch (type) {
        case QS_F32: return 4;
        case QS_F16: case QS_BF16: return 2;
        case QS_Q4_0: return 18;
        case QS_Q5_0: return 22;
        case QS_Q8_0: return 34;
        case QS_Q4_K: return 144;
        case QS_Q5_K: return 176;
        case QS_Q6_K: return 210;
        default: return 0;
    }
}

/* Generate block `blk` of a tensor of `type` whose elements are sigma*N(0,1)
 * from stream `key`; writes qs_block_bytes(type) bytes to `out`. */
QS_HD void qs_gen_block(int type, uint64_t key, float sigma, uint64_t blk, uint8_t* out) {
    float x[256];
    int n = qs_block_elems(type);
    uint64_t base = blk * (uint64_t)n;
    for (int i = 0; i < n; ++i) x[i] = QS_MUL(qs_normal(key, base + (uint64_t)i), sigma);
    switch (type) {
        case QS_F32: { uint32_t u = qs_f2u(x[0]); out[0] = (uint8_t)u; out[1] = (uint8_t)(u >> 8); out[2] = (uint8_t)(u >> 16); out[3] = (uint8_t)(u >> 24); break; }
        case QS_F16: { uint16_t h = qs_f2h(x[0]); out[0] = (uint8_t)h; out[1] = (uint8_t)(h >> 8); break; }
        case QS_BF16: { uint16_t h = qs_f2bf(x[0]); out[0] = (uint8_t)h; out[1] = (uint8_t)(h >> 8); break; }
        case QS_Q4_0: qs_encode_q4_0(x, out); break;
        case QS_Q5_0: qs_encode_q5_0(x, out); break;
        case QS_Q8_0: qs_encode_q8_0(x, out); break;
        case QS_Q4_K: qs_encode_q4_k(x, out); break;
        case QS_Q5_K: qs_encode_q5_k(x, out); break;
        case QS_Q6_K: qs_encode_q6_k(x, out); break;
        default: break;
    }
}

#endif /* QMOE_SYNTH_H */
