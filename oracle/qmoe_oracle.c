/*
 * qmoe_oracle.c -- CPU restatement of the reference MoE block.
 *
 * TEST INFRASTRUCTURE ONLY.  Nothing in the product links or calls this file:
 * it is loaded by tests/, by __graft_entry__.smoke() and by bench.py's CPU
 * baseline leg, always as the checker (or as the timed CPU baseline), never as
 * the thing measured on the GPU.
 *
 * Every function restates one piece of the reference (sahan974/qwen-3.5-cuda)
 * and cites it.  Arithmetic follows the reference's own order so that, where
 * the reference is deterministic, the oracle reproduces it bit for bit:
 *   - or_dequant            src/cuda/matmul_q4.cu:13-129
 *   - or_gemv               src/cuda/matmul_q4.cu:131-167 (256-thread block:
 *                           per-thread fmaf chain over k = t, t+256, ...;
 *                           __shfl_down tree 16,8,4,2,1 per warp; warp 0
 *                           reduces the 8 warp partials with the same tree)
 *   - or_topk               src/cuda/moe.cu:7-52
 *   - or_silu_mul           src/cuda/moe.cu:61-67
 *   - or_add                src/cuda/moe.cu:76-81   (out += a*x, one fma)
 *   - or_shared_add         src/cuda/moe.cu:90-96   (out += x*sigmoid(g))
 *   - or_moe_forward        src/layer_moe.cpp:95-155 (validation :114-124)
 *   - or_rmsnorm            src/cuda/ops.cu:25-65 (pre-MoE norm, model.cpp:208);
 *                           the reference scales by rsqrtf, a hardware
 *                           approximation, here 1/sqrtf (within 2 ulp)
 *   - or_route_batch        layer_moe.cpp:98-99 + moe.cu:7-52 for T tokens
 *   - or_dispatch           no counterpart in the reference (single token);
 *                           stable counting sort of (token, slot) pairs by
 *                           expert, key order (expert, token, slot).
 *
 * Parity pins: the quant decoders are checked against the known-answer
 * blocks of the reference's tests/kernel_tests.cu:116-223 and the top-k
 * against tests/kernel_tests.cu:424-453 (tests/golden/).  Expert compute has
 * no reference test; it is pinned by running the reference's own CUDA path
 * (oracle/_ref, built from the reference sources) on the GPU box.
 *
 * Build: see oracle/build_oracle.sh (gcc -O2 -fopenmp -ffp-contract=off).
 * Floating-point contraction is OFF so every fmaf below is explicit.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

#define OR_EXPORT __attribute__((visibility("default")))

/* status codes shared with the product's C-ABI (include/qmoe.h) */
enum {
    OR_OK = 0,
    OR_ERR_ARG = 1,
    OR_ERR_TYPE = 2,
    OR_ERR_SHAPE = 3,
    OR_ERR_ROUTING = 10,       /* invalid / non-finite routing result (layer_moe.cpp:116-118) */
    OR_ERR_NOT_NORMALIZED = 11 /* route weights do not sum to 1 (layer_moe.cpp:122-124) */
};

static int g_threads = 1;

/* 1 inside a parallel region of this file (the token-parallel batch entry
 * points), where the row-parallel GEMV runs on the calling thread alone. */
static int or_in_parallel(void) {
#ifdef _OPENMP
    return omp_in_parallel();
#else
    return 0;
#endif
}

OR_EXPORT void or_set_threads(int n) { g_threads = n < 1 ? 1 : n; }
OR_EXPORT int or_max_threads(void) {
#ifdef _OPENMP
    return omp_get_max_threads();
#else
    return 1;
#endif
}

/* ---- fp16 -> f32 (matmul_q4.cu:13-16 uses __half2float, exact) ---- */
static float or_h2f(const uint8_t* p) {
    uint16_t h = (uint16_t)(p[0] | (p[1] << 8));
    uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1Fu, m = h & 0x3FFu;
    union { uint32_t u; float f; } v;
    if (e == 0x1F) { v.u = sign | 0x7F800000u | (m << 13); return v.f; }
    if (e == 0) {
        float r = ldexpf((float)m, -24);
        return sign ? -r : r;
    }
    v.u = sign | ((e + 112u) << 23) | (m << 13);
    return v.f;
}

static float or_bf2f(const uint8_t* p) {
    union { uint32_t u; float f; } v;
    v.u = ((uint32_t)p[0] | ((uint32_t)p[1] << 8)) << 16;
    return v.f;
}

/* matmul_q4.cu:18-26 */
static void or_scale_min_k4(int j, const uint8_t* q, uint8_t* d, uint8_t* m) {
    if (j < 4) {
        *d = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *d = (uint8_t)((q[j + 4] & 0x0f) | ((q[j - 4] >> 6) << 4));
        *m = (uint8_t)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
    }
}

/* matmul_q4.cu:30-129: value of element `index` of a tensor of GGML `type`. */
OR_EXPORT float or_dequant(const uint8_t* data, int type, uint64_t index) {
    if (type == 0) { float f; memcpy(&f, data + index * 4, 4); return f; }
    if (type == 1) return or_h2f(data + index * 2);
    if (type == 30) return or_bf2f(data + index * 2);
    if (type == 8) {
        const uint8_t* b = data + (index / 32) * 34;
        return or_h2f(b) * (float)(int8_t)b[2 + index % 32];
    }
    if (type == 2) {
        const uint8_t* b = data + (index / 32) * 18;
        int i = (int)(index % 32);
        int q = (i < 16) ? (b[2 + i] & 15) : (b[2 + i - 16] >> 4);
        return or_h2f(b) * (float)(q - 8);
    }
    if (type == 6) {
        const uint8_t* b = data + (index / 32) * 22;
        int i = (int)(index % 32);
        uint32_t qh = (uint32_t)b[2] | ((uint32_t)b[3] << 8) | ((uint32_t)b[4] << 16) | ((uint32_t)b[5] << 24);
        int j = i & 15;
        int high = (i < 16) ? ((qh >> j) & 1) : ((qh >> (j + 16)) & 1);
        int low = (i < 16) ? (b[6 + j] & 15) : (b[6 + j] >> 4);
        return or_h2f(b) * (float)((low | (high << 4)) - 16);
    }
    if (type == 12 || type == 13) {
        const int bb = (type == 12) ? 144 : 176;
        const uint8_t* b = data + (index / 256) * bb;
        const int i = (int)(index % 256);
        const float d = or_h2f(b), dmin = or_h2f(b + 2);
        uint8_t sc, mn;
        or_scale_min_k4(i / 32, b + 4, &sc, &mn);
        const int group64 = i / 64, in64 = i % 64, lane = in64 & 31;
        if (type == 12) {
            const uint8_t q = b[16 + group64 * 32 + lane];
            return d * (float)sc * (float)((in64 < 32) ? (q & 15) : (q >> 4)) - dmin * (float)mn;
        }
        const uint8_t q = b[48 + group64 * 32 + lane];
        const uint8_t mask = (uint8_t)(1u << (2 * group64 + (in64 >= 32)));
        const int value = ((in64 < 32) ? (q & 15) : (q >> 4)) + ((b[16 + lane] & mask) ? 16 : 0);
        return d * (float)sc * (float)value - dmin * (float)mn;
    }
    if (type == 14) {
        const uint8_t* b = data + (index / 256) * 210;
        const int i = (int)(index % 256);
        const uint8_t* ql = b;
        const uint8_t* qh = b + 128;
        const int8_t* scales = (const int8_t*)(b + 192);
        const int half = i / 128, r = i % 128, lane = r & 31, quarter = r / 32;
        const uint8_t lo = (quarter == 0) ? (ql[half * 64 + lane] & 15)
                         : (quarter == 1) ? (ql[half * 64 + 32 + lane] & 15)
                         : (quarter == 2) ? (ql[half * 64 + lane] >> 4)
                                          : (ql[half * 64 + 32 + lane] >> 4);
        const uint8_t hi = (qh[half * 32 + lane] >> (2 * quarter)) & 3;
        const int si = half * 8 + (lane / 16) + 2 * quarter;
        return or_h2f(b + 208) * (float)scales[si] * (float)((int)(lo | (hi << 4)) - 32);
    }
    return 0.0f;
}

/* matmul_q4.cu:179-183 */
OR_EXPORT int or_type_supported(int t) {
    return t == 0 || t == 1 || t == 30 || t == 2 || t == 6 || t == 8 || t == 12 || t == 13 || t == 14;
}

/* One output row with the reference's reduction order (matmul_q4.cu:140-167,
 * launched with 256 threads at :197).  The shuffle tree leaves in lane 0
 * v[0] after v[i] += v[i+off] for off = 16, 8, 4, 2, 1. */
static float or_tree32(float* v) {
    for (int off = 16; off; off >>= 1)
        for (int i = 0; i < off; ++i) v[i] = v[i] + v[i + off];
    return v[0];
}

static float or_gemv_row(const uint8_t* w, int type, const float* x, int K, uint64_t base) {
    float part[256];
    for (int t = 0; t < 256; ++t) {
        float s = 0.0f;
        for (int k = t; k < K; k += 256) s = fmaf(or_dequant(w, type, base + (uint64_t)k), x[k], s);
        part[t] = s;
    }
    float warp[32];
    for (int wi = 0; wi < 8; ++wi) warp[wi] = or_tree32(part + 32 * wi);
    for (int i = 8; i < 32; ++i) warp[i] = 0.0f;
    return or_tree32(warp);
}

/* y[M] = rows [offset/K, offset/K + M) of W times x[K] (matmul_q4.cu:185-207). */
OR_EXPORT int or_gemv(const uint8_t* w, int type, uint64_t num_elements, const float* x, float* y,
                      int M, int K, uint64_t element_offset) {
    if (!w) return OR_ERR_ARG;
    if (!or_type_supported(type)) return OR_ERR_TYPE;
    if (M <= 0 || K <= 0 || element_offset + (uint64_t)M * (uint64_t)K > num_elements) return OR_ERR_SHAPE;
#pragma omp parallel for num_threads(g_threads) if (g_threads > 1 && M >= 64 && !or_in_parallel()) schedule(static)
    for (int row = 0; row < M; ++row)
        y[row] = or_gemv_row(w, type, x, K, element_offset + (uint64_t)row * (uint64_t)K);
    return OR_OK;
}

/* ops.cu:25-65: sum of squares with the 256-thread GEMV reduction structure
 * (fmaf chain per thread, shuffle trees), scale = 1/sqrt(mean + eps) (the
 * reference uses rsqrtf), out = (x * scale) * w. */
OR_EXPORT void or_rmsnorm(const float* x, const float* w, float* out, int n, float eps) {
    float part[256];
    for (int t = 0; t < 256; ++t) {
        float s = 0.0f;
        for (int i = t; i < n; i += 256) s = fmaf(x[i], x[i], s);
        part[t] = s;
    }
    float warp[32];
    for (int wi = 0; wi < 8; ++wi) warp[wi] = or_tree32(part + 32 * wi);
    for (int i = 8; i < 32; ++i) warp[i] = 0.0f;
    float ss = or_tree32(warp);
    float scale = 1.0f / sqrtf(ss / (float)n + eps);
    for (int i = 0; i < n; ++i) out[i] = (x[i] * scale) * w[i];
}

/* matmul_q4.cu:209-227 */
OR_EXPORT int or_dequantize_row(const uint8_t* w, int type, uint64_t num_elements, float* out, int row, int cols) {
    if (!w || !or_type_supported(type)) return OR_ERR_TYPE;
    uint64_t start = (uint64_t)row * (uint64_t)cols;
    if (row < 0 || cols <= 0 || start + (uint64_t)cols > num_elements) return OR_ERR_SHAPE;
    for (int i = 0; i < cols; ++i) out[i] = or_dequant(w, type, start + (uint64_t)i);
    return OR_OK;
}

/* moe.cu:7-52: finite check; k argmax passes (strict >, ascending i, so the
 * lowest index wins ties); softmax over the selected logits. */
OR_EXPORT void or_topk(const float* x, int* idx, float* w, int n, int k) {
    for (int i = 0; i < n; ++i) {
        if (!isfinite(x[i])) {
            idx[0] = -1;
            w[0] = NAN;
            return;
        }
    }
    for (int j = 0; j < k; ++j) {
        float best = -INFINITY;
        int bi = -1;
        for (int i = 0; i < n; ++i) {
            int used = 0;
            for (int p = 0; p < j; ++p) used |= (idx[p] == i);
            if (!used && x[i] > best) {
                best = x[i];
                bi = i;
            }
        }
        idx[j] = bi;
        w[j] = best;
    }
    float mx = w[0];
    for (int j = 1; j < k; ++j) mx = fmaxf(mx, w[j]);
    float sum = 0;
    for (int j = 0; j < k; ++j) {
        w[j] = expf(w[j] - mx);
        sum += w[j];
    }
    for (int j = 0; j < k; ++j) w[j] /= sum;
}

/* moe.cu:61-67 */
OR_EXPORT void or_silu_mul(const float* g, const float* u, float* h, int n) {
    for (int i = 0; i < n; ++i) {
        float silu_g = g[i] / (1.0f + expf(-g[i]));
        h[i] = silu_g * u[i];
    }
}

/* moe.cu:76-81: out[i] += a * x[i], contracted to one fma by nvcc. */
OR_EXPORT void or_add(float* out, const float* x, float a, int n) {
    for (int i = 0; i < n; ++i) out[i] = fmaf(a, x[i], out[i]);
}

/* moe.cu:90-96: out[i] += x[i] * sigmoid(gate[0]), one fma. */
OR_EXPORT void or_shared_add(float* out, const float* x, const float* gate, int n) {
    float sg = 1.0f / (1.0f + expf(-gate[0]));
    for (int i = 0; i < n; ++i) out[i] = fmaf(x[i], sg, out[i]);
}

/* Tensor view: raw GGUF payload + type + element count. */
typedef struct {
    const uint8_t* data;
    int type;
    uint64_t num_elements;
} or_tensor;

typedef struct {
    or_tensor router, gate_exps, up_exps, down_exps, shared_gate_inp, shared_gate, shared_up, shared_down;
    const float* expert_bias; /* optional per-expert logit bias (benchmark config 3; not in the reference) */
} or_block;

/* One token through the MoE block: layer_moe.cpp:95-155.
 * Optional debug outputs: logits[E], h[k][F] (silu(g)*u per slot), hs[Fs],
 * sgate (scalar).  Returns OR_OK or the routing error codes. */
OR_EXPORT int or_moe_forward(const or_block* W, int d, int E, int k, int F, int Fs,
                             const float* x, float* out, int* idx, float* wts,
                             float* logits_out, float* h_out, float* hs_out, float* sgate_out) {
    float* logits = (float*)malloc(sizeof(float) * (size_t)E);
    float* gate = (float*)malloc(sizeof(float) * (size_t)(F > Fs ? F : Fs));
    float* up = (float*)malloc(sizeof(float) * (size_t)(F > Fs ? F : Fs));
    float* hid = (float*)malloc(sizeof(float) * (size_t)(F > Fs ? F : Fs));
    float* eo = (float*)malloc(sizeof(float) * (size_t)d);
    float* accum = (float*)malloc(sizeof(float) * (size_t)d);
    int st = OR_OK;

    /* 1. routing (layer_moe.cpp:98-99) */
    or_gemv(W->router.data, W->router.type, W->router.num_elements, x, logits, E, d, 0);
    if (W->expert_bias)
        for (int e = 0; e < E; ++e) logits[e] = logits[e] + W->expert_bias[e];
    if (logits_out) memcpy(logits_out, logits, sizeof(float) * (size_t)E);
    or_topk(logits, idx, wts, E, k);

    /* 3. validation (layer_moe.cpp:114-124) */
    float route_sum = 0.0f;
    for (int j = 0; j < k; ++j) {
        if (idx[j] < 0 || idx[j] >= E || !isfinite(wts[j]) || wts[j] < 0.0f) { st = OR_ERR_ROUTING; break; }
        route_sum += wts[j];
    }
    if (st == OR_OK && (!isfinite(route_sum) || fabsf(route_sum - 1.0f) > 1e-4f)) st = OR_ERR_NOT_NORMALIZED;
    if (st != OR_OK) goto done;

    /* 4. routed experts in selection order (layer_moe.cpp:107, 127-142) */
    for (int i = 0; i < d; ++i) accum[i] = 0.0f;
    {
        uint64_t gu_stride = (uint64_t)d * (uint64_t)F;
        uint64_t down_stride = (uint64_t)F * (uint64_t)d;
        for (int j = 0; j < k; ++j) {
            int e = idx[j];
            or_gemv(W->gate_exps.data, W->gate_exps.type, W->gate_exps.num_elements, x, gate, F, d, (uint64_t)e * gu_stride);
            or_gemv(W->up_exps.data, W->up_exps.type, W->up_exps.num_elements, x, up, F, d, (uint64_t)e * gu_stride);
            or_silu_mul(gate, up, hid, F);
            if (h_out) memcpy(h_out + (size_t)j * (size_t)F, hid, sizeof(float) * (size_t)F);
            or_gemv(W->down_exps.data, W->down_exps.type, W->down_exps.num_elements, hid, eo, d, F, (uint64_t)e * down_stride);
            or_add(accum, eo, wts[j], d);
        }
    }
    /* 5-6. shared expert (layer_moe.cpp:145-154) */
    {
        float sgate;
        or_gemv(W->shared_gate_inp.data, W->shared_gate_inp.type, W->shared_gate_inp.num_elements, x, &sgate, 1, d, 0);
        if (sgate_out) *sgate_out = sgate;
        or_gemv(W->shared_gate.data, W->shared_gate.type, W->shared_gate.num_elements, x, gate, Fs, d, 0);
        or_gemv(W->shared_up.data, W->shared_up.type, W->shared_up.num_elements, x, up, Fs, d, 0);
        or_silu_mul(gate, up, hid, Fs);
        if (hs_out) memcpy(hs_out, hid, sizeof(float) * (size_t)Fs);
        or_gemv(W->shared_down.data, W->shared_down.type, W->shared_down.num_elements, hid, eo, d, Fs, 0);
        or_shared_add(accum, eo, &sgate, d);
    }
    memcpy(out, accum, sizeof(float) * (size_t)d);
done:
    free(logits); free(gate); free(up); free(hid); free(eo); free(accum);
    return st;
}

/* Router logits (+ optional bias) and top-k of T tokens (layer_moe.cpp:98-99,
 * moe.cu:7-52), the tokens in parallel (each token's arithmetic is the
 * single-token order above, so the result does not depend on the threads).
 * logits[T][E], idx/wts[T][k]. */
OR_EXPORT void or_route_batch(const uint8_t* router, int type, uint64_t num_elements, const float* bias,
                              int d, int E, int k, int T, const float* x, float* logits, int* idx, float* wts) {
#pragma omp parallel for num_threads(g_threads) if (g_threads > 1 && T > 1) schedule(dynamic, 8)
    for (int t = 0; t < T; ++t) {
        float* lg = logits + (size_t)t * E;
        or_gemv(router, type, num_elements, x + (size_t)t * d, lg, E, d, 0);
        if (bias)
            for (int e = 0; e < E; ++e) lg[e] = lg[e] + bias[e];
        or_topk(lg, idx + (size_t)t * k, wts + (size_t)t * k, E, k);
    }
}

/* T tokens (the reference has no batched path: a batch is T independent
 * calls of MoeLayer::forward).  With more than one thread and T > 1 the
 * tokens run in parallel, each with the single-token arithmetic, so the
 * results are the same as one after another.  Returns the first error code
 * in token order; status[t] (optional) receives each token's code. */
OR_EXPORT int or_moe_forward_batch(const or_block* W, int d, int E, int k, int F, int Fs, int T,
                                   const float* x, float* out, int* idx, float* wts, int* status,
                                   float* logits_out, float* h_out, float* hs_out, float* sgate_out) {
    int first = OR_OK;
    int* codes = (int*)malloc(sizeof(int) * (size_t)(T > 0 ? T : 1));
#pragma omp parallel for num_threads(g_threads) if (g_threads > 1 && T > 1) schedule(dynamic, 1)
    for (int t = 0; t < T; ++t) {
        codes[t] = or_moe_forward(W, d, E, k, F, Fs, x + (size_t)t * d, out + (size_t)t * d,
                                idx + (size_t)t * k, wts + (size_t)t * k,
                                logits_out ? logits_out + (size_t)t * E : NULL,
                                h_out ? h_out + (size_t)t * k * F : NULL,
                                hs_out ? hs_out + (size_t)t * Fs : NULL,
                                sgate_out ? sgate_out + t : NULL);
    }
    for (int t = 0; t < T; ++t) {
        if (status) status[t] = codes[t];
        if (codes[t] != OR_OK && first == OR_OK) first = codes[t];
    }
    free(codes);
    return first;
}

/* Token->expert permutation (new; no reference counterpart).  Pairs p = t*k+j
 * with a valid expert id are ordered by (expert, t, j): a stable counting sort.
 * offsets[E+1]: first pair of each expert; perm[pos] = p; inv_perm[p] = pos
 * (-1 for pairs whose id is out of range). Returns the number of valid pairs. */
OR_EXPORT int or_dispatch(const int* idx, int T, int k, int E, int* offsets, int* perm, int* inv_perm) {
    int P = T * k;
    int* cnt = (int*)calloc((size_t)E + 1, sizeof(int));
    for (int p = 0; p < P; ++p)
        if (idx[p] >= 0 && idx[p] < E) cnt[idx[p]]++;
    offsets[0] = 0;
    for (int e = 0; e < E; ++e) offsets[e + 1] = offsets[e] + cnt[e];
    for (int e = 0; e < E; ++e) cnt[e] = offsets[e];
    for (int p = 0; p < P; ++p) {
        int e = idx[p];
        if (e >= 0 && e < E) {
            int pos = cnt[e]++;
            perm[pos] = p;
            if (inv_perm) inv_perm[p] = pos;
        } else if (inv_perm) {
            inv_perm[p] = -1;
        }
    }
    int n = offsets[E];
    free(cnt);
    return n;
}
