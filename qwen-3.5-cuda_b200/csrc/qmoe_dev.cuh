// Device helpers shared by the qmoe kernels (sm_100a).
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>

namespace qmoe {

// ---------------------------------------------------------------------------
// Error word bits (device side of qmoe_check_errors).
// ---------------------------------------------------------------------------
enum : uint32_t {
    EF_ROUTING = 1u,        // non-finite logits / invalid id or weight (layer_moe.cpp:116-118)
    EF_NOT_NORMALIZED = 2u, // |sum(w) - 1| > 1e-4 (layer_moe.cpp:122-124)
    EF_TIMEOUT = 4u,        // a bounded wait gave up
};

// Control block at the start of every workspace (uint32 words).
enum : int {
    CTRL_ARRIVE = 0,     // arrival counter for the router's last-CTA step
    CTRL_ERROR = 1,      // error flags (EF_*)
    CTRL_ERR_TOKEN = 2,  // first failing token (atomicMin), 0xFFFFFFFF = none
    CTRL_N_ACTIVE = 3,   // number of experts with >= 1 routed pair
    CTRL_N_PAIRS = 4,    // number of valid pairs
    CTRL_WORDS = 64
};

// ---------------------------------------------------------------------------
// Small math / bit helpers
// ---------------------------------------------------------------------------
__device__ __forceinline__ float h2f_bits(uint32_t h16) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(h16 & 0xFFFFu)));
}

__device__ __forceinline__ int dp4a_uu(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_su(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.u32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// ---------------------------------------------------------------------------
// Shared-memory addressing, mbarriers and 1-D bulk copies (TMA, no tensor map)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after `limit` polls, records EF_TIMEOUT and returns false.
constexpr uint32_t kWaitLimit = 1u << 24;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* ctrl) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (ctrl) atomicOr(ctrl + CTRL_ERROR, EF_TIMEOUT);
    return false;
}

// global -> shared bulk copy (16-byte aligned addresses, size multiple of 16),
// completion signalled on `bar` as transaction bytes.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// Copies [src, src+bytes) of global memory into shared memory at `dst`, where
// `src` may be unaligned: the 16-byte aligned superset [lo, hi) is bulk-copied
// (hi clipped to `limit`, the end of the source allocation), any tail past the
// last full 16-byte chunk is copied with plain loads by the calling thread.
// Returns the transaction bytes that will arrive on `bar`, and sets *skew to
// the offset of `src` inside the staged window.  `dst` must be 16-byte aligned
// and have room for bytes + 32.  Called by ONE thread.
__device__ __forceinline__ uint32_t stage_bytes(uint8_t* dst, const uint8_t* src, uint64_t bytes,
                                                const uint8_t* limit, uint64_t* bar, uint32_t* skew) {
    uintptr_t s = reinterpret_cast<uintptr_t>(src);
    uintptr_t lo = s & ~static_cast<uintptr_t>(15);
    uintptr_t hi = (s + bytes + 15) & ~static_cast<uintptr_t>(15);
    uintptr_t lim = reinterpret_cast<uintptr_t>(limit);
    uintptr_t hi_full = hi <= lim ? hi : (lim & ~static_cast<uintptr_t>(15));
    *skew = static_cast<uint32_t>(s - lo);
    uint32_t tx = 0;
    if (hi_full > lo) {
        tx = static_cast<uint32_t>(hi_full - lo);
        bulk_g2s(dst, reinterpret_cast<const void*>(lo), tx, bar);
    }
    // tail (only when the window would run past the allocation end)
    for (uintptr_t a = hi_full > lo ? hi_full : lo; a < s + bytes; ++a)
        dst[a - lo] = *reinterpret_cast<const uint8_t*>(a);
    return tx;
}

// ---------------------------------------------------------------------------
// Shared-memory loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(const void* p) { return *reinterpret_cast<const uint4*>(p); }
__device__ __forceinline__ uint32_t lds32(const void* p) { return *reinterpret_cast<const uint32_t*>(p); }

// 16 bytes from a shared address with any 2-byte alignment: two aligned
// 16-byte loads and a byte funnel shift.
__device__ __forceinline__ uint4 lds128_any(const uint8_t* p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    uint32_t off = static_cast<uint32_t>(a & 15u);
    const uint8_t* base = p - off;
    uint4 v0 = lds128(base);
    if (off == 0) return v0;
    uint4 v1 = lds128(base + 16);
    uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint32_t sh = (off & 3u) * 8u;
    uint32_t s[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) s[i] = __funnelshift_r(w[i], w[i + 1], sh);
    uint32_t q = off >> 2;  // 0..3
    uint4 r;
    r.x = q == 0 ? s[0] : q == 1 ? s[1] : q == 2 ? s[2] : s[3];
    r.y = q == 0 ? s[1] : q == 1 ? s[2] : q == 2 ? s[3] : s[4];
    r.z = q == 0 ? s[2] : q == 1 ? s[3] : q == 2 ? s[4] : s[5];
    r.w = q == 0 ? s[3] : q == 1 ? s[4] : q == 2 ? s[5] : s[6];
    return r;
}

// 4 bytes from a shared address with 2-byte alignment.
__device__ __forceinline__ uint32_t lds32_any(const uint8_t* p) {
    uintptr_t a = reinterpret_cast<uintptr_t>(p);
    uint32_t off = static_cast<uint32_t>(a & 3u);
    const uint8_t* base = p - off;
    uint32_t w0 = lds32(base);
    if (off == 0) return w0;
    uint32_t w1 = lds32(base + 4);
    return __funnelshift_r(w0, w1, off * 8u);
}

// ---------------------------------------------------------------------------
// 24-bit fixed-point activation planes.
//
// An activation vector v[K] (K a multiple of 32) is stored per 32-element
// block b as integers X = rint(v * 2^sh_b), |X| < 2^22, with sh_b chosen from
// the block's largest magnitude, split into three byte planes
// X = P0 + 256*P1 + 65536*P2 (P0, P1 unsigned, P2 signed).  Meta per 16
// elements: float2 {2^-sh_b, sum of the 16 original values}.  A quantised
// weight row then dots against the planes with dp4a in exact integer
// arithmetic; the result differs from an F32 dot product by at most
// |v|max * 2^-23 per element, i.e. F32-level accuracy.
// ---------------------------------------------------------------------------
struct XPlanesView {
    const uint8_t* p0;
    const uint8_t* p1;
    const uint8_t* p2;
    const float2* meta;  // [K/16]
};

// Quantises one 32-element block held one element per lane (all 32 lanes
// participate).  Writes the lane's three plane bytes and, from lanes 0 and 16,
// the meta of the two 16-element halves.
__device__ __forceinline__ void xq_block32(float v, uint8_t* p0, uint8_t* p1, uint8_t* p2, float2* meta16,
                                           int lane) {
    float a = fabsf(v);
    float amax = a;
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    // fmaxf drops NaN: detect non-finite separately
    bool bad = !isfinite(v);
    bad = __any_sync(0xffffffffu, bad);
    float s16 = v;
#pragma unroll
    for (int o = 8; o; o >>= 1) s16 += __shfl_xor_sync(0xffffffffu, s16, o);
    uint32_t eb = __float_as_uint(amax) >> 23;  // biased exponent (sign is 0)
    int sh = eb == 0 ? 126 : 21 - (static_cast<int>(eb) - 127);
    sh = sh > 126 ? 126 : sh;
    float mul = __uint_as_float(static_cast<uint32_t>(sh + 127) << 23);
    float scale = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
    int X = bad ? 0 : __float2int_rn(v * mul);
    if (bad) scale = __uint_as_float(0x7FC00000u);
    *p0 = static_cast<uint8_t>(X & 255);
    *p1 = static_cast<uint8_t>((X >> 8) & 255);
    *p2 = static_cast<uint8_t>((X >> 16) & 255);
    if ((lane & 15) == 0) meta16[lane >> 4] = make_float2(scale, s16);
}

// 64 consecutive elements (one "unit") of a plane view, as 16 words per plane.
struct XUnit64 {
    uint32_t x0[16], x1[16], x2[16];
};

__device__ __forceinline__ void load_xunit64(XUnit64& u, const XPlanesView& xv, int e0) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 a = lds128(xv.p0 + e0 + 16 * q);
        uint4 b = lds128(xv.p1 + e0 + 16 * q);
        uint4 c = lds128(xv.p2 + e0 + 16 * q);
        u.x0[4 * q] = a.x; u.x0[4 * q + 1] = a.y; u.x0[4 * q + 2] = a.z; u.x0[4 * q + 3] = a.w;
        u.x1[4 * q] = b.x; u.x1[4 * q + 1] = b.y; u.x1[4 * q + 2] = b.z; u.x1[4 * q + 3] = b.w;
        u.x2[4 * q] = c.x; u.x2[4 * q + 1] = c.y; u.x2[4 * q + 2] = c.z; u.x2[4 * q + 3] = c.w;
    }
}

// Four 16-element runs starting at e[0..3] (Q6_K units).
__device__ __forceinline__ void load_xunit_runs(XUnit64& u, const XPlanesView& xv, const int e[4]) {
#pragma unroll
    for (int q = 0; q < 4; ++q) {
        uint4 a = lds128(xv.p0 + e[q]);
        uint4 b = lds128(xv.p1 + e[q]);
        uint4 c = lds128(xv.p2 + e[q]);
        u.x0[4 * q] = a.x; u.x0[4 * q + 1] = a.y; u.x0[4 * q + 2] = a.z; u.x0[4 * q + 3] = a.w;
        u.x1[4 * q] = b.x; u.x1[4 * q + 1] = b.y; u.x1[4 * q + 2] = b.z; u.x1[4 * q + 3] = b.w;
        u.x2[4 * q] = c.x; u.x2[4 * q + 1] = c.y; u.x2[4 * q + 2] = c.z; u.x2[4 * q + 3] = c.w;
    }
}

// Combines the three plane partial sums into sum(q * X) (one rounding).
__device__ __forceinline__ float planes_combine(int P0, int P1, int P2) {
    int p12 = P1 + (P2 << 8);
    return fmaf(256.0f, static_cast<float>(p12), static_cast<float>(P0));
}

}  // namespace qmoe
