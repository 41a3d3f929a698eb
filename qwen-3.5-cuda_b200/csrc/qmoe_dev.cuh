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
    EF_ALIGN = 8u,          // a bulk copy with a misaligned address or size was skipped
};

// Control block at the start of every workspace (uint32 words).
enum : int {
    CTRL_ARRIVE = 0,     // arrival counter for the router's last-CTA step
    CTRL_ERROR = 1,      // error flags (EF_*)
    CTRL_ERR_TOKEN = 2,  // first failing token (atomicMin), 0xFFFFFFFF = none
    CTRL_N_ACTIVE = 3,   // number of experts with >= 1 routed pair
    CTRL_N_PAIRS = 4,    // number of valid pairs
    CTRL_GRID_CTR = 6,   // words 6-7: 64-bit arrival count of the fused expert kernel's grid barrier
    CTRL_SINK = 8,       // words 8-9: device address of a host-mapped error word (0 = none)
    CTRL_WORDS = 64
};

// Records error flags in the workspace error word and, when the caller has
// registered one (qmoe_workspace_set_error_sink), in its host-mapped word, so
// that a host can notice an error without synchronising the stream.
__device__ __forceinline__ void raise_error(uint32_t* ctrl, uint32_t flag) {
    atomicOr(ctrl + CTRL_ERROR, flag);
    const unsigned long long sink = *reinterpret_cast<volatile unsigned long long*>(ctrl + CTRL_SINK);
    if (sink) atomicOr_system(reinterpret_cast<unsigned int*>(sink), flag);
}

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

// try_wait with a suspend-time hint: the warp sleeps in the barrier unit until
// the phase completes (or ~100 us pass) instead of re-issuing the test.
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(100000u)
        : "memory");
    return ok != 0;
}

// Bounded wait: gives up after kWaitLimit tries (each one suspends for up to
// the hint above), records EF_TIMEOUT and returns false.
constexpr uint32_t kWaitLimit = 1u << 14;
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t* ctrl) {
    for (uint32_t i = 0; i < kWaitLimit; ++i)
        if (mbar_try_wait(bar, parity)) return true;
    if (ctrl) raise_error(ctrl, EF_TIMEOUT);
    return false;
}

// L2 prefetch of a global range (no shared-memory destination).
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// global -> shared bulk copy (16-byte aligned addresses, size multiple of 16),
// completion signalled on `bar` as transaction bytes.  A misaligned request is
// not issued: EF_ALIGN is recorded and the waiter times out instead of the
// copy faulting.
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint32_t* ctrl) {
    if (((smem_u32(smem_dst) | static_cast<uint32_t>(reinterpret_cast<uintptr_t>(gmem_src)) | bytes) & 15u) != 0) {
        if (ctrl) raise_error(ctrl, EF_ALIGN);
        return;
    }
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(smem_dst)),
        "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ uint64_t gtimer() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Programmatic dependent launch (PDL).  wait: block until the grids this
// launch depends on have completed and their memory is visible (a no-op when
// the launch has no programmatic dependency).  launch_dependents: allow the
// next kernel in the stream to start its prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------------------
// Shared-memory accesses through 32-bit shared-window addresses (explicit
// ld.shared / st.shared: the hot loops never go through generic addressing).
// volatile keeps them ordered after the mbarrier waits that publish the data.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(uint32_t a) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
    uint32_t v;
    asm volatile("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ uint32_t lds16(uint32_t a) {
    unsigned short v;
    asm volatile("ld.shared.u16 %0, [%1];" : "=h"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float ldsf(uint32_t a) {
    float v;
    asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(a));
    return v;
}
__device__ __forceinline__ float2 ldsf2(uint32_t a) {
    float2 v;
    asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(a));
    return v;
}
__device__ __forceinline__ void sts8(uint32_t a, uint32_t v) {
    asm volatile("st.shared.u8 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void stsf(uint32_t a, float v) {
    asm volatile("st.shared.f32 [%0], %1;" ::"r"(a), "f"(v) : "memory");
}
__device__ __forceinline__ void stsf2(uint32_t a, float x, float y) {
    asm volatile("st.shared.v2.f32 [%0], {%1, %2};" ::"r"(a), "f"(x), "f"(y) : "memory");
}

// 16 bytes from a shared address with any 2-byte alignment: two aligned
// 16-byte loads and a byte funnel shift.
__device__ __forceinline__ uint4 lds128_any(uint32_t a) {
    const uint32_t off = a & 15u;
    const uint32_t base = a - off;
    const uint4 v0 = lds128(base);
    if (off == 0) return v0;
    const uint4 v1 = lds128(base + 16);
    const uint32_t w[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    const uint32_t sh = (off & 3u) * 8u;
    uint32_t s[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) s[i] = __funnelshift_r(w[i], w[i + 1], sh);
    const uint32_t q = off >> 2;  // 0..3
    uint4 r;
    r.x = q == 0 ? s[0] : q == 1 ? s[1] : q == 2 ? s[2] : s[3];
    r.y = q == 0 ? s[1] : q == 1 ? s[2] : q == 2 ? s[3] : s[4];
    r.z = q == 0 ? s[2] : q == 1 ? s[3] : q == 2 ? s[4] : s[5];
    r.w = q == 0 ? s[3] : q == 1 ? s[4] : q == 2 ? s[5] : s[6];
    return r;
}

// 4 bytes from a shared address with 2-byte alignment.
__device__ __forceinline__ uint32_t lds32_any(uint32_t a) {
    const uint32_t off = a & 3u;
    const uint32_t w0 = lds32(a - off);
    if (off == 0) return w0;
    const uint32_t w1 = lds32(a - off + 4);
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
    uint32_t p0, p1, p2;  // shared addresses of the three planes
    uint32_t meta;        // shared address of float2 meta[K/16]
};

// Quantises one 32-element block held one element per lane (all 32 lanes
// participate).  Writes the lane's three plane bytes and, from lanes 0 and 16,
// the meta of the two 16-element halves.  The largest magnitude comes from one
// redux over the IEEE bits (non-negative floats order like unsigned ints;
// anything >= 0x7F800000 is inf/NaN).
// Byte position of element e inside one activation plane.  The 16-byte
// chunk c = e/16 is stored at chunk c ^ ((c/8) % 8): the eight lanes of a
// quarter-warp that read the four 16-element runs of eight consecutive
// 64-element units then hit eight different 16-byte bank groups.
__device__ __forceinline__ uint32_t pswz(uint32_t e) {
    const uint32_t c = e >> 4;
    return ((c ^ ((c >> 3) & 7u)) << 4) | (e & 15u);
}

// Combines the three plane partial sums into sum(q * X) (one rounding).
__device__ __forceinline__ float planes_combine(int P0, int P1, int P2) {
    int p12 = P1 + (P2 << 8);
    return fmaf(256.0f, static_cast<float>(p12), static_cast<float>(P0));
}

// 24-bit planes of four consecutive elements e0..e0+3 per lane,
// where the 8 lanes 8m..8m+7 of a warp hold one 32-block: block maximum over
// the 8 lanes, 16-run sums over 4 lanes, one 32-bit store per plane.
__device__ __forceinline__ void write_planes4(float4 v, uint8_t* base, int K, int e0, int lane) {
    uint32_t ab = max(max(__float_as_uint(v.x) & 0x7FFFFFFFu, __float_as_uint(v.y) & 0x7FFFFFFFu),
                      max(__float_as_uint(v.z) & 0x7FFFFFFFu, __float_as_uint(v.w) & 0x7FFFFFFFu));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) ab = max(ab, __shfl_xor_sync(0xffffffffu, ab, o));
    float s16 = (v.x + v.y) + (v.z + v.w);
    s16 += __shfl_xor_sync(0xffffffffu, s16, 1);
    s16 += __shfl_xor_sync(0xffffffffu, s16, 2);
    const bool bad = ab >= 0x7F800000u;
    const uint32_t eb = ab >> 23;
    int sh = eb == 0 ? 126 : 21 - (static_cast<int>(eb) - 127);
    sh = sh > 126 ? 126 : sh;
    const float mul = __uint_as_float(static_cast<uint32_t>(sh + 127) << 23);
    float scale = __uint_as_float(static_cast<uint32_t>(127 - sh) << 23);
    if (bad) scale = __uint_as_float(0x7FC00000u);
    const uint32_t X0 = bad ? 0u : static_cast<uint32_t>(__float2int_rn(v.x * mul));
    const uint32_t X1 = bad ? 0u : static_cast<uint32_t>(__float2int_rn(v.y * mul));
    const uint32_t X2 = bad ? 0u : static_cast<uint32_t>(__float2int_rn(v.z * mul));
    const uint32_t X3 = bad ? 0u : static_cast<uint32_t>(__float2int_rn(v.w * mul));
    const uint32_t w0 = (X0 & 255u) | ((X1 & 255u) << 8) | ((X2 & 255u) << 16) | ((X3 & 255u) << 24);
    const uint32_t w1 = ((X0 >> 8) & 255u) | (((X1 >> 8) & 255u) << 8) | (((X2 >> 8) & 255u) << 16) | (((X3 >> 8) & 255u) << 24);
    const uint32_t w2 = ((X0 >> 16) & 255u) | (((X1 >> 16) & 255u) << 8) | (((X2 >> 16) & 255u) << 16) | (((X3 >> 16) & 255u) << 24);
    const uint32_t o = pswz(static_cast<uint32_t>(e0));
    *reinterpret_cast<uint32_t*>(base + o) = w0;
    *reinterpret_cast<uint32_t*>(base + K + o) = w1;
    *reinterpret_cast<uint32_t*>(base + 2 * K + o) = w2;
    if ((lane & 3) == 0) reinterpret_cast<float2*>(base + 3 * K)[e0 >> 4] = make_float2(scale, s16);
}

}  // namespace qmoe
