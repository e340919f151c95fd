// Shared device code of the B200 HardShell backend: the exact integer rules of HardShell
// (crates/hardshell/src/int.rs) for device and host, and thin PTX wrappers for sm_100a
// (mbarrier, TMA, tcgen05).
#pragma once

#include <cstdint>
#include <cstring>
#include <cuda_runtime.h>

#define HS_HD __host__ __device__ __forceinline__

namespace hs {

typedef __int128 i128;
typedef unsigned __int128 u128;

constexpr int32_t RESIDUAL_LIMIT = (1 << 30) - 1;  // gpt2/mod.rs:113
constexpr int64_t SCORE_LIMIT = 1LL << 40;         // gpt2/mod.rs:116

// int.rs:110 shift_round for |p| < 2^max_shift: floor((p + 2^(s-1)) / 2^s).
HS_HD i128 shift_round128(i128 p, uint32_t s, uint32_t max_shift) {
    if (s == 0) return p;
    if (s > max_shift) return 0;
    u128 sum = (u128)p + ((u128)1 << (s - 1));
    return ((i128)sum) >> s;
}

// int.rs:63 rescale(x, m, s) for an i64 x: exact, with the product in 128 bits.
HS_HD i128 rescale128(int64_t x, int32_t m, uint32_t s) { return shift_round128((i128)x * (i128)m, s, 95); }

// rescale for |x * m| < 2^63 (the GEMM epilogues: |acc + b| < 2^32, |m| <= 2^31): the result
// floor((p + 2^(s-1)) / 2^s) written as (p >> s) + bit (s-1) of p, so no step overflows.
// For s >= 64 the exact result is 0 because |p| < 2^63 <= 2^(s-1).
HS_HD int64_t rescale64(int64_t x, int32_t m, uint32_t s) {
    int64_t p = x * (int64_t)m;
    if (s == 0) return p;
    if (s >= 64) return 0;
    return (p >> s) + ((p >> (s - 1)) & 1);
}

// int.rs:138 clamp_wide / int.rs:131 clamp (lo wins when the bounds cross).
HS_HD int64_t clamp64(int64_t x, int64_t lo, int64_t hi) {
    int64_t u = x < hi ? x : hi;
    return u > lo ? u : lo;
}
HS_HD int64_t clamp128(i128 x, int64_t lo, int64_t hi) {
    i128 u = x < (i128)hi ? x : (i128)hi;
    i128 c = u > (i128)lo ? u : (i128)lo;
    return (int64_t)c;
}

// int.rs:41 floor_div for b > 0.
HS_HD int64_t floor_div64(int64_t a, int64_t b) {
    int64_t q = a / b, r = a % b;
    return (r != 0 && (r < 0)) ? q - 1 : q;
}

// int.rs:213 isqrt_u128: digit by digit, two bits per round.
HS_HD u128 isqrt128(u128 x) {
    u128 bit = (u128)1 << 126;
    while (bit > x) bit >>= 2;
    u128 rem = x, res = 0;
    while (bit != 0) {
        u128 trial = res + bit;
        if (rem >= trial) {
            rem -= trial;
            res = (res >> 1) + bit;
        } else {
            res >>= 1;
        }
        bit >>= 2;
    }
    return res;
}

__device__ __forceinline__ double u128_to_double(u128 x) {
    return (double)(uint64_t)(x >> 64) * 18446744073709551616.0 + (double)(uint64_t)x;
}

__device__ __forceinline__ double u128_to_double_signed(i128 x) {
    return x < 0 ? -u128_to_double((u128)(-x)) : u128_to_double((u128)x);
}

// 2^-s as a double (exact for 0 <= s <= 1022).
__device__ __forceinline__ double exp2_neg(int s) {
    return __longlong_as_double((long long)(1023 - s) << 52);
}

// clamp(rescale(acc, m, s), -127, 127) (int.rs:63 with the attention output clamp) for
// |acc| < 2^53, with msc = m * 2^-s (exact). The double z = acc * msc + 1/2 has one rounding, so
// for |z| < 1024 it is within 2^-43 of the exact value and its floor is the result unless the
// fraction is within 2^-40 of an integer; those values, and s > 95, take the exact 128-bit rule.
__device__ __forceinline__ int32_t rescale_clamp127(int64_t acc, int32_t m, int s, double msc) {
    const double z = fma((double)acc, msc, 0.5);
    const double fl = floor(z);
    const double fr = z - fl;
    if (s <= 95) {
        if (fabs(z) >= 1024.0) return z > 0 ? 127 : -127;
        if (fr > 9.094947017729282e-13 && fr < 1.0 - 9.094947017729282e-13) return min(max((int32_t)fl, -127), 127);
    }
    return (int32_t)clamp128(rescale128(acc, m, (uint32_t)s), -127, 127);
}

// floor(x / d) for a 128-bit x whose quotient fits in 64 bits, d >= 1: a double estimate and an
// exact integer correction (the estimate is within a few units; each correction is exact).
__device__ __forceinline__ uint64_t udiv128_small(u128 x, uint64_t d) {
    double qd = u128_to_double(x) / (double)d;
    uint64_t q = qd >= 18446744073709551615.0 ? ~0ULL : (uint64_t)qd;
    u128 qw = (u128)q * d;
    while (qw > x) {
        q -= 1;
        qw -= d;
    }
    while (x - qw >= d) {
        q += 1;
        qw += d;
    }
    return q;
}

// 2^k as a double, exact for 0 <= k <= 1023.
HS_HD double pow2_double(int k) {
    const uint64_t bits = (uint64_t)(1023 + k) << 52;
    double d;
    memcpy(&d, &bits, sizeof d);
    return d;
}

// ceil(2^sh / s) for 1 <= s < 2^44, sh <= 108, when the quotient is at most 2^62. The double
// estimate x of 2^sh / s has a relative error below 2^-52, so x is within 2^11 of the quotient and
// the residual R = 2^sh - x s is below 2^56 in magnitude: the low word of its 128-bit two's
// complement is its value. One signed 64-bit division brings |R| below s, and one unit step makes
// x the least value with x s >= 2^sh. No loop, on the device and the host alike.
HS_HD uint64_t ceil_pow2_div(int sh, uint64_t s) {
    uint64_t x = (uint64_t)((1.0 / (double)s) * pow2_double(sh));
    int64_t R = (int64_t)(uint64_t)(((u128)1 << sh) - (u128)x * s);
    const int64_t d = R / (int64_t)s;
    x += (uint64_t)d;
    R -= d * (int64_t)s;
    if (R > 0) x += 1;
    return x;
}

// floor(x / d) for a 128-bit x and a 32-bit d >= 1, with three 64-bit divisions.
__device__ __forceinline__ u128 udiv128_u32(u128 x, uint32_t d) {
    uint64_t hi = (uint64_t)(x >> 64), lo = (uint64_t)x;
    if (hi == 0) return lo / d;
    uint64_t qh = hi / d, r = hi % d;
    uint64_t t1 = (r << 32) | (lo >> 32);
    uint64_t q1 = t1 / d;
    r = t1 % d;
    uint64_t t0 = (r << 32) | (lo & 0xFFFFFFFFull);
    uint64_t q0 = t0 / d;
    return ((u128)qh << 64) | ((u128)q1 << 32) | q0;
}

// floor(sqrt(x)) for x < 2^100: the double square root as an estimate, then exact integer
// corrections (int.rs:213 isqrt_u128 defines the value).
__device__ __forceinline__ uint64_t isqrt_u128_fast(u128 x) {
    uint64_t r = (uint64_t)sqrt(u128_to_double(x));
    while ((u128)r * r > x) r--;
    while ((u128)(r + 1) * (r + 1) <= x) r++;
    return r;
}

// ---- sm_100a PTX wrappers ----

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                     smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t phase) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, "
        "p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(phase)
        : "memory");
    return ok != 0;
}

// A bounded wait: true when the phase completed; false (and the error word set) after about
// `limit` polls. Every wait of the kernels is bounded, so a fault can never hang the GPU.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t phase, int* err, int code) {
    for (uint32_t i = 0; i < (1u << 26); i++) {
        if (mbar_try_wait(bar, phase)) return true;
        if (i > 64) __nanosleep(32);
        if ((i & 1023) == 0 && *(volatile int*)err != 0) return false;
    }
    atomicCAS(err, 0, code);
    return false;
}

// TMA: a 2D tiled load of box {c0, c1} into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(tmap), "r"(c0), "r"(c1), "r"(smem_u32(bar))
        : "memory");
}

// A 2D tiled TMA store from shared memory (a bulk async-group of the issuing thread). The x
// coordinate times the element size is a multiple of 16 bytes and both coordinates are >= 0 at
// every call site; the tensor map clips what lies past its extent.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int c0, int c1) {
    asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
                 "r"(smem_u32(src)), "r"(c0), "r"(c1)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until the issued bulk stores have read their shared-memory source (it may be reused).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// Wait until all but the most recent bulk store group have read their shared-memory source.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
// Wait until the issued bulk stores are complete.
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Order this thread's generic-proxy shared-memory writes before later async-proxy (TMA) reads.
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// An untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global
// to this CTA's shared memory, completing on `bar` (no multicast).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// tcgen05: TMEM allocation (a whole warp), MMA, commit, loads and fences.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] x B[smem desc]^T, kind::i8 (s8/u8 in, s32 accumulators).
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                       uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}

// 32 lanes x 32 bits, 16 columns: thread t of the warp gets columns c..c+15 of lane (base + t).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
}
// 32 lanes x 32 bits, 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
        "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}

// A named barrier among `count` threads (count a multiple of 32).
__device__ __forceinline__ void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The shared-memory matrix descriptor of tcgen05 for a K-major tile written by TMA with the
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart (stride byte offset),
// descriptor version 1 (bits 46-47), layout type 2 = SWIZZLE_128B (bits 61-63).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);   // start address, bits 0-13
    d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
    d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset, bits 32-45
    d |= (uint64_t)1 << 46;                     // version
    d |= (uint64_t)2 << 61;                     // SWIZZLE_128B
    return d;
}

// The instruction descriptor of tcgen05.mma kind::i8: s32 accumulators, A and B K-major.
HS_HD uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

}  // namespace hs
