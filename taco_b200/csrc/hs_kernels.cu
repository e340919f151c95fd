// The CUDA-core kernels of the B200 HardShell backend: embeddings, LayerNorm, the dp4a GEMM
// (reference and small passes), the KV-cache store, causal integer attention and the coder op.
// Every value is exact integer arithmetic with the rules of crates/hardshell/src/int.rs.
#include <cuda_runtime.h>

#include <cstdint>
#include <type_traits>

#include "hs_common.cuh"
#include "hs_kernels.cuh"

namespace hs {

namespace {

__device__ __forceinline__ int64_t warp_max64(int64_t v) {
    for (int o = 16; o > 0; o >>= 1) {
        int64_t w = __shfl_xor_sync(0xffffffffu, v, o);
        v = w > v ? w : v;
    }
    return v;
}
__device__ __forceinline__ uint64_t warp_sum64(uint64_t v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
__device__ __forceinline__ int64_t warp_sums64(int64_t v) {
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// Block reductions for up to 1024 threads (blockDim a multiple of 32). `sh` holds 32 slots.
__device__ int64_t block_max64(int64_t v, int64_t* sh) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_max64(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    int64_t r = lane < nw ? sh[lane] : INT64_MIN;
    r = warp_max64(r);
    return r;
}
__device__ uint64_t block_sum64(uint64_t v, uint64_t* sh) {
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    v = warp_sum64(v);
    __syncthreads();
    if (lane == 0) sh[w] = v;
    __syncthreads();
    uint64_t r = lane < nw ? sh[lane] : 0;
    return warp_sum64(r);
}

// ---- embeddings (crates/hardshell/src/gpt2/ops.rs:52 embed) ----

__global__ void k_embed(const RowInfo* rows, int R, const int8_t* wte, int ldw, const int32_t* em, int es,
                        const int8_t* wpe, const int32_t* pm, int ps, int d, int32_t* x) {
    int r = blockIdx.x;  // rows in x: a pass can have more than 65,535 of them
    int j = blockIdx.y * blockDim.x + threadIdx.x;
    if (r >= R || j >= d) return;
    uint32_t tok = rows[r].token, pos = rows[r].pos;
    int64_t a = rescale64(wte[(size_t)tok * ldw + j], em[tok], es);
    int64_t b = rescale64(wpe[(size_t)pos * d + j], pm[pos], ps);
    x[(size_t)r * d + j] = (int32_t)clamp64(a + b, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
}

// ---- LayerNorm (crates/hardshell/src/layernorm.rs:201-256), one block per row ----

// A LayerNorm output: i8 (out_lo == nullptr), or an i16 value (ln_f_bits = 16) stored as two i8
// planes, hi = floor(v / 256) in `out` and lo = (v mod 256) - 128 in `out_lo`, so that
// v = 256 hi + lo + 128 (the limb split of crates/hardshell-cuda/kernels/hardshell.cu:549-556).
__device__ __forceinline__ void ln_put(int64_t y, int8_t* out, int8_t* out_lo, size_t idx) {
    if (!out_lo) {
        out[idx] = (int8_t)clamp64(y, -127, 127);
        return;
    }
    const int32_t v = (int32_t)clamp64(y, -32767, 32767);
    out[idx] = (int8_t)(v >> 8);
    out_lo[idx] = (int8_t)((v & 255) - 128);
}

__global__ void k_layernorm(const int32_t* x, int R, int d, LnDev ln, int ln_k, int ln_j, uint64_t eps, int8_t* out,
                            int ldo, int8_t* out_lo) {
    __shared__ int64_t sh[32];
    __shared__ uint64_t shu[64];
    int r = blockIdx.x;
    if (r >= R) return;
    const int32_t* xr = x + (size_t)r * d;
    int64_t s = 0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) s += xr[j];
    s = warp_sums64(s);
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5, nw = blockDim.x >> 5;
    if (lane == 0) sh[w] = s;
    __syncthreads();
    int64_t sum = 0;
    for (int i = 0; i < nw; i++) sum += sh[i];
    int64_t mean = floor_div64(sum, d);
    u128 sq = 0;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        int64_t c = (int64_t)xr[j] - mean;
        uint64_t a = c < 0 ? (uint64_t)(-c) : (uint64_t)c;
        sq += (u128)a * a;
    }
    // Reduce the 128-bit sums with the two halves and a carry.
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t lo = (uint64_t)sq, hi = (uint64_t)(sq >> 64);
        uint64_t lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
        uint64_t hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
        sq += ((u128)hi2 << 64) | lo2;
    }
    __syncthreads();
    if (lane == 0) {
        shu[2 * w] = (uint64_t)sq;
        shu[2 * w + 1] = (uint64_t)(sq >> 64);
    }
    __syncthreads();
    u128 sum_sq = 0;
    for (int i = 0; i < nw; i++) sum_sq += ((u128)shu[2 * i + 1] << 64) | shu[2 * i];
    u128 var = sum_sq / (u128)d;
    u128 root = isqrt128((var << (2 * ln_j)) + (u128)eps);
    if (root < 1) root = 1;
    i128 inv = (i128)(((u128)1 << ln_k) / root);
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        i128 t = (i128)((int64_t)xr[j] - mean) * inv * (i128)ln.g[j];
        i128 y;
        if (ln.beta_frac == 0) {
            y = shift_round128((i128)((u128)t * (u128)(i128)ln.m), ln.s, 126) + (i128)ln.b[j];
        } else {
            i128 c = (i128)ln.b[j] << (ln.s - ln.beta_frac);
            y = shift_round128((i128)((u128)t * (u128)(i128)ln.m + (u128)c), ln.s, 126);
        }
        ln_put((int64_t)clamp128(y, -32767, 32767), out, out_lo, (size_t)r * ldo + j);
    }
}

// ---- residual add + LayerNorm, one warp per row ----
//
// x = clamp(x + delta, -R, R) (the residual step of reference.rs:224-231; the delta of the GEMM is
// already clamped to i32, which gives the same value because |x| <= R), then the LayerNorm of
// layernorm.rs:201-256 with t * m = (x - mean) * g * (inv * m): the per-row factor inv * m is one
// 128-bit value, so an output costs one 64 x 128-bit product, a shift and a clamp. The row stays in
// registers (RPL values per lane).
template <int RPL>
__global__ void __launch_bounds__(256, RPL <= 32 ? 4 : 1) k_resid_ln(int32_t* x, const int32_t* delta, int R, int d, LnDev ln, int ln_k,
                                                  int ln_j, uint64_t eps, int8_t* out, int ldo, int8_t* out_lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= R) return;
    int32_t* xr = x + (size_t)r * d;
    int32_t v[RPL];
    int64_t sum = 0;
#pragma unroll
    for (int i = 0; i < RPL; i++) {
        int j = lane + 32 * i;
        int32_t xv = 0;
        if (j < d) {
            xv = xr[j];
            if (delta) {
                xv = (int32_t)clamp64((int64_t)xv + delta[(size_t)r * d + j], -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
                xr[j] = xv;
            }
        }
        v[i] = xv;
        sum += xv;
    }
    sum = warp_sums64(sum);
    const int64_t mean = floor_div64(sum, d);
    uint64_t lo = 0, hi = 0;
#pragma unroll
    for (int i = 0; i < RPL; i++) {
        int j = lane + 32 * i;
        if (j < d) {
            int64_t c = (int64_t)v[i] - mean;
            uint64_t a = c < 0 ? (uint64_t)(-c) : (uint64_t)c;
            uint64_t sq = a * a;  // |c| < 2^32, so c^2 < 2^64
            lo += sq;
            hi += lo < sq ? 1 : 0;
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
        uint64_t hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
        lo += lo2;
        hi += hi2 + (lo < lo2 ? 1 : 0);
    }
    const u128 sum_sq = ((u128)hi << 64) | lo;
    const u128 var = udiv128_u32(sum_sq, (uint32_t)d);  // var < 2^64 (layernorm.rs bounds)
    const u128 sq_arg = (var << (2 * ln_j)) + (u128)eps;  // < 2^97
    uint64_t root = isqrt_u128_fast(sq_arg);
    if (root < 1) root = 1;
    const i128 inv = (i128)((1ULL << ln_k) / root);     // 2^K <= 2^48
    const i128 u = inv * (i128)ln.m;  // |u| < 2^80
    const int s = ln.s;
    // The estimate t ~ cg * u / 2^s in double: cg is exact (|cg| < 2^47) and ud has a relative
    // error of at most 2^-53, so for |t| < 2^20 the estimate of t + 1/2 is within 2^-31 of the
    // exact value and its floor is exact unless the fraction is within 2^-30 of an integer. Those
    // values, |t| >= 2^20, and the beta_frac form take the exact 128-bit rule below.
    const bool est_ok = ln.beta_frac == 0 && s <= 126;
    const double ud = u128_to_double_signed(u) * exp2_neg(s);
#pragma unroll
    for (int i = 0; i < RPL; i++) {
        int j = lane + 32 * i;
        if (j >= d) continue;
        int64_t cg = ((int64_t)v[i] - mean) * (int64_t)ln.g[j];  // |cg| < 2^47
        int64_t yv;
        bool done = false;
        if (est_ok) {
            const double z = fma((double)cg, ud, 0.5);
            if (fabs(z) < 1048576.0) {
                const double fl = floor(z);
                const double fr = z - fl;
                if (fr > 9.313225746154785e-10 && fr < 1.0 - 9.313225746154785e-10) {
                    yv = (int64_t)fl + (int64_t)ln.b[j];
                    done = true;
                }
            }
        }
        if (!done) {
            i128 p = (i128)cg * u;  // t * m, |p| < 2^126
            i128 y;
            if (ln.beta_frac == 0) {
                y = shift_round128(p, s, 126) + (i128)ln.b[j];
            } else {
                i128 cb = (i128)ln.b[j] << (s - ln.beta_frac);
                y = shift_round128((i128)((u128)p + (u128)cb), s, 126);
            }
            yv = clamp128(y, -32767, 32767);
        }
        ln_put(yv, out, out_lo, (size_t)r * ldo + j);
    }
}

// The exact LayerNorm output rule for one value (layernorm.rs:201-256): kept out of line, as the
// vector kernel below takes it only for values whose double estimate is too close to call.
__device__ __noinline__ int64_t ln_exact(int64_t cg, i128 u, int s, int32_t b, int beta_frac) {
    i128 p = (i128)cg * u;
    i128 y;
    if (beta_frac == 0) {
        y = shift_round128(p, s, 126) + (i128)b;
    } else {
        i128 cb = (i128)b << (s - beta_frac);
        y = shift_round128((i128)((u128)p + (u128)cb), s, 126);
    }
    return (int64_t)clamp128(y, -32767, 32767);
}

// The same fused step for rows of exactly 128 * NV values (GPT-2: NV = 6): each lane holds groups
// of four consecutive values, so every load and store is a 16-byte vector (the output a 4-byte
// word), and the row width is a compile-time constant, so the divisions by it become
// multiplications. A row is taken by WPR warps (warp w of the row: the groups w * NV / WPR ..),
// whose sums meet in shared memory (s_red: WPR * 3 words) when WPR > 1.
template <int NV, int WPR>
__device__ __forceinline__ void resid_ln_row(int32_t* x, const int32_t* delta, int r, int w, int lane, const LnDev& ln,
                                             int ln_k, int ln_j, uint64_t eps, int8_t* out, int ldo,
                                             int8_t* out_lo, uint64_t* s_red) {
    constexpr int D = 128 * NV;
    constexpr int NW = NV / WPR;  // 16-byte groups per lane
    static_assert(NV % WPR == 0, "the warps of a row take equal parts");
    int4* xr = reinterpret_cast<int4*>(x + (size_t)r * D) + 32 * NW * w + lane;
    int4 v[NW];
#pragma unroll
    for (int i = 0; i < NW; i++) v[i] = xr[32 * i];
    if (delta) {
        const int4* dr = reinterpret_cast<const int4*>(delta + (size_t)r * D) + 32 * NW * w + lane;
        int4 dv[NW];
#pragma unroll
        for (int i = 0; i < NW; i++) dv[i] = __ldcs(dr + 32 * i);
        // clamp(x + delta, -R, R): |x| <= R < 2^31, so the saturating 32-bit sum clamped to
        // [-R, R] is exact.
        auto radd = [](int32_t a, int32_t b) {
            int32_t t;
            asm("add.sat.s32 %0, %1, %2;" : "=r"(t) : "r"(a), "r"(b));
            return min(max(t, -RESIDUAL_LIMIT), RESIDUAL_LIMIT);
        };
#pragma unroll
        for (int i = 0; i < NW; i++) {
            v[i].x = radd(v[i].x, dv[i].x);
            v[i].y = radd(v[i].y, dv[i].y);
            v[i].z = radd(v[i].z, dv[i].z);
            v[i].w = radd(v[i].w, dv[i].w);
            xr[32 * i] = v[i];
        }
    }
    // Pairs of values (|x| <= R < 2^30) add in 32 bits without overflow.
    int64_t sum = 0;
#pragma unroll
    for (int i = 0; i < NW; i++) sum += (int64_t)(v[i].x + v[i].y) + (int64_t)(v[i].z + v[i].w);
    sum = warp_sums64(sum);
    if constexpr (WPR > 1) {
        if (lane == 0) s_red[w] = (uint64_t)sum;
        __syncthreads();
        sum = 0;
#pragma unroll
        for (int k = 0; k < WPR; k++) sum += (int64_t)s_red[k];
    }
    const int64_t mean = floor_div64(sum, D);
    // |x - mean| < 2^31, so (x - mean)^2 < 2^62 is one 32x32 -> 64 multiply, and three of them add in
    // 64 bits without overflow; the 128-bit total carries between the groups of three.
    const int32_t mean32 = (int32_t)mean;
    uint64_t lo = 0, hi = 0;
    auto sq = [&](int32_t xv) {
        const int32_t c = xv - mean32;
        return (uint64_t)((int64_t)c * (int64_t)c);
    };
    auto acc3 = [&](uint64_t t) {
        lo += t;
        hi += lo < t ? 1 : 0;
    };
    int32_t xs_all[4 * NW];
#pragma unroll
    for (int i = 0; i < NW; i++) {
        xs_all[4 * i] = v[i].x;
        xs_all[4 * i + 1] = v[i].y;
        xs_all[4 * i + 2] = v[i].z;
        xs_all[4 * i + 3] = v[i].w;
    }
#pragma unroll
    for (int k = 0; k < 4 * NW; k += 3) {
        uint64_t t = sq(xs_all[k]);
        if (k + 1 < 4 * NW) t += sq(xs_all[k + 1]);
        if (k + 2 < 4 * NW) t += sq(xs_all[k + 2]);
        acc3(t);
    }
    for (int o = 16; o > 0; o >>= 1) {
        uint64_t lo2 = __shfl_xor_sync(0xffffffffu, lo, o);
        uint64_t hi2 = __shfl_xor_sync(0xffffffffu, hi, o);
        lo += lo2;
        hi += hi2 + (lo < lo2 ? 1 : 0);
    }
    if constexpr (WPR > 1) {
        if (lane == 0) {
            s_red[WPR + 2 * w] = lo;
            s_red[WPR + 2 * w + 1] = hi;
        }
        __syncthreads();
        lo = 0;
        hi = 0;
#pragma unroll
        for (int k = 0; k < WPR; k++) {
            const uint64_t lo2 = s_red[WPR + 2 * k];
            lo += lo2;
            hi += s_red[WPR + 2 * k + 1] + (lo < lo2 ? 1 : 0);
        }
    }
    const u128 sum_sq = ((u128)hi << 64) | lo;
    const u128 var = udiv128_u32(sum_sq, (uint32_t)D);
    const u128 sq_arg = (var << (2 * ln_j)) + (u128)eps;
    uint64_t root = isqrt_u128_fast(sq_arg);
    if (root < 1) root = 1;
    // floor(2^K / root) (K <= 48): the correctly rounded double quotient, then exact corrections.
    const uint64_t num = 1ULL << ln_k;
    uint64_t q = (uint64_t)((double)num / (double)root);
    while (q * root > num) q--;
    while ((q + 1) * root <= num) q++;
    const i128 u = (i128)q * (i128)ln.m;  // |u| < 2^80
    const int s = ln.s;
    const bool est_ok = ln.beta_frac == 0 && s <= 126;
    const double ud = u128_to_double_signed(u) * exp2_neg(s);
    uint32_t* orow = reinterpret_cast<uint32_t*>(out + (size_t)r * ldo) + 32 * NW * w + lane;
    uint32_t* lrow = out_lo ? reinterpret_cast<uint32_t*>(out_lo + (size_t)r * ldo) + 32 * NW * w + lane : nullptr;
#pragma unroll
    for (int i = 0; i < NW; i++) {
        const int j0 = 128 * (NW * w + i) + 4 * lane;
        const uint2 graw = *reinterpret_cast<const uint2*>(ln.g + j0);
        const int4 bv = *reinterpret_cast<const int4*>(ln.b + j0);
        const int32_t xs[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
        const int32_t gs[4] = {(int16_t)(graw.x & 0xFFFF), (int16_t)(graw.x >> 16), (int16_t)(graw.y & 0xFFFF),
                               (int16_t)(graw.y >> 16)};
        const int32_t bs[4] = {bv.x, bv.y, bv.z, bv.w};
        uint32_t word = 0, lword = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t cg = (int64_t)(xs[k] - mean32) * (int64_t)gs[k];  // |cg| < 2^47
            int64_t yv;
            bool done = false;
            if (est_ok) {
                const double z = fma((double)cg, ud, 0.5);
                if (fabs(z) < 1048576.0) {
                    const double fl = floor(z);
                    const double fr = z - fl;
                    if (fr > 9.313225746154785e-10 && fr < 1.0 - 9.313225746154785e-10) {
                        yv = (int64_t)fl + (int64_t)bs[k];
                        done = true;
                    }
                }
            }
            if (!done) yv = ln_exact(cg, u, s, bs[k], ln.beta_frac);
            if (!lrow) {
                word |= (uint32_t)(uint8_t)(int8_t)clamp64(yv, -127, 127) << (8 * k);
            } else {
                // An i16 output as two planes (ln_put).
                const int32_t v = (int32_t)clamp64(yv, -32767, 32767);
                word |= (uint32_t)(uint8_t)(int8_t)(v >> 8) << (8 * k);
                lword |= (uint32_t)(uint8_t)(int8_t)((v & 255) - 128) << (8 * k);
            }
        }
        orow[32 * i] = word;
        if (lrow) lrow[32 * i] = lword;
    }
}


// One warp per row, 8 rows per block (passes with many rows).
template <int NV>
__global__ void __launch_bounds__(256, 4) k_resid_ln_v(int32_t* x, const int32_t* delta, int R, LnDev ln, int ln_k,
                                                       int ln_j, uint64_t eps, int8_t* out, int ldo, int8_t* out_lo) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r = blockIdx.x * 8 + warp;
    if (r >= R) return;
    resid_ln_row<NV, 1>(x, delta, r, 0, lane, ln, ln_k, ln_j, eps, out, ldo, out_lo, nullptr);
}

// WPR warps per row, one row per block (passes of few rows, such as a decode step: more warps in
// flight and a shorter chain per warp).
template <int NV, int WPR>
__global__ void __launch_bounds__(32 * WPR) k_resid_ln_split(int32_t* x, const int32_t* delta, int R, LnDev ln,
                                                             int ln_k, int ln_j, uint64_t eps, int8_t* out, int ldo,
                                                             int8_t* out_lo) {
    __shared__ uint64_t s_red[3 * WPR];
    const int r = blockIdx.x;  // every thread of the block takes part in the barriers
    resid_ln_row<NV, WPR>(x, delta, r, threadIdx.x >> 5, threadIdx.x & 31, ln, ln_k, ln_j, eps, out, ldo, out_lo,
                          s_red);
}

__global__ void k_resid_add(int32_t* x, const int32_t* delta, size_t n) {
    size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i < n) x[i] = (int32_t)clamp64((int64_t)x[i] + delta[i], -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
}

// ---- the GEMM epilogue for one element (shared by the dp4a GEMM) ----

__device__ __forceinline__ void epi_store(int mode, const EpiArgs& e, int r, int n, int32_t acc) {
    if (mode == EPI_RAW) {
        e.out32[(size_t)r * e.ldo + n] = acc;
        return;
    }
    int64_t v = (int64_t)acc + (int64_t)e.b[n];
    int64_t y = rescale64(v, e.m[n], e.s);
    if (mode == EPI_ACT) {
        e.out8[(size_t)r * e.ldo + n] = (int8_t)clamp64(y, -127, 127);
    } else if (mode == EPI_GELU) {
        int64_t in = clamp64(y, -e.gelu_off, e.gelu_off - 1);
        e.out8[(size_t)r * e.ldo + n] = e.gelu[in + e.gelu_off];
    } else if (mode == EPI_RESID) {
        int32_t* xp = &e.x[(size_t)r * e.ldx + n];
        *xp = (int32_t)clamp64((int64_t)*xp + y, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
    } else if (mode == EPI_DELTA) {
        e.out32[(size_t)r * e.ldo + n] = (int32_t)clamp64(y, INT32_MIN, INT32_MAX);
    } else if (mode == EPI_QKV) {
        int8_t o = (int8_t)clamp64(y, -127, 127);
        const RowInfo ri = e.rows[r];
        if (n < e.d) {
            e.out8[(size_t)r * e.ldo + n] = o;
        } else {
            const int j = n < 2 * e.d ? n - e.d : n - 2 * e.d;
            const int h = j / e.hd, c = j - h * e.hd;
            const size_t head = ((size_t)ri.slot * e.L + e.layer) * e.H + h;
            if (n < 2 * e.d) e.kc[(head * e.n_ctx + ri.pos) * e.hd + c] = o;
            else e.vc[(head * e.hd + c) * e.n_ctx + ri.pos] = o;
        }
    }
}

// ---- the dp4a GEMM: a block of 256 threads computes 8 rows x 256 columns ----

constexpr int SG_ROWS = 8;

__global__ void __launch_bounds__(256) k_gemm_simple(int mode, const int8_t* A, int lda, int R, LinearDev W,
                                                     EpiArgs e) {
    __shared__ int4 sa[SG_ROWS][8];  // 8 rows x 128 bytes of K
    __shared__ int64_t red[SG_ROWS][8];
    int n = blockIdx.y * 256 + threadIdx.x;
    int r0 = blockIdx.x * SG_ROWS;  // row groups in x: up to 2^20 rows
    int32_t acc[SG_ROWS];
#pragma unroll
    for (int i = 0; i < SG_ROWS; i++) acc[i] = 0;
    const int8_t* wrow = W.w + (size_t)(n < W.Np ? n : 0) * W.Kp;
    for (int k0 = 0; k0 < W.Kp; k0 += 128) {
        __syncthreads();
        if (threadIdx.x < SG_ROWS * 8) {
            int rr = threadIdx.x >> 3, c = threadIdx.x & 7;
            int r = r0 + rr;
            int4 v = make_int4(0, 0, 0, 0);
            if (r < R) v = *reinterpret_cast<const int4*>(A + (size_t)r * lda + k0 + 16 * c);
            sa[rr][c] = v;
        }
        __syncthreads();
#pragma unroll
        for (int c = 0; c < 8; c++) {
            int4 wv = *reinterpret_cast<const int4*>(wrow + k0 + 16 * c);
#pragma unroll
            for (int i = 0; i < SG_ROWS; i++) {
                int4 av = sa[i][c];
                acc[i] = __dp4a(wv.x, av.x, acc[i]);
                acc[i] = __dp4a(wv.y, av.y, acc[i]);
                acc[i] = __dp4a(wv.z, av.z, acc[i]);
                acc[i] = __dp4a(wv.w, av.w, acc[i]);
            }
        }
    }
    if (mode != EPI_LOGITS) {
        if (n < e.N)
            for (int i = 0; i < SG_ROWS; i++)
                if (r0 + i < R) epi_store(mode, e, r0 + i, n, acc[i]);
        return;
    }
    // Logits: l = clamp(rescale(acc, m[n], s), +-2^40); per row the max over each 128 columns
    // of the block (one logits tile: warps 0-3 and warps 4-7), then d16 = min(tmax - l, last).
    int64_t l[SG_ROWS];
    int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
#pragma unroll
    for (int i = 0; i < SG_ROWS; i++) {
        l[i] = n < e.N ? clamp64(rescale64(acc[i], e.m[n], e.s), -SCORE_LIMIT, SCORE_LIMIT) : -SCORE_LIMIT;
        int64_t mx = warp_max64(l[i]);
        if (lane == 0) red[i][w] = mx;
    }
    __syncthreads();
    const int hq = w >> 2;  // which 128 columns
    const int tile = blockIdx.y * 2 + hq;  // column groups of 256 in y
#pragma unroll
    for (int i = 0; i < SG_ROWS; i++) {
        int64_t tm = red[i][4 * hq];
        for (int q = 1; q < 4; q++) tm = red[i][4 * hq + q] > tm ? red[i][4 * hq + q] : tm;
        int r = r0 + i;
        if (r < R) {
            if (n < e.N) {
                int64_t dd = tm - l[i];
                e.d16[(size_t)r * e.ldd + n] = (uint16_t)(dd < e.last ? dd : e.last);
            }
            if ((threadIdx.x & 127) == 0 && tile < e.ldt) e.tmax[(size_t)r * e.ldt + tile] = tm;
        }
    }
}

// ---- the KV cache: keys [slot, layer, head, pos, hd]; values transposed [slot, layer, head, hd, pos]
// (the values layout of crates/hardshell/src/gpt2/attention.rs:48, so p.v is a dot product along
// the positions of one channel) ----

// One block per (32-row group, 64 channels): 8 threads per row, 8 channels each. Every byte
// lands in its own 32-byte sector of vc (one position of a channel row), so the stores are
// spread over all SMs instead of the few CTAs of the QKV GEMM that hold the v columns.
constexpr int VS_CH = 64;
__global__ void __launch_bounds__(256) k_v_scatter(const RowInfo* rows, int R, const int8_t* vstage, int ldv, int d,
                                                   int H, int hd, int L, int layer, int n_ctx, int8_t* vc) {
    const int r0 = blockIdx.x * 32, lane = threadIdx.x & 31;
    // Every warp reads the group's rows itself (no block barrier needed).
    if (vt_run_warp(rows, r0, R, n_ctx, lane)) return;
    const int r = r0 + (threadIdx.x >> 3);
    if (r >= R) return;
    const RowInfo ri = rows[r];
    const int c0 = blockIdx.y * VS_CH + (threadIdx.x & 7) * 8;
#pragma unroll
    for (int k = 0; k < 8; k++) {
        const int j = c0 + k;
        if (j < d) {
            const int h = j / hd, c = j - h * hd;
            const size_t head = ((size_t)ri.slot * L + layer) * H + h;
            vc[(head * hd + c) * n_ctx + ri.pos] = vstage[(size_t)r * ldv + j];
        }
    }
}

// ---- causal attention of one row and one head (crates/hardshell/src/gpt2/reference.rs:252-284) ----

constexpr int ATT_THREADS = 128;

// attention.rs:36 digits: p = d0 + 2^8 d1 + 2^16 d2 + 2^24 d3 with each d in -128..127.
__device__ __forceinline__ void balanced_digits(int64_t p, int8_t* d) {
    int64_t rest = p;
#pragma unroll
    for (int k = 0; k < 4; k++) {
        int64_t digit = ((rest + 128) & 255) - 128;
        d[k] = (int8_t)digit;
        rest = (rest - digit) >> 8;
    }
}

// The general kernel (any head width): scalar loops. The fast kernel below takes hd % 16 == 0.
__global__ void __launch_bounds__(ATT_THREADS) k_attention(const RowInfo* rows, int R, const int8_t* qkv, int ldq,
                                                           const int8_t* kc, const int8_t* vc, int L, int layer,
                                                           int H, int hd, int n_ctx, int d, int32_t sm, int ss,
                                                           int32_t om, int os, const int32_t* table, int tlen,
                                                           int P, int8_t* att, int lda, const int* rowlist) {
    extern __shared__ int64_t s_sc[];  // n_ctx scores, then weights, then p
    __shared__ int64_t red[32];
    __shared__ uint64_t redu[32];
    __shared__ int8_t q[1024];
    __shared__ int64_t part[ATT_THREADS];
    int h = blockIdx.y, r = rowlist ? rowlist[blockIdx.x] : (int)blockIdx.x;
    if (r >= R) return;
    uint32_t slot = rows[r].slot;
    int n = (int)rows[r].pos + 1;
    for (int c = threadIdx.x; c < hd; c += ATT_THREADS) q[c] = qkv[(size_t)r * ldq + h * hd + c];
    __syncthreads();
    size_t head = (((size_t)slot * L + layer) * H + h) * n_ctx * (size_t)hd;
    const int8_t* K = kc + head;
    const int8_t* Vt = vc + head;
    int64_t mx = INT64_MIN;
    for (int j = threadIdx.x; j < n; j += ATT_THREADS) {
        const int8_t* kr = K + (size_t)j * hd;
        int32_t dot = 0;
        for (int c = 0; c < hd; c++) dot += (int32_t)q[c] * (int32_t)kr[c];
        int64_t sc = clamp64(rescale64(dot, sm, ss), -SCORE_LIMIT, SCORE_LIMIT);
        s_sc[j] = sc;
        mx = sc > mx ? sc : mx;
    }
    mx = block_max64(mx, red);
    // softmax.rs:78: e = table[min(max - s, len - 1)], p = floor((e << P) / sum(e)).
    uint64_t sum = 0;
    int64_t last = tlen - 1;
    for (int j = threadIdx.x; j < n; j += ATT_THREADS) {
        int64_t dd = mx - s_sc[j];
        int64_t e = table[dd < last ? dd : last];
        s_sc[j] = e;
        sum += (uint64_t)e;
    }
    sum = block_sum64(sum, redu);
    if (sum == 0) sum = 1;
    uint64_t rec = (~0ULL) / sum;
    for (int j = threadIdx.x; j < n; j += ATT_THREADS) {
        uint64_t x = (uint64_t)s_sc[j] << P;
        uint64_t qv = __umul64hi(x, rec);
        while ((qv + 1) * sum <= x) qv++;
        s_sc[j] = (int64_t)qv;
    }
    __syncthreads();
    // acc[c] = sum_j p_j v_j[c] in i64; groups of hd threads split the keys.
    int groups = hd <= ATT_THREADS ? ATT_THREADS / hd : 1;
    for (int c0 = 0; c0 < hd; c0 += ATT_THREADS) {
        int c = c0 + (hd <= ATT_THREADS ? threadIdx.x % hd : threadIdx.x);
        int g = hd <= ATT_THREADS ? threadIdx.x / hd : 0;
        int64_t acc = 0;
        if (c < hd && g < groups)
            for (int j = g; j < n; j += groups) acc += s_sc[j] * (int64_t)Vt[(size_t)c * n_ctx + j];
        part[threadIdx.x] = acc;
        __syncthreads();
        if (threadIdx.x < (hd <= ATT_THREADS ? hd : ATT_THREADS) && c < hd) {
            int64_t t = 0;
            if (hd <= ATT_THREADS) {
                for (int gg = 0; gg < groups; gg++) t += part[gg * hd + c];
            } else {
                t = part[threadIdx.x];
            }
            att[(size_t)r * lda + h * hd + c] = (int8_t)clamp128(rescale128(t, om, os), -127, 127);
        }
        __syncthreads();
    }
}

// The fast kernel for a head width HD (a multiple of 16) and n_ctx % 4 == 0: q.k with dp4a over
// 16-byte key loads, and p.v as four dp4a dot products per channel over the balanced base-256
// digits of p (attention.rs:36), four positions per instruction along the transposed values.
// Exact: each digit dot has at most n_ctx terms of magnitude <= 2^14.
template <int HD>
__global__ void __launch_bounds__(ATT_THREADS) k_attention_vec(const RowInfo* rows, int R, const int8_t* qkv,
                                                               int ldq, const int8_t* kc, const int8_t* vc, int L,
                                                               int layer, int H, int n_ctx, int32_t sm, int ss,
                                                               int32_t om, int os, const int32_t* table, int tlen,
                                                               int P, int8_t* att, int lda, const int* rowlist) {
    extern __shared__ __align__(16) uint8_t smem_att[];
    int64_t* s_sc = reinterpret_cast<int64_t*>(smem_att);             // n_ctx: scores, then e
    int4* s_dig = reinterpret_cast<int4*>(smem_att + 8 * (size_t)n_ctx);  // n_ctx / 4 quads x 4 planes
    __shared__ int64_t red[32];
    __shared__ uint64_t redu[32];
    const int h = blockIdx.y, r = rowlist ? rowlist[blockIdx.x] : (int)blockIdx.x;
    if (r >= R) return;
    const uint32_t slot = rows[r].slot;
    const int n = (int)rows[r].pos + 1;
    const int nq = (n + 3) >> 2;
    int32_t qw[HD / 4];
    {
        const int4* qp = reinterpret_cast<const int4*>(qkv + (size_t)r * ldq + h * HD);
#pragma unroll
        for (int i = 0; i < HD / 16; i++) {
            int4 v = qp[i];
            qw[4 * i] = v.x;
            qw[4 * i + 1] = v.y;
            qw[4 * i + 2] = v.z;
            qw[4 * i + 3] = v.w;
        }
    }
    const size_t head = ((size_t)slot * L + layer) * H + h;
    const int4* K = reinterpret_cast<const int4*>(kc + head * n_ctx * HD);
    const int8_t* Vt = vc + head * HD * n_ctx;
    int64_t mx = INT64_MIN;
    for (int j = threadIdx.x; j < n; j += ATT_THREADS) {
        int32_t dot = 0;
#pragma unroll
        for (int i = 0; i < HD / 16; i++) {
            int4 k4 = K[(size_t)j * (HD / 16) + i];
            dot = __dp4a(qw[4 * i], k4.x, dot);
            dot = __dp4a(qw[4 * i + 1], k4.y, dot);
            dot = __dp4a(qw[4 * i + 2], k4.z, dot);
            dot = __dp4a(qw[4 * i + 3], k4.w, dot);
        }
        int64_t sc = clamp64(rescale64(dot, sm, ss), -SCORE_LIMIT, SCORE_LIMIT);
        s_sc[j] = sc;
        mx = sc > mx ? sc : mx;
    }
    mx = block_max64(mx, red);
    uint64_t sum = 0;
    const int64_t last = tlen - 1;
    for (int j = threadIdx.x; j < n; j += ATT_THREADS) {
        int64_t dd = mx - s_sc[j];
        int64_t e = table[dd < last ? dd : last];
        s_sc[j] = e;
        sum += (uint64_t)e;
    }
    sum = block_sum64(sum, redu);
    if (sum == 0) sum = 1;
    const uint64_t rec = (~0ULL) / sum;
    int8_t* dig = reinterpret_cast<int8_t*>(s_dig);
    for (int j = threadIdx.x; j < 4 * nq; j += ATT_THREADS) {
        int8_t dk[4] = {0, 0, 0, 0};
        if (j < n) {
            uint64_t x = (uint64_t)s_sc[j] << P;
            uint64_t qv = __umul64hi(x, rec);
            while ((qv + 1) * sum <= x) qv++;
            balanced_digits((int64_t)qv, dk);
        }
        int qd = j >> 2, i = j & 3;
#pragma unroll
        for (int k = 0; k < 4; k++) dig[16 * (size_t)qd + 4 * k + i] = dk[k];
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int c = warp; c < HD; c += ATT_THREADS / 32) {
        const int32_t* vrow = reinterpret_cast<const int32_t*>(Vt + (size_t)c * n_ctx);
        int32_t a0 = 0, a1 = 0, a2 = 0, a3 = 0;
        for (int qd = lane; qd < nq; qd += 32) {
            int32_t v = vrow[qd];
            int4 dg = s_dig[qd];
            a0 = __dp4a(dg.x, v, a0);
            a1 = __dp4a(dg.y, v, a1);
            a2 = __dp4a(dg.z, v, a2);
            a3 = __dp4a(dg.w, v, a3);
        }
        for (int o = 16; o > 0; o >>= 1) {
            a0 += __shfl_xor_sync(0xffffffffu, a0, o);
            a1 += __shfl_xor_sync(0xffffffffu, a1, o);
            a2 += __shfl_xor_sync(0xffffffffu, a2, o);
            a3 += __shfl_xor_sync(0xffffffffu, a3, o);
        }
        if (lane == 0) {
            int64_t acc = ((((int64_t)a3 * 256 + a2) * 256 + a1) * 256) + a0;
            att[(size_t)r * lda + h * HD + c] = (int8_t)rescale_clamp127(acc, om, (int)os, (double)om * exp2_neg((int)os));
        }
    }
}

// ---- the coder op (crates/taco-coder/src/freq.rs:103 from_weights, interval.rs:82-100) ----

constexpr int CODER_THREADS = 256;
constexpr int CODER_WARPS = CODER_THREADS / 32;
constexpr int CODER_MAX_STEPS = 32;  // steps of 256 symbols per warp: V <= 8 * 32 * 256 = 65536

// One block per row. d16 is read as groups of 8 symbols (one 16-byte load). Every weight is a
// table entry, table[min(d, last)] for the symbol's distance d from the row max, so pass 1 only
// counts the symbols at each distance (shared-memory atomics; the clamped tail has its own
// register count) and W = sum over d of count[d] * table[d]. The table is not increasing and its
// first entry is its largest, and the row max has distance 0, so the largest weight is table[0]:
// the largest symbol (freq.rs:107-117, lowest id on a tie) is the lowest id whose distance is at
// most `head`, the last index with table[head] == table[0]. F[d] = 1 + floor(table[d] * spare / W)
// replaces the counts in place, and sum(f) = sum over d of count[d] * F[d].
// An encode query (kind 0) then sums f over the symbols below its token: one block reduction. A
// decode query walks warp -> step -> lane -> symbol, each level a parallel scan: warp w owns the
// groups [w * gpw, (w + 1) * gpw), lane l the groups w * gpw + l + 32 k (k = the step).
__global__ void __launch_bounds__(CODER_THREADS) k_coder(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt,
                                                         int tsh, int R, int V, const uint64_t* table, int tlen,
                                                         int head, uint32_t bits, const RowInfo* rows, uint64_t* out,
                                                         int* err) {
    extern __shared__ __align__(16) uint32_t F[];  // counts, then 1 + floor(table[j] * spare / W), j <= dmax
    __shared__ int64_t red[32];
    __shared__ uint64_t redu[32];
    __shared__ uint64_t wsum[CODER_WARPS];
    __shared__ uint64_t steps[CODER_WARPS][CODER_MAX_STEPS];
    const int r = blockIdx.x;
    if (r >= R) return;
    const uint16_t* dr = d16 + (size_t)r * ldd;
    const int64_t* tr = tmax + (size_t)r * ldt;
    const int VT = (V + (1 << tsh) - 1) >> tsh;  // logits tiles of 2^tsh columns
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int32_t last = tlen - 1;
    const uint64_t total = 1ULL << bits;
    const uint64_t spare = total - (uint64_t)V;
    const int ng = (V + 7) / 8, ng_full = V / 8;
    for (int j = threadIdx.x; j < tlen / 4; j += CODER_THREADS) reinterpret_cast<uint4*>(F)[j] = make_uint4(0, 0, 0, 0);
    for (int j = 4 * (tlen / 4) + threadIdx.x; j < tlen; j += CODER_THREADS) F[j] = 0;
    // The row max.
    int64_t mx = INT64_MIN;
    for (int t = threadIdx.x; t < VT; t += CODER_THREADS) mx = tr[t] > mx ? tr[t] : mx;
    mx = block_max64(mx, red);  // (its barriers also order the clearing of F)
    // The distance offset of the tile of symbol v0, clamped to last (then every distance is last).
    auto tile_off = [&](int v0) -> int32_t {
        const int64_t o = mx - tr[v0 >> tsh];
        return o < (int64_t)last ? (int32_t)o : last;
    };
    // Pass 1: the distance counts (and, for a decode query, the largest symbol: an encode query
    // finds out where it lies in its prefix pass instead). Two distances at a time in the
    // halfwords of a word: min(off + d, last) is a saturating halfword add, which stops at
    // 65535 > last, then a halfword min, both exact. The clamped ones count in F[last].
    const RowInfo q = rows[r];
    int best = V;
    const uint32_t last2 = (uint32_t)last * 0x10001u;
    const uint32_t head2 = (uint32_t)(head < last ? head : last) * 0x10001u;
    // The largest distance counted, two halfwords at a time (the highest bin that occurs).
    uint32_t dm2 = 0;
    // Groups of 8 symbols, CODER_UNROLL groups per thread and round so that several 16-byte loads
    // are in flight before the counting.
    auto count_group = [&](int v0, uint4 raw, auto track) {
        const int32_t off = tile_off(v0);
        if (off == last) {
            atomicAdd(&F[last], 8u);
            dm2 = last2;
            if constexpr (decltype(track)::value) best = head >= last && v0 < best ? v0 : best;
            return;
        }
        const uint32_t off2 = (uint32_t)off * 0x10001u;
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t near[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t p = __vminu2(__vaddus2(u[k], off2), last2);
            atomicAdd(&F[p & 0xFFFFu], 1u);
            atomicAdd(&F[p >> 16], 1u);
            dm2 = __vmaxu2(dm2, p);
            if constexpr (decltype(track)::value) near[k] = __vcmpleu2(p, head2);
        }
        if constexpr (decltype(track)::value) {
            if ((near[0] | near[1] | near[2] | near[3]) != 0) {
                int first = 8;
#pragma unroll
                for (int k = 3; k >= 0; k--) {
                    if (near[k] >> 16) first = 2 * k + 1;
                    if (near[k] & 0xFFFFu) first = 2 * k;
                }
                best = v0 + first < best ? v0 + first : best;
            }
        }
    };
    constexpr int CODER_UNROLL = 4;
    auto pass1 = [&](auto track) {
        int g0 = threadIdx.x;
        for (; g0 + (CODER_UNROLL - 1) * CODER_THREADS < ng_full; g0 += CODER_UNROLL * CODER_THREADS) {
            uint4 raw[CODER_UNROLL];
#pragma unroll
            for (int k = 0; k < CODER_UNROLL; k++)
                raw[k] = *reinterpret_cast<const uint4*>(dr + 8 * (g0 + k * CODER_THREADS));
#pragma unroll
            for (int k = 0; k < CODER_UNROLL; k++) count_group(8 * (g0 + k * CODER_THREADS), raw[k], track);
        }
        for (; g0 < ng_full; g0 += CODER_THREADS)
            count_group(8 * g0, *reinterpret_cast<const uint4*>(dr + 8 * g0), track);
    };
    if (q.kind == 0) pass1(std::false_type{});
    else pass1(std::true_type{});
    if (ng_full < ng && threadIdx.x == ng_full % CODER_THREADS) {
        const int v0 = 8 * ng_full;
        const int32_t off = tile_off(v0);
        for (int v = v0; v < V; v++) {
            int32_t dd = off + (int32_t)dr[v];
            dd = dd < last ? dd : last;
            atomicAdd(&F[dd], 1u);
            dm2 = (uint32_t)dd > (dm2 & 0xFFFFu) ? (dm2 & 0xFFFF0000u) | (uint32_t)dd : dm2;
            best = dd <= head && v < best ? v : best;
        }
    }
    __syncthreads();  // the counts are complete
    const uint64_t n_last = F[last];
    // The largest distance that occurs: the highest counted bin.
    int32_t dmax = (int32_t)max(dm2 & 0xFFFFu, dm2 >> 16);
    dmax = (int32_t)block_max64(dmax, red);
    const int largest_found = (int)-block_max64(-(int64_t)best, red);
    // W = sum over the distances of count * table (< 2^16 * 2^40: fits in 64 bits).
    uint64_t W = 0;
    for (int j = threadIdx.x; j <= dmax; j += CODER_THREADS)
        W += (uint64_t)(j == last ? (uint32_t)n_last : F[j]) * table[j];
    W = block_sum64(W, redu);
    const bool all_zero = W == 0;
    const int largest = all_zero ? 0 : largest_found;
    const uint32_t f_flat = (uint32_t)(1 + spare / (uint64_t)V);  // all-zero rule: every weight is 1
    // F for the distances that occur (every table entry is <= table[0] <= W, so the quotient is
    // below 2^32), and sum(f).
    uint64_t sum_f = 0;
    if (all_zero) {
        sum_f = (uint64_t)V * f_flat;
    } else {
        // floor(t * spare / W) for a table entry t <= table[0] <= W (so the quotient is at most
        // spare < 2^32): t * (spare / W) in double, the reciprocal ratio taken once per row, is
        // within 2^-19 of the quotient, so its floor is q or q - 1; the remainder t * spare - q W
        // computed mod 2^64 is exact because |t * spare - q W| < 2 W <= 2^57 (t <= 2^40, V <= 2^16),
        // and at most a few exact steps put q right.
        const double ratio = (double)spare / (double)W;
        auto fdiv = [&](uint64_t t) -> uint64_t {
            uint64_t q = (uint64_t)((double)t * ratio);
            int64_t rm = (int64_t)(t * spare - q * W);
            for (int k = 0; k < 4 && rm < 0; k++) {
                q -= 1;
                rm += (int64_t)W;
            }
            for (int k = 0; k < 4 && rm >= (int64_t)W; k++) {
                q += 1;
                rm -= (int64_t)W;
            }
            // The error bound above makes one step enough; a remainder still out of [0, W) means
            // the bound failed for this table, and the call fails instead of coding a wrong q.
            if (rm < 0 || rm >= (int64_t)W) atomicCAS(err, 0, ERR_CODER_DIVISION);
            return q;
        };
        for (int j = threadIdx.x; j <= dmax; j += CODER_THREADS) {
            const uint32_t c = j == last ? (uint32_t)n_last : F[j];
            if (c) {
                const uint32_t f = (uint32_t)(1 + fdiv(table[j]));
                F[j] = f;
                sum_f += (uint64_t)c * f;
            }
        }
        sum_f = block_sum64(sum_f, redu);  // (its barriers also publish F)
    }
    const uint64_t rem = total - sum_f;  // the remainder goes to the largest symbol (freq.rs:150)
    auto f_of = [&](int32_t off, uint32_t d) -> uint32_t {
        int32_t dd = off + (int32_t)d;
        return all_zero ? f_flat : F[dd < last ? dd : last];
    };
    if (q.kind == 0) {
        // Encode: start = sum of f below the token (+ rem if the largest symbol is below it). The
        // largest symbol is the lowest id at a distance <= head, so it lies below the token if any
        // symbol below does, and is the token if none does and the token does.
        const int s = (int)q.value;
        const int gs = s / 8;
        uint64_t pre = 0;
        bool below = false;
        auto group_sum = [&](int v0, uint4 raw) {
            const uint32_t off2 = (uint32_t)tile_off(v0) * 0x10001u;
            const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
            uint32_t gsum = 0;  // 8 frequencies: at most total - (V - 8) < 2^32 for V > 8
            uint32_t dm = last2;
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t p = __vminu2(__vaddus2(u[k], off2), last2);  // as in pass 1
                dm = __vminu2(dm, p);
                gsum += F[p & 0xFFFFu] + F[p >> 16];
            }
            pre += all_zero ? 8ull * f_flat : gsum;
            const uint32_t dmin = min(dm & 0xFFFFu, dm >> 16);
            below |= dmin <= (uint32_t)head;
        };
        int gj = threadIdx.x;
        for (; gj + (CODER_UNROLL - 1) * CODER_THREADS < gs; gj += CODER_UNROLL * CODER_THREADS) {
            uint4 raw[CODER_UNROLL];
#pragma unroll
            for (int k = 0; k < CODER_UNROLL; k++)
                raw[k] = *reinterpret_cast<const uint4*>(dr + 8 * (gj + k * CODER_THREADS));
#pragma unroll
            for (int k = 0; k < CODER_UNROLL; k++) group_sum(8 * (gj + k * CODER_THREADS), raw[k]);
        }
        for (; gj < gs; gj += CODER_THREADS) group_sum(8 * gj, *reinterpret_cast<const uint4*>(dr + 8 * gj));
        if (threadIdx.x == CODER_THREADS - 1) {
            const int32_t off = tile_off(8 * gs);
            for (int v = 8 * gs; v < s; v++) {
                int32_t dd = off + (int32_t)dr[v];
                dd = dd < last ? dd : last;
                below |= dd <= head;
                pre += f_of(off, dr[v]);
            }
        }
        pre = block_sum64(pre, redu);
        below = __syncthreads_or(below) != 0;
        if (threadIdx.x == 0) {
            int32_t ds = tile_off(s) + (int32_t)dr[s];
            ds = ds < last ? ds : last;
            // all_zero: every weight is 1 and symbol 0 is the largest.
            const bool lt = all_zero ? s > 0 : below;
            const bool eq = all_zero ? s == 0 : (!below && ds <= head);
            const uint64_t start = pre + (lt ? rem : 0);
            const uint64_t freq = f_of(tile_off(s), dr[s]) + (eq ? rem : 0);
            out[3 * (size_t)r] = (uint64_t)s;
            out[3 * (size_t)r + 1] = start;
            out[3 * (size_t)r + 2] = freq;
        }
        return;
    }
    // Decode. f of one group of 8 symbols (0 past V).
    auto group_f = [&](int gi, uint32_t (&f)[8]) {
        const int v0 = 8 * gi;
        const uint4 raw = *reinterpret_cast<const uint4*>(dr + v0);
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
        const int32_t off = tile_off(v0);
#pragma unroll
        for (int i = 0; i < 8; i++) f[i] = v0 + i < V ? f_of(off, (u[i >> 1] >> (16 * (i & 1))) & 0xFFFF) : 0u;
    };
    // Pass 2: per warp and step (32 groups), the sum of f.
    const int gpw = (ng + CODER_WARPS - 1) / CODER_WARPS;
    const int ga = min(ng, w * gpw), gb = min(ng, ga + gpw);
    const int nsteps = (gb - ga + 31) / 32;
    uint64_t wtotal = 0;
    for (int k = 0; k < nsteps; k++) {
        const int gi = ga + 32 * k + lane;
        uint64_t s = 0;
        if (gi < gb) {
            uint32_t f[8];
            group_f(gi, f);
#pragma unroll
            for (int i = 0; i < 8; i++) s += f[i];
        }
        s = warp_sum64(s);
        if (lane == 0) steps[w][k] = s;
        wtotal += s;
    }
    if (lane == 0) wsum[w] = wtotal;
    __syncthreads();
    uint64_t before = 0;
    for (int i = 0; i < w; i++) before += wsum[i];
    const int a = 8 * ga, b = min(V, 8 * gb);
    // A(v) = sum of f below v + (rem if v > largest): the start of symbol v.
    auto adj = [&](int v) -> uint64_t { return (uint64_t)v > (uint64_t)largest ? rem : 0; };
    const uint64_t Aa = before + adj(a);
    const uint64_t Ab = b >= V ? total : before + wtotal + adj(b);
    const bool mine = a < b && q.value >= Aa && q.value < Ab;
    if (!mine) return;
    // Level 1: the step. Lane k holds the exclusive prefix of the step sums.
    uint64_t st = lane < nsteps ? steps[w][lane] : 0;
    uint64_t incl = st;
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const uint64_t excl = incl - st;
    // The last step whose start is <= target (starts include rem past the largest symbol).
    int kstep;
    {
        const int v0 = 8 * (ga + 32 * lane);
        const bool ok = lane < nsteps && before + excl + adj(v0) <= q.value;
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        kstep = 31 - __clz(m);
    }
    const uint64_t step_base = before + __shfl_sync(0xffffffffu, excl, kstep);
    // Level 2: the lane (group of 8) within the step.
    const int gi = ga + 32 * kstep + lane;
    uint32_t f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (gi < gb) group_f(gi, f);
    uint64_t gs = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) gs += f[i];
    uint64_t ginc = gs;
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t t = __shfl_up_sync(0xffffffffu, ginc, o);
        if (lane >= o) ginc += t;
    }
    const uint64_t gstart = step_base + ginc - gs;  // sum of f below this group (no rem)
    int owner;
    {
        const bool ok = gi < gb && gstart + adj(8 * gi) <= q.value;
        const unsigned m = __ballot_sync(0xffffffffu, ok);
        owner = 31 - __clz(m);
    }
    if (lane != owner) return;
    // Level 3: the symbol within the group (this lane).
    uint64_t acc = gstart;
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
        const int v = 8 * gi + i;
        if (v >= V) break;
        const uint64_t start = acc + adj(v);
        const uint64_t freq = f[i] + (v == largest ? rem : 0);
        const bool hit = q.value >= start && q.value < start + freq;
        if (hit) {
            out[3 * (size_t)r] = (uint64_t)v;
            out[3 * (size_t)r + 1] = start;
            out[3 * (size_t)r + 2] = freq;
            return;
        }
        acc += f[i];
    }
}

__global__ void k_weights(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                          const uint64_t* table, int tlen, uint64_t* wout) {
    __shared__ int64_t red[32];
    int r = blockIdx.x;
    if (r >= R) return;
    const uint16_t* dr = d16 + (size_t)r * ldd;
    const int64_t* tr = tmax + (size_t)r * ldt;
    int VT = (V + (1 << tsh) - 1) >> tsh;
    int64_t mx = INT64_MIN;
    for (int t = threadIdx.x; t < VT; t += blockDim.x) mx = tr[t] > mx ? tr[t] : mx;
    mx = block_max64(mx, red);
    const int64_t last = tlen - 1;
    for (int v = threadIdx.x; v < V; v += blockDim.x) {
        int64_t dd = mx - tr[v >> tsh] + (int64_t)dr[v];
        wout[(size_t)r * V + v] = table[dd < last ? dd : last];
    }
}

// ---- the mixed coder op of the profile logs (crates/hardshell-cuda/src/mixed.rs:1-20) ----

// floor(t * spare / W) for 0 < t <= W (so the quotient is at most spare < 2^32): the double
// estimate is within one or two of it, and exact 128-bit products put it right.
// A q that the 8 steps do not put right sets the error word (the call fails, nothing is coded
// with it).
__device__ __forceinline__ uint64_t mix_fdiv(uint64_t t, uint64_t spare, uint64_t W, double ratio, int* err) {
    uint64_t q = (uint64_t)((double)t * ratio);
    q = q < spare ? q : spare;
    const u128 x = (u128)t * spare;
    for (int k = 0; k < 8 && (u128)q * W > x; k++) q--;
    for (int k = 0; k < 8 && (u128)(q + 1) * W <= x; k++) q++;
    if ((u128)q * W > x || (u128)(q + 1) * W <= x) atomicCAS(err, 0, ERR_CODER_DIVISION);
    return q;
}

// One block per row, on the d16/tmax output of the logits GEMM as k_coder. Every GPT-2 weight
// is table[min(d, last)] for the symbol's distance d from the row max, and so is every mixed
// weight of a symbol other than the prediction p: g(d) = max(1, (table[d] * m) >> k) with the
// row's mix record (taco-match mixer.rs:491-516 apply), max(1, table[d]) without a prediction
// (mixer.rs:265-269), table[d] for a plain row. g does not increase with d, because the table
// does not. Pass 1 counts the symbols at each distance.
//
// Phase 0, the statistics of the GPT-2 weights (mixed.rs step 1): out = {W, w[p] (0 for a table
// word), top}, top the lowest id at a distance <= head (the first largest weight, table[0]).
// Phase 1: p leaves its bin; W' = sum over d of count[d] g(d) + w'[p], F[d] = 1 + floor(g(d)
// spare / W') and f_p = 1 + floor(w'[p] spare / W') (freq.rs:103-157 from_weights). The largest
// mixed weight is max(g(dmin), w'[p]), dmin the nearest distance of the other symbols. The
// largest symbol (the lowest id on a tie) is p if w'[p] is the largest weight, or the lowest
// other symbol at a distance <= gh (the last distance with g(d) == g(dmin)) if g(dmin) is and
// that symbol is lower. An encode or decode query is then answered as in k_coder.
__global__ void __launch_bounds__(CODER_THREADS) k_coder_mix(const uint16_t* d16, int ldd, const int64_t* tmax,
                                                             int ldt, int tsh, int R, int V, const uint64_t* table,
                                                             int tlen, int head, uint32_t bits, const RowInfo* rows,
                                                             const MixRow* mix, int phase, uint64_t* out,
                                                             int* err) {
    extern __shared__ __align__(16) uint32_t F[];  // counts, then F[d] of the distances that occur
    __shared__ int64_t red[32];
    __shared__ uint64_t redu[32];
    __shared__ uint64_t wsum[CODER_WARPS];
    __shared__ uint64_t steps[CODER_WARPS][CODER_MAX_STEPS];
    const int r = blockIdx.x;
    if (r >= R) return;
    const uint16_t* dr = d16 + (size_t)r * ldd;
    const int64_t* tr = tmax + (size_t)r * ldt;
    const int VT = (V + (1 << tsh) - 1) >> tsh;
    const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
    const int32_t last = tlen - 1;
    const uint64_t total = 1ULL << bits;
    const uint64_t spare = total - (uint64_t)V;
    const int ng = (V + 7) / 8;
    const MixRow mr = mix[r];
    const bool has_p = mr.p < (uint32_t)V;
    const int p = has_p ? (int)mr.p : -1;
    for (int j = threadIdx.x; j < tlen; j += CODER_THREADS) F[j] = 0;
    int64_t mx = INT64_MIN;
    for (int t = threadIdx.x; t < VT; t += CODER_THREADS) mx = tr[t] > mx ? tr[t] : mx;
    mx = block_max64(mx, red);  // (its barriers also order the clearing of F)
    auto tile_off = [&](int v0) -> int32_t {
        const int64_t o = mx - tr[v0 >> tsh];
        return o < (int64_t)last ? (int32_t)o : last;
    };
    // The distances of the 8 symbols of group gi, two per word: min(off + d, last) as a
    // saturating halfword add and a halfword min (as k_coder). The row stride is a multiple of 8,
    // so the last group loads whole; its halfwords past V are not symbols.
    const uint32_t last2 = (uint32_t)last * 0x10001u;
    auto group_dist = [&](int gi, uint32_t (&pd)[4]) {
        const int v0 = 8 * gi;
        const uint4 raw = *reinterpret_cast<const uint4*>(dr + v0);
        const uint32_t off2 = (uint32_t)tile_off(v0) * 0x10001u;
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
        for (int k = 0; k < 4; k++) pd[k] = __vminu2(__vaddus2(u[k], off2), last2);
    };
    // Bit i: symbol 8 gi + i is at a distance <= lim (lim2 = lim in both halfwords).
    auto near_mask = [&](const uint32_t (&pd)[4], uint32_t lim2) -> uint32_t {
        uint32_t nm = 0;
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const uint32_t c = __vcmpleu2(pd[k], lim2);
            nm |= ((c & 1u) << (2 * k)) | (((c >> 16) & 1u) << (2 * k + 1));
        }
        return nm;
    };
    // Pass 1: the counts, and in phase 0 the lowest symbol at a distance <= head. Whole groups
    // as k_coder's pass 1 (several 16-byte loads in flight, a group whose tile is clamped counted
    // at once); the last, partial group by one thread.
    const int32_t hd = head < last ? head : last;
    const uint32_t head2 = (uint32_t)hd * 0x10001u;
    const int ng_full = V / 8;
    int best = V;
    auto count_group = [&](int v0, uint4 raw, auto track) {
        const int32_t off = tile_off(v0);
        if (off == last) {
            atomicAdd(&F[last], 8u);
            if constexpr (decltype(track)::value) best = hd >= last && v0 < best ? v0 : best;
            return;
        }
        const uint32_t off2 = (uint32_t)off * 0x10001u;
        const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
        uint32_t pd[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            pd[k] = __vminu2(__vaddus2(u[k], off2), last2);
            atomicAdd(&F[pd[k] & 0xFFFFu], 1u);
            atomicAdd(&F[pd[k] >> 16], 1u);
        }
        if constexpr (decltype(track)::value) {
            if (v0 < best) {
                const uint32_t nm = near_mask(pd, head2);
                if (nm) best = v0 + __ffs(nm) - 1;
            }
        }
    };
    constexpr int UNROLL = 4;
    auto pass1 = [&](auto track) {
        int g0 = threadIdx.x;
        for (; g0 + (UNROLL - 1) * CODER_THREADS < ng_full; g0 += UNROLL * CODER_THREADS) {
            uint4 raw[UNROLL];
#pragma unroll
            for (int k = 0; k < UNROLL; k++) raw[k] = *reinterpret_cast<const uint4*>(dr + 8 * (g0 + k * CODER_THREADS));
#pragma unroll
            for (int k = 0; k < UNROLL; k++) count_group(8 * (g0 + k * CODER_THREADS), raw[k], track);
        }
        for (; g0 < ng_full; g0 += CODER_THREADS)
            count_group(8 * g0, *reinterpret_cast<const uint4*>(dr + 8 * g0), track);
    };
    if (phase == 0) pass1(std::true_type{});
    else pass1(std::false_type{});
    if (ng_full < ng && threadIdx.x == ng_full % CODER_THREADS) {
        uint32_t pd[4];
        group_dist(ng_full, pd);
        const int v0 = 8 * ng_full;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (v0 + i < V) {
                const uint32_t d = (pd[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
                atomicAdd(&F[d], 1u);
                if (phase == 0 && d <= (uint32_t)hd && v0 + i < best) best = v0 + i;
            }
    }
    int32_t d_p = 0;
    if (has_p) {
        const int32_t dd = tile_off(p) + (int32_t)dr[p];
        d_p = dd < last ? dd : last;
    }
    if (phase == 1 && has_p && threadIdx.x == 0) atomicSub(&F[d_p], 1u);
    __syncthreads();  // the counts are complete
    if (phase == 0) {
        uint64_t W = 0;  // < 2^16 * 2^40
        for (int j = threadIdx.x; j < tlen; j += CODER_THREADS) W += (uint64_t)F[j] * table[j];
        W = block_sum64(W, redu);
        const int top = (int)-block_max64(-(int64_t)best, red);
        if (threadIdx.x == 0) {
            out[3 * (size_t)r] = W;
            out[3 * (size_t)r + 1] = has_p ? table[d_p] : 0;
            out[3 * (size_t)r + 2] = W == 0 ? 0 : (uint64_t)top;
        }
        return;
    }
    const bool plain = mr.p == MIX_PLAIN;
    const uint64_t mm = has_p ? (uint64_t)mr.m : 1;
    const uint32_t kk = has_p ? mr.k : 0;
    auto g = [&](int32_t d) -> uint64_t {
        const uint64_t t = table[d];
        if (plain) return t;
        const uint64_t x = (uint64_t)(((u128)t * mm) >> kk);  // < 2^62 for t <= R (mixed.rs:17-19)
        return x > 1 ? x : 1;
    };
    // The nearest and the farthest distance of the other symbols.
    int32_t lo = INT32_MAX, hi = -1;
    for (int j = threadIdx.x; j < tlen; j += CODER_THREADS)
        if (F[j]) {
            lo = j < lo ? j : lo;
            hi = j > hi ? j : hi;
        }
    lo = (int32_t)-block_max64(-(int64_t)lo, red);
    hi = (int32_t)block_max64(hi, red);
    const bool has_o = hi >= 0;
    const uint64_t wpm = has_p ? mr.wp : 0;
    uint64_t W = 0;  // W' < 2^63 (mixed.rs:17-19)
    if (has_o)
        for (int j = lo + threadIdx.x; j <= hi; j += CODER_THREADS)
            if (F[j]) W += (uint64_t)F[j] * g(j);
    W = block_sum64(W, redu) + wpm;
    const bool all_zero = W == 0;  // a plain row whose weights are all 0: every weight counts 1
    const uint64_t Wo = has_o ? g(lo) : 0;
    // gh: g does not increase, so g(d) == g(lo) exactly on [lo, gh]; a binary search.
    __shared__ int32_t s_gh;
    if (threadIdx.x == 0) {
        int32_t a = lo, b = last;
        while (has_o && a < b) {
            const int32_t mid = a + (b - a + 1) / 2;
            if (g(mid) == Wo) a = mid;
            else b = mid - 1;
        }
        s_gh = has_o ? a : -1;
    }
    __syncthreads();
    const int32_t gh = s_gh;
    const uint64_t Wmax = Wo > wpm ? Wo : wpm;
    const bool cand_p = has_p && wpm == Wmax;
    const bool cand_o = has_o && Wo == Wmax;
    const uint32_t f_flat = (uint32_t)(1 + spare / (uint64_t)V);
    uint64_t f_p = 0, sum_f;
    if (all_zero) {
        sum_f = (uint64_t)V * f_flat;
    } else {
        const double ratio = (double)spare / (double)W;
        sum_f = 0;
        if (has_o)
            for (int j = lo + threadIdx.x; j <= hi; j += CODER_THREADS) {
                const uint32_t c = F[j];
                if (c) {
                    const uint32_t f = (uint32_t)(1 + mix_fdiv(g(j), spare, W, ratio, err));
                    F[j] = f;
                    sum_f += (uint64_t)c * f;
                }
            }
        sum_f = block_sum64(sum_f, redu);  // (its barriers also publish F)
        if (has_p) {
            f_p = 1 + mix_fdiv(wpm, spare, W, ratio, err);
            sum_f += f_p;
        }
    }
    const uint64_t rem = total - sum_f;  // the remainder goes to the largest symbol (freq.rs:150)
    // f of a symbol at distance d other than p (a bin that p alone occupied holds 0).
    auto fd = [&](uint32_t d) -> uint64_t { return all_zero ? f_flat : F[d]; };
    const RowInfo q = rows[r];
    if (q.kind == 0) {
        // Encode: start = sum of f below the token (+ rem if the largest symbol is below it), as
        // k_coder: 8 frequencies per group summed in 32 bits. In p's group, p's slot takes f_p in
        // place of its bin's F, in 32-bit modular arithmetic: the true sum of 8 distinct symbols is
        // below 2^32 (every other symbol has f >= 1, and V > 8). `below`: some symbol other than p
        // below s is at a distance <= gh.
        const int s = (int)q.value;
        const int gs = s / 8;
        const int gp = has_p ? p / 8 : -1;
        uint64_t pre = 0;
        bool below = false;
        const uint32_t gh2 = (uint32_t)(gh < 0 ? 0 : gh) * 0x10001u;
        if (!all_zero) {
            auto group_sum = [&](int gi, uint4 raw) {
                const int v0 = 8 * gi;
                const uint32_t off2 = (uint32_t)tile_off(v0) * 0x10001u;
                const uint32_t u[4] = {raw.x, raw.y, raw.z, raw.w};
                uint32_t pd[4], gsum = 0, dm = last2;
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    pd[k] = __vminu2(__vaddus2(u[k], off2), last2);
                    dm = __vminu2(dm, pd[k]);
                    gsum += F[pd[k] & 0xFFFFu] + F[pd[k] >> 16];
                }
                if (gi == gp) {
                    gsum += (uint32_t)f_p - F[d_p];
                    below |= (near_mask(pd, gh2) & ~(1u << (p - v0))) != 0;
                } else {
                    below |= (int32_t)min(dm & 0xFFFFu, dm >> 16) <= gh;
                }
                pre += gsum;
            };
            constexpr int UNROLL = 4;
            int gj = threadIdx.x;
            for (; gj + (UNROLL - 1) * CODER_THREADS < gs; gj += UNROLL * CODER_THREADS) {
                uint4 raw[UNROLL];
#pragma unroll
                for (int k = 0; k < UNROLL; k++) raw[k] = *reinterpret_cast<const uint4*>(dr + 8 * (gj + k * CODER_THREADS));
#pragma unroll
                for (int k = 0; k < UNROLL; k++) group_sum(gj + k * CODER_THREADS, raw[k]);
            }
            for (; gj < gs; gj += CODER_THREADS) group_sum(gj, *reinterpret_cast<const uint4*>(dr + 8 * gj));
            if (threadIdx.x == CODER_THREADS - 1 && 8 * gs < s) {
                uint32_t pd[4];
                group_dist(gs, pd);
#pragma unroll
                for (int i = 0; i < 8; i++) {
                    const int v = 8 * gs + i;
                    if (v < s) {
                        const uint32_t d = (pd[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
                        if (v == p) {
                            pre += f_p;
                        } else {
                            pre += F[d];
                            below |= (int32_t)d <= gh;
                        }
                    }
                }
            }
        }
        pre = block_sum64(pre, redu);
        below = __syncthreads_or(below) != 0;
        if (threadIdx.x == 0) {
            uint64_t start, freq;
            if (all_zero) {  // every weight is 1 and symbol 0 is the largest
                start = (uint64_t)s * f_flat + (s > 0 ? rem : 0);
                freq = f_flat + (s == 0 ? rem : 0);
            } else {
                const bool s_is_p = has_p && s == p;
                const int32_t ds0 = tile_off(s) + (int32_t)dr[s];
                const int32_t ds = ds0 < last ? ds0 : last;
                const bool lt = (cand_p && p < s) || (cand_o && below);
                const bool cs = s_is_p ? cand_p : (cand_o && ds <= gh);
                start = pre + (lt ? rem : 0);
                freq = (s_is_p ? f_p : (uint64_t)F[ds]) + (!lt && cs ? rem : 0);
            }
            out[3 * (size_t)r] = (uint64_t)s;
            out[3 * (size_t)r + 1] = start;
            out[3 * (size_t)r + 2] = freq;
        }
        return;
    }
    // Decode. The largest symbol first: the lowest other symbol at a distance <= gh (each thread
    // scans its groups in order, so its first hit is its lowest), or p.
    int largest = 0;
    if (!all_zero) {
        int lo_o = V;
        if (cand_o) {
            const uint32_t gh2 = (uint32_t)gh * 0x10001u;
            for (int gi = threadIdx.x; gi < ng; gi += CODER_THREADS) {
                uint32_t pd[4];
                group_dist(gi, pd);
                const int v0 = 8 * gi;
                uint32_t nm = near_mask(pd, gh2) & (V - v0 >= 8 ? 0xFFu : (1u << (V - v0)) - 1);
                if (p >= v0 && p < v0 + 8) nm &= ~(1u << (p - v0));
                if (nm) {
                    lo_o = v0 + __ffs(nm) - 1;
                    break;
                }
            }
            lo_o = (int)-block_max64(-(int64_t)lo_o, red);
        }
        largest = cand_p && p < lo_o ? p : lo_o;
    }
    // f of one group of 8 symbols (0 past V).
    auto group_f = [&](int gi, uint32_t (&f)[8]) {
        uint32_t pd[4];
        group_dist(gi, pd);
        const int v0 = 8 * gi;
#pragma unroll
        for (int i = 0; i < 8; i++) {
            const int v = v0 + i;
            const uint32_t d = (pd[i >> 1] >> (16 * (i & 1))) & 0xFFFFu;
            f[i] = v >= V ? 0u : (uint32_t)(v == p ? f_p : fd(d));
        }
    };
    // The walk of k_coder: warp -> step -> lane -> symbol. Pass 2: per warp and step (32
    // groups), the sum of f.
    const int gpw = (ng + CODER_WARPS - 1) / CODER_WARPS;
    const int ga = min(ng, w * gpw), gb = min(ng, ga + gpw);
    const int nsteps = (gb - ga + 31) / 32;
    uint64_t wtotal = 0;
    for (int k = 0; k < nsteps; k++) {
        const int gi = ga + 32 * k + lane;
        uint64_t s = 0;
        if (gi < gb) {
            uint32_t f[8];
            group_f(gi, f);
#pragma unroll
            for (int i = 0; i < 8; i++) s += f[i];
        }
        s = warp_sum64(s);
        if (lane == 0) steps[w][k] = s;
        wtotal += s;
    }
    if (lane == 0) wsum[w] = wtotal;
    __syncthreads();
    uint64_t before = 0;
    for (int i = 0; i < w; i++) before += wsum[i];
    const int a = 8 * ga, b = min(V, 8 * gb);
    // A(v) = sum of f below v + (rem if v > largest): the start of symbol v.
    auto adj = [&](int v) -> uint64_t { return (uint64_t)v > (uint64_t)largest ? rem : 0; };
    const uint64_t Aa = before + adj(a);
    const uint64_t Ab = b >= V ? total : before + wtotal + adj(b);
    const bool mine = a < b && q.value >= Aa && q.value < Ab;
    if (!mine) return;
    // Level 1: the step. Lane k holds the exclusive prefix of the step sums.
    uint64_t st = lane < nsteps ? steps[w][lane] : 0;
    uint64_t incl = st;
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t t = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += t;
    }
    const uint64_t excl = incl - st;
    int kstep;
    {
        const int v0 = 8 * (ga + 32 * lane);
        const bool ok = lane < nsteps && before + excl + adj(v0) <= q.value;
        kstep = 31 - __clz(__ballot_sync(0xffffffffu, ok));
    }
    const uint64_t step_base = before + __shfl_sync(0xffffffffu, excl, kstep);
    // Level 2: the lane (group of 8) within the step.
    const int gi = ga + 32 * kstep + lane;
    uint32_t f[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (gi < gb) group_f(gi, f);
    uint64_t gsum = 0;
#pragma unroll
    for (int i = 0; i < 8; i++) gsum += f[i];
    uint64_t ginc = gsum;
    for (int o = 1; o < 32; o <<= 1) {
        uint64_t t = __shfl_up_sync(0xffffffffu, ginc, o);
        if (lane >= o) ginc += t;
    }
    const uint64_t gstart = step_base + ginc - gsum;
    int owner;
    {
        const bool ok = gi < gb && gstart + adj(8 * gi) <= q.value;
        owner = 31 - __clz(__ballot_sync(0xffffffffu, ok));
    }
    if (lane != owner) return;
    // Level 3: the symbol within the group (this lane).
    uint64_t acc = gstart;
#pragma unroll 1
    for (int i = 0; i < 8; i++) {
        const int v = 8 * gi + i;
        if (v >= V) break;
        const uint64_t start = acc + adj(v);
        const uint64_t freq = f[i] + (v == largest ? rem : 0);
        if (q.value >= start && q.value < start + freq) {
            out[3 * (size_t)r] = (uint64_t)v;
            out[3 * (size_t)r + 1] = start;
            out[3 * (size_t)r + 2] = freq;
            return;
        }
        acc += f[i];
    }
}

}  // namespace

cudaError_t configure_core_kernels() {
    cudaError_t e = cudaFuncSetAttribute(k_attention, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_ATTN_CTX * 8);
    if (e != cudaSuccess) return e;
    const int vsmem = 8 * MAX_ATTN_CTX + 16 * (MAX_ATTN_CTX / 4 + 1);
    e = cudaFuncSetAttribute(k_attention_vec<64>, cudaFuncAttributeMaxDynamicSharedMemorySize, vsmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_attention_vec<16>, cudaFuncAttributeMaxDynamicSharedMemorySize, vsmem);
    if (e != cudaSuccess) return e;
    e = cudaFuncSetAttribute(k_coder_mix, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_LOGIT_TABLE * 4);
    if (e != cudaSuccess) return e;
    return cudaFuncSetAttribute(k_coder, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_LOGIT_TABLE * 4);
}

void launch_embed(const RowInfo* rows, int R, const int8_t* wte, int ldw, const int32_t* em, int es,
                  const int8_t* wpe, const int32_t* pm, int ps, int d, int32_t* x, cudaStream_t st) {
    if (R <= 0) return;
    dim3 grid(R, (d + 255) / 256);
    k_embed<<<grid, 256, 0, st>>>(rows, R, wte, ldw, em, es, wpe, pm, ps, d, x);
}

void launch_layernorm(const int32_t* x, int R, int d, const LnDev& ln, int ln_k, int ln_j, uint64_t eps,
                      int8_t* out, int ldo, cudaStream_t st, int8_t* out_lo) {
    if (R <= 0) return;
    k_layernorm<<<R, 256, 0, st>>>(x, R, d, ln, ln_k, ln_j, eps, out, ldo, out_lo);
}

// Up to this many rows a LayerNorm row is split over three warps (the decode steps of an unfold).
constexpr int LN_SPLIT_ROWS = 4096;

void launch_resid_layernorm(int32_t* x, const int32_t* delta, int R, int d, const LnDev& ln, int ln_k, int ln_j,
                            uint64_t eps, int8_t* out, int ldo, cudaStream_t st, int8_t* out_lo) {
    if (R <= 0) return;
    int blocks = (R + 7) / 8;
    if (d == 768 && ldo % 4 == 0 && R <= LN_SPLIT_ROWS) {
        k_resid_ln_split<6, 3><<<R, 96, 0, st>>>(x, delta, R, ln, ln_k, ln_j, eps, out, ldo, out_lo);
    } else if (d == 768 && ldo % 4 == 0) {
        k_resid_ln_v<6><<<blocks, 256, 0, st>>>(x, delta, R, ln, ln_k, ln_j, eps, out, ldo, out_lo);
    } else if (d <= 32 * 24) {
        k_resid_ln<24><<<blocks, 256, 0, st>>>(x, delta, R, d, ln, ln_k, ln_j, eps, out, ldo, out_lo);
    } else if (d <= 32 * 64) {
        k_resid_ln<64><<<blocks, 256, 0, st>>>(x, delta, R, d, ln, ln_k, ln_j, eps, out, ldo, out_lo);
    } else {
        // Wide rows: the residual step as its own pass, then the block-per-row LayerNorm.
        if (delta) {
            size_t n = (size_t)R * d;
            k_resid_add<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, delta, n);
        }
        k_layernorm<<<R, 256, 0, st>>>(x, R, d, ln, ln_k, ln_j, eps, out, ldo, out_lo);
    }
}

void launch_gemm_simple(int mode, const int8_t* A, int lda, int R, const LinearDev& W, const EpiArgs& e,
                        cudaStream_t st) {
    if (R <= 0) return;
    dim3 grid((R + SG_ROWS - 1) / SG_ROWS, W.Np / 256);
    k_gemm_simple<<<grid, 256, 0, st>>>(mode, A, lda, R, W, e);
}

void launch_v_scatter(const RowInfo* rows, int R, const int8_t* vstage, int ldv, int d, int H, int hd, int L,
                      int layer, int n_ctx, int8_t* vc, cudaStream_t st) {
    if (R <= 0) return;
    dim3 grid((R + 31) / 32, (d + VS_CH - 1) / VS_CH);
    k_v_scatter<<<grid, 256, 0, st>>>(rows, R, vstage, ldv, d, H, hd, L, layer, n_ctx, vc);
}

void launch_attention(const RowInfo* rows, int R, const int* rowlist, int n, const int8_t* qkv, int ldq,
                      const int8_t* kc, const int8_t* vc, int L, int layer, int H, int hd, int n_ctx, int d,
                      int32_t sm, int ss, int32_t om, int os, const int32_t* table, int tlen, int P, int8_t* att,
                      int lda, cudaStream_t st) {
    if (R <= 0 || n <= 0) return;
    dim3 grid(n, H);  // rows in x (a pass can have more than 65,535), heads in y
    // The vector kernel needs 16-byte aligned q rows and 4-byte aligned value rows.
    bool vec_ok = (n_ctx % 4) == 0 && (ldq % 16) == 0;
    size_t vsmem = 8 * (size_t)n_ctx + 16 * (size_t)(n_ctx / 4 + 1);
    if (vec_ok && hd == 64) {
        k_attention_vec<64><<<grid, ATT_THREADS, vsmem, st>>>(rows, R, qkv, ldq, kc, vc, L, layer, H, n_ctx, sm, ss,
                                                               om, os, table, tlen, P, att, lda, rowlist);
        return;
    }
    if (vec_ok && hd == 16) {
        k_attention_vec<16><<<grid, ATT_THREADS, vsmem, st>>>(rows, R, qkv, ldq, kc, vc, L, layer, H, n_ctx, sm, ss,
                                                               om, os, table, tlen, P, att, lda, rowlist);
        return;
    }
    size_t smem = (size_t)n_ctx * sizeof(int64_t);
    k_attention<<<grid, ATT_THREADS, smem, st>>>(rows, R, qkv, ldq, kc, vc, L, layer, H, hd, n_ctx, d, sm, ss, om,
                                                  os, table, tlen, P, att, lda, rowlist);
}

void launch_coder(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                  const uint64_t* table, int tlen, int head, uint32_t bits, const RowInfo* rows, uint64_t* out,
                  int* err, cudaStream_t st) {
    if (R <= 0) return;
    k_coder<<<R, CODER_THREADS, (size_t)tlen * 4, st>>>(d16, ldd, tmax, ldt, tsh, R, V, table, tlen, head, bits,
                                                         rows, out, err);
}

void launch_coder_mix(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                      const uint64_t* table, int tlen, int head, uint32_t bits, const RowInfo* rows,
                      const MixRow* mix, int phase, uint64_t* out, int* err, cudaStream_t st) {
    if (R <= 0) return;
    k_coder_mix<<<R, CODER_THREADS, (size_t)tlen * 4, st>>>(d16, ldd, tmax, ldt, tsh, R, V, table, tlen, head, bits,
                                                             rows, mix, phase, out, err);
}

void launch_weights(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                    const uint64_t* table, int tlen, uint64_t* w, cudaStream_t st) {
    if (R <= 0) return;
    k_weights<<<R, 256, 0, st>>>(d16, ldd, tmax, ldt, tsh, R, V, table, tlen, w);
}

}  // namespace hs
