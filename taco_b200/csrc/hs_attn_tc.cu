// Prefill attention of the B200 HardShell backend on the tensor cores (tcgen05).
//
// One CTA per (group, head): a group is up to 128 rows of one slot at consecutive positions
// pos0 .. pos0 + count - 1, attending causally to the keys 0 .. pos0 + count - 1 of its slot.
// The integer softmax of crates/hardshell/src/softmax.rs:78 needs the exact row max before any
// weight and the exact row sum before any probability, so the scores S = Q K^T are computed
// twice per 128-key chunk on the tensor cores (cheap: K = 64):
//   pass 1: S -> the max and min dot of each row (score() is monotone in the dot, so the max
//           score is max(score(maxdot), score(mindot)), as in the reference GPU kernel);
//   pass 2: S -> the table index d = min(max - score, len - 1) -> e = attn_exp[d] -> the row sum;
//           each key's d (u16) goes to this SM's slot of a scratch buffer in global memory;
//   pass 3: d back from the scratch (no third S) -> p = floor(e * 2^P / sum) (an exact
//           multiply-shift), split into four unsigned bytes p = p0 + 2^8 p1 + 2^16 p2 + 2^24 p3,
//           written to shared memory as four u8 A operands; O_k += P_k V (u8 x s8) in TMEM.
// The scratch slot is picked by %smid: a CTA needs more than half of an SM's shared memory, so at
// most one runs on an SM at a time, and the slots of all SMs (n_ctx u16 per row, 256 KB at
// n_ctx = 1024) stay in L2 between the two passes.
// Then acc = sum_k 2^(8k) O_k (exact: each O_k has at most n_ctx terms below 2^15) and
// att = clamp(rescale(acc, out_m, out_s), -127, 127) (crates/hardshell/src/gpt2/reference.rs:252-284).
//
// Operands come in by TMA (no multicast): Q [128 x 64] and K chunks [128 x 64] with the 64-byte
// swizzle, V^T chunks [64 x 128] with the 128-byte swizzle from the transposed values cache.
// (A fold pass runs this kernel on 96 % of its rows, so one S pass less is most of a pass.)
// Warps 0..15 do the softmax: TMEM lane group warp % 4 (32 rows) and key quarter warp / 4 (32
// of the 128 keys of a chunk). Warp 16 is the TMA producer, warp 17 owns TMEM and issues the
// MMAs: S of chunk i + 1 is issued before P V of chunk i, and P is double-buffered, so the
// softmax warps always have work while the tensor core runs. Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "hs_common.cuh"
#include "hs_kernels.cuh"

namespace hs {

namespace {

constexpr int GM = 128;        // rows of a group (TMEM lanes)
constexpr int KC = 128;        // keys per chunk
constexpr int HDIM = 64;       // head width of this kernel
constexpr int EW = 16;         // softmax warps
constexpr int ETH = 32 * EW;   // softmax threads
constexpr int ATHREADS = ETH + 64;
constexpr int Q_BYTES = GM * HDIM;        // 8 KB
constexpr int K_BYTES = KC * HDIM;        // 8 KB
constexpr int V_BYTES = HDIM * KC;        // 8 KB
constexpr int P_BYTES = 4 * GM * KC;      // 64 KB (four planes), double-buffered
constexpr int TABLE_MAX = 8192;           // attn_exp entries kept in shared memory
// The scratch slot of one SM: per 128-key chunk, key quarter, 16-byte word (8 keys) and row, the
// u16 table indices of 8 keys, so that a warp's 32 rows store and load 512 contiguous bytes.
constexpr size_t SCR_CHUNK_BYTES = 4 * 4 * GM * 16;  // 32 KB per chunk of 128 keys
constexpr size_t ASMEM =
    (size_t)Q_BYTES + 2 * K_BYTES + 2 * V_BYTES + 2 * P_BYTES + 4 * TABLE_MAX + 8 * GM * 8 + 512 + 1024;

struct __align__(8) ABars {
    uint64_t q_full;
    uint64_t k_full[2], k_empty[2];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full[2], s_empty[2];
    uint64_t p_full[2], p_empty[2];
    uint64_t o_full;
    uint64_t t_full;  // the exp table in shared memory
    uint32_t tmem_base;
};

// The shared-memory descriptor of a K-major tile with the 64-byte swizzle (rows of 64 bytes,
// 8-row groups 512 bytes apart), descriptor version 1, layout type 4 = SWIZZLE_64B.
__device__ __forceinline__ uint64_t sdesc_sw64(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(512 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)4 << 61;
    return d;
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ int64_t score_of(int32_t dot, int32_t sm, int ss, bool fast, int64_t h) {
    int64_t y = fast ? (((int64_t)dot * (int64_t)sm + h) >> ss) : rescale64(dot, sm, (uint32_t)ss);
    return clamp64(y, -SCORE_LIMIT, SCORE_LIMIT);
}

// The table index min(max - score, last). NARROW (21 <= ss <= 62): |dot| <= 64 * 2^14 = 2^20 and
// |sm| <= 2^31, so |score| < 2^30 (no clamp at 2^40) and the distance fits in 32 bits. The
// distance is never negative (max is the row's largest score); the unsigned comparison keeps the
// index inside the table for any input all the same, at no cost.
template <bool NARROW>
__device__ __forceinline__ int32_t dist_of(int64_t M, int32_t dot, int32_t sm, int ss, bool fast, int64_t h,
                                           int32_t last) {
    if (NARROW) {
        int32_t dd = (int32_t)M - (int32_t)(((int64_t)dot * (int64_t)sm + h) >> ss);
        return (uint32_t)dd < (uint32_t)last ? dd : last;
    } else {
        int64_t dd = M - score_of(dot, sm, ss, fast, h);
        return (int32_t)((uint64_t)dd < (uint64_t)last ? dd : (int64_t)last);
    }
}

template <bool NARROW, bool SSHI>
__global__ void __launch_bounds__(ATHREADS, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnGroup* groups, int L, int layer, int H,
                   int n_ctx, int32_t sm, int ss, int32_t om, int os, const int32_t* table, int tlen, int P,
                   int8_t* att, int lda, uint8_t* scratch, int scr_slots, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint32_t smid;
    asm("mov.u32 %0, %%smid;" : "=r"(smid));
    if (smid >= (uint32_t)scr_slots) {  // the same for every thread of the CTA: nothing started yet
        if (threadIdx.x == 0) atomicCAS(err, 0, ERR_ATTN_SCRATCH);
        return;
    }
    // Aligned to 1,024 bytes by an offset from the __shared__ array itself (not through an
    // integer cast), so every access below stays a shared-memory access with 32-bit addresses.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sQ = smem;
    uint8_t* sK = sQ + Q_BYTES;                 // 2 x 8 KB
    uint8_t* sV = sK + 2 * K_BYTES;             // 2 x 8 KB
    uint8_t* sP = sV + 2 * V_BYTES;             // 2 x 4 planes x 16 KB
    int32_t* sT = reinterpret_cast<int32_t*>(sP + 2 * P_BYTES);
    int64_t* sX = reinterpret_cast<int64_t*>(sT + TABLE_MAX);  // [2][4][GM] row exchange
    ABars* bars = reinterpret_cast<ABars*>(sX + 8 * GM);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const AttnGroup grp = groups[blockIdx.x];
    const int h = blockIdx.y;
    const int n_keys = (int)grp.pos0 + (int)grp.count;
    const int nch = (n_keys + KC - 1) / KC;
    const size_t head = ((size_t)grp.slot * L + layer) * H + h;

    if (threadIdx.x == 0) {
        mbar_init(&bars->q_full, 1);
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars->k_full[i], 1);
            mbar_init(&bars->k_empty[i], 1);
            mbar_init(&bars->v_full[i], 1);
            mbar_init(&bars->v_empty[i], 1);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->s_empty[i], ETH);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars->p_full[i], ETH);
            mbar_init(&bars->p_empty[i], 1);
        }
        mbar_init(&bars->o_full, 1);
        mbar_init(&bars->t_full, 1);
        fence_barrier_init();
    }
    if (warp == EW + 1) {
        tmem_alloc(&bars->tmem_base, 512);
        tmem_relinquish();
        tc_fence_before();
    }
    const int tl = tlen < TABLE_MAX ? tlen : TABLE_MAX;
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == EW) {
        // TMA producer: Q, then K chunks for the three passes, with the V^T chunks in pass 3.
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
            // The exp table (its buffer is padded to 16 bytes), needed from pass 2 on.
            const uint32_t tbytes = (uint32_t)((tl * 4 + 15) & ~15);
            mbar_arrive_expect_tx(&bars->t_full, tbytes);
            bulk_load(sT, table, tbytes, &bars->t_full);
            mbar_arrive_expect_tx(&bars->q_full, Q_BYTES);
            tma_load_2d(sQ, &tmQ, &bars->q_full, h * HDIM, (int)grp.first_row);
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0;
            bool ok = true;
            // V^T chunk c of pass 3 (both buffers are free at the start: chunks 0 and 1 load first).
            auto load_v = [&](int c) -> bool {
                if (!mbar_wait(&bars->v_empty[vs], vph ^ 1, err, 12)) return false;
                mbar_arrive_expect_tx(&bars->v_full[vs], V_BYTES);
                tma_load_2d(sV + vs * V_BYTES, &tmV, &bars->v_full[vs], c * KC, (int)(head * HDIM));
                if (++vs == 2) {
                    vs = 0;
                    vph ^= 1;
                }
                return true;
            };
            for (int c = 0; c < nch && c < 2 && ok; c++) ok = load_v(c);
            for (int it = 0; it < 2 * nch && ok; it++) {
                int c = it % nch;
                if (!mbar_wait(&bars->k_empty[ks], kph ^ 1, err, 11)) break;
                mbar_arrive_expect_tx(&bars->k_full[ks], K_BYTES);
                tma_load_2d(sK + ks * K_BYTES, &tmK, &bars->k_full[ks], 0, (int)(head * n_ctx) + c * KC);
                if (++ks == 2) {
                    ks = 0;
                    kph ^= 1;
                }
            }
            for (int c = 2; c < nch && ok; c++) ok = load_v(c);
        }
    } else if (warp == EW + 1) {
        // MMA issuer: S of every chunk of passes 1 and 2, then the P V of each chunk of pass 3 as
        // its planes are written (P is double-buffered).
        if (lane == 0) {
            const uint32_t id_s = idesc_i8(GM, KC, true, true);
            const uint32_t id_pv = idesc_i8(GM, HDIM, false, true);
            bool ok = mbar_wait(&bars->q_full, 0, err, 13);
            tc_fence_after();
            const uint32_t qa = smem_u32(sQ);
            int ks = 0, vs = 0;
            uint32_t kph = 0, vph = 0;
            auto do_pv = [&](int c) -> bool {
                const int pb = c & 1;
                if (!mbar_wait(&bars->p_full[pb], (c >> 1) & 1, err, 16)) return false;
                if (!mbar_wait(&bars->v_full[vs], vph, err, 17)) return false;
                tc_fence_after();
                const uint32_t vb = smem_u32(sV + vs * V_BYTES);
#pragma unroll
                for (int pl = 0; pl < 4; pl++) {
                    const uint32_t pa = smem_u32(sP + pb * P_BYTES + pl * (GM * KC));
                    const uint32_t o = tmem + 2 * KC + pl * HDIM;
#pragma unroll
                    for (int k = 0; k < KC / 32; k++)
                        mma_i8(o, sdesc_sw128(pa + 32 * k), sdesc_sw128(vb + 32 * k), id_pv, (c > 0 || k > 0) ? 1u : 0u);
                }
                mma_commit(&bars->v_empty[vs]);
                mma_commit(&bars->p_empty[pb]);
                if (++vs == 2) {
                    vs = 0;
                    vph ^= 1;
                }
                return true;
            };
            for (int it = 0; it < 2 * nch && ok; it++) {
                const int sb = it & 1;
                const uint32_t sph = (it >> 1) & 1;
                if (!mbar_wait(&bars->s_empty[sb], sph ^ 1, err, 14)) break;
                if (!mbar_wait(&bars->k_full[ks], kph, err, 15)) break;
                tc_fence_after();
                const uint32_t kb = smem_u32(sK + ks * K_BYTES);
                const uint32_t d = tmem + sb * KC;
#pragma unroll
                for (int k = 0; k < HDIM / 32; k++)
                    mma_i8(d, sdesc_sw64(qa + 32 * k), sdesc_sw64(kb + 32 * k), id_s, k != 0 ? 1u : 0u);
                mma_commit(&bars->k_empty[ks]);
                mma_commit(&bars->s_full[sb]);
                if (++ks == 2) {
                    ks = 0;
                    kph ^= 1;
                }
            }
            for (int c = 0; c < nch && ok; c++) ok = do_pv(c);
            mma_commit(&bars->o_full);
        }
    } else {
        // Softmax warps: one row per thread, 32 keys of each chunk (quarter qt = warp / 4).
        const int g = warp & 3, qt = warp >> 2;
        const int row = g * 32 + lane;
        const int rpos = (int)grp.pos0 + row;  // rows past the group compute harmless values
        const uint32_t tbase = tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(qt * 32);
        const bool fast = ss >= 0 && ss <= 62;
        const int64_t hround = (fast && ss > 0) ? (1LL << (ss - 1)) : 0;
        const int32_t last = tl - 1;
        // The last position of this warp's 32 rows: a key slice past it is masked for every lane.
        const int wlast = (int)grp.pos0 + g * 32 + 31;
        // The first: a key slice at or below it is whole for every lane. The choice between the
        // whole and the masked path is the warp's, so the diagonal slice takes the masked path
        // once instead of both paths diverged.
        const int wfirst = (int)grp.pos0 + g * 32;
        // The table index min(M - score(dot), last); NARROW: the score is the low word of the
        // 64-bit shift (one shift of the high word when ss >= 32, a funnel shift below).
        auto dist = [&](int64_t M, int32_t dot) -> int32_t {
            if constexpr (NARROW) {
                const int64_t t = (int64_t)dot * (int64_t)sm + hround;
                int32_t score;
                if constexpr (SSHI) score = (int32_t)(t >> 32) >> (ss - 32);
                else score = (int32_t)__funnelshift_r((uint32_t)t, (uint32_t)((uint64_t)t >> 32), ss);
                const int32_t dd = (int32_t)M - score;
                return (uint32_t)dd < (uint32_t)last ? dd : last;
            } else {
                return dist_of<false>(M, dot, sm, ss, fast, hround, last);
            }
        };
        int it = 0;
        // Pass 1: the max and min dot over the row's causal keys.
        int32_t maxd = INT32_MIN, mind = INT32_MAX;
        for (int c = 0; c < nch; c++, it++) {
            const int sb = it & 1;
            mbar_wait(&bars->s_full[sb], (it >> 1) & 1, err, 21);
            __syncwarp();
            tc_fence_after();
            uint32_t v[32];
            tmem_ld32(tbase + sb * KC, v);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars->s_empty[sb]);
            const int j0 = c * KC + qt * 32;
            if (j0 > wlast) {
                // every key of this slice is masked for this warp's rows
            } else if (j0 + 31 <= wfirst) {
                // A max/min tree instead of one dependent chain of 32 steps.
                int32_t mx[8], mn[8];
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    mx[q] = max(max((int32_t)v[4 * q], (int32_t)v[4 * q + 1]), max((int32_t)v[4 * q + 2], (int32_t)v[4 * q + 3]));
                    mn[q] = min(min((int32_t)v[4 * q], (int32_t)v[4 * q + 1]), min((int32_t)v[4 * q + 2], (int32_t)v[4 * q + 3]));
                }
#pragma unroll
                for (int q = 0; q < 4; q++) {
                    mx[q] = max(mx[q], mx[q + 4]);
                    mn[q] = min(mn[q], mn[q + 4]);
                }
                maxd = max(maxd, max(max(mx[0], mx[1]), max(mx[2], mx[3])));
                mind = min(mind, min(min(mn[0], mn[1]), min(mn[2], mn[3])));
            } else {
#pragma unroll
                for (int q = 0; q < 32; q++) {
                    if (j0 + q <= rpos) {
                        int32_t dv = (int32_t)v[q];
                        maxd = dv > maxd ? dv : maxd;
                        mind = dv < mind ? dv : mind;
                    }
                }
            }
        }
        sX[(0 * 4 + qt) * GM + row] = maxd;
        sX[(1 * 4 + qt) * GM + row] = mind;
        named_bar(1, ETH);
#pragma unroll
        for (int o = 0; o < 4; o++) {
            int64_t a = sX[(0 * 4 + o) * GM + row], b = sX[(1 * 4 + o) * GM + row];
            maxd = (int32_t)(a > maxd ? a : maxd);
            mind = (int32_t)(b < mind ? b : mind);
        }
        int64_t M = INT64_MIN;
        if (maxd >= mind) {
            int64_t s1 = score_of(maxd, sm, ss, fast, hround), s2 = score_of(mind, sm, ss, fast, hround);
            M = s1 > s2 ? s1 : s2;
        }
        // Pass 2: the row sum of e, and each key's table index into this SM's scratch slot (the
        // thread's 32 keys of a chunk as four 16-byte words, word k of the warp's 32 rows at 512
        // contiguous bytes). The same thread reads them back in pass 3.
        const size_t slot_bytes = (size_t)((n_ctx + KC - 1) / KC) * SCR_CHUNK_BYTES;  // the same for every CTA
        uint4* scr = reinterpret_cast<uint4*>(scratch + (size_t)smid * slot_bytes) + qt * 4 * GM + row;
        mbar_wait(&bars->t_full, 0, err, 26);
        uint64_t sum = 0;
        for (int c = 0; c < nch; c++, it++) {
            const int sb = it & 1;
            mbar_wait(&bars->s_full[sb], (it >> 1) & 1, err, 22);
            __syncwarp();
            tc_fence_after();
            uint32_t v[32];
            tmem_ld32(tbase + sb * KC, v);
            tmem_ld_wait();
            tc_fence_before();
            mbar_arrive(&bars->s_empty[sb]);
            const int j0 = c * KC + qt * 32;
            if (j0 > wlast) continue;  // masked for every lane: nothing stored, nothing read back
            uint32_t dk[16];
#pragma unroll
            for (int q = 0; q < 32; q += 2) {
                const uint32_t d0 = (uint32_t)dist(M, (int32_t)v[q]), d1 = (uint32_t)dist(M, (int32_t)v[q + 1]);
                dk[q >> 1] = d0 | (d1 << 16);
            }
            uint4* w = scr + (size_t)c * (SCR_CHUNK_BYTES / 16);
#pragma unroll
            for (int k = 0; k < 4; k++) __stcg(w + k * GM, make_uint4(dk[4 * k], dk[4 * k + 1], dk[4 * k + 2], dk[4 * k + 3]));
            if (j0 + 31 <= wfirst) {
                // Four partial sums: independent chains for the look-ups and adds.
                uint64_t ps[4] = {0, 0, 0, 0};
#pragma unroll
                for (int q = 0; q < 32; q++) ps[q & 3] += (uint32_t)sT[(dk[q >> 1] >> (16 * (q & 1))) & 0xFFFFu];
                sum += (ps[0] + ps[1]) + (ps[2] + ps[3]);
            } else {
#pragma unroll
                for (int q = 0; q < 32; q++)
                    if (j0 + q <= rpos) sum += (uint32_t)sT[(dk[q >> 1] >> (16 * (q & 1))) & 0xFFFFu];
            }
        }
        // Pass 3's first table indices are on their way while the sums are exchanged.
        auto load_idx = [&](int c, uint4* dst) {
            if (c < nch && c * KC + qt * 32 <= wlast) {
                const uint4* r = scr + (size_t)c * (SCR_CHUNK_BYTES / 16);
#pragma unroll
                for (int k = 0; k < 4; k++) dst[k] = __ldcg(r + k * GM);
            }
        };
        uint4 nxt[4] = {};
        load_idx(0, nxt);
        named_bar(1, ETH);  // everyone has read sX (pass 1) before it is reused
        sX[qt * GM + row] = (int64_t)sum;
        named_bar(1, ETH);
        sum = 0;
#pragma unroll
        for (int o = 0; o < 4; o++) sum += (uint64_t)sX[o * GM + row];
        if (sum == 0) sum = 1;
        // p = floor(e * 2^P / sum) for every e < 2^31 as floor(e * mg / 2^(31 + l)): the numerators
        // e * 2^P have N = 31 + P <= 61 bits, 2^l >= sum and mg = ceil(2^(N + l) / sum) <= 2^(N + 1),
        // so the quotient is exact (Granlund and Montgomery, "Division by invariant integers using
        // multiplication", 1994, Theorem 4.2). With mg = mh 2^32 + ml and u = e mh + (e ml >> 32),
        // p = u >> (l - 1): two 32x32 multiplies per key.
        int l = 64 - __clzll((long long)(sum - 1));
        if (l < 1) l = 1;
        const uint64_t mg = ceil_pow2_div(31 + P + l, sum);
        const uint32_t mh = (uint32_t)(mg >> 32), ml = (uint32_t)mg;
        const int psh = l - 1;
        // Pass 3: the table indices back from the scratch (the next chunk's loads in flight while
        // this one is used), p, its four byte planes into shared memory (128-byte swizzle,
        // K-major), P V.
        const uint32_t rsw = (uint32_t)(row & 7);
        for (int c = 0; c < nch; c++) {
            const int j0 = c * KC + qt * 32;
            uint32_t dk[16];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                dk[4 * k] = nxt[k].x;
                dk[4 * k + 1] = nxt[k].y;
                dk[4 * k + 2] = nxt[k].z;
                dk[4 * k + 3] = nxt[k].w;
            }
            load_idx(c + 1, nxt);
            auto prob = [&](int q) -> uint32_t {
                const uint32_t e = (uint32_t)sT[(dk[q >> 1] >> (16 * (q & 1))) & 0xFFFFu];
                const uint64_t t = (uint64_t)e * ml;
                const uint64_t u = (uint64_t)e * mh + (t >> 32);
                return (uint32_t)(u >> psh);
            };
            uint32_t pv[32];
            if (j0 > wlast) {
#pragma unroll
                for (int q = 0; q < 32; q++) pv[q] = 0u;
            } else if (j0 + 31 <= wfirst) {
#pragma unroll
                for (int q = 0; q < 32; q++) pv[q] = prob(q);
            } else {
#pragma unroll
                for (int q = 0; q < 32; q++) pv[q] = j0 + q <= rpos ? prob(q) : 0u;
            }
            // The four byte planes of each 4-key word: a 4x4 byte transpose with byte permutes.
            uint32_t pw[4][8];  // [plane][4-key word] of this thread's 32 keys
#pragma unroll
            for (int w = 0; w < 8; w++) {
                const uint32_t a = __byte_perm(pv[4 * w], pv[4 * w + 1], 0x5140);
                const uint32_t b2 = __byte_perm(pv[4 * w], pv[4 * w + 1], 0x7362);
                const uint32_t c2 = __byte_perm(pv[4 * w + 2], pv[4 * w + 3], 0x5140);
                const uint32_t d2 = __byte_perm(pv[4 * w + 2], pv[4 * w + 3], 0x7362);
                pw[0][w] = __byte_perm(a, c2, 0x5410);
                pw[1][w] = __byte_perm(a, c2, 0x7632);
                pw[2][w] = __byte_perm(b2, d2, 0x5410);
                pw[3][w] = __byte_perm(b2, d2, 0x7632);
            }
            // The P V of chunk c - 2 (the same buffer) must be done before its planes are overwritten.
            const int pb = c & 1;
            mbar_wait(&bars->p_empty[pb], ((c >> 1) & 1) ^ 1, err, 24);
            __syncwarp();
            uint8_t* prow = sP + pb * P_BYTES + (row >> 3) * 1024 + (row & 7) * 128;
#pragma unroll
            for (int pl = 0; pl < 4; pl++) {
                uint8_t* base = prow + pl * (GM * KC);
#pragma unroll
                for (int cc = 0; cc < 2; cc++) {
                    const uint32_t chunk = (uint32_t)(qt * 2 + cc);  // 16-byte chunk of the 128-byte row
                    *reinterpret_cast<uint4*>(base + ((chunk ^ rsw) << 4)) =
                        make_uint4(pw[pl][4 * cc], pw[pl][4 * cc + 1], pw[pl][4 * cc + 2], pw[pl][4 * cc + 3]);
                }
            }
            fence_proxy_async();
            mbar_arrive(&bars->p_full[pb]);
        }
        // O: acc = sum_k 2^(8k) O_k for this thread's 16 channels, then the output rescale.
        mbar_wait(&bars->o_full, 0, err, 25);
        __syncwarp();
        tc_fence_after();
        const bool row_ok = row < (int)grp.count;
        uint32_t o[4][16];
#pragma unroll
        for (int pl = 0; pl < 4; pl++)
            tmem_ld16(tmem + ((uint32_t)(g * 32) << 16) + 2 * KC + pl * HDIM + qt * 16, o[pl]);
        tmem_ld_wait();
        if (row_ok) {
            // att = clamp(rescale(acc, om, os), -127, 127), |acc| <= 2^30 * 128 (rescale_clamp127): the
            // double estimates of all 16 values first, branch-free, so their latencies overlap; the
            // values too close to a rounding boundary take the exact rule afterwards.
            const double omsc = (double)om * exp2_neg(os);
            int64_t accs[16];
            int32_t ys[16];
            uint32_t slow = os > 95 ? 0xFFFFu : 0u;
#pragma unroll
            for (int q = 0; q < 16; q++) {
                accs[q] = ((((int64_t)(int32_t)o[3][q] * 256 + (int32_t)o[2][q]) * 256 + (int32_t)o[1][q]) * 256) +
                          (int32_t)o[0][q];
                const double z = fma((double)accs[q], omsc, 0.5);
                const double zc = fmin(fmax(z, -1024.0), 1024.0);
                const double fl = floor(zc);
                const double fr = zc - fl;
                ys[q] = min(max((int32_t)fl, -127), 127);
                const bool near = fabs(z) < 1024.0 && !(fr > 9.094947017729282e-13 && fr < 1.0 - 9.094947017729282e-13);
                slow |= (uint32_t)near << q;
            }
            if (slow) {
#pragma unroll
                for (int q = 0; q < 16; q++)
                    if ((slow >> q) & 1) ys[q] = (int32_t)clamp128(rescale128(accs[q], om, (uint32_t)os), -127, 127);
            }
            uint32_t packed[4];
#pragma unroll
            for (int w = 0; w < 4; w++)
                packed[w] = __byte_perm(__byte_perm(ys[4 * w], ys[4 * w + 1], 0x0040),
                                        __byte_perm(ys[4 * w + 2], ys[4 * w + 3], 0x0040), 0x5410);
            *reinterpret_cast<uint4*>(att + (size_t)(grp.first_row + row) * lda + h * HDIM + qt * 16) =
                make_uint4(packed[0], packed[1], packed[2], packed[3]);
        }
        tc_fence_before();
    }
    __syncthreads();
    if (warp == EW + 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem, 512);
    }
}

// ---- decode attention: one warp per (row, head) ----
//
// The rows of a pass that are not in a prefill group (batched decode: one row per stream). Each
// warp reads the row's K [n x 64] and V^T [64 x n] of one head once, which is all the DRAM traffic
// there is: the dots (dp4a) into shared memory with the max and min dot, then e and the sum, then
// p (the exact multiply-shift of the prefill kernel) as four unsigned byte planes in place, then
// P V with u8 x s8 dp4a over 8 channels at a time: each lane takes 16 keys per step, one 16-byte
// load per channel row (a warp reads 512 contiguous bytes of a row), and accumulates its keys'
// part of the 8 channels x 4 planes; a butterfly reduce-scatter leaves lane l with value l, and
// lane 4c gathers the four planes of channel c. The dots pass keeps 2 keys per lane in flight,
// so that 5 blocks fit on an SM. No block-wide synchronisation.
constexpr int DEC_WARPS = 4;

__device__ __forceinline__ int32_t dp4a_us(uint32_t a, uint32_t b, int32_t c) {
    int32_t d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

template <bool NARROW, bool SSHI>
__global__ void __launch_bounds__(32 * DEC_WARPS, 5) k_attention_dec(const RowInfo* rows, const int* rowlist, int nrows,
                                                                   const int8_t* qkv, int ldq, const int8_t* kc,
                                                                   const int8_t* vc, int L, int layer, int H,
                                                                   int n_ctx, int32_t sm, int ss, int32_t om, int os,
                                                                   const int32_t* table, int tlen, int P, int8_t* att,
                                                                   int lda) {
    extern __shared__ __align__(16) uint32_t s_dec[];  // [DEC_WARPS][n_ctx]: dots, then e, then p planes
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int item = blockIdx.x * DEC_WARPS + warp;
    if (item >= nrows * H) return;
    const int h = item % H;
    const int r = rowlist ? rowlist[item / H] : item / H;
    const RowInfo ri = rows[r];
    const int n = (int)ri.pos + 1;
    uint32_t* sb = s_dec + (size_t)warp * n_ctx;
    const size_t head = ((size_t)ri.slot * L + layer) * H + h;
    const int4* K = reinterpret_cast<const int4*>(kc + head * n_ctx * HDIM);
    const int8_t* Vt = vc + head * HDIM * n_ctx;
    int32_t qw[16];
    {
        const int4* qp = reinterpret_cast<const int4*>(qkv + (size_t)r * ldq + h * HDIM);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int4 v = qp[i];
            qw[4 * i] = v.x;
            qw[4 * i + 1] = v.y;
            qw[4 * i + 2] = v.z;
            qw[4 * i + 3] = v.w;
        }
    }
    // Pass 1: the dots (2 keys per lane in flight).
    int32_t maxd = INT32_MIN, mind = INT32_MAX;
    for (int j0 = 0; j0 < n; j0 += 64) {
        int4 kv[2][4];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int j = j0 + 32 * u + lane;
            if (j < n) {
#pragma unroll
                for (int i = 0; i < 4; i++) kv[u][i] = K[(size_t)j * 4 + i];
            }
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int j = j0 + 32 * u + lane;
            if (j < n) {
                int32_t dot = 0;
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    dot = __dp4a(qw[4 * i], kv[u][i].x, dot);
                    dot = __dp4a(qw[4 * i + 1], kv[u][i].y, dot);
                    dot = __dp4a(qw[4 * i + 2], kv[u][i].z, dot);
                    dot = __dp4a(qw[4 * i + 3], kv[u][i].w, dot);
                }
                sb[j] = (uint32_t)dot;
                maxd = max(maxd, dot);
                mind = min(mind, dot);
            }
        }
    }
    for (int o = 16; o > 0; o >>= 1) {
        maxd = max(maxd, __shfl_xor_sync(0xffffffffu, maxd, o));
        mind = min(mind, __shfl_xor_sync(0xffffffffu, mind, o));
    }
    const bool fast = ss >= 0 && ss <= 62;
    const int64_t hround = (fast && ss > 0) ? (1LL << (ss - 1)) : 0;
    const int32_t last = (tlen < TABLE_MAX ? tlen : TABLE_MAX) - 1;
    const int64_t s1 = score_of(maxd, sm, ss, fast, hround), s2 = score_of(mind, sm, ss, fast, hround);
    const int64_t M = s1 > s2 ? s1 : s2;
    auto dist = [&](int32_t dot) -> int32_t {
        if constexpr (NARROW) {
            const int64_t t = (int64_t)dot * (int64_t)sm + hround;
            int32_t score;
            if constexpr (SSHI) score = (int32_t)(t >> 32) >> (ss - 32);
            else score = (int32_t)__funnelshift_r((uint32_t)t, (uint32_t)((uint64_t)t >> 32), ss);
            const int32_t dd = (int32_t)M - score;
            return (uint32_t)dd < (uint32_t)last ? dd : last;
        } else {
            return dist_of<false>(M, dot, sm, ss, fast, hround, last);
        }
    };
    __syncwarp();
    // Pass 2: e in place and the sum.
    uint64_t sum = 0;
    for (int j = lane; j < n; j += 32) {
        const uint32_t e = (uint32_t)__ldg(table + dist((int32_t)sb[j]));
        sb[j] = e;
        sum += e;
    }
    for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
    if (sum == 0) sum = 1;
    int l = 64 - __clzll((long long)(sum - 1));
    if (l < 1) l = 1;
    const uint64_t mg = ceil_pow2_div(31 + P + l, sum);
    const uint32_t mh = (uint32_t)(mg >> 32), ml = (uint32_t)mg;
    const int psh = l - 1;
    __syncwarp();
    // Pass 3: p as four byte planes of each quad of keys, in place (keys past n give 0).
    const int nq = (n + 15) >> 4 << 2;  // whole 16-key groups (n_ctx % 16 == 0), zeros past n
    for (int qd = lane; qd < nq; qd += 32) {
        uint32_t pv[4];
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int j = 4 * qd + k;
            uint32_t p = 0;
            if (j < n) {
                const uint32_t e = sb[j];
                const uint64_t t = (uint64_t)e * ml;
                const uint64_t u = (uint64_t)e * mh + (t >> 32);
                p = (uint32_t)(u >> psh);
            }
            pv[k] = p;
        }
        const uint32_t a = __byte_perm(pv[0], pv[1], 0x5140), b2 = __byte_perm(pv[0], pv[1], 0x7362);
        const uint32_t c2 = __byte_perm(pv[2], pv[3], 0x5140), d2 = __byte_perm(pv[2], pv[3], 0x7362);
        *reinterpret_cast<uint4*>(sb + 4 * qd) = make_uint4(__byte_perm(a, c2, 0x5410), __byte_perm(a, c2, 0x7632),
                                                            __byte_perm(b2, d2, 0x5410), __byte_perm(b2, d2, 0x7632));
    }
    __syncwarp();
    // P V, 8 channels at a time.
    const double omsc = (double)om * exp2_neg(os);
#pragma unroll 1
    for (int c0 = 0; c0 < HDIM; c0 += 8) {
        int32_t acc[32];  // [channel][plane]
#pragma unroll
        for (int i = 0; i < 32; i++) acc[i] = 0;
        // Each lane takes 16 keys (4 quads) per step: one 16-byte load per channel row.
        for (int qg = lane; 4 * qg < nq; qg += 32) {
            uint4 vv[8];
#pragma unroll
            for (int c = 0; c < 8; c++)
                vv[c] = __ldg(reinterpret_cast<const uint4*>(Vt + (size_t)(c0 + c) * n_ctx) + qg);
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint4 pw = *reinterpret_cast<const uint4*>(sb + 16 * qg + 4 * k);
#pragma unroll
                for (int c = 0; c < 8; c++) {
                    const uint32_t v = k == 0 ? vv[c].x : k == 1 ? vv[c].y : k == 2 ? vv[c].z : vv[c].w;
                    acc[4 * c] = dp4a_us(pw.x, v, acc[4 * c]);
                    acc[4 * c + 1] = dp4a_us(pw.y, v, acc[4 * c + 1]);
                    acc[4 * c + 2] = dp4a_us(pw.z, v, acc[4 * c + 2]);
                    acc[4 * c + 3] = dp4a_us(pw.w, v, acc[4 * c + 3]);
                }
            }
        }
        // Butterfly reduce-scatter over the 32 values: after offset o the lane keeps the half of
        // its values picked by its bit o, summed with its partner's; lane l ends with value l.
#pragma unroll
        for (int o = 16, half = 16; o > 0; o >>= 1, half >>= 1) {
            const bool up = (lane & o) != 0;
#pragma unroll
            for (int k = 0; k < half; k++) {
                const int32_t send = up ? acc[k] : acc[k + half];
                const int32_t keep = up ? acc[k + half] : acc[k];
                acc[k] = keep + __shfl_xor_sync(0xffffffffu, send, o);
            }
        }
        // Value l = 4 c + plane: lane 4 c gathers channel c's four planes.
        const int32_t p1 = __shfl_down_sync(0xffffffffu, acc[0], 1);
        const int32_t p2 = __shfl_down_sync(0xffffffffu, acc[0], 2);
        const int32_t p3 = __shfl_down_sync(0xffffffffu, acc[0], 3);
        if ((lane & 3) == 0) {
            // Each plane sum is at most n * 255 * 128 < 2^31 in magnitude.
            const int64_t a = ((((int64_t)p3 * 256 + p2) * 256 + p1) * 256) + acc[0];
            att[(size_t)r * lda + h * HDIM + c0 + (lane >> 2)] = (int8_t)rescale_clamp127(a, om, os, omsc);
        }
    }
}

}  // namespace

cudaError_t configure_attn_tc() {
    const void* fns[3] = {(const void*)k_attention_tc<true, true>, (const void*)k_attention_tc<true, false>,
                          (const void*)k_attention_tc<false, false>};
    for (const void* f : fns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)ASMEM);
        if (e != cudaSuccess) return e;
    }
    const void* dfns[3] = {(const void*)k_attention_dec<true, true>, (const void*)k_attention_dec<true, false>,
                           (const void*)k_attention_dec<false, false>};
    for (const void* f : dfns) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             DEC_WARPS * 4 * MAX_ATTN_CTX);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

bool attention_dec_supported(int hd, int n_ctx, int ldq, int tlen) {
    return hd == HDIM && n_ctx % 16 == 0 && ldq % 16 == 0 && tlen <= TABLE_MAX;
}

void launch_attention_dec(const RowInfo* rows, const int* rowlist, int nrows, const int8_t* qkv, int ldq,
                          const int8_t* kc, const int8_t* vc, int L, int layer, int H, int n_ctx, int32_t sm, int ss,
                          int32_t om, int os, const int32_t* table, int tlen, int P, int8_t* att, int lda,
                          cudaStream_t st) {
    if (nrows <= 0) return;
    const int grid = (nrows * H + DEC_WARPS - 1) / DEC_WARPS;
    const size_t smem = (size_t)DEC_WARPS * n_ctx * 4;
    if (ss >= 32 && ss <= 62)
        k_attention_dec<true, true><<<grid, 32 * DEC_WARPS, smem, st>>>(rows, rowlist, nrows, qkv, ldq, kc, vc, L,
                                                                       layer, H, n_ctx, sm, ss, om, os, table, tlen,
                                                                       P, att, lda);
    else if (ss >= 21 && ss < 32)
        k_attention_dec<true, false><<<grid, 32 * DEC_WARPS, smem, st>>>(rows, rowlist, nrows, qkv, ldq, kc, vc, L,
                                                                        layer, H, n_ctx, sm, ss, om, os, table, tlen,
                                                                        P, att, lda);
    else
        k_attention_dec<false, false><<<grid, 32 * DEC_WARPS, smem, st>>>(rows, rowlist, nrows, qkv, ldq, kc, vc, L,
                                                                         layer, H, n_ctx, sm, ss, om, os, table,
                                                                         tlen, P, att, lda);
}

bool attention_tc_supported(int hd, int n_ctx, int tlen) {
    return hd == HDIM && n_ctx % 16 == 0 && n_ctx <= 8192 && tlen <= TABLE_MAX;
}

// %nsmid: SM ids run from 0 to this bound minus one (not necessarily every id in between).
__global__ void k_sm_id_bound(int* out) {
    uint32_t n;
    asm("mov.u32 %0, %%nsmid;" : "=r"(n));
    *out = (int)n;
}

cudaError_t attn_scratch_slots(int* slots, cudaStream_t st) {
    int* d = nullptr;
    cudaError_t e = cudaMalloc(&d, sizeof(int));
    if (e != cudaSuccess) return e;
    k_sm_id_bound<<<1, 1, 0, st>>>(d);
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaMemcpyAsync(slots, d, sizeof(int), cudaMemcpyDeviceToHost, st);
    if (e == cudaSuccess) e = cudaStreamSynchronize(st);
    cudaError_t f = cudaFree(d);
    return e != cudaSuccess ? e : f;
}

size_t attn_scratch_bytes(int slots, int n_ctx) {
    return (size_t)slots * (size_t)((n_ctx + KC - 1) / KC) * SCR_CHUNK_BYTES;
}

void launch_attention_tc(const void* tmQ, const void* tmK, const void* tmV, const AttnGroup* groups, int n_groups,
                         int L, int layer, int H, int n_ctx, int32_t sm, int ss, int32_t om, int os,
                         const int32_t* table, int tlen, int P, int8_t* att, int lda, uint8_t* scratch, int scr_slots,
                         int* err, cudaStream_t st) {
    if (n_groups <= 0) return;
    dim3 grid(n_groups, H);
    const CUtensorMap& q = *reinterpret_cast<const CUtensorMap*>(tmQ);
    const CUtensorMap& k = *reinterpret_cast<const CUtensorMap*>(tmK);
    const CUtensorMap& v = *reinterpret_cast<const CUtensorMap*>(tmV);
    if (ss >= 32 && ss <= 62)
        k_attention_tc<true, true><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, L, layer, H, n_ctx, sm, ss, om, os,
                                                                 table, tlen, P, att, lda, scratch, scr_slots, err);
    else if (ss >= 21 && ss < 32)
        k_attention_tc<true, false><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, L, layer, H, n_ctx, sm, ss, om, os,
                                                                  table, tlen, P, att, lda, scratch, scr_slots, err);
    else
        k_attention_tc<false, false><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, L, layer, H, n_ctx, sm, ss, om,
                                                                   os, table, tlen, P, att, lda, scratch, scr_slots, err);
}

}  // namespace hs
