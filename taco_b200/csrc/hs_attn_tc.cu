// Prefill attention of the B200 HardShell backend on the tensor cores (tcgen05).
//
// The unit of work is a tile: one (group, head). A group is up to 128 rows of one slot at
// consecutive positions pos0 .. pos0 + count - 1, attending causally to the keys
// 0 .. pos0 + count - 1 of its slot. The kernel is persistent: one CTA per SM takes the tiles
// t = blockIdx.x, blockIdx.x + gridDim.x, ... in the host's order (groups longest first, the
// heads of a group consecutive).
// The integer softmax of crates/hardshell/src/softmax.rs:78 needs the exact row max before any
// weight and the exact row sum before any probability, so a tile runs three passes over its
// 128-key chunks, with S = Q K^T computed twice on the tensor cores (cheap: K = 64):
//   pass 1: S -> the max dot of each row when the score multiplier is >= 0, else the min dot
//           (score() is monotone in the dot, rising or falling with the multiplier's sign, so the
//           max score is the score of that extreme);
//   pass 2: S -> the table index d = min(max - score, len - 1) -> e = attn_exp[d] -> the row sum;
//           each key's d (u16) goes to this CTA's slot of a scratch buffer in global memory;
//   pass 3: d back from the scratch (no third S) -> p = floor(e * 2^P / sum) (an exact
//           multiply-shift), split into four unsigned bytes p = p0 + 2^8 p1 + 2^16 p2 + 2^24 p3,
//           written to shared memory as four u8 A operands; O_k += P_k V (u8 x s8) in TMEM.
// Then acc = sum_k 2^(8k) O_k (exact: each O_k has at most n_ctx terms below 2^15) and
// att = clamp(rescale(acc, out_m, out_s), -127, 127) (crates/hardshell/src/gpt2/reference.rs:252-284).
//
// Tiles overlap. Pass 3 reads no S, so the first two S of the next tile are computed while the
// softmax warps run pass 3; and a tile's output (its epilogue) is read from TMEM after the pass 1
// of the next tile, when its last P V products are done. The softmax warps run, per tile t:
// pass 1 (t), epilogue (t - 1), pass 2 (t), pass 3 (t). The P V of tile t + 1 starts only after
// every softmax thread has written its first P planes, so after its epilogue of tile t.
//
// Operands come in by TMA (no multicast): Q [128 x 64] (Q_STAGES buffers) and K chunks [128 x 64]
// with the 64-byte swizzle, V^T chunks [64 x 128] with the 128-byte swizzle from the transposed
// values cache. Warps 0..15 do the softmax: TMEM lane group warp % 4 (32 rows) and key quarter
// warp / 4 (32 of the 128 keys of a chunk). Warp 16 loads Q and K, warp 17 owns TMEM and issues
// the MMAs (S two items ahead of the softmax, across tiles), warp 18 loads V: a producer waiting
// for a K buffer never holds up a V load that the softmax needs first. The scratch slot of a CTA
// is 32 KB per 128-key chunk of n_ctx (256 KB at n_ctx = 1024); a thread reads back only what it
// wrote itself, and the slots of the resident CTAs stay in L2 between the passes. Every wait is
// bounded.
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
constexpr int W_QK = EW;       // the Q and K producer warp
constexpr int W_MMA = EW + 1;  // the TMEM owner and MMA issuer
constexpr int W_V = EW + 2;    // the V producer warp
constexpr int ATHREADS = ETH + 96;
constexpr int Q_BYTES = GM * HDIM;        // 8 KB
constexpr int K_BYTES = KC * HDIM;        // 8 KB
constexpr int Q_STAGES = 2;               // Q of this tile and of the next
constexpr int K_STAGES = 3;               // K chunks in flight: pass 1 is bound by their latency
constexpr int V_BYTES = HDIM * KC;        // 8 KB
constexpr int P_BYTES = 4 * GM * KC;      // 64 KB (four planes), double-buffered
constexpr int TABLE_MAX = 8192;           // attn_exp entries kept in shared memory
// The row exchange: max and min dots (i32 [8][GM]) and the sums (i64 [4][GM]) apart, so that a
// warp's pass 1 of the next tile never writes where a slower warp still reads this tile's sums.
constexpr int XBYTES = 8 * GM * 4 + 4 * GM * 8;
// The scratch slot of one CTA: per 128-key chunk, key quarter, 16-byte word (4 keys) and row, the
// u32 weights e of 4 keys, so that a warp's 32 rows store and load 512 contiguous bytes.
constexpr size_t SCR_CHUNK_BYTES = 4 * 8 * GM * 16;  // 64 KB per chunk of 128 keys
constexpr size_t ASMEM = (size_t)Q_STAGES * Q_BYTES + (size_t)K_STAGES * K_BYTES + 2 * V_BYTES + 2 * P_BYTES +
                         4 * TABLE_MAX + XBYTES + 512 + 1024;
static_assert(ASMEM <= 232448, "the attention CTA's shared memory exceeds the 227 KB per block");

struct __align__(8) ABars {
    uint64_t q_full[Q_STAGES], q_empty[Q_STAGES];
    uint64_t k_full[K_STAGES], k_empty[K_STAGES];
    uint64_t v_full[2], v_empty[2];
    uint64_t s_full[2], s_empty[2];
    uint64_t p_full[2], p_empty[2];
    uint64_t o_full;
    uint64_t t_full;  // the exp table in shared memory
    uint32_t tmem_base;
};
static_assert(sizeof(ABars) <= 512, "the barriers exceed their shared-memory slot");

__device__ __forceinline__ int tile_chunks(const AttnGroup& g) { return ((int)g.pos0 + (int)g.count + KC - 1) / KC; }


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


// 32 lanes x 32 bits, 8 columns: thread t of the warp gets columns c..c+7 of lane (base + t).
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr));
}

template <bool NARROW, bool SSHI>
__global__ void __launch_bounds__(ATHREADS, 1)
    k_attention_tc(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                   const __grid_constant__ CUtensorMap tmV, const AttnGroup* groups, int T, int L, int layer, int H,
                   int n_ctx, int32_t sm, int ss, int32_t om, int os, const int32_t* table, int tlen, int P,
                   int8_t* att, int lda, uint8_t* scratch, int scr_slots, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    if (blockIdx.x >= (uint32_t)scr_slots) {  // the same for every thread of the CTA: nothing started yet
        if (threadIdx.x == 0) atomicCAS(err, 0, ERR_ATTN_SCRATCH);
        return;
    }
    // Aligned to 1,024 bytes by an offset from the __shared__ array itself (not through an
    // integer cast), so every access below stays a shared-memory access with 32-bit addresses.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    uint8_t* sQ = smem;                         // 2 x 8 KB
    uint8_t* sK = sQ + Q_STAGES * Q_BYTES;      // K_STAGES x 8 KB
    uint8_t* sV = sK + K_STAGES * K_BYTES;      // 2 x 8 KB
    uint8_t* sP = sV + 2 * V_BYTES;             // 2 x 4 planes x 16 KB
    int32_t* sT = reinterpret_cast<int32_t*>(sP + 2 * P_BYTES);
    int32_t* sXm = sT + TABLE_MAX;                                // [8][GM] max, min dots
    int64_t* sXs = reinterpret_cast<int64_t*>(sXm + 8 * GM);      // [4][GM] sums
    ABars* bars = reinterpret_cast<ABars*>(sXs + 4 * GM);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int t0 = (int)blockIdx.x, tstep = (int)gridDim.x;
    const int n_mine = t0 < T ? (T - t0 + tstep - 1) / tstep : 0;  // this CTA's tiles

    if (threadIdx.x == 0) {
        for (int i = 0; i < Q_STAGES; i++) {
            mbar_init(&bars->q_full[i], 1);
            mbar_init(&bars->q_empty[i], 1);
        }
        for (int i = 0; i < K_STAGES; i++) {
            mbar_init(&bars->k_full[i], 1);
            mbar_init(&bars->k_empty[i], 1);
        }
        for (int i = 0; i < 2; i++) {
            mbar_init(&bars->v_full[i], 1);
            mbar_init(&bars->v_empty[i], 1);
            mbar_init(&bars->s_full[i], 1);
            mbar_init(&bars->s_empty[i], ETH);
            mbar_init(&bars->p_full[i], ETH);
            mbar_init(&bars->p_empty[i], 1);
        }
        mbar_init(&bars->o_full, 1);
        mbar_init(&bars->t_full, 1);
        fence_barrier_init();
    }
    if (warp == W_MMA) {
        tmem_alloc(&bars->tmem_base, 512);
        tmem_relinquish();
        tc_fence_before();
    }
    const int tl = tlen < TABLE_MAX ? tlen : TABLE_MAX;
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = bars->tmem_base;

    if (warp == W_QK) {
        // Q of each tile (buffer seq & 1, free once the tile before the last has its S), then the
        // K chunks of its passes 1 and 2, in the order the MMA issuer uses them.
        if (lane == 0) {
            prefetch_tmap(&tmQ);
            prefetch_tmap(&tmK);
            // The exp table (its buffer is padded to 16 bytes), needed from pass 2 on.
            const uint32_t tbytes = (uint32_t)((tl * 4 + 15) & ~15);
            mbar_arrive_expect_tx(&bars->t_full, tbytes);
            bulk_load(sT, table, tbytes, &bars->t_full);
            int ks = 0;
            uint32_t kph = 0;
            bool ok = true;
            for (int seq = 0; seq < n_mine && ok; seq++) {
                const int t = t0 + seq * tstep;
                const AttnGroup grp = groups[t / H];
                const int h = t % H, nch = tile_chunks(grp);
                const size_t head = ((size_t)grp.slot * L + layer) * H + h;
                const int qb = seq % Q_STAGES;
                if (!mbar_wait(&bars->q_empty[qb], ((seq / Q_STAGES) & 1) ^ 1, err, 10)) break;
                mbar_arrive_expect_tx(&bars->q_full[qb], Q_BYTES);
                tma_load_2d(sQ + qb * Q_BYTES, &tmQ, &bars->q_full[qb], h * HDIM, (int)grp.first_row);
                for (int it = 0; it < 2 * nch; it++) {
                    const int c = it < nch ? it : it - nch;
                    if (!mbar_wait(&bars->k_empty[ks], kph ^ 1, err, 11)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&bars->k_full[ks], K_BYTES);
                    tma_load_2d(sK + ks * K_BYTES, &tmK, &bars->k_full[ks], 0, (int)(head * n_ctx) + c * KC);
                    if (++ks == K_STAGES) {
                        ks = 0;
                        kph ^= 1;
                    }
                }
            }
        }
    } else if (warp == W_V) {
        // The V^T chunks of each tile's pass 3.
        if (lane == 0) {
            prefetch_tmap(&tmV);
            int vs = 0;
            uint32_t vph = 0;
            bool ok = true;
            for (int seq = 0; seq < n_mine && ok; seq++) {
                const int t = t0 + seq * tstep;
                const AttnGroup grp = groups[t / H];
                const int h = t % H, nch = tile_chunks(grp);
                const size_t head = ((size_t)grp.slot * L + layer) * H + h;
                for (int c = 0; c < nch; c++) {
                    if (!mbar_wait(&bars->v_empty[vs], vph ^ 1, err, 12)) {
                        ok = false;
                        break;
                    }
                    mbar_arrive_expect_tx(&bars->v_full[vs], V_BYTES);
                    tma_load_2d(sV + vs * V_BYTES, &tmV, &bars->v_full[vs], c * KC, (int)(head * HDIM));
                    if (++vs == 2) {
                        vs = 0;
                        vph ^= 1;
                    }
                }
            }
        }
    } else if (warp == W_MMA) {
        // MMA issuer. The S items (pass 1 then pass 2 of each tile, nch chunks each) run two ahead
        // of the softmax warps' use, across tiles: each S item the softmax warps take frees the
        // S buffer of the item two later. After the S items of tile t's passes (which include the
        // first two of tile t + 1), the P V of tile t as its planes are written, then o_full.
        if (lane == 0) {
            const uint32_t id_s = idesc_i8(GM, KC, true, true);
            const uint32_t id_pv = idesc_i8(GM, HDIM, false, true);
            // The S stream: tile s_seq, item s_j of its 2 s_nch.
            int s_seq = 0, s_j = 0, s_nch = n_mine > 0 ? tile_chunks(groups[t0 / H]) : 0;
            int ks = 0, sit = 0;
            uint32_t kph = 0;
            auto issue_s = [&]() -> bool {
                if (s_seq >= n_mine) return true;  // no S item left
                const int sb = sit & 1, qb = s_seq % Q_STAGES;
                if (s_j == 0 && !mbar_wait(&bars->q_full[qb], (s_seq / Q_STAGES) & 1, err, 13)) return false;
                if (!mbar_wait(&bars->s_empty[sb], ((sit >> 1) & 1) ^ 1, err, 14)) return false;
                if (!mbar_wait(&bars->k_full[ks], kph, err, 15)) return false;
                tc_fence_after();
                const uint32_t qa = smem_u32(sQ + qb * Q_BYTES);
                const uint32_t kb = smem_u32(sK + ks * K_BYTES);
                const uint32_t d = tmem + sb * KC;
#pragma unroll
                for (int k = 0; k < HDIM / 32; k++)
                    mma_i8(d, sdesc_sw64(qa + 32 * k), sdesc_sw64(kb + 32 * k), id_s, k != 0 ? 1u : 0u);
                mma_commit(&bars->k_empty[ks]);
                mma_commit(&bars->s_full[sb]);
                if (++ks == K_STAGES) {
                    ks = 0;
                    kph ^= 1;
                }
                sit++;
                if (++s_j == 2 * s_nch) {
                    mma_commit(&bars->q_empty[qb]);  // Q of this tile is read
                    s_j = 0;
                    if (++s_seq < n_mine) s_nch = tile_chunks(groups[(t0 + s_seq * tstep) / H]);
                }
                return true;
            };
            bool ok = issue_s() && issue_s();
            int vs = 0, pit = 0;
            uint32_t vph = 0;
            for (int seq = 0; seq < n_mine && ok; seq++) {
                const int nch = tile_chunks(groups[(t0 + seq * tstep) / H]);
                for (int j = 0; j < 2 * nch && ok; j++) ok = issue_s();
                for (int c = 0; c < nch && ok; c++, pit++) {
                    const int pb = pit & 1;
                    if (!mbar_wait(&bars->p_full[pb], (pit >> 1) & 1, err, 16)) ok = false;
                    else if (!mbar_wait(&bars->v_full[vs], vph, err, 17)) ok = false;
                    if (!ok) break;
                    tc_fence_after();
                    const uint32_t vb = smem_u32(sV + vs * V_BYTES);
#pragma unroll
                    for (int pl = 0; pl < 4; pl++) {
                        const uint32_t pa = smem_u32(sP + pb * P_BYTES + pl * (GM * KC));
                        const uint32_t o = tmem + 2 * KC + pl * HDIM;
#pragma unroll
                        for (int k = 0; k < KC / 32; k++)
                            mma_i8(o, sdesc_sw128(pa + 32 * k), sdesc_sw128(vb + 32 * k), id_pv,
                                   (c > 0 || k > 0) ? 1u : 0u);
                    }
                    mma_commit(&bars->v_empty[vs]);
                    mma_commit(&bars->p_empty[pb]);
                    if (++vs == 2) {
                        vs = 0;
                        vph ^= 1;
                    }
                }
                if (ok) mma_commit(&bars->o_full);
            }
        }
    } else {
        // Softmax warps: one row per thread, 32 keys of each chunk (quarter qt = warp / 4).
        const int g = warp & 3, qt = warp >> 2;
        const int row = g * 32 + lane;
        const uint32_t tbase = tmem + ((uint32_t)(g * 32) << 16) + (uint32_t)(qt * 32);
        const bool fast = ss >= 0 && ss <= 62;
        const int64_t hround = (fast && ss > 0) ? (1LL << (ss - 1)) : 0;
        const int32_t last = tl - 1;
        const double omsc = (double)om * exp2_neg(os);
        // This thread's words of the CTA's scratch slot (the same size for every CTA).
        const size_t slot_bytes = (size_t)((n_ctx + KC - 1) / KC) * SCR_CHUNK_BYTES;
        uint4* scr = reinterpret_cast<uint4*>(scratch + (size_t)blockIdx.x * slot_bytes) + qt * 8 * GM + row;
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
        // The epilogue of a tile: acc = sum_k 2^(8k) O_k for this thread's 16 channels, then the
        // output rescale. o_full completes once per tile, so the tile's sequence number gives the
        // phase.
        auto epilogue = [&](int eseq, uint32_t first_row, uint32_t count, int eh) {
            mbar_wait(&bars->o_full, (uint32_t)(eseq & 1), err, 25);
            __syncwarp();
            tc_fence_after();
            // Two halves of 8 channels, so that the loads and the estimates of one half fit in the
            // registers that the next tile's live values leave.
            uint32_t packed[4];
#pragma unroll
            for (int half = 0; half < 2; half++) {
                uint32_t o[4][8];
#pragma unroll
                for (int pl = 0; pl < 4; pl++)
                    tmem_ld8(tmem + ((uint32_t)(g * 32) << 16) + 2 * KC + pl * HDIM + qt * 16 + half * 8, o[pl]);
                tmem_ld_wait();
                // att = clamp(rescale(acc, om, os), -127, 127), |acc| <= 2^30 * 128 (rescale_clamp127):
                // the double estimates of all 8 values first, branch-free, so their latencies overlap;
                // the values too close to a rounding boundary take the exact rule afterwards.
                int64_t accs[8];
                int32_t ys[8];
                uint32_t slow = os > 95 ? 0xFFu : 0u;
#pragma unroll
                for (int q = 0; q < 8; q++) {
                    accs[q] = ((((int64_t)(int32_t)o[3][q] * 256 + (int32_t)o[2][q]) * 256 + (int32_t)o[1][q]) * 256) +
                              (int32_t)o[0][q];
                    const double z = fma((double)accs[q], omsc, 0.5);
                    const double zc = fmin(fmax(z, -1024.0), 1024.0);
                    const double fl = floor(zc);
                    const double fr = zc - fl;
                    ys[q] = min(max((int32_t)fl, -127), 127);
                    const bool near =
                        fabs(z) < 1024.0 && !(fr > 9.094947017729282e-13 && fr < 1.0 - 9.094947017729282e-13);
                    slow |= (uint32_t)near << q;
                }
                if (slow) {
#pragma unroll
                    for (int q = 0; q < 8; q++)
                        if ((slow >> q) & 1) ys[q] = (int32_t)clamp128(rescale128(accs[q], om, (uint32_t)os), -127, 127);
                }
#pragma unroll
                for (int w = 0; w < 2; w++)
                    packed[2 * half + w] = __byte_perm(__byte_perm(ys[4 * w], ys[4 * w + 1], 0x0040),
                                                       __byte_perm(ys[4 * w + 2], ys[4 * w + 3], 0x0040), 0x5410);
            }
            tc_fence_before();
            if (row < (int)count)
                *reinterpret_cast<uint4*>(att + (size_t)(first_row + row) * lda + eh * HDIM + qt * 16) =
                    make_uint4(packed[0], packed[1], packed[2], packed[3]);
        };
        int sit = 0, pit = 0;  // S items taken, P chunks written (across tiles)
        uint32_t prev_first = 0, prev_count = 0;
        int prev_h = 0;
        for (int seq = 0; seq <= n_mine; seq++) {
            if (seq == n_mine) {
                if (seq > 0) epilogue(seq - 1, prev_first, prev_count, prev_h);
                break;
            }
            const int t = t0 + seq * tstep;
            const AttnGroup grp = groups[t / H];
            const int h = t % H, nch = tile_chunks(grp);
            const int rpos = (int)grp.pos0 + row;  // rows past the group compute harmless values
            // The last position of this warp's 32 rows: a key slice past it is masked for every lane.
            const int wlast = (int)grp.pos0 + g * 32 + 31;
            // The first: a key slice at or below it is whole for every lane. The choice between the
            // whole and the masked path is the warp's, so the diagonal slice takes the masked path
            // once instead of both paths diverged.
            const int wfirst = (int)grp.pos0 + g * 32;
            // Pass 1: the extreme dot over the row's causal keys. score() is monotone in the dot,
            // rising with it when sm >= 0 and falling when sm < 0 (the same for every row), so the
            // max score is score(max dot) or score(min dot): one of the two is tracked.
            auto pass1 = [&](auto ext, const int32_t ident) -> int32_t {
                int32_t xd = ident;
                for (int c = 0; c < nch; c++, sit++) {
                    const int sb = sit & 1;
                    mbar_wait(&bars->s_full[sb], (sit >> 1) & 1, err, 21);
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
                        // A tree instead of one dependent chain of 32 steps.
                        int32_t t[8];
#pragma unroll
                        for (int q = 0; q < 8; q++)
                            t[q] = ext(ext((int32_t)v[4 * q], (int32_t)v[4 * q + 1]), ext((int32_t)v[4 * q + 2], (int32_t)v[4 * q + 3]));
#pragma unroll
                        for (int q = 0; q < 4; q++) t[q] = ext(t[q], t[q + 4]);
                        xd = ext(xd, ext(ext(t[0], t[1]), ext(t[2], t[3])));
                    } else {
#pragma unroll
                        for (int q = 0; q < 32; q++)
                            if (j0 + q <= rpos) xd = ext(xd, (int32_t)v[q]);
                    }
                }
                sXm[qt * GM + row] = xd;
                named_bar(1, ETH);
#pragma unroll
                for (int o = 0; o < 4; o++) xd = ext(xd, sXm[o * GM + row]);
                return xd;
            };
            const bool rising = sm >= 0;
            const int32_t ident = rising ? INT32_MIN : INT32_MAX;
            const int32_t xd = rising ? pass1([](int32_t a, int32_t b) { return max(a, b); }, INT32_MIN)
                                      : pass1([](int32_t a, int32_t b) { return min(a, b); }, INT32_MAX);
            // |dot| <= 2^20, so the identity means that the row has no key (a row past the group).
            const int64_t M = xd != ident ? score_of(xd, sm, ss, fast, hround) : INT64_MIN;
            // The tile before: its last P V products ran while this pass 1 did.
            if (seq > 0) epilogue(seq - 1, prev_first, prev_count, prev_h);
            prev_first = grp.first_row;
            prev_count = grp.count;
            prev_h = h;
            // Pass 2: the row sum of e, and each key's table index into this CTA's scratch slot (the
            // thread's 32 keys of a chunk as four 16-byte words, word k of the warp's 32 rows at 512
            // contiguous bytes). The same thread reads them back in pass 3.
            if (seq == 0) mbar_wait(&bars->t_full, 0, err, 26);
            uint64_t sum = 0;
            for (int c = 0; c < nch; c++, sit++) {
                const int sb = sit & 1;
                mbar_wait(&bars->s_full[sb], (sit >> 1) & 1, err, 22);
                __syncwarp();
                tc_fence_after();
                uint32_t v[32];
                tmem_ld32(tbase + sb * KC, v);
                tmem_ld_wait();
                tc_fence_before();
                mbar_arrive(&bars->s_empty[sb]);
                const int j0 = c * KC + qt * 32;
                if (j0 > wlast) continue;  // masked for every lane: nothing stored, nothing read back
                uint32_t ev[32];
#pragma unroll
                for (int q = 0; q < 32; q++) ev[q] = (uint32_t)sT[dist(M, (int32_t)v[q])];
                uint4* w = scr + (size_t)c * (SCR_CHUNK_BYTES / 16);
#pragma unroll
                for (int k = 0; k < 8; k++)
                    __stcg(w + k * GM, make_uint4(ev[4 * k], ev[4 * k + 1], ev[4 * k + 2], ev[4 * k + 3]));
                if (j0 + 31 <= wfirst) {
                    // Four partial sums: independent chains for the adds.
                    uint64_t ps[4] = {0, 0, 0, 0};
#pragma unroll
                    for (int q = 0; q < 32; q++) ps[q & 3] += ev[q];
                    sum += (ps[0] + ps[1]) + (ps[2] + ps[3]);
                } else {
#pragma unroll
                    for (int q = 0; q < 32; q++)
                        if (j0 + q <= rpos) sum += ev[q];
                }
            }
            // Pass 3's first weights are on their way while the sums are exchanged. Pass 3 goes by
            // half slices of 16 keys (hc = 2 c + half): the 16 weights of one half come back from
            // the scratch while the half before is used.
            auto load_half = [&](int hc, uint4* dst) {
                const int c = hc >> 1;
                if (c < nch && c * KC + qt * 32 <= wlast) {
                    const uint4* r = scr + (size_t)c * (SCR_CHUNK_BYTES / 16) + (size_t)(hc & 1) * 4 * GM;
#pragma unroll
                    for (int k = 0; k < 4; k++) dst[k] = __ldcg(r + k * GM);
                }
            };
            uint4 nxt[4] = {};
            load_half(0, nxt);
            sXs[qt * GM + row] = (int64_t)sum;
            named_bar(1, ETH);
            sum = 0;
#pragma unroll
            for (int o = 0; o < 4; o++) sum += (uint64_t)sXs[o * GM + row];
            if (sum == 0) sum = 1;
            // p = floor(e * 2^P / sum) for every e < 2^31 as floor(e * mg / 2^(31 + l)): the
            // numerators e * 2^P have N = 31 + P <= 61 bits, 2^l >= sum and mg = ceil(2^(N + l) / sum)
            // <= 2^(N + 1), so the quotient is exact (Granlund and Montgomery, "Division by invariant
            // integers using multiplication", 1994, Theorem 4.2). With mg = mh 2^32 + ml and
            // u = e mh + (e ml >> 32), p = u >> (l - 1): one wide and one high-word multiply per key
            // (the high word alone: 10 % off pass 3 against two wide products).
            int l = 64 - __clzll((long long)(sum - 1));
            if (l < 1) l = 1;
            const uint64_t mg = ceil_pow2_div(31 + P + l, sum);
            const uint32_t mh = (uint32_t)(mg >> 32), ml = (uint32_t)mg;
            const int psh = l - 1;
            auto prob = [&](uint32_t e) -> uint32_t {
                const uint64_t u = (uint64_t)e * mh + __umulhi(e, ml);  // the high word of e ml: 32 bits
                return (uint32_t)(u >> psh);
            };
            // Pass 3: the weights back from the scratch, p, its four byte planes into shared memory
            // (128-byte swizzle, K-major), P V.
            const uint32_t rsw = (uint32_t)(row & 7);
            uint8_t* prow0 = sP + (row >> 3) * 1024 + (row & 7) * 128;
            for (int hc = 0; hc < 2 * nch; hc++) {
                const int c = hc >> 1, half = hc & 1;
                const int j0 = c * KC + qt * 32 + half * 16;  // the first key of this half slice
                uint32_t ev[16];
#pragma unroll
                for (int k = 0; k < 4; k++) {
                    ev[4 * k] = nxt[k].x;
                    ev[4 * k + 1] = nxt[k].y;
                    ev[4 * k + 2] = nxt[k].z;
                    ev[4 * k + 3] = nxt[k].w;
                }
                load_half(hc + 1, nxt);
                uint32_t pv[16];
                if (j0 > wlast) {
#pragma unroll
                    for (int q = 0; q < 16; q++) pv[q] = 0u;
                } else if (j0 + 15 <= wfirst) {
#pragma unroll
                    for (int q = 0; q < 16; q++) pv[q] = prob(ev[q]);
                } else {
#pragma unroll
                    for (int q = 0; q < 16; q++) pv[q] = j0 + q <= rpos ? prob(ev[q]) : 0u;
                }
                // The four byte planes of each 4-key word: a 4x4 byte transpose with byte permutes.
                uint32_t pw[4][4];  // [plane][4-key word] of this half slice
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const uint32_t a = __byte_perm(pv[4 * w], pv[4 * w + 1], 0x5140);
                    const uint32_t b2 = __byte_perm(pv[4 * w], pv[4 * w + 1], 0x7362);
                    const uint32_t c2 = __byte_perm(pv[4 * w + 2], pv[4 * w + 3], 0x5140);
                    const uint32_t d2 = __byte_perm(pv[4 * w + 2], pv[4 * w + 3], 0x7362);
                    pw[0][w] = __byte_perm(a, c2, 0x5410);
                    pw[1][w] = __byte_perm(a, c2, 0x7632);
                    pw[2][w] = __byte_perm(b2, d2, 0x5410);
                    pw[3][w] = __byte_perm(b2, d2, 0x7632);
                }
                // The P V of two chunks before (the same buffer) must be done before its planes are
                // overwritten.
                const int pb = pit & 1;
                if (half == 0) {
                    mbar_wait(&bars->p_empty[pb], ((pit >> 1) & 1) ^ 1, err, 24);
                    __syncwarp();
                }
                const uint32_t chunk = (uint32_t)(qt * 2 + half);  // 16-byte chunk of the 128-byte row
                uint8_t* prow = prow0 + pb * P_BYTES + ((chunk ^ rsw) << 4);
#pragma unroll
                for (int pl = 0; pl < 4; pl++)
                    *reinterpret_cast<uint4*>(prow + pl * (GM * KC)) = make_uint4(pw[pl][0], pw[pl][1], pw[pl][2], pw[pl][3]);
                if (half == 1) {
                    fence_proxy_async();
                    mbar_arrive(&bars->p_full[pb]);
                    pit++;
                }
            }
        }
    }
    __syncthreads();
    if (warp == W_MMA) {
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
constexpr int DEC_SHORT = 64;  // the longest context of the lane-per-channel P V

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
    const int nq = (n + 15) >> 4 << 2;  // whole 16-key groups (n_ctx % 16 == 0), zeros past n
    // The dots, the softmax and p as four byte planes in shared memory (passes 1 to 3).
    auto planes = [&]() {
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
        for (int qd = lane; qd < nq; qd += 32) {
            uint32_t pv[4];
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const int j = 4 * qd + k;
                uint32_t p = 0;
                if (j < n) {
                    const uint32_t e = sb[j];
                    const uint64_t u = (uint64_t)e * mh + __umulhi(e, ml);
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
    };
    const double omsc = (double)om * exp2_neg(os);
    // A short context (n <= DEC_SHORT): lane l takes channels 2l and 2l + 1 in P V, and their V^T
    // rows (at most 4 x 16 bytes each) are loaded first, so that their latency overlaps the K
    // loads and the softmax instead of following it. Bytes past n multiply p = 0.
    if (n <= DEC_SHORT) {
        uint4 vsh[2][4];
        const int nv = (n + 15) >> 4;
#pragma unroll
        for (int ch = 0; ch < 2; ch++) {
            const uint4* vr = reinterpret_cast<const uint4*>(Vt + (size_t)(2 * lane + ch) * n_ctx);
#pragma unroll
            for (int i = 0; i < 4; i++) vsh[ch][i] = i < nv ? __ldg(vr + i) : make_uint4(0u, 0u, 0u, 0u);
        }
        planes();
        // P V of channels 2 lane and 2 lane + 1: the p words of each quad of keys are the same for
        // every lane (broadcast reads), so no reduction across lanes follows.
        int32_t a[2][4] = {};
#pragma unroll
        for (int qd = 0; qd < DEC_SHORT / 4; qd++) {
            if (qd < nq) {
                const uint4 pw = *reinterpret_cast<const uint4*>(sb + 4 * qd);
#pragma unroll
                for (int ch = 0; ch < 2; ch++) {
                    const uint4 vq = vsh[ch][qd >> 2];
                    const uint32_t v = (qd & 3) == 0 ? vq.x : (qd & 3) == 1 ? vq.y : (qd & 3) == 2 ? vq.z : vq.w;
                    a[ch][0] = dp4a_us(pw.x, v, a[ch][0]);
                    a[ch][1] = dp4a_us(pw.y, v, a[ch][1]);
                    a[ch][2] = dp4a_us(pw.z, v, a[ch][2]);
                    a[ch][3] = dp4a_us(pw.w, v, a[ch][3]);
                }
            }
        }
#pragma unroll
        for (int ch = 0; ch < 2; ch++) {
            // Each plane sum is at most n * 255 * 128 < 2^31 in magnitude.
            const int64_t acc = ((((int64_t)a[ch][3] * 256 + a[ch][2]) * 256 + a[ch][1]) * 256) + a[ch][0];
            att[(size_t)r * lda + h * HDIM + 2 * lane + ch] = (int8_t)rescale_clamp127(acc, om, os, omsc);
        }
        return;
    }
    planes();
    // P V, 8 channels at a time.
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

size_t attn_scratch_bytes(int slots, int n_ctx) {
    return (size_t)slots * (size_t)((n_ctx + KC - 1) / KC) * SCR_CHUNK_BYTES;
}

void launch_attention_tc(const void* tmQ, const void* tmK, const void* tmV, const AttnGroup* groups, int n_groups,
                         int L, int layer, int H, int n_ctx, int32_t sm, int ss, int32_t om, int os,
                         const int32_t* table, int tlen, int P, int8_t* att, int lda, uint8_t* scratch, int scr_slots,
                         int* err, cudaStream_t st) {
    if (n_groups <= 0 || scr_slots <= 0) return;
    // One persistent CTA per SM (a CTA takes more than half of an SM's shared memory), at most one
    // per tile and per scratch slot.
    const int T = n_groups * H;
    const int grid = T < scr_slots ? T : scr_slots;
    const CUtensorMap& q = *reinterpret_cast<const CUtensorMap*>(tmQ);
    const CUtensorMap& k = *reinterpret_cast<const CUtensorMap*>(tmK);
    const CUtensorMap& v = *reinterpret_cast<const CUtensorMap*>(tmV);
    if (ss >= 32 && ss <= 62)
        k_attention_tc<true, true><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, T, L, layer, H, n_ctx, sm, ss, om,
                                                                 os, table, tlen, P, att, lda, scratch, scr_slots, err);
    else if (ss >= 21 && ss < 32)
        k_attention_tc<true, false><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, T, L, layer, H, n_ctx, sm, ss, om,
                                                                  os, table, tlen, P, att, lda, scratch, scr_slots, err);
    else
        k_attention_tc<false, false><<<grid, ATHREADS, ASMEM, st>>>(q, k, v, groups, T, L, layer, H, n_ctx, sm, ss, om,
                                                                   os, table, tlen, P, att, lda, scratch, scr_slots,
                                                                   err);
}

}  // namespace hs
