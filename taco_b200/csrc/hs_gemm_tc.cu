// The int8 GEMM of the B200 HardShell backend on the 5th-generation tensor cores.
//
// out = epilogue(A . W^T): A is [rows, Kp] int8 (activations), W is [Np, Kp] int8 (weights),
// both K-major, loaded by TMA with the 128-byte swizzle (no multicast). tcgen05.mma kind::i8
// accumulates exact s32 sums in TMEM; the epilogue warps read TMEM and apply the fixed-point
// requantisation of HardShell (crates/hardshell/src/gpt2/ops.rs:107-169 linear, :213 logits)
// before any value leaves the SM.
//
// Persistent kernel, one CTA per SM, 10 warps:
//   warp 0      TMA producer (one thread): A and B tiles into a ring of 3 or 4 stages;
//   warp 1      TMEM owner and MMA issuer (one thread);
//   warps 2..9  epilogue: TMEM lane group (warp % 4) and column half ((warp - 2) / 4), so each
//               thread owns 128 of the 256 accumulator columns of one row.
// The accumulator is double-buffered in TMEM (2 x 256 columns), so the epilogue of one tile runs
// while the MMAs of the next tile fill the other buffer. The per-column multiplier and the bias
// folded with the rounding constant (c = b * m + 2^(s-1)) are staged in shared memory once per
// tile, so an output costs one 32x32->64 multiply-add and one shift. Every wait is bounded.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "hs_common.cuh"
#include "hs_kernels.cuh"

namespace hs {

namespace {

constexpr int BM = TILE_M;   // 128 rows (TMEM lanes)
constexpr int BN = TILE_N;   // 256 columns (one MMA instruction N)
constexpr int BK = TILE_K;   // 128 bytes of K per stage (one swizzle atom row)
constexpr int UMMA_K = 32;   // K of one kind::i8 instruction
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int GELU_SMEM = 65536;

constexpr int VT_STRIDE = 36;                  // bytes per row of a warp's 32 x 32 transpose tile
constexpr int VT_TILE = 32 * VT_STRIDE;

// The epilogue of EPI_DELTA, EPI_GELU and EPI_LOGITS stores through TMA, so the stores leave as
// whole row segments instead of 32 scattered 16-byte pieces per instruction. DELTA and LOGITS:
// each epilogue warp stages blocks of 32 rows x 128 bytes (the 128-byte swizzle) in two 4 KB
// buffers, one TMA store per block; they run with 3 stages to make room. GELU, whose 64 KB table
// fills shared memory: one buffer of 32 rows x 32 bytes (the 32-byte swizzle).
//
// Epilogue warps: 8 (two per TMEM lane group), or 12 for QKV (three per lane group),
// whose epilogue bounds its K = 768 GEMM: 14 warps still leave 128 registers per thread (at
// most 4 warps per SM sub-partition), and a warp's share of a tile drops from 4 to 3 or 2 of the
// 8 chunks of 32 columns, in contiguous ranges.
template <int MODE>
struct Cfg {
    static constexpr int EPI_WARPS = MODE == EPI_QKV ? 12 : 8;
    static constexpr int EPI_THREADS = 32 * EPI_WARPS;
    static constexpr int THREADS = 64 + EPI_THREADS;
    static constexpr int STAGES = (MODE == EPI_GELU || MODE == EPI_DELTA || MODE == EPI_LOGITS || MODE == EPI_QKV) ? 3 : 4;
    static constexpr int EXTRA = MODE == EPI_GELU ? GELU_SMEM : (MODE == EPI_QKV ? EPI_WARPS * VT_TILE : 0);
    static constexpr int STORE_WARP =
        (MODE == EPI_DELTA || MODE == EPI_LOGITS) ? 8192 : (MODE == EPI_GELU ? 1024 : (MODE == EPI_QKV ? 2048 : 0));
    static constexpr int WSUM = (MODE == EPI_DELTA || MODE == EPI_LOGITS) ? 2 * BN * 8 : 0;  // s_w (WIDE)
    static constexpr size_t SMEM =
        (size_t)STAGES * STAGE_BYTES + EXTRA + EPI_WARPS * STORE_WARP + 2 * BN * 12 + WSUM + 256 + 1024;
};

struct __align__(8) Bars {
    uint64_t full[4];
    uint64_t empty[4];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
};

__device__ __forceinline__ int64_t rescale_fast(uint32_t acc, int32_t m, int64_t c, int s, bool fast) {
    // fast (0 <= s <= 62): floor((acc * m + b * m + 2^(s-1)) / 2^s) with c = b * m + 2^(s-1);
    // |acc * m| <= 2^61 and |c| < 2^62 + 2^61, so the sum fits in an i64 and the shift is the floor.
    // Otherwise c holds b and the general rule runs (int.rs:63).
    if (fast) return ((int64_t)(int32_t)acc * (int64_t)m + c) >> s;
    return rescale64((int64_t)(int32_t)acc + c, m, (uint32_t)s);
}

// S32: the host has bounded every output of this linear below 2^30 in magnitude (and the shift is
// in 0..=62), so the rescaled value is the low word of the 64-bit shift and the clamps are 32-bit.
template <bool S32>
__device__ __forceinline__ auto rescale_e(uint32_t acc, int32_t m, int64_t c, int s, bool fast) {
    if constexpr (S32) return (int32_t)(((int64_t)(int32_t)acc * (int64_t)m + c) >> s);
    else return rescale_fast(acc, m, c, s, fast);
}
template <class T>
__device__ __forceinline__ T clamp_e(T y, int64_t lo, int64_t hi) {
    if constexpr (sizeof(T) == 4) return min(max(y, (T)lo), (T)hi);
    else return clamp64(y, lo, hi);
}

// The 32 rescaled values of one chunk on the S32 path: one 32x32->64 multiply-add and one shift
// each (SHI: s >= 32, so the result is the high word shifted; else a funnel shift), with the
// column parameters read as 16-byte vectors.
template <bool SHI>
__device__ __forceinline__ void rescale_chunk32(const uint32_t (&v)[32], const int32_t* pm, const int64_t* pc, int s,
                                                int32_t (&y)[32]) {
#pragma unroll
    for (int q = 0; q < 32; q += 4) {
        const int4 m4 = *reinterpret_cast<const int4*>(pm + q);
        const longlong2 c01 = *reinterpret_cast<const longlong2*>(pc + q);
        const longlong2 c23 = *reinterpret_cast<const longlong2*>(pc + q + 2);
        const int32_t mm[4] = {m4.x, m4.y, m4.z, m4.w};
        const int64_t cc[4] = {c01.x, c01.y, c23.x, c23.y};
#pragma unroll
        for (int k = 0; k < 4; k++) {
            const int64_t t = (int64_t)(int32_t)v[q + k] * (int64_t)mm[k] + cc[k];
            if constexpr (SHI) y[q + k] = (int32_t)(t >> 32) >> (s - 32);
            else y[q + k] = (int32_t)__funnelshift_r((uint32_t)t, (uint32_t)((uint64_t)t >> 32), s);
        }
    }
}

// Four values already in [-128, 127] as the bytes of one word (byte permutes).
__device__ __forceinline__ uint32_t pack4_i8(int32_t a, int32_t b, int32_t c, int32_t d) {
    return __byte_perm(__byte_perm(a, b, 0x0040), __byte_perm(c, d, 0x0040), 0x5410);
}

// EPI_QKV: one value at column n of a row of (slot, pos): q to out8, k and v to the caches (v
// to the staging rows instead when `stage`).
__device__ __forceinline__ void qkv_store(const EpiArgs& e, int row, const RowInfo& ri, int n, int8_t o, bool stage) {
    if (n < e.d) {
        e.out8[(size_t)row * e.ldo + n] = o;
        return;
    }
    if (stage && n >= 2 * e.d) {
        e.vstage[(size_t)row * e.ldv + (n - 2 * e.d)] = o;
        return;
    }
    const int j = n < 2 * e.d ? n - e.d : n - 2 * e.d;
    const int h = j / e.hd, c = j - h * e.hd;
    const size_t head = ((size_t)ri.slot * e.L + e.layer) * e.H + h;
    if (n < 2 * e.d) e.kc[(head * e.n_ctx + ri.pos) * e.hd + c] = o;
    else e.vc[(head * e.hd + c) * e.n_ctx + ri.pos] = o;
}

// WIDE (version 2 models): the activations are i16, as two i8 planes (tmA: hi, tmA2: lo). Tiles
// are 128 x 128; each stage holds both A planes and a 128-row B tile (the same 48 KB), the MMA warp
// accumulates hi and lo into two TMEM accumulators of 128 columns, and the epilogue recombines
// v = 256 acc_hi + acc_lo + 128 sum_k W[n][k] exactly in i64 (hardshell.cu:798-830 wide_dot).
// NN: tiles of 64 columns (passes of few rows, so that the tiles fill the SMs); else 256 (128 for
// WIDE).
template <int MODE, bool S32, bool WIDE, bool NN = false>
__global__ void __launch_bounds__(Cfg<MODE>::THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmA2,
              const __grid_constant__ CUtensorMap tmB, const __grid_constant__ CUtensorMap tmC,
              const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV, int MT, int NT,
              int KB, EpiArgs e, int* err) {
    constexpr int STAGES = Cfg<MODE>::STAGES;
    constexpr int EPI_WARPS = Cfg<MODE>::EPI_WARPS;
    constexpr int EPI_THREADS = Cfg<MODE>::EPI_THREADS;
    constexpr int THREADS = Cfg<MODE>::THREADS;
    constexpr int NPART = EPI_WARPS / 4;  // epilogue warps per TMEM lane group
    constexpr int TN = WIDE ? 128 : (NN ? 64 : BN);  // columns of one tile
    static_assert(!(WIDE && NN), "the version 2 tiles are 128 columns");
    static_assert(!WIDE || EPI_WARPS == 8, "the version 2 epilogues take 8 warps");
    static_assert(MODE != EPI_LOGITS || EPI_WARPS == 8, "the logits epilogue takes 8 warps");
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    // Aligned to 1,024 bytes by an offset from the __shared__ array itself (not through an
    // integer cast), so every access below stays a shared-memory access with 32-bit addresses.
    uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
    int8_t* s_gelu = reinterpret_cast<int8_t*>(smem + (size_t)STAGES * STAGE_BYTES);
    uint8_t* s_store = smem + (size_t)STAGES * STAGE_BYTES + Cfg<MODE>::EXTRA;  // [EPI_WARPS][STORE_WARP]
    int64_t* s_c = reinterpret_cast<int64_t*>(s_store + EPI_WARPS * Cfg<MODE>::STORE_WARP);  // [2][BN]
    int32_t* s_m = reinterpret_cast<int32_t*>(s_c + 2 * BN);                                 // [2][BN]
    int64_t* s_w = reinterpret_cast<int64_t*>(s_m + 2 * BN);                                 // [2][BN] (WIDE)
    Bars* bars = reinterpret_cast<Bars*>(s_w + (WIDE ? 2 * BN : 0));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        if (WIDE) prefetch_tmap(&tmA2);
        prefetch_tmap(&tmB);
        if (MODE == EPI_QKV && e.kv_tma) {
            prefetch_tmap(&tmC);
            prefetch_tmap(&tmK);
            prefetch_tmap(&tmV);
        }
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], EPI_THREADS);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
    }
    if (MODE == EPI_GELU) {
        // The GELU table (256 or 65536 i8 entries) in shared memory for the epilogue look-ups.
        const int n = 2 * e.gelu_off;
        for (int i = threadIdx.x * 16; i < n; i += THREADS * 16)
            *reinterpret_cast<int4*>(s_gelu + i) = *reinterpret_cast<const int4*>(e.gelu + i);
    }
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = bars->tmem_base;
    const int tiles = MT * NT;

    if (warp == 0) {
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
                int mt = t % MT, nt = t / MT;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(&bars->empty[stage], phase ^ 1, err, 1)) {
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + (size_t)stage * STAGE_BYTES;
                    mbar_arrive_expect_tx(&bars->full[stage], WIDE ? STAGE_BYTES : A_BYTES + TN * BK);
                    tma_load_2d(sa, &tmA, &bars->full[stage], kb * BK, e.a_row0 + mt * BM);
                    if (WIDE) {
                        // [A hi | A lo | B (128 rows)]: 16 + 16 + 16 KB.
                        tma_load_2d(sa + A_BYTES, &tmA2, &bars->full[stage], kb * BK, e.a_row0 + mt * BM);
                        tma_load_2d(sa + 2 * A_BYTES, &tmB, &bars->full[stage], kb * BK, nt * TN);
                    } else {
                        tma_load_2d(sa + A_BYTES, &tmB, &bars->full[stage], kb * BK, nt * TN);
                    }
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(BM, TN, true, true);
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            int i = 0;
            for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, i++) {
                int acc = i & 1;
                uint32_t aphase = (i >> 1) & 1;
                if (!mbar_wait(&bars->tempty[acc], aphase ^ 1, err, 2)) break;
                tc_fence_after();
                uint32_t d = tmem_base + acc * BN;
                for (int kb = 0; kb < KB; kb++) {
                    if (!mbar_wait(&bars->full[stage], phase, err, 3)) {
                        ok = false;
                        break;
                    }
                    tc_fence_after();
                    uint32_t sa = smem_u32(smem + (size_t)stage * STAGE_BYTES);
                    if (WIDE) {
                        // hi plane into columns [0, 128), lo plane into [128, 256) of this buffer.
                        const uint32_t sl = sa + A_BYTES, sb = sa + 2 * A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / UMMA_K; k++) {
                            mma_i8(d, sdesc_sw128(sa + k * UMMA_K), sdesc_sw128(sb + k * UMMA_K), idesc,
                                   (kb | k) != 0 ? 1u : 0u);
                            mma_i8(d + TN, sdesc_sw128(sl + k * UMMA_K), sdesc_sw128(sb + k * UMMA_K), idesc,
                                   (kb | k) != 0 ? 1u : 0u);
                        }
                    } else {
                        uint32_t sb = sa + A_BYTES;
#pragma unroll
                        for (int k = 0; k < BK / UMMA_K; k++) {
                            mma_i8(d, sdesc_sw128(sa + k * UMMA_K), sdesc_sw128(sb + k * UMMA_K), idesc,
                                   (kb | k) != 0 ? 1u : 0u);
                        }
                    }
                    mma_commit(&bars->empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
                if (ok) mma_commit(&bars->tfull[acc]);
            }
        }
    } else {
        const int et = threadIdx.x - 64;        // 0 .. EPI_THREADS - 1
        const int g = warp & 3;                 // TMEM lane group this warp may read
        const int part = (warp - 2) >> 2;       // 0 .. NPART - 1 within the lane group
        const int half = part;                  // (the 8-warp epilogues: which 128 columns)
        const int row_in_tile = g * 32 + lane;
        const int s = e.s;
        const bool fast = s >= 0 && s <= 62;
        const int64_t hround = (fast && s > 0) ? (1LL << (s - 1)) : 0;
        // One 32-row x 32-byte piece (this lane's row: lo, hi) to the output through TMA at
        // element column x and row y. Warp-collective.
        uint8_t* my_store = s_store + (warp - 2) * Cfg<MODE>::STORE_WARP;
        auto store_piece = [&](uint4 lo, uint4 hi, int x, int y) {
            if (lane == 0) bulk_wait_read();
            __syncwarp();
            const uint32_t sw = (uint32_t)((lane >> 2) & 1);
            *reinterpret_cast<uint4*>(my_store + lane * 32 + (sw << 4)) = lo;
            *reinterpret_cast<uint4*>(my_store + lane * 32 + ((sw ^ 1) << 4)) = hi;
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmC, my_store, x, y);
                bulk_commit();
            }
        };
        // EPI_QKV: one 32-row x 32-byte piece through the TMA store map `map` (the 32-byte swizzle),
        // alternating between two 1 KB buffers. Warp-collective.
        uint32_t qpieces = 0;
        auto store_piece2 = [&](const CUtensorMap* map, const uint32_t (&pk)[8], int x, int y) {
            uint8_t* buf = my_store + (qpieces & 1) * 1024;
            if (lane == 0) bulk_wait_read1();  // the store that last used this buffer has read it
            __syncwarp();
            const uint32_t sw = (uint32_t)((lane >> 2) & 1);
            *reinterpret_cast<uint4*>(buf + lane * 32 + (sw << 4)) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
            *reinterpret_cast<uint4*>(buf + lane * 32 + ((sw ^ 1) << 4)) = make_uint4(pk[4], pk[5], pk[6], pk[7]);
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(map, buf, x, y);
                bulk_commit();
            }
            qpieces++;
        };
        // One 32-row x 128-byte block (this lane's row: 8 x 16 bytes) through TMA at element column
        // x and row y (the 128-byte swizzle), alternating between two buffers. Warp-collective.
        uint32_t blocks = 0;
        auto store_block = [&](const uint4 (&b)[8], int x, int y) {
            uint8_t* buf = my_store + (blocks & 1) * 4096;
            if (lane == 0) bulk_wait_read1();  // the store that last used this buffer has read it
            __syncwarp();
#pragma unroll
            for (int j = 0; j < 8; j++) *reinterpret_cast<uint4*>(buf + lane * 128 + ((j ^ (lane & 7)) << 4)) = b[j];
            fence_async_smem();
            __syncwarp();
            if (lane == 0) {
                tma_store_2d(&tmC, buf, x, y);
                bulk_commit();
            }
            blocks++;
        };
        // The column parameters of a tile, staged in shared memory (double-buffered by the
        // accumulator parity). Each thread's loads for the next tile are issued before the
        // current tile's work and written to its buffer at the top of the next iteration, so the
        // global load latency is not paid between tiles. WIDE: the raw bias (the epilogue
        // rescales in 128 bits) and the weight row sums.
        int32_t pf_m = 0, pf_b = 0;
        int64_t pf_w = 0;
        auto fetch_params = [&](int t) {
            const int n = (t / MT) * TN + et;
            pf_m = 0;
            pf_b = 0;
            pf_w = 0;
            if (et < TN && t < tiles && n < e.N) {
                pf_m = e.m[n];
                if (MODE != EPI_LOGITS && MODE != EPI_RAW) pf_b = e.b[n];
                if (WIDE) pf_w = e.wsum[n];
            }
        };
        fetch_params(blockIdx.x);
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, i++) {
            const int mt = t % MT, nt = t / MT;
            const int acc = i & 1;
            const uint32_t aphase = (i >> 1) & 1;
            const int col0 = nt * TN;
            // Buffer `acc` was last read for tile i - 2, which every epilogue warp finished before
            // the barrier of tile i - 1.
            if (et < TN) {
                const int64_t b = pf_b;
                s_m[acc * BN + et] = pf_m;
                s_c[acc * BN + et] = (fast && !WIDE) ? b * (int64_t)pf_m + hround : b;
                if (WIDE) s_w[acc * BN + et] = pf_w;
            }
            named_bar(1, EPI_THREADS);
            fetch_params(t + gridDim.x);
            // On a timeout the error word is set and every later wait returns at once; the warps keep
            // taking part in the named barriers, so no thread can wait on a barrier forever.
            mbar_wait(&bars->tfull[acc], aphase, err, 4);
            __syncwarp();
            tc_fence_after();
            const int row = mt * BM + row_in_tile;
            const bool row_ok = row < e.R;
            // EPI_QKV: are this warp's 32 rows 32 consecutive positions of one slot, starting at a
            // multiple of 16 (the transposed v store)? Warp-uniform.
            bool vt_ok = false, vt_stage = false;
            uint32_t vt_slot = 0, vt_pos0 = 0;
            if (MODE == EPI_QKV) {
                const int r0 = mt * BM + g * 32;
                vt_ok = vt_run_warp(e.rows, r0, e.R, e.n_ctx, lane);
                if (vt_ok) {
                    const RowInfo a0 = e.rows[r0];
                    vt_slot = a0.slot;
                    vt_pos0 = a0.pos;
                }
                vt_stage = !vt_ok && e.vstage != nullptr;
            }
            const uint32_t taddr = tmem_base + ((uint32_t)(g * 32) << 16) + (uint32_t)(acc * BN);
            const int32_t* pm = s_m + acc * BN;
            const int64_t* pc = s_c + acc * BN;
            if constexpr (WIDE) {
                // This thread: row `row`, columns half * 64 .. + 63 of the 128-column tile; hi at
                // TMEM columns [0, 128), lo at [128, 256).
                const int64_t* pw = s_w + acc * BN;
                auto value = [&](uint32_t hi, uint32_t lo, int n) -> int64_t {
                    return 256 * (int64_t)(int32_t)hi + (int64_t)(int32_t)lo + 128 * pw[n];
                };
                if constexpr (MODE == EPI_LOGITS) {
                    // One logits tile of LOGIT_TILE_WIDE = 64 columns per thread: the running max per
                    // 16-column chunk and the packed distance fix-up of the 8-bit path.
                    const uint32_t lastv = (uint32_t)e.last;
                    const uint32_t last2 = lastv | (lastv << 16);
                    uint32_t pk[32];
                    int64_t mc[4];
                    int64_t run = -SCORE_LIMIT;
#pragma unroll
                    for (int ch = 0; ch < 4; ch++) {
                        const int c0 = half * 64 + ch * 16;
                        uint32_t vh[16], vl[16];
                        __syncwarp();
                        tmem_ld16(taddr + c0, vh);
                        tmem_ld16(taddr + TN + c0, vl);
                        tmem_ld_wait();
                        int64_t l[16];
#pragma unroll
                        for (int q = 0; q < 16; q++) {
                            l[q] = col0 + c0 + q < e.N
                                       ? (int64_t)clamp128(rescale128(value(vh[q], vl[q], c0 + q), pm[c0 + q], (uint32_t)s),
                                                           -SCORE_LIMIT, SCORE_LIMIT)
                                       : -SCORE_LIMIT;
                            run = l[q] > run ? l[q] : run;
                        }
                        mc[ch] = run;
#pragma unroll
                        for (int q = 0; q < 16; q += 2) {
                            const int64_t d0 = run - l[q], d1 = run - l[q + 1];
                            const uint32_t a0 = d0 < (int64_t)lastv ? (uint32_t)d0 : lastv;
                            const uint32_t a1 = d1 < (int64_t)lastv ? (uint32_t)d1 : lastv;
                            pk[ch * 8 + (q >> 1)] = a0 | (a1 << 16);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&bars->tempty[acc]);
                    if (col0 + half * 64 < e.N) {
#pragma unroll
                        for (int ch = 0; ch < 4; ch++) {
                            const int64_t sh = run - mc[ch];
                            const uint32_t a = sh < (int64_t)lastv ? (uint32_t)sh : lastv;
                            const uint32_t a2 = a | (a << 16);
#pragma unroll
                            for (int w = 0; w < 8; w++)
                                pk[ch * 8 + w] = __vminu2(__vadd2(pk[ch * 8 + w], a2), last2);
                        }
                        // 64 columns of u16 = one 128-byte block; columns past N are clipped.
                        uint4 blk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) blk[j] = make_uint4(pk[4 * j], pk[4 * j + 1], pk[4 * j + 2], pk[4 * j + 3]);
                        store_block(blk, col0 + half * 64, mt * BM + g * 32);
                        const int tile = nt * 2 + half;
                        if (row_ok && tile < e.ldt) e.tmax[(size_t)row * e.ldt + tile] = run;
                    }
                    continue;
                } else if constexpr (MODE == EPI_DELTA) {
#pragma unroll 1
                    for (int c0 = half * 64; c0 < half * 64 + 64; c0 += 32) {
                        uint32_t vh[32], vl[32];
                        __syncwarp();
                        tmem_ld32(taddr + c0, vh);
                        tmem_ld32(taddr + TN + c0, vl);
                        tmem_ld_wait();
                        const int colb = col0 + c0;
                        if (colb >= e.N) continue;
                        int32_t o[32];
#pragma unroll
                        for (int q = 0; q < 32; q++)
                            o[q] = (int32_t)clamp128(rescale128(value(vh[q], vl[q], c0 + q) + pc[c0 + q], pm[c0 + q],
                                                                (uint32_t)s),
                                                     INT32_MIN, INT32_MAX);
                        uint4 blk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) blk[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                        store_block(blk, colb, mt * BM + g * 32);
                    }
                    tc_fence_before();
                    mbar_arrive(&bars->tempty[acc]);
                    continue;
                }
            }
            if (MODE == EPI_LOGITS) {
                // One TMEM pass over this thread's 128 columns (one logits tile). Per 16-column chunk:
                // the running max M_c after the chunk and the distances min(M_c - l, last) as packed
                // u16 pairs in registers. Then every chunk moves to the tile max M with saturating
                // packed adds: min(d' + min(M - M_c, last), last) = min(M - l, last), because d' and
                // the shift are each clamped at last only when the true value is at least last.
                const uint32_t lastv = (uint32_t)e.last;
                const uint32_t last2 = lastv | (lastv << 16);
                uint32_t pk[64];
                const int tile = nt * 2 + half;
                if (S32 && col0 + BN <= e.N) {
                    // Every logit is below 2^30 in magnitude (the host's bound), so the clamp at
                    // 2^40 is the identity and the max and the distances fit in 32 bits.
                    int32_t mc32[8];
                    int32_t run32 = INT32_MIN;
#pragma unroll
                    for (int ch = 0; ch < 8; ch++) {
                        const int c0 = half * 128 + ch * 16;
                        uint32_t v[16];
                        __syncwarp();
                        tmem_ld16(taddr + c0, v);
                        tmem_ld_wait();
                        int32_t l[16];
#pragma unroll
                        for (int q = 0; q < 16; q++) {
                            l[q] = (int32_t)(((int64_t)(int32_t)v[q] * (int64_t)pm[c0 + q] + pc[c0 + q]) >> s);
                            run32 = l[q] > run32 ? l[q] : run32;
                        }
                        mc32[ch] = run32;
#pragma unroll
                        for (int q = 0; q < 16; q += 2) {
                            const uint32_t a0 = min((uint32_t)(run32 - l[q]), lastv);
                            const uint32_t a1 = min((uint32_t)(run32 - l[q + 1]), lastv);
                            pk[ch * 8 + (q >> 1)] = a0 | (a1 << 16);
                        }
                    }
                    tc_fence_before();
                    mbar_arrive(&bars->tempty[acc]);
#pragma unroll
                    for (int ch = 0; ch < 8; ch++) {
                        const uint32_t a = min((uint32_t)(run32 - mc32[ch]), lastv);
                        const uint32_t a2 = a | (a << 16);
#pragma unroll
                        for (int w = 0; w < 8; w++) pk[ch * 8 + w] = __vminu2(__vadd2(pk[ch * 8 + w], a2), last2);
                    }
                    // Two 128-byte blocks of 64 u16 columns. Rows past R land in the padding rows of
                    // d16 (never read).
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        uint4 blk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            blk[j] = make_uint4(pk[32 * h2 + 4 * j], pk[32 * h2 + 4 * j + 1], pk[32 * h2 + 4 * j + 2],
                                                pk[32 * h2 + 4 * j + 3]);
                        store_block(blk, col0 + half * 128 + 64 * h2, mt * BM + g * 32);
                    }
                    if (row_ok && tile < e.ldt) e.tmax[(size_t)row * e.ldt + tile] = run32;
                    continue;
                }
                int64_t mc[8];
                int64_t run = -SCORE_LIMIT;
#pragma unroll
                for (int ch = 0; ch < 8; ch++) {
                    const int c0 = half * 128 + ch * 16;
                    uint32_t v[16];
                    __syncwarp();
                    tmem_ld16(taddr + c0, v);
                    tmem_ld_wait();
                    int64_t l[16];
#pragma unroll
                    for (int q = 0; q < 16; q++) {
                        l[q] = col0 + c0 + q < e.N
                                   ? clamp64(rescale_fast(v[q], pm[c0 + q], pc[c0 + q], s, fast), -SCORE_LIMIT,
                                             SCORE_LIMIT)
                                   : -SCORE_LIMIT;
                        run = l[q] > run ? l[q] : run;
                    }
                    mc[ch] = run;
#pragma unroll
                    for (int q = 0; q < 16; q += 2) {
                        const int64_t d0 = run - l[q], d1 = run - l[q + 1];
                        const uint32_t a0 = d0 < (int64_t)lastv ? (uint32_t)d0 : lastv;
                        const uint32_t a1 = d1 < (int64_t)lastv ? (uint32_t)d1 : lastv;
                        pk[ch * 8 + (q >> 1)] = a0 | (a1 << 16);
                    }
                }
                // The accumulator is read: hand it back to the MMA warp before the stores.
                tc_fence_before();
                mbar_arrive(&bars->tempty[acc]);
                if (col0 + half * 128 < e.N) {
#pragma unroll
                    for (int ch = 0; ch < 8; ch++) {
                        const int64_t sh = run - mc[ch];
                        const uint32_t a = sh < (int64_t)lastv ? (uint32_t)sh : lastv;
                        const uint32_t a2 = a | (a << 16);
#pragma unroll
                        for (int w = 0; w < 8; w++) pk[ch * 8 + w] = __vminu2(__vadd2(pk[ch * 8 + w], a2), last2);
                    }
                    // Columns past N are clipped by the tensor map; blocks wholly past N are skipped.
#pragma unroll
                    for (int h2 = 0; h2 < 2; h2++) {
                        if (col0 + half * 128 + 64 * h2 >= e.N) continue;
                        uint4 blk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++)
                            blk[j] = make_uint4(pk[32 * h2 + 4 * j], pk[32 * h2 + 4 * j + 1], pk[32 * h2 + 4 * j + 2],
                                                pk[32 * h2 + 4 * j + 3]);
                        store_block(blk, col0 + half * 128 + 64 * h2, mt * BM + g * 32);
                    }
                    if (row_ok && tile < e.ldt) e.tmax[(size_t)row * e.ldt + tile] = run;
                }
                continue;
            } else {
                // This warp's chunks of 32 columns: a contiguous range (4 of the 8 with 8 warps;
                // 3, 3 and 2 with 12).
                constexpr int CPP = (TN / 32 + NPART - 1) / NPART;
                const int c_end = min(TN, 32 * CPP * (part + 1));
                for (int c0 = 32 * CPP * part; c0 < c_end; c0 += 32) {
                    uint32_t v[32];
                    __syncwarp();
                    tmem_ld32(taddr + c0, v);
                    tmem_ld_wait();
                    const int colb = col0 + c0;
                    if (colb >= e.N) continue;
                    // GELU and DELTA store through TMA (warp-collective): rows past R land in the
                    // padding rows of the output, which nothing reads.
                    // EPI_QKV: the TMA stores are warp-collective too; its other stores check row_ok.
                    if (MODE != EPI_GELU && MODE != EPI_DELTA && MODE != EPI_QKV && !row_ok) continue;
                    const bool full = colb + 32 <= e.N;
                    // The rescaled values: 32-bit on the S32 path, computed for the whole chunk.
                    int32_t y32[32];
                    if constexpr (S32) {
                        if (s >= 32) rescale_chunk32<true>(v, pm + c0, pc + c0, s, y32);
                        else rescale_chunk32<false>(v, pm + c0, pc + c0, s, y32);
                    }
                    auto Y = [&](int q) {
                        if constexpr (S32) return y32[q];
                        else return rescale_fast(v[q], pm[c0 + q], pc[c0 + q], s, fast);
                    };
                    if (MODE == EPI_QKV) {
                        const RowInfo ri = e.rows[row];  // rows past R read stale entries of the table
                        int8_t o[32];
#pragma unroll
                        for (int q = 0; q < 32; q++)
                            o[q] = (int8_t)clamp_e(Y(q), -127, 127);
                        uint32_t pk[8];
#pragma unroll
                        for (int q = 0; q < 8; q++)
                            pk[q] = (uint32_t)(uint8_t)o[4 * q] | (uint32_t)(uint8_t)o[4 * q + 1] << 8 |
                                    (uint32_t)(uint8_t)o[4 * q + 2] << 16 | (uint32_t)(uint8_t)o[4 * q + 3] << 24;
                        // The 32 x 32-byte pieces of whole runs leave by TMA (kv_tma): q rows to the qkv
                        // buffer (rows past R land in its padding rows), and, for a warp whose 32 rows
                        // are 32 consecutive positions of one slot, key rows and the transposed value
                        // rows straight into the caches.
                        if (e.kv_tma && full && colb + 32 <= e.d) {
                            store_piece2(&tmC, pk, colb, mt * BM + g * 32);
                            continue;
                        }
                        if (e.kv_tma && full && vt_ok && colb >= e.d && colb < 2 * e.d) {
                            const int j = colb - e.d, h = j / e.hd, c = j - h * e.hd;
                            const size_t head = ((size_t)vt_slot * e.L + e.layer) * e.H + h;
                            store_piece2(&tmK, pk, c, (int)(head * e.n_ctx + vt_pos0));
                            continue;
                        }
                        if (e.kv_tma && full && vt_ok && colb >= 2 * e.d) {
                            // The 32 x 32 transpose through shared memory; lane l then holds the 32
                            // positions of channel colb - 2d + l, which leave as one TMA piece.
                            uint8_t* tile = reinterpret_cast<uint8_t*>(s_gelu) + (warp - 2) * VT_TILE;
#pragma unroll
                            for (int q = 0; q < 8; q++) *reinterpret_cast<uint32_t*>(tile + lane * VT_STRIDE + 4 * q) = pk[q];
                            __syncwarp();
                            uint32_t tk[8];
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                tk[q] = (uint32_t)tile[(4 * q) * VT_STRIDE + lane] |
                                        (uint32_t)tile[(4 * q + 1) * VT_STRIDE + lane] << 8 |
                                        (uint32_t)tile[(4 * q + 2) * VT_STRIDE + lane] << 16 |
                                        (uint32_t)tile[(4 * q + 3) * VT_STRIDE + lane] << 24;
                            __syncwarp();
                            const int j = colb - 2 * e.d, h = j / e.hd, c = j - h * e.hd;
                            const size_t head = ((size_t)vt_slot * e.L + e.layer) * e.H + h;
                            store_piece2(&tmV, tk, (int)vt_pos0, (int)(head * e.hd + c));
                            continue;
                        }
                        if (!row_ok) continue;
                        if (full && colb + 32 <= e.d && (e.ldo & 15) == 0) {
                            // A whole 32-byte run of q.
                            uint32_t pk[8];
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                pk[q] = (uint32_t)(uint8_t)o[4 * q] | (uint32_t)(uint8_t)o[4 * q + 1] << 8 |
                                        (uint32_t)(uint8_t)o[4 * q + 2] << 16 | (uint32_t)(uint8_t)o[4 * q + 3] << 24;
                            uint4* dst = reinterpret_cast<uint4*>(e.out8 + (size_t)row * e.ldo + colb);
                            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                        } else if (full && (e.hd & 31) == 0 && (e.d & 31) == 0 && colb >= e.d && colb < 2 * e.d) {
                            // A whole 32-byte run of one key row.
                            const int j = colb - e.d, h = j / e.hd, c = j - h * e.hd;
                            const size_t head = ((size_t)ri.slot * e.L + e.layer) * e.H + h;
                            uint32_t pk[8];
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                pk[q] = (uint32_t)(uint8_t)o[4 * q] | (uint32_t)(uint8_t)o[4 * q + 1] << 8 |
                                        (uint32_t)(uint8_t)o[4 * q + 2] << 16 | (uint32_t)(uint8_t)o[4 * q + 3] << 24;
                            uint4* dst = reinterpret_cast<uint4*>(e.kc + (head * e.n_ctx + ri.pos) * e.hd + c);
                            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                        } else if (full && vt_stage && colb >= 2 * e.d && (e.ldv & 15) == 0 &&
                                   colb + 32 <= 3 * e.d) {
                            // A whole 32-byte run of v of one row, to the staging rows.
                            uint32_t pk[8];
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                pk[q] = (uint32_t)(uint8_t)o[4 * q] | (uint32_t)(uint8_t)o[4 * q + 1] << 8 |
                                        (uint32_t)(uint8_t)o[4 * q + 2] << 16 | (uint32_t)(uint8_t)o[4 * q + 3] << 24;
                            uint4* dst = reinterpret_cast<uint4*>(e.vstage + (size_t)row * e.ldv + (colb - 2 * e.d));
                            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                        } else if (full && vt_ok && colb >= 2 * e.d) {
                            // 32 channels of v for 32 consecutive positions: transpose the 32 x 32
                            // bytes through shared memory, then each lane writes one channel's 32
                            // positions (two 16-byte stores into the transposed values cache).
                            uint8_t* tile = reinterpret_cast<uint8_t*>(s_gelu) + (warp - 2) * VT_TILE;
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                *reinterpret_cast<uint32_t*>(tile + lane * VT_STRIDE + 4 * q) =
                                    (uint32_t)(uint8_t)o[4 * q] | (uint32_t)(uint8_t)o[4 * q + 1] << 8 |
                                    (uint32_t)(uint8_t)o[4 * q + 2] << 16 | (uint32_t)(uint8_t)o[4 * q + 3] << 24;
                            __syncwarp();
                            uint32_t pk[8];
#pragma unroll
                            for (int q = 0; q < 8; q++)
                                pk[q] = (uint32_t)tile[(4 * q) * VT_STRIDE + lane] |
                                        (uint32_t)tile[(4 * q + 1) * VT_STRIDE + lane] << 8 |
                                        (uint32_t)tile[(4 * q + 2) * VT_STRIDE + lane] << 16 |
                                        (uint32_t)tile[(4 * q + 3) * VT_STRIDE + lane] << 24;
                            __syncwarp();
                            const int j = colb - 2 * e.d + lane, h = j / e.hd, c = j - h * e.hd;
                            const size_t head = ((size_t)vt_slot * e.L + e.layer) * e.H + h;
                            uint4* dst = reinterpret_cast<uint4*>(e.vc + (head * e.hd + c) * e.n_ctx + vt_pos0);
                            dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                            dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; q++)
                                if (colb + q < e.N) qkv_store(e, row, ri, colb + q, o[q], vt_stage);
                        }
                    } else if (MODE == EPI_ACT || MODE == EPI_GELU) {
                        uint32_t packed[8];
#pragma unroll
                        for (int w = 0; w < 8; w++) {
                            int32_t o4[4];
#pragma unroll
                            for (int k = 0; k < 4; k++) {
                                const auto y = Y(4 * w + k);
                                if (MODE == EPI_ACT) {
                                    o4[k] = (int32_t)clamp_e(y, -127, 127);
                                } else {
                                    const auto in = clamp_e(y, -e.gelu_off, e.gelu_off - 1);
                                    o4[k] = s_gelu[in + e.gelu_off];
                                }
                            }
                            packed[w] = pack4_i8(o4[0], o4[1], o4[2], o4[3]);
                        }
                        int8_t* dst = e.out8 + (size_t)row * e.ldo + colb;
                        if (MODE == EPI_GELU) {
                            store_piece(make_uint4(packed[0], packed[1], packed[2], packed[3]),
                                        make_uint4(packed[4], packed[5], packed[6], packed[7]), colb, mt * BM + g * 32);
                        } else if (full && (e.ldo & 15) == 0) {
                            reinterpret_cast<uint4*>(dst)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                            reinterpret_cast<uint4*>(dst)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; q++)
                                if (colb + q < e.N) dst[q] = (int8_t)(packed[q >> 2] >> (8 * (q & 3)));
                        }
                    } else if (MODE == EPI_GELU16) {
                        // i16 GELU outputs as two i8 planes (hi, lo): v = 256 hi + lo + 128.
                        uint32_t ph[8], pl[8];
#pragma unroll
                        for (int q = 0; q < 8; q++) ph[q] = pl[q] = 0;
#pragma unroll
                        for (int q = 0; q < 32; q++) {
                            const auto y = Y(q);
                            const auto in = clamp_e(y, -e.gelu_off, e.gelu_off - 1);
                            const int32_t g16 = __ldg(e.gelu16 + (int64_t)in + e.gelu_off);
                            ph[q >> 2] |= (uint32_t)(uint8_t)(int8_t)(g16 >> 8) << (8 * (q & 3));
                            pl[q >> 2] |= (uint32_t)(uint8_t)(int8_t)((g16 & 255) - 128) << (8 * (q & 3));
                        }
                        int8_t* dh = e.out8 + (size_t)row * e.ldo + colb;
                        int8_t* dl = e.out8_lo + (size_t)row * e.ldo + colb;
                        if (full && (e.ldo & 15) == 0) {
                            reinterpret_cast<uint4*>(dh)[0] = make_uint4(ph[0], ph[1], ph[2], ph[3]);
                            reinterpret_cast<uint4*>(dh)[1] = make_uint4(ph[4], ph[5], ph[6], ph[7]);
                            reinterpret_cast<uint4*>(dl)[0] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
                            reinterpret_cast<uint4*>(dl)[1] = make_uint4(pl[4], pl[5], pl[6], pl[7]);
                        } else {
#pragma unroll
                            for (int q = 0; q < 32; q++)
                                if (colb + q < e.N) {
                                    dh[q] = (int8_t)(ph[q >> 2] >> (8 * (q & 3)));
                                    dl[q] = (int8_t)(pl[q >> 2] >> (8 * (q & 3)));
                                }
                        }
                    } else if (MODE == EPI_DELTA) {
                        int32_t o[32];
#pragma unroll
                        for (int q = 0; q < 32; q++) {
                            if constexpr (S32) o[q] = y32[q];
                            else o[q] = (int32_t)clamp64(Y(q), INT32_MIN, INT32_MAX);
                        }
                        uint4 blk[8];
#pragma unroll
                        for (int j = 0; j < 8; j++) blk[j] = make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                        store_block(blk, colb, mt * BM + g * 32);
                    } else if (MODE == EPI_RAW) {
                        int32_t* dst = e.out32 + (size_t)row * e.ldo + colb;
#pragma unroll
                        for (int q = 0; q < 32; q++)
                            if (colb + q < e.N) dst[q] = (int32_t)v[q];
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&bars->tempty[acc]);
        }
        // The TMA stores of this warp are complete before the CTA (and its shared memory) ends.
        if (Cfg<MODE>::STORE_WARP > 0 && lane == 0) bulk_wait_all();
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

template <int MODE>
void launch_mode(const void* tmA, const void* tmA2, const void* tmB, const void* tmC, const void* tmK,
                 const void* tmV, int MT, int NT, int KB, const EpiArgs& e, int grid, int* err, cudaStream_t st,
                 bool narrow) {
    const CUtensorMap& a = *reinterpret_cast<const CUtensorMap*>(tmA);
    const CUtensorMap& b = *reinterpret_cast<const CUtensorMap*>(tmB);
    const CUtensorMap& c = *reinterpret_cast<const CUtensorMap*>(tmC ? tmC : tmB);
    const CUtensorMap& k = *reinterpret_cast<const CUtensorMap*>(tmK ? tmK : tmB);
    const CUtensorMap& v = *reinterpret_cast<const CUtensorMap*>(tmV ? tmV : tmB);
    if constexpr (MODE == EPI_DELTA || MODE == EPI_LOGITS) {
        if (tmA2) {
            const CUtensorMap& a2 = *reinterpret_cast<const CUtensorMap*>(tmA2);
            k_gemm_tc<MODE, false, true><<<grid, Cfg<MODE>::THREADS, Cfg<MODE>::SMEM, st>>>(a, a2, b, c, k, v, MT, NT, KB, e, err);
            return;
        }
    }
    if constexpr (MODE == EPI_ACT || MODE == EPI_GELU || MODE == EPI_DELTA || MODE == EPI_QKV) {
        if (narrow) {
            if (e.small && e.s >= 0 && e.s <= 62)
                k_gemm_tc<MODE, true, false, true><<<grid, Cfg<MODE>::THREADS, Cfg<MODE>::SMEM, st>>>(a, a, b, c, k, v, MT,
                                                                                                 NT, KB, e, err);
            else
                k_gemm_tc<MODE, false, false, true><<<grid, Cfg<MODE>::THREADS, Cfg<MODE>::SMEM, st>>>(a, a, b, c, k, v, MT,
                                                                                                  NT, KB, e, err);
            return;
        }
    }
    if (MODE != EPI_RAW && e.small && e.s >= 0 && e.s <= 62)
        k_gemm_tc<MODE, true, false><<<grid, Cfg<MODE>::THREADS, Cfg<MODE>::SMEM, st>>>(a, a, b, c, k, v, MT, NT, KB, e, err);
    else
        k_gemm_tc<MODE, false, false><<<grid, Cfg<MODE>::THREADS, Cfg<MODE>::SMEM, st>>>(a, a, b, c, k, v, MT, NT, KB, e, err);
}

template <int MODE>
cudaError_t configure_mode() {
    cudaError_t r = cudaFuncSetAttribute(k_gemm_tc<MODE, true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)Cfg<MODE>::SMEM);
    if (r != cudaSuccess) return r;
    r = cudaFuncSetAttribute(k_gemm_tc<MODE, false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             (int)Cfg<MODE>::SMEM);
    if (r != cudaSuccess) return r;
    if constexpr (MODE == EPI_DELTA || MODE == EPI_LOGITS)
        r = cudaFuncSetAttribute(k_gemm_tc<MODE, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Cfg<MODE>::SMEM);
    if (r != cudaSuccess) return r;
    if constexpr (MODE == EPI_ACT || MODE == EPI_GELU || MODE == EPI_DELTA || MODE == EPI_QKV) {
        r = cudaFuncSetAttribute(k_gemm_tc<MODE, true, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Cfg<MODE>::SMEM);
        if (r != cudaSuccess) return r;
        r = cudaFuncSetAttribute(k_gemm_tc<MODE, false, false, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 (int)Cfg<MODE>::SMEM);
    }
    return r;
}

}  // namespace

cudaError_t configure_tc_kernels() {
    cudaError_t e;
    if ((e = configure_mode<EPI_ACT>()) != cudaSuccess) return e;
    if ((e = configure_mode<EPI_GELU>()) != cudaSuccess) return e;
    if ((e = configure_mode<EPI_LOGITS>()) != cudaSuccess) return e;
    if ((e = configure_mode<EPI_RAW>()) != cudaSuccess) return e;
    if ((e = configure_mode<EPI_QKV>()) != cudaSuccess) return e;
    if ((e = configure_mode<EPI_GELU16>()) != cudaSuccess) return e;
    return configure_mode<EPI_DELTA>();
}

void launch_gemm_tc(int mode, const void* tmA, const void* tmB, const void* tmC, int R, int Np, int Kp,
                    const EpiArgs& e, int num_sms, int* err, cudaStream_t st, const void* tmA2, const void* tmK,
                    const void* tmV, const void* tmB64) {
    if (R <= 0) return;
    int MT = (R + BM - 1) / BM, NT = Np / (tmA2 ? 128 : BN), KB = Kp / BK;
    // 256-column tiles for at most half the SMs (a decode step): 64-column tiles, four times as many
    // CTAs. (With 96 tiles on 148 SMs, the fc GEMM of a 1,024-row step, the narrow tiles were 12 %
    // slower; with 24, proj and mlp, 17-19 % faster.)
    const bool narrow = tmB64 != nullptr && !tmA2 && Np % 64 == 0 && 2 * MT * NT <= num_sms &&
                        (mode == EPI_ACT || mode == EPI_GELU || mode == EPI_DELTA || mode == EPI_QKV);
    if (narrow) {
        NT = Np / 64;
        tmB = tmB64;
    }
    int tiles = MT * NT;
    int grid = tiles < num_sms ? tiles : num_sms;
    switch (mode) {
        case EPI_ACT: launch_mode<EPI_ACT>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, narrow); break;
        case EPI_GELU: launch_mode<EPI_GELU>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, narrow); break;
        case EPI_LOGITS: launch_mode<EPI_LOGITS>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, false); break;
        case EPI_RAW: launch_mode<EPI_RAW>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, false); break;
        case EPI_DELTA: launch_mode<EPI_DELTA>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, narrow); break;
        case EPI_QKV: launch_mode<EPI_QKV>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, narrow); break;
        case EPI_GELU16: launch_mode<EPI_GELU16>(tmA, tmA2, tmB, tmC, tmK, tmV, MT, NT, KB, e, grid, err, st, false); break;
        default: break;
    }
}

}  // namespace hs
