// The int8 GEMM of the B200 HardShell backend on the 5th-generation tensor cores.
//
// out = epilogue(A . W^T): A is [rows, Kp] int8 (activations), W is [Np, Kp] int8 (weights),
// both K-major, loaded by TMA with the 128-byte swizzle (no multicast). tcgen05.mma kind::i8
// accumulates exact s32 sums in TMEM; the epilogue warps read TMEM and apply the fixed-point
// requantisation of HardShell (crates/hardshell/src/gpt2/ops.rs:107-169 linear, :213 logits)
// before any value leaves the SM.
//
// Persistent kernel, one CTA per SM, 6 warps:
//   warp 0      TMA producer (one thread): A and B tiles into a 4-stage ring;
//   warp 1      TMEM owner and MMA issuer (one thread);
//   warps 2..5  epilogue: each thread owns one accumulator row (TMEM lane).
// The accumulator is double-buffered in TMEM (2 x 256 columns), so the epilogue of one tile runs
// while the MMAs of the next tile fill the other buffer. Every wait is bounded.
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
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK;
constexpr int B_BYTES = BN * BK;
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
constexpr int TMEM_COLS = 2 * BN;
constexpr int THREADS = 192;
constexpr size_t SMEM_BYTES = (size_t)STAGES * STAGE_BYTES + 1024 + 256;

struct __align__(8) Bars {
    uint64_t full[STAGES];
    uint64_t empty[STAGES];
    uint64_t tfull[2];
    uint64_t tempty[2];
    uint32_t tmem_base;
};

__device__ __forceinline__ void epi_chunk(int mode, const EpiArgs& e, int row, int col, const uint32_t (&v)[16]) {
    const bool row_ok = row < e.R;
    if (!row_ok) return;
    if (mode == EPI_RAW) {
#pragma unroll
        for (int i = 0; i < 16; i++)
            if (col + i < e.N) e.out32[(size_t)row * e.ldo + col + i] = (int32_t)v[i];
        return;
    }
    if (mode == EPI_ACT || mode == EPI_GELU) {
        uint32_t packed[4] = {0, 0, 0, 0};
#pragma unroll
        for (int i = 0; i < 16; i++) {
            int n = col + i < e.N ? col + i : e.N - 1;
            int64_t y = rescale64((int64_t)(int32_t)v[i] + (int64_t)e.b[n], e.m[n], e.s);
            int8_t o;
            if (mode == EPI_ACT) {
                o = (int8_t)clamp64(y, -127, 127);
            } else {
                int64_t in = clamp64(y, -e.gelu_off, e.gelu_off - 1);
                o = e.gelu[in + e.gelu_off];
            }
            packed[i >> 2] |= (uint32_t)(uint8_t)o << (8 * (i & 3));
        }
        int8_t* dst = e.out8 + (size_t)row * e.ldo + col;
        if (col + 16 <= e.N && (e.ldo & 15) == 0) {
            *reinterpret_cast<uint4*>(dst) = make_uint4(packed[0], packed[1], packed[2], packed[3]);
        } else {
#pragma unroll
            for (int i = 0; i < 16; i++)
                if (col + i < e.N) dst[i] = (int8_t)(packed[i >> 2] >> (8 * (i & 3)));
        }
        return;
    }
    if (mode == EPI_RESID) {
        int32_t* xp = e.x + (size_t)row * e.ldx + col;
        if (col + 16 <= e.N && (e.ldx & 3) == 0) {
#pragma unroll
            for (int q = 0; q < 4; q++) {
                int4 xv = reinterpret_cast<int4*>(xp)[q];
                int32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
                for (int i = 0; i < 4; i++) {
                    int n = col + 4 * q + i;
                    int64_t y = rescale64((int64_t)(int32_t)v[4 * q + i] + (int64_t)e.b[n], e.m[n], e.s);
                    xs[i] = (int32_t)clamp64((int64_t)xs[i] + y, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
                }
                reinterpret_cast<int4*>(xp)[q] = make_int4(xs[0], xs[1], xs[2], xs[3]);
            }
        } else {
            for (int i = 0; i < 16; i++) {
                int n = col + i;
                if (n >= e.N) break;
                int64_t y = rescale64((int64_t)(int32_t)v[i] + (int64_t)e.b[n], e.m[n], e.s);
                xp[i] = (int32_t)clamp64((int64_t)xp[i] + y, -RESIDUAL_LIMIT, RESIDUAL_LIMIT);
            }
        }
    }
}

__device__ __forceinline__ int64_t logit_of(const EpiArgs& e, int n, uint32_t acc) {
    return clamp64(rescale64((int64_t)(int32_t)acc, e.m[n], e.s), -SCORE_LIMIT, SCORE_LIMIT);
}

__global__ void __launch_bounds__(THREADS, 1)
    k_gemm_tc(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, int mode, int MT,
              int NT, int KB, EpiArgs e, int* err) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
    Bars* bars = reinterpret_cast<Bars*>(smem + (size_t)STAGES * STAGE_BYTES);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (warp == 0 && lane == 0) {
        prefetch_tmap(&tmA);
        prefetch_tmap(&tmB);
        for (int s = 0; s < STAGES; s++) {
            mbar_init(&bars->full[s], 1);
            mbar_init(&bars->empty[s], 1);
        }
        for (int a = 0; a < 2; a++) {
            mbar_init(&bars->tfull[a], 1);
            mbar_init(&bars->tempty[a], 128);
        }
        fence_barrier_init();
    }
    if (warp == 1) {
        tmem_alloc(&bars->tmem_base, TMEM_COLS);
        tmem_relinquish();
        tc_fence_before();
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
                    mbar_arrive_expect_tx(&bars->full[stage], STAGE_BYTES);
                    tma_load_2d(sa, &tmA, &bars->full[stage], kb * BK, mt * BM);
                    tma_load_2d(sa + A_BYTES, &tmB, &bars->full[stage], kb * BK, nt * BN);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1;
                    }
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(BM, BN, true, true);
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
                    uint32_t sb = sa + A_BYTES;
#pragma unroll
                    for (int k = 0; k < BK / UMMA_K; k++) {
                        mma_i8(d, sdesc_sw128(sa + k * UMMA_K), sdesc_sw128(sb + k * UMMA_K), idesc,
                               (kb | k) != 0 ? 1u : 0u);
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
        // Epilogue: TMEM lane group g = warp % 4 (the lanes a warp may read), one row per thread.
        const int g = warp & 3;
        const int row_in_tile = g * 32 + lane;
        int i = 0;
        for (int t = blockIdx.x; t < tiles; t += gridDim.x, i++) {
            int mt = t % MT, nt = t / MT;
            int acc = i & 1;
            uint32_t aphase = (i >> 1) & 1;
            bool ready = mbar_wait(&bars->tfull[acc], aphase, err, 4);
            __syncwarp();
            if (!__all_sync(0xffffffffu, ready)) break;
            tc_fence_after();
            const int row = mt * BM + row_in_tile;
            const uint32_t taddr = tmem_base + ((uint32_t)(g * 32) << 16) + (uint32_t)(acc * BN);
            const int col0 = nt * BN;
            if (mode != EPI_LOGITS) {
#pragma unroll 1
                for (int c = 0; c < BN; c += 16) {
                    uint32_t v[16];
                    __syncwarp();
                    tmem_ld16(taddr + c, v);
                    tmem_ld_wait();
                    if (col0 + c < e.N) epi_chunk(mode, e, row, col0 + c, v);
                }
            } else {
                // Pass 1: the max of this row over the tile; pass 2: d16 = min(tmax - l, last).
                int64_t tm = INT64_MIN;
#pragma unroll 1
                for (int c = 0; c < BN; c += 16) {
                    uint32_t v[16];
                    __syncwarp();
                    tmem_ld16(taddr + c, v);
                    tmem_ld_wait();
#pragma unroll
                    for (int q = 0; q < 16; q++) {
                        int n = col0 + c + q;
                        if (n < e.N) {
                            int64_t l = logit_of(e, n, v[q]);
                            tm = l > tm ? l : tm;
                        }
                    }
                }
#pragma unroll 1
                for (int c = 0; c < BN; c += 16) {
                    uint32_t v[16];
                    __syncwarp();
                    tmem_ld16(taddr + c, v);
                    tmem_ld_wait();
                    if (row < e.R && col0 + c < e.N) {
                        uint32_t packed[8];
#pragma unroll
                        for (int q = 0; q < 16; q += 2) {
                            int n0 = col0 + c + q, n1 = n0 + 1;
                            uint32_t a0 = 0, a1 = 0;
                            if (n0 < e.N) {
                                int64_t dd = tm - logit_of(e, n0, v[q]);
                                a0 = (uint32_t)(dd < e.last ? dd : e.last);
                            }
                            if (n1 < e.N) {
                                int64_t dd = tm - logit_of(e, n1, v[q + 1]);
                                a1 = (uint32_t)(dd < e.last ? dd : e.last);
                            }
                            packed[q >> 1] = a0 | (a1 << 16);
                        }
                        uint16_t* dst = e.d16 + (size_t)row * e.ldd + col0 + c;
                        // d16 rows are padded to a multiple of 256 columns, so 16 entries fit.
                        reinterpret_cast<uint4*>(dst)[0] = make_uint4(packed[0], packed[1], packed[2], packed[3]);
                        reinterpret_cast<uint4*>(dst)[1] = make_uint4(packed[4], packed[5], packed[6], packed[7]);
                    }
                }
                if (row < e.R) e.tmax[(size_t)row * e.ldt + nt] = tm;
            }
            tc_fence_before();
            mbar_arrive(&bars->tempty[acc]);
        }
    }
    __syncthreads();
    if (warp == 1) {
        __syncwarp();
        tc_fence_after();
        tmem_dealloc(tmem_base, TMEM_COLS);
    }
}

}  // namespace

cudaError_t configure_tc_kernels() {
    return cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)SMEM_BYTES);
}

void launch_gemm_tc(int mode, const void* tmA, const void* tmB, int R, int Np, int Kp, const EpiArgs& e,
                    int num_sms, int* err, cudaStream_t st) {
    if (R <= 0) return;
    int MT = (R + BM - 1) / BM, NT = Np / BN, KB = Kp / BK;
    int tiles = MT * NT;
    int grid = tiles < num_sms ? tiles : num_sms;
    k_gemm_tc<<<grid, THREADS, SMEM_BYTES, st>>>(*reinterpret_cast<const CUtensorMap*>(tmA),
                                                 *reinterpret_cast<const CUtensorMap*>(tmB), mode, MT, NT, KB, e,
                                                 err);
}

}  // namespace hs
