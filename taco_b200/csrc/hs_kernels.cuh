// Launchers of the CUDA-core kernels of the B200 HardShell backend (hs_kernels.cu) and of the
// tcgen05 GEMM (hs_gemm_tc.cu). Every launcher takes the stream of its batch.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

#include "hs_device.hpp"

namespace hs {

// Set the shared-memory limits of the kernels for the current device (once per device).
cudaError_t configure_core_kernels();
cudaError_t configure_tc_kernels();

struct ModelConsts {
    int d, f, V, H, hd, L, n_ctx;
    int Dp, Fp, QKVp, Vp, VT;
    int tsh;        // log2 of the logits tile width: 7 (128 columns), 6 for a 16-bit ln_f
    bool lnf_wide;  // ln_f_bits = 16: the final LayerNorm output is i16 (two i8 planes)
    int ln_k, ln_j;
    uint64_t ln_eps;
    int softmax_p;
};

void launch_embed(const RowInfo* rows, int R, const int8_t* wte, int ldw, const int32_t* em, int es,
                  const int8_t* wpe, const int32_t* pm, int ps, int d, int32_t* x, cudaStream_t st);

// out_lo != nullptr: 16-bit outputs (ln_f_bits = 16) as two i8 planes, hi in `out` and lo in
// `out_lo` (v = 256 hi + lo + 128).
void launch_layernorm(const int32_t* x, int R, int d, const LnDev& ln, int ln_k, int ln_j, uint64_t eps,
                      int8_t* out, int ldo, cudaStream_t st, int8_t* out_lo = nullptr);

// x = clamp(x + delta, -R, R) (delta may be null), then out = LayerNorm(x) (i8).
void launch_resid_layernorm(int32_t* x, const int32_t* delta, int R, int d, const LnDev& ln, int ln_k, int ln_j,
                            uint64_t eps, int8_t* out, int ldo, cudaStream_t st, int8_t* out_lo = nullptr);

// out = epilogue(W . A^T) on CUDA cores (dp4a); the reference kernel of the tensor-core GEMM and
// the path for passes of a few rows.
void launch_gemm_simple(int mode, const int8_t* A, int lda, int R, const LinearDev& W, const EpiArgs& e,
                        cudaStream_t st);

// The same GEMM on the 5th-generation tensor cores (tcgen05, TMEM accumulators, TMA).
// `tmA` and `tmB` are CUtensorMap objects (128-byte aligned, 128 bytes each). EPI_DELTA and
// EPI_LOGITS store their output through `tmC` with 32-row x 128-byte boxes (128-byte swizzle),
// EPI_GELU with 32-row x 32-byte boxes (32-byte swizzle), over all the rows of the output buffer;
// the other modes take nullptr.
// tmA2 != nullptr (EPI_DELTA and EPI_LOGITS of version 2 models): tmA and tmA2 are the hi and lo
// planes of i16 activations, tmB has 128-row boxes and the tiles are 128 x 128.
// EPI_QKV with e.kv_tma: tmC, tmK and tmV are the 32-row x 32-byte store maps (32-byte swizzle) of
// the qkv buffer, the keys cache [heads * n_ctx, hd] and the transposed values cache
// [heads * hd, n_ctx].
void launch_gemm_tc(int mode, const void* tmA, const void* tmB, const void* tmC, int R, int Np, int Kp,
                    const EpiArgs& e, int num_sms, int* err, cudaStream_t st, const void* tmA2 = nullptr,
                    const void* tmK = nullptr, const void* tmV = nullptr, const void* tmB64 = nullptr);

#ifdef __CUDACC__
// vt_run_host for the warp whose lane l holds row r0 + l (warp-uniform result).
__device__ __forceinline__ bool vt_run_warp(const RowInfo* rows, int r0, int R, int n_ctx, int lane) {
    if (r0 + 31 >= R || (n_ctx & 15) != 0) return false;
    const RowInfo a0 = rows[r0], me = rows[r0 + lane];
    const bool mine = me.slot == a0.slot && me.pos == a0.pos + (uint32_t)lane;
    return __all_sync(0xffffffffu, mine) && (a0.pos & 15) == 0;
}
#endif

// The range decoder of the batched unfold (hs_decode.cu): the states of n blocks, one step's rows
// (the live blocks are the first R), the consumption of one step's intervals, the targets of a
// host-run step, and the failed flags.
void launch_dec_init(DecState* st, const uint8_t* payload, const uint64_t* offsets, const uint64_t* lengths,
                     uint32_t* prev, uint32_t eot, int n, cudaStream_t s);
void launch_dec_begin(const DecState* st, int R, const uint32_t* slot_of, const uint32_t* pos_of,
                      uint32_t steps_since, const uint32_t* prev, uint32_t bits, RowInfo* rows, cudaStream_t s);
void launch_dec_end(DecState* st, int R, const uint64_t* intervals, uint32_t bits, uint32_t V, const uint8_t* payload,
                    uint32_t* prev, uint32_t* out, const uint64_t* out_off, uint32_t step, cudaStream_t s);
void launch_dec_targets(const DecState* st, int R, uint32_t bits, uint64_t* targets, cudaStream_t s);
void launch_dec_gather(const uint32_t* out, const uint64_t* out_off, const uint32_t* counts, int L, uint32_t s0,
                       uint32_t s1, uint32_t* dst, cudaStream_t s);
void launch_dec_status(const DecState* st, int n, uint32_t* status, cudaStream_t s);

// The v of the rows in 32-row groups that are not vt_run, from the QKV epilogue's row-major
// staging (stride ldv) into the transposed values cache of one layer.
void launch_v_scatter(const RowInfo* rows, int R, const int8_t* vstage, int ldv, int d, int H, int hd, int L,
                      int layer, int n_ctx, int8_t* vc, cudaStream_t st);

// Attention of the rows `rowlist[0..n)` (all R rows when rowlist is null) on CUDA cores: the
// decode path and the rows that are not in a prefill group.
void launch_attention(const RowInfo* rows, int R, const int* rowlist, int n, const int8_t* qkv, int ldq,
                      const int8_t* kc, const int8_t* vc, int L, int layer, int H, int hd, int n_ctx, int d,
                      int32_t sm, int ss, int32_t om, int os, const int32_t* table, int tlen, int P, int8_t* att,
                      int lda, cudaStream_t st);

// Prefill attention of whole groups on the tensor cores (hs_attn_tc.cu). tmQ covers the qkv
// buffer (box 64 x 128, 64-byte swizzle), tmK the keys cache (64 x 128, 64-byte swizzle), tmV the
// transposed values cache (128 x 64, 128-byte swizzle).
cudaError_t configure_attn_tc();
bool attention_tc_supported(int hd, int n_ctx, int tlen);
// The rows of a pass outside the prefill groups (batched decode) with one warp per (row, head):
// head width 64, n_ctx % 16 == 0, 16-byte aligned q rows.
bool attention_dec_supported(int hd, int n_ctx, int ldq, int tlen);
void launch_attention_dec(const RowInfo* rows, const int* rowlist, int nrows, const int8_t* qkv, int ldq,
                          const int8_t* kc, const int8_t* vc, int L, int layer, int H, int n_ctx, int32_t sm, int ss,
                          int32_t om, int os, const int32_t* table, int tlen, int P, int8_t* att, int lda,
                          cudaStream_t st);

// The prefill attention's scratch: one slot per persistent CTA (the launch uses at most
// scr_slots CTAs; one per SM is the most that fit), attn_scratch_bytes(slots, n_ctx) bytes in all.
size_t attn_scratch_bytes(int slots, int n_ctx);
void launch_attention_tc(const void* tmQ, const void* tmK, const void* tmV, const AttnGroup* groups, int n_groups,
                         int L, int layer, int H, int n_ctx, int32_t sm, int ss, int32_t om, int os,
                         const int32_t* table, int tlen, int P, int8_t* att, int lda, uint8_t* scratch, int scr_slots,
                         int* err, cudaStream_t st);

// The coder op: from the d16/tmax output of the logits GEMM, the interval of each row's query
// in the table of taco_coder::FreqTable::from_weights(weights, bits). out: 3 u64 per row. `head`
// is the last index j with table[j] == table[0] (the table is not increasing).
void launch_coder(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                  const uint64_t* table, int tlen, int head, uint32_t bits, const RowInfo* rows, uint64_t* out,
                  int* err, cudaStream_t st);

// The mixed coder op of the profile logs, in two phases around a host step. Phase 0 (the stats
// kernel): out = {W, w[p], top} of the GPT-2 weights of each row, p = mix[r].p. Phase 1: the
// interval of each row's query in the table from_weights(w', bits) of the mixed weights w' that
// mix[r] describes. One block per row, as launch_coder.
void launch_coder_mix(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                      const uint64_t* table, int tlen, int head, uint32_t bits, const RowInfo* rows,
                      const MixRow* mix, int phase, uint64_t* out, int* err, cudaStream_t st);

// The full weights of each row (run_weights): w[r, v] = table[min(max - logit, last)].
void launch_weights(const uint16_t* d16, int ldd, const int64_t* tmax, int ldt, int tsh, int R, int V,
                    const uint64_t* table, int tlen, uint64_t* w, cudaStream_t st);

}  // namespace hs
