// The host runtime of the B200 HardShell backend and its C ABI (include/hardshell_b200.h).
//
// It restates the CUDA engine of the reference (crates/hardshell-cuda) B200-first:
// - the device: one CUDA context per GPU, one stream per batch (device.rs);
// - the model: the validated .hsm uploaded once, every weight matrix padded to the GEMM tiles
//   (K to 128 bytes, N to 256 rows) with its TMA descriptor (model.rs);
// - the batch: slots with their KV caches, the pass planner with the context restart and
//   overlap (batch/plan.rs:60-120), one forward pass per plan pass, and the coder op, so that only
//   32 bytes per input come back (batch.rs:463-570). Positions change only after every pass ran.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <string>
#include <unordered_map>
#include <deque>
#include <vector>

#include "../../include/hardshell_b200.h"
#include "hs_device.hpp"
#include "hs_kernels.cuh"
#include "hs_host.hpp"
#include "hsm_file.hpp"
#include "sha256.hpp"

using namespace hs;

namespace {

thread_local std::string g_err;

int fail(int code, const std::string& msg) {
    g_err = msg;
    return code;
}

}  // namespace

int hs::host_fail(int code, const std::string& msg) { return fail(code, msg); }

namespace {

#define CK(call)                                                                                     \
    do {                                                                                             \
        cudaError_t e_ = (call);                                                                     \
        if (e_ != cudaSuccess)                                                                       \
            return fail(HS_CUDA, std::string(#call) + " failed: " + cudaGetErrorString(e_));         \
    } while (0)

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The GEMM path: the tensor-core kernel, or the dp4a kernel (HS_GEMM=simple, for tests).
bool use_tc_default() {
    const char* v = getenv("HS_GEMM");
    return !(v && strcmp(v, "simple") == 0);
}

// The prefill attention path: tensor cores for groups of rows (default), or CUDA cores for every
// row (HS_ATTN=vec, for tests).
bool use_attn_tc_default() {
    const char* v = getenv("HS_ATTN");
    return !(v && strcmp(v, "vec") == 0);
}

// The smallest group of consecutive rows of one slot that takes the tensor-core attention.
constexpr int ATTN_TC_MIN_ROWS = 16;

}  // namespace

struct hs_dev {
    int ordinal = 0;
    int num_sms = 0;
    std::string name;
    int* d_err = nullptr;
    EncodeTiledFn encode = nullptr;
};

namespace {

int set_device(hs_dev* d) {
    CK(cudaSetDevice(d->ordinal));
    return HS_OK;
}

// A 2D int8 tensor map over [rows, cols] (cols contiguous): box {box_cols, box_rows} with the
// 128-byte swizzle (box_cols = 128) or the 64-byte swizzle (box_cols = 64).
int make_tmap(hs_dev* dev, CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows,
              uint32_t box_cols = TILE_K) {
    cuuint64_t gdim[2] = {cols, rows};
    cuuint64_t gstride[1] = {cols};
    cuuint32_t box[2] = {box_cols, box_rows};
    cuuint32_t estr[2] = {1, 1};
    if (((uintptr_t)base & 15) != 0 || (cols & 15) != 0)
        return fail(HS_UNSUPPORTED, "a TMA tensor needs 16-byte aligned rows");
    CUtensorMapSwizzle sw = box_cols == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
    CUresult r = dev->encode(tm, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HS_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return HS_OK;
}

// The store tensor map of a GEMM epilogue: [rows, cols] elements of `esize` bytes with a row pitch
// of `ld` elements, boxes of 32 rows x box_bytes (32 or 128) with the swizzle of that width.
int make_store_tmap(hs_dev* dev, CUtensorMap* tm, const void* base, CUtensorMapDataType type, int esize,
                    uint64_t rows, uint64_t cols, uint64_t ld, int box_bytes) {
    cuuint64_t gdim[2] = {cols, rows};
    cuuint64_t gstride[1] = {ld * (uint64_t)esize};
    cuuint32_t box[2] = {(cuuint32_t)(box_bytes / esize), 32};
    cuuint32_t estr[2] = {1, 1};
    if (((uintptr_t)base & 15) != 0 || (gstride[0] & 15) != 0)
        return fail(HS_UNSUPPORTED, "a TMA tensor needs 16-byte aligned rows");
    CUresult r = dev->encode(tm, type, 2, const_cast<void*>(base), gdim, gstride, box, estr,
                             CU_TENSOR_MAP_INTERLEAVE_NONE,
                             box_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_32B,
                             CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(HS_CUDA, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return HS_OK;
}

template <typename T>
int dalloc(T** p, size_t count, std::vector<void*>& owned) {
    void* q = nullptr;
    size_t bytes = std::max<size_t>(count * sizeof(T), 16);
    CK(cudaMalloc(&q, bytes));
    CK(cudaMemset(q, 0, bytes));
    owned.push_back(q);
    *p = (T*)q;
    return HS_OK;
}

template <typename T>
int upload(T** p, const T* src, size_t count, std::vector<void*>& owned) {
    int rc = dalloc(p, count, owned);
    if (rc) return rc;
    if (count) CK(cudaMemcpy(*p, src, count * sizeof(T), cudaMemcpyHostToDevice));
    return HS_OK;
}

struct DevLinear {
    LinearDev ld{};
    bool small = false;  // every rescaled output is below 2^30 in magnitude (32-bit epilogue)
    // A linear over i16 activations (version 2): the row sums sum_k W[n][k] and a tensor map with
    // 128-row boxes (the 128 x 128 tiles of the two-plane GEMM).
    int64_t* wsum = nullptr;
    alignas(128) CUtensorMap tm;
    alignas(128) CUtensorMap tm128;
    alignas(128) CUtensorMap tm64;  // 64-row boxes: the 64-column tiles of passes of few rows
};

}  // namespace

struct hs_model {
    hs_dev* dev = nullptr;
    std::vector<void*> owned;
    ModelConsts c{};
    uint32_t eot = 0, version = 1;
    uint8_t hash[32] = {0};
    uint64_t weight_bytes = 0;
    bool use_tc = true;
    bool attn_tc = false;
    bool attn_dec = false;  // the warp-per-(row, head) decode attention for rows outside the groups
    int8_t* wte = nullptr;
    int32_t* em = nullptr;
    int es = 0;
    int32_t* lm = nullptr;
    int ls = 0;
    int8_t* wpe = nullptr;
    int32_t* pm = nullptr;
    int ps = 0;
    std::vector<LayerDev> layers;
    std::vector<std::unique_ptr<DevLinear>> lins;  // 4 per layer (qkv, proj, fc, mlp), then the LM head
    LnDev lnf{};
    int32_t* attn_exp = nullptr;
    int attn_len = 0;
    uint64_t* logits_exp = nullptr;
    int logits_len = 0;
    int logits_head = 0;  // the last index j with logits_exp[j] == logits_exp[0]

    ~hs_model() {
        if (dev && cudaSetDevice(dev->ordinal) != cudaSuccess) cudaGetLastError();
        for (void* p : owned) cudaFree(p);
    }
};

// The bookkeeping of one slot's inputs for a truncation (crates/hardshell/src/gpt2/stream.rs
// StreamState): the inputs since the last reset, the first input position of the current
// context (0, or K + 1 after a restart), one more than the highest position the current context
// wrote, and `first` of the context before the last restart (-1: none).
struct StreamSt {
    uint32_t len = 0, first = 0, written = 0;
    int32_t prev_first = -1;
};

struct hs_batch {
    hs_model* model = nullptr;
    int slots = 0, max_rows = 0, Rcap = 0;
    uint16_t overlap = 0;
    std::vector<int> pos;
    std::vector<uint32_t> hist;  // [slots, n_ctx]
    std::vector<uint32_t> hist_work;  // the planning copy of hist during a call (swapped in on commit)
    std::vector<StreamSt> streams;              // per slot
    std::vector<std::vector<uint32_t>> prev;    // per slot: the full context before the last restart
    std::vector<void*> owned;
    cudaStream_t stream = nullptr;
    int8_t* kc = nullptr;
    int8_t* vc = nullptr;
    RowInfo* d_rows = nullptr;
    int32_t* x = nullptr;
    int8_t* a = nullptr;
    int8_t* qkv = nullptr;
    int8_t* att = nullptr;
    int8_t* g = nullptr;
    // Version 2: the lo planes of the i16 ln_f output and of the i16 GELU outputs.
    int8_t* a_lo = nullptr;
    int8_t* g_lo = nullptr;
    int32_t* dbuf = nullptr;  // the residual delta of the last proj/mlp GEMM
    // The logits of the mixed coder op (a whole pass; made on the first mixed call).
    uint16_t* d16 = nullptr;
    int64_t* tmax = nullptr;
    // The logits of the other paths: the LM head and the coder run in chunks of `lchunk` rows,
    // so the distances of a chunk (lchunk x 50,432 x 2 bytes) stay in L2 between the GEMM that
    // writes them and the coder that reads them.
    uint16_t* d16c = nullptr;
    int64_t* tmaxc = nullptr;
    int lchunk = 0;
    uint64_t* intervals = nullptr;
    uint64_t* weights = nullptr;
    // The host copies of a pass (pinned, two halves: run() prepares the next pass in one half
    // while the GPU works on the pass it uploaded from the other); the pointers below are the
    // current half.
    RowInfo* h_rows_base = nullptr;
    uint64_t* h_intervals_base = nullptr;
    AttnGroup* h_groups_base = nullptr;
    int* h_rowlist_base = nullptr;
    RowInfo* h_rows = nullptr;
    uint64_t* h_intervals = nullptr;
    AttnGroup* h_groups = nullptr;
    int* h_rowlist = nullptr;
    cudaEvent_t pass_done[2] = {nullptr, nullptr};  // recorded after a pass's read back, per half
    AttnGroup* d_groups = nullptr;   // the prefill groups of the pass
    uint8_t* attn_scr = nullptr;     // the prefill attention's scratch, one slot per persistent CTA
    int attn_scr_slots = 0;
    int* d_rowlist = nullptr;        // the other rows of the pass
    int n_groups = 0, n_rowlist = 0;
    bool v_scatter = false;  // some 32-row group of the pass is not a transposed v run
    // The mixed coder op (made on its first use): the mix records of a pass, the statistics of
    // its rows and the intervals of GPT-2 alone (run_coded_dual), with pinned host copies.
    // Mixed passes run two deep (the host mixer of pass k beside the forward pass of pass k + 1),
    // so pass k uses half k & 1 of the row table and of the logits (d16, tmax and the store map
    // of d16); half 0 is the batch's own, half 1 is made with the mixed buffers. The pinned host
    // buffers have a half per pass parity too: h_mix holds the table words [2][Rcap] of the
    // statistics kernel, then the mix records [2][Rcap].
    MixRow* d_mix = nullptr;
    uint64_t* d_stats = nullptr;
    uint64_t* d_plain = nullptr;
    MixRow* h_mix = nullptr;
    uint64_t* h_stats = nullptr;  // [2][3 Rcap]
    uint64_t* h_plain = nullptr;  // [2][3 Rcap]
    cudaEvent_t stats_done[2] = {nullptr, nullptr};
    RowInfo* mx_rows[2] = {nullptr, nullptr};
    uint16_t* mx_d16[2] = {nullptr, nullptr};
    int64_t* mx_tmax[2] = {nullptr, nullptr};
    alignas(128) CUtensorMap mx_ts_d16[2];
    uint64_t bytes = 0;
    // Per-op device time (CUDA events on the batch stream) when profiling is on.
    bool profiling = false;
    std::vector<cudaEvent_t> ev_pool;
    std::vector<std::pair<int, int>> ev_pending;  // (op, index of the begin event; end = +1)
    std::vector<double> op_ms;
    std::vector<uint64_t> op_launches, op_flops;
    alignas(128) CUtensorMap tm_a;
    alignas(128) CUtensorMap tm_att;
    alignas(128) CUtensorMap tm_g;
    alignas(128) CUtensorMap tm_q;   // qkv rows, 64-byte boxes (attention Q)
    alignas(128) CUtensorMap tm_k;   // the keys cache
    alignas(128) CUtensorMap tm_v;   // the transposed values cache
    alignas(128) CUtensorMap ts_delta;  // epilogue stores: the residual delta (i32)
    alignas(128) CUtensorMap ts_g;      // the GELU output (i8)
    // The QKV epilogue's stores (32 x 32-byte boxes): q into the qkv buffer, keys and transposed
    // values into the caches; kv_tma when they exist (the cache layouts allow them).
    alignas(128) CUtensorMap ts_q, ts_kc, ts_vt;
    bool kv_tma = false;
    alignas(128) CUtensorMap ts_d16;    // the logit distances (u16) of the mixed op
    alignas(128) CUtensorMap ts_d16c;   // the logit distances (u16) of a chunk
    alignas(128) CUtensorMap tm_a_lo;   // version 2: the lo plane of the ln_f output
    alignas(128) CUtensorMap tm_g_lo;   // version 2: the lo plane of the GELU output

    ~hs_batch() {
        if (model && cudaSetDevice(model->dev->ordinal) != cudaSuccess) cudaGetLastError();
        for (cudaEvent_t e : ev_pool) cudaEventDestroy(e);
        if (stream) cudaStreamDestroy(stream);
        for (void* p : owned) cudaFree(p);
        for (cudaEvent_t e : pass_done)
            if (e) cudaEventDestroy(e);
        if (h_rows_base) cudaFreeHost(h_rows_base);
        if (h_intervals_base) cudaFreeHost(h_intervals_base);
        if (h_groups_base) cudaFreeHost(h_groups_base);
        if (h_rowlist_base) cudaFreeHost(h_rowlist_base);
        for (cudaEvent_t e : stats_done)
            if (e) cudaEventDestroy(e);
        if (h_mix) cudaFreeHost(h_mix);
        if (h_stats) cudaFreeHost(h_stats);
        if (h_plain) cudaFreeHost(h_plain);
    }
};

namespace {

// The ops of one pass, for the profile (the reference's CudaBatch::profile op names).
// OP_PASS spans a whole pass (first kernel to the coder, gaps included); it is not a launch.
enum Op { OP_EMBED, OP_LN, OP_GEMM_QKV, OP_KV, OP_ATTN, OP_GEMM_PROJ, OP_GEMM_FC, OP_GEMM_MLP, OP_GEMM_LOGITS,
          OP_CODER, OP_DECODER, OP_PASS, OP_COUNT };
const char* OP_NAMES[OP_COUNT] = {"embed", "layernorm", "gemm_qkv", "kv_store", "attention", "gemm_proj",
                                  "gemm_fc", "gemm_mlp", "gemm_logits", "coder", "decoder", "pass"};

// Kernel launches of this process (the bench reports the launches of its timed region). Several
// host threads launch at once in the multi-GPU fold and unfold, so the count is atomic.
std::atomic<unsigned long long> g_launches{0};

struct ProfScope {
    hs_batch* b;
    int op;
    int idx = -1;
    ProfScope(hs_batch* b_, int op_, uint64_t flops) : b(b_), op(op_) {
        if (op != OP_PASS) g_launches.fetch_add(1, std::memory_order_relaxed);
        if (!b->profiling) return;
        b->op_launches[op]++;
        b->op_flops[op] += flops;
        size_t need = 2 * (b->ev_pending.size() + 1);
        while (b->ev_pool.size() < need) {
            cudaEvent_t e;
            cudaEventCreate(&e);
            b->ev_pool.push_back(e);
        }
        idx = (int)(2 * b->ev_pending.size());
        b->ev_pending.push_back({op, idx});
        cudaEventRecord(b->ev_pool[idx], b->stream);
    }
    ~ProfScope() {
        if (idx >= 0) cudaEventRecord(b->ev_pool[idx + 1], b->stream);
    }
};

// After a synchronised pass: add the elapsed time of every recorded op.
void prof_collect(hs_batch* b) {
    for (auto& p : b->ev_pending) {
        float ms = 0;
        if (cudaEventElapsedTime(&ms, b->ev_pool[p.second], b->ev_pool[p.second + 1]) == cudaSuccess)
            b->op_ms[p.first] += ms;
    }
    b->ev_pending.clear();
}

int upload_linear(hs_model* m, const hsm::Linear& L, DevLinear& D, bool wide_in = false) {
    int N = L.rows, K = L.cols;
    int Np = round_up(N, TILE_N), Kp = round_up(K, TILE_K);
    std::vector<int8_t> w((size_t)Np * Kp, 0);
    for (int n = 0; n < N; n++) memcpy(&w[(size_t)n * Kp], &L.w[(size_t)n * K], K);
    std::vector<int32_t> b(Np, 0), mm(Np, 0);
    std::copy(L.b.begin(), L.b.end(), b.begin());
    std::copy(L.rs.m.begin(), L.rs.m.end(), mm.begin());
    int8_t* dw;
    int32_t *db, *dm;
    int rc = upload(&dw, w.data(), w.size(), m->owned);
    if (!rc) rc = upload(&db, b.data(), b.size(), m->owned);
    if (!rc) rc = upload(&dm, mm.data(), mm.size(), m->owned);
    if (rc) return rc;
    D.ld = LinearDev{dw, N, K, Np, Kp, db, dm, (int)L.rs.s};
    // An i8 activation is at most 128 in magnitude, so |acc_n| <= 128 * sum_k |W[n][k]| and an
    // output is at most (|acc_n| * |m_n| + |b_n * m_n| + 2^(s-1)) / 2^s + 1 in magnitude.
    D.small = false;
    const int s = (int)L.rs.s;
    if (s >= 0 && s <= 62) {
        unsigned __int128 worst = 0;
        for (int n = 0; n < N; n++) {
            uint64_t l1 = 0;
            for (int k = 0; k < K; k++) l1 += (uint64_t)std::abs((int)L.w[(size_t)n * K + k]);
            const uint64_t am = (uint64_t)std::abs((int64_t)L.rs.m[n]);
            const uint64_t ab = (uint64_t)std::abs((int64_t)L.b[n]);
            const unsigned __int128 t = (unsigned __int128)128 * l1 * am + (unsigned __int128)ab * am;
            worst = t > worst ? t : worst;
        }
        worst += s > 0 ? (unsigned __int128)1 << (s - 1) : 0;
        D.small = (worst >> s) + 1 < ((unsigned __int128)1 << 30);
    }
    m->weight_bytes += w.size() + 8 * (size_t)Np;
    if (wide_in) {
        std::vector<int64_t> ws(Np, 0);
        for (int n = 0; n < N; n++)
            for (int k = 0; k < K; k++) ws[n] += L.w[(size_t)n * K + k];
        if ((rc = upload(&D.wsum, ws.data(), ws.size(), m->owned))) return rc;
        if ((rc = make_tmap(m->dev, &D.tm128, dw, Np, Kp, 128))) return rc;
    }
    if ((rc = make_tmap(m->dev, &D.tm64, dw, Np, Kp, 64))) return rc;
    return make_tmap(m->dev, &D.tm, dw, Np, Kp, TILE_N);
}

int upload_ln(hs_model* m, const hsm::LayerNormP& L, LnDev& D) {
    int16_t* g;
    int32_t* b;
    int rc = upload(&g, L.g.data(), L.g.size(), m->owned);
    if (!rc) rc = upload(&b, L.b.data(), L.b.size(), m->owned);
    if (rc) return rc;
    D = LnDev{g, b, L.m, (int)L.s, (int)L.beta_frac};
    return HS_OK;
}

// The forward pass of R rows (the rows are in b->d_rows): the layers and ln_f into b->a; the
// LM head is logits() (run_logits_chunks or the mixed pass).
int forward(hs_batch* b, int R) {
    hs_model* m = b->model;
    const ModelConsts& c = m->c;
    cudaStream_t st = b->stream;
    {
        ProfScope p(b, OP_EMBED, 0);
        launch_embed(b->d_rows, R, m->wte, c.Dp, m->em, m->es, m->wpe, m->pm, m->ps, c.d, b->x, st);
    }
    // The attention work of this pass: 2 * 2 * hd * (pos + 1) per row and head (q.k and p.v).
    uint64_t attn_ops = 0;
    for (int r = 0; r < R; r++) attn_ops += 4ULL * c.d * (b->h_rows[r].pos + 1);
    // tmA2: the lo plane of i16 activations (version 2); then the tiles are 128 x 128.
    auto gemm = [&](int op, int mode, const int8_t* A, int lda, const CUtensorMap* tmA, const DevLinear& W,
                    EpiArgs e, const CUtensorMap* tmC, const CUtensorMap* tmA2 = nullptr) {
        ProfScope p(b, op, 2ULL * R * W.ld.N * W.ld.K);
        e.small = W.small ? 1 : 0;
        e.wsum = W.wsum;
        const bool qkv_tma = mode == EPI_QKV && b->kv_tma;
        e.kv_tma = qkv_tma ? 1 : 0;
        if (m->use_tc)
            launch_gemm_tc(mode, tmA, tmA2 ? &W.tm128 : &W.tm, qkv_tma ? &b->ts_q : tmC, R, W.ld.Np, W.ld.Kp, e,
                           m->dev->num_sms, m->dev->d_err, st, tmA2, qkv_tma ? &b->ts_kc : nullptr,
                           qkv_tma ? &b->ts_vt : nullptr, &W.tm64);
        else
            launch_gemm_simple(mode, A, lda, R, W.ld, e, st);
    };
    for (int l = 0; l < c.L; l++) {
        const LayerDev& Ld = m->layers[l];
        const DevLinear& qkv = *m->lins[4 * l];
        const DevLinear& proj = *m->lins[4 * l + 1];
        const DevLinear& fc = *m->lins[4 * l + 2];
        const DevLinear& mlp = *m->lins[4 * l + 3];
        {
            // The residual of the previous layer's MLP joins x here (none before layer 0).
            ProfScope p(b, OP_LN, 0);
            launch_resid_layernorm(b->x, l == 0 ? nullptr : b->dbuf, R, c.d, Ld.ln1, c.ln_k, c.ln_j, c.ln_eps, b->a,
                                   c.Dp, st);
        }
        EpiArgs e{};
        e.R = R;
        e.N = 3 * c.d;
        e.b = qkv.ld.b;
        e.m = qkv.ld.m;
        e.s = qkv.ld.s;
        e.out8 = b->qkv;
        e.ldo = c.QKVp;
        // q to the qkv buffer, k and v straight into the caches of this layer (no separate store).
        e.rows = b->d_rows;
        e.kc = b->kc;
        e.vc = b->vc;
        e.L = c.L;
        e.layer = l;
        e.H = c.H;
        e.hd = c.hd;
        e.n_ctx = c.n_ctx;
        e.d = c.d;
        // On tensor cores the v of rows outside transposed runs (decode rows, ragged groups) is
        // staged row-major in the attention output buffer, free until attention writes it, and
        // placed by the scatter kernel over all SMs.
        if (m->use_tc) {
            e.vstage = b->att;
            e.ldv = c.Dp;
        }
        gemm(OP_GEMM_QKV, EPI_QKV, b->a, c.Dp, &b->tm_a, qkv, e, nullptr);
        if (m->use_tc && b->v_scatter) {
            ProfScope p(b, OP_KV, 0);
            launch_v_scatter(b->d_rows, R, b->att, c.Dp, c.d, c.H, c.hd, c.L, l, c.n_ctx, b->vc, st);
        }
        {
            ProfScope p(b, OP_ATTN, attn_ops);
            launch_attention_tc(&b->tm_q, &b->tm_k, &b->tm_v, b->d_groups, b->n_groups, c.L, l, c.H, c.n_ctx,
                                Ld.score_m, Ld.score_s, Ld.out_m, Ld.out_s, m->attn_exp, m->attn_len, c.softmax_p,
                                b->att, c.Dp, b->attn_scr, b->attn_scr_slots, m->dev->d_err, st);
            const int* rl = b->n_groups ? b->d_rowlist : nullptr;
            const int nr = b->n_groups ? b->n_rowlist : R;
            if (m->attn_dec)
                launch_attention_dec(b->d_rows, rl, nr, b->qkv, c.QKVp, b->kc, b->vc, c.L, l, c.H, c.n_ctx, Ld.score_m,
                                     Ld.score_s, Ld.out_m, Ld.out_s, m->attn_exp, m->attn_len, c.softmax_p, b->att,
                                     c.Dp, st);
            else
                launch_attention(b->d_rows, R, rl, nr, b->qkv, c.QKVp, b->kc, b->vc, c.L, l, c.H, c.hd, c.n_ctx, c.d,
                                 Ld.score_m, Ld.score_s, Ld.out_m, Ld.out_s, m->attn_exp, m->attn_len, c.softmax_p,
                                 b->att, c.Dp, st);
        }
        e = EpiArgs{};
        e.R = R;
        e.N = c.d;
        e.b = proj.ld.b;
        e.m = proj.ld.m;
        e.s = proj.ld.s;
        e.out32 = b->dbuf;
        e.ldo = c.d;
        gemm(OP_GEMM_PROJ, EPI_DELTA, b->att, c.Dp, &b->tm_att, proj, e, &b->ts_delta);
        {
            ProfScope p(b, OP_LN, 0);
            launch_resid_layernorm(b->x, b->dbuf, R, c.d, Ld.ln2, c.ln_k, c.ln_j, c.ln_eps, b->a, c.Dp, st);
        }
        e = EpiArgs{};
        e.R = R;
        e.N = c.f;
        e.b = fc.ld.b;
        e.m = fc.ld.m;
        e.s = fc.ld.s;
        e.out8 = b->g;
        e.ldo = c.Fp;
        e.gelu = Ld.gelu;
        e.gelu_off = Ld.gelu_off;
        const bool gwide = Ld.gelu16 != nullptr;
        if (gwide) {
            e.gelu16 = Ld.gelu16;
            e.out8_lo = b->g_lo;
            gemm(OP_GEMM_FC, EPI_GELU16, b->a, c.Dp, &b->tm_a, fc, e, nullptr);
        } else {
            gemm(OP_GEMM_FC, EPI_GELU, b->a, c.Dp, &b->tm_a, fc, e, &b->ts_g);
        }
        e = EpiArgs{};
        e.R = R;
        e.N = c.d;
        e.b = mlp.ld.b;
        e.m = mlp.ld.m;
        e.s = mlp.ld.s;
        e.out32 = b->dbuf;
        e.ldo = c.d;
        gemm(OP_GEMM_MLP, EPI_DELTA, b->g, c.Fp, &b->tm_g, mlp, e, &b->ts_delta, gwide ? &b->tm_g_lo : nullptr);
    }
    {
        ProfScope p(b, OP_LN, 0);
        launch_resid_layernorm(b->x, b->dbuf, R, c.d, m->lnf, c.ln_k, c.ln_j, c.ln_eps, b->a, c.Dp, st,
                               c.lnf_wide ? b->a_lo : nullptr);
    }
    return HS_OK;
}

// The LM head of rows r0 .. r0 + n - 1 of the pass (ln_f output in b->a): the logit distances
// and tile maxima of those rows into rows 0 .. n - 1 of d16 / tmax (store map ts).
void logits(hs_batch* b, int r0, int n, uint16_t* d16, int64_t* tmax, const CUtensorMap* ts) {
    hs_model* m = b->model;
    const ModelConsts& c = m->c;
    const DevLinear& lmh = *m->lins[4 * c.L];
    ProfScope p(b, OP_GEMM_LOGITS, 2ULL * n * lmh.ld.N * lmh.ld.K);
    EpiArgs e{};
    e.R = n;
    e.N = c.V;
    e.m = lmh.ld.m;
    e.s = lmh.ld.s;
    e.d16 = d16;
    e.ldd = c.Vp;
    e.tmax = tmax;
    e.ldt = c.VT;
    e.last = m->logits_len - 1;
    e.small = lmh.small ? 1 : 0;
    e.wsum = lmh.wsum;
    e.a_row0 = r0;
    if (m->use_tc)
        launch_gemm_tc(EPI_LOGITS, &b->tm_a, c.lnf_wide ? &lmh.tm128 : &lmh.tm, ts, n, lmh.ld.Np, lmh.ld.Kp, e,
                       m->dev->num_sms, m->dev->d_err, b->stream, c.lnf_wide ? &b->tm_a_lo : nullptr);
    else
        launch_gemm_simple(EPI_LOGITS, b->a + (size_t)r0 * c.Dp, c.Dp, n, lmh.ld, e, b->stream);
}

// The LM head and the op on its logits, chunk by chunk (lchunk rows): op(r0, n) runs on the
// chunk's d16c / tmaxc right after its GEMM, while they are in L2.
template <class Op>
void run_logits_chunks(hs_batch* b, int R, Op op) {
    for (int r0 = 0; r0 < R; r0 += b->lchunk) {
        const int n = std::min(b->lchunk, R - r0);
        logits(b, r0, n, b->d16c, b->tmaxc, &b->ts_d16c);
        op(r0, n);
    }
}

int check_device_error(hs_batch* b) {
    hs_dev* dev = b->model->dev;
    CK(cudaStreamSynchronize(b->stream));
    CK(cudaGetLastError());
    int herr = 0;
    CK(cudaMemcpy(&herr, dev->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr != 0) {
        cudaMemset(dev->d_err, 0, sizeof(int));
        if (herr == ERR_CODER_DIVISION)
            return fail(HS_CUDA, "the coder op's frequency division did not converge (code " + std::to_string(herr) + ")");
        if (herr == ERR_ATTN_SCRATCH)
            return fail(HS_CUDA, "the prefill attention ran a CTA without a scratch slot (code " +
                                     std::to_string(herr) + ")");
        return fail(HS_CUDA, "a kernel wait timed out (code " + std::to_string(herr) + ")");
    }
    return HS_OK;
}

// The prefill groups of a pass (the reference's attention row groups, batch.rs att_groups): runs
// of rows of one slot at consecutive positions, cut at 128 rows. Runs of at least
// ATTN_TC_MIN_ROWS rows go to the tensor-core kernel; the other rows to the CUDA-core kernel.
void plan_groups(hs_batch* b, int R) {
    b->n_groups = 0;
    b->n_rowlist = 0;
    if (!b->model->attn_tc) return;
    int r = 0;
    while (r < R) {
        const RowInfo& f = b->h_rows[r];
        int e = r + 1;
        while (e < R && e - r < 128 && b->h_rows[e].slot == f.slot && b->h_rows[e].pos == f.pos + (uint32_t)(e - r)) e++;
        if (e - r >= ATTN_TC_MIN_ROWS) {
            b->h_groups[b->n_groups++] = AttnGroup{(uint32_t)r, (uint32_t)(e - r), f.slot, f.pos};
        } else {
            for (int q = r; q < e; q++) b->h_rowlist[b->n_rowlist++] = q;
        }
        r = e;
    }
    // Longest first: a group's work grows with its last key, and the CTAs start in launch order.
    std::stable_sort(b->h_groups, b->h_groups + b->n_groups, [](const AttnGroup& x, const AttnGroup& y) {
        return x.pos0 + x.count > y.pos0 + y.count;
    });
}

struct PlanRow {
    uint32_t slot, token, pos;
    long input;  // -1: a restart row
};

// batch/plan.rs:60-120: the passes of a call, with the restart rows of a full context. The
// positions and histories change in copies; the caller commits them after the passes ran.
// The stream states and kept contexts of the slots that a call touches, committed with the
// positions (batch/plan.rs:68-116).
// The stream states of a call, committed only when every pass ran: a copy of each slot's state
// (slot-indexed, so that an input costs no look-up) and the contexts saved by restarts.
struct StreamPlan {
    std::vector<StreamSt> st;
    std::unordered_map<uint32_t, std::vector<uint32_t>> prev;
};

// The passes of a call (crates/hardshell-cuda/src/batch/plan.rs:60-120), made as the call runs
// them: advance(want) takes inputs until `want` passes are complete or the inputs end, so the
// host plans pass k + 1 while the GPU runs pass k. A pass is cut at max_rows rows and before a
// context restart of a slot already in it. The positions, histories and stream states are
// copies, committed only when every pass ran. The passes are a deque, so a pass stays where it
// is while later ones are added.
struct Planner {
    const hs_batch* b;
    const uint32_t* slots;
    const uint32_t* tokens;
    const uint32_t n;
    uint32_t i = 0;
    const int n_ctx, k;
    const uint32_t eot;
    std::deque<std::vector<PlanRow>> passes;
    std::vector<int> pos;
    std::vector<uint32_t>& hist;
    StreamPlan sp;
    std::vector<char> in_pass;
    std::vector<PlanRow> cur;
    bool done = false;

    Planner(const hs_batch* b_, const uint32_t* slots_, const uint32_t* tokens_, uint32_t n_,
            std::vector<uint32_t>& hist_work)
        : b(b_), slots(slots_), tokens(tokens_), n(n_), n_ctx(b_->model->c.n_ctx),
          k(std::min<int>(b_->overlap, b_->model->c.n_ctx - 2)), eot(b_->model->eot), pos(b_->pos), hist(hist_work),
          in_pass(b_->slots, 0) {
        hist.assign(b->hist.begin(), b->hist.end());  // into a buffer kept by the batch: no new pages
        sp.st = b->streams;
        cur.reserve(row_reserve());
    }
    size_t row_reserve() const { return std::min<size_t>((size_t)b->max_rows, (size_t)n + 64); }
    void flush() {
        if (!cur.empty()) {
            passes.push_back(std::move(cur));
            cur = std::vector<PlanRow>();
            cur.reserve(row_reserve());
        }
        std::fill(in_pass.begin(), in_pass.end(), 0);
    }
    void push(PlanRow r) {
        if ((int)cur.size() >= b->max_rows) flush();
        in_pass[r.slot] = 1;
        cur.push_back(r);
    }
    void advance(size_t want) {
        while (!done && passes.size() < want) {
            if (i == n) {
                flush();
                done = true;
                break;
            }
            const uint32_t s = slots[i];
            uint32_t* h = &hist[(size_t)s * n_ctx];
            int at = pos[s];
            StreamSt& ss = sp.st[s];
            if (at >= n_ctx) {
                if (in_pass[s]) flush();
                // The full context before the restart, for a truncation (stream.rs restart).
                sp.prev[s].assign(h, h + n_ctx);
                ss.prev_first = (int32_t)ss.first;
                ss.first = (uint32_t)k + 1;
                ss.written = (uint32_t)k + 1;
                memmove(h + 1, h + (n_ctx - k), sizeof(uint32_t) * k);
                h[0] = eot;
                for (int q = 0; q <= k; q++) push({s, h[q], (uint32_t)q, -1});
                at = k + 1;
            }
            h[at] = tokens[i];
            push({s, tokens[i], (uint32_t)at, (long)i});
            pos[s] = at + 1;
            ss.len++;
            ss.written = std::max(ss.written, (uint32_t)at + 1);
            i++;
        }
    }
};

// The host side of a mixed call (crates/hardshell-cuda/src/batch/mixed.rs:25-35 Mixing): the
// table word of each input, the host mixer, and for run_coded_dual the intervals of GPT-2 alone.
struct MixCall {
    const uint32_t* tables;
    hs_mixer_fn fn;
    void* user;
    hs_interval* plain;
};

// The mix record of a row with a predicted token p (crates/hardshell-cuda/src/mixed.rs:60-90
// mix_record, the rule 5 values of taco_match::Mixer apply): R = max(W - w[p], 1), m = 2^16 - q,
// k = max(0, bitlen(R) + 16 - 62), and w'[p] = max(1, (R * q) >> k) (below 2^62).
int mix_record(const hs_mix_stats& st, uint32_t p, uint32_t q, MixRow* out) {
    if (q == 0 || q >= (1u << 16)) return fail(HS_UNSUPPORTED, "the mixer probability q must be in 1..=65535");
    if (st.predicted > st.total) return fail(HS_UNSUPPORTED, "the weight of the prediction is above the sum");
    const uint64_t r = std::max<uint64_t>(st.total - st.predicted, 1);
    const int bitlen = 64 - __builtin_clzll(r);
    const uint32_t k = bitlen + 16 > 62 ? (uint32_t)(bitlen + 16 - 62) : 0;
    const unsigned __int128 x = ((unsigned __int128)r * q) >> k;
    *out = MixRow{p, k, (1u << 16) - q, 0, std::max<uint64_t>((uint64_t)x, 1), 0};
    return HS_OK;
}

// Runs the passes; with `out` the coder answers (3 u64 per input), else the weights. With `mix`
// the answers are those of the mixed coder op, pass by pass with the host mixer between the
// statistics and the mixed table.
int run(hs_batch* b, const uint32_t* slots, const uint32_t* tokens, const uint32_t* kinds, const uint64_t* values,
        uint32_t n, uint32_t bits, hs_interval* out, uint64_t* wout, const MixCall* mix = nullptr) {
    hs_model* m = b->model;
    const ModelConsts& c = m->c;
    for (uint32_t i = 0; i < n; i++) {
        if (slots[i] >= (uint32_t)b->slots)
            return fail(HS_BAD_SLOT, "slot " + std::to_string(slots[i]) + " is not valid in a batch of " +
                                         std::to_string(b->slots) + " slots");
        if (tokens[i] >= (uint32_t)c.V)
            return fail(HS_TOKEN_RANGE, "token " + std::to_string(tokens[i]) + " is not in the vocabulary of " +
                                            std::to_string(c.V) + " tokens");
    }
    if (out) {
        if (bits == 0 || bits > 32 || (uint64_t)c.V > (1ULL << bits))
            return fail(HS_UNSUPPORTED, "freq_bits must be in 1..=32 and 2^freq_bits >= vocab");
        for (uint32_t i = 0; i < n; i++) {
            bool ok = (kinds[i] == 0 && values[i] < (uint64_t)c.V) || (kinds[i] == 1 && values[i] < (1ULL << bits));
            if (!ok) return fail(HS_UNSUPPORTED, "a coder token or target is out of range");
        }
    }
    if (mix) {
        for (uint32_t i = 0; i < n; i++) {
            const uint32_t t = mix->tables[i];
            if (t >= (uint32_t)c.V && t != MIX_NONE && t != MIX_PLAIN)
                return fail(HS_UNSUPPORTED, "a predicted token is out of range");
        }
    }
    int rc = set_device(m->dev);
    if (rc) return rc;
    // An earlier failed API call of this thread (already reported to its caller) leaves its code
    // behind; clear it, so that the launch checks below report only this call's own errors. A
    // device fault is sticky and still shows.
    cudaGetLastError();
    if (mix && !b->d_mix) {
        // The buffers of the mixed coder op, made on the first mixed call: the second half of the
        // row table and of the logits (with its store map), the mix records, the statistics.
        const size_t Rc = (size_t)b->Rcap;
        if ((rc = dalloc(&b->d16, Rc * c.Vp, b->owned)) || (rc = dalloc(&b->tmax, Rc * c.VT, b->owned)) ||
            (rc = make_store_tmap(m->dev, &b->ts_d16, b->d16, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (int)Rc, c.V, c.Vp,
                                  128)))
            return rc;
        b->bytes += Rc * (2 * (size_t)c.Vp + 8 * (size_t)c.VT);
        b->mx_rows[0] = b->d_rows;
        b->mx_d16[0] = b->d16;
        b->mx_tmax[0] = b->tmax;
        b->mx_ts_d16[0] = b->ts_d16;
        if ((rc = dalloc(&b->mx_rows[1], Rc, b->owned)) || (rc = dalloc(&b->mx_d16[1], Rc * c.Vp, b->owned)) ||
            (rc = dalloc(&b->mx_tmax[1], Rc * c.VT, b->owned)) ||
            (rc = make_store_tmap(m->dev, &b->mx_ts_d16[1], b->mx_d16[1], CU_TENSOR_MAP_DATA_TYPE_UINT16, 2,
                                  (int)Rc, c.V, c.Vp, 128)) ||
            (rc = dalloc(&b->d_mix, Rc, b->owned)) || (rc = dalloc(&b->d_stats, 3 * Rc, b->owned)) ||
            (rc = dalloc(&b->d_plain, 3 * Rc, b->owned)))
            return rc;
        b->bytes += Rc * (sizeof(RowInfo) + 2 * (size_t)c.Vp + 8 * (size_t)c.VT + sizeof(MixRow) + 48);
        CK(cudaMallocHost(&b->h_mix, sizeof(MixRow) * 4 * Rc));
        CK(cudaMallocHost(&b->h_stats, sizeof(uint64_t) * 6 * Rc));
        CK(cudaMallocHost(&b->h_plain, sizeof(uint64_t) * 6 * Rc));
        for (cudaEvent_t& e : b->stats_done) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    }
    // The batch's own buffers are current again when the call ends, however it ends.
    struct MixHalfRestore {
        hs_batch* b;
        ~MixHalfRestore() {
            if (!b->mx_rows[0]) return;
            b->d_rows = b->mx_rows[0];
            b->d16 = b->mx_d16[0];
            b->tmax = b->mx_tmax[0];
            b->ts_d16 = b->mx_ts_d16[0];
        }
    } mix_restore{b};
    auto use_mix_half = [&](size_t k) {
        const int h = (int)(k & 1);
        b->d_rows = b->mx_rows[h];
        b->d16 = b->mx_d16[h];
        b->tmax = b->mx_tmax[h];
        b->ts_d16 = b->mx_ts_d16[h];
    };
    if (wout && !b->weights) {
        // The weights buffer of run_weights: made on the first use (vocab u64 per row).
        if ((rc = dalloc(&b->weights, (size_t)b->Rcap * c.V, b->owned))) return rc;
        b->bytes += (uint64_t)b->Rcap * c.V * 8;
    }
    Planner plan(b, slots, tokens, n, b->hist_work);
    auto& passes = plan.passes;
    // Coder answers: pass k uses half k & 1 of the host buffers, and the host prepares pass k + 1
    // while the GPU runs pass k. Before a half is filled again (pass k + 2), the answers of the
    // pass that used it are copied out. The device buffers are reused in stream order.
    auto use_half = [&](size_t k) {
        const size_t h = k & 1, Rc = (size_t)b->Rcap;
        b->h_rows = b->h_rows_base + h * Rc;
        b->h_groups = b->h_groups_base + h * Rc;
        b->h_rowlist = b->h_rowlist_base + h * Rc;
        b->h_intervals = b->h_intervals_base + h * 3 * Rc;
    };
    auto answers_out = [&](size_t k) -> int {
        CK(cudaEventSynchronize(b->pass_done[k & 1]));
        const uint64_t* hi = b->h_intervals_base + (k & 1) * 3 * (size_t)b->Rcap;
        const auto& pass = passes[k];
        for (size_t r = 0; r < pass.size(); r++) {
            long in = pass[r].input;
            if (in < 0) continue;
            hs_interval& iv = out[in];
            iv.symbol = (uint32_t)hi[3 * r];
            iv.start = hi[3 * r + 1];
            iv.freq = hi[3 * r + 2];
            iv.is_last = iv.symbol + 1 == (uint32_t)c.V;
            iv.reserved = 0;
        }
        return HS_OK;
    };
    auto plain_out = [&](size_t k) {
        const uint64_t* hp = b->h_plain + (k & 1) * 3 * (size_t)b->Rcap;
        const auto& pass = passes[k];
        for (size_t r = 0; r < pass.size(); r++) {
            long in = pass[r].input;
            if (in < 0) continue;
            hs_interval& iv = mix->plain[in];
            iv.symbol = (uint32_t)hp[3 * r];
            iv.start = hp[3 * r + 1];
            iv.freq = hp[3 * r + 2];
            iv.is_last = iv.symbol + 1 == (uint32_t)c.V;
            iv.reserved = 0;
        }
    };
    // The second half of mixed pass j (batch/mixed.rs:145-180 mix_pass), after the forward pass of
    // pass j + 1 is in the stream: the host mixer for each input of pass j with a predicted token,
    // in input order, on the statistics read back; the mix records up; the coder of GPT-2 alone
    // (run_coded_dual) and the mixed coder on the logits of pass j (half j & 1).
    auto finish = [&](size_t j) -> int {
        const auto& pass = passes[j];
        const int R = (int)pass.size();
        const size_t h = j & 1, Rc = (size_t)b->Rcap;
        CK(cudaEventSynchronize(b->stats_done[h]));
        const uint64_t* st = b->h_stats + h * 3 * Rc;
        MixRow* rec = b->h_mix + (2 + h) * Rc;
        for (int r = 0; r < R; r++) {
            const long in = pass[r].input;
            const uint32_t t = in >= 0 ? mix->tables[in] : MIX_NONE;
            rec[r] = MixRow{t, 0, 0, 0, 0, 0};
            if (in < 0 || t >= (uint32_t)c.V) continue;
            const hs_mix_stats ms{st[3 * r], st[3 * r + 1], (uint32_t)st[3 * r + 2], 0};
            const uint32_t q = mix->fn(mix->user, (uint32_t)in, &ms);
            if ((rc = mix_record(ms, t, q, &rec[r]))) return rc;
        }
        // The answers of pass j - 2 left before this pass's read back reuses their half (their
        // copy is ahead of the statistics of pass j in the stream, so this does not wait).
        if (j >= 2) {
            if ((rc = answers_out(j - 2))) return rc;
            if (mix->plain) plain_out(j - 2);
        }
        ProfScope pass_scope(b, OP_PASS, 0);
        CK(cudaMemcpyAsync(b->d_mix, rec, sizeof(MixRow) * R, cudaMemcpyHostToDevice, b->stream));
        {
            ProfScope p(b, OP_CODER, 0);
            if (mix->plain)
                launch_coder(b->mx_d16[h], c.Vp, b->mx_tmax[h], c.VT, c.tsh, R, c.V, m->logits_exp, m->logits_len,
                             m->logits_head, bits, b->mx_rows[h], b->d_plain, m->dev->d_err, b->stream);
            launch_coder_mix(b->mx_d16[h], c.Vp, b->mx_tmax[h], c.VT, c.tsh, R, c.V, m->logits_exp, m->logits_len,
                             m->logits_head, bits, b->mx_rows[h], b->d_mix, 1, b->intervals, m->dev->d_err,
                             b->stream);
        }
        if (mix->plain)
            CK(cudaMemcpyAsync(b->h_plain + h * 3 * Rc, b->d_plain, sizeof(uint64_t) * 3 * R, cudaMemcpyDeviceToHost,
                               b->stream));
        CK(cudaMemcpyAsync(b->h_intervals_base + h * 3 * Rc, b->intervals, sizeof(uint64_t) * 3 * R,
                           cudaMemcpyDeviceToHost, b->stream));
        CK(cudaEventRecord(b->pass_done[h], b->stream));
        return HS_OK;
    };
    for (size_t k = 0;; k++) {
        plan.advance(k + 1);  // pass k (planned while the GPU runs pass k - 1)
        if (k >= passes.size()) break;
        const auto& pass = passes[k];
        if (out && !mix && k >= 2 && (rc = answers_out(k - 2))) return rc;
        use_half(k);
        if (mix) use_mix_half(k);
        int R = (int)pass.size();
        for (int r = 0; r < R; r++) {
            const PlanRow& p = pass[r];
            RowInfo ri{p.slot, p.token, p.pos, 0, 0};
            if (out && p.input >= 0) {
                ri.kind = kinds[p.input];
                ri.value = values[p.input];
            }
            b->h_rows[r] = ri;
        }
        CK(cudaMemcpyAsync(b->d_rows, b->h_rows, sizeof(RowInfo) * R, cudaMemcpyHostToDevice, b->stream));
        plan_groups(b, R);
        b->v_scatter = false;
        for (int r0 = 0; r0 < R && !b->v_scatter; r0 += 32)
            b->v_scatter = !vt_run_host(b->h_rows, r0, R, b->model->c.n_ctx);
        if (b->n_groups) {
            CK(cudaMemcpyAsync(b->d_groups, b->h_groups, sizeof(AttnGroup) * b->n_groups, cudaMemcpyHostToDevice,
                               b->stream));
            if (b->n_rowlist)
                CK(cudaMemcpyAsync(b->d_rowlist, b->h_rowlist, sizeof(int) * b->n_rowlist, cudaMemcpyHostToDevice,
                                   b->stream));
        }
        std::unique_ptr<ProfScope> pass_scope(new ProfScope(b, OP_PASS, (uint64_t)R));
        rc = forward(b, R);
        if (rc) return rc;
        if (out && mix) {
            logits(b, 0, R, b->d16, b->tmax, &b->ts_d16);
            // The first half of a mixed pass: the statistics of its rows, read back into half k & 1;
            // then the second half of the previous pass.
            MixRow* pw = b->h_mix + (k & 1) * (size_t)b->Rcap;
            for (int r = 0; r < R; r++) {
                const long in = pass[r].input;
                pw[r] = MixRow{in >= 0 ? mix->tables[in] : MIX_NONE, 0, 0, 0, 0, 0};
            }
            CK(cudaMemcpyAsync(b->d_mix, pw, sizeof(MixRow) * R, cudaMemcpyHostToDevice, b->stream));
            {
                ProfScope p(b, OP_CODER, 0);
                launch_coder_mix(b->d16, c.Vp, b->tmax, c.VT, c.tsh, R, c.V, m->logits_exp, m->logits_len,
                                 m->logits_head, bits, b->d_rows, b->d_mix, 0, b->d_stats, m->dev->d_err,
                                 b->stream);
            }
            pass_scope.reset();
            CK(cudaMemcpyAsync(b->h_stats + (k & 1) * 3 * (size_t)b->Rcap, b->d_stats, sizeof(uint64_t) * 3 * R,
                               cudaMemcpyDeviceToHost, b->stream));
            CK(cudaEventRecord(b->stats_done[k & 1], b->stream));
            if (k >= 1 && (rc = finish(k - 1))) return rc;
        } else if (out) {
            run_logits_chunks(b, R, [&](int r0, int nr) {
                ProfScope p(b, OP_CODER, 0);
                launch_coder(b->d16c, c.Vp, b->tmaxc, c.VT, c.tsh, nr, c.V, m->logits_exp, m->logits_len,
                             m->logits_head, bits, b->d_rows + r0, b->intervals + 3 * (size_t)r0, m->dev->d_err,
                             b->stream);
            });
            pass_scope.reset();
            CK(cudaMemcpyAsync(b->h_intervals, b->intervals, sizeof(uint64_t) * 3 * R, cudaMemcpyDeviceToHost,
                               b->stream));
            CK(cudaEventRecord(b->pass_done[k & 1], b->stream));
        } else {
            run_logits_chunks(b, R, [&](int r0, int nr) {
                ProfScope p(b, OP_CODER, 0);
                launch_weights(b->d16c, c.Vp, b->tmaxc, c.VT, c.tsh, nr, c.V, m->logits_exp, m->logits_len,
                               b->weights + (size_t)r0 * c.V, b->stream);
            });
            pass_scope.reset();
            // The weights of this pass leave before the next pass overwrites them.
            rc = check_device_error(b);
            if (rc) return rc;
            for (int r = 0; r < R; r++) {
                long in = pass[r].input;
                if (in < 0) continue;
                CK(cudaMemcpy(wout + (size_t)in * c.V, b->weights + (size_t)r * c.V, sizeof(uint64_t) * c.V,
                              cudaMemcpyDeviceToHost));
            }
        }
    }
    if (out && mix && !passes.empty() && (rc = finish(passes.size() - 1))) return rc;
    rc = check_device_error(b);
    if (rc) return rc;
    if (b->profiling) prof_collect(b);
    if (out) {
        for (size_t k = passes.size() >= 2 ? passes.size() - 2 : 0; k < passes.size(); k++) {
            if ((rc = answers_out(k))) return rc;
            if (mix && mix->plain) plain_out(k);
        }
    }
    // Every pass ran: commit the positions and histories (batch/plan.rs:120 commit).
    b->pos = plan.pos;
    b->hist.swap(b->hist_work);
    b->streams.swap(plan.sp.st);
    for (auto& kv : plan.sp.prev) b->prev[kv.first] = std::move(kv.second);
    return HS_OK;
}

// hs_batch_decode_blocks: n coded blocks unfolded at once, the decoder of each on the device
// (hs_decode.cu). Block i runs in slot slots[i] from position 0, takes EOT as its first input
// and every decoded symbol as the next one (crates/taco/src/gpu_unfold.rs:100-160). The blocks
// are ordered by token count, longest first, so the blocks still running at a step are a prefix
// of that order. A step where no running block needs a context restart is enqueued without a
// host wait: the rows come from the decoder states (k_dec_begin), then the forward pass, the
// coder op and the interval check (k_dec_end). A step with a restart takes the host path of
// run_coded with the targets read back, after the histories of the slots are brought up to date.
int decode_blocks(hs_batch* b, uint32_t n, const uint32_t* slots, const uint8_t* payload, uint64_t payload_len,
                  const uint64_t* offsets, const uint64_t* lengths, const uint32_t* counts, uint32_t bits,
                  uint32_t* tokens_out, uint64_t tokens_cap, const uint64_t* token_offsets, uint32_t* status) {
    hs_model* m = b->model;
    const ModelConsts& c = m->c;
    if (n == 0) return HS_OK;
    if (bits == 0 || bits > 32 || (uint64_t)c.V > (1ULL << bits))
        return fail(HS_UNSUPPORTED, "freq_bits must be in 1..=32 and 2^freq_bits >= vocab");
    if (n > (uint32_t)b->max_rows) return fail(HS_UNSUPPORTED, "more blocks than the batch's max_rows");
    std::vector<char> seen(b->slots, 0);
    uint64_t total = 0;
    for (uint32_t i = 0; i < n; i++) {
        if (slots[i] >= (uint32_t)b->slots)
            return fail(HS_BAD_SLOT, "slot " + std::to_string(slots[i]) + " is not valid in a batch of " +
                                         std::to_string(b->slots) + " slots");
        if (seen[slots[i]]) return fail(HS_BAD_ARGUMENT, "two blocks in one slot");
        seen[slots[i]] = 1;
        if (offsets[i] > payload_len || lengths[i] > payload_len - offsets[i])
            return fail(HS_LENGTH_MISMATCH, "a block lies outside the payload");
        if (token_offsets[i] > tokens_cap || counts[i] > tokens_cap - token_offsets[i])
            return fail(HS_LENGTH_MISMATCH, "a block's tokens lie outside the output");
        total += counts[i];
    }
    int rc = set_device(m->dev);
    if (rc) return rc;
    cudaGetLastError();
    cudaStream_t st = b->stream;
    const int n_ctx = c.n_ctx;
    std::vector<uint32_t> order(n);
    for (uint32_t i = 0; i < n; i++) order[i] = i;
    std::stable_sort(order.begin(), order.end(), [&](uint32_t x, uint32_t y) { return counts[x] > counts[y]; });
    // Per-call device buffers, in block order (`order`).
    std::vector<void*> owned;
    struct Guard {
        std::vector<void*>& o;
        ~Guard() {
            for (void* p : o) cudaFree(p);
        }
    } guard{owned};
    std::vector<uint64_t> h_off(n), h_len(n), h_oo(n);
    std::vector<uint32_t> h_cnt(n), h_slot(n), h_pos(n, 0);
    uint64_t acc = 0;
    for (uint32_t k = 0; k < n; k++) {
        const uint32_t i = order[k];
        h_off[k] = offsets[i];
        h_len[k] = lengths[i];
        h_cnt[k] = counts[i];
        h_slot[k] = slots[i];
        h_oo[k] = acc;
        acc += counts[i];
    }
    uint8_t* d_payload = nullptr;
    uint64_t *d_off = nullptr, *d_len = nullptr, *d_oo = nullptr, *d_tg = nullptr, *d_iv = nullptr;
    uint32_t *d_cnt = nullptr, *d_slot = nullptr, *d_pos = nullptr, *d_prev = nullptr, *d_out = nullptr,
             *d_gather = nullptr, *d_status = nullptr;
    DecState* d_st = nullptr;
    if ((rc = upload(&d_payload, payload, payload_len, owned)) || (rc = upload(&d_off, h_off.data(), n, owned)) ||
        (rc = upload(&d_len, h_len.data(), n, owned)) || (rc = upload(&d_oo, h_oo.data(), n, owned)) ||
        (rc = upload(&d_cnt, h_cnt.data(), n, owned)) || (rc = upload(&d_slot, h_slot.data(), n, owned)) ||
        (rc = dalloc(&d_pos, n, owned)) || (rc = dalloc(&d_prev, n, owned)) || (rc = dalloc(&d_out, total, owned)) ||
        (rc = dalloc(&d_tg, n, owned)) || (rc = dalloc(&d_iv, 3 * (size_t)n, owned)) ||
        (rc = dalloc(&d_status, n, owned)) || (rc = dalloc(&d_st, n, owned)))
        return rc;
    launch_dec_init(d_st, d_payload, d_off, d_len, d_prev, m->eot, (int)n, st);
    for (uint32_t k = 0; k < n; k++) {
        b->pos[h_slot[k]] = 0;
        b->streams[h_slot[k]] = StreamSt{};
        std::fill(b->hist.begin() + (size_t)h_slot[k] * n_ctx, b->hist.begin() + (size_t)(h_slot[k] + 1) * n_ctx, 0u);
    }
    // The steps since the last host sync run at positions h_pos[k] + (step - s_sync); sync_hist
    // reads their symbols back and writes the inputs of those rows into the histories.
    uint32_t s_sync = 0;
    std::vector<uint32_t> last_sym(n, m->eot);  // the input of the block's next row
    std::vector<uint32_t> h_gather;
    auto live_at = [&](uint32_t step) {
        uint32_t L = 0;
        while (L < n && h_cnt[L] > step) L++;
        return L;
    };
    auto sync_hist = [&](uint32_t step) -> int {
        if (step <= s_sync) return HS_OK;
        const uint32_t L = live_at(s_sync), w = step - s_sync;
        if (L == 0) return HS_OK;
        if (!d_gather || h_gather.size() < (size_t)L * w) {
            h_gather.assign((size_t)L * w, 0);
            int r2 = dalloc(&d_gather, (size_t)L * w, owned);
            if (r2) return r2;
        }
        launch_dec_gather(d_out, d_oo, d_cnt, (int)L, s_sync, step, d_gather, st);
        CK(cudaMemcpyAsync(h_gather.data(), d_gather, sizeof(uint32_t) * L * w, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        for (uint32_t k = 0; k < L; k++) {
            uint32_t* h = &b->hist[(size_t)h_slot[k] * n_ctx];
            const uint32_t e = std::min(step, h_cnt[k]);
            StreamSt& ss = b->streams[h_slot[k]];
            for (uint32_t s2 = s_sync; s2 < e; s2++) {
                const uint32_t p2 = h_pos[k] + (s2 - s_sync);
                h[p2] = last_sym[k];
                last_sym[k] = h_gather[(size_t)k * w + (s2 - s_sync)];
                ss.len++;
                ss.written = std::max(ss.written, p2 + 1);
            }
            b->pos[h_slot[k]] = (int)(h_pos[k] + (e - s_sync));
            h_pos[k] = (uint32_t)b->pos[h_slot[k]];
        }
        s_sync = step;
        return HS_OK;
    };
    const uint32_t S = h_cnt[0];
    bool upload_pos = true;
    for (uint32_t step = 0; step < S; step++) {
        const uint32_t L = live_at(step);
        bool restart = false;
        for (uint32_t k = 0; k < L && !restart; k++) restart = h_pos[k] + (step - s_sync) >= (uint32_t)n_ctx;
        if (!restart) {
            if (upload_pos) {
                CK(cudaMemcpyAsync(d_pos, h_pos.data(), sizeof(uint32_t) * n, cudaMemcpyHostToDevice, st));
                upload_pos = false;
            }
            {
                ProfScope p(b, OP_DECODER, 0);
                launch_dec_begin(d_st, (int)L, d_slot, d_pos, step - s_sync, d_prev, bits, b->d_rows, st);
            }
            b->n_groups = 0;
            b->n_rowlist = 0;
            b->v_scatter = true;
            for (uint32_t k = 0; k < L; k++) b->h_rows[k].pos = h_pos[k] + (step - s_sync);  // host statistics only
            {
                std::unique_ptr<ProfScope> pass_scope(new ProfScope(b, OP_PASS, (uint64_t)L));
                rc = forward(b, (int)L);
                if (rc) return rc;
                run_logits_chunks(b, (int)L, [&](int r0, int nr) {
                    ProfScope p(b, OP_CODER, 0);
                    launch_coder(b->d16c, c.Vp, b->tmaxc, c.VT, c.tsh, nr, c.V, m->logits_exp, m->logits_len,
                                 m->logits_head, bits, b->d_rows + r0, b->intervals + 3 * (size_t)r0, m->dev->d_err,
                                 st);
                });
            }
            {
                ProfScope p(b, OP_DECODER, 0);
                launch_dec_end(d_st, (int)L, b->intervals, bits, (uint32_t)c.V, d_payload, d_prev, d_out, d_oo, step, st);
            }
            if (b->profiling) {
                // Keep the event pool bounded: collect the profile of the enqueued steps now and then.
                if ((step & 63) == 63) {
                    if ((rc = check_device_error(b))) return rc;
                    prof_collect(b);
                }
            }
            continue;
        }
        // A restart step: bring the histories up to date, then run it through run_coded.
        if ((rc = check_device_error(b)) || (rc = sync_hist(step))) return rc;
        launch_dec_targets(d_st, (int)L, bits, d_tg, st);
        std::vector<uint64_t> tg(L);
        CK(cudaMemcpyAsync(tg.data(), d_tg, sizeof(uint64_t) * L, cudaMemcpyDeviceToHost, st));
        CK(cudaStreamSynchronize(st));
        std::vector<uint32_t> in_slot(h_slot.begin(), h_slot.begin() + L), in_tok(last_sym.begin(), last_sym.begin() + L),
            kinds(L, 1);
        std::vector<hs_interval> ivs(L);
        if ((rc = run(b, in_slot.data(), in_tok.data(), kinds.data(), tg.data(), L, bits, ivs.data(), nullptr)))
            return rc;
        std::vector<uint64_t> h_iv(3 * (size_t)L);
        for (uint32_t k = 0; k < L; k++) {
            h_iv[3 * k] = ivs[k].symbol;
            h_iv[3 * k + 1] = ivs[k].start;
            h_iv[3 * k + 2] = ivs[k].freq;
            last_sym[k] = ivs[k].symbol;
            h_pos[k] = (uint32_t)b->pos[h_slot[k]];
        }
        CK(cudaMemcpyAsync(d_iv, h_iv.data(), sizeof(uint64_t) * 3 * L, cudaMemcpyHostToDevice, st));
        launch_dec_end(d_st, (int)L, d_iv, bits, (uint32_t)c.V, d_payload, d_prev, d_out, d_oo, step, st);
        CK(cudaStreamSynchronize(st));  // the host copies of h_iv and h_pos stay valid until here
        s_sync = step + 1;
        upload_pos = true;
    }
    if ((rc = check_device_error(b)) || (rc = sync_hist(S))) return rc;
    if (b->profiling) prof_collect(b);
    std::vector<uint32_t> all(total), fl(n);
    launch_dec_status(d_st, (int)n, d_status, st);
    if (total) CK(cudaMemcpyAsync(all.data(), d_out, sizeof(uint32_t) * total, cudaMemcpyDeviceToHost, st));
    CK(cudaMemcpyAsync(fl.data(), d_status, sizeof(uint32_t) * n, cudaMemcpyDeviceToHost, st));
    CK(cudaStreamSynchronize(st));
    for (uint32_t k = 0; k < n; k++) {
        const uint32_t i = order[k];
        memcpy(tokens_out + token_offsets[i], all.data() + h_oo[k], sizeof(uint32_t) * counts[i]);
        if (status) status[i] = fl[k];
    }
    return HS_OK;
}

// Rows with no coder answer (the rebuild rows of a truncation): passes of at most max_rows rows,
// each synchronised before the host buffers are filled again.
int run_rows(hs_batch* b, const std::vector<PlanRow>& rows) {
    for (size_t r0 = 0; r0 < rows.size(); r0 += (size_t)b->max_rows) {
        const int R = (int)std::min(rows.size() - r0, (size_t)b->max_rows);
        for (int r = 0; r < R; r++) {
            const PlanRow& p = rows[r0 + r];
            b->h_rows[r] = RowInfo{p.slot, p.token, p.pos, 0, 0};
        }
        CK(cudaMemcpyAsync(b->d_rows, b->h_rows, sizeof(RowInfo) * R, cudaMemcpyHostToDevice, b->stream));
        plan_groups(b, R);
        b->v_scatter = false;
        for (int q0 = 0; q0 < R && !b->v_scatter; q0 += 32) b->v_scatter = !vt_run_host(b->h_rows, q0, R, b->model->c.n_ctx);
        if (b->n_groups) {
            CK(cudaMemcpyAsync(b->d_groups, b->h_groups, sizeof(AttnGroup) * b->n_groups, cudaMemcpyHostToDevice,
                               b->stream));
            if (b->n_rowlist)
                CK(cudaMemcpyAsync(b->d_rowlist, b->h_rowlist, sizeof(int) * b->n_rowlist, cudaMemcpyHostToDevice,
                                   b->stream));
        }
        int rc = forward(b, R);
        if (rc || (rc = check_device_error(b))) return rc;
    }
    return HS_OK;
}

// CudaBatch::truncate (crates/hardshell-cuda/src/batch/stream.rs:46-77) with the rules of
// StreamState::plan_truncate / commit_truncate (crates/hardshell/src/gpt2/stream.rs:118-160):
// inside the current context only the position moves back; before the last restart the slot
// takes the kept history of the old context and runs its rows again at the positions that the
// new context wrote (the rebuilt cache entries are the old ones, bit for bit); before the restart
// before the last one it is an error. The slot does not change on an error.
int truncate_slot(hs_batch* b, uint32_t slot, uint64_t len) {
    if (slot >= (uint32_t)b->slots)
        return fail(HS_BAD_SLOT, "slot " + std::to_string(slot) + " is not valid in a batch of " +
                                     std::to_string(b->slots) + " slots");
    const int n_ctx = b->model->c.n_ctx;
    StreamSt ss = b->streams[slot];
    const uint64_t pos = (uint64_t)b->pos[slot];
    auto bad = [&]() {
        return fail(HS_MODEL, "BadTruncate: length " + std::to_string(len) + " for a stream of " +
                                  std::to_string(ss.len) + " inputs");
    };
    if (len > ss.len) return bad();
    const uint64_t drop = ss.len - len;
    const uint64_t here = pos > ss.first ? pos - ss.first : 0;
    if (drop <= here) {
        b->streams[slot].len = (uint32_t)len;
        b->pos[slot] = (int)(pos - drop);
        return HS_OK;
    }
    if (ss.prev_first < 0) return bad();
    const uint64_t before = drop - here;
    if (before > (uint64_t)(n_ctx - ss.prev_first)) return bad();
    const uint32_t target = (uint32_t)(n_ctx - before);
    const std::vector<uint32_t>& old = b->prev[slot];
    if (old.size() != (size_t)n_ctx) return bad();
    int rc = set_device(b->model->dev);
    if (rc) return rc;
    cudaGetLastError();
    std::vector<PlanRow> rows;
    for (uint32_t p = 0; p < std::min(target, ss.written); p++) rows.push_back({slot, old[p], p, -1});
    if ((rc = run_rows(b, rows))) return rc;
    std::copy(old.begin(), old.end(), b->hist.begin() + (size_t)slot * n_ctx);
    StreamSt& st = b->streams[slot];
    st.len = (uint32_t)len;
    st.first = (uint32_t)ss.prev_first;
    st.prev_first = -1;
    st.written = (uint32_t)n_ctx;
    b->pos[slot] = (int)target;
    return HS_OK;
}

}  // namespace

extern "C" {

// Helpers for the other translation units of the library (not in the public header).
int hs_internal_tmap(hs_dev* dev, void* tm, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    return make_tmap(dev, (CUtensorMap*)tm, base, rows, cols, box_rows);
}
int hs_internal_dev_info(hs_dev* dev, int* num_sms, int** d_err) {
    int rc = set_device(dev);
    if (rc) return rc;
    *num_sms = dev->num_sms;
    *d_err = dev->d_err;
    return HS_OK;
}
int hs_internal_fail(int code, const char* msg) { return fail(code, msg); }

int hs_last_error(char* buf, size_t cap) {
    if (!buf || cap == 0) return HS_BAD_ARGUMENT;
    size_t n = std::min(cap - 1, g_err.size());
    memcpy(buf, g_err.data(), n);
    buf[n] = 0;
    return HS_OK;
}

// HS_FAIL_OPEN: a comma-separated list of ordinals whose open fails on the host, before any CUDA
// call (a test of the callers' fallback without a fault of any GPU).
static bool open_fails_by_request(int ordinal) {
    const char* v = getenv("HS_FAIL_OPEN");
    if (!v) return false;
    for (const char* p = v; *p;) {
        char* end = nullptr;
        const long o = strtol(p, &end, 10);
        if (end == p) break;
        if (o == ordinal) return true;
        p = *end == ',' ? end + 1 : end;
        if (*end != ',') break;
    }
    return false;
}

int hs_open(int ordinal, hs_dev** out) {
    if (!out) return fail(HS_BAD_ARGUMENT, "null output");
    *out = nullptr;
    if (open_fails_by_request(ordinal))
        return fail(HS_NO_DEVICE, "device " + std::to_string(ordinal) + " refused by HS_FAIL_OPEN");
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess || count == 0)
        return fail(HS_NO_DEVICE, std::string("no CUDA device: ") + (e != cudaSuccess ? cudaGetErrorString(e) : "none"));
    if (ordinal < 0 || ordinal >= count) return fail(HS_NO_DEVICE, "no CUDA device " + std::to_string(ordinal));
    cudaDeviceProp prop;
    CK(cudaGetDeviceProperties(&prop, ordinal));
    if (prop.major < 10)
        return fail(HS_UNSUPPORTED, "the kernels are sm_100a: the GPU needs compute capability 10.0");
    CK(cudaSetDevice(ordinal));
    auto d = std::make_unique<hs_dev>();
    d->ordinal = ordinal;
    d->num_sms = prop.multiProcessorCount;
    d->name = prop.name;
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    CK(cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q));
    if (!fn || q != cudaDriverEntryPointSuccess) return fail(HS_CUDA, "cuTensorMapEncodeTiled is not available");
    d->encode = (EncodeTiledFn)fn;
    CK(cudaMalloc(&d->d_err, sizeof(int)));
    CK(cudaMemset(d->d_err, 0, sizeof(int)));
    CK(configure_core_kernels());
    CK(configure_tc_kernels());
    CK(configure_attn_tc());
    *out = d.release();
    return HS_OK;
}

void hs_dev_free(hs_dev* d) {
    if (!d) return;
    if (cudaSetDevice(d->ordinal) != cudaSuccess) cudaGetLastError();
    if (d->d_err) cudaFree(d->d_err);
    delete d;
}

int hs_mem_info(hs_dev* d, uint64_t* free_bytes, uint64_t* total_bytes) {
    if (!d || !free_bytes || !total_bytes) return fail(HS_BAD_ARGUMENT, "null argument");
    int rc = set_device(d);
    if (rc) return rc;
    size_t f = 0, t = 0;
    CK(cudaMemGetInfo(&f, &t));
    *free_bytes = f;
    *total_bytes = t;
    return HS_OK;
}

int hs_dev_name(hs_dev* d, char* buf, size_t cap) {
    if (!d || !buf || cap == 0) return fail(HS_BAD_ARGUMENT, "null argument");
    size_t n = std::min(cap - 1, d->name.size());
    memcpy(buf, d->name.data(), n);
    buf[n] = 0;
    return HS_OK;
}

int hs_model_check(const uint8_t* file, size_t len, hs_model_info* out) {
    if (!file || !out) return fail(HS_BAD_ARGUMENT, "null argument");
    hsm::Model M;
    std::string err;
    if (!hsm::load_model(file, len, M, err)) return fail(HS_MODEL, "the model file is not valid: " + err);
    memset(out, 0, sizeof(*out));
    out->n_layer = (uint32_t)M.n_layer;
    out->n_head = (uint32_t)M.n_head;
    out->d_model = (uint32_t)M.d_model;
    out->d_ff = (uint32_t)M.d_ff;
    out->vocab = (uint32_t)M.vocab;
    out->n_ctx = (uint32_t)M.n_ctx;
    out->eot_token = M.eot;
    out->version = M.version;
    out->cache_bytes_per_slot = 2ULL * M.n_layer * M.n_ctx * M.d_model;
    sha256(file, len, out->hash);
    return HS_OK;
}

int hs_model_load(hs_dev* dev, const uint8_t* file, size_t len, hs_model** out) {
    if (!dev || !file || !out) return fail(HS_BAD_ARGUMENT, "null argument");
    *out = nullptr;
    hsm::Model M;
    std::string err;
    if (!hsm::load_model(file, len, M, err)) return fail(HS_MODEL, "the model file is not valid: " + err);
    if (M.is_wide() && !use_tc_default())
        return fail(HS_UNSUPPORTED, "the CUDA-core GEMM path (HS_GEMM=simple) does not run the i16 activations "
                                    "of hsm format version 2");
    if (M.vocab < 2) return fail(HS_UNSUPPORTED, "the vocabulary needs at least 2 tokens");
    if (M.vocab > MAX_CODER_VOCAB)
        return fail(HS_UNSUPPORTED, "the coder op of this backend takes at most 65536 tokens");
    if ((int)M.logits_exp.size() > MAX_LOGIT_TABLE)
        return fail(HS_UNSUPPORTED, "the logit table is longer than 16384 entries");
    if (M.n_ctx > MAX_ATTN_CTX) return fail(HS_UNSUPPORTED, "the context is longer than 8192 positions");
    if (M.head_dim > 1024) return fail(HS_UNSUPPORTED, "the head width is more than 1024");
    int rc = set_device(dev);
    if (rc) return rc;
    auto m = std::make_unique<hs_model>();
    m->dev = dev;
    m->use_tc = use_tc_default();
    m->attn_tc = use_attn_tc_default() && attention_tc_supported(M.head_dim, M.n_ctx, (int)M.attn_exp.size());
    m->attn_dec = use_attn_tc_default() &&
                  attention_dec_supported(M.head_dim, M.n_ctx, round_up(3 * M.d_model, 16), (int)M.attn_exp.size());
    sha256(file, len, m->hash);
    m->eot = M.eot;
    m->version = M.version;
    ModelConsts& c = m->c;
    c.d = M.d_model;
    c.f = M.d_ff;
    c.V = M.vocab;
    c.H = M.n_head;
    c.hd = M.head_dim;
    c.L = M.n_layer;
    c.n_ctx = M.n_ctx;
    c.Dp = round_up(c.d, TILE_K);
    c.Fp = round_up(c.f, TILE_K);
    c.QKVp = round_up(3 * c.d, 16);
    c.Vp = round_up(c.V, TILE_N);
    c.lnf_wide = M.ln_f_bits == 16;
    c.tsh = c.lnf_wide ? 6 : 7;  // LOGIT_TILE_WIDE or LOGIT_TILE columns per logits tile
    c.VT = (c.V + (1 << c.tsh) - 1) >> c.tsh;
    c.ln_k = (int)M.ln_k;
    c.ln_j = (int)M.ln_j;
    c.ln_eps = M.ln_eps;
    c.softmax_p = (int)M.softmax_p;
    // The token embedding doubles as the LM head: [Vp, Dp], rows padded with zeros.
    hsm::Linear lm;
    lm.rows = c.V;
    lm.cols = c.d;
    lm.w = M.wte;
    lm.b.assign(c.V, 0);
    lm.rs = M.logit;
    for (int l = 0; l < c.L; l++) {
        const hsm::Block& B = M.blocks[l];
        LayerDev Ld{};
        for (const hsm::Linear* L : {&B.c_attn, &B.c_proj, &B.c_fc, &B.mlp_proj}) {
            m->lins.emplace_back(new DevLinear());
            // mlp_proj reads the i16 GELU output of a version 2 layer (two planes).
            rc = upload_linear(m.get(), *L, *m->lins.back(), L == &B.mlp_proj && B.gelu_wide);
            if (rc) return rc;
        }
        Ld.qkv = m->lins[4 * l]->ld;
        Ld.proj = m->lins[4 * l + 1]->ld;
        Ld.fc = m->lins[4 * l + 2]->ld;
        Ld.mlp = m->lins[4 * l + 3]->ld;
        if ((rc = upload_ln(m.get(), B.ln_1, Ld.ln1)) || (rc = upload_ln(m.get(), B.ln_2, Ld.ln2))) return rc;
        Ld.score_m = B.score_m;
        Ld.score_s = (int)B.score_s;
        Ld.out_m = B.out_m;
        Ld.out_s = (int)B.out_s;
        int8_t* gl;
        if ((rc = upload(&gl, B.gelu8.data(), B.gelu8.size(), m->owned))) return rc;
        Ld.gelu = gl;
        Ld.gelu16 = nullptr;
        if (B.gelu_wide) {
            int16_t* g16;
            if ((rc = upload(&g16, B.gelu16.data(), B.gelu16.size(), m->owned))) return rc;
            Ld.gelu16 = g16;
        }
        Ld.gelu_off = (int)B.gelu_offset;
        m->layers.push_back(Ld);
    }
    m->lins.emplace_back(new DevLinear());
    if ((rc = upload_linear(m.get(), lm, *m->lins.back(), c.lnf_wide))) return rc;
    m->wte = const_cast<int8_t*>(m->lins.back()->ld.w);
    m->es = (int)M.embed.s;
    m->ls = (int)M.logit.s;
    if ((rc = upload(&m->em, M.embed.m.data(), M.embed.m.size(), m->owned))) return rc;
    m->lm = const_cast<int32_t*>(m->lins.back()->ld.m);
    if ((rc = upload(&m->wpe, M.wpe.data(), M.wpe.size(), m->owned))) return rc;
    if ((rc = upload(&m->pm, M.pos.m.data(), M.pos.m.size(), m->owned))) return rc;
    m->ps = (int)M.pos.s;
    if ((rc = upload_ln(m.get(), M.ln_f, m->lnf))) return rc;
    {
        // Padded to a multiple of 4 entries: the attention kernel copies it in 16-byte units.
        std::vector<int32_t> t(M.attn_exp);
        t.resize((t.size() + 3) & ~(size_t)3, 0);
        if ((rc = upload(&m->attn_exp, t.data(), t.size(), m->owned))) return rc;
    }
    m->attn_len = (int)M.attn_exp.size();
    if ((rc = upload(&m->logits_exp, M.logits_exp.data(), M.logits_exp.size(), m->owned))) return rc;
    m->logits_len = (int)M.logits_exp.size();
    while (m->logits_head + 1 < m->logits_len && M.logits_exp[m->logits_head + 1] == M.logits_exp[0]) m->logits_head++;
    m->weight_bytes += M.wpe.size() + 8 * M.logits_exp.size() + 4 * M.attn_exp.size();
    CK(cudaDeviceSynchronize());
    *out = m.release();
    return HS_OK;
}

void hs_model_free(hs_model* m) { delete m; }

int hs_model_get_info(hs_model* m, hs_model_info* out) {
    if (!m || !out) return fail(HS_BAD_ARGUMENT, "null argument");
    const ModelConsts& c = m->c;
    out->n_layer = c.L;
    out->n_head = c.H;
    out->d_model = c.d;
    out->d_ff = c.f;
    out->vocab = c.V;
    out->n_ctx = c.n_ctx;
    out->eot_token = m->eot;
    out->version = m->version;
    out->cache_bytes_per_slot = 2ULL * c.L * c.n_ctx * c.d;
    out->weight_bytes = m->weight_bytes;
    memcpy(out->hash, m->hash, 32);
    return HS_OK;
}

int hs_batch_new(hs_model* m, uint32_t slots, uint32_t max_rows, hs_batch** out) {
    if (!m || !out) return fail(HS_BAD_ARGUMENT, "null argument");
    *out = nullptr;
    if (slots == 0 || max_rows == 0) return fail(HS_UNSUPPORTED, "a batch needs at least one slot and one row");
    if (max_rows < 2) max_rows = 2;  // a restart needs two rows in one pass
    if (max_rows > (1u << 20)) return fail(HS_UNSUPPORTED, "max_rows is more than 2^20");
    int rc = set_device(m->dev);
    if (rc) return rc;
    auto b = std::make_unique<hs_batch>();
    b->model = m;
    b->slots = (int)slots;
    b->max_rows = (int)max_rows;
    b->Rcap = round_up((int)max_rows, TILE_M);
    const ModelConsts& c = m->c;
    b->pos.assign(slots, 0);
    b->hist.assign((size_t)slots * c.n_ctx, 0);
    b->streams.assign(slots, StreamSt{});
    b->prev.assign(slots, {});
    CK(cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking));
    size_t cache = (size_t)slots * c.L * c.n_ctx * c.d;
    size_t R = b->Rcap;
    if ((rc = dalloc(&b->kc, cache, b->owned)) || (rc = dalloc(&b->vc, cache, b->owned)) ||
        (rc = dalloc(&b->d_rows, R, b->owned)) || (rc = dalloc(&b->x, R * c.d, b->owned)) ||
        (rc = dalloc(&b->a, R * c.Dp, b->owned)) || (rc = dalloc(&b->qkv, R * c.QKVp, b->owned)) ||
        (rc = dalloc(&b->att, R * c.Dp, b->owned)) || (rc = dalloc(&b->g, R * c.Fp, b->owned)) ||
        (rc = dalloc(&b->dbuf, R * c.d, b->owned)) ||
        (rc = dalloc(&b->intervals, 3 * R, b->owned)))
        return rc;
    // The chunk of the LM head: the whole pass by default. Chunks small enough for their
    // distances to stay in L2 (HS_LOGIT_CHUNK rows, a multiple of 128) were measured slower on a
    // B200: at 512, 768 and 1024 rows the fold ran at 6.8, 7.0 and 7.3 MB/s against 8.1 MB/s
    // unchunked, the logits GEMM and the coder paying their start-up and last wave per chunk.
    {
        int ch = (int)R;
        if (const char* v = getenv("HS_LOGIT_CHUNK")) ch = std::max(128, atoi(v) / 128 * 128);
        b->lchunk = (int)std::min<size_t>(R, (size_t)ch);
    }
    const size_t LC = (size_t)b->lchunk;
    if ((rc = dalloc(&b->d16c, LC * c.Vp, b->owned)) || (rc = dalloc(&b->tmaxc, LC * c.VT, b->owned))) return rc;
    if ((rc = dalloc(&b->d_groups, R, b->owned)) || (rc = dalloc(&b->d_rowlist, R, b->owned))) return rc;
    bool gelu_wide = false;
    for (const LayerDev& Ld : m->layers) gelu_wide |= Ld.gelu16 != nullptr;
    if (c.lnf_wide) {
        if ((rc = dalloc(&b->a_lo, R * c.Dp, b->owned))) return rc;
        if ((rc = make_tmap(m->dev, &b->tm_a_lo, b->a_lo, R, c.Dp, TILE_M))) return rc;
    }
    if (gelu_wide) {
        if ((rc = dalloc(&b->g_lo, R * c.Fp, b->owned))) return rc;
        if ((rc = make_tmap(m->dev, &b->tm_g_lo, b->g_lo, R, c.Fp, TILE_M))) return rc;
    }
    CK(cudaMallocHost(&b->h_groups_base, sizeof(AttnGroup) * 2 * R));
    CK(cudaMallocHost(&b->h_rowlist_base, sizeof(int) * 2 * R));
    CK(cudaMallocHost(&b->h_rows_base, sizeof(RowInfo) * 2 * R));
    CK(cudaMallocHost(&b->h_intervals_base, sizeof(uint64_t) * 3 * 2 * R));
    for (cudaEvent_t& e : b->pass_done) CK(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
    b->h_groups = b->h_groups_base;
    b->h_rowlist = b->h_rowlist_base;
    b->h_rows = b->h_rows_base;
    b->h_intervals = b->h_intervals_base;
    b->bytes = 2 * cache + R * (sizeof(RowInfo) + 8 * c.d + 2 * c.Dp + c.QKVp + c.Fp + 24 + (c.lnf_wide ? c.Dp : 0) +
                                (gelu_wide ? c.Fp : 0)) +
               LC * (2 * c.Vp + 8 * c.VT);
    if ((rc = make_store_tmap(m->dev, &b->ts_delta, b->dbuf, CU_TENSOR_MAP_DATA_TYPE_INT32, 4, R, c.d, c.d, 128)) ||
        (rc = make_store_tmap(m->dev, &b->ts_g, b->g, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, R, c.f, c.Fp, 32)) ||
        (rc = make_store_tmap(m->dev, &b->ts_d16c, b->d16c, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, (int)LC, c.V, c.Vp,
                              128)))
        return rc;
    if ((rc = make_tmap(m->dev, &b->tm_a, b->a, R, c.Dp, TILE_M)) ||
        (rc = make_tmap(m->dev, &b->tm_att, b->att, R, c.Dp, TILE_M)) ||
        (rc = make_tmap(m->dev, &b->tm_g, b->g, R, c.Fp, TILE_M)))
        return rc;
    if (m->use_tc && (c.n_ctx % 16) == 0 && (c.hd % 32) == 0 && (c.d % 32) == 0 && (c.QKVp % 16) == 0) {
        const uint64_t heads = (uint64_t)slots * c.L * c.H;
        if ((rc = make_store_tmap(m->dev, &b->ts_q, b->qkv, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, R, 3 * c.d, c.QKVp, 32)) ||
            (rc = make_store_tmap(m->dev, &b->ts_kc, b->kc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, heads * c.n_ctx, c.hd,
                                  c.hd, 32)) ||
            (rc = make_store_tmap(m->dev, &b->ts_vt, b->vc, CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, heads * c.hd, c.n_ctx,
                                  c.n_ctx, 32)))
            return rc;
        b->kv_tma = getenv("HS_QKV_TMA") == nullptr || atoi(getenv("HS_QKV_TMA")) != 0;
    }
    if (m->attn_tc) {
        // The prefill attention's scratch (the exp-table index of every key of the rows of one
        // tile, one slot per persistent CTA, one CTA per SM): 256 KB per SM at n_ctx = 1024.
        b->attn_scr_slots = m->dev->num_sms;
        // HS_ATTN_CTAS=<n> caps the persistent grid (a test hook: a few CTAs then run many tiles
        // each, with every length of tile after every other).
        if (const char* v = getenv("HS_ATTN_CTAS")) {
            const int n = atoi(v);
            if (n > 0 && n < b->attn_scr_slots) b->attn_scr_slots = n;
        }
        const size_t scr = attn_scratch_bytes(b->attn_scr_slots, c.n_ctx);
        if ((rc = dalloc(&b->attn_scr, scr, b->owned))) return rc;
        b->bytes += scr;
        uint64_t heads = (uint64_t)slots * c.L * c.H;
        if ((rc = make_tmap(m->dev, &b->tm_q, b->qkv, R, c.QKVp, 128, 64)) ||
            (rc = make_tmap(m->dev, &b->tm_k, b->kc, heads * c.n_ctx, c.hd, 128, 64)) ||
            (rc = make_tmap(m->dev, &b->tm_v, b->vc, heads * c.hd, c.n_ctx, 64, 128)))
            return rc;
    }
    *out = b.release();
    return HS_OK;
}

void hs_batch_free(hs_batch* b) { delete b; }

int hs_batch_set_overlap(hs_batch* b, uint16_t k) {
    if (!b) return fail(HS_BAD_ARGUMENT, "null argument");
    if ((int)k + 2 > b->model->c.n_ctx)
        return fail(HS_INVALID_OVERLAP, "the overlap " + std::to_string(k) + " is more than n_ctx - 2");
    b->overlap = k;
    return HS_OK;
}

int hs_batch_reset(hs_batch* b, uint32_t slot) {
    if (!b) return fail(HS_BAD_ARGUMENT, "null argument");
    if (slot < (uint32_t)b->slots) {
        b->pos[slot] = 0;
        b->streams[slot] = StreamSt{};
    }
    return HS_OK;
}

uint32_t hs_batch_position(hs_batch* b, uint32_t slot) {
    if (!b || slot >= (uint32_t)b->slots) return 0;
    return (uint32_t)b->pos[slot];
}

uint64_t hs_batch_gpu_bytes(hs_batch* b) { return b ? b->bytes : 0; }

int hs_batch_set_profiling(hs_batch* b, int on) {
    if (!b) return fail(HS_BAD_ARGUMENT, "null argument");
    b->profiling = on != 0;
    b->op_ms.assign(OP_COUNT, 0.0);
    b->op_launches.assign(OP_COUNT, 0);
    b->op_flops.assign(OP_COUNT, 0);
    b->ev_pending.clear();
    return HS_OK;
}

int hs_batch_profile(hs_batch* b, hs_op_profile* out, int cap) {
    if (!b || (cap > 0 && !out)) return fail(HS_BAD_ARGUMENT, "null argument");
    if (!b->profiling) return 0;
    int n = 0;
    for (int op = 0; op < OP_COUNT && n < cap; op++) {
        hs_op_profile& p = out[n++];
        memset(&p, 0, sizeof(p));
        strncpy(p.name, OP_NAMES[op], sizeof(p.name) - 1);
        p.ms = b->op_ms[op];
        p.launches = b->op_launches[op];
        p.ops = b->op_flops[op];
    }
    return n;
}

uint64_t hs_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int hs_batch_run_coded(hs_batch* b, const uint32_t* slots, const uint32_t* tokens, const uint32_t* kinds,
                       const uint64_t* values, uint32_t n, uint32_t freq_bits, hs_interval* out) {
    if (!b || (n && (!slots || !tokens || !kinds || !values || !out))) return fail(HS_BAD_ARGUMENT, "null argument");
    return run(b, slots, tokens, kinds, values, n, freq_bits, out, nullptr);
}

int hs_batch_run_coded_mixed(hs_batch* b, const uint32_t* slots, const uint32_t* tokens, const uint32_t* kinds,
                             const uint64_t* values, const uint32_t* tables, uint32_t n, uint32_t freq_bits,
                             hs_mixer_fn mixer, void* user, hs_interval* out) {
    if (!b || !mixer || (n && (!slots || !tokens || !kinds || !values || !tables || !out)))
        return fail(HS_BAD_ARGUMENT, "null argument");
    const MixCall mc{tables, mixer, user, nullptr};
    return run(b, slots, tokens, kinds, values, n, freq_bits, out, nullptr, &mc);
}

int hs_batch_run_coded_dual(hs_batch* b, const uint32_t* slots, const uint32_t* tokens, const uint32_t* coded,
                            const uint32_t* predictions, uint32_t n, uint32_t freq_bits, hs_mixer_fn mixer,
                            void* user, hs_interval* plain_out, hs_interval* mixed_out) {
    if (!b || !mixer || (n && (!slots || !tokens || !coded || !predictions || !plain_out || !mixed_out)))
        return fail(HS_BAD_ARGUMENT, "null argument");
    // batch/mixed.rs prediction_words: a token or none (no plain word).
    for (uint32_t i = 0; i < n; i++)
        if (predictions[i] == MIX_PLAIN) return fail(HS_UNSUPPORTED, "a predicted token is out of range");
    const std::vector<uint32_t> kinds(n, 0);
    const std::vector<uint64_t> values(coded, coded + n);
    const MixCall mc{predictions, mixer, user, plain_out};
    return run(b, slots, tokens, kinds.data(), values.data(), n, freq_bits, mixed_out, nullptr, &mc);
}

int hs_batch_stream_len(hs_batch* b, uint32_t slot, uint64_t* len) {
    if (!b || !len) return fail(HS_BAD_ARGUMENT, "null argument");
    if (slot >= (uint32_t)b->slots)
        return fail(HS_BAD_SLOT, "slot " + std::to_string(slot) + " is not valid in a batch of " +
                                     std::to_string(b->slots) + " slots");
    *len = b->streams[slot].len;
    return HS_OK;
}

int hs_batch_room(hs_batch* b, uint32_t slot, uint64_t* room) {
    if (!b || !room) return fail(HS_BAD_ARGUMENT, "null argument");
    if (slot >= (uint32_t)b->slots)
        return fail(HS_BAD_SLOT, "slot " + std::to_string(slot) + " is not valid in a batch of " +
                                     std::to_string(b->slots) + " slots");
    const int n_ctx = b->model->c.n_ctx, k = std::min<int>(b->overlap, n_ctx - 2), p = b->pos[slot];
    *room = p >= n_ctx ? (uint64_t)std::max(0, n_ctx - k - 1) : (uint64_t)(n_ctx - p);
    return HS_OK;
}

int hs_batch_truncate(hs_batch* b, uint32_t slot, uint64_t len) {
    if (!b) return fail(HS_BAD_ARGUMENT, "null argument");
    return truncate_slot(b, slot, len);
}

int hs_batch_decode_blocks(hs_batch* b, uint32_t n, const uint32_t* slots, const uint8_t* payload,
                           uint64_t payload_len, const uint64_t* offsets, const uint64_t* lengths,
                           const uint32_t* counts, uint32_t freq_bits, uint32_t* tokens_out, uint64_t tokens_cap,
                           const uint64_t* token_offsets, uint32_t* status) {
    if (!b || (n && (!slots || !offsets || !lengths || !counts || !token_offsets || (!payload && payload_len) ||
                     (!tokens_out && tokens_cap))))
        return fail(HS_BAD_ARGUMENT, "null argument");
    return decode_blocks(b, n, slots, payload, payload_len, offsets, lengths, counts, freq_bits, tokens_out, tokens_cap,
                         token_offsets, status);
}

int hs_batch_run_weights(hs_batch* b, const uint32_t* slots, const uint32_t* tokens, uint32_t n, uint64_t* out) {
    if (!b || (n && (!slots || !tokens || !out))) return fail(HS_BAD_ARGUMENT, "null argument");
    return run(b, slots, tokens, nullptr, nullptr, n, 32, nullptr, out);
}

// ---- op-level entry points ----

int hs_op_linear_act(hs_dev* dev, int path, const int8_t* A, const int8_t* W, const int32_t* bias, const int32_t* mult,
                     uint32_t shift, uint32_t M, uint32_t N, uint32_t K, int8_t* out8, int32_t* raw32) {
    if (!dev || !A || !W || (!raw32 && (!bias || !mult || !out8))) return fail(HS_BAD_ARGUMENT, "null argument");
    if (M == 0 || N == 0 || K == 0 || K > 65536) return fail(HS_UNSUPPORTED, "shape out of range");
    int rc = set_device(dev);
    if (rc) return rc;
    std::vector<void*> owned;
    struct Guard {
        std::vector<void*>& o;
        ~Guard() {
            for (void* p : o) cudaFree(p);
        }
    } guard{owned};
    int Mp = round_up((int)M, TILE_M), Np = round_up((int)N, TILE_N), Kp = round_up((int)K, TILE_K);
    std::vector<int8_t> ha((size_t)Mp * Kp, 0), hw((size_t)Np * Kp, 0);
    for (uint32_t r = 0; r < M; r++) memcpy(&ha[(size_t)r * Kp], A + (size_t)r * K, K);
    for (uint32_t n = 0; n < N; n++) memcpy(&hw[(size_t)n * Kp], W + (size_t)n * K, K);
    std::vector<int32_t> hb(Np, 0), hm(Np, 0);
    if (!raw32) {
        std::copy(bias, bias + N, hb.begin());
        std::copy(mult, mult + N, hm.begin());
    }
    int8_t *da, *dw, *dout;
    int32_t *db, *dm, *d32;
    if ((rc = upload(&da, ha.data(), ha.size(), owned)) || (rc = upload(&dw, hw.data(), hw.size(), owned)) ||
        (rc = upload(&db, hb.data(), hb.size(), owned)) || (rc = upload(&dm, hm.data(), hm.size(), owned)) ||
        (rc = dalloc(&dout, (size_t)M * N, owned)) || (rc = dalloc(&d32, (size_t)M * N, owned)))
        return rc;
    LinearDev L{dw, (int)N, (int)K, Np, Kp, db, dm, (int)shift};
    EpiArgs e{};
    e.R = (int)M;
    e.N = (int)N;
    e.b = db;
    e.m = dm;
    e.s = (int)shift;
    e.out8 = dout;
    e.ldo = (int)N;
    e.out32 = d32;
    int mode = raw32 ? EPI_RAW : EPI_ACT;
    cudaStream_t st = 0;
    if (path == 0) {
        if (N % 16 != 0) return fail(HS_UNSUPPORTED, "the tensor-core path needs N % 16 == 0 for aligned stores");
        alignas(128) CUtensorMap ta, tb;
        if ((rc = make_tmap(dev, &ta, da, Mp, Kp, TILE_M)) || (rc = make_tmap(dev, &tb, dw, Np, Kp, TILE_N)))
            return rc;
        launch_gemm_tc(mode, &ta, &tb, nullptr, (int)M, Np, Kp, e, dev->num_sms, dev->d_err, st);
    } else {
        launch_gemm_simple(mode, da, Kp, (int)M, L, e, st);
    }
    CK(cudaGetLastError());
    CK(cudaDeviceSynchronize());
    int herr = 0;
    CK(cudaMemcpy(&herr, dev->d_err, sizeof(int), cudaMemcpyDeviceToHost));
    if (herr) {
        cudaMemset(dev->d_err, 0, sizeof(int));
        if (herr == ERR_CODER_DIVISION)
            return fail(HS_CUDA, "the coder op's frequency division did not converge (code " + std::to_string(herr) + ")");
        return fail(HS_CUDA, "a kernel wait timed out (code " + std::to_string(herr) + ")");
    }
    if (raw32) CK(cudaMemcpy(raw32, d32, sizeof(int32_t) * M * N, cudaMemcpyDeviceToHost));
    else CK(cudaMemcpy(out8, dout, (size_t)M * N, cudaMemcpyDeviceToHost));
    return HS_OK;
}

}  // extern "C"

hs_model* hs::batch_model(hs_batch* b) { return b->model; }
uint32_t hs::batch_slots(const hs_batch* b) { return (uint32_t)b->slots; }
uint32_t hs::batch_max_rows(const hs_batch* b) { return (uint32_t)b->max_rows; }
