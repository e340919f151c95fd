// The fold of the profile text above the C ABI: bytes in, a .taco container out
// (crates/taco/src/fold.rs fold_with and code_segment, codec.rs BlockEncoder, and the container
// writer of crates/taco-format/src/writer.rs). The model's part is hs_batch_run_coded on the GPU;
// the rest is host code: the tokenizer, the zstd frame, the range encoder with the stop rule, the
// choice of the smallest stored form, and the container.
//
// The steps of one fold:
// 1. The input divides into blocks of the block size (the last one shorter).
// 2. On host threads, each block is tokenized (its tokens must join to its bytes) and compressed
//    into one zstd frame (level 19, content size, no checksum, no dictionary id; zstd_block.rs).
// 3. On the GPU, the blocks run in rounds of up to `slots` blocks, one slot each from a fresh
//    context: the inputs EOT, t0 .. t(n-2) with the encode queries t0 .. t(n-1), the context
//    restarting with the overlap K (codec.rs:1-24, the order of the encoder's calls).
// 4. On host threads, each block's intervals go through the range encoder until the payload (the
//    varint token count, then the coder bytes) is sure to reach the bound min(block length, zstd
//    frame length): then the block has no coded form (codec.rs:70-131, the stop rule).
// 5. Each block is stored in its smallest form: raw, then zstd, then coded, ties to the earlier
//    (writer.rs:89 choose_smallest), and the container is written (header version 2).
#include <dlfcn.h>
#include <unistd.h>

#include <algorithm>
#include <functional>
#include <memory>
#include <atomic>
#include <chrono>
#include <condition_variable>
#include <mutex>
#include <cerrno>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <thread>
#include <vector>

#include "hardshell_b200.h"
#include "hs_host.hpp"
#include "sha256.hpp"

namespace {

constexpr uint32_t DEFAULT_BLOCK_SIZE = 16 * 1024;  // crates/taco/src/lib.rs:101
constexpr uint32_t SPREAD_BLOCKS = 64;              // lib.rs:138
constexpr uint32_t SPREAD_MIN_BLOCK = 4 * 1024;     // lib.rs:145
constexpr uint32_t MAX_BLOCK_SIZE = 64u << 20;      // crates/taco-format: the largest block size
constexpr size_t HEADER_LEN = 104;                  // version 2 header
constexpr uint32_t FREQ_BITS = 32;                  // codec.rs:35
constexpr int ZSTD_LEVEL = 19;                      // crates/taco-format/src/zstd_block.rs:23
constexpr uint8_t KIND_RAW = 0, KIND_CODED = 1, KIND_ZSTD = 2;
constexpr uint64_t MAX_BLOCKS = 0xFFFFFFFFull;      // the block count is a u32 (header.rs)
constexpr uint64_t LEN_UNKNOWN = HS_LEN_UNKNOWN;    // a fold input or an unfold container of unknown length

// The blocks of `len` bytes in blocks of `bs` (the last one shorter), with no overflow for any
// length (the reference's block_count is checked arithmetic too).
constexpr uint64_t blocks_of(uint64_t len, uint64_t bs) { return len / bs + (len % bs != 0); }

// ---- zstd, from the system library (opened once) ----

struct Zstd {
    void* lib = nullptr;
    void* (*create)() = nullptr;
    size_t (*free_ctx)(void*) = nullptr;
    size_t (*set_param)(void*, int, int) = nullptr;
    size_t (*compress2)(void*, void*, size_t, const void*, size_t) = nullptr;
    size_t (*bound)(size_t) = nullptr;
    unsigned (*is_error)(size_t) = nullptr;
    unsigned (*version)() = nullptr;
    void* (*dcreate)() = nullptr;
    size_t (*dfree)(void*) = nullptr;
    size_t (*dset_param)(void*, int, int) = nullptr;
    size_t (*decompress)(void*, void*, size_t, const void*, size_t) = nullptr;
    unsigned long long (*content_size)(const void*, size_t) = nullptr;
    size_t (*frame_size)(const void*, size_t) = nullptr;
    bool ok = false;

    Zstd() {
        lib = dlopen("libzstd.so.1", RTLD_NOW | RTLD_LOCAL);
        if (!lib) return;
        create = (void* (*)())dlsym(lib, "ZSTD_createCCtx");
        free_ctx = (size_t(*)(void*))dlsym(lib, "ZSTD_freeCCtx");
        set_param = (size_t(*)(void*, int, int))dlsym(lib, "ZSTD_CCtx_setParameter");
        compress2 = (size_t(*)(void*, void*, size_t, const void*, size_t))dlsym(lib, "ZSTD_compress2");
        bound = (size_t(*)(size_t))dlsym(lib, "ZSTD_compressBound");
        is_error = (unsigned (*)(size_t))dlsym(lib, "ZSTD_isError");
        version = (unsigned (*)())dlsym(lib, "ZSTD_versionNumber");
        dcreate = (void* (*)())dlsym(lib, "ZSTD_createDCtx");
        dfree = (size_t(*)(void*))dlsym(lib, "ZSTD_freeDCtx");
        dset_param = (size_t(*)(void*, int, int))dlsym(lib, "ZSTD_DCtx_setParameter");
        decompress = (size_t(*)(void*, void*, size_t, const void*, size_t))dlsym(lib, "ZSTD_decompressDCtx");
        content_size = (unsigned long long (*)(const void*, size_t))dlsym(lib, "ZSTD_getFrameContentSize");
        frame_size = (size_t(*)(const void*, size_t))dlsym(lib, "ZSTD_findFrameCompressedSize");
        ok = create && free_ctx && set_param && compress2 && bound && is_error && version && dcreate && dfree &&
             dset_param && decompress && content_size && frame_size;
    }
};

const Zstd& zstd() {
    static const Zstd z;
    return z;
}

// compress_zstd (zstd_block.rs:64-79): one frame at level 19 with the content size, no
// checksum and no dictionary id. The parameter ids are those of zstd.h (ZSTD_c_compressionLevel
// 100, ZSTD_c_contentSizeFlag 200, ZSTD_c_checksumFlag 201, ZSTD_c_dictIDFlag 202).
bool compress_zstd(const uint8_t* data, size_t len, std::vector<uint8_t>& out) {
    const Zstd& z = zstd();
    void* cctx = z.create();
    if (!cctx) return false;
    bool ok = true;
    const int params[4][2] = {{100, ZSTD_LEVEL}, {200, 1}, {201, 0}, {202, 0}};
    for (const auto& p : params) ok = ok && !z.is_error(z.set_param(cctx, p[0], p[1]));
    if (ok) {
        out.resize(z.bound(len));
        const size_t n = z.compress2(cctx, out.data(), out.size(), data, len);
        ok = !z.is_error(n);
        out.resize(ok ? n : 0);
    }
    z.free_ctx(cctx);
    return ok;
}

// The bounded decoder of a zstd block (zstd_block.rs): exactly one frame, whose header gives
// the content size, equal to the block's original length; a window of at most 2^23 bytes
// (ZSTD_d_windowLogMax, id 100); the output written into the block's own bytes only.
bool decompress_zstd(const uint8_t* frame, size_t n, uint8_t* out, size_t original_len) {
    const Zstd& z = zstd();
    static const uint8_t magic[4] = {0x28, 0xB5, 0x2F, 0xFD};
    if (n < 4 || memcmp(frame, magic, 4) != 0) return false;
    if (z.content_size(frame, n) != (unsigned long long)original_len) return false;
    const size_t fs = z.frame_size(frame, n);
    if (z.is_error(fs) || fs != n) return false;
    void* dctx = z.dcreate();
    if (!dctx) return false;
    bool ok = !z.is_error(z.dset_param(dctx, 100, 23));
    if (ok) {
        const size_t got = z.decompress(dctx, out, original_len, frame, n);
        ok = !z.is_error(got) && got == original_len;
    }
    z.dfree(dctx);
    return ok;
}

// ---- the range encoder (crates/taco-coder/src/encoder.rs) ----

// A 64-bit window over a 128-bit low with a carry, bytes out with the pending run of 0xFF, and
// the length of the output up to its last non-zero byte (the smallest final length).
struct RangeEncoder {
    unsigned __int128 low = 0;
    uint64_t range = ~0ULL;  // INITIAL_RANGE
    uint8_t cache = 0;
    size_t pending = 0;
    std::vector<uint8_t> out;
    size_t nonzero_len = 0;
    static constexpr uint64_t TOP = 1ULL << 56;

    void shift_low() {
        const uint8_t carry = (uint8_t)((low >> 64) & 1);
        const uint64_t window = (uint64_t)low;
        if (pending == 0 || window < 0xFF00000000000000ULL || carry != 0) {
            if (pending > 0) {
                const uint8_t first = (uint8_t)(cache + carry);
                out.push_back(first);
                if (first != 0) nonzero_len = out.size();
                const uint8_t fill = (uint8_t)(0xFF + carry);
                out.insert(out.end(), pending - 1, fill);
                if (fill != 0 && pending > 1) nonzero_len = out.size();
            }
            cache = (uint8_t)(window >> 56);
            pending = 0;
        }
        pending++;
        low = (unsigned __int128)(window << 8);
    }

    void encode(uint64_t start, uint64_t freq, bool is_last, uint32_t bits) {
        const uint64_t r = range >> bits;
        const uint64_t offset = r * start;
        low += offset;
        range = is_last ? range - offset : r * freq;
        while (range < TOP) {
            range <<= 8;
            shift_low();
        }
    }

    // The shortest tail that keeps the code inside [low, low + range): low rounded up to a
    // multiple of 2^64, or else of 2^56; two more bytes out; trailing zero bytes dropped.
    std::vector<uint8_t> finish() {
        const unsigned __int128 end = low + range;
        for (int k : {64, 56}) {
            const unsigned __int128 mask = ((unsigned __int128)1 << k) - 1;
            const unsigned __int128 v = (low + mask) & ~mask;
            if (v < end) {
                low = v;
                break;
            }
        }
        shift_low();
        shift_low();
        while (!out.empty() && out.back() == 0) out.pop_back();
        return std::move(out);
    }
};

void write_varint(uint64_t v, std::vector<uint8_t>& out) {  // payload.rs:20: LEB128
    while (v >= 0x80) {
        out.push_back((uint8_t)(v | 0x80));
        v >>= 7;
    }
    out.push_back((uint8_t)v);
}

size_t varint_len(uint64_t v) {
    size_t n = 1;
    while (v >= 0x80) {
        v >>= 7;
        n++;
    }
    return n;
}

struct FoldBlock {
    size_t off = 0, len = 0;
    std::vector<uint32_t> tokens;
    std::vector<uint8_t> zstd;
    bool zstd_ok = false;
    uint8_t kind = KIND_RAW;
    std::vector<uint8_t> stored;  // the stored bytes of a zstd or coded block
};

// Runs f(i) for i in [0, n) on up to `threads` host threads.
template <typename F>
void parallel_for(size_t n, unsigned threads, F&& f) {
    threads = std::max(1u, std::min<unsigned>(threads, (unsigned)std::max<size_t>(n, 1)));
    std::atomic<size_t> next{0};
    auto work = [&]() {
        for (size_t i; (i = next.fetch_add(1)) < n;) f(i);
    };
    std::vector<std::thread> pool;
    for (unsigned t = 1; t < threads; t++) pool.emplace_back(work);
    work();
    for (auto& t : pool) t.join();
}

}  // namespace

extern "C" {

uint64_t hs_fold_bound(uint64_t len, uint32_t block_size) {
    // Block size 0: the fold takes the default or, with `spread`, a size down to 4 KiB; the
    // smallest gives the most table entries.
    const uint64_t bs = block_size ? block_size : SPREAD_MIN_BLOCK;
    const uint64_t nb = blocks_of(len, bs);
    if (len > UINT64_MAX - HEADER_LEN || nb > (UINT64_MAX - HEADER_LEN - len) / 5) return UINT64_MAX;
    return HEADER_LEN + 5 * nb + len;
}

}  // extern "C"

namespace {

// A context window of a block: inputs start .. start + count - 1 of the block's token stream.
struct Window {
    size_t block, start, count;
};

// The windows of a fold and the range encoders of its blocks, shared by the GPU threads.
//
// The windows are dealt in waves: window 0 of every block, then window 1 of every block, and so
// on. After each round of a GPU, the encoder of each block takes the intervals of its windows in
// order as they complete (codec.rs BlockEncoder::push_interval), and a block whose encoder stopped
// (its payload reached min(block length, zstd length): codec.rs:70-131, ADR 0007 section 5.2) has
// no later window started, as the reference's GPU fold leaves them in its queue
// (crates/taco/src/gpu_fold.rs:200-204). The container does not depend on that order: a stopped
// block is stored raw or as zstd whatever ran after its stop.
class WindowFeed {
  public:
    WindowFeed(std::vector<Window> windows, std::vector<FoldBlock>& blocks, size_t n_blocks)
        : windows_(std::move(windows)), blocks_(blocks), iv_(windows_.size()), done_(windows_.size(), 0),
          st_(n_blocks), locks_(n_blocks) {
        for (size_t w = 0; w < windows_.size(); w++) {
            BlockState& bs = st_[windows_[w].block];
            if (bs.windows.empty()) {
                const FoldBlock& fb = blocks_[windows_[w].block];
                bs.prefix = varint_len(fb.tokens.size());
                bs.stop = std::min(fb.len, fb.zstd.size());
            }
            bs.windows.push_back(w);
        }
    }

    const std::vector<Window>& windows() const { return windows_; }
    std::vector<hs_interval>& intervals(size_t w) { return iv_[w]; }

    // Up to n windows of blocks whose encoders have not stopped, in wave order.
    void take(size_t n, std::vector<size_t>& out) {
        out.clear();
        std::lock_guard<std::mutex> lk(mu_);
        while (out.size() < n && next_ < order_.size()) {
            const size_t w = order_[next_++];
            if (!st_[windows_[w].block].stopped.load(std::memory_order_relaxed)) out.push_back(w);
        }
    }

    // The windows `ws` completed (their intervals are in intervals(w)): each block's encoder takes
    // the intervals of its next windows in order; a window whose block stopped is dropped.
    void complete(const std::vector<size_t>& ws) {
        for (size_t w : ws) {
            const size_t b = windows_[w].block;
            std::lock_guard<std::mutex> lk(locks_[b]);
            BlockState& bs = st_[b];
            done_[w] = 1;
            while (!bs.stopped && bs.taken < bs.windows.size() && done_[bs.windows[bs.taken]]) {
                const size_t v = bs.windows[bs.taken++];
                for (const hs_interval& iv : iv_[v]) {
                    bs.enc.encode(iv.start, iv.freq, iv.is_last != 0, FREQ_BITS);
                    if (bs.prefix + bs.enc.nonzero_len >= bs.stop) {
                        bs.stopped = true;
                        break;
                    }
                }
                std::vector<hs_interval>().swap(iv_[v]);
            }
            if (bs.stopped) std::vector<hs_interval>().swap(iv_[w]);
        }
    }

    // The wave order of the windows (set once, before the GPU stage).
    void order_by_waves() {
        order_.clear();
        for (size_t k = 0;; k++) {
            bool any = false;
            for (const BlockState& bs : st_)
                if (k < bs.windows.size()) {
                    order_.push_back(bs.windows[k]);
                    any = true;
                }
            if (!any) break;
        }
        next_ = 0;
    }

    // After the GPU stage: the payload of block b (the varint count, then the coder bytes), or
    // false if its encoder stopped. Every window of a live block has been taken.
    bool finish(size_t b, std::vector<uint8_t>& coded) {
        BlockState& bs = st_[b];
        if (bs.windows.empty() || bs.stopped || bs.taken != bs.windows.size()) return false;
        write_varint(blocks_[b].tokens.size(), coded);
        const std::vector<uint8_t> tail = bs.enc.finish();
        coded.insert(coded.end(), tail.begin(), tail.end());
        return true;
    }

    size_t rows_run() const { return rows_run_.load(); }
    void add_rows(size_t n) { rows_run_ += n; }

  private:
    struct BlockState {
        std::vector<size_t> windows;  // this block's windows, in order
        size_t taken = 0;             // windows whose intervals the encoder took
        size_t prefix = 0, stop = 0;
        RangeEncoder enc;
        std::atomic<bool> stopped{false};
    };
    std::vector<Window> windows_;
    std::vector<FoldBlock>& blocks_;
    std::vector<std::vector<hs_interval>> iv_;
    std::vector<uint8_t> done_;
    std::vector<BlockState> st_;
    std::vector<std::mutex> locks_;
    std::vector<size_t> order_;
    size_t next_ = 0;
    std::mutex mu_;
    std::atomic<size_t> rows_run_{0};
};

// The GPU stage on one batch whose overlap is K: rounds of up to `slots` windows from the feed,
// one fresh slot each, slot-major rows. A window runs as EOT, its K overlap inputs (answers not
// used) and its own inputs, the rows of the context restart (crates/taco/src/gpu_fold.rs
// Window::rows); the answers of its own inputs go to the feed's encoders.
int run_windows(hs_batch* batch, uint32_t eot, size_t K, WindowFeed& feed, const std::vector<FoldBlock>& blocks) {
    const uint32_t slots = hs::batch_slots(batch);
    const std::vector<Window>& windows = feed.windows();
    std::vector<uint32_t> s_slot, s_tok, s_kind;
    std::vector<uint64_t> s_val;
    std::vector<hs_interval> ivs;
    std::vector<size_t> first, mine;
    int rc;
    for (;;) {
        feed.take(slots, mine);
        if (mine.empty()) return HS_OK;
        s_slot.clear();
        s_tok.clear();
        s_val.clear();
        first.assign(mine.size(), 0);
        for (size_t m = 0; m < mine.size(); m++) {
            const Window& win = windows[mine[m]];
            const std::vector<uint32_t>& t = blocks[win.block].tokens;
            const uint32_t slot = (uint32_t)m;
            if ((rc = hs_batch_reset(batch, slot))) return rc;
            auto row = [&](size_t j) {  // input j of the block, coding t_j
                s_slot.push_back(slot);
                s_tok.push_back(j ? t[j - 1] : eot);
                s_val.push_back(t[j]);
            };
            if (win.start > 0) {
                s_slot.push_back(slot);  // the restart's EOT row
                s_tok.push_back(eot);
                s_val.push_back(0);
                for (size_t j = win.start - K; j < win.start; j++) row(j);
            }
            first[m] = s_slot.size();
            for (size_t j = win.start; j < win.start + win.count; j++) row(j);
        }
        s_kind.assign(s_slot.size(), 0);
        ivs.resize(s_slot.size());
        if ((rc = hs_batch_run_coded(batch, s_slot.data(), s_tok.data(), s_kind.data(), s_val.data(),
                                     (uint32_t)s_slot.size(), FREQ_BITS, ivs.data())))
            return rc;
        // Every answer is checked as the reference checks the coder op's intervals on the host
        // (crates/taco/src/lanes.rs:119-128, interval.rs CodeInterval::new): a frequency of 0, an
        // interval past the total or a wrong last-symbol flag is a fault of the device, and fails
        // the fold here instead of reaching the range encoder (whose range a zero frequency would
        // leave at 0).
        constexpr uint64_t TOTAL = 1ull << FREQ_BITS;
        for (const hs_interval& iv : ivs)
            if (iv.freq == 0 || iv.start > TOTAL || iv.freq > TOTAL - iv.start ||
                (iv.is_last != 0) != (iv.start + iv.freq == TOTAL))
                return hs::host_fail(HS_CUDA, "the coder op gave a bad interval (start " + std::to_string(iv.start) +
                                                  ", freq " + std::to_string(iv.freq) + ")");
        feed.add_rows(s_slot.size());
        for (size_t m = 0; m < mine.size(); m++) {
            const Window& win = windows[mine[m]];
            feed.intervals(mine[m]).assign(ivs.begin() + first[m], ivs.begin() + first[m] + win.count);
        }
        feed.complete(mine);
    }
}

// ---- the GPU side of a fold: the caller's batch, or one host thread per GPU ----

class GpuRunner {
  public:
    virtual ~GpuRunner() = default;
    // Runs the windows of the feed until it is empty (every window taken has completed).
    virtual int run(WindowFeed& feed, const std::vector<FoldBlock>& blocks) = 0;
};

// The batch of hs_fold, on the caller's thread (its device handle belongs to that thread).
class OneGpu : public GpuRunner {
  public:
    OneGpu(hs_batch* batch, uint32_t eot, size_t K) : batch_(batch), eot_(eot), K_(K) {}
    int run(WindowFeed& feed, const std::vector<FoldBlock>& blocks) override {
        return run_windows(batch_, eot_, K_, feed, blocks);
    }

  private:
    hs_batch* batch_;
    uint32_t eot_;
    size_t K_;
};

// hs_fold_multi: one host thread per GPU for the whole fold (crates/taco/src/gpu_fold.rs:128-186).
// Each thread opens its device (a device handle belongs to its thread), loads the model and makes
// its batch once; then it runs the windows of each segment's feed with the others, all taking
// rounds from the one feed, so a faster GPU takes more. A GPU that cannot be opened, load the
// model or hold the batch gives its share to the others, as the reference's backend choice falls
// back from a device that fails (crates/taco/src/backend.rs:288-342). An error while windows run
// fails the fold (the windows it had taken never complete). A thread's error message is
// thread-local; it comes back with its status.
class MultiGpu : public GpuRunner {
  public:
    struct Config {
        const int* ordinals;
        uint32_t n;
        const uint8_t* model_file;
        size_t model_len;
        const uint8_t* hash;
        uint32_t vocab, eot, n_ctx, slots, max_rows;
        size_t K;
    };

    explicit MultiGpu(const Config& c) : c_(c), rcs_(c.n, HS_OK), msgs_(c.n), live_(c.n, 0) {}

    ~MultiGpu() override {
        {
            std::lock_guard<std::mutex> lk(mu_);
            quit_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }

    // Starts the threads, each of which opens its GPU. The opening overlaps the host's work on
    // the first segment; run() waits for it, so a fold that needs no window opens no GPU.
    void start() {
        for (uint32_t g = 0; g < c_.n; g++) threads_.emplace_back([this, g] { worker(g); });
    }

    // The GPUs that did not open (after every GPU tried).
    uint32_t failed() {
        std::unique_lock<std::mutex> lk(mu_);
        wait_tried(lk);
        return failed_;
    }

    int run(WindowFeed& feed, const std::vector<FoldBlock>& blocks) override {
        std::unique_lock<std::mutex> lk(mu_);
        wait_tried(lk);
        if (failed_ == c_.n)
            return hs::host_fail(rcs_[0], "no GPU of the fold opened; GPU " + std::to_string(c_.ordinals[0]) + ": " +
                                              msgs_[0]);
        feed_ = &feed;
        blocks_ = &blocks;
        busy_ = c_.n - failed_;
        gen_++;
        cv_.notify_all();
        cv_.wait(lk, [&] { return busy_ == 0; });
        for (uint32_t g = 0; g < c_.n; g++)
            if (live_[g] && rcs_[g])
                return hs::host_fail(rcs_[g], "GPU " + std::to_string(c_.ordinals[g]) + ": " + msgs_[g]);
        return HS_OK;
    }

  private:
    void wait_tried(std::unique_lock<std::mutex>& lk) {  // under mu_
        cv_.wait(lk, [&] { return tried_ == c_.n; });
        uint32_t ok = 0;
        for (uint32_t g = 0; g < c_.n; g++) ok += live_[g];
        failed_ = c_.n - ok;
    }

    void note(uint32_t g, int rc) {  // under mu_
        char buf[1024];
        hs_last_error(buf, sizeof buf);
        msgs_[g] = buf;
        rcs_[g] = rc;
    }

    void worker(uint32_t g) {
        hs_dev* dev = nullptr;
        hs_model* model = nullptr;
        hs_batch* batch = nullptr;
        int rc = hs_open(c_.ordinals[g], &dev);
        if (!rc) rc = hs_model_load(dev, c_.model_file, c_.model_len, &model);
        hs_model_info mi;
        if (!rc && !(rc = hs_model_get_info(model, &mi))) {
            if (memcmp(mi.hash, c_.hash, 32) != 0 || mi.n_ctx != c_.n_ctx || mi.eot_token != c_.eot ||
                mi.vocab != c_.vocab)
                rc = hs::host_fail(HS_MODEL, "the loaded model is not the model file");
        }
        if (!rc) rc = hs_batch_new(model, c_.slots, c_.max_rows, &batch);
        if (!rc) rc = hs_batch_set_overlap(batch, (uint16_t)c_.K);
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (rc) note(g, rc);
            live_[g] = rc == HS_OK;
            tried_++;
        }
        cv_.notify_all();
        uint64_t seen = 0;
        while (!rc) {
            WindowFeed* feed;
            const std::vector<FoldBlock>* blocks;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
                if (quit_) break;
                seen = gen_;
                feed = feed_;
                blocks = blocks_;
            }
            const int r = run_windows(batch, c_.eot, c_.K, *feed, *blocks);
            {
                std::lock_guard<std::mutex> lk(mu_);
                if (r) note(g, r);
                busy_--;
            }
            cv_.notify_all();
            rc = r;
        }
        if (batch) hs_batch_free(batch);
        if (model) hs_model_free(model);
        if (dev) hs_dev_free(dev);
    }

    Config c_;
    std::vector<int> rcs_;
    std::vector<std::string> msgs_;
    std::vector<char> live_;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_;
    uint32_t tried_ = 0, failed_ = 0, busy_ = 0;
    uint64_t gen_ = 0;
    bool quit_ = false;
    WindowFeed* feed_ = nullptr;
    const std::vector<FoldBlock>* blocks_ = nullptr;
};

// ---- the input and the output of a fold ----

// The input bytes in order: read() gives up to cap bytes, 0 only at the end, < 0 on an error.
struct Source {
    virtual ~Source() = default;
    virtual int64_t read(uint8_t* buf, size_t cap) = 0;
};

// Where the parts of the container go (stream.rs Layout): the stored blocks in order, the
// table entries in order, and the header last, which completes the container. Each call gives 0,
// or non-zero on an error. A sink that needs the input length before the first block (it puts
// the blocks after a table whose size follows from the length) says so with needs_len() and
// receives the offset of the first stored byte in begin().
struct Sink {
    virtual ~Sink() = default;
    virtual bool needs_len() const { return false; }
    virtual int begin(uint64_t /*data_off*/) { return 0; }
    virtual int block(const uint8_t* p, size_t n) = 0;
    virtual int table(const uint8_t* p, size_t n) = 0;
    virtual int header(const uint8_t* p, size_t n) = 0;
    // What failed, after a call gave non-zero.
    virtual std::string why() const { return "the output sink failed"; }
};

// A seekable output (stream.rs SeekLayout): write() puts n bytes at offset `at`. The header and
// the table have their places at the start; the blocks follow the table.
struct SeekSink : Sink {
    uint64_t block_at = 0, table_at = HEADER_LEN;
    virtual int write(uint64_t at, const uint8_t* p, size_t n) = 0;
    bool needs_len() const override { return true; }
    int begin(uint64_t data_off) override {
        block_at = data_off;
        return 0;
    }
    int block(const uint8_t* p, size_t n) override {
        block_at += n;
        return write(block_at - n, p, n);
    }
    int table(const uint8_t* p, size_t n) override {
        table_at += n;
        return write(table_at - n, p, n);
    }
    int header(const uint8_t* p, size_t n) override { return write(0, p, n); }
};

struct MemSource : Source {
    const uint8_t* p;
    size_t left;
    MemSource(const uint8_t* d, size_t n) : p(d), left(n) {}
    int64_t read(uint8_t* buf, size_t cap) override {
        const size_t n = std::min(cap, left);
        if (n) memcpy(buf, p, n);
        p += n;
        left -= n;
        return (int64_t)n;
    }
};

// The caller's buffer; writes past its end are dropped and remembered (the caller gets the
// length it needs).
struct MemSink : SeekSink {
    uint8_t* out;
    size_t cap;
    bool overflow = false;
    MemSink(uint8_t* o, size_t c) : out(o), cap(c) {}
    int write(uint64_t at, const uint8_t* p, size_t n) override {
        if (!out || at > cap || n > cap - at) overflow = true;
        else if (n) memcpy(out + at, p, n);
        return 0;
    }
};

struct CallbackSource : Source {
    hs_source_fn fn;
    void* user;
    int64_t read(uint8_t* buf, size_t cap) override { return fn(user, buf, cap); }
    CallbackSource(hs_source_fn f, void* u) : fn(f), user(u) {}
};

struct CallbackSink : SeekSink {
    hs_sink_fn fn;
    void* user;
    int write(uint64_t at, const uint8_t* p, size_t n) override { return fn(user, at, p, n); }
    CallbackSink(hs_sink_fn f, void* u) : fn(f), user(u) {}
};

// The method "spool" for an output that cannot seek (stream.rs SpoolLayout and TempFile): the
// stored blocks and the table go to two temporary files in a directory of the caller; at the end
// the header goes to the writer, then the table and the blocks are copied after it. Each file is
// unlinked as soon as it is made (mkstemp, name .taco-spool-<pid>-<part>-XXXXXX), so it vanishes
// when the fold ends, after an error or a crash too; the reference deletes its files when the
// fold ends.
class SpoolSink : public Sink {
  public:
    SpoolSink(hs_write_fn fn, void* user) : fn_(fn), user_(user) {}
    ~SpoolSink() override {
        if (blocks_) fclose(blocks_);
        if (table_) fclose(table_);
    }
    // Makes the two files in `dir` (NULL: $TMPDIR, else /tmp). HS_IO if it cannot.
    int open(const char* dir) {
        std::string d = dir ? dir : "";
        if (d.empty()) {
            const char* t = getenv("TMPDIR");
            d = t && *t ? t : "/tmp";
        }
        if (!make(d, "blocks", &blocks_) || !make(d, "table", &table_))
            return hs::host_fail(HS_IO, "cannot make a temporary file in " + d + ": " + why_);
        return HS_OK;
    }
    int block(const uint8_t* p, size_t n) override { return put(blocks_, p, n); }
    int table(const uint8_t* p, size_t n) override { return put(table_, p, n); }
    int header(const uint8_t* p, size_t n) override {
        if (fn_(user_, p, n)) return fail("the output writer failed");
        return copy(table_) || copy(blocks_);
    }
    std::string why() const override { return why_.empty() ? "the output writer failed" : why_; }

  private:
    bool make(const std::string& dir, const char* part, FILE** f) {
        std::string path = dir + "/.taco-spool-" + std::to_string((long)getpid()) + "-" + part + "-XXXXXX";
        const int fd = mkstemp(&path[0]);
        if (fd < 0) {
            why_ = strerror(errno);
            return false;
        }
        unlink(path.c_str());
        *f = fdopen(fd, "w+b");
        if (!*f) {
            why_ = strerror(errno);
            ::close(fd);
            return false;
        }
        setvbuf(*f, nullptr, _IOFBF, 1 << 20);
        return true;
    }
    int fail(const std::string& w) {
        why_ = w;
        return 1;
    }
    int put(FILE* f, const uint8_t* p, size_t n) {
        if (n && fwrite(p, 1, n, f) != n) return fail(std::string("a temporary file failed: ") + strerror(errno));
        return 0;
    }
    int copy(FILE* f) {
        if (fflush(f) || fseeko(f, 0, SEEK_SET)) return fail(std::string("a temporary file failed: ") + strerror(errno));
        std::vector<uint8_t> buf(1 << 20);
        for (;;) {
            const size_t k = fread(buf.data(), 1, buf.size(), f);
            if (k && fn_(user_, buf.data(), k)) return fail("the output writer failed");
            if (k < buf.size()) return ferror(f) ? fail("a temporary file failed on reading") : 0;
        }
    }

    hs_write_fn fn_;
    void* user_;
    FILE* blocks_ = nullptr;
    FILE* table_ = nullptr;
    std::string why_;
};

// The blocks of one segment and their input bytes. A fold holds two segments at a time: the
// one on the GPUs and the next one, which the host threads tokenize and compress meanwhile.
struct Segment {
    uint64_t first = 0;  // index of the segment's first block
    std::vector<uint8_t> data;
    std::vector<FoldBlock> blocks;  // off is relative to data
    int rc = HS_OK;
    std::string msg;
    double ms = 0;
};

// The largest input of one segment, and its most blocks (crates/taco/src/stream.rs:56-63 has 64
// MiB and 256 blocks). The bytes do not depend on the segment size (stream.rs:19-20). Here a
// segment holds up to 4,096 blocks, so that 8 GPUs of 512 slots have windows enough to fill their
// passes; the memory stays bounded by the 64 MiB of input per segment (its tokens, zstd frames
// and payloads), two segments at a time.
constexpr uint64_t SEGMENT_BYTES = 64ull << 20;
constexpr uint64_t SEGMENT_BLOCKS = 4096;

double ms_since(std::chrono::steady_clock::time_point t0) {
    return std::chrono::duration<double, std::milli>(std::chrono::steady_clock::now() - t0).count();
}

// Tokens and zstd frames of a segment's blocks on the host threads.
void prep_segment(Segment& seg, const hs_tokenizer* tok, unsigned threads) {
    const auto t0 = std::chrono::steady_clock::now();
    std::atomic<int64_t> bad_tokens{-1}, bad_zstd{-1};
    parallel_for(seg.blocks.size(), threads, [&](size_t i) {
        FoldBlock& b = seg.blocks[i];
        const uint8_t* in = seg.data.data() + b.off;
        hs::tokenize(tok, in, b.len, b.tokens);
        if (!hs::tokens_restore(tok, b.tokens.data(), b.tokens.size(), in, b.len)) bad_tokens = (int64_t)i;
        b.zstd_ok = compress_zstd(in, b.len, b.zstd);
        if (!b.zstd_ok) bad_zstd = (int64_t)i;
    });
    if (bad_tokens >= 0) {
        seg.rc = HS_MODEL;
        seg.msg = "the tokens of block " + std::to_string(seg.first + bad_tokens.load()) +
                  " do not give its bytes back (TokenizerRoundTrip)";
    } else if (bad_zstd >= 0) {
        seg.rc = HS_CUDA;
        seg.msg = "zstd failed on block " + std::to_string(seg.first + bad_zstd.load());
    }
    seg.ms = ms_since(t0);
}

struct FoldStatsAcc {
    uint64_t tokens = 0, coded = 0, zstd = 0, rows = 0;
    double prep_ms = 0, gpu_ms = 0, finish_ms = 0;
};

// The fold of fold_with, segment by segment (crates/taco/src/fold.rs code_segment over the
// segments of stream.rs StreamFold::run, for to_seekable and to_writer): the stored blocks and
// the table entries go to the sink as each segment ends, the header (with the input's length,
// block count and SHA-256) last. `len` may be LEN_UNKNOWN (to_writer with no input length): then
// the segments are read until the input ends, and the block size is the set one or the default
// (the spread rule needs the length). Per segment:
// 2. tokens and zstd frames on the host threads (for the next segment while the GPUs run this one);
// 3. the context windows on the GPUs, each block's range encoder taking its intervals as they
//    complete (WindowFeed);
// 4.-5. each block's payload if its encoder did not stop, and its smallest stored form.
int fold_stream_impl(const uint8_t model_hash[32], uint32_t n_ctx, GpuRunner& gpu,
                     const hs_tokenizer* tok, Source& src, uint64_t len, Sink& sink, const hs_fold_options* opt,
                     uint64_t* out_len, hs_fold_stats* stats) {
    if (!zstd().ok) return hs::host_fail(HS_UNSUPPORTED, "the zstd library (libzstd.so.1) is not available");
    // FoldOptions::block_size_for (fold.rs:159-170): a set size, or 16 KiB; with `spread`, the
    // power of two that makes about 64 blocks, within 4 KiB .. 16 KiB.
    const bool known = len != LEN_UNKNOWN;
    uint64_t bs = opt->block_size ? opt->block_size : DEFAULT_BLOCK_SIZE;
    if (opt->spread && !opt->block_size && known) {
        uint64_t per = (len + SPREAD_BLOCKS - 1) / SPREAD_BLOCKS, p2 = 1;
        while (p2 < per) p2 <<= 1;
        bs = std::min<uint64_t>(std::max<uint64_t>(p2, SPREAD_MIN_BLOCK), DEFAULT_BLOCK_SIZE);
    }
    if (bs == 0 || bs > MAX_BLOCK_SIZE) return hs::host_fail(HS_UNSUPPORTED, "the block size is out of range");
    // The block count: from the length, or (length unknown) counted as the segments arrive.
    const uint64_t nblocks = known ? blocks_of(len, bs) : 0;
    if (nblocks > MAX_BLOCKS) return hs::host_fail(HS_UNSUPPORTED, "more than 2^32 - 1 blocks");
    if (!known && sink.needs_len())
        return hs::host_fail(HS_BAD_ARGUMENT, "a seekable output needs the input length");
    const unsigned threads = opt->threads ? opt->threads : std::max(1u, std::thread::hardware_concurrency());
    const size_t K = std::min<size_t>(opt->overlap, n_ctx - 2);
    const uint64_t seg_blocks = std::min<uint64_t>(std::max<uint64_t>(SEGMENT_BYTES / bs, 1), SEGMENT_BLOCKS);
    hs::Sha256 sum;
    FoldStatsAcc acc;
    uint64_t total_len = 0, total_blocks = 0, stored_total = 0;
    int rc;
    auto io = [](const std::string& what) { return hs::host_fail(HS_IO, what); };
    if (known && sink.begin(HEADER_LEN + 5 * nblocks)) return io(sink.why());
    // Reads the input bytes of the segment that starts at block `first`: the segment's share of
    // `len`, or (length unknown) up to a full segment, fewer only at the end of the input. The
    // buffer grows with the bytes that arrive (stream.rs read_up_to).
    auto read_segment = [&](uint64_t first, Segment& seg) -> int {
        seg.first = first;
        const uint64_t want = known ? std::min<uint64_t>(seg_blocks * bs, len - first * bs) : seg_blocks * bs;
        seg.data.clear();
        if (known) seg.data.resize((size_t)want);
        uint64_t got = 0;
        while (got < want) {
            if (seg.data.size() == got)
                seg.data.resize((size_t)std::min<uint64_t>(want, std::max<uint64_t>(2 * got, 1u << 20)));
            const int64_t r = src.read(seg.data.data() + got, (size_t)(seg.data.size() - got));
            if (r < 0) return io("the input source failed");
            if (r == 0) {
                if (known) return io("the input is shorter than its length");
                break;
            }
            got += (uint64_t)r;
        }
        seg.data.resize((size_t)got);
        const uint64_t nb = blocks_of(got, bs);
        if (first + nb > MAX_BLOCKS) return hs::host_fail(HS_UNSUPPORTED, "more than 2^32 - 1 blocks");
        sum.update(seg.data.data(), (size_t)got);
        total_len += got;
        seg.blocks.assign((size_t)nb, FoldBlock());
        for (uint64_t i = 0; i < nb; i++) {
            seg.blocks[i].off = (size_t)(i * bs);
            seg.blocks[i].len = (size_t)std::min<uint64_t>(bs, got - i * bs);
        }
        seg.rc = HS_OK;
        seg.msg.clear();
        return HS_OK;
    };
    auto cur = std::make_unique<Segment>(), next = std::make_unique<Segment>();
    if ((rc = read_segment(0, *cur))) return rc;
    if (!cur->blocks.empty()) {
        prep_segment(*cur, tok, threads);
        acc.prep_ms += cur->ms;
    }
    std::vector<uint8_t> table;
    while (!cur->blocks.empty()) {
        if (cur->rc) return hs::host_fail(cur->rc, cur->msg);
        const uint64_t first = cur->first;
        // The next segment: read here (the source is called on the caller's thread only), then
        // tokenized and compressed on the host threads while the GPUs run this one. With the
        // length unknown, a full segment may have one after it; a read that finds the end of the
        // input gives an empty one.
        std::thread helper;
        bool more = known ? first + seg_blocks < nblocks : cur->data.size() == seg_blocks * bs;
        if (more) {
            if ((rc = read_segment(first + seg_blocks, *next))) return rc;
            more = !next->blocks.empty();
            if (more) helper = std::thread([&] { prep_segment(*next, tok, threads); });
        }
        struct Join {
            std::thread& t;
            ~Join() {
                if (t.joinable()) t.join();
            }
        } join{helper};
        // 3. The windows (gpu_fold.rs windows_of). A block's inputs are x_0 = EOT, x_j = t_(j-1)
        // (input j codes t_j). In one slot its context restarts after every n_ctx positions with
        // EOT and the last K inputs (crates/hardshell/src/gpt2/context.rs), so the block divides
        // into context windows: window 0 is inputs 0 .. n_ctx - 1, each later window the next
        // n_ctx - K - 1 inputs. Each window runs in a fresh slot of its own (run_windows), so the
        // windows of all blocks run side by side in full passes. A block whose payload prefix
        // already reaches its bound needs none (BlockEncoder::stopped).
        std::vector<FoldBlock>& blocks = cur->blocks;
        std::vector<Window> windows;
        for (size_t i = 0; i < blocks.size(); i++) {
            const FoldBlock& b = blocks[i];
            if (b.tokens.empty() || varint_len(b.tokens.size()) >= std::min(b.len, b.zstd.size())) continue;
            for (size_t s0 = 0; s0 < b.tokens.size();) {
                const size_t c = std::min(b.tokens.size() - s0, s0 == 0 ? (size_t)n_ctx : n_ctx - K - 1);
                windows.push_back({i, s0, c});
                s0 += c;
            }
        }
        WindowFeed feed(std::move(windows), blocks, blocks.size());
        feed.order_by_waves();
        auto t0 = std::chrono::steady_clock::now();
        if (!feed.windows().empty() && (rc = gpu.run(feed, blocks))) return rc;
        acc.gpu_ms += ms_since(t0);
        // 4.-5. The payloads of the blocks whose encoders did not stop, then the smallest form.
        t0 = std::chrono::steady_clock::now();
        parallel_for(blocks.size(), threads, [&](size_t i) {
            FoldBlock& b = blocks[i];
            std::vector<uint8_t> coded;
            const bool live = feed.finish(i, coded);
            size_t best = b.len;
            if (b.zstd.size() < best) {
                best = b.zstd.size();
                b.kind = KIND_ZSTD;
                b.stored = std::move(b.zstd);
            }
            if (live && coded.size() < best) {
                b.kind = KIND_CODED;
                b.stored = std::move(coded);
            }
        });
        acc.rows += feed.rows_run();
        // The segment's table entries and stored blocks (writer.rs:245-300).
        table.clear();
        for (const FoldBlock& b : blocks) {
            const uint32_t sl = (uint32_t)(b.kind == KIND_RAW ? b.len : b.stored.size());
            table.push_back(b.kind);
            for (int k = 0; k < 4; k++) table.push_back((uint8_t)(sl >> (8 * k)));
            if (sink.block(b.kind == KIND_RAW ? cur->data.data() + b.off : b.stored.data(), sl))
                return io(sink.why());
            stored_total += sl;
            acc.tokens += b.tokens.size();
            acc.coded += b.kind == KIND_CODED;
            acc.zstd += b.kind == KIND_ZSTD;
        }
        if (sink.table(table.data(), table.size())) return io(sink.why());
        total_blocks += blocks.size();
        acc.finish_ms += ms_since(t0);
        if (!more) break;
        helper.join();
        acc.prep_ms += next->ms;
        std::swap(cur, next);
    }
    if (known) {
        uint8_t extra;
        const int64_t r = src.read(&extra, 1);
        if (r < 0) return io("the input source failed");
        if (r > 0) return io("the input is longer than its length");
    }
    // The header (header.rs, version 2, profile text).
    uint8_t h[HEADER_LEN] = {0};
    auto put16 = [&](size_t o, uint16_t v) { memcpy(h + o, &v, 2); };
    auto put32 = [&](size_t o, uint32_t v) { memcpy(h + o, &v, 4); };
    auto put64 = [&](size_t o, uint64_t v) { memcpy(h + o, &v, 8); };
    memcpy(h, "TACO", 4);
    put16(4, 2);  // version
    put16(6, 0);  // flags
    memcpy(h + 8, model_hash, 32);
    put64(40, total_len);
    sum.final(h + 48);
    put32(80, (uint32_t)bs);
    put32(84, (uint32_t)total_blocks);
    const uint16_t k = (uint16_t)opt->overlap;
    h[88] = 0;                 // profile text
    h[89] = 0;                 // reserved
    put16(90, k ? 2 : 0);      // coding parts: bit 1 = the overlap
    memcpy(h + 92 + 2, &k, 2);  // coding parameters: the overlap
    if (sink.header(h, HEADER_LEN)) return io(sink.why());
    const uint64_t container_len = HEADER_LEN + 5 * total_blocks + stored_total;
    *out_len = container_len;
    if (stats) {
        memset(stats, 0, sizeof(*stats));
        stats->original_len = total_len;
        stats->container_len = container_len;
        stats->blocks = total_blocks;
        stats->block_size = (uint32_t)bs;
        stats->tokens = acc.tokens;
        stats->coded_blocks = acc.coded;
        stats->zstd_blocks = acc.zstd;
        stats->gpu_rows = acc.rows;
        stats->prep_ms = acc.prep_ms;
        stats->gpu_ms = acc.gpu_ms;
        stats->finish_ms = acc.finish_ms;
    }
    return HS_OK;
}

// FoldPlan::new (fold.rs:388-395): the tokenizer must have the model's vocabulary.
int check_tokenizer(const hs_tokenizer* tok, uint32_t vocab) {
    uint32_t tv, te, tc;
    hs::tokenizer_info(tok, &tv, &te, &tc);
    if (tv != vocab)
        return hs::host_fail(HS_MODEL, "the tokenizer has " + std::to_string(tv) + " tokens, the model " +
                                           std::to_string(vocab) + " (TokenizerMismatch)");
    return HS_OK;
}

// The one-GPU fold of a batch (hs_fold, hs_fold_stream).
int fold_one(hs_batch* batch, const hs_tokenizer* tok, Source& src, uint64_t len, Sink& sink,
             const hs_fold_options* opt, uint64_t* out_len, hs_fold_stats* stats) {
    hs_model_info info;
    int rc = hs_model_get_info(hs::batch_model(batch), &info);
    if (rc || (rc = check_tokenizer(tok, info.vocab))) return rc;
    if (opt->overlap > 0xFFFF) return hs::host_fail(HS_INVALID_OVERLAP, "the overlap is out of range");
    if ((rc = hs_batch_set_overlap(batch, (uint16_t)opt->overlap))) return rc;
    OneGpu gpu(batch, info.eot_token, std::min<size_t>(opt->overlap, info.n_ctx - 2));
    return fold_stream_impl(info.hash, info.n_ctx, gpu, tok, src, len, sink, opt, out_len, stats);
}

// The fold on several GPUs (hs_fold_multi, hs_fold_stream_multi).
int fold_many(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len, uint32_t slots,
              uint32_t max_rows, const hs_tokenizer* tok, Source& src, uint64_t len, Sink& sink,
              const hs_fold_options* opt, uint64_t* out_len, hs_fold_stats* stats) {
    // The windows are cut with the model's context length and EOT token, as hs_fold cuts them
    // with those of its batch's model (gpu_fold.rs windows_of, Window::rows); the tokenizer only
    // has to share the model's vocabulary (FoldPlan::new, fold.rs:388-395).
    uint32_t vocab, eot, n_ctx;
    {
        std::string err;
        if (!hs::model_file_info(model_file, model_len, &vocab, &eot, &n_ctx, err))
            return hs::host_fail(HS_MODEL, "the model file is not valid: " + err);
    }
    int rc = check_tokenizer(tok, vocab);
    if (rc) return rc;
    if (opt->overlap > 0xFFFF || opt->overlap > n_ctx - 2)
        return hs::host_fail(HS_INVALID_OVERLAP, "the overlap must be at most n_ctx - 2");
    uint8_t hash[32];
    hs::sha256(model_file, model_len, hash);  // the model hash of the container (model.rs:359)
    // HS_FOLD_WORKERS_PER_GPU (default 2): host threads per GPU, each with its own batch, so that
    // one thread's host work between its rounds (rows, planning, range coding) overlaps another
    // thread's passes on the same GPU (the 256 MiB mixed input on one B200: 41.1 s with two,
    // 45.4 s with one; the same container).
    uint32_t per = 2;
    if (const char* v = getenv("HS_FOLD_WORKERS_PER_GPU")) per = (uint32_t)std::min(8, std::max(1, atoi(v)));
    std::vector<int> ords;
    for (uint32_t k = 0; k < per; k++) ords.insert(ords.end(), ordinals, ordinals + n_gpus);
    MultiGpu gpu({ords.data(), (uint32_t)ords.size(), model_file, model_len, hash, vocab, eot, n_ctx, slots,
                  max_rows, opt->overlap});
    gpu.start();
    rc = fold_stream_impl(hash, n_ctx, gpu, tok, src, len, sink, opt, out_len, stats);
    if (!rc && stats) stats->gpus_failed = gpu.failed() / per;  // a GPU's workers fail together
    return rc;
}

int mem_result(const MemSink& sink, uint64_t total, size_t cap, size_t* out_len) {
    *out_len = (size_t)total;
    if (sink.overflow)
        return hs::host_fail(HS_BAD_ARGUMENT, "the output holds " + std::to_string(cap) + " bytes, " +
                                                  std::to_string(total) + " needed (hs_fold_bound)");
    return HS_OK;
}

}  // namespace

extern "C" {

int hs_fold(hs_batch* batch, const hs_tokenizer* tok, const uint8_t* input, size_t len, const hs_fold_options* opt,
            uint8_t* out, size_t cap, size_t* out_len, hs_fold_stats* stats) {
    if (!batch || !tok || !opt || !out_len || (len && !input)) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    MemSource src(input, len);
    MemSink sink(out, cap);
    uint64_t total = 0;
    const int rc = fold_one(batch, tok, src, len, sink, opt, &total, stats);
    return rc ? rc : mem_result(sink, total, cap, out_len);
}

int hs_fold_stream(hs_batch* batch, const hs_tokenizer* tok, uint64_t len, hs_source_fn source, void* source_user,
                   hs_sink_fn sink, void* sink_user, const hs_fold_options* opt, uint64_t* out_len,
                   hs_fold_stats* stats) {
    if (!batch || !tok || !opt || !out_len || !source || !sink) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackSource src(source, source_user);
    CallbackSink snk(sink, sink_user);
    return fold_one(batch, tok, src, len, snk, opt, out_len, stats);
}

int hs_fold_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                  uint32_t slots, uint32_t max_rows, const hs_tokenizer* tok, const uint8_t* input, size_t len,
                  const hs_fold_options* opt, uint8_t* out, size_t cap, size_t* out_len, hs_fold_stats* stats) {
    if (!ordinals || !n_gpus || !model_file || !tok || !opt || !out_len || (len && !input))
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    MemSource src(input, len);
    MemSink sink(out, cap);
    uint64_t total = 0;
    const int rc =
        fold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, src, len, sink, opt, &total, stats);
    return rc ? rc : mem_result(sink, total, cap, out_len);
}

int hs_fold_stream_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                         uint32_t slots, uint32_t max_rows, const hs_tokenizer* tok, uint64_t len,
                         hs_source_fn source, void* source_user, hs_sink_fn sink, void* sink_user,
                         const hs_fold_options* opt, uint64_t* out_len, hs_fold_stats* stats) {
    if (!ordinals || !n_gpus || !model_file || !tok || !opt || !out_len || !source || !sink)
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackSource src(source, source_user);
    CallbackSink snk(sink, sink_user);
    return fold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, src, len, snk, opt, out_len,
                     stats);
}
int hs_fold_spool(hs_batch* batch, const hs_tokenizer* tok, uint64_t len, hs_source_fn source, void* source_user,
                  hs_write_fn write, void* write_user, const char* spool_dir, const hs_fold_options* opt,
                  uint64_t* out_len, hs_fold_stats* stats) {
    if (!batch || !tok || !opt || !out_len || !source || !write) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackSource src(source, source_user);
    SpoolSink snk(write, write_user);
    int rc = snk.open(spool_dir);
    if (rc) return rc;
    return fold_one(batch, tok, src, len, snk, opt, out_len, stats);
}
int hs_fold_spool_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                        uint32_t slots, uint32_t max_rows, const hs_tokenizer* tok, uint64_t len, hs_source_fn source,
                        void* source_user, hs_write_fn write, void* write_user, const char* spool_dir,
                        const hs_fold_options* opt, uint64_t* out_len, hs_fold_stats* stats) {
    if (!ordinals || !n_gpus || !model_file || !tok || !opt || !out_len || !source || !write)
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackSource src(source, source_user);
    SpoolSink snk(write, write_user);
    int rc = snk.open(spool_dir);
    if (rc) return rc;
    return fold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, src, len, snk, opt, out_len,
                     stats);
}

uint32_t hs_zstd_version(void) { return zstd().ok ? zstd().version() : 0; }

}  // extern "C"

// ---- unfold ----

namespace {

// Positional reads of a container: read() fills n bytes from offset `at`; 0, or non-zero on an
// error.
struct ReadAt {
    virtual ~ReadAt() = default;
    virtual int read(uint64_t at, uint8_t* p, size_t n) = 0;
    // Whether a read failed in the caller's source (an I/O error, not a short container).
    virtual bool failed() const { return false; }
    // The bytes before `end` (the header and the table) will be read again; the later ones once.
    virtual void keep(uint64_t /*end*/) {}
};

// The original bytes in order: write() takes n bytes; 0, or non-zero on an error.
struct Writer {
    virtual ~Writer() = default;
    virtual int write(const uint8_t* p, size_t n) = 0;
};

struct MemReadAt : ReadAt {
    const uint8_t* d;
    uint64_t n;
    MemReadAt(const uint8_t* p, uint64_t len) : d(p), n(len) {}
    int read(uint64_t at, uint8_t* p, size_t k) override {
        if (at > n || k > n - at) return 1;
        if (k) memcpy(p, d + at, k);
        return 0;
    }
};

struct MemWriter : Writer {
    uint8_t* out;
    size_t at = 0, cap;
    MemWriter(uint8_t* o, size_t c) : out(o), cap(c) {}
    int write(const uint8_t* p, size_t n) override {
        if (n > cap - at) return 1;
        if (n) memcpy(out + at, p, n);
        at += n;
        return 0;
    }
};

struct CallbackReadAt : ReadAt {
    hs_read_at_fn fn;
    void* user;
    CallbackReadAt(hs_read_at_fn f, void* u) : fn(f), user(u) {}
    int read(uint64_t at, uint8_t* p, size_t n) override { return fn(user, at, p, n); }
};

// A container that arrives through a pipe (stream.rs PipeSource), read in one pass. The bytes
// below keep_to (the header and the block table) are kept in memory as they arrive, so that they
// can be read again by offset; the bytes after them (the stored blocks) are read in order, each
// once. read() gives 0, 1 if the container ends first or the read would skip bytes or go back
// before them, 2 if the source failed. The kept bytes grow only with the bytes that arrive, so a
// false block count in a header costs no memory before its table exists (stream.rs:566-568).
struct PipeReadAt : ReadAt {
    hs_source_fn fn;
    void* user;
    std::vector<uint8_t> kept;
    uint64_t pos = 0;  // the bytes taken from the source
    uint64_t keep_to = UINT64_MAX;
    bool bad = false;
    PipeReadAt(hs_source_fn f, void* u) : fn(f), user(u) {}
    bool failed() const override { return bad; }
    void keep(uint64_t end) override { keep_to = end; }
    int read(uint64_t at, uint8_t* p, size_t n) override {
        size_t done = 0;
        if (at < kept.size()) {
            done = (size_t)std::min<uint64_t>(n, kept.size() - at);
            memcpy(p, kept.data() + at, done);
        }
        if (done == n) return 0;
        if (at + done != pos) return 1;
        while (done < n) {
            const int64_t r = fn(user, p + done, n - done);
            if (r < 0 || (uint64_t)r > n - done) {
                bad = true;
                return 2;
            }
            if (r == 0) return 1;
            if (pos < keep_to) {
                const uint64_t k = std::min<uint64_t>((uint64_t)r, keep_to - pos);
                kept.insert(kept.end(), p + done, p + done + k);
            }
            pos += (uint64_t)r;
            done += (size_t)r;
        }
        return 0;
    }
};

struct CallbackWriter : Writer {
    hs_write_fn fn;
    void* user;
    CallbackWriter(hs_write_fn f, void* u) : fn(f), user(u) {}
    int write(const uint8_t* p, size_t n) override { return fn(user, p, n); }
};

// The header of a container (crates/taco-format/src/header.rs:220-330), checked.
struct Header {
    uint16_t version = 0;
    size_t hlen = 0;
    uint8_t model_hash[32];
    uint64_t original_len = 0;
    uint8_t checksum[32];
    uint32_t block_size = 0, count = 0;
    uint8_t profile = 0, mixer_rule = 0;
    uint16_t overlap = 0;
    bool needs_model = false;
};

int bad_container(const std::string& why) { return hs::host_fail(HS_FORMAT, "the container is not valid: " + why); }

int parse_header(ReadAt& in, uint64_t n, Header& c) {
    uint8_t d[HEADER_LEN];
    if (n < 6 || in.read(0, d, 6)) return bad_container("truncated header");
    auto rd16 = [&](size_t o) { uint16_t v; memcpy(&v, d + o, 2); return v; };
    auto rd32 = [&](size_t o) { uint32_t v; memcpy(&v, d + o, 4); return v; };
    auto rd64 = [&](size_t o) { uint64_t v; memcpy(&v, d + o, 8); return v; };
    if (memcmp(d, "TACO", 4) != 0) return bad_container("bad magic");
    c.version = rd16(4);
    if (c.version != 1 && c.version != 2) return bad_container("unsupported version " + std::to_string(c.version));
    c.hlen = c.version == 1 ? 88 : HEADER_LEN;
    if (n < c.hlen || in.read(0, d, c.hlen)) return bad_container("truncated header");
    if (rd16(6) != 0) return bad_container("unknown flags");
    memcpy(c.model_hash, d + 8, 32);
    c.original_len = rd64(40);
    memcpy(c.checksum, d + 48, 32);
    c.block_size = rd32(80);
    c.count = rd32(84);
    if (c.block_size == 0 || c.block_size > MAX_BLOCK_SIZE) return bad_container("block size out of range");
    if ((uint64_t)c.count != blocks_of(c.original_len, c.block_size)) return bad_container("wrong block count");
    if (c.version == 2) {
        c.profile = d[88];
        const uint8_t reserved = d[89];
        const uint16_t bits = rd16(90);
        const uint8_t* params = d + 92;
        if (c.profile > 1 || reserved != 0 || (bits & ~3u)) return bad_container("bad version 2 fields");
        if (c.profile == 0 && (bits & 1)) return bad_container("the text profile has no mixer");
        if (bits & 1) {
            if (params[0] != 1 && params[0] != 2) return bad_container("unknown mixer rule");
            c.mixer_rule = params[0];
        } else if (params[0] != 0) {
            return bad_container("mixer rule without the mixer bit");
        }
        uint16_t k;
        memcpy(&k, params + 2, 2);
        if ((bits & 2) && k == 0) return bad_container("overlap bit with K = 0");
        if (!(bits & 2) && k != 0) return bad_container("overlap without the overlap bit");
        c.overlap = k;
        if (params[1] != 0) return bad_container("non-zero coding parameters");
        for (int i = 4; i < 12; i++)
            if (params[i] != 0) return bad_container("non-zero coding parameters");
    }
    c.needs_model = std::any_of(c.model_hash, c.model_hash + 32, [](uint8_t b) { return b != 0; });
    return HS_OK;
}

constexpr uint32_t TABLE_GROUP = 4096;  // table entries read at a time (stream.rs:66)

// Reads the table entries [first, first + n) into kinds / stored, and checks each entry's rules
// (reader.rs): the kind, a raw block stores its original length, any other kind is smaller, a
// coded or mixed block needs a model, a mixed block needs the mixer bit.
int read_table(ReadAt& in, const Header& c, uint32_t first, uint32_t n, std::vector<uint8_t>& kinds,
               std::vector<uint32_t>& stored) {
    std::vector<uint8_t> raw((size_t)n * 5);
    if (n && in.read(c.hlen + 5 * (uint64_t)first, raw.data(), raw.size())) return bad_container("truncated block table");
    kinds.resize(n);
    stored.resize(n);
    for (uint32_t j = 0; j < n; j++) {
        const uint32_t i = first + j;
        const uint8_t kind = raw[5 * (size_t)j];
        uint32_t sl;
        memcpy(&sl, &raw[5 * (size_t)j + 1], 4);
        const uint64_t olen = std::min<uint64_t>(c.block_size, c.original_len - (uint64_t)i * c.block_size);
        if (kind > 3 || (c.version == 1 && kind > 1)) return bad_container("unknown block kind");
        if (kind == KIND_RAW && sl != olen) return bad_container("a raw block stores its original bytes");
        if (kind != KIND_RAW && sl >= olen) return bad_container("a coded, mixed or zstd block is not smaller than its bytes");
        if ((kind == KIND_CODED || kind == 3) && !c.needs_model) return bad_container("a coded block needs a model");
        if (kind == 3 && c.mixer_rule == 0) return bad_container("a mixed block needs the mixer bit");
        kinds[j] = kind;
        stored[j] = sl;
    }
    return HS_OK;
}

// The coded blocks of one unfold segment, for the GPU side: the segment's stored bytes, its
// blocks' offsets and lengths, the indices (in the segment) of its coded blocks, and the buffer of
// the restored bytes.
struct CodedJob {
    const Header* c;
    const hs_tokenizer* tok;
    uint32_t eot;
    const uint8_t* data;
    size_t data_len;
    const std::vector<uint64_t>* at;
    const std::vector<uint32_t>* stored;
    const std::vector<uint32_t>* coded;
    uint64_t first, seg_len;
    uint8_t* restored;
};

// Decodes the coded blocks coded[r0 .. r1) of the job on `batch` (slots 0 .. r1 - r0 - 1): the
// varint token count (1 .. the block length), then the coder bytes on the device
// (hs_batch_decode_blocks: codec.rs:370-520 BlockDecoder), then the tokens' bytes. A corrupt
// block gives HS_CORRUPT with its index in *bad and the reason in *why (no error is recorded, so
// several threads can each report theirs); another failure returns its status with the thread's
// last error set.
int decode_round(hs_batch* batch, const CodedJob& J, size_t r0, size_t r1, uint64_t* bad, std::string* why) {
    const Header& c = *J.c;
    const size_t mm = r1 - r0;
    std::vector<uint32_t> slots(mm), counts(mm), status(mm);
    std::vector<uint64_t> offs(mm), lens(mm), toff(mm);
    auto corrupt = [&](uint32_t j, const char* reason) {
        *bad = J.first + j;
        *why = reason;
        return (int)HS_CORRUPT;
    };
    uint64_t ntok = 0;
    for (size_t q = 0; q < mm; q++) {
        const uint32_t j = (*J.coded)[r0 + q];
        const uint8_t* p = J.data + (*J.at)[j];
        const size_t sl = (*J.stored)[j];
        uint64_t count = 0;
        size_t k = 0;
        for (int shift = 0;; shift += 7, k++) {
            if (k >= sl || shift > 63) return corrupt(j, "the token count is not valid");
            count |= (uint64_t)(p[k] & 0x7F) << shift;
            if (!(p[k] & 0x80)) break;
        }
        k++;
        const size_t olen = (size_t)std::min<uint64_t>(c.block_size, J.seg_len - (uint64_t)j * c.block_size);
        if (count == 0 || count > olen) return corrupt(j, "the token count does not agree with the block length");
        slots[q] = (uint32_t)q;
        counts[q] = (uint32_t)count;
        offs[q] = (*J.at)[j] + k;
        lens[q] = sl - k;
        toff[q] = ntok;
        ntok += count;
    }
    std::vector<uint32_t> toks(std::max<uint64_t>(ntok, 1));
    int rc = hs_batch_decode_blocks(batch, (uint32_t)mm, slots.data(), J.data, J.data_len, offs.data(), lens.data(),
                                    counts.data(), FREQ_BITS, toks.data(), ntok, toff.data(), status.data());
    if (rc) return rc;
    for (size_t q = 0; q < mm; q++) {
        const uint32_t j = (*J.coded)[r0 + q];
        if (status[q]) return corrupt(j, "an interval does not hold its target");
        const size_t o = (size_t)j * c.block_size;
        const size_t olen = (size_t)std::min<uint64_t>(c.block_size, J.seg_len - o);
        size_t w = 0;
        for (uint32_t t = 0; t < counts[q]; t++) {
            size_t nb;
            const uint32_t id = toks[toff[q] + t];
            const uint8_t* bytes = hs::token_bytes(J.tok, id, &nb);
            if (id == J.eot || nb == 0 || nb > olen - w) return corrupt(j, "the tokens do not give the block length");
            memcpy(J.restored + o + w, bytes, nb);
            w += nb;
        }
        if (w != olen) return corrupt(j, "the tokens do not give the block length");
    }
    return HS_OK;
}

int corrupt_block(uint64_t i, const std::string& why) {
    return hs::host_fail(HS_CORRUPT, "block " + std::to_string(i) + " is corrupt: " + why);
}

// The GPU side of an unfold: decodes every coded block of a job.
class UnfoldGpu {
  public:
    virtual ~UnfoldGpu() = default;
    virtual int set_overlap(uint16_t k) = 0;
    virtual int run(const CodedJob& J) = 0;
};

// hs_unfold: the caller's batch, rounds of up to min(slots, max_rows) blocks in order.
class OneDecoder : public UnfoldGpu {
  public:
    explicit OneDecoder(hs_batch* b) : b_(b) {}
    int set_overlap(uint16_t k) override { return hs_batch_set_overlap(b_, k); }
    int run(const CodedJob& J) override {
        const size_t per = std::max<size_t>(1, std::min(hs::batch_slots(b_), hs::batch_max_rows(b_)));
        for (size_t r0 = 0; r0 < J.coded->size(); r0 += per) {
            uint64_t bad = 0;
            std::string why;
            const int rc = decode_round(b_, J, r0, std::min(J.coded->size(), r0 + per), &bad, &why);
            if (rc == HS_CORRUPT) return corrupt_block(bad, why);
            if (rc) return rc;
        }
        return HS_OK;
    }

  private:
    hs_batch* b_;
};

// hs_unfold_multi: worker threads (each with its device, model and batch, made once) take rounds of
// the job's coded blocks from one counter, as the GPU fold's threads take windows
// (crates/taco/src/gpu_unfold.rs:74-200 deals the blocks of a job to the lanes). Several corrupt
// blocks report the one with the lowest index, so the error does not depend on the dealing
// (unfold.rs decode_group). Workers that cannot open give their share to the others. The workers
// start at the first segment with coded blocks: a container of raw and zstd blocks opens no GPU.
class MultiDecoder : public UnfoldGpu {
  public:
    MultiDecoder(const std::vector<int>& ords, const uint8_t* model_file, size_t model_len, const uint8_t* hash,
                 uint32_t slots, uint32_t max_rows)
        : ords_(ords), file_(model_file), len_(model_len), hash_(hash), slots_(slots), rows_(max_rows),
          rcs_(ords.size(), HS_OK), msgs_(ords.size()), live_(ords.size(), 0) {}

    ~MultiDecoder() override {
        {
            std::lock_guard<std::mutex> lk(mu_);
            quit_ = true;
        }
        cv_.notify_all();
        for (auto& t : threads_) t.join();
    }

    int start() {
        for (size_t g = 0; g < ords_.size(); g++) threads_.emplace_back([this, g] { worker(g); });
        std::unique_lock<std::mutex> lk(mu_);
        cv_.wait(lk, [&] { return tried_ == ords_.size(); });
        size_t ok = 0;
        for (char l : live_) ok += l;
        if (!ok) return hs::host_fail(rcs_[0], "no GPU of the unfold opened: " + msgs_[0]);
        n_live_ = ok;
        return HS_OK;
    }

    int set_overlap(uint16_t k) override {
        overlap_ = k;
        return HS_OK;
    }

    int run(const CodedJob& J) override {
        if (!started_) {
            started_ = true;
            if ((start_rc_ = start())) return start_rc_;
        }
        if (start_rc_) return start_rc_;
        std::unique_lock<std::mutex> lk(mu_);
        job_ = &J;
        next_ = 0;
        bad_ = UINT64_MAX;
        busy_ = n_live_;
        gen_++;
        cv_.notify_all();
        cv_.wait(lk, [&] { return busy_ == 0; });
        for (size_t g = 0; g < ords_.size(); g++)
            if (live_[g] && rcs_[g]) return hs::host_fail(rcs_[g], "GPU " + std::to_string(ords_[g]) + ": " + msgs_[g]);
        if (bad_ != UINT64_MAX) return corrupt_block(bad_, bad_why_);
        return HS_OK;
    }

  private:
    void note(size_t g, int rc) {  // under mu_
        char buf[1024];
        hs_last_error(buf, sizeof buf);
        msgs_[g] = buf;
        rcs_[g] = rc;
    }

    void worker(size_t g) {
        hs_dev* dev = nullptr;
        hs_model* model = nullptr;
        hs_batch* batch = nullptr;
        int rc = hs_open(ords_[g], &dev);
        if (!rc) rc = hs_model_load(dev, file_, len_, &model);
        hs_model_info mi;
        if (!rc && !(rc = hs_model_get_info(model, &mi)) && memcmp(mi.hash, hash_, 32) != 0)
            rc = hs::host_fail(HS_MODEL, "the loaded model is not the model file");
        if (!rc) rc = hs_batch_new(model, slots_, rows_, &batch);
        {
            std::lock_guard<std::mutex> lk(mu_);
            if (rc) note(g, rc);
            live_[g] = rc == HS_OK;
            tried_++;
        }
        cv_.notify_all();
        uint64_t seen = 0;
        while (!rc) {
            const CodedJob* J;
            {
                std::unique_lock<std::mutex> lk(mu_);
                cv_.wait(lk, [&] { return quit_ || gen_ != seen; });
                if (quit_) break;
                seen = gen_;
                J = job_;
            }
            int r = hs_batch_set_overlap(batch, overlap_);
            const size_t per = std::max<size_t>(1, std::min<size_t>(slots_, rows_));
            uint64_t my_bad = UINT64_MAX;
            std::string my_why;
            while (!r) {
                const size_t r0 = next_.fetch_add(per);
                if (r0 >= J->coded->size()) break;
                uint64_t bad = 0;
                std::string why;
                const int d = decode_round(batch, *J, r0, std::min(J->coded->size(), r0 + per), &bad, &why);
                if (d == HS_CORRUPT) {
                    if (bad < my_bad) my_bad = bad, my_why = why;
                } else {
                    r = d;
                }
            }
            {
                std::lock_guard<std::mutex> lk(mu_);
                if (r) note(g, r);
                if (my_bad < bad_) bad_ = my_bad, bad_why_ = my_why;
                busy_--;
            }
            cv_.notify_all();
            rc = r;
        }
        if (batch) hs_batch_free(batch);
        if (model) hs_model_free(model);
        if (dev) hs_dev_free(dev);
    }

    std::vector<int> ords_;
    const uint8_t* file_;
    size_t len_;
    const uint8_t* hash_;
    uint32_t slots_, rows_;
    std::vector<int> rcs_;
    std::vector<std::string> msgs_;
    std::vector<char> live_;
    std::vector<std::thread> threads_;
    std::mutex mu_;
    std::condition_variable cv_;
    size_t tried_ = 0, n_live_ = 0, busy_ = 0;
    uint64_t gen_ = 0;
    bool quit_ = false;
    uint16_t overlap_ = 0;
    const CodedJob* job_ = nullptr;
    bool started_ = false;
    int start_rc_ = HS_OK;
    std::atomic<size_t> next_{0};
    uint64_t bad_ = UINT64_MAX;
    std::string bad_why_;
};

// taco::unfold segment by segment (crates/taco/src/stream.rs StreamUnfold::from_seekable and
// from_reader): the whole table is checked before any output, and with a known length `n` the
// container length too; then each segment's stored bytes are read, its raw blocks copied, its
// zstd blocks decoded on the host, its coded blocks on the GPUs, and its bytes written out; the
// SHA-256 of all of them is checked at the end. With n = LEN_UNKNOWN (a pipe) a missing byte is
// an error where the segment that needs it is read, and a byte after the last block an error at
// the end, so the output can hold restored bytes before the error. `hash` and `eot` are those of
// the model (the container must name it, if it names one).
int unfold_stream_impl(UnfoldGpu& gpu, const uint8_t* hash, uint32_t eot, const hs_tokenizer* tok, ReadAt& in,
                       uint64_t n, Writer& out) {
    const bool known = n != LEN_UNKNOWN;
    Header c;
    int rc = parse_header(in, n, c);
    if (rc) return rc;
    // unfold.rs:157-180 checked_model: a container that names a model needs that model.
    if (c.needs_model && memcmp(c.model_hash, hash, 32) != 0)
        return hs::host_fail(HS_MODEL_MISMATCH, "the container was folded with another model");
    std::vector<uint8_t> kinds;
    std::vector<uint32_t> stored;
    const uint64_t table_end = c.hlen + 5 * (uint64_t)c.count;
    if (n < table_end) return bad_container("truncated block table");
    in.keep(table_end);
    uint64_t total = table_end;
    for (uint32_t g = 0; g < c.count; g += TABLE_GROUP) {
        const uint32_t m = std::min<uint32_t>(TABLE_GROUP, c.count - g);
        if ((rc = read_table(in, c, g, m, kinds, stored))) return rc;
        for (uint32_t j = 0; j < m; j++) {
            if (kinds[j] == 3)
                return hs::host_fail(HS_UNSUPPORTED, "block " + std::to_string(g + j) +
                                                         " is a mixed block (profile logs): its unfold needs the "
                                                         "match model and the mixer of the caller");
            total += stored[j];
        }
    }
    if (known && total > n) return bad_container("truncated block");
    if (known && total < n) return bad_container("extra bytes after the last block");
    if ((rc = gpu.set_overlap(c.overlap))) return rc;
    const uint64_t seg_blocks = std::min<uint64_t>(std::max<uint64_t>(SEGMENT_BYTES / c.block_size, 1), SEGMENT_BLOCKS);
    hs::Sha256 sum;
    std::vector<uint8_t> data, restored;
    std::vector<uint64_t> at;
    uint64_t pos = table_end;
    for (uint64_t first = 0; first < c.count; first += seg_blocks) {
        const uint32_t m = (uint32_t)std::min<uint64_t>(seg_blocks, c.count - first);
        if ((rc = read_table(in, c, (uint32_t)first, m, kinds, stored))) return rc;
        at.resize(m);
        uint64_t seg_stored = 0;
        for (uint32_t j = 0; j < m; j++) {
            at[j] = seg_stored;
            seg_stored += stored[j];
        }
        data.resize((size_t)seg_stored);
        if (seg_stored && in.read(pos, data.data(), data.size())) return bad_container("truncated block");
        pos += seg_stored;
        const uint64_t o0 = first * c.block_size;
        const uint64_t seg_len = std::min<uint64_t>((uint64_t)m * c.block_size, c.original_len - o0);
        restored.resize((size_t)seg_len);
        // Raw and zstd blocks on the host; the coded ones collected for the GPUs.
        std::vector<uint32_t> coded;
        for (uint32_t j = 0; j < m; j++) {
            const size_t o = (size_t)j * c.block_size;
            const size_t olen = (size_t)std::min<uint64_t>(c.block_size, seg_len - o);
            if (kinds[j] == KIND_RAW) memcpy(restored.data() + o, data.data() + at[j], olen);
            else if (kinds[j] == KIND_ZSTD &&
                     !decompress_zstd(data.data() + at[j], stored[j], restored.data() + o, olen))
                // A format error in the reference (unfold.rs:93, FormatError::CorruptZstdBlock),
                // not a corrupt coded block.
                return bad_container("the zstd frame of block " + std::to_string(first + j) +
                                     " does not give the block (CorruptZstdBlock)");
            else if (kinds[j] == KIND_CODED) coded.push_back(j);
        }
        if (!coded.empty()) {
            const CodedJob J{&c, tok, eot, data.data(), data.size(), &at, &stored, &coded, first, seg_len,
                             restored.data()};
            if ((rc = gpu.run(J))) return rc;
        }
        sum.update(restored.data(), restored.size());
        if (out.write(restored.data(), restored.size())) return hs::host_fail(HS_IO, "the output writer failed");
    }
    if (!known) {
        uint8_t one;
        if (in.read(pos, &one, 1) == 0) return bad_container("extra bytes after the last block");
        if (in.failed()) return hs::host_fail(HS_IO, "the input source failed");
    }
    uint8_t got[32];
    sum.final(got);
    if (memcmp(got, c.checksum, 32) != 0)
        return hs::host_fail(HS_CORRUPT, "the restored bytes do not have the container's SHA-256");
    return HS_OK;
}

// hs_unfold, hs_unfold_stream and hs_unfold_pipe on the caller's batch.
int unfold_one(hs_batch* batch, const hs_tokenizer* tok, ReadAt& in, uint64_t n, Writer& out) {
    hs_model_info info;
    int rc = hs_model_get_info(hs::batch_model(batch), &info);
    if (rc) return rc;
    OneDecoder gpu(batch);
    rc = unfold_stream_impl(gpu, info.hash, info.eot_token, tok, in, n, out);
    if (rc && in.failed()) return hs::host_fail(HS_IO, "the input source failed");
    return rc;
}

// hs_unfold_multi, hs_unfold_stream_multi and hs_unfold_pipe_multi: worker threads on the GPUs of
// `ordinals`, which start at the first segment with coded blocks.
int unfold_many(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len, uint32_t slots,
                uint32_t max_rows, const hs_tokenizer* tok, ReadAt& in, uint64_t n, Writer& out) {
    uint32_t vocab, eot, n_ctx;
    {
        std::string err;
        if (!hs::model_file_info(model_file, model_len, &vocab, &eot, &n_ctx, err))
            return hs::host_fail(HS_MODEL, "the model file is not valid: " + err);
    }
    int rc = check_tokenizer(tok, vocab);
    if (rc) return rc;
    uint8_t hash[32];
    hs::sha256(model_file, model_len, hash);
    // Two worker threads per GPU, as the fold (HS_FOLD_WORKERS_PER_GPU).
    uint32_t per = 2;
    if (const char* v = getenv("HS_FOLD_WORKERS_PER_GPU")) per = (uint32_t)std::min(8, std::max(1, atoi(v)));
    std::vector<int> ords;
    for (uint32_t k = 0; k < per; k++) ords.insert(ords.end(), ordinals, ordinals + n_gpus);
    MultiDecoder gpu(ords, model_file, model_len, hash, slots, max_rows);
    rc = unfold_stream_impl(gpu, hash, eot, tok, in, n, out);
    if (rc && in.failed()) return hs::host_fail(HS_IO, "the input source failed");
    return rc;
}

}  // namespace

extern "C" {

int hs_unfold(hs_batch* batch, const hs_tokenizer* tok, const uint8_t* container, size_t len, uint8_t* out,
              size_t cap, size_t* out_len) {
    if (!batch || !tok || !out_len || (len && !container)) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    MemReadAt in(container, len);
    Header c;
    int rc = parse_header(in, len, c);
    if (rc) return rc;
    *out_len = (size_t)c.original_len;
    if (cap < c.original_len || (!out && c.original_len))
        return hs::host_fail(HS_BAD_ARGUMENT, "the output holds " + std::to_string(cap) + " bytes, " +
                                                  std::to_string(c.original_len) + " needed");
    MemWriter w(out, cap);
    return unfold_one(batch, tok, in, len, w);
}

int hs_unfold_stream(hs_batch* batch, const hs_tokenizer* tok, uint64_t len, hs_read_at_fn read_at, void* read_user,
                     hs_write_fn write, void* write_user, uint64_t* out_len) {
    if (!batch || !tok || !read_at || !write || !out_len) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackReadAt in(read_at, read_user);
    Header c;
    int rc = parse_header(in, len, c);
    if (rc) return rc;
    *out_len = c.original_len;
    CallbackWriter w(write, write_user);
    return unfold_one(batch, tok, in, len, w);
}

int hs_unfold_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len, uint32_t slots,
                    uint32_t max_rows, const hs_tokenizer* tok, const uint8_t* container, size_t len, uint8_t* out,
                    size_t cap, size_t* out_len) {
    if (!ordinals || !n_gpus || !model_file || !tok || !out_len || (len && !container))
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    MemReadAt in(container, len);
    Header c;
    int rc = parse_header(in, len, c);
    if (rc) return rc;
    *out_len = (size_t)c.original_len;
    if (cap < c.original_len || (!out && c.original_len))
        return hs::host_fail(HS_BAD_ARGUMENT, "the output holds " + std::to_string(cap) + " bytes, " +
                                                  std::to_string(c.original_len) + " needed");
    MemWriter w(out, cap);
    return unfold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, in, len, w);
}

int hs_unfold_stream_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                           uint32_t slots, uint32_t max_rows, const hs_tokenizer* tok, uint64_t len,
                           hs_read_at_fn read_at, void* read_user, hs_write_fn write, void* write_user,
                           uint64_t* out_len) {
    if (!ordinals || !n_gpus || !model_file || !tok || !read_at || !write || !out_len)
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    CallbackReadAt in(read_at, read_user);
    Header c;
    int rc = parse_header(in, len, c);
    if (rc) return rc;
    *out_len = c.original_len;
    CallbackWriter w(write, write_user);
    return unfold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, in, len, w);
}

int hs_unfold_pipe(hs_batch* batch, const hs_tokenizer* tok, hs_source_fn source, void* source_user, hs_write_fn write,
                   void* write_user, uint64_t* out_len) {
    if (!batch || !tok || !source || !write || !out_len) return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    PipeReadAt in(source, source_user);
    Header c;
    int rc = parse_header(in, LEN_UNKNOWN, c);
    if (rc) return in.failed() ? hs::host_fail(HS_IO, "the input source failed") : rc;
    *out_len = c.original_len;
    CallbackWriter w(write, write_user);
    return unfold_one(batch, tok, in, LEN_UNKNOWN, w);
}

int hs_unfold_pipe_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                         uint32_t slots, uint32_t max_rows, const hs_tokenizer* tok, hs_source_fn source,
                         void* source_user, hs_write_fn write, void* write_user, uint64_t* out_len) {
    if (!ordinals || !n_gpus || !model_file || !tok || !source || !write || !out_len)
        return hs::host_fail(HS_BAD_ARGUMENT, "null argument");
    PipeReadAt in(source, source_user);
    Header c;
    int rc = parse_header(in, LEN_UNKNOWN, c);
    if (rc) return in.failed() ? hs::host_fail(HS_IO, "the input source failed") : rc;
    *out_len = c.original_len;
    CallbackWriter w(write, write_user);
    return unfold_many(ordinals, n_gpus, model_file, model_len, slots, max_rows, tok, in, LEN_UNKNOWN, w);
}

}  // extern "C"
