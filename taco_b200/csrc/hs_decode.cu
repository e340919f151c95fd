// The range decoder of taco-coder on the device, for the batched unfold of coded blocks.
//
// The reference unfolds a coded block on the host (crates/taco/src/gpu_unfold.rs:100-160 with
// crates/taco/src/codec.rs BlockDecoder): for every token it asks the decoder for the target
// t = min(code / (range >> bits), 2^bits - 1) (crates/taco-coder/src/decoder.rs:75-80), runs the
// coder op with a decode query for t, checks that the returned interval holds t and consumes it
// (decoder.rs:91-106), and feeds the symbol back as the next input. Here the decoder state of
// every block lives in device memory and these kernels do both halves around the forward pass
// and the coder op, so the host need not wait for each step.
//
// The arithmetic is the reference's, unchanged: INITIAL_RANGE = 2^64 - 1, TOP = 2^56, the first
// 8 bytes read big-endian into `code`, zero bytes past the end of the input, renormalisation by
// bytes while range < TOP (decoder.rs:29-35, 139-146).
#include <cuda_runtime.h>

#include <cstdint>

#include "hs_common.cuh"
#include "hs_kernels.cuh"

namespace hs {

namespace {

constexpr uint64_t DEC_TOP = 1ULL << 56;

__device__ __forceinline__ uint8_t dec_byte(DecState& d, const uint8_t* payload) {
    if (d.pos < d.len) return payload[d.base + d.pos++];
    return 0;
}

__device__ __forceinline__ uint64_t dec_target(const DecState& d, uint32_t bits) {
    // range >= 2^56 and bits <= 32, so r >= 2^24.
    const uint64_t r = d.range >> bits;
    const uint64_t t = d.code / r;
    const uint64_t top = (bits >= 64 ? ~0ULL : (1ULL << bits)) - 1;
    return t < top ? t : top;
}

__global__ void k_dec_init(DecState* st, const uint8_t* payload, const uint64_t* offsets, const uint64_t* lengths,
                           uint32_t* prev, uint32_t eot, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    DecState d;
    d.base = offsets[i];
    d.len = lengths[i];
    d.pos = 0;
    d.code = 0;
    d.range = ~0ULL;
    d.failed = 0;
    d.pad = 0;
    for (int k = 0; k < 8; k++) d.code = (d.code << 8) | dec_byte(d, payload);
    st[i] = d;
    prev[i] = eot;
}

// The rows of one step: block i (i < R, the live blocks are a prefix) decodes in slot slot_of[i]
// at position pos_of[i] + steps_since, with the previous symbol (or EOT) as its input and its
// target as a decode query.
__global__ void k_dec_begin(const DecState* st, int R, const uint32_t* slot_of, const uint32_t* pos_of,
                            uint32_t steps_since, const uint32_t* prev, uint32_t bits, RowInfo* rows) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R) return;
    RowInfo ri;
    ri.slot = slot_of[i];
    ri.token = prev[i];
    ri.pos = pos_of[i] + steps_since;
    ri.kind = 1;
    ri.value = dec_target(st[i], bits);
    rows[i] = ri;
}

// The second half of a decode (decoder.rs:91-106): the interval of row i must hold the block's
// target; then the state takes it and reads its bytes. A block whose interval does not hold its
// target is marked failed and keeps its state (its later symbols mean nothing; the host reports
// the block as failed). The symbol becomes the block's next input and its output token.
__global__ void k_dec_end(DecState* st, int R, const uint64_t* intervals, uint32_t bits, uint32_t V,
                          const uint8_t* payload, uint32_t* prev, uint32_t* out, const uint64_t* out_off,
                          uint32_t step) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= R) return;
    DecState d = st[i];
    const uint32_t sym = (uint32_t)intervals[3 * (size_t)i];
    const uint64_t start = intervals[3 * (size_t)i + 1];
    const uint64_t freq = intervals[3 * (size_t)i + 2];
    if (!d.failed) {
        const uint64_t t = dec_target(d, bits);
        if (t < start || t - start >= freq) {
            d.failed = 1;
        } else {
            const uint64_t r = d.range >> bits;
            const uint64_t offset = r * start;
            d.code -= offset;
            d.range = sym + 1 == V ? d.range - offset : r * freq;
            while (d.range < DEC_TOP) {
                d.range <<= 8;
                d.code = (d.code << 8) | dec_byte(d, payload);
            }
        }
    }
    st[i] = d;
    prev[i] = sym;
    out[out_off[i] + step] = sym;
}

// The targets of the first R blocks into a plain array (the host path of a restart step).
__global__ void k_dec_targets(const DecState* st, int R, uint32_t bits, uint64_t* targets) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < R) targets[i] = dec_target(st[i], bits);
}

// The symbols of steps [s0, s1) of the first L blocks, packed [L][s1 - s0] for one read back
// (0 past a block's end).
__global__ void k_dec_gather(const uint32_t* out, const uint64_t* out_off, const uint32_t* counts, int L, uint32_t s0,
                             uint32_t s1, uint32_t* dst) {
    const uint32_t w = s1 - s0;
    const size_t k = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (k >= (size_t)L * w) return;
    const int i = (int)(k / w);
    const uint32_t s = s0 + (uint32_t)(k - (size_t)i * w);
    dst[k] = s < counts[i] ? out[out_off[i] + s] : 0u;
}

// The failed flags of the n blocks.
__global__ void k_dec_status(const DecState* st, int n, uint32_t* status) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) status[i] = st[i].failed;
}

}  // namespace

void launch_dec_init(DecState* st, const uint8_t* payload, const uint64_t* offsets, const uint64_t* lengths,
                     uint32_t* prev, uint32_t eot, int n, cudaStream_t s) {
    if (n > 0) k_dec_init<<<(n + 127) / 128, 128, 0, s>>>(st, payload, offsets, lengths, prev, eot, n);
}

void launch_dec_begin(const DecState* st, int R, const uint32_t* slot_of, const uint32_t* pos_of,
                      uint32_t steps_since, const uint32_t* prev, uint32_t bits, RowInfo* rows, cudaStream_t s) {
    if (R > 0) k_dec_begin<<<(R + 127) / 128, 128, 0, s>>>(st, R, slot_of, pos_of, steps_since, prev, bits, rows);
}

void launch_dec_end(DecState* st, int R, const uint64_t* intervals, uint32_t bits, uint32_t V, const uint8_t* payload,
                    uint32_t* prev, uint32_t* out, const uint64_t* out_off, uint32_t step, cudaStream_t s) {
    if (R > 0)
        k_dec_end<<<(R + 127) / 128, 128, 0, s>>>(st, R, intervals, bits, V, payload, prev, out, out_off, step);
}

void launch_dec_targets(const DecState* st, int R, uint32_t bits, uint64_t* targets, cudaStream_t s) {
    if (R > 0) k_dec_targets<<<(R + 127) / 128, 128, 0, s>>>(st, R, bits, targets);
}

void launch_dec_gather(const uint32_t* out, const uint64_t* out_off, const uint32_t* counts, int L, uint32_t s0,
                       uint32_t s1, uint32_t* dst, cudaStream_t s) {
    const size_t total = (size_t)L * (s1 - s0);
    if (total > 0) k_dec_gather<<<(unsigned)((total + 255) / 256), 256, 0, s>>>(out, out_off, counts, L, s0, s1, dst);
}

void launch_dec_status(const DecState* st, int n, uint32_t* status, cudaStream_t s) {
    if (n > 0) k_dec_status<<<(n + 127) / 128, 128, 0, s>>>(st, n, status);
}

}  // namespace hs
