/* The C ABI of the B200 HardShell backend (libhardshell_b200.so).
 *
 * It replaces the CUDA engine of the reference, crates/hardshell-cuda, behind the interface that
 * crates/taco uses for a GPU backend (the `Lanes` trait, crates/taco/src/lanes.rs:61-113). Every
 * entry point names the reference function it replaces. Plain pointers and sizes only: the caller
 * owns every host array, the library copies in and out and owns the device memory.
 *
 * Handles nest as in the reference: a device outlives its models, a model outlives its batches.
 * A device handle is bound to the host thread that opened it (crates/hardshell-cuda/src/device.rs:9:
 * "use it on one thread"); use one thread per GPU.
 *
 * Every function returns a status (HS_OK = 0) unless its comment says otherwise; on an error,
 * hs_last_error() gives the message of the calling thread. After a failed run, no slot position
 * changed (crates/hardshell-cuda/src/batch.rs:443-446).
 */
#ifndef HARDSHELL_B200_H
#define HARDSHELL_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes; they mirror crates/hardshell-cuda/src/error.rs:9-50 (enum Error). */
enum hs_status {
    HS_OK = 0,
    HS_NO_DEVICE = 1,       /* Error::NoDevice: no driver or no such device */
    HS_CUDA = 2,            /* Error::Cuda: a CUDA call or a kernel failed */
    HS_UNSUPPORTED = 3,     /* Error::Unsupported: the device, model or request shape */
    HS_MODEL = 4,           /* Error::Model: the model file is not valid */
    HS_BAD_SLOT = 5,        /* Error::BadSlot */
    HS_LENGTH_MISMATCH = 6, /* Error::LengthMismatch */
    HS_TOKEN_RANGE = 7,     /* Error::Model(TokenOutOfRange) */
    HS_INVALID_OVERLAP = 8, /* Error::Model(InvalidOverlap) */
    HS_BAD_ARGUMENT = 9,    /* a null pointer or a size out of range */
    HS_FORMAT = 10,         /* TacoError::Format: the container breaks a rule of the format */
    HS_CORRUPT = 11,        /* TacoError::CorruptBlock / ChecksumMismatch: a block or the output is wrong */
    HS_MODEL_MISMATCH = 12, /* TacoError::ModelHashMismatch: the container names another model */
    HS_IO = 13              /* TacoError::Io / StreamError: a source, sink or writer of the caller failed,
                               or the input is shorter or longer than its length */
};

typedef struct hs_dev hs_dev;
typedef struct hs_model hs_model;
typedef struct hs_batch hs_batch;

/* The answer of the coder op for one input: a symbol and its interval in the table of
 * taco_coder::FreqTable::from_weights(weights, freq_bits) (crates/hardshell-cuda/src/batch.rs:47
 * CoderInterval). is_last is 1 when the symbol is the last symbol of the table. 32 bytes. */
typedef struct hs_interval {
    uint32_t symbol;
    uint32_t is_last;
    uint64_t start;
    uint64_t freq;
    uint64_t reserved;
} hs_interval;

/* Model dimensions (crates/hardshell/src/gpt2/model.rs:87 Dims and the header constants). */
typedef struct hs_model_info {
    uint32_t n_layer, n_head, d_model, d_ff, vocab, n_ctx, eot_token, version;
    uint64_t cache_bytes_per_slot; /* crates/hardshell-cuda/src/model.rs:395 */
    uint64_t weight_bytes;         /* crates/hardshell-cuda/src/model.rs:389 */
    uint8_t hash[32];              /* SHA-256 of the model file (model.rs:359) */
} hs_model_info;

/* CudaDevice::open (crates/hardshell-cuda/src/device.rs:29). HS_NO_DEVICE without a device,
 * HS_UNSUPPORTED below compute capability 10.0 (the kernels are sm_100a). For tests of the
 * callers' fallback, the environment variable HS_FAIL_OPEN (a comma-separated list of ordinals)
 * makes the open of those ordinals fail with HS_NO_DEVICE before any CUDA call. */
int hs_open(int ordinal, hs_dev** out);
void hs_dev_free(hs_dev* dev);
/* CudaDevice::memory (device.rs:58): free and total bytes. */
int hs_mem_info(hs_dev* dev, uint64_t* free_bytes, uint64_t* total_bytes);
/* CudaDevice::name (device.rs:43): the device name, NUL-terminated, cut to `cap` bytes. */
int hs_dev_name(hs_dev* dev, char* buf, size_t cap);

/* CudaModel::load (crates/hardshell-cuda/src/model.rs:242): validates the .hsm bytes as
 * hardshell::gpt2::Model::load does (crates/hardshell/src/gpt2/model.rs:292) and uploads the
 * weights. The bytes are copied. HS_MODEL for an invalid file, HS_UNSUPPORTED for a valid model
 * this backend does not run (see the message). */
int hs_model_load(hs_dev* dev, const uint8_t* file, size_t len, hs_model** out);
/* hardshell::gpt2::Model::load (crates/hardshell/src/gpt2/model.rs:292) on the host alone: the
 * checks of hs_model_load without a device or an upload. HS_MODEL for an invalid file; else the
 * dimensions, version, cache bytes per slot and SHA-256 (weight_bytes is 0: it depends on the
 * device layout). */
int hs_model_check(const uint8_t* file, size_t len, hs_model_info* out);
void hs_model_free(hs_model* model);
int hs_model_get_info(hs_model* model, hs_model_info* out);

/* CudaBatch::new (crates/hardshell-cuda/src/batch.rs:237): `slots` sessions with their KV
 * caches and passes of at most `max_rows` rows (a max_rows of 1 becomes 2). */
int hs_batch_new(hs_model* model, uint32_t slots, uint32_t max_rows, hs_batch** out);
void hs_batch_free(hs_batch* batch);
/* CudaBatch::set_overlap (batch.rs:354): the context overlap K <= n_ctx - 2 of every slot. */
int hs_batch_set_overlap(hs_batch* batch, uint16_t k);
/* CudaBatch::reset (batch.rs:397): empties the context of `slot`. */
int hs_batch_reset(hs_batch* batch, uint32_t slot);
/* CudaBatch::position (batch.rs:391): the tokens in the context of `slot` (0 if not valid). */
uint32_t hs_batch_position(hs_batch* batch, uint32_t slot);
/* CudaBatch::gpu_bytes (batch.rs:385). */
uint64_t hs_batch_gpu_bytes(hs_batch* batch);

/* CudaBatch::run_coded (batch.rs:463): runs the n inputs (slots[i], tokens[i]) and answers
 * query i: kinds[i] = 0 (Encode) gives the interval of token values[i]; kinds[i] = 1 (Decode)
 * gives the symbol whose interval holds target values[i] < 2^freq_bits. The rows of one slot run
 * at consecutive positions (prefill); a full context starts again with the overlap. Only the
 * intervals come back (32 bytes per input). */
int hs_batch_run_coded(hs_batch* batch, const uint32_t* slots, const uint32_t* tokens, const uint32_t* kinds,
                       const uint64_t* values, uint32_t n, uint32_t freq_bits, hs_interval* out);

/* CudaBatch::run_weights (batch.rs:447): the vocab weights of every input, n * vocab u64. */
int hs_batch_run_weights(hs_batch* batch, const uint32_t* slots, const uint32_t* tokens, uint32_t n,
                         uint64_t* out);

/* The mixed coder op of the profile `logs` (crates/hardshell-cuda/src/mixed.rs, batch/mixed.rs).
 * The table word of an input: a predicted token (the table of the mixed weights of
 * taco_match::Mixer::mix, mixer.rs:491-516), HS_MIX_NONE (a mixed table without a prediction:
 * the weights max(1, w)) or HS_MIX_PLAIN (the table of GPT-2 alone, as hs_batch_run_coded). */
#define HS_MIX_NONE 0xFFFFFFFFu
#define HS_MIX_PLAIN 0xFFFFFFFEu

/* What the host mixer needs from the GPT-2 weights w of one input (mixed.rs:36-47 MixStats):
 * total = sum(w), predicted = w[p], top = the token with the largest weight (the lowest id on a
 * tie, 0 if every weight is 0). 24 bytes. */
typedef struct hs_mix_stats {
    uint64_t total;
    uint64_t predicted;
    uint32_t top;
    uint32_t reserved;
} hs_mix_stats;

/* The host mixer: gives q, the probability of the predicted token in units of 2^-16 (1..=65535),
 * for input `input` from its statistics (rules 2 to 4 of the mixer: W = total, w[p] = predicted,
 * agreement = top == p). Called in input order, once for each input with a predicted token, so
 * the caller can update its mixer state between calls. A q outside 1..=65535 fails the call. */
typedef uint32_t (*hs_mixer_fn)(void* user, uint32_t input, const hs_mix_stats* stats);

/* CudaBatch::run_coded_mixed (batch/mixed.rs:71-109): runs the inputs as hs_batch_run_coded, but
 * answers query i in the table that tables[i] names. For each pass: the forward pass, the
 * statistics of every row (one more kernel and a read back of 24 bytes per row), the mixer calls,
 * the mix records (32 bytes per row up), and the mixed coder kernel. Errors: those of
 * hs_batch_run_coded; HS_UNSUPPORTED if a table word is not a token, HS_MIX_NONE or HS_MIX_PLAIN,
 * or if `mixer` gives a q outside 1..=65535. After an error no position changed, but `mixer` can
 * have been called: the caller must drop its mixer state. */
int hs_batch_run_coded_mixed(hs_batch* batch, const uint32_t* slots, const uint32_t* tokens, const uint32_t* kinds,
                             const uint64_t* values, const uint32_t* tables, uint32_t n, uint32_t freq_bits,
                             hs_mixer_fn mixer, void* user, hs_interval* out);

/* CudaBatch::run_coded_dual (batch/mixed.rs:109-135): the two intervals of coded[i] for the
 * encoder of the profile `logs`, in the table of GPT-2 alone (plain_out[i]) and in the mixed
 * table of predictions[i] (mixed_out[i]; a token or HS_MIX_NONE). `mixer` is called as for
 * hs_batch_run_coded_mixed. */
int hs_batch_run_coded_dual(hs_batch* batch, const uint32_t* slots, const uint32_t* tokens, const uint32_t* coded,
                            const uint32_t* predictions, uint32_t n, uint32_t freq_bits, hs_mixer_fn mixer,
                            void* user, hs_interval* plain_out, hs_interval* mixed_out);

/* CudaBatch::stream_len (batch/stream.rs:17-21): the inputs of `slot` since its last reset (the
 * EOT row of a block start is one input; the rows of a context restart are not). */
int hs_batch_stream_len(hs_batch* batch, uint32_t slot, uint64_t* len);
/* CudaBatch::room (batch/stream.rs:23-33, StreamState::room): the inputs `slot` can take before
 * its next context restart; a draft of at most this many rows never needs a rebuild at a
 * truncation. */
int hs_batch_room(hs_batch* batch, uint32_t slot, uint64_t* room);
/* CudaBatch::truncate (batch/stream.rs:35-77), the engine side of speculative decoding: the
 * slot keeps its first `len` inputs and then gives the weights of a slot that ran only those,
 * bit for bit (crates/hardshell/src/gpt2/stream.rs rules). Inside the current context only the
 * position moves back; before the last context restart the slot takes back the old context and
 * runs the rows that the new context overwrote again (no read back). Errors: HS_BAD_SLOT;
 * HS_MODEL (BadTruncate) if len is more than the stream length or before the restart before
 * the last one. The slot does not change on an error. */
int hs_batch_truncate(hs_batch* batch, uint32_t slot, uint64_t len);

/* The unfold of n coded blocks with the range decoder on the device. It replaces the host loop
 * of crates/taco/src/gpu_unfold.rs:100-160 (codec.rs BlockDecoder over run_coded with Decode
 * queries, one host round trip per token) for the coded blocks of a job. Block i is reset into
 * slot slots[i] (distinct slots), takes EOT as its first input and each decoded symbol as its
 * next one, and decodes counts[i] tokens from its range-coded bytes
 * payload[offsets[i] .. offsets[i] + lengths[i]) (the bytes after the block's varint count),
 * each with the coder op at freq_bits (taco-coder decoder.rs target / decode_interval).
 * tokens_out[token_offsets[i] + j] receives its j-th symbol (the caller maps tokens to bytes
 * and checks the block's length, as BlockDecoder::finish does). status[i] (may be NULL) is 0, or
 * 1 if an interval did not hold its target (the reference's TargetNotInInterval: the block is
 * corrupt; its tokens mean nothing). At most max_rows blocks per call. No counterpart call in the
 * reference: it is the GPU range coder of its "next" list. On an error the positions of the
 * call's slots are unspecified: reset them before reuse. */
int hs_batch_decode_blocks(hs_batch* batch, uint32_t n, const uint32_t* slots, const uint8_t* payload,
                           uint64_t payload_len, const uint64_t* offsets, const uint64_t* lengths,
                           const uint32_t* counts, uint32_t freq_bits, uint32_t* tokens_out, uint64_t tokens_cap,
                           const uint64_t* token_offsets, uint32_t* status);

/* ---- the host glue of the fold: no GPU needed ---- */

/* The tokenizer of a model (crates/taco/src/tokenizer/mod.rs Tokenizer::for_vocabulary): GPT-2
 * byte-level BPE over the vocabulary and the merges of the .hsm file. Any byte string tokenizes,
 * and the bytes of the tokens join to the input. HS_MODEL if the file is not valid, a byte has no
 * single token, or a merge is refused (the MergeFault cases of mod.rs:33-47). */
typedef struct hs_tokenizer hs_tokenizer;
int hs_tokenizer_new(const uint8_t* file, size_t len, hs_tokenizer** out);
void hs_tokenizer_free(hs_tokenizer* tokenizer);
/* Tokenizer::encode (mod.rs:180-200): the tokens of data[0 .. len) into out (at most len
 * tokens); *n = the token count. HS_BAD_ARGUMENT (with *n set) if cap is too small. */
int hs_tokenize(const hs_tokenizer* tokenizer, const uint8_t* data, size_t len, uint32_t* out, size_t cap,
                size_t* n);
/* The pieces of the pre-tokenizer (tokenizer/pretokenize.rs Pieces, and the single bytes outside
 * the well-formed UTF-8 runs): the end offset of each piece, in order. */
int hs_tokenizer_pieces(const hs_tokenizer* tokenizer, const uint8_t* data, size_t len, uint64_t* ends,
                        size_t cap, size_t* n);

/* The options of a fold (crates/taco/src/fold.rs FoldOptions, profile text). block_size 0 is
 * the default 16 KiB (lib.rs:101); with `spread` and no block size, the power of two that gives
 * about 64 blocks, within 4 KiB .. 16 KiB (fold.rs:159-170). overlap is the context overlap K
 * (the text profile's default is 0). threads: host threads for the tokenizer, zstd and the range
 * encoder (0 = all). */
typedef struct hs_fold_options {
    uint32_t block_size;
    uint32_t overlap;
    uint32_t spread;
    uint32_t threads;
} hs_fold_options;

/* FoldStats (fold.rs): the counts of one fold. */
typedef struct hs_fold_stats {
    uint64_t original_len, container_len, blocks, coded_blocks, zstd_blocks, tokens;
    uint32_t block_size;
    uint32_t gpus_failed; /* hs_fold_multi: the GPUs that did not open and gave their windows away */
    uint64_t gpu_rows;    /* the rows that ran on the GPUs (windows of stopped blocks never start) */
    /* Wall time of the stages, summed over the segments: the host threads' tokens and zstd frames
     * (overlapped with the GPU stage of the previous segment), the GPU stage (passes and the range
     * encoders), and the payloads, the stored forms and the writes. */
    double prep_ms, gpu_ms, finish_ms;
} hs_fold_stats;

/* The largest container of a fold of `len` bytes with this block size (0: the default or the
 * `spread` size, whichever gives the larger bound). UINT64_MAX if it does not fit in 64 bits. */
uint64_t hs_fold_bound(uint64_t len, uint32_t block_size);

/* taco::fold_with on the CUDA engine (fold.rs:334-360), profile text: the .taco container
 * (version 2) of input[0 .. len) with the model of `batch`. Each block is stored raw, as a zstd
 * frame or coded by the model, whichever is smallest (writer.rs:89). The coder intervals come from
 * hs_batch_run_coded: each block's context windows run in fresh slots, in waves (window 0 of every
 * block, then window 1, ...), and each block's range encoder takes its windows' intervals as they
 * complete; the later windows of a block whose encoder stopped do not run (gpu_fold.rs:200-204).
 * The tokenizer, zstd and the range encoder run on host threads. zstd comes from the system
 * library (libzstd.so.1, hs_zstd_version); the reference pins zstd 1.5.7, and a zstd frame of
 * another version can differ in its bytes (it decodes to the same block). *out_len = the container
 * length; HS_BAD_ARGUMENT if it is more than cap (see hs_fold_bound). The batch keeps the fold's
 * overlap, and its slots the contexts of the last windows. */
int hs_fold(hs_batch* batch, const hs_tokenizer* tokenizer, const uint8_t* input, size_t len,
            const hs_fold_options* options, uint8_t* out, size_t cap, size_t* out_len, hs_fold_stats* stats);

/* hs_fold on several GPUs of this host (crates/taco/src/gpu_fold.rs:128-186): one host thread
 * per GPU opens device ordinals[g], loads the model file, makes a batch of `slots` slots and
 * passes of `max_rows` rows, and runs the context windows dealt to it round-robin; the host
 * stages are shared; the GPUs take rounds of windows from one queue. The windows follow the
 * model file's context length and EOT token; the
 * tokenizer must have the model's vocabulary (HS_MODEL). A GPU that cannot be opened, load the
 * model or hold the batch gives its windows to the GPUs that can (stats->gpus_failed counts it),
 * as the reference falls back from a device that fails (crates/taco/src/backend.rs:288-342); with
 * no GPU left the call fails with the first GPU's error when the first windows are to run. The
 * GPUs open while the host tokenizes and compresses the first segment. An error while windows run
 * fails the call with that GPU's status and message. The container is the bytes hs_fold gives on
 * one GPU. */
int hs_fold_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                  uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, const uint8_t* input,
                  size_t len, const hs_fold_options* options, uint8_t* out, size_t cap, size_t* out_len,
                  hs_fold_stats* stats);

/* ---- streams: inputs of any size with bounded memory (crates/taco/src/stream.rs) ----
 *
 * The bytes are those of hs_fold and hs_unfold; the work moves in segments of blocks (at most 64
 * MiB of input and 4,096 blocks each), and a fold or unfold holds about two segments: the one on
 * the GPUs and the next one on the host threads. The callbacks are called on the caller's thread
 * only, in order. */

/* The input of a fold: fills buf with up to cap bytes and gives their count; 0 only at the end
 * of the input; < 0 on an error (the call fails with HS_IO). */
typedef int64_t (*hs_source_fn)(void* user, uint8_t* buf, size_t cap);
/* The output of a fold, seekable: writes buf[0 .. n) at offset `at`; 0, or non-zero on an error. */
typedef int (*hs_sink_fn)(void* user, uint64_t at, const uint8_t* buf, size_t n);
/* The container of an unfold: reads n bytes at offset `at` into buf; 0, or non-zero on an error. */
typedef int (*hs_read_at_fn)(void* user, uint64_t at, uint8_t* buf, size_t n);
/* The output of an unfold, in order: takes buf[0 .. n); 0, or non-zero on an error. */
typedef int (*hs_write_fn)(void* user, const uint8_t* buf, size_t n);

/* StreamFold::to_seekable (stream.rs:419-428): the fold of hs_fold of the `len` bytes that
 * `source` gives, into `sink`. The sink receives the block table and the stored blocks of each
 * segment as it ends, and the header (which holds the input's SHA-256) last; *out_len = the
 * container length. HS_IO if the source gives fewer or more than `len` bytes or a callback fails. */
int hs_fold_stream(hs_batch* batch, const hs_tokenizer* tokenizer, uint64_t len, hs_source_fn source,
                   void* source_user, hs_sink_fn sink, void* sink_user, const hs_fold_options* options,
                   uint64_t* out_len, hs_fold_stats* stats);

/* hs_fold_stream on several GPUs of this host, as hs_fold_multi. */
int hs_fold_stream_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                         uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, uint64_t len,
                         hs_source_fn source, void* source_user, hs_sink_fn sink, void* sink_user,
                         const hs_fold_options* options, uint64_t* out_len, hs_fold_stats* stats);

/* The length of a fold input that is not known before it ends (a pipe). */
#define HS_LEN_UNKNOWN UINT64_MAX

/* StreamFold::to_writer (stream.rs:430-452), the method "spool": the fold of hs_fold of the bytes
 * that `source` gives, into `write`, an output that cannot seek (a pipe). The stored blocks and
 * the table go to two temporary files in `spool_dir` (NULL: $TMPDIR, else /tmp), named
 * .taco-spool-<pid>-blocks-XXXXXX and -table-XXXXXX and unlinked as soon as they are made, so
 * they vanish when the call ends, after an error or a crash too; at the end the header, the
 * table and the blocks go to `write` in that order. The spool holds about the container's size.
 * `len` is the input length, or HS_LEN_UNKNOWN: then the source is read until it ends, and the
 * block size is options->block_size or the default (`spread` needs the length and is ignored).
 * HS_IO if the source gives fewer or more than a known `len` bytes, a temporary file cannot be
 * made or written, or a callback fails; HS_UNSUPPORTED past 2^32 - 1 blocks. The container is
 * the bytes of hs_fold_stream. hs_fold_stream refuses HS_LEN_UNKNOWN (HS_BAD_ARGUMENT): a
 * seekable output needs the table's size before the first block. */
int hs_fold_spool(hs_batch* batch, const hs_tokenizer* tokenizer, uint64_t len, hs_source_fn source,
                  void* source_user, hs_write_fn write, void* write_user, const char* spool_dir,
                  const hs_fold_options* options, uint64_t* out_len, hs_fold_stats* stats);

/* hs_fold_spool on several GPUs of this host, as hs_fold_multi. The GPUs open while the host
 * works on the first segment, and a fold whose blocks need no model window (blocks too short to
 * code) runs on no GPU. */
int hs_fold_spool_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                        uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, uint64_t len,
                        hs_source_fn source, void* source_user, hs_write_fn write, void* write_user,
                        const char* spool_dir, const hs_fold_options* options, uint64_t* out_len,
                        hs_fold_stats* stats);

/* StreamUnfold::from_seekable (stream.rs): the unfold of hs_unfold of the `len`-byte container
 * that `read_at` reads, into `write`. The header, the whole block table and the container length
 * are checked before any output; then each segment's bytes go to `write` in order. *out_len = the
 * original length (from the header). The SHA-256 is checked at the end: HS_CORRUPT then means
 * that the bytes already written are wrong. */
int hs_unfold_stream(hs_batch* batch, const hs_tokenizer* tokenizer, uint64_t len, hs_read_at_fn read_at,
                     void* read_user, hs_write_fn write, void* write_user, uint64_t* out_len);

/* hs_unfold_stream with the worker threads of hs_unfold_multi. */
int hs_unfold_stream_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                           uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, uint64_t len,
                           hs_read_at_fn read_at, void* read_user, hs_write_fn write, void* write_user,
                           uint64_t* out_len);

/* StreamUnfold::from_reader (stream.rs:809-827): the unfold of hs_unfold of the container that
 * `source` gives in one pass (a pipe), into `write`. The header and the whole block table are
 * read and checked before any output (they stay in memory: 5 bytes per block); the stored blocks
 * are then read in order. A missing byte is HS_FORMAT where the segment that needs it is read,
 * a byte after the last block HS_FORMAT at the end, so `write` can have taken restored bytes
 * before an error; the output is complete and correct only if the call returns HS_OK. HS_IO if
 * the source fails. *out_len = the original length (from the header). */
int hs_unfold_pipe(hs_batch* batch, const hs_tokenizer* tokenizer, hs_source_fn source, void* source_user,
                   hs_write_fn write, void* write_user, uint64_t* out_len);

/* taco::unfold on the CUDA engine (crates/taco/src/unfold.rs, profile text): the original bytes of
 * a .taco container (version 1 or 2) into out[0 .. *out_len). The header and the block table are
 * checked as crates/taco-format/src/reader.rs checks them (HS_FORMAT); a container that names a
 * model must name the model of `batch` (HS_MODEL_MISMATCH). Raw blocks are copied, zstd blocks
 * decoded (one frame, content size = the block length, window <= 8 MiB), coded blocks decoded on
 * the GPU by hs_batch_decode_blocks in rounds of min(slots, max_rows) blocks and turned into
 * bytes with the tokenizer's vocabulary; a block whose decoding fails or whose tokens do not give
 * its length, or output whose SHA-256 is not the header's, is HS_CORRUPT; a zstd frame that does
 * not give exactly its block is HS_FORMAT (FormatError::CorruptZstdBlock). Mixed blocks (profile
 * logs) are HS_UNSUPPORTED: their unfold needs the caller's match model and mixer. *out_len = the
 * original length; HS_BAD_ARGUMENT if it is more than cap. */
int hs_unfold(hs_batch* batch, const hs_tokenizer* tokenizer, const uint8_t* container, size_t len, uint8_t* out,
              size_t cap, size_t* out_len);

/* hs_unfold on several GPUs of this host: worker threads (two per GPU of `ordinals`, each with its
 * device, the model file loaded and a batch of `slots` slots and `max_rows` rows) take rounds of
 * each segment's coded blocks, as the reference deals the blocks of an unfold job to its lanes
 * (crates/taco/src/gpu_unfold.rs:74-200); raw and zstd blocks stay on the host. The output and the
 * errors are those of hs_unfold (several corrupt blocks report the lowest index). The workers
 * start at the first segment with coded blocks, so a container without any opens no GPU. */
int hs_unfold_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                    uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, const uint8_t* container,
                    size_t len, uint8_t* out, size_t cap, size_t* out_len);

/* hs_unfold_pipe with the worker threads of hs_unfold_multi. */
int hs_unfold_pipe_multi(const int* ordinals, uint32_t n_gpus, const uint8_t* model_file, size_t model_len,
                         uint32_t slots, uint32_t max_rows, const hs_tokenizer* tokenizer, hs_source_fn source,
                         void* source_user, hs_write_fn write, void* write_user, uint64_t* out_len);

/* The version of the zstd library that hs_fold uses (major * 10000 + minor * 100 + patch), or 0
 * if it is not available. */
uint32_t hs_zstd_version(void);

/* The message of the last error of the calling thread (NUL-terminated, cut to `cap`). */
int hs_last_error(char* buf, size_t cap);

/* The per-op device time of the passes that ran since profiling was switched on, as
 * CudaBatch::profile gives it (crates/hardshell-cuda/src/batch.rs:488-499): the reference marks
 * each op with a %globaltimer stamp, this backend brackets each launch with CUDA events on the
 * batch stream. `ops` is the algorithmic integer work of the op (2 per multiply-add). */
typedef struct hs_op_profile {
    char name[32];
    double ms;
    uint64_t launches;
    uint64_t ops;
} hs_op_profile;

/* Switches the profile on (1) or off (0) and clears it (batch.rs:488 profile). */
int hs_batch_set_profiling(hs_batch* batch, int on);
/* Fills up to `cap` op entries; returns their number (0 when profiling is off), or < 0 on error. */
int hs_batch_profile(hs_batch* batch, hs_op_profile* out, int cap);
/* The number of kernel launches of this library in this process (for the benchmark). */
uint64_t hs_launch_count(void);

/* ---- op-level entry points: the kernels alone, for tests and measurements ----
 * (the reference's op-level path, crates/hardshell-cuda/src/batch/record.rs, and its GEMM tests,
 * crates/hardshell-cuda/tests/ops.rs). Host buffers in and out. */

/* out[m][n] = clamp(rescale(A[m] . W[n] + bias[n], mult[n], shift), -127, 127) for int8
 * A [M, K] and W [N, K], exact int32 accumulation (crates/hardshell/src/gpt2/ops.rs:434
 * LinearOut::Act). path 0 = tensor cores (tcgen05), 1 = CUDA cores (dp4a).
 * With raw32 != NULL the int32 accumulators are written there instead (out8 may be NULL). */
int hs_op_linear_act(hs_dev* dev, int path, const int8_t* A, const int8_t* W, const int32_t* bias,
                     const int32_t* mult, uint32_t shift, uint32_t M, uint32_t N, uint32_t K, int8_t* out8,
                     int32_t* raw32);

/* No counterpart in the reference: hs_op_linear_act for callers that cannot allocate device
 * memory at call time (another allocator owns the rest of HBM, or cudaFree's device-wide
 * synchronisation would stall their other streams). Same arguments, results and errors, but the
 * padded operands, parameters and result are staged in one static __device__ array of
 * HS_STATIC_SCRATCH_BYTES per GPU (held until exit); shapes that need more are refused with
 * HS_UNSUPPORTED. It calls no cudaMalloc or cudaFree. The first call on a device resolves the
 * array's address (cudaGetSymbolAddress) and creates the library's non-blocking stream for that
 * device, on which every call runs (not the legacy default stream): make that first call before
 * any stream capture. Calls share the array, so calls that overlap on one GPU race: serialise
 * them. */
#define HS_STATIC_SCRATCH_BYTES (32u << 20)
int hs_op_linear_act_noalloc(hs_dev* dev, int path, const int8_t* A, const int8_t* W, const int32_t* bias,
                             const int32_t* mult, uint32_t shift, uint32_t M, uint32_t N, uint32_t K, int8_t* out8,
                             int32_t* raw32);

/* A device-resident GEMM benchmark: the same op on device buffers it allocates, with inputs
 * from a seed, timed with CUDA events over `iters` launches after `warmup`. Fills the mean
 * launch time in microseconds. For bench.py. */
int hs_op_linear_bench(hs_dev* dev, int path, uint32_t M, uint32_t N, uint32_t K, uint64_t seed, int warmup,
                       int iters, double* us_per_launch);

#ifdef __cplusplus
}
#endif

#endif /* HARDSHELL_B200_H */
