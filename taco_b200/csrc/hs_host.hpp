// Host-side helpers shared by the C-ABI files of the backend.
#pragma once

#include <string>

namespace hs {

// Records `msg` as the calling thread's last error (hs_last_error) and returns `code`.
int host_fail(int code, const std::string& msg);

}  // namespace hs

#include <cstddef>
#include <cstdint>
#include <vector>

struct hs_model;
struct hs_batch;
struct hs_tokenizer;

namespace hs {

// The model of a batch, and its slot count.
hs_model* batch_model(hs_batch* b);
uint32_t batch_slots(const hs_batch* b);
uint32_t batch_max_rows(const hs_batch* b);

// The vocabulary size, EOT token and context length of a model file (false with a message if the
// file is not a valid model).
bool model_file_info(const uint8_t* file, size_t len, uint32_t* vocab, uint32_t* eot, uint32_t* n_ctx,
                     std::string& err);

// The vocabulary size, EOT token and context length of the tokenizer's model.
void tokenizer_info(const hs_tokenizer* t, uint32_t* vocab, uint32_t* eot, uint32_t* n_ctx);

// The bytes of token `id` (empty for an id out of range).
const uint8_t* token_bytes(const hs_tokenizer* t, uint32_t id, size_t* n);

// Tokenizer::encode, and the check of crates/taco/src/codec.rs:55 tokens_restore: the bytes of
// `tokens` (none of them EOT or empty) join to data[0 .. len).
void tokenize(const hs_tokenizer* t, const uint8_t* data, size_t len, std::vector<uint32_t>& out);
bool tokens_restore(const hs_tokenizer* t, const uint32_t* tokens, size_t n, const uint8_t* data, size_t len);

}  // namespace hs
