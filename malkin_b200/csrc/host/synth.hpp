#pragma once
#include <cstdint>
#include <string>

namespace mkb {

struct SynthSpec {
  int n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, n_ctx_train;
  float rope_base, rms_eps;
  int tied;
  uint32_t type_default, type_attn_v, type_ffn_down, type_output, type_embd;
  float sigma;
  uint64_t seed;
  int has_eos = 0, eos_token_id = 0;  // tokenizer.ggml.eos_token_id when has_eos
};

// Writes a synthetic Qwen3 model (see synth.cpp) to path.
void write_synth_gguf(const std::string& path, const SynthSpec& spec, int n_threads);
// Quantizes rows x cols floats into GGUF rows of `type` (Q8_0, Q4_K, Q6_K, F32).
void quantize_rows(uint32_t type, const float* x, uint8_t* y, int64_t rows, int64_t cols);

}  // namespace mkb
