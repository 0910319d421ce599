// Synthetic Qwen3 GGUF writer: the stand-in for "seeded N(0, sigma) weights, norms 1.0, quantized, written as GGUF"
// (malkin ships no weight quantizer and no GGUF writer). Tensor names, shapes and metadata keys are the ones
// malkin's read_config / Model constructor bind (model.cpp:78-135). Quantizers: Q8_0 (per-32 absmax), Q4_K and
// Q6_K (simple min/max and absmax fits; the format, not the fit, is what both sides must agree on: they read the
// same bytes). Every row's values depend only on (seed, tensor index, row), so the file is identical for any
// thread count.
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <string>
#include <thread>
#include <vector>

#include "gguf.hpp"
#include "synth.hpp"

namespace mkb {

namespace {

uint64_t splitmix64(uint64_t& s) {
  uint64_t z = (s += 0x9E3779B97F4A7C15ull);
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

// n values ~ N(0, sigma): Box-Muller on a splitmix64 stream.
void normal_row(uint64_t seed, uint64_t tensor, uint64_t row, float sigma, float* out, int64_t n) {
  uint64_t s = seed * 0x632BE59BD9B4E019ull ^ (tensor + 1) * 0x8CB92BA72F3D8DD7ull ^ (row + 1) * 0xD6E8FEB86659FD93ull;
  splitmix64(s);
  for (int64_t i = 0; i < n; i += 2) {
    const uint64_t a = splitmix64(s), b = splitmix64(s);
    const float u1 = (static_cast<float>(a >> 40) + 1.0f) * (1.0f / 16777216.0f);  // (0, 1]
    const float u2 = static_cast<float>(b >> 40) * (1.0f / 16777216.0f);            // [0, 1)
    const float r = std::sqrt(-2.0f * std::log(u1)) * sigma;
    const float t = 6.28318530717958647692f * u2;
    out[i] = r * std::cos(t);
    if (i + 1 < n) out[i + 1] = r * std::sin(t);
  }
}

void put16(uint8_t* p, uint16_t v) { std::memcpy(p, &v, 2); }

// Q8_0 block: fp16 d = absmax / 127, q = round(x / d) (the ggml Q8_0 rule).
void quant_q8_0(const float* x, uint8_t* y, int64_t k) {
  for (int64_t b = 0; b < k / 32; ++b, x += 32, y += 34) {
    float amax = 0.0f;
    for (int i = 0; i < 32; ++i) amax = std::max(amax, std::fabs(x[i]));
    const float d = amax / 127.0f, id = d != 0.0f ? 1.0f / d : 0.0f;
    put16(y, fp32_to_fp16(d));
    for (int i = 0; i < 32; ++i) {
      const int q = static_cast<int>(std::lround(x[i] * id));
      y[2 + i] = static_cast<uint8_t>(static_cast<int8_t>(std::clamp(q, -127, 127)));
    }
  }
}

// Q4_K super-block (144 bytes): fp16 d, fp16 dmin, 12 bytes of 6-bit (scale, min) per 32-value sub-block packed as
// scale_min_k4 unpacks them (kernels.h:18-26), then 128 bytes of nibbles (quant.cpp:77-90 layout).
void quant_q4_k(const float* x, uint8_t* y, int64_t k) {
  for (int64_t sb = 0; sb < k / 256; ++sb, x += 256, y += 144) {
    float scale[8], mn[8];
    for (int j = 0; j < 8; ++j) {
      float lo = 0.0f, hi = -INFINITY;
      for (int l = 0; l < 32; ++l) {
        lo = std::min(lo, x[32 * j + l]);
        hi = std::max(hi, x[32 * j + l]);
      }
      scale[j] = std::max(hi - lo, 0.0f) / 15.0f;
      mn[j] = -lo;
    }
    const float smax = *std::max_element(scale, scale + 8), mmax = *std::max_element(mn, mn + 8);
    const uint16_t dh = fp32_to_fp16(smax / 63.0f), mh = fp32_to_fp16(mmax / 63.0f);
    const float d = fp16_to_fp32(dh), dmin = fp16_to_fp32(mh);
    int sc[8], m[8];
    for (int j = 0; j < 8; ++j) {
      sc[j] = d > 0.0f ? std::clamp(static_cast<int>(std::lround(scale[j] / d)), 0, 63) : 0;
      m[j] = dmin > 0.0f ? std::clamp(static_cast<int>(std::lround(mn[j] / dmin)), 0, 63) : 0;
    }
    put16(y, dh);
    put16(y + 2, mh);
    uint8_t* s = y + 4;
    for (int j = 0; j < 4; ++j) {
      s[j] = static_cast<uint8_t>(sc[j] | ((sc[j + 4] >> 4) << 6));
      s[j + 4] = static_cast<uint8_t>(m[j] | ((m[j + 4] >> 4) << 6));
      s[j + 8] = static_cast<uint8_t>((sc[j + 4] & 0xF) | ((m[j + 4] & 0xF) << 4));
    }
    uint8_t* qs = y + 16;
    std::memset(qs, 0, 128);
    for (int j = 0; j < 8; ++j) {
      const float step = d * static_cast<float>(sc[j]), off = dmin * static_cast<float>(m[j]);
      for (int l = 0; l < 32; ++l) {
        const int q = step > 0.0f ? std::clamp(static_cast<int>(std::lround((x[32 * j + l] + off) / step)), 0, 15) : 0;
        qs[32 * (j / 2) + l] |= static_cast<uint8_t>(q << ((j & 1) ? 4 : 0));
      }
    }
  }
}

// Q6_K super-block (210 bytes): ql[128] low nibbles, qh[64] 2-bit highs, int8 scale per 16 values, fp16 d
// (quant.cpp:108-128 layout): value p has scale sc[p / 16] and 6-bit q stored +32.
void quant_q6_k(const float* x, uint8_t* y, int64_t k) {
  for (int64_t sb = 0; sb < k / 256; ++sb, x += 256, y += 210) {
    float scale[16];
    for (int i = 0; i < 16; ++i) {
      float amax = 0.0f;
      for (int l = 0; l < 16; ++l) amax = std::max(amax, std::fabs(x[16 * i + l]));
      scale[i] = amax / 31.0f;
    }
    const float smax = *std::max_element(scale, scale + 16);
    const uint16_t dh = fp32_to_fp16(smax / 127.0f);
    const float d = fp16_to_fp32(dh);
    std::memset(y, 0, 210);
    uint8_t* ql = y;
    uint8_t* qh = y + 128;
    auto* scs = reinterpret_cast<int8_t*>(y + 192);
    for (int i = 0; i < 16; ++i) {
      const int s = d > 0.0f ? std::clamp(static_cast<int>(std::lround(scale[i] / d)), -128, 127) : 0;
      scs[i] = static_cast<int8_t>(s);
    }
    for (int p = 0; p < 256; ++p) {
      const float step = d * static_cast<float>(scs[p / 16]);
      const int q = step != 0.0f ? std::clamp(static_cast<int>(std::lround(x[p] / step)) + 32, 0, 63) : 32;
      const int n = p / 128, r = p % 128, c = r / 32, l = r % 32;
      ql[64 * n + l + 32 * (c & 1)] |= static_cast<uint8_t>((q & 0xF) << (c >= 2 ? 4 : 0));
      qh[32 * n + l] |= static_cast<uint8_t>((q >> 4) << (2 * c));
    }
    put16(y + 208, dh);
  }
}

// IEEE binary16 with round-to-nearest-even (subnormals kept; overflow to infinity).
uint16_t to_f16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u, e8 = (x >> 23) & 0xFFu;
  uint32_t mant = x & 0x7FFFFFu;
  if (e8 == 0xFF) return static_cast<uint16_t>(sign | 0x7C00u | (mant ? 0x200u : 0u));
  const int e = static_cast<int>(e8) - 127 + 15;
  if (e >= 31) return static_cast<uint16_t>(sign | 0x7C00u);
  uint32_t r, rem, half;
  if (e <= 0) {  // subnormal half: shift the implicit-one mantissa right
    if (e < -10) return static_cast<uint16_t>(sign);
    mant |= 0x800000u;
    const int shift = 14 - e;
    r = mant >> shift;
    rem = mant & ((1u << shift) - 1);
    half = 1u << (shift - 1);
  } else {
    r = (static_cast<uint32_t>(e) << 10) | (mant >> 13);
    rem = mant & 0x1FFFu;
    half = 0x1000u;
  }
  if (rem > half || (rem == half && (r & 1u))) ++r;  // a carry may move into the exponent, as rounding does
  return static_cast<uint16_t>(sign | r);
}

// bfloat16: the top 16 bits of the float, rounded to nearest even.
uint16_t to_bf16(float f) {
  uint32_t x;
  std::memcpy(&x, &f, 4);
  if ((x & 0x7F800000u) == 0x7F800000u) return static_cast<uint16_t>((x >> 16) | ((x & 0xFFFFu) ? 0x40u : 0u));
  return static_cast<uint16_t>((x + 0x7FFFu + ((x >> 16) & 1u)) >> 16);
}

void quantize_row(uint32_t type, const float* x, uint8_t* y, int64_t k) {
  switch (type) {
    case kF16:
      for (int64_t i = 0; i < k; ++i) {
        const uint16_t h = to_f16(x[i]);
        std::memcpy(y + 2 * i, &h, 2);
      }
      return;
    case kBF16:
      for (int64_t i = 0; i < k; ++i) {
        const uint16_t h = to_bf16(x[i]);
        std::memcpy(y + 2 * i, &h, 2);
      }
      return;
    case kQ8_0:
      return quant_q8_0(x, y, k);
    case kQ4_K:
      return quant_q4_k(x, y, k);
    case kQ6_K:
      return quant_q6_k(x, y, k);
    case kF32:
      std::memcpy(y, x, static_cast<size_t>(k) * 4);
      return;
    default:
      throw std::runtime_error(std::string("synth: cannot quantize to ") + type_name(type));
  }
}

}  // namespace

void quantize_rows(uint32_t type, const float* x, uint8_t* y, int64_t rows, int64_t cols) {
  const size_t rb = row_bytes(type, cols);
  for (int64_t r = 0; r < rows; ++r) quantize_row(type, x + r * cols, y + r * rb, cols);
}

void write_synth_gguf(const std::string& path, const SynthSpec& s, int n_threads) {
  if (s.n_layer <= 0 || s.n_embd <= 0 || s.n_ff <= 0 || s.n_head <= 0 || s.n_head_kv <= 0 || s.head_dim <= 0 ||
      s.n_vocab <= 0 || s.n_head % s.n_head_kv || s.head_dim % 32)
    throw std::runtime_error("synth: bad model shape");
  GgufWriter w;
  w.add_str("general.architecture", "qwen3");
  w.add_str("general.name", "malkin-b200-synthetic");
  w.add_u32("qwen3.block_count", static_cast<uint32_t>(s.n_layer));
  w.add_u32("qwen3.context_length", static_cast<uint32_t>(s.n_ctx_train));
  w.add_u32("qwen3.embedding_length", static_cast<uint32_t>(s.n_embd));
  w.add_u32("qwen3.feed_forward_length", static_cast<uint32_t>(s.n_ff));
  w.add_u32("qwen3.attention.head_count", static_cast<uint32_t>(s.n_head));
  w.add_u32("qwen3.attention.head_count_kv", static_cast<uint32_t>(s.n_head_kv));
  w.add_u32("qwen3.attention.key_length", static_cast<uint32_t>(s.head_dim));
  w.add_u32("qwen3.attention.value_length", static_cast<uint32_t>(s.head_dim));
  w.add_f32("qwen3.rope.freq_base", s.rope_base);
  w.add_f32("qwen3.attention.layer_norm_rms_epsilon", s.rms_eps);
  w.add_str("tokenizer.ggml.model", "gpt2");
  {
    std::vector<std::string> toks(static_cast<size_t>(s.n_vocab));
    for (int i = 0; i < s.n_vocab; ++i) toks[static_cast<size_t>(i)] = "<t" + std::to_string(i) + ">";
    w.add_str_array("tokenizer.ggml.tokens", toks);
  }
  if (s.has_eos) {
    if (s.eos_token_id < 0 || s.eos_token_id >= s.n_vocab) throw std::runtime_error("synth: eos_token_id out of range");
    w.add_u32("tokenizer.ggml.eos_token_id", static_cast<uint32_t>(s.eos_token_id));
  }
  const int64_t E = s.n_embd, F = s.n_ff, HD = static_cast<int64_t>(s.n_head) * s.head_dim,
                KD = static_cast<int64_t>(s.n_head_kv) * s.head_dim, V = s.n_vocab;
  struct Job {
    int idx;
    uint32_t type;
    int64_t rows, cols;
    bool ones;
  };
  std::vector<Job> jobs;
  auto mat = [&](const std::string& name, uint32_t type, int64_t cols, int64_t rows) {
    jobs.push_back({w.add_tensor(name, type, {cols, rows}), type, rows, cols, false});
  };
  auto vec = [&](const std::string& name, int64_t n) { jobs.push_back({w.add_tensor(name, kF32, {n}), kF32, 1, n, true}); };
  mat("token_embd.weight", s.tied ? s.type_output : s.type_embd, E, V);
  vec("output_norm.weight", E);
  if (!s.tied) mat("output.weight", s.type_output, E, V);
  for (int i = 0; i < s.n_layer; ++i) {
    const std::string p = "blk." + std::to_string(i) + ".";
    vec(p + "attn_norm.weight", E);
    vec(p + "ffn_norm.weight", E);
    vec(p + "attn_q_norm.weight", s.head_dim);
    vec(p + "attn_k_norm.weight", s.head_dim);
    mat(p + "attn_q.weight", s.type_default, E, HD);
    mat(p + "attn_k.weight", s.type_default, E, KD);
    mat(p + "attn_v.weight", s.type_attn_v, E, KD);
    mat(p + "attn_output.weight", s.type_default, HD, E);
    mat(p + "ffn_gate.weight", s.type_default, E, F);
    mat(p + "ffn_up.weight", s.type_default, E, F);
    mat(p + "ffn_down.weight", s.type_ffn_down, F, E);
  }
  w.open(path);
  // Work items: (job, row chunk) of about 2 M values each.
  struct Item {
    size_t job;
    int64_t r0, r1;
  };
  std::vector<Item> items;
  for (size_t j = 0; j < jobs.size(); ++j) {
    const int64_t per = std::max<int64_t>(1, (int64_t{1} << 21) / jobs[j].cols);
    for (int64_t r = 0; r < jobs[j].rows; r += per) items.push_back({j, r, std::min(jobs[j].rows, r + per)});
  }
  std::atomic<size_t> next{0};
  std::atomic<bool> failed{false};
  std::string error;
  auto worker = [&] {
    std::vector<float> buf;
    try {
      for (size_t it; (it = next.fetch_add(1)) < items.size() && !failed.load();) {
        const Item& item = items[it];
        const Job& jb = jobs[item.job];
        uint8_t* dst = w.data(jb.idx);
        const size_t rb = row_bytes(jb.type, jb.cols);
        buf.resize(static_cast<size_t>(jb.cols));
        for (int64_t r = item.r0; r < item.r1; ++r) {
          if (jb.ones) {
            std::fill(buf.begin(), buf.end(), 1.0f);
          } else {
            normal_row(s.seed, static_cast<uint64_t>(jb.idx), static_cast<uint64_t>(r), s.sigma, buf.data(), jb.cols);
          }
          quantize_row(jb.type, buf.data(), dst + static_cast<size_t>(r) * rb, jb.cols);
        }
      }
    } catch (const std::exception& e) {
      if (!failed.exchange(true)) error = e.what();
    }
  };
  int nt = n_threads > 0 ? n_threads : static_cast<int>(std::thread::hardware_concurrency());
  nt = std::max(1, std::min<int>(nt, static_cast<int>(items.size())));
  std::vector<std::thread> pool;
  for (int i = 0; i < nt; ++i) pool.emplace_back(worker);
  for (auto& t : pool) t.join();
  w.close();
  if (failed) throw std::runtime_error("synth: " + error);
}

}  // namespace mkb
