// TEST INFRASTRUCTURE ONLY (oracle): C entry points over malkin's own, unmodified CPU path.
//
// oracle/Makefile compiles this file together with the reference's sources, where they lie, into
// oracle/_ref/libmalkin_ref.so. Only tests/, __graft_entry__.smoke() and bench.py's reference arm load it,
// as the checker or as the timed CPU baseline; the product (malkin_b200) never links or calls it.
//
// What is exposed (reference citations are src/<file>:<line> in kekzl/malkin v0.2.0):
//   model      GgufFile + Model(f, n_ctx, n_seq) + Model::forward(const BatchToken*, n, logits)   model.cpp:112,280
//              Model::move_kv                                                                     model.cpp:432
//   quant      quantize_row_q8 (kern::quantize_row_q8), quantize_i8, dequantize_row, matmul        quant.cpp:132-351
//   attention  kern::attend_gqa (tree ancestors as extra keys)                                    kernels_avx512.cpp:282
//   sampler    Sampler::distribution / draw / verify                                              sampler.cpp:22-97
//   accept     Engine::accept_greedy / accept_sampled restated over Model::move_kv and Sampler,   engine.cpp:441-507
//              because they are private members of Engine; emit() is taken as "continue" (no
//              end-of-generation token, no stop string).
//   engine     malkin's Engine itself (generate with continuous batching and a draft model, and      engine.cpp:100-559
//              perplexity), compiled with ref_tokenizer.cpp standing in for the pcre2 tokenizer.
#include <cstddef>
#include <cstdint>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include <omp.h>

#include <thread>

#include "cpu.h"
#include "engine.h"
#include "gguf.h"
#include "kernels.h"
#include "model.h"
#include "quant.h"
#include "sampler.h"

#include "../include/malkin_b200.h"

using namespace malkin;

// The C ABI's structs mirror malkin's: a BatchToken array and the sampling parameters cross the boundary as they are
// (model.h:25-30, sampler.h:10-18; mk_sampling stops before SamplingParams::seed, the host owns the RNG).
#define MK_SAME_FIELD(A, B, fa, fb) \
  static_assert(offsetof(A, fa) == offsetof(B, fb) && sizeof(A::fa) == sizeof(B::fb), #A "." #fa " != " #B "." #fb)
static_assert(sizeof(mk_batch_token) == sizeof(BatchToken) && alignof(mk_batch_token) == alignof(BatchToken));
MK_SAME_FIELD(mk_batch_token, BatchToken, id, id);
MK_SAME_FIELD(mk_batch_token, BatchToken, seq, seq);
MK_SAME_FIELD(mk_batch_token, BatchToken, pos, pos);
MK_SAME_FIELD(mk_batch_token, BatchToken, logits, logits);
MK_SAME_FIELD(mk_batch_token, BatchToken, kv, kv);
MK_SAME_FIELD(mk_batch_token, BatchToken, parent, parent);
MK_SAME_FIELD(mk_sampling, SamplingParams, temperature, temperature);
MK_SAME_FIELD(mk_sampling, SamplingParams, top_p, top_p);
MK_SAME_FIELD(mk_sampling, SamplingParams, top_k, top_k);
MK_SAME_FIELD(mk_sampling, SamplingParams, min_p, min_p);
MK_SAME_FIELD(mk_sampling, SamplingParams, presence_penalty, presence_penalty);
MK_SAME_FIELD(mk_sampling, SamplingParams, frequency_penalty, frequency_penalty);
static_assert(sizeof(mk_sampling) == offsetof(SamplingParams, seed));
#undef MK_SAME_FIELD

namespace {

struct RefModel {
  std::unique_ptr<GgufFile> file;
  std::unique_ptr<Model> model;
};

void put_err(char* err, int len, const char* what) {
  if (err && len > 0) {
    std::strncpy(err, what, static_cast<size_t>(len) - 1);
    err[len - 1] = 0;
  }
}

SamplingParams params_of(float temp, float top_p, int top_k, float min_p, float pres, float freq, uint64_t seed) {
  SamplingParams p;
  p.temperature = temp;
  p.top_p = top_p;
  p.top_k = top_k;
  p.min_p = min_p;
  p.presence_penalty = pres;
  p.frequency_penalty = freq;
  p.seed = seed;
  return p;
}

Dist dist_of(const float* p, const int32_t* ids, int n) {
  Dist d;
  for (int i = 0; i < n; ++i) d.emplace_back(p[i], ids[i]);
  return d;
}

}  // namespace

extern "C" {

// "" when this CPU can run the reference (AVX-512 F/BW/VL/DQ + VNNI + BF16), else the missing features.
const char* ref_missing_features() {
  static std::string s;
  s = cpu_missing_features();
  return s.c_str();
}

int ref_physical_cores() { return cpu_physical_cores(); }

void ref_set_threads(int n) { omp_set_num_threads(n > 0 ? n : 1); }

void* ref_model_open(const char* path, int n_ctx, int n_seq, int wide, char* err, int errlen) {
  try {
    auto r = std::make_unique<RefModel>();
    r->file = std::make_unique<GgufFile>(path);
    r->model = std::make_unique<Model>(*r->file, n_ctx, n_seq);
    if (wide) r->model->pack_wide();
    return r.release();
  } catch (const std::exception& e) {
    put_err(err, errlen, e.what());
    return nullptr;
  }
}

void ref_model_close(void* h) { delete static_cast<RefModel*>(h); }

// n_layer n_embd n_ff n_head n_head_kv head_dim n_vocab n_ctx n_seq; f: rope_base rms_eps
void ref_model_cfg(void* h, int* out, float* f) {
  const Model& m = *static_cast<RefModel*>(h)->model;
  const ModelConfig& c = m.cfg();
  const int v[9] = {c.n_layer, c.n_embd, c.n_ff, c.n_head, c.n_head_kv, c.head_dim, c.n_vocab, m.n_ctx(), m.n_seq()};
  std::memcpy(out, v, sizeof v);
  f[0] = c.rope_base;
  f[1] = c.rms_eps;
}

// Model::forward(const BatchToken*, n, logits) (model.cpp:280-323); 0 = ok, -1 = exception (message in err).
int ref_model_forward(void* h, int n, const int32_t* id, const int32_t* seq, const int32_t* pos, const int32_t* logits,
                      const int32_t* kv, const int32_t* parent, float* out, char* err, int errlen) {
  try {
    std::vector<BatchToken> b(static_cast<size_t>(n));
    for (int t = 0; t < n; ++t) {
      b[t].id = id[t];
      b[t].seq = seq[t];
      b[t].pos = pos[t];
      b[t].logits = logits[t] != 0;
      b[t].kv = kv[t];
      b[t].parent = parent[t];
    }
    static_cast<RefModel*>(h)->model->forward(b.data(), n, out);
    return 0;
  } catch (const std::exception& e) {
    put_err(err, errlen, e.what());
    return -1;
  }
}

void ref_model_move_kv(void* h, int from, int to, int seq) { static_cast<RefModel*>(h)->model->move_kv(from, to, seq); }

// ---- quant.h ----

void ref_quantize_row_q8(const float* x, void* blocks, int64_t k) {
  quantize_row_q8(x, static_cast<BlockQ8*>(blocks), k);
}

float ref_quantize_i8(const float* x, int n, int8_t* q) { return quantize_i8(x, n, q); }

int ref_dequantize_row(int type, const void* src, float* dst, int64_t k) {
  try {
    dequantize_row(static_cast<GgmlType>(type), src, dst, k);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

float ref_fp16_to_fp32(uint16_t h) { return fp16_to_fp32(h); }

// y[t * rows + r] = W[r] . x[t] through malkin's matmul (quant.cpp:330-351): mode 0 = row path (vec_dot),
// 1 = compact panels (pack_weight), 2 = compact + wide panels (wide used when n > kWideMinTokens).
int ref_matmul(int type, const uint8_t* w, int64_t rows, int64_t cols, int mode, const float* x, int n, float* y) {
  try {
    Weight wt;
    wt.type = static_cast<GgmlType>(type);
    wt.data = w;
    wt.rows = rows;
    wt.cols = cols;
    wt.row_bytes = ggml_row_size(wt.type, cols);
    std::unique_ptr<PackedBuffer> compact, wide;
    if (mode >= 1) compact = std::make_unique<PackedBuffer>(pack_weight(wt, false));
    if (mode >= 2) wide = std::make_unique<PackedBuffer>(pack_weight(wt, true));
    std::vector<BlockQ8> xq;
    if (weight_type_quantized(wt.type)) quantize_acts(x, n, cols, xq);
    matmul(wt, x, xq.empty() ? nullptr : xq.data(), n, y);
    return 0;
  } catch (const std::exception&) {
    return -1;
  }
}

// kern::attend_gqa for one token and one KV head (kernels_avx512.cpp:282): k / v point at key row 0 of the head,
// stride bytes between rows, the row's scale soff bytes after the head's first value.
void ref_attend_gqa(const float* q, int G, int D, const int8_t* k, const int8_t* v, int64_t stride, int64_t soff,
                    int n, float scale, float* out, const int* extra, int ne) {
  std::vector<float> scratch(static_cast<size_t>(G) * (n + ne) + 64);
  kern::attend_gqa(q, G, D, k, v, static_cast<size_t>(stride), static_cast<ptrdiff_t>(soff), n, scale, out,
                   scratch.data(), extra, ne);
}

void ref_silu_mul(int64_t n, float* g, const float* u) { kern::silu_mul(n, g, u); }

// ---- sampler.h ----

// The uniform stream Sampler draws from (sampler.h:39, sampler.cpp:66 / 82): n values of
// std::uniform_real_distribution<double>(0, 1) over std::mt19937_64(seed).
void ref_uniforms(uint64_t seed, int n, double* out) {
  std::mt19937_64 rng(seed);
  for (int i = 0; i < n; ++i) out[i] = std::uniform_real_distribution<double>(0.0, 1.0)(rng);
}

void* ref_sampler_new(float temp, float top_p, int top_k, float min_p, float pres, float freq, uint64_t seed) {
  return new Sampler(params_of(temp, top_p, top_k, min_p, pres, freq, seed));
}

void ref_sampler_free(void* s) { delete static_cast<Sampler*>(s); }

void ref_sampler_accept(void* s, int32_t id) { static_cast<Sampler*>(s)->accept(id); }

// Sampler::distribution (sampler.cpp:22-62); logits modified in place as in the reference. Returns entries written.
int ref_sampler_distribution(void* s, float* logits, int n_vocab, float* p, int32_t* ids, int cap) {
  Dist d;
  static_cast<Sampler*>(s)->distribution(logits, n_vocab, d);
  const int n = static_cast<int>(d.size()) < cap ? static_cast<int>(d.size()) : cap;
  for (int i = 0; i < n; ++i) {
    p[i] = d[i].first;
    ids[i] = d[i].second;
  }
  return static_cast<int>(d.size());
}

int32_t ref_sampler_draw(void* s, const float* p, const int32_t* ids, int n) {
  return static_cast<Sampler*>(s)->draw(dist_of(p, ids, n));
}

int32_t ref_sampler_sample(void* s, float* logits, int n_vocab) { return static_cast<Sampler*>(s)->sample(logits, n_vocab); }

int32_t ref_sampler_verify(void* s, const float* pp, const int32_t* pid, int np, const float* qp, const int32_t* qid,
                           int nq, int32_t d, int* accepted) {
  bool a = false;
  const int32_t t = static_cast<Sampler*>(s)->verify(dist_of(pp, pid, np), dist_of(qp, qid, nq), d, a);
  *accepted = a ? 1 : 0;
  return t;
}

// Engine::accept_greedy (engine.cpp:441-479) for one slot whose root row is logits[0]. cache_len: the slot's KV
// length before the step (P = cache_len, the root's KV row); on return cache_len + 1 + accepted.
// Writes the accepted ids, returns the accepted count; *next = next token; *k = adapted draft length.
int ref_accept_greedy(void* model, void* sampler, float* logits, int n_vocab, int kk, const int32_t* chain,
                      const int32_t* alt, int seq, int* cache_len, int32_t* accepted_ids, int32_t* next, int* k,
                      int n_draft) {
  Model* m = model ? static_cast<RefModel*>(model)->model.get() : nullptr;
  Sampler& smp = *static_cast<Sampler*>(sampler);
  const int P = *cache_len;
  int size = P + 1;  // s.cache.push_back(q.next) in Engine::accept (engine.cpp:428)
  auto row = [&](int t) { return logits + static_cast<size_t>(t) * n_vocab; };
  Dist dist;
  int cur = 0, done = 0, acc = 0;
  bool bonus_ready = false;
  for (int i = 0; i < kk; ++i) {
    smp.distribution(row(cur), n_vocab, dist);
    const int32_t a = dist[0].second;
    int slot = -1;
    if (a == chain[i])
      slot = 1 + 2 * i;
    else if (a == alt[i])
      slot = 2 + 2 * i;
    if (slot < 0) {
      *next = a;
      bonus_ready = true;
      break;
    }
    if (m) m->move_kv(P + slot, size, seq);
    ++size;
    accepted_ids[acc++] = a;
    cur = slot;
    smp.accept(a);  // emit() -> sampler.accept (engine.cpp:64); generation continues
    done = i + 1;
    if (slot == 2 + 2 * i) break;
  }
  if (!bonus_ready) {
    smp.distribution(row(cur), n_vocab, dist);
    *next = dist[0].second;
  }
  if (done == kk && kk == *k && cur == 2 * kk - 1)
    *k = std::min(*k + 1, n_draft);
  else if (2 * done < kk)
    *k = std::max(1, *k - 1);
  *cache_len = size;
  return acc;
}

// Engine::accept_sampled (engine.cpp:482-507) for one slot: logits rows 0..kk (chain laid out [next, d0, ...]);
// q_p / q_id: kk draft distributions of q_n[i] entries each, packed back to back.
int ref_accept_sampled(void* sampler, float* logits, int n_vocab, int kk, const int32_t* chain, const float* q_p,
                       const int32_t* q_id, const int* q_n, int32_t* accepted_ids, int32_t* next, int* k, int n_draft) {
  Sampler& smp = *static_cast<Sampler*>(sampler);
  auto row = [&](int t) { return logits + static_cast<size_t>(t) * n_vocab; };
  Dist dist;
  int i = 0, off = 0, acc = 0;
  for (; i < kk; ++i) {
    smp.distribution(row(i), n_vocab, dist);
    bool ok = false;
    const int32_t t = smp.verify(dist, dist_of(q_p + off, q_id + off, q_n[i]), chain[i], ok);
    off += q_n[i];
    if (!ok) {
      *next = t;
      break;
    }
    accepted_ids[acc++] = t;
    smp.accept(t);
  }
  if (i == kk) *next = smp.sample(row(kk), n_vocab);
  if (i == kk && kk == *k)
    *k = std::min(*k + 1, n_draft);
  else if (2 * i < kk)
    *k = std::max(1, *k - 1);
  return acc;
}

// ---- Engine (engine.cpp) ----
void* ref_engine_open(const char* model, const char* draft, int n_ctx, int parallel, int n_draft, int threads, char* err,
                      int errlen) {
  try {
    EngineOptions o;
    o.model_path = model;
    o.n_ctx = n_ctx;
    o.threads = threads;
    o.threads_batch = threads;
    o.draft_path = draft ? draft : "";
    o.n_draft = n_draft;
    o.parallel = parallel;
    return new Engine(o);
  } catch (const std::exception& e) {
    put_err(err, errlen, e.what());
    return nullptr;
  }
}

void ref_engine_close(void* h) { delete static_cast<Engine*>(h); }

// n requests through Engine::generate, each on its own thread started together (continuous batching) or one after
// another (sequential). sampling: n x (temperature, top_p, top_k, min_p). Per request: its tokens (read back from
// the generated text, at most cap) in out[i * cap ..], their count in out_n[i], and stats[i * 6 ..] = prompt,
// cached, completion tokens, drafted, accepted, finish (1 stop, 2 length, 3 cancelled). 0 = ok, -1 = exception.
int ref_engine_generate(void* h, int n, int sequential, const int32_t* prompts, const int32_t* plen,
                        const int32_t* max_tokens, const float* sampling, const uint64_t* seeds, int cap, int32_t* out,
                        int32_t* out_n, int32_t* stats, char* err, int errlen) {
  Engine& e = *static_cast<Engine*>(h);
  std::vector<GenRequest> reqs(static_cast<size_t>(n));
  size_t off = 0;
  for (int i = 0; i < n; ++i) {
    GenRequest& r = reqs[static_cast<size_t>(i)];
    r.prompt.assign(prompts + off, prompts + off + plen[i]);
    off += static_cast<size_t>(plen[i]);
    r.max_tokens = max_tokens[i];
    r.sampling = params_of(sampling[4 * i], sampling[4 * i + 1], static_cast<int>(sampling[4 * i + 2]),
                           sampling[4 * i + 3], 0.0f, 0.0f, seeds[i]);
  }
  std::vector<GenResult> res(static_cast<size_t>(n));
  std::vector<std::string> errs(static_cast<size_t>(n));
  auto run = [&](int i) {
    try {
      res[static_cast<size_t>(i)] = e.generate(reqs[static_cast<size_t>(i)], nullptr);
    } catch (const std::exception& x) {
      errs[static_cast<size_t>(i)] = x.what();
    }
  };
  if (sequential) {
    for (int i = 0; i < n; ++i) run(i);
  } else {
    std::vector<std::thread> th;
    for (int i = 0; i < n; ++i) th.emplace_back(run, i);
    for (auto& t : th) t.join();
  }
  for (int i = 0; i < n; ++i) {
    if (!errs[static_cast<size_t>(i)].empty()) {
      put_err(err, errlen, errs[static_cast<size_t>(i)].c_str());
      return -1;
    }
    const GenResult& r = res[static_cast<size_t>(i)];
    const auto ids = e.tokenizer().encode(r.text, false);
    const int m = std::min<int>(cap, static_cast<int>(ids.size()));
    std::copy(ids.begin(), ids.begin() + m, out + static_cast<size_t>(i) * cap);
    out_n[i] = m;
    int32_t* st = stats + 6 * i;
    st[0] = r.prompt_tokens;
    st[1] = r.cached_tokens;
    st[2] = r.completion_tokens;
    st[3] = r.drafted;
    st[4] = r.accepted;
    st[5] = r.finish_reason == "stop" ? 1 : (r.finish_reason == "length" ? 2 : 3);
  }
  return 0;
}

// Engine::perplexity over token ids (the text is their pieces, read back by the stand-in tokenizer).
int ref_engine_perplexity(void* h, const int32_t* toks, int n, int window, double* nll, int* scored, char* err,
                          int errlen) {
  try {
    Engine& e = *static_cast<Engine*>(h);
    *nll = e.perplexity(e.tokenizer().decode(std::vector<int32_t>(toks, toks + n)), window, scored);
    return 0;
  } catch (const std::exception& x) {
    put_err(err, errlen, x.what());
    return -1;
  }
}

}  // extern "C"
