// Host-side launchers of the CUDA kernels (plain C++ signatures, usable from g++-compiled host code).
#pragma once
#include <cuda_runtime_api.h>

#include <cstddef>
#include <cstdint>

#define MK_TOPK_CAP 64

namespace mkb {

constexpr int kMaxDevices = 64;  // per-device tables (kernel attributes, scratch addresses)

// Token tiles (8 tokens each) of the activation layout for a batch of n tokens: an even count (the tensor-core
// GEMM reads tokens in groups of 16), and whole GEMM passes of 18 tiles once n exceeds one pass, so every pass
// reads initialised (zero) tiles.
inline int act_tiles(int n) {
  const int t = (n + 7) / 8;
  return t <= 18 ? (t + 1) / 2 * 2 : (t + 17) / 18 * 18;
}

// Status-word code of an activation outside the fp16 range of the split-fp16 GEMM operand (bounded-wait timeouts use
// codes 1-10 and 16 up).
// Quantized activations in the GEMM layout (layout.hpp). nt8 = token tiles of the current batch (layout stride).
struct ActQ {
  uint8_t* qx = nullptr;
  uint8_t* qc = nullptr;  // tensor-core order of the same int8 values (nullable)
  float* dx = nullptr;
  float* dsx = nullptr;
  uint32_t* sh = nullptr;
  int nt8 = 0;
  float* xf = nullptr;  // the float values before quantization, [token][ldxf] (nullable; F32/F16/BF16 weights read it)
  int64_t ldxf = 0;
};

// Device weight in the panel layout, or (Q8_0) in the tensor-core tile layout.
constexpr int kLayoutPanels = 0, kLayoutTc = 1, kLayoutRows = 2;  // rows: F32 / F16 / BF16 GGUF rows as they are
struct DevWeight {
  uint32_t type = 0;
  const uint8_t* data = nullptr;
  int64_t rows = 0;    // valid rows
  int64_t cols = 0;    // values per row (this shard)
  int64_t panels = 0;  // ceil(rows / 16)
  int kunits = 0;      // cols / 32 (Q8_0) or cols / 256 (K-quants)
  int layout = kLayoutPanels;
};


// ---- quantization (quant.cu) ----
// x rows [n][ldx] -> act (blocks of K values); rows n..npad-1 zero-filled. K % 32 == 0.
void launch_quant_rows(const float* x, int64_t ldx, int n, int K, const ActQ& act, cudaStream_t s);
// Split-K output slices: n_slices buffers, `stride` floats apart, summed in slice order by the consumer.
struct Slices {
  const float* p = nullptr;
  int n = 0;
  int64_t stride = 0;
};
// rmsnorm (model.cpp:46-49) then quantize. rows: row indices into x (nullptr = 0..n-1). add: residual
// contributions added into x first, in slice order (x[r] += add[0][r] + add[1][r] + ..., written back).
void launch_rmsnorm_quant(float* x, int64_t ldx, Slices add, const int32_t* rows, const float* w, float eps, int n,
                          int K, const ActQ& act, cudaStream_t s);
// gu rows [n][ld] (slices): gate at [0, F), up at [F, 2F): SiLU(gate) * up (kernels_avx512.cpp:271-280), quantized.
void launch_silu_quant(Slices gu, int64_t ld, int F, int n, const ActQ& act, cudaStream_t s);
// dst[t * ld + i] = sum of slices (tensor parallel: the local partial before the allreduce).
void launch_sum_slices(Slices src, int64_t ld, int n, int cols, float* dst, cudaStream_t s);
// malkin BlockQ8 output (40-byte blocks) for tests.
void launch_quant_blockq8(const float* x, int n, int64_t K, void* blocks, cudaStream_t s);
// quantize_i8 rows (quant.cpp:134-140).
void launch_quant_i8(const float* x, int n, int len, int8_t* q, float* scale, cudaStream_t s);
void launch_silu_mul(float* g, const float* u, int64_t n, cudaStream_t s);

// ---- GEMM (gemm.cu) ----
// Slice s (of split) gets y[s * slice + t * ldy + r] = sum over slice s's k-range of W[r] . x[t], t < n, r < rows
// (plain stores). split 1 keeps malkin's block order. status: device word for bounded-wait failures (nullable).
void launch_gemm(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                 int* status, cudaStream_t s);
// F32 / F16 / BF16 weights (kLayoutRows): y[t][r] = malkin's vec_dot row path on the float activations act.xf.
void launch_gemm_rows(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, cudaStream_t s);
// Split that fills the GPU for this weight (>= 1), and the slices a split request produces.
int gemm_split_for(const DevWeight& w, int num_sms);
int gemm_slices(const DevWeight& w, int split);
// Kernel-shape tuning: times every kernel shape of w's layout (panel tile and token pass; tensor-core pass size) for
// n tokens on stream s with the operands launch_gemm would get (y is overwritten with the product, which every shape
// computes bit-identically, so the choice never changes a result) and keeps the fastest for (device, weight shape,
// token tiles); split-1 launches of that shape use it from then on. L2 is flushed before every timed launch, so the
// weights stream from HBM as they do inside a forward. No-op when the shape is tuned already, s is capturing, or
// MALKIN_B200_GEMM_TUNE=0; otherwise it allocates a 256 MiB flush buffer on first use and synchronizes s.
void gemm_tune(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int* status, cudaStream_t s);
// The tuned (or, while tuning, the forced) shape for w at n tokens: a panel variant index or tensor-core pass
// tokens; -1 if none.
int gemm_choice(const DevWeight& w, int n);
// out[(r * n + t) * nblk + b]: exact int dot of block b (Q6_K: 16-value halves).
void launch_block_dots(const DevWeight& w, const ActQ& act, int n, int32_t* out, int* status, cudaStream_t s);

// ---- tensor-core Q8_0 GEMM (tcgen05 kind::i8, gemm_tc.cu), reached through launch_gemm / launch_block_dots ----
// malkin's exact int8 block dots and per-block float epilogue; bit-identical to malkin at split 1 (token passes
// fill the SMs instead of K slices).
void launch_gemm_tc(const DevWeight& w, const ActQ& act, int n, float* y, int64_t ldy, int64_t slice, int split,
                    int32_t* dots, int* status, cudaStream_t s);
int gemm_tc_split_for(const DevWeight& w, int num_sms);
int gemm_tc_slices(const DevWeight& w, int split);
int gemm_tc_max_tokens();  // largest pass size (tokens)

// ---- tensor-parallel sum over NVLink peer memory (tp_reduce.cu) ----
// Rank r's exchange buffer: data[r] = two halves of `cap` floats, flags[r] = one int per rank (the last epoch that
// rank published into r); the pointers of the other ranks are their CUDA IPC mappings in this process.
constexpr int kMaxTp = 8;
constexpr int kErrTpWait = 12;  // status code: a rank's partial never arrived
constexpr uint32_t kTpWaitPolls = 1u << 24;  // polls of about 64 ns: about a second at most
struct TpExchange {
  float* data[kMaxTp] = {};
  int* flags[kMaxTp] = {};
  float* red[kMaxTp] = {};   // two-shot: rank r's reduced rows (two halves of `cap` floats)
  int* flags2[kMaxTp] = {};  // two-shot: the last epoch rank q reduced its rows for, in rank r's buffer
  int* epoch = nullptr;          // this rank's call counter (device)
  unsigned* counter = nullptr;   // this rank's CTA arrival counters (device): publish, reduce
  unsigned* counter2 = nullptr;
  int rank = 0, size = 1;
  int64_t cap = 0;
  uint32_t wait_polls = kTpWaitPolls;  // a flag wait gives up after this many polls (status kErrTpWait)
};
// publish: this rank's split-K slices, summed in slice order, into its half of the exchange; gather: the sum over
// ranks in rank order into dst (n x cols, cols % 4 == 0). Run both, in this order, on every rank.
void launch_tp_publish(const TpExchange& x, Slices src, int64_t ld, int n, int cols, cudaStream_t s);
// Exact tensor parallel: dst[t][r * el + e] = src[r][t][e] (the all-gathered output-feature slices of tp ranks).
void launch_tp_concat(const float* src, int tp, int n, int el, float* dst, cudaStream_t s);
void launch_tp_gather(const TpExchange& x, int n, int cols, float* dst, int* status, cudaStream_t s);
// Two-shot alternative to gather (after publish): reduce sums this rank's 1/size of the rows over the ranks (rank
// order) into its red half; allgather copies every rank's reduced rows into dst. Same sums, bit for bit; each rank
// reads 2 (size - 1) / size of the data from peers instead of (size - 1) times it.
void launch_tp_reduce(const TpExchange& x, int n, int cols, int* status, cudaStream_t s);
void launch_tp_allgather(const TpExchange& x, int n, int cols, float* dst, int* status, cudaStream_t s);

// ---- fixed scratch of the allocation-free entry point (noalloc.cu) ----
// Bytes of the per-device scratch, and its address on the current device (nullptr and *err set on failure).
size_t noalloc_scratch_bytes();
uint8_t* noalloc_scratch(cudaError_t* err);

// ---- attention (attention.cu) ----
struct AttnLayer {
  int8_t* k;   // [kvh][n_rows][D]
  int8_t* v;
  float* ks;   // [kvh][n_rows]
  float* vs;
  int64_t n_rows;  // rows per head (n_seq * n_ctx)
};
// Per token: RoPE table row rpos, KV row kv_at (absolute). y: [n][ldy] = q heads | k heads | v heads, as GEMM
// slices: columns before v_col0 have qk.n slices, the v columns v_n slices (same stride).
void launch_qkv_post(Slices qk, int v_n, int64_t v_col0, int64_t ldy, int n, int H, int KV, int D, const float* q_norm,
                     const float* k_norm, float eps, const float* rope_cs, const int32_t* rpos, const int32_t* kv_at,
                     float* q_out, const AttnLayer& L, cudaStream_t s);

// Attention work description (host-built, device tables).
struct AttnPlan {
  int n = 0;                    // tokens
  int n_sg = 0;                 // query sub-groups (consecutive tokens of one sequence, at most attn_qmax() / G)
  int kchunks = 0;              // key chunks of the score kernel's grid (attn_key_chunks of the context length)
  const int32_t* sg_first = nullptr;  // [n_sg + 1] token ranges
  const int32_t* kv_base = nullptr;   // [n]
  const int32_t* n_keys = nullptr;    // [n]
  const int32_t* anc_off = nullptr;   // [n + 1]
  const int32_t* anc = nullptr;       // extra key rows (relative to kv_base)
  const int32_t* tok_sg = nullptr;    // [n] sub-group of each token
  const int32_t* sg_maxk = nullptr;   // [n_sg] longest key prefix (n_keys) among the sub-group's tokens
  float* st = nullptr;                // key-major score / probability tables, one per (sub-group, KV head)
  const int32_t* st_off = nullptr;    // [n_sg] float offset of each sub-group's tables (attn_st_floats each)
  float* ex = nullptr;                // [n][H][ex_stride] the extra keys' scores, then probabilities
  int ex_stride = 0;                  // >= the most extra keys of any token
  float* inv = nullptr;               // [n][H] 1 / sum of e_j
  float* exmax = nullptr;             // [n][H] the largest extra-key score
  float* att = nullptr;               // [n][H][D] output when the caller passes none (workspace)
  int* status = nullptr;              // device word for bounded-wait failures (nullable)
};
// Query vectors (rows x G) one sub-group may hold.
int attn_qmax();
// Key chunks of the score kernel for a context of n_ctx keys.
int attn_key_chunks(int n_ctx);
// Floats of the score / probability tables of one sub-group of `rows` tokens with keys 0 .. maxk - 1 (all KV heads).
int64_t attn_st_floats(int rows, int G, int KV, int maxk);
// out: [n][H][D] floats (nullable); act: the same rows quantized into the GEMM activation layouts (act.qx nullable).
void launch_attention(const float* q, int H, int KV, int D, float scale, const AttnLayer& L, const AttnPlan& p,
                      float* out, const ActQ& act, cudaStream_t s);

// ---- misc (misc.cu) ----
// Token embedding rows (GGUF Q8_0 / Q4_K / Q6_K / F32 / F16 rows) -> x [n][E].
void launch_embed(const uint8_t* tab, uint32_t type, size_t row_bytes, int E, const int32_t* ids, int n, float* x,
                  cudaStream_t s);
// Sequential KV row moves (Model::move_kv semantics, in list order) for every layer and head.
struct KvCacheRef {
  int8_t* k;
  int8_t* v;
  float* ks;
  float* vs;
  int n_layer, kvh, D;
  int64_t n_rows;  // per head per layer
};
// n_lists move lists (list l: count[l] moves from[l * stride + m] -> to[l * stride + m], absolute rows).
void launch_move_kv(const KvCacheRef& c, const int32_t* from, const int32_t* to, const int32_t* count, int n_lists,
                    int stride, cudaStream_t s);

// ---- accept (accept.cu) ----
// Per logits row: (max value, lowest index of it) over V values, index offset vbase (vocab shard).
void launch_argmax(const float* logits, int64_t ld, int m, int V, int vbase, float* best_v, int32_t* best_i,
                   cudaStream_t s);
// Same, written at row * kc (candidate-list layout).
void launch_argmax_kc(const float* logits, int64_t ld, int m, int V, int vbase, int kc, float* best_v,
                      int32_t* best_i, cudaStream_t s);
// Per logits row r: sum[r] = sum over this shard's V values of exp(double(l - mx[r])), tl[r] = the logit of token
// tgt[r] if vbase <= tgt[r] < vbase + V, else 0 (perplexity).
void launch_row_lse(const float* logits, int64_t ld, int m, int V, int vbase, const float* mx, const int32_t* tgt,
                    double* sum, float* tl, cudaStream_t s);
// Per logits row: top-k (value desc, index asc) candidates, stride kc per row; k <= 64.
void launch_topk(const float* logits, int64_t ld, int m, int V, int vbase, int k, int kc, float* cand_v,
                 int32_t* cand_i, cudaStream_t s);
// Tensor parallel: per row, merge tp lists of k candidates ([rank][row][kc]) into the top k ([row][kc]).
void launch_merge_cand(const float* in_v, const int32_t* in_i, int tp, int m, int k, int kc, float* out_v,
                       int32_t* out_i, cudaStream_t s);

// One request of mk_accept, device side.
struct AcceptReq {
  int32_t kk, greedy, seq, cache_len;
  int32_t row0;                // logits row of the root; tree node t at row0 + t (rows contiguous)
  int32_t chain_off;           // into chain / alt
  int32_t q_off, qn_off;       // into q_p / q_id, q_n
  int32_t u_off, n_u;          // into uniforms
  int32_t top_k;
  float temperature, top_p, min_p;
};
struct AcceptOut {
  int32_t n_acc, next, cache_len, u_used, last_node, status;
  int32_t ids[32];
};
// Greedy / sampled acceptance of n_req requests over per-row candidates (cand_v / cand_i, kc per row, sorted
// value desc, index asc). Greedy requests emit their KV moves into from/to/count (list r, stride 32) with
// sequence row base seq * n_ctx.
void launch_accept(const AcceptReq* reqs, int n_req, const float* cand_v, const int32_t* cand_i, int kc,
                   const int32_t* chain, const int32_t* alt, const float* q_p, const int32_t* q_id, const int32_t* q_n,
                   const double* uniforms, int n_ctx, AcceptOut* out, int32_t* from, int32_t* to, int32_t* count,
                   cudaStream_t s);
}  // namespace mkb
