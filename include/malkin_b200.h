/*
 * malkin_b200 — C ABI of the B200 (sm_100a) speculative-verify path.
 *
 * The path: one target-model forward pass that scores every request's draft tree (Qwen3 dense, GGUF
 * Q8_0 / Q4_K / Q6_K weights, int8 KV cache), then greedy or exact-rejection acceptance of the drafted
 * tokens, on device. Every entry point returns an int status (MK_OK = 0, negative = error) and never
 * throws; mk_last_error() holds the message of the calling thread's last failure.
 *
 * Each entry point names the reference interface it replaces (kekzl/malkin v0.2.0, src/<file>:<line>).
 * Pointers are host pointers unless the parameter name starts with "dev_". Device pointers must be on the
 * current CUDA device (mk_ctx calls: the context's device).
 */
#ifndef MALKIN_B200_H
#define MALKIN_B200_H

#include <stdbool.h>
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MK_OK 0
#define MK_ERR_ARG (-1)         /* bad argument: same cases malkin throws std::runtime_error for */
#define MK_ERR_CUDA (-2)        /* CUDA runtime failure */
#define MK_ERR_NCCL (-3)        /* NCCL failure (tensor parallel) */
#define MK_ERR_UNSUPPORTED (-4) /* valid for malkin, not implemented on this path (e.g. sampling penalties) */
#define MK_ERR_STATE (-5)       /* call order (e.g. forward before alloc_kv) */
#define MK_ERR_IO (-6)          /* file / GGUF parse error */
#define MK_ERR_TIMEOUT (-7)     /* a device-side bounded wait gave up (status read back from the kernel) */

/* ggml type ids as stored in GGUF (gguf.h:12-29). Weights: Q8_0, Q4_K, Q6_K; norms F32. */
#define MK_TYPE_F32 0
#define MK_TYPE_F16 1
#define MK_TYPE_Q8_0 8
#define MK_TYPE_Q4_K 12
#define MK_TYPE_Q6_K 14

#define MK_MAX_DRAFT 32 /* draft tokens per request per step (malkin: n_draft <= kMaxBatch - 1, adaptive <= 8) */

/* Message of the calling thread's last failed call ("" if none). */
const char* mk_last_error(void);
/* Library version string. */
const char* mk_version(void);

/* ---------------------------------------------------------------------------------------------------------
 * Synthetic model writer. malkin has no weight quantizer or GGUF writer; this is the stand-in the benchmark
 * configurations name ("N(0, sigma) seeded weights, norms 1.0, quantized, written as GGUF"). The file is a
 * GGUF v3 that malkin's own GgufFile + read_config (gguf.cpp:205-249, model.cpp:78-101) load unchanged.
 * ------------------------------------------------------------------------------------------------------- */
typedef struct mk_synth_spec {
  int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, n_ctx_train;
  float rope_base, rms_eps;
  int32_t tied;           /* 1: no output.weight (LM head = token_embd, model.cpp:116-117) */
  int32_t type_default;   /* weight type of every matrix not named below */
  int32_t type_attn_v;    /* attn_v.weight */
  int32_t type_ffn_down;  /* ffn_down.weight */
  int32_t type_output;    /* output.weight (or token_embd.weight when tied) */
  int32_t type_embd;      /* token_embd.weight when not tied */
  float sigma;            /* weights ~ N(0, sigma) */
  uint64_t seed;
  int32_t has_eos;        /* 1: write eos_token_id as tokenizer.ggml.eos_token_id (an end-of-generation token) */
  int32_t eos_token_id;
} mk_synth_spec;

/* Writes the model to path with n_threads host threads (0 = all). */
int mk_synth_gguf(const char* path, const mk_synth_spec* spec, int n_threads);

/* ---------------------------------------------------------------------------------------------------------
 * Model context: one per process and GPU (tensor-parallel rank). Replaces malkin::Model (model.h:33-97).
 * ------------------------------------------------------------------------------------------------------- */
typedef struct mk_ctx mk_ctx;

/* One token of a multi-sequence batch; layout-compatible with malkin::BatchToken (model.h:25-30):
 * plain (parent < 0): RoPE position and KV row pos, attends to positions 0..pos of its sequence;
 * tree (parent = batch index of a token of the same sequence, parent < own index): KV row kv, attends to the
 * keys of its parent plus itself. logits: write n_vocab logits for this token. */
typedef struct mk_batch_token {
  int32_t id;
  int32_t seq;
  int32_t pos;
  bool logits;
  int32_t kv;
  int32_t parent;
} mk_batch_token;

typedef struct mk_model_config {
  int32_t n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_ctx_train, n_vocab;
  float rope_base, rms_eps;
  int32_t n_ctx, n_seq;   /* after mk_alloc_kv */
  int32_t tp_rank, tp_size;
  int64_t weight_bytes;   /* GGUF bytes of the matrices this rank streams per forward (incl. LM head shard) */
} mk_model_config;

/* Creates a context on CUDA device `device`. Tensor parallel: tp_size ranks (1, 2, 4, 8), one process per GPU;
 * nccl_id = the 128-byte ncclUniqueId rank 0 created with mk_nccl_unique_id (NULL when tp_size == 1). */
int mk_init(int device, int tp_rank, int tp_size, const void* nccl_id, mk_ctx** out);
/* Fills 128 bytes with a fresh ncclUniqueId (rank 0 calls it and ships it to the other ranks). */
int mk_nccl_unique_id(void* out128);
/* Releases every device resource of the context (NCCL communicator included). */
int mk_shutdown(mk_ctx* ctx);

/* GgufFile + Model(const GgufFile&, n_ctx = 0, n_seq) (gguf.cpp:205, model.cpp:112-152): parses the GGUF,
 * repacks this rank's shard of every matrix into the device panel layout (Model::pack, model.cpp:163-178) and
 * uploads it. The file can be unmapped once this returns. */
int mk_load_gguf(mk_ctx* ctx, const char* path);
/* Model::alloc_kv (model.cpp:197-202): int8 KV cache for n_seq sequences of n_ctx positions, in HBM.
 * max_batch: largest forward batch (malkin: kMaxBatch = 256, model.h:35); 0 = 256. Under tensor parallelism it is
 * collective (every rank calls it with the same arguments): it maps the ranks' exchange buffers into each other
 * with CUDA IPC for the rank sum, so the ranks must be separate processes. */
int mk_alloc_kv(mk_ctx* ctx, int n_ctx, int n_seq, int max_batch);
int mk_model_config_get(const mk_ctx* ctx, mk_model_config* out);

/* The slice of a qwen3 GGUF that tensor-parallel rank tp_rank of tp_size holds (host only, no device; no counterpart
 * in malkin, which runs on one host): q heads [head0, head0 + heads) and kv heads [kv_head0, ...) of the row-split
 * q / k / v, ffn rows [ffn0, ffn0 + ffn) of gate / up in whole ffn_down blocks, output features [embd0, embd0 + embd)
 * of attn_output and ffn_down (each over its whole input, so every sum keeps malkin's block order; the ranks
 * all-gather the quantized inputs of those two and the output slices), vocabulary rows [vocab0, vocab0 + vocab) of
 * the LM head. */
typedef struct mk_tp_shard {
  int32_t head0, heads, kv_head0, kv_heads, ffn0, ffn;
  int64_t vocab0, vocab;
  int32_t embd0, embd;
} mk_tp_shard;
int mk_tp_shard_of(const char* gguf_path, int tp_size, int tp_rank, mk_tp_shard* out);

/* Self-check of the tensor-parallel rank sum (no counterpart in malkin, which has no tensor parallelism). Runs rank 0's
 * own exchange kernels (publish + gather; twoshot != 0: publish + reduce + allgather) on the current device for
 * n_calls consecutive calls, against size - 1 (1..7) peers emulated by the host: before each call the host writes
 * every present peer's partial and the flags it would release. absent[k] (NULL: none) names a peer (1..size-1) that
 * does not take part in call k, or -1; rank 0's waits then give up after wait_polls polls of about 64 ns each.
 * host_parts: n_calls x size x n x cols floats (cols % 4 == 0), rank r's partial of call k; host_out: n_calls x n x
 * cols, the sum over ranks in rank order that rank 0 received; call_status[k]: MK_OK, or MK_ERR_TIMEOUT when a wait of
 * call k gave up. Shows that a wait that runs out reaches the caller and that the calls after it are still right. */
int mk_tp_exchange_check(int size, int twoshot, int n, int cols, int n_calls, const int* absent, int wait_polls,
                         const float* host_parts, float* host_out, int* call_status);

/* Model::forward(const BatchToken*, n, float* logits) (model.cpp:280-323): same validation, same key sets
 * (prefix + tree ancestors), same KV writes. Logits of the rows with .logits set stay on the device for
 * mk_accept; host_logits (nullable) also receives them, n_vocab floats per row in batch order. */
int mk_forward(mk_ctx* ctx, const mk_batch_token* batch, int n, float* host_logits);

/* Model::move_kv (model.cpp:432-440): copies KV row `from` to row `to` of sequence seq, all layers. */
int mk_move_kv(mk_ctx* ctx, int from, int to, int seq);

/* Sampling parameters (sampler.h:10-18). Penalties must be 0 on this path (MK_ERR_UNSUPPORTED otherwise). */
typedef struct mk_sampling {
  float temperature; /* <= 0: greedy */
  float top_p;
  int32_t top_k;     /* <= 0: whole vocabulary (here: limited to MK_MAX_TOPK) */
  float min_p;
  float presence_penalty;
  float frequency_penalty;
} mk_sampling;

#define MK_MAX_TOPK 64

/* One decoding slot's proposal (engine.h:126-131). Greedy: the tree [next, c0, a0, c1, a1, ...] laid out by
 * Engine::build_batch (engine.cpp:362-379) starting at batch index root; sampled: the chain [next, d0, ...]. */
typedef struct mk_proposal {
  int32_t seq;        /* slot = KV sequence */
  int32_t kk;         /* draft tokens (0: plain decode or the first token after a prompt) */
  int32_t root;       /* batch index of the slot's next token in the last mk_forward batch */
  int32_t cache_len;  /* P: KV rows valid before this step (the root's KV row) */
  mk_sampling sampling;
  const int32_t* chain;   /* kk chain tokens */
  const int32_t* alt;     /* greedy: kk runner-up tokens */
  /* sampled: draft distribution of each chain token, q_n[i] (prob, id) entries each, packed back to back */
  const float* q_p;
  const int32_t* q_id;
  const int32_t* q_n;
  /* sampled: this request's uniform stream (std::uniform_real_distribution<double>(0,1) of its mt19937_64),
   * consumed in Sampler order; at most kk + 1 values are used (mk_accept_result.uniforms_used says how many) */
  const double* uniforms;
  int32_t n_uniforms;
} mk_proposal;

typedef struct mk_accept_result {
  int32_t n_accepted;                /* drafted tokens kept */
  int32_t accepted[MK_MAX_DRAFT];    /* their ids, in order */
  int32_t next;                      /* next token (bonus / correction / sample) */
  int32_t cache_len;                 /* KV rows valid after the step: P + 1 + n_accepted */
  int32_t uniforms_used;
  int32_t last_node;                 /* greedy: tree node the walk ended on (0 root, 1 + 2i chain i, 2 + 2i alt i);
                                        Engine::accept_greedy's `cur`, for the adaptive draft length */
} mk_accept_result;

/* Engine::accept_greedy / accept_sampled + Sampler::distribution / verify / draw (engine.cpp:441-507,
 * sampler.cpp:22-97) over the device logits of the last mk_forward, with Model::move_kv of the accepted tree
 * path on device (greedy). No logits cross to the host. The host keeps emit(): EOG / stop strings / budget. */
int mk_accept(mk_ctx* ctx, const mk_proposal* props, int n_props, mk_accept_result* out);

/* The uniform stream a malkin Sampler draws from (sampler.h:39 std::mt19937_64 seeded with `seed`,
 * sampler.cpp:66 / 82 std::uniform_real_distribution<double>(0, 1)): values skip .. skip + n - 1. The host keeps
 * one stream per request and passes the unconsumed tail to mk_accept. */
int mk_rng_uniforms(uint64_t seed, int64_t skip, int n, double* out);

/* One verify step: mk_forward (no host logits) + mk_accept, as one call (Engine::step's model part,
 * engine.cpp:397-421 minus the host-side emit). */
int mk_verify_step(mk_ctx* ctx, const mk_batch_token* batch, int n, const mk_proposal* props, int n_props,
                   mk_accept_result* out);

/* ---------------------------------------------------------------------------------------------------------
 * Engine: continuous batching with speculative decoding over device models, malkin::Engine (engine.h:47-141,
 * engine.cpp:191-559) at the token level. One target context and an optional draft context (same vocabulary,
 * same n_ctx and n_seq, on the same GPU); one KV sequence per slot. Each mk_engine_step is Engine::worker_loop's
 * admission plus Engine::step: waiting requests go to idle slots with the longest common prompt prefix, decoding
 * slots get an adaptive draft length (plan_drafts), the draft proposes (greedy: top-1 chain and top-2 siblings;
 * sampled: a chain drawn from the draft's distribution with its own seed + 1 stream), one target batch holds the
 * trees / chains and then prompt chunks, acceptance runs on the device, emission on the host.
 * Detokenization, stop strings and chat templates stay with the caller: it passes the end-of-generation ids and
 * ends a request with mk_engine_cancel (malkin's on_text returning false). Calls on one engine are not thread-safe.
 * ------------------------------------------------------------------------------------------------------- */
#define MK_FINISH_STOP 1      /* end-of-generation token (finish_reason "stop") */
#define MK_FINISH_LENGTH 2    /* max_tokens reached or the context is full ("length") */
#define MK_FINISH_CANCELLED 3 /* mk_engine_cancel ("cancelled") */

typedef struct mk_gen_request { /* GenRequest (engine.h:29-34) with token ids */
  const int32_t* prompt;
  int32_t n_prompt;           /* 1 .. n_ctx - 1 */
  int32_t max_tokens;         /* 0: until the context ends */
  mk_sampling sampling;       /* temperature <= 0: greedy; else top_k 1 .. MK_MAX_TOPK; penalties 0 */
  uint64_t seed;              /* SamplingParams::seed (sampler.h:17); 0: random */
  const int32_t* eog;         /* end-of-generation token ids (Tokenizer::is_eog) */
  int32_t n_eog;
} mk_gen_request;

typedef struct mk_gen_event {
  int32_t request;
  int32_t token;   /* an emitted token, or -1 when the request finished */
  int32_t finish;  /* 0 for a token, else MK_FINISH_* */
} mk_gen_event;

typedef struct mk_gen_stats { /* GenResult's counters (engine.h:36-42) */
  int32_t prompt_tokens, cached_tokens, completion_tokens, drafted, accepted;
  int32_t finish; /* 0 while running */
} mk_gen_stats;

typedef struct mk_engine mk_engine;

/* draft may be NULL (plain decoding). n_draft: largest draft length (0: malkin's default 8; at most MK_MAX_DRAFT). */
int mk_engine_create(mk_ctx* target, mk_ctx* draft, int n_draft, mk_engine** out);
int mk_engine_destroy(mk_engine* e);
/* Queues a request (Engine::generate, engine.cpp:227-242); MK_ERR_ARG for an empty prompt or one that fills the
 * context, MK_ERR_UNSUPPORTED for penalties or a top_k the device accept cannot take. */
int mk_engine_submit(mk_engine* e, const mk_gen_request* r, int32_t* request_id);
/* One step; then up to cap queued events in emission order (tokens of a request in order, its finish last). Events
 * that do not fit stay queued for the next call (cap 0 just steps). */
int mk_engine_step(mk_engine* e, mk_gen_event* events, int cap, int* n_events);
/* Queued events without stepping. */
int mk_engine_events(mk_engine* e, mk_gen_event* events, int cap, int* n_events);
/* 1 while any request is waiting or in flight, else 0. */
int mk_engine_busy(const mk_engine* e, int* busy);
/* Ends the request at its next emitted token (a waiting one at the next step) with MK_FINISH_CANCELLED. */
int mk_engine_cancel(mk_engine* e, int32_t request_id);
int mk_engine_stats(const mk_engine* e, int32_t request_id, mk_gen_stats* out);
/* Engine::perplexity (engine.cpp:525-559) over token ids: mean negative log-likelihood of the second half of each
 * window of `window` tokens (at most n_ctx); bos >= 0 replaces each window's first token (Tokenizer::add_bos).
 * Uses sequence 0; no request may be in flight (MK_ERR_STATE). */
int mk_engine_perplexity(mk_engine* e, const int32_t* tokens, int n, int window, int32_t bos, double* mean_nll,
                         int* scored);

/* Per-stage device time of the last forward, ms, in the 8 MALKIN_PROFILE stages (model.cpp:52-76):
 * norm+qkv, qk-norm/rope/kv, attention, wo+res+norm, gate+up, silu+quant, down, output. Enabled by
 * mk_set_profile(ctx, 1) (forward then runs without its CUDA graph). */
int mk_set_profile(mk_ctx* ctx, int on);
int mk_stage_times(const mk_ctx* ctx, float* ms8);
/* Kernel launches issued by the last mk_forward / mk_accept / mk_verify_step (graph nodes counted). */
int64_t mk_last_launch_count(const mk_ctx* ctx);
/* Host->device and device->host bytes the context copied since the previous call of this function. */
int mk_last_io_bytes(mk_ctx* ctx, int64_t* h2d, int64_t* d2h);
/* The CUDA stream the context launches on (cudaStream_t), for callers that time with events. */
void* mk_stream(const mk_ctx* ctx);

/* ---------------------------------------------------------------------------------------------------------
 * Kernel-level entry points (the kern:: / quant.h seam, kernels.h:28-84, quant.h:44-75), on the current device,
 * on device buffers; for parity tests and callers that keep their own model. stream: cudaStream_t or NULL.
 * ------------------------------------------------------------------------------------------------------- */
typedef struct mk_weight mk_weight;

/* pack_weight_into (quant.cpp:218-229): repacks rows x cols GGUF rows of `type` (host, row-major) into the
 * device panel layout on the current device. */
int mk_weight_upload(int type, const void* host_rows, int64_t rows, int64_t cols, mk_weight** out);
int mk_weight_free(mk_weight* w);
int64_t mk_weight_device_bytes(const mk_weight* w);

/* quantize_row_q8 over n rows (quant.cpp:132, 193-199, kernels_avx512.cpp:66-80): dev_x n x k floats (row stride
 * k), dev_blocks n * k/32 malkin BlockQ8 {float d; int16 s[2]; int8 qs[32]} (40 bytes each). */
int mk_quantize_q8(const float* dev_x, int n, int64_t k, void* dev_blocks, void* stream);

/* matmul (quant.cpp:330-351): dev_y[t * rows + r] = W[r] . x[t], activations quantized to Q8 blocks on device.
 * split_k = 1 keeps malkin's per-row block order (results bit-identical to its compact panel kernels);
 * 0 = choose for speed. */
int mk_matmul(const mk_weight* w, const float* dev_x, int n, float* dev_y, int split_k, void* stream);

/* mk_matmul without any device allocation (no counterpart in the reference, which multiplies on the host): the
 * quantized activations, split-K partial sums and status word live in a fixed 16 MiB scratch array of this library
 * (a __device__ variable, one per device), so the call makes no cudaMalloc / cudaFree and never waits on the whole
 * device the way cudaFree does. For callers that must not allocate per call: engines that reserve all HBM for the
 * KV cache at start-up, and latency-bound loops that must not stall other streams. Same arguments and results as
 * mk_matmul. Limits: about 76 bytes per token per 32 values of activations must fit (for example 256 tokens x
 * 16384 values); split_k = 0 lowers the split until the partial sums fit, an
 * explicit split_k whose partial sums do not fit is rejected with MK_ERR_ARG. Calls on one device share the scratch:
 * calls that overlap in time (other streams, other threads) race, so serialise them. Each call synchronizes `stream`
 * before it returns (it reads the kernels' status word back). The first call on each device looks up the scratch
 * address and keeps it; make that first call before any stream capture. The kept address belongs to the device's
 * primary context and does not survive cudaDeviceReset: a process that resets a device must not call this entry
 * point on that device afterwards. */
int mk_matmul_noalloc(const mk_weight* w, const float* dev_x, int n, float* dev_y, int split_k, void* stream);

/* Exact integer block dot products of the GEMM (gemm_avx512.cpp:83-98, 130-141, 179-199): dev_out[(r * n + t) *
 * nblk + b] = sum of w * x over block b (Q8_0, Q4_K: 32 values; Q6_K: 16 values, nblk = cols/16). */
int mk_block_dots(const mk_weight* w, const float* dev_x, int n, int32_t* dev_out, void* stream);

/* quantize_i8 (quant.cpp:134-140) of n rows of len values: dev_q int8, dev_scale one float per row. */
int mk_quantize_i8(const float* dev_x, int n, int len, int8_t* dev_q, float* dev_scale, void* stream);

/* kern::silu_mul (kernels_avx512.cpp:271-280) in place on dev_g (n values). */
int mk_silu_mul(float* dev_g, const float* dev_u, int64_t n, void* stream);

/* Tree-masked GQA attention (Model::attention + kern::attend_gqa, model.cpp:204-247, kernels_avx512.cpp:229-307)
 * on caller buffers: n query tokens x H heads x D (dev_q, float); KV cache of one layer in this library's
 * head-major layout: dev_k / dev_v int8 [KV][n_rows][D], dev_ks / dev_vs float [KV][n_rows];
 * per token: dev_kv_base (first row of its sequence), dev_n_keys (contiguous keys from kv_base), extra key rows
 * (relative to kv_base) dev_anc[dev_anc_off[t] .. dev_anc_off[t+1]). dev_out n x H x D. */
int mk_attention(const float* dev_q, int n, int H, int KV, int D, const int8_t* dev_k, const int8_t* dev_v,
                 const float* dev_ks, const float* dev_vs, int64_t n_rows, const int32_t* dev_kv_base,
                 const int32_t* dev_n_keys, const int32_t* dev_anc_off, const int32_t* dev_anc, float* dev_out,
                 void* stream);

#ifdef __cplusplus
}
#endif

#endif /* MALKIN_B200_H */
