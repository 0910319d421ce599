// Qwen3 dense decoder on one B200 (one tensor-parallel rank): the B200 counterpart of malkin::Model
// (model.h:33-97). Weights live in HBM in the device panel layout; the int8 KV cache is HBM-resident; a forward
// pass is a fixed kernel sequence replayed as a CUDA graph per batch shape.
#pragma once
#include <cuda_runtime_api.h>

#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <stdexcept>
#include <tuple>
#include <vector>

#include "../../../include/malkin_b200.h"
#include "../kernels/kernels.hpp"
#include "gguf.hpp"

namespace mkb {

struct ModelCfg {
  int n_layer = 0, n_embd = 0, n_ff = 0, n_head = 0, n_head_kv = 0, head_dim = 0, n_ctx_train = 0, n_vocab = 0;
  float rope_base = 10000.0f, rms_eps = 1e-6f;
};

// cudaMalloc'd bytes, freed on destruction.
class DevBuf {
 public:
  DevBuf() = default;
  explicit DevBuf(size_t bytes);
  ~DevBuf();
  DevBuf(const DevBuf&) = delete;
  DevBuf& operator=(const DevBuf&) = delete;
  DevBuf(DevBuf&& o) noexcept : p_(o.p_), n_(o.n_) { o.p_ = nullptr, o.n_ = 0; }
  DevBuf& operator=(DevBuf&& o) noexcept;
  template <typename T = void>
  T* get() const {
    return static_cast<T*>(p_);
  }
  size_t size() const { return n_; }

 private:
  void* p_ = nullptr;
  size_t n_ = 0;
};

// Error kinds, mapped to the C ABI status codes by api.cpp.
struct ArgError : std::runtime_error {          // MK_ERR_ARG: malkin throws for the same inputs
  using std::runtime_error::runtime_error;
};
struct UnsupportedError : std::runtime_error {  // MK_ERR_UNSUPPORTED
  using std::runtime_error::runtime_error;
};
struct StateError : std::runtime_error {        // MK_ERR_STATE
  using std::runtime_error::runtime_error;
};
struct CudaError : std::runtime_error {         // MK_ERR_CUDA
  using std::runtime_error::runtime_error;
};
struct NcclError : std::runtime_error {         // MK_ERR_NCCL
  using std::runtime_error::runtime_error;
};
struct TimeoutError : std::runtime_error {      // MK_ERR_TIMEOUT: a device-side bounded wait gave up
  using std::runtime_error::runtime_error;
};

// Throws CudaError with the CUDA error string.
void cuda_check(cudaError_t e, const char* what);
// Throws for a nonzero device status word: UnsupportedError for an activation outside the fp16 range of the
// split-fp16 GEMM (malkin's f32 path has no such limit), TimeoutError for a bounded wait that gave up.
void throw_device_status(int code, const std::string& what);

// The config of a qwen3 GGUF (read_config, model.cpp:78-101), and the slice of it one tensor-parallel rank holds:
// q / kv heads (column split), ffn rows in whole k-units of ffn_down, vocabulary rows (split of the LM head).
ModelCfg read_config(const GgufReader& f);
// mk_tp_exchange_check (tp_check.cpp): rank 0's rank-sum kernels against host-emulated peers on one device.
void tp_exchange_check(int size, bool twoshot, int n, int cols, int n_calls, const int* absent, uint32_t wait_polls,
                       const float* parts, float* out, int* call_status);
struct TpShard {
  int head0 = 0, heads = 0, kv_head0 = 0, kv_heads = 0, ffn0 = 0, ffn = 0;
  int64_t vocab0 = 0, vocab = 0;
  int embd0 = 0, embd = 0;  // output features of attn_output / ffn_down
};
TpShard tp_shard(const ModelCfg& c, int ffn_unit, int tp, int rank);

class Model {
 public:
  Model(int device, int tp_rank, int tp_size, const void* nccl_id);
  ~Model();

  void load(const std::string& path);
  void alloc_kv(int n_ctx, int n_seq, int max_batch);
  void forward(const mk_batch_token* batch, int n, float* host_logits);
  void move_kv(int from, int to, int seq);
  void accept(const mk_proposal* props, int n_props, mk_accept_result* out);
  // Top-k candidates (value desc, index asc; k <= MK_MAX_TOPK) of every logits row of the last forward, on the host:
  // rows x k values and token ids (tensor parallel: merged over the vocabulary shards).
  void candidates(int k, std::vector<float>* v, std::vector<int32_t>* ids);
  // Per logits row r of the last forward with targets[r] >= 0: log(sum exp(l - mx)) + mx - l[targets[r]], the
  // negative log-likelihood Engine::perplexity adds (engine.cpp:545-552); rows with targets[r] < 0 get 0.
  void row_nll(const int32_t* targets, double* nll);
  int max_batch() const { return max_batch_; }
  int last_logit_rows() const { return last_m_; }

  const ModelCfg& cfg() const { return cfg_; }
  int n_ctx() const { return n_ctx_; }
  int n_seq() const { return n_seq_; }
  int tp_rank() const { return tp_rank_; }
  int tp_size() const { return tp_size_; }
  int64_t weight_bytes() const { return weight_bytes_; }
  cudaStream_t stream() const { return stream_; }
  void set_profile(bool on) { profile_ = on; }
  const float* stage_ms() const { return stage_ms_; }
  int64_t last_launches() const { return last_launches_; }
  // Host->device and device->host bytes copied since the previous call (then reset).
  void io_bytes(int64_t* h2d, int64_t* d2h) {
    *h2d = h2d_bytes_;
    *d2h = d2h_bytes_;
    h2d_bytes_ = d2h_bytes_ = 0;
  }

 private:
  struct Layer {
    DevWeight qkv[3];
    int64_t qkv_col[3] = {0, 0, 0};
    int qkv_split[3] = {1, 1, 1};  // split-K slices of each GEMM (fixed per weight)
    int n_qkv = 0;
    DevWeight wo;
    int wo_split = 1;
    DevWeight gu[2];
    int64_t gu_col[2] = {0, 0};
    int gu_split[2] = {1, 1};
    int n_gu = 0;
    DevWeight down;
    int down_split = 1;
    const float *attn_norm = nullptr, *ffn_norm = nullptr, *q_norm = nullptr, *k_norm = nullptr;
  };

  void run_forward(int n, int m);               // kernel sequence (captured or direct)
  void tune_gemms(int n, int m);                // measured kernel shapes for n rows (m output rows), before capture
  // y slices = W x: slice s at y + s * slice (split-K partial sums, summed in order by the consumer)
  void gemm(const DevWeight& w, int split, int n, float* y, int64_t ldy, int64_t slice);
  void allreduce(float* buf, size_t count);
  // The rank sum of row-split partials (split-K slices) into p_: peer-memory kernels when the exchange is set up,
  // else slice sum + ncclAllReduce.
  void tp_sum(Slices parts, int n);
  // Exact tensor parallel: the activation blocks [start[r], start[r] + count[r]) that rank r quantized, from every
  // rank to every rank (what weight w reads), and the gathered output slices part_ [n][El_] -> p_ [n][E].
  void act_gather(const std::vector<int64_t>& start, const std::vector<int64_t>& count, const DevWeight& w);
  void out_gather(int n);
  ActQ act_at(int64_t block) const;  // act_ from 32-value block `block` on
  void setup_tp_exchange(size_t floats);
  void close_tp_exchange();
  void stage(int i);                             // profile lap
  void ensure_meta(size_t anc_cap);
  void check_status();  // throws TimeoutError if a kernel recorded a failed bounded wait

  ModelCfg cfg_;
  int device_ = 0, tp_rank_ = 0, tp_size_ = 1, num_sms_ = 148;
  void* nccl_ = nullptr;  // ncclComm_t
  // tensor-parallel exchange over peer memory (tp_reduce.cu): own buffer, peers' IPC mappings, kernel arguments
  DevBuf tpx_;
  void* tpx_peer_[kMaxTp] = {};
  TpExchange tpx_args_;
  bool tpx_on_ = false;
  bool tpx_twoshot_ = false;
  // tensor-parallel split of attn_output / ffn_down: by output features over the whole input (exact, default), or
  // by input columns with the rank sum of partials (MALKIN_B200_TP_SPLIT=rows: not malkin's block order)
  bool any_float_ = false;  // some matrix is F32 / F16 / BF16: the producers also keep the float activations
  bool tp_rows_ = false;
  int E0_ = 0, El_ = 0;                           // this rank's output features of attn_output / ffn_down
  std::vector<int64_t> head_blk0_, head_blks_;   // every rank's 32-value blocks of the attention output
  std::vector<int64_t> ffn_blk0_, ffn_blks_;     // every rank's 32-value blocks of the ffn activations
  float* tpg_ = nullptr;                          // [tp][n][El_] gathered output slices
  cudaStream_t stream_ = nullptr;
  bool loaded_ = false;

  // shard geometry
  int Hl_ = 0, KVl_ = 0, Fl_ = 0, F0_ = 0;  // local q heads, kv heads, ffn rows and first ffn row
  int64_t Vl_ = 0, V0_ = 0;                  // local vocab rows, first row
  int64_t qkv_ld_ = 0;                       // columns of y_qkv
  int64_t weight_bytes_ = 0;

  // weights
  DevBuf wbuf_;
  std::vector<Layer> layers_;
  DevWeight lm_head_;
  const float* out_norm_ = nullptr;
  const uint8_t* embd_ = nullptr;
  uint32_t embd_type_ = 0;
  size_t embd_row_bytes_ = 0;
  std::vector<float> inv_freq_;

  // KV cache + activations
  int n_ctx_ = 0, n_seq_ = 0, max_batch_ = 0;
  DevBuf kv_, rope_, scratch_;
  std::vector<AttnLayer> kv_layers_;
  float *x_ = nullptr, *yqkv_ = nullptr, *q_ = nullptr, *att_ = nullptr, *ygu_ = nullptr, *p_ = nullptr,
        *part_ = nullptr, *logits_ = nullptr;
  int64_t qkv_slice_ = 0, gu_slice_ = 0, part_slice_ = 0;  // floats between split-K slices
  int* status_ = nullptr;                                  // device word: bounded-wait failures
  ActQ act_;
  float* cand_v_ = nullptr;
  int32_t* cand_i_ = nullptr;
  float* gath_v_ = nullptr;
  int32_t* gath_i_ = nullptr;

  // per-forward metadata (device + pinned host staging, one copy per forward)
  DevBuf meta_;
  int32_t* meta_host_ = nullptr;
  size_t meta_cap_ = 0;  // int32 entries
  int32_t *d_ids_ = nullptr, *d_rpos_ = nullptr, *d_kvat_ = nullptr, *d_kvbase_ = nullptr, *d_nkeys_ = nullptr,
          *d_ancoff_ = nullptr, *d_sgfirst_ = nullptr, *d_toksg_ = nullptr, *d_outrows_ = nullptr, *d_sgmaxk_ = nullptr, *d_stoff_ = nullptr, *d_anc_ = nullptr;
  DevBuf attn_ws_;             // attention score tables, extra-key scores, 1 / sums, output rows
  int64_t attn_st_cap_ = 0;     // floats of the score tables
  int attn_ex_stride_ = 0;
  AttnPlan plan_;
  int sg_rows_ = 0;


  // last forward: logits row of each batch index (-1: none), tokens
  std::vector<int> lrow_;
  int last_n_ = 0, last_m_ = 0;

  // accept tables
  DevBuf acc_dev_;
  void* acc_host_ = nullptr;
  size_t acc_cap_ = 0;

  // graphs keyed by (n, m, n_sg)
  std::map<std::tuple<int, int, int>, cudaGraphExec_t> graphs_;
  std::map<std::tuple<int, int, int>, int64_t> graph_nodes_;
  bool profile_ = false;
  std::vector<cudaEvent_t> pev_;  // profile: one event per stage boundary of every layer
  std::vector<int> pstage_;
  size_t pk_ = 0;
  float stage_ms_[8] = {};
  int64_t last_launches_ = 0;
  int64_t h2d_bytes_ = 0, d2h_bytes_ = 0;  // host <-> device bytes since the last io_bytes() read
};

}  // namespace mkb
