#include "model.hpp"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <stdexcept>
#include <string>

#include "gguf.hpp"
#include "layout.hpp"
#include "nccl_dl.hpp"
#include "repack.hpp"

namespace mkb {

void cuda_check(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw CudaError(std::string("cuda: ") + what + ": " + cudaGetErrorString(e));
}

namespace {

void nccl_check(ncclResult_t r, const char* what) {
  if (r != ncclSuccess) throw NcclError(std::string("nccl: ") + what + ": " + dl_error_string(r));
}

size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

}  // namespace

DevBuf::DevBuf(size_t bytes) {
  if (bytes) cuda_check(cudaMalloc(&p_, bytes), "cudaMalloc");
  n_ = bytes;
}

DevBuf::~DevBuf() {
  if (p_) cudaFree(p_);
}

DevBuf& DevBuf::operator=(DevBuf&& o) noexcept {
  if (this != &o) {
    if (p_) cudaFree(p_);
    p_ = o.p_;
    n_ = o.n_;
    o.p_ = nullptr;
    o.n_ = 0;
  }
  return *this;
}

Model::Model(int device, int tp_rank, int tp_size, const void* nccl_id)
    : device_(device), tp_rank_(tp_rank), tp_size_(tp_size) {
  if (tp_size < 1 || tp_size > 8 || tp_rank < 0 || tp_rank >= tp_size) throw ArgError("init: bad tensor-parallel rank");
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  cuda_check(cudaDeviceGetAttribute(&num_sms_, cudaDevAttrMultiProcessorCount, device), "sm count");
  cuda_check(cudaStreamCreateWithFlags(&stream_, cudaStreamNonBlocking), "stream");
  if (tp_size > 1) {
    if (!nccl_id) throw ArgError("init: tensor parallel needs an NCCL unique id");
    ncclUniqueId id;
    std::memcpy(&id, nccl_id, sizeof id);
    ncclComm_t comm;
    nccl_check(dl_comm_init_rank(&comm, tp_size, id, tp_rank), "ncclCommInitRank");
    nccl_ = comm;
  }
}

Model::~Model() {
  cudaSetDevice(device_);
  for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g);
  graphs_.clear();
  close_tp_exchange();
  if (nccl_) dl_comm_destroy(static_cast<ncclComm_t>(nccl_));
  if (meta_host_) cudaFreeHost(meta_host_);
  if (acc_host_) cudaFreeHost(acc_host_);
  for (auto& e : pev_)
    if (e) cudaEventDestroy(e);
  if (stream_) cudaStreamDestroy(stream_);
}

// ---------------------------------------------------------------------------------------------------------------
// load: read_config (model.cpp:78-101) + Model::Model (model.cpp:112-152) + pack (model.cpp:163-178), per shard.
// ---------------------------------------------------------------------------------------------------------------
ModelCfg read_config(const GgufReader& f) {
  const std::string arch = f.meta_text("general.architecture").value_or("");
  if (arch != "qwen3") throw ArgError("architecture '" + arch + "' unsupported (supported: qwen3)");
  auto need = [&](const std::string& k) {
    auto v = f.meta_int("qwen3." + k);
    if (!v) throw ArgError("model: metadata qwen3." + k + " missing");
    return static_cast<int>(*v);
  };
  ModelCfg c;
  c.n_layer = need("block_count");
  c.n_embd = need("embedding_length");
  c.n_ff = need("feed_forward_length");
  c.n_head = need("attention.head_count");
  c.n_head_kv = static_cast<int>(f.meta_int("qwen3.attention.head_count_kv").value_or(c.n_head));
  c.head_dim = static_cast<int>(f.meta_int("qwen3.attention.key_length").value_or(c.n_embd / c.n_head));
  c.n_ctx_train = static_cast<int>(f.meta_int("qwen3.context_length").value_or(4096));
  c.rope_base = static_cast<float>(f.meta_real("qwen3.rope.freq_base").value_or(10000.0));
  c.rms_eps = static_cast<float>(f.meta_real("qwen3.attention.layer_norm_rms_epsilon").value_or(1e-6));
  if (c.head_dim % 32 || c.n_head % c.n_head_kv) throw ArgError("model: unsupported head layout");
  if (c.n_head / c.n_head_kv > 8)
    throw UnsupportedError("unsupported: more than 8 query heads per KV head (" + std::to_string(c.n_head) + " / " +
                           std::to_string(c.n_head_kv) + ")");
  if (c.head_dim != 64 && c.head_dim != 128 && c.head_dim != 256)
    throw UnsupportedError("unsupported: head_dim " + std::to_string(c.head_dim) + " (64, 128, 256)");
  const TensorView* out = f.find("output.weight");
  if (!out) out = f.find("token_embd.weight");  // tied embeddings
  if (!out) throw ArgError("model: tensor token_embd.weight missing");
  c.n_vocab = static_cast<int>(out->rows());
  return c;
}

TpShard tp_shard(const ModelCfg& c, int ffn_unit, int tp, int rank) {
  if (tp < 1 || rank < 0 || rank >= tp) throw ArgError("tensor parallel: bad rank " + std::to_string(rank) + " of " +
                                                       std::to_string(tp));
  if (c.n_head % tp || c.n_head_kv % tp)
    throw ArgError("tensor parallel: " + std::to_string(tp) + " ranks do not divide the heads");
  if (ffn_unit <= 0 || c.n_ff % ffn_unit) throw ArgError("model: n_ff not a multiple of the ffn_down block");
  TpShard s;
  s.heads = c.n_head / tp;
  s.head0 = rank * s.heads;
  s.kv_heads = c.n_head_kv / tp;
  s.kv_head0 = rank * s.kv_heads;
  // ffn rows in whole k-units of ffn_down (32 or 256 values), as even as the units allow
  const int nfu = c.n_ff / ffn_unit;
  const int fu0 = static_cast<int>(static_cast<int64_t>(rank) * nfu / tp);
  const int fu1 = static_cast<int>(static_cast<int64_t>(rank + 1) * nfu / tp);
  s.ffn0 = fu0 * ffn_unit;
  s.ffn = (fu1 - fu0) * ffn_unit;
  s.vocab0 = static_cast<int64_t>(rank) * c.n_vocab / tp;
  s.vocab = static_cast<int64_t>(rank + 1) * c.n_vocab / tp - s.vocab0;
  if (c.n_embd % (kPanelRows * tp))
    throw ArgError("tensor parallel: " + std::to_string(tp) + " ranks do not divide n_embd in 16-row panels");
  s.embd = c.n_embd / tp;
  s.embd0 = rank * s.embd;
  return s;
}

void Model::load(const std::string& path) {
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  GgufReader f(path);
  ModelCfg c = read_config(f);
  auto weight = [&](const std::string& name, bool required) -> const TensorView* {
    const TensorView* t = f.find(name);
    if (!t) {
      if (required) throw ArgError("model: tensor " + name + " missing");
      return nullptr;
    }
    return t;
  };
  auto norm = [&](const std::string& name, int64_t n) {
    const TensorView* t = f.find(name);
    if (!t) throw ArgError("model: tensor " + name + " missing");
    if (t->type != kF32 || t->nelements() != n)
      throw ArgError("model: norm " + name + " not F32[" + std::to_string(n) + "]");
    return t;
  };
  const TensorView* tok = weight("token_embd.weight", true);
  const TensorView* out = weight("output.weight", false);
  if (!out) out = tok;  // tied embeddings
  cfg_ = c;
  const int tp = tp_size_, r = tp_rank_;
  const int D = c.head_dim, E = c.n_embd;

  any_float_ = false;
  auto check_mat = [&](const TensorView* t) {
    if (!repack_supported(t->type))
      throw UnsupportedError(std::string("unsupported: tensor ") + t->name + " has type " + type_name(t->type) +
                               " (this path streams F32 F16 BF16 Q8_0 Q4_K Q6_K)");
    if (float_type(t->type)) {
      if (tp > 1) throw UnsupportedError("unsupported: F32 / F16 / BF16 matrices under tensor parallelism");
      any_float_ = true;
    }
  };
  // shard geometry (tensor parallel): heads, ffn rows in whole k-units of ffn_down, vocabulary rows
  const TensorView* down0 = weight("blk.0.ffn_down.weight", true);
  check_mat(down0);
  const TpShard sh = tp_shard(c, kunit_values(down0->type), tp, r);
  Hl_ = sh.heads;
  KVl_ = sh.kv_heads;
  F0_ = sh.ffn0;
  Fl_ = sh.ffn;
  V0_ = sh.vocab0;
  Vl_ = sh.vocab;
  {
    const char* e = std::getenv("MALKIN_B200_TP_SPLIT");
    tp_rows_ = tp > 1 && e && std::string(e) == "rows";
  }
  const bool exact_tp = tp > 1 && !tp_rows_;
  E0_ = exact_tp ? sh.embd0 : 0;
  El_ = exact_tp ? sh.embd : E;
  head_blk0_.assign(static_cast<size_t>(tp), 0);
  head_blks_.assign(static_cast<size_t>(tp), 0);
  ffn_blk0_.assign(static_cast<size_t>(tp), 0);
  ffn_blks_.assign(static_cast<size_t>(tp), 0);
  for (int rr = 0; rr < tp; ++rr) {
    const TpShard o = tp_shard(c, kunit_values(down0->type), tp, rr);
    head_blk0_[static_cast<size_t>(rr)] = static_cast<int64_t>(o.head0) * D / 32;
    head_blks_[static_cast<size_t>(rr)] = static_cast<int64_t>(o.heads) * D / 32;
    ffn_blk0_[static_cast<size_t>(rr)] = o.ffn0 / 32;
    ffn_blks_[static_cast<size_t>(rr)] = o.ffn / 32;
  }
  const int64_t HDl = static_cast<int64_t>(Hl_) * D, KDl = static_cast<int64_t>(KVl_) * D;

  // Device byte plan.
  struct Piece {
    const TensorView* t;
    int64_t r0, nr, c0, nc;
    size_t off;  // in wbuf
    int layout;
  };
  std::vector<Piece> pieces;
  size_t total = 0;
  auto add_piece = [&](const TensorView* t, int64_t r0, int64_t nr, int64_t c0, int64_t nc) -> size_t {
    check_mat(t);
    const int u = kunit_values(t->type);
    if (c0 % u || nc % u) throw ArgError("tensor parallel: shard of " + t->name + " not block aligned");
    total = align_up(total, 256);
    const int layout = weight_layout(t->type, nr, nc);
    pieces.push_back({t, r0, nr, c0, nc, total, layout});
    total += repack_layout_bytes(t->type, layout, nr, nc / u);
    weight_bytes_ += static_cast<int64_t>(nr) * static_cast<int64_t>(row_bytes(t->type, nc));
    return pieces.size() - 1;
  };
  weight_bytes_ = 0;
  struct LayerPlan {
    int qkv[3], nqkv, wo, gu[2], ngu, down;
    const TensorView *an, *fn, *qn, *kn;
  };
  std::vector<LayerPlan> lp(static_cast<size_t>(c.n_layer));
  for (int i = 0; i < c.n_layer; ++i) {
    const std::string p = "blk." + std::to_string(i) + ".";
    LayerPlan& L = lp[static_cast<size_t>(i)];
    L.an = norm(p + "attn_norm.weight", E);
    L.fn = norm(p + "ffn_norm.weight", E);
    L.qn = norm(p + "attn_q_norm.weight", D);
    L.kn = norm(p + "attn_k_norm.weight", D);
    const TensorView* wq = weight(p + "attn_q.weight", true);
    const TensorView* wk = weight(p + "attn_k.weight", true);
    const TensorView* wv = weight(p + "attn_v.weight", true);
    const TensorView* wo = weight(p + "attn_output.weight", true);
    const TensorView* wg = weight(p + "ffn_gate.weight", true);
    const TensorView* wu = weight(p + "ffn_up.weight", true);
    const TensorView* wd = weight(p + "ffn_down.weight", true);
    if (wq->cols() != E || wk->cols() != E || wv->cols() != E || wg->cols() != E || wu->cols() != E ||
        wo->cols() != static_cast<int64_t>(c.n_head) * D || wd->cols() != c.n_ff || wq->rows() != static_cast<int64_t>(c.n_head) * D ||
        wk->rows() != static_cast<int64_t>(c.n_head_kv) * D || wv->rows() != static_cast<int64_t>(c.n_head_kv) * D ||
        wg->rows() != c.n_ff || wu->rows() != c.n_ff || wo->rows() != E || wd->rows() != E)
      throw ArgError("model: layer " + std::to_string(i) + " tensor shapes do not match the config");
    if (wd->type != down0->type) throw UnsupportedError("unsupported: ffn_down types differ across layers");
    L.qkv[0] = static_cast<int>(add_piece(wq, r * HDl, HDl, 0, E));
    L.qkv[1] = static_cast<int>(add_piece(wk, r * KDl, KDl, 0, E));
    L.qkv[2] = static_cast<int>(add_piece(wv, r * KDl, KDl, 0, E));
    L.nqkv = 3;
    // attn_output / ffn_down: this rank's output features over the whole input (exact), or all features over this
    // rank's input columns (row split)
    L.wo = static_cast<int>(exact_tp ? add_piece(wo, E0_, El_, 0, static_cast<int64_t>(c.n_head) * D)
                                     : add_piece(wo, 0, E, r * HDl, HDl));
    L.gu[0] = static_cast<int>(add_piece(wg, F0_, Fl_, 0, E));
    L.gu[1] = static_cast<int>(add_piece(wu, F0_, Fl_, 0, E));
    L.ngu = 2;
    L.down = static_cast<int>(exact_tp ? add_piece(wd, E0_, El_, 0, c.n_ff) : add_piece(wd, 0, E, F0_, Fl_));
  }
  const int lm_piece = static_cast<int>(add_piece(out, V0_, Vl_, 0, E));
  // Embedding table (GGUF rows, replicated) and norms (F32) after the matrices.
  total = align_up(total, 256);
  const size_t embd_off = total;
  embd_type_ = tok->type;
  if (type_size(embd_type_).block == 0 || !repack_supported(embd_type_))
    throw UnsupportedError(std::string("unsupported: token_embd type ") + type_name(embd_type_));
  embd_row_bytes_ = row_bytes(tok->type, tok->cols());
  if (tok->cols() != E) throw ArgError("model: token_embd width != n_embd");
  total += tok->nbytes;
  const TensorView* onorm = norm("output_norm.weight", E);
  total = align_up(total, 256);
  const size_t norm_off = total;
  total += static_cast<size_t>(c.n_layer) * (2 * E + 2 * D) * 4 + static_cast<size_t>(E) * 4;

  wbuf_ = DevBuf(total);
  uint8_t* base = wbuf_.get<uint8_t>();
  std::vector<uint8_t> staging;
  for (const Piece& pc : pieces) {
    const int u = kunit_values(pc.t->type);
    const size_t rb = row_bytes(pc.t->type, pc.t->cols());
    const size_t nbytes = repack_layout_bytes(pc.t->type, pc.layout, pc.nr, pc.nc / u);
    staging.resize(nbytes);
    repack_layout(pc.t->type, pc.layout, pc.t->data + static_cast<size_t>(pc.r0) * rb, rb, pc.nr, pc.c0 / u,
                  pc.nc / u, staging.data(), 0);
    cuda_check(cudaMemcpy(base + pc.off, staging.data(), nbytes, cudaMemcpyHostToDevice), "upload weights");
  }
  cuda_check(cudaMemcpy(base + embd_off, tok->data, tok->nbytes, cudaMemcpyHostToDevice), "upload embeddings");
  embd_ = base + embd_off;
  float* nb = reinterpret_cast<float*>(base + norm_off);
  auto put_norm = [&](const TensorView* t, int64_t n) {
    cuda_check(cudaMemcpy(nb, t->data, static_cast<size_t>(n) * 4, cudaMemcpyHostToDevice), "upload norms");
    const float* p = nb;
    nb += n;
    return p;
  };
  auto dev = [&](int idx) {
    const Piece& pc = pieces[static_cast<size_t>(idx)];
    DevWeight w;
    w.type = pc.t->type;
    w.data = base + pc.off;
    w.rows = pc.nr;
    w.cols = pc.nc;
    w.panels = (pc.nr + kPanelRows - 1) / kPanelRows;
    w.kunits = static_cast<int>(pc.nc / kunit_values(pc.t->type));
    w.layout = pc.layout;
    return w;
  };
  // Fuse consecutive same-type pieces (q|k|v, gate|up) into one weight: their panels (tiles) are adjacent in wbuf.
  auto fuse = [&](const int* idx, int cnt, DevWeight* outw, int64_t* cols, int& nout) {
    nout = 0;
    int64_t col = 0;
    for (int i = 0; i < cnt; ++i) {
      DevWeight w = dev(idx[i]);
      const bool adjacent =
          nout > 0 && outw[nout - 1].type == w.type && outw[nout - 1].layout == w.layout &&
          outw[nout - 1].data + repack_layout_bytes(w.type, w.layout, outw[nout - 1].rows, w.kunits) == w.data &&
          outw[nout - 1].rows % layout_row_quantum(w.layout) == 0;
      if (adjacent) {
        outw[nout - 1].rows += w.rows;
        outw[nout - 1].panels = (outw[nout - 1].rows + kPanelRows - 1) / kPanelRows;
      } else {
        outw[nout] = w;
        cols[nout] = col;
        ++nout;
      }
      col += w.rows;
    }
  };
  layers_.assign(static_cast<size_t>(c.n_layer), Layer{});
  for (int i = 0; i < c.n_layer; ++i) {
    const LayerPlan& P = lp[static_cast<size_t>(i)];
    Layer& L = layers_[static_cast<size_t>(i)];
    fuse(P.qkv, P.nqkv, L.qkv, L.qkv_col, L.n_qkv);
    for (int j = 0; j < L.n_qkv; ++j) L.qkv_split[j] = gemm_split_for(L.qkv[j], num_sms_);
    if (L.n_qkv == 3) L.qkv_split[1] = L.qkv_split[0];  // q and k columns are summed with one slice count
    L.wo = dev(P.wo);
    L.wo_split = gemm_split_for(L.wo, num_sms_);
    fuse(P.gu, P.ngu, L.gu, L.gu_col, L.n_gu);
    for (int j = 0; j < L.n_gu; ++j) L.gu_split[j] = gemm_split_for(L.gu[j], num_sms_);
    L.down = dev(P.down);
    L.down_split = gemm_split_for(L.down, num_sms_);
    L.attn_norm = put_norm(P.an, E);
    L.ffn_norm = put_norm(P.fn, E);
    L.q_norm = put_norm(P.qn, D);
    L.k_norm = put_norm(P.kn, D);
  }
  out_norm_ = put_norm(onorm, E);
  lm_head_ = dev(lm_piece);
  qkv_ld_ = HDl + 2 * KDl;
  inv_freq_.clear();
  for (int i = 0; i < D / 2; ++i) inv_freq_.push_back(std::pow(c.rope_base, -2.0f * static_cast<float>(i) / static_cast<float>(D)));
  loaded_ = true;
}

// ---------------------------------------------------------------------------------------------------------------
// alloc_kv (model.cpp:197-202) + scratch for max_batch tokens (model.cpp:139-151).
// ---------------------------------------------------------------------------------------------------------------
void Model::alloc_kv(int n_ctx, int n_seq, int max_batch) {
  if (!loaded_) throw StateError("alloc_kv before load");
  if (n_ctx <= 0 || n_seq <= 0) throw ArgError("alloc_kv: n_ctx and n_seq must be positive");
  if (max_batch <= 0) max_batch = 256;
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g);
  graphs_.clear();
  const ModelCfg& c = cfg_;
  const int D = c.head_dim, E = c.n_embd;
  n_ctx_ = n_ctx;
  n_seq_ = n_seq;
  max_batch_ = max_batch;
  const int64_t R = static_cast<int64_t>(n_seq) * n_ctx;
  const size_t plane = static_cast<size_t>(c.n_layer) * KVl_ * R;
  kv_ = DevBuf(plane * (2 * static_cast<size_t>(D) + 2 * sizeof(float)));
  cuda_check(cudaMemset(kv_.get(), 0, kv_.size()), "kv memset");
  int8_t* kbase = kv_.get<int8_t>();
  int8_t* vbase = kbase + plane * D;
  float* ksb = reinterpret_cast<float*>(vbase + plane * D);
  float* vsb = ksb + plane;
  kv_layers_.resize(static_cast<size_t>(c.n_layer));
  for (int il = 0; il < c.n_layer; ++il) {
    const size_t lo = static_cast<size_t>(il) * KVl_ * R;
    kv_layers_[static_cast<size_t>(il)] = {kbase + lo * D, vbase + lo * D, ksb + lo, vsb + lo, R};
  }
  // RoPE table [pos][cos D/2 | sin D/2], the reference's float angles and libm cos / sin (model.cpp:336-340).
  {
    std::vector<float> tab(static_cast<size_t>(n_ctx) * D);
    for (int p = 0; p < n_ctx; ++p) {
      for (int i = 0; i < D / 2; ++i) {
        const float a = static_cast<float>(p) * inv_freq_[static_cast<size_t>(i)];
        tab[static_cast<size_t>(p) * D + i] = std::cos(a);
        tab[static_cast<size_t>(p) * D + D / 2 + i] = std::sin(a);
      }
    }
    rope_ = DevBuf(tab.size() * 4);
    cuda_check(cudaMemcpy(rope_.get(), tab.data(), tab.size() * 4, cudaMemcpyHostToDevice), "rope table");
  }
  const int NT8 = act_tiles(max_batch);
  const int NB = NT8 * 8;  // token rows of the activation buffers (whole GEMM passes)
  const int64_t HD = static_cast<int64_t>(Hl_) * D;
  const bool exact_tp = tp_size_ > 1 && !tp_rows_;
  // activation blocks: the widest GEMM input (exact tensor parallel: the whole attention output and ffn width)
  const int64_t kmax = exact_tp ? std::max<int64_t>({E, static_cast<int64_t>(c.n_head) * D, c.n_ff})
                                : std::max<int64_t>({E, HD, Fl_});
  const int64_t blocks = kmax / 32;
  int s_qkv = 1, s_gu = 1, s_part = 1;
  for (const Layer& L : layers_) {
    for (int j = 0; j < L.n_qkv; ++j) s_qkv = std::max(s_qkv, L.qkv_split[j]);
    for (int j = 0; j < L.n_gu; ++j) s_gu = std::max(s_gu, L.gu_split[j]);
    s_part = std::max({s_part, L.wo_split, L.down_split});
  }
  qkv_slice_ = static_cast<int64_t>(NB) * qkv_ld_;
  gu_slice_ = static_cast<int64_t>(NB) * 2 * Fl_;
  part_slice_ = static_cast<int64_t>(NB) * E;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t o = off;
    off = align_up(off + bytes, 256);
    return o;
  };
  const size_t o_x = take(static_cast<size_t>(NB) * E * 4), o_y = take(static_cast<size_t>(s_qkv) * qkv_slice_ * 4),
               o_q = take(static_cast<size_t>(NB) * HD * 4), o_att = take(static_cast<size_t>(NB) * HD * 4),
               o_gu = take(static_cast<size_t>(s_gu) * gu_slice_ * 4), o_p = take(static_cast<size_t>(NB) * E * 4),
               o_part = take(static_cast<size_t>(s_part) * part_slice_ * 4),
               o_lg = take(static_cast<size_t>(NB) * Vl_ * 4), o_qx = take(static_cast<size_t>(blocks) * NB * 32),
               o_qc = take(static_cast<size_t>(blocks) * NB * 32),
               o_dx = take(static_cast<size_t>(blocks) * NB * 4), o_dsx = take(static_cast<size_t>(blocks) * NB * 4),
               o_sh = take(static_cast<size_t>(blocks) * NB * 4),
               o_cv = take(static_cast<size_t>(NB) * MK_TOPK_CAP * 4), o_ci = take(static_cast<size_t>(NB) * MK_TOPK_CAP * 4),
               o_gv = take(static_cast<size_t>(tp_size_) * NB * MK_TOPK_CAP * 4),
               o_gi = take(static_cast<size_t>(tp_size_) * NB * MK_TOPK_CAP * 4), o_st = take(256),
               o_tpg = take(exact_tp ? static_cast<size_t>(NB) * E * 4 : 0),
               o_xf = take(any_float_ ? static_cast<size_t>(NB) * kmax * 4 : 0);
  scratch_ = DevBuf(off);
  cuda_check(cudaMemset(scratch_.get(), 0, off), "scratch memset");
  uint8_t* sb = scratch_.get<uint8_t>();
  x_ = reinterpret_cast<float*>(sb + o_x);
  yqkv_ = reinterpret_cast<float*>(sb + o_y);
  q_ = reinterpret_cast<float*>(sb + o_q);
  att_ = reinterpret_cast<float*>(sb + o_att);
  ygu_ = reinterpret_cast<float*>(sb + o_gu);
  p_ = reinterpret_cast<float*>(sb + o_p);
  part_ = reinterpret_cast<float*>(sb + o_part);
  logits_ = reinterpret_cast<float*>(sb + o_lg);
  act_.qx = sb + o_qx;
  // the Q8_0 tensor-core GEMM reads the int8 copy in the UMMA core-matrix order
  act_.qc = sb + o_qc;
  act_.dx = reinterpret_cast<float*>(sb + o_dx);
  act_.dsx = reinterpret_cast<float*>(sb + o_dsx);
  act_.sh = reinterpret_cast<uint32_t*>(sb + o_sh);
  cand_v_ = reinterpret_cast<float*>(sb + o_cv);
  cand_i_ = reinterpret_cast<int32_t*>(sb + o_ci);
  gath_v_ = reinterpret_cast<float*>(sb + o_gv);
  gath_i_ = reinterpret_cast<int32_t*>(sb + o_gi);
  status_ = reinterpret_cast<int*>(sb + o_st);
  tpg_ = exact_tp ? reinterpret_cast<float*>(sb + o_tpg) : nullptr;
  act_.xf = any_float_ ? reinterpret_cast<float*>(sb + o_xf) : nullptr;  // F32 / F16 / BF16 matrices read the floats
  act_.ldxf = kmax;
  if (!exact_tp) setup_tp_exchange(static_cast<size_t>(NB) * E);
  // attention plan geometry
  const int G = c.n_head / c.n_head_kv;
  sg_rows_ = std::max(1, attn_qmax() / G);
  // attention workspace: the key-major score tables of every sub-group (at most one per token, each row padded to
  // att_nqp slots, plus a chunk-maximum row per 128 keys), the extra keys' scores, 1 / sums and the output rows
  {
    const int GA = (G + 1) / 2 * 2;
    attn_st_cap_ = static_cast<int64_t>(KVl_) * (n_ctx + attn_key_chunks(n_ctx)) * max_batch * (GA + 4);
    attn_ex_stride_ = max_batch;
    const int64_t ex = static_cast<int64_t>(max_batch) * Hl_ * attn_ex_stride_;
    const int64_t inv = static_cast<int64_t>(max_batch) * Hl_ * 2, att = static_cast<int64_t>(max_batch) * Hl_ * D;
    attn_ws_ = DevBuf(static_cast<size_t>(attn_st_cap_ + ex + inv + att) * sizeof(float));  // inv + exmax
  }
  meta_cap_ = 0;
  ensure_meta(static_cast<size_t>(max_batch) * 16);
}

void Model::ensure_meta(size_t anc_cap) {
  const size_t MB = static_cast<size_t>(max_batch_);
  const size_t need = 11 * MB + 3 + anc_cap;
  if (need <= meta_cap_) return;
  for (auto& [k, g] : graphs_) cudaGraphExecDestroy(g);
  graphs_.clear();
  const size_t cap = std::max(need, meta_cap_ * 2);
  meta_ = DevBuf(cap * 4);
  if (meta_host_) cudaFreeHost(meta_host_);
  meta_host_ = nullptr;
  cuda_check(cudaMallocHost(reinterpret_cast<void**>(&meta_host_), cap * 4), "pinned meta");
  meta_cap_ = cap;
  int32_t* m = meta_.get<int32_t>();
  d_ids_ = m;
  d_rpos_ = m + MB;
  d_kvat_ = m + 2 * MB;
  d_kvbase_ = m + 3 * MB;
  d_nkeys_ = m + 4 * MB;
  d_ancoff_ = m + 5 * MB;
  d_sgfirst_ = m + 6 * MB + 1;
  d_toksg_ = m + 7 * MB + 2;
  d_outrows_ = m + 8 * MB + 2;
  d_sgmaxk_ = m + 9 * MB + 2;
  d_stoff_ = m + 10 * MB + 2;
  d_anc_ = m + 11 * MB + 3;
}

void Model::stage(int i) {
  if (!profile_) return;
  if (pk_ == pev_.size()) {
    cudaEvent_t e;
    cuda_check(cudaEventCreate(&e), "event");
    pev_.push_back(e);
    pstage_.push_back(-1);
  }
  cuda_check(cudaEventRecord(pev_[pk_], stream_), "event record");
  pstage_[pk_++] = i;
}

// Exchange buffers for the peer-memory rank sum: allocated and zeroed here, their CUDA IPC handles allgathered over
// NCCL (which also orders every rank's zeroing before any rank's first publish), the peers' handles opened. Every
// rank must be able to map every peer; the ranks agree on that with a min-allreduce and fall back to NCCL together
// otherwise (also when MALKIN_B200_TP_REDUCE=nccl). MALKIN_B200_TP_REDUCE=twoshot selects reduce + allgather
// instead of the one-shot gather when every rank sets it.
void Model::setup_tp_exchange(size_t floats) {
  close_tp_exchange();
  if (tp_size_ <= 1) return;
  auto comm = static_cast<ncclComm_t>(nccl_);
  const size_t cap = (floats + 63) / 64 * 64;
  // [data: 2 halves | red: 2 halves | flags[kMaxTp] | flags2[kMaxTp] | epoch, counter, counter2 (32 B apart)]
  const size_t bytes = 4 * cap * sizeof(float) + 2 * kMaxTp * sizeof(int) + 128;
  tpx_ = DevBuf(bytes);
  cuda_check(cudaMemsetAsync(tpx_.get(), 0, bytes, stream_), "tp exchange memset");
  cudaIpcMemHandle_t mine{};
  int ok = 1;
  const char* e = std::getenv("MALKIN_B200_TP_REDUCE");
  if (e && std::string(e) == "nccl") ok = 0;
  tpx_twoshot_ = e && std::string(e) == "twoshot";
  if (ok && cudaIpcGetMemHandle(&mine, tpx_.get()) != cudaSuccess) {
    cudaGetLastError();
    ok = 0;
  }
  DevBuf hbuf(static_cast<size_t>(tp_size_) * sizeof mine + 2 * sizeof(int));
  auto* hb = hbuf.get<uint8_t>();
  cuda_check(cudaMemcpyAsync(hb + tp_rank_ * sizeof mine, &mine, sizeof mine, cudaMemcpyHostToDevice, stream_),
             "ipc handle upload");
  nccl_check(dl_all_gather(hb + tp_rank_ * sizeof mine, hb, sizeof mine, ncclUint8, comm, stream_), "ipc allgather");
  std::vector<cudaIpcMemHandle_t> all(static_cast<size_t>(tp_size_));
  cuda_check(cudaMemcpyAsync(all.data(), hb, all.size() * sizeof mine, cudaMemcpyDeviceToHost, stream_),
             "ipc handle download");
  cuda_check(cudaStreamSynchronize(stream_), "ipc exchange");
  for (int r = 0; r < tp_size_ && ok; ++r) {
    if (r == tp_rank_) continue;
    void* p = nullptr;
    if (cudaIpcOpenMemHandle(&p, all[static_cast<size_t>(r)], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
      cudaGetLastError();
      ok = 0;
    } else {
      tpx_peer_[r] = p;
    }
  }
  // every rank takes the same path: peer exchange only if every rank mapped every peer, two-shot only if every
  // rank asked for it
  int agree[2] = {ok, tpx_twoshot_ ? 1 : 0};
  int* d_ok = reinterpret_cast<int*>(hb + tp_size_ * sizeof mine);
  cuda_check(cudaMemcpyAsync(d_ok, agree, sizeof agree, cudaMemcpyHostToDevice, stream_), "tp ok upload");
  nccl_check(dl_all_reduce(d_ok, d_ok, 2, ncclInt32, ncclMin, comm, stream_), "tp ok allreduce");
  cuda_check(cudaMemcpyAsync(agree, d_ok, sizeof agree, cudaMemcpyDeviceToHost, stream_), "tp ok download");
  cuda_check(cudaStreamSynchronize(stream_), "tp ok");
  const int all_ok = agree[0];
  tpx_twoshot_ = agree[1] != 0;
  if (!all_ok) {
    close_tp_exchange();
    return;
  }
  TpExchange& x = tpx_args_;
  x = TpExchange{};
  for (int r = 0; r < tp_size_; ++r) {
    auto* base = static_cast<uint8_t*>(r == tp_rank_ ? tpx_.get() : tpx_peer_[r]);
    x.data[r] = reinterpret_cast<float*>(base);
    x.red[r] = reinterpret_cast<float*>(base + 2 * cap * sizeof(float));
    x.flags[r] = reinterpret_cast<int*>(base + 4 * cap * sizeof(float));
    x.flags2[r] = x.flags[r] + kMaxTp;
  }
  auto* own = tpx_.get<uint8_t>() + 4 * cap * sizeof(float) + 2 * kMaxTp * sizeof(int);
  x.epoch = reinterpret_cast<int*>(own);
  x.counter = reinterpret_cast<unsigned*>(own + 32);
  x.counter2 = reinterpret_cast<unsigned*>(own + 64);
  x.rank = tp_rank_;
  x.size = tp_size_;
  x.cap = static_cast<int64_t>(cap);
  tpx_on_ = true;
}

void Model::close_tp_exchange() {
  for (auto& p : tpx_peer_) {
    if (p) cudaIpcCloseMemHandle(p);
    p = nullptr;
  }
  tpx_ = DevBuf();
  tpx_on_ = false;
}

void Model::tp_sum(Slices parts, int n) {
  const int E = cfg_.n_embd;
  if (tpx_on_) {
    launch_tp_publish(tpx_args_, parts, E, n, E, stream_);
    if (tpx_twoshot_) {
      launch_tp_reduce(tpx_args_, n, E, status_, stream_);
      launch_tp_allgather(tpx_args_, n, E, p_, status_, stream_);
    } else {
      launch_tp_gather(tpx_args_, n, E, p_, status_, stream_);
    }
  } else {
    launch_sum_slices(parts, E, n, E, p_, stream_);
    allreduce(p_, static_cast<size_t>(n) * E);
  }
}

ActQ Model::act_at(int64_t block) const {
  ActQ v = act_;
  const int64_t npad = static_cast<int64_t>(act_.nt8) * 8;
  v.qx = act_.qx + block * npad * 32;
  v.qc = act_.qc ? act_.qc + block * npad * 32 : nullptr;
  v.dx = act_.dx + block * npad;
  v.dsx = act_.dsx + block * npad;
  v.sh = act_.sh + block * npad;
  return v;
}

void Model::act_gather(const std::vector<int64_t>& start, const std::vector<int64_t>& count, const DevWeight& w) {
  auto comm = static_cast<ncclComm_t>(nccl_);
  const size_t npad = static_cast<size_t>(act_.nt8) * 8;
  nccl_check(dl_group_start(), "group");
  for (int rr = 0; rr < tp_size_; ++rr) {  // rank rr's blocks, broadcast in place (block-major: one range each)
    const size_t b0 = static_cast<size_t>(start[static_cast<size_t>(rr)]);
    const size_t nb = static_cast<size_t>(count[static_cast<size_t>(rr)]);
    if (nb == 0) continue;
    uint8_t* q = (w.layout == kLayoutTc ? act_.qc : act_.qx) + b0 * npad * 32;
    nccl_check(dl_broadcast(q, q, nb * npad * 32, ncclUint8, rr, comm, stream_), "broadcast");
    nccl_check(dl_broadcast(act_.dx + b0 * npad, act_.dx + b0 * npad, nb * npad, ncclFloat, rr, comm, stream_),
               "broadcast");
    if (w.type == kQ4_K)
      nccl_check(dl_broadcast(act_.dsx + b0 * npad, act_.dsx + b0 * npad, nb * npad, ncclFloat, rr, comm, stream_),
                 "broadcast");
    if (w.type == kQ6_K)
      nccl_check(dl_broadcast(act_.sh + b0 * npad, act_.sh + b0 * npad, nb * npad, ncclUint32, rr, comm, stream_),
                 "broadcast");
  }
  nccl_check(dl_group_end(), "group");
}

void Model::out_gather(int n) {
  nccl_check(dl_all_gather(part_, tpg_, static_cast<size_t>(n) * El_, ncclFloat, static_cast<ncclComm_t>(nccl_),
                           stream_),
             "allgather");
  launch_tp_concat(tpg_, tp_size_, n, El_, p_, stream_);
}

void Model::allreduce(float* buf, size_t count) {
  nccl_check(dl_all_reduce(buf, buf, count, ncclFloat, ncclSum, static_cast<ncclComm_t>(nccl_), stream_),
             "allreduce");
}

void Model::gemm(const DevWeight& w, int split, int n, float* y, int64_t ldy, int64_t slice) {
  launch_gemm(w, act_, n, y, ldy, slice, split, status_, stream_);
}

void Model::tune_gemms(int n, int m) {
  const Layer& L = layers_[0];  // every layer has the same shapes
  act_.nt8 = act_tiles(n);
  for (int i = 0; i < L.n_qkv; ++i)
    if (L.qkv_split[i] == 1) gemm_tune(L.qkv[i], act_, n, yqkv_ + L.qkv_col[i], qkv_ld_, status_, stream_);
  if (L.wo_split == 1) gemm_tune(L.wo, act_, n, part_, El_, status_, stream_);
  for (int i = 0; i < L.n_gu; ++i)
    if (L.gu_split[i] == 1)
      gemm_tune(L.gu[i], act_, n, ygu_ + L.gu_col[i], 2 * static_cast<int64_t>(Fl_), status_, stream_);
  if (L.down_split == 1) gemm_tune(L.down, act_, n, part_, El_, status_, stream_);
  if (m > 0) {
    act_.nt8 = act_tiles(m);
    gemm_tune(lm_head_, act_, m, logits_, Vl_, status_, stream_);
  }
}

void Model::run_forward(int n, int m) {
  const ModelCfg& c = cfg_;
  const int D = c.head_dim, E = c.n_embd;
  const float scale = 1.0f / std::sqrt(static_cast<float>(D));
  const int nt8 = act_tiles(n);
  if (profile_) {
    pk_ = 0;
    stage(-1);
  }
  launch_embed(embd_, embd_type_, embd_row_bytes_, E, d_ids_, n, x_, stream_);
  const bool tp = tp_size_ > 1, gx = tp && !tp_rows_;  // gx: exact split (gathered inputs and output slices)
  Slices pending;  // residual contributions not yet added into x (the previous down projection)
  for (int il = 0; il < c.n_layer; ++il) {
    const Layer& L = layers_[static_cast<size_t>(il)];
    act_.nt8 = nt8;
    launch_rmsnorm_quant(x_, E, pending, nullptr, L.attn_norm, c.rms_eps, n, E, act_, stream_);
    for (int i = 0; i < L.n_qkv; ++i) gemm(L.qkv[i], L.qkv_split[i], n, yqkv_ + L.qkv_col[i], qkv_ld_, qkv_slice_);
    stage(0);
    // q / k columns come from the first weight (fused q|k|v, or q then k), v from the last
    const int64_t v_col0 = L.n_qkv == 3 ? L.qkv_col[2] : (L.n_qkv == 2 ? L.qkv_col[1] : qkv_ld_);
    const int v_n = L.n_qkv >= 2 ? L.qkv_split[L.n_qkv - 1] : L.qkv_split[0];
    launch_qkv_post(Slices{yqkv_, L.qkv_split[0], qkv_slice_}, v_n, v_col0, qkv_ld_, n, Hl_, KVl_, D, L.q_norm,
                    L.k_norm, c.rms_eps, rope_.get<float>(), d_rpos_, d_kvat_, q_, kv_layers_[static_cast<size_t>(il)],
                    stream_);
    stage(1);
    act_.nt8 = nt8;
    const size_t rk = static_cast<size_t>(tp_rank_);
    launch_attention(q_, Hl_, KVl_, D, scale, kv_layers_[static_cast<size_t>(il)], plan_, nullptr,
                     gx ? act_at(head_blk0_[rk]) : act_, stream_);
    if (gx) act_gather(head_blk0_, head_blks_, L.wo);
    stage(2);
    gemm(L.wo, L.wo_split, n, part_, El_, part_slice_);
    Slices wo_add{part_, L.wo_split, part_slice_};
    if (gx) {
      out_gather(n);
      wo_add = Slices{p_, 1, 0};
    } else if (tp) {
      tp_sum(wo_add, n);
      wo_add = Slices{p_, 1, 0};
    }
    launch_rmsnorm_quant(x_, E, wo_add, nullptr, L.ffn_norm, c.rms_eps, n, E, act_, stream_);
    stage(3);
    for (int i = 0; i < L.n_gu; ++i) gemm(L.gu[i], L.gu_split[i], n, ygu_ + L.gu_col[i], 2 * static_cast<int64_t>(Fl_), gu_slice_);
    stage(4);
    launch_silu_quant(Slices{ygu_, L.gu_split[0], gu_slice_}, 2 * static_cast<int64_t>(Fl_), Fl_, n,
                      gx ? act_at(ffn_blk0_[rk]) : act_, stream_);
    if (gx) act_gather(ffn_blk0_, ffn_blks_, L.down);
    stage(5);
    gemm(L.down, L.down_split, n, part_, El_, part_slice_);
    pending = Slices{part_, L.down_split, part_slice_};
    if (gx) {
      out_gather(n);
      pending = Slices{p_, 1, 0};
    } else if (tp) {
      tp_sum(pending, n);
      pending = Slices{p_, 1, 0};
    }
    stage(6);
  }
  if (m > 0) {
    act_.nt8 = act_tiles(m);
    launch_rmsnorm_quant(x_, E, pending, d_outrows_, out_norm_, c.rms_eps, m, E, act_, stream_);
    gemm(lm_head_, 1, m, logits_, Vl_, 0);
  }
  stage(7);
}

// ---------------------------------------------------------------------------------------------------------------
// forward (model.cpp:280-323)
// ---------------------------------------------------------------------------------------------------------------
void Model::forward(const mk_batch_token* batch, int n, float* host_logits) {
  if (!loaded_ || n_ctx_ == 0) throw StateError("forward before load / alloc_kv");
  if (n <= 0 || n > max_batch_) throw ArgError("forward: batch size out of range");
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  const ModelCfg& c = cfg_;
  std::vector<int32_t> ids(n), rpos(n), kvat(n), kvbase(n), nkeys(n), ancoff(n + 1), toksg(n), outrows;
  std::vector<int32_t> anc, sgfirst;
  lrow_.assign(static_cast<size_t>(n), -1);
  for (int t = 0; t < n; ++t) {
    const mk_batch_token& b = batch[t];
    const int kv = b.parent < 0 ? b.pos : b.kv;
    if (b.seq < 0 || b.seq >= n_seq_ || b.pos < 0 || b.pos >= n_ctx_ || kv < 0 || kv >= n_ctx_)
      throw ArgError("forward: bad slot");
    if (b.parent >= t || (b.parent >= 0 && batch[b.parent].seq != b.seq)) throw ArgError("forward: bad tree parent");
    if (b.id < 0 || b.id >= c.n_vocab) throw ArgError("forward: token id out of range");
    ids[t] = b.id;
    rpos[t] = b.pos;
    kvbase[t] = b.seq * n_ctx_;
    kvat[t] = kvbase[t] + kv;
    if (b.logits) {
      lrow_[static_cast<size_t>(t)] = static_cast<int>(outrows.size());
      outrows.push_back(t);
    }
  }
  for (int t = 0; t < n; ++t) {
    const mk_batch_token& b = batch[t];
    ancoff[t] = static_cast<int32_t>(anc.size());
    if (b.parent < 0) {
      nkeys[t] = b.pos + 1;
    } else {
      nkeys[t] = nkeys[b.parent];
      for (int i = ancoff[b.parent]; i < ancoff[b.parent + 1]; ++i) anc.push_back(anc[static_cast<size_t>(i)]);
      anc.push_back(kvat[t] - kvbase[t]);
    }
    ancoff[t + 1] = static_cast<int32_t>(anc.size());
  }
  // attention sub-groups: runs of one sequence, at most sg_rows_ rows
  std::vector<int32_t> sgmaxk;
  for (int t = 0; t < n; ++t) {
    if (t == 0 || kvbase[t] != kvbase[t - 1] || t - sgfirst.back() >= sg_rows_) {
      sgfirst.push_back(t);
      sgmaxk.push_back(0);
    }
    toksg[t] = static_cast<int32_t>(sgfirst.size()) - 1;
    sgmaxk.back() = std::max(sgmaxk.back(), nkeys[t]);
  }
  const int n_sg = static_cast<int>(sgfirst.size());
  sgfirst.push_back(n);
  // offsets of the sub-groups' attention score tables
  std::vector<int32_t> stoff(static_cast<size_t>(n_sg) + 1, 0);
  {
    int64_t off = 0;
    for (int g = 0; g < n_sg; ++g) {
      stoff[static_cast<size_t>(g)] = static_cast<int32_t>(off);
      off += attn_st_floats(sgfirst[static_cast<size_t>(g) + 1] - sgfirst[static_cast<size_t>(g)],
                            cfg_.n_head / cfg_.n_head_kv, KVl_, sgmaxk[static_cast<size_t>(g)]);
    }
    if (off > attn_st_cap_ || off > INT32_MAX) throw ArgError("forward: attention workspace exceeded");
    stoff[static_cast<size_t>(n_sg)] = static_cast<int32_t>(off);
  }
  const int m = static_cast<int>(outrows.size());
  ensure_meta(anc.size());
  // pinned staging -> one copy
  const size_t MB = static_cast<size_t>(max_batch_);
  int32_t* h = meta_host_;
  std::copy(ids.begin(), ids.end(), h);
  std::copy(rpos.begin(), rpos.end(), h + MB);
  std::copy(kvat.begin(), kvat.end(), h + 2 * MB);
  std::copy(kvbase.begin(), kvbase.end(), h + 3 * MB);
  std::copy(nkeys.begin(), nkeys.end(), h + 4 * MB);
  std::copy(ancoff.begin(), ancoff.end(), h + 5 * MB);
  std::copy(sgfirst.begin(), sgfirst.end(), h + 6 * MB + 1);
  std::copy(toksg.begin(), toksg.end(), h + 7 * MB + 2);
  std::copy(outrows.begin(), outrows.end(), h + 8 * MB + 2);
  std::copy(sgmaxk.begin(), sgmaxk.end(), h + 9 * MB + 2);
  std::copy(stoff.begin(), stoff.end(), h + 10 * MB + 2);
  std::copy(anc.begin(), anc.end(), h + 11 * MB + 3);
  cuda_check(cudaMemcpyAsync(meta_.get(), h, (11 * MB + 3 + anc.size()) * 4, cudaMemcpyHostToDevice, stream_),
             "meta upload");
  h2d_bytes_ += static_cast<int64_t>((11 * MB + 3 + anc.size()) * 4);
  plan_.n = n;
  plan_.n_sg = n_sg;
  plan_.kchunks = attn_key_chunks(n_ctx_);
  plan_.sg_first = d_sgfirst_;
  plan_.kv_base = d_kvbase_;
  plan_.n_keys = d_nkeys_;
  plan_.anc_off = d_ancoff_;
  plan_.anc = d_anc_;
  plan_.tok_sg = d_toksg_;
  plan_.sg_maxk = d_sgmaxk_;
  {
    float* ws = attn_ws_.get<float>();
    plan_.st = ws;
    plan_.st_off = d_stoff_;
    plan_.ex = ws + attn_st_cap_;
    plan_.ex_stride = attn_ex_stride_;
    plan_.inv = plan_.ex + static_cast<size_t>(max_batch_) * Hl_ * attn_ex_stride_;
    plan_.exmax = plan_.inv + static_cast<size_t>(max_batch_) * Hl_;
    plan_.att = plan_.exmax + static_cast<size_t>(max_batch_) * Hl_;
  }
  plan_.status = status_;

  // kernel shapes measured on first sight of a batch shape (scratch operands; every shape gives identical results)
  if (profile_ || graphs_.find(std::make_tuple(n, m, n_sg)) == graphs_.end()) tune_gemms(n, m);
  if (profile_) {
    run_forward(n, m);
    cuda_check(cudaStreamSynchronize(stream_), "forward");
    for (float& v : stage_ms_) v = 0.0f;
    for (size_t k = 1; k < pk_; ++k) {
      float ms = 0;
      cuda_check(cudaEventElapsedTime(&ms, pev_[k - 1], pev_[k]), "event time");
      if (pstage_[k] >= 0 && pstage_[k] < 8) stage_ms_[pstage_[k]] += ms;
    }
    last_launches_ = -1;
  } else {
    const auto key = std::make_tuple(n, m, n_sg);
    auto it = graphs_.find(key);
    if (it == graphs_.end()) {
      cudaGraph_t g;
      cuda_check(cudaStreamBeginCapture(stream_, cudaStreamCaptureModeThreadLocal), "begin capture");
      try {
        run_forward(n, m);
      } catch (...) {
        cudaStreamEndCapture(stream_, &g);
        if (g) cudaGraphDestroy(g);
        throw;
      }
      cuda_check(cudaStreamEndCapture(stream_, &g), "end capture");
      cudaGraphExec_t ge;
      cuda_check(cudaGraphInstantiate(&ge, g, 0), "graph instantiate");
      size_t nodes = 0;
      cudaGraphGetNodes(g, nullptr, &nodes);
      std::vector<cudaGraphNode_t> nv(nodes);
      cudaGraphGetNodes(g, nv.data(), &nodes);
      size_t kernels = 0;
      for (auto nd : nv) {
        cudaGraphNodeType ty;
        if (cudaGraphNodeGetType(nd, &ty) == cudaSuccess && ty == cudaGraphNodeTypeKernel) ++kernels;
      }
      nodes = kernels;
      cudaGraphDestroy(g);
      if (graphs_.size() >= 16) {
        cudaGraphExecDestroy(graphs_.begin()->second);
        graphs_.erase(graphs_.begin());
      }
      it = graphs_.emplace(key, ge).first;
      graph_nodes_[key] = static_cast<int64_t>(nodes);
    }
    cuda_check(cudaGraphLaunch(it->second, stream_), "graph launch");
    last_launches_ = graph_nodes_[key];
  }
  last_n_ = n;
  last_m_ = m;
  if (host_logits && m > 0) {
    if (tp_size_ == 1) {
      cuda_check(cudaMemcpyAsync(host_logits, logits_, static_cast<size_t>(m) * c.n_vocab * 4, cudaMemcpyDeviceToHost,
                                 stream_),
                 "logits download");
      d2h_bytes_ += static_cast<int64_t>(m) * c.n_vocab * 4;
      cuda_check(cudaStreamSynchronize(stream_), "forward");
      check_status();
    } else {
      // gather every rank's vocab shard: [rank][m][Vl_r] -> host rows of n_vocab
      cuda_check(cudaStreamSynchronize(stream_), "forward");
      const int64_t vmax = (c.n_vocab + tp_size_ - 1) / tp_size_ + 1;
      DevBuf gb(static_cast<size_t>(tp_size_) * m * vmax * 4), sb(static_cast<size_t>(m) * vmax * 4);
      cuda_check(cudaMemset(sb.get(), 0, sb.size()), "memset");
      cuda_check(cudaMemcpy2D(sb.get(), vmax * 4, logits_, Vl_ * 4, Vl_ * 4, m, cudaMemcpyDeviceToDevice), "pack");
      nccl_check(dl_all_gather(sb.get(), gb.get(), static_cast<size_t>(m) * vmax, ncclFloat,
                               static_cast<ncclComm_t>(nccl_), stream_),
                 "allgather logits");
      cuda_check(cudaStreamSynchronize(stream_), "allgather");
      std::vector<float> all(static_cast<size_t>(tp_size_) * m * vmax);
      cuda_check(cudaMemcpy(all.data(), gb.get(), all.size() * 4, cudaMemcpyDeviceToHost), "logits download");
      for (int rk = 0; rk < tp_size_; ++rk) {
        const int64_t v0 = static_cast<int64_t>(rk) * c.n_vocab / tp_size_;
        const int64_t vl = static_cast<int64_t>(rk + 1) * c.n_vocab / tp_size_ - v0;
        for (int row = 0; row < m; ++row)
          std::memcpy(host_logits + static_cast<size_t>(row) * c.n_vocab + v0,
                      all.data() + (static_cast<size_t>(rk) * m + row) * vmax, static_cast<size_t>(vl) * 4);
      }
    }
  }
}

void throw_device_status(int code, const std::string& what) {
  throw TimeoutError(what + ": device pipeline wait gave up (code " + std::to_string(code) + ")");
}

void Model::check_status() {
  int st = 0;
  cuda_check(cudaMemcpy(&st, status_, sizeof st, cudaMemcpyDeviceToHost), "status");
  if (st != 0) {
    cuda_check(cudaMemset(status_, 0, sizeof st), "status reset");
    throw_device_status(st, "forward (results of this step are invalid)");
  }
}

void Model::candidates(int k, std::vector<float>* v, std::vector<int32_t>* ids) {
  if (last_n_ == 0) throw StateError("candidates before forward");
  if (k < 1 || k > MK_MAX_TOPK) throw ArgError("candidates: k outside 1.." + std::to_string(MK_MAX_TOPK));
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  constexpr int kc = MK_TOPK_CAP;
  const int m = last_m_;
  v->assign(static_cast<size_t>(m) * k, 0.0f);
  ids->assign(static_cast<size_t>(m) * k, 0);
  if (m == 0) return;
  const int K = static_cast<int>(std::min<int64_t>(k, Vl_));
  if (K > 1)
    launch_topk(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), K, kc, cand_v_, cand_i_, stream_);
  else
    launch_argmax_kc(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), kc, cand_v_, cand_i_, stream_);
  if (tp_size_ > 1) {
    auto comm = static_cast<ncclComm_t>(nccl_);
    nccl_check(dl_group_start(), "group");
    nccl_check(dl_all_gather(cand_v_, gath_v_, static_cast<size_t>(m) * kc, ncclFloat, comm, stream_), "allgather");
    nccl_check(dl_all_gather(cand_i_, gath_i_, static_cast<size_t>(m) * kc, ncclInt32, comm, stream_), "allgather");
    nccl_check(dl_group_end(), "group");
    launch_merge_cand(gath_v_, gath_i_, tp_size_, m, k, kc, cand_v_, cand_i_, stream_);
  }
  std::vector<float> hv(static_cast<size_t>(m) * kc);
  std::vector<int32_t> hi(static_cast<size_t>(m) * kc);
  cuda_check(cudaMemcpyAsync(hv.data(), cand_v_, hv.size() * 4, cudaMemcpyDeviceToHost, stream_), "candidates");
  cuda_check(cudaMemcpyAsync(hi.data(), cand_i_, hi.size() * 4, cudaMemcpyDeviceToHost, stream_), "candidates");
  cuda_check(cudaStreamSynchronize(stream_), "candidates");
  d2h_bytes_ += static_cast<int64_t>(hv.size() * 8);
  for (int r = 0; r < m; ++r)
    for (int j = 0; j < k; ++j) {
      (*v)[static_cast<size_t>(r) * k + j] = hv[static_cast<size_t>(r) * kc + j];
      (*ids)[static_cast<size_t>(r) * k + j] = hi[static_cast<size_t>(r) * kc + j];
    }
}

void Model::row_nll(const int32_t* targets, double* nll) {
  if (last_n_ == 0) throw StateError("row_nll before forward");
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  const int m = last_m_;
  if (m == 0) return;
  const size_t MB = static_cast<size_t>(max_batch_);
  // scratch: row maxima and target logits in the candidate values, targets in the candidate ids, the argmax
  // indices and the double sums in the gather buffers
  float* mx = cand_v_;
  float* tl = cand_v_ + MB * 32;
  int32_t* tgt = cand_i_;
  double* sum = reinterpret_cast<double*>(gath_v_);
  cuda_check(cudaMemcpyAsync(tgt, targets, static_cast<size_t>(m) * 4, cudaMemcpyHostToDevice, stream_), "targets");
  h2d_bytes_ += static_cast<int64_t>(m) * 4;
  launch_argmax(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), mx, gath_i_, stream_);
  auto comm = static_cast<ncclComm_t>(nccl_);
  if (tp_size_ > 1) nccl_check(dl_all_reduce(mx, mx, m, ncclFloat, ncclMax, comm, stream_), "allreduce max");
  launch_row_lse(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), mx, tgt, sum, tl, stream_);
  if (tp_size_ > 1) {
    nccl_check(dl_group_start(), "group");
    nccl_check(dl_all_reduce(sum, sum, m, ncclDouble, ncclSum, comm, stream_), "allreduce sum");
    nccl_check(dl_all_reduce(tl, tl, m, ncclFloat, ncclSum, comm, stream_), "allreduce logit");
    nccl_check(dl_group_end(), "group");
  }
  std::vector<float> hmx(static_cast<size_t>(m)), htl(static_cast<size_t>(m));
  std::vector<double> hs(static_cast<size_t>(m));
  cuda_check(cudaMemcpyAsync(hmx.data(), mx, static_cast<size_t>(m) * 4, cudaMemcpyDeviceToHost, stream_), "nll");
  cuda_check(cudaMemcpyAsync(htl.data(), tl, static_cast<size_t>(m) * 4, cudaMemcpyDeviceToHost, stream_), "nll");
  cuda_check(cudaMemcpyAsync(hs.data(), sum, static_cast<size_t>(m) * 8, cudaMemcpyDeviceToHost, stream_), "nll");
  cuda_check(cudaStreamSynchronize(stream_), "nll");
  d2h_bytes_ += static_cast<int64_t>(m) * 16;
  for (int r = 0; r < m; ++r)
    nll[r] = targets[r] < 0 ? 0.0 : std::log(hs[static_cast<size_t>(r)]) + hmx[static_cast<size_t>(r)] -
                                          htl[static_cast<size_t>(r)];
}

void Model::move_kv(int from, int to, int seq) {
  if (n_ctx_ == 0) throw StateError("move_kv before alloc_kv");
  if (seq < 0 || seq >= n_seq_ || from < 0 || from >= n_ctx_ || to < 0 || to >= n_ctx_) throw ArgError("move_kv: bad row");
  if (from == to) return;
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  int32_t h[3] = {seq * n_ctx_ + from, seq * n_ctx_ + to, 1};
  DevBuf d(sizeof h);
  cuda_check(cudaMemcpyAsync(d.get(), h, sizeof h, cudaMemcpyHostToDevice, stream_), "move_kv");
  KvCacheRef kc{kv_layers_[0].k, kv_layers_[0].v, kv_layers_[0].ks, kv_layers_[0].vs, cfg_.n_layer, KVl_, cfg_.head_dim,
                static_cast<int64_t>(n_seq_) * n_ctx_};
  int32_t* dp = d.get<int32_t>();
  launch_move_kv(kc, dp, dp + 1, dp + 2, 1, 1, stream_);
  cuda_check(cudaStreamSynchronize(stream_), "move_kv");
}

// ---------------------------------------------------------------------------------------------------------------
// accept: Engine::accept_greedy / accept_sampled on device (engine.cpp:441-507)
// ---------------------------------------------------------------------------------------------------------------
void Model::accept(const mk_proposal* props, int np, mk_accept_result* res) {
  if (last_n_ == 0) throw StateError("accept before forward");
  if (np <= 0) return;
  cuda_check(cudaSetDevice(device_), "cudaSetDevice");
  bool any_sampled = false;
  int K = 1;
  size_t n_chain = 0, n_q = 0, n_qn = 0, n_u = 0;
  for (int i = 0; i < np; ++i) {
    const mk_proposal& p = props[i];
    const bool greedy = p.sampling.temperature <= 0.0f;
    if (p.sampling.presence_penalty != 0.0f || p.sampling.frequency_penalty != 0.0f)
      throw UnsupportedError("unsupported: presence / frequency penalties on the device accept path");
    if (p.seq < 0 || p.seq >= n_seq_) throw ArgError("accept: bad sequence");
    if (p.kk < 0 || p.kk > MK_MAX_DRAFT) throw ArgError("accept: draft length out of range");
    if (p.cache_len < 0 || p.cache_len + 1 + p.kk > n_ctx_) throw ArgError("accept: context full");
    const int rows = greedy ? 2 * p.kk + 1 : p.kk + 1;
    if (p.root < 0 || p.root + rows > last_n_) throw ArgError("accept: proposal rows outside the last batch");
    const int r0 = lrow_[static_cast<size_t>(p.root)];
    for (int t = 0; t < rows; ++t)
      if (r0 < 0 || lrow_[static_cast<size_t>(p.root + t)] != r0 + t) throw ArgError("accept: proposal rows without logits");
    if (p.kk > 0 && !p.chain) throw ArgError("accept: missing chain");
    if (greedy && p.kk > 0 && !p.alt) throw ArgError("accept: missing alt");
    if (!greedy) {
      any_sampled = true;
      if (p.sampling.top_k <= 0 || p.sampling.top_k > MK_MAX_TOPK)
        throw UnsupportedError("unsupported: top_k outside 1.." + std::to_string(MK_MAX_TOPK) + " on the device path");
      K = std::max(K, p.sampling.top_k);
      if (p.kk > 0 && (!p.q_p || !p.q_id || !p.q_n)) throw ArgError("accept: missing draft distributions");
      for (int j = 0; j < p.kk; ++j) n_q += static_cast<size_t>(p.q_n[j]);
      n_qn += static_cast<size_t>(p.kk);
      if (p.n_uniforms > 0 && !p.uniforms) throw ArgError("accept: missing uniforms");
      n_u += static_cast<size_t>(std::max(0, p.n_uniforms));
    }
    n_chain += static_cast<size_t>(p.kk);
  }
  K = std::min<int64_t>(K, Vl_);
  constexpr int kc = MK_TOPK_CAP;
  const int m = last_m_;
  if (any_sampled)
    launch_topk(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), K, kc, cand_v_, cand_i_, stream_);
  else
    launch_argmax_kc(logits_, Vl_, m, static_cast<int>(Vl_), static_cast<int>(V0_), kc, cand_v_, cand_i_, stream_);
  if (tp_size_ > 1) {
    const int kk = any_sampled ? K : 1;
    auto comm = static_cast<ncclComm_t>(nccl_);
    nccl_check(dl_group_start(), "group");
    nccl_check(dl_all_gather(cand_v_, gath_v_, static_cast<size_t>(m) * kc, ncclFloat, comm, stream_), "allgather");
    nccl_check(dl_all_gather(cand_i_, gath_i_, static_cast<size_t>(m) * kc, ncclInt32, comm, stream_), "allgather");
    nccl_check(dl_group_end(), "group");
    launch_merge_cand(gath_v_, gath_i_, tp_size_, m, kk, kc, cand_v_, cand_i_, stream_);
  }
  // tables: reqs | outs | from | to | count | chain | alt | q_n | q_id | q_p | uniforms
  const size_t o_req = 0, o_out = align_up(o_req + np * sizeof(AcceptReq), 16),
               o_from = align_up(o_out + np * sizeof(AcceptOut), 16), o_to = o_from + np * 32 * 4,
               o_cnt = o_to + np * 32 * 4, o_chain = align_up(o_cnt + np * 4, 16), o_alt = o_chain + n_chain * 4,
               o_qn = o_alt + n_chain * 4, o_qid = o_qn + n_qn * 4, o_qp = o_qid + n_q * 4,
               o_u = align_up(o_qp + n_q * 4, 16), total = align_up(o_u + n_u * 8 + 16, 256);
  if (total > acc_cap_) {
    acc_dev_ = DevBuf(total * 2);
    if (acc_host_) cudaFreeHost(acc_host_);
    acc_host_ = nullptr;
    cuda_check(cudaMallocHost(&acc_host_, total * 2), "pinned accept");
    acc_cap_ = total * 2;
  }
  auto* hb = static_cast<uint8_t*>(acc_host_);
  auto* reqs = reinterpret_cast<AcceptReq*>(hb + o_req);
  auto* chain = reinterpret_cast<int32_t*>(hb + o_chain);
  auto* alt = reinterpret_cast<int32_t*>(hb + o_alt);
  auto* qn = reinterpret_cast<int32_t*>(hb + o_qn);
  auto* qid = reinterpret_cast<int32_t*>(hb + o_qid);
  auto* qp = reinterpret_cast<float*>(hb + o_qp);
  auto* uu = reinterpret_cast<double*>(hb + o_u);
  size_t ci = 0, qi = 0, qni = 0, ui = 0;
  for (int i = 0; i < np; ++i) {
    const mk_proposal& p = props[i];
    AcceptReq& R = reqs[i];
    R.kk = p.kk;
    R.greedy = p.sampling.temperature <= 0.0f ? 1 : 0;
    R.seq = p.seq;
    R.cache_len = p.cache_len;
    R.row0 = lrow_[static_cast<size_t>(p.root)];
    R.chain_off = static_cast<int32_t>(ci);
    R.q_off = static_cast<int32_t>(qi);
    R.qn_off = static_cast<int32_t>(qni);
    R.u_off = static_cast<int32_t>(ui);
    R.n_u = R.greedy ? 0 : std::max(0, p.n_uniforms);
    R.top_k = std::min<int>(p.sampling.top_k, static_cast<int>(Vl_ * tp_size_));
    R.temperature = p.sampling.temperature;
    R.top_p = p.sampling.top_p;
    R.min_p = p.sampling.min_p;
    for (int j = 0; j < p.kk; ++j) {
      chain[ci + static_cast<size_t>(j)] = p.chain[j];
      alt[ci + static_cast<size_t>(j)] = R.greedy ? p.alt[j] : -1;
    }
    ci += static_cast<size_t>(p.kk);
    if (!R.greedy) {
      for (int j = 0; j < p.kk; ++j) {
        qn[qni++] = p.q_n[j];
        for (int e = 0; e < p.q_n[j]; ++e) {
          qp[qi] = p.q_p[qi - static_cast<size_t>(R.q_off) + 0];
          qid[qi] = p.q_id[qi - static_cast<size_t>(R.q_off)];
          ++qi;
        }
      }
      for (int j = 0; j < R.n_u; ++j) uu[ui++] = p.uniforms[j];
    }
  }
  uint8_t* db = acc_dev_.get<uint8_t>();
  cuda_check(cudaMemcpyAsync(db, hb, total, cudaMemcpyHostToDevice, stream_), "accept upload");
  h2d_bytes_ += static_cast<int64_t>(total);
  auto* d_out = reinterpret_cast<AcceptOut*>(db + o_out);
  auto* d_from = reinterpret_cast<int32_t*>(db + o_from);
  auto* d_to = reinterpret_cast<int32_t*>(db + o_to);
  auto* d_cnt = reinterpret_cast<int32_t*>(db + o_cnt);
  launch_accept(reinterpret_cast<AcceptReq*>(db + o_req), np, cand_v_, cand_i_, kc,
                reinterpret_cast<int32_t*>(db + o_chain), reinterpret_cast<int32_t*>(db + o_alt),
                reinterpret_cast<float*>(db + o_qp), reinterpret_cast<int32_t*>(db + o_qid),
                reinterpret_cast<int32_t*>(db + o_qn), reinterpret_cast<double*>(db + o_u), n_ctx_, d_out, d_from, d_to,
                d_cnt, stream_);
  KvCacheRef kc_ref{kv_layers_[0].k, kv_layers_[0].v, kv_layers_[0].ks, kv_layers_[0].vs, cfg_.n_layer, KVl_,
                    cfg_.head_dim, static_cast<int64_t>(n_seq_) * n_ctx_};
  launch_move_kv(kc_ref, d_from, d_to, d_cnt, np, 32, stream_);
  auto* h_out = reinterpret_cast<AcceptOut*>(hb + o_out);
  cuda_check(cudaMemcpyAsync(h_out, d_out, np * sizeof(AcceptOut), cudaMemcpyDeviceToHost, stream_), "accept download");
  auto* h_status = reinterpret_cast<int*>(hb + o_cnt);  // the count region is free on the host side
  cuda_check(cudaMemcpyAsync(h_status, status_, sizeof(int), cudaMemcpyDeviceToHost, stream_), "status download");
  d2h_bytes_ += static_cast<int64_t>(np * sizeof(AcceptOut));
  cuda_check(cudaStreamSynchronize(stream_), "accept");
  if (*h_status != 0) {
    const int code = *h_status;
    cuda_check(cudaMemset(status_, 0, sizeof(int)), "status reset");
    throw_device_status(code, "verify step (results of this step are invalid)");
  }
  for (int i = 0; i < np; ++i) {
    const AcceptOut& o = h_out[i];
    if (o.status != 0) throw ArgError("accept: uniform stream too short for request " + std::to_string(i));
    mk_accept_result& r = res[i];
    r.n_accepted = o.n_acc;
    for (int j = 0; j < o.n_acc; ++j) r.accepted[j] = o.ids[j];
    r.next = o.next;
    r.cache_len = o.cache_len;
    r.uniforms_used = o.u_used;
    r.last_node = o.last_node;
  }
}

}  // namespace mkb
