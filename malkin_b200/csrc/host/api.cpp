// The C ABI (include/malkin_b200.h): status codes instead of exceptions, thread-local error text.
#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <memory>
#include <random>
#include <stdexcept>
#include <string>
#include <vector>

#include "../../../include/malkin_b200.h"
#include "engine.hpp"
#include "gguf.hpp"
#include "layout.hpp"
#include "model.hpp"
#include "nccl_dl.hpp"
#include "repack.hpp"
#include "synth.hpp"

struct mk_ctx {
  std::unique_ptr<mkb::Model> model;
};

struct mk_engine {
  std::unique_ptr<mkb::Engine> engine;
  std::vector<mk_gen_event> queue;  // events not yet handed out
  size_t head = 0;
};

struct mk_weight {
  mkb::DevWeight w;
  mkb::DevBuf buf;
  int device = 0;
};

static_assert(sizeof(mk_batch_token) == 24, "mk_batch_token must match malkin::BatchToken");

namespace {

thread_local std::string g_error;

template <typename F>
int guard(int io_code, F&& f) {
  try {
    g_error.clear();
    f();
    return MK_OK;
  } catch (const mkb::ArgError& e) {
    g_error = e.what();
    return MK_ERR_ARG;
  } catch (const mkb::UnsupportedError& e) {
    g_error = e.what();
    return MK_ERR_UNSUPPORTED;
  } catch (const mkb::StateError& e) {
    g_error = e.what();
    return MK_ERR_STATE;
  } catch (const mkb::CudaError& e) {
    g_error = e.what();
    return MK_ERR_CUDA;
  } catch (const mkb::NcclError& e) {
    g_error = e.what();
    return MK_ERR_NCCL;
  } catch (const mkb::TimeoutError& e) {
    g_error = e.what();
    return MK_ERR_TIMEOUT;
  } catch (const std::exception& e) {
    g_error = e.what();
    return io_code;
  } catch (...) {
    g_error = "unknown error";
    return io_code;
  }
}

mkb::Model& model_of(mk_ctx* c) {
  if (!c || !c->model) throw mkb::StateError("null context");
  return *c->model;
}

cudaStream_t as_stream(void* s) { return static_cast<cudaStream_t>(s); }

int current_device() {
  int d = 0;
  mkb::cuda_check(cudaGetDevice(&d), "cudaGetDevice");
  return d;
}

// Temporary quantized-activation buffers for the kernel-level entry points: int8 qx | the same int8 values in the
// tensor-core order (qc) | dx | dsx | sh.
struct TmpAct {
  mkb::DevBuf buf;
  mkb::ActQ act;
  TmpAct(int n, int64_t K) {
    const int nt8 = mkb::act_tiles(n), npad = nt8 * 8;
    const int64_t blocks = K / 32;
    const size_t qx = static_cast<size_t>(blocks) * npad * 32, f = static_cast<size_t>(blocks) * npad * 4;
    const size_t tc = qx;
    buf = mkb::DevBuf(qx + tc + 3 * f + 256);
    auto* p = buf.get<uint8_t>();
    act.qx = p;
    act.qc = p + qx;
    act.dx = reinterpret_cast<float*>(p + qx + tc);
    act.dsx = act.dx + blocks * npad;
    act.sh = reinterpret_cast<uint32_t*>(act.dsx + blocks * npad);
    act.nt8 = nt8;
  }
};

}  // namespace

extern "C" {

const char* mk_last_error(void) { return g_error.c_str(); }

const char* mk_version(void) { return "malkin_b200 0.1.0 (sm_100a)"; }

int mk_synth_gguf(const char* path, const mk_synth_spec* spec, int n_threads) {
  return guard(MK_ERR_IO, [&] {
    if (!path || !spec) throw mkb::ArgError("synth: null argument");
    mkb::SynthSpec s{spec->n_layer,   spec->n_embd,    spec->n_ff,         spec->n_head,
                     spec->n_head_kv, spec->head_dim,  spec->n_vocab,      spec->n_ctx_train,
                     spec->rope_base, spec->rms_eps,   spec->tied,         static_cast<uint32_t>(spec->type_default),
                     static_cast<uint32_t>(spec->type_attn_v), static_cast<uint32_t>(spec->type_ffn_down),
                     static_cast<uint32_t>(spec->type_output), static_cast<uint32_t>(spec->type_embd), spec->sigma,
                     spec->seed, spec->has_eos, spec->eos_token_id};
    mkb::write_synth_gguf(path, s, n_threads);
  });
}

int mk_nccl_unique_id(void* out128) {
  return guard(MK_ERR_NCCL, [&] {
    if (!out128) throw mkb::ArgError("null id buffer");
    ncclUniqueId id;
    if (mkb::dl_get_unique_id(&id) != ncclSuccess) throw mkb::NcclError("ncclGetUniqueId failed");
    static_assert(sizeof(id) == 128, "ncclUniqueId size");
    std::memcpy(out128, &id, sizeof id);
  });
}

int mk_init(int device, int tp_rank, int tp_size, const void* nccl_id, mk_ctx** out) {
  return guard(MK_ERR_CUDA, [&] {
    if (!out) throw mkb::ArgError("null output");
    *out = nullptr;
    auto c = std::make_unique<mk_ctx>();
    c->model = std::make_unique<mkb::Model>(device, tp_rank, tp_size, nccl_id);
    *out = c.release();
  });
}

int mk_shutdown(mk_ctx* ctx) {
  return guard(MK_ERR_CUDA, [&] { delete ctx; });
}

int mk_load_gguf(mk_ctx* ctx, const char* path) {
  return guard(MK_ERR_IO, [&] {
    if (!path) throw mkb::ArgError("null path");
    model_of(ctx).load(path);
  });
}

int mk_alloc_kv(mk_ctx* ctx, int n_ctx, int n_seq, int max_batch) {
  return guard(MK_ERR_ARG, [&] { model_of(ctx).alloc_kv(n_ctx, n_seq, max_batch); });
}

int mk_tp_shard_of(const char* gguf_path, int tp_size, int tp_rank, mk_tp_shard* out) {
  return guard(MK_ERR_ARG, [&] {
    if (!gguf_path || !out) throw mkb::ArgError("tp_shard: null argument");
    mkb::GgufReader f(gguf_path);
    const mkb::ModelCfg c = mkb::read_config(f);
    const mkb::TensorView* down0 = f.find("blk.0.ffn_down.weight");
    if (!down0) throw mkb::ArgError("model: tensor blk.0.ffn_down.weight missing");
    if (!mkb::repack_supported(down0->type)) throw mkb::UnsupportedError("tp_shard: unsupported ffn_down type");
    const mkb::TpShard sh = mkb::tp_shard(c, mkb::kunit_values(down0->type), tp_size, tp_rank);
    *out = mk_tp_shard{sh.head0, sh.heads, sh.kv_head0, sh.kv_heads, sh.ffn0, sh.ffn, sh.vocab0, sh.vocab, sh.embd0,
                       sh.embd};
  });
}

int mk_tp_exchange_check(int size, int twoshot, int n, int cols, int n_calls, const int* absent, int wait_polls,
                         const float* host_parts, float* host_out, int* call_status) {
  return guard(MK_ERR_ARG, [&] {
    if (wait_polls <= 0) throw mkb::ArgError("tp_exchange_check: wait_polls must be positive");
    mkb::tp_exchange_check(size, twoshot != 0, n, cols, n_calls, absent, static_cast<uint32_t>(wait_polls), host_parts,
                           host_out, call_status);
  });
}

int mk_model_config_get(const mk_ctx* ctx, mk_model_config* out) {
  return guard(MK_ERR_ARG, [&] {
    if (!out) throw mkb::ArgError("null output");
    const mkb::Model& m = model_of(const_cast<mk_ctx*>(ctx));
    const mkb::ModelCfg& c = m.cfg();
    *out = mk_model_config{c.n_layer, c.n_embd, c.n_ff, c.n_head, c.n_head_kv, c.head_dim, c.n_ctx_train, c.n_vocab,
                           c.rope_base, c.rms_eps, m.n_ctx(), m.n_seq(), m.tp_rank(), m.tp_size(), m.weight_bytes()};
  });
}

int mk_forward(mk_ctx* ctx, const mk_batch_token* batch, int n, float* host_logits) {
  return guard(MK_ERR_ARG, [&] {
    if (!batch && n > 0) throw mkb::ArgError("null batch");
    model_of(ctx).forward(batch, n, host_logits);
  });
}

int mk_move_kv(mk_ctx* ctx, int from, int to, int seq) {
  return guard(MK_ERR_ARG, [&] { model_of(ctx).move_kv(from, to, seq); });
}

int mk_accept(mk_ctx* ctx, const mk_proposal* props, int n_props, mk_accept_result* out) {
  return guard(MK_ERR_ARG, [&] {
    if (n_props > 0 && (!props || !out)) throw mkb::ArgError("null proposals / results");
    model_of(ctx).accept(props, n_props, out);
  });
}

int mk_verify_step(mk_ctx* ctx, const mk_batch_token* batch, int n, const mk_proposal* props, int n_props,
                   mk_accept_result* out) {
  return guard(MK_ERR_ARG, [&] {
    mkb::Model& m = model_of(ctx);
    if (!batch) throw mkb::ArgError("null batch");
    m.forward(batch, n, nullptr);
    if (n_props > 0) {
      if (!props || !out) throw mkb::ArgError("null proposals / results");
      m.accept(props, n_props, out);
    }
  });
}

int mk_rng_uniforms(uint64_t seed, int64_t skip, int n, double* out) {
  return guard(MK_ERR_ARG, [&] {
    if (n < 0 || skip < 0 || (n > 0 && !out)) throw mkb::ArgError("rng: bad argument");
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<double> u(0.0, 1.0);
    for (int64_t i = 0; i < skip; ++i) (void)u(rng);
    for (int i = 0; i < n; ++i) out[i] = u(rng);
  });
}

int mk_set_profile(mk_ctx* ctx, int on) {
  return guard(MK_ERR_ARG, [&] { model_of(ctx).set_profile(on != 0); });
}

int mk_stage_times(const mk_ctx* ctx, float* ms8) {
  return guard(MK_ERR_ARG, [&] {
    const float* s = model_of(const_cast<mk_ctx*>(ctx)).stage_ms();
    for (int i = 0; i < 8; ++i) ms8[i] = s[i];
  });
}

int64_t mk_last_launch_count(const mk_ctx* ctx) {
  if (!ctx || !ctx->model) return -1;
  return ctx->model->last_launches();
}

int mk_last_io_bytes(mk_ctx* ctx, int64_t* h2d, int64_t* d2h) {
  return guard(MK_ERR_ARG, [&] {
    if (!h2d || !d2h) throw mkb::ArgError("null output");
    model_of(ctx).io_bytes(h2d, d2h);
  });
}

void* mk_stream(const mk_ctx* ctx) {
  if (!ctx || !ctx->model) return nullptr;
  return ctx->model->stream();
}

// ---- kernel-level entry points ----

int mk_weight_upload(int type, const void* host_rows, int64_t rows, int64_t cols, mk_weight** out) {
  return guard(MK_ERR_ARG, [&] {
    if (!host_rows || !out || rows <= 0 || cols <= 0) throw mkb::ArgError("weight_upload: bad argument");
    if (!mkb::repack_supported(static_cast<uint32_t>(type))) throw mkb::UnsupportedError("weight_upload: unsupported type");
    const int u = mkb::kunit_values(static_cast<uint32_t>(type));
    if (cols % u) throw mkb::ArgError("weight_upload: cols not a multiple of the block");
    auto w = std::make_unique<mk_weight>();
    w->device = current_device();
    const size_t rb = mkb::row_bytes(static_cast<uint32_t>(type), cols);
    const int layout = mkb::weight_layout(static_cast<uint32_t>(type), rows, cols);
    const size_t bytes = mkb::repack_layout_bytes(static_cast<uint32_t>(type), layout, rows, cols / u);
    std::vector<uint8_t> staging(bytes);
    mkb::repack_layout(static_cast<uint32_t>(type), layout, static_cast<const uint8_t*>(host_rows), rb, rows, 0,
                       cols / u, staging.data(), 0);
    w->buf = mkb::DevBuf(bytes);
    mkb::cuda_check(cudaMemcpy(w->buf.get(), staging.data(), bytes, cudaMemcpyHostToDevice), "upload");
    w->w.type = static_cast<uint32_t>(type);
    w->w.data = w->buf.get<uint8_t>();
    w->w.rows = rows;
    w->w.cols = cols;
    w->w.panels = (rows + mkb::kPanelRows - 1) / mkb::kPanelRows;
    w->w.kunits = static_cast<int>(cols / u);
    w->w.layout = layout;
    *out = w.release();
  });
}

int mk_weight_free(mk_weight* w) {
  return guard(MK_ERR_CUDA, [&] { delete w; });
}

int64_t mk_weight_device_bytes(const mk_weight* w) { return w ? static_cast<int64_t>(w->buf.size()) : -1; }

int mk_quantize_q8(const float* dev_x, int n, int64_t k, void* dev_blocks, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (n <= 0 || k <= 0 || k % 32) throw mkb::ArgError("quantize_q8: bad shape");
    mkb::launch_quant_blockq8(dev_x, n, k, dev_blocks, as_stream(stream));
    mkb::cuda_check(cudaGetLastError(), "quantize_q8");
  });
}

int mk_matmul(const mk_weight* w, const float* dev_x, int n, float* dev_y, int split_k, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (!w || n <= 0) throw mkb::ArgError("matmul: bad argument");
    cudaStream_t s = as_stream(stream);
    mkb::DevBuf status(sizeof(int));
    mkb::cuda_check(cudaMemsetAsync(status.get(), 0, sizeof(int), s), "memset");
    TmpAct t(n, w->w.cols);
    mkb::launch_quant_rows(dev_x, w->w.cols, n, static_cast<int>(w->w.cols), t.act, s);
    t.act.xf = const_cast<float*>(dev_x);  // F32 / F16 / BF16 weights read the floats themselves
    t.act.ldxf = w->w.cols;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int split = mkb::gemm_slices(w->w, split_k > 0 ? split_k : mkb::gemm_split_for(w->w, sms));
    const int64_t slice = static_cast<int64_t>(n) * w->w.rows;
    mkb::DevBuf slices(split > 1 ? static_cast<size_t>(split) * slice * 4 : 0);
    float* out = split > 1 ? slices.get<float>() : dev_y;
    if (split == 1) mkb::gemm_tune(w->w, t.act, n, out, w->w.rows, status.get<int>(), s);
    mkb::launch_gemm(w->w, t.act, n, out, w->w.rows, slice, split, status.get<int>(), s);
    if (split > 1) mkb::launch_sum_slices(mkb::Slices{out, split, slice}, w->w.rows, n, static_cast<int>(w->w.rows), dev_y, s);
    mkb::cuda_check(cudaGetLastError(), "matmul");
    int st = 0;
    mkb::cuda_check(cudaMemcpyAsync(&st, status.get(), sizeof st, cudaMemcpyDeviceToHost, s), "status");
    mkb::cuda_check(cudaStreamSynchronize(s), "matmul");
    if (st != 0) mkb::throw_device_status(st, "matmul");
  });
}

int mk_matmul_noalloc(const mk_weight* w, const float* dev_x, int n, float* dev_y, int split_k, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (!w || !dev_x || !dev_y || n <= 0 || split_k < 0) throw mkb::ArgError("matmul_noalloc: bad argument");
    if (current_device() != w->device)
      throw mkb::ArgError("matmul_noalloc: the weight lives on device " + std::to_string(w->device) +
                          ", the current device is " + std::to_string(current_device()));
    cudaError_t e = cudaSuccess;
    uint8_t* base = mkb::noalloc_scratch(&e);
    mkb::cuda_check(e, "matmul_noalloc: scratch address");
    const size_t cap = mkb::noalloc_scratch_bytes();
    auto up = [](size_t b) { return (b + 255) / 256 * 256; };
    // [status | qx | tensor-core copy qc | dx | dsx | sh | split-K slices]
    const int nt8 = mkb::act_tiles(n), npad = nt8 * 8;
    const int64_t blocks = w->w.cols / 32;
    const size_t qx = up(static_cast<size_t>(blocks) * npad * 32), f = up(static_cast<size_t>(blocks) * npad * 4);
    const size_t tc = qx;
    const size_t act_end = 256 + qx + tc + 3 * f;
    if (act_end > cap)
      throw mkb::ArgError("matmul_noalloc: " + std::to_string(n) + " tokens x " + std::to_string(w->w.cols) +
                          " values need " + std::to_string(act_end) + " bytes of activations; the fixed scratch holds " +
                          std::to_string(cap) + " (about 76 bytes per token per 32 values)");
    const int64_t slice = static_cast<int64_t>(n) * w->w.rows;
    const size_t room = cap - act_end;
    auto fits = [&](int split) { return split <= 1 || static_cast<size_t>(split) * slice * 4 <= room; };
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int split = mkb::gemm_slices(w->w, split_k > 0 ? split_k : mkb::gemm_split_for(w->w, sms));
    if (!fits(split)) {
      if (split_k > 0)
        throw mkb::ArgError("matmul_noalloc: split_k " + std::to_string(split_k) + " needs " +
                            std::to_string(static_cast<size_t>(split) * slice * 4) +
                            " bytes of partial sums; the fixed scratch has " + std::to_string(room) + " left");
      while (split > 1 && !fits(split)) split = mkb::gemm_slices(w->w, split - 1);
      if (!fits(split)) split = 1;
    }
    cudaStream_t s = as_stream(stream);
    int* status = reinterpret_cast<int*>(base);
    mkb::ActQ act;
    act.qx = base + 256;
    act.qc = act.qx + qx;
    act.dx = reinterpret_cast<float*>(act.qx + qx + tc);
    act.dsx = reinterpret_cast<float*>(reinterpret_cast<uint8_t*>(act.dx) + f);
    act.sh = reinterpret_cast<uint32_t*>(reinterpret_cast<uint8_t*>(act.dsx) + f);
    act.nt8 = nt8;
    act.xf = const_cast<float*>(dev_x);  // F32 / F16 / BF16 weights read the floats themselves
    act.ldxf = w->w.cols;
    float* slices = reinterpret_cast<float*>(base + act_end);
    // the status word must start at zero; activations and slices are fully written before they are read
    mkb::cuda_check(cudaMemsetAsync(status, 0, sizeof(int), s), "matmul_noalloc: clear status");
    mkb::launch_quant_rows(dev_x, w->w.cols, n, static_cast<int>(w->w.cols), act, s);
    float* out = split > 1 ? slices : dev_y;
    mkb::launch_gemm(w->w, act, n, out, w->w.rows, slice, split, status, s);
    if (split > 1) mkb::launch_sum_slices(mkb::Slices{out, split, slice}, w->w.rows, n, static_cast<int>(w->w.rows), dev_y, s);
    mkb::cuda_check(cudaGetLastError(), "matmul_noalloc");
    int st = 0;
    mkb::cuda_check(cudaMemcpyAsync(&st, status, sizeof st, cudaMemcpyDeviceToHost, s), "matmul_noalloc: status");
    mkb::cuda_check(cudaStreamSynchronize(s), "matmul_noalloc");
    if (st != 0) mkb::throw_device_status(st, "matmul_noalloc");
  });
}

int mk_block_dots(const mk_weight* w, const float* dev_x, int n, int32_t* dev_out, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (!w || n <= 0) throw mkb::ArgError("block_dots: bad argument");
    if (mkb::float_type(w->w.type)) throw mkb::UnsupportedError("block_dots: F32 / F16 / BF16 weights have no int8 dots");
    cudaStream_t s = as_stream(stream);
    mkb::DevBuf status(sizeof(int));
    mkb::cuda_check(cudaMemsetAsync(status.get(), 0, sizeof(int), s), "memset");
    TmpAct t(n, w->w.cols);
    mkb::launch_quant_rows(dev_x, w->w.cols, n, static_cast<int>(w->w.cols), t.act, s);
    mkb::launch_block_dots(w->w, t.act, n, dev_out, status.get<int>(), s);
    mkb::cuda_check(cudaGetLastError(), "block_dots");
    int st = 0;
    mkb::cuda_check(cudaMemcpyAsync(&st, status.get(), sizeof st, cudaMemcpyDeviceToHost, s), "status");
    mkb::cuda_check(cudaStreamSynchronize(s), "block_dots");
    if (st != 0) mkb::throw_device_status(st, "block_dots");
  });
}

int mk_quantize_i8(const float* dev_x, int n, int len, int8_t* dev_q, float* dev_scale, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (n <= 0 || len <= 0) throw mkb::ArgError("quantize_i8: bad shape");
    mkb::launch_quant_i8(dev_x, n, len, dev_q, dev_scale, as_stream(stream));
    mkb::cuda_check(cudaGetLastError(), "quantize_i8");
  });
}

int mk_silu_mul(float* dev_g, const float* dev_u, int64_t n, void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (n <= 0) throw mkb::ArgError("silu_mul: bad length");
    mkb::launch_silu_mul(dev_g, dev_u, n, as_stream(stream));
    mkb::cuda_check(cudaGetLastError(), "silu_mul");
  });
}

int mk_attention(const float* dev_q, int n, int H, int KV, int D, const int8_t* dev_k, const int8_t* dev_v,
                 const float* dev_ks, const float* dev_vs, int64_t n_rows, const int32_t* dev_kv_base,
                 const int32_t* dev_n_keys, const int32_t* dev_anc_off, const int32_t* dev_anc, float* dev_out,
                 void* stream) {
  return guard(MK_ERR_ARG, [&] {
    if (n <= 0 || H <= 0 || KV <= 0 || H % KV || H / KV > 8 || (D != 64 && D != 128 && D != 256))
      throw mkb::ArgError("attention: bad shape (H a multiple of KV, at most 8 query heads per KV head, D 64 / 128 / 256)");
    cudaStream_t s = as_stream(stream);
    std::vector<int32_t> kvb(n), nk(n), ao(n + 1);
    mkb::cuda_check(cudaMemcpy(kvb.data(), dev_kv_base, n * 4, cudaMemcpyDeviceToHost), "attention");
    mkb::cuda_check(cudaMemcpy(nk.data(), dev_n_keys, n * 4, cudaMemcpyDeviceToHost), "attention");
    mkb::cuda_check(cudaMemcpy(ao.data(), dev_anc_off, (n + 1) * 4, cudaMemcpyDeviceToHost), "attention");
    const int G = H / KV, rows = std::max(1, mkb::attn_qmax() / G);
    std::vector<int32_t> sgf, tsg(n), sgm;
    int maxk = 1, maxex = 1;
    for (int t = 0; t < n; ++t) {
      maxex = std::max(maxex, ao[t + 1] - ao[t]);
      if (t == 0 || kvb[t] != kvb[t - 1] || t - sgf.back() >= rows) {
        sgf.push_back(t);
        sgm.push_back(0);
      }
      tsg[t] = static_cast<int32_t>(sgf.size()) - 1;
      sgm.back() = std::max(sgm.back(), nk[t]);
      maxk = std::max(maxk, nk[t]);
    }
    const int n_sg = static_cast<int>(sgf.size());
    sgf.push_back(n);
    std::vector<int32_t> stoff(static_cast<size_t>(n_sg) + 1, 0);
    int64_t st_total = 0;
    for (int g = 0; g < n_sg; ++g) {
      stoff[static_cast<size_t>(g)] = static_cast<int32_t>(st_total);
      st_total += mkb::attn_st_floats(sgf[static_cast<size_t>(g) + 1] - sgf[static_cast<size_t>(g)], G, KV,
                                      sgm[static_cast<size_t>(g)]);
    }
    if (st_total > INT32_MAX) throw mkb::ArgError("attention: score tables too large");
    stoff[static_cast<size_t>(n_sg)] = static_cast<int32_t>(st_total);
    mkb::AttnPlan p;
    p.n = n;
    p.n_sg = n_sg;
    p.kchunks = mkb::attn_key_chunks(maxk);
    mkb::DevBuf tabs((sgf.size() + tsg.size() + sgm.size() + stoff.size()) * 4);
    mkb::cuda_check(cudaMemcpy(tabs.get(), sgf.data(), sgf.size() * 4, cudaMemcpyHostToDevice), "attention");
    mkb::cuda_check(cudaMemcpy(tabs.get<int32_t>() + sgf.size(), tsg.data(), tsg.size() * 4, cudaMemcpyHostToDevice),
                    "attention");
    mkb::cuda_check(cudaMemcpy(tabs.get<int32_t>() + sgf.size() + tsg.size(), sgm.data(), sgm.size() * 4,
                               cudaMemcpyHostToDevice),
                    "attention");
    mkb::cuda_check(cudaMemcpy(tabs.get<int32_t>() + sgf.size() + tsg.size() + sgm.size(), stoff.data(),
                               stoff.size() * 4, cudaMemcpyHostToDevice),
                    "attention");
    const int64_t exs = (maxex + 3) / 4 * 4;
    const size_t ws_floats = static_cast<size_t>(st_total) + static_cast<size_t>(n) * H * exs +
                             static_cast<size_t>(n) * H * 2 + static_cast<size_t>(n) * H * D;
    mkb::DevBuf ws(ws_floats * 4);
    p.sg_first = tabs.get<int32_t>();
    p.tok_sg = tabs.get<int32_t>() + sgf.size();
    p.sg_maxk = tabs.get<int32_t>() + sgf.size() + tsg.size();
    p.kv_base = dev_kv_base;
    p.n_keys = dev_n_keys;
    p.anc_off = dev_anc_off;
    p.anc = dev_anc;
    p.st = ws.get<float>();
    p.st_off = tabs.get<int32_t>() + sgf.size() + tsg.size() + sgm.size();
    p.ex = p.st + st_total;
    p.ex_stride = static_cast<int>(exs);
    p.inv = p.ex + static_cast<size_t>(n) * H * exs;
    p.exmax = p.inv + static_cast<size_t>(n) * H;
    p.att = p.exmax + static_cast<size_t>(n) * H;
    mkb::AttnLayer L{const_cast<int8_t*>(dev_k), const_cast<int8_t*>(dev_v), const_cast<float*>(dev_ks),
                     const_cast<float*>(dev_vs), n_rows};
    mkb::launch_attention(dev_q, H, KV, D, 1.0f / std::sqrt(static_cast<float>(D)), L, p, dev_out, mkb::ActQ{}, s);
    mkb::cuda_check(cudaGetLastError(), "attention");
    mkb::cuda_check(cudaStreamSynchronize(s), "attention");
  });
}

}  // extern "C"

// ---------------------------------------------------------------------------------------------------------------
// engine
// ---------------------------------------------------------------------------------------------------------------
namespace {

void drain(mk_engine* e, mk_gen_event* events, int cap, int* n_events) {
  int n = 0;
  while (n < cap && e->head < e->queue.size()) events[n++] = e->queue[e->head++];
  if (e->head == e->queue.size()) e->queue.clear(), e->head = 0;
  if (n_events) *n_events = n;
}

}  // namespace

int mk_engine_create(mk_ctx* target, mk_ctx* draft, int n_draft, mk_engine** out) {
  return guard(MK_ERR_ARG, [&] {
    if (!target || !out || n_draft < 0) throw mkb::ArgError("engine_create: bad argument");
    auto e = std::make_unique<mk_engine>();
    e->engine = std::make_unique<mkb::Engine>(&model_of(target), draft ? &model_of(draft) : nullptr, n_draft);
    *out = e.release();
  });
}

int mk_engine_destroy(mk_engine* e) {
  return guard(MK_ERR_ARG, [&] { delete e; });
}

int mk_engine_submit(mk_engine* e, const mk_gen_request* r, int32_t* request_id) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || !r) throw mkb::ArgError("engine_submit: bad argument");
    const int id = e->engine->submit(*r);
    if (request_id) *request_id = id;
  });
}

int mk_engine_step(mk_engine* e, mk_gen_event* events, int cap, int* n_events) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || cap < 0 || (cap > 0 && !events)) throw mkb::ArgError("engine_step: bad argument");
    e->engine->step(&e->queue);
    drain(e, events, cap, n_events);
  });
}

int mk_engine_events(mk_engine* e, mk_gen_event* events, int cap, int* n_events) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || cap < 0 || (cap > 0 && !events)) throw mkb::ArgError("engine_events: bad argument");
    drain(e, events, cap, n_events);
  });
}

int mk_engine_busy(const mk_engine* e, int* busy) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || !busy) throw mkb::ArgError("engine_busy: bad argument");
    *busy = e->engine->busy() ? 1 : 0;
  });
}

int mk_engine_cancel(mk_engine* e, int32_t request_id) {
  return guard(MK_ERR_ARG, [&] {
    if (!e) throw mkb::ArgError("engine_cancel: bad argument");
    e->engine->cancel(request_id);
  });
}

int mk_engine_stats(const mk_engine* e, int32_t request_id, mk_gen_stats* out) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || !out) throw mkb::ArgError("engine_stats: bad argument");
    *out = e->engine->stats(request_id);
  });
}

int mk_engine_perplexity(mk_engine* e, const int32_t* tokens, int n, int window, int32_t bos, double* mean_nll,
                         int* scored) {
  return guard(MK_ERR_ARG, [&] {
    if (!e || !tokens || !mean_nll) throw mkb::ArgError("engine_perplexity: bad argument");
    *mean_nll = e->engine->perplexity(tokens, n, window, bos, scored);
  });
}
