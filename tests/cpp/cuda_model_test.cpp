// The binding INTEGRATION.md shows, compiled and run: malkin's own headers (gguf.h, model.h: BatchToken, Model) and
// include/malkin_b200.h in one C++ program. CudaModel below is the snippet's backend. It runs a prompt and a greedy
// draft-tree verify on the GPU, malkin's CPU Model runs the same BatchToken arrays, and the program checks that the
// logits are bit-identical and that mk_accept's walk and KV compaction give malkin's Engine::accept_greedy result.
// Built by oracle/Makefile (it needs the reference headers and oracle/_ref/libmalkin_ref.so); run by
// tests/test_gpu_integration.py with a synthetic GGUF path. Prints "ok" and exits 0 on success.
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf.h"
#include "model.h"
#include "malkin_b200.h"

using namespace malkin;

// ---- the INTEGRATION.md backend ----
struct CudaModel {
  mk_ctx* ctx = nullptr;
  static void check(int rc) {
    if (rc != MK_OK) throw std::runtime_error(mk_last_error());
  }
  CudaModel(const std::string& path, int n_ctx, int n_seq, int device = 0) {
    check(mk_init(device, 0, 1, nullptr, &ctx));
    check(mk_load_gguf(ctx, path.c_str()));
    if (n_ctx > 0) check(mk_alloc_kv(ctx, n_ctx, n_seq, Model::kMaxBatch));
  }
  ~CudaModel() { mk_shutdown(ctx); }
  void forward(const BatchToken* b, int n, float* logits) {
    check(mk_forward(ctx, reinterpret_cast<const mk_batch_token*>(b), n, logits));
  }
  void move_kv(int from, int to, int seq) { check(mk_move_kv(ctx, from, to, seq)); }
};

static int argmax(const float* l, int n) {
  int b = 0;
  for (int i = 1; i < n; ++i)
    if (l[i] > l[b]) b = i;
  return b;
}

int main(int argc, char** argv) {
  if (argc < 2) {
    std::fprintf(stderr, "usage: %s model.gguf\n", argv[0]);
    return 2;
  }
  try {
    const std::string path = argv[1];
    const int n_ctx = 64;
    CudaModel gpu(path, n_ctx, 1);
    GgufFile file(path);
    Model cpu(file, n_ctx, 1);
    const int V = cpu.cfg().n_vocab;
    // prompt: 10 tokens, logits of the last
    std::vector<BatchToken> prompt;
    for (int i = 0; i < 10; ++i) prompt.push_back({(i * 37 + 5) % V, 0, i, i == 9});
    std::vector<float> gl(static_cast<size_t>(V)), cl(static_cast<size_t>(V));
    gpu.forward(prompt.data(), 10, gl.data());
    cpu.forward(prompt.data(), 10, cl.data());
    if (std::memcmp(gl.data(), cl.data(), gl.size() * 4) != 0) throw std::runtime_error("prompt logits differ");
    const int next = argmax(cl.data(), V), P = 10, kk = 3;
    // greedy tree as Engine::build_batch lays it out: [next, c0, a0, c1, a1, c2, a2]; the chain follows the target
    // for two tokens (c0 = its argmax after next, c1 = its argmax after c0), then a token it will not pick
    std::vector<int32_t> chain(kk), alt(kk);
    auto tree = [&] {
      std::vector<BatchToken> b;
      b.push_back({next, 0, P, true});
      for (int i = 0; i < kk; ++i) {
        const int par = i == 0 ? 0 : 2 * i - 1;
        b.push_back({chain[i], 0, P + 1 + i, true, P + 1 + 2 * i, par});
        b.push_back({alt[i], 0, P + 1 + i, true, P + 2 + 2 * i, par});
      }
      return b;
    };
    std::vector<float> tl(static_cast<size_t>(2 * kk + 1) * V), tg(tl.size());
    for (int i = 0; i < kk; ++i) chain[i] = (i * 11 + 3) % V, alt[i] = (i * 17 + 9) % V;
    for (int d = 0; d < 2; ++d) {  // fill the chain from the target's own argmax, depth by depth
      auto b = tree();
      cpu.forward(b.data(), static_cast<int>(b.size()), tl.data());
      chain[d] = argmax(tl.data() + static_cast<size_t>(d == 0 ? 0 : 2 * d - 1) * V, V);
    }
    auto b = tree();
    cpu.forward(b.data(), static_cast<int>(b.size()), tl.data());
    gpu.forward(b.data(), static_cast<int>(b.size()), tg.data());
    if (std::memcmp(tl.data(), tg.data(), tl.size() * 4) != 0) throw std::runtime_error("tree logits differ");
    // malkin's greedy walk (Engine::accept_greedy) on the CPU logits
    std::vector<int32_t> want;
    int cur = 0, want_next = -1;
    for (int i = 0; i < kk; ++i) {
      const int a = argmax(tl.data() + static_cast<size_t>(cur) * V, V);
      const int slot = a == chain[i] ? 1 + 2 * i : (a == alt[i] ? 2 + 2 * i : -1);
      if (slot < 0) {
        want_next = a;
        break;
      }
      cpu.move_kv(P + slot, P + 1 + static_cast<int>(want.size()), 0);
      want.push_back(a);
      cur = slot;
      if (slot == 2 + 2 * i) break;
    }
    if (want_next < 0) want_next = argmax(tl.data() + static_cast<size_t>(cur) * V, V);
    // the device: the INTEGRATION.md accept call on the same (already forwarded) batch
    mk_proposal q{};
    q.seq = 0;
    q.kk = kk;
    q.root = 0;
    q.cache_len = P;
    q.sampling = {0.0f, 1.0f, 1, 0.0f, 0.0f, 0.0f};
    q.chain = chain.data();
    q.alt = alt.data();
    mk_accept_result res{};
    CudaModel::check(mk_accept(gpu.ctx, &q, 1, &res));
    if (res.n_accepted != static_cast<int>(want.size()) || res.next != want_next)
      throw std::runtime_error("accept differs: " + std::to_string(res.n_accepted) + " vs " +
                               std::to_string(want.size()));
    for (size_t i = 0; i < want.size(); ++i)
      if (res.accepted[i] != want[i]) throw std::runtime_error("accepted id differs");
    // the compacted KV: both sides continue with the bonus token at row P + 1 + n_accepted
    const int row = P + 1 + res.n_accepted;
    BatchToken nb{res.next, 0, row, true};
    cpu.forward(&nb, 1, cl.data());
    gpu.forward(&nb, 1, gl.data());
    if (std::memcmp(gl.data(), cl.data(), gl.size() * 4) != 0) throw std::runtime_error("post-accept logits differ");
    std::printf("ok: %d accepted, next %d\n", res.n_accepted, res.next);
    return 0;
  } catch (const std::exception& e) {
    std::fprintf(stderr, "FAIL: %s\n", e.what());
    return 1;
  }
}
