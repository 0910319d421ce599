// Continuous-batching speculative decoder over device models: the B200 counterpart of malkin::Engine
// (engine.h:47-141, engine.cpp:191-559) without its text layer. One target Model and an optional draft Model (same
// vocabulary) on the same GPU; one KV sequence per slot. A step is Engine::step: admit waiting requests into idle
// slots (longest common prefix reuse), plan the draft length per decoding slot (adaptive k), run the draft proposal
// (greedy: top-1 chain + top-2 siblings; sampled: a chain drawn from the draft distribution), lay out one target
// batch (trees / chains, then prompt chunks), forward it, then accept on the device and emit on the host.
// Tokens leave as ids: detokenization, stop strings and chat formatting stay with the host, which ends a request
// with cancel() (malkin's on_text returning false).
#pragma once
#include <cstdint>
#include <deque>
#include <memory>
#include <random>
#include <vector>

#include "../../../include/malkin_b200.h"
#include "model.hpp"

namespace mkb {

class Engine {
 public:
  // target: the verified model; draft: nullptr for plain decoding. n_draft: largest draft length (malkin's
  // --draft-max, default 8; at most MK_MAX_DRAFT). Both models need alloc_kv with the same n_seq (the slots).
  Engine(Model* target, Model* draft, int n_draft);

  int submit(const mk_gen_request& r);                // Engine::generate's queueing (engine.cpp:227-242)
  void step(std::vector<mk_gen_event>* events);       // Engine::worker_loop's admit + step (engine.cpp:191-225)
  bool busy() const { return busy_ > 0 || !pending_.empty(); }
  void cancel(int id);
  mk_gen_stats stats(int id) const;
  // Engine::perplexity (engine.cpp:525-559) over token ids: windows of `window` tokens (at most n_ctx), the second
  // half of each scored; bos >= 0 replaces each window's first token. Uses slot 0; no request may be in flight.
  double perplexity(const int32_t* toks, int n, int window, int32_t bos, int* scored);

 private:
  struct Request {
    int id = 0;
    std::vector<int32_t> prompt, eog;
    int budget = 0;
    mk_sampling sp{};
    bool greedy = true;
    std::mt19937_64 rng, drng;  // the target and draft Samplers' engines (seed, seed + 1; 0: random)
    std::deque<double> ubuf;    // target uniforms drawn from rng and not yet consumed
    bool decoding = false, cancelled = false;
    int k = 4;  // adaptive draft length
    int32_t next = 0;
    mk_gen_stats st{};
  };
  struct Slot {
    std::vector<int32_t> cache;   // tokens whose target KV is valid
    std::unique_ptr<Request> req;  // null: idle
    uint64_t used = 0;
    std::vector<int32_t> dcache;  // tokens whose draft KV is valid
    std::vector<float> dv;        // draft candidates of the slot's last draft logits row
    std::vector<int32_t> di;
  };
  struct Proposal {
    int seq = 0, kk = 0, root = 0;
    bool greedy = true;
    std::vector<int32_t> chain, alt;
    std::vector<std::vector<std::pair<float, int32_t>>> qd;  // sampled: draft distribution of each chain token
  };

  void admit(std::unique_ptr<Request> r);
  bool plan_drafts();
  void propose();
  int build_batch();
  bool emit(Request& q, int32_t id, size_t cached, std::vector<mk_gen_event>* ev);
  void finish(Slot& s, std::vector<mk_gen_event>* ev);
  void draft_flush(std::vector<mk_batch_token>& batch, int k);
  void ensure_uniforms(Request& q, size_t n);

  Model* target_;
  Model* draft_;
  int n_draft_ = 8;
  std::vector<Slot> slots_;
  std::vector<std::unique_ptr<Request>> pending_;
  std::vector<mk_gen_stats> done_;  // finished requests' stats by id
  int busy_ = 0, next_id_ = 0;
  uint64_t admitted_ = 0;
  std::vector<mk_batch_token> batch_;
  std::vector<int> batch_seq_, batch_root_;  // prompt-finishing slots and their batch indices
  std::vector<Proposal> props_;
};

}  // namespace mkb
