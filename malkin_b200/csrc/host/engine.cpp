// Continuous-batching speculative decoder (engine.hpp). Every decision follows malkin's Engine (engine.cpp:191-559):
// admission, draft lengths, batch layout, acceptance, emission and the adaptive draft length; the numbers that feed
// the decisions (logits, top-k candidates, acceptance walks) come from the device models.
#include "engine.hpp"

#include <algorithm>
#include <cmath>
#include <string>

namespace mkb {

namespace {

using Dist = std::vector<std::pair<float, int32_t>>;

// Sampler::distribution (sampler.cpp:22-62) at temperature > 0 over the row's top-k candidates (value desc): the same
// float exponentials and double sums, min-p then nucleus.
void distribution_of(const float* v, const int32_t* id, int k, const mk_sampling& sp, Dist* out) {
  out->clear();
  std::vector<float> e(static_cast<size_t>(k));
  const float mx = v[0];
  double sum = 0;
  for (int j = 0; j < k; ++j) {
    e[static_cast<size_t>(j)] = std::exp((v[j] - mx) / sp.temperature);
    sum += e[static_cast<size_t>(j)];
  }
  const double floor = static_cast<double>(sp.min_p) * e[0];
  double kept = 0;
  int n = 0;
  for (; n < k; ++n) {
    if (n > 0 && e[static_cast<size_t>(n)] < floor) break;
    kept += e[static_cast<size_t>(n)];
    if (kept >= sp.top_p * sum) {
      ++n;
      break;
    }
  }
  n = std::max(n, 1);
  double total = 0;
  for (int j = 0; j < n; ++j) total += e[static_cast<size_t>(j)];
  for (int j = 0; j < n; ++j) out->emplace_back(static_cast<float>(e[static_cast<size_t>(j)] / total), id[j]);
}

// Sampler::draw (sampler.cpp:64-72).
int32_t draw_from(const Dist& d, std::mt19937_64& rng) {
  if (d.size() == 1) return d[0].second;
  double r = std::uniform_real_distribution<double>(0.0, 1.0)(rng);
  for (const auto& [p, id] : d) {
    r -= p;
    if (r <= 0) return id;
  }
  return d.back().second;
}

}  // namespace

Engine::Engine(Model* target, Model* draft, int n_draft) : target_(target), draft_(draft) {
  if (!target_ || target_->n_ctx() == 0) throw StateError("engine: the target model needs weights and a KV cache");
  if (draft_) {
    if (draft_->n_ctx() == 0) throw StateError("engine: the draft model needs a KV cache");
    if (draft_->n_seq() != target_->n_seq() || draft_->n_ctx() != target_->n_ctx())
      throw ArgError("engine: draft and target need the same n_ctx and n_seq");
    if (draft_->cfg().n_vocab != target_->cfg().n_vocab)
      throw ArgError("engine: draft model vocabulary differs from the target");
  }
  if (n_draft > 0) n_draft_ = std::min({n_draft, target_->max_batch() - 1, MK_MAX_DRAFT});
  slots_.resize(static_cast<size_t>(target_->n_seq()));
}

int Engine::submit(const mk_gen_request& rq) {
  const int n_ctx = target_->n_ctx();
  if (!rq.prompt || rq.n_prompt <= 0) throw ArgError("empty prompt");
  if (rq.n_prompt >= n_ctx)
    throw ArgError("prompt has " + std::to_string(rq.n_prompt) + " tokens, context is " + std::to_string(n_ctx));
  const int V = target_->cfg().n_vocab;
  for (int i = 0; i < rq.n_prompt; ++i)
    if (rq.prompt[i] < 0 || rq.prompt[i] >= V) throw ArgError("prompt token out of range");
  if (rq.sampling.presence_penalty != 0.0f || rq.sampling.frequency_penalty != 0.0f)
    throw UnsupportedError("unsupported: presence / frequency penalties on the device path");
  const bool greedy = rq.sampling.temperature <= 0.0f;
  if (!greedy && (rq.sampling.top_k < 1 || rq.sampling.top_k > MK_MAX_TOPK))
    throw UnsupportedError("unsupported: top_k outside 1.." + std::to_string(MK_MAX_TOPK) + " on the device path");
  auto r = std::make_unique<Request>();
  r->id = next_id_++;
  r->prompt.assign(rq.prompt, rq.prompt + rq.n_prompt);
  if (rq.eog && rq.n_eog > 0) r->eog.assign(rq.eog, rq.eog + rq.n_eog);
  r->budget = rq.max_tokens > 0 ? rq.max_tokens : n_ctx;
  r->sp = rq.sampling;
  r->greedy = greedy;
  // Sampler(p) seeds its engine with p.seed (0: random); the draft Sampler with seed + 1 (engine.cpp:42-45)
  r->rng.seed(rq.seed ? rq.seed : std::random_device{}());
  r->drng.seed(rq.seed ? rq.seed + 1 : std::random_device{}());
  r->st.prompt_tokens = rq.n_prompt;
  pending_.push_back(std::move(r));
  done_.resize(static_cast<size_t>(next_id_));
  return next_id_ - 1;
}

void Engine::cancel(int id) {
  for (Slot& s : slots_)
    if (s.req && s.req->id == id) s.req->cancelled = true;  // ends at its next emitted token, as on_text does
  for (auto& r : pending_)
    if (r && r->id == id) r->cancelled = true;
}

mk_gen_stats Engine::stats(int id) const {
  for (const Slot& s : slots_)
    if (s.req && s.req->id == id) return s.req->st;
  for (const auto& r : pending_)
    if (r && r->id == id) return r->st;
  if (id < 0 || id >= static_cast<int>(done_.size())) throw ArgError("engine: unknown request");
  return done_[static_cast<size_t>(id)];
}

// Engine::admit (engine.cpp:244-268): the idle slot with the longest common prefix, least recently used on ties.
void Engine::admit(std::unique_ptr<Request> r) {
  const auto& prompt = r->prompt;
  int best = -1;
  size_t best_common = 0;
  for (int i = 0; i < static_cast<int>(slots_.size()); ++i) {
    const Slot& s = slots_[static_cast<size_t>(i)];
    if (s.req) continue;
    size_t c = 0;
    while (c < s.cache.size() && c < prompt.size() && s.cache[c] == prompt[c]) ++c;
    if (best < 0 || c > best_common || (c == best_common && s.used < slots_[static_cast<size_t>(best)].used)) {
      best = i;
      best_common = c;
    }
  }
  Slot& s = slots_[static_cast<size_t>(best)];
  best_common = std::min(best_common, prompt.size() - 1);  // the last prompt token is evaluated for its logits
  s.cache.resize(best_common);
  r->st.cached_tokens = static_cast<int32_t>(best_common);
  r->st.finish = MK_FINISH_LENGTH;
  s.used = ++admitted_;
  r->k = std::min(4, n_draft_);
  s.req = std::move(r);
  ++busy_;
}

// Engine::plan_drafts (engine.cpp:336-358).
bool Engine::plan_drafts() {
  const int n_ctx = target_->n_ctx();
  props_.clear();
  for (size_t i = 0; i < slots_.size(); ++i) {
    if (!slots_[i].req || !slots_[i].req->decoding) continue;
    props_.emplace_back();
    props_.back().seq = static_cast<int>(i);
  }
  const int nd = static_cast<int>(props_.size());
  bool drafting = false;
  for (Proposal& p : props_) {
    const Slot& s = slots_[static_cast<size_t>(p.seq)];
    const Request& q = *s.req;
    p.greedy = q.greedy;
    if (!draft_) continue;
    const int left = q.budget - q.st.completion_tokens, free = n_ctx - static_cast<int>(s.cache.size()) - 2;
    const int cap = target_->max_batch() / nd - 1;
    p.kk = std::max(0, std::min({q.k, left, p.greedy ? free / 2 : free, p.greedy ? cap / 2 : cap}));
    drafting = drafting || p.kk > 0;
  }
  return drafting;
}

void Engine::draft_flush(std::vector<mk_batch_token>& b, int k) {
  if (b.empty()) return;
  draft_->forward(b.data(), static_cast<int>(b.size()), nullptr);
  std::vector<float> v;
  std::vector<int32_t> ids;
  draft_->candidates(k, &v, &ids);
  size_t row = 0;
  for (const mk_batch_token& t : b) {
    if (!t.logits) continue;
    Slot& s = slots_[static_cast<size_t>(t.seq)];
    s.dv.assign(v.begin() + static_cast<ptrdiff_t>(row * k), v.begin() + static_cast<ptrdiff_t>((row + 1) * k));
    s.di.assign(ids.begin() + static_cast<ptrdiff_t>(row * k), ids.begin() + static_cast<ptrdiff_t>((row + 1) * k));
    ++row;
  }
  b.clear();
}

// Engine::propose (engine.cpp:270-334): catch the draft KV up to cache + next (common prefix reuse), then rounds in
// which every proposing slot picks its next draft token and all of them are fed in one pass.
void Engine::propose() {
  const int dmax = draft_->max_batch();
  int K = 1;
  for (const Proposal& p : props_)
    if (p.kk > 0) K = std::max(K, p.greedy ? 2 : slots_[static_cast<size_t>(p.seq)].req->sp.top_k);
  std::vector<mk_batch_token> b;
  for (const Proposal& p : props_) {
    if (p.kk == 0) continue;
    Slot& s = slots_[static_cast<size_t>(p.seq)];
    const size_t len = s.cache.size() + 1;
    size_t common = 0;
    while (common < s.dcache.size() && common < s.cache.size() && s.dcache[common] == s.cache[common]) ++common;
    if (common == s.cache.size() && common < s.dcache.size() && s.dcache[common] == s.req->next) ++common;
    common = std::min(common, len - 1);  // the last token is evaluated for its logits
    s.dcache.resize(common);
    for (size_t pos = common; pos < len; ++pos) {
      const int32_t id = pos < s.cache.size() ? s.cache[pos] : s.req->next;
      b.push_back({id, p.seq, static_cast<int32_t>(pos), pos + 1 == len, -1, -1});
      s.dcache.push_back(id);
      if (static_cast<int>(b.size()) == dmax) draft_flush(b, K);
    }
  }
  draft_flush(b, K);
  for (int i = 0;; ++i) {
    bool more = false;
    for (Proposal& p : props_) {
      if (i >= p.kk) continue;
      Slot& s = slots_[static_cast<size_t>(p.seq)];
      int32_t a = 0;
      if (p.greedy) {  // top-1 chain, top-2 alternative
        a = s.di[0];
        p.alt.push_back(s.di[1]);
      } else {
        p.qd.emplace_back();
        const int k = s.req->sp.top_k;
        distribution_of(s.dv.data(), s.di.data(), k, s.req->sp, &p.qd.back());
        a = draw_from(p.qd.back(), s.req->drng);
      }
      p.chain.push_back(a);
      if (i + 1 < p.kk) {
        b.push_back({a, p.seq, static_cast<int32_t>(s.dcache.size()), true, -1, -1});
        s.dcache.push_back(a);
        more = true;
      }
    }
    draft_flush(b, K);
    if (!more) break;
  }
}

// Engine::build_batch (engine.cpp:360-395): greedy [next, chain0, alt0, chain1, alt1, ...] at KV rows P, P + 1, ...
// (chain i and alt i at RoPE position P + 1 + i under chain i - 1); sampled [next, d0, d1, ...]; then prompt chunks
// in slot order up to the batch limit.
int Engine::build_batch() {
  batch_.clear();
  batch_seq_.clear();
  batch_root_.clear();
  for (Proposal& p : props_) {
    const Slot& s = slots_[static_cast<size_t>(p.seq)];
    const int P = static_cast<int>(s.cache.size());
    p.root = static_cast<int>(batch_.size());
    batch_.push_back({s.req->next, p.seq, P, true, -1, -1});
    for (int i = 0; i < p.kk; ++i) {
      if (p.greedy) {
        const int par = i == 0 ? p.root : p.root + 2 * i - 1;
        batch_.push_back({p.chain[static_cast<size_t>(i)], p.seq, P + 1 + i, true, P + 1 + 2 * i, par});
        batch_.push_back({p.alt[static_cast<size_t>(i)], p.seq, P + 1 + i, true, P + 2 + 2 * i, par});
      } else {
        batch_.push_back({p.chain[static_cast<size_t>(i)], p.seq, P + 1 + i, true, -1, -1});
      }
    }
  }
  const int decode_rows = static_cast<int>(batch_.size());
  const int maxb = target_->max_batch();
  for (size_t i = 0; i < slots_.size(); ++i) {
    const Slot& s = slots_[i];
    if (!s.req || s.req->decoding) continue;
    const auto& prompt = s.req->prompt;
    const int from = static_cast<int>(s.cache.size());
    const int take = std::min(maxb - static_cast<int>(batch_.size()), static_cast<int>(prompt.size()) - from);
    for (int pos = from; pos < from + take; ++pos) {
      const bool last = pos + 1 == static_cast<int>(prompt.size());
      batch_.push_back({prompt[static_cast<size_t>(pos)], static_cast<int32_t>(i), pos, last, -1, -1});
      if (last) {
        batch_seq_.push_back(static_cast<int>(i));
        batch_root_.push_back(static_cast<int>(batch_.size()) - 1);
      }
    }
  }
  return decode_rows;
}

// Request::emit (engine.cpp:59-97) at token level: end-of-generation id, cancellation, budget, context end.
bool Engine::emit(Request& q, int32_t id, size_t cached, std::vector<mk_gen_event>* ev) {
  if (std::find(q.eog.begin(), q.eog.end(), id) != q.eog.end()) {
    q.st.finish = MK_FINISH_STOP;
    return false;
  }
  ++q.st.completion_tokens;
  ev->push_back({q.id, id, 0});
  if (q.cancelled) return false;
  if (q.st.completion_tokens >= q.budget) return false;
  return static_cast<int>(cached) + 1 < target_->n_ctx();
}

void Engine::finish(Slot& s, std::vector<mk_gen_event>* ev) {
  Request& q = *s.req;
  if (q.cancelled) q.st.finish = MK_FINISH_CANCELLED;
  done_[static_cast<size_t>(q.id)] = q.st;
  ev->push_back({q.id, -1, q.st.finish});
  s.req.reset();
  --busy_;
}

void Engine::ensure_uniforms(Request& q, size_t n) {
  while (q.ubuf.size() < n) q.ubuf.push_back(std::uniform_real_distribution<double>(0.0, 1.0)(q.rng));
}

// Engine::worker_loop's admission (engine.cpp:201-203) then Engine::step (engine.cpp:397-421) and Engine::accept /
// accept_greedy / accept_sampled (engine.cpp:423-507), the walks done on the device by Model::accept.
void Engine::step(std::vector<mk_gen_event>* ev) {
  for (auto it = pending_.begin(); it != pending_.end();) {  // requests cancelled before admission end now
    if ((*it)->cancelled) {
      Request& q = **it;
      q.st.finish = MK_FINISH_CANCELLED;
      done_[static_cast<size_t>(q.id)] = q.st;
      ev->push_back({q.id, -1, MK_FINISH_CANCELLED});
      it = pending_.erase(it);
    } else {
      ++it;
    }
  }
  const size_t take = std::min(pending_.size(), slots_.size() - static_cast<size_t>(busy_));
  for (size_t i = 0; i < take; ++i) admit(std::move(pending_[i]));
  pending_.erase(pending_.begin(), pending_.begin() + static_cast<ptrdiff_t>(take));
  if (busy_ == 0) return;
  if (plan_drafts()) propose();
  const int decode_rows = build_batch(), n = static_cast<int>(batch_.size());
  if (n == 0) return;
  const int n_ctx = target_->n_ctx();
  target_->forward(batch_.data(), n, nullptr);
  for (int t = decode_rows; t < n; ++t) slots_[static_cast<size_t>(batch_[static_cast<size_t>(t)].seq)].cache.push_back(batch_[static_cast<size_t>(t)].id);

  // one device acceptance for every slot: first tokens of finished prompts (kk = 0), then the decoding slots
  std::vector<mk_proposal> mp;
  std::vector<std::vector<float>> qp(props_.size());
  std::vector<std::vector<int32_t>> qi(props_.size()), qn(props_.size());
  std::vector<std::vector<double>> un(batch_seq_.size() + props_.size());
  auto uniforms_for = [&](Request& q, size_t need, std::vector<double>& u) {
    if (q.greedy) return;
    ensure_uniforms(q, need);
    u.assign(q.ubuf.begin(), q.ubuf.begin() + static_cast<ptrdiff_t>(need));
  };
  for (size_t j = 0; j < batch_seq_.size(); ++j) {
    Slot& s = slots_[static_cast<size_t>(batch_seq_[j])];
    mk_proposal p{};
    p.seq = batch_seq_[j];
    p.root = batch_root_[j];
    p.cache_len = static_cast<int32_t>(s.cache.size()) - 1;
    p.sampling = s.req->sp;
    uniforms_for(*s.req, 1, un[j]);
    p.uniforms = un[j].empty() ? nullptr : un[j].data();
    p.n_uniforms = static_cast<int32_t>(un[j].size());
    mp.push_back(p);
  }
  for (size_t i = 0; i < props_.size(); ++i) {
    const Proposal& pr = props_[i];
    Slot& s = slots_[static_cast<size_t>(pr.seq)];
    mk_proposal p{};
    p.seq = pr.seq;
    p.kk = pr.kk;
    p.root = pr.root;
    p.cache_len = static_cast<int32_t>(s.cache.size());
    p.sampling = s.req->sp;
    p.chain = pr.chain.data();
    p.alt = pr.greedy ? pr.alt.data() : nullptr;
    if (!pr.greedy) {
      for (const Dist& d : pr.qd) {
        qn[i].push_back(static_cast<int32_t>(d.size()));
        for (const auto& [pp, id] : d) qp[i].push_back(pp), qi[i].push_back(id);
      }
      p.q_p = qp[i].data();
      p.q_id = qi[i].data();
      p.q_n = qn[i].data();
    }
    std::vector<double>& u = un[batch_seq_.size() + i];
    uniforms_for(*s.req, static_cast<size_t>(pr.kk) + 1, u);
    p.uniforms = u.empty() ? nullptr : u.data();
    p.n_uniforms = static_cast<int32_t>(u.size());
    mp.push_back(p);
  }
  std::vector<mk_accept_result> res(mp.size());
  if (!mp.empty()) target_->accept(mp.data(), static_cast<int>(mp.size()), res.data());
  auto consume = [](Request& q, int used) {
    for (int u = 0; u < used && !q.ubuf.empty(); ++u) q.ubuf.pop_front();
  };

  // prompts that finished: first token (Sampler::sample on the prompt's last row)
  for (size_t j = 0; j < batch_seq_.size(); ++j) {
    Slot& s = slots_[static_cast<size_t>(batch_seq_[j])];
    Request& q = *s.req;
    consume(q, res[j].uniforms_used);
    q.decoding = true;
    q.next = res[j].next;
    if (!emit(q, q.next, s.cache.size(), ev)) finish(s, ev);
  }
  // decoding slots: the accepted path, then the next token
  for (size_t i = 0; i < props_.size(); ++i) {
    const Proposal& pr = props_[i];
    const mk_accept_result& r = res[batch_seq_.size() + i];
    Slot& s = slots_[static_cast<size_t>(pr.seq)];
    Request& q = *s.req;
    consume(q, r.uniforms_used);
    s.cache.push_back(q.next);
    q.st.drafted += pr.kk;
    bool go = true;
    int done = 0;
    for (int a = 0; a < r.n_accepted; ++a) {
      s.cache.push_back(r.accepted[a]);
      ++q.st.accepted;
      go = emit(q, r.accepted[a], s.cache.size(), ev);
      if (!go) break;
      done = a + 1;
    }
    if (go) q.next = r.next;
    if (pr.kk > 0) {  // adapt the draft length: grow after a fully accepted chain, shrink when most drafts fail
      const bool full = pr.greedy ? done == pr.kk && r.last_node == 2 * pr.kk - 1 : done == pr.kk;
      if (full && pr.kk == q.k)
        q.k = std::min(q.k + 1, n_draft_);
      else if (2 * done < pr.kk)
        q.k = std::max(1, q.k - 1);
    }
    if (go) go = emit(q, q.next, s.cache.size(), ev);
    if (!go) finish(s, ev);
  }
  (void)n_ctx;
}

double Engine::perplexity(const int32_t* toks, int n, int window, int32_t bos, int* scored) {
  if (busy()) throw StateError("perplexity: requests in flight");
  if (!toks || n <= 0 || window <= 1) throw ArgError("perplexity: bad arguments");
  window = std::min(window, target_->n_ctx());
  const int n_chunks = n / window;
  if (n_chunks == 0) throw ArgError("text shorter than one window");
  const int maxb = target_->max_batch();
  const int first = window / 2;
  double nll = 0;
  int count = 0;
  std::vector<mk_batch_token> b;
  std::vector<int32_t> tg;
  std::vector<double> rn;
  for (int c = 0; c < n_chunks; ++c) {
    std::vector<int32_t> chunk(toks + static_cast<ptrdiff_t>(c) * window, toks + static_cast<ptrdiff_t>(c + 1) * window);
    if (bos >= 0) chunk[0] = bos;
    for (int i = 0; i < window; i += maxb) {
      const int nb = std::min(maxb, window - i);
      b.clear();
      tg.assign(static_cast<size_t>(nb), -1);
      for (int t = 0; t < nb; ++t) {
        const int j = i + t;
        b.push_back({chunk[static_cast<size_t>(j)], 0, j, true, -1, -1});
        if (j >= first && j + 1 < window) tg[static_cast<size_t>(t)] = chunk[static_cast<size_t>(j) + 1];
      }
      target_->forward(b.data(), nb, nullptr);
      rn.assign(static_cast<size_t>(nb), 0.0);
      target_->row_nll(tg.data(), rn.data());
      for (int t = 0; t < nb; ++t)
        if (tg[static_cast<size_t>(t)] >= 0) {
          nll += rn[static_cast<size_t>(t)];
          ++count;
        }
    }
  }
  slots_[0].cache.clear();  // perplexity used sequence 0
  if (scored) *scored = count;
  return nll / count;
}

}  // namespace mkb
