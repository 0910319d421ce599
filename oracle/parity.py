"""TEST INFRASTRUCTURE ONLY (checker): parity of the device verify step against malkin's own CPU path (oracle/_ref).

Used by tests/test_gpu_parity.py and by bench.py's reference leg, after its timed region; the product never imports
it. One parity case on a loaded model (device side: a malkin_b200 Model, any tensor-parallel size; reference side:
malkin's Model + Sampler compiled from its sources, see ref_harness.cpp):

  1. R requests, seeded uniform prompts of `prefix` tokens, prefilled (chunks of at most 256 rows on the reference
     side, malkin's kMaxBatch, model.h:35); logits of each prompt's last token.
  2. Greedy tree verify: root = the device's greedy next token, a chain of kk drafts by the 0.55 greedy-match rule
     (at each depth, with seeded probability 0.55, the target's greedy token at the chain node above, else a uniform
     token) and one uniform sibling per depth, laid out as Engine::build_batch does (engine.cpp:362-379); greedy
     accept with KV compaction (Engine::accept_greedy, engine.cpp:441-479).
  3. Sampled chain verify at temperature 0.8 (chain only, kk + 1 rows, engine.cpp:366-378): the draft distribution
     of depth i is Dirichlet(1) over the target's top-8 tokens at chain node i and the drafted token is drawn from it;
     accept with a seeded mt19937_64 uniform stream per request (Engine::accept_sampled + Sampler, engine.cpp:482-507,
     sampler.cpp:22-97).

Drafts, q and uniforms are inputs shared by both sides. Checks: max-abs logits after the final norm (prefill rows,
tree rows, chain rows) <= 2e-2; greedy accepted ids / next / cache length identical for every request whose
reference tree logits have a top-1 margin above 1e-2 at every node; sampled decisions identical given the same
logits and uniforms (malkin's accept run on the device's logits), and counted on malkin's own logits.
"""
from __future__ import annotations

from typing import Dict, List

import numpy as np

TOL_LOGITS = 2e-2
MARGIN = 1e-2
SAMPLING = dict(temperature=0.8, top_p=0.95, top_k=40, min_p=0.05)


def tree_rows(reqs, kk):
    """Engine::build_batch greedy layout (engine.cpp:362-379): per request [next, c0, a0, c1, a1, ...]."""
    rows, roots = [], []
    for seq, P, nxt, chain, alt in reqs:
        root = len(rows)
        roots.append(root)
        rows.append((int(nxt), seq, P, 1, -1, -1))
        for i in range(kk):
            par = root if i == 0 else root + 2 * i - 1
            rows.append((int(chain[i]), seq, P + 1 + i, 1, P + 1 + 2 * i, par))
            rows.append((int(alt[i]), seq, P + 1 + i, 1, P + 2 + 2 * i, par))
    return rows, roots


def chain_rows(reqs, kk):
    """Sampled layout (engine.cpp:366-378): per request [next, d0, ..., d_{kk-1}] as plain rows."""
    rows, roots = [], []
    for seq, P, nxt, chain in reqs:
        roots.append(len(rows))
        rows.append((int(nxt), seq, P, 1, -1, -1))
        rows += [(int(chain[i]), seq, P + 1 + i, 1, -1, -1) for i in range(kk)]
    return rows, roots


def _forward_chunks(fwd, rows, max_rows):
    """Forward a batch in chunks of at most max_rows rows. Plain (prompt) rows split anywhere; a batch with tree rows
    splits on whole requests, so every parent stays in its child's chunk (rows are grouped by request)."""
    tree = any(r[5] >= 0 for r in rows)
    out, i = [], 0
    while i < len(rows):
        j = min(len(rows), i + max_rows)
        if tree and j < len(rows):  # back off to the first row of a request
            while j > i + 1 and rows[j][1] == rows[j - 1][1]:
                j -= 1
        chunk = [(a, b, c, d, e, (f - i if f >= 0 else f)) for (a, b, c, d, e, f) in rows[i:j]]
        lg = fwd(chunk)
        if lg is not None:
            out.append(lg)
        i = j
    return np.concatenate(out) if out else np.zeros((0, 0), np.float32)


def device_leg(mk, m, requests: int, prefix: int, kk: int, seed: int = 1, max_batch: int = 256,
               sampled: bool = True) -> Dict:
    """Runs the case on the device model `m` (every tensor-parallel rank calls it with the same arguments)."""
    V = m.config().n_vocab
    R, P = requests, prefix
    rng = np.random.default_rng(seed)
    prompts = rng.integers(0, V, (R, P))
    pre = [(int(prompts[s, i]), s, i, int(i == P - 1), -1, -1) for s in range(R) for i in range(P)]
    fwd = lambda rows: m.forward([mk.BatchToken(*r) for r in rows])  # noqa: E731
    pre_logits = _forward_chunks(fwd, pre, max_batch)
    nexts = [int(np.argmax(pre_logits[s])) for s in range(R)]
    # greedy tree: 0.55 greedy-match chain, built depth by depth from the device's argmax
    flips = rng.random((R, kk)) < 0.55
    chains = rng.integers(0, V, (R, kk))
    alts = rng.integers(0, V, (R, kk))
    for d in range(kk):
        rows, roots = tree_rows([(s, P, nexts[s], chains[s], alts[s]) for s in range(R)], kk)
        lg = fwd(rows)
        for s in range(R):
            if flips[s, d]:
                chains[s, d] = int(np.argmax(lg[roots[s] + (0 if d == 0 else 2 * d - 1)]))
    rows, roots = tree_rows([(s, P, nexts[s], chains[s], alts[s]) for s in range(R)], kk)
    tree_logits = fwd(rows)
    res = m.accept([mk.Proposal(seq=s, root=roots[s], cache_len=P, chain=chains[s], alt=alts[s]) for s in range(R)])
    greedy = [(list(r.ids), int(r.next), int(r.cache_len)) for r in res]
    out = dict(R=R, P=P, kk=kk, V=V, prompts=prompts, pre_rows=pre, pre_logits=pre_logits, nexts=nexts,
               chains=chains.copy(), alts=alts, tree_rows=rows, tree_roots=roots, tree_logits=tree_logits,
               greedy=greedy)
    if not sampled:
        return out
    # sampled chain: depth by depth, q = Dirichlet(1) over the top-8 at chain node i, the draft drawn from q
    dchain = np.zeros((R, kk), dtype=np.int64)
    qs: List[List[List[tuple]]] = [[] for _ in range(R)]
    for d in range(kk):
        crow, croots = chain_rows([(s, P, nexts[s], dchain[s]) for s in range(R)], kk)
        lg = fwd(crow)
        for s in range(R):
            top = np.argsort(-lg[croots[s] + d], kind="stable")[:8]
            w = rng.dirichlet(np.ones(8)).astype(np.float32)
            qs[s].append([(float(p), int(t)) for p, t in zip(w, top)])
            cdf = np.cumsum(w.astype(np.float64))
            dchain[s, d] = int(top[min(7, int(np.searchsorted(cdf, rng.random() * cdf[-1], side="right")))])
    crow, croots = chain_rows([(s, P, nexts[s], dchain[s]) for s in range(R)], kk)
    chain_logits = fwd(crow)
    useeds = [1000 + 7 * s + seed for s in range(R)]
    samp = mk.Sampling(**SAMPLING)
    res = m.accept([mk.Proposal(seq=s, root=croots[s], cache_len=P, chain=dchain[s], sampling=samp, q=qs[s],
                                uniforms=mk.rng_uniforms(useeds[s], 2 * kk + 4)) for s in range(R)])
    out.update(dchain=dchain, q=qs, chain_rows=crow, chain_roots=croots, chain_logits=chain_logits, useeds=useeds,
               sampled=[(list(r.ids), int(r.next), int(r.uniforms_used)) for r in res])
    return out


def reference_leg(ref, rm, d: Dict) -> Dict:
    """Runs the same inputs through malkin's CPU path: `ref` an oracle.Ref, `rm` an oracle.RefModel with at least R
    sequences of prefix + 2 kk + 2 positions."""
    R, P, kk = d["R"], d["P"], d["kk"]
    fwd = rm.forward
    pre_logits = _forward_chunks(fwd, d["pre_rows"], 256)
    tree_logits = _forward_chunks(fwd, d["tree_rows"], 256)
    greedy = []
    per = 2 * kk + 1
    for s in range(R):
        smp = ref.sampler(temperature=0.0, seed=1)
        rt = d["tree_roots"][s]
        ids, nxt, cl = ref.accept_greedy(smp, tree_logits[rt:rt + per], d["chains"][s], d["alts"][s], model=rm, seq=s,
                                         cache_len=P, n_draft=kk)
        ref.free_sampler(smp)
        greedy.append(([int(x) for x in ids], int(nxt), int(cl)))
    out = dict(pre_logits=pre_logits, tree_logits=tree_logits, greedy=greedy)
    if "chain_rows" not in d:
        return out
    chain_logits = _forward_chunks(fwd, d["chain_rows"], 256)
    on_ref, on_dev = [], []
    for s in range(R):
        rt = d["chain_roots"][s]
        for logits, dst in ((chain_logits, on_ref), (d["chain_logits"], on_dev)):
            smp = ref.sampler(seed=d["useeds"][s], **SAMPLING)
            ids, nxt = ref.accept_sampled(smp, logits[rt:rt + kk + 1], d["dchain"][s], d["q"][s], n_draft=kk)
            ref.free_sampler(smp)
            dst.append(([int(x) for x in ids], int(nxt)))
    out.update(chain_logits=chain_logits, sampled_ref_logits=on_ref, sampled_dev_logits=on_dev)
    return out


def compare(d: Dict, r: Dict) -> Dict:
    """The parity block: max-abs logits, greedy identity where the margin allows, sampled decision identity."""
    mx = max(float(np.abs(d[k] - r[k]).max()) for k in ("pre_logits", "tree_logits", "chain_logits") if k in r)
    kk, per = d["kk"], 2 * d["kk"] + 1
    g_cmp = g_same = 0
    for s, (dev, ref) in enumerate(zip(d["greedy"], r["greedy"])):
        rt = d["tree_roots"][s]
        srt = np.sort(r["tree_logits"][rt:rt + per], axis=-1)
        same = np.array_equal(d["tree_logits"][rt:rt + per], r["tree_logits"][rt:rt + per])
        if same or np.all(srt[:, -1] - srt[:, -2] > MARGIN):  # identical logits: every walk must match
            g_cmp += 1
            g_same += int(dev == ref)
    out = {"max_abs_logits": mx, "tol": TOL_LOGITS, "greedy_compared": g_cmp, "greedy_identical": g_same,
           "greedy_ok": g_same == g_cmp, "accepted_greedy": sum(len(x[0]) for x in d["greedy"])}
    if "sampled" in d:
        dev = [(ids, nxt) for ids, nxt, _ in d["sampled"]]
        out["sampled_identical_same_logits"] = sum(int(a == b) for a, b in zip(dev, r["sampled_dev_logits"]))
        out["sampled_identical_ref_logits"] = sum(int(a == b) for a, b in zip(dev, r["sampled_ref_logits"]))
        out["sampled_requests"] = len(dev)
        out["sampled_ok"] = out["sampled_identical_same_logits"] == len(dev)
        out["accepted_sampled"] = sum(len(x[0]) for x in d["sampled"])
    out["ok"] = bool(mx <= TOL_LOGITS and out["greedy_ok"] and out.get("sampled_ok", True))
    return out
