"""The parity harness (oracle/parity.py) on the CPU: malkin's own CPU path (oracle/_ref) stands in for the device
model, so both legs compute the same thing and the comparison must report exact agreement. Checks the harness's
batching (prompt chunks, request-aligned tree chunks), tree / chain layouts, accept plumbing and comparison logic
that the GPU parity tests and the benchmark's reference leg rely on."""
from types import SimpleNamespace

import numpy as np


class RefAsDevice:
    """The device-model interface device_leg uses (config / forward / accept), served by malkin's CPU path; sampled
    accepts go through the oracle's restatement with the proposal's uniforms."""

    def __init__(self, ref, rm, oracle):
        self.ref, self.rm, self.oracle = ref, rm, oracle
        self.last = None

    def config(self):
        return SimpleNamespace(n_vocab=self.rm.n_vocab)

    def forward(self, batch):
        rows = [(t.id, t.seq, t.pos, int(t.logits), t.kv, t.parent) for t in batch]
        assert all(r[3] for r in rows) or all(r[5] < 0 for r in rows)
        self.last = self.rm.forward(rows)
        return self.last

    def accept(self, props):
        out = []
        for p in props:
            n = len(p.chain)
            if p.sampling.temperature <= 0:
                smp = self.ref.sampler(temperature=0.0, seed=1)
                ids, nxt, cl = self.ref.accept_greedy(smp, self.last[p.root:p.root + 2 * n + 1], p.chain, p.alt,
                                                      model=self.rm, seq=p.seq, cache_len=p.cache_len, n_draft=n)
                self.ref.free_sampler(smp)
                out.append(SimpleNamespace(ids=ids, next=nxt, cache_len=cl, uniforms_used=0))
            else:
                q = [list(zip(p.q_p[o:o + k].tolist(), p.q_id[o:o + k].tolist()))
                     for o, k in zip(np.concatenate([[0], np.cumsum(p.q_n)[:-1]]).astype(int), p.q_n)]
                ids, nxt, used = self.oracle.accept_sampled(self.last[p.root:p.root + n + 1], p.chain, q, p.uniforms)
                out.append(SimpleNamespace(ids=ids, next=nxt, cache_len=p.cache_len + 1 + len(ids),
                                           uniforms_used=used))
        return out


def test_parity_harness_reports_exact_agreement(mk, ref, oracle, model_paths):
    from oracle import RefModel
    from oracle.parity import compare, device_leg, reference_leg
    path = model_paths["q8"]
    R, P, kk = 3, 19, 4
    dev = RefAsDevice(ref, RefModel(ref, path, P + 2 * kk + 4, R), oracle)
    d = device_leg(mk, dev, R, P, kk, seed=5, max_batch=8)  # 8-row chunks: prompts split mid-request
    r = reference_leg(ref, RefModel(ref, path, P + 2 * kk + 4, R), d)
    c = compare(d, r)
    assert c["max_abs_logits"] == 0.0
    assert c["greedy_compared"] >= 1 and c["greedy_ok"]
    assert c["sampled_ok"] and c["sampled_identical_ref_logits"] == R
    assert c["ok"]
    assert len(d["tree_rows"]) == R * (2 * kk + 1) and len(d["chain_rows"]) == R * (kk + 1)
    # the 0.55 rule drafted some greedy tokens, so some drafts were accepted
    assert c["accepted_greedy"] > 0


def test_parity_compare_flags_a_planted_difference(mk, ref, oracle, model_paths):
    """A logit moved by more than the tolerance in the oracle-side copy must fail the comparison."""
    from oracle import RefModel
    from oracle.parity import compare, device_leg, reference_leg
    path = model_paths["q8"]
    dev = RefAsDevice(ref, RefModel(ref, path, 40, 2), oracle)
    d = device_leg(mk, dev, 2, 9, 3, seed=2, sampled=False)
    r = reference_leg(ref, RefModel(ref, path, 40, 2), d)
    assert compare(d, r)["ok"]
    r["tree_logits"] = r["tree_logits"].copy()
    r["tree_logits"][1, 7] += 0.05
    c = compare(d, r)
    assert not c["ok"] and abs(c["max_abs_logits"] - 0.05) < 1e-6
