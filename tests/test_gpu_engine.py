"""The device engine (mk_engine_*: continuous batching, draft-model speculation, adaptive draft length, emission,
perplexity) against malkin's own Engine (engine.cpp, compiled into oracle/_ref with a stand-in tokenizer) on the
same synthetic GGUF files: every request's generated tokens identical, and the drafted / accepted / completion
counts and finish reasons identical, greedy and sampled (temperature 0.8, seeded), with no draft, the target as its
own draft (every draft accepted, the draft length grows to its cap) and an unrelated draft (drafts rejected, the
draft length shrinks). Perplexity agrees to 1e-9 relative (the device sums exp in double in another order)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SPEC = dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64, n_vocab=1000, n_ctx_train=512)
N_CTX = 256
PARALLEL = 3
REQS = [  # four requests on three slots: the last waits for a free slot and reuses its prefix
    dict(prompt=[11, 12, 13, 14, 15], max_tokens=20),
    dict(prompt=[11, 12, 13, 99], max_tokens=25),
    dict(prompt=[500, 501, 502], max_tokens=15, temperature=0.8, top_p=0.95, top_k=40, min_p=0.05, seed=9),
    dict(prompt=list(range(300, 340)), max_tokens=12),
]


@pytest.fixture(scope="module")
def files(tmp_path_factory, mk):
    d = tmp_path_factory.mktemp("engine")
    return dict(target=mk.synth_gguf(str(d / "t.gguf"), seed=3, **SPEC),
                draft=mk.synth_gguf(str(d / "d.gguf"), seed=5, **dict(SPEC, n_layer=1)), dir=d)


def device_run(mk, target, draft, reqs, n_draft=0, sequential=False, eog=()):
    t = mk.Model().load(target).alloc_kv(N_CTX, PARALLEL)
    dm = mk.Model().load(draft).alloc_kv(N_CTX, PARALLEL) if draft else None
    e = mk.Engine(t, dm, n_draft)
    toks = {}
    ids = []
    for q in reqs:
        smp = mk.Sampling(q.get("temperature", 0.0), q.get("top_p", 0.95), q.get("top_k", 40), q.get("min_p", 0.05))
        ids.append(e.submit(q["prompt"], q["max_tokens"], smp, q.get("seed", 1), eog))
        if sequential:
            toks.update(e.run())
    toks.update(e.run())
    out = []
    for i in ids:
        s = e.stats(i)
        out.append((toks.get(i, []), (s.prompt_tokens, s.completion_tokens, s.drafted, s.accepted, s.finish)))
    e.close()
    return out


def reference_run(ref, target, draft, reqs, n_draft=0):
    from oracle import RefEngine
    e = RefEngine(ref, target, N_CTX, parallel=PARALLEL, draft=draft, n_draft=n_draft, threads=4)
    res = e.generate(reqs)
    return [(t, (s[0], s[2], s[3], s[4], s[5])) for t, s in res]


@pytest.mark.parametrize("draft", ["none", "self", "other"])
def test_engine_matches_malkin_engine(mk, ref, torch_cuda, files, draft):
    dpath = {"none": None, "self": files["target"], "other": files["draft"]}[draft]
    dev = device_run(mk, files["target"], dpath, REQS)
    want = reference_run(ref, files["target"], dpath, REQS)
    for i, (d, w) in enumerate(zip(dev, want)):
        assert d[0] == w[0], (i, d[0], w[0])
        assert d[1] == w[1], (i, d[1], w[1])
    if draft == "self":  # greedy drafts from the target itself are always accepted
        assert all(d[1][3] == d[1][2] > 0 for d, q in zip(dev, REQS) if "temperature" not in q)
    if draft == "none":
        assert all(d[1][2] == 0 for d in dev)


def test_engine_batched_equals_sequential(mk, torch_cuda, files):
    """The tools/check_parallel.sh property: requests decoded together give the tokens they give alone."""
    a = device_run(mk, files["target"], files["draft"], REQS, sequential=False)
    b = device_run(mk, files["target"], files["draft"], REQS, sequential=True)
    assert [x[0] for x in a] == [x[0] for x in b]


def test_engine_speculation_keeps_greedy_output(mk, torch_cuda, files):
    greedy = [q for q in REQS if "temperature" not in q]
    plain = device_run(mk, files["target"], None, greedy)
    for dpath in (files["target"], files["draft"]):
        spec = device_run(mk, files["target"], dpath, greedy, n_draft=6)
        assert [x[0] for x in spec] == [x[0] for x in plain]


def test_engine_end_of_generation(mk, ref, torch_cuda, files):
    """A request stops at an end-of-generation token (finish "stop"), as malkin's Tokenizer::is_eog ends it."""
    plain = device_run(mk, files["target"], None, REQS[:2])
    eos = plain[0][0][6]
    path = mk.synth_gguf(str(files["dir"] / "t_eos.gguf"), seed=3, eos_token_id=eos, **SPEC)
    dev = device_run(mk, path, files["draft"], REQS, eog=[eos])
    want = reference_run(ref, path, files["draft"], REQS)
    assert [x[0] for x in dev] == [x[0] for x in want]
    assert [x[1] for x in dev] == [x[1] for x in want]
    assert dev[0][1][4] == mk.FINISH_STOP and len(dev[0][0]) == plain[0][0].index(eos)


def test_engine_cancel(mk, torch_cuda, files):
    t = mk.Model().load(files["target"]).alloc_kv(N_CTX, PARALLEL)
    e = mk.Engine(t)
    a = e.submit([1, 2, 3], 50)
    b = e.submit([4, 5, 6], 50)
    e.cancel(b)  # still waiting: ends at the next step without tokens
    ev = e.step()
    assert (b, -1, mk.FINISH_CANCELLED) in ev
    e.cancel(a)  # ends at its next emitted token
    toks = e.run()
    s = e.stats(a)
    assert s.finish == mk.FINISH_CANCELLED and 1 <= s.completion_tokens <= 3
    assert len(toks.get(a, [])) <= 2


def test_engine_rejects_bad_requests(mk, torch_cuda, files):
    t = mk.Model().load(files["target"]).alloc_kv(N_CTX, PARALLEL)
    e = mk.Engine(t)
    with pytest.raises(mk.MalkinError):
        e.submit([], 5)
    with pytest.raises(mk.MalkinError):
        e.submit(list(range(N_CTX)), 5)  # fills the context
    with pytest.raises(mk.MalkinError):
        e.submit([1, 2], 5, mk.Sampling(temperature=0.8, top_k=0))  # whole-vocabulary sampling: not on the device


def test_perplexity_matches_malkin(mk, ref, torch_cuda, files):
    from oracle import RefEngine
    toks = np.random.default_rng(4).integers(0, SPEC["n_vocab"], 300).tolist()
    t = mk.Model().load(files["target"]).alloc_kv(N_CTX, PARALLEL)
    nll, n = mk.Engine(t).perplexity(toks, 128)
    want, wn = RefEngine(ref, files["target"], N_CTX, parallel=PARALLEL, threads=4).perplexity(toks, 128)
    assert n == wn == 2 * (128 - 1 - 64)
    assert abs(nll - want) <= 1e-9 * abs(want)
