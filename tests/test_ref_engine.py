"""The engine checker (malkin's Engine compiled into oracle/_ref with the stand-in tokenizer) on CPU: it generates,
speculates and scores perplexity through the harness, and shows the properties the device engine is held to -
requests decoded together give the tokens they give alone, the target as its own draft has every greedy draft
accepted, and speculation never changes greedy output."""
import pytest

SPEC = dict(n_layer=2, n_embd=128, n_ff=256, n_head=4, n_head_kv=2, head_dim=32, n_vocab=500, n_ctx_train=256)
REQS = [dict(prompt=[11, 12, 13], max_tokens=10), dict(prompt=[11, 12, 40, 41], max_tokens=12),
        dict(prompt=[7, 8], max_tokens=9, temperature=0.8, seed=5)]


@pytest.fixture(scope="module")
def files(tmp_path_factory, mk):
    d = tmp_path_factory.mktemp("refengine")
    return (mk.synth_gguf(str(d / "t.gguf"), seed=2, **SPEC),
            mk.synth_gguf(str(d / "d.gguf"), seed=8, **dict(SPEC, n_layer=1)))


def test_reference_engine_properties(ref, files):
    from oracle import RefEngine
    t, d = files
    plain = RefEngine(ref, t, 128, parallel=3, threads=2).generate(REQS)
    alone = RefEngine(ref, t, 128, parallel=3, threads=2).generate(REQS, sequential=True)
    assert [x[0] for x in plain] == [x[0] for x in alone]
    assert [len(x[0]) for x in plain] == [q["max_tokens"] for q in REQS]
    self_draft = RefEngine(ref, t, 128, parallel=3, draft=t, threads=2).generate(REQS)
    other = RefEngine(ref, t, 128, parallel=3, draft=d, threads=2).generate(REQS)
    for i, q in enumerate(REQS):
        if "temperature" in q:
            continue
        assert self_draft[i][0] == plain[i][0] == other[i][0]
        assert self_draft[i][1][4] == self_draft[i][1][3] > 0  # accepted == drafted
    nll, n = RefEngine(ref, t, 128, threads=2).perplexity(list(range(100, 356)), 64)
    assert n == 4 * (64 - 1 - 32) and 0 < nll < 20
