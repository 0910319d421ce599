"""Model-level parity of the sm_100a path through the C ABI: prefill and tree-verify logits bit-identical to malkin's
(golden) - every float operation runs in malkin's order - greedy accepted paths identical, KV compaction (move_kv)
correct (the next step matches), sampled decisions identical given the same uniforms."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2  # the north star's max-abs logits tolerance; the path is bit-exact, so the tests require equality


def load(mk, path, n_ctx=64, n_seq=2, max_batch=256):
    return mk.Model(0).load(path).alloc_kv(n_ctx, n_seq, max_batch)


def batch_of(mk, rows):
    return mk.make_batch(mk.BatchToken(int(r[0]), int(r[1]), int(r[2]), bool(r[3]), int(r[4]), int(r[5])) for r in rows)


def margin_ok(logits_rows):
    s = np.sort(logits_rows, axis=-1)
    return bool(np.all(s[:, -1] - s[:, -2] > 1e-2))


@pytest.mark.parametrize("name", ["q8", "kq"])
def test_verify_step_matches_reference(mk, golden, model_paths, name, torch_cuda):
    m = load(mk, model_paths[name])
    pl = m.forward(batch_of(mk, golden[f"m_{name}_pre"]))
    assert np.array_equal(pl, golden[f"m_{name}_pre_logits"])
    tree = golden[f"m_{name}_tree"]
    tl = m.forward(batch_of(mk, tree))
    gl = golden[f"m_{name}_tree_logits"]
    assert np.array_equal(tl, gl)
    kk = 4
    props = []
    for root in golden[f"m_{name}_roots"]:
        chain = [int(tree[root + 1 + 2 * i][0]) for i in range(kk)]
        alt = [int(tree[root + 2 + 2 * i][0]) for i in range(kk)]
        props.append(mk.Proposal(seq=int(tree[root][1]), root=int(root), cache_len=int(tree[root][2]), chain=chain,
                                 alt=alt))
    res = m.accept(props)
    for j, (r, root) in enumerate(zip(res, golden[f"m_{name}_roots"])):
        n = int(golden[f"m_{name}_acc_n"][j])
        assert r.ids == list(golden[f"m_{name}_acc_ids"][j][:n])
        assert r.next == int(golden[f"m_{name}_acc_next"][j])
        assert r.cache_len == int(golden[f"m_{name}_acc_cache"][j])
    # next step reads the compacted KV rows
    l2 = m.forward(batch_of(mk, golden[f"m_{name}_step2"]))
    assert np.array_equal(l2, golden[f"m_{name}_step2_logits"])
    m.close()


def test_verify_step_matches_oracle_fresh(mk, oracle, model_paths, torch_cuda):
    """Fresh seeded batch: device forward + accept vs the oracle forward + accept on the same inputs."""
    from oracle import OracleModel
    path = model_paths["q8"]
    m = load(mk, path, n_ctx=96, n_seq=3)
    om = OracleModel(oracle, path, 96, 3)
    rng = np.random.default_rng(11)
    pre = []
    for seq, L in enumerate((20, 33, 7)):
        pre += [(int(t), seq, i, int(i == L - 1), -1, -1) for i, t in enumerate(rng.integers(0, 1000, L))]
    a = m.forward(batch_of(mk, pre))
    b = om.forward(pre)
    assert np.array_equal(a, b)
    lens = (20, 33, 7)
    rows, props = [], []
    for seq in range(3):
        P, root, kk = lens[seq], len(rows), 3
        greedy = int(np.argmax(b[seq]))
        rows.append((greedy, seq, P, 1, -1, -1))
        chain = [int(x) for x in rng.integers(0, 1000, kk)]
        alt = [int(x) for x in rng.integers(0, 1000, kk)]
        for i in range(kk):
            par = root if i == 0 else root + 2 * i - 1
            rows.append((chain[i], seq, P + 1 + i, 1, P + 1 + 2 * i, par))
            rows.append((alt[i], seq, P + 1 + i, 1, P + 2 + 2 * i, par))
        props.append((seq, root, P, chain, alt))
    ta = m.forward(batch_of(mk, rows))
    tb = om.forward(rows)
    assert np.array_equal(ta, tb)
    res = m.accept([mk.Proposal(seq=s, root=r, cache_len=P, chain=c, alt=al) for s, r, P, c, al in props])
    for (s, r, P, c, al), got in zip(props, res):
        ids, nxt, _ = oracle.accept_greedy(ta[r:r + 7], c, al)  # identical logits -> identical walk
        assert got.ids == ids and got.next == nxt


def test_sampled_accept_identical_decisions(mk, oracle, model_paths, torch_cuda):
    """Engine::accept_sampled on device vs the oracle on the same logits and the same uniform stream."""
    path = model_paths["q8"]
    m = load(mk, path, n_ctx=64, n_seq=4)
    rng = np.random.default_rng(3)
    pre = []
    for seq in range(4):
        pre += [(int(t), seq, i, int(i == 9), -1, -1) for i, t in enumerate(rng.integers(0, 1000, 10))]
    m.forward(batch_of(mk, pre))
    kk = 5
    rows, props = [], []
    for seq in range(4):
        root = len(rows)
        chain = [int(x) for x in rng.integers(0, 1000, kk)]
        rows.append((int(rng.integers(0, 1000)), seq, 10, 1, -1, -1))
        rows += [(chain[i], seq, 11 + i, 1, -1, -1) for i in range(kk)]
        props.append((seq, root, chain))
    lg = m.forward(batch_of(mk, rows))
    for trial in range(3):
        mprops, want = [], []
        for seq, root, chain in props:
            q = []
            for i in range(kk):
                top = np.argsort(-lg[root + i], kind="stable")[:8]
                w8 = rng.dirichlet(np.ones(8)).astype(np.float32)
                q.append([(float(p), int(t)) for p, t in zip(w8, top)])
                if trial > 0 and i < len(chain):
                    chain[i] = int(top[int(rng.integers(0, 3))])
            U = mk.rng_uniforms(500 + 17 * seq + trial, 16)
            s = mk.Sampling(temperature=0.8, top_p=0.95, top_k=40, min_p=0.05)
            mprops.append(mk.Proposal(seq=seq, root=root, cache_len=10, chain=chain, sampling=s, q=q, uniforms=U))
            want.append(oracle.accept_sampled(lg[root:root + kk + 1], chain, q, U))
        res = m.accept(mprops)
        for got, (ids, nxt, used) in zip(res, want):
            assert got.ids == ids and got.next == nxt and got.uniforms_used == used


def test_batch_validation_errors(mk, model_paths, torch_cuda):
    """Model::forward's checks (model.cpp:280-305): errors, not crashes; the context stays usable."""
    m = load(mk, model_paths["q8"], n_ctx=16, n_seq=1)
    cases = [
        [mk.BatchToken(1, 1, 0, True)],                 # bad sequence
        [mk.BatchToken(1, 0, 16, True)],                # pos >= n_ctx
        [mk.BatchToken(1000, 0, 0, True)],              # token id out of range
        [mk.BatchToken(1, 0, 0, True), mk.BatchToken(2, 0, 1, True, 1, 1)],  # parent >= own index
        [mk.BatchToken(1, 0, 0, True), mk.BatchToken(2, 0, 1, True, 16, 0)],  # tree kv row out of range
    ]
    for c in cases:
        with pytest.raises(mk.MalkinError) as e:
            m.forward(c)
        assert e.value.code == mk.MK_ERR_ARG
    with pytest.raises(mk.MalkinError):
        m.forward([mk.BatchToken(1, 0, 0, True)] * 300)  # > max_batch
    out = m.forward([mk.BatchToken(1, 0, 0, True)])
    assert out.shape == (1, 1000) and np.isfinite(out).all()
    with pytest.raises(mk.MalkinError) as e:
        m.accept([mk.Proposal(seq=0, root=0, cache_len=0, sampling=mk.Sampling(presence_penalty=0.5), chain=[],
                              uniforms=[0.5])])
    assert e.value.code == mk.MK_ERR_UNSUPPORTED


def test_continuous_batch_equals_separate(mk, model_paths, torch_cuda):
    """Two sequences in one forward == each alone (rows of one sequence never see the other's keys)."""
    path = model_paths["kq"]
    rng = np.random.default_rng(8)
    ta = [(int(t), 0, i, 1, -1, -1) for i, t in enumerate(rng.integers(0, 1000, 6))]
    tb = [(int(t), 1, i, 1, -1, -1) for i, t in enumerate(rng.integers(0, 1000, 9))]
    m1 = load(mk, path)
    both = m1.forward(batch_of(mk, ta + tb))
    m2 = load(mk, path)
    a = m2.forward(batch_of(mk, ta))
    b = m2.forward(batch_of(mk, tb))
    # every row's arithmetic is independent of the other rows in the batch
    assert np.array_equal(both, np.concatenate([a, b]))


def test_profile_and_launch_count(mk, model_paths, torch_cuda):
    m = load(mk, model_paths["q8"])
    b = [mk.BatchToken(5, 0, 0, True)]
    m.forward(b)
    assert m.last_launch_count() > 10
    m.set_profile(True)
    m.forward(b)
    st = m.stage_times()
    assert len(st) == 8 and all(t >= 0 for t in st) and sum(st) > 0


FLOAT_MODELS = {  # malkin's row path for F32 / F16 / BF16 matrices (quant.cpp:171-191, 330-351)
    "f16": dict(type_default=1), "bf16": dict(type_default=30), "f32": dict(type_default=0),
    "mixed": dict(type_default=8, type_attn_v=0, type_ffn_down=1, type_output=30),
}


@pytest.mark.parametrize("name", list(FLOAT_MODELS))
def test_float_weight_models_match_malkin(mk, ref, torch_cuda, tmp_path, name):
    """F32 / F16 / BF16 matrices (alone, and mixed with Q8_0): prefill and tree-verify logits bit-identical to malkin's
    CPU Model, which runs them through vec_dot's dot_f32 / dot_f16 / dot_bf16 (16 fma lanes, then reduce_add)."""
    from oracle import RefModel
    path = mk.synth_gguf(str(tmp_path / f"{name}.gguf"), n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2,
                         head_dim=64, n_vocab=1000, n_ctx_train=256, seed=6, **FLOAT_MODELS[name])
    m = load(mk, path, n_ctx=64, n_seq=1)
    rm = RefModel(ref, path, 64, 1)
    pre = [(int(t), 0, i, 1, -1, -1) for i, t in enumerate(np.random.default_rng(3).integers(0, 1000, 12))]
    assert np.array_equal(m.forward(batch_of(mk, pre)), rm.forward(pre))
    tree = [(17, 0, 12, 1, -1, -1), (23, 0, 13, 1, 13, 0), (5, 0, 13, 1, 14, 0), (99, 0, 14, 1, 15, 1)]
    assert np.array_equal(m.forward(batch_of(mk, tree)), rm.forward(tree))
