"""The oracle (our C restatement of malkin's verify path) pinned against malkin's own outputs: the committed golden
fixtures (made from oracle/_ref by tests/golden/make_golden.py) and, where the reference runs here, live."""
import hashlib

import numpy as np
import pytest

from oracle import OracleModel

TYPES = (8, 12, 14)


def test_quantize_q8_bit_exact(oracle, golden):
    for x, want in zip(golden["q8_x"], golden["q8_blocks"]):
        got = oracle.quantize_row_q8(x).view(np.uint8)
        assert np.array_equal(got.reshape(-1), want.reshape(-1))


def test_quantize_i8_bit_exact(oracle, golden):
    for x, q, d in zip(golden["i8_x"], golden["i8_q"], golden["i8_d"]):
        gq, gd = oracle.quantize_i8(x)
        assert np.array_equal(gq, q) and np.float32(gd) == d


@pytest.mark.parametrize("t", TYPES)
def test_dequantize_bit_exact(oracle, golden, t):
    w = golden[f"mm{t}_w"]
    for i, want in enumerate(golden[f"mm{t}_deq"]):
        assert np.array_equal(oracle.dequantize_row(t, w[i], 512), want)


@pytest.mark.parametrize("t", TYPES)
def test_matmul_bit_exact_vs_compact_panels(oracle, golden, t):
    """Same float operations in the same block order as k_q8_0 / k_q45_k / k_q6_k (gemm_avx512.cpp:67-205)."""
    w, x = golden[f"mm{t}_w"], golden[f"mm{t}_x"]
    y = oracle.matmul(t, w, 35, 512, x)
    assert np.array_equal(y, golden[f"mm{t}_y"])
    # the row path (vec_dot) sums in a different order: same values within float rounding
    yr = golden[f"mm{t}_yrow"]
    assert np.abs(y - yr).max() <= 1e-5 * max(1.0, np.abs(yr).max()) * 50


@pytest.mark.parametrize("t", TYPES)
def test_block_dots_reconstruct_matmul(oracle, golden, t):
    """The exact integer block dots, scaled as malkin scales them, reproduce the bit-exact matmul."""
    w, x = golden[f"mm{t}_w"], golden[f"mm{t}_x"][:3]
    dots = oracle.block_dots(t, w, 35, 512, x)
    xq = [oracle.quantize_row_q8(r) for r in x]
    ref = golden[f"mm{t}_y"][:3]
    # float(dot) exact; recompute the Q8_0 case with the reference formula in float32
    if t == 8:
        for r in range(35):
            for tok in range(3):
                acc = np.float32(0)
                for b in range(16):
                    dw = np.frombuffer(w[r, 34 * b:34 * b + 2].tobytes(), np.float16)[0].astype(np.float32)
                    s = np.float32(dw * xq[tok]["d"][b])
                    acc = np.float32(np.fma(np.float32(dots[r, tok, b]), s, acc)) if hasattr(np, "fma") else \
                        np.float32(np.float64(dots[r, tok, b]) * np.float64(s) + np.float64(acc))
                assert abs(acc - ref[tok, r]) <= 1e-6 * max(1.0, abs(ref[tok, r]))
    assert dots.dtype == np.int32 and np.abs(dots).max() < 2 ** 22


def test_silu_matches(oracle, golden):
    y = oracle.silu_mul(golden["silu_g"], golden["silu_u"])
    np.testing.assert_allclose(y, golden["silu_y"], rtol=1e-6, atol=1e-7)


def test_attention_tree_keys(oracle, golden):
    for i in range(4):
        G, D, n = map(int, golden[f"att{i}_shape"])
        out = oracle.attend(golden[f"att{i}_q"], G, D, golden[f"att{i}_k"], golden[f"att{i}_v"], golden[f"att{i}_ks"],
                            golden[f"att{i}_vs"], n, golden[f"att{i}_extra"], np.float32(1.0 / np.sqrt(D)))
        assert np.array_equal(out, golden[f"att{i}_out"])


def test_distribution_matches(oracle, golden):
    for row, p, ids in zip(golden["dist_logits"], golden["dist_p"], golden["dist_id"]):
        gp, gid = oracle.distribution(row)
        n = int((ids >= 0).sum())
        assert len(gp) == n and np.array_equal(gid, ids[:n])
        np.testing.assert_array_equal(gp, p[:n])


def test_accept_sampled_decisions(oracle, golden):
    """Same accept / reject decisions and tokens as Sampler::verify given the same uniform stream."""
    U_all = {}
    from oracle import Ref
    for c in range(len(golden["as_seed"])):
        seed = int(golden["as_seed"][c])
        q = [[(float(p), int(t)) for p, t in zip(golden["as_qp"][c, i], golden["as_qid"][c, i])] for i in range(4)]
        import malkin_b200 as mk
        U = mk.rng_uniforms(seed, 16)
        ids, nxt, used = oracle.accept_sampled(golden["as_logits"][c], golden["as_chain"][c], q, U)
        n = int(golden["as_n"][c])
        assert ids == list(golden["as_ids"][c][:n]) and nxt == int(golden["as_next"][c])
        U_all[c] = used


@pytest.mark.parametrize("name", ["q8", "kq"])
def test_model_forward_and_accept(oracle, golden, model_paths, name):
    path = model_paths[name]
    with open(path, "rb") as f:
        assert hashlib.sha256(f.read()).digest() == golden[f"m_{name}_sha"].tobytes(), "synthetic model not reproducible"
    m = OracleModel(oracle, path, 64, 2)
    pl = m.forward([tuple(r) for r in golden[f"m_{name}_pre"]])
    # the restatement reproduces malkin's float operations in malkin's order: logits bit-identical
    assert np.array_equal(pl, golden[f"m_{name}_pre_logits"])
    tree = [tuple(r) for r in golden[f"m_{name}_tree"]]
    tl = m.forward(tree)
    assert np.array_equal(tl, golden[f"m_{name}_tree_logits"])
    roots = golden[f"m_{name}_roots"]
    kk = 4
    for j, root in enumerate(roots):
        seq, P = tree[root][1], tree[root][2]
        chain = [tree[root + 1 + 2 * i][0] for i in range(kk)]
        alt = [tree[root + 2 + 2 * i][0] for i in range(kk)]
        ids, nxt, _ = oracle.accept_greedy(tl[root:root + 2 * kk + 1], chain, alt, model=m, seq=seq, cache_len=P)
        n = int(golden[f"m_{name}_acc_n"][j])
        assert ids == list(golden[f"m_{name}_acc_ids"][j][:n]) and nxt == int(golden[f"m_{name}_acc_next"][j])
    l2 = m.forward([tuple(r) for r in golden[f"m_{name}_step2"]])
    assert np.array_equal(l2, golden[f"m_{name}_step2_logits"])


def test_oracle_vs_reference_live(oracle, ref):
    """Where malkin's CPU path runs here: fresh random inputs, oracle vs reference."""
    rng = np.random.default_rng(7)
    for _ in range(4):
        x = rng.standard_normal(1024).astype(np.float32) * rng.uniform(0.01, 10)
        assert oracle.quantize_row_q8(x).tobytes() == ref.quantize_row_q8(x).tobytes()
    from make_golden import random_rows
    for t in TYPES:
        w = random_rows(rng, t, 21, 768 if t == 8 else 768)
        x = rng.uniform(-2, 2, (11, 768)).astype(np.float32)
        assert np.array_equal(oracle.matmul(t, w, 21, 768, x), ref.matmul(t, w, 21, 768, x, mode=1))
    lg = rng.normal(0, 2, 3000).astype(np.float32)
    s = ref.sampler(seed=3)
    p, ids = ref.distribution(s, lg)
    ref.free_sampler(s)
    gp, gid = oracle.distribution(lg)
    assert np.array_equal(gid, ids) and np.array_equal(gp, p)
    assert np.array_equal(ref.uniforms(99, 8), __import__("malkin_b200").rng_uniforms(99, 8))
