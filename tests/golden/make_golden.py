"""Generates tests/golden/golden.npz: known answers from malkin's own CPU path (oracle/_ref, the reference sources
compiled unchanged) on seeded inputs. Run where the reference is mounted and the CPU has AVX-512 VNNI / BF16:

    python tests/golden/make_golden.py

Model cases store the synthetic-model spec (the product's writer regenerates the same bytes anywhere; the file's
SHA-256 is stored to prove it) plus the batches and malkin's logits / accept results.
"""
from __future__ import annotations

import hashlib
import os
import sys
import tempfile

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)

import malkin_b200 as mk  # noqa: E402  (synthetic GGUF writer only)
from oracle import Ref, RefModel  # noqa: E402

OUT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden.npz")

# Model specs used by the golden model cases and the GPU parity tests.
SPECS = {
    "q8": dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=128, n_vocab=1000,
               type_default=mk.TYPE_Q8_0, seed=0),
    "kq": dict(n_layer=2, n_embd=512, n_ff=1024, n_head=4, n_head_kv=2, head_dim=128, n_vocab=1000,
               type_default=mk.TYPE_Q4_K, type_attn_v=mk.TYPE_Q6_K, type_ffn_down=mk.TYPE_Q6_K,
               type_output=mk.TYPE_Q6_K, type_embd=mk.TYPE_Q4_K, seed=5),
}


def sha(path: str) -> str:
    with open(path, "rb") as f:
        return hashlib.sha256(f.read()).hexdigest()


def random_rows(rng, t: int, rows: int, k: int) -> np.ndarray:
    """Random GGUF rows with sane fp16 scales (as test_quant.cpp:22-59 builds them)."""
    rb = mk.row_bytes(t, k)
    w = rng.integers(0, 256, (rows, rb), dtype=np.uint8)

    def f16(v):
        return np.frombuffer(np.float16(v).tobytes(), np.uint8)

    for r in range(rows):
        if t == mk.TYPE_Q8_0:
            for b in range(k // 32):
                w[r, 34 * b:34 * b + 2] = f16(rng.uniform(0.001, 0.02))
        elif t == mk.TYPE_Q4_K:
            for b in range(k // 256):
                w[r, 144 * b:144 * b + 2] = f16(rng.uniform(0.001, 0.02))
                w[r, 144 * b + 2:144 * b + 4] = f16(rng.uniform(0.001, 0.02))
        elif t == mk.TYPE_Q6_K:
            for b in range(k // 256):
                w[r, 210 * b + 208:210 * b + 210] = f16(rng.uniform(0.001, 0.02))
    return w


def tree_batch(rng, reqs, V):
    """Engine::build_batch greedy layout (engine.cpp:362-379) for [(seq, P, next, chain, alt)]."""
    b = []
    roots = []
    for seq, P, nxt, chain, alt in reqs:
        root = len(b)
        roots.append(root)
        b.append((nxt, seq, P, 1, -1, -1))
        for i in range(len(chain)):
            par = root if i == 0 else root + 2 * i - 1
            b.append((int(chain[i]), seq, P + 1 + i, 1, P + 1 + 2 * i, par))
            b.append((int(alt[i]), seq, P + 1 + i, 1, P + 2 + 2 * i, par))
    return b, roots


def main() -> None:
    r = Ref()
    rng = np.random.default_rng(42)
    g = {}
    # quantize_row_q8: random rows plus edge rows (zeros, one spike, exact .5 ties after scaling)
    x = rng.uniform(-3, 3, (6, 256)).astype(np.float32)
    x[1] = 0.0
    x[2] = 0.0
    x[2, 7] = 5.0
    x[3] = np.arange(256, dtype=np.float32) / 2.0 - 64.0
    g["q8_x"] = x
    g["q8_blocks"] = np.stack([r.quantize_row_q8(row).view(np.uint8) for row in x])
    # quantize_i8 (KV rows)
    xi = rng.uniform(-2, 2, (5, 128)).astype(np.float32)
    xi[4] = 0.0
    g["i8_x"] = xi
    qs = [r.quantize_i8(row) for row in xi]
    g["i8_q"] = np.stack([q for q, _ in qs])
    g["i8_d"] = np.asarray([d for _, d in qs], dtype=np.float32)
    # dequantize_row + matmul (compact panels and row path) per weight type
    for t in (mk.TYPE_Q8_0, mk.TYPE_Q4_K, mk.TYPE_Q6_K):
        rows, cols, n = 35, 512, 19
        w = random_rows(rng, t, rows, cols)
        xx = rng.uniform(-2, 2, (n, cols)).astype(np.float32)
        g[f"mm{t}_w"] = w
        g[f"mm{t}_x"] = xx
        g[f"mm{t}_deq"] = np.stack([r.dequantize_row(t, w[i], cols) for i in range(4)])
        g[f"mm{t}_y"] = r.matmul(t, w, rows, cols, xx, mode=1)
        g[f"mm{t}_yrow"] = r.matmul(t, w, rows, cols, xx, mode=0)
    # silu_mul
    gg = rng.uniform(-6, 6, 512).astype(np.float32)
    uu = rng.uniform(-2, 2, 512).astype(np.float32)
    g["silu_g"], g["silu_u"], g["silu_y"] = gg, uu, r.silu_mul(gg, uu)
    # attention with tree extra keys (test_quant.cpp:138-211 cases)
    att = []
    for G, D, n, ne in ((1, 64, 1, 0), (2, 128, 7, 3), (4, 128, 300, 5), (4, 64, 33, 9)):
        rows = n + ne + 4
        q = rng.uniform(-3, 3, G * D).astype(np.float32)
        k = rng.integers(-127, 128, (rows, D)).astype(np.int8)
        v = rng.integers(-127, 128, (rows, D)).astype(np.int8)
        ks = rng.uniform(0.005, 0.03, rows).astype(np.float32)
        vs = rng.uniform(0.005, 0.03, rows).astype(np.float32)
        extra = rng.choice(np.arange(n, rows), ne, replace=False).astype(np.int32) if ne else np.zeros(0, np.int32)
        scale = np.float32(1.0 / np.sqrt(D))
        out = r.attend(q, G, D, k, v, ks, vs, n, extra, scale)
        att.append((G, D, n, q, k, v, ks, vs, extra, out))
    for i, (G, D, n, q, k, v, ks, vs, extra, out) in enumerate(att):
        g[f"att{i}_shape"] = np.asarray([G, D, n], dtype=np.int32)
        g[f"att{i}_q"], g[f"att{i}_k"], g[f"att{i}_v"] = q, k, v
        g[f"att{i}_ks"], g[f"att{i}_vs"], g[f"att{i}_extra"], g[f"att{i}_out"] = ks, vs, extra, out
    # sampler: uniforms, distribution, verify-chain decisions
    g["rng_seed"] = np.asarray([1234], dtype=np.uint64)
    g["rng_u"] = r.uniforms(1234, 64)
    lg = rng.normal(0, 2, (6, 1000)).astype(np.float32)
    g["dist_logits"] = lg
    dp, di = [], []
    for row in lg:
        s = r.sampler(seed=7)
        p, ids = r.distribution(s, row)
        r.free_sampler(s)
        dp.append(np.pad(p, (0, 40 - len(p))))
        di.append(np.pad(ids, (0, 40 - len(ids)), constant_values=-1))
    g["dist_p"], g["dist_id"] = np.stack(dp), np.stack(di)
    # accept_sampled on fixed logits rows with draft distributions over each row's top-8 (Dirichlet(1))
    acc_cases = []
    for case in range(12):
        kk = 4
        lrows = rng.normal(0, 1.5, (kk + 1, 1000)).astype(np.float32)
        chain, q = [], []
        for i in range(kk):
            top = np.argsort(-lrows[i], kind="stable")[:8]
            w8 = rng.dirichlet(np.ones(8)).astype(np.float32)
            q.append([(float(p), int(t)) for p, t in zip(w8, top)])
            chain.append(int(rng.choice(top, p=w8 / w8.sum())))
        seed = 100 + case
        s = r.sampler(seed=seed)
        ids, nxt = r.accept_sampled(s, lrows, chain, q)
        r.free_sampler(s)
        acc_cases.append((lrows, chain, q, seed, ids, nxt))
    g["as_logits"] = np.stack([c[0] for c in acc_cases])
    g["as_chain"] = np.asarray([c[1] for c in acc_cases], dtype=np.int32)
    g["as_qp"] = np.asarray([[[p for p, _ in d] for d in c[2]] for c in acc_cases], dtype=np.float32)
    g["as_qid"] = np.asarray([[[t for _, t in d] for d in c[2]] for c in acc_cases], dtype=np.int32)
    g["as_seed"] = np.asarray([c[3] for c in acc_cases], dtype=np.uint64)
    g["as_n"] = np.asarray([len(c[4]) for c in acc_cases], dtype=np.int32)
    g["as_ids"] = np.asarray([c[4] + [-1] * (4 - len(c[4])) for c in acc_cases], dtype=np.int32)
    g["as_next"] = np.asarray([c[5] for c in acc_cases], dtype=np.int32)
    # model cases: prefill two sequences, then a greedy tree verify of both, then accept with move_kv
    with tempfile.TemporaryDirectory() as td:
        for name, spec in SPECS.items():
            path = os.path.join(td, name + ".gguf")
            mk.synth_gguf(path, **spec)
            g[f"m_{name}_sha"] = np.frombuffer(bytes.fromhex(sha(path)), np.uint8)
            V = spec["n_vocab"]
            n_ctx = 64
            m = RefModel(r, path, n_ctx, 2)
            lens = (12, 9)
            pre = []
            for seq, L in enumerate(lens):
                toks = rng.integers(0, V, L)
                pre += [(int(t), seq, i, int(i == L - 1), -1, -1) for i, t in enumerate(toks)]
            pl = m.forward(pre)
            nexts = [int(np.argmax(pl[0])), int(np.argmax(pl[1]))]
            kk = 4
            reqs = []
            for seq, L in enumerate(lens):
                chain = rng.integers(0, V, kk)
                alt = rng.integers(0, V, kk)
                reqs.append((seq, L, nexts[seq], chain, alt))
            b, roots = tree_batch(rng, reqs, V)
            tl = m.forward(b)
            # make chain[0] the target's greedy continuation of request 0 so the walk accepts at least one node
            reqs[0] = (reqs[0][0], reqs[0][1], reqs[0][2], np.concatenate([[int(np.argmax(tl[roots[0]]))],
                                                                            reqs[0][3][1:]]), reqs[0][4])
            b, roots = tree_batch(rng, reqs, V)
            tl = m.forward(b)
            accs = []
            for (seq, P, nxt, chain, alt), root in zip(reqs, roots):
                s = r.sampler(temperature=0.0, seed=1)
                ids, nx, cl = r.accept_greedy(s, tl[root:root + 2 * kk + 1], chain, alt, model=m, seq=seq,
                                              cache_len=P)
                r.free_sampler(s)
                accs.append((ids, nx, cl))
            # next step after the accept (KV compacted by move_kv): plain decode of each request's next token
            step2 = [(a[1], seq, a[2], 1, -1, -1) for seq, a in enumerate(accs)]
            l2 = m.forward(step2)
            g[f"m_{name}_pre"] = np.asarray(pre, dtype=np.int32)
            g[f"m_{name}_pre_logits"] = pl
            g[f"m_{name}_tree"] = np.asarray(b, dtype=np.int32)
            g[f"m_{name}_tree_logits"] = tl
            g[f"m_{name}_roots"] = np.asarray(roots, dtype=np.int32)
            g[f"m_{name}_acc_n"] = np.asarray([len(a[0]) for a in accs], dtype=np.int32)
            g[f"m_{name}_acc_ids"] = np.asarray([a[0] + [-1] * (kk - len(a[0])) for a in accs], dtype=np.int32)
            g[f"m_{name}_acc_next"] = np.asarray([a[1] for a in accs], dtype=np.int32)
            g[f"m_{name}_acc_cache"] = np.asarray([a[2] for a in accs], dtype=np.int32)
            g[f"m_{name}_step2"] = np.asarray(step2, dtype=np.int32)
            g[f"m_{name}_step2_logits"] = l2
            del m
    np.savez_compressed(OUT, **g)
    print(f"wrote {OUT}: {os.path.getsize(OUT)} bytes, {len(g)} arrays")


if __name__ == "__main__":
    main()
