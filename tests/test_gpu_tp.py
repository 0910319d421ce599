"""Tensor parallel on 2 / 4 / 8 GPUs (skipped with fewer): one process per GPU over NCCL, q / k / v / gate / up
split by heads / ffn rows, vocabulary-split LM head with gathered candidates. Default (exact) split: attn_output /
ffn_down by output features over the whole gathered input, so the logits and greedy accepts are bit-identical to the
single-GPU path (and so to malkin). Opt-in row split (MALKIN_B200_TP_SPLIT=rows): wo / down by input columns with a
rank sum (peer-memory one-shot or two-shot exchange, or NCCL allreduce) - 2e-2 max-abs logits, identical accepted
paths where the top-1 margin exceeds 1e-2. On one GPU: the exchange kernels against host-emulated peers, including
a peer that never arrives (the bounded wait must reach the caller as MK_ERR_TIMEOUT and leave the next calls
correct)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2
# a model every tensor-parallel size divides: heads, KV heads, E / (16 tp), ffn blocks and vocabulary panels
TP_SPEC = dict(n_layer=2, n_embd=512, n_ff=1024, n_head=8, n_head_kv=8, head_dim=64, n_vocab=1024, seed=11)


@pytest.fixture(scope="module")
def tp_model(tmp_path_factory, mk):
    return mk.synth_gguf(str(tmp_path_factory.mktemp("tp") / "tp.gguf"), type_default=mk.TYPE_Q8_0, **TP_SPEC)


def _batches(rng):
    pre, rows, props = [], [], []
    lens = (20, 13)
    for seq, L in enumerate(lens):
        pre += [(int(t), seq, i, int(i == L - 1), -1, -1) for i, t in enumerate(rng.integers(0, 1000, L))]
    kk = 3
    for seq, P in enumerate(lens):
        root = len(rows)
        chain = [int(x) for x in rng.integers(0, 1000, kk)]
        alt = [int(x) for x in rng.integers(0, 1000, kk)]
        rows.append((int(rng.integers(0, 1000)), seq, P, 1, -1, -1))
        for i in range(kk):
            par = root if i == 0 else root + 2 * i - 1
            rows.append((chain[i], seq, P + 1 + i, 1, P + 1 + 2 * i, par))
            rows.append((alt[i], seq, P + 1 + i, 1, P + 2 + 2 * i, par))
        props.append((seq, root, P, chain, alt))
    return pre, rows, props


def _run(mk, path, device, rank, world, nccl_id, seed):
    from test_gpu_model import batch_of
    m = mk.Model(device, rank, world, nccl_id).load(path).alloc_kv(64, 2, 64)
    pre, rows, props = _batches(np.random.default_rng(seed))
    pl = m.forward(batch_of(mk, pre))
    tl = m.forward(batch_of(mk, rows))
    res = m.accept([mk.Proposal(seq=s, root=r, cache_len=P, chain=c, alt=a) for s, r, P, c, a in props])
    acc = [(x.ids, x.next, x.cache_len) for x in res]
    m.close()
    return pl, tl, acc


def _child(rank, world, nccl_id, path, seed, q, mode):
    import os
    import sys
    if mode != "exact":
        os.environ["MALKIN_B200_TP_SPLIT"] = "rows"
        os.environ["MALKIN_B200_TP_REDUCE"] = mode
    sys.path[:0] = ["tests", "tests/golden"]
    import malkin_b200 as mk
    try:
        q.put((rank, _run(mk, path, rank, rank, world, nccl_id, seed), None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


@pytest.mark.parametrize("world", [2, 4, 8])
@pytest.mark.parametrize("mode", ["exact", "oneshot", "twoshot", "nccl"])
def test_tp_matches_single_gpu(mk, tp_model, torch_cuda, world, mode):
    torch = torch_cuda
    if torch.cuda.device_count() < world:
        pytest.skip(f"tensor parallel over {world} ranks needs {world} GPUs")
    import torch.multiprocessing as mp
    path, seed = tp_model, 7
    ref_pl, ref_tl, ref_acc = _run(mk, path, 0, 0, 1, None, seed)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    nccl_id = mk.nccl_unique_id()
    procs = [ctx.Process(target=_child, args=(r, world, nccl_id, path, seed, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(world):
        rank, res, err = q.get(timeout=300)
        assert err is None, err
        out[rank] = res
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(world):  # every rank returns the full logits and the same accepts
        pl, tl, acc = out[rank]
        if mode == "exact":
            assert np.array_equal(pl, ref_pl) and np.array_equal(tl, ref_tl)
            assert acc == ref_acc
            continue
        assert np.abs(pl - ref_pl).max() < TOL
        assert np.abs(tl - ref_tl).max() < TOL
        s = np.sort(ref_tl, axis=-1)
        for j, (a, b) in enumerate(zip(acc, ref_acc)):
            root = j * 7
            if np.all(s[root:root + 7, -1] - s[root:root + 7, -2] > 1e-2):
                assert a == b


@pytest.mark.parametrize("twoshot", [False, True])
@pytest.mark.parametrize("size", [2, 8])
def test_tp_exchange_timeout_then_correct(mk, torch_cuda, twoshot, size):
    """Rank 0's exchange kernels on one GPU against host-emulated peers: call 1 complete, call 2 with peer 1 absent
    (its flag is never set: the bounded wait gives up and the call reports MK_ERR_TIMEOUT), calls 3 and 4 complete
    again and must give the exact rank-order sums, which shows the arrival counters and epochs were left consistent."""
    rng = np.random.default_rng(size + 10 * twoshot)
    calls, n, cols = 4, 17, 4096
    parts = rng.standard_normal((calls, size, n, cols)).astype(np.float32)
    out, st = mk.tp_exchange_check(parts, twoshot=twoshot, absent=[-1, 1, -1, -1], wait_polls=1 << 14)
    assert list(st) == [mk.MK_OK, mk.MK_ERR_TIMEOUT, mk.MK_OK, mk.MK_OK]
    for k in (0, 2, 3):
        want = parts[k, 0].copy()
        for r in range(1, size):
            want = (want + parts[k, r]).astype(np.float32)
        assert np.array_equal(out[k], want), k
