"""Tensor parallel on 2 GPUs (skipped with fewer): one process per GPU over NCCL, q / k / v / gate / up column-split,
wo / down row-split with an allreduce, vocabulary-split LM head with gathered candidates. Logits and greedy accepts
must match the single-GPU path (2e-2 max-abs logits; identical accepted paths where the top-1 margin exceeds 1e-2)."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 2e-2


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


def _child(rank, world, nccl_id, path, seed, q):
    import sys
    sys.path[:0] = ["tests", "tests/golden"]
    import malkin_b200 as mk
    try:
        q.put((rank, _run(mk, path, rank, rank, world, nccl_id, seed), None))
    except Exception as e:  # reported to the parent, which fails the test
        q.put((rank, None, repr(e)))


def test_tp2_matches_single_gpu(mk, model_paths, torch_cuda):
    torch = torch_cuda
    if torch.cuda.device_count() < 2:
        pytest.skip("tensor parallel needs 2 GPUs")
    import torch.multiprocessing as mp
    path, seed = model_paths["q8"], 7
    ref_pl, ref_tl, ref_acc = _run(mk, path, 0, 0, 1, None, seed)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    nccl_id = mk.nccl_unique_id()
    procs = [ctx.Process(target=_child, args=(r, 2, nccl_id, path, seed, q)) for r in range(2)]
    for p in procs:
        p.start()
    out = {}
    for _ in range(2):
        rank, res, err = q.get(timeout=300)
        assert err is None, err
        out[rank] = res
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank in range(2):  # every rank returns the full logits and the same accepts
        pl, tl, acc = out[rank]
        assert np.abs(pl - ref_pl).max() < TOL
        assert np.abs(tl - ref_tl).max() < TOL
        s = np.sort(ref_tl, axis=-1)
        for j, (a, b) in enumerate(zip(acc, ref_acc)):
            root = j * 7
            if np.all(s[root:root + 7, -1] - s[root:root + 7, -2] > 1e-2):
                assert a == b
