"""Tensor-parallel host logic on CPU: the shard plan each rank derives from the GGUF (mk_tp_shard_of, the geometry
Model::load uses), checked across world_size-2 gloo ranks and for every tp size, plus the max-over-ranks reduction
bench.py uses for timing. Column split of q / k / v by head, ffn split in whole ffn_down blocks, vocabulary split of
the LM head; every dimension must be covered exactly once, in rank order."""
import os
import socket

import pytest

SPECS = {
    # 9 Q8_0 ffn units of 32 values: uneven at tp 2 (4 + 5 units) and tp 4
    "q8": dict(n_layer=1, n_embd=256, n_ff=288, n_head=8, n_head_kv=8, head_dim=64, n_vocab=1001, seed=3),
    # 3 Q6_K ffn_down units of 256 values
    "kq": dict(n_layer=1, n_embd=512, n_ff=768, n_head=8, n_head_kv=4, head_dim=64, n_vocab=999, seed=4),
}


def _models(mk, tmp_path):
    out = {}
    for name, spec in SPECS.items():
        spec = dict(spec)
        if name == "q8":
            spec["type_default"] = mk.TYPE_Q8_0
        else:
            spec.update(type_default=mk.TYPE_Q4_K, type_ffn_down=mk.TYPE_Q6_K, type_output=mk.TYPE_Q6_K,
                        type_embd=mk.TYPE_Q4_K)
        out[name] = mk.synth_gguf(str(tmp_path / f"{name}.gguf"), **spec)
    return out


def _check_partition(shards, spec, unit):
    n_head, n_kv, n_ff, n_vocab = spec["n_head"], spec["n_head_kv"], spec["n_ff"], spec["n_vocab"]
    for field0, field, total in (("head0", "heads", n_head), ("kv_head0", "kv_heads", n_kv), ("ffn0", "ffn", n_ff),
                                 ("vocab0", "vocab", n_vocab), ("embd0", "embd", spec["n_embd"])):
        pos = 0
        for s in shards:
            assert s[field0] == pos, (field0, shards)
            pos += s[field]
        assert pos == total, (field, shards)
    for s in shards:
        assert s["ffn0"] % unit == 0 and s["ffn"] % unit == 0
        assert s["heads"] == n_head // len(shards) and s["kv_heads"] == n_kv // len(shards)
        assert s["embd"] == spec["n_embd"] // len(shards) and s["embd"] % 16 == 0  # whole 16-row panels
    sizes = [s["ffn"] // unit for s in shards]
    assert max(sizes) - min(sizes) <= 1  # as even as whole blocks allow


def _as_dict(s):
    return {k: getattr(s, k) for k, _ in s._fields_}


def test_shard_plan_every_tp_size(mk, tmp_path):
    paths = _models(mk, tmp_path)
    for name, unit in (("q8", 32), ("kq", 256)):
        for tp in (1, 2, 4, 8):
            if SPECS[name]["n_head_kv"] % tp:
                with pytest.raises(mk.MalkinError, match="divide the heads"):
                    mk.tp_shard_of(paths[name], tp, 0)
                continue
            _check_partition([_as_dict(mk.tp_shard_of(paths[name], tp, r)) for r in range(tp)], SPECS[name], unit)
    with pytest.raises(mk.MalkinError, match="bad rank"):
        mk.tp_shard_of(paths["q8"], 2, 2)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, paths, q):
    import torch.distributed as dist
    import malkin_b200 as mk
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        got = {name: _as_dict(mk.tp_shard_of(path, world, rank)) for name, path in paths.items()}
        allg = [None] * world
        dist.all_gather_object(allg, got)
        import torch
        t = torch.tensor([1.5 + rank], dtype=torch.float64)  # per-rank step time -> max over ranks
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        if rank == 0:
            q.put((allg, float(t.item())))
    finally:
        dist.destroy_process_group()


def test_shard_plan_across_gloo_ranks(mk, tmp_path):
    import torch.multiprocessing as mp
    paths = _models(mk, tmp_path)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, paths, q)) for r in range(2)]
    for p in procs:
        p.start()
    allg, tmax = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert tmax == 2.5
    for name, unit in (("q8", 32), ("kq", 256)):
        _check_partition([allg[r][name] for r in range(2)], SPECS[name], unit)
