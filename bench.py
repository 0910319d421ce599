"""Speculative-verify benchmark: accepted tok/s of malkin's tree-verify step (target forward over every request's
draft tree + greedy acceptance + KV compaction) for a synthetic Qwen3 model, on 1..8 B200s (tensor parallel).

    python bench.py [--gpus N --steps K --warmup W --config 8b]            # this repository's CUDA path
    python bench.py --impl reference [...]                                  # malkin's own CPU path (oracle/_ref)
    torchrun --nproc-per-node N bench.py --gpus N ...                       # N > 1: one rank per GPU

One JSON line on rank 0. A step = one verify pass (forward + accept + move_kv) over a fixed state: every request has
`prompt` tokens of KV (prefilled on the GPU) and the same drafted tree each step, so every step does identical work.
Drafts follow the configuration's rule: at each depth the chain token is the target's greedy token with probability
0.55 (seeded coin flips), otherwise uniform; siblings are uniform. The accepted count per step is therefore fixed by
the seed (accepted = the leading run of matching flips per request, + 1 bonus token each).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

METRIC = "accepted tok/s, Qwen3-8B-arch Q8_0, 8 req x 16-node trees, 1/2/4/8 B200; HBM GB/s"

Q8_0, Q4_K, Q6_K = 8, 12, 14
CONFIGS = {
    # name: model shape, weight types, requests, prompt tokens, draft depth (tree = root + chain + siblings)
    "0.6b": dict(model=dict(n_layer=28, n_embd=1024, n_ff=3072, n_head=16, n_head_kv=8, tied=True,
                            type_default=Q8_0), requests=1, prompt=512, kk=8),
    "4b": dict(model=dict(n_layer=36, n_embd=2560, n_ff=9728, n_head=32, n_head_kv=8, tied=True, type_default=Q4_K,
                          type_attn_v=Q6_K, type_ffn_down=Q6_K, type_output=Q6_K), requests=1, prompt=4096, kk=8),
    "8b": dict(model=dict(n_layer=36, n_embd=4096, n_ff=12288, n_head=32, n_head_kv=8, tied=False,
                          type_default=Q8_0), requests=8, prompt=2048, kk=8),
    "14b": dict(model=dict(n_layer=40, n_embd=5120, n_ff=17408, n_head=40, n_head_kv=8, tied=False,
                           type_default=Q6_K), requests=4, prompt=8192, kk=16),
    "32b": dict(model=dict(n_layer=64, n_embd=5120, n_ff=25600, n_head=64, n_head_kv=8, tied=False,
                           type_default=Q4_K), requests=32, prompt=8192, kk=8),
    # two layers of the 8B shapes (full vocabulary): the small case for ncu captures of the 8B kernels
    "8b-l2": dict(model=dict(n_layer=2, n_embd=4096, n_ff=12288, n_head=32, n_head_kv=8, tied=False,
                             type_default=Q8_0), requests=8, prompt=2048, kk=8),
    # small case for quick checks
    "tiny": dict(model=dict(n_layer=4, n_embd=1024, n_ff=3072, n_head=16, n_head_kv=8, tied=False,
                            type_default=Q8_0), requests=2, prompt=256, kk=8),
}
BLOCK = {Q8_0: (32, 34), Q4_K: (256, 144), Q6_K: (256, 210)}


def model_path(name: str) -> str:
    """Synthetic model file: MALKIN_B200_MODEL_DIR, else /dev/shm when it has room, else the temp dir."""
    import shutil
    d = os.environ.get("MALKIN_B200_MODEL_DIR")
    if not d:
        need = 2.5 * weight_bytes_of(CONFIGS[name])["total"]
        d = os.path.join(tempfile.gettempdir(), "malkin_b200")
        try:
            if os.path.isdir("/dev/shm") and shutil.disk_usage("/dev/shm").free > need:
                d = "/dev/shm/malkin_b200"
        except OSError:
            pass
    os.makedirs(d, exist_ok=True)
    return os.path.join(d, f"qwen3-{name}-synthetic-seed0.gguf")


def spec_of(cfg: dict) -> dict:
    m = dict(cfg["model"])
    return dict(head_dim=128, n_vocab=151936, n_ctx_train=40960, rope_base=1e6, sigma=0.02, seed=0, **m)


def ensure_model(name: str, child: bool = False) -> str:
    """Writes the synthetic GGUF once per box (rank 0); other ranks wait on the marker file. child=True writes it from
    a separate process (`bench.py --write-model NAME`), so the calling process never maps this repository's library
    (the reference arm measures malkin alone)."""
    path = model_path(name)
    if not os.path.exists(path + ".done"):
        if child:
            subprocess.run([sys.executable, os.path.abspath(__file__), "--write-model", name], check=True)
            return path
        import malkin_b200 as mk
        tmp = path + f".tmp{os.getpid()}"
        mk.synth_gguf(tmp, **spec_of(CONFIGS[name]))
        os.replace(tmp, path)
        open(path + ".done", "w").close()
    return path


def weight_bytes_of(cfg: dict) -> dict:
    """GGUF bytes of the streamed matrices (incl. LM head), per layer group and total."""
    m = spec_of(cfg)
    E, F, HD, KD, V, L = m["n_embd"], m["n_ff"], m["n_head"] * 128, m["n_head_kv"] * 128, m["n_vocab"], m["n_layer"]
    td = m["type_default"]
    tv, tdn = m.get("type_attn_v", td), m.get("type_ffn_down", td)
    tout = m.get("type_output", td)

    def rb(t, rows, cols):
        b, s = BLOCK[t]
        return rows * (cols // b) * s
    qkv = rb(td, HD + KD, E) + rb(tv, KD, E)
    wo = rb(td, E, HD)
    gu = 2 * rb(td, F, E)
    down = rb(tdn, E, F)
    out = rb(tout, V, E)
    return dict(qkv=qkv * L, wo=wo * L, gate_up=gu * L, down=down * L, output=out, total=(qkv + wo + gu + down) * L + out)


def kv_bytes_per_token(cfg: dict) -> int:
    m = spec_of(cfg)
    return m["n_layer"] * 2 * m["n_head_kv"] * (128 + 4)


def build_tree(reqs, kk):
    """Engine::build_batch greedy layout (engine.cpp:362-379): per request [next, c0, a0, c1, a1, ...]."""
    rows, roots = [], []
    for seq, P, nxt, chain, alt in reqs:
        root = len(rows)
        roots.append(root)
        rows.append((nxt, seq, P, 1, -1, -1))
        for i in range(kk):
            par = root if i == 0 else root + 2 * i - 1
            rows.append((int(chain[i]), seq, P + 1 + i, 1, P + 1 + 2 * i, par))
            rows.append((int(alt[i]), seq, P + 1 + i, 1, P + 2 + 2 * i, par))
    return rows, roots


def draft_plan(cfg: dict, V: int):
    """Seeded coin flips (p = 0.55) and uniform fallback / sibling tokens; expected accepted tokens per step."""
    rng = np.random.default_rng(2)
    R, kk = cfg["requests"], cfg["kk"]
    flips = rng.random((R, kk)) < 0.55
    chains = rng.integers(0, V, (R, kk))
    alts = rng.integers(0, V, (R, kk))
    lead = [int(np.argmin(np.append(f, False))) for f in flips]  # leading run of True
    return flips, chains, alts, sum(lead) + R


def clocks_start():
    try:
        out = open(os.path.join(tempfile.gettempdir(), f"clocks{os.getpid()}.csv"), "w")
        p = subprocess.Popen(["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                              "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                              "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits", "-lms", "100"],
                             stdout=out, stderr=subprocess.DEVNULL)
        t_end = time.time() + 3.0  # the sampler is running (its first line written) before the timed region starts
        while time.time() < t_end and os.path.getsize(out.name) == 0 and p.poll() is None:
            time.sleep(0.02)
        return p, out
    except Exception:
        return None, None


def clocks_stop(handle, devices):
    p, out = handle
    if p is None:
        return None
    size_at_stop = os.path.getsize(out.name)
    p.terminate()
    p.wait()
    out.close()
    note = None
    if size_at_stop == 0:  # a region shorter than the sampling interval: one reading right after it
        note = "timed region shorter than the 100 ms sampling interval: one reading right after it"
        try:
            with open(out.name, "w") as f:
                subprocess.run(["nvidia-smi", "--query-gpu=index,clocks.sm,clocks.max.sm,power.draw,"
                                "clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
                                "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
                                "clocks_event_reasons.sw_power_cap", "--format=csv,noheader,nounits"],
                               stdout=f, stderr=subprocess.DEVNULL, timeout=20)
        except Exception:
            pass
    sm, mx, reasons = [], 0.0, set()
    names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
    want = {str(d) for d in devices}
    for line in open(out.name):
        f = [x.strip() for x in line.split(",")]
        if len(f) < 9 or f[0] not in want:
            continue
        try:
            sm.append(float(f[1]))
            mx = float(f[2])
        except ValueError:
            continue
        for n, v in zip(names, f[5:9]):
            if v.lower() == "active":
                reasons.add(n)
    os.unlink(out.name)
    if not sm:
        return None
    res = {"sm_mhz": float(np.median(sm)), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm),
           "gpus": sorted(int(d) for d in want)}
    if note:
        res["note"] = note
    return res


def peaks():
    try:
        return json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json"))), "of measured"
    except Exception:
        return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0}, "of fallback"


def profiled_traffic(name: str):
    """DRAM bytes per launch of a kernel from its committed ncu summary (profiles/<name>.md, a line
    'dram_bytes_per_launch: <int>'), or None."""
    try:
        for line in open(os.path.join(ROOT, "profiles", name + ".md")):
            if line.strip().startswith("dram_bytes_per_launch:"):
                return int(line.split(":", 1)[1].strip().split()[0])
    except (OSError, ValueError):
        pass
    return None


def fp32_floor(cfg: dict, world: int, n: int, gu_ms: float, clocks):
    """The gate+up GEMM's other bound: malkin's exact block order needs a float epilogue per (row, token, 32-value
    block) - float(dot), d_w * d_x, fma (Q8_0: 3 FMA-pipe lane operations) - at 128 FMA lanes per SM."""
    s = spec_of(cfg)
    if s["type_default"] != Q8_0 or gu_ms <= 0:
        return None
    rows = 2 * s["n_ff"] // world
    ops = rows * n * (s["n_embd"] // 32) * 3
    mhz = (clocks or {}).get("sm_mhz") or 1965.0
    floor_us = ops / (148 * 128 * mhz * 1e6) * 1e6
    launch_us = gu_ms * 1e3 / s["n_layer"]
    return {"lane_ops_per_launch": ops, "floor_us": floor_us, "launch_us": launch_us, "frac": floor_us / launch_us}


def reference_model(path: str, cfg: dict):
    """malkin's CPU path (oracle/_ref) with the configuration's weights loaded and KV for its requests, all physical
    cores; (ref, model, load seconds) or (None, reason, 0)."""
    from oracle import Ref, RefModel
    why = Ref.available()
    if why:
        return None, why, 0.0
    r = Ref()
    r.set_threads(r.physical_cores())
    t0 = time.perf_counter()
    m = RefModel(r, path, cfg["prompt"] + 2 * cfg["kk"] + 8, cfg["requests"])
    return r, m, time.perf_counter() - t0


def cpu_baseline_sample(path: str, cfg: dict, accepted_per_step: int, steps: int = 1, loaded=None):
    """malkin's own CPU path (oracle/_ref) on the same weights and tree shape, all physical cores. The KV prefix rows
    exist but are not prefilled: malkin's cache is LazyBytes (gguf.cpp:281-296), anonymous pages never written, so its
    attention reads zero pages rather than DRAM-resident keys and the time is optimistic for the CPU."""
    r, m, load_s = loaded if loaded else reference_model(path, cfg)
    if r is None:
        return None, m
    cores = r.physical_cores()
    R, P, kk = cfg["requests"], cfg["prompt"], cfg["kk"]
    V = spec_of(cfg)["n_vocab"]
    _, chains, alts, _ = draft_plan(cfg, V)
    rng = np.random.default_rng(3)
    reqs = [(s, P, int(rng.integers(0, V)), chains[s], alts[s]) for s in range(R)]
    rows, roots = build_tree(reqs, kk)
    # malkin caps a forward at kMaxBatch = 256 rows: larger trees batches split on whole requests
    per = max(1, 256 // (2 * kk + 1))
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        for s0 in range(0, R, per):
            sub = [rw for rw in rows if s0 <= rw[1] < s0 + per]
            base = min(i for i, rw in enumerate(rows) if rw[1] == s0)
            sub = [(a, b, c, d, e, (f - base if f >= 0 else f)) for (a, b, c, d, e, f) in sub]
            lg = m.forward(sub)
            s = r.sampler(temperature=0.0, seed=1)
            for j, seq in enumerate(range(s0, min(R, s0 + per))):
                rt = j * (2 * kk + 1)
                r.accept_greedy(s, lg[rt:rt + 2 * kk + 1], chains[seq], alts[seq], model=None)
            r.free_sampler(s)
        times.append(time.perf_counter() - t0)
    t = min(times)
    return dict(value=accepted_per_step / t, unit="tok/s", cores=cores, kind="reference",
                sample=f"{steps} verify step(s) of the {R}x{2 * kk + 1}-row tree batch (ms/step {t * 1e3:.1f}, "
                       f"model load {load_s:.1f} s); prefix KV rows not prefilled: malkin's lazily allocated cache "
                       f"pages are never written, so its attention reads zero pages (optimistic for the CPU); "
                       f"accepted/step from the seeded draft rule"), None


def run_reference(args, cfg):
    """--impl reference: malkin's CPU path on this config (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    V = spec_of(cfg)["n_vocab"]
    _, _, _, A = draft_plan(cfg, V)
    path = ensure_model(args.config, child=True)
    base, why = cpu_baseline_sample(path, cfg, A, steps=max(1, min(args.steps, 2)))
    line = {"impl": "reference", "metric": METRIC, "unit": "tok/s", "higher_is_better": True,
            "n_gpus": args.gpus, "steps": max(1, min(args.steps, 2)), "warmup": 0, "dtype": "int8 x int8 -> fp32",
            "data": "synthetic", "config": config_json(args, cfg)}
    if base is None:
        line.update({"unavailable": f"malkin CPU path cannot run here: {why}"})
    else:
        line.update({"value": base["value"], "ms_per_step": A / base["value"] * 1e3, "cpu_baseline": base,
                     "e2e": {"value": base["value"], "unit": "tok/s", "h2d_bytes_per_step": 0,
                             "d2h_bytes_per_step": 0}})
    print(json.dumps(line), flush=True)


def config_json(args, cfg):
    m = spec_of(cfg)
    out = {"workload": f"qwen3-{args.config} architecture synthetic, {cfg['requests']} req x {2 * cfg['kk']}-node "
                       f"trees (chain {cfg['kk']} + siblings), {cfg['prompt']}-token KV prefix, greedy accept",
           "weights": "Q8_0" if m["type_default"] == Q8_0 else ("Q4_K" if m["type_default"] == Q4_K else "Q6_K"),
           "requests": cfg["requests"], "rows_per_step": cfg["requests"] * (2 * cfg["kk"] + 1),
           "prompt": cfg["prompt"], "parallelism": f"tp{args.gpus}",
           "q8_gemm": os.environ.get("MALKIN_B200_Q8_GEMM", "exact"),
           "l2": "inputs larger than L2 (weights stream from HBM every step)"}
    if args.gpus > 1 and os.environ.get("MALKIN_B200_TP_SPLIT", "") == "rows":
        out["tp_split"] = "rows (wo / down by input columns, rank sum)"
        out["tp_reduce"] = {"nccl": "ncclAllReduce", "twoshot": "peer memory, two-shot"}.get(
            os.environ.get("MALKIN_B200_TP_REDUCE", ""), "peer memory, one-shot")
    elif args.gpus > 1:
        out["tp_split"] = "exact (wo / down by output features over gathered inputs, NCCL broadcasts + all-gather)"
    return out


# ---------------------------------------------------------------------------------------------------------------
# Kernel probes (for ncu captures of one kernel at the 8B verify shapes; not part of the timed benchmark)
# ---------------------------------------------------------------------------------------------------------------
PROBE_GEMM_SHAPES = {  # name: (rows, cols, weight type); the 8B Q8_0 matrices, then the 4B and 14B K-quant ones
    "gate+up": (24576, 4096, Q8_0), "down": (4096, 12288, Q8_0), "qkv": (6144, 4096, Q8_0), "wo": (4096, 4096, Q8_0),
    "lm_head": (151936, 4096, Q8_0), "gate+up_q4k_4b": (19456, 2560, Q4_K), "down_q6k_4b": (2560, 9728, Q6_K),
    "gate+up_q6k_14b": (34816, 5120, Q6_K), "down_q6k_14b": (5120, 17408, Q6_K),
    "down_tp2": (2048, 12288, Q8_0), "down_tp8": (512, 12288, Q8_0),
    "q_q4k_4b": (4096, 2560, Q4_K), "wo_q4k_4b": (2560, 4096, Q4_K), "v_q6k_4b": (1024, 2560, Q6_K),
    "gate+up_06b": (6144, 1024, Q8_0), "down_06b": (1024, 3072, Q8_0), "qkv_06b": (4096, 1024, Q8_0)}


def probe_gemm(shapes, layouts, n: int, reps: int) -> None:
    """mk_matmul on seeded random weights of the named shapes, n tokens. The first call measures the kernel shapes
    (gemm_tune); the reps after it run between cudaProfilerStart / Stop, so `ncu --profile-from-start off` sees only
    the chosen kernel."""
    import torch
    import malkin_b200 as mk
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    from make_golden import random_rows
    rng = np.random.default_rng(0)
    for name in shapes:
        rows, cols, t = PROBE_GEMM_SHAPES[name]
        w = random_rows(rng, t, min(rows, 4096), cols)
        if rows > w.shape[0]:  # tile the seeded rows up to the full shape (the data does not change the timing)
            w = np.tile(w, (rows // w.shape[0] + 1, 1))[:rows]
        x = torch.from_numpy(rng.uniform(-3, 3, (n, cols)).astype(np.float32)).cuda()
        y = torch.zeros((n, rows), device="cuda")
        for layout in layouts:
            os.environ.pop("MALKIN_B200_Q8_LAYOUT", None)
            if layout != "auto":
                os.environ["MALKIN_B200_Q8_LAYOUT"] = layout
            W = mk.Weight(t, w, rows, cols)
            W.matmul(x.data_ptr(), n, y.data_ptr(), split_k=0)
            torch.cuda.synchronize()
            torch.cuda.profiler.start()
            for _ in range(reps):
                W.matmul(x.data_ptr(), n, y.data_ptr(), split_k=0)
            torch.cuda.synchronize()
            torch.cuda.profiler.stop()
            print(json.dumps({"probe": "gemm", "shape": name, "type": t, "layout": layout, "rows": rows, "cols": cols,
                              "n": n}))
            del W


PROBE_ATTN_SHAPES = {  # name: (requests, rows per request, prefix keys, q heads, kv heads)
    "8b": (8, 17, 2048, 32, 8), "0.6b": (1, 17, 512, 16, 8), "4b": (1, 17, 4096, 32, 8), "14b": (4, 33, 8192, 40, 8)}


def probe_attention(reps: int, shape: str = "8b") -> None:
    """Tree attention (mk_attention) at a configuration's verify shape: requests x tree rows, prefix + 1 contiguous
    keys plus each node's ancestors, D = 128, seeded int8 KV. The reps run between cudaProfilerStart / Stop."""
    import torch
    import malkin_b200 as mk
    reqs, tok, P, H, KV = PROBE_ATTN_SHAPES[shape]
    D, n_ctx = 128, P + 2 * tok + 8
    n_rows, n = reqs * n_ctx, reqs * tok
    rng = np.random.default_rng(0)
    q = torch.from_numpy(rng.standard_normal((n, H, D)).astype(np.float32)).cuda()
    k = torch.from_numpy(rng.integers(-127, 128, (KV, n_rows, D)).astype(np.int8)).cuda()
    v = torch.from_numpy(rng.integers(-127, 128, (KV, n_rows, D)).astype(np.int8)).cuda()
    ks = torch.from_numpy(rng.uniform(0.001, 0.02, (KV, n_rows)).astype(np.float32)).cuda()
    vs = torch.from_numpy(rng.uniform(0.001, 0.02, (KV, n_rows)).astype(np.float32)).cuda()
    kv_base, n_keys, anc_off, anc = [], [], [0], []
    for r in range(reqs):
        for t in range(tok):
            kv_base.append(r * n_ctx)
            n_keys.append(P + 1)
            anc += [P + 1 + 2 * i for i in range((t + 1) // 2)]
            anc_off.append(len(anc))
    ti = lambda a: torch.tensor(a, dtype=torch.int32).cuda()  # noqa: E731
    kvb, nk, ao, an = ti(kv_base), ti(n_keys), ti(anc_off), ti(anc)
    out = torch.zeros((n, H, D), device="cuda")
    torch.cuda.synchronize()
    torch.cuda.profiler.start()
    for _ in range(reps):
        mk.attention(q.data_ptr(), n, H, KV, D, k.data_ptr(), v.data_ptr(), ks.data_ptr(), vs.data_ptr(), n_rows,
                     kvb.data_ptr(), nk.data_ptr(), ao.data_ptr(), an.data_ptr(), out.data_ptr())
    torch.cuda.synchronize()
    torch.cuda.profiler.stop()
    print(json.dumps({"probe": "attention", "shape": shape, "n": n, "heads": H, "kv_heads": KV, "keys": P + 1}))


PARITY_PREFIX = {"0.6b": 512, "4b": 256, "8b": 128, "14b": 64, "32b": 64, "8b-l2": 128, "tiny": 64}


def parity_leg(mk, m, cfg, loaded, rank, world, max_batch):
    """Parity of this run's model against malkin's CPU path on a short-prefix case of the configuration's batch
    (oracle/parity.py): every rank runs the device side (collective under tensor parallelism), rank 0 the reference
    side. Returns the comparison (rank 0) or None."""
    from oracle.parity import compare, device_leg, reference_leg
    name = next(k for k, v in CONFIGS.items() if v is cfg)
    R, kk, P = cfg["requests"], cfg["kk"], PARITY_PREFIX.get(name, 64)
    try:
        d = device_leg(mk, m, R, P, kk, seed=11, max_batch=max_batch, sampled=True)
    except Exception as e:
        return {"ok": False, "error": f"device side: {e}"}
    if rank != 0:
        return None
    r, rm, _ = loaded if loaded else (None, "reference leg skipped", 0.0)
    if r is None:
        return {"ok": None, "unavailable": str(rm)}
    try:
        c = compare(d, reference_leg(r, rm, d))
    except Exception as e:
        return {"ok": False, "error": f"reference side: {e}"}
    c["case"] = (f"{R} req x {P}-token prefix (the timed run's {cfg['prompt']}), {2 * kk + 1}-row trees greedy + "
                 f"{kk + 1}-row chains sampled at temperature 0.8, tp{world}")
    return c


def sampled_variant(mk, m, cfg, nexts, P, timed, steps):
    """Times the configuration's sampled mode (temperature 0.8 rejection accept over chain-only rows) on the same
    state: drafts drawn from Dirichlet(1) weights over the target's top-8 at each chain node, seeded uniforms; every
    step consumes the same uniforms, so every step does identical work."""
    from oracle.parity import SAMPLING, chain_rows
    R, kk = cfg["requests"], cfg["kk"]
    rng = np.random.default_rng(4)
    dchain = np.zeros((R, kk), dtype=np.int64)
    qs = [[] for _ in range(R)]
    for d in range(kk):
        rows, roots = chain_rows([(s, P, nexts[s], dchain[s]) for s in range(R)], kk)
        lg = m.forward([mk.BatchToken(*r) for r in rows])
        for s in range(R):
            top = np.argsort(-lg[roots[s] + d], kind="stable")[:8]
            w = rng.dirichlet(np.ones(8)).astype(np.float32)
            qs[s].append([(float(p), int(t)) for p, t in zip(w, top)])
            cdf = np.cumsum(w.astype(np.float64))
            dchain[s, d] = int(top[min(7, int(np.searchsorted(cdf, rng.random() * cdf[-1], side="right")))])
    rows, roots = chain_rows([(s, P, nexts[s], dchain[s]) for s in range(R)], kk)
    batch = mk.make_batch(mk.BatchToken(*r) for r in rows)
    samp = mk.Sampling(**SAMPLING)
    props = [mk.Proposal(seq=s, root=roots[s], cache_len=P, chain=dchain[s], sampling=samp, q=qs[s],
                         uniforms=mk.rng_uniforms(77 + s, 2 * kk + 4)) for s in range(R)]
    for _ in range(3):
        m.verify_step(batch, props)
    res, ms, launches = timed(batch, props, profile_range=True)
    A = sum(r.n_accepted + 1 for r in res)
    ms_step = ms / steps
    return {"value": A / (ms_step / 1e3), "unit": "tok/s", "ms_per_step": ms_step, "accepted_per_step": A,
            "rows_per_step": len(rows), "gpu_launches": launches,
            "mode": "temperature 0.8 rejection accept, top_p 0.95, top_k 40, min_p 0.05, chain-only rows"}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=100)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="8b", choices=sorted(CONFIGS))
    ap.add_argument("--impl", default="malkin_b200", choices=["malkin_b200", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--probe", choices=["gemm", "attention"], help="run one kernel probe instead of the benchmark")
    ap.add_argument("--probe-shapes", default="gate+up,qkv", help="gemm probe: " + ",".join(PROBE_GEMM_SHAPES))
    ap.add_argument("--probe-layouts", default="auto", help="gemm probe: auto,tc,panels")
    ap.add_argument("--probe-n", type=int, default=136)
    ap.add_argument("--probe-reps", type=int, default=3)
    ap.add_argument("--probe-attn", default="8b", choices=["8b", "0.6b", "4b", "14b"], help="attention probe shape")
    ap.add_argument("--no-parity", action="store_true", help="skip the parity leg against malkin's CPU path")
    ap.add_argument("--write-model", metavar="CONFIG", help="write the configuration's synthetic GGUF and exit")
    args = ap.parse_args()
    if args.write_model:
        print(ensure_model(args.write_model))
        return
    if args.probe == "gemm":
        return probe_gemm(args.probe_shapes.split(","), args.probe_layouts.split(","), args.probe_n, args.probe_reps)
    if args.probe == "attention":
        return probe_attention(args.probe_reps, args.probe_attn)
    args.warmup = max(3, args.warmup)
    cfg = CONFIGS[args.config]
    if args.impl == "reference":
        return run_reference(args, cfg)

    import torch
    import torch.distributed as dist

    import malkin_b200 as mk

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE {world}")
    torch.cuda.set_device(local)
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=300))
    # model file (rank 0 writes, everyone waits)
    if rank == 0:
        path = ensure_model(args.config)
    if world > 1:
        dist.barrier()
    path = model_path(args.config)
    nid = None
    if world > 1:
        obj = [mk.nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(obj, src=0)
        nid = obj[0]
    R, P, kk = cfg["requests"], cfg["prompt"], cfg["kk"]
    rows_per_step = R * (2 * kk + 1)
    n_ctx = P + 2 * kk + 8
    max_batch = max(256, rows_per_step)
    t0 = time.perf_counter()
    m = mk.Model(local, rank, world, nid).load(path).alloc_kv(n_ctx, R, max_batch)
    load_s = time.perf_counter() - t0
    mc = m.config()
    V = mc.n_vocab
    # prefill: seeded prompts, chunks of max_batch tokens, logits for each prompt's last token
    rng = np.random.default_rng(1)
    prompts = rng.integers(0, V, (R, P))
    toks = [(int(prompts[s, i]), s, i, int(i == P - 1), -1, -1) for s in range(R) for i in range(P)]
    nexts = {}
    t0 = time.perf_counter()
    for c0 in range(0, len(toks), max_batch):
        chunk = toks[c0:c0 + max_batch]
        lg = m.forward([mk.BatchToken(*r) for r in chunk])
        j = 0
        for r in chunk:
            if r[3]:
                nexts[r[1]] = int(np.argmax(lg[j]))
                j += 1
    prefill_s = time.perf_counter() - t0
    # drafts by the 0.55 greedy-match rule: depth by depth, the target's greedy token at the chain node above
    flips, chains, alts, A_pred = draft_plan(cfg, V)
    chains = chains.copy()
    for d in range(kk):
        reqs = [(s, P, nexts[s], chains[s], alts[s]) for s in range(R)]
        rows, roots = build_tree(reqs, kk)
        lg = m.forward([mk.BatchToken(*r) for r in rows])
        for s in range(R):
            node = 0 if d == 0 else 2 * d - 1
            if flips[s, d]:
                chains[s, d] = int(np.argmax(lg[roots[s] + node]))
    reqs = [(s, P, nexts[s], chains[s], alts[s]) for s in range(R)]
    rows, roots = build_tree(reqs, kk)
    batch = mk.make_batch(mk.BatchToken(*r) for r in rows)
    props = [mk.Proposal(seq=s, root=roots[s], cache_len=P, chain=chains[s], alt=alts[s]) for s in range(R)]

    res = m.verify_step(batch, props)
    A = sum(r.n_accepted + 1 for r in res)
    for _ in range(args.warmup):
        m.verify_step(batch, props)
    stream = torch.cuda.ExternalStream(m.stream)

    def timed(b, ps, profile_range=False):
        """K steps on the library's stream between device events, after a barrier; max over ranks. profile_range:
        the steps run between cudaProfilerStart / Stop (`ncu --profile-from-start off` lists only them)."""
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        if profile_range:
            torch.cuda.profiler.start()
        n_launch = 0
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            out = m.verify_step(b, ps)
            n_launch += m.last_launch_count() + 3  # forward graph kernels + candidates, accept, move_kv
        e1.record(stream)
        e1.synchronize()
        torch.cuda.synchronize()
        if profile_range:
            torch.cuda.profiler.stop()
        if world > 1:
            dist.barrier()
        t_ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([t_ms], dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            t_ms = float(t.item())
        return out, t_ms, n_launch

    # the clock sampler starts before the first barrier (its start-up must not delay one rank's first step)
    clk = clocks_start() if rank == 0 else (None, None)
    res, ms, launches = timed(batch, props, profile_range=True)
    clocks = clocks_stop(clk, list(range(world))) if rank == 0 else None
    A_step = sum(r.n_accepted + 1 for r in res)
    ms_step = ms / args.steps
    value = A_step / (ms_step / 1e3)
    # sampled mode of the same configuration (temperature 0.8 rejection accept): chain-only rows, kk + 1 per request
    # (engine.cpp:366-378); drafts drawn from Dirichlet(1) weights over the target's top-8 at each chain node
    sampled = sampled_variant(mk, m, cfg, nexts, P, timed, args.steps)
    # e2e: the same steps through the public API from host inputs, host wall clock (inputs rebuilt every step)
    m.io_bytes()
    if world > 1:
        dist.barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        b = mk.make_batch(mk.BatchToken(*r) for r in rows)
        ps = [mk.Proposal(seq=s, root=roots[s], cache_len=P, chain=chains[s], alt=alts[s]) for s in range(R)]
        res2 = m.verify_step(b, ps)
    e2e_s = time.perf_counter() - t0
    h2d, d2h = m.io_bytes()
    if world > 1:
        t = torch.tensor([e2e_s], dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_s = float(t.item())
    # roofline: stage-profiled forwards (CUDA events per stage on the launching stream)
    m.set_profile(True)
    st = np.zeros(8)
    for _ in range(3):
        m.forward(batch, want_logits=False)
        st += np.asarray(m.stage_times())
    st /= 3
    m.set_profile(False)
    wb = weight_bytes_of(cfg)
    pk, pk_src = peaks()
    gu_bytes = wb["gate_up"] / world
    gu_gbs = gu_bytes / (st[4] / 1e3) / 1e9 if st[4] > 0 else None
    step_bytes = wb["total"] / world + (R * P + rows_per_step) * kv_bytes_per_token(cfg) / world + \
        rows_per_step * V * 4 / world
    line = {
        "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
        "scaling": "strong", "vs_baseline": None, "dtype": "int8 x int8 -> fp32 (Q8 activations, GGUF weights)",
        "data": "synthetic (seeded N(0,0.02) weights, seeded prompts and drafts)", "config": config_json(args, cfg),
        "accepted_per_step": A_step, "accepted_predicted": A_pred, "verified_rows_per_s": rows_per_step / ms_step * 1e3,
        "step_hbm_gbs": step_bytes * world / (ms_step / 1e3) / 1e9,
        "e2e": {"value": A_step * args.steps / e2e_s, "unit": "tok/s", "h2d_bytes_per_step": h2d // args.steps,
                "d2h_bytes_per_step": d2h // args.steps},
        "gpu_launches": launches,
        "roofline": {"kernel": "gate+up weight-streaming GEMM (k_gemm<Q8_0>, mma.sync panels, tuned shape)",
                     "bound": "hbm",
                     "achieved": gu_gbs, "peak": pk["hbm_gbs"], "unit": "GB/s",
                     "frac": (gu_gbs / pk["hbm_gbs"]) if gu_gbs else None, "peak_source": pk_src,
                     "traffic": profiled_traffic("gemm_q8_gate_up_8b") if args.config == "8b" and world == 1 else None,
                     "traffic_source": "profiles/gemm_q8_gate_up_8b.md (ncu, one launch at the 8B gate+up shape)",
                     "algorithmic_bytes_per_launch": gu_bytes / spec_of(cfg)["n_layer"],
                     "fp32_epilogue": fp32_floor(cfg, world, rows_per_step, st[4], clocks),
                     "stage_ms": {k: float(v) for k, v in zip(
                         ["norm+qkv", "qk-norm/rope/kv", "attention", "wo+res+norm", "gate+up", "silu+quant", "down",
                          "output"], st)}},
        "roofline_step": {"bytes_per_step": step_bytes * world, "roofline_ms": step_bytes / (pk["hbm_gbs"] * 1e9) * 1e3,
                          "frac": (step_bytes / (pk["hbm_gbs"] * 1e9)) / (ms_step / 1e3)},
        "clocks": clocks, "load_s": load_s, "prefill_s": prefill_s,
    }
    if sampled:
        line["sampled"] = sampled
    # Reference leg (after every timed region): malkin's CPU path on rank 0 times the CPU baseline (N = 1) and
    # checks parity on a short-prefix case of the same model and batch shape (every N; all ranks run the device side).
    loaded = None
    if rank == 0 and not (args.no_cpu_baseline and args.no_parity):
        try:
            loaded = reference_model(path, cfg)
        except Exception as e:  # the reference leg is reported, never fatal
            loaded = (None, str(e), 0.0)
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        try:
            base, why = cpu_baseline_sample(path, cfg, A_step, loaded=loaded)
        except Exception as e:
            base, why = None, str(e)
        line["cpu_baseline"] = base if base else {"value": None, "unit": "tok/s", "kind": "reference",
                                                  "sample": f"unavailable: {why}"}
    if not args.no_parity:
        line["parity"] = parity_leg(mk, m, cfg, loaded if rank == 0 else None, rank, world, max_batch)
        if world > 1:
            dist.barrier()  # the other ranks wait for rank 0's reference side before the communicator goes away
    if rank == 0:
        print(json.dumps(line), flush=True)
    m.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
