"""Parity at the benchmark configurations' model shapes: the sm_100a path through the C ABI against malkin's own CPU
path (oracle/_ref, run on the GPU box's host cores) on the same seeded GGUF and the same inputs (oracle/parity.py):
logits bit-identical (every float operation in malkin's order; the north star's bound is max-abs <= 2e-2), greedy
accepted paths identical, sampled (temperature 0.8) accept decisions identical given the same uniforms.

Shapes (full vocabulary 151936, full layer counts, the configurations' weight types):
  0.6b  Qwen3-0.6B Q8_0, 1 request, 512-token prompt, one 17-row tree and one 9-row sampled chain (configuration 1
        in full);
  4b    Qwen3-4B Q4_K_M-style (Q4_K, Q6_K for attn_v / ffn_down / output), 1 request, 256-token prefix (the
        configuration's 4096 is shortened so malkin's CPU prefill stays within seconds), one 17-row tree;
  8b    Qwen3-8B Q8_0, 8 requests x 128-token prefix (2048 shortened), 136 tree rows and 72 sampled chain rows;
  14b   Qwen3-14B Q6_K, 4 requests x 64-token prefix (8192 shortened), 33-row trees (kk = 16).
The per-step work that does not depend on the prefix (every weight GEMM, the LM head, accept) is the
configuration's; the attention reads fewer keys."""
import os
import sys

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

CASES = {
    "0.6b": dict(requests=1, prefix=512, kk=8, sampled=True),
    "4b": dict(requests=1, prefix=256, kk=8, sampled=False),
    "8b": dict(requests=8, prefix=128, kk=8, sampled=True),
    "14b": dict(requests=4, prefix=64, kk=16, sampled=False),
}


@pytest.mark.parametrize("name", list(CASES))
def test_parity_at_config_shape(mk, ref, torch_cuda, name):
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    import bench
    from oracle import RefModel
    from oracle.parity import compare, device_leg, reference_leg
    case = CASES[name]
    path = bench.ensure_model(name)
    R, P, kk = case["requests"], case["prefix"], case["kk"]
    n_ctx = P + 2 * kk + 8
    m = mk.Model(0).load(path).alloc_kv(n_ctx, R, 256)
    try:
        d = device_leg(mk, m, R, P, kk, seed=1, sampled=case["sampled"])
    finally:
        m.close()
    ref.set_threads(ref.physical_cores())
    r = reference_leg(ref, RefModel(ref, path, n_ctx, R), d)
    c = compare(d, r)
    print(name, c)
    assert c["max_abs_logits"] == 0.0, c
    assert c["greedy_ok"] and c["greedy_compared"] == R, c
    if case["sampled"]:
        assert c["sampled_ok"] and c["sampled_identical_ref_logits"] == R, c
