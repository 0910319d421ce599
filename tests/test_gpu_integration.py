"""INTEGRATION.md's C++ binding, compiled against malkin's own headers (oracle/_ref/cuda_model_test, built from
tests/cpp/cuda_model_test.cpp by oracle/Makefile) and run on a synthetic model: the GPU forward behind malkin's
BatchToken gives malkin's CPU logits bit for bit, and mk_accept's greedy walk with KV compaction gives
Engine::accept_greedy's result (the program compares both sides in one process)."""
import os
import subprocess

import pytest

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BIN = os.path.join(ROOT, "oracle", "_ref", "cuda_model_test")


def test_cpp_binding_matches_malkin(mk, ref, torch_cuda, tmp_path):
    assert os.path.exists(BIN), "oracle/_ref/cuda_model_test not built (oracle/Makefile ref target)"
    for seed, spec in ((1, dict(n_layer=2, n_embd=256, n_ff=512, n_head=4, n_head_kv=2, head_dim=64)),
                       (2, dict(n_layer=3, n_embd=512, n_ff=1024, n_head=8, n_head_kv=4, head_dim=64))):
        path = mk.synth_gguf(str(tmp_path / f"m{seed}.gguf"), n_vocab=1000, n_ctx_train=256, seed=seed, **spec)
        p = subprocess.run([BIN, path], capture_output=True, text=True, timeout=300)
        assert p.returncode == 0 and p.stdout.startswith("ok"), p.stdout + p.stderr
