"""The C ABI library without a GPU: it loads, exports every entry point include/malkin_b200.h declares, its host-only
entry points work, and calls that need a device fail with a status code instead of crashing."""
import ctypes
import os
import re

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def header_functions():
    src = open(os.path.join(ROOT, "include", "malkin_b200.h")).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mk_[a-z0-9_]+)\s*\(", src)))


def test_exports_every_declared_symbol(mk):
    names = header_functions()
    assert len(names) >= 25
    for n in names:
        assert hasattr(mk.lib, n), f"libmalkin_b200.so does not export {n}"
    assert set(names) == set(mk.EXPORTS)


def test_version_and_error(mk):
    assert "sm_100a" in mk.version()
    assert mk.lib.mk_last_error() is not None


def test_rng_stream_matches_golden(mk, golden):
    assert np.array_equal(mk.rng_uniforms(int(golden["rng_seed"][0]), 64), golden["rng_u"])
    # skip = consuming a prefix
    assert np.array_equal(mk.rng_uniforms(1234, 10, skip=5), golden["rng_u"][5:15])


def test_synth_is_deterministic_and_loadable(mk, tmp_path, oracle):
    a = mk.synth_gguf(str(tmp_path / "a.gguf"), n_layer=1, n_embd=256, n_ff=256, n_head=2, n_head_kv=1, n_vocab=300,
                      seed=9, n_threads=1)
    b = mk.synth_gguf(str(tmp_path / "b.gguf"), n_layer=1, n_embd=256, n_ff=256, n_head=2, n_head_kv=1, n_vocab=300,
                      seed=9, n_threads=7)
    assert open(a, "rb").read() == open(b, "rb").read()
    from oracle import OracleModel
    m = OracleModel(oracle, a, 16, 1)
    assert (m.n_layer, m.n_embd, m.n_vocab, m.head_dim) == (1, 256, 300, 128)


def gguf_tensors(path):
    """Minimal GGUF v3 walker (test-side, independent of the library's reader): {name: (type, ne, bytes)}."""
    import struct
    data = open(path, "rb").read()
    pos = 0

    def take(fmt):
        nonlocal pos
        v = struct.unpack_from("<" + fmt, data, pos)
        pos += struct.calcsize("<" + fmt)
        return v[0] if len(v) == 1 else v

    def text():
        nonlocal pos
        n = take("Q")
        s = data[pos:pos + n].decode()
        pos += n
        return s

    width = {0: 1, 1: 1, 2: 2, 3: 2, 4: 4, 5: 4, 6: 4, 7: 1, 10: 8, 11: 8, 12: 8}
    magic, version, n_t, n_kv = take("I"), take("I"), take("Q"), take("Q")
    assert magic == 0x46554747 and version == 3
    align = 32
    for _ in range(n_kv):
        key, t = text(), take("I")
        if t == 8:
            text()
        elif t == 9:
            et, cnt = take("I"), take("Q")
            for _ in range(cnt):
                text() if et == 8 else take({1: "B", 4: "I", 5: "i", 6: "f"}.get(et, "Q"))
        else:
            v = struct.unpack_from("<" + {1: "B", 2: "H", 4: "I", 5: "i", 6: "f", 7: "B", 10: "Q"}.get(t, "B"), data,
                                   pos)[0]
            pos += width[t]
            if key == "general.alignment":
                align = v
    infos = []
    for _ in range(n_t):
        name, nd = text(), take("I")
        ne = [take("Q") for _ in range(nd)]
        infos.append((name, ne, take("I"), take("Q")))
    start = (pos + align - 1) // align * align
    from malkin_b200 import row_bytes
    out = {}
    for name, ne, t, off in infos:
        nb = row_bytes(t, ne[0]) * int(np.prod(ne[1:], dtype=np.int64))
        out[name] = (t, ne, data[start + off:start + off + nb])
    return out


def test_synth_quantizers_roundtrip(mk, tmp_path, oracle):
    """The writer's Q8_0 / Q4_K / Q6_K rows, dequantized by the oracle's restatement of malkin's dequantize_row
    (quant.cpp:70-128), have the statistics of the N(0, sigma) draws they were quantized from: mean within 4 standard
    errors of 0 and standard deviation within 2 % (Q8_0, Q6_K) / 4 % (Q4_K) of sigma = 0.02."""
    sigma = 0.02
    for t, tol in ((mk.TYPE_Q8_0, 0.02), (mk.TYPE_Q4_K, 0.04), (mk.TYPE_Q6_K, 0.02)):
        p = mk.synth_gguf(str(tmp_path / f"t{t}.gguf"), n_layer=1, n_embd=512, n_ff=512, n_head=2, n_head_kv=1,
                          n_vocab=300, type_default=t, seed=1)
        typ, ne, raw = gguf_tensors(p)["token_embd.weight"]
        assert typ == t and ne == [512, 300]
        rb = mk.row_bytes(t, 512)
        vals = np.concatenate([oracle.dequantize_row(t, np.frombuffer(raw[r * rb:(r + 1) * rb], np.uint8), 512)
                               for r in range(300)]).astype(np.float64)
        se = sigma / np.sqrt(vals.size)
        assert abs(vals.mean()) < 4 * se, (t, vals.mean())
        assert abs(vals.std() / sigma - 1) < tol, (t, vals.std())
        # no degenerate blocks: every row has spread, and values use the type's range
        assert np.all(vals.reshape(300, 512).std(axis=1) > 0.5 * sigma)


def test_gguf_reader_rejects_malformed_files(mk, tmp_path):
    """The library's GGUF reader (the one mk_load_gguf uses) fails with MK_ERR_ARG and a 'gguf:' message on a bad
    magic, a truncated header, an unsupported version and a tensor that points past the end of the file."""
    good = mk.synth_gguf(str(tmp_path / "g.gguf"), n_layer=1, n_embd=256, n_ff=256, n_head=2, n_head_kv=1,
                         n_vocab=300, seed=3)
    assert mk.tp_shard_of(good, 1, 0).ffn == 256
    data = open(good, "rb").read()
    cases = {
        "magic": b"GGUX" + data[4:],
        "truncated": data[:200],
        "version": data[:4] + (2).to_bytes(4, "little") + data[8:],
        "data": data[:-4096],
    }
    for name, blob in cases.items():
        p = tmp_path / f"{name}.gguf"
        p.write_bytes(blob)
        with __import__("pytest").raises(mk.MalkinError) as e:
            mk.tp_shard_of(str(p), 1, 0)
        assert e.value.code == mk.MK_ERR_ARG and "gguf:" in str(e.value), (name, str(e.value))


def test_device_calls_fail_cleanly_without_gpu(mk):
    import torch
    if torch.cuda.is_available():
        return
    h = ctypes.c_void_p()
    rc = mk.lib.mk_init(0, 0, 1, None, ctypes.byref(h))
    assert rc == mk.MK_ERR_CUDA and mk.lib.mk_last_error()
    # null context: state error, no crash
    assert mk.lib.mk_forward(None, None, 0, None) in (mk.MK_ERR_STATE, mk.MK_ERR_ARG)
