"""TEST INFRASTRUCTURE ONLY: the CPU checkers of the malkin_b200 CUDA path.

`Oracle` binds liboracle.so, our plain-C restatement of malkin's verify path (malkin_oracle.c); `Ref` binds
_ref/libmalkin_ref.so, malkin's own CPU path compiled unchanged from its sources plus ref_harness.cpp. Only tests/,
__graft_entry__.smoke() and bench.py's CPU-baseline / reference arm import this package; the product never does.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from typing import Dict, List, Optional, Sequence, Tuple

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ORACLE_PATH = os.path.join(HERE, "liboracle.so")
REF_PATH = os.path.join(HERE, "_ref", "libmalkin_ref.so")

BLOCK_Q8 = np.dtype([("d", "<f4"), ("s", "<i2", (2,)), ("qs", "i1", (32,))])
assert BLOCK_Q8.itemsize == 40

_P_I32 = ctypes.POINTER(ctypes.c_int32)
_P_F32 = ctypes.POINTER(ctypes.c_float)
_P_F64 = ctypes.POINTER(ctypes.c_double)
_vp = ctypes.c_void_p


def reference_src() -> str:
    """The reference's src/ directory: $MALKIN_REF_SRC, else a checkout named `reference` beside this repository
    ("" when neither exists)."""
    env = os.environ.get("MALKIN_REF_SRC")
    if env:
        return env
    sib = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "src")
    return sib if os.path.isdir(sib) else ""


def build(ref: bool = True) -> None:
    """Compiles liboracle.so (always) and _ref (when the reference sources are found)."""
    subprocess.run(["make", "-C", HERE, os.path.join(HERE, "liboracle.so")] +
                   (["ref", f"REF={reference_src()}"] if ref else []), check=True, stdout=subprocess.DEVNULL)


def _p(a: np.ndarray, t):
    return a.ctypes.data_as(t)


class _Sampling(ctypes.Structure):
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("min_p", ctypes.c_float),
                ("top_k", ctypes.c_int)]


def _batch_arrays(batch: Sequence[Tuple]) -> List[np.ndarray]:
    """batch rows (id, seq, pos, logits, kv, parent) -> six int32 arrays."""
    a = np.asarray([tuple(int(v) for v in b) for b in batch], dtype=np.int32).reshape(-1, 6)
    return [np.ascontiguousarray(a[:, i]) for i in range(6)]


class Oracle:
    """liboracle.so: plain-C restatement (malkin_oracle.c)."""

    def __init__(self, path: str = ORACLE_PATH):
        if not os.path.exists(path):
            build(ref=False)
        L = self.lib = ctypes.CDLL(path)
        L.orc_quantize_row_q8.argtypes = [_vp, _vp, ctypes.c_int64]
        L.orc_quantize_i8.argtypes = [_vp, ctypes.c_int, _vp]
        L.orc_quantize_i8.restype = ctypes.c_float
        L.orc_dequantize_row.argtypes = [ctypes.c_int, _vp, _vp, ctypes.c_int64]
        L.orc_block_dots.argtypes = [ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int, _vp]
        L.orc_matmul.argtypes = [ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, _vp, ctypes.c_int, _vp]
        L.orc_silu_mul.argtypes = [ctypes.c_int64, _vp, _vp]
        L.orc_attend.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, ctypes.c_int64, ctypes.c_int, _vp,
                                 ctypes.c_int, ctypes.c_float, _vp]
        L.orc_model_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int]
        L.orc_model_open.restype = _vp
        L.orc_model_close.argtypes = [_vp]
        L.orc_model_cfg.argtypes = [_vp, _vp]
        L.orc_model_forward.argtypes = [_vp, ctypes.c_int] + [_vp] * 7
        L.orc_model_move_kv.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.orc_distribution.argtypes = [_vp, ctypes.c_int, _Sampling, _vp, _vp]
        L.orc_accept_greedy.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp,
                                        _vp, _vp]
        L.orc_accept_sampled.argtypes = [_vp, ctypes.c_int, _Sampling, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                         _vp]

    def quantize_row_q8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(x.size // 32, dtype=BLOCK_Q8)
        self.lib.orc_quantize_row_q8(x.ctypes.data, y.ctypes.data, x.size)
        return y

    def quantize_i8(self, x: np.ndarray) -> Tuple[np.ndarray, float]:
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.zeros(x.size, dtype=np.int8)
        d = self.lib.orc_quantize_i8(x.ctypes.data, x.size, q.ctypes.data)
        return q, d

    def dequantize_row(self, t: int, row: np.ndarray, k: int) -> np.ndarray:
        y = np.zeros(k, dtype=np.float32)
        row = np.ascontiguousarray(row, dtype=np.uint8)
        assert self.lib.orc_dequantize_row(t, row.ctypes.data, y.ctypes.data, k) == 0
        return y

    def block_dots(self, t: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        n = x.shape[0]
        xq = np.concatenate([self.quantize_row_q8(r) for r in x])
        nblk = cols // 32 * (2 if t == 14 else 1)
        out = np.zeros((rows, n, nblk), dtype=np.int32)
        self.lib.orc_block_dots(t, np.ascontiguousarray(w).ctypes.data, rows, cols, xq.ctypes.data, n, out.ctypes.data)
        return out

    def matmul(self, t: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        y = np.zeros((x.shape[0], rows), dtype=np.float32)
        self.lib.orc_matmul(t, np.ascontiguousarray(w).ctypes.data, rows, cols, x.ctypes.data, x.shape[0],
                            y.ctypes.data)
        return y

    def silu_mul(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.array(g, dtype=np.float32)
        u = np.ascontiguousarray(u, dtype=np.float32)
        self.lib.orc_silu_mul(g.size, g.ctypes.data, u.ctypes.data)
        return g

    def attend(self, q, G, D, k, v, ks, vs, n, extra, scale) -> np.ndarray:
        """One token, G heads of one KV head: k / v int8 [rows, D], ks / vs float [rows]."""
        q = np.ascontiguousarray(q, dtype=np.float32)
        extra = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
        out = np.zeros(G * D, dtype=np.float32)
        k, v = np.ascontiguousarray(k, dtype=np.int8), np.ascontiguousarray(v, dtype=np.int8)
        ks, vs = np.ascontiguousarray(ks, dtype=np.float32), np.ascontiguousarray(vs, dtype=np.float32)
        self.lib.orc_attend(q.ctypes.data, G, D, k.ctypes.data, v.ctypes.data, ks.ctypes.data, vs.ctypes.data, D, n,
                            extra.ctypes.data if extra.size else None, int(extra.size), scale, out.ctypes.data)
        return out

    def distribution(self, logits: np.ndarray, temperature=0.8, top_p=0.95, top_k=40, min_p=0.05):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        V = logits.size
        cap = top_k if 0 < top_k < V else V
        p = np.zeros(cap, dtype=np.float32)
        ids = np.zeros(cap, dtype=np.int32)
        n = self.lib.orc_distribution(logits.ctypes.data, V, _Sampling(temperature, top_p, min_p, top_k),
                                      p.ctypes.data, ids.ctypes.data)
        return p[:n], ids[:n]

    def accept_greedy(self, logits: np.ndarray, chain, alt, model: Optional["OracleModel"] = None, seq=0,
                      cache_len=0):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        chain = np.asarray(chain, dtype=np.int32)
        alt = np.asarray(alt, dtype=np.int32)
        acc = np.zeros(max(1, len(chain)), dtype=np.int32)
        nxt, last = ctypes.c_int32(), ctypes.c_int32()
        n = self.lib.orc_accept_greedy(model.h if model else None, logits.ctypes.data, logits.shape[-1], len(chain),
                                       chain.ctypes.data, alt.ctypes.data, seq, cache_len, acc.ctypes.data,
                                       ctypes.byref(nxt), ctypes.byref(last))
        return list(acc[:n]), nxt.value, last.value

    def accept_sampled(self, logits: np.ndarray, chain, q, uniforms, temperature=0.8, top_p=0.95, top_k=40,
                       min_p=0.05):
        logits = np.ascontiguousarray(logits, dtype=np.float32)
        chain = np.asarray(chain, dtype=np.int32)
        q_n = np.asarray([len(d) for d in q], dtype=np.int32)
        q_p = np.asarray([p for d in q for (p, _) in d] or [0], dtype=np.float32)
        q_id = np.asarray([i for d in q for (_, i) in d] or [0], dtype=np.int32)
        U = np.ascontiguousarray(uniforms, dtype=np.float64)
        acc = np.zeros(max(1, len(chain)), dtype=np.int32)
        nxt, used = ctypes.c_int32(), ctypes.c_int32()
        n = self.lib.orc_accept_sampled(logits.ctypes.data, logits.shape[-1],
                                        _Sampling(temperature, top_p, min_p, top_k), len(chain), chain.ctypes.data,
                                        q_p.ctypes.data, q_id.ctypes.data, q_n.ctypes.data, U.ctypes.data,
                                        acc.ctypes.data, ctypes.byref(nxt), ctypes.byref(used))
        return list(acc[:n]), nxt.value, used.value


class OracleModel:
    """Model on the C oracle (orc_model_*)."""

    def __init__(self, oracle: Oracle, path: str, n_ctx: int, n_seq: int = 1):
        self.o = oracle
        self.h = oracle.lib.orc_model_open(path.encode(), n_ctx, n_seq)
        if not self.h:
            raise RuntimeError(f"oracle: cannot load {path}")
        c = np.zeros(9, dtype=np.int32)
        oracle.lib.orc_model_cfg(self.h, c.ctypes.data)
        (self.n_layer, self.n_embd, self.n_ff, self.n_head, self.n_head_kv, self.head_dim, self.n_vocab, self.n_ctx,
         self.n_seq) = map(int, c)

    def __del__(self):
        if getattr(self, "h", None):
            self.o.lib.orc_model_close(self.h)
            self.h = None

    def forward(self, batch: Sequence[Tuple]) -> np.ndarray:
        arrs = _batch_arrays(batch)
        m = int(arrs[3].astype(bool).sum())
        out = np.zeros((max(m, 1), self.n_vocab), dtype=np.float32)
        rc = self.o.lib.orc_model_forward(self.h, len(batch), *[a.ctypes.data for a in arrs], out.ctypes.data)
        if rc != 0:
            raise ValueError("oracle: batch rejected")
        return out[:m]

    def move_kv(self, frm: int, to: int, seq: int = 0) -> None:
        self.o.lib.orc_model_move_kv(self.h, frm, to, seq)


class Ref:
    """_ref/libmalkin_ref.so: malkin's own CPU path (needs an AVX-512 VNNI / BF16 host to run)."""

    def __init__(self, path: str = REF_PATH):
        if not os.path.exists(path):
            raise FileNotFoundError(path)
        L = self.lib = ctypes.CDLL(path)
        L.ref_missing_features.restype = ctypes.c_char_p
        missing = L.ref_missing_features().decode()
        if missing:
            raise RuntimeError(f"reference CPU path needs {missing}")
        L.ref_physical_cores.restype = ctypes.c_int
        L.ref_set_threads.argtypes = [ctypes.c_int]
        L.ref_model_open.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_char_p,
                                     ctypes.c_int]
        L.ref_model_open.restype = _vp
        L.ref_model_close.argtypes = [_vp]
        L.ref_model_cfg.argtypes = [_vp, _vp, _vp]
        L.ref_model_forward.argtypes = [_vp, ctypes.c_int] + [_vp] * 7 + [ctypes.c_char_p, ctypes.c_int]
        L.ref_model_move_kv.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
        L.ref_quantize_row_q8.argtypes = [_vp, _vp, ctypes.c_int64]
        L.ref_quantize_i8.argtypes = [_vp, ctypes.c_int, _vp]
        L.ref_quantize_i8.restype = ctypes.c_float
        L.ref_dequantize_row.argtypes = [ctypes.c_int, _vp, _vp, ctypes.c_int64]
        L.ref_matmul.argtypes = [ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.c_int, _vp, ctypes.c_int, _vp]
        L.ref_attend_gqa.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int64, ctypes.c_int64,
                                     ctypes.c_int, ctypes.c_float, _vp, _vp, ctypes.c_int]
        L.ref_silu_mul.argtypes = [ctypes.c_int64, _vp, _vp]
        L.ref_uniforms.argtypes = [ctypes.c_uint64, ctypes.c_int, _vp]
        L.ref_sampler_new.argtypes = [ctypes.c_float, ctypes.c_float, ctypes.c_int, ctypes.c_float, ctypes.c_float,
                                      ctypes.c_float, ctypes.c_uint64]
        L.ref_sampler_new.restype = _vp
        L.ref_sampler_free.argtypes = [_vp]
        L.ref_sampler_distribution.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp, ctypes.c_int]
        L.ref_accept_greedy.argtypes = [_vp, _vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_int, _vp, _vp,
                                        _vp, _vp, ctypes.c_int]
        L.ref_accept_sampled.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp, _vp, _vp, _vp,
                                         ctypes.c_int]
        L.ref_engine_open.argtypes = [ctypes.c_char_p, ctypes.c_char_p] + [ctypes.c_int] * 4 + [ctypes.c_char_p,
                                                                                                ctypes.c_int]
        L.ref_engine_open.restype = _vp
        L.ref_engine_close.argtypes = [_vp]
        L.ref_engine_generate.argtypes = [_vp, ctypes.c_int, ctypes.c_int] + [_vp] * 5 + [ctypes.c_int] + [_vp] * 3 + [
            ctypes.c_char_p, ctypes.c_int]
        L.ref_engine_perplexity.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, _vp, _vp, ctypes.c_char_p,
                                            ctypes.c_int]

    @staticmethod
    def available() -> Optional[str]:
        """None when the reference library loads and runs here, else the reason."""
        try:
            Ref()
            return None
        except Exception as e:  # missing build or ISA
            return str(e)

    def set_threads(self, n: int) -> None:
        self.lib.ref_set_threads(n)

    def physical_cores(self) -> int:
        return int(self.lib.ref_physical_cores())

    def quantize_row_q8(self, x: np.ndarray) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32)
        y = np.zeros(x.size // 32, dtype=BLOCK_Q8)
        self.lib.ref_quantize_row_q8(x.ctypes.data, y.ctypes.data, x.size)
        return y

    def quantize_i8(self, x: np.ndarray):
        x = np.ascontiguousarray(x, dtype=np.float32)
        q = np.zeros(x.size, dtype=np.int8)
        d = self.lib.ref_quantize_i8(x.ctypes.data, x.size, q.ctypes.data)
        return q, d

    def dequantize_row(self, t: int, row: np.ndarray, k: int) -> np.ndarray:
        y = np.zeros(k, dtype=np.float32)
        row = np.ascontiguousarray(row, dtype=np.uint8)
        assert self.lib.ref_dequantize_row(t, row.ctypes.data, y.ctypes.data, k) == 0
        return y

    def matmul(self, t: int, w: np.ndarray, rows: int, cols: int, x: np.ndarray, mode: int = 1) -> np.ndarray:
        x = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, cols)
        y = np.zeros((x.shape[0], rows), dtype=np.float32)
        assert self.lib.ref_matmul(t, np.ascontiguousarray(w).ctypes.data, rows, cols, mode, x.ctypes.data, x.shape[0],
                                   y.ctypes.data) == 0
        return y

    def silu_mul(self, g: np.ndarray, u: np.ndarray) -> np.ndarray:
        g = np.array(g, dtype=np.float32)
        u = np.ascontiguousarray(u, dtype=np.float32)
        self.lib.ref_silu_mul(g.size, g.ctypes.data, u.ctypes.data)
        return g

    def attend(self, q, G, D, k, v, ks, vs, n, extra, scale) -> np.ndarray:
        """Same call as Oracle.attend: packs rows in malkin's KV layout (D int8 values then the float scale)."""
        rows = k.shape[0]
        stride = D + 8  # one head: D values, then 4 pad bytes, then the scale at D + 4 (soff = D + 4)
        kb = np.zeros((rows, stride), dtype=np.int8)
        vb = np.zeros((rows, stride), dtype=np.int8)
        kb[:, :D] = k
        vb[:, :D] = v
        kb[:, D + 4:D + 8] = np.asarray(ks, dtype=np.float32).view(np.int8).reshape(rows, 4)
        vb[:, D + 4:D + 8] = np.asarray(vs, dtype=np.float32).view(np.int8).reshape(rows, 4)
        q = np.ascontiguousarray(q, dtype=np.float32)
        extra = np.ascontiguousarray(np.asarray(extra, dtype=np.int32))
        out = np.zeros(G * D, dtype=np.float32)
        self.lib.ref_attend_gqa(q.ctypes.data, G, D, kb.ctypes.data, vb.ctypes.data, stride, D + 4, n, scale,
                                out.ctypes.data, extra.ctypes.data if extra.size else None, int(extra.size))
        return out

    def uniforms(self, seed: int, n: int) -> np.ndarray:
        out = np.zeros(n, dtype=np.float64)
        self.lib.ref_uniforms(seed, n, out.ctypes.data)
        return out

    def sampler(self, temperature=0.8, top_p=0.95, top_k=40, min_p=0.05, seed=1) -> int:
        return self.lib.ref_sampler_new(temperature, top_p, top_k, min_p, 0.0, 0.0, seed)

    def free_sampler(self, s: int) -> None:
        self.lib.ref_sampler_free(s)

    def distribution(self, sampler: int, logits: np.ndarray):
        logits = np.array(logits, dtype=np.float32)
        cap = logits.size
        p = np.zeros(cap, dtype=np.float32)
        ids = np.zeros(cap, dtype=np.int32)
        n = self.lib.ref_sampler_distribution(sampler, logits.ctypes.data, logits.size, p.ctypes.data, ids.ctypes.data,
                                              cap)
        return p[:n], ids[:n]

    def accept_greedy(self, sampler: int, logits: np.ndarray, chain, alt, model: Optional["RefModel"] = None, seq=0,
                      cache_len=0, k=8, n_draft=8):
        logits = np.array(logits, dtype=np.float32)
        chain = np.asarray(chain, dtype=np.int32)
        alt = np.asarray(alt, dtype=np.int32)
        acc = np.zeros(max(1, len(chain)), dtype=np.int32)
        cl, nx, kk = ctypes.c_int(cache_len), ctypes.c_int32(), ctypes.c_int(k)
        n = self.lib.ref_accept_greedy(model.h if model else None, sampler, logits.ctypes.data, logits.shape[-1],
                                       len(chain), chain.ctypes.data, alt.ctypes.data, seq, ctypes.byref(cl),
                                       acc.ctypes.data, ctypes.byref(nx), ctypes.byref(kk), n_draft)
        return list(acc[:n]), nx.value, cl.value

    def accept_sampled(self, sampler: int, logits: np.ndarray, chain, q, k=8, n_draft=8):
        logits = np.array(logits, dtype=np.float32)
        chain = np.asarray(chain, dtype=np.int32)
        q_n = np.asarray([len(d) for d in q] or [0], dtype=np.int32)
        q_p = np.asarray([p for d in q for (p, _) in d] or [0], dtype=np.float32)
        q_id = np.asarray([i for d in q for (_, i) in d] or [0], dtype=np.int32)
        acc = np.zeros(max(1, len(chain)), dtype=np.int32)
        nx, kk = ctypes.c_int32(), ctypes.c_int(k)
        n = self.lib.ref_accept_sampled(sampler, logits.ctypes.data, logits.shape[-1], len(chain), chain.ctypes.data,
                                        q_p.ctypes.data, q_id.ctypes.data, q_n.ctypes.data, acc.ctypes.data,
                                        ctypes.byref(nx), ctypes.byref(kk), n_draft)
        return list(acc[:n]), nx.value


class RefModel:
    """malkin::Model through the reference library."""

    def __init__(self, ref: Ref, path: str, n_ctx: int, n_seq: int = 1, wide: bool = False):
        self.r = ref
        err = ctypes.create_string_buffer(512)
        self.h = ref.lib.ref_model_open(path.encode(), n_ctx, n_seq, int(wide), err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())
        c = np.zeros(9, dtype=np.int32)
        f = np.zeros(2, dtype=np.float32)
        ref.lib.ref_model_cfg(self.h, c.ctypes.data, f.ctypes.data)
        (self.n_layer, self.n_embd, self.n_ff, self.n_head, self.n_head_kv, self.head_dim, self.n_vocab, self.n_ctx,
         self.n_seq) = map(int, c)

    def __del__(self):
        if getattr(self, "h", None):
            self.r.lib.ref_model_close(self.h)
            self.h = None

    def forward(self, batch: Sequence[Tuple]) -> np.ndarray:
        arrs = _batch_arrays(batch)
        m = int(arrs[3].astype(bool).sum())
        out = np.zeros((max(m, 1), self.n_vocab), dtype=np.float32)
        err = ctypes.create_string_buffer(512)
        rc = self.r.lib.ref_model_forward(self.h, len(batch), *[a.ctypes.data for a in arrs], out.ctypes.data, err,
                                          512)
        if rc != 0:
            raise ValueError(err.value.decode())
        return out[:m]

    def move_kv(self, frm: int, to: int, seq: int = 0) -> None:
        self.r.lib.ref_model_move_kv(self.h, frm, to, seq)


class RefEngine:
    """malkin::Engine (engine.cpp) through the reference library: continuous batching, the draft model's
    speculative trees / chains, adaptive draft length, perplexity. Token i's text is "<ti>" (the synthetic models'
    vocabulary), so generated text reads back as token ids."""

    def __init__(self, ref: Ref, path: str, n_ctx: int, parallel: int = 1, draft: Optional[str] = None,
                 n_draft: int = 0, threads: int = 0):
        self.r = ref
        err = ctypes.create_string_buffer(512)
        self.h = ref.lib.ref_engine_open(path.encode(), draft.encode() if draft else None, n_ctx, parallel, n_draft,
                                         threads, err, 512)
        if not self.h:
            raise RuntimeError(err.value.decode())

    def __del__(self):
        if getattr(self, "h", None):
            self.r.lib.ref_engine_close(self.h)
            self.h = None

    def generate(self, requests: Sequence[Dict], sequential: bool = False, cap: int = 4096):
        """requests: dicts with prompt, max_tokens, and optionally temperature, top_p, top_k, min_p, seed (greedy
        by default). Returns [(tokens, stats)] with stats = (prompt, cached, completion, drafted, accepted, finish)."""
        n = len(requests)
        prompts = np.concatenate([np.asarray(q["prompt"], dtype=np.int32) for q in requests])
        plen = np.array([len(q["prompt"]) for q in requests], dtype=np.int32)
        mt = np.array([q.get("max_tokens", 0) for q in requests], dtype=np.int32)
        smp = np.array([[q.get("temperature", 0.0), q.get("top_p", 0.95), q.get("top_k", 40), q.get("min_p", 0.05)]
                        for q in requests], dtype=np.float32)
        seeds = np.array([q.get("seed", 1) for q in requests], dtype=np.uint64)
        out = np.zeros((n, cap), dtype=np.int32)
        out_n = np.zeros(n, dtype=np.int32)
        st = np.zeros((n, 6), dtype=np.int32)
        err = ctypes.create_string_buffer(512)
        rc = self.r.lib.ref_engine_generate(self.h, n, int(sequential), prompts.ctypes.data, plen.ctypes.data,
                                            mt.ctypes.data, smp.ctypes.data, seeds.ctypes.data, cap, out.ctypes.data,
                                            out_n.ctypes.data, st.ctypes.data, err, 512)
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return [(out[i, :out_n[i]].tolist(), tuple(int(x) for x in st[i])) for i in range(n)]

    def perplexity(self, tokens: Sequence[int], window: int):
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nll = ctypes.c_double()
        scored = ctypes.c_int()
        err = ctypes.create_string_buffer(512)
        rc = self.r.lib.ref_engine_perplexity(self.h, t.ctypes.data, len(t), window, ctypes.byref(nll),
                                              ctypes.byref(scored), err, 512)
        if rc != 0:
            raise RuntimeError(err.value.decode())
        return nll.value, scored.value
