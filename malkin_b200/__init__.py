"""malkin_b200 — B200-native (sm_100a) speculative-verify path of kekzl/malkin.

Python mirror of the C ABI in include/malkin_b200.h (ctypes over the in-tree libmalkin_b200.so). The names follow
malkin's C++ API: Model(load GGUF, alloc_kv, forward(BatchToken batch), move_kv), the engine's accept step, and the
Sampler's uniform stream. Importing fails loudly when the CUDA library has not been built: there is no CPU
fallback on this path.
"""
from __future__ import annotations

import ctypes
import os
from typing import Dict, Iterable, List, Optional, Sequence, Tuple

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmalkin_b200.so")

if not os.path.exists(LIB_PATH):
    raise ImportError(
        f"{LIB_PATH} is missing: build it with `make -C malkin_b200/csrc` (or __graft_entry__.build())")
lib = ctypes.CDLL(LIB_PATH)

MK_OK = 0
MK_ERR_ARG = -1
MK_ERR_CUDA = -2
MK_ERR_NCCL = -3
MK_ERR_UNSUPPORTED = -4
MK_ERR_STATE = -5
MK_ERR_IO = -6
MK_ERR_TIMEOUT = -7

TYPE_F32, TYPE_F16, TYPE_Q8_0, TYPE_Q4_K, TYPE_Q6_K, TYPE_BF16 = 0, 1, 8, 12, 14, 30
MAX_DRAFT = 32
MAX_TOPK = 64

# ggml block geometry (elements, bytes) per type
BLOCK = {TYPE_F32: (1, 4), TYPE_F16: (1, 2), TYPE_BF16: (1, 2), TYPE_Q8_0: (32, 34), TYPE_Q4_K: (256, 144),
         TYPE_Q6_K: (256, 210)}


def row_bytes(t: int, n: int) -> int:
    b, s = BLOCK[t]
    assert n % b == 0
    return n // b * s


class MalkinError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"[{code}] {msg}")
        self.code = code


def _check(rc: int) -> None:
    if rc != MK_OK:
        raise MalkinError(rc, lib.mk_last_error().decode())


# ---- C structs ----
class SynthSpec(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_vocab", "n_ctx_train")] + [
        ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float), ("tied", ctypes.c_int32),
        ("type_default", ctypes.c_int32), ("type_attn_v", ctypes.c_int32), ("type_ffn_down", ctypes.c_int32),
        ("type_output", ctypes.c_int32), ("type_embd", ctypes.c_int32), ("sigma", ctypes.c_float),
        ("seed", ctypes.c_uint64), ("has_eos", ctypes.c_int32), ("eos_token_id", ctypes.c_int32)]


class BatchToken(ctypes.Structure):
    """malkin::BatchToken (model.h:25-30)."""
    _fields_ = [("id", ctypes.c_int32), ("seq", ctypes.c_int32), ("pos", ctypes.c_int32), ("logits", ctypes.c_bool),
                ("kv", ctypes.c_int32), ("parent", ctypes.c_int32)]

    def __init__(self, id=0, seq=0, pos=0, logits=False, kv=-1, parent=-1):
        super().__init__(id, seq, pos, logits, kv, parent)


assert ctypes.sizeof(BatchToken) == 24


class ModelConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_int32) for n in
                ("n_layer", "n_embd", "n_ff", "n_head", "n_head_kv", "head_dim", "n_ctx_train", "n_vocab")] + [
        ("rope_base", ctypes.c_float), ("rms_eps", ctypes.c_float), ("n_ctx", ctypes.c_int32),
        ("n_seq", ctypes.c_int32), ("tp_rank", ctypes.c_int32), ("tp_size", ctypes.c_int32),
        ("weight_bytes", ctypes.c_int64)]


class Sampling(ctypes.Structure):
    """SamplingParams (sampler.h:10-18); penalties must be 0."""
    _fields_ = [("temperature", ctypes.c_float), ("top_p", ctypes.c_float), ("top_k", ctypes.c_int32),
                ("min_p", ctypes.c_float), ("presence_penalty", ctypes.c_float),
                ("frequency_penalty", ctypes.c_float)]

    def __init__(self, temperature=0.8, top_p=0.95, top_k=40, min_p=0.05, presence_penalty=0.0,
                 frequency_penalty=0.0):
        super().__init__(temperature, top_p, top_k, min_p, presence_penalty, frequency_penalty)


_P_I32 = ctypes.POINTER(ctypes.c_int32)
_P_F32 = ctypes.POINTER(ctypes.c_float)
_P_F64 = ctypes.POINTER(ctypes.c_double)


class _Proposal(ctypes.Structure):
    _fields_ = [("seq", ctypes.c_int32), ("kk", ctypes.c_int32), ("root", ctypes.c_int32),
                ("cache_len", ctypes.c_int32), ("sampling", Sampling), ("chain", _P_I32), ("alt", _P_I32),
                ("q_p", _P_F32), ("q_id", _P_I32), ("q_n", _P_I32), ("uniforms", _P_F64),
                ("n_uniforms", ctypes.c_int32)]


class AcceptResult(ctypes.Structure):
    _fields_ = [("n_accepted", ctypes.c_int32), ("accepted", ctypes.c_int32 * MAX_DRAFT), ("next", ctypes.c_int32),
                ("cache_len", ctypes.c_int32), ("uniforms_used", ctypes.c_int32), ("last_node", ctypes.c_int32)]

    @property
    def ids(self) -> List[int]:
        return list(self.accepted[: self.n_accepted])


class Proposal:
    """One decoding slot's proposal (engine.h:126-131). Greedy: tree [next, c0, a0, c1, a1, ...] from batch index
    root; sampled (temperature > 0): chain [next, d0, ...] with draft distributions q and the slot's uniforms."""

    def __init__(self, seq: int, root: int, cache_len: int, chain: Sequence[int] = (),
                 alt: Optional[Sequence[int]] = None, sampling: Optional[Sampling] = None,
                 q: Optional[Sequence[Sequence[tuple]]] = None, uniforms: Optional[Sequence[float]] = None):
        self.sampling = sampling or Sampling(temperature=0.0)
        self.seq, self.root, self.cache_len = seq, root, cache_len
        self.chain = np.ascontiguousarray(np.asarray(chain, dtype=np.int32).reshape(-1))
        self.alt = np.ascontiguousarray(np.asarray(alt if alt is not None else [-1] * len(self.chain), dtype=np.int32))
        q = q or []
        self.q_n = np.asarray([len(d) for d in q], dtype=np.int32)
        self.q_p = np.asarray([p for d in q for (p, _) in d], dtype=np.float32)
        self.q_id = np.asarray([i for d in q for (_, i) in d], dtype=np.int32)
        self.uniforms = np.asarray(uniforms if uniforms is not None else [], dtype=np.float64)

    def _c(self) -> _Proposal:
        def ptr(a, t):
            return a.ctypes.data_as(t) if a.size else ctypes.cast(None, t)
        return _Proposal(self.seq, len(self.chain), self.root, self.cache_len, self.sampling,
                         ptr(self.chain, _P_I32), ptr(self.alt, _P_I32), ptr(self.q_p, _P_F32),
                         ptr(self.q_id, _P_I32), ptr(self.q_n, _P_I32), ptr(self.uniforms, _P_F64),
                         int(self.uniforms.size))


# ---- signatures ----
_vp = ctypes.c_void_p
lib.mk_last_error.restype = ctypes.c_char_p
lib.mk_version.restype = ctypes.c_char_p
lib.mk_synth_gguf.argtypes = [ctypes.c_char_p, ctypes.POINTER(SynthSpec), ctypes.c_int]
lib.mk_nccl_unique_id.argtypes = [_vp]
lib.mk_init.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, ctypes.POINTER(_vp)]
lib.mk_shutdown.argtypes = [_vp]
lib.mk_load_gguf.argtypes = [_vp, ctypes.c_char_p]
lib.mk_alloc_kv.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
lib.mk_model_config_get.argtypes = [_vp, ctypes.POINTER(ModelConfig)]
lib.mk_forward.argtypes = [_vp, ctypes.POINTER(BatchToken), ctypes.c_int, _P_F32]
lib.mk_move_kv.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int]
lib.mk_accept.argtypes = [_vp, ctypes.POINTER(_Proposal), ctypes.c_int, ctypes.POINTER(AcceptResult)]
lib.mk_verify_step.argtypes = [_vp, ctypes.POINTER(BatchToken), ctypes.c_int, ctypes.POINTER(_Proposal), ctypes.c_int,
                               ctypes.POINTER(AcceptResult)]
lib.mk_rng_uniforms.argtypes = [ctypes.c_uint64, ctypes.c_int64, ctypes.c_int, _P_F64]
lib.mk_set_profile.argtypes = [_vp, ctypes.c_int]
lib.mk_stage_times.argtypes = [_vp, _P_F32]
lib.mk_last_launch_count.argtypes = [_vp]
lib.mk_last_launch_count.restype = ctypes.c_int64
lib.mk_last_io_bytes.argtypes = [_vp, ctypes.POINTER(ctypes.c_int64), ctypes.POINTER(ctypes.c_int64)]
lib.mk_stream.argtypes = [_vp]
lib.mk_stream.restype = _vp
lib.mk_weight_upload.argtypes = [ctypes.c_int, _vp, ctypes.c_int64, ctypes.c_int64, ctypes.POINTER(_vp)]
lib.mk_weight_free.argtypes = [_vp]
lib.mk_weight_device_bytes.argtypes = [_vp]
lib.mk_weight_device_bytes.restype = ctypes.c_int64
lib.mk_quantize_q8.argtypes = [_vp, ctypes.c_int, ctypes.c_int64, _vp, _vp]
lib.mk_matmul.argtypes = [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp]


class TpShard(ctypes.Structure):
    """mk_tp_shard: the slice of the model one tensor-parallel rank holds."""
    _fields_ = [("head0", ctypes.c_int32), ("heads", ctypes.c_int32), ("kv_head0", ctypes.c_int32),
                ("kv_heads", ctypes.c_int32), ("ffn0", ctypes.c_int32), ("ffn", ctypes.c_int32),
                ("vocab0", ctypes.c_int64), ("vocab", ctypes.c_int64), ("embd0", ctypes.c_int32), ("embd", ctypes.c_int32)]


lib.mk_tp_shard_of.argtypes = [ctypes.c_char_p, ctypes.c_int, ctypes.c_int, ctypes.POINTER(TpShard)]


def tp_shard_of(path: str, tp_size: int, tp_rank: int) -> TpShard:
    """Shard geometry of rank tp_rank of tp_size for the GGUF at path (host only)."""
    out = TpShard()
    _check(lib.mk_tp_shard_of(path.encode(), tp_size, tp_rank, ctypes.byref(out)))
    return out
lib.mk_matmul_noalloc.argtypes = [_vp, _vp, ctypes.c_int, _vp, ctypes.c_int, _vp]
lib.mk_block_dots.argtypes = [_vp, _vp, ctypes.c_int, _vp, _vp]
lib.mk_quantize_i8.argtypes = [_vp, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp]
lib.mk_silu_mul.argtypes = [_vp, _vp, ctypes.c_int64, _vp]
lib.mk_attention.argtypes = [_vp, ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, _vp, _vp, _vp, _vp,
                             ctypes.c_int64, _vp, _vp, _vp, _vp, _vp, _vp]

# Every symbol include/malkin_b200.h declares (tests check the library exports them all).
EXPORTS = ("mk_last_error", "mk_version", "mk_synth_gguf", "mk_init", "mk_nccl_unique_id", "mk_shutdown",
           "mk_load_gguf", "mk_alloc_kv", "mk_model_config_get", "mk_forward", "mk_move_kv", "mk_accept",
           "mk_rng_uniforms", "mk_verify_step", "mk_set_profile", "mk_stage_times", "mk_last_launch_count",
           "mk_stream", "mk_last_io_bytes", "mk_tp_shard_of", "mk_tp_exchange_check", "mk_weight_upload", "mk_weight_free", "mk_weight_device_bytes", "mk_quantize_q8",
           "mk_matmul", "mk_matmul_noalloc", "mk_block_dots", "mk_quantize_i8", "mk_silu_mul", "mk_attention",
           "mk_engine_create", "mk_engine_destroy", "mk_engine_submit", "mk_engine_step", "mk_engine_events",
           "mk_engine_busy", "mk_engine_cancel", "mk_engine_stats", "mk_engine_perplexity")


def version() -> str:
    return lib.mk_version().decode()


def synth_gguf(path: str, n_layer: int, n_embd: int, n_ff: int, n_head: int, n_head_kv: int, head_dim: int = 128,
               n_vocab: int = 151936, n_ctx_train: int = 40960, rope_base: float = 1e6, rms_eps: float = 1e-6,
               tied: bool = False, type_default: int = TYPE_Q8_0, type_attn_v: Optional[int] = None,
               type_ffn_down: Optional[int] = None, type_output: Optional[int] = None,
               type_embd: Optional[int] = None, sigma: float = 0.02, seed: int = 0, n_threads: int = 0,
               eos_token_id: Optional[int] = None) -> str:
    """Writes a synthetic Qwen3 GGUF (seeded N(0, sigma) weights, norms 1.0) and returns its path. eos_token_id: an
    end-of-generation token written as tokenizer.ggml.eos_token_id."""
    s = SynthSpec(n_layer, n_embd, n_ff, n_head, n_head_kv, head_dim, n_vocab, n_ctx_train, rope_base, rms_eps,
                  int(tied), type_default, type_attn_v if type_attn_v is not None else type_default,
                  type_ffn_down if type_ffn_down is not None else type_default,
                  type_output if type_output is not None else type_default,
                  type_embd if type_embd is not None else type_default, sigma, seed,
                  int(eos_token_id is not None), eos_token_id or 0)
    _check(lib.mk_synth_gguf(path.encode(), ctypes.byref(s), n_threads))
    return path


def rng_uniforms(seed: int, n: int, skip: int = 0) -> np.ndarray:
    """Values skip..skip+n-1 of the uniform stream a malkin Sampler with this seed draws."""
    out = np.empty(n, dtype=np.float64)
    _check(lib.mk_rng_uniforms(seed, skip, n, out.ctypes.data_as(_P_F64)))
    return out


lib.mk_tp_exchange_check.argtypes = [ctypes.c_int] * 5 + [ctypes.c_void_p, ctypes.c_int] + [ctypes.c_void_p] * 3


def tp_exchange_check(parts: np.ndarray, twoshot: bool = False, absent: Optional[Sequence[int]] = None,
                      wait_polls: int = 1 << 24):
    """Rank 0's tensor-parallel exchange kernels against host-emulated peers (mk_tp_exchange_check).
    parts: [calls, size, n, cols] float32. Returns (sums [calls, n, cols], status per call)."""
    parts = np.ascontiguousarray(parts, dtype=np.float32)
    calls, size, n, cols = parts.shape
    out = np.zeros((calls, n, cols), dtype=np.float32)
    st = np.zeros(calls, dtype=np.int32)
    ab = None if absent is None else np.ascontiguousarray(absent, dtype=np.int32)
    _check(lib.mk_tp_exchange_check(size, int(twoshot), n, cols, calls, None if ab is None else ab.ctypes.data,
                                    wait_polls, parts.ctypes.data, out.ctypes.data, st.ctypes.data))
    return out, st


def nccl_unique_id() -> bytes:
    buf = ctypes.create_string_buffer(128)
    _check(lib.mk_nccl_unique_id(buf))
    return buf.raw


def make_batch(tokens: Iterable[BatchToken]) -> ctypes.Array:
    toks = list(tokens)
    arr = (BatchToken * len(toks))()
    for i, t in enumerate(toks):
        arr[i] = t
    return arr


class Model:
    """malkin::Model on one GPU / tensor-parallel rank (model.h:33-97)."""

    def __init__(self, device: int = 0, tp_rank: int = 0, tp_size: int = 1, nccl_id: Optional[bytes] = None):
        self._h = _vp()
        idbuf = ctypes.create_string_buffer(nccl_id, 128) if nccl_id else None
        _check(lib.mk_init(device, tp_rank, tp_size, idbuf, ctypes.byref(self._h)))

    def close(self) -> None:
        if self._h:
            _check(lib.mk_shutdown(self._h))
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def load(self, path: str) -> "Model":
        _check(lib.mk_load_gguf(self._h, path.encode()))
        return self

    def alloc_kv(self, n_ctx: int, n_seq: int = 1, max_batch: int = 256) -> "Model":
        _check(lib.mk_alloc_kv(self._h, n_ctx, n_seq, max_batch))
        return self

    def config(self) -> ModelConfig:
        c = ModelConfig()
        _check(lib.mk_model_config_get(self._h, ctypes.byref(c)))
        return c

    def forward(self, batch, want_logits: bool = True) -> Optional[np.ndarray]:
        """Model::forward(const BatchToken*, n, logits): returns [rows with .logits, n_vocab] float32 (or None)."""
        b = batch if isinstance(batch, ctypes.Array) else make_batch(batch)
        m = sum(1 for t in b if t.logits)
        out = None
        ptr = ctypes.cast(None, _P_F32)
        if want_logits and m:
            out = np.empty((m, self.config().n_vocab), dtype=np.float32)
            ptr = out.ctypes.data_as(_P_F32)
        _check(lib.mk_forward(self._h, b, len(b), ptr))
        return out

    def move_kv(self, frm: int, to: int, seq: int = 0) -> None:
        _check(lib.mk_move_kv(self._h, frm, to, seq))

    def accept(self, proposals: Sequence[Proposal]) -> List[AcceptResult]:
        cp = (_Proposal * len(proposals))(*[p._c() for p in proposals])
        res = (AcceptResult * len(proposals))()
        _check(lib.mk_accept(self._h, cp, len(proposals), res))
        return list(res)

    def verify_step(self, batch, proposals: Sequence[Proposal]) -> List[AcceptResult]:
        b = batch if isinstance(batch, ctypes.Array) else make_batch(batch)
        cp = (_Proposal * len(proposals))(*[p._c() for p in proposals])
        res = (AcceptResult * len(proposals))()
        _check(lib.mk_verify_step(self._h, b, len(b), cp, len(proposals), res))
        return list(res)

    def set_profile(self, on: bool) -> None:
        _check(lib.mk_set_profile(self._h, int(on)))

    def stage_times(self) -> List[float]:
        ms = (ctypes.c_float * 8)()
        _check(lib.mk_stage_times(self._h, ms))
        return list(ms)

    def last_launch_count(self) -> int:
        return int(lib.mk_last_launch_count(self._h))

    def io_bytes(self):
        """(host->device, device->host) bytes copied since the previous call."""
        h, d = ctypes.c_int64(), ctypes.c_int64()
        _check(lib.mk_last_io_bytes(self._h, ctypes.byref(h), ctypes.byref(d)))
        return h.value, d.value

    @property
    def stream(self) -> int:
        return int(lib.mk_stream(self._h) or 0)


FINISH_STOP, FINISH_LENGTH, FINISH_CANCELLED = 1, 2, 3


class GenRequest(ctypes.Structure):
    """GenRequest (engine.h:29-34) with token ids."""
    _fields_ = [("prompt", ctypes.c_void_p), ("n_prompt", ctypes.c_int32), ("max_tokens", ctypes.c_int32),
                ("sampling", Sampling), ("seed", ctypes.c_uint64), ("eog", ctypes.c_void_p),
                ("n_eog", ctypes.c_int32)]


class GenEvent(ctypes.Structure):
    _fields_ = [("request", ctypes.c_int32), ("token", ctypes.c_int32), ("finish", ctypes.c_int32)]


class GenStats(ctypes.Structure):
    """GenResult's counters (engine.h:36-42); finish 0 while running."""
    _fields_ = [(n, ctypes.c_int32) for n in
                ("prompt_tokens", "cached_tokens", "completion_tokens", "drafted", "accepted", "finish")]


lib.mk_engine_create.argtypes = [_vp, _vp, ctypes.c_int, ctypes.POINTER(_vp)]
lib.mk_engine_destroy.argtypes = [_vp]
lib.mk_engine_submit.argtypes = [_vp, ctypes.POINTER(GenRequest), ctypes.POINTER(ctypes.c_int32)]
lib.mk_engine_step.argtypes = [_vp, ctypes.POINTER(GenEvent), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
lib.mk_engine_events.argtypes = [_vp, ctypes.POINTER(GenEvent), ctypes.c_int, ctypes.POINTER(ctypes.c_int)]
lib.mk_engine_busy.argtypes = [_vp, ctypes.POINTER(ctypes.c_int)]
lib.mk_engine_cancel.argtypes = [_vp, ctypes.c_int32]
lib.mk_engine_stats.argtypes = [_vp, ctypes.c_int32, ctypes.POINTER(GenStats)]
lib.mk_engine_perplexity.argtypes = [_vp, _vp, ctypes.c_int, ctypes.c_int, ctypes.c_int32,
                                     ctypes.POINTER(ctypes.c_double), ctypes.POINTER(ctypes.c_int)]


class Engine:
    """malkin::Engine (engine.h:47-141) at the token level over a target Model and an optional draft Model."""

    def __init__(self, target: "Model", draft: Optional["Model"] = None, n_draft: int = 0):
        self._h = _vp()
        self._keep = (target, draft)
        _check(lib.mk_engine_create(target._h, draft._h if draft is not None else None, n_draft,
                                    ctypes.byref(self._h)))
        self._ev = (GenEvent * 4096)()

    def close(self) -> None:
        if self._h:
            _check(lib.mk_engine_destroy(self._h))
            self._h = _vp()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def submit(self, prompt: Sequence[int], max_tokens: int = 0, sampling: Optional[Sampling] = None, seed: int = 0,
               eog: Sequence[int] = ()) -> int:
        p = np.ascontiguousarray(prompt, dtype=np.int32)
        e = np.ascontiguousarray(eog, dtype=np.int32)
        r = GenRequest(p.ctypes.data, len(p), max_tokens, sampling or Sampling(temperature=0.0), seed,
                       e.ctypes.data if len(e) else None, len(e))
        rid = ctypes.c_int32()
        _check(lib.mk_engine_submit(self._h, ctypes.byref(r), ctypes.byref(rid)))
        return rid.value

    def step(self) -> List[Tuple[int, int, int]]:
        """One Engine::step; returns (request, token, finish) events (token -1 with the finish code at the end)."""
        out, n = [], ctypes.c_int()
        _check(lib.mk_engine_step(self._h, self._ev, len(self._ev), ctypes.byref(n)))
        while True:
            out += [(e.request, e.token, e.finish) for e in self._ev[:n.value]]
            if n.value < len(self._ev):
                return out
            _check(lib.mk_engine_events(self._h, self._ev, len(self._ev), ctypes.byref(n)))

    def busy(self) -> bool:
        b = ctypes.c_int()
        _check(lib.mk_engine_busy(self._h, ctypes.byref(b)))
        return bool(b.value)

    def cancel(self, request: int) -> None:
        _check(lib.mk_engine_cancel(self._h, request))

    def stats(self, request: int) -> GenStats:
        s = GenStats()
        _check(lib.mk_engine_stats(self._h, request, ctypes.byref(s)))
        return s

    def run(self) -> Dict[int, List[int]]:
        """Steps until every request finished; returns each request's tokens."""
        toks: Dict[int, List[int]] = {}
        while self.busy():
            for r, t, f in self.step():
                toks.setdefault(r, [])
                if f == 0:
                    toks[r].append(t)
        return toks

    def perplexity(self, tokens: Sequence[int], window: int, bos: int = -1) -> Tuple[float, int]:
        """Engine::perplexity over token ids: (mean negative log-likelihood, tokens scored)."""
        t = np.ascontiguousarray(tokens, dtype=np.int32)
        nll, n = ctypes.c_double(), ctypes.c_int()
        _check(lib.mk_engine_perplexity(self._h, t.ctypes.data, len(t), window, bos, ctypes.byref(nll),
                                        ctypes.byref(n)))
        return nll.value, n.value


class Weight:
    """One GGUF matrix repacked into the device panel layout on the current device (pack_weight_into)."""

    def __init__(self, type_: int, rows_bytes: np.ndarray, rows: int, cols: int):
        self._h = _vp()
        a = np.ascontiguousarray(rows_bytes, dtype=np.uint8)
        assert a.size == rows * row_bytes(type_, cols)
        _check(lib.mk_weight_upload(type_, a.ctypes.data, rows, cols, ctypes.byref(self._h)))
        self.type, self.rows, self.cols = type_, rows, cols

    def __del__(self):
        if getattr(self, "_h", None):
            lib.mk_weight_free(self._h)
            self._h = _vp()

    @property
    def device_bytes(self) -> int:
        return int(lib.mk_weight_device_bytes(self._h))

    def matmul(self, dev_x: int, n: int, dev_y: int, split_k: int = 0, stream: int = 0) -> None:
        _check(lib.mk_matmul(self._h, dev_x, n, dev_y, split_k, stream or None))

    def matmul_noalloc(self, dev_x: int, n: int, dev_y: int, split_k: int = 0, stream: int = 0) -> None:
        """matmul through the fixed per-device scratch (mk_matmul_noalloc): no device allocation per call."""
        _check(lib.mk_matmul_noalloc(self._h, dev_x, n, dev_y, split_k, stream or None))

    def block_dots(self, dev_x: int, n: int, dev_out: int, stream: int = 0) -> None:
        _check(lib.mk_block_dots(self._h, dev_x, n, dev_out, stream or None))


def quantize_q8(dev_x: int, n: int, k: int, dev_blocks: int, stream: int = 0) -> None:
    _check(lib.mk_quantize_q8(dev_x, n, k, dev_blocks, stream or None))


def quantize_i8(dev_x: int, n: int, length: int, dev_q: int, dev_scale: int, stream: int = 0) -> None:
    _check(lib.mk_quantize_i8(dev_x, n, length, dev_q, dev_scale, stream or None))


def silu_mul(dev_g: int, dev_u: int, n: int, stream: int = 0) -> None:
    _check(lib.mk_silu_mul(dev_g, dev_u, n, stream or None))


def attention(dev_q: int, n: int, H: int, KV: int, D: int, dev_k: int, dev_v: int, dev_ks: int, dev_vs: int,
              n_rows: int, dev_kv_base: int, dev_n_keys: int, dev_anc_off: int, dev_anc: int, dev_out: int,
              stream: int = 0) -> None:
    _check(lib.mk_attention(dev_q, n, H, KV, D, dev_k, dev_v, dev_ks, dev_vs, n_rows, dev_kv_base, dev_n_keys,
                            dev_anc_off, dev_anc, dev_out, stream or None))
