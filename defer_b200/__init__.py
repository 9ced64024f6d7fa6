"""defer_b200 — B200 backend of convo-lang/defer's token loop.

Python mirror of the reference crate's public API (src/lib.rs:40-44) over the
C ABI in include/defer_b200.h:

    Model.load / forward / forward_ext / new_cache      (src/model.rs)
    KvCache len / truncate / clone / keys / values /
            fingerprint / bit_eq                        (src/model.rs:184-243)
    Session new / prompt / step / generate / checkout /
            checkpoint / history / rng_word_pos         (src/engine.rs)
    seed_from_u64, words_per_sample, sample_logits      (src/engine.rs, src/sampler.rs)
    DeferCheckpoint, WalHeader, WalWriter, WalLog       (src/checkpoint.rs, src/wal.rs)
    ablation_attribution, log_softmax_at                (src/attribution.rs)

plus the batched drivers (replay_batch, generate_batch) that advance many
sessions per device step. Every call runs the CUDA path; there is no CPU
fallback.
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from typing import Callable, List, Optional, Sequence

import numpy as np

from . import _lib
from ._lib import CheckpointFields, DeferConfig, TOKEN_CB, WalHeaderC

__all__ = [
    "DeferError", "IoError", "ParseError", "ModelError", "CheckpointError", "WalError", "TokenizerError",
    "DivergenceError", "CudaError", "DeviceTimeoutError", "InvalidArgumentError",
    "Config", "Model", "KvCache", "Session", "DeferCheckpoint", "WalHeader", "WalWriter", "WalLog",
    "seed_from_u64", "chacha8_words", "words_per_sample", "sample_logits", "log_softmax_at",
    "ablation_attribution", "replay_batch", "generate_batch",
]


# ------------------------------------------------------------------ errors
class DeferError(Exception):
    """DeferError (src/error.rs:5-14); `code` is the C ABI status."""
    code = 0


class IoError(DeferError):
    code = 1


class ParseError(DeferError):
    code = 2


class ModelError(DeferError):
    code = 3


class CheckpointError(DeferError):
    code = 4


class WalError(DeferError):
    code = 5


class TokenizerError(DeferError):
    code = 6


class DivergenceError(DeferError):
    code = 7


class CudaError(DeferError):
    code = 8


class DeviceTimeoutError(DeferError):
    code = 9


class InvalidArgumentError(DeferError):
    code = 10


_ERRORS = {c.code: c for c in (IoError, ParseError, ModelError, CheckpointError, WalError, TokenizerError,
                               DivergenceError, CudaError, DeviceTimeoutError, InvalidArgumentError)}


def _L():
    return _lib.load()


def _check(rc: int):
    if rc != 0:
        msg = (_L().defer_last_error() or b"").decode(errors="replace")
        raise _ERRORS.get(rc, DeferError)(msg)


def _u8(b: bytes):
    b = bytes(b)
    return (ctypes.c_uint8 * max(len(b), 1)).from_buffer_copy(b if b else b"\0")


def _u32arr(xs: Sequence[int]):
    a = np.ascontiguousarray(np.asarray(list(xs) if not isinstance(xs, np.ndarray) else xs,
                                        dtype=np.uint32).reshape(-1))
    if a.size == 0:
        a = np.zeros(1, np.uint32)
    return a, a.ctypes.data_as(_lib.c_u32p)


def _f32p(a: np.ndarray):
    return a.ctypes.data_as(_lib.c_f32p)


# ------------------------------------------------------------------ model
@dataclass
class Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    max_seq_len: int
    rms_norm_eps: float
    rope_theta: float
    tie_word_embeddings: bool
    activation: str
    has_bias: bool
    weights_bf16: bool
    bos_token_id: Optional[int]
    eos_token_ids: List[int]
    weight_bytes: int
    device: int
    sm_count: int

    @property
    def kv_dim(self):
        return self.num_kv_heads * self.head_dim

    @property
    def q_dim(self):
        return self.num_heads * self.head_dim


class Model:
    """Model (src/model.rs:271-520) resident on one B200."""

    def __init__(self, handle):
        self._h = handle
        c = DeferConfig()
        _check(_L().defer_model_config(self._h, ctypes.byref(c)))
        n = ctypes.c_size_t(0)
        _check(_L().defer_model_eos_tokens(self._h, None, 0, ctypes.byref(n)))
        eos = (ctypes.c_uint32 * max(n.value, 1))()
        _check(_L().defer_model_eos_tokens(self._h, eos, n.value, ctypes.byref(n)))
        self.config = Config(c.vocab_size, c.hidden_size, c.intermediate_size, c.num_layers, c.num_heads,
                             c.num_kv_heads, c.head_dim, c.max_seq_len, c.rms_norm_eps, c.rope_theta,
                             bool(c.tie_word_embeddings), "gelu" if c.gelu else "silu", bool(c.has_bias),
                             bool(c.weights_bf16), None if c.bos_token_id < 0 else int(c.bos_token_id),
                             list(eos)[:n.value], int(c.weight_bytes), c.device, c.sm_count)
        sig = (ctypes.c_uint8 * 32)()
        _check(_L().defer_model_signature(self._h, sig))
        self.signature = bytes(sig)

    @staticmethod
    def load(path: str, device: int = 0) -> "Model":
        h = ctypes.c_void_p()
        _check(_L().defer_model_load(os.fsencode(path), device, ctypes.byref(h)))
        return Model(h)

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _L().defer_model_free(h)
            self._h = None

    def new_cache(self, cap: int = 0) -> "KvCache":
        h = ctypes.c_void_p()
        _check(_L().defer_cache_new(self._h, cap, ctypes.byref(h)))
        return KvCache(h, self, owned=True)

    def forward_ext(self, token: int, cache: "KvCache", masked: Sequence[int] = (), logits: bool = True):
        out = np.empty(self.config.vocab_size, np.float32) if logits else None
        m = (ctypes.c_size_t * max(len(masked), 1))(*masked)
        _check(_L().defer_forward(self._h, cache._h, int(token), m, len(masked), _f32p(out) if logits else None))
        return out

    def forward(self, token: int, cache: "KvCache"):
        return self.forward_ext(token, cache, ())

    def timing(self, reset: bool = False) -> dict:
        """Totals of the token-loop runs since the last reset: device_ms
        (CUDA events on the model's stream), runs, launches, tokens and
        algorithmic hbm_bytes."""
        ms = ctypes.c_double(0)
        b = ctypes.c_double(0)
        r, l, t = ctypes.c_uint64(0), ctypes.c_uint64(0), ctypes.c_uint64(0)
        _check(_L().defer_model_timing(self._h, ctypes.byref(ms), ctypes.byref(r), ctypes.byref(l), ctypes.byref(t),
                                       ctypes.byref(b), 1 if reset else 0))
        return {"device_ms": ms.value, "runs": r.value, "launches": l.value, "tokens": t.value,
                "hbm_bytes": b.value}

    def trace_next_run(self, step: int):
        """Instrumentation: the next dataflow token-loop run records a
        per-stage time trace of its step `step` (see trace())."""
        _check(_L().defer_debug_trace_arm(self._h, int(step)))

    def trace(self) -> np.ndarray:
        """The last trace as uint64 [ctas, stages, 24] globaltimer ns: slot 0
        stage entry, 1 inputs received, 2 + w phase warp w done, 10-21 warp
        0's sub-stage marks (see defer_debug_trace_arm; 0 = not reached)."""
        n = ctypes.c_size_t(0)
        c, st = ctypes.c_int32(0), ctypes.c_int32(0)
        _check(_L().defer_debug_trace_read(self._h, None, 0, ctypes.byref(n), ctypes.byref(c), ctypes.byref(st)))
        out = np.zeros(max(n.value, 1), np.uint64)
        _check(_L().defer_debug_trace_read(self._h, out.ctypes.data_as(ctypes.POINTER(ctypes.c_uint64)), out.size,
                                           ctypes.byref(n), ctypes.byref(c), ctypes.byref(st)))
        return out[:n.value].reshape(c.value, st.value, -1) if n.value else out[:0]

    def stall_next_run(self, wait_us: int = 1000):
        """Fault drill: the next token-loop run withholds one hand-off with
        its bounded waits cut to wait_us, and raises DeviceTimeoutError."""
        _check(_L().defer_debug_stall(self._h, int(wait_us)))


class KvCache:
    """KvCache (src/model.rs:184-243) in HBM."""

    def __init__(self, handle, model: Model, owned: bool, keepalive=None):
        self._h = handle
        self.model = model
        self._owned = owned
        self._keep = keepalive
        self.kv_dim = model.config.kv_dim

    def __del__(self):
        h = getattr(self, "_h", None)
        if h and self._owned:
            _L().defer_cache_free(h)
        self._h = None

    def __len__(self):
        return _L().defer_cache_len(self._h)

    def len(self):
        return len(self)

    def truncate(self, n: int):
        _check(_L().defer_cache_truncate(self._h, n))

    def clone(self) -> "KvCache":
        h = ctypes.c_void_p()
        _check(_L().defer_cache_clone(self._h, ctypes.byref(h)))
        return KvCache(h, self.model, owned=True)

    def layer(self, l: int):
        n = len(self) * self.kv_dim
        k = np.empty(max(n, 1), np.float32)
        v = np.empty(max(n, 1), np.float32)
        _check(_L().defer_cache_download(self._h, l, _f32p(k), _f32p(v)))
        return k[:n], v[:n]

    def keys(self, l: int) -> np.ndarray:
        return self.layer(l)[0]

    def values(self, l: int) -> np.ndarray:
        return self.layer(l)[1]

    def fingerprint(self) -> bytes:
        out = (ctypes.c_uint8 * 32)()
        _check(_L().defer_cache_fingerprint(self._h, out))
        return bytes(out)

    def bit_eq(self, other: "KvCache") -> bool:
        e = ctypes.c_int(0)
        _check(_L().defer_cache_bit_eq(self._h, other._h, ctypes.byref(e)))
        return bool(e.value)


# ----------------------------------------------------------- sampler / PRNG
def seed_from_u64(seed: int) -> bytes:
    out = (ctypes.c_uint8 * 32)()
    _L().defer_seed_from_u64(seed & 0xFFFFFFFFFFFFFFFF, out)
    return bytes(out)


def chacha8_words(seed: bytes, start: int, n: int) -> np.ndarray:
    out = np.empty(max(n, 1), np.uint32)
    _check(_L().defer_chacha8_words(_u8(seed), start, n, out.ctypes.data_as(_lib.c_u32p)))
    return out[:n]


def words_per_sample(temperature: float) -> int:
    return 0 if temperature == 0.0 else 1


def sample_logits(logits, temperature: float, word: int = 0, device: int = 0):
    """sample_token (src/sampler.rs:78-109) on the device; returns (token, margin)."""
    a = np.ascontiguousarray(logits, np.float32)
    tok = ctypes.c_uint32(0)
    mg = ctypes.c_float(0)
    _check(_L().defer_sample_logits(device, _f32p(a), a.size, temperature, word & 0xFFFFFFFF, ctypes.byref(tok),
                                    ctypes.byref(mg)))
    return tok.value, mg.value


def log_softmax_at(logits, idx: int) -> float:
    a = np.ascontiguousarray(logits, np.float32)
    return _L().defer_log_softmax_at(_f32p(a), a.size, idx)


# ------------------------------------------------------------- checkpoint
@dataclass
class DeferCheckpoint:
    """DeferCheckpoint (src/checkpoint.rs:26-108)."""
    model_signature: bytes
    base_seed: bytes
    temperature: float
    history_tokens: List[int]
    prompt_len: int
    rng_word_pos: int

    def generated_tokens(self):
        return self.history_tokens[self.prompt_len:]

    def _fields(self):
        f = CheckpointFields()
        ctypes.memmove(f.model_signature, bytes(self.model_signature), 32)
        ctypes.memmove(f.base_seed, bytes(self.base_seed), 32)
        f.temperature = self.temperature
        f.prompt_len = self.prompt_len
        f.rng_word_pos_lo = self.rng_word_pos & 0xFFFFFFFFFFFFFFFF
        f.rng_word_pos_hi = self.rng_word_pos >> 64
        arr, p = _u32arr(self.history_tokens)
        f.history_tokens = p
        f.n_tokens = len(self.history_tokens)
        return f, arr

    def to_bytes(self) -> bytes:
        f, keep = self._fields()
        n = ctypes.c_size_t(0)
        _check(_L().defer_checkpoint_encode(ctypes.byref(f), None, 0, ctypes.byref(n)))
        buf = (ctypes.c_uint8 * n.value)()
        _check(_L().defer_checkpoint_encode(ctypes.byref(f), buf, n.value, ctypes.byref(n)))
        return bytes(buf)

    @staticmethod
    def from_bytes(b: bytes) -> "DeferCheckpoint":
        f = CheckpointFields()
        _check(_L().defer_checkpoint_decode(_u8(b), len(b), ctypes.byref(f), None, 0))
        toks = np.empty(max(f.n_tokens, 1), np.uint32)
        _check(_L().defer_checkpoint_decode(_u8(b), len(b), ctypes.byref(f), toks.ctypes.data_as(_lib.c_u32p),
                                            toks.size))
        return DeferCheckpoint(bytes(f.model_signature), bytes(f.base_seed), float(np.float32(f.temperature)),
                               [int(t) for t in toks[:f.n_tokens]], int(f.prompt_len),
                               int(f.rng_word_pos_lo) | (int(f.rng_word_pos_hi) << 64))

    def save(self, path: str):
        b = self.to_bytes()
        _check(_L().defer_checkpoint_save(_u8(b), len(b), os.fsencode(path)))

    @staticmethod
    def load(path: str) -> "DeferCheckpoint":
        n = ctypes.c_size_t(0)
        _check(_L().defer_checkpoint_load(os.fsencode(path), None, 0, ctypes.byref(n)))
        buf = (ctypes.c_uint8 * n.value)()
        _check(_L().defer_checkpoint_load(os.fsencode(path), buf, n.value, ctypes.byref(n)))
        return DeferCheckpoint.from_bytes(bytes(buf))


# ------------------------------------------------------------------- WAL
@dataclass
class WalHeader:
    """WalHeader (src/wal.rs:45-84)."""
    model_signature: bytes
    base_seed: bytes
    temperature: float
    prompt_len: int
    start_rng_word_pos: int
    prefix_tokens: List[int]

    @staticmethod
    def from_checkpoint(c: DeferCheckpoint) -> "WalHeader":
        return WalHeader(c.model_signature, c.base_seed, c.temperature, c.prompt_len, c.rng_word_pos,
                         list(c.history_tokens))


class WalWriter:
    """WalWriter (src/wal.rs:212-255)."""

    def __init__(self, h):
        self._h = h

    @staticmethod
    def create(path: str, header: WalHeader, durable: bool = False) -> "WalWriter":
        c = WalHeaderC()
        ctypes.memmove(c.model_signature, bytes(header.model_signature), 32)
        ctypes.memmove(c.base_seed, bytes(header.base_seed), 32)
        c.temperature = header.temperature
        c.prompt_len = header.prompt_len
        c.start_rng_word_pos_lo = header.start_rng_word_pos & 0xFFFFFFFFFFFFFFFF
        c.start_rng_word_pos_hi = header.start_rng_word_pos >> 64
        arr, p = _u32arr(header.prefix_tokens)
        c.prefix_tokens = p
        c.n_prefix = len(header.prefix_tokens)
        h = ctypes.c_void_p()
        _check(_L().defer_wal_create(os.fsencode(path), ctypes.byref(c), 1 if durable else 0, ctypes.byref(h)))
        return WalWriter(h)

    @staticmethod
    def resume(path: str, durable: bool = False):
        h = ctypes.c_void_p()
        _check(_L().defer_wal_resume(os.fsencode(path), 1 if durable else 0, ctypes.byref(h)))
        return WalLog.read(path), WalWriter(h)

    def append(self, token: int, rng_word_pos: int):
        _check(_L().defer_wal_append(self._h, token, rng_word_pos & 0xFFFFFFFFFFFFFFFF, rng_word_pos >> 64))

    def close(self):
        if getattr(self, "_h", None):
            _L().defer_wal_close(self._h)
            self._h = None

    def __del__(self):
        self.close()

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()


@dataclass
class WalLog:
    """WalLog (src/wal.rs:106-210), collapsed through the C ABI."""
    checkpoint: DeferCheckpoint
    n_records: int
    torn_tail: bool
    valid_len: int

    @staticmethod
    def parse(b: bytes) -> "WalLog":
        n = ctypes.c_size_t(0)
        nrec = ctypes.c_size_t(0)
        torn = ctypes.c_int(0)
        vl = ctypes.c_uint64(0)
        _check(_L().defer_wal_to_checkpoint(_u8(b), len(b), None, 0, ctypes.byref(n), ctypes.byref(nrec),
                                            ctypes.byref(torn), ctypes.byref(vl)))
        buf = (ctypes.c_uint8 * n.value)()
        _check(_L().defer_wal_to_checkpoint(_u8(b), len(b), buf, n.value, ctypes.byref(n), ctypes.byref(nrec),
                                            ctypes.byref(torn), ctypes.byref(vl)))
        return WalLog(DeferCheckpoint.from_bytes(bytes(buf)), nrec.value, bool(torn.value), vl.value)

    @staticmethod
    def read(path: str) -> "WalLog":
        with open(path, "rb") as f:
            return WalLog.parse(f.read())

    @property
    def records(self):
        """(step, token, rng_word_pos) of every valid record."""
        c = self.checkpoint
        start = len(c.history_tokens) - self.n_records
        wps = words_per_sample(c.temperature)
        base = c.rng_word_pos - self.n_records * wps
        return [(start + i, c.history_tokens[start + i], base + (i + 1) * wps) for i in range(self.n_records)]

    def to_checkpoint(self) -> DeferCheckpoint:
        return self.checkpoint


# ---------------------------------------------------------------- session
class Session:
    """Session (src/engine.rs:23-274) with its KV cache and logits in HBM."""

    def __init__(self, model: Model, base_seed: bytes, temperature: float, _handle=None):
        self.model = model
        if _handle is None:
            h = ctypes.c_void_p()
            _check(_L().defer_session_new(model._h, _u8(base_seed), temperature, ctypes.byref(h)))
            _handle = h
        self._h = _handle

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            _L().defer_session_free(h)
            self._h = None

    def prompt(self, tokens: Sequence[int]):
        arr, p = _u32arr(tokens)
        _check(_L().defer_session_prompt(self._h, p, len(tokens)))

    def step(self) -> int:
        t = ctypes.c_uint32(0)
        _check(_L().defer_session_step(self._h, ctypes.byref(t)))
        return t.value

    def generate(self, max_tokens: int, stop: Sequence[int] = (),
                 on_token: Optional[Callable[["Session", int], None]] = None) -> List[int]:
        sarr, sp = _u32arr(stop)
        out = np.empty(max(max_tokens, 1), np.uint32)
        n = ctypes.c_size_t(0)
        err = []

        def cb(_user, token, _pos):
            if on_token is None:
                return 0
            try:
                on_token(self, int(token))
                return 0
            except DeferError as e:  # propagate the callback's own error kind
                err.append(e)
                return e.code or IoError.code
            except Exception as e:  # noqa: BLE001
                err.append(e)
                return IoError.code

        cfun = TOKEN_CB(cb)
        rc = _L().defer_session_generate(self._h, max_tokens, sp, len(stop), cfun, None,
                                         out.ctypes.data_as(_lib.c_u32p), ctypes.byref(n))
        if rc != 0 and err:
            raise err[0]
        _check(rc)
        return [int(t) for t in out[:n.value]]

    @staticmethod
    def checkout(model: Model, ckpt: DeferCheckpoint) -> "Session":
        b = ckpt.to_bytes()
        h = ctypes.c_void_p()
        _check(_L().defer_session_checkout(model._h, _u8(b), len(b), ctypes.byref(h)))
        return Session(model, ckpt.base_seed, ckpt.temperature, _handle=h)

    def checkpoint(self) -> DeferCheckpoint:
        n = ctypes.c_size_t(0)
        _check(_L().defer_session_checkpoint(self._h, None, 0, ctypes.byref(n)))
        buf = (ctypes.c_uint8 * n.value)()
        _check(_L().defer_session_checkpoint(self._h, buf, n.value, ctypes.byref(n)))
        return DeferCheckpoint.from_bytes(bytes(buf))

    def history(self) -> List[int]:
        n = ctypes.c_size_t(0)
        _check(_L().defer_session_history(self._h, None, 0, ctypes.byref(n)))
        out = np.empty(max(n.value, 1), np.uint32)
        _check(_L().defer_session_history(self._h, out.ctypes.data_as(_lib.c_u32p), n.value, ctypes.byref(n)))
        return [int(t) for t in out[:n.value]]

    def prompt_len(self) -> int:
        return _L().defer_session_prompt_len(self._h)

    def generated(self) -> List[int]:
        return self.history()[self.prompt_len():]

    def rng_word_pos(self) -> int:
        return _L().defer_session_rng_word_pos(self._h)

    def last_logits(self) -> np.ndarray:
        out = np.empty(self.model.config.vocab_size, np.float32)
        _check(_L().defer_session_last_logits(self._h, _f32p(out)))
        return out

    def cache(self) -> KvCache:
        return KvCache(_L().defer_session_cache(self._h), self.model, owned=False, keepalive=self)

    def margins(self) -> np.ndarray:
        n = ctypes.c_size_t(0)
        _check(_L().defer_session_margins(self._h, None, 0, ctypes.byref(n)))
        out = np.empty(max(n.value, 1), np.float32)
        _check(_L().defer_session_margins(self._h, _f32p(out), n.value, ctypes.byref(n)))
        return out[:n.value]


# --------------------------------------------------------- batch drivers
@dataclass
class ReplayResult:
    status: int
    div_step: int
    div_token: int
    fingerprint: Optional[bytes]


def replay_batch(model: Model, ckpts: Sequence[DeferCheckpoint], batch: int = 64, fingerprints: bool = False):
    """Verified checkout of many checkpoints at once; returns (results, device_ms)."""
    n = len(ckpts)
    raw = [c.to_bytes() for c in ckpts]
    bufs = [_u8(b) for b in raw]
    lens = (ctypes.c_size_t * max(n, 1))(*[len(b) for b in raw])
    ptrs = (_lib.c_u8p * max(n, 1))(*[ctypes.cast(b, _lib.c_u8p) for b in bufs])
    st = (ctypes.c_int32 * max(n, 1))()
    ds = (ctypes.c_int32 * max(n, 1))()
    dt = (ctypes.c_uint32 * max(n, 1))()
    fp = (ctypes.c_uint8 * (32 * max(n, 1)))() if fingerprints else None
    ms = ctypes.c_double(0)
    _check(_L().defer_replay_batch(model._h, ptrs, lens, n, batch, st, ds, dt, fp, ctypes.byref(ms)))
    res = [ReplayResult(st[i], ds[i], dt[i], bytes(fp[32 * i:32 * i + 32]) if fingerprints else None)
           for i in range(n)]
    return res, ms.value


def generate_batch(model: Model, prompts: Sequence[Sequence[int]], seeds: Sequence[bytes],
                   temperatures: Sequence[float], max_tokens: Sequence[int], batch: int = 64):
    """Session::new + prompt + generate for many sessions; returns (tokens, device_ms)."""
    n = len(prompts)
    keep = [_u32arr(p) for p in prompts]
    pp = (_lib.c_u32p * max(n, 1))(*[k[1] for k in keep])
    pl = (ctypes.c_size_t * max(n, 1))(*[len(p) for p in prompts])
    sd = (ctypes.c_uint8 * (32 * max(n, 1)))(*b"".join(bytes(s) for s in seeds))
    tp = (ctypes.c_float * max(n, 1))(*temperatures)
    mt = (ctypes.c_size_t * max(n, 1))(*max_tokens)
    outs = [np.empty(max(m, 1), np.uint32) for m in max_tokens]
    op = (_lib.c_u32p * max(n, 1))(*[o.ctypes.data_as(_lib.c_u32p) for o in outs])
    no = (ctypes.c_size_t * max(n, 1))()
    ms = ctypes.c_double(0)
    _check(_L().defer_generate_batch(model._h, pp, pl, sd, tp, mt, n, batch, op, no, ctypes.byref(ms)))
    return [[int(t) for t in outs[i][:no[i]]] for i in range(n)], ms.value


def verify(model: Model, seed: bytes, temperature: float, prompt: Sequence[int], runs: int = 10,
           max_tokens: int = 32, stop: Sequence[int] = ()):
    """`defer verify` (src/main.rs:620-666): `runs` identical sessions and a
    checkout of run 0, all bit-identical; returns (tokens, KV fingerprint)
    or raises DivergenceError."""
    pa, pp = _u32arr(prompt)
    sa, sp = _u32arr(stop)
    out = np.empty(max(max_tokens, 1), np.uint32)
    n = ctypes.c_size_t(0)
    fp = (ctypes.c_uint8 * 32)()
    _check(_L().defer_verify(model._h, _u8(seed), temperature, pp, len(prompt), runs, max_tokens, sp, len(stop),
                             out.ctypes.data_as(_lib.c_u32p), ctypes.byref(n), fp))
    return [int(t) for t in out[:n.value]], bytes(fp)


def tc_gemm(x: np.ndarray, w: np.ndarray, w_bf16: bool = False, device: int = 0) -> np.ndarray:
    """The tensor-core contraction of the batched attribution step on its
    own: x [m, k] . w [n, k]^T (m <= 128) as split-bf16 tcgen05 MMAs."""
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    m, k = x.shape
    n = w.shape[0]
    y = np.empty((m, n), np.float32)
    _check(_L().defer_debug_tc_gemm(device, _f32p(x), m, _f32p(w), n, k, 1 if w_bf16 else 0, _f32p(y)))
    return y


def ablation_attribution(model: Model, context: Sequence[int], target: int, positions: Sequence[int],
                         batch: int = 128):
    """attribution::ablation_attribution (src/attribution.rs:224-264):
    returns (base_logprob, [(position, token, ablated_logprob, delta)])."""
    arr, p = _u32arr(context)
    pos = (ctypes.c_size_t * max(len(positions), 1))(*positions)
    out = (ctypes.c_double * max(len(positions), 1))()
    base = ctypes.c_double(0)
    _check(_L().defer_ablation(model._h, p, len(context), target, pos, len(positions), batch, ctypes.byref(base),
                               out))
    return base.value, [(int(q), int(context[q]), out[i], base.value - out[i]) for i, q in enumerate(positions)]
