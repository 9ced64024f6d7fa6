"""CPU ORACLE — test infrastructure only.

Python half of the CPU restatement of convo-lang/defer's reference path.
The arithmetic (ops, forward pass, sampler, ChaCha8) lives in ``oracle.c``
(built by ``oracle/Makefile`` into ``oracle/_build/liboracle.so``); this
module restates the byte-level parts of the reference on top of it:

* safetensors reading/writing (safetensors.rs:142-299), SHA-256 signature
* ``Config::from_json`` / ``Config::to_json`` (model.rs:44-160)
* ``Session`` prompt / step / generate / checkpoint / checkout (engine.rs)
* WAL and checkpoint formats (wal.rs, checkpoint.rs), CRC-32 (crc32.rs)
* the tiny synthetic model writer (synthetic.rs)
* leave-one-out ablation (attribution.rs:224-264)

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline
leg may import this module. It is the checker, never the product.

Parity status: pinned against the reference's own known-answer tests
(tests/test_oracle.py); the ChaCha8 / seed_from_u64 / gen::<f32>
restatement of the third-party rand crates is pinned at the ChaCha block
function (independent ChaCha20 and the published ChaCha8 vector) but not at
seed_from_u64, so interchange with WALs written by the real Rust binary is
unpinned.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import math
import os
import struct
import subprocess
from dataclasses import dataclass, field
from typing import Callable, List, Optional, Sequence

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

_lib = None


def build() -> str:
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = ctypes.CDLL(LIB_PATH)
        f32p = ctypes.POINTER(ctypes.c_float)
        sz = ctypes.c_size_t
        vp = ctypes.c_void_p
        L.or_linear.argtypes = [f32p, f32p, f32p, f32p, sz, sz]
        L.or_dot.argtypes = [f32p, f32p, sz]
        L.or_dot.restype = ctypes.c_float
        L.or_rmsnorm.argtypes = [f32p, f32p, f32p, sz, ctypes.c_float]
        L.or_layernorm.argtypes = [f32p, f32p, f32p, f32p, sz, ctypes.c_float]
        L.or_matmul_sequential.argtypes = [f32p, f32p, f32p, sz, sz, sz]
        L.or_silu.argtypes = [ctypes.c_float]
        L.or_silu.restype = ctypes.c_float
        L.or_gelu.argtypes = [ctypes.c_float]
        L.or_gelu.restype = ctypes.c_float
        L.or_softmax_inplace.argtypes = [f32p, sz]
        L.or_chacha_block.argtypes = [ctypes.POINTER(ctypes.c_uint32), ctypes.POINTER(ctypes.c_uint32), ctypes.c_int]
        L.or_chacha_sizeof.restype = sz
        L.or_chacha_init.argtypes = [vp, ctypes.c_char_p]
        L.or_chacha_next_u32.argtypes = [vp]
        L.or_chacha_next_u32.restype = ctypes.c_uint32
        L.or_chacha_word_pos.argtypes = [vp]
        L.or_chacha_word_pos.restype = ctypes.c_uint64
        L.or_chacha_gen_f32.argtypes = [vp]
        L.or_chacha_gen_f32.restype = ctypes.c_float
        L.or_chacha_gen_range_f32.argtypes = [vp, ctypes.c_float, ctypes.c_float]
        L.or_chacha_gen_range_f32.restype = ctypes.c_float
        L.or_u32_to_unit_f32.argtypes = [ctypes.c_uint32]
        L.or_u32_to_unit_f32.restype = ctypes.c_float
        L.or_seed_from_u64.argtypes = [ctypes.c_uint64, ctypes.c_char_p]
        L.or_argmax.argtypes = [f32p, sz]
        L.or_argmax.restype = sz
        L.or_softmax_with_temperature.argtypes = [f32p, sz, ctypes.c_float, f32p]
        L.or_cdf_scan.argtypes = [f32p, sz, ctypes.c_float]
        L.or_cdf_scan.restype = sz
        L.or_sample_token_word.argtypes = [f32p, sz, ctypes.c_float, ctypes.c_uint32, f32p]
        L.or_sample_token_word.restype = sz
        L.or_model_new.argtypes = [sz, sz, sz, sz, sz, sz, sz, sz, ctypes.c_float, ctypes.c_float, ctypes.c_int]
        L.or_model_new.restype = vp
        L.or_model_set_globals.argtypes = [vp, f32p, f32p, f32p]
        L.or_model_set_layer.argtypes = [vp, sz] + [f32p] * 12
        L.or_model_free.argtypes = [vp]
        L.or_model_inv_freq.argtypes = [vp]
        L.or_model_inv_freq.restype = f32p
        L.or_rope_tables.argtypes = [vp, sz, f32p, f32p]
        L.or_cache_new.argtypes = [vp, sz]
        L.or_cache_new.restype = vp
        L.or_cache_free.argtypes = [vp]
        L.or_cache_len.argtypes = [vp]
        L.or_cache_len.restype = sz
        L.or_cache_truncate.argtypes = [vp, sz]
        L.or_cache_set_len.argtypes = [vp, sz]
        L.or_cache_copy.argtypes = [vp, vp]
        L.or_cache_keys.argtypes = [vp, sz]
        L.or_cache_keys.restype = f32p
        L.or_cache_values.argtypes = [vp, sz]
        L.or_cache_values.restype = f32p
        L.or_forward.argtypes = [vp, vp, ctypes.c_uint32, ctypes.POINTER(ctypes.c_size_t), sz, f32p,
                                 ctypes.c_char_p, sz]
        L.or_forward.restype = ctypes.c_int
        L.or_log_softmax_at.argtypes = [f32p, sz, sz]
        L.or_log_softmax_at.restype = ctypes.c_double
        L.or_crc32.argtypes = [ctypes.c_char_p, sz]
        L.or_crc32.restype = ctypes.c_uint32
        _lib = L
    return _lib


def fp(a: Optional[np.ndarray]):
    if a is None:
        return None
    assert a.dtype == np.float32 and a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))


# ----------------------------------------------------------------- errors
class DeferError(Exception):
    kind = "Model"


class IoError(DeferError):
    kind = "Io"


class ParseError(DeferError):
    kind = "Parse"


class ModelError(DeferError):
    kind = "Model"


class CheckpointError(DeferError):
    kind = "Checkpoint"


class WalError(DeferError):
    kind = "Wal"


class DivergenceError(DeferError):
    kind = "Divergence"


# ------------------------------------------------------------------ ops.rs
def linear(x, w, bias=None) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    w = np.ascontiguousarray(w, np.float32)
    out_dim = w.size // x.size
    out = np.zeros(out_dim, np.float32)
    lib().or_linear(fp(out), fp(x), fp(w), fp(None if bias is None else np.ascontiguousarray(bias, np.float32)),
                    x.size, out_dim)
    return out


def rmsnorm(x, w, eps: float) -> np.ndarray:
    x = np.ascontiguousarray(x, np.float32)
    out = np.zeros_like(x)
    lib().or_rmsnorm(fp(out), fp(x), fp(np.ascontiguousarray(w, np.float32)), x.size, eps)
    return out


def softmax(x: Sequence[float]) -> np.ndarray:
    a = np.array(x, np.float32)
    lib().or_softmax_inplace(fp(a), a.size)
    return a


# ------------------------------------------------------------- ChaCha8Rng
class ChaCha8Rng:
    """rand_chacha 0.3.1 ChaCha8Rng restated (words consumed in order)."""

    def __init__(self, seed: bytes):
        assert len(seed) == 32
        self._buf = ctypes.create_string_buffer(lib().or_chacha_sizeof())
        lib().or_chacha_init(self._buf, bytes(seed))
        self.seed = bytes(seed)

    @classmethod
    def seed_from_u64(cls, s: int) -> "ChaCha8Rng":
        return cls(seed_from_u64(s))

    def next_u32(self) -> int:
        return lib().or_chacha_next_u32(self._buf)

    def gen_f32(self) -> float:
        return lib().or_chacha_gen_f32(self._buf)

    def gen_range_f32(self, lo: float, hi: float) -> float:
        return lib().or_chacha_gen_range_f32(self._buf, lo, hi)

    def get_word_pos(self) -> int:
        return lib().or_chacha_word_pos(self._buf)


def seed_from_u64(s: int) -> bytes:
    """engine.rs:19-21 (rand_core 0.6.4 PCG32 seed fill)."""
    out = ctypes.create_string_buffer(32)
    lib().or_seed_from_u64(s & 0xFFFFFFFFFFFFFFFF, out)
    return out.raw


def chacha_block(state16: Sequence[int], rounds: int) -> List[int]:
    inp = (ctypes.c_uint32 * 16)(*state16)
    out = (ctypes.c_uint32 * 16)()
    lib().or_chacha_block(inp, out, rounds)
    return list(out)


def keystream_words(seed: bytes, start: int, n: int) -> np.ndarray:
    r = ChaCha8Rng(seed)
    for _ in range(start):
        r.next_u32()
    return np.array([r.next_u32() for _ in range(n)], np.uint32)


# -------------------------------------------------------------- sampler.rs
def words_per_sample(t: float) -> int:
    return 0 if t == 0.0 else 1


def argmax(logits) -> int:
    a = np.ascontiguousarray(logits, np.float32)
    return lib().or_argmax(fp(a), a.size)


def softmax_with_temperature(logits, t: float) -> np.ndarray:
    a = np.ascontiguousarray(logits, np.float32)
    p = np.zeros_like(a)
    lib().or_softmax_with_temperature(fp(a), a.size, t, fp(p))
    return p


def sample_token_word(logits, t: float, word: int) -> int:
    """sampler.rs:78-109 with the one PRNG word already drawn."""
    a = np.ascontiguousarray(logits, np.float32)
    if a.size == 0:
        raise AssertionError("cannot sample from empty logits")
    if not (t >= 0.0 and math.isfinite(t)):
        raise AssertionError("temperature must be finite and >= 0")
    p = np.zeros_like(a)
    return lib().or_sample_token_word(fp(a), a.size, t, word & 0xFFFFFFFF, fp(p))


def sample_token(logits, t: float, rng: ChaCha8Rng) -> int:
    a = np.ascontiguousarray(logits, np.float32)
    if a.size == 0:
        raise AssertionError("cannot sample from empty logits")
    if not (t >= 0.0 and math.isfinite(t)):
        raise AssertionError("temperature must be finite and >= 0")
    if t == 0.0:
        return argmax(a)
    return sample_token_word(a, t, rng.next_u32())


def unit_f32(word: int) -> float:
    return lib().or_u32_to_unit_f32(word & 0xFFFFFFFF)


def crc32(b: bytes) -> int:
    return lib().or_crc32(bytes(b), len(b))


# ------------------------------------------------------------ safetensors
_DT = {"F32": 4, "F16": 2, "BF16": 2, "F64": 8}


def _convert(dtype: str, raw: bytes) -> np.ndarray:
    """safetensors.rs:77-104 — every dtype to f32, exactly."""
    if dtype == "F32":
        return np.frombuffer(raw, "<f4").astype(np.float32)
    if dtype == "F16":
        return np.frombuffer(raw, "<f2").astype(np.float32)
    if dtype == "BF16":
        return (np.frombuffer(raw, "<u2").astype(np.uint32) << 16).view(np.float32)
    if dtype == "F64":
        return np.frombuffer(raw, "<f8").astype(np.float32)
    raise ModelError(f"unsupported safetensors dtype {dtype}")


@dataclass
class SafeTensors:
    names: List[str]
    tensors: dict
    metadata: List[tuple]
    signature: bytes

    def meta(self, key):
        for k, v in self.metadata:
            if k == key:
                return v
        return None

    @staticmethod
    def load(path: str) -> "SafeTensors":
        """safetensors.rs:142-237: one pass, SHA-256 over every byte."""
        with open(path, "rb") as f:
            data = f.read()
        sig = hashlib.sha256(data).digest()
        if len(data) < 8:
            raise ModelError("invalid safetensors header length")
        hl = struct.unpack_from("<Q", data, 0)[0]
        if hl > 100 * 1024 * 1024 or 8 + hl > len(data):
            raise ModelError("invalid safetensors header length")
        try:
            hdr = json.loads(data[8:8 + hl].decode("utf-8"), object_pairs_hook=list)
        except UnicodeDecodeError:
            raise ModelError("safetensors header is not UTF-8")
        if not isinstance(hdr, list):
            raise ModelError("safetensors header is not an object")
        metadata, entries = [], []
        for name, v in hdr:
            if name == "__metadata__":
                if isinstance(v, list):
                    metadata = [(k, s) for k, s in v if isinstance(s, str)]
                continue
            v = dict(v)
            dt = v["dtype"]
            if dt not in _DT:
                raise ModelError(f"unsupported safetensors dtype {dt}")
            shape = [int(s) for s in v["shape"]]
            s, e = v["data_offsets"]
            numel = int(np.prod(shape)) if shape else 1
            if e < s or e - s != numel * _DT[dt]:
                raise ModelError(f"size mismatch for tensor {name}")
            entries.append((s, name, dt, shape, e))
        entries.sort(key=lambda t: (t[0], t[1]))
        base = 8 + hl
        data_len = len(data) - base
        pos = 0
        names, tensors = [], {}
        for s, name, dt, shape, e in entries:
            if s < pos or e > data_len:
                raise ModelError(f"overlapping/out of range tensor {name}")
            arr = _convert(dt, data[base + s:base + e])
            if len(shape) > 3:
                shape = [arr.size // max(shape[-1], 1), shape[-1]]
            tensors[name] = arr.reshape(shape) if shape else arr
            names.append(name)
            pos = e
        return SafeTensors(names, tensors, metadata, sig)


def json_quote(s: str) -> str:
    """json.rs:77-94."""
    out = ['"']
    for c in s:
        if c == '"':
            out.append('\\"')
        elif c == "\\":
            out.append("\\\\")
        elif c == "\n":
            out.append("\\n")
        elif c == "\r":
            out.append("\\r")
        elif c == "\t":
            out.append("\\t")
        elif ord(c) < 0x20:
            out.append("\\u%04x" % ord(c))
        else:
            out.append(c)
    out.append('"')
    return "".join(out)


def write_safetensors(path: str, tensors, metadata=()) -> None:
    """safetensors.rs:252-299 — F32 tensors in the given order."""
    parts = []
    if metadata:
        parts.append('"__metadata__":{' + ",".join(f"{json_quote(k)}:{json_quote(v)}" for k, v in metadata) + "}")
    off = 0
    for name, shape, data in tensors:
        n = int(np.prod(shape))
        assert n == np.asarray(data).size
        parts.append(f'{json_quote(name)}:{{"dtype":"F32","shape":[{",".join(str(d) for d in shape)}],'
                     f'"data_offsets":[{off},{off + n * 4}]}}')
        off += n * 4
    header = "{" + ",".join(parts) + "}"
    while len(header.encode()) % 8:
        header += " "
    hb = header.encode()
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for _, _, data in tensors:
            f.write(np.ascontiguousarray(data, "<f4").tobytes())


# ------------------------------------------------------------- model.rs
def _rust_exp_f32(x: float) -> str:
    """Rust `{:e}` of an f32: shortest round-trip digits, e.g. 1e-5."""
    s = np.format_float_scientific(np.float32(x), unique=True, trim="-")
    mant, exp = s.split("e")
    mant = mant.rstrip(".")
    return f"{mant}e{int(exp)}"


def _rust_disp_f32(x: float) -> str:
    return np.format_float_positional(np.float32(x), unique=True, trim="-")


@dataclass
class Config:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rms_norm_eps: float
    rope_theta: float
    max_seq_len: int
    tie_word_embeddings: bool
    activation: str = "silu"
    bos_token_id: Optional[int] = None
    eos_token_ids: List[int] = field(default_factory=list)

    @property
    def kv_dim(self):
        return self.num_kv_heads * self.head_dim

    @property
    def q_dim(self):
        return self.num_heads * self.head_dim

    @staticmethod
    def from_json(v: dict, st: SafeTensors) -> "Config":
        """model.rs:44-118."""
        def num(k):
            x = v.get(k)
            ok = isinstance(x, (int, float)) and not isinstance(x, bool) and x >= 0 and float(x).is_integer()
            return int(x) if ok else None

        def flt(k):
            x = v.get(k)
            return float(x) if isinstance(x, (int, float)) and not isinstance(x, bool) else None

        def missing(k):
            return ModelError(f"config is missing `{k}`")

        embed = st.tensors.get("model.embed_tokens.weight", st.tensors.get("embed_tokens.weight"))
        vg = hg = None
        if embed is not None and embed.ndim == 2:
            vg, hg = embed.shape
        hidden = num("hidden_size") if num("hidden_size") is not None else hg
        if hidden is None:
            raise missing("hidden_size")
        vocab = num("vocab_size") if num("vocab_size") is not None else vg
        if vocab is None:
            raise missing("vocab_size")
        nl = num("num_hidden_layers")
        if nl is None:
            nl = 0
            while f"model.layers.{nl}.input_layernorm.weight" in st.tensors:
                nl += 1
            if nl == 0:
                raise missing("num_hidden_layers")
        inter = num("intermediate_size")
        if inter is None:
            t = st.tensors.get("model.layers.0.mlp.gate_proj.weight")
            if t is None:
                raise missing("intermediate_size")
            inter = t.shape[0]
        nh = num("num_attention_heads")
        if nh is None:
            raise missing("num_attention_heads")
        nkv = num("num_key_value_heads") if num("num_key_value_heads") is not None else nh
        hd = num("head_dim") if num("head_dim") is not None else hidden // nh
        act = v.get("hidden_act", "silu")
        if not isinstance(act, str):
            act = "silu"
        if act in ("silu", "swish"):
            act = "silu"
        elif act.startswith("gelu"):
            act = "gelu"
        else:
            raise ModelError(f"unsupported activation {act}")
        eos = v.get("eos_token_id")
        if isinstance(eos, list):
            eos_ids = [int(x) for x in eos if isinstance(x, int) and x >= 0]
        elif isinstance(eos, int) and eos >= 0:
            eos_ids = [eos]
        else:
            eos_ids = []
        has_lm_head = "lm_head.weight" in st.tensors
        tie = v.get("tie_word_embeddings")
        tie = (tie if isinstance(tie, bool) else (not has_lm_head)) or not has_lm_head
        eps = flt("rms_norm_eps")
        theta = flt("rope_theta")
        bos = v.get("bos_token_id")
        cfg = Config(vocab, hidden, inter, nl, nh, nkv, hd,
                     float(np.float32(eps if eps is not None else 1e-6)),
                     float(np.float32(theta if theta is not None else 10000.0)),
                     num("max_position_embeddings") if num("max_position_embeddings") is not None else 4096,
                     tie, act, bos if isinstance(bos, int) else None, eos_ids)
        if cfg.num_kv_heads == 0 or cfg.num_heads % cfg.num_kv_heads != 0:
            raise ModelError("num_attention_heads must be a multiple of num_key_value_heads")
        if cfg.head_dim % 2 != 0:
            raise ModelError("head_dim must be even for RoPE")
        return cfg

    def to_json(self) -> str:
        """model.rs:129-160."""
        s = ('{"architectures":["LlamaForCausalLM"],'
             f'"vocab_size":{self.vocab_size},"hidden_size":{self.hidden_size},'
             f'"intermediate_size":{self.intermediate_size},"num_hidden_layers":{self.num_layers},'
             f'"num_attention_heads":{self.num_heads},"num_key_value_heads":{self.num_kv_heads},'
             f'"head_dim":{self.head_dim},"rms_norm_eps":{_rust_exp_f32(self.rms_norm_eps)},'
             f'"rope_theta":{_rust_disp_f32(self.rope_theta)},'
             f'"max_position_embeddings":{self.max_seq_len},'
             f'"tie_word_embeddings":{"true" if self.tie_word_embeddings else "false"},'
             f'"hidden_act":"{"silu" if self.activation == "silu" else "gelu_pytorch_tanh"}"')
        if self.bos_token_id is not None:
            s += f',"bos_token_id":{self.bos_token_id}'
        if self.eos_token_ids:
            s += ',"eos_token_id":[' + ",".join(str(x) for x in self.eos_token_ids) + "]"
        return s + "}"


class KvCache:
    """model.rs:184-243 backed by the C cache (capacity fixed up front)."""

    def __init__(self, model: "Model", cap: Optional[int] = None):
        self.model = model
        self.cap = cap if cap is not None else model.config.max_seq_len
        self.ptr = lib().or_cache_new(model.ptr, self.cap)
        self.kv_dim = model.config.kv_dim

    def __del__(self):
        p = getattr(self, "ptr", None)
        if p:
            lib().or_cache_free(p)
            self.ptr = None

    def __len__(self):
        return lib().or_cache_len(self.ptr)

    def truncate(self, n: int):
        lib().or_cache_truncate(self.ptr, n)

    def set_len(self, n: int):
        """Timing samples only: length n <= cap without computing the rows
        in between (see or_cache_set_len)."""
        lib().or_cache_set_len(self.ptr, n)

    def clone(self) -> "KvCache":
        c = KvCache(self.model, self.cap)
        lib().or_cache_copy(c.ptr, self.ptr)
        return c

    def keys(self, layer: int) -> np.ndarray:
        n = len(self) * self.kv_dim
        p = lib().or_cache_keys(self.ptr, layer)
        return np.ctypeslib.as_array(p, shape=(max(n, 1),))[:n].copy()

    def values(self, layer: int) -> np.ndarray:
        n = len(self) * self.kv_dim
        p = lib().or_cache_values(self.ptr, layer)
        return np.ctypeslib.as_array(p, shape=(max(n, 1),))[:n].copy()

    def bit_eq(self, other: "KvCache") -> bool:
        if len(self) != len(other) or self.kv_dim != other.kv_dim:
            return False
        for l in range(self.model.config.num_layers):
            if self.keys(l).tobytes() != other.keys(l).tobytes():
                return False
            if self.values(l).tobytes() != other.values(l).tobytes():
                return False
        return True

    def fingerprint(self) -> bytes:
        """model.rs:233-242."""
        h = hashlib.sha256()
        h.update(struct.pack("<Q", len(self)))
        for l in range(self.model.config.num_layers):
            h.update(self.keys(l).astype("<f4").tobytes())
            h.update(self.values(l).astype("<f4").tobytes())
        return h.digest()


class Model:
    """model.rs:271-363 on top of the C forward pass."""

    def __init__(self, config: Config, st: SafeTensors):
        c = config
        self.config = c
        self.signature = st.signature
        embed_name = "model.embed_tokens.weight" if "model.embed_tokens.weight" in st.tensors else "embed_tokens.weight"
        has_bias = "model.layers.0.self_attn.q_proj.bias" in st.tensors
        self._keep = []

        def take(name, shape):
            t = st.tensors.get(name)
            if t is None:
                raise ModelError(f"missing tensor {name}")
            if t.size != int(np.prod(shape)):
                raise ModelError(f"tensor {name} has shape {list(t.shape)}, expected {list(shape)}")
            a = np.ascontiguousarray(t.reshape(-1), np.float32)
            self._keep.append(a)
            return a

        h, q, kv, ff = c.hidden_size, c.q_dim, c.kv_dim, c.intermediate_size
        self.embed = take(embed_name, (c.vocab_size, h))
        self.ptr = lib().or_model_new(c.vocab_size, h, ff, c.num_layers, c.num_heads, c.num_kv_heads, c.head_dim,
                                      c.max_seq_len, c.rms_norm_eps, c.rope_theta, 1 if c.activation == "gelu" else 0)
        self.layers = []
        for i in range(c.num_layers):
            p = f"model.layers.{i}"
            L = dict(
                attn_norm=take(f"{p}.input_layernorm.weight", (h,)),
                wq=take(f"{p}.self_attn.q_proj.weight", (q, h)),
                bq=take(f"{p}.self_attn.q_proj.bias", (q,)) if has_bias else None,
                wk=take(f"{p}.self_attn.k_proj.weight", (kv, h)),
                bk=take(f"{p}.self_attn.k_proj.bias", (kv,)) if has_bias else None,
                wv=take(f"{p}.self_attn.v_proj.weight", (kv, h)),
                bv=take(f"{p}.self_attn.v_proj.bias", (kv,)) if has_bias else None,
                wo=take(f"{p}.self_attn.o_proj.weight", (h, q)),
                ffn_norm=take(f"{p}.post_attention_layernorm.weight", (h,)),
                w_gate=take(f"{p}.mlp.gate_proj.weight", (ff, h)),
                w_up=take(f"{p}.mlp.up_proj.weight", (ff, h)),
                w_down=take(f"{p}.mlp.down_proj.weight", (h, ff)),
            )
            self.layers.append(L)
            lib().or_model_set_layer(self.ptr, i, *[fp(L[k]) for k in (
                "attn_norm", "wq", "bq", "wk", "bk", "wv", "bv", "wo", "ffn_norm", "w_gate", "w_up", "w_down")])
        self.norm = take("model.norm.weight", (h,))
        self.lm_head = None if c.tie_word_embeddings else take("lm_head.weight", (c.vocab_size, h))
        lib().or_model_set_globals(self.ptr, fp(self.embed), fp(self.norm), fp(self.lm_head))

    def __del__(self):
        p = getattr(self, "ptr", None)
        if p:
            lib().or_model_free(p)
            self.ptr = None

    @staticmethod
    def load(path: str) -> "Model":
        """model.rs:286-299."""
        st = SafeTensors.load(path)
        s = st.meta("defer.config")
        if s is not None:
            v = dict(json.loads(s))
        else:
            p = os.path.join(os.path.dirname(path), "config.json")
            try:
                with open(p) as f:
                    v = json.load(f)
            except OSError:
                v = {}
        return Model(Config.from_json(v, st), st)

    def inv_freq(self) -> np.ndarray:
        p = lib().or_model_inv_freq(self.ptr)
        return np.ctypeslib.as_array(p, shape=(self.config.head_dim // 2,)).copy()

    def rope_tables(self, pos: int):
        half = self.config.head_dim // 2
        cs = np.zeros(half, np.float32)
        sn = np.zeros(half, np.float32)
        lib().or_rope_tables(self.ptr, pos, fp(cs), fp(sn))
        return cs, sn

    def new_cache(self, cap: Optional[int] = None) -> KvCache:
        return KvCache(self, cap)

    def forward_ext(self, token: int, cache: KvCache, masked: Sequence[int] = ()) -> np.ndarray:
        logits = np.zeros(self.config.vocab_size, np.float32)
        m = (ctypes.c_size_t * max(len(masked), 1))(*masked)
        err = ctypes.create_string_buffer(256)
        rc = lib().or_forward(self.ptr, cache.ptr, token, m, len(masked), fp(logits), err, 256)
        if rc != 0:
            raise ModelError(err.value.decode())
        return logits

    def forward(self, token: int, cache: KvCache) -> np.ndarray:
        return self.forward_ext(token, cache, ())


# ------------------------------------------------------------ checkpoint.rs
@dataclass
class DeferCheckpoint:
    model_signature: bytes
    base_seed: bytes
    temperature: float
    history_tokens: List[int]
    prompt_len: int
    rng_word_pos: int

    def generated_tokens(self):
        return self.history_tokens[self.prompt_len:]

    def to_bytes(self) -> bytes:
        """checkpoint.rs:44-60."""
        b = bytearray(b"DEFERCKP")
        b += struct.pack("<I", 1)
        b += self.model_signature + self.base_seed
        b += struct.pack("<f", self.temperature)
        b += struct.pack("<I", self.prompt_len)
        b += self.rng_word_pos.to_bytes(16, "little")
        b += struct.pack("<Q", len(self.history_tokens))
        for t in self.history_tokens:
            b += struct.pack("<I", t)
        b += struct.pack("<I", crc32(bytes(b)))
        return bytes(b)

    @staticmethod
    def from_bytes(b: bytes) -> "DeferCheckpoint":
        """checkpoint.rs:62-90."""
        FIXED = 8 + 4 + 32 + 32 + 4 + 4 + 16 + 8
        if len(b) < FIXED + 4 or b[:8] != b"DEFERCKP":
            raise CheckpointError("not a defer checkpoint")
        body, tail = b[:-4], b[-4:]
        if crc32(body) != struct.unpack("<I", tail)[0]:
            raise CheckpointError("checksum mismatch (file corrupt)")
        if struct.unpack_from("<I", body, 8)[0] != 1:
            raise CheckpointError("unsupported checkpoint version")
        sig = body[12:44]
        seed = body[44:76]
        temp = struct.unpack_from("<f", body, 76)[0]
        plen = struct.unpack_from("<I", body, 80)[0]
        rng = int.from_bytes(body[84:100], "little")
        n = struct.unpack_from("<Q", body, 100)[0]
        if len(body) != FIXED + 4 * n:
            raise CheckpointError("length mismatch")
        toks = list(struct.unpack_from(f"<{n}I", body, 108))
        if plen > n:
            raise CheckpointError("prompt_len exceeds history length")
        return DeferCheckpoint(sig, seed, temp, toks, plen, rng)


# ------------------------------------------------------------------ wal.rs
RECORD_SIZE = 29


@dataclass
class WalHeader:
    model_signature: bytes
    base_seed: bytes
    temperature: float
    prompt_len: int
    start_rng_word_pos: int
    prefix_tokens: List[int]

    def to_bytes(self) -> bytes:
        """wal.rs:55-71."""
        b = bytearray(b"DEFERWAL")
        b += struct.pack("<I", 1)
        b += self.model_signature + self.base_seed
        b += struct.pack("<f", self.temperature)
        b += struct.pack("<I", self.prompt_len)
        b += self.start_rng_word_pos.to_bytes(16, "little")
        b += struct.pack("<I", len(self.prefix_tokens))
        for t in self.prefix_tokens:
            b += struct.pack("<I", t)
        b += struct.pack("<I", crc32(bytes(b)))
        return bytes(b)

    @staticmethod
    def from_checkpoint(c: DeferCheckpoint) -> "WalHeader":
        return WalHeader(c.model_signature, c.base_seed, c.temperature, c.prompt_len, c.rng_word_pos,
                         list(c.history_tokens))


def wal_record_bytes(step: int, token: int, rng_word_pos: int) -> bytes:
    """wal.rs:94-103."""
    b = bytes([1]) + struct.pack("<II", step, token) + rng_word_pos.to_bytes(16, "little")
    return b + struct.pack("<I", crc32(b))


@dataclass
class WalLog:
    header: WalHeader
    records: List[tuple]
    valid_len: int
    torn_tail: bool

    @staticmethod
    def parse(b: bytes) -> "WalLog":
        """wal.rs:123-194."""
        FIXED = 8 + 4 + 32 + 32 + 4 + 4 + 16 + 4
        if len(b) < FIXED + 4 or b[:8] != b"DEFERWAL":
            raise WalError("not a defer WAL")
        if struct.unpack_from("<I", b, 8)[0] != 1:
            raise WalError("unsupported WAL version")
        sig, seed = b[12:44], b[44:76]
        temp = struct.unpack_from("<f", b, 76)[0]
        plen = struct.unpack_from("<I", b, 80)[0]
        start = int.from_bytes(b[84:100], "little")
        n = struct.unpack_from("<I", b, 100)[0]
        hend = FIXED + 4 * n
        if len(b) < hend + 4:
            raise WalError("truncated WAL header")
        prefix = list(struct.unpack_from(f"<{n}I", b, 104))
        if crc32(b[:hend]) != struct.unpack_from("<I", b, hend)[0]:
            raise WalError("WAL header checksum mismatch")
        hdr = WalHeader(sig, seed, temp, plen, start, prefix)
        if plen > n:
            raise WalError("prompt_len exceeds prefix length")
        recs = []
        off = hend + 4
        exp_step, exp_rng = n, start
        torn = False
        while off < len(b):
            if len(b) - off < RECORD_SIZE:
                torn = True
                break
            r = b[off:off + RECORD_SIZE]
            if r[0] != 1 or crc32(r[:25]) != struct.unpack_from("<I", r, 25)[0]:
                torn = True
                break
            step, tok = struct.unpack_from("<II", r, 1)
            rng = int.from_bytes(r[9:25], "little")
            exp_rng += words_per_sample(temp)
            if step != exp_step or rng != exp_rng:
                raise WalError(f"record {len(recs)} is inconsistent (step {step} / rng {rng}, expected "
                               f"{exp_step} / {exp_rng})")
            exp_step += 1
            recs.append((step, tok, rng))
            off += RECORD_SIZE
        return WalLog(hdr, recs, off, torn)

    def to_checkpoint(self) -> DeferCheckpoint:
        h = self.header
        return DeferCheckpoint(h.model_signature, h.base_seed, h.temperature,
                               list(h.prefix_tokens) + [r[1] for r in self.records], h.prompt_len,
                               self.records[-1][2] if self.records else h.start_rng_word_pos)


# --------------------------------------------------------------- engine.rs
class Session:
    """engine.rs:23-274 (tracing paths excluded)."""

    def __init__(self, model: Model, base_seed: bytes, temperature: float, cache_cap: Optional[int] = None):
        if not (temperature >= 0.0 and math.isfinite(temperature)):
            raise ModelError("temperature must be finite and >= 0")
        self.model = model
        self.cache = model.new_cache(cache_cap)
        self.rng = ChaCha8Rng(base_seed)
        self.base_seed = bytes(base_seed)
        self.temperature = float(np.float32(temperature))
        self.history: List[int] = []
        self.prompt_len = 0
        self.logits: Optional[np.ndarray] = None

    def prompt(self, tokens: Sequence[int]):
        if len(self.history) != self.prompt_len:
            raise ModelError("cannot add prompt tokens after generation started")
        for t in tokens:
            self.feed(t)
        self.prompt_len = len(self.history)

    def feed(self, token: int):
        self.logits = self.model.forward(token, self.cache)
        self.history.append(token)

    def sample(self) -> int:
        if self.logits is None:
            raise ModelError("no context: provide a non-empty prompt")
        return sample_token(self.logits, self.temperature, self.rng)

    def step(self) -> int:
        t = self.sample()
        self.feed(t)
        return t

    def generate(self, max_tokens: int, stop: Sequence[int] = (),
                 on_token: Optional[Callable[["Session", int], None]] = None) -> List[int]:
        out = []
        for _ in range(max_tokens):
            t = self.step()
            out.append(t)
            if on_token:
                on_token(self, t)
            if t in stop:
                break
        return out

    def generated(self):
        return self.history[self.prompt_len:]

    def rng_word_pos(self) -> int:
        return self.rng.get_word_pos()

    def checkpoint(self) -> DeferCheckpoint:
        return DeferCheckpoint(self.model.signature, self.base_seed, self.temperature, list(self.history),
                               self.prompt_len, self.rng_word_pos())

    @staticmethod
    def checkout(model: Model, ck: DeferCheckpoint, cache_cap: Optional[int] = None) -> "Session":
        """engine.rs:241-274."""
        if ck.model_signature != model.signature:
            raise CheckpointError(f"model signature mismatch: checkpoint {ck.model_signature.hex()} vs loaded "
                                  f"{model.signature.hex()}")
        plen = ck.prompt_len
        if plen > len(ck.history_tokens):
            raise CheckpointError("prompt_len exceeds history")
        expected = (len(ck.history_tokens) - plen) * words_per_sample(ck.temperature)
        if ck.rng_word_pos != expected:
            raise CheckpointError(f"rng_word_pos {ck.rng_word_pos} inconsistent with "
                                  f"{len(ck.history_tokens) - plen} sampled tokens (expected {expected})")
        s = Session(model, ck.base_seed, ck.temperature, cache_cap)
        s.prompt(ck.history_tokens[:plen])
        for i in range(plen, len(ck.history_tokens)):
            rec = ck.history_tokens[i]
            got = s.sample()
            if got != rec:
                raise DivergenceError(f"replay sampled token {got} at position {i}, checkpoint recorded {rec}")
            s.feed(rec)
        return s


# ---------------------------------------------------------- attribution.rs
def log_softmax_at(logits, idx: int) -> float:
    a = np.ascontiguousarray(logits, np.float32)
    return lib().or_log_softmax_at(fp(a), a.size, idx)


def ablation_attribution(model: Model, context: Sequence[int], target: int, positions: Sequence[int]):
    """attribution.rs:224-264 — returns (base_logprob, [(p, token, ablated, delta)])."""
    n = len(context)
    if n == 0:
        raise ModelError("cannot ablate an empty context")
    if target >= model.config.vocab_size:
        raise ModelError(f"target token {target} out of range")
    for p in positions:
        if p + 1 >= n:
            raise ModelError(f"position {p} can not be ablated (must be < {n - 1}; the query token itself is "
                             "excluded)")
    full = model.new_cache(n)
    base = None
    for t in context:
        base = model.forward(t, full)
    base_lp = log_softmax_at(base, target)
    scores = []
    for p in positions:
        cache = full.clone()
        cache.truncate(p + 1)
        logits = None
        for t in context[p + 1:]:
            logits = model.forward_ext(t, cache, [p])
        lp = log_softmax_at(logits, target)
        scores.append((p, context[p], lp, base_lp - lp))
    return base_lp, scores


# ---------------------------------------------------------- synthetic.rs
def tiny_config() -> Config:
    """synthetic.rs:12-29."""
    return Config(256, 64, 160, 2, 4, 2, 16, float(np.float32(1e-5)), 10000.0, 1024, False, "silu")


def write_tiny_model(path: str, config: Config, seed: int) -> None:
    """synthetic.rs:32-59 — ChaCha8 gen_range(-1,1) * 1.7/sqrt(fan_in)."""
    rng = ChaCha8Rng.seed_from_u64(seed)
    c = config

    def mat(rows, cols, scale):
        scale = np.float32(scale)
        vals = np.empty(rows * cols, np.float32)
        for i in range(rows * cols):
            vals[i] = np.float32(rng.gen_range_f32(-1.0, 1.0)) * scale
        return vals

    def s(fan_in):
        return np.float32(1.7) / np.sqrt(np.float32(fan_in))

    h, q, kv, ff, v = c.hidden_size, c.q_dim, c.kv_dim, c.intermediate_size, c.vocab_size
    t = [("model.embed_tokens.weight", [v, h], mat(v, h, 1.0))]
    for i in range(c.num_layers):
        p = f"model.layers.{i}"
        t.append((f"{p}.input_layernorm.weight", [h], np.ones(h, np.float32)))
        t.append((f"{p}.self_attn.q_proj.weight", [q, h], mat(q, h, s(h))))
        t.append((f"{p}.self_attn.k_proj.weight", [kv, h], mat(kv, h, s(h))))
        t.append((f"{p}.self_attn.v_proj.weight", [kv, h], mat(kv, h, s(h))))
        t.append((f"{p}.self_attn.o_proj.weight", [h, q], mat(h, q, s(q))))
        t.append((f"{p}.post_attention_layernorm.weight", [h], np.ones(h, np.float32)))
        t.append((f"{p}.mlp.gate_proj.weight", [ff, h], mat(ff, h, s(h))))
        t.append((f"{p}.mlp.up_proj.weight", [ff, h], mat(ff, h, s(h))))
        t.append((f"{p}.mlp.down_proj.weight", [h, ff], mat(h, ff, s(ff))))
    t.append(("model.norm.weight", [h], np.ones(h, np.float32)))
    if not c.tie_word_embeddings:
        t.append(("lm_head.weight", [v, h], mat(v, h, np.float32(3.0) * s(h))))
    write_safetensors(path, t, [("defer.config", c.to_json())])
