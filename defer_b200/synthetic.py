"""Synthetic Llama weights for tests and benchmarks (no checkpoints are
available offline).

* ``write_normal_model``: every matrix and embedding N(0, 0.02) in fp32 (or
  rounded to bf16 and stored BF16), RMSNorm weights 1.0 (as in HF init and
  the reference's src/synthetic.rs:44,49,54). Tensor i (file order) is drawn
  from numpy's PCG64 stream seeded with (seed, i), so tensors can be made in
  parallel and regenerated independently.
* ``write_tiny_model``: the reference's test model (src/synthetic.rs:12-59):
  ChaCha8 ``gen_range(-1, 1) * 1.7 / sqrt(fan_in)`` weights, written in the
  reference's safetensors layout with the config in ``defer.config``.

The named shapes are the ones the benchmark configurations use.
"""
from __future__ import annotations

import json
import os
import struct
from concurrent.futures import ThreadPoolExecutor
from dataclasses import dataclass

import numpy as np


@dataclass
class Shape:
    vocab_size: int
    hidden_size: int
    intermediate_size: int
    num_layers: int
    num_heads: int
    num_kv_heads: int
    head_dim: int
    rope_theta: float
    tie_word_embeddings: bool
    rms_norm_eps: float = 1e-5
    max_position_embeddings: int = 4096
    bf16: bool = False

    def config_json(self) -> str:
        return json.dumps({
            "architectures": ["LlamaForCausalLM"], "vocab_size": self.vocab_size,
            "hidden_size": self.hidden_size, "intermediate_size": self.intermediate_size,
            "num_hidden_layers": self.num_layers, "num_attention_heads": self.num_heads,
            "num_key_value_heads": self.num_kv_heads, "head_dim": self.head_dim,
            "rms_norm_eps": self.rms_norm_eps, "rope_theta": self.rope_theta,
            "max_position_embeddings": self.max_position_embeddings,
            "tie_word_embeddings": self.tie_word_embeddings, "hidden_act": "silu"}, separators=(",", ":"))

    def params(self) -> int:
        h, q, kv, ff, v = (self.hidden_size, self.num_heads * self.head_dim, self.num_kv_heads * self.head_dim,
                           self.intermediate_size, self.vocab_size)
        per = 2 * h + q * h + 2 * kv * h + h * q + 3 * ff * h
        return v * h * (1 if self.tie_word_embeddings else 2) + self.num_layers * per + h


SHAPES = {
    # SmolLM2-135M shape (configs 1-3)
    "smollm2-135m": Shape(49152, 576, 1536, 30, 9, 3, 64, 100000.0, True, max_position_embeddings=4097),
    # SmolLM2-1.7B shape (config 4)
    "smollm2-1.7b": Shape(49152, 2048, 8192, 24, 32, 32, 64, 130000.0, True, max_position_embeddings=4097),
    # Llama-3-8B shape, bf16-stored (config 5)
    "llama3-8b": Shape(128256, 4096, 14336, 32, 32, 8, 128, 500000.0, False, max_position_embeddings=4097,
                       bf16=True),
    # the 8B shape's widths with 2 layers (parity tests of config 5's arithmetic)
    "test-8b-width": Shape(128256, 4096, 14336, 2, 32, 8, 128, 500000.0, False, max_position_embeddings=4097,
                           bf16=True),
    # small shapes for fast tests
    "test-small": Shape(512, 128, 352, 3, 4, 2, 32, 10000.0, True, max_position_embeddings=1024),
    "test-gqa4": Shape(1000, 256, 512, 2, 8, 2, 32, 500000.0, False, max_position_embeddings=512),
    "test-bf16": Shape(768, 256, 512, 2, 4, 1, 64, 10000.0, False, max_position_embeddings=512, bf16=True),
}


def tensor_list(s: Shape):
    """(name, shape, kind) in file order; kind is 'normal' or 'ones'."""
    h, q, kv, ff, v = (s.hidden_size, s.num_heads * s.head_dim, s.num_kv_heads * s.head_dim,
                       s.intermediate_size, s.vocab_size)
    t = [("model.embed_tokens.weight", (v, h), "normal")]
    for i in range(s.num_layers):
        p = f"model.layers.{i}"
        t += [(f"{p}.input_layernorm.weight", (h,), "ones"),
              (f"{p}.self_attn.q_proj.weight", (q, h), "normal"),
              (f"{p}.self_attn.k_proj.weight", (kv, h), "normal"),
              (f"{p}.self_attn.v_proj.weight", (kv, h), "normal"),
              (f"{p}.self_attn.o_proj.weight", (h, q), "normal"),
              (f"{p}.post_attention_layernorm.weight", (h,), "ones"),
              (f"{p}.mlp.gate_proj.weight", (ff, h), "normal"),
              (f"{p}.mlp.up_proj.weight", (ff, h), "normal"),
              (f"{p}.mlp.down_proj.weight", (h, ff), "normal")]
    t.append(("model.norm.weight", (h,), "ones"))
    if not s.tie_word_embeddings:
        t.append(("lm_head.weight", (v, h), "normal"))
    return t


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even fp32 -> bf16 bit patterns (finite inputs)."""
    u = np.ascontiguousarray(a, np.float32).view(np.uint32)
    r = ((u >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    return ((u + r) >> np.uint32(16)).astype(np.uint16)


def _make(seed: int, idx: int, shape, kind: str, bf16: bool) -> bytes:
    n = int(np.prod(shape))
    if kind == "ones":
        a = np.ones(n, np.float32)
    else:
        g = np.random.Generator(np.random.PCG64([seed, idx]))
        a = g.standard_normal(n, dtype=np.float32)
        a *= np.float32(0.02)
    if bf16:
        return f32_to_bf16_bits(a).astype("<u2").tobytes()
    return a.astype("<f4").tobytes()


def write_normal_model(path: str, shape: Shape, seed: int = 0, threads: int = 0) -> str:
    """Writes the safetensors file (config in `defer.config`); returns path."""
    tl = tensor_list(shape)
    dt, esz = ("BF16", 2) if shape.bf16 else ("F32", 4)
    entries = {"__metadata__": {"defer.config": shape.config_json()}}
    off = 0
    for name, shp, _ in tl:
        n = int(np.prod(shp)) * esz
        entries[name] = {"dtype": dt, "shape": list(shp), "data_offsets": [off, off + n]}
        off += n
    header = json.dumps(entries, separators=(",", ":"))
    header += " " * ((8 - len(header) % 8) % 8)
    hb = header.encode()
    tmp = path + ".tmp"
    threads = threads or min(16, os.cpu_count() or 1)
    with open(tmp, "wb") as f, ThreadPoolExecutor(threads) as ex:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        futs = []
        for i, (name, shp, kind) in enumerate(tl):
            futs.append(ex.submit(_make, seed, i, shp, kind, shape.bf16))
            if len(futs) >= 2 * threads:
                f.write(futs.pop(0).result())
        for fu in futs:
            f.write(fu.result())
    os.replace(tmp, path)
    return path


def model_path(name: str, directory: str, seed: int = 0) -> str:
    """Path of the cached synthetic model `name`, writing it if absent."""
    os.makedirs(directory, exist_ok=True)
    p = os.path.join(directory, f"{name}-seed{seed}.safetensors")
    if not os.path.exists(p):
        write_normal_model(p, SHAPES[name], seed)
    return p


# ------------------------------------------------------------ tiny model
def _json_quote(s: str) -> str:
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


# Config::to_json of synthetic::tiny_config (src/model.rs:129-160,
# src/synthetic.rs:12-29).
TINY_CONFIG_JSON = ('{"architectures":["LlamaForCausalLM"],"vocab_size":256,"hidden_size":64,'
                    '"intermediate_size":160,"num_hidden_layers":2,"num_attention_heads":4,'
                    '"num_key_value_heads":2,"head_dim":16,"rms_norm_eps":1e-5,"rope_theta":10000,'
                    '"max_position_embeddings":1024,"tie_word_embeddings":false,"hidden_act":"silu"}')


def write_tiny_model(path: str, seed: int) -> str:
    """src/synthetic.rs:12-59 (tiny_config + write_model): one ChaCha8 word
    per weight, gen_range(-1, 1) = ((word >> 9 | 1.0f bits) - 1) * 2 - 1."""
    from . import chacha8_words, seed_from_u64

    h, q, kv, ff, v, L = 64, 64, 32, 160, 256, 2
    counts = [v * h]
    for _ in range(L):
        counts += [q * h, kv * h, kv * h, h * q, ff * h, ff * h, h * ff]
    counts.append(v * h)
    words = chacha8_words(seed_from_u64(seed), 0, sum(counts))
    one = ((words >> np.uint32(9)) | np.uint32(0x3F800000)).view(np.float32)
    unit = (one - np.float32(1.0)) * np.float32(2.0) + np.float32(-1.0)
    cur = [0]

    def mat(n, scale):
        a = unit[cur[0]:cur[0] + n] * np.float32(scale)
        cur[0] += n
        return a.astype(np.float32)

    def s(fan_in):
        return np.float32(1.7) / np.sqrt(np.float32(fan_in))

    t = [("model.embed_tokens.weight", [v, h], mat(v * h, 1.0))]
    for i in range(L):
        p = f"model.layers.{i}"
        t += [(f"{p}.input_layernorm.weight", [h], np.ones(h, np.float32)),
              (f"{p}.self_attn.q_proj.weight", [q, h], mat(q * h, s(h))),
              (f"{p}.self_attn.k_proj.weight", [kv, h], mat(kv * h, s(h))),
              (f"{p}.self_attn.v_proj.weight", [kv, h], mat(kv * h, s(h))),
              (f"{p}.self_attn.o_proj.weight", [h, q], mat(h * q, s(q))),
              (f"{p}.post_attention_layernorm.weight", [h], np.ones(h, np.float32)),
              (f"{p}.mlp.gate_proj.weight", [ff, h], mat(ff * h, s(h))),
              (f"{p}.mlp.up_proj.weight", [ff, h], mat(ff * h, s(h))),
              (f"{p}.mlp.down_proj.weight", [h, ff], mat(h * ff, s(ff)))]
    t.append(("model.norm.weight", [h], np.ones(h, np.float32)))
    t.append(("lm_head.weight", [v, h], mat(v * h, np.float32(3.0) * s(h))))
    # safetensors.rs:252-299 header layout
    parts = ['"__metadata__":{' + _json_quote("defer.config") + ":" + _json_quote(TINY_CONFIG_JSON) + "}"]
    off = 0
    for name, shp, data in t:
        n = int(np.prod(shp)) * 4
        parts.append(f'{_json_quote(name)}:{{"dtype":"F32","shape":[{",".join(map(str, shp))}],'
                     f'"data_offsets":[{off},{off + n}]}}')
        off += n
    header = "{" + ",".join(parts) + "}"
    header += " " * ((8 - len(header) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(header)))
        f.write(header.encode())
        for _, _, data in t:
            f.write(data.astype("<f4").tobytes())
    return path
