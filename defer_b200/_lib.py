"""ctypes binding of include/defer_b200.h (libdefer_b200.so, built in-tree).

There is no fallback: if the library is missing the import fails loudly.
"""
from __future__ import annotations

import ctypes
import os

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libdefer_b200.so")

c_u8p = ctypes.POINTER(ctypes.c_uint8)
c_u32p = ctypes.POINTER(ctypes.c_uint32)
c_f32p = ctypes.POINTER(ctypes.c_float)
c_f64p = ctypes.POINTER(ctypes.c_double)
c_szp = ctypes.POINTER(ctypes.c_size_t)
c_i32p = ctypes.POINTER(ctypes.c_int32)
vp = ctypes.c_void_p
sz = ctypes.c_size_t


class DeferConfig(ctypes.Structure):
    _fields_ = [(n, ctypes.c_uint32) for n in (
        "vocab_size", "hidden_size", "intermediate_size", "num_layers",
        "num_heads", "num_kv_heads", "head_dim", "max_seq_len")] + [
        ("rms_norm_eps", ctypes.c_float), ("rope_theta", ctypes.c_float),
        ("tie_word_embeddings", ctypes.c_int32), ("gelu", ctypes.c_int32),
        ("has_bias", ctypes.c_int32), ("weights_bf16", ctypes.c_int32),
        ("bos_token_id", ctypes.c_int64), ("weight_bytes", ctypes.c_uint64),
        ("device", ctypes.c_int32), ("sm_count", ctypes.c_int32)]


class CheckpointFields(ctypes.Structure):
    _fields_ = [("model_signature", ctypes.c_uint8 * 32), ("base_seed", ctypes.c_uint8 * 32),
                ("temperature", ctypes.c_float), ("prompt_len", ctypes.c_uint32),
                ("rng_word_pos_lo", ctypes.c_uint64), ("rng_word_pos_hi", ctypes.c_uint64),
                ("history_tokens", c_u32p), ("n_tokens", sz)]


class WalHeaderC(ctypes.Structure):
    _fields_ = [("model_signature", ctypes.c_uint8 * 32), ("base_seed", ctypes.c_uint8 * 32),
                ("temperature", ctypes.c_float), ("prompt_len", ctypes.c_uint32),
                ("start_rng_word_pos_lo", ctypes.c_uint64), ("start_rng_word_pos_hi", ctypes.c_uint64),
                ("prefix_tokens", c_u32p), ("n_prefix", sz)]


TOKEN_CB = ctypes.CFUNCTYPE(ctypes.c_int, vp, ctypes.c_uint32, ctypes.c_uint64)

# (name, restype, argtypes) of every entry point declared in the header.
SIGNATURES = [
    ("defer_last_error", ctypes.c_char_p, []),
    ("defer_model_load", ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(vp)]),
    ("defer_model_free", None, [vp]),
    ("defer_model_config", ctypes.c_int, [vp, ctypes.POINTER(DeferConfig)]),
    ("defer_model_signature", ctypes.c_int, [vp, c_u8p]),
    ("defer_model_eos_tokens", ctypes.c_int, [vp, c_u32p, sz, c_szp]),
    ("defer_forward", ctypes.c_int, [vp, vp, ctypes.c_uint32, c_szp, sz, c_f32p]),
    ("defer_forward_noalloc", ctypes.c_int, [vp, vp, vp, ctypes.c_uint32, ctypes.c_uint32, ctypes.c_uint32, vp,
                                             vp]),
    ("defer_cache_new", ctypes.c_int, [vp, ctypes.c_uint32, ctypes.POINTER(vp)]),
    ("defer_cache_free", None, [vp]),
    ("defer_cache_len", sz, [vp]),
    ("defer_cache_truncate", ctypes.c_int, [vp, sz]),
    ("defer_cache_clone", ctypes.c_int, [vp, ctypes.POINTER(vp)]),
    ("defer_cache_download", ctypes.c_int, [vp, ctypes.c_uint32, c_f32p, c_f32p]),
    ("defer_cache_fingerprint", ctypes.c_int, [vp, c_u8p]),
    ("defer_cache_bit_eq", ctypes.c_int, [vp, vp, ctypes.POINTER(ctypes.c_int)]),
    ("defer_seed_from_u64", None, [ctypes.c_uint64, c_u8p]),
    ("defer_chacha8_words", ctypes.c_int, [c_u8p, ctypes.c_uint64, sz, c_u32p]),
    ("defer_words_per_sample", ctypes.c_uint64, [ctypes.c_float]),
    ("defer_sample_logits", ctypes.c_int, [ctypes.c_int, c_f32p, sz, ctypes.c_float, ctypes.c_uint32, c_u32p,
                                           c_f32p]),
    ("defer_session_new", ctypes.c_int, [vp, c_u8p, ctypes.c_float, ctypes.POINTER(vp)]),
    ("defer_session_free", None, [vp]),
    ("defer_session_prompt", ctypes.c_int, [vp, c_u32p, sz]),
    ("defer_session_step", ctypes.c_int, [vp, c_u32p]),
    ("defer_session_generate", ctypes.c_int, [vp, sz, c_u32p, sz, TOKEN_CB, vp, c_u32p, c_szp]),
    ("defer_session_checkout", ctypes.c_int, [vp, c_u8p, sz, ctypes.POINTER(vp)]),
    ("defer_session_checkpoint", ctypes.c_int, [vp, c_u8p, sz, c_szp]),
    ("defer_session_history", ctypes.c_int, [vp, c_u32p, sz, c_szp]),
    ("defer_session_prompt_len", sz, [vp]),
    ("defer_session_rng_word_pos", ctypes.c_uint64, [vp]),
    ("defer_session_last_logits", ctypes.c_int, [vp, c_f32p]),
    ("defer_session_cache", vp, [vp]),
    ("defer_session_margins", ctypes.c_int, [vp, c_f32p, sz, c_szp]),
    ("defer_checkpoint_encode", ctypes.c_int, [ctypes.POINTER(CheckpointFields), c_u8p, sz, c_szp]),
    ("defer_checkpoint_decode", ctypes.c_int, [c_u8p, sz, ctypes.POINTER(CheckpointFields), c_u32p, sz]),
    ("defer_checkpoint_save", ctypes.c_int, [c_u8p, sz, ctypes.c_char_p]),
    ("defer_checkpoint_load", ctypes.c_int, [ctypes.c_char_p, c_u8p, sz, c_szp]),
    ("defer_wal_create", ctypes.c_int, [ctypes.c_char_p, ctypes.POINTER(WalHeaderC), ctypes.c_int,
                                        ctypes.POINTER(vp)]),
    ("defer_wal_resume", ctypes.c_int, [ctypes.c_char_p, ctypes.c_int, ctypes.POINTER(vp)]),
    ("defer_wal_append", ctypes.c_int, [vp, ctypes.c_uint32, ctypes.c_uint64, ctypes.c_uint64]),
    ("defer_wal_close", None, [vp]),
    ("defer_wal_to_checkpoint", ctypes.c_int, [c_u8p, sz, c_u8p, sz, c_szp, c_szp, ctypes.POINTER(ctypes.c_int),
                                               ctypes.POINTER(ctypes.c_uint64)]),
    ("defer_verify", ctypes.c_int, [vp, c_u8p, ctypes.c_float, c_u32p, sz, ctypes.c_uint32, sz, c_u32p, sz, c_u32p,
                                    c_szp, c_u8p]),
    ("defer_replay_batch", ctypes.c_int, [vp, ctypes.POINTER(c_u8p), c_szp, sz, ctypes.c_int, c_i32p, c_i32p,
                                          c_u32p, c_u8p, c_f64p]),
    ("defer_generate_batch", ctypes.c_int, [vp, ctypes.POINTER(c_u32p), c_szp, c_u8p, c_f32p, c_szp, sz,
                                            ctypes.c_int, ctypes.POINTER(c_u32p), c_szp, c_f64p]),
    ("defer_ablation", ctypes.c_int, [vp, c_u32p, sz, ctypes.c_uint32, c_szp, sz, ctypes.c_int, c_f64p, c_f64p]),
    ("defer_model_timing", ctypes.c_int, [vp, c_f64p, ctypes.POINTER(ctypes.c_uint64),
                                          ctypes.POINTER(ctypes.c_uint64), ctypes.POINTER(ctypes.c_uint64), c_f64p,
                                          ctypes.c_int]),
    ("defer_debug_trace_arm", ctypes.c_int, [vp, ctypes.c_int32]),
    ("defer_debug_trace_read", ctypes.c_int, [vp, ctypes.POINTER(ctypes.c_uint64), sz, c_szp, c_i32p, c_i32p]),
    ("defer_debug_stall", ctypes.c_int, [vp, ctypes.c_uint32]),
    ("defer_debug_tc_gemm", ctypes.c_int, [ctypes.c_int, c_f32p, ctypes.c_uint32, c_f32p, ctypes.c_uint32,
                                           ctypes.c_uint32, ctypes.c_int32, c_f32p]),
    ("defer_log_softmax_at", ctypes.c_double, [c_f32p, sz, sz]),
]

_lib = None


def load() -> ctypes.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m defer_b200.build` "
                              "(there is no CPU fallback)")
        L = ctypes.CDLL(LIB_PATH)
        for name, res, args in SIGNATURES:
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib
