"""CPU oracle runs of the benchmark-config parity tests (test
infrastructure). Each function runs in a spawned worker process, so the
long single-threaded oracle runs of several configurations overlap each
other and the GPU work of the tests."""
from __future__ import annotations

import os
import sys

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _oracle():
    if ROOT not in sys.path:
        sys.path.insert(0, ROOT)
    from oracle import oracle as O
    return O


def _kv(O, cache, layers):
    return [(cache.keys(l).copy(), cache.values(l).copy()) for l in range(layers)]


def greedy_run(path, prompt, n):
    """Oracle session at T = 0 (sampler.rs:24-40 argmax): the generated
    tokens, the logits after every fed token and the final KV cache."""
    O = _oracle()
    m = O.Model.load(path)
    c = m.new_cache(len(prompt) + n + 1)
    logits = []
    lo = None
    for t in prompt:
        lo = m.forward(t, c)
        logits.append(lo)
    toks = []
    for _ in range(n):
        t = O.argmax(lo)
        toks.append(int(t))
        lo = m.forward(t, c)
        logits.append(lo)
    return toks, np.stack(logits), _kv(O, c, m.config.num_layers)


def edge_report(O, lo, t, word, got):
    """Where the oracle's sampler (sequential fp32 CDF, sampler.rs:95-104)
    chooses another token than `got`: both choices, the distance of r to the
    sequential fp32 CDF edge between them (seq_edge), to the exact float64
    edge, and how far the sequential CDF has drifted from the exact one."""
    want = int(O.sample_token_word(lo, t, word))
    if want == got:
        return None
    s = lo.astype(np.float32) / np.float32(t)
    s64 = s.astype(np.float64)
    e64 = np.where(np.isnan(s64), 0.0, np.exp(s64 - np.nanmax(s64)))
    c_exact = np.cumsum(e64 / e64.sum())
    e32 = np.where(np.isnan(s), np.float32(0), np.exp(s - np.nanmax(s))).astype(np.float32)
    z32 = np.add.accumulate(e32, dtype=np.float32)[-1]
    p32 = e32 * (np.float32(1.0) / z32)
    c_seq = np.add.accumulate(p32, dtype=np.float32).astype(np.float64)
    r = float(O.unit_f32(word))
    k = min(want, got)
    return {"oracle": want, "gpu": got, "edge": abs(r - c_exact[k]), "drift": abs(c_seq[k] - c_exact[k]),
            "seq_edge": abs(r - c_seq[k])}


def teacher_forced(path, tokens, n_prompt, t, seed, check_steps, want_kv):
    """Feeds the recorded `tokens` (a GPU session's history) through the
    oracle, as Session::checkout does (engine.rs:241-274) but without
    stopping: at every generated position the oracle samples with the
    session's PRNG word, and every choice that differs from the recorded
    token is reported (edge_report). Returns the reports, the logits after
    the fed positions listed in check_steps, and the final KV if asked."""
    O = _oracle()
    m = O.Model.load(path)
    c = m.new_cache(len(tokens) + 1)
    words = O.keystream_words(seed, 0, max(len(tokens) - n_prompt, 1))
    checks = set(check_steps)
    kept = {}
    reports = []
    lo = None
    for i, tok in enumerate(tokens):
        if i >= n_prompt:
            r = edge_report(O, lo, t, int(words[i - n_prompt]), int(tok))
            if r is not None:
                r["step"] = i
                reports.append(r)
        lo = m.forward(int(tok), c)
        if i in checks:
            kept[i] = lo.copy()
    kv = _kv(O, c, m.config.num_layers) if want_kv else None
    return reports, kept, kv


def ablation(path, context, target, positions):
    """attribution.rs:224-264 on the oracle: base log-probability, the
    ablated ones, and the base logits."""
    O = _oracle()
    m = O.Model.load(path)
    base, scores = O.ablation_attribution(m, context, target, positions)
    c = m.new_cache(len(context))
    lo = None
    for t in context:
        lo = m.forward(t, c)
    return base, [s[2] for s in scores], lo
