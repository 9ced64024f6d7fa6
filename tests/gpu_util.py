"""Helpers shared by the GPU parity tests: model fixtures and the
tolerances of the parity contract.

Tolerances (fp32 on both sides, different summation orders):
  * logits: max |gpu - cpu| <= 1e-4 * (max - min of the cpu logits)
  * KV entries: max |gpu - cpu| <= 1e-5 * max |cpu| per layer and K/V
  * tokens: identical, except where the CPU sampler's decision sits within
    rounding distance of a boundary (greedy top-2 gap or the CDF margin of r)
"""
import os

import numpy as np

from defer_b200 import synthetic
from oracle import oracle as O

LOGIT_TOL = 1e-4
KV_TOL = 1e-5


def model_file(directory: str, name: str, seed: int = 0) -> str:
    if name == "tiny":
        p = os.path.join(directory, f"tiny-{seed}.safetensors")
        if not os.path.exists(p):
            synthetic.write_tiny_model(p, seed)
        return p
    return synthetic.model_path(name, directory, seed)


def logits_close(gpu: np.ndarray, cpu: np.ndarray):
    rng = float(cpu.max() - cpu.min())
    err = float(np.abs(gpu.astype(np.float64) - cpu.astype(np.float64)).max())
    return err <= LOGIT_TOL * rng, err, rng


def kv_close(gpu_cache, cpu_cache, layers: int):
    worst = 0.0
    for l in range(layers):
        kg, vg = gpu_cache.layer(l)
        ko, vo = cpu_cache.keys(l), cpu_cache.values(l)
        for g, o in ((kg, ko), (vg, vo)):
            if o.size == 0:
                continue
            scale = float(np.abs(o).max()) or 1.0
            worst = max(worst, float(np.abs(g.astype(np.float64) - o).max()) / scale)
    return worst <= KV_TOL, worst


def greedy_gap(logits: np.ndarray) -> float:
    """Distance between the two largest logits (how close argmax is to a tie)."""
    a = np.sort(logits[~np.isnan(logits)])
    return float(a[-1] - a[-2]) if a.size > 1 else float("inf")


def cdf_margin(logits: np.ndarray, t: float, word: int) -> float:
    """Distance of r to the nearest CDF edge of the CPU sampler's choice."""
    if t == 0.0:
        return greedy_gap(logits)
    p = O.softmax_with_temperature(logits, t).astype(np.float64)
    c = np.cumsum(p)
    r = float(O.unit_f32(word))
    i = int(np.searchsorted(c, r, side="right"))
    lo = c[i - 1] if i > 0 else 0.0
    hi = c[i] if i < c.size else c[-1]
    return min(abs(hi - r), abs(r - lo))
