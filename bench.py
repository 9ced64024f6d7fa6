#!/usr/bin/env python
"""Benchmark of the B200 token loop on the reference's headline workload.

Workload (config 2): SmolLM2-135M-shape Llama, random-init fp32 weights
N(0, 0.02) from seed 0; one session per GPU at temperature 0.7 with ChaCha8
seed 42 (+ rank); a 32-token uniform-random prompt; decode to a 2048-token
context while appending every token to a WAL on the host; then a verified
checkout (replay with Divergence checks) of that WAL.

One step = that whole session loop: 32 prompt + 2016 generated + 2048
replayed = 4096 single-token forward passes (each with its sampler step).

  value : tokens per second of the step on the device (CUDA events recorded
          on the engine's stream around every token-loop launch; weights and
          caches resident in HBM), summed over ranks, time = max over ranks.
  e2e   : the same tokens per wall-clock second through the public API with
          host buffers (prompt / WAL / checkpoint bytes in, tokens out),
          including every host<->device copy and the WAL file writes.
  config1 : 5-token prompt, 64 greedy tokens, one session per GPU, with its
          HBM roofline (the single-session decode target).
  batched_replay : config 3 (512 sessions, prompts 16-256 tokens, seeds
          0..511, T=0.8, 512 generated tokens each) on the same ranks: each
          rank generates the checkpoints of its contiguous token-balanced
          block with the batched token loop, then the timed batched verified
          replay; aggregate tokens / max-over-ranks device time, with both
          roofline bounds (HBM bytes, fp32 SIMT flops) and the binding one.
  ablation : config 4 (1.7B shape, leave-one-out attribution over a
          128-token context, 127 variants batched).
  cpu_baseline / --impl reference : the single-threaded CPU oracle of the
          reference's path on bounded samples of the same workload.

python bench.py [--gpus N] [--steps K] [--warmup W] [--impl b200|reference]
"""
from __future__ import annotations

import argparse
import json
import multiprocessing as mp
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

MODEL = "smollm2-135m"
PROMPT_LEN = 32
CONTEXT = 2048
TEMPERATURE = 0.7
SEED = 42
FALLBACK_HBM_GBS = 6650.0
WORKLOAD = ("config2: SmolLM2-135M-shape fp32 Llama (synthetic N(0,0.02) seed 0), T=0.7, ChaCha8 seed 42+rank, "
            "32-token prompt -> 2048-token context with a host WAL, then verified WAL replay; "
            "1 session per GPU")


def model_dir() -> str:
    return os.environ.get("DEFER_BENCH_DIR", os.path.join(tempfile.gettempdir(), "defer_bench"))


def prompt_tokens(vocab: int):
    import numpy as np
    return [int(t) for t in np.random.default_rng(2).integers(0, vocab, PROMPT_LEN)]


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    except Exception:  # noqa: BLE001
        return FALLBACK_HBM_GBS, "fallback"


def tensor_peak():
    """Sustained dense bf16 tensor throughput (TFLOP/s) for a kernel timed
    inside a long step, from MEASURED_PEAKS.json."""
    try:
        d = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
        return float(d["bf16_tflops_sustained"]), "measured (sustained)"
    except Exception:  # noqa: BLE001
        return 1400.0, "fallback (sustained)"


def traffic_per_token():
    """DRAM bytes per token of the token-loop kernel from the committed ncu
    summary (profiles/traffic.json), or None."""
    try:
        d = json.load(open(os.path.join(ROOT, "profiles", "traffic.json")))
        return d.get(MODEL)
    except Exception:  # noqa: BLE001
        return None


class Clocks:
    """Samples nvidia-smi every 200 ms while the timed region runs."""

    def __init__(self, device: int):
        self.device = device
        self.proc = None
        self.path = os.path.join(tempfile.gettempdir(), f"defer_clocks_{os.getpid()}.csv")

    def __enter__(self):
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits",
                                          "-i", str(self.device), "-lms", "200"],
                                         stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except OSError:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        try:
            rows = [r.split(",") for r in open(self.path).read().strip().splitlines()]
        except OSError:
            return None
        sm, mx, reasons = [], 0.0, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            if len(r) < 8:
                continue
            try:
                sm.append(float(r[1]))
                mx = max(mx, float(r[2]))
            except ValueError:
                continue
            for n, v in zip(names, r[4:8]):
                if v.strip().lower() == "active":
                    reasons.add(n)
        if not sm:
            return None
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": mx, "reasons": sorted(reasons), "samples": len(sm)}


# ------------------------------------------------------------ CPU legs
SAMPLE_FORWARDS = 16  # forwards per CPU sample step


def workload_positions(n: int):
    """Positions of a stratified sample of n forwards of the workload. It
    feeds positions 0..2047 twice (the generation, then the verified replay),
    so its position mix is uniform over 0..2047; forward k of the sample
    runs at the middle of the k-th of n equal position ranges."""
    return [int((k + 0.5) * CONTEXT / n) for k in range(n)]


def _cpu_sample_worker(args):
    """The oracle (the reference's CPU path restated in C, single-threaded
    like the reference) on one core: `steps` timed sample steps after `warm`
    untimed ones, each SAMPLE_FORWARDS forwards at workload_positions (the
    cache length is set per forward: the CPU cost of a forward at position p
    does not depend on the cached values), each followed by the sampler
    (T = 0.7) where the workload samples from those logits. Returns
    (forwards, seconds)."""
    path, steps, warm, seed, core = args
    if core is not None:
        try:
            os.sched_setaffinity(0, {core})
        except OSError:
            pass
    sys.path.insert(0, ROOT)
    import numpy as np
    from oracle import oracle as O
    m = O.Model.load(path)
    rng = np.random.default_rng(seed)
    toks = [int(t) for t in rng.integers(0, m.config.vocab_size, SAMPLE_FORWARDS)]
    words = [int(w) for w in rng.integers(0, 2 ** 32, SAMPLE_FORWARDS, dtype=np.uint64)]
    c = m.new_cache(CONTEXT + 1)
    pos = workload_positions(SAMPLE_FORWARDS)

    def one_step():
        for k, p in enumerate(pos):
            c.set_len(p)
            lo = m.forward(toks[k], c)
            if PROMPT_LEN - 1 <= p < CONTEXT - 1:  # these logits are sampled (generation and replay)
                O.sample_token_word(lo, TEMPERATURE, words[k])

    for _ in range(warm):
        one_step()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    return steps * SAMPLE_FORWARDS, time.perf_counter() - t0


def cpu_model_name():
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_sample(path: str, steps: int, warm: int, sessions: int):
    """`sessions` independent single-threaded oracle sessions, one per core
    (spawned processes); returns (forwards per second, cores, forwards,
    seconds)."""
    ctx = mp.get_context("spawn")
    cores = sorted(os.sched_getaffinity(0))[:max(1, sessions)]
    with ctx.Pool(len(cores)) as pool:
        res = pool.map(_cpu_sample_worker, [(path, steps, warm, SEED + i, c) for i, c in enumerate(cores)])
    fw = sum(r[0] for r in res)
    secs = max(r[1] for r in res)
    return fw / secs, len(cores), fw, secs


def cpu_sample_text(steps: int, sessions: int) -> str:
    return (f"{sessions} session(s), one single-threaded oracle process pinned per core (the reference is "
            f"single-threaded); per step {SAMPLE_FORWARDS} forwards at positions stratified over 0..{CONTEXT - 1} "
            f"(the workload's position mix: generation and replay each feed 0..{CONTEXT - 1}), each followed by "
            f"the T=0.7 sampler where the workload samples; {steps} timed step(s); the workload's mean cost per "
            f"forward is extrapolated from the sample; CPU: {cpu_model_name()}")


def bench_config(world: int) -> dict:
    """The workload description both arms print (the same dict)."""
    return {"workload": WORKLOAD, "tokens_per_step_per_gpu": 2 * CONTEXT,
            "l2": "weights 538 MB per token > 126 MB L2: inputs larger than L2, no flush",
            "parallelism": f"{world} independent session(s), one per GPU, no collective"}


METRIC = "decode tok/s (single-session token loop)"


# ------------------------------------------------------------------- arms
def run_reference(args):
    """The reference's CPU implementation of the path (the oracle port; the
    Rust crate cannot be built here) on the host cores: one single-threaded
    session per GPU of the other arm, each timed on a bounded sample of the
    config-2 workload per step. Under torchrun only rank 0 runs."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", str(args.gpus)))
    if rank != 0:
        return 0
    from defer_b200 import synthetic
    path = synthetic.model_path(MODEL, model_dir(), 0)
    value, cores, fw, secs = cpu_sample(path, args.steps, args.warmup, world)
    sample = cpu_sample_text(args.steps, world)
    line = {"impl": "reference", "metric": METRIC, "value": value, "unit": "tok/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * secs / max(args.steps, 1),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": value / world / 17.0, "dtype": "fp32",
            "data": "synthetic", "config": bench_config(world),
            "cpu_baseline": {"value": value, "unit": "tok/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)
    return 0


def session_step(D, m, prompt, seed_bytes, wal_path):
    """One step through the public API: prompt, generate to CONTEXT with a
    host WAL, then checkout from the WAL bytes. Returns (tokens, h2d, d2h)."""
    s = D.Session(m, seed_bytes, TEMPERATURE)
    s.prompt(prompt)
    hdr = D.WalHeader(m.signature, seed_bytes, TEMPERATURE, len(prompt), 0, prompt)
    w = D.WalWriter.create(wal_path, hdr)
    gen = CONTEXT - len(prompt)
    t0 = m.timing()
    out = s.generate(gen, on_token=lambda sess, t: w.append(t, sess.rng_word_pos()))
    t1 = m.timing()
    w.close()
    ck = D.WalLog.read(wal_path).to_checkpoint()
    r = D.Session.checkout(m, ck)
    t2 = m.timing()
    assert r.history() == s.history() and len(out) == gen
    tokens = len(prompt) + gen + CONTEXT
    # host->device: program tokens + PRNG words of each run; device->host:
    # tokens, margins and slot state read back after each run
    h2d = 4 * (len(prompt) + 2 * gen + CONTEXT + gen)
    d2h = 4 * (len(prompt) + 2 * gen + CONTEXT + 2 * gen)
    phases = {k: (t1[k] - t0[k], t2[k] - t1[k]) for k in ("device_ms", "hbm_bytes", "tokens", "launches")}
    return tokens, h2d, d2h, phases


# ------------------------------------------------ single-session greedy (config 1)
CONFIG1_WORKLOAD = ("config1: the same 135M-shape model; 5-token uniform-random prompt (seed 1), greedy decode of "
                    "64 tokens, one session per GPU (dataflow token-loop kernel)")


def config1_measure(D, m, reps, world, max_over_ranks, sum_over_ranks):
    """Config 1 on every rank: `reps` timed sessions after 2 untimed ones.
    value = tokens fed (5 + 64 per session) per second of device time; the
    roofline is the algorithmic bytes of those steps (weights once per token
    plus the KV read and written) over the same time."""
    import numpy as np
    prompt = [int(t) for t in np.random.default_rng(1).integers(0, m.config.vocab_size, 5)]

    def one():
        s = D.Session(m, D.seed_from_u64(0), 0.0)
        s.prompt(prompt)
        out = s.generate(64)
        assert len(out) == 64
        return out

    ref = one()
    one()
    m.timing(reset=True)
    t0 = time.perf_counter()
    for _ in range(reps):
        assert one() == ref  # bit-reproducible run to run
    wall = time.perf_counter() - t0
    tm = m.timing(reset=True)
    dev_s = max_over_ranks(tm["device_ms"] / 1e3)
    tokens = sum_over_ranks(tm["tokens"])
    peak, peak_kind = peaks()
    achieved = sum_over_ranks(tm["hbm_bytes"]) / dev_s / 1e9
    return {"metric": "decode tok/s (config 1, single-session greedy)", "value": tokens / dev_s, "unit": "tok/s",
            "us_per_token": 1e6 * dev_s / (69 * reps),
            "sessions": reps, "tokens": int(tokens), "device_s": dev_s,
            "config": {"workload": CONFIG1_WORKLOAD},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / world / peak,
                         "peak_kind": peak_kind, "target_frac": 0.70,
                         "kernel": "k_flow (dataflow token loop: one launch for the prompt, one for the 64 tokens)"},
            "e2e": {"value": tokens / max_over_ranks(wall), "unit": "tok/s",
                    "h2d_bytes_per_step": 4 * (5 + 64), "d2h_bytes_per_step": 4 * 2 * 64}}


# -------------------------------------------------- batched replay (config 3)
REPLAY_T = 0.8
REPLAY_WORKLOAD = ("config3: the same 135M-shape model; {n} independent sessions (prompt lengths uniform 16-256, "
                   "token IDs uniform, ChaCha8 seeds 0..{n1}, T=0.8, {gen} generated tokens each); their "
                   "checkpoints generated by the batched token loop, then a batched verified replay (every "
                   "recorded token re-sampled and compared), sessions partitioned over the GPUs in contiguous "
                   "token-balanced blocks, no collective on the data path")
FP32_FMA_PER_SM_CLK = 128  # fp32 FMA lanes per SM per clock (sm_100)


def replay_sessions(n: int, vocab: int):
    import numpy as np
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(16, 257, n)]
    return [[int(t) for t in rng.integers(0, vocab, k)] for k in lens]


def batched_replay(D, m, args, rank, world, max_over_ranks, sum_over_ranks, barrier, sms, clk_mhz):
    """Config 3 on this rank's block: generate the checkpoints (batched token
    loop), then the timed batched verified replay. Returns the JSON object."""
    from defer_b200.partition import partition
    n, gen = args.replay_sessions, args.replay_gen
    prompts = replay_sessions(n, m.config.vocab_size)
    blocks = partition([len(p) + gen for p in prompts], world)
    mine = list(blocks[rank])
    batch = max(1, min(len(mine), args.replay_batch))
    pr = [prompts[i] for i in mine]
    seeds = [D.seed_from_u64(i) for i in mine]
    toks, gen_ms = D.generate_batch(m, pr, seeds, [REPLAY_T] * len(mine), [gen] * len(mine), batch=batch)
    cks = [D.DeferCheckpoint(m.signature, seeds[k], REPLAY_T, pr[k] + toks[k], len(pr[k]), len(toks[k]))
           for k in range(len(mine))]
    tokens = sum(len(c.history_tokens) for c in cks)
    m.timing(reset=True)
    barrier()
    t0 = time.perf_counter()
    res, ms = D.replay_batch(m, cks, batch=batch) if cks else ([], 0.0)
    wall = time.perf_counter() - t0
    barrier()
    tmr = m.timing(reset=True)
    launches = tmr["launches"]
    failures = sum(1 for r in res if r.status != 0)
    dev_s = max_over_ranks(ms / 1e3)
    wall_s = max_over_ranks(wall)
    gen_s = max_over_ranks(gen_ms / 1e3)
    all_tokens = sum_over_ranks(tokens)
    all_fail = sum_over_ranks(failures)
    value = all_tokens / dev_s
    c = m.config
    H, FF, QD, KVD = c.hidden_size, c.intermediate_size, c.q_dim, c.kv_dim
    mac = c.num_layers * (H * (QD + 2 * KVD) + QD * H + 3 * FF * H) + c.vocab_size * H  # projections + head
    # attention at position p: scores and the weighted value sum, 2 * 2 * L * NH * HD * (p + 1) flops
    att = sum(len(ck.history_tokens) * (len(ck.history_tokens) + 1) // 2 for ck in cks)
    flops = 2.0 * mac * tokens + 4.0 * c.num_layers * c.num_heads * c.head_dim * att
    all_flops = sum_over_ranks(flops)
    peak_tf = world * sms * FP32_FMA_PER_SM_CLK * 2 * clk_mhz * 1e6 / 1e12
    achieved_tf = all_flops / dev_s / 1e12
    # HBM: weights once per batched step plus every slot's KV read and written (the engine's algorithmic bytes)
    hbm_peak, hbm_kind = peaks()
    achieved_gbs = sum_over_ranks(tmr["hbm_bytes"]) / dev_s / 1e9
    simt = {"bound": "fp32 simt", "achieved": achieved_tf, "peak": peak_tf, "unit": "TFLOP/s",
            "frac": achieved_tf / peak_tf, "peak_kind": f"nominal: {sms} SMs x {FP32_FMA_PER_SM_CLK} fp32 FMA/clk "
                                                        f"x 2 x {clk_mhz:.0f} MHz per GPU",
            "flops": all_flops, "note": "projections, lm_head and attention; the batched GEMMs keep the "
                                        "reference's fp32 arithmetic"}
    hbm = {"bound": "hbm", "achieved": achieved_gbs, "peak": hbm_peak * world, "unit": "GB/s",
           "frac": achieved_gbs / (hbm_peak * world), "peak_kind": hbm_kind,
           "bytes": sum_over_ranks(tmr["hbm_bytes"]), "note": "weights once per batched step plus the KV read "
                                                                "and written by every slot"}
    binding = simt if simt["frac"] >= hbm["frac"] else hbm
    # host->device: the checkpoint bytes; device->host: status, step, token per session
    h2d = sum(len(c.to_bytes()) for c in cks)
    d2h = 12 * len(cks)
    return {"metric": "batched replay tok/s (verified checkout of many WALs)", "value": value, "unit": "tok/s",
            "n_gpus": world, "scaling": "strong", "sessions": n, "tokens": int(all_tokens),
            "divergences": int(all_fail),
            "batch_per_gpu": batch, "device_s": dev_s, "generate_tok_s": all_tokens / gen_s,
            "gpu_launches": launches, "rank_tokens": tokens, "rank_device_s": ms / 1e3,
            "config": {"workload": REPLAY_WORKLOAD.format(n=n, n1=n - 1, gen=gen),
                       "parallelism": f"{world} GPU(s), contiguous token-balanced session blocks"},
            "roofline": dict(binding, other=hbm if binding is simt else simt),
            "e2e": {"value": all_tokens / wall_s, "unit": "tok/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h}}


# ------------------------------------------------ 8B-shape WAL replay (config 5)
C5_SESSIONS = 8
C5_CONTEXT = 4096
C5_PROMPT = 32
C5_T = 0.8
C5_WORKLOAD = ("config5: Llama-3-8B-shape (hidden 4096, 32 layers, 32/8 heads x 128, FFN 14336, vocab 128256 "
               "untied), random-init N(0,0.02) weights stored bf16 and computed fp32; per GPU 8 sessions "
               "(32-token uniform-random prompt, ChaCha8 seeds 1000+8*rank.., T=0.8, sampled to a 4096-token "
               "context by the batched token loop), whose 4096-position checkpoints are replayed together with "
               "every sampled token verified")


def config5_measure(D, rank, world, max_over_ranks, sum_over_ranks, barrier):
    """Config 5 on every rank (8 sessions per GPU): load, generate the WAL
    histories, then the timed batched verified replay. Returns the object."""
    import numpy as np
    from defer_b200 import synthetic
    t0 = time.perf_counter()
    if rank == 0:  # one writer per box, the other ranks wait for the file
        synthetic.model_path("llama3-8b", model_dir(), 0)
    barrier()
    path = synthetic.model_path("llama3-8b", model_dir(), 0)
    gen_file_s = time.perf_counter() - t0
    t0 = time.perf_counter()
    m = D.Model.load(path, device=int(os.environ.get("LOCAL_RANK", "0")))
    load_s = time.perf_counter() - t0
    V = m.config.vocab_size
    rng = np.random.default_rng(50 + rank)
    prompts = [[int(t) for t in rng.integers(0, V, C5_PROMPT)] for _ in range(C5_SESSIONS)]
    seeds = [D.seed_from_u64(1000 + C5_SESSIONS * rank + i) for i in range(C5_SESSIONS)]
    toks, gen_ms = D.generate_batch(m, prompts, seeds, [C5_T] * C5_SESSIONS, [C5_CONTEXT - C5_PROMPT] * C5_SESSIONS,
                                    batch=C5_SESSIONS)
    cks = [D.DeferCheckpoint(m.signature, seeds[k], C5_T, prompts[k] + toks[k], C5_PROMPT, len(toks[k]))
           for k in range(C5_SESSIONS)]
    tokens = sum(len(c.history_tokens) for c in cks)
    m.timing(reset=True)
    barrier()
    t0 = time.perf_counter()
    res, ms = D.replay_batch(m, cks, batch=C5_SESSIONS)
    wall = time.perf_counter() - t0
    barrier()
    tm = m.timing(reset=True)
    dev_s = max_over_ranks(ms / 1e3)
    all_tokens = sum_over_ranks(tokens)
    fails = sum_over_ranks(sum(1 for r in res if r.status != 0))
    peak, kind = peaks()
    achieved = sum_over_ranks(tm["hbm_bytes"]) / dev_s / 1e9
    weight_bytes = m.config.weight_bytes
    del m  # frees the 8B weights and caches before the next measurement
    return {"metric": "batched replay tok/s (8B shape, 8 sessions per GPU)", "value": all_tokens / dev_s,
            "unit": "tok/s", "n_gpus": world, "scaling": "weak", "sessions_per_gpu": C5_SESSIONS,
            "tokens": int(all_tokens), "divergences": int(fails), "device_s": dev_s,
            "gpu_launches": tm["launches"],
            "generate_tok_s": all_tokens / max_over_ranks(gen_ms / 1e3), "load_s": load_s,
            "file_write_s": gen_file_s, "weights_bytes": weight_bytes,
            "config": {"workload": C5_WORKLOAD},
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s",
                         "frac": achieved / world / peak, "peak_kind": kind,
                         "note": "15.01 GB of bf16 weights once per step plus every session's KV read and written"},
            "e2e": {"value": all_tokens / max_over_ranks(wall), "unit": "tok/s",
                    "h2d_bytes_per_step": sum(len(c.to_bytes()) for c in cks), "d2h_bytes_per_step": 12 * len(cks)}}


# ------------------------------------------------ ablation attribution (config 4)
ABLATION_WORKLOAD = ("config4: SmolLM2-1.7B-shape fp32 Llama (synthetic N(0,0.02) seed 0); leave-one-out "
                     "attribution over a 128-token uniform-random context: base run plus 127 ablated variants "
                     "(every position but the query, attribution.rs:237), each replayed from its masked "
                     "position with one masked cache per variant, variants batched in one token loop")


def ablation_measure(D, rank, sms, clk_mhz, barrier):
    """Config 4 on this rank: returns the JSON object (device time of the
    ablation's token-loop launches)."""
    import numpy as np
    from defer_b200 import synthetic
    if rank == 0:  # one writer per box, the other ranks wait for the file
        synthetic.model_path("smollm2-1.7b", model_dir(), 0)
    barrier()
    m = D.Model.load(synthetic.model_path("smollm2-1.7b", model_dir(), 0),
                     device=int(os.environ.get("LOCAL_RANK", "0")))
    ctx = [int(t) for t in np.random.default_rng(4 + rank).integers(0, m.config.vocab_size, 128)]
    positions = list(range(len(ctx) - 1))
    D.ablation_attribution(m, ctx[:16], ctx[16], list(range(15)))  # warm-up
    m.timing(reset=True)
    t0 = time.perf_counter()
    base, rows = D.ablation_attribution(m, ctx, ctx[-1], positions)
    wall = time.perf_counter() - t0
    tm = m.timing(reset=True)
    n = len(ctx)
    forwards = n + sum(n - p - 1 for p in positions)  # base + every variant's replay from p + 1
    c = m.config
    H, FF, QD, KVD = c.hidden_size, c.intermediate_size, c.q_dim, c.kv_dim
    mac = c.num_layers * (H * (QD + 2 * KVD) + QD * H + 3 * FF * H) + c.vocab_size * H
    dev_s = tm["device_ms"] / 1e3
    useful = forwards * 2.0 * mac  # the model's projection flops
    # the tensor-core step computes each product as 3 split-bf16 MMAs (2 for bf16-stored weights)
    terms = 2 if m.config.weights_bf16 else 3
    tc = os.environ.get("DEFER_B200_TC", "") != "0" and m.config.hidden_size >= 1024
    peak_tc, kind_tc = tensor_peak()
    achieved = useful / dev_s / 1e12
    roof = ({"bound": "tensor", "achieved": achieved * terms, "peak": peak_tc, "unit": "TFLOP/s",
             "frac": achieved * terms / peak_tc, "peak_kind": kind_tc,
             "useful_tflops": achieved, "note": f"executed MMA flops = {terms} split-bf16 products per fp32 product"}
            if tc else
            {"bound": "fp32 simt", "achieved": achieved, "peak": sms * FP32_FMA_PER_SM_CLK * 2 * clk_mhz * 1e6 / 1e12,
             "unit": "TFLOP/s", "peak_kind": f"nominal: {sms} SMs x {FP32_FMA_PER_SM_CLK} fp32 FMA/clk x 2 x "
                                             f"{clk_mhz:.0f} MHz"})
    if "frac" not in roof:
        roof["frac"] = roof["achieved"] / roof["peak"]
    return {"metric": "ablation forwards/s (leave-one-out attribution)", "value": forwards / dev_s,
            "unit": "forwards/s", "variants": len(positions), "forwards": forwards, "device_s": dev_s,
            "wall_s": wall, "gpu_launches": tm["launches"], "base_logprob": base,
            "path": "tensor-core step (tcgen05, split bf16)" if tc else "CUDA-core step",
            "config": {"workload": ABLATION_WORKLOAD}, "roofline": roof}


def run_b200(args):
    import numpy as np  # noqa: F401
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    dist = None
    if world > 1:
        import datetime

        import torch
        import torch.distributed as tdist
        torch.cuda.set_device(local)
        tdist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300),
                                 device_id=torch.device(f"cuda:{local}"))
        dist = tdist

    # single-session runs use the dataflow token-loop kernel; fail loudly if it does not apply
    os.environ.setdefault("DEFER_B200_LOOP", "flow")
    import defer_b200 as D
    from defer_b200 import synthetic

    def barrier():
        if dist:
            dist.barrier()

    def max_over_ranks(x: float) -> float:
        if not dist:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def sum_over_ranks(x: float) -> float:
        if not dist:
            return x
        import torch
        t = torch.tensor([x], dtype=torch.float64, device=f"cuda:{local}")
        dist.all_reduce(t, op=dist.ReduceOp.SUM)
        return float(t.item())

    if rank == 0:
        path = synthetic.model_path(MODEL, model_dir(), 0)
    barrier()
    path = synthetic.model_path(MODEL, model_dir(), 0)

    # CPU baseline first (spawned pool, before this process touches the GPU)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        v, cores, fw, secs = cpu_sample(path, args.cpu_steps, 1, 1)
        cpu = {"value": v, "unit": "tok/s", "cores": cores, "kind": "port",
               "sample": cpu_sample_text(args.cpu_steps, 1) + f" ({fw} forwards in {secs:.1f} s)"}

    m = D.Model.load(path, device=local)
    prompt = prompt_tokens(m.config.vocab_size)
    seed_bytes = D.seed_from_u64(SEED + rank)
    wal = os.path.join(tempfile.gettempdir(), f"defer_bench_{os.getpid()}.wal")
    for _ in range(args.warmup):
        session_step(D, m, prompt, seed_bytes, wal)

    barrier()
    m.timing(reset=True)
    with Clocks(local) as clk:
        barrier()
        t0 = time.perf_counter()
        tokens = h2d = d2h = 0
        ph = {"device_ms": [0.0, 0.0], "hbm_bytes": [0.0, 0.0], "tokens": [0, 0], "launches": [0, 0]}
        for _ in range(args.steps):
            t, a, b, p = session_step(D, m, prompt, seed_bytes, wal)
            tokens += t
            h2d += a
            d2h += b
            for k in ph:
                ph[k][0] += p[k][0]
                ph[k][1] += p[k][1]
        wall = time.perf_counter() - t0
        barrier()
    tm = m.timing(reset=True)
    clocks = clk.summary()
    c1 = config1_measure(D, m, args.config1_reps, world, max_over_ranks, sum_over_ranks)
    m.timing(reset=True)
    os.environ.pop("DEFER_B200_LOOP", None)  # wide batches below take the grid-barrier token loop
    replay = None
    if args.replay_sessions > 0:
        import torch
        sms = torch.cuda.get_device_properties(local).multi_processor_count
        clk_mhz = (clocks or {}).get("sm_max_mhz") or 1965.0
        replay = batched_replay(D, m, args, rank, world, max_over_ranks, sum_over_ranks, barrier, sms, clk_mhz)
        m.timing(reset=True)
    config5 = None
    if not args.no_config5:
        config5 = config5_measure(D, rank, world, max_over_ranks, sum_over_ranks, barrier)
    ablation = None
    if not args.no_ablation:
        import torch
        sms = torch.cuda.get_device_properties(local).multi_processor_count
        clk_mhz = (clocks or {}).get("sm_max_mhz") or 1965.0
        ablation = ablation_measure(D, rank, sms, clk_mhz, barrier)
    try:
        os.unlink(wal)
    except OSError:
        pass

    dev_s = max_over_ranks(tm["device_ms"] / 1e3)
    wall_s = max_over_ranks(wall)
    all_tokens = sum_over_ranks(tokens)
    value = all_tokens / dev_s
    e2e = all_tokens / wall_s
    peak, peak_kind = peaks()
    # The dominant kernel is the single-session decode (k_flow): the
    # generation launch of every step, 2016 tokens at positions 32..2047.
    gen_ms, gen_bytes, gen_tok = ph["device_ms"][0], ph["hbm_bytes"][0], ph["tokens"][0]
    achieved = gen_bytes / (gen_ms / 1e3) / 1e9
    tpt = traffic_per_token()
    roofline = {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                "peak_kind": peak_kind, "kernel": "k_flow (dataflow token loop): the generation launch of each step",
                "bytes_per_launch": gen_bytes / args.steps, "tokens_per_launch": gen_tok / args.steps,
                "traffic": (tpt * gen_tok / args.steps) if tpt else None,
                "launch_ms": gen_ms / args.steps, "us_per_token": 1e3 * gen_ms / max(gen_tok, 1)}
    rep_ms, rep_bytes, rep_tok = ph["device_ms"][1], ph["hbm_bytes"][1], ph["tokens"][1]
    checkout_obj = {"what": "position-parallel verified checkout of the WAL (lanes of one cache, grid-barrier kernel)",
              "tokens_per_step": rep_tok / args.steps, "ms_per_step": rep_ms / args.steps,
              "tok_s": rep_tok / (rep_ms / 1e3) if rep_ms else None,
              "launches_per_step": ph["launches"][1] / args.steps,
              "hbm_gbs": rep_bytes / (rep_ms / 1e3) / 1e9 if rep_ms else None}
    if rank == 0:
        assert tokens == 2 * CONTEXT * args.steps
        line = {"metric": METRIC, "value": value, "unit": "tok/s",
                "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
                "ms_per_step": 1000.0 * dev_s / args.steps, "higher_is_better": True, "scaling": "weak",
                "vs_baseline": value / world / 17.0, "dtype": "fp32", "data": "synthetic",
                "config": bench_config(world),
                "roofline": roofline, "checkout": checkout_obj, "cpu_baseline": cpu, "config1": c1,
                "e2e": {"value": e2e, "unit": "tok/s", "h2d_bytes_per_step": h2d // max(args.steps, 1),
                        "d2h_bytes_per_step": d2h // max(args.steps, 1)},
                "gpu_launches": tm["launches"], "clocks": clocks, "batched_replay": replay,
                "ablation": ablation, "config5": config5,
                "device": {"tokens": tokens, "device_ms": tm["device_ms"], "runs": tm["runs"]}}
        print(json.dumps(line), flush=True)
    if dist:
        dist.destroy_process_group()
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=3)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--cpu-steps", type=int, default=8,
                    help=f"sample steps ({SAMPLE_FORWARDS} forwards each) of the CPU baseline")
    ap.add_argument("--config1-reps", type=int, default=10, help="timed repetitions of config 1")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--replay-sessions", type=int, default=512,
                    help="sessions of the batched replay measurement (config 3); 0 skips it")
    ap.add_argument("--replay-gen", type=int, default=512, help="generated tokens per replay session")
    ap.add_argument("--replay-batch", type=int, default=512, help="slots per GPU of the batched replay")
    ap.add_argument("--no-config5", action="store_true", help="skip config 5 (8B shape, 8 replayed sessions)")
    ap.add_argument("--no-ablation", action="store_true",
                    help="skip config 4 (1.7B-shape leave-one-out attribution, 127 variants)")
    ap.add_argument("--profile-case", nargs="?", const="single", choices=["single", "batched", "ablation", "tc-gemm"],
                    help="no measurement: a small case for profiles. single: the 135M model, 16-token "
                         "prompt, then one launch of 32 sampled tokens (dataflow kernel). batched: "
                         "--profile-slots sessions with --profile-prompt prompts and 2 sampled tokens "
                         "in one batch on the per-stage launch path (one kernel per stage). ablation: "
                         "config 4's leave-one-out attribution on the 1.7B shape over a 24-token "
                         "context (tensor-core step). tc-gemm: three tensor-core GEMMs of 128 slots x "
                         "the 1.7B shape's gate/up matrix (16384 x 2048, fp32 weights)")
    ap.add_argument("--profile-slots", type=int, default=512)
    ap.add_argument("--profile-prompt", type=int, default=128)
    ap.add_argument("--profile-gen", type=int, default=2, help="sampled tokens per session of --profile-case batched")
    ap.add_argument("--trace", action="store_true",
                    help="no measurement: per-stage critical-path breakdown of the dataflow kernel from "
                         "globaltimer stamps of one traced step (--profile-prompt tokens of context)")
    ap.add_argument("--trace-out", default=None, help="with --trace: also save the raw stamps (.npy)")
    a = ap.parse_args(argv)
    if a.impl == "reference":
        return run_reference(a)
    if a.trace:
        return profile_trace(a.profile_prompt, a.trace_out)
    if a.profile_case == "batched":
        return profile_case_batched(a.profile_slots, a.profile_prompt, a.profile_gen)
    if a.profile_case == "ablation":
        return profile_case_ablation()
    if a.profile_case == "tc-gemm":
        return profile_case_tc_gemm()
    if a.profile_case:
        return profile_case()
    return run_b200(a)


def profile_case():
    """Two token-loop launches on the benchmark model: a 16-token prompt, then
    32 sampled tokens (the launch profiles capture)."""
    os.environ.setdefault("DEFER_B200_LOOP", "flow")
    import numpy as np
    import defer_b200 as D
    from defer_b200 import synthetic
    m = D.Model.load(synthetic.model_path(MODEL, model_dir(), 0))
    s = D.Session(m, D.seed_from_u64(1), 0.7)
    s.prompt([int(t) for t in np.random.default_rng(1).integers(0, m.config.vocab_size, 16)])
    s.generate(32)
    print(json.dumps({"profile_case": "ok", **m.timing()}))
    return 0


def profile_case_ablation():
    """Config 4's attribution on the 1.7B shape over a 24-token context."""
    import numpy as np
    import defer_b200 as D
    from defer_b200 import synthetic
    m = D.Model.load(synthetic.model_path("smollm2-1.7b", model_dir(), 0))
    ctx = [int(t) for t in np.random.default_rng(4).integers(0, m.config.vocab_size, 24)]
    base, _ = D.ablation_attribution(m, ctx, ctx[-1], list(range(len(ctx) - 1)))
    print(json.dumps({"profile_case": "ablation", "base_logprob": base, **m.timing()}))
    return 0


def profile_case_tc_gemm():
    """Three tensor-core GEMMs: 128 slots x the 1.7B gate/up matrix."""
    import numpy as np
    import defer_b200 as D
    rng = np.random.default_rng(0)
    x = rng.standard_normal((128, 2048)).astype(np.float32)
    w = (rng.standard_normal((16384, 2048)) * 0.02).astype(np.float32)
    for _ in range(3):
        y = D.tc_gemm(x, w)
    print(json.dumps({"profile_case": "tc-gemm", "checksum": float(np.abs(y).sum())}))
    return 0


STAGE_KINDS = ("qkv", "attn", "o", "gateup", "down")


def stage_names(L: int):
    names = ["select"]
    for l in range(L):
        names += [f"{k}{l}" for k in STAGE_KINDS]
    return names + ["head", "sum1", "sum2"]


def trace_summary(tr, L: int):
    """Critical path of one traced step of the dataflow kernel. tr[c, k, :]
    holds globaltimer ns of CTA c in stage k: entry, inputs received, then
    each phase warp's finish. For stage k with producer stage p: end(k) =
    last finish over CTAs; span = end(k) - end(p) (its share of the step);
    handoff = a CTA's receipt minus end(p) (last producer store to the
    consumer holding every input); compute = a CTA's last warp finish minus
    its receipt; tail = end(k) minus the median CTA's finish. `select`: the
    sampling CTAs' time to poll the previous logits' statistics, to sample,
    and to finish the stage, from their entry."""
    import numpy as np
    tr = np.asarray(tr, dtype=np.int64)
    names = stage_names(L)
    done = tr[:, :, 2:9].max(axis=2)  # the 7 phase warps
    recv = tr[:, :, 1]
    ends = done.max(axis=0)
    prod = {0: None}
    for l in range(L):
        q = 1 + 5 * l
        prod[q] = 0 if l == 0 else q - 1
        for j in range(1, 5):
            prod[q + j] = q + j - 1
    prod[1 + 5 * L] = 5 * L
    prod[2 + 5 * L] = 1 + 5 * L
    prod[3 + 5 * L] = 2 + 5 * L
    rows = {}
    for k, name in enumerate(names):
        p = prod.get(k)
        if p is None or ends[k] == 0 or ends[p] == 0:
            continue
        part = (done[:, k] > 0) & (recv[:, k] > 0)
        if not part.any():
            continue
        ho = (recv[part, k] - ends[p]) / 1e3
        cp = (done[part, k] - recv[part, k]) / 1e3
        kind = name.rstrip("0123456789")
        r = rows.setdefault(kind, {"n": 0, "span": [], "handoff_med": [], "handoff_max": [], "compute_med": [],
                                   "compute_max": [], "tail": [], "ctas": [], "mark10": [], "mark11": [],
                                   "mark12": [], "mark13": [], "mark14": [], "mark15": []})
        for mk in (10, 11, 12, 13, 14, 15):  # warp 0's sub-stage marks, from the receipt
            ok = part & (tr[:, k, mk] > 0)
            if ok.any():
                r[f"mark{mk}"].append(float(np.median((tr[ok, k, mk] - recv[ok, k]) / 1e3)))
        r["n"] += 1
        r["span"].append((ends[k] - ends[p]) / 1e3)
        r["handoff_med"].append(float(np.median(ho)))
        r["handoff_max"].append(float(ho.max()))
        r["compute_med"].append(float(np.median(cp)))
        r["compute_max"].append(float(cp.max()))
        r["tail"].append((ends[k] - np.median(done[part, k])) / 1e3)
        r["ctas"].append(int(part.sum()))
    out = {}
    for kind, r in rows.items():
        out[kind] = {"stages": r["n"], **{key: round(float(np.mean(v)), 3) for key, v in r.items()
                                          if key != "n" and len(v)}}
    own = (tr[:, 0, 11] > 0) & (tr[:, 0, 10] > 0)  # CTAs that sampled a slot's token in SELECT
    if own.any():
        sel = tr[own, 0, :]
        out["select"] = {"ctas": int(own.sum()),
                         "inputs_polled": round(float(np.median(sel[:, 10] - sel[:, 0])) / 1e3, 3),
                         "sampler": round(float(np.median(sel[:, 11] - sel[:, 10])) / 1e3, 3),
                         "sum_rows": round(float(np.median(sel[:, 12] - sel[:, 10])) / 1e3, 3),
                         "sum_walk": round(float(np.median(sel[:, 13] - sel[:, 12])) / 1e3, 3),
                         "cdf_rows": round(float(np.median(sel[:, 14] - sel[:, 13])) / 1e3, 3),
                         "cdf_walk": round(float(np.median(sel[:, 15] - sel[:, 14])) / 1e3, 3),
                         "last_sum_records": round(float(tr[:, 0, 12].max() - np.median(sel[:, 10])) / 1e3, 3),
                         "sum_polled": round(float(np.median(sel[:, 16] - sel[:, 12])) / 1e3, 3),
                         "sum_decoded": round(float(np.median(sel[:, 17] - sel[:, 16])) / 1e3, 3),
                         "sum_walked": round(float(np.median(sel[:, 18] - sel[:, 17])) / 1e3, 3),
                         "cdf_polled": round(float(np.median(sel[:, 19] - sel[:, 14])) / 1e3, 3),
                         "cdf_decoded": round(float(np.median(sel[:, 20] - sel[:, 19])) / 1e3, 3),
                         "cdf_walked": round(float(np.median(sel[:, 21] - sel[:, 20])) / 1e3, 3),
                         "done": round(float(np.median(done[own, 0] - sel[:, 0])) / 1e3, 3)}
    t0 = tr[:, 0, 0][tr[:, 0, 0] > 0].min() if (tr[:, 0, 0] > 0).any() else 0
    last = int(max(i for i in range(len(names)) if ends[i] > 0))
    return {"step_us": round((ends[last] - t0) / 1e3, 3), "last_stage": names[last], "per_kind_us": out}


def profile_trace(context: int, out: str = None):
    """Traces one generated step of the benchmark session (dataflow
    kernel) at about `context` positions and prints the per-stage
    breakdown (trace_summary) as JSON."""
    os.environ.setdefault("DEFER_B200_LOOP", "flow")
    import numpy as np
    import defer_b200 as D
    from defer_b200 import synthetic
    m = D.Model.load(synthetic.model_path(MODEL, model_dir(), 0))
    s = D.Session(m, D.seed_from_u64(1), TEMPERATURE)
    s.prompt([int(t) for t in np.random.default_rng(1).integers(0, m.config.vocab_size, context)])
    s.generate(8)  # warm-up launch
    m.timing(reset=True)
    m.trace_next_run(16)
    s.generate(32)
    tm = m.timing(reset=True)
    tr = m.trace()
    if out:
        np.save(out, tr)
    res = trace_summary(tr, m.config.num_layers)
    res.update({"profile": "trace", "context": context + 8 + 16, "launch_us_per_token": 1e3 * tm["device_ms"] / 32})
    print(json.dumps(res), flush=True)
    return 0


def profile_case_batched(n: int, plen: int, gen: int = 2):
    """n sessions (plen-token uniform prompts, T=0.8, `gen` sampled tokens) as
    one batch on the per-stage launch path, so that ncu sees every stage of
    the batched step as its own kernel."""
    os.environ["DEFER_B200_PHASED"] = "1"
    import numpy as np
    import defer_b200 as D
    from defer_b200 import synthetic
    m = D.Model.load(synthetic.model_path(MODEL, model_dir(), 0))
    rng = np.random.default_rng(3)
    prompts = [[int(t) for t in rng.integers(0, m.config.vocab_size, plen)] for _ in range(n)]
    seeds = [D.seed_from_u64(i) for i in range(n)]
    _, ms = D.generate_batch(m, prompts, seeds, [0.8] * n, [gen] * n, batch=n)
    print(json.dumps({"profile_case": "batched", "slots": n, "steps": plen + gen, "device_ms": ms}))
    return 0


if __name__ == "__main__":
    sys.exit(main())
