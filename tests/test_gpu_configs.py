"""Oracle parity on the benchmark configurations themselves, at their real
lengths, through the C ABI:

  config 1: 135M shape, 5-token prompt (seed 1), 64 greedy tokens: tokens
            identical, logits within tolerance after every fed token, KV
            within tolerance at the end.
  config 2: 135M shape, T = 0.7, ChaCha8 seed 42, 32-token prompt, decoded
            to a 2048-token context, then teacher-forced through the oracle:
            logits at every 8th position and the last 64, KV at the end, and
            every sampled token the oracle's sequential-CDF sampler would
            choose differently (its logits differ from the GPU's by rounding)
            within a few ulps of an edge of that sampler's own CDF. The
            disagreement rate is reported.
  config 3: 512 sessions (prompts 16-256, seeds 0..511, T = 0.8, 512
            generated tokens each) replayed in one batch with no divergence;
            the sessions with the shortest and the longest prompt are
            teacher-forced through the oracle as in config 2.
  config 4: 1.7B shape, leave-one-out ablation over a 128-token context at
            the positions next to the query (p = 124, 125, 126): base and
            ablated log-probabilities and the base logits.
  config 5: the 8B shape's widths (bf16-stored weights, untied 128256-token
            head, 32/8 heads x 128) on 2 layers: logits and KV over 40
            positions, sampled tokens, and the batched verified replay.

The oracle runs are long and single-threaded, so a module fixture starts
them in spawned worker processes as soon as their inputs exist.
"""
import json
import multiprocessing as mp
import os
import tempfile
from concurrent.futures import ProcessPoolExecutor

import numpy as np
import pytest

import defer_b200 as D
from tests import oracle_jobs as J
from tests.gpu_util import KV_TOL, LOGIT_TOL, kv_close, logits_close, model_file

pytestmark = pytest.mark.gpu

# where the per-configuration parity records (disagreement rates, worst
# errors) are written: DEFER_PARITY_OUT, else a folder in the temp dir
OUT = os.environ.get("DEFER_PARITY_OUT", os.path.join(tempfile.gettempdir(), "defer_parity"))


def _tokens(vocab, n, seed):
    return [int(t) for t in np.random.default_rng(seed).integers(0, vocab, n)]


def _config3_prompts(n, vocab):
    rng = np.random.default_rng(3)
    lens = [int(x) for x in rng.integers(16, 257, n)]
    return [[int(t) for t in rng.integers(0, vocab, k)] for k in lens]


class Runs:
    pass


@pytest.fixture(scope="module")
def runs(tmp_path_factory):
    d = os.environ.get("DEFER_BENCH_DIR") or str(tmp_path_factory.mktemp("configs"))
    r = Runs()
    r.p135 = model_file(d, "smollm2-135m")
    r.p17 = model_file(d, "smollm2-1.7b")
    pool = ProcessPoolExecutor(max_workers=6, mp_context=mp.get_context("spawn"))
    r.gm = D.Model.load(r.p135)
    V = r.gm.config.vocab_size
    # config 1: independent of the GPU run
    r.c1_prompt = _tokens(V, 5, 1)
    r.c1_job = pool.submit(J.greedy_run, r.p135, r.c1_prompt, 64)
    # config 4
    r.c4_ctx = _tokens(V, 128, 4)
    r.c4_pos = [124, 125, 126]
    r.c4_job = pool.submit(J.ablation, r.p17, r.c4_ctx, r.c4_ctx[-1], r.c4_pos)
    # config 2: the GPU session, then its history teacher-forced through the oracle
    r.c2_seed = D.seed_from_u64(42)
    s = D.Session(r.gm, r.c2_seed, 0.7)
    r.c2_prompt = _tokens(V, 32, 2)
    s.prompt(r.c2_prompt)
    s.generate(2048 - 32)
    r.c2_hist = s.history()
    r.c2_session = s
    r.c2_checks = sorted(set(range(0, 2048, 8)) | set(range(2048 - 64, 2048)))
    r.c2_job = pool.submit(J.teacher_forced, r.p135, r.c2_hist, 32, 0.7, r.c2_seed, r.c2_checks, True)
    # config 3: the 512 sessions by the batched token loop; two teacher-forced
    prompts = _config3_prompts(512, V)
    seeds = [D.seed_from_u64(i) for i in range(512)]
    toks, _ = D.generate_batch(r.gm, prompts, seeds, [0.8] * 512, [512] * 512, batch=512)
    r.c3_cks = [D.DeferCheckpoint(r.gm.signature, seeds[k], 0.8, prompts[k] + toks[k], len(prompts[k]),
                                  len(toks[k])) for k in range(512)]
    lens = [len(p) for p in prompts]
    r.c3_pick = [int(np.argmin(lens)), int(np.argmax(lens))]
    r.c3_jobs = {}
    for k in r.c3_pick:
        hist = prompts[k] + toks[k]
        checks = sorted(set(range(0, len(hist), 32)) | {len(hist) - 1})
        r.c3_jobs[k] = (hist, len(prompts[k]), seeds[k], checks,
                        pool.submit(J.teacher_forced, r.p135, hist, len(prompts[k]), 0.8, seeds[k], checks, True))
    yield r
    pool.shutdown(wait=False, cancel_futures=True)


def _gpu_teacher_forced(gm, hist, checks):
    """The GPU forward over a recorded history; logits at the checked steps."""
    c = gm.new_cache(len(hist) + 1)
    want = set(checks)
    out = {}
    for i, t in enumerate(hist):
        lo = gm.forward_ext(t, c, (), logits=i in want)
        if i in want:
            out[i] = lo
    return out, c


def _check_logits(gpu, cpu, label):
    worst = 0.0
    for i in sorted(cpu):
        ok, err, rng = logits_close(gpu[i], cpu[i])
        assert ok, f"{label}: step {i} logits err {err} vs range {rng}"
        worst = max(worst, err / rng)
    return worst


def _check_edges(reports, label, sampled):
    # The device sampler is the reference's sequential-CDF sampler bit for
    # bit (test_gpu_parity checks it on identical logits), so a differing
    # choice comes from the forward's own rounding differences (logits within
    # ~1e-6 of their range): r then lies within a few fp32 ulps of the edge
    # between the two tokens in the oracle's own sequential CDF. With ~V
    # edges in [0, 1) such near-ties occur at a rate of roughly V x 1e-7
    # per sampled token.
    for r in reports:
        assert r["seq_edge"] <= 1e-6, f"{label}: {r}"
    assert len(reports) <= max(3, 0.02 * sampled), f"{label}: {len(reports)} of {sampled}"


def _record(name, obj):
    try:
        os.makedirs(OUT, exist_ok=True)
        with open(os.path.join(OUT, f"parity_{name}.json"), "w") as f:
            json.dump(obj, f, indent=1)
    except OSError:
        pass


def test_config1_greedy_stream_logits_and_kv(runs):
    gm = runs.gm
    s = D.Session(gm, D.seed_from_u64(0), 0.0)
    s.prompt(runs.c1_prompt)
    gen = s.generate(64)
    otoks, ologits, okv = runs.c1_job.result()
    assert gen == otoks  # identical greedy stream, no near-tie escape
    hist = runs.c1_prompt + gen
    glog, _ = _gpu_teacher_forced(gm, hist, range(len(hist)))
    worst = _check_logits(glog, {i: ologits[i] for i in range(len(hist))}, "config1")
    assert s.last_logits().tobytes() == glog[len(hist) - 1].tobytes()  # session path == forward path
    kv = 0.0
    for l in range(gm.config.num_layers):
        kg, vg = s.cache().layer(l)
        for g, o in ((kg, okv[l][0]), (vg, okv[l][1])):
            kv = max(kv, float(np.abs(g.astype(np.float64) - o).max()) / float(np.abs(o).max()))
    assert kv <= KV_TOL, kv
    _record("config1", {"tokens": len(gen), "identical": True, "worst_logit_err_over_range": worst,
                        "worst_kv_rel": kv, "logit_tol": LOGIT_TOL, "kv_tol": KV_TOL})


def test_config2_teacher_forced_over_2048_positions(runs):
    gm = runs.gm
    hist = runs.c2_hist
    assert len(hist) == 2048
    glog, gc = _gpu_teacher_forced(gm, hist, runs.c2_checks)
    assert gc.fingerprint() == runs.c2_session.cache().fingerprint()  # forward path == session path
    reports, ologits, okv = runs.c2_job.result()
    worst = _check_logits(glog, ologits, "config2")
    kv = 0.0
    for l in range(gm.config.num_layers):
        kg, vg = gc.layer(l)
        for g, o in ((kg, okv[l][0]), (vg, okv[l][1])):
            kv = max(kv, float(np.abs(g.astype(np.float64) - o).max()) / float(np.abs(o).max()))
    assert kv <= KV_TOL, kv
    _check_edges(reports, "config2", 2048 - 32)
    rate = len(reports) / (2048 - 32)
    _record("config2", {"sampled": 2048 - 32, "oracle_disagreements": len(reports), "rate": rate,
                        "reports": reports, "worst_logit_err_over_range": worst, "worst_kv_rel": kv})
    # the verified replay of the GPU's own history never diverges
    r = D.Session.checkout(gm, runs.c2_session.checkpoint())
    assert r.cache().fingerprint() == gc.fingerprint()


def test_config3_batched_replay_and_two_sessions_teacher_forced(runs):
    gm = runs.gm
    res, _ = D.replay_batch(gm, runs.c3_cks, batch=512, fingerprints=True)
    assert all(x.status == 0 for x in res), [(i, x.status, x.div_step) for i, x in enumerate(res) if x.status][:5]
    out = {}
    for k in runs.c3_pick:
        hist, n_prompt, seed, checks, job = runs.c3_jobs[k]
        glog, gc = _gpu_teacher_forced(gm, hist, checks)
        assert gc.fingerprint() == res[k].fingerprint  # batched replay == single-session forward
        reports, ologits, okv = job.result()
        worst = _check_logits(glog, ologits, f"config3 session {k}")
        ok, kv = kv_close(gc, _KvView(okv), gm.config.num_layers)
        assert ok, kv
        _check_edges(reports, f"config3 session {k}", len(hist) - n_prompt)
        out[k] = {"tokens": len(hist), "prompt": n_prompt, "oracle_disagreements": len(reports),
                  "reports": reports, "worst_logit_err_over_range": worst, "worst_kv_rel": kv}
    _record("config3", out)


class _KvView:
    """The oracle job's KV lists with the oracle cache's accessors."""

    def __init__(self, kv):
        self.kv = kv

    def keys(self, l):
        return self.kv[l][0]

    def values(self, l):
        return self.kv[l][1]


def test_config5_shape_forward_and_replay(tmp_path):
    """Config 5's arithmetic (8B widths, bf16-stored weights, untied head
    over 128256 tokens, GQA 32/8 x 128) on a 2-layer model: logits and KV
    against the oracle over 40 positions, sampled tokens against the
    oracle's choices, and the batched verified replay of two sessions."""
    path = model_file(str(tmp_path), "test-8b-width")
    gm, om = D.Model.load(path), O_model(path)
    assert gm.config.weights_bf16 and not gm.config.tie_word_embeddings
    toks = _tokens(gm.config.vocab_size, 40, 12)
    gc, oc = gm.new_cache(), om.new_cache()
    worst = 0.0
    for i, t in enumerate(toks):
        ok, err, rng = logits_close(gm.forward(t, gc), om.forward(t, oc))
        assert ok, (i, err, rng)
        worst = max(worst, err / rng)
    ok, kv = kv_close(gc, oc, gm.config.num_layers)
    assert ok, kv
    prompts = [_tokens(gm.config.vocab_size, 8, 20 + i) for i in range(2)]
    seeds = [D.seed_from_u64(900 + i) for i in range(2)]
    gen, _ = D.generate_batch(gm, prompts, seeds, [0.8, 0.8], [24, 24], batch=2)
    cks = [D.DeferCheckpoint(gm.signature, seeds[k], 0.8, prompts[k] + gen[k], 8, len(gen[k])) for k in range(2)]
    res, _ = D.replay_batch(gm, cks, batch=2)
    assert all(r.status == 0 for r in res)
    reports, _, _ = J.teacher_forced(path, prompts[0] + gen[0], 8, 0.8, seeds[0], [], False)
    _check_edges(reports, "config5 shape", 24)
    _record("config5", {"positions": len(toks), "worst_logit_err_over_range": worst, "worst_kv_rel": kv,
                        "sampled": 24, "oracle_disagreements": len(reports)})


def O_model(path):
    from oracle import oracle as O
    return O.Model.load(path)


def test_config4_ablation_next_to_the_query(runs):
    gm = D.Model.load(runs.p17)
    ctx = runs.c4_ctx
    base, rows = D.ablation_attribution(gm, ctx, ctx[-1], runs.c4_pos)
    obase, olps, ologits = runs.c4_job.result()
    s = D.Session(gm, D.seed_from_u64(0), 0.0)
    s.prompt(ctx)
    ok, err, rng = logits_close(s.last_logits(), ologits)
    assert ok, (err, rng)
    # log p = l_t - logsumexp(l): with logits within LOGIT_TOL * range, each
    # log-probability is within twice that
    tol = 2 * LOGIT_TOL * rng
    assert abs(base - obase) <= tol, (base, obase, tol)
    for (_, _, lp, _), olp in zip(rows, olps):
        assert abs(lp - olp) <= tol, (lp, olp, tol)
    _record("config4", {"positions": runs.c4_pos, "base": [base, obase], "ablated": [[r[2] for r in rows], olps],
                        "tol": tol})
