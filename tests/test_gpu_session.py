"""The reference's integration suites (tests/verification.rs,
tests/attribution.rs ablation) run on the CUDA path, plus the batched
drivers against the single-session path."""
import os

import numpy as np
import pytest

import defer_b200 as D
from oracle import oracle as O
from tests.gpu_util import logits_close, model_file

pytestmark = pytest.mark.gpu

PROMPT = [ord(c) for c in "The alignment problem can be solved by"]
TEMPERATURE = 0.7
SEED = 42424242


@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("tiny"))
    p = model_file(d, "tiny", 1234)
    return D.Model.load(p), p, d


def generate(m, t, seed, n, prompt=PROMPT):
    s = D.Session(m, D.seed_from_u64(seed), t)
    s.prompt(prompt)
    out = s.generate(n)
    return out, s


def test_runs_have_zero_deviation(tiny):  # tests/verification.rs:45-59
    m, _, _ = tiny
    ref, rs = generate(m, TEMPERATURE, SEED, 48)
    fp, lg = rs.cache().fingerprint(), rs.last_logits().tobytes()
    for _ in range(10):
        out, s = generate(m, TEMPERATURE, SEED, 48)
        assert out == ref
        assert s.cache().fingerprint() == fp
        assert s.last_logits().tobytes() == lg
        assert s.rng_word_pos() == 48


def test_reloading_weights_is_deterministic(tiny):  # tests/verification.rs:61-69
    m, p, _ = tiny
    ref, _ = generate(m, TEMPERATURE, SEED, 32)
    for _ in range(2):
        m2 = D.Model.load(p)
        assert m2.signature == m.signature
        assert generate(m2, TEMPERATURE, SEED, 32)[0] == ref


def test_seeds_and_temperatures_matter(tiny):  # tests/verification.rs:71-81
    m, _, _ = tiny
    assert generate(m, TEMPERATURE, SEED, 32)[0] != generate(m, TEMPERATURE, SEED + 1, 32)[0]
    g1, s1 = generate(m, 0.0, 1, 32)
    g2, _ = generate(m, 0.0, 2, 32)
    assert g1 == g2 and s1.rng_word_pos() == 0


def test_checkout_kv_cache_is_bit_identical(tiny, tmp_path):  # tests/verification.rs:83-107
    m, _, _ = tiny
    for t in (0.0, TEMPERATURE, 1.5):
        _, live = generate(m, t, SEED, 40)
        ck = live.checkpoint()
        p = str(tmp_path / f"t{t}.ckpt")
        ck.save(p)
        loaded = D.DeferCheckpoint.load(p)
        assert loaded == ck
        restored = D.Session.checkout(m, loaded)
        fresh = D.Session(m, ck.base_seed, t)
        fresh.prompt(ck.history_tokens)
        assert restored.cache().bit_eq(live.cache())
        assert restored.cache().bit_eq(fresh.cache())
        assert restored.last_logits().tobytes() == live.last_logits().tobytes()
        assert restored.rng_word_pos() == live.rng_word_pos()


def test_resumed_generation_matches_uninterrupted(tiny):  # tests/verification.rs:109-117
    m, _, _ = tiny
    full, _ = generate(m, TEMPERATURE, SEED, 60)
    _, partial = generate(m, TEMPERATURE, SEED, 25)
    resumed = D.Session.checkout(m, partial.checkpoint())
    resumed.generate(35)
    assert resumed.generated() == full


def test_checkout_rejects_wrong_model_and_tampering(tiny):  # tests/verification.rs:119-135
    m, _, _ = tiny
    _, s = generate(m, TEMPERATURE, SEED, 10)
    bad = s.checkpoint()
    bad.model_signature = bytes([bad.model_signature[0] ^ 1]) + bad.model_signature[1:]
    with pytest.raises(D.CheckpointError):
        D.Session.checkout(m, bad)
    tam = s.checkpoint()
    tam.history_tokens[-1] = (tam.history_tokens[-1] + 1) % 256
    with pytest.raises(D.DivergenceError):
        D.Session.checkout(m, tam)
    br = s.checkpoint()
    br.rng_word_pos += 1
    with pytest.raises(D.CheckpointError):
        D.Session.checkout(m, br)


def test_wal_reconstructs_session(tiny, tmp_path):  # tests/verification.rs:137-180
    m, _, _ = tiny
    seed = D.seed_from_u64(SEED)
    path = str(tmp_path / "gen.wal")
    s = D.Session(m, seed, TEMPERATURE)
    s.prompt(PROMPT)
    header = D.WalHeader(m.signature, seed, TEMPERATURE, len(PROMPT), 0, PROMPT)
    w = D.WalWriter.create(path, header)
    s.generate(30, on_token=lambda sess, t: w.append(t, sess.rng_word_pos()))
    w.close()
    with open(path, "ab") as f:  # crash mid-record
        f.write(bytes([0x01, 0xAA, 0xBB]))
    log = D.WalLog.read(path)
    assert log.torn_tail and log.n_records == 30
    ck = log.to_checkpoint()
    assert ck == s.checkpoint()
    restored = D.Session.checkout(m, ck)
    assert restored.cache().bit_eq(s.cache())
    _, w = D.WalWriter.resume(path)
    restored.generate(5, on_token=lambda sess, t: w.append(t, sess.rng_word_pos()))
    w.close()
    log = D.WalLog.read(path)
    assert not log.torn_tail
    assert log.to_checkpoint() == restored.checkpoint()


def test_prompt_after_generation_and_bad_tokens(tiny):
    m, _, _ = tiny
    _, s = generate(m, TEMPERATURE, SEED, 2)
    with pytest.raises(D.ModelError):
        s.prompt([1])
    s2 = D.Session(m, D.seed_from_u64(1), 0.5)
    with pytest.raises(D.ModelError):
        s2.prompt([1, 2, 300])  # token id out of range: the first two are fed
    assert s2.history() == [1, 2]
    with pytest.raises(D.ModelError):
        D.Session(m, D.seed_from_u64(1), -1.0)
    with pytest.raises(D.ModelError):
        D.Session(m, D.seed_from_u64(1), 0.5).step()  # no context


def test_stop_tokens_and_callback_errors(tiny):
    m, _, _ = tiny
    ref, _ = generate(m, TEMPERATURE, SEED, 40)
    stop = ref[10]
    out, s = D.Session(m, D.seed_from_u64(SEED), TEMPERATURE), None
    out.prompt(PROMPT)
    got = out.generate(40, stop=[stop])
    assert got == ref[:ref.index(stop) + 1]
    assert len(out.history()) == len(PROMPT) + len(got)
    # a failing callback stops generation at that token; the state equals a
    # session that generated exactly that many tokens
    s = D.Session(m, D.seed_from_u64(SEED), TEMPERATURE)
    s.prompt(PROMPT)
    seen = []

    def cb(sess, t):
        seen.append(t)
        if len(seen) == 7:
            raise D.WalError("disk full")
    with pytest.raises(D.WalError):
        s.generate(40, on_token=cb)
    _, s7 = generate(m, TEMPERATURE, SEED, 7)
    assert s.history() == s7.history() and s.rng_word_pos() == 7
    assert s.cache().bit_eq(s7.cache())
    assert s.last_logits().tobytes() == s7.last_logits().tobytes()


def test_model_forward_cache_api(tiny):
    m, p, _ = tiny
    om = O.Model.load(p)
    c, oc = m.new_cache(), om.new_cache()
    for t in PROMPT[:12]:
        assert logits_close(m.forward(t, c), om.forward(t, oc))[0]
    c2 = c.clone()
    assert c2.bit_eq(c) and len(c2) == 12
    c2.truncate(5)
    assert len(c2) == 5 and not c2.bit_eq(c)
    with pytest.raises(D.ModelError):
        m.forward(256, c)


# ------------------------------------------------------------ batched paths
def test_replay_batch_equals_single_checkout(tiny):
    m, _, _ = tiny
    cks, fps = [], []
    rng = np.random.default_rng(0)
    for i in range(11):
        plen = int(rng.integers(3, 30))
        prompt = [int(t) for t in rng.integers(0, 256, plen)]
        _, s = generate(m, [0.0, 0.8, 1.3][i % 3], i, int(rng.integers(1, 40)), prompt)
        cks.append(s.checkpoint())
        fps.append(s.cache().fingerprint())
    tam = D.DeferCheckpoint(**{**cks[4].__dict__})
    tam.history_tokens = list(tam.history_tokens)
    tam.history_tokens[-1] = (tam.history_tokens[-1] + 1) % 256
    for batch in (1, 4, 16):
        res, ms = D.replay_batch(m, cks + [tam], batch=batch, fingerprints=True)
        for i in range(11):
            assert res[i].status == 0 and res[i].fingerprint == fps[i], (batch, i)
        assert res[11].status == D.DivergenceError.code
        assert res[11].div_step == len(tam.history_tokens) - 1


def test_sharded_replay_blocks_equal_one_batched_replay(tiny):
    """Row e: each rank's block of a partition (here two ranks run one after
    the other on one GPU) gives exactly the outcomes and KV fingerprints of
    one batched replay of everything."""
    from defer_b200.partition import replay_sharded
    m, _, _ = tiny
    rng = np.random.default_rng(5)
    cks = []
    for i in range(9):
        prompt = [int(t) for t in rng.integers(0, 256, int(rng.integers(3, 25)))]
        _, s = generate(m, [0.0, 0.8, 1.3][i % 3], 50 + i, int(rng.integers(1, 30)), prompt)
        cks.append(s.checkpoint())
    whole, _ = D.replay_batch(m, cks, batch=8, fingerprints=True)
    parts = []
    for rank in range(2):
        out, ms, blocks = replay_sharded(m, cks, rank, 2, batch=4)
        assert ms > 0.0
        parts.extend(out)
    assert [b for blk in blocks for b in blk] == list(range(9))
    assert [(r.status, r.fingerprint) for r in parts] == [(r.status, r.fingerprint) for r in whole]


def test_generate_batch_equals_sessions(tiny):
    m, _, _ = tiny
    rng = np.random.default_rng(1)
    prompts = [[int(t) for t in rng.integers(0, 256, int(rng.integers(2, 20)))] for _ in range(9)]
    seeds = [D.seed_from_u64(100 + i) for i in range(9)]
    temps = [0.0, 0.7, 1.0] * 3
    maxt = [int(rng.integers(1, 30)) for _ in range(9)]
    outs, _ = D.generate_batch(m, prompts, seeds, temps, maxt, batch=5)
    for i in range(9):
        s = D.Session(m, seeds[i], temps[i])
        s.prompt(prompts[i])
        assert s.generate(maxt[i]) == outs[i]


def test_ablation_matches_oracle_and_masked_forward(tiny):  # tests/attribution.rs:96-129
    m, p, _ = tiny
    om = O.Model.load(p)
    _, s = generate(m, 0.8, 5, 4)
    h = s.history()
    ctx, target = h[:-1], h[-1]
    positions = list(range(len(ctx) - 1))
    base, r = D.ablation_attribution(m, ctx, target, positions, batch=16)
    base2, r2 = D.ablation_attribution(m, ctx, target, positions, batch=3)
    assert base == base2 and r == r2  # deterministic, independent of the batch width
    obase, orr = O.ablation_attribution(om, ctx, target, positions)
    assert abs(base - obase) < 1e-3
    for (pg, _, lg, _), (po, _, lo, _) in zip(r, orr):
        assert pg == po and abs(lg - lo) < 1e-3
    assert any(x[3] != 0.0 for x in r)
    # prefix reuse equals a full masked recompute, bit for bit
    for q in (0, len(ctx) // 2, len(ctx) - 2):
        c = m.new_cache()
        for t in ctx:
            logits = m.forward_ext(t, c, [q])
        assert D.log_softmax_at(logits, target) == r[q][2]
    with pytest.raises(D.ModelError):
        D.ablation_attribution(m, ctx, target, [len(ctx) - 1])


def test_verify_runs_and_checkout_agree_with_the_oracle(tiny):  # src/main.rs:620-666
    m, p, _ = tiny
    toks, fp = D.verify(m, D.seed_from_u64(SEED), TEMPERATURE, PROMPT, runs=4, max_tokens=32)
    assert len(toks) == 32
    om = O.Model.load(p)
    os_ = O.Session(om, O.seed_from_u64(SEED), TEMPERATURE)
    os_.prompt(PROMPT)
    assert os_.generate(32) == toks  # the reference's stream on its own test model
    live = D.Session(m, D.seed_from_u64(SEED), TEMPERATURE)
    live.prompt(PROMPT)
    live.generate(32)
    assert live.cache().fingerprint() == fp
    with pytest.raises(D.InvalidArgumentError):
        D.verify(m, D.seed_from_u64(SEED), TEMPERATURE, PROMPT, runs=0)
