"""Position-parallel checkout (Session::checkout, engine.rs:241-274, with the
recorded positions spread over lanes of one cache) against the checkout that
advances one position per step (DEFER_B200_REPLAY_LANES=1): the same KV
bits, last logits, sampler margins and rng position, and for a tampered
history the same Divergence position and sampled token."""
import os
import re

import numpy as np
import pytest

import defer_b200 as D
from tests.gpu_util import model_file

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def mdir(tmp_path_factory):
    return str(tmp_path_factory.mktemp("lanes"))


def _lanes(n, fn):
    old = os.environ.get("DEFER_B200_REPLAY_LANES")
    os.environ["DEFER_B200_REPLAY_LANES"] = str(n)
    try:
        return fn()
    finally:
        if old is None:
            os.environ.pop("DEFER_B200_REPLAY_LANES", None)
        else:
            os.environ["DEFER_B200_REPLAY_LANES"] = old


def _state(m, ck):
    s = D.Session.checkout(m, ck)
    return (s.cache().fingerprint(), s.last_logits().tobytes(), s.margins().tobytes(), s.rng_word_pos(),
            s.history())


def _divergence(m, ck):
    with pytest.raises(D.DivergenceError) as e:
        D.Session.checkout(m, ck)
    return re.findall(r"\d+", str(e.value))[:2]  # sampled token, position


@pytest.mark.parametrize("name,t,n_prompt,n_gen", [("test-small", 0.8, 12, 200), ("test-gqa4", 0.0, 70, 90),
                                                    ("smollm2-135m", 0.7, 32, 300)])
def test_lane_checkout_equals_sequential_checkout(mdir, name, t, n_prompt, n_gen):
    m = D.Model.load(model_file(mdir, name))
    prompt = [int(x) for x in np.random.default_rng(8).integers(0, m.config.vocab_size, n_prompt)]
    s = D.Session(m, D.seed_from_u64(77), t)
    s.prompt(prompt)
    s.generate(n_gen)
    ck = s.checkpoint()
    want = _lanes(1, lambda: _state(m, ck))
    assert want[0] == s.cache().fingerprint()
    for lanes in (7, 64, 256):
        assert _lanes(lanes, lambda: _state(m, ck)) == want, lanes
    # a tampered token: the first divergence in position order is reported
    n = len(ck.history_tokens)
    for pos in (n_prompt, n_prompt + n_gen // 2, n - 1):
        tam = s.checkpoint()
        tam.history_tokens[pos] = (tam.history_tokens[pos] + 1) % m.config.vocab_size
        if pos + 7 < n:
            tam.history_tokens[pos + 7] = (tam.history_tokens[pos + 7] + 3) % m.config.vocab_size
        ref = _lanes(1, lambda: _divergence(m, tam))
        assert int(ref[1]) == pos
        for lanes in (5, 64):
            assert _lanes(lanes, lambda: _divergence(m, tam)) == ref


def test_lane_checkout_then_generation_continues(mdir):
    m = D.Model.load(model_file(mdir, "test-small"))
    prompt = [int(x) for x in np.random.default_rng(9).integers(0, m.config.vocab_size, 20)]
    full = D.Session(m, D.seed_from_u64(5), 0.9)
    full.prompt(prompt)
    whole = full.generate(160)
    part = D.Session(m, D.seed_from_u64(5), 0.9)
    part.prompt(prompt)
    part.generate(100)
    r = _lanes(32, lambda: D.Session.checkout(m, part.checkpoint()))
    assert r.generate(60) == whole[100:]
    assert r.cache().fingerprint() == full.cache().fingerprint()
