"""Device-side failure detection without a GPU fault: every spin-wait of the
persistent token-loop kernels is bounded, and a wait that runs out sets the
status word, which the host raises as DeviceTimeoutError. The drill arms one
run from the host: CTA 0 withholds its first hand-off of step 0 (the
dataflow kernel's step header, the grid-barrier kernel's first arrival) and
every bounded wait is cut to about a millisecond. Nothing faults, traps or
hangs; the next run on the same model must be unaffected.
"""
import os

import numpy as np
import pytest

import defer_b200 as D
from tests.gpu_util import model_file

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def model(tmp_path_factory):
    d = str(tmp_path_factory.mktemp("faults"))
    return D.Model.load(model_file(d, "test-small"))


def _with_loop(loop, fn):
    old = os.environ.get("DEFER_B200_LOOP")
    os.environ["DEFER_B200_LOOP"] = loop
    try:
        return fn()
    finally:
        if old is None:
            os.environ.pop("DEFER_B200_LOOP", None)
        else:
            os.environ["DEFER_B200_LOOP"] = old


def _run(m, prompt, n):
    s = D.Session(m, D.seed_from_u64(5), 0.8)
    s.prompt(prompt)
    return s.generate(n), s.cache().fingerprint()


@pytest.mark.parametrize("loop", ["flow", "barrier"])
def test_withheld_handoff_times_out_and_the_next_run_is_clean(model, loop):
    prompt = [int(t) for t in np.random.default_rng(7).integers(0, model.config.vocab_size, 20)]
    want = _with_loop(loop, lambda: _run(model, prompt, 12))

    def drill():
        s = D.Session(model, D.seed_from_u64(5), 0.8)
        model.stall_next_run(wait_us=1000)
        with pytest.raises(D.DeviceTimeoutError):
            s.prompt(prompt)

    _with_loop(loop, drill)
    # the drill is consumed by that one run: the same model runs normally
    # and gives the same tokens and KV bits as before the drill
    assert _with_loop(loop, lambda: _run(model, prompt, 12)) == want


def test_stall_argument_is_checked(model):
    with pytest.raises(D.InvalidArgumentError):
        model.stall_next_run(wait_us=0)
