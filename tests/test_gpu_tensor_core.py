"""The tensor-core (tcgen05) contraction of the batched attribution step.

The GEMM alone against a float64 product: split-bf16 operands with fp32
accumulation keep each output within a few 1e-6 of sum |x| |w| for fp32
weights (two terms per operand leave 2^-17 of each product) and within
about fp32 rounding for bf16-stored weights (three activation terms leave
2^-27), for shapes that pad rows and K and several K splits.
Then the attribution batch on the tensor-core step (DEFER_B200_TC=1): the
same log-probabilities for every batch width (each slot's rows of the
contraction are independent of the others), within the parity tolerance
of the CPU oracle (attribution.rs:224-264), and a position ablated alone
gives the bits it gives inside a wide batch.
"""
import os

import numpy as np
import pytest

import defer_b200 as D
from oracle import oracle as O
from tests.gpu_util import model_file

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("m,n,k", [(128, 64, 64), (5, 200, 576), (127, 1000, 2048), (33, 128, 8192), (1, 64, 100)])
def test_tc_gemm_matches_float64(m, n, k):
    rng = np.random.default_rng(m * 1000 + n + k)
    x = rng.standard_normal((m, k)).astype(np.float32)
    w = (rng.standard_normal((n, k)) * 0.02).astype(np.float32)
    y = D.tc_gemm(x, w)
    ref = x.astype(np.float64) @ w.astype(np.float64).T
    scale = np.abs(x).astype(np.float64) @ np.abs(w).astype(np.float64).T
    err = np.abs(y - ref) / scale
    assert err.max() < 2e-5, err.max()
    assert np.median(err) < 2e-6, np.median(err)


def test_tc_gemm_bf16_weights_and_row_independence():
    rng = np.random.default_rng(3)
    x = rng.standard_normal((100, 1024)).astype(np.float32)
    w = (rng.standard_normal((320, 1024)) * 0.02).astype(np.float32)
    wb = (w.view(np.uint32) & 0xFFFF0000).view(np.float32)  # bf16-exact values
    y = D.tc_gemm(x, wb, w_bf16=True)
    ref = x.astype(np.float64) @ wb.astype(np.float64).T
    scale = np.abs(x).astype(np.float64) @ np.abs(wb).astype(np.float64).T
    err = np.abs(y - ref) / scale
    assert err.max() < 3e-6, err.max()
    assert np.median(err) < 3e-7, np.median(err)
    # a row's result does not depend on the other rows of the tile
    y7 = D.tc_gemm(x[7:8], wb, w_bf16=True)
    assert y7.tobytes() == y[7:8].tobytes()
    y2 = D.tc_gemm(x[40:90], wb, w_bf16=True)
    assert y2.tobytes() == y[40:90].tobytes()


@pytest.fixture
def force_tc():
    old = os.environ.get("DEFER_B200_TC")
    os.environ["DEFER_B200_TC"] = "1"
    yield
    if old is None:
        os.environ.pop("DEFER_B200_TC", None)
    else:
        os.environ["DEFER_B200_TC"] = old


@pytest.mark.parametrize("name", ["tiny", "test-gqa4"])
def test_tc_ablation_matches_oracle(tmp_path, force_tc, name):
    path = model_file(str(tmp_path), name)
    m, om = D.Model.load(path), O.Model.load(path)
    ctx = [int(t) for t in np.random.default_rng(6).integers(0, m.config.vocab_size, 40)]
    target = ctx[-1]
    positions = list(range(len(ctx) - 1))
    base, r = D.ablation_attribution(m, ctx, target, positions, batch=128)
    base2, r2 = D.ablation_attribution(m, ctx, target, positions, batch=5)
    assert base == base2 and r == r2  # deterministic, independent of the batch width
    for q in (0, 17, len(ctx) - 2):  # a position ablated alone: the same bits
        b1, r1 = D.ablation_attribution(m, ctx, target, [q], batch=1)
        assert b1 == base and r1[0] == r[q]
    obase, orr = O.ablation_attribution(om, ctx, target, positions)
    c = om.new_cache()
    for t in ctx:
        lo = om.forward(t, c)
    tol = 2e-4 * float(lo.max() - lo.min())
    assert abs(base - obase) < tol, (base, obase, tol)
    for (pg, _, lg, _), (po, _, lo_, _) in zip(r, orr):
        assert pg == po and abs(lg - lo_) < tol, (pg, lg, lo_, tol)
