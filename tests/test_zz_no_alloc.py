"""The allocation-free forward step (defer_forward_noalloc) against the
ordinary one (defer_forward), through the C ABI.

It serves callers that must not allocate device memory while they run (a
server whose pool already owns the free HBM, a loop that must stay out of
the driver's allocator): they hand in the KV cache and logits buffers, and
the step's scratch comes from a fixed array inside the library. Its logits
and KV entries must equal the ordinary step's bit for bit (every token-loop
path of this library computes the same arithmetic), and one step is also
checked against the CPU oracle at the parity tolerance. After its first
call on a device (the set-up) it must not change the device's free memory.
This file is collected last so that a failure here cannot hide any other
test; it must pass alone in a fresh process and after the whole suite.
"""
import ctypes

import numpy as np
import pytest

import defer_b200 as D
from defer_b200 import _lib
from oracle import oracle as O
from tests.gpu_util import logits_close, model_file

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def torch():
    import torch as t
    assert t.cuda.is_available()
    return t


def _noalloc(model, k, v, cap, pos, token, logits):
    return _lib.load().defer_forward_noalloc(model._h, ctypes.c_void_p(k.data_ptr()), ctypes.c_void_p(v.data_ptr()),
                                             cap, pos, token, ctypes.c_void_p(logits.data_ptr()), None)


@pytest.mark.parametrize("name", ["test-gqa4", "tiny"])
def test_noalloc_step_matches_forward(tmp_path, torch, name):
    path = model_file(str(tmp_path), name)
    m = D.Model.load(path)
    c = m.config
    cap = 96
    n = c.num_layers * c.num_kv_heads * cap * c.head_dim
    # the caller's own buffers (here from torch's pool, allocated up front)
    k = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
    v = torch.full((n,), float("nan"), dtype=torch.float32, device="cuda")
    logits = torch.empty(c.vocab_size, dtype=torch.float32, device="cuda")
    ref = m.new_cache(cap)
    om = O.Model.load(path)
    oc = om.new_cache()
    toks = [int(t) for t in np.random.default_rng(3).integers(0, c.vocab_size, 70)]
    for pos, t in enumerate(toks):  # consecutive calls, crossing a 64-position attention chunk
        rc = _noalloc(m, k, v, cap, pos, t, logits)
        assert rc == 0, _lib.load().defer_last_error()
        torch.cuda.synchronize()
        want = m.forward(t, ref)
        got = logits.cpu().numpy()
        assert np.array_equal(got.view(np.uint32), want.view(np.uint32)), f"pos {pos}: logits differ in bits"
        if pos in (0, len(toks) - 1):
            ok, err, rng = logits_close(got, om.forward(t, oc))
            assert ok, (pos, err, rng)
        elif pos < len(toks) - 1:
            om.forward(t, oc)
    # the ordinary path's first calls allocated its own buffers above; the
    # allocation-free step itself took nothing after its set-up call
    torch.cuda.synchronize()
    before = torch.cuda.mem_get_info()[0]
    for pos in range(len(toks), len(toks) + 2):
        assert _noalloc(m, k, v, cap, pos, toks[0], logits) == 0, _lib.load().defer_last_error()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == before
    # the KV entries written by the two paths are the same bits
    kk = k.cpu().numpy().reshape(c.num_layers, c.num_kv_heads, cap, c.head_dim)[:, :, :len(toks)]
    vv = v.cpu().numpy().reshape(c.num_layers, c.num_kv_heads, cap, c.head_dim)[:, :, :len(toks)]
    for layer in range(c.num_layers):
        rk, rv = ref.layer(layer)
        rk = rk.reshape(len(toks), c.num_kv_heads, c.head_dim).transpose(1, 0, 2)
        rv = rv.reshape(len(toks), c.num_kv_heads, c.head_dim).transpose(1, 0, 2)
        assert np.array_equal(kk[layer].view(np.uint32), rk.view(np.uint32))
        assert np.array_equal(vv[layer].view(np.uint32), rv.view(np.uint32))


def test_noalloc_rejects_oversized_scratch_and_bad_input(tmp_path, torch):
    m = D.Model.load(model_file(str(tmp_path), "test-gqa4"))
    buf = torch.zeros(16, dtype=torch.float32, device="cuda")
    L = _lib.load()
    rc = _noalloc(m, buf, buf, 1 << 24, 0, 1, buf)
    assert rc == D.InvalidArgumentError.code
    assert b"limit" in L.defer_last_error()
    assert _noalloc(m, buf, buf, 8, 0, m.config.vocab_size, buf) == D.ModelError.code
    assert _noalloc(m, buf, buf, 8, 8, 1, buf) == D.ModelError.code
