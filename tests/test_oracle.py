"""Pins the CPU oracle against the reference's own known-answer tests and
published vectors (the reference cannot be compiled here). Each test names
the reference test it restates."""
import hashlib
import json
import math
import os
import struct

import numpy as np
import pytest

from oracle import oracle as O


# ------------------------------------------------------------- ops.rs tests
def test_matmul_small():  # ops.rs:189-196
    out = np.zeros(4, np.float32)
    a = np.array([1, 2, 3, 4, 5, 6], np.float32)
    b = np.array([7, 8, 9, 10, 11, 12], np.float32)
    O.lib().or_matmul_sequential(O.fp(out), O.fp(a), O.fp(b), 2, 2, 3)
    assert out.tolist() == [58.0, 64.0, 139.0, 154.0]


def test_linear_matches_matmul():  # ops.rs:198-206
    out = O.linear([1.0, 0.5, -1.0], np.array([1, 2, 3, 4, 5, 6], np.float32), [0.5, -0.5])
    assert out.tolist() == [1.0 + 1.0 - 3.0 + 0.5, 4.0 + 2.5 - 6.0 - 0.5]


def test_blocked_linear_is_bit_identical_to_reference():  # ops.rs:208-224
    ind, outd = 37, 11
    w = np.array([np.float32((i * 7919) % 1000) * np.float32(1e-3) - np.float32(0.5) for i in range(ind * outd)],
                 np.float32)
    x = np.array([np.float32((i * 104729) % 997) * np.float32(1e-2) - np.float32(4.0) for i in range(ind)],
                 np.float32)
    b = np.array([np.float32(i) * np.float32(0.1) for i in range(outd)], np.float32)
    out = O.linear(x, w, b)
    for o in range(outd):
        s = np.float32(0.0)
        for i in range(ind):
            s = np.float32(s + np.float32(w[o * ind + i] * x[i]))
        s = np.float32(s + b[o])
        assert out[o].view(np.uint32) == s.view(np.uint32)


def test_norms():  # ops.rs:226-238
    x = np.array([1, 2, 3, 4], np.float32)
    out = O.rmsnorm(x, np.ones(4, np.float32), 0.0)
    rms = math.sqrt(30.0 / 4.0)
    assert np.all(np.abs(out - x / rms) < 1e-6)
    ln = np.zeros(4, np.float32)
    O.lib().or_layernorm(O.fp(ln), O.fp(x), O.fp(np.ones(4, np.float32)), O.fp(np.zeros(4, np.float32)), 4, 0.0)
    assert abs(float(ln.sum())) < 1e-5


def test_activations_and_softmax():  # ops.rs:240-252
    assert O.lib().or_silu(0.0) == 0.0
    assert abs(O.lib().or_gelu(1.0) - 0.841192) < 1e-4
    v = O.softmax([1.0, 2.0, 3.0])
    assert abs(float(v.sum()) - 1.0) < 1e-6 and v[2] > v[1] > v[0]


# --------------------------------------------------------- sampler.rs tests
def test_greedy_ties_pick_lowest_index():  # sampler.rs:116-121
    assert O.argmax([1.0, 3.0, 3.0, 2.0]) == 1
    assert O.argmax([float("nan"), 0.0, 0.0]) == 1
    assert O.argmax([float("-inf")] * 3) == 0


def test_greedy_does_not_touch_rng():  # sampler.rs:123-130
    rng = O.ChaCha8Rng.seed_from_u64(1)
    for _ in range(10):
        O.sample_token([0.1, 0.2, 0.3], 0.0, rng)
    assert rng.get_word_pos() == 0


def test_exactly_one_word_per_sample():  # sampler.rs:132-145
    rng = O.ChaCha8Rng.seed_from_u64(7)
    cases = [[0.0, 1.0, 2.0], [float("-inf")] * 2, [float("nan"), 5.0], [1e30, -1e30, 1e30]]
    for i, l in enumerate(cases):
        O.sample_token(l, 0.7, rng)
        assert rng.get_word_pos() == i + 1


def test_reproducible_and_distributed():  # sampler.rs:147-162
    logits = [0.0, 1.0, 2.0, 3.0]

    def run():
        rng = O.ChaCha8Rng.seed_from_u64(42)
        return [O.sample_token(logits, 1.0, rng) for _ in range(2000)]

    a = run()
    assert a == run()
    c = np.bincount(a, minlength=4)
    assert c[3] > c[2] > c[1] > c[0] > 0


def test_cdf_scan_edge_cases():
    # r beyond the rounded CDF total returns the last non-zero index (sampler.rs:106-108)
    p = np.array([0.25, 0.0, 0.25, 0.5, 0.0], np.float32)
    assert O.lib().or_cdf_scan(O.fp(p), 5, 0.9999999) == 3
    assert O.lib().or_cdf_scan(O.fp(p), 5, 0.0) == 0
    assert O.lib().or_cdf_scan(O.fp(p), 5, 0.25) == 2


# -------------------------------------------------- crc32 / sha256 / ChaCha
def test_crc32_check_value():  # crc32.rs:33-35
    assert O.crc32(b"123456789") == 0xCBF43926


def test_chacha_block_matches_independent_chacha20():
    """The block function (round count as a parameter) equals the ChaCha20
    of the `cryptography` package at 20 rounds."""
    from cryptography.hazmat.primitives.ciphers import Cipher, algorithms
    for key in (bytes(range(32)), bytes(32), hashlib.sha256(b"k").digest()):
        for counter in (0, 1, 7):
            st = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + list(struct.unpack("<8I", key)) + \
                 [counter, 0, 0, 0]
            mine = b"".join(struct.pack("<I", w) for w in O.chacha_block(st, 20))
            nonce = struct.pack("<I", counter) + bytes(12)
            ref = Cipher(algorithms.ChaCha20(key, nonce), mode=None).encryptor().update(bytes(64))
            assert mine == ref


CHACHA8_ZERO_BLOCK = ("3e00ef2f895f40d67f5bb8e81f09a5a12c840ec3ce9a7f3b181be188ef711a1e"
                      "984ce172b9216f419f445367456d5619314a42a3da86b001387bfdb80e0cfe42")


def test_chacha8_published_vector():
    """ChaCha8, all-zero key and IV, first keystream block (the 8-round
    known-answer vector published for ChaCha with a zero key and IV)."""
    st = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + [0] * 12
    got = b"".join(struct.pack("<I", w) for w in O.chacha_block(st, 8)).hex()
    assert got == CHACHA8_ZERO_BLOCK


def test_chacha8rng_word_stream_is_block_order():
    seed = O.seed_from_u64(5)
    r = O.ChaCha8Rng(seed)
    words = [r.next_u32() for _ in range(40)]
    key = list(struct.unpack("<8I", seed))
    exp = []
    for blk in range(3):
        st = [0x61707865, 0x3320646E, 0x79622D32, 0x6B206574] + key + [blk, 0, 0, 0]
        exp += O.chacha_block(st, 8)
    assert words == exp[:40]
    assert r.get_word_pos() == 40


def test_gen_f32_uses_top_24_bits():
    assert O.unit_f32(0xFFFFFFFF) == np.float32(16777215 / 16777216)
    assert O.unit_f32(0x000000FF) == 0.0
    assert O.unit_f32(0x00000100) == np.float32(2.0 ** -24)


# ------------------------------------------------------ safetensors.rs tests
def test_half_conversions():  # safetensors.rs:305-313
    def f16(h):
        return float(O._convert("F16", struct.pack("<H", h))[0])
    assert f16(0x3C00) == 1.0 and f16(0xC000) == -2.0 and f16(0x7BFF) == 65504.0
    assert f16(0x0001) == float(np.float32(5.9604645e-8))
    assert math.isinf(f16(0x7C00))
    assert float(O._convert("BF16", struct.pack("<H", 0x3F80))[0]) == 1.0


def test_write_then_read(tmp_path):  # safetensors.rs:315-333
    p = str(tmp_path / "t.safetensors")
    O.write_safetensors(p, [("b", [2, 2], np.array([1, 2, 3, 4], np.float32)),
                            ("a", [3], np.array([-1.0, 0.5, 9.0], np.float32))], [("k", "v")])
    st = O.SafeTensors.load(p)
    assert st.names == ["b", "a"]
    assert list(st.tensors["b"].shape) == [2, 2]
    assert st.tensors["a"].tolist() == [-1.0, 0.5, 9.0]
    assert st.meta("k") == "v"
    assert st.signature == hashlib.sha256(open(p, "rb").read()).digest()


# ------------------------------------------------- checkpoint / WAL tests
def test_checkpoint_roundtrip_and_corruption():  # checkpoint.rs:142-156
    c = O.DeferCheckpoint(bytes([7] * 32), bytes([9] * 32), float(np.float32(0.7)), [1, 2, 3, 40000], 2, 2)
    b = bytearray(c.to_bytes())
    assert len(b) == 112 + 4 * 4
    assert O.DeferCheckpoint.from_bytes(bytes(b)) == c
    b[50] ^= 1
    with pytest.raises(O.CheckpointError):
        O.DeferCheckpoint.from_bytes(bytes(b))


def test_wal_write_read_torn_resume():  # wal.rs:272-301
    h = O.WalHeader(bytes([1] * 32), bytes([2] * 32), 0.5, 3, 0, [10, 11, 12])
    b = h.to_bytes() + b"".join(O.wal_record_bytes(3 + i, t, i + 1) for i, t in enumerate([5, 6, 7]))
    log = O.WalLog.parse(b + bytes([1, 2, 3, 4, 5]))
    assert log.torn_tail and len(log.records) == 3
    ck = log.to_checkpoint()
    assert ck.history_tokens == [10, 11, 12, 5, 6, 7] and ck.rng_word_pos == 3
    log2 = O.WalLog.parse(b + O.wal_record_bytes(6, 8, 4))
    assert not log2.torn_tail and log2.records[-1][1] == 8
    assert len(O.wal_record_bytes(0, 0, 0)) == 29


def test_wal_inconsistent_record_is_an_error():
    h = O.WalHeader(bytes(32), bytes(32), 0.5, 1, 0, [1])
    with pytest.raises(O.WalError):
        O.WalLog.parse(h.to_bytes() + O.wal_record_bytes(1, 5, 2))


# --------------------------------------------- model invariants (tiny model)
@pytest.fixture(scope="module")
def tiny(tmp_path_factory):
    p = str(tmp_path_factory.mktemp("tiny") / "tiny.safetensors")
    O.write_tiny_model(p, O.tiny_config(), 1234)
    return O.Model.load(p), p


PROMPT = [ord(c) for c in "The alignment problem can be solved by"]


def _gen(m, t, seed, n):
    s = O.Session(m, O.seed_from_u64(seed), t)
    s.prompt(PROMPT)
    out = s.generate(n)
    return out, s


def test_runs_are_deterministic(tiny):  # tests/verification.rs:45-59 (fewer runs)
    m, _ = tiny
    a, s1 = _gen(m, 0.7, 42424242, 24)
    for _ in range(3):
        b, s2 = _gen(m, 0.7, 42424242, 24)
        assert a == b and s1.cache.fingerprint() == s2.cache.fingerprint()
        assert s1.logits.tobytes() == s2.logits.tobytes()
        assert s2.rng_word_pos() == 24


def test_seeds_and_greedy(tiny):  # tests/verification.rs:71-81
    m, _ = tiny
    assert _gen(m, 0.7, 1, 16)[0] != _gen(m, 0.7, 2, 16)[0]
    g1, s1 = _gen(m, 0.0, 1, 16)
    g2, _ = _gen(m, 0.0, 2, 16)
    assert g1 == g2 and s1.rng_word_pos() == 0


def test_checkout_is_bit_identical(tiny):  # tests/verification.rs:83-107
    m, _ = tiny
    for t in (0.0, 0.7, 1.5):
        _, live = _gen(m, t, 42424242, 20)
        ck = O.DeferCheckpoint.from_bytes(live.checkpoint().to_bytes())
        restored = O.Session.checkout(m, ck)
        fresh = O.Session(m, ck.base_seed, t)
        fresh.prompt(ck.history_tokens)
        assert restored.cache.bit_eq(live.cache) and restored.cache.bit_eq(fresh.cache)
        assert restored.logits.tobytes() == live.logits.tobytes()
        assert restored.rng_word_pos() == live.rng_word_pos()


def test_checkout_rejects_wrong_model_and_tampering(tiny):  # tests/verification.rs:119-135
    m, _ = tiny
    _, s = _gen(m, 0.7, 42424242, 8)
    bad = s.checkpoint()
    bad.model_signature = bytes([bad.model_signature[0] ^ 1]) + bad.model_signature[1:]
    with pytest.raises(O.CheckpointError):
        O.Session.checkout(m, bad)
    tam = s.checkpoint()
    tam.history_tokens[-1] = (tam.history_tokens[-1] + 1) % 256
    with pytest.raises(O.DivergenceError):
        O.Session.checkout(m, tam)
    br = s.checkpoint()
    br.rng_word_pos += 1
    with pytest.raises(O.CheckpointError):
        O.Session.checkout(m, br)


def test_ablation_prefix_reuse_equals_full_recompute(tiny):  # tests/attribution.rs:96-129
    m, _ = tiny
    _, s = _gen(m, 0.8, 5, 4)
    h = s.history
    ctx, target = h[:-1], h[-1]
    positions = list(range(len(ctx) - 1))[:8]
    base, r1 = O.ablation_attribution(m, ctx, target, positions)
    _, r2 = O.ablation_attribution(m, ctx, target, positions)
    assert r1 == r2 and any(x[3] != 0.0 for x in r1)
    for p in (0, 5):
        c = m.new_cache()
        for t in ctx:
            logits = m.forward_ext(t, c, [p])
        assert O.log_softmax_at(logits, target) == r1[p][2]
    c1, c2 = m.new_cache(), m.new_cache()
    for t in ctx[:6]:
        assert m.forward(t, c1).tobytes() == m.forward_ext(t, c2, []).tobytes()
    with pytest.raises(O.ModelError):
        O.ablation_attribution(m, ctx, target, [len(ctx) - 1])


def test_golden_fixture(tiny):
    """Oracle regression anchor: tests/golden/oracle_tiny.json (made by
    tests/golden/make_golden.py from this oracle)."""
    g = json.load(open(os.path.join(os.path.dirname(__file__), "golden", "oracle_tiny.json")))
    m, _ = tiny
    assert m.signature.hex() == g["signature"]
    assert O.seed_from_u64(42).hex() == g["seed_from_u64_42"]
    assert O.keystream_words(O.seed_from_u64(42), 0, 8).tolist() == g["chacha8_words_seed42"]
    for case in g["cases"]:
        out, s = _gen(m, case["temperature"], case["seed"], case["n"])
        assert out == case["tokens"]
        assert s.cache.fingerprint().hex() == case["kv_fingerprint"]
        assert hashlib.sha256(s.logits.astype("<f4").tobytes()).hexdigest() == case["logits_sha256"]
