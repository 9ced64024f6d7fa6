"""Host-side parts of the B200 library, checked without a GPU: the C ABI
loads and exports every declared symbol; the byte/integer code (ChaCha8,
seed_from_u64, checkpoint and WAL formats, CRC, log-softmax, the synthetic
tiny-model writer) is bit-exact against the oracle."""
import ctypes
import os
import re
import struct

import numpy as np
import pytest

import defer_b200 as D
from defer_b200 import _lib, synthetic
from oracle import oracle as O

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def declared_symbols():
    src = open(os.path.join(ROOT, "include", "defer_b200.h")).read()
    return sorted(set(re.findall(r"DEFER_API[^;(]*?\b(defer_\w+)\s*\(", src)))


def test_library_exports_every_declared_symbol():
    lib = ctypes.CDLL(_lib.LIB_PATH)
    names = declared_symbols()
    assert len(names) >= 40
    for n in names:
        assert hasattr(lib, n), n
    # the binding covers the header exactly
    assert sorted(s[0] for s in _lib.SIGNATURES) == names


def test_seed_and_chacha_words_match_oracle():
    for s in (0, 1, 42, 2**63 + 5, 42424242):
        assert D.seed_from_u64(s) == O.seed_from_u64(s)
    seed = D.seed_from_u64(42)
    assert D.chacha8_words(seed, 0, 100).tolist() == O.keystream_words(seed, 0, 100).tolist()
    assert D.chacha8_words(seed, 37, 21).tolist() == O.keystream_words(seed, 0, 58)[37:].tolist()
    assert D.words_per_sample(0.0) == 0 and D.words_per_sample(0.7) == 1


def _ck():
    return D.DeferCheckpoint(bytes(range(32)), bytes([9] * 32), float(np.float32(0.7)), [1, 2, 3, 40000, 7],
                             2, 3)


def test_checkpoint_bytes_match_oracle(tmp_path):
    c = _ck()
    b = c.to_bytes()
    ob = O.DeferCheckpoint(c.model_signature, c.base_seed, c.temperature, c.history_tokens, c.prompt_len,
                           c.rng_word_pos).to_bytes()
    assert b == ob and len(b) == 112 + 4 * 5
    assert D.DeferCheckpoint.from_bytes(b) == c
    p = str(tmp_path / "x.ckpt")
    c.save(p)
    assert open(p, "rb").read() == b
    assert D.DeferCheckpoint.load(p) == c
    assert not os.path.exists(str(tmp_path / "x.ckpt.tmp"))


@pytest.mark.parametrize("name,tmp", [(".hidden", ".hidden.ckpt.tmp"), ("run.ckpt", "run.ckpt.tmp"),
                                      ("plain", "plain.ckpt.tmp"), ("d.x/.hidden", "d.x/.hidden.ckpt.tmp")])
def test_checkpoint_temp_name_follows_with_extension(tmp_path, monkeypatch, name, tmp):
    # Path::with_extension("ckpt.tmp") (checkpoint.rs:94): a directory in the
    # way makes the final rename fail, so the temp file stays to be seen
    monkeypatch.chdir(tmp_path)
    os.makedirs(name)
    with pytest.raises(D.DeferError):
        _ck().save(name)
    assert os.path.isfile(tmp), sorted(os.listdir("."))


@pytest.mark.parametrize("mutate,err", [
    (lambda b: b.__setitem__(50, b[50] ^ 1), D.CheckpointError),
    (lambda b: b.__setitem__(0, ord("X")), D.CheckpointError),
    (lambda b: b.__delitem__(slice(-9, -5)), D.CheckpointError),
])
def test_checkpoint_corruption_is_rejected(mutate, err):
    b = bytearray(_ck().to_bytes())
    mutate(b)
    with pytest.raises(err):
        D.DeferCheckpoint.from_bytes(bytes(b))


def test_wal_writer_and_parser_match_oracle(tmp_path):
    p = str(tmp_path / "g.wal")
    h = D.WalHeader(bytes([1] * 32), bytes([2] * 32), 0.5, 3, 0, [10, 11, 12])
    with D.WalWriter.create(p, h, durable=True) as w:
        for i, t in enumerate([5, 6, 7]):
            w.append(t, i + 1)
    raw = open(p, "rb").read()
    oh = O.WalHeader(h.model_signature, h.base_seed, h.temperature, h.prompt_len, 0, h.prefix_tokens)
    assert raw == oh.to_bytes() + b"".join(O.wal_record_bytes(3 + i, t, i + 1) for i, t in enumerate([5, 6, 7]))
    # torn tail (wal.rs:282-292) and resume (wal.rs:294-300)
    with open(p, "ab") as f:
        f.write(bytes([1, 2, 3, 4, 5]))
    log = D.WalLog.read(p)
    assert log.torn_tail and log.n_records == 3
    assert log.to_checkpoint().history_tokens == [10, 11, 12, 5, 6, 7]
    assert log.to_checkpoint().rng_word_pos == 3
    assert log.records == [(3, 5, 1), (4, 6, 2), (5, 7, 3)]
    log2, w = D.WalWriter.resume(p, durable=True)
    w.append(8, 4)
    w.close()
    log3 = D.WalLog.read(p)
    assert not log3.torn_tail and log3.records[-1][1] == 8
    assert O.WalLog.parse(open(p, "rb").read()).records[-1] == (6, 8, 4)


def test_wal_errors():
    h = O.WalHeader(bytes(32), bytes(32), 0.5, 1, 0, [1])
    with pytest.raises(D.WalError):
        D.WalLog.parse(h.to_bytes() + O.wal_record_bytes(1, 5, 2))  # rng position skips a word
    with pytest.raises(D.WalError):
        D.WalLog.parse(b"DEFERCKP" + bytes(200))
    b = bytearray(h.to_bytes())
    b[20] ^= 1
    with pytest.raises(D.WalError):
        D.WalLog.parse(bytes(b))


def test_tiny_model_file_matches_oracle_writer(tmp_path):
    a, b = str(tmp_path / "a.safetensors"), str(tmp_path / "b.safetensors")
    synthetic.write_tiny_model(a, 1234)
    O.write_tiny_model(b, O.tiny_config(), 1234)
    assert open(a, "rb").read() == open(b, "rb").read()


def test_log_softmax_matches_oracle():
    rng = np.random.default_rng(0)
    for n in (3, 100, 49152):
        l = rng.standard_normal(n).astype(np.float32) * 3
        i = int(rng.integers(n))
        assert D.log_softmax_at(l, i) == O.log_softmax_at(l, i)
    l = np.array([1.0, float("nan"), 3.0], np.float32)
    assert D.log_softmax_at(l, 2) == O.log_softmax_at(l, 2)


def test_bf16_rounding_is_nearest_even():
    x = np.array([1.0, 1.00390625, 1.005859375, -2.5, 3.0e-3], np.float32)
    bits = synthetic.f32_to_bf16_bits(x)
    back = (bits.astype(np.uint32) << 16).view(np.float32)
    assert np.all(np.abs(back - x) <= np.abs(x) * 2.0 ** -8)
    assert struct.unpack("<H", bits[1].tobytes())[0] == 0x3F80  # tie rounds to even


def test_missing_library_fails_loudly(monkeypatch):
    monkeypatch.setattr(_lib, "_lib", None)
    monkeypatch.setattr(_lib, "LIB_PATH", "/nonexistent/libdefer_b200.so")
    with pytest.raises(ImportError):
        _lib.load()
