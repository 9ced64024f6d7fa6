"""Writes tests/golden/oracle_tiny.json: token streams, KV fingerprints and
logits digests of the CPU oracle on the reference's tiny test model
(src/synthetic.rs, seed 1234) with the prompt of tests/verification.rs.

    python tests/golden/make_golden.py
"""
import hashlib
import json
import os
import sys
import tempfile

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
sys.path.insert(0, ROOT)
from oracle import oracle as O  # noqa: E402

PROMPT = [ord(c) for c in "The alignment problem can be solved by"]


def main():
    d = tempfile.mkdtemp()
    p = os.path.join(d, "tiny.safetensors")
    O.write_tiny_model(p, O.tiny_config(), 1234)
    m = O.Model.load(p)
    cases = []
    for t, seed, n in [(0.0, 1, 24), (0.7, 42424242, 24), (1.5, 7, 24)]:
        s = O.Session(m, O.seed_from_u64(seed), t)
        s.prompt(PROMPT)
        out = s.generate(n)
        cases.append({"temperature": t, "seed": seed, "n": n, "tokens": out,
                      "kv_fingerprint": s.cache.fingerprint().hex(),
                      "logits_sha256": hashlib.sha256(s.logits.astype("<f4").tobytes()).hexdigest()})
    words = O.keystream_words(O.seed_from_u64(42), 0, 8).tolist()
    out = {"model": "reference tiny model (synthetic.rs, seed 1234)", "signature": m.signature.hex(),
           "prompt": PROMPT, "cases": cases, "seed_from_u64_42": O.seed_from_u64(42).hex(),
           "chacha8_words_seed42": words}
    with open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "oracle_tiny.json"), "w") as f:
        json.dump(out, f, indent=1)
    print(json.dumps(out)[:300])


if __name__ == "__main__":
    main()
