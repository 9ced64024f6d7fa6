"""Session-level data parallelism across GPUs: the deterministic
partition of sessions over ranks, and the sharded verified replay run as
two gloo ranks on the CPU (the oracle's checkout as the per-rank worker, so
no GPU is needed). The GPU worker is the batched replay the GPU tests cover."""
import os
import pickle
import socket
import tempfile

import numpy as np
import pytest

from defer_b200.partition import partition, replay_sharded


def test_partition_blocks_cover_every_session_once_in_order():
    rng = np.random.default_rng(0)
    for n in (0, 1, 3, 17, 512):
        w = [int(x) for x in rng.integers(16, 800, n)]
        for world in (1, 2, 3, 4, 8):
            blocks = partition(w, world)
            assert len(blocks) == world
            flat = [i for b in blocks for i in b]
            assert flat == list(range(n))
            assert all(b.step == 1 for b in blocks)
            if n:
                total, biggest = sum(w), max(w)
                for b in blocks:  # balanced to within one session
                    assert sum(w[i] for i in b) <= total / world + biggest


def test_partition_is_deterministic_and_rejects_bad_input():
    w = [5, 1, 9, 9, 2, 7]
    assert partition(w, 3) == partition(list(w), 3)
    assert [len(b) for b in partition([0, 0, 0, 0], 2)] == [2, 2]
    with pytest.raises(ValueError):
        partition(w, 0)
    with pytest.raises(ValueError):
        partition([1, -1], 2)


# ------------------------------------------------------------ two gloo ranks
def _make_checkpoints(tmp):
    from oracle import oracle as O
    cfg = O.tiny_config()
    path = os.path.join(tmp, "tiny.safetensors")
    O.write_tiny_model(path, cfg, 1234)
    m = O.Model.load(path)
    cks = []
    for i, (plen, gen, t) in enumerate([(5, 6, 0.7), (3, 4, 0.0), (8, 3, 1.1), (4, 7, 0.7), (6, 2, 0.9)]):
        s = O.Session(m, O.seed_from_u64(100 + i), t)
        s.prompt([int(x) for x in np.random.default_rng(i).integers(0, cfg.vocab_size, plen)])
        s.generate(gen)
        cks.append(s.checkpoint())
    bad = pickle.loads(pickle.dumps(cks[3]))  # a recorded token that was never sampled
    k = bad.prompt_len + 2
    bad.history_tokens[k] = (bad.history_tokens[k] + 1) % cfg.vocab_size
    cks[3] = bad
    return path, cks


def _oracle_worker(model, cks, batch):
    from oracle import oracle as O
    out = []
    for ck in cks:
        try:
            s = O.Session.checkout(model, ck)
            out.append((0, s.cache.fingerprint()))
        except O.DivergenceError as e:
            out.append((7, str(e)))
    return out, float(len(cks))


def _rank_main(rank, world, port, path, ck_file, out_file):
    import torch.distributed as dist
    from oracle import oracle as O
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        cks = pickle.load(open(ck_file, "rb"))
        model = O.Model.load(path)
        res = replay_sharded(model, cks, rank, world, batch=4, group=dist.group.WORLD, worker=_oracle_worker)
        pickle.dump(res, open(out_file.format(rank), "wb"))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_sharded_replay_over_two_gloo_ranks_equals_one_process():
    import torch.multiprocessing as mp
    from oracle import oracle as O
    with tempfile.TemporaryDirectory() as tmp:
        path, cks = _make_checkpoints(tmp)
        ck_file = os.path.join(tmp, "cks.pkl")
        pickle.dump(cks, open(ck_file, "wb"))
        out_file = os.path.join(tmp, "out{}.pkl")
        mp.start_processes(_rank_main, args=(2, _free_port(), path, ck_file, out_file), nprocs=2,
                           join=True, start_method="spawn")
        single, _, blocks1 = replay_sharded(O.Model.load(path), cks, 0, 1, worker=_oracle_worker)
        r0 = pickle.load(open(out_file.format(0), "rb"))
        r1 = pickle.load(open(out_file.format(1), "rb"))
    assert r0[0] == r1[0] == single          # same outcomes, session order, on every rank
    assert [s for s, _ in single] == [0, 0, 0, 7, 0]  # the tampered record diverges
    assert r0[2] == r1[2] and len(r0[2]) == 2 and all(len(b) for b in r0[2])
    assert r0[1] == r1[1] == max(len(b) for b in r0[2])  # device time = max over ranks
