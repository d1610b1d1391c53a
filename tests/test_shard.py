"""Multi-GPU host logic on the CPU: the document plan and the final gather, as 2 gloo ranks."""
import os
import socket

import numpy as np
import pytest

from conftest import pkg

S = pkg("shard")


def test_assign_covers_every_document_once_and_balances():
    rng = np.random.default_rng(0)
    lens = rng.integers(128, 2209, size=64).tolist()
    for world in (1, 2, 4, 8):
        shards = S.assign(lens, world)
        flat = sorted(i for s in shards for i in s)
        assert flat == list(range(64))
        loads = [sum(S.doc_cost(lens[i]) for i in s) for s in shards]
        assert max(loads) <= 1.15 * (sum(loads) / world) + max(S.doc_cost(l) for l in lens)
    # Deterministic: every rank computes the same plan.
    assert S.assign(lens, 4) == S.assign(list(lens), 4)


def test_assign_edge_cases():
    assert S.assign([], 3) == [[], [], []]
    assert S.assign([5], 4)[0] == [0]
    with pytest.raises(ValueError):
        S.assign([1], 0)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, lens, q):
    import importlib
    import sys

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sh = importlib.import_module("embeddinggemma2-rust_b200.shard")
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    shards = sh.assign(lens, world)
    # Stand-in for the per-rank embedding pass: a deterministic function of the document.
    local = np.stack([np.full(8, lens[i] * 10 + i, np.float32) for i in shards[rank]]) if shards[rank] else np.zeros((0, 8), np.float32)
    out = sh.gather(local, shards, rank, len(lens), dist)
    q.put((rank, out))
    dist.destroy_process_group()


def test_two_rank_gather_restores_input_order():
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    lens = [700, 3, 2208, 17, 130, 1100, 9]
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, lens, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.stack([np.full(8, l * 10 + i, np.float32) for i, l in enumerate(lens)])
    for r in range(2):
        np.testing.assert_array_equal(results[r], want)


# ---- failure detection and re-queue (host-side faults; no GPU involved) ----

class _InputError(Exception):
    code = -1  # EG2_ERR_INVALID, as lib.Eg2Error carries it


def _fake_worker(tag, fail_on_call=None, bad_token=None):
    """A stand-in GPU worker: embeds a document as [len, first id, tag]. It raises a device-style error
    on its `fail_on_call`-th call, and an input error for any batch holding `bad_token`."""
    calls = {"n": 0}

    def embed(seqs):
        calls["n"] += 1
        if fail_on_call is not None and calls["n"] == fail_on_call:
            raise RuntimeError(f"worker {tag}: device lost")
        if bad_token is not None and any(bad_token in s for s in seqs):
            raise _InputError("token id out of range")
        return np.stack([np.array([len(s), s[0], 0.0], np.float32) for s in seqs])

    return embed


def _docs(n=23, seed=3):
    rng = np.random.default_rng(seed)
    return [rng.integers(0, 1000, size=int(l)).astype(np.uint32) for l in rng.integers(1, 3000, size=n)]


def _check(res, seqs):
    for s, r in zip(seqs, res):
        assert r[0] == len(s) and r[1] == s[0]


def test_reassign_gives_orphans_to_survivors_only():
    lens = [700, 3, 2208, 17, 130, 1100, 9, 400]
    shards = S.assign(lens, 3)
    extra = S.reassign(lens, shards, {1})
    assert extra[1] == [] and sorted(extra[0] + extra[2]) == shards[1]
    assert S.reassign(lens, shards, {1}) == extra  # every survivor computes the same plan
    with pytest.raises(RuntimeError):
        S.reassign(lens, shards, {0, 1, 2})


def test_dispatch_requeues_a_failed_gpu():
    seqs = _docs()
    res, rep = S.dispatch([_fake_worker(0), _fake_worker(1, fail_on_call=1), _fake_worker(2)], seqs)
    _check(res, seqs)
    assert rep["failed_workers"] == [1] and rep["rounds"] == 2 and rep["input_errors"] == []


def test_dispatch_cascading_failures_end_on_the_last_gpu():
    seqs = _docs(seed=4)
    res, rep = S.dispatch([_fake_worker(0), _fake_worker(1, fail_on_call=1), _fake_worker(2, fail_on_call=2)], seqs)
    _check(res, seqs)
    assert rep["failed_workers"] == [1, 2]


def test_dispatch_input_error_fails_only_its_document():
    seqs = _docs(seed=5)
    seqs[7] = np.array([5, 999999, 6], np.uint32)
    res, rep = S.dispatch([_fake_worker(0, bad_token=999999), _fake_worker(1, bad_token=999999)], seqs)
    assert isinstance(res[7], S.DocumentError)
    _check([r for i, r in enumerate(res) if i != 7], [s for i, s in enumerate(seqs) if i != 7])
    assert rep["failed_workers"] == [] and rep["input_errors"] == [7]


def test_dispatch_every_gpu_failing_raises():
    with pytest.raises(RuntimeError):
        S.dispatch([_fake_worker(0, fail_on_call=1), _fake_worker(1, fail_on_call=1)], _docs())


def _takeover_worker(rank, world, port, lens, mode, q):
    import importlib
    import sys
    from datetime import timedelta

    import torch.distributed as dist

    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    sh = importlib.import_module("embeddinggemma2-rust_b200.shard")
    store = dist.TCPStore("127.0.0.1", port, world, rank == 0, timeout=timedelta(seconds=60))
    if mode.get(rank) == "never_joins":
        q.put((rank, "left"))
        return

    def embed(idx):
        if mode.get(rank) == "raises":
            raise RuntimeError("device lost")
        return np.stack([np.full(4, lens[i] * 10 + i, np.float32) for i in idx])

    out = sh.run_rank_with_takeover(rank, world, store, lens, embed, timeout_s=5.0)
    q.put((rank, out))
    if rank == 0:
        # The store lives in rank 0: keep it up until the other survivors have read their results.
        import time
        time.sleep(2.0)


@pytest.mark.parametrize("mode", [{1: "raises"}, {2: "never_joins"}, {}])
def test_ranks_take_over_a_failed_rank(mode):
    import multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    lens = [700, 3, 2208, 17, 130, 1100, 9, 400, 64]
    port = _free_port()
    procs = [ctx.Process(target=_takeover_worker, args=(r, 3, port, lens, mode, q)) for r in range(3)]
    for p in procs:
        p.start()
    results = dict(q.get(timeout=120) for _ in procs)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    want = np.stack([np.full(4, l * 10 + i, np.float32) for i, l in enumerate(lens)])
    for r in range(3):
        if mode.get(r) == "raises":
            assert results[r] is None
        elif mode.get(r) == "never_joins":
            assert results[r] == "left"
        else:
            np.testing.assert_array_equal(results[r], want)
