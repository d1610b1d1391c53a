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
