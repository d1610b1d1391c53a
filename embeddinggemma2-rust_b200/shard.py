"""Sharding documents across GPUs (one process per GPU) and gathering their embeddings.

The path shards by document: attention is block-diagonal per sequence (src/text.rs:183-202), so every
document is independent and ranks never exchange activations. Documents are assigned longest-first to the
least-loaded rank (LPT) by estimated cost — projection work grows with the length, global-layer
attention with its square — and each rank embeds its share in one packed pass. The embeddings come back
to every rank (or rank 0) in input order through ``torch.distributed`` (gloo on CPU, NCCL on GPUs): the
only communication is this final gather of [n_docs, dims] floats.
"""
from __future__ import annotations

import heapq

import numpy as np


def doc_cost(length: int, window: int = 512) -> float:
    """Relative cost of one document: per-token GEMM work plus attention pairs (20 sliding layers
    with radius `window`, 4 global layers; weights as in the FLOP count of the benchmark)."""
    gemm = 273_416_192.0 * length
    i = np.arange(length)
    sliding_pairs = float((np.minimum(i + window, length - 1) - np.maximum(i - window, 0) + 1).sum())
    attn = 20 * 4 * 1024 * sliding_pairs + 4 * 4 * 2048 * float(length) ** 2
    return gemm + attn


def assign(lens, world: int) -> list[list[int]]:
    """Indices of the documents each rank embeds: longest-first to the least-loaded rank. Ties go to
    the lower rank and equal lengths keep input order, so every rank computes the same plan."""
    if world <= 0:
        raise ValueError("world must be positive")
    order = sorted(range(len(lens)), key=lambda i: (-int(lens[i]), i))
    heap = [(0.0, r) for r in range(world)]
    shards: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        load, r = heapq.heappop(heap)
        shards[r].append(i)
        heapq.heappush(heap, (load + doc_cost(int(lens[i])), r))
    for s in shards:
        s.sort()
    return shards


def gather(local: np.ndarray, shards: list[list[int]], rank: int, n_docs: int, dist) -> np.ndarray:
    """All-gather each rank's [len(shards[rank]), D] embeddings and scatter them back into input order."""
    import torch

    d = local.shape[1] if local.ndim == 2 else 0
    world = len(shards)
    width = max(len(s) for s in shards)
    buf = torch.zeros((width, d), dtype=torch.float32)
    buf[: local.shape[0]] = torch.from_numpy(np.ascontiguousarray(local, dtype=np.float32))
    backend = dist.get_backend()
    if backend == "nccl":
        buf = buf.cuda()
    parts = [torch.zeros_like(buf) for _ in range(world)]
    dist.all_gather(parts, buf)
    out = np.zeros((n_docs, d), dtype=np.float32)
    for r in range(world):
        p = parts[r].cpu().numpy()
        for j, i in enumerate(shards[r]):
            out[i] = p[j]
    return out


# ---------------------------------------------------------------------------------------------
# Failure detection and re-queue. The reference's server catches a failed batch and re-runs its jobs
# one by one, so one bad request cannot fail the others it was merged with (src/serve.rs:537-543,
# :570-595). Across GPUs the same idea: a shard whose GPU reports a device failure (CUDA error, a
# bounded wait that ran out, out of memory) is re-queued on the GPUs still healthy; a shard that fails
# on its input (EG2_ERR_INVALID: an id out of range, an empty sequence) is re-run document by document
# on the same GPU, so only the bad documents fail.
# ---------------------------------------------------------------------------------------------
INVALID_INPUT = -1  # EG2_ERR_INVALID


def is_input_error(exc: BaseException) -> bool:
    """A failure caused by the documents themselves, not by the GPU."""
    return getattr(exc, "code", None) == INVALID_INPUT


def reassign(lens, shards: list[list[int]], failed) -> list[list[int]]:
    """The documents of the `failed` ranks, added longest-first to the least-loaded surviving rank
    (loads counted from each survivor's own shard). Deterministic: every survivor computes the same
    plan. Raises when no rank survives."""
    failed = set(failed)
    alive = [r for r in range(len(shards)) if r not in failed]
    if not alive:
        raise RuntimeError("every rank failed")
    heap = [(sum(doc_cost(int(lens[i])) for i in shards[r]), r) for r in alive]
    heapq.heapify(heap)
    extra: list[list[int]] = [[] for _ in shards]
    orphans = sorted((i for r in failed for i in shards[r]), key=lambda i: (-int(lens[i]), i))
    for i in orphans:
        load, r = heapq.heappop(heap)
        extra[r].append(i)
        heapq.heappush(heap, (load + doc_cost(int(lens[i])), r))
    for s in extra:
        s.sort()
    return extra


class DocumentError:
    """Placeholder result of a document that failed on its own input."""

    def __init__(self, exc: BaseException):
        self.exc = exc

    def __repr__(self):
        return f"DocumentError({self.exc!r})"


def _run_shard(embed, seqs, idx):
    """embed(list of sequences) -> [n, D]; on an input error, document by document."""
    try:
        out = embed([seqs[i] for i in idx]) if idx else None
        return {i: out[j] for j, i in enumerate(idx)}
    except Exception as e:  # noqa: BLE001 - classified below
        if not is_input_error(e) or len(idx) <= 1:
            if is_input_error(e):
                return {idx[0]: DocumentError(e)}
            raise
        res = {}
        for i in idx:
            try:
                res[i] = embed([seqs[i]])[0]
            except Exception as e1:  # noqa: BLE001
                if not is_input_error(e1):
                    raise
                res[i] = DocumentError(e1)
        return res


def dispatch(workers, seqs, max_rounds: int | None = None):
    """Embed `seqs` over several GPUs driven from one process, one host thread per GPU (one library
    context each; contexts on different GPUs run concurrently). `workers[r]` is a callable
    list-of-sequences -> [n, D] array bound to GPU r.

    Returns (results in input order, report). A worker that raises anything but an input error is
    marked failed and its documents are re-queued on the remaining workers (repeatedly, until every
    document is done or no worker is left). A document whose input is invalid yields a DocumentError
    in its slot instead of failing the others."""
    import threading

    lens = [len(s) for s in seqs]
    world = len(workers)
    shards = assign(lens, world)
    done: dict[int, object] = {}
    failed: set[int] = set()
    errors: dict[int, str] = {}
    pending = shards
    rounds = 0
    while True:
        rounds += 1
        results: dict[int, dict] = {}
        threads = []

        def work(r, idx):
            try:
                results[r] = _run_shard(workers[r], seqs, idx)
            except BaseException as e:  # noqa: BLE001 - any device-side failure
                errors[r] = f"{type(e).__name__}: {e}"

        for r in range(world):
            if r in failed or not pending[r]:
                continue
            t = threading.Thread(target=work, args=(r, pending[r]), daemon=True)
            threads.append(t)
            t.start()
        for t in threads:
            t.join()
        newly = {r for r in range(world) if r not in failed and pending[r] and r not in results}
        for r, res in results.items():
            done.update(res)
        if not newly:
            break
        failed |= newly
        if max_rounds is not None and rounds >= max_rounds:
            break
        # Re-queue what the failed workers held on the survivors (their own shards are already done).
        orphan_shards = [[i for i in pending[r] if i not in done] if r in newly else [] for r in range(world)]
        pending = reassign(lens, orphan_shards, failed)
    missing = [i for i in range(len(seqs)) if i not in done]
    if missing:
        raise RuntimeError(f"{len(missing)} document(s) not embedded: every GPU failed ({errors})")
    report = {"failed_workers": sorted(failed), "errors": errors, "rounds": rounds,
              "input_errors": sorted(i for i, v in done.items() if isinstance(v, DocumentError))}
    return [done[i] for i in range(len(seqs))], report


def run_rank_with_takeover(rank: int, world: int, store, lens, embed, timeout_s: float = 30.0, poll_s: float = 0.05):
    """Multi-process form (one process per GPU): each rank embeds its shard and publishes the result
    and its status in a key-value store (a torch.distributed TCPStore); a rank that fails leaves. The
    others learn of it on the host -- a 'failed' status, or no status within `timeout_s` (a rank that
    died or never joined) -- and take over its documents with the deterministic `reassign` plan. No
    collective is used, so a missing rank cannot block the others. Returns the [n, D] embeddings in
    input order on every surviving rank, or None on a rank that failed."""
    import pickle
    import time

    shards = assign(lens, world)

    def publish(tag, res):
        store.set(f"{tag}/{rank}", pickle.dumps({i: np.asarray(v, np.float32) for i, v in res.items()}))

    try:
        mine = shards[rank]
        out = embed(mine) if mine else np.zeros((0, 0), np.float32)
        publish("res", {i: out[j] for j, i in enumerate(mine)})
        store.set(f"status/{rank}", "ok")
    except Exception as e:  # noqa: BLE001 - the rank leaves; the others take over
        store.set(f"status/{rank}", f"failed: {type(e).__name__}")
        return None

    def status(r, deadline):
        while True:
            try:
                if store.check([f"status/{r}"]):
                    return store.get(f"status/{r}").decode()
            except Exception:  # noqa: BLE001
                pass
            if time.monotonic() > deadline:
                return "missing"
            time.sleep(poll_s)

    deadline = time.monotonic() + timeout_s
    st = {r: status(r, deadline) for r in range(world)}
    failed = {r for r, v in st.items() if v != "ok"}
    results: dict[int, np.ndarray] = {}
    for r in range(world):
        if r not in failed:
            results.update(pickle.loads(store.get(f"res/{r}")))
    if failed:
        extra = reassign(lens, shards, failed)
        mine = extra[rank]
        if mine:
            out = embed(mine)
            publish("takeover", {i: out[j] for j, i in enumerate(mine)})
        store.set(f"takeover_done/{rank}", "1")
        for r in range(world):
            if r in failed:
                continue
            store.wait([f"takeover_done/{r}"])
            if extra[r]:
                results.update(pickle.loads(store.get(f"takeover/{r}")))
    n = len(lens)
    d = next(iter(results.values())).shape[0] if results else 0
    out = np.zeros((n, d), np.float32)
    for i, v in results.items():
        out[i] = v
    missing = [i for i in range(n) if i not in results]
    if missing:
        raise RuntimeError(f"documents {missing[:8]} were not embedded")
    return out
