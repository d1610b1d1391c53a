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
