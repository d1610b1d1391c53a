"""Oracle outputs for the workloads too large to run through the CPU oracle inside a GPU test.

The CPU oracle (oracle/, the C restatement of the reference's CPU f32 path, src/text.rs:136-235)
needs minutes for these, so its results are computed once here and committed; the GPU tests compare
the library against them. Each case is a workload of BASELINE.json's configs on the seeded random-init
checkpoint (``weights.make_random_checkpoint(seed=0)``):

* ``c1``: one sequence of 512 token ids, uniform over the vocabulary, seed 0;
* ``c3``: 64 documents with lengths uniform in [128, 2208] and uniform ids, seed 7 -- the same
  draw as bench.py's mixed-length leg;
* ``c4``: one sequence of 11,774 uniform ids, seed 11774 (configs[3], the reference's long case,
  README.md:46).

Stored per case: the token-id lengths, the ids' generator, and the 768-d mean-pooled L2-normalised
embeddings (f32); the Matryoshka cuts follow from them (src/model.rs:677-688). The checkpoint's
SHA-256 is stored too, so a test can tell when the generator's checkpoint no longer matches.

Run (CPU; about 10 minutes on 8 cores):  python tests/golden/make_oracle_fixtures.py
"""
from __future__ import annotations

import hashlib
import importlib
import sys
import tempfile
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parents[2]
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))
wmod = importlib.import_module("embeddinggemma2-rust_b200.weights")

OUT = Path(__file__).resolve().parent / "oracle_fixtures.npz"
VOCAB = 262144


def case_ids(name: str) -> list[np.ndarray]:
    """The token ids of a case (the same draws bench.py and the tests make)."""
    if name == "c1":
        return [np.random.default_rng(0).integers(0, VOCAB, size=512).astype(np.uint32)]
    if name == "c3":
        rng = np.random.default_rng(7)
        lens = rng.integers(128, 2208 + 1, size=64)
        return [rng.integers(0, VOCAB, size=int(n)).astype(np.uint32) for n in lens]
    if name == "c4":
        return [np.random.default_rng(11774).integers(0, VOCAB, size=11774).astype(np.uint32)]
    raise KeyError(name)


def checkpoint_sha256(model_dir: Path) -> str:
    h = hashlib.sha256()
    with open(Path(model_dir) / "model.safetensors", "rb") as f:
        for chunk in iter(lambda: f.read(1 << 24), b""):
            h.update(chunk)
    return h.hexdigest()


def main() -> None:
    import oracle as O

    out = {}
    with tempfile.TemporaryDirectory() as d:
        wmod.make_random_checkpoint(d, seed=0, vision=False)
        out["checkpoint_sha256"] = np.array(checkpoint_sha256(Path(d)))
        m = O.OracleText(d)
        for name in ("c1", "c4", "c3"):
            seqs = case_ids(name)
            t0 = time.perf_counter()
            # One sequence per oracle pass: the oracle's result for a sequence does not depend on its
            # neighbours, and single passes keep the peak memory small.
            emb = np.concatenate([m.embed_ids([s]) for s in seqs], axis=0).astype(np.float32)
            print(f"{name}: {len(seqs)} sequence(s), {sum(len(s) for s in seqs)} tokens, "
                  f"{time.perf_counter() - t0:.1f} s", flush=True)
            out[f"{name}_lens"] = np.array([len(s) for s in seqs], dtype=np.int64)
            out[f"{name}_emb"] = emb
    np.savez_compressed(OUT, **out)
    print(OUT)


if __name__ == "__main__":
    main()
