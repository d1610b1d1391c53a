"""Failure detection across GPU workers (backend.embed_on_gpus / shard.dispatch), with the failure made
on the host: a worker that raises as a lost GPU would. Its documents are re-queued on the healthy
context and the results equal a plain call; an invalid document fails alone. Two contexts on cuda:0
stand in for two GPUs (no kernel of one waits on the other)."""
import numpy as np
import pytest

from conftest import pkg

B = pkg("backend")
L = pkg("lib")

pytestmark = pytest.mark.gpu


class _LostGpu:
    """A TextBackend stand-in whose device is gone: every call raises a CUDA-class error."""

    def __init__(self, dev):
        self.dev = dev

    def embed_ids(self, seqs, dims):
        raise L.Eg2Error(-3, "device lost (injected on the host)")


def test_requeue_on_the_healthy_gpu(dev_bf16, model_dir):
    rng = np.random.default_rng(8)
    seqs = [rng.integers(0, 262144, size=int(n)).astype(np.uint32) for n in rng.integers(1, 900, size=12)]
    want = B.TextBackend(dev_bf16).embed_ids(seqs)
    got, rep = B.embed_on_gpus([_LostGpu(dev_bf16), B.TextBackend(dev_bf16)], seqs)
    assert rep["failed_workers"] == [0]
    # The re-queued documents ran as one call on the healthy context: compare within the profile
    # (their pass composition differs from the single call's, so the last bits may too).
    assert np.abs(got[768] - want[768]).max() < 4e-3


def test_invalid_document_fails_alone(dev_bf16, model_dir):
    other = B.Device(model_dir, 0, "bf16")
    try:
        rng = np.random.default_rng(9)
        seqs = [rng.integers(0, 262144, size=int(n)).astype(np.uint32) for n in (40, 300, 7, 1200)]
        seqs[2] = np.array([1, 262144 + 5, 2], np.uint32)  # id out of range
        got, rep = B.embed_on_gpus([B.TextBackend(dev_bf16), B.TextBackend(other)], seqs)
        assert rep["failed_workers"] == [] and rep["input_errors"] == [2]
        assert np.isnan(got[768][2]).all() and np.isfinite(got[768][[0, 1, 3]]).all()
        alone = B.TextBackend(dev_bf16).embed_ids([seqs[3]])[768][0]
        assert np.abs(got[768][3] - alone).max() < 4e-3
    finally:
        other.close()
