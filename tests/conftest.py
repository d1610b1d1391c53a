"""Shared fixtures. GPU tests carry ``@pytest.mark.gpu``; everything else runs on the CPU.

The checkpoint is the seeded random-init one (``weights.make_random_checkpoint``), generated once
per session into a temporary directory.
"""
from __future__ import annotations

import importlib
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
for p in (str(ROOT), str(ROOT / "oracle")):
    if p not in sys.path:
        sys.path.insert(0, p)

PKG = "embeddinggemma2-rust_b200"


def pkg(mod: str = ""):
    return importlib.import_module(PKG + ("." + mod if mod else ""))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 (sm_100a) GPU")


@pytest.fixture(scope="session")
def model_dir(tmp_path_factory) -> Path:
    d = tmp_path_factory.mktemp("eg2_model")
    pkg("weights").make_random_checkpoint(d, seed=0, vision=True)
    return d


@pytest.fixture(scope="session")
def oracle_text(model_dir):
    import oracle

    return oracle.OracleText(model_dir)


@pytest.fixture(scope="session")
def oracle_vision(model_dir):
    import oracle

    return oracle.OracleVision(model_dir)


def _gpu_device(model_dir, precision):
    import torch

    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    return pkg("backend").Device(model_dir, 0, precision)


@pytest.fixture(scope="session")
def dev_bf16(model_dir):
    d = _gpu_device(model_dir, "bf16")
    yield d
    d.close()


@pytest.fixture(scope="session")
def dev_tf32(model_dir):
    d = _gpu_device(model_dir, "tf32")
    yield d
    d.close()


@pytest.fixture(scope="session")
def dev_f32(model_dir):
    d = _gpu_device(model_dir, "f32")
    yield d
    d.close()
