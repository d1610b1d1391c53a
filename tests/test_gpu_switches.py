"""Launch-mode switches change how work is scheduled, never the arithmetic: a pass run with programmatic
dependent launch turned off (EG2_NO_PDL=1) gives the same bits as the default run, for a mix of long and
short documents (fused epilogues, the K-split path of short passes, CUDA-graph replay). Each variant
runs in its own process because the library reads the switch once."""
import json
import os
import subprocess
import sys

import numpy as np
import pytest

from conftest import ROOT

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import importlib, json, sys
import numpy as np
sys.path.insert(0, sys.argv[1])
B = importlib.import_module("embeddinggemma2-rust_b200.backend")
dev = B.Device(sys.argv[2], 0, "bf16")
tb = B.TextBackend(dev)
rng = np.random.default_rng(11)
out = {}
for name, lens in (("long", [700, 33, 1200]), ("short", [17, 40])):
    seqs = [rng.integers(0, 262144, size=n).astype(np.uint32) for n in lens]
    emb = tb.embed_ids(seqs)
    out[name] = np.asarray(emb[768]).astype(np.float32).view(np.uint32).tolist()
json.dump(out, open(sys.argv[3], "w"))
"""


def run_variant(tmp_path, model_dir, env_extra, tag):
    script = tmp_path / "embed_variant.py"
    script.write_text(SCRIPT)
    out = tmp_path / f"{tag}.json"
    env = dict(os.environ)
    env.pop("EG2_NO_PDL", None)
    env.update(env_extra)
    subprocess.run([sys.executable, str(script), str(ROOT), str(model_dir), str(out)], env=env, check=True,
                   timeout=600)
    return json.load(open(out))


def test_no_pdl_is_bit_identical(tmp_path, model_dir):
    base = run_variant(tmp_path, model_dir, {}, "default")
    nopdl = run_variant(tmp_path, model_dir, {"EG2_NO_PDL": "1"}, "nopdl")
    for name in ("long", "short"):
        a = np.array(base[name], dtype=np.uint32)
        b = np.array(nopdl[name], dtype=np.uint32)
        assert a.shape == b.shape and a.size > 0
        np.testing.assert_array_equal(a, b, err_msg=name)
