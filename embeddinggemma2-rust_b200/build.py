"""Build libeg2_b200.so (sm_100a) in-tree with nvcc.

One translation unit (csrc/eg2_lib.cu includes the kernel and runtime sources). The library links
the CUDA runtime statically and reaches the driver's cuTensorMapEncodeTiled through
cudaGetDriverEntryPoint, so it needs no -lcuda and no torch.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "_lib" / "libeg2_b200.so"
SOURCES = ["eg2_lib.cu", "common.cuh", "kernels.h", "json.h", "gemm_tc.cu", "simt.cu", "rowops.cu", "attention_tc.cu", "noalloc.cu", "probe.cu", "runtime.cu"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def host_compiler() -> list[str]:
    # The system g++ matches the CUDA 12.9 host-compiler requirements.
    gxx = "/usr/bin/g++"
    return ["-ccbin", gxx] if Path(gxx).exists() else []


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + [HERE.parent / "include" / "eg2.h", Path(__file__)]
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    OUT.parent.mkdir(parents=True, exist_ok=True)
    tmp = OUT.with_suffix(".so.tmp")
    cmd = [
        nvcc(), *host_compiler(),
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
        "-Xcompiler", "-fPIC", "-shared",
        "-Xptxas", "-v" if verbose else "-O3",
        "-o", str(tmp), str(CSRC / "eg2_lib.cu"),
    ]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("nvcc failed building libeg2_b200.so")
    if verbose:
        sys.stderr.write(r.stderr)
    tmp.replace(OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
