"""Build recipe for libcab_b200.so (sm_100a only).

``python cab_build.py`` compiles ``csrc/cab_lib.cu`` (one translation unit holding every
kernel) with nvcc into ``cab_attention/libcab_b200.so`` next to the Python package, so the
library travels with the source tree. The CUDA runtime is linked statically and the
driver is reached through ``cudaGetDriverEntryPoint`` at run time, so the library loads
on a machine without a GPU driver (its compute entry points then fail with
CAB_ERR_LAUNCH).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
CSRC = HERE / "csrc"
OUT = HERE / "cab_attention" / "libcab_b200.so"
INCLUDE = HERE.parent / "include"


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found")
    return cand


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + \
        sorted(INCLUDE.glob("*.h"))


def needs_build() -> bool:
    if not OUT.exists():
        return True
    t = OUT.stat().st_mtime
    return any(s.stat().st_mtime > t for s in sources())


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return OUT
    cmd = [
        nvcc_path(), "-std=c++17", "-O3", "-lineinfo",
        "-gencode", "arch=compute_100a,code=sm_100a",
        "-shared", "-Xcompiler", "-fPIC,-fvisibility=hidden",
        "-cudart", "static",
        "-I", str(INCLUDE),
        "-o", str(OUT) + ".tmp",
        str(CSRC / "cab_lib.cu"),
    ]
    if verbose:
        cmd.insert(4, "-Xptxas=-v")
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError("nvcc failed:\n" + res.stdout + res.stderr)
    if verbose:
        sys.stderr.write(res.stderr)
    os.replace(str(OUT) + ".tmp", OUT)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
    print(OUT)
