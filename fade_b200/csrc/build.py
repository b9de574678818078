"""Build libfade_sm100.so in-tree with nvcc (sm_100a only).

Run as ``python -m fade_b200.csrc.build`` or through ``__graft_entry__.build()``.
The library is a plain C-ABI shared object: no torch headers, CUDA runtime
linked statically, compiled without --use_fast_math (the quantisers are
bit-exact with IEEE division and round-to-nearest-even).
"""

from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

CSRC = Path(__file__).resolve().parent
PKG = CSRC.parent
LIB_NAME = "libfade_sm100.so"
SOURCES = ("abi.cu", "quant.cu", "rotate.cu", "rope.cu", "decode.cu")

NVCC_FLAGS = [
    "-O3",
    "-std=c++17",
    "-gencode",
    "arch=compute_100a,code=sm_100a",
    "-lineinfo",
    "-Xcompiler",
    "-fPIC",
    "--expt-relaxed-constexpr",
]


def nvcc_path() -> str:
    cand = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not Path(cand).exists():
        raise RuntimeError("nvcc not found; libfade_sm100.so cannot be built")
    return cand


def lib_path() -> Path:
    return PKG / LIB_NAME


def needs_build() -> bool:
    out = lib_path()
    if not out.exists():
        return True
    mtime = out.stat().st_mtime
    deps = [CSRC / s for s in SOURCES] + list(CSRC.glob("*.cuh")) + list((PKG.parent / "include").glob("*.h"))
    return any(p.exists() and p.stat().st_mtime > mtime for p in deps)


def build(force: bool = False, verbose: bool = False) -> Path:
    out = lib_path()
    if not force and not needs_build():
        return out
    nvcc = nvcc_path()
    objdir = PKG / "_build"
    objdir.mkdir(exist_ok=True)
    objs = []
    procs = []
    for src in SOURCES:
        obj = objdir / (Path(src).stem + ".o")
        cmd = [nvcc, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            print(" ".join(cmd), file=sys.stderr)
        procs.append((src, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
        objs.append(str(obj))
    for src, p in procs:
        txt, _ = p.communicate()
        if p.returncode != 0:
            raise RuntimeError(f"nvcc failed on {src}:\n{txt.decode(errors='replace')}")
    tmp = out.with_suffix(".so.tmp")
    cmd = [nvcc, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", str(tmp)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}{r.stderr}")
    os.replace(tmp, out)
    return out


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True))
