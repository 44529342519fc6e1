"""Build libllattn.so (sm_100a) in-tree with nvcc.

    python build.py            # incremental: rebuilds objects whose sources changed
    python build.py --clean    # drop objects first

Objects go to csrc/_build/, the library to the package directory, next to
the Python code that loads it. Flags: -gencode arch=compute_100a,code=sm_100a
-lineinfo -O3; LLATTN_CHECK_BOUNDS=1 in the environment adds the device-side
bounds checks of the tensor-core kernels (error word instead of a trap).
"""

from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

CSRC = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.dirname(CSRC)
ROOT = os.path.dirname(PKG)
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(CSRC, "_build")
LIB = os.path.join(PKG, "libllattn.so")
SOURCES = ["api.cu", "pool.cu", "latent.cu", "local_simt.cu", "gate.cu", "local_sm100.cu", "decode.cu", "profile.cu"]
NVCC = os.environ.get("NVCC", shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc")


def flags() -> list[str]:
    f = ["-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo", "-O3", "-std=c++17",
         "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden", "--expt-relaxed-constexpr",
         "-I" + INCLUDE, "-I" + CSRC]
    if os.environ.get("LLATTN_CHECK_BOUNDS") == "1":
        f.append("-DLLATTN_CHECK_BOUNDS=1")
    if os.environ.get("LLATTN_TRACE", "0") not in ("", "0"):
        # diagnostic builds: 1 = forward, 2 = dK/dV, 3 = gate backward phase timestamps
        f.append("-DLLATTN_TRACE=" + os.environ["LLATTN_TRACE"])
    if os.environ.get("LLATTN_PTXAS_V") == "1":
        f += ["-Xptxas", "-v"]
    return f


def _digest(src: str, fl: list[str]) -> str:
    h = hashlib.sha256(" ".join(fl).encode())
    for name in sorted(os.listdir(CSRC)) + sorted(os.listdir(INCLUDE)):
        if name.endswith((".cuh", ".h")):
            path = os.path.join(CSRC if name.endswith(".cuh") else INCLUDE, name)
            with open(path, "rb") as fh:
                h.update(fh.read())
    with open(src, "rb") as fh:
        h.update(fh.read())
    return h.hexdigest()[:16]


def _compile(name: str, fl: list[str]) -> str:
    src = os.path.join(CSRC, name)
    obj = os.path.join(BUILD, name.replace(".cu", f".{_digest(src, fl)}.o"))
    if not os.path.exists(obj):
        cmd = [NVCC, *fl, "-c", src, "-o", obj + ".tmp"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {name}:\n{r.stdout}\n{r.stderr}")
        if r.stderr.strip() and os.environ.get("LLATTN_PTXAS_V") == "1":
            sys.stderr.write(r.stderr)
        os.replace(obj + ".tmp", obj)
        stem = name.replace(".cu", ".")
        for old in os.listdir(BUILD):  # drop objects of earlier versions of this source
            if old.startswith(stem) and old.endswith(".o") and os.path.join(BUILD, old) != obj:
                os.remove(os.path.join(BUILD, old))
    return obj


def build(clean: bool = False) -> str:
    if clean and os.path.isdir(BUILD):
        shutil.rmtree(BUILD)
    os.makedirs(BUILD, exist_ok=True)
    fl = flags()
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda n: _compile(n, fl), SOURCES))
    tmp = LIB + ".tmp"
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", *objs, "-o", tmp,
           "-Xcompiler", "-fPIC"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(clean="--clean" in sys.argv))
