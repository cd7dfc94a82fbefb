"""Builds libjanus_b200.so from csrc/*.cu with nvcc for sm_100a (in-tree, next to this file).

    python -m janus_b200.build            # incremental: rebuilds when a source or header is newer than the library
"""

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

HERE = Path(__file__).resolve().parent
SRC = HERE / "csrc"
INCLUDE = HERE.parent / "include"
LIB = HERE / "libjanus_b200.so"
OBJ = HERE / "_build"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-I", str(INCLUDE)]


def nvcc():
    home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = Path(home) / "bin" / "nvcc"
    return str(path) if path.exists() else "nvcc"


def sources():
    return sorted(SRC.glob("*.cu"))


def _stale(target, deps):
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose=False, force=False, extra=()):
    headers = list(SRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    OBJ.mkdir(exist_ok=True)
    jobs = []
    for cu in sources():
        obj = OBJ / (cu.stem + ".o")
        if force or _stale(obj, [cu, *headers]):
            jobs.append([nvcc(), *ARCH, *FLAGS, *extra, "-c", str(cu), "-o", str(obj)])

    def run(cmd):
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
        if verbose and (r.stdout or r.stderr):
            print(r.stdout, r.stderr, sep="\n", flush=True)

    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as pool:
        list(pool.map(run, jobs))
    objs = [OBJ / (cu.stem + ".o") for cu in sources()]
    if force or jobs or _stale(LIB, objs):
        run([nvcc(), *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"])
    return LIB


if __name__ == "__main__":
    build(verbose="-v" in sys.argv, force="-f" in sys.argv)
    print(LIB)
