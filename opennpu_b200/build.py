"""Build libonpu.so (the CUDA library behind the onpu_* C ABI) in-tree, for sm_100a only.

    python -m opennpu_b200.build            # incremental
    python -m opennpu_b200.build --force

Objects go to opennpu_b200/_build/, the library to opennpu_b200/_lib/libonpu.so. nvcc
cross-compiles without a GPU, so this runs on the CPU-only build host too.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "_lib" / "libonpu.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-ffp-contract=off", f"-I{ROOT / 'include'}",
          f"-I{CSRC}"]


def sources():
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp"))


def headers():
    return sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.hpp")) + \
        sorted((ROOT / "include").glob("*.h"))


def _compile(src, obj, verbose):
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"] if verbose else []
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{r.stdout}\n{r.stderr}")
    return r.stderr


def build(force=False, verbose=False, jobs=None):
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    newest_header = max((h.stat().st_mtime for h in headers()), default=0)
    todo = []
    objs = []
    for src in sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append((src, obj))
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count()) as ex:
        for (src, _), log in zip(todo, ex.map(lambda so: _compile(so[0], so[1], verbose), todo)):
            if verbose and log:
                print(f"== {src.name}\n{log}")
    if todo or not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true")
    a = ap.parse_args(argv)
    print(build(a.force, a.verbose))


if __name__ == "__main__":
    sys.exit(main())
