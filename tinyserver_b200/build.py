"""Build libqwen3fused.so (the sm_100a kernels + C ABI) in-tree with nvcc.

    python -m tinyserver_b200.build [--force] [--verbose-ptxas]

Objects go to tinyserver_b200/_build/, the library to
tinyserver_b200/lib/libqwen3fused.so.  The CUDA runtime is linked statically,
so the library only needs the driver at run time; it shares the primary
context (and therefore streams and device pointers) with torch.
"""

from __future__ import annotations

import argparse
import concurrent.futures as cf
import fcntl
import glob
import hashlib
import os
import shutil
import subprocess

PKG = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(PKG)
CSRC = os.path.join(PKG, "csrc")
INCLUDE = os.path.join(ROOT, "include")
BUILD = os.path.join(PKG, "_build")
LIB = os.path.join(PKG, "lib", "libqwen3fused.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O2",
              "--expt-relaxed-constexpr", "-I", INCLUDE, "-I", CSRC]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found: cannot build libqwen3fused.so")


def sources() -> list[str]:
    return sorted(glob.glob(os.path.join(CSRC, "*.cu")))


def _deps() -> list[str]:
    return sources() + glob.glob(os.path.join(CSRC, "*.cuh")) + \
        glob.glob(os.path.join(INCLUDE, "*.h"))


def source_hash() -> str:
    """Hash of every source the library is built from (file names and bytes)."""
    h = hashlib.sha256()
    for p in sorted(_deps()):
        h.update(os.path.basename(p).encode())
        with open(p, "rb") as f:
            h.update(f.read())
    return h.hexdigest()


STAMP = LIB + ".srchash"


def is_stale() -> bool:
    """Whether the library is missing or was built from other sources.  The
    sources' hash decides, not mtimes, which a copy of the tree to another
    machine does not preserve."""
    if not os.path.exists(LIB) or not os.path.exists(STAMP):
        return True
    with open(STAMP) as f:
        return f.read().strip() != source_hash()


def _compile(src: str, verbose_ptxas: bool) -> str:
    obj = os.path.join(BUILD, os.path.basename(src)[:-3] + ".o")
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", src, "-o", obj]
    if verbose_ptxas:
        cmd += ["-Xptxas", "-v"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    if verbose_ptxas:
        print(r.stderr)
    return obj


def build(force: bool = False, verbose_ptxas: bool = False) -> str:
    """Compile every csrc/*.cu for sm_100a and link the shared library, then
    record the sources' hash beside it.  Processes that build at the same time
    (the ranks of one job) take turns on a file lock, and a process that gets
    the lock after another built the same sources does nothing."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(os.path.dirname(LIB), exist_ok=True)
    with open(LIB + ".lock", "w") as lock:
        fcntl.flock(lock, fcntl.LOCK_EX)
        if not force and not verbose_ptxas and not is_stale():
            return LIB
        want = source_hash()
        with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
            objs = list(ex.map(lambda s: _compile(s, verbose_ptxas), sources()))
        tmp = f"{LIB}.tmp{os.getpid()}"
        cmd = [nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", tmp, *objs]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
        with open(STAMP, "w") as f:
            f.write(want)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose_ptxas=args.verbose_ptxas))


if __name__ == "__main__":
    main()
