"""Build of ``libnnop_b200.so`` (the C-ABI library) for sm_100a.

Every ``csrc/*.cu`` is compiled separately with nvcc (in parallel) and linked
into ``onionop.jl_b200/lib/libnnop_b200.so``.  The library links the CUDA
runtime statically and has no torch dependency, so any host language can load
it (Julia ``ccall``, Python ``ctypes``).
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import pathlib
import shutil
import subprocess

PKG_ROOT = pathlib.Path(__file__).resolve().parent.parent      # onionop.jl_b200/
CSRC = PKG_ROOT / "csrc"
LIB_DIR = PKG_ROOT / "lib"
LIB_PATH = LIB_DIR / "libnnop_b200.so"
BUILD_DIR = PKG_ROOT / "_build"
INCLUDE = PKG_ROOT.parent / "include"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-O2",
    "--expt-relaxed-constexpr", "-I", str(INCLUDE), "-I", str(CSRC),
]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def sources() -> list[pathlib.Path]:
    return sorted(CSRC.glob("*.cu"))


def _needs_rebuild(obj: pathlib.Path, src: pathlib.Path) -> bool:
    if not obj.exists():
        return True
    deps = [src] + list(CSRC.glob("*.cuh")) + list(INCLUDE.glob("*.h"))
    mt = obj.stat().st_mtime
    return any(d.stat().st_mtime > mt for d in deps)


def build(verbose: bool = False, force: bool = False, extra_flags: list[str] | None = None) -> pathlib.Path:
    """Compile and link the library; returns its path.  Raises on failure."""
    BUILD_DIR.mkdir(exist_ok=True)
    LIB_DIR.mkdir(exist_ok=True)
    flags = NVCC_FLAGS + (extra_flags or [])
    objs = []
    jobs = []
    for src in sources():
        obj = BUILD_DIR / (src.stem + ".o")
        objs.append(obj)
        if force or _needs_rebuild(obj, src):
            jobs.append([nvcc(), *flags, "-c", str(src), "-o", str(obj)])

    def run(cmd):
        r = subprocess.run(cmd, capture_output=True, text=True)
        return cmd, r

    failed = []
    if jobs:
        with cf.ThreadPoolExecutor(max_workers=min(len(jobs), os.cpu_count() or 4)) as ex:
            for cmd, r in ex.map(run, jobs):
                if verbose or r.returncode != 0:
                    print(" ".join(cmd))
                    print(r.stdout, r.stderr)
                if r.returncode != 0:
                    failed.append(cmd[-3])
    if failed:
        raise RuntimeError(f"nvcc failed for: {failed}")
    relink = force or bool(jobs) or not LIB_PATH.exists()
    if relink:
        cmd = [nvcc(), *ARCH, "-shared", "-o", str(LIB_PATH), *map(str, objs)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB_PATH


if __name__ == "__main__":
    import sys
    print(build(verbose="-v" in sys.argv, force="-f" in sys.argv))
