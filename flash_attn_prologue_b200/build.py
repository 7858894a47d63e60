"""Builds libflash_prologue.so (the C-ABI library) in-tree with nvcc for sm_100a.

Usage: python -m flash_attn_prologue_b200.build [--force] [-j JOBS]

Each csrc/*.cu compiles to an object under _build/ (in parallel), then the
objects link into flash_attn_prologue_b200/libflash_prologue.so. A source is
recompiled when it or any csrc header / include/*.h is newer than its object.
"""
import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
INCLUDE = ROOT / "include"
BUILD = ROOT / "_build"
LIB = PKG / "libflash_prologue.so"

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3,-fvisibility=hidden",
              "--expt-relaxed-constexpr", "-Xptxas", "-v,-warn-spills"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: set NVCC or put the CUDA toolkit on PATH")


def _deps_mtime() -> float:
    files = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + list(INCLUDE.glob("*.h"))
    return max((f.stat().st_mtime for f in files), default=0.0)


def _compile(src: Path, obj: Path, extra, log_dir: Path):
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, *extra, "-I", str(INCLUDE), "-c", str(src), "-o", str(obj)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    (log_dir / (src.stem + ".ptxas.txt")).write_text(res.stdout + res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr[-4000:]}")
    return obj


def build(force: bool = False, jobs: int = 0) -> Path:
    BUILD.mkdir(exist_ok=True)
    extra = []
    deps = _deps_mtime()
    srcs = sorted(CSRC.glob("*.cu"))
    todo = []
    objs = []
    for src in srcs:
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, deps):
            todo.append((src, obj))
    if todo:
        workers = jobs or min(len(todo), os.cpu_count() or 4)
        with cf.ThreadPoolExecutor(max_workers=workers) as ex:
            list(ex.map(lambda so: _compile(so[0], so[1], extra, BUILD), todo))
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        tmp = LIB.with_suffix(".so.tmp")
        cmd = [nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", *map(str, objs), "-o", str(tmp)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"link failed:\n{res.stderr[-4000:]}")
        os.replace(tmp, LIB)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("-j", "--jobs", type=int, default=0)
    args = ap.parse_args(argv)
    lib = build(force=args.force, jobs=args.jobs)
    print(lib)


if __name__ == "__main__":
    sys.exit(main())
