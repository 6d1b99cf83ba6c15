"""Builds libjishui_b200.so (all sm_100a kernels + the C ABI) in-tree with nvcc.

Each ``csrc/*.cu`` file is compiled to an object under ``_build/`` (in parallel,
skipped when up to date) and linked into ``midstream_llm_b200/libjishui_b200.so``.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = ROOT / "_build"
LIB = PKG / "libjishui_b200.so"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libjishui_b200.so")


def _flags(debug: bool) -> list[str]:
    f = ARCH + ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC", "-I", str(ROOT / "include"),
                "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]
    if debug:
        f += ["-DJX_DEBUG"]
    return f


def _sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu"))


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted(CSRC.glob("*.h")) + sorted((ROOT / "include").glob("*.h"))


def _compile(src: Path, obj: Path, flags: list[str], verbose: bool) -> tuple[Path, str]:
    cmd = [_nvcc(), *flags, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return src, r.stdout + r.stderr


def build(force: bool = False, debug: bool = False, verbose: bool = False, jobs: int | None = None) -> Path:
    """Compiles the kernels if any source changed; returns the path of the shared library."""
    BUILD.mkdir(exist_ok=True)
    flags = _flags(debug)
    newest_header = max((h.stat().st_mtime for h in _headers()), default=0.0)
    todo = []
    objs = []
    for src in _sources():
        obj = BUILD / (src.stem + ".o")
        objs.append(obj)
        if force or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append((src, obj))
    if todo:
        with cf.ThreadPoolExecutor(max_workers=jobs or min(8, len(todo))) as ex:
            for src, log in ex.map(lambda t: _compile(t[0], t[1], flags, verbose), todo):
                if verbose and log.strip():
                    print(f"== {src.name}\n{log}", file=sys.stderr)
    if todo or not LIB.exists() or LIB.stat().st_mtime < max(o.stat().st_mtime for o in objs):
        cmd = [_nvcc(), *ARCH, "-shared", "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objs), "-lcudart"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    import argparse

    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("-v", "--verbose", action="store_true", help="print ptxas register/spill reports")
    a = ap.parse_args()
    print(build(force=a.force, debug=a.debug, verbose=a.verbose))
