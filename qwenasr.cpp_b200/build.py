"""Build recipe of the native library (CUDA sm_100a kernels + C++ host runtime).

    python qwenasr.cpp_b200/build.py          # incremental
    python qwenasr.cpp_b200/build.py --clean

Produces qwenasr.cpp_b200/libqwenasr_b200.so in-tree (objects under
qwenasr.cpp_b200/_build/).  nvcc cross-compiles for sm_100a without a GPU.
"""
from __future__ import annotations

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
BUILD = PKG / "_build"
LIB = PKG / "libqwenasr_b200.so"
BIN = PKG / "bin"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "-Xcompiler", "-Wall,-Wextra,-Wshadow",
          f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CSRC / 'adapter'}", "--expt-relaxed-constexpr"]


def sources() -> list[Path]:
    out = sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cpp")) + sorted((CSRC / "adapter").glob("*.cpp"))
    return [p for p in out if p.is_file()]


def headers_mtime() -> float:
    hs = list(CSRC.rglob("*.h")) + list(CSRC.rglob("*.cuh")) + list((ROOT / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def compile_one(src: Path, hdr_time: float, verbose_ptxas: bool) -> Path:
    obj = BUILD / (src.relative_to(CSRC).as_posix().replace("/", "__") + ".o")
    if obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_time):
        return obj
    cmd = [NVCC, *ARCH, *COMMON, "-c", str(src), "-o", str(obj)]
    if verbose_ptxas and src.suffix == ".cu":
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{res.stdout}\n{res.stderr}")
    if verbose_ptxas and res.stderr:
        (BUILD / (obj.name + ".ptxas.txt")).write_text(res.stderr)
    return obj


def build(clean: bool = False, verbose_ptxas: bool = False, jobs: int | None = None) -> Path:
    if clean and BUILD.exists():
        shutil.rmtree(BUILD)
    BUILD.mkdir(parents=True, exist_ok=True)
    hdr = headers_mtime()
    srcs = sources()
    with cf.ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 4)) as ex:
        objs = list(ex.map(lambda s: compile_one(s, hdr, verbose_ptxas), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if LIB.exists() and LIB.stat().st_mtime >= newest and not clean:
        build_tools()   # a tool's own source may have changed
        return LIB
    tmp = LIB.with_suffix(".so.tmp")
    cmd = [NVCC, *ARCH, "-shared", "-o", str(tmp), *map(str, objs), "-lpthread"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"link failed:\n{res.stdout}\n{res.stderr}")
    os.replace(tmp, LIB)
    build_tools()
    return LIB


def build_tools() -> None:
    """CLI harnesses in csrc/tools, linked against the library (rpath $ORIGIN/..)."""
    BIN.mkdir(exist_ok=True)
    for src in sorted((CSRC / "tools").glob("*.cpp")):
        exe = BIN / src.stem
        if exe.exists() and exe.stat().st_mtime >= max(src.stat().st_mtime, LIB.stat().st_mtime):
            continue
        cmd = ["g++", "-O2", "-std=c++17", f"-I{ROOT / 'include'}", f"-I{CSRC}", f"-I{CSRC / 'adapter'}",
               str(src), "-o", str(exe), f"-L{PKG}", "-lqwenasr_b200", "-Wl,-rpath,$ORIGIN/.."]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"tool build failed for {src.name}:\n{res.stdout}\n{res.stderr}")


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--clean", action="store_true")
    ap.add_argument("--ptxas", action="store_true", help="keep -Xptxas -v reports in _build/")
    a = ap.parse_args()
    print(build(clean=a.clean, verbose_ptxas=a.ptxas))
    sys.exit(0)
