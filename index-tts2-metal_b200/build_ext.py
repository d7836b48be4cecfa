"""Build libitts_cfm.so (the C-ABI library) with nvcc for sm_100a, in-tree.

    python index-tts2-metal_b200/build_ext.py [--force] [--jobs N]

Objects go to index-tts2-metal_b200/_build/, the library to
index-tts2-metal_b200/lib/libitts_cfm.so. A translation unit is rebuilt when
it or any header under csrc/ or include/ is newer than its object.
"""
from __future__ import annotations

import argparse
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "lib" / "libitts_cfm.so"
CLI = PKG / "lib" / "mtts_cfm"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ARCH + ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "-I", str(REPO / "include"),
                "-I", str(CSRC), "--expt-relaxed-constexpr"]


def _sources() -> list[Path]:
    return sorted(list(CSRC.glob("*.cu")) + list(CSRC.glob("*.cpp")))


def _headers_mtime() -> float:
    hs = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + list((REPO / "include").glob("*.h"))
    return max((h.stat().st_mtime for h in hs), default=0.0)


def _compile(src: Path, force: bool, hdr_mtime: float) -> Path:
    obj = BUILD / (src.name + ".o")
    if not force and obj.exists() and obj.stat().st_mtime >= max(src.stat().st_mtime, hdr_mtime):
        return obj
    cmd = [NVCC] + FLAGS + ["-c", str(src), "-o", str(obj)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src.name}:\n{r.stdout}\n{r.stderr}")
    return obj


def build(force: bool = False, jobs: int | None = None) -> Path:
    BUILD.mkdir(parents=True, exist_ok=True)
    LIB.parent.mkdir(parents=True, exist_ok=True)
    srcs = _sources()
    hm = _headers_mtime()
    with ThreadPoolExecutor(max_workers=jobs or min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(lambda s: _compile(s, force, hm), srcs))
    newest = max(o.stat().st_mtime for o in objs)
    if force or not LIB.exists() or LIB.stat().st_mtime < newest:
        cmd = [NVCC] + ARCH + ["-shared", "-o", str(LIB)] + [str(o) for o in objs] + ["-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    # C++ host driver over the C ABI (links the library with an $ORIGIN rpath).
    cli_src = PKG / "cli" / "mtts_cfm.cpp"
    if force or not CLI.exists() or CLI.stat().st_mtime < max(LIB.stat().st_mtime, cli_src.stat().st_mtime,
                                                                (REPO / "include" / "itts_cfm.hpp").stat().st_mtime):
        cmd = [os.environ.get("CXX", "g++"), "-O2", "-std=c++17", "-I", str(REPO / "include"), str(cli_src), "-o",
               str(CLI), "-L", str(LIB.parent), "-litts_cfm", "-Wl,-rpath,$ORIGIN"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"cli build failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    a = ap.parse_args()
    print(build(a.force, a.jobs))
    sys.exit(0)
