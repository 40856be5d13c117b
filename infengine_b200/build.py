"""Build recipe for the in-tree CUDA libraries (sm_100a only).

    python -m infengine_b200.build          # builds what is out of date
    python -m infengine_b200.build --force  # rebuilds everything

Products (git-ignored, shipped with the tree):
  infengine_b200/libinfengine_b200.so   C-ABI of include/infengine_b200.h
  infengine_b200/libinfengine_dropin.so C++ drop-in for the reference's
                                        kernels/*.cuh entry points (links the above)
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OBJ = PKG / "_build"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CFLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-fvisibility=hidden",
    "-I", str(ROOT / "include"), "--expt-relaxed-constexpr",
]

CORE_SOURCES = ["capi.cu", "skinny.cu", "gemm_tc.cu", "noalloc.cu", "comm.cu", "attention.cu", "p2p.cu", "norm.cu",
                "engine.cu", "loader.cu", "attention_tc.cu"]
DROPIN_SOURCES = ["dropin.cu"]

LIB_CORE = PKG / "libinfengine_b200.so"
LIB_DROPIN = PKG / "libinfengine_dropin.so"


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(" ".join(cmd) + "\n" + r.stdout + r.stderr)
        raise RuntimeError(f"build step failed: {cmd[-1]}")
    if r.stderr.strip():
        sys.stderr.write(r.stderr)


def _newer(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return False
    t = target.stat().st_mtime
    return all(d.stat().st_mtime <= t for d in deps)


def _headers() -> list[Path]:
    return sorted(CSRC.glob("*.cuh")) + sorted((ROOT / "include").rglob("*.h*"))


def _compile(src: str, force: bool, extra: list[str] | None = None) -> Path:
    OBJ.mkdir(exist_ok=True)
    s = CSRC / src
    o = OBJ / (Path(src).stem + ".o")
    if force or not _newer(o, [s, *_headers()]):
        _run([NVCC, *CFLAGS, *(extra or []), "-c", str(s), "-o", str(o)])
    return o


def build(force: bool = False, verbose: bool = False) -> list[Path]:
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        core_objs = list(ex.map(lambda s: _compile(s, force), CORE_SOURCES))
        dropin_objs = list(ex.map(lambda s: _compile(s, force), DROPIN_SOURCES))
    if force or not _newer(LIB_CORE, core_objs):
        _run([NVCC, *ARCH, "-shared", "--cudart", "static", "-o", str(LIB_CORE), *map(str, core_objs),
              "-ldl", "-Xlinker", "-Bsymbolic"])
    if force or not _newer(LIB_DROPIN, dropin_objs + [LIB_CORE]):
        _run([NVCC, *ARCH, "-shared", "-o", str(LIB_DROPIN), *map(str, dropin_objs),
              "-L", str(PKG), "-linfengine_b200", "-Xlinker", "-rpath,$ORIGIN", "--cudart", "static", "-ldl",
              "-Xlinker", "-Bsymbolic"])
    if verbose:
        print(f"built {LIB_CORE.name}, {LIB_DROPIN.name}")
    return [LIB_CORE, LIB_DROPIN]


def ptxas_report(src: str = "skinny.cu") -> str:
    """Registers / spills / shared memory per kernel (nvcc -Xptxas -v)."""
    r = subprocess.run([NVCC, *CFLAGS, "-Xptxas", "-v", "-c", str(CSRC / src), "-o", os.devnull],
                       capture_output=True, text=True)
    return r.stderr


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--ptxas", default=None, help="print -Xptxas -v for one source file")
    a = ap.parse_args()
    if a.ptxas:
        print(ptxas_report(a.ptxas))
    else:
        build(force=a.force, verbose=True)
