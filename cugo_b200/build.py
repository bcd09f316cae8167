"""Builds the native library in-tree: cugo_b200/lib/libcugo_b200.so (sm_100a only).

    python -m cugo_b200.build [--force]

The library is torch-free: CUDA sources under cugo_b200/csrc/ compiled by nvcc with
the CUDA runtime linked statically, exporting the C ABI of include/cugo_b200.h.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB_DIR = PKG / "lib"
LIB = LIB_DIR / "libcugo_b200.so"

SOURCES = ["env_kernels.cu", "drivers.cu", "policy_kernels.cu", "mlp_kernels.cu", "seq_kernels.cu",
           "rollout_kernels.cu", "update_kernels.cu"]
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--cudart", "static",
              "-Xcompiler", "-fvisibility=hidden"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the cugo_b200 native library needs the CUDA toolkit")


def _inputs() -> list[Path]:
    files = [CSRC / s for s in SOURCES]
    files += sorted(CSRC.rglob("*.cuh")) + [ROOT / "include" / "cugo_b200.h", Path(__file__)]
    return [f for f in files if f.exists()]


def up_to_date() -> bool:
    if not LIB.exists():
        return False
    newest = max(f.stat().st_mtime for f in _inputs())
    return LIB.stat().st_mtime >= newest


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and up_to_date():
        return LIB
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    objs = []
    tmp = LIB_DIR / "obj"
    tmp.mkdir(exist_ok=True)
    for src in SOURCES:
        obj = tmp / (Path(src).stem + ".o")
        cmd = [nvcc(), *ARCH_FLAGS, *NVCC_FLAGS, "-c", str(CSRC / src), "-o", str(obj)]
        if verbose:
            cmd.insert(1, "-Xptxas=-v")
            print(" ".join(cmd), file=sys.stderr)
        subprocess.run(cmd, check=True)
        objs.append(str(obj))
    out = LIB.with_suffix(".so.tmp")
    cmd = [nvcc(), *ARCH_FLAGS, "--cudart", "static", "-shared", *objs, "-o", str(out)]
    subprocess.run(cmd, check=True)
    out.replace(LIB)
    return LIB


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    print(build(force=args.force, verbose=args.verbose))


if __name__ == "__main__":
    main()
