"""Builds oracle/_ref/libcugo_ref.so from the reference's sources (TEST
INFRASTRUCTURE ONLY): `make -C oracle REF=<reference>`.  Needs the reference tree
(present in the build container, absent on GPU boxes, which use the prebuilt file)."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent
DEFAULT_REF = Path(os.environ.get("CUGO_REFERENCE", "/root/reference"))


def reference_present(ref: Path = DEFAULT_REF) -> bool:
    return (ref / "include" / "cugo" / "game" / "torch50.h").is_file()


def build(ref: Path = DEFAULT_REF) -> Path:
    lib = HERE / "_ref" / "libcugo_ref.so"
    if not reference_present(ref):
        if lib.is_file():
            return lib
        raise RuntimeError(f"reference sources not found at {ref} and no prebuilt {lib}")
    subprocess.run(["make", "-s", "-C", str(HERE), f"REF={ref}"], check=True)
    return lib
