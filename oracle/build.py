"""Builds oracle/_ref/libcugo_ref.so from the reference's sources (TEST
INFRASTRUCTURE ONLY): `make -C oracle REF=<reference>`.  Needs the reference tree
(present in the build container, absent on GPU boxes, which use the prebuilt file).

The reference tree is found through CUGO_REFERENCE, else as a directory named
`reference` beside this repository's root."""
from __future__ import annotations

import os
import subprocess
from pathlib import Path

HERE = Path(__file__).resolve().parent


def reference_root() -> Path:
    """The reference checkout: $CUGO_REFERENCE, else <repository root>/../reference."""
    env = os.environ.get("CUGO_REFERENCE")
    return Path(env) if env else HERE.parent.parent / "reference"


DEFAULT_REF = reference_root()


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
