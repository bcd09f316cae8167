"""Stages the reference's own Python modules and builds the reference's own CUDA
extension into baseline/_ref/ (git-ignored; it travels to the GPU box with the
snapshot, as oracle/_ref does).  TEST AND BENCHMARK INFRASTRUCTURE ONLY: the
product never imports anything from here.

    python -m baseline.build_ref            # stage + build (needs the reference tree)

  baseline/_ref/python/*.py        the reference's python/ modules, copied unmodified
                                   (cugo_ppo50, cugo_eval50, cugo_seq_selfplay50, ...)
  baseline/_ref/torch50_ext/       the reference extension (python/csrc/torch50_ext.cpp
                                   and .cu, include/ headers) built by
                                   torch.utils.cpp_extension with the flags of the
                                   reference loader (python/cugo_torch50_ext.py:141-193:
                                   -O3 -std=c++20 for host and device code) for sm_100,
                                   the architecture that loader selects on a B200
                                   (TORCH_CUDA_ARCH_LIST = the device capability, 10.0)

On the GPU box (no reference tree) `reference_python()` and `load_reference_extension()`
use the staged files.  The reference tree is found through CUGO_REFERENCE, else as a
directory named `reference` beside this repository's root.
"""
from __future__ import annotations

import importlib.machinery
import importlib.util
import os
import shutil
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
REF_OUT = HERE / "_ref"
PY_OUT = REF_OUT / "python"
EXT_DIR = REF_OUT / "torch50_ext"
EXT_NAME = "cugo_torch50_ext_v6"  # the reference loader's module name


def reference_root() -> Path:
    env = os.environ.get("CUGO_REFERENCE")
    return Path(env) if env else HERE.parent.parent / "reference"


def reference_present(ref: Path | None = None) -> bool:
    ref = ref or reference_root()
    return (ref / "python" / "csrc" / "torch50_ext.cu").is_file()


def stage(ref: Path | None = None) -> Path:
    """Copies the reference's python/*.py (unmodified) into baseline/_ref/python."""
    ref = ref or reference_root()
    PY_OUT.mkdir(parents=True, exist_ok=True)
    for src in sorted((ref / "python").glob("*.py")):
        shutil.copy2(src, PY_OUT / src.name)
    return PY_OUT


def extension_path() -> Path:
    return EXT_DIR / f"{EXT_NAME}.so"


def build_extension(ref: Path | None = None, verbose: bool = False) -> Path:
    """The reference extension for sm_100 with its loader's flags (no intermediates kept)."""
    ref = ref or reference_root()
    from torch.utils import cpp_extension

    EXT_DIR.mkdir(parents=True, exist_ok=True)
    os.environ["TORCH_CUDA_ARCH_LIST"] = "10.0"
    os.environ.setdefault("MAX_JOBS", "4")
    csrc = ref / "python" / "csrc"
    cpp_extension.load(
        name=EXT_NAME,
        sources=[str(csrc / "torch50_ext.cpp"), str(csrc / "torch50_ext.cu")],
        extra_include_paths=[str(ref / "include")],
        extra_cflags=["-O3", "-std=c++20"],
        extra_cuda_cflags=["-O3", "-std=c++20"],
        build_directory=str(EXT_DIR),
        with_cuda=True,
        verbose=verbose,
        is_python_module=True,
    )
    # Only the module is kept: object files and ninja state stay out of the snapshot.
    for f in EXT_DIR.iterdir():
        if f.name != extension_path().name:
            if f.is_dir():
                shutil.rmtree(f)
            else:
                f.unlink()
    return extension_path()


def reference_python() -> Path:
    """Directory of the staged reference modules (put it on sys.path to import them)."""
    if not (PY_OUT / "cugo_ppo50.py").is_file():
        raise RuntimeError(f"reference modules not staged in {PY_OUT} (python -m baseline.build_ref)")
    return PY_OUT


def load_reference_extension():
    """The reference's extension module built by build_extension()."""
    path = extension_path()
    if not path.is_file():
        raise RuntimeError(f"reference extension not built: {path} (python -m baseline.build_ref)")
    import torch  # noqa: F401  (the module links against torch's libraries)

    if EXT_NAME in sys.modules:
        return sys.modules[EXT_NAME]
    loader = importlib.machinery.ExtensionFileLoader(EXT_NAME, str(path))
    spec = importlib.util.spec_from_file_location(EXT_NAME, str(path), loader=loader)
    mod = importlib.util.module_from_spec(spec)
    loader.exec_module(mod)
    sys.modules[EXT_NAME] = mod
    return mod


def available() -> bool:
    return extension_path().is_file() and (PY_OUT / "cugo_ppo50.py").is_file()


def build(verbose: bool = False) -> None:
    if not reference_present():
        if available():
            return
        raise RuntimeError(f"reference tree not found at {reference_root()} and nothing staged")
    stage()
    if not extension_path().is_file():
        build_extension(verbose=verbose)


if __name__ == "__main__":
    build(verbose="--verbose" in sys.argv)
    print(PY_OUT)
    print(extension_path())
