"""Ahead-of-time build of the sm_100a library and its PyTorch binding, in-tree.

Replaces the reference's JIT loader (src/mini_flash_attention/_cuda.py:11-37, which set
TORCH_CUDA_ARCH_LIST to the detected GPU and compiled at first call). Here:

1. ``libmfa_b200.so``: the CUDA kernels and the C ABI (include/mfa_b200.h), compiled by nvcc
   for ``-gencode arch=compute_100a,code=sm_100a`` only. It depends on no torch library.
2. ``mfa_b200_C*.so``: the pybind11/ATen binding (csrc/mfa_binding.cpp), compiled with
   torch.utils.cpp_extension as host-only C++ and linked against (1).

Both land in the package directory so that they travel with the source tree. Cross-compiles
without a GPU. Usage: ``python -m mini_flash_attention._build [--force] [--verbose]``.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_ROOT = PKG_DIR.parent                      # mini-flash-attention_b200/
CSRC = SRC_ROOT / "csrc"
REPO_ROOT = SRC_ROOT.parent
INCLUDE = REPO_ROOT / "include"
BUILD_DIR = SRC_ROOT / "_build"
LIB_NAME = "libmfa_b200.so"
EXT_NAME = "mfa_b200_C"

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH_FLAGS + ["-O3", "-lineinfo", "-std=c++17", "-Xptxas", "-v"]

LIB_SOURCES = [CSRC / "mfa_capi.cu"]
LIB_DEPS = LIB_SOURCES + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "mfa_b200.h"]
BINDING_SOURCES = [CSRC / "mfa_binding.cpp"]


def _nvcc() -> str:
    found = shutil.which("nvcc")
    if found:
        return found
    cand = Path(os.environ.get("CUDA_HOME", "/usr/local/cuda")) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    raise RuntimeError("nvcc not found (set CUDA_HOME or PATH)")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build_library(force: bool = False, verbose: bool = False) -> Path:
    """Compile the kernels + C ABI into ``libmfa_b200.so`` (sm_100a)."""
    out = PKG_DIR / LIB_NAME
    if not force and not _stale(out, LIB_DEPS):
        return out
    BUILD_DIR.mkdir(parents=True, exist_ok=True)
    tmp = BUILD_DIR / (LIB_NAME + ".tmp")
    cmd = [_nvcc(), *NVCC_FLAGS, "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", f"-I{INCLUDE}",
           "-Xlinker", f"-soname={LIB_NAME}",
           *[str(s) for s in LIB_SOURCES], "-o", str(tmp)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if verbose or res.returncode != 0:
        sys.stdout.write(res.stdout)
        sys.stderr.write(res.stderr)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}): {' '.join(cmd)}")
    (BUILD_DIR / "ptxas_lib.txt").write_text(res.stderr)
    os.replace(tmp, out)
    return out


def preload_library() -> ctypes.CDLL:
    """Load ``libmfa_b200.so`` globally so the binding's DT_NEEDED entry resolves to it."""
    return ctypes.CDLL(str(PKG_DIR / LIB_NAME), mode=ctypes.RTLD_GLOBAL)


def _existing_binding() -> Path | None:
    hits = sorted(PKG_DIR.glob(f"{EXT_NAME}*.so"))
    return hits[0] if hits else None


def build_binding(force: bool = False, verbose: bool = False) -> Path:
    """Compile the pybind11/ATen binding against libmfa_b200.so."""
    lib = PKG_DIR / LIB_NAME
    existing = _existing_binding()
    if (not force and existing is not None
            and not _stale(existing, BINDING_SOURCES + [INCLUDE / "mfa_b200.h", lib])):
        return existing
    from torch.utils import cpp_extension  # heavy import, only when actually building

    preload_library()
    bdir = BUILD_DIR / "binding"
    bdir.mkdir(parents=True, exist_ok=True)
    cpp_extension.load(
        name=EXT_NAME,
        sources=[str(s) for s in BINDING_SOURCES],
        extra_include_paths=[str(INCLUDE)],
        extra_cflags=["-O3", "-std=c++17"],
        extra_ldflags=[f"-L{PKG_DIR}", f"-l:{LIB_NAME}"],
        build_directory=str(bdir),
        with_cuda=True,
        verbose=verbose,
        is_python_module=True,
    )
    built = bdir / f"{EXT_NAME}.so"
    if not built.exists():
        raise RuntimeError(f"binding build produced no {built}")
    for old in PKG_DIR.glob(f"{EXT_NAME}*.so"):
        old.unlink()
    dst = PKG_DIR / f"{EXT_NAME}.so"
    shutil.copy2(built, dst)
    return dst


def build(force: bool = False, verbose: bool = False) -> None:
    build_library(force=force, verbose=verbose)
    build_binding(force=force, verbose=verbose)


def main() -> None:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args()
    build(force=args.force, verbose=args.verbose)
    print(f"built {PKG_DIR / LIB_NAME} and {_existing_binding()}")


if __name__ == "__main__":
    main()
