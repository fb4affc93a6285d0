"""Recipe: compile the reference's own CUDA kernels into oracle/_ref/libmfa_ref.so.

Test infrastructure only. Compiles, unmodified and in place, the reference sources
  src/mini_flash_attention/flash_attn_cuda.cu       (CuTe / SM80 mma.sync kernel)
  src/mini_flash_attention/flash_attn_wmma_cuda.cu  (WMMA kernel)
with the flags of the reference loader (src/mini_flash_attention/_cuda.py:32-33:
-O3 --use_fast_math) for sm_100a, plus oracle/ref_shim.cu (a C-ABI wrapper of our own).

The reference's CUTLASS submodule (third_party/cutlass) is not vendored and its pinned commit
is unknown; the CuTe headers used instead are the CUTLASS 4.x tree shipped inside the
flashinfer wheel of this image (only stable CuTe APIs are used by the kernel,
flash_attn_cuda.cu:5-12). The WMMA unit defines its launcher under the CuTe launcher's name
(flash_attn_wmma_cuda.cu:253), so it is renamed with a -D define at compile time.

The reference checkout is taken from --reference-root, else $MFA_REFERENCE_ROOT, else a
directory named `reference` beside this repository; without one nothing is built. The built
library travels with the tree, the sources are never copied into it.
Usage: python oracle/build_ref.py [--force] [--reference-root DIR]
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT_DIR = HERE / "_ref"
OUT_LIB = OUT_DIR / "libmfa_ref.so"


def reference_sources(root: str | os.PathLike | None = None) -> Path:
    """src/mini_flash_attention of the reference checkout (see the module docstring)."""
    if root is None:
        root = os.environ.get("MFA_REFERENCE_ROOT") or HERE.parent.parent / "reference"
    return Path(root) / "src" / "mini_flash_attention"


def cutlass_include() -> Path:
    env = os.environ.get("MFA_CUTLASS_INCLUDE")
    cands = [Path(env)] if env else []
    try:
        import flashinfer  # noqa: F401  (only to locate its data directory)
        cands.append(Path(flashinfer.__file__).resolve().parent / "data" / "cutlass" / "include")
    except Exception:  # noqa: BLE001
        pass
    site = Path(sys.prefix) / "lib" / f"python{sys.version_info.major}.{sys.version_info.minor}"
    cands.append(site / "site-packages" / "flashinfer" / "data" / "cutlass" / "include")
    for c in cands:
        if (c / "cute" / "tensor.hpp").exists():
            return c
    raise RuntimeError("no CuTe headers found (set MFA_CUTLASS_INCLUDE)")


def available(root: str | os.PathLike | None = None) -> bool:
    return (reference_sources(root) / "flash_attn_cuda.cu").exists()


def build(force: bool = False, reference_root: str | os.PathLike | None = None) -> Path | None:
    if not available(reference_root):
        return None
    ref_src = reference_sources(reference_root)
    srcs = [ref_src / "flash_attn_cuda.cu", ref_src / "flash_attn_wmma_cuda.cu",
            ref_src / "utils.cuh", HERE / "ref_shim.cu", Path(__file__)]
    if (not force and OUT_LIB.exists()
            and all(s.stat().st_mtime <= OUT_LIB.stat().st_mtime for s in srcs)):
        return OUT_LIB
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    OUT_DIR.mkdir(exist_ok=True)
    inc = cutlass_include()
    common = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O3", "--use_fast_math",
              "-std=c++17", "-Xcompiler", "-fPIC", f"-I{inc}", f"-I{ref_src}"]
    objs = []
    units = [
        (ref_src / "flash_attn_cuda.cu", []),
        (ref_src / "flash_attn_wmma_cuda.cu",
         ["-Dlaunch_flash_attn_forward=launch_flash_attn_forward_wmma"]),
        (HERE / "ref_shim.cu", []),
    ]
    for src, extra in units:
        obj = OUT_DIR / (src.stem + ".o")
        cmd = common + extra + ["-c", str(src), "-o", str(obj)]
        res = subprocess.run(cmd, capture_output=True, text=True)
        if res.returncode != 0:
            raise RuntimeError(f"reference build failed: {' '.join(cmd)}\n{res.stderr}")
        objs.append(str(obj))
    cmd = [nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", *objs,
           "-o", str(OUT_LIB)]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"reference link failed:\n{res.stderr}")
    for o in objs:
        Path(o).unlink()
    return OUT_LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--reference-root", default=None)
    a = ap.parse_args()
    print(build(force=a.force, reference_root=a.reference_root)
          or "reference sources not present; nothing built")
