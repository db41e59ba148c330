"""In-tree build of libslmopt.so (the CUDA kernels and the C ABI) for sm_100a.

The shared library lands next to this file so it travels with the source
tree; nothing is installed into site-packages.  nvcc cross-compiles without a
GPU.  Flags that matter for exactness:

* ``--fmad=false`` and explicit ``__f*_rn`` intrinsics: no FMA contraction in
  the AdamW recurrence;
* ``-prec-div=true -prec-sqrt=true -ftz=false``: IEEE division, square root and
  subnormals, as the reference's Rust f32 arithmetic;
* ``-Xcompiler -ffp-contract=off``: the host-side scalar work (powi, the lr
  schedule) rounds once per operation as well.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
SRC_ROOT = PKG_DIR.parent
CSRC = SRC_ROOT / "csrc"
REPO_ROOT = SRC_ROOT.parent
INCLUDE = REPO_ROOT / "include"
LIB_NAME = "libslmopt.so"
LIB_PATH = PKG_DIR / LIB_NAME

SOURCES = ["kernels.cu", "api.cu", "zero1.cu", "noalloc.cu", "sha256.cpp", "hostcopy.cpp"]
HEADERS = ["slmopt_internal.h", "handle.h", "sha256.h", "hostcopy.h"]

ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = [
    "-O3",
    "-lineinfo",
    "-std=c++17",
    "--fmad=false",
    "-prec-div=true",
    "-prec-sqrt=true",
    "-ftz=false",
    "-Xcompiler",
    "-fPIC,-O2,-ffp-contract=off",
    "-shared",
]


def nvcc_path() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found: the CUDA toolkit is required to build libslmopt.so")


def nccl_paths() -> tuple[Path, Path]:
    """(include dir, lib dir) of the NCCL that torch ships (the one a torch
    process has loaded), else the system NCCL."""
    try:
        import nvidia.nccl  # namespace package from the nvidia-nccl wheel

        root = Path(list(nvidia.nccl.__path__)[0])
        if (root / "include" / "nccl.h").exists() and (root / "lib" / "libnccl.so.2").exists():
            return root / "include", root / "lib"
    except Exception:
        pass
    return Path("/usr/include"), Path("/usr/lib/x86_64-linux-gnu")


def _inputs() -> list[Path]:
    return [CSRC / s for s in SOURCES] + [CSRC / h for h in HEADERS] + [INCLUDE / "slmopt.h"]


def is_stale() -> bool:
    if not LIB_PATH.exists():
        return True
    built = LIB_PATH.stat().st_mtime
    return any(p.stat().st_mtime > built for p in _inputs())


def build(force: bool = False, verbose: bool = False, extra_flags: list[str] | None = None) -> Path:
    """Compile libslmopt.so if any source is newer than it (or ``force``)."""
    if not force and not is_stale():
        return LIB_PATH
    out_tmp = LIB_PATH.with_suffix(".so.tmp")
    nccl_inc, nccl_lib = nccl_paths()
    cmd = (
        [nvcc_path()]
        + ARCH_FLAGS
        + NVCC_FLAGS
        + (extra_flags or [])
        + ["-I", str(INCLUDE), "-I", str(nccl_inc), "-o", str(out_tmp)]
        + [str(CSRC / s) for s in SOURCES]
        + ["-L", str(nccl_lib), "-l:libnccl.so.2", "-Xlinker", f"-rpath={nccl_lib}"]
    )
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode != 0:
        raise RuntimeError(f"nvcc failed ({res.returncode}):\n{res.stdout}\n{res.stderr}")
    if verbose and (res.stdout or res.stderr):
        print(res.stdout + res.stderr, file=sys.stderr)
    out_tmp.replace(LIB_PATH)
    return LIB_PATH


if __name__ == "__main__":
    force = "--force" in sys.argv
    extra = ["-Xptxas", "-v"] if "--ptxas-v" in sys.argv else None
    print(build(force=force or extra is not None, verbose=True, extra_flags=extra))
