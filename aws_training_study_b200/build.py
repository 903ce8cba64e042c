"""Build the sm_100a extension ``libpcp_attn.so`` in-tree with nvcc.

    python -m aws_training_study_b200.build [--verbose-ptxas]

The library is a plain C-ABI shared object (include/pcp_attn.h) loaded with
ctypes; it links the NCCL that ships with PyTorch (nvidia-nccl wheel) so the
process uses one NCCL build.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_DIR = Path(__file__).resolve().parent
REPO = PKG_DIR.parent
CSRC = PKG_DIR / "csrc"
INCLUDE = REPO / "include"
LIB_NAME = "libpcp_attn.so"
LIB_PATH = PKG_DIR / LIB_NAME
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nccl_dirs() -> tuple[Path, Path]:
    import nvidia.nccl  # the wheel PyTorch links against

    root = Path(list(nvidia.nccl.__path__)[0])
    return root / "include", root / "lib"


def _nvcc() -> str:
    cuda_home = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    cand = Path(cuda_home) / "bin" / "nvcc"
    if cand.exists():
        return str(cand)
    found = shutil.which("nvcc")
    if not found:
        raise RuntimeError("nvcc not found (set CUDA_HOME)")
    return found


def sources() -> list[Path]:
    return sorted(CSRC.glob("*.cu")) + sorted(CSRC.glob("*.cuh")) + [INCLUDE / "pcp_attn.h"]


def needs_build() -> bool:
    if not LIB_PATH.exists():
        return True
    mtime = LIB_PATH.stat().st_mtime
    return any(src.stat().st_mtime > mtime for src in sources())


def build(force: bool = False, verbose_ptxas: bool = False, quiet: bool = False) -> Path:
    if not force and not needs_build():
        return LIB_PATH
    nccl_inc, nccl_lib = _nccl_dirs()
    cmd = [
        _nvcc(),
        *ARCH_FLAGS,
        "-lineinfo",
        "-O3",
        "-std=c++17",
        "--shared",
        "-Xcompiler",
        "-fPIC,-O2,-Wall",
        "-I",
        str(INCLUDE),
        "-I",
        str(nccl_inc),
        str(CSRC / "pcp_attn.cu"),
        "-o",
        str(LIB_PATH) + ".tmp",
        f"-L{nccl_lib}",
        "-l:libnccl.so.2",
        f"-Xlinker=-rpath,{nccl_lib}",
    ]
    if verbose_ptxas:
        cmd.insert(1, "-Xptxas=-v")
    if not quiet:
        print(" ".join(cmd), flush=True)
    subprocess.run(cmd, check=True)
    os.replace(str(LIB_PATH) + ".tmp", LIB_PATH)
    return LIB_PATH


def main(argv: list[str] | None = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose-ptxas", action="store_true")
    args = ap.parse_args(argv)
    build(force=args.force or args.verbose_ptxas, verbose_ptxas=args.verbose_ptxas)
    print(f"built {LIB_PATH}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
