"""Build recipe for the package's native libraries (run by __graft_entry__.build()).

  libg4b200.so  -- CUDA kernels + the C ABI of include/g4.h, sm_100a only
  libg4synth.so -- host quantizers used to make synthetic GGUF block streams

Objects go to gemma4.kt_b200/_build/, the shared libraries next to this file
(in-tree, so they travel with the repository snapshot to a GPU host).
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT = PKG / "_build"
INCLUDE = ROOT / "include"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = shutil.which("nvcc") or os.path.join(CUDA_HOME, "bin", "nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "--expt-relaxed-constexpr",
    "-Xcompiler", "-fPIC,-O3", "-I", str(INCLUDE), "-I", str(CSRC),
]

CU_SOURCES = ["g4_capi.cu", "g4_gemv.cu", "g4_moe.cu", "g4_moe_tc.cu", "g4_decode.cu", "g4_gemv_dec.cu", "g4_gemv_mma.cu", "g4_block.cu"]
CU_HEADERS = ["g4_common.cuh", "g4_gemv.cuh", "g4_gemv_rows.cuh", "g4_internal.h", "g4_ctx.h", "g4_moe_tc.h", "g4_fuse.cuh"]


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        sys.stderr.write(r.stdout + r.stderr)
        raise RuntimeError("build step failed: " + " ".join(cmd))


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.exists() and d.stat().st_mtime > t for d in deps)


def build_cuda(verbose: bool = False) -> Path:
    OUT.mkdir(exist_ok=True)
    headers = [CSRC / h for h in CU_HEADERS] + [INCLUDE / "g4.h"]
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        if not s.exists():
            continue
        o = OUT / (src + ".o")
        if _stale(o, [s] + headers + [Path(__file__)]):
            cmd = [NVCC, *NVCC_FLAGS, "-c", str(s), "-o", str(o)]
            if verbose:
                cmd.insert(1, "-Xptxas=-v")
            _run(cmd)
        objs.append(o)
    lib = PKG / "libg4b200.so"
    if _stale(lib, objs):
        _run([NVCC, *ARCH, "-shared", "-o", str(lib), *map(str, objs), "-ldl", "-lcudart"])
    return lib


def build_synth() -> Path:
    src = CSRC / "g4_synth.c"
    lib = PKG / "libg4synth.so"
    if _stale(lib, [src]):
        _run(["gcc", "-O3", "-fPIC", "-shared", "-std=c11", "-o", str(lib), str(src), "-lm", "-lpthread"])
    return lib


def build_all(verbose: bool = False) -> None:
    build_cuda(verbose)
    build_synth()


if __name__ == "__main__":
    build_all(verbose="-v" in sys.argv)
    print("built", PKG / "libg4b200.so", PKG / "libg4synth.so")
