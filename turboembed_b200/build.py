"""Build libturbo_b200.so in-tree with nvcc for sm_100a.

    python -m turboembed_b200.build        # or: python turboembed_b200/build.py

Objects go to turboembed_b200/_build/ and are rebuilt only when a source or
header is newer. The library links the CUDA runtime statically, as the
reference's backend does (core/build.rs:146-186), so the .so needs only the
driver on the machine that loads it.
"""
import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
LIB = PKG / "libturbo_b200.so"
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(ROOT / "include"),
         "--expt-relaxed-constexpr"]
SOURCES = ["backend.cpp", "hooks.cpp", "rowwise.cu", "gemm_simt.cu", "gemm_tc.cu", "attention.cu", "attention_tc.cu",
           "noalloc.cu", "quantize.cu", "gemm_tf32.cu", "devrows.cu", "attention_tf32.cu", "attention_fa.cu"]
HEADERS = [CSRC / "kernels.h", CSRC / "common.cuh", CSRC / "tcgen05.cuh", CSRC / "softmax.cuh", ROOT / "include/turbo_b200.h", ROOT / "include/turbo/turbo_abi.h"]


def _stale(obj: Path, src: Path) -> bool:
    if not obj.exists():
        return True
    t = obj.stat().st_mtime
    return any(p.stat().st_mtime > t for p in [src, *HEADERS])


def _compile(name: str) -> Path:
    src = CSRC / name
    obj = BUILD / (name + ".o")
    if _stale(obj, src):
        cmd = [NVCC, *ARCH, *FLAGS, "-c", str(src), "-o", str(obj)]
        if name.endswith(".cpp"):
            cmd[1:1] = ["-x", "cu"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"nvcc failed on {name}:\n{r.stderr}")
    return obj


def build(verbose: bool = False) -> Path:
    BUILD.mkdir(exist_ok=True)
    with ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 1)) as ex:
        objs = list(ex.map(_compile, SOURCES))
    if not LIB.exists() or any(o.stat().st_mtime > LIB.stat().st_mtime for o in objs):
        cmd = [NVCC, *ARCH, "-shared", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stderr}")
    if verbose:
        print(LIB)
    return LIB


if __name__ == "__main__":
    build(verbose=True)
    sys.exit(0)
