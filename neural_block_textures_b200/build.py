"""Builds libntc_b200.so (the CUDA kernels, the host engine, the C ABI and the ntc_cuda::Trainer
class) in-tree with nvcc for sm_100a. Run `python -m neural_block_textures_b200.build`."""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
OUT_DIR = PKG / "_lib"
BUILD_DIR = PKG / "_build"
LIB = OUT_DIR / "libntc_b200.so"
SOURCES = ["kernels_mlp.cu", "kernels_tc.cu", "kernels_latent.cu", "kernels_snap.cu", "kernels_stats.cu", "engine.cu",
           "ntcb_format.cpp", "ntcb_decoder.cu",
           "static_scratch.cu", "nccl_link.cpp", "p2p_exchange.cu", "device_cache.cu"]
GENCODE = ["-gencode", "arch=compute_100a,code=sm_100a"]
# No fast-math: the noise (logf / cosf / sqrtf), the sigmoid (expf) and every division must be CUDA's
# IEEE / accurate versions for parity with the reference backend.
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr", "-Xptxas", "-warn-spills"]


def nvcc() -> str:
    cand = os.environ.get("NVCC") or shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    return cand


def _deps(src: Path) -> list[Path]:
    return [src, *sorted(CSRC.glob("*.cuh")), *sorted(CSRC.glob("*.h")), *sorted((ROOT / "include").glob("*.h"))]


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _compile(src: str, verbose: bool) -> Path:
    s = CSRC / src
    obj = BUILD_DIR / (src + ".o")
    if not _stale(obj, _deps(s)):
        return obj
    cmd = [nvcc(), *GENCODE, *NVCC_FLAGS, "-c", str(s), "-o", str(obj)]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose:
        sys.stderr.write(r.stderr)
    return obj


def build(verbose: bool = False) -> Path:
    OUT_DIR.mkdir(exist_ok=True)
    BUILD_DIR.mkdir(exist_ok=True)
    with cf.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if _stale(LIB, objs):
        cmd = [nvcc(), *GENCODE, "-shared", "-Xcompiler", "-fPIC", "-o", str(LIB), *map(str, objs), "-cudart", "static"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
    return LIB


if __name__ == "__main__":
    print(build(verbose="-v" in sys.argv))
