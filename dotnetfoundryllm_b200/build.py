"""Build recipe for the native libraries (in-tree, so the .so files travel with
the source tree to the GPU host).

- ``_lib/libfoundry_cuda.so``: the sm_100a kernels and the C ABI of
  ``include/foundry_cuda.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``).
- ``_lib/libfoundry_gen.so``: the seeded synthetic-GGUF payload generator
  (host C + OpenMP).

``python -m dotnetfoundryllm_b200.build`` builds both; ``build(force=True)``
rebuilds unconditionally.
"""
from __future__ import annotations

import os
import shutil
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

PKG = Path(__file__).resolve().parent
ROOT = PKG.parent
CSRC = PKG / "csrc"
LIB = PKG / "_lib"
OBJ = PKG / "_build"

CUDA_SOURCES = ["fl_matvec.cu", "fl_misc.cu", "fl_token.cu", "fl_token_hd64.cu", "fl_token_hd128.cu",
                "fl_token_hd256.cu", "fl_prefill.cu", "fl_sample.cu", "fl_tc_gemm.cu", "fl_runtime.cu"]
HOST_SOURCES = ["fl_repack.cpp"]
HEADERS = ["fl_layout.h", "fl_decode.h", "fl_device.cuh", "fl_kernels.h", "fl_repack.h", "fl_mv_core.cuh", "fl_dequant.cuh",
           "fl_token.cuh"]

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _gcc() -> str:
    for cand in ("/usr/bin/gcc", shutil.which("gcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("gcc not found")


def _gxx() -> str:
    for cand in ("/usr/bin/g++", shutil.which("g++")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("g++ not found")


def _stale(target: Path, deps: list[Path]) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build step failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def build_cuda(force: bool = False, verbose_ptxas: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    OBJ.mkdir(exist_ok=True)
    out = LIB / "libfoundry_cuda.so"
    hdrs = [CSRC / h for h in HEADERS] + [ROOT / "include" / "foundry_cuda.h"]
    nvcc = _nvcc()
    jobs = []
    objs = []
    for src in CUDA_SOURCES:
        o = OBJ / (src + ".o")
        objs.append(o)
        if force or _stale(o, [CSRC / src] + hdrs):
            cmd = [nvcc, *ARCH, "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-c",
                   "-I", str(CSRC), "-I", str(ROOT / "include"), str(CSRC / src), "-o", str(o)]
            if verbose_ptxas:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    for src in HOST_SOURCES:
        o = OBJ / (src + ".o")
        objs.append(o)
        if force or _stale(o, [CSRC / src] + hdrs):
            jobs.append([_gxx(), "-O2", "-std=c++17", "-fPIC", "-ffp-contract=off", "-c", "-I", str(CSRC),
                         str(CSRC / src), "-o", str(o)])
    with ThreadPoolExecutor(max_workers=max(1, min(len(jobs), os.cpu_count() or 4))) as ex:
        list(ex.map(_run, jobs))
    if force or jobs or _stale(out, objs):
        _run([nvcc, *ARCH, "-shared", "-o", str(out), *map(str, objs), "-lcudart", "-lpthread"])
    return out


def build_gen(force: bool = False) -> Path:
    LIB.mkdir(exist_ok=True)
    out = LIB / "libfoundry_gen.so"
    src = CSRC / "ggufgen.c"
    if force or _stale(out, [src]):
        _run([_gcc(), "-O2", "-std=gnu11", "-fPIC", "-shared", "-fopenmp", "-ffp-contract=off",
              str(src), "-o", str(out), "-lm"])
    return out


def build(force: bool = False) -> None:
    build_gen(force)
    build_cuda(force)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
    print("built", *(p.name for p in LIB.glob("*.so")))
