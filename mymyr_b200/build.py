"""Builds the device library in-tree: mymyr_b200/lib/libmymyr_b200.so (C ABI of include/mymyr_b200.h).

CUDA sources are compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``); the host task
compiler by g++. The library links the CUDA runtime statically, so it loads with nothing but the driver.

    python -m mymyr_b200.build            # or __graft_entry__.build()
"""

from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

ROOT = Path(__file__).resolve().parent
REPO = ROOT.parent
CSRC = ROOT / "csrc"
LIB_DIR = ROOT / "lib"
LIB = LIB_DIR / "libmymyr_b200.so"
OBJ_DIR = REPO / "_build" / "mymyr_b200"

CU_SOURCES = ["api.cu", "expand.cu", "brfs.cu", "dbrfs.cu", "comm.cu", "astar.cu", "env.cu", "jit.cu"]
CPP_SOURCES = ["compile.cpp", "codegen.cpp", "relax.cpp"]
# device sources compiled at run time (NVRTC), embedded into the library as strings
EMBEDDED = {"b2_jit_core_source": "core.cuh", "b2_jit_kernels_source": "jit_kernels.cuh"}
CUDA_LIB = "/usr/local/cuda/lib64"
# NVRTC is loaded with dlopen at the first compile (jit.cu); the library links only the static CUDA runtime

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def _run(cmd: list[str]) -> None:
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"command failed ({r.returncode}): {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")


def _stale(out: Path, deps: list[Path]) -> bool:
    if not out.exists():
        return True
    t = out.stat().st_mtime
    return any(d.stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> Path:
    OBJ_DIR.mkdir(parents=True, exist_ok=True)
    LIB_DIR.mkdir(parents=True, exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.hpp")) + [REPO / "include" / "mymyr_b200.h"]
    inc = ["-I", str(REPO / "include"), "-I", str(CSRC)]
    jobs = []
    objs = []
    for src in CU_SOURCES:
        s = CSRC / src
        o = OBJ_DIR / (src + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++20", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
                   *inc, "-c", str(s), "-o", str(o)]
            if ptxas_verbose:
                cmd.insert(1, "-Xptxas=-v")
            jobs.append(cmd)
    for src in CPP_SOURCES:
        s = CSRC / src
        o = OBJ_DIR / (src + ".o")
        objs.append(o)
        if _stale(o, [s] + headers):
            jobs.append(["g++", "-std=c++20", "-O2", "-fPIC", "-Wall", *inc, "-c", str(s), "-o", str(o)])
    emb_src = OBJ_DIR / "jit_sources.cpp"
    emb_obj = OBJ_DIR / "jit_sources.cpp.o"
    objs.append(emb_obj)
    if _stale(emb_obj, [CSRC / f for f in EMBEDDED.values()]):
        parts = []
        for sym, f in EMBEDDED.items():
            text = (CSRC / f).read_text()
            assert ")B2SRC" not in text
            parts.append(f'extern "C" const char {sym}[] = R"B2SRC({text})B2SRC";\n')
        emb_src.write_text("".join(parts))
        jobs.append(["g++", "-std=c++20", "-O1", "-fPIC", "-c", str(emb_src), "-o", str(emb_obj)])
    with cf.ThreadPoolExecutor(max_workers=max(1, min(8, os.cpu_count() or 1))) as ex:
        list(ex.map(_run, jobs))
    if jobs or not LIB.exists():
        tmp = LIB.with_suffix(".so.tmp")
        _run([nvcc(), *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs), "-ldl"])
        tmp.replace(LIB)
    if verbose:
        print(f"built {LIB}")
    return LIB


if __name__ == "__main__":
    build(verbose=True, ptxas_verbose="-v" in sys.argv)
