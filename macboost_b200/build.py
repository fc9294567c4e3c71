"""Build libmacboostc.so in-tree: sm_100a CUDA kernels + C++ host engine + C ABI.

    python -m macboost_b200.build [--force]

The library links the CUDA runtime statically and exports only the
``macboost_*`` symbols of include/macboost_c.h (a linker version script), so
it loads next to any other CUDA runtime in the same process.  No PyTorch.
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
BUILD = PKG / "_build"
LIB = PKG / "libmacboostc.so"
CLI = PKG / "macboost"          # the `macboost` command (C++ over the C ABI)

CXX_SOURCES = ["model.cpp", "forest.cpp", "forest_codes.cpp", "shap.cpp", "engine.cpp",
               "table.cpp", "binned.cpp", "capi.cpp"]
CU_SOURCES = ["kernels.cu", "kernels_complete.cu", "kernels_complete_fixed.cu",
              "kernels_explicit.cu", "kernels_codes.cu", "kernels_shap.cu", "kernels_binned.cu",
              "noalloc.cu"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def _nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found (set NVCC)")


def _cuda_home(nvcc: str) -> Path:
    return Path(nvcc).resolve().parent.parent


def _sources():
    return ([CSRC / s for s in CXX_SOURCES] + [CSRC / s for s in CU_SOURCES]
            + sorted(CSRC.glob("*.h")) + sorted(CSRC.glob("*.cuh")) + [ROOT / "include" / "macboost_c.h", Path(__file__)])


def needs_build() -> bool:
    if not LIB.exists() or not CLI.exists():
        return True
    t = min(LIB.stat().st_mtime, CLI.stat().st_mtime)
    return any(p.stat().st_mtime > t for p in _sources() + [CSRC / "cli_main.cpp"])


def build(force: bool = False, verbose: bool = False) -> Path:
    if not force and not needs_build():
        return LIB
    nvcc = _nvcc()
    cuda = _cuda_home(nvcc)
    BUILD.mkdir(exist_ok=True)
    objs = []
    jobs = []
    for s in CU_SOURCES:
        o = BUILD / (Path(s).stem + ".cu.o")
        jobs.append([nvcc, "-std=c++17", *ARCH, "-lineinfo", "-O3", "-Xptxas", "-v",
                     "-Xcompiler", "-fPIC,-fvisibility=hidden", "-I", str(CSRC),
                     "-c", str(CSRC / s), "-o", str(o)])
        objs.append(o)
    cxx = os.environ.get("CXX", "g++")
    for s in CXX_SOURCES:
        o = BUILD / (Path(s).stem + ".o")
        jobs.append([cxx, "-std=c++17", "-O2", "-fPIC", "-Wall", "-Wextra", "-fno-fast-math",
                     "-I", str(cuda / "include"), "-I", str(CSRC), "-c", str(CSRC / s),
                     "-o", str(o)])
        objs.append(o)
    procs = [subprocess.Popen(j, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
             for j in jobs]
    failed = []
    for j, p in zip(jobs, procs):
        out, _ = p.communicate()
        if verbose or p.returncode:
            sys.stdout.write(out)
        if p.returncode:
            failed.append(" ".join(j))
    if failed:
        raise RuntimeError("compilation failed:\n" + "\n".join(failed))
    vscript = BUILD / "exports.map"
    vscript.write_text("{\n  global: macboost_*;\n  local: *;\n};\n")
    tmp = LIB.with_suffix(f".so.tmp{os.getpid()}")
    link = [nvcc, *ARCH, "-shared", "-cudart", "static", "-o", str(tmp), *map(str, objs),
            "-Xlinker", f"--version-script={vscript}", "-Xlinker", "-Bsymbolic",
            "-Xlinker", "--exclude-libs,ALL", "-lpthread", "-ldl", "-lrt"]
    r = subprocess.run(link, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode:
        sys.stdout.write(r.stdout)
        raise RuntimeError("link failed: " + " ".join(link))
    os.replace(tmp, LIB)
    build_cli(cxx)
    return LIB


def build_cli(cxx: str = "g++") -> Path:
    """The `macboost` executable: main.swift's inference commands in C++,
    linked to libmacboostc.so beside it (rpath $ORIGIN)."""
    tmp = CLI.with_name(f"macboost.tmp{os.getpid()}")
    cmd = [cxx, "-std=c++17", "-O2", "-Wall", "-Wextra", str(CSRC / "cli_main.cpp"),
           "-o", str(tmp), f"-L{PKG}", "-lmacboostc", "-Wl,-rpath,$ORIGIN"]
    r = subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True)
    if r.returncode:
        sys.stdout.write(r.stdout)
        raise RuntimeError("CLI build failed: " + " ".join(cmd))
    os.replace(tmp, CLI)
    return CLI


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
    print(LIB)
