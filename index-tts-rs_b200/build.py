"""Builds the in-tree shared libraries of the package.

  libitts_gpt.so   -- the decoder (CUDA, sm_100a) behind include/itts_gpt.h
  libitts_synth.so -- seeded synthetic weights (host only; benchmarks and tests)

Objects go to _build/ (not committed); the .so files sit next to this file so a
snapshot of the repository carries them to a GPU machine.
"""
from __future__ import annotations

import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
BUILD = PKG / "_build"
INCLUDE = PKG.parent / "include"
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CU_SOURCES = ["decode.cu", "decode_wide.cu", "codec.cu", "mk_decode.cu", "xk_decode.cu", "prefill.cu", "prefill_batch.cu", "gemm_tc.cu", "sample.cu", "api.cu"]


def _nvcc() -> str:
    for c in (os.environ.get("NVCC"), "/usr/local/cuda/bin/nvcc", shutil.which("nvcc")):
        if c and Path(c).exists():
            return c
    raise RuntimeError("nvcc not found")


def _host_cxx() -> str:
    return "/usr/bin/g++" if Path("/usr/bin/g++").exists() else "g++"


def _run(cmd):
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"build failed: {' '.join(cmd)}\n{r.stdout}\n{r.stderr}")
    return r.stdout + r.stderr


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build(verbose: bool = False, ptxas_verbose: bool = False) -> dict:
    BUILD.mkdir(exist_ok=True)
    nvcc = _nvcc()
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [INCLUDE / "itts_gpt.h"]
    flags = ARCH + ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-ccbin",
                    _host_cxx(), f"-I{INCLUDE}"]
    if ptxas_verbose:
        flags += ["-Xptxas", "-v"]
    logs = {}

    def compile_one(src):
        obj = BUILD / (src + ".o")
        if _stale(obj, [CSRC / src] + headers) or ptxas_verbose:
            logs[src] = _run([nvcc] + flags + ["-c", str(CSRC / src), "-o", str(obj)])
        return obj

    with cf.ThreadPoolExecutor(max_workers=len(CU_SOURCES)) as ex:
        objs = list(ex.map(compile_one, CU_SOURCES))
    lib = PKG / "libitts_gpt.so"
    if _stale(lib, objs):
        _run([nvcc] + ARCH + ["-shared", "-o", str(lib)] + [str(o) for o in objs] +
             ["-lcudart", "-Xlinker", "--no-undefined"])
    synth = PKG / "libitts_synth.so"
    if _stale(synth, [CSRC / "synth.cpp"]):
        _run([_host_cxx(), "-O3", "-fopenmp", "-fPIC", "-shared", "-ffp-contract=off",
              str(CSRC / "synth.cpp"), "-o", str(synth)])
    if verbose:
        for k, v in logs.items():
            print(f"== {k}\n{v}")
    return logs


if __name__ == "__main__":
    out = build(verbose=True, ptxas_verbose="-v" in sys.argv)
    print("built", PKG / "libitts_gpt.so")
