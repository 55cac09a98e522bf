"""Build libkmamba_b200.so in-tree with nvcc for sm_100a (no JIT cache).

Each source compiles to its own object under bissimamba_b200/_build (in
parallel, rebuilt only when the source or a header is newer), then one link
step writes the shared library next to this file."""
from __future__ import annotations

import os
import subprocess
import sys
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OBJ = os.path.join(HERE, "_build")
OUT = os.path.join(HERE, "libkmamba_b200.so")
SOURCES = ["capi.cu", "scannd_generic.cu", "scannd_tma.cu", "scannd_strips.cu", "scannd_bwd.cu", "scannd_bwd_strips.cu", "convnd.cu", "convnd_fused.cu",
           "blockscan.cu", "block.cu", "proj_tc.cu", "gemm_tc.cu", "block_gemm.cu", "model.cu", "distributed.cu", "kser.cpp", "wavefront.cpp"]
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-O3", "-std=c++17", "-gencode", "arch=compute_100a,code=sm_100a", "-lineinfo",
         "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr", "-ccbin", "/usr/bin/g++"]


def _nccl_dir():
    """NCCL of the image: the copy PyTorch loads (nvidia-nccl wheel), so one
    process never holds two NCCL versions; else the system one."""
    try:
        import nvidia.nccl
        d = list(nvidia.nccl.__path__)[0]
        if os.path.exists(os.path.join(d, "include", "nccl.h")):
            return d
    except ImportError:
        pass
    return None


_NCCL = _nccl_dir()
if _NCCL:
    FLAGS += ["-I" + os.path.join(_NCCL, "include")]
    LIBS = ["-L" + os.path.join(_NCCL, "lib"), "-l:libnccl.so.2",
            "-Xlinker", "-rpath=" + os.path.join(_NCCL, "lib")]
else:
    LIBS = ["-lnccl"]


def _headers():
    hs = [os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith((".cuh", ".h"))]
    inc = os.path.join(HERE, "..", "include")
    hs += [os.path.join(inc, f) for f in os.listdir(inc)]
    return hs


def _obj(src):
    return os.path.join(OBJ, os.path.splitext(src)[0] + ".o")


def needs_build() -> bool:
    if not os.path.exists(OUT):
        return True
    t = os.path.getmtime(OUT)
    if os.path.isdir(OBJ) and any(not os.path.exists(_obj(s)) for s in SOURCES):
        return True
    deps = [os.path.join(CSRC, s) for s in SOURCES] + _headers()
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src, verbose):
    cmd = [NVCC] + FLAGS + (["-Xptxas=-v"] if verbose else []) + ["-c", "-o", _obj(src), os.path.join(CSRC, src)]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed on {src}:\n{r.stdout}\n{r.stderr}")
    return r.stderr if verbose else ""


def build(force: bool = False, verbose: bool = False) -> str:
    if not force and not needs_build():
        return OUT
    os.makedirs(OBJ, exist_ok=True)
    hdr_t = max(os.path.getmtime(h) for h in _headers())
    todo = []
    for s in SOURCES:
        o = _obj(s)
        if force or not os.path.exists(o) or os.path.getmtime(o) < max(os.path.getmtime(os.path.join(CSRC, s)), hdr_t):
            todo.append(s)
    with ThreadPoolExecutor(max_workers=min(len(todo), os.cpu_count() or 4) or 1) as ex:
        for msg in ex.map(lambda s: _compile(s, verbose), todo):
            if msg:
                print(msg)
    cmd = [NVCC, "-shared", "-gencode", "arch=compute_100a,code=sm_100a", "-ccbin", "/usr/bin/g++", "-o", OUT]
    cmd += [_obj(s) for s in SOURCES] + LIBS
    subprocess.run(cmd, check=True)
    return OUT


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose="-v" in sys.argv)
