"""Build libspilltune_b200.so in-tree with nvcc for sm_100a.

    python -m spilltune_b200.build          # or spilltune_b200.build.build()

The library is plain C ABI (include/spilltune_b200.h) with the CUDA runtime
linked statically, so it loads into any process (torch or not) on a B200 host.
"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libspilltune_b200.so")
SOURCES = ["fl_capi.cu", "fl_dequant.cu", "fl_lora.cu", "fl_lora_down.cu", "fl_gemm.cu", "fl_gemm_bwd.cu", "fl_smallm.cu", "fl_smallm_bwd.cu", "fl_noalloc.cu", "fl_moe.cu", "fl_head.cu", "fl_split.cu"]
HEADERS = ["fl_ptx.cuh", "fl_codebook.cuh", "fl_host.h"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc_path():
    p = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(p):
        raise RuntimeError("nvcc not found; the CUDA toolkit is required to build libspilltune_b200")
    return p


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(ROOT, "include", "spilltune_b200.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, verbose=False, extra=()):
    if not force and not _stale():
        return LIB
    tmp = LIB + ".tmp"
    cmd = [nvcc_path(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC,-O2",
           "-I", os.path.join(ROOT, "include"), "-o", tmp,
           *[os.path.join(CSRC, s) for s in SOURCES], *extra]
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.run(cmd, check=True)
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True,
          extra=("-Xptxas", "-v") if "--ptxas-v" in sys.argv else ())
    print(LIB)
