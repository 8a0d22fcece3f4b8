"""Build the rung's native code in-tree: gemm-ladder_b200/lib/libbwgemm.so (sm_100a, cross-compiled by nvcc; no GPU
needed).  ``python gemm-ladder_b200/build.py [--force] [--trace] [--next]``; --trace builds lib/libbwgemm_trace.so,
the same library with the per-block timeline compiled in (-DBW_TRACE: per block, %globaltimer stamps of its phases,
read back with bw_trace_read); --next builds lib/libbwgemm_next.so, the library with the options built but not on by
default (the K split over clusters of 2 to 8 blocks, the TMA-store epilogue), for A/B runs: BWGEMM_LIB=libbwgemm_next.so
selects it.  (Stream-K over a part wave of pair tiles and swap-AB on SM pairs were measured slower and stay off; the
host emulator still builds and checks them.)"""
import os
import shutil
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
CSRC = os.path.join(HERE, "csrc")
LIB_DIR = os.path.join(HERE, "lib")
LIB = os.path.join(LIB_DIR, "libbwgemm.so")
TRACE_LIB = os.path.join(LIB_DIR, "libbwgemm_trace.so")
NEXT_LIB = os.path.join(LIB_DIR, "libbwgemm_next.so")
NEXT_DEFINES = ["-DBW_KSPLIT=1", "-DBW_EPI_TMA=1"]
INCLUDE = os.path.join(ROOT, "include")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", *ARCH, "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
              f"-I{INCLUDE}", f"-I{CSRC}"]


def nvcc():
    for cand in (shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and os.path.exists(cand):
            return cand
    raise RuntimeError("nvcc not found")


def sources():
    out = [os.path.join(INCLUDE, "bwgemm.h")]
    for f in sorted(os.listdir(CSRC)):
        if f.endswith((".cu", ".cuh", ".h")):
            out.append(os.path.join(CSRC, f))
    return out


def up_to_date(lib=LIB):
    if not os.path.exists(lib):
        return False
    t = os.path.getmtime(lib)
    return all(os.path.getmtime(s) <= t for s in sources())


def build(force=False, verbose=False, trace=False, next_options=False):
    """Compile libbwgemm.so (trace: libbwgemm_trace.so; next_options: libbwgemm_next.so; both:
    libbwgemm_next_trace.so) if a source is newer than it (or force)."""
    lib = (os.path.join(LIB_DIR, "libbwgemm_next_trace.so") if trace and next_options else TRACE_LIB if trace
           else NEXT_LIB if next_options else LIB)
    if not force and up_to_date(lib):
        return lib
    os.makedirs(LIB_DIR, exist_ok=True)
    defines = (["-DBW_TRACE"] if trace else []) + (NEXT_DEFINES if next_options else [])
    cmd = [nvcc(), *NVCC_FLAGS, *defines, os.path.join(CSRC, "bwgemm.cu"), "-o", lib + ".tmp"]
    if verbose:
        print(" ".join(cmd))
    subprocess.check_call(cmd)
    os.replace(lib + ".tmp", lib)
    return lib


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose=True, trace="--trace" in sys.argv,
                next_options="--next" in sys.argv))
