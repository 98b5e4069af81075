"""Build libbreeze_ql.so in-tree for sm_100a with nvcc.

Usage: ``python -m breeze_engine_b200.build [--force] [--debug]``.  The output
sits next to this file so it travels with the repository snapshot; nothing is
installed into site-packages or a JIT cache.
"""
import argparse
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
LIB = os.path.join(HERE, "libbreeze_ql.so")
SOURCES = ["ql_api.cu", "ql_quant.cu", "ql_prepack.cu", "ql_gemv.cu", "ql_gemv4.cu", "ql_gemm.cu", "ql_gemm16.cu", "ql_gemmw.cu",
           "ql_norm.cu", "ql_peer.cu"]
HEADERS = ["ql_common.cuh", "ql_internal.h", "ql_tcgen05.cuh", "ql_quant.cuh"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]


def nvcc():
    cuda = os.environ.get("CUDA_HOME", "/usr/local/cuda")
    path = os.path.join(cuda, "bin", "nvcc")
    return path if os.path.exists(path) else "nvcc"


def _stale():
    if not os.path.exists(LIB):
        return True
    t = os.path.getmtime(LIB)
    deps = [os.path.join(CSRC, f) for f in SOURCES + HEADERS]
    deps.append(os.path.join(os.path.dirname(HERE), "include", "breeze_ql.h"))
    deps.append(os.path.abspath(__file__))
    return any(os.path.getmtime(d) > t for d in deps if os.path.exists(d))


def build(force=False, debug=False, verbose=False):
    """Compile every source for sm_100a into one shared library (in-tree)."""
    if not force and not _stale():
        return LIB
    tmp = LIB + f".{os.getpid()}.tmp"
    cmd = [nvcc(), *ARCH, "-O3", "-lineinfo", "-std=c++17", "-shared", "-Xcompiler", "-fPIC",
           "-Xcompiler", "-fvisibility=hidden", "-Xcompiler", "-fopenmp", "--expt-relaxed-constexpr",
           "-I", os.path.join(os.path.dirname(HERE), "include"),
           *([] if not debug else ["-DQL_DEBUG"]),
           *([] if not verbose else ["-Xptxas", "-v"]),
           *[os.path.join(CSRC, s) for s in SOURCES], "-lgomp", "-o", tmp]
    try:
        subprocess.run(cmd, check=True)
        os.replace(tmp, LIB)
    finally:
        if os.path.exists(tmp):
            os.unlink(tmp)
    return LIB


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__)
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--debug", action="store_true")
    ap.add_argument("--verbose", action="store_true", help="print ptxas register/smem usage")
    args = ap.parse_args(argv)
    print(build(force=args.force, debug=args.debug, verbose=args.verbose))
    return 0


if __name__ == "__main__":
    sys.exit(main())
