"""Builds libfa_b200.so (the sm_100a kernels + C ABI) in-tree with nvcc.

The library lands in tilelang_fa_v100/_lib/ next to the Python package that loads
it, so it travels with the source tree.  Objects are compiled in parallel into
_build/ (git-ignored) and re-used when the sources and headers are unchanged.
"""
import concurrent.futures
import hashlib
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
BUILD = os.path.join(HERE, "_build")
LIB_DIR = os.path.join(HERE, "tilelang_fa_v100", "_lib")
LIB = os.path.join(LIB_DIR, "libfa_b200.so")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ARCH + [
    "-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "-Xcompiler", "-O3",
    "--expt-relaxed-constexpr", "-I", CSRC, "-I", INCLUDE,
]


def _nvcc():
    cand = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")
    return cand if os.path.exists(cand) else "nvcc"


def _sources():
    return sorted(os.path.join(CSRC, f) for f in os.listdir(CSRC) if f.endswith(".cu"))


def _headers_digest():
    h = hashlib.sha256()
    for d in (CSRC, INCLUDE):
        for f in sorted(os.listdir(d)):
            if f.endswith((".cuh", ".h")):
                with open(os.path.join(d, f), "rb") as fh:
                    h.update(f.encode() + fh.read())
    h.update(" ".join(NVCC_FLAGS).encode())
    return h.hexdigest()[:16]


def _compile(src, digest, ptxas_verbose):
    with open(src, "rb") as fh:
        key = hashlib.sha256(fh.read() + digest.encode()).hexdigest()[:16]
    obj = os.path.join(BUILD, os.path.basename(src) + "." + key + ".o")
    if os.path.exists(obj) and not ptxas_verbose:
        return obj, ""
    cmd = [_nvcc()] + NVCC_FLAGS + (["-Xptxas", "-v"] if ptxas_verbose else []) + ["-c", src, "-o", obj]
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("nvcc failed for %s:\n%s\n%s" % (src, r.stdout, r.stderr))
    return obj, r.stderr


def build(verbose=False, ptxas_verbose=False):
    """Compiles every csrc/*.cu for sm_100a and links libfa_b200.so; returns its path."""
    os.makedirs(BUILD, exist_ok=True)
    os.makedirs(LIB_DIR, exist_ok=True)
    digest = _headers_digest()
    srcs = _sources()
    with concurrent.futures.ThreadPoolExecutor(max_workers=min(8, len(srcs))) as ex:
        results = list(ex.map(lambda s: _compile(s, digest, ptxas_verbose), srcs))
    objs = [o for o, _ in results]
    if verbose or ptxas_verbose:
        for (_, log), s in zip(results, srcs):
            if log:
                print("== %s\n%s" % (os.path.basename(s), log), file=sys.stderr)
    tmp = LIB + ".tmp"
    if os.environ.get("FA_CUDART", "static") == "shared":
        rt = ["-cudart", "shared", "-Xlinker", "-rpath=/usr/local/cuda/lib64"]
    else:
        rt = ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]
    cmd = [_nvcc()] + ARCH + ["-shared", "-o", tmp] + objs + rt
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError("link failed:\n%s\n%s" % (r.stdout, r.stderr))
    os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(verbose=True, ptxas_verbose="-v" in sys.argv))
