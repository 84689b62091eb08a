"""In-tree build of ``pax_b200/libpax_b200.so`` for sm_100a.

Compiles each translation unit under ``pax_b200/csrc`` with nvcc
(``-gencode arch=compute_100a,code=sm_100a -lineinfo``) into
``pax_b200/_build`` and links them into one shared library next to this
file, so the library travels with the source tree.  Objects are rebuilt when
any source or header is newer.  Run ``python -m pax_b200.build``.
"""
from __future__ import annotations

import concurrent.futures
import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD_DIR = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libpax_b200.so")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

SOURCES = ["gemm_tc_f16.cu", "gemm_tc_f32.cu", "gemm_tc.cu", "gemm_skinny.cu", "gemm_simt.cu", "peer_sync.cu",
           "host_bridge.cpp", "fp16_ops.cpp"]
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-O3", "--expt-relaxed-constexpr", "-I", INCLUDE]
# Host-only translation unit: cpu_gemm_ref is built with the same host flags
# as the reference's own CPU build (oracle/Makefile) so their fp32 results
# agree bit for bit.
HOST_FLAGS = {"host_bridge.cpp": ["-Xcompiler", "-march=x86-64-v3,-ffp-contract=fast"]}


def _headers() -> list[str]:
    return (glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(CSRC, "*.h"))
            + glob.glob(os.path.join(INCLUDE, "*.h")))


def _stale(target: str, deps: list[str]) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(d) > t for d in deps)


def _compile(src: str, verbose: bool) -> str:
    obj = os.path.join(BUILD_DIR, os.path.splitext(src)[0] + ".o")
    path = os.path.join(CSRC, src)
    if not _stale(obj, [path] + _headers()):
        return obj
    cmd = [NVCC, *ARCH, *FLAGS, *HOST_FLAGS.get(src, []), "-c", path, "-o", obj]
    if verbose:
        cmd.insert(1, "-Xptxas=-v")
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"nvcc failed for {src}:\n{r.stdout}\n{r.stderr}")
    if verbose and (r.stdout or r.stderr):
        print(r.stdout + r.stderr, file=sys.stderr)
    return obj


def build(force: bool = False, verbose: bool = False) -> str:
    """Compile and link the library; returns its path."""
    os.makedirs(BUILD_DIR, exist_ok=True)
    if force:
        for o in glob.glob(os.path.join(BUILD_DIR, "*.o")):
            os.remove(o)
    with concurrent.futures.ThreadPoolExecutor(max_workers=len(SOURCES)) as ex:
        objs = list(ex.map(lambda s: _compile(s, verbose), SOURCES))
    if force or _stale(LIB, objs):
        tmp = LIB + ".tmp"
        cmd = [NVCC, *ARCH, "-shared", "-o", tmp, *objs, "-Xlinker", "--no-undefined"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"link failed:\n{r.stdout}\n{r.stderr}")
        os.replace(tmp, LIB)
    return LIB


if __name__ == "__main__":
    print(build(force="--force" in sys.argv, verbose="-v" in sys.argv))
