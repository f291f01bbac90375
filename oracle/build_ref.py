"""ORACLE — test infrastructure only. Recipe that compiles the reference
(OpWorks) from its own sources, in place under the reference tree, into
oracle/_ref/ (git-ignored; travels to the GPU box with the snapshot):

    oracle/_ref/libopworks_llama_ref.so  <- <ref>/src/llama_c_api.cu
    oracle/_ref/libopworks_ops_ref.so    <- oracle/ref_ops_shim.cu + <ref>/include

Only nvcc on those few files is used (no CMake, no reference build system).
The libraries are checkers: GPU tests compare our kernels with them on the same
inputs, and bench.py may time them alongside our own path.
"""

from __future__ import annotations

import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
OUT = os.path.join(HERE, "_ref")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
FLAGS = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC", "-shared", "-gencode", "arch=compute_100a,code=sm_100a",
         "-w"]


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def build(ref_root, force=False, verbose=True):
    os.makedirs(OUT, exist_ok=True)
    inc = os.path.join(ref_root, "include")
    jobs = []
    llama = os.path.join(OUT, "libopworks_llama_ref.so")
    src = os.path.join(ref_root, "src", "llama_c_api.cu")
    if os.path.exists(src) and (force or _stale(llama, [src])):
        jobs.append((llama, [NVCC] + FLAGS + ["-I", inc, src, "-o", llama]))
    ops = os.path.join(OUT, "libopworks_ops_ref.so")
    shim = os.path.join(HERE, "ref_ops_shim.cu")
    if force or _stale(ops, [shim]):
        jobs.append((ops, [NVCC] + FLAGS + ["-I", inc, shim, "-o", ops]))
    procs = [(t, subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)) for t, c in jobs]
    for t, p in procs:
        out, _ = p.communicate()
        if p.returncode != 0:
            print(f"reference build of {t} failed (checker unavailable):\n{out.decode(errors='replace')}",
                  file=sys.stderr)
        elif verbose:
            print(f"built {os.path.relpath(t, os.path.dirname(HERE))}", file=sys.stderr)


if __name__ == "__main__":
    build(sys.argv[1] if len(sys.argv) > 1 else "/root/reference", force="--force" in sys.argv)
