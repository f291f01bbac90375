"""Builds the in-tree shared libraries (nvcc for sm_100a, g++ for the oracle).

    python -m opworks_b200.build            # everything that is stale
    python -m opworks_b200.build --force    # rebuild all

Outputs live next to the sources so they travel with the repository:
    opworks_b200/lib/libopworks_ops.so     operator C ABI   (include/opworks_ops.h)
    opworks_b200/lib/libopworks_llama.so   Llama C ABI      (include/opworks_llama.h)

The test checkers (CPU oracle, reference builds) have their own recipe,
oracle/build_ref.py; __graft_entry__.build() runs both.
"""

from __future__ import annotations

import glob
import os
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
INC = os.path.join(ROOT, "include")
CSRC = os.path.join(ROOT, "opworks_b200", "csrc")
LIBDIR = os.path.join(ROOT, "opworks_b200", "lib")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-std=c++17", "-O3", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "-shared",
              "--expt-relaxed-constexpr",
              "-Xcudafe", "--diag_suppress=177"] + ARCH


def _headers():
    return glob.glob(os.path.join(INC, "**", "*"), recursive=True)


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.isfile(s))


def _targets():
    hdrs = _headers()
    out = []
    out.append((os.path.join(LIBDIR, "libopworks_ops.so"),
                [NVCC] + NVCC_FLAGS + ["-I", INC, os.path.join(CSRC, "ops_c_api.cu"), "-o",
                                       os.path.join(LIBDIR, "libopworks_ops.so")],
                hdrs + [os.path.join(CSRC, "ops_c_api.cu")]))
    llama_srcs = sorted(glob.glob(os.path.join(CSRC, "llama*.cu")))
    if llama_srcs:
        out.append((os.path.join(LIBDIR, "libopworks_llama.so"),
                    [NVCC] + NVCC_FLAGS + ["-I", INC] + llama_srcs + ["-o", os.path.join(LIBDIR, "libopworks_llama.so")],
                    hdrs + llama_srcs))
    return out


def build(force=False, verbose=True):
    os.makedirs(LIBDIR, exist_ok=True)
    jobs = []
    for target, cmd, srcs in _targets():
        if force or _stale(target, srcs):
            jobs.append((target, cmd, subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)))
    t0 = time.time()
    failed = []
    for target, cmd, proc in jobs:
        out, _ = proc.communicate()
        text = out.decode(errors="replace")
        if proc.returncode != 0:
            failed.append((target, text))
        elif verbose:
            print(f"built {os.path.relpath(target, ROOT)}", file=sys.stderr)
    if failed:
        for target, text in failed:
            print(f"--- build of {target} failed:\n{text}", file=sys.stderr)
        raise RuntimeError("build failed: " + ", ".join(os.path.basename(t) for t, _ in failed))
    if verbose and jobs:
        print(f"build: {len(jobs)} target(s) in {time.time() - t0:.1f}s", file=sys.stderr)


if __name__ == "__main__":
    build(force="--force" in sys.argv)
