"""ORACLE — test infrastructure only. Builds the checkers the tests use; the
product never loads any of it.

    oracle/liboracle.so                   <- oracle/oracle.cpp (g++, OpenMP)
    tests/native/lib<name>.so             <- tests/native/<name>.cu (test-only hooks)

and, when the reference (OpWorks) source tree is available, from its own
sources (nvcc on a few files; no CMake, no reference build system), into
oracle/_ref/ (git-ignored; travels to the GPU box with the snapshot):

    libopworks_llama_ref.so   <- <ref>/src/llama_c_api.cu
    libopworks_ops_ref.so     <- oracle/ref_ops_shim.cu over <ref>/include
    suite/                    <- the reference's OWN test sources, unchanged,
                                 compiled against THIS repository's include/:
        framework             tests/unit/framework.cu + multi_tu.cu
        ops_test              tests/model/ops_test.cu
        test_<op>.so          tests/integration/<op>.cu (the solve() adapters)
        llama_test.o, llama_bf16_test.o   compile-only (their HF fixtures are absent)
        ops_fixtures.opw      the reference's scripts/llama/export_reference.py
                              build_op_fixtures() on a reduced hidden size
        manifest.json         per artifact: command, and every header nvcc -M
                              reports (none may lie under <ref>/include)

The reference tree is located by reference_root(): an explicit argument,
else the OPWORKS_REFERENCE environment variable, else a directory named
`reference` beside this repository's root.

    python oracle/build_ref.py [<reference root>] [--force]
"""

from __future__ import annotations

import importlib.util
import json
import os
import shlex
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(HERE)
OUT = os.path.join(HERE, "_ref")
SUITE = os.path.join(OUT, "suite")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
LIB_FLAGS = ["-std=c++17", "-O3", "-Xcompiler", "-fPIC", "-shared", "-w"] + ARCH
SUITE_FLAGS = ["-std=c++17", "-O3", "-w", "--expt-relaxed-constexpr"] + ARCH
# our include/ for <opworks>; tests/ so that the sources' "../include/..." lands in our include/
SUITE_INC = ["-I", os.path.join(REPO, "include"), "-I", os.path.join(REPO, "tests")]
INTEGRATION_OPS = ["vector_add", "relu", "reduction", "softmax", "layer_normalization", "matrix_multiplication"]
# build_op_fixtures() config: Llama-3.2-1B attention shapes and vocabulary with a
# reduced hidden size, so the pack (dominated by the vocab x hidden embedding
# table) stays 66 MB instead of 1 GB
FIXTURE_CFG = {
    "hidden_size": 128, "intermediate_size": 512, "head_dim": 64, "num_attention_heads": 32,
    "num_key_value_heads": 8, "rms_norm_eps": 1e-5, "vocab_size": 128256, "rope_theta": 500000.0,
    "rope_scaling": {"rope_type": "llama3", "factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                     "original_max_position_embeddings": 8192},
}


def reference_root(explicit=None):
    """The reference source tree, or None when it is not available."""
    for cand in (explicit, os.environ.get("OPWORKS_REFERENCE"), os.path.join(os.path.dirname(REPO), "reference")):
        if cand and os.path.isdir(os.path.join(cand, "include")):
            return os.path.abspath(cand)
    return None


def _stale(target, sources):
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources if os.path.isfile(s))


def _run_all(jobs, verbose, what):
    """jobs: [(target, cmd)]; runs them in parallel, returns {target: ok}."""
    procs = [(t, c, subprocess.Popen(c, stdout=subprocess.PIPE, stderr=subprocess.STDOUT)) for t, c in jobs]
    ok = {}
    for t, c, p in procs:
        out, _ = p.communicate()
        ok[t] = p.returncode == 0
        if not ok[t]:
            print(f"{what} build of {t} failed:\n{out.decode(errors='replace')}", file=sys.stderr)
        elif verbose:
            print(f"built {os.path.relpath(t, REPO)}", file=sys.stderr)
    return ok


def build_oracle(force=False, verbose=True):
    src = os.path.join(HERE, "oracle.cpp")
    lib = os.path.join(HERE, "liboracle.so")
    if force or _stale(lib, [src]):
        ok = _run_all([(lib, ["g++", "-O3", "-march=x86-64-v3", "-fopenmp", "-std=c++17", "-shared", "-fPIC", src,
                              "-o", lib])], verbose, "oracle")
        if not ok[lib]:
            raise RuntimeError("oracle build failed")


def build_test_hooks(force=False, verbose=True):
    """tests/native/*.cu -> tests/native/lib<name>.so: test-only entry points
    that drive single product kernels (included from include/) in ways the
    product's C ABI never does, e.g. a bounded wait that runs out."""
    native = os.path.join(REPO, "tests", "native")
    ours = [os.path.join(dp, f) for dp, _, fs in os.walk(os.path.join(REPO, "include")) for f in fs]
    jobs = []
    for name in sorted(os.listdir(native)) if os.path.isdir(native) else []:
        if not name.endswith(".cu"):
            continue
        src = os.path.join(native, name)
        lib = os.path.join(native, "lib" + name[:-3] + ".so")
        if force or _stale(lib, [src] + ours):
            jobs.append((lib, [NVCC] + LIB_FLAGS + ["-lineinfo", "-I", os.path.join(REPO, "include"), src,
                                                    "-o", lib]))
    ok = _run_all(jobs, verbose, "test hook")
    if not all(ok.values()):
        raise RuntimeError("test hook build failed")


def _headers(cmd_sources, extra_flags):
    """Every header nvcc -M reports for the sources (host-side dependency scan)."""
    out = subprocess.run([NVCC, "-M", "-std=c++17"] + ARCH + extra_flags + cmd_sources, stdout=subprocess.PIPE,
                         stderr=subprocess.DEVNULL, text=True)
    if out.returncode != 0:
        return None
    deps = out.stdout.replace("\\\n", " ").split(":", 1)[-1].split()
    return sorted({os.path.abspath(d) for d in deps if not d.startswith("/usr") and not d.endswith(".cu")})


def _fixture_pack(ref, path):
    spec = importlib.util.spec_from_file_location("ref_export_reference",
                                                  os.path.join(ref, "scripts", "llama", "export_reference.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, os.path.join(ref, "scripts", "llama"))
    try:
        spec.loader.exec_module(mod)
        mod.build_op_fixtures(dict(FIXTURE_CFG)).write(path)
    finally:
        sys.path.pop(0)


def build_reference(ref, force=False, verbose=True):
    os.makedirs(SUITE, exist_ok=True)
    inc = os.path.join(ref, "include")
    jobs = []
    llama = os.path.join(OUT, "libopworks_llama_ref.so")
    src = os.path.join(ref, "src", "llama_c_api.cu")
    if os.path.exists(src) and (force or _stale(llama, [src])):
        jobs.append((llama, [NVCC] + LIB_FLAGS + ["-I", inc, src, "-o", llama]))
    ops = os.path.join(OUT, "libopworks_ops_ref.so")
    shim = os.path.join(HERE, "ref_ops_shim.cu")
    if force or _stale(ops, [shim]):
        jobs.append((ops, [NVCC] + LIB_FLAGS + ["-I", inc, shim, "-o", ops]))
    _run_all(jobs, verbose, "reference")

    # the reference's own tests against our headers
    ours = [os.path.join(dp, f) for dp, _, fs in os.walk(os.path.join(REPO, "include")) for f in fs]
    t = lambda *p: os.path.join(ref, "tests", *p)  # noqa: E731
    units = [("framework", [t("unit", "framework.cu"), t("unit", "multi_tu.cu")], []),
             ("ops_test", [t("model", "ops_test.cu")], [])]
    units += [(f"test_{op}.so", [t("integration", f"{op}.cu")], ["-shared", "-Xcompiler", "-fPIC"])
              for op in INTEGRATION_OPS]
    units += [(f"{name}.o", [t("model", f"{name}.cu")], ["-c"]) for name in ("llama_test", "llama_bf16_test")]
    suite_jobs, manifest = [], {"reference_include": inc, "our_include": os.path.join(REPO, "include"), "units": {}}
    for name, srcs, extra in units:
        if not all(os.path.exists(s) for s in srcs):
            continue
        target = os.path.join(SUITE, name)
        cmd = [NVCC] + SUITE_FLAGS + extra + SUITE_INC + srcs + ["-o", target]
        manifest["units"][name] = {"sources": srcs, "command": shlex.join(cmd),
                                   "headers": _headers(srcs[:1], SUITE_INC)}
        if force or _stale(target, srcs + ours):
            suite_jobs.append((target, cmd))
    ok = _run_all(suite_jobs, verbose, "reference suite")
    for name in manifest["units"]:
        target = os.path.join(SUITE, name)
        manifest["units"][name]["built"] = ok.get(target, os.path.exists(target))
    pack = os.path.join(SUITE, "ops_fixtures.opw")
    if force or not os.path.exists(pack):
        try:
            _fixture_pack(ref, pack)
            if verbose:
                print(f"built {os.path.relpath(pack, REPO)}", file=sys.stderr)
        except Exception as e:  # torch or the reference script unavailable: the GPU test skips
            print(f"reference op fixtures not generated: {e}", file=sys.stderr)
    manifest["ops_fixtures"] = {"config": FIXTURE_CFG, "built": os.path.exists(pack)}
    with open(os.path.join(SUITE, "manifest.json"), "w") as f:
        json.dump(manifest, f, indent=1)


def build(ref=None, force=False, verbose=True):
    build_oracle(force, verbose)
    build_test_hooks(force, verbose)
    root = reference_root(ref)
    if root is not None:
        build_reference(root, force, verbose)
    elif verbose:
        print("reference tree not found (argument, OPWORKS_REFERENCE or ../reference): "
              "reference checkers not rebuilt", file=sys.stderr)


if __name__ == "__main__":
    args = [a for a in sys.argv[1:] if not a.startswith("--")]
    build(args[0] if args else None, force="--force" in sys.argv)
