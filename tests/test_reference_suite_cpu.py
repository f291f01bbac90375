"""The drop-in header boundary, checked with the reference's OWN test sources:
tests/unit/framework.cu + multi_tu.cu, tests/model/ops_test.cu,
tests/model/llama_test.cu, llama_bf16_test.cu and the six
tests/integration/*.cu adapters of OpWorks, compiled unchanged for sm_100a
against this repository's include/ by oracle/build_ref.py (into
oracle/_ref/suite/, with a manifest of the commands and of every header nvcc
reported).

On CPU: every unit built, no header came from the reference's include/ (our
include/ supplied <opworks> and the "../include/..." headers), and the
framework binary, run without a GPU, exits with the reference's own "no CUDA
device" skip code 77 (tests/unit/framework.cu:224-231). The binaries run on
the GPU in tests/test_reference_suite_gpu.py.
"""

import json
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUITE = os.path.join(ROOT, "oracle", "_ref", "suite")
MANIFEST = os.path.join(SUITE, "manifest.json")
UNITS = ["framework", "ops_test", "llama_test.o", "llama_bf16_test.o"] + [
    f"test_{op}.so" for op in ("vector_add", "relu", "reduction", "softmax", "layer_normalization",
                               "matrix_multiplication")]


@pytest.fixture(scope="module")
def manifest():
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    try:
        import build_ref

        if build_ref.reference_root() is not None:
            build_ref.build(verbose=False)  # no-op when up to date
    finally:
        sys.path.pop(0)
    if not os.path.exists(MANIFEST):
        pytest.skip("the reference tree is not available and its suite was never built here")
    with open(MANIFEST) as f:
        return json.load(f)


def test_every_reference_unit_built_against_our_headers(manifest):
    ours = manifest["our_include"]
    theirs = manifest["reference_include"]
    for name in UNITS:
        unit = manifest["units"].get(name)
        assert unit is not None, f"{name} missing from the manifest"
        assert unit["built"] and os.path.exists(os.path.join(SUITE, name)), f"{name} did not compile"
        headers = unit["headers"]
        assert headers, name
        assert not [h for h in headers if h.startswith(theirs + os.sep)], name
        assert any(h.startswith(ours + os.sep) for h in headers), name
        # the include path names our include/, never the reference's
        assert f"-I {ours}" in unit["command"] and theirs not in unit["command"], name


def test_reference_framework_binary_skips_cleanly_without_a_gpu(manifest):
    binary = os.path.join(SUITE, "framework")
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    rc = subprocess.run([binary], env=env, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, timeout=120).returncode
    assert rc == 77, rc
