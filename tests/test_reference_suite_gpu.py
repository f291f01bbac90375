"""The reference's OWN test programs, compiled unchanged against this
repository's include/ (oracle/_ref/suite/, built by oracle/build_ref.py where
the reference tree is available; the binaries travel with the repository):

* tests/unit/framework.cu + multi_tu.cu: exit code 0 (the reference's
  contracts, ownership, boundaries, streams, graph replay, reduction, row ops
  and matmul checks, tests/unit/framework.cu:224-240);
* tests/model/ops_test.cu on fixtures written by the reference's own
  build_op_fixtures() (scripts/llama/export_reference.py:93-175): "all
  operator tests passed" (tests/model/ops_test.cu:359-374);
* the six tests/integration/*.cu `solve()` adapters (the LeetGPU-style C
  ABI): called through ctypes on device buffers and checked against the CPU
  oracle with the operator tolerances.
"""

import ctypes
import os
import subprocess

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu
torch = pytest.importorskip("torch")

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
SUITE = os.path.join(ROOT, "oracle", "_ref", "suite")


def need(name):
    path = os.path.join(SUITE, name)
    if not os.path.exists(path):
        pytest.skip(f"{name} was not built (oracle/_ref/suite: the reference tree was unavailable at build time)")
    return path


def run(cmd):
    return subprocess.run(cmd, stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True, timeout=600)


def test_reference_framework_suite_passes():
    out = run([need("framework")])
    assert out.returncode == 0, out.stdout[-3000:]
    assert "PASS" in out.stdout


def test_reference_ops_test_passes_on_reference_fixtures():
    out = run([need("ops_test"), need("ops_fixtures.opw")])
    assert out.returncode == 0, out.stdout[-3000:]
    assert "all operator tests passed" in out.stdout, out.stdout[-3000:]


def _adapter(op):
    lib = ctypes.CDLL(need(f"test_{op}.so"))
    lib.solve.restype = None
    return lib.solve


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr())


def _close(a, e, tol=1e-5):
    a, e = np.asarray(a, np.float64), np.asarray(e, np.float64)
    rel = np.abs(a - e) / (1 + np.abs(e))
    assert np.all(rel <= tol), f"max rel err {rel.max():.3g}"


def test_reference_integration_adapters():
    rng = np.random.default_rng(11)
    keep = []  # device inputs must outlive the calls (the caching allocator reuses freed blocks)

    def dev(a):
        keep.append(torch.from_numpy(np.ascontiguousarray(a, np.float32)).cuda())
        return keep[-1]

    n = 1_000_003
    a, b = rng.standard_normal(n).astype(np.float32), rng.standard_normal(n).astype(np.float32)
    out = torch.empty(n, device="cuda")
    solve = _adapter("vector_add")
    solve.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_size_t]
    solve(_ptr(dev(a)), _ptr(dev(b)), _ptr(out), n)
    assert np.array_equal(out.cpu().numpy(), a + b)

    solve = _adapter("relu")
    solve.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    solve(_ptr(dev(a)), _ptr(out), n)
    assert np.array_equal(out.cpu().numpy(), np.maximum(a, 0))

    solve = _adapter("reduction")
    solve.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    x = rng.uniform(-1, 1, 1 << 24).astype(np.float32)
    s = torch.empty(1, device="cuda")
    solve(_ptr(dev(x)), _ptr(s), x.size)
    # fp32 accumulation over 2^24 terms: relative to the sum of magnitudes
    assert abs(float(s.cpu()[0]) - oracle.reduce_sum(x)) <= 1e-5 * (1 + np.abs(x).sum() / 1000)

    solve = _adapter("softmax")
    solve.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int]
    x = (rng.standard_normal(4099) * 4).astype(np.float32)
    o = torch.empty(x.size, device="cuda")
    solve(_ptr(dev(x)), _ptr(o), x.size)
    _close(o.cpu().numpy(), oracle.softmax(x[None, :])[0])

    solve = _adapter("layer_normalization")
    solve.argtypes = [ctypes.c_void_p] * 4 + [ctypes.c_int, ctypes.c_int, ctypes.c_float]
    x = rng.standard_normal((64, 2048)).astype(np.float32)
    g = rng.uniform(0.5, 1.5, 2048).astype(np.float32)
    be = (rng.standard_normal(2048) * 0.1).astype(np.float32)
    o = torch.empty(x.size, device="cuda")
    solve(_ptr(dev(x)), _ptr(dev(g)), _ptr(dev(be)), _ptr(o), 64, 2048, 1e-5)
    _close(o.cpu().numpy().reshape(64, 2048), oracle.layer_norm(x, g, be, 1e-5))

    solve = _adapter("matrix_multiplication")
    solve.argtypes = [ctypes.c_void_p] * 3 + [ctypes.c_int] * 3
    A = (rng.standard_normal((96, 300)) / 300 ** 0.5).astype(np.float32)
    B = (rng.standard_normal((300, 200)) / 300 ** 0.5).astype(np.float32)
    o = torch.empty(96 * 200, device="cuda")
    solve(_ptr(dev(A)), _ptr(dev(B)), _ptr(o), 96, 300, 200)
    _close(o.cpu().numpy().reshape(96, 200), oracle.mat_mul(A, B))
