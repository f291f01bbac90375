"""Kernel-level timings through the C ABIs: CUDA events on the launching
stream, warm-up first, L2 flushed (a 256 MB read) before every timed launch,
median over the timed launches.

    python -m opworks_b200.microbench c1        # config C1 operator shapes
    python -m opworks_b200.microbench decode    # decode-step kernels (C3 shapes)
    python -m opworks_b200.microbench prefill   # one 8192-token prefill (C4)
    python -m opworks_b200.microbench pair      # two-SM prefill GEMMs at the C4 shapes

`c1` times our operators and, when the reference was built from its own
sources into oracle/_ref (libopworks_ops_ref.so), the reference's kernels on
the same inputs. `decode` times the paged decode attention, the bf16x2
projection GEMMs and the fused sampler at the C3 shapes; it is also the
command the ncu captures under profiles/ were taken with.
"""

from __future__ import annotations

import argparse
import ctypes
import json
import os

import numpy as np

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_OPS = os.path.join(ROOT, "oracle", "_ref", "libopworks_ops_ref.so")


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class Timer:
    """Median CUDA-event time (ms) of fn(), with an L2 flush before each launch.

    The flush READS a 256 MB buffer (twice the L2): the cache is left holding
    clean lines, so the timed kernel pays no write-back of the flush's own
    data (a write flush would leave ~126 MB of dirty lines behind)."""

    def __init__(self, torch):
        self.torch = torch
        self.flush_buf = torch.ones(64 * 1024 * 1024, dtype=torch.float32, device="cuda")  # 256 MB > L2
        self.flush_out = torch.empty(1, dtype=torch.float32, device="cuda")

    def __call__(self, fn, iters=20, warmup=3):
        torch = self.torch
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize()
        times = []
        for _ in range(iters):
            torch.sum(self.flush_buf, dim=0, keepdim=True, out=self.flush_out)
            # a ~50 us device spin after the flush keeps the host's launch of
            # fn ahead of the GPU, so the events bracket device time only
            torch.cuda._sleep(100_000)
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            fn()
            e.record()
            torch.cuda.synchronize()
            times.append(s.elapsed_time(e))
        return float(np.median(times))


def _ref_ops():
    if not os.path.exists(REF_OPS):
        return None
    lib = ctypes.CDLL(REF_OPS)
    P, I, F = ctypes.c_void_p, ctypes.c_int, ctypes.c_float
    sigs = {"ref_softmax": [P, P, I, I], "ref_layer_norm": [P, P, P, P, I, I, F], "ref_mat_mul_relu": [P, P, P, I, I, I],
            "ref_reduce_sum": [P, P, I], "ref_reduce_sum_ws": [P, P, I, P, I], "ref_sync": []}
    for name, args in sigs.items():
        fn = getattr(lib, name)
        fn.argtypes = args
        fn.restype = None
    lib.ref_reduction_workspace_size.argtypes = [I]
    lib.ref_reduction_workspace_size.restype = I
    return lib


def c1(iters=20):
    """Config C1: softmax 4096x1024, layer_norm 4096x2048, mat_mul
    1024x2048 @ 2048x1024 + ReLU, Sum over 2^24 floats (seeded inputs)."""
    import torch

    import opworks_b200

    ops = opworks_b200.ops_lib()
    ref = _ref_ops()
    hbm, tc, src = measured_peaks()
    t = Timer(torch)
    g = torch.Generator(device="cpu")
    out = []

    def row(name, bytes_=None, flops=None, ours=None, theirs=None):
        r = {"op": name, "ours_us": round(ours * 1e3, 2)}
        if bytes_ is not None:
            r["bytes"] = bytes_
            r["ours_gbs"] = round(bytes_ / (ours / 1e3) / 1e9, 1)
            r["ours_frac_hbm"] = round(r["ours_gbs"] / hbm, 4)
        if flops is not None:
            r["flops"] = flops
            r["ours_tflops"] = round(flops / (ours / 1e3) / 1e12, 1)
            r["ours_frac_bf16_peak"] = round(r["ours_tflops"] / tc, 4)
        if theirs is not None:
            r["reference_us"] = round(theirs * 1e3, 2)
            r["speedup"] = round(theirs / ours, 2)
        out.append(r)

    g.manual_seed(1)
    x = (torch.randn(4096, 1024, generator=g) * 4).cuda()
    y = torch.empty_like(x)
    ours = t(lambda: ops.softmax(x, y, 4096, 1024, 0), iters)
    theirs = t(lambda: ref.ref_softmax(x.data_ptr(), y.data_ptr(), 4096, 1024), iters) if ref else None
    row("softmax 4096x1024", bytes_=2 * x.numel() * 4, ours=ours, theirs=theirs)

    g.manual_seed(2)
    x = torch.randn(4096, 2048, generator=g).cuda()
    gam = (0.5 + torch.rand(2048, generator=g)).cuda()
    bet = (0.1 * torch.randn(2048, generator=g)).cuda()
    y = torch.empty_like(x)
    ours = t(lambda: ops.layer_norm(x, y, gam, bet, 4096, 2048, 1e-5, 0), iters)
    theirs = (t(lambda: ref.ref_layer_norm(x.data_ptr(), y.data_ptr(), gam.data_ptr(), bet.data_ptr(), 4096, 2048,
                                           1e-5), iters) if ref else None)
    row("layer_norm 4096x2048", bytes_=2 * x.numel() * 4, ours=ours, theirs=theirs)

    g.manual_seed(3)
    M, N, K = 1024, 2048, 1024
    A = (torch.randn(M, N, generator=g) / np.sqrt(2048)).cuda()
    B = (torch.randn(N, K, generator=g) / np.sqrt(2048)).cuda()
    C = torch.empty(M, K, device="cuda")
    ours = t(lambda: ops.mat_mul(A, B, C, M, N, K, 1, 0.0, 0), iters)
    theirs = t(lambda: ref.ref_mat_mul_relu(A.data_ptr(), B.data_ptr(), C.data_ptr(), M, N, K), iters) if ref else None
    row("mat_mul 1024x2048x1024 + ReLU (3xTF32)", flops=2 * M * N * K, ours=ours, theirs=theirs)

    g.manual_seed(4)
    n = 1 << 24
    x = (torch.rand(n, generator=g) * 2 - 1).cuda()
    o = torch.empty(1, device="cuda")
    ws = torch.empty(max(1, ops.lib.opw_reduction_workspace_size(n)), device="cuda")
    ours = t(lambda: ops.reduce(0, x, o, n, ws, ws.numel(), 0), iters)
    # the reference's allocation-free overload with its own workspace size
    # (its convenience overload allocates and frees scratch on every call)
    theirs = None
    if ref:
        rws = torch.empty(max(1, ref.ref_reduction_workspace_size(n)), device="cuda")
        theirs = t(lambda: ref.ref_reduce_sum_ws(x.data_ptr(), o.data_ptr(), n, rws.data_ptr(), rws.numel()), iters)
    row("reduce sum 2^24", bytes_=n * 4, ours=ours, theirs=theirs)
    return {"peak_source": src, "hbm_gbs": hbm, "bf16_tflops": tc, "ops": out}


def decode(only="all", iters=20):
    """C3 decode-step kernels: paged decode attention (32 seqs x ctx 2176, 8 KV
    heads), bf16x2 GEMMs with 32 token rows, fused sampler (32 x 128256)."""
    import torch

    import opworks_b200

    ops = opworks_b200.ops_lib()
    hbm, _, _ = measured_peaks()
    t = Timer(torch)
    res = {}
    if only in ("all", "attention"):
        B, ctx, kvh, qh = 32, 2176, 8, 32
        bps = (ctx + 15) // 16
        nblk = B * bps
        g = torch.Generator(device="cuda")
        g.manual_seed(11)
        k = torch.randn(nblk, kvh, 16, 64, device="cuda", generator=g)
        v = torch.randn(nblk, kvh, 16, 64, device="cuda", generator=g)
        table = torch.randperm(nblk, device="cuda", generator=g).int().view(B, bps)
        lens = torch.full((B,), ctx, dtype=torch.int32, device="cuda")
        q = torch.randn(B, qh * 64, device="cuda", generator=g)
        out = torch.empty_like(q)
        ms = t(lambda: ops.paged_attention_decode(q, k, v, table, bps, lens, B, ctx, qh, kvh, out, 0), iters)
        b = B * ctx * kvh * 64 * 4 * 2
        res["attention"] = {"us": round(ms * 1e3, 1), "bytes": b, "gbs": round(b / ms / 1e6, 1),
                            "frac_hbm": round(b / ms / 1e6 / hbm, 4)}
    if only in ("all", "gemm"):
        raw = ops.raw("gemm_bf16x2")
        res["gemm"] = []
        for N, K in [(3072, 2048), (2048, 2048), (16384, 2048), (2048, 8192), (128256, 2048)]:
            M = 32
            W = torch.randn(N, K, device="cuda").to(torch.bfloat16)
            xh = torch.randn(M, K, device="cuda").to(torch.bfloat16)
            xl = (torch.randn(M, K, device="cuda") * 1e-3).to(torch.bfloat16)
            o = torch.empty(64 * M * N, device="cuda")
            used = [0]

            def f():
                used[0] = raw(W.view(torch.int16), xh.view(torch.int16), xl.view(torch.int16), o, N, K, M, 0, 0)

            ms = t(f, iters)
            b = N * K * 2
            res["gemm"].append({"N": N, "K": K, "M": M, "splits": used[0], "us": round(ms * 1e3, 1),
                                "weight_gbs": round(b / ms / 1e6, 1)})
    if only in ("all", "sample"):
        rows, V = 32, 128256
        g = torch.Generator(device="cuda")
        g.manual_seed(12)
        lg = torch.randn(rows, V, device="cuda", generator=g)
        tt = torch.full((rows,), 0.7, device="cuda")
        pp = torch.full((rows,), 0.9, device="cuda")
        u = torch.rand(rows, dtype=torch.float64, device="cuda", generator=g)
        o = torch.empty(rows, dtype=torch.int32, device="cuda")
        ms = t(lambda: ops.sample(lg, rows, V, tt, pp, u, o, 0), iters)
        res["sample"] = {"rows": rows, "vocab": V, "us": round(ms * 1e3, 1)}
    return res


def pair(M=8192, iters=10):
    """Two-SM GEMM (the prefill projections' kernel) at the C4 shapes: M
    token rows against the QKV, O, gate/up and down weights, with two
    activation terms (16-bit weights x hi + lo; the tensor cores execute
    twice the useful 2*M*N*K) and with one fp16 term. TFLOP/s counts the
    useful 2*M*N*K."""
    import torch

    import opworks_b200

    ops = opworks_b200.ops_lib()
    _, tc, src = measured_peaks()
    t = Timer(torch)
    raw = ops.raw("gemm_bf16x2_pair")
    res = []
    for name, N, K in [("qkv", 3072, 2048), ("o", 2048, 2048), ("gate_up", 16384, 2048), ("down", 2048, 8192)]:
        W = (torch.randn(N, K, device="cuda") / K**0.5).to(torch.bfloat16)
        x = torch.randn(M, K, device="cuda")
        xh = x.to(torch.bfloat16)
        xl = (x - xh.float()).to(torch.bfloat16)
        o = torch.empty(M, N, device="cuda")
        ms = t(lambda: raw(W.view(torch.int16), xh.view(torch.int16), xl.view(torch.int16), o, N, K, M, 0), iters)
        W16, x16 = W.float().to(torch.float16), x.to(torch.float16)
        ms1 = t(lambda: ops.raw("gemm_f16x2_pair")(W16.view(torch.int16), x16.view(torch.int16), 0, o, N, K, M, 0),
                iters)
        f = 2.0 * M * N * K
        res.append({"gemm": name, "M": M, "N": N, "K": K, "us": round(ms * 1e3, 1),
                    "useful_tflops": round(f / ms / 1e9, 1), "mma_frac_of_bf16_peak": round(2 * f / ms / 1e9 / tc, 3),
                    "one_term_us": round(ms1 * 1e3, 1), "one_term_tflops": round(f / ms1 / 1e9, 1),
                    "one_term_frac_of_bf16_peak": round(f / ms1 / 1e9 / tc, 3)})
    return {"peak_source": src, "bf16_tflops": tc, "gemms": res}


def tf32_peak(n=8192, burst_iters=10, sustain_s=3.0):
    """Measured TF32 tensor-core peak (the denominator for this library's
    TF32 kernels: prefill attention, split-TF32 GEMMs): torch.matmul of n^3
    fp32 with TF32 allowed (cuBLAS), best of `burst_iters` (burst) and back
    to back for `sustain_s` seconds (sustained), 2 n^3 flops each."""
    import torch

    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = True
    try:
        a = torch.randn(n, n, device="cuda")
        b = torch.randn(n, n, device="cuda")
        c = torch.empty(n, n, device="cuda")
        for _ in range(3):
            torch.matmul(a, b, out=c)
        torch.cuda.synchronize()
        best = float("inf")
        for _ in range(burst_iters):
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            torch.matmul(a, b, out=c)
            e.record()
            torch.cuda.synchronize()
            best = min(best, s.elapsed_time(e))
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = max(1, int(sustain_s * 1e3 / best))
        s.record()
        for _ in range(reps):
            torch.matmul(a, b, out=c)
        e.record()
        torch.cuda.synchronize()
        flop = 2.0 * n ** 3
        return {"tf32_tflops": round(flop / best / 1e9, 1),
                "tf32_tflops_sustained": round(flop * reps / s.elapsed_time(e) / 1e9, 1),
                "how": f"torch.matmul fp32 {n}^3 with allow_tf32 (cuBLAS): best of {burst_iters}, and {reps} back to back"}
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


def prefill(T=8192, iters=2):
    """Config C4: one T-token prefill of the random-init Llama-3.2-1B on the
    fast path (tensor-core GEMMs and attention), CUDA events on the engine
    stream; returns ms and tokens/s."""
    import torch

    from opworks_b200 import pack
    from opworks_b200.llama import LlamaBatch, Model

    path = pack.ensure_random_llama_pack()
    with Model(path, weight_sets=1, max_positions=max(8192, T)) as m, LlamaBatch(m, 1, T, "fast", prefill_rows=T) as eng:
        ids = np.random.default_rng(8).integers(0, m.vocab, T).astype(np.int32)
        eng.prefill(0, ids[:512])  # warm: module loads
        st = torch.cuda.ExternalStream(eng.stream())
        times = []
        for _ in range(iters):
            eng.reset(0)
            torch.cuda.synchronize()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record(st)
            eng.prefill(0, ids)
            b.record(st)
            torch.cuda.synchronize()
            times.append(a.elapsed_time(b))
    ms = float(min(times))
    return {"tokens": T, "ms": round(ms, 2), "tok_s": round(T / (ms / 1e3), 1)}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["c1", "decode", "prefill", "pair"])
    ap.add_argument("--tokens", type=int, default=8192)
    ap.add_argument("--only", default="all", choices=["all", "attention", "gemm", "sample"])
    ap.add_argument("--iters", type=int, default=20)
    a = ap.parse_args()
    if a.what == "c1":
        r = c1(a.iters)
    elif a.what == "prefill":
        r = prefill(a.tokens, max(1, min(a.iters, 3)))
    elif a.what == "pair":
        r = pair(a.tokens, a.iters)
    else:
        r = decode(a.only, a.iters)
    print(json.dumps(r))


if __name__ == "__main__":
    main()
