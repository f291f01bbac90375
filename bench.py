#!/usr/bin/env python3
"""Llama-3.2-1B (random-init) batch-32 decode at context 2048 on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

Workload (one batch per GPU, request-partitioned so
N GPUs run N independent batches with no collective on the data path):
  * weights: OPWPACK1 float32 pack, N(0, 0.02) projections / embedding,
    RMSNorm gains 1.0, tied LM head (generated once per box under
    $OPWORKS_PACK_DIR, default /tmp/opworks_packs); the engine uses the fp16
    copy made at load (fast path), the fp32 KV cache is paged (16-token blocks)
  * 32 sequences per GPU, each prefilled with 2048 uniform random token ids
  * W warm-up + K timed decode steps, every sequence sampling with T = 0.7,
    top-p = 0.9 on the device (seeded counter RNG); a step = one batched
    forward of 32 tokens through libopworks_llama.so's opw_llama_batch_decode

Reported (one JSON line from rank 0):
  value      decode tokens/s over all GPUs, device time (CUDA events on the
             engine stream around the K steps, max over ranks)
  e2e        same metric by host wall clock around the K C-ABI calls, host
             token buffers in and out (H2D/D2H inside the timed region)
  roofline   the dominant kernel of a decode step (CUDA-event time of each
             kernel group while re-running the last step), algorithmic bytes
             / time against the measured HBM copy bandwidth
  cpu_baseline  the C++ oracle's batched decode step on the host cores
             (bounded sample: a few steps), rank 0 at N = 1
  prefill    C3 prefill (32 x 2048 tokens) and C4 (one 8192-token prompt)
  c5         config C5 serving at this N: 256 requests partitioned over the
             ranks (strong scaling: total generated tok/s, per-rank busy time)
  c2_session C2 through the 11-symbol session ABI (our library and the
             reference's, float32 and bfloat16 packs)
`--impl reference` times the reference algorithm's CPU restatement (the
OpWorks reference has no CPU path of its own) on the same workload.
"""

from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time

import numpy as np

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

BATCH = 32
CTX = 2048
TEMPERATURE = 0.7
TOP_P = 0.9
METRIC = "Llama-3.2-1B decode tok/s (bs32, ctx2k)"
UNIT = "tok/s"


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=252)
    ap.add_argument("--warmup", type=int, default=4)
    ap.add_argument("--impl", choices=["ours", "reference"], default="ours")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill-8k", action="store_true")
    ap.add_argument("--no-extras", action="store_true", help="skip the C1 operator and reference-CUDA sections")
    ap.add_argument("--batch", type=int, default=BATCH, help="sequences per GPU (C3: 32; smaller for profiling)")
    ap.add_argument("--ctx", type=int, default=CTX, help="prefilled context (C3: 2048; smaller for profiling)")
    ap.add_argument("--profile-iters", type=int, default=3)
    ap.add_argument("--parallel", choices=["rp", "tp"], default="rp",
                    help="rp: request-partitioned replicas (default, weak scaling); tp: one tensor-parallel engine "
                         "over all ranks (global batch fixed, strong scaling)")
    ap.add_argument("--tp-reduce", choices=["nccl", "p2p"], default="p2p",
                    help="--parallel tp: NCCL all-reduce, or peer stores from the GEMM epilogue + rank-order sum")
    ap.add_argument("--workload", choices=["c3", "c5"], default="c3",
                    help="c3: batched decode (default, the headline); c5: 256-request serving, "
                         "request-partitioned over the ranks")
    ap.add_argument("--c5-max-batch", type=int, default=64, help="KV slots per GPU for c5 continuous batching")
    ap.add_argument("--no-c5", action="store_true", help="skip the C5 serving block of the c3 line")
    return ap.parse_args()


def measured_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 100 ms."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index):
        self.gpu = gpu_index
        self.rows = []
        self.proc = None
        self.thread = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", "-i", str(self.gpu), f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "100"], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        self.thread = threading.Thread(target=self._read, daemon=True)
        self.thread.start()

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) >= 9:
                self.rows.append(parts)

    def stop(self):
        if self.proc:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()
        if self.thread:
            self.thread.join(timeout=5)

    def summary(self):
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"], "samples": 0}
        sm = [float(r[1]) for r in self.rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in self.rows if r[2].replace(".", "").isdigit()]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in self.rows for i in range(4) if r[5 + i].lower() == "active"})
        power = [float(r[3]) for r in self.rows if r[3].replace(".", "").isdigit()]
        return {"sm_mhz": float(np.median(sm)) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(self.rows), "power_w_max": max(power) if power else None}


def algorithmic_bytes(label, cfg, batch, ctx_mean):
    """Minimal HBM bytes of one decode step's kernel group (all launches)."""
    L, H, I, V = cfg["layers"], cfg["hidden"], cfg["intermediate"], cfg["vocab"]
    qw, kvw = cfg["q_heads"] * cfg["head_dim"], cfg["kv_heads"] * cfg["head_dim"]
    act = lambda n: batch * n
    table = {
        "gemm_qkv": L * ((qw + 2 * kvw) * H * 2 + act(H) * 2 + act(qw + 2 * kvw) * 4),
        "gemm_o": L * (H * qw * 2 + act(qw) * 2 + act(H) * 4),
        "gemm_gate_up": L * (2 * I * H * 2 + act(H) * 2 + act(2 * I) * 4),
        "gemm_down": L * (H * I * 2 + act(I) * 2 + act(H) * 4),
        # fused fast path: 16-bit weights, two-term 16-bit activations in (4 bytes
        # per element), fused epilogue traffic out
        "gemm_qkv_rope_kv_write": L * ((qw + 2 * kvw) * H * 2 + act(H) * 4 + act(qw + 2 * kvw) * 4),
        # residual epilogues: hidden read + write, next operand h * gain out
        "gemm_o_residual": L * (H * qw * 2 + act(qw) * 4 + act(H) * 12),
        "gemm_gate_up_silu": L * (2 * I * H * 2 + act(H) * 4 + act(I) * 4),
        "gemm_down_residual": L * (H * I * 2 + act(I) * 4 + act(H) * 12),
        "attention": L * (batch * ctx_mean * kvw * 4 * 2 + act(qw) * 4 + act(qw) * 2),
        "lm_head": V * H * 2 + act(H) * 4 + act(V) * 4,
    }
    return table.get(label)


def step_bytes(cfg, batch, ctx_mean):
    tot = 0
    for lab in ("gemm_qkv_rope_kv_write", "gemm_o_residual", "gemm_gate_up_silu", "gemm_down_residual", "attention",
                "lm_head"):
        tot += algorithmic_bytes(lab, cfg, batch, ctx_mean)
    return tot


def scaled_traffic(label, tr, batch, ctx, kv_share=1.0):
    """DRAM bytes per launch from an ncu capture (profiles/traffic.json),
    scaled to this launch by the units it processes: attention traffic grows
    with batch x context x the KV heads this GPU holds (kv_share of them), a
    GEMM's does not change."""
    if not isinstance(tr, dict) or "dram_bytes_per_launch" not in tr:
        return None
    b = float(tr["dram_bytes_per_launch"])
    if label == "attention":
        b *= (batch * ctx) / float(tr["batch"] * tr["ctx"]) * kv_share
    elif kv_share != 1.0:
        return None  # the capture holds the full weight matrices
    return int(b)


def load_traffic():
    p = os.path.join(ROOT, "profiles", "traffic.json")
    if os.path.exists(p):
        with open(p) as f:
            return json.load(f)
    return {}


# ----------------------------------------------------------------- our arm


def _kernel_group(name, prev_group):
    """Kernel group of one launch of a decode step, from its (demangled) name."""
    if "embed" in name:
        return "embed_rmsnorm"
    if "attn" in name:
        return "attention"
    if "QkvTile" in name:
        return "gemm_qkv_rope_kv_write"
    if "SiluMulTile" in name:
        return "gemm_gate_up_silu"
    if "ResidualTile" in name:  # O right after attention, down after gate/up
        return "gemm_o_residual" if prev_group == "attention" else "gemm_down_residual"
    if "LogitsTile" in name:
        return "lm_head"
    if "sample" in name:
        return "sample"
    return name.split("(")[0][-40:]


def in_graph_kernel_times(step_fn, steps=3):
    """Per-group device time of the last of `steps` graph-replayed decode
    steps, from a CUPTI kernel trace (torch.profiler). With programmatic
    dependent launch a kernel starts before its predecessor ends and waits
    inside, so each launch is charged from the later of its own start and the
    previous launch's end to its own end: the charges add up to the step's
    span. Returns [{kernel, ms_per_step, launches_per_step}] and the span."""
    import torch
    from torch.profiler import ProfilerActivity, profile

    torch.cuda.synchronize()
    with profile(activities=[ProfilerActivity.CUDA]) as prof:
        for _ in range(steps):
            step_fn()
        torch.cuda.synchronize()
    ev = sorted((e for e in prof.events() if e.device_type == torch.autograd.DeviceType.CUDA
                 and e.name and "Memcpy" not in e.name and "Memset" not in e.name),
                key=lambda e: e.time_range.start)
    starts = [i for i, e in enumerate(ev) if "embed" in e.name]
    if not starts:
        return None
    last = ev[starts[-1]:]
    rows, order, prev_end, prev_group = {}, [], None, None
    for e in last:
        g = _kernel_group(e.name, prev_group)
        t0, t1 = e.time_range.start, e.time_range.end
        charge = t1 - (max(t0, prev_end) if prev_end is not None else t0)
        if g not in rows:
            rows[g] = [0.0, 0]
            order.append(g)
        rows[g][0] += max(charge, 0.0) / 1e3
        rows[g][1] += 1
        prev_end = t1 if prev_end is None else max(prev_end, t1)
        prev_group = g
    span_ms = (prev_end - last[0].time_range.start) / 1e3
    return {"span_ms": round(span_ms, 4),
            "timing": "CUPTI kernel trace of the graph-replayed step; each launch charged from max(its start, "
                      "previous launch end) to its end (programmatic-launch overlap counted once)",
            "groups": [{"kernel": g, "ms_per_step": round(rows[g][0], 4), "launches_per_step": rows[g][1]}
                       for g in order]}


def run_ours(args):
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))

    def barrier():
        if world > 1:
            dist.barrier()

    def allmax(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    from opworks_b200 import pack
    from opworks_b200.llama import LlamaBatch, Model

    if rank == 0:
        pack_path = pack.ensure_random_llama_pack()
    barrier()
    pack_path = pack.ensure_random_llama_pack()  # cached path on every rank

    K, W = args.steps, args.warmup
    MULTI = 64  # extra steps of the host-sync-free multi-step decode (extras)
    # positions: W warm-up steps, 1 or K (warm multi-step), K (timed), K
    # (e2e), 3 (in-graph trace), MULTI (extras), 1 spare
    max_seq = ((CTX + W + 3 * K + 3 + MULTI + 1 + 15) // 16) * 16
    t_load = time.perf_counter()
    model = Model(pack_path, weight_sets=1, max_positions=max(8192, max_seq), device=local)
    t_load = time.perf_counter() - t_load
    cfg = {"layers": model.layers, "hidden": model.hidden, "intermediate": model.intermediate,
           "q_heads": model.q_heads, "kv_heads": model.kv_heads, "head_dim": model.head_dim, "vocab": model.vocab}
    tp = args.parallel == "tp" and world > 1
    # bytes this GPU moves: a tensor-parallel rank holds 1 / world of the
    # heads and MLP columns (embedding and LM head stay whole)
    rcfg = dict(cfg)
    if tp:
        for key in ("q_heads", "kv_heads", "intermediate"):
            rcfg[key] = cfg[key] // world
    if tp:
        from opworks_b200.llama import nccl_unique_id

        box = [nccl_unique_id() if rank == 0 else None]
        dist.broadcast_object_list(box, src=0)
        eng = LlamaBatch(model, BATCH, max_seq, "fast", prefill_rows=CTX, tp=(rank, world, box[0]))
        if args.tp_reduce == "p2p":
            handles = [None] * world
            dist.all_gather_object(handles, eng.tp_ipc_handle())
            eng.tp_open_peers(handles)
    else:
        eng = LlamaBatch(model, BATCH, max_seq, "fast", prefill_rows=CTX)
    shard = 0 if tp else rank  # tensor-parallel ranks serve the same sequences
    stream = torch.cuda.ExternalStream(eng.stream())

    rng = np.random.default_rng(6 + 1000 * shard)
    prompts = rng.integers(0, model.vocab, (BATCH, CTX)).astype(np.int32)
    seeds = (7_000 + np.arange(BATCH) + 1_000_000 * shard).astype(np.uint64)
    slots = np.arange(BATCH, dtype=np.int32)

    # ---- prefill (C3: 32 x 2048 tokens), timed on the engine stream
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    prev = np.array([eng.prefill(int(s), prompts[s], TEMPERATURE, TOP_P, -1.0, int(seeds[s])) for s in slots],
                    np.int32)
    e1.record(stream)
    torch.cuda.synchronize()
    prefill_ms = allmax(e0.elapsed_time(e1))

    step = 1

    def decode_once():
        nonlocal prev, step
        prev = eng.decode(slots, prev, temperature=TEMPERATURE, top_p=TOP_P, seeds=seeds, steps=step)
        step += 1

    # `value`: K steps with every step's sampled tokens fed back on the device
    # (one opw_llama_batch_decode_multi call: K replays of the step graph, the
    # sampler writing each row's next inputs, inputs resident, one D2H of the
    # K x 32 tokens at the end). Tensor-parallel runs keep the per-step call.
    multi_value = not tp

    def decode_k(k=K):
        nonlocal prev, step
        toks, _ = eng.decode_multi(slots, prev, k, temperature=TEMPERATURE, top_p=TOP_P, seeds=seeds, steps0=step)
        prev = toks[-1]
        step += k

    for _ in range(W):
        decode_once()
    if multi_value:
        # warm: the multi-step graph is captured here (one graph serves calls
        # of up to 256 steps; longer calls regrow its buffers once)
        decode_k(1 if K <= 256 else K)
    torch.cuda.synchronize()

    clocks = ClockSampler(local if "CUDA_VISIBLE_DEVICES" not in os.environ else local)
    clocks.start()
    time.sleep(0.3)  # let the sampler attach before the timed region
    barrier()
    torch.cuda.synchronize()
    s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    ctx0 = step - 1  # positions decoded after the prefill so far
    if multi_value:
        # a ~0.5 ms device spin ahead of the start event: the host's enqueue
        # of the timed call (input staging, K graph launches) lands before
        # the GPU reaches it, so the events bracket device work only
        with torch.cuda.stream(stream):
            torch.cuda._sleep(1_000_000)
    s0.record(stream)
    if multi_value:
        decode_k()
    else:
        for _ in range(K):
            decode_once()
    s1.record(stream)
    torch.cuda.synchronize()
    barrier()
    dev_ms = allmax(s0.elapsed_time(s1))
    # e2e: the public per-step call (H2D of the step's tokens and sampling
    # inputs, graph replay, D2H of the sampled tokens, blocking), host clock
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    for _ in range(K):
        decode_once()
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    clocks.stop()
    barrier()
    wall = allmax(wall)

    ctx_mean = CTX + ctx0 + K / 2.0
    groups = 1 if tp else world  # independent sequence groups across the ranks
    value = BATCH * K * groups / (dev_ms / 1e3)
    e2e_value = BATCH * K * groups / wall
    h2d, d2h = eng.io_bytes(BATCH)

    # ---- per-kernel device time of the last step (roofline)
    kernels = eng.profile(BATCH, args.profile_iters)
    ctx_prof = CTX + step - 1  # context of the profiled step
    kernels_in_graph = in_graph_kernel_times(decode_once)
    if kernels_in_graph is not None:
        for g in kernels_in_graph["groups"]:
            b = algorithmic_bytes(g["kernel"], rcfg, BATCH, CTX + step - 1)  # after the traced steps
            g["gbs"] = round(b / (g["ms_per_step"] / 1e3) / 1e9, 1) if b and g["ms_per_step"] > 0 else None

    # ---- host-sync-free multi-step decode (extras): MULTI more steps in
    # chunks of 16 graph replays with device-side token feedback, host clock
    multi = None
    if not args.no_extras:
        chunk = 16

        def multi_chunk():
            nonlocal prev, step
            toks, _ = eng.decode_multi(slots, prev, chunk, temperature=TEMPERATURE, top_p=TOP_P, seeds=seeds,
                                       steps0=step)
            prev = toks[-1]
            step += chunk

        multi_chunk()  # warm: the 16-step graph is captured here
        torch.cuda.synchronize()
        t0m = time.perf_counter()
        for _ in range(MULTI // chunk - 1):
            multi_chunk()
        wall_m = allmax(time.perf_counter() - t0m)
        n_m = (MULTI // chunk - 1) * chunk
        multi = {"value": round(BATCH * n_m * groups / wall_m, 1), "unit": UNIT, "steps": n_m, "chunk": chunk,
                 "timing": "host wall clock around opw_llama_batch_decode_multi calls (one H2D before and one "
                           "D2H after each chunk)"}
    hbm_peak, tc_peak, peak_src = measured_peaks()
    ctx_now = ctx_prof
    traffic = load_traffic()
    rows = []
    for label, ms, launches in kernels:
        b = algorithmic_bytes(label, rcfg, BATCH, ctx_now)
        rows.append({"kernel": label, "ms_per_step": round(ms, 4), "launches_per_step": launches,
                     "gbs": round(b / (ms / 1e3) / 1e9, 1) if b and ms > 0 else None})
    # launch groups: attention = split-KV partial (+ combine kernel when the
    # KV range is split: fewer (sequence, kv head) pairs than 2 CTAs per SM)
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    attn_kernels = 1 if (2 * sms) // (BATCH * cfg["kv_heads"]) <= 1 else 2
    gpu_launches_per_step = sum(k[2] * (attn_kernels if k[0] == "attention" else 1) for k in kernels)
    dom = max((r for r in rows if r["gbs"] is not None), key=lambda r: r["ms_per_step"])
    dom_bytes = algorithmic_bytes(dom["kernel"], rcfg, BATCH, ctx_now) / dom["launches_per_step"]
    dom_ms = dom["ms_per_step"] / dom["launches_per_step"]
    achieved = dom_bytes / (dom_ms / 1e3) / 1e9
    tr = traffic.get(dom["kernel"])
    roofline = {"bound": "hbm", "kernel": dom["kernel"], "achieved": round(achieved, 1), "peak": hbm_peak,
                "unit": "GB/s", "frac": round(achieved / hbm_peak, 4),
                "traffic": scaled_traffic(dom["kernel"], tr, BATCH, ctx_now, rcfg["kv_heads"] / cfg["kv_heads"]),
                "algorithmic_bytes_per_launch": int(dom_bytes), "avg_launch_ms": round(dom_ms, 5),
                "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"}
    sb = step_bytes(rcfg, BATCH, ctx_mean)
    step_roofline = {"bytes_per_step": int(sb), "achieved_gbs": round(sb / (dev_ms / K / 1e3) / 1e9, 1),
                     "frac_of_hbm": round(sb / (dev_ms / K / 1e3) / 1e9 / hbm_peak, 4)}

    # ---- C4: one 8192-token prefill (rank 0 at N = 1)
    prefill8k = None
    if not args.no_prefill_8k and world == 1:
        eng8 = LlamaBatch(model, 1, 8192, "fast", prefill_rows=8192)
        ids8 = np.random.default_rng(8).integers(0, model.vocab, 8192).astype(np.int32)
        eng8.prefill(0, ids8[:512])  # warm (module loads)
        eng8.reset(0)
        st8 = torch.cuda.ExternalStream(eng8.stream())
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(st8)
        eng8.prefill(0, ids8)
        b.record(st8)
        torch.cuda.synchronize()
        ms8 = a.elapsed_time(b)
        gemm_flop = 8192 * 2 * (model.layers * (model.hidden * (model.q_heads + 2 * model.kv_heads) * model.head_dim
                                                + model.hidden * model.q_heads * model.head_dim
                                                + 3 * model.hidden * model.intermediate))
        attn_flop = 4 * model.q_heads * model.head_dim * (8192 * 8193 / 2) * model.layers
        prefill8k = {"tokens": 8192, "ms": round(ms8, 2), "tok_s": round(8192 / (ms8 / 1e3), 1),
                     "tflops_useful": round((gemm_flop + attn_flop) / (ms8 / 1e3) / 1e12, 1),
                     "frac_of_bf16_peak": round((gemm_flop + attn_flop) / (ms8 / 1e3) / 1e12 / tc_peak, 4),
                     "gemm_tflop": round(gemm_flop / 1e12, 2), "attention_tflop": round(attn_flop / 1e12, 2)}
        eng8.close()

    # ---- C5: 256-request serving, strong scaling over the ranks (every
    # rank; request-partitioned, no collective on the data path)
    c5 = None
    if not args.no_c5 and not tp:
        c5 = c5_serve(model, args, rank, world, torch.device("cuda", local))

    # ---- C2: batch 1, 128-token prompt, then greedy decode (fast path, our
    # batched ABI with one slot; host wall clock per blocking call)
    c2 = None
    if world == 1 and not args.no_extras:
        with LlamaBatch(model, 1, 128 + 128 + 8, "fast", prefill_rows=128) as e2:
            ids2 = np.random.default_rng(5).integers(0, model.vocab, 128).astype(np.int32)
            e2.prefill(0, ids2)  # warm: module loads and graph capture happen here
            e2.decode([0], [0])
            e2.reset(0)
            t = time.perf_counter()
            tok = e2.prefill(0, ids2)
            ttft = time.perf_counter() - t
            t = time.perf_counter()
            for _ in range(128):
                tok = int(e2.decode([0], [tok])[0])
            dec = time.perf_counter() - t
        c2 = {"prompt": 128, "ttft_ms": round(ttft * 1e3, 2), "decode_steps": 128,
              "decode_tok_s": round(128 / dec, 1), "precision": "fast (fp16 weights)",
              "timing": "host wall clock per blocking call"}

    # ---- C1 operator configs, ours and the reference's kernels (rank 0, N = 1)
    c1 = None
    if world == 1 and not args.no_extras:
        from opworks_b200 import microbench

        c1 = microbench.c1(iters=10)
        # the TF32 denominator: prefill attention and the split-TF32 mat_mul
        c1["tf32_peak"] = microbench.tf32_peak()
        tf = c1["tf32_peak"]["tf32_tflops"]
        for op in c1.get("ops", []):
            if "ours_tflops" in op:
                op["ours_frac_tf32_peak"] = round(op["ours_tflops"] / tf, 4)
                op["tf32_mma_frac_of_tf32_peak"] = round(3 * op["ours_tflops"] / tf, 4)  # 3 MMAs per K step

    cpu = None
    ref_cuda = None
    c2_session = None
    if rank == 0 and world == 1:
        eng.close()
        model.close()
        if not args.no_extras:
            ref_cuda = reference_cuda_path(pack_path)
            c2_session = session_c2_block(pack_path)
        if not args.no_cpu_baseline:
            cpu = cpu_baseline(pack_path)
            if not args.no_extras:
                cpu["other_configs"] = cpu_extras(pack_path)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 1), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
            "ms_per_step": round(dev_ms / K, 4), "higher_is_better": True, "scaling": "strong" if tp else "weak",
            "vs_baseline": None,
            "dtype": "f16",
            "data": "synthetic: random-init weights N(0,0.02) (norm gains 1.0), uniform random token ids",
            "config": {"workload": f"C3 batched decode: Llama-3.2-1B random-init, {BATCH} sequences per GPU "
                                   f"prefilled to {CTX} random ids, T=0.7 top-p=0.9 device sampling, fp32 paged KV "
                                   "(16-token blocks)",
                       "model": "Llama-3.2-1B (16 layers, 2048 hidden, 32/8 heads, 128256 vocab)",
                       "global_batch": BATCH * groups, "seq_len": CTX, "ctx_range": [CTX + ctx0, CTX + ctx0 + K],
                       "parallelism": (f"tp{world}: tensor-parallel heads / MLP columns, "
                                       + ("NCCL all-reduce" if args.tp_reduce == "nccl" else
                                          "peer stores from the GEMM epilogue + rank-order sum")
                                       + " after o and down" if tp else
                                       f"request-partitioned x{world} (no collective)"),
                       "precision": "fp16 weights (rounded from the fp32 pack) and two-term fp16 GEMM operands, "
                                    "fp32 accumulation / residual / KV cache / attention / softmax, sampling fp64",
                       "l2": "inputs larger than L2: every step streams 2.47 GB of weights + ~4.5 GB of KV",
                       "cuda_graph": True,
                       "timed_step": ("K replays of the step graph in one decode_multi call, sampled tokens fed "
                                      "back on the device by the sampler, CUDA events on the engine stream"
                                      if multi_value else "K blocking per-step decode calls, CUDA events"),
                       "e2e_step": "K blocking opw_llama_batch_decode calls (H2D of the step's inputs, graph "
                                   "replay, D2H of the sampled tokens), host wall clock"},
            "roofline": roofline, "step_roofline": step_roofline,
            "e2e": {"value": round(e2e_value, 1), "unit": UNIT, "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "gpu_launches": gpu_launches_per_step * K, "gpu_launches_per_step": gpu_launches_per_step,
            "clocks": clocks.summary(),
            "prefill": {"c3_tokens": BATCH * CTX, "c3_ms": round(prefill_ms, 1),
                        "c3_tok_s": round(BATCH * CTX * groups / (prefill_ms / 1e3), 1), "c4": prefill8k},
            "kernels": rows,
            "kernels_timing": "CUDA events recorded between kernel groups inside the captured step; the event "
                              "nodes serialise the programmatic-launch overlap, so the groups add up to more "
                              "than the step (kernels_in_graph has the overlapped step)",
            "kernels_in_graph": kernels_in_graph, "load_s": round(t_load, 2),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        if c1 is not None:
            line["c1_ops"] = c1
        if c2 is not None:
            line["c2"] = c2
        if c5 is not None:
            line["c5"] = c5
        if multi is not None:
            line["multi_step_decode"] = multi
        if ref_cuda is not None:
            line["reference_cuda"] = ref_cuda
        if c2_session is not None:
            line["c2_session"] = c2_session
        print(json.dumps(line), flush=True)
    try:
        eng.close()
        model.close()
    except Exception:
        pass
    if world > 1:
        dist.destroy_process_group()


# ------------------------------------- the reference's own CUDA path (same GPU)

REF_LLAMA = os.path.join(ROOT, "oracle", "_ref", "libopworks_llama_ref.so")


def session_c2(lib, pack_path, steps=64, reps=3):
    """C2 through the reference's 11-symbol session ABI, timed the way the
    reference's scripts/llama/benchmark.py:53-68 times it: reset, prefill of
    a 128-token prompt (TTFT, host wall clock), then `steps` blocking
    decode_step calls (tokens/s); the median of `reps` repetitions. `lib` is
    a ctypes library with the ABI (ours or the reference's)."""
    import ctypes
    import statistics

    P, I, S = ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p
    for name, res, args in (("opw_llama_load", P, [S, S, I]), ("opw_llama_create_session", P, [P, I, S, I]),
                            ("opw_llama_reset_session", I, [P, S, I]),
                            ("opw_llama_prefill", ctypes.c_int32, [P, ctypes.POINTER(ctypes.c_int32), I, S, I]),
                            ("opw_llama_decode_step", ctypes.c_int32, [P, ctypes.c_int32, S, I]),
                            ("opw_llama_destroy_session", None, [P]), ("opw_llama_free", None, [P])):
        fn = getattr(lib, name)
        fn.restype, fn.argtypes = res, args
    err = ctypes.create_string_buffer(512)
    t = time.perf_counter()
    m = lib.opw_llama_load(pack_path.encode(), err, 512)
    load_s = time.perf_counter() - t
    if not m:
        return {"unavailable": err.value.decode(errors="replace")}
    prompt = np.random.default_rng(5).integers(0, 128256, 128).astype(np.int32)
    arr = (ctypes.c_int32 * 128)(*prompt.tolist())
    s = lib.opw_llama_create_session(m, 128 + steps + 8, err, 512)
    ttfts, rates = [], []
    try:
        for _ in range(reps + 1):  # the first repetition warms up
            lib.opw_llama_reset_session(s, err, 512)
            t0 = time.perf_counter()
            tok = lib.opw_llama_prefill(s, arr, 128, err, 512)
            t1 = time.perf_counter()
            for _ in range(steps):
                tok = lib.opw_llama_decode_step(s, tok, err, 512)
            t2 = time.perf_counter()
            if tok < 0:
                return {"unavailable": err.value.decode(errors="replace")}
            ttfts.append(t1 - t0)
            rates.append(steps / (t2 - t1))
    finally:
        lib.opw_llama_destroy_session(s)
        lib.opw_llama_free(m)
    return {"ttft_ms": round(statistics.median(ttfts[1:]) * 1e3, 2),
            "decode_tok_s": round(statistics.median(rates[1:]), 1), "load_s": round(load_s, 2),
            "prompt": 128, "decode_steps": steps, "reps": reps}


def session_c2_block(fp32_pack):
    """C2 via the session ABI: our library and the reference's, on the float32
    pack (our session default: the accurate fp32 path) and on a bfloat16 pack
    of the same draw (LlamaModelBF16: our fast path)."""
    import ctypes

    from opworks_b200 import llama, pack

    bf16_pack = pack.ensure_random_llama_pack(dtype="bfloat16")
    out = {"method": "reference scripts/llama/benchmark.py:53-68 (host wall clock, blocking calls), median of 3",
           "ours_fp32_pack": session_c2(llama.lib(), fp32_pack),
           "ours_bf16_pack": session_c2(llama.lib(), bf16_pack)}
    if os.path.exists(REF_LLAMA):
        ref = ctypes.CDLL(REF_LLAMA)
        out["reference_fp32_pack"] = session_c2(ref, fp32_pack)
        out["reference_bf16_pack"] = session_c2(ref, bf16_pack)
    return out


def reference_cuda_path(pack_path, c3_sessions=2, c3_steps=8, c2_steps=64):
    """The reference's CUDA library (built from its own sources into
    oracle/_ref) through its C ABI on the same GPU and pack: C2 (128-token
    prompt, then greedy decode, batch 1) and C3-style decode at context 2048.
    The reference has no batched decode: C3 serving is one session step after
    another (round robin), so its C3 throughput is one token per session
    step; it is measured on `c3_sessions` sessions and is the same for 32."""
    if not os.path.exists(REF_LLAMA):
        return None
    import ctypes

    lib = ctypes.CDLL(REF_LLAMA)
    lib.opw_llama_load.restype = ctypes.c_void_p
    lib.opw_llama_load.argtypes = [ctypes.c_char_p, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_create_session.restype = ctypes.c_void_p
    lib.opw_llama_create_session.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_prefill.restype = ctypes.c_int32
    lib.opw_llama_prefill.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_char_p,
                                      ctypes.c_int]
    lib.opw_llama_decode_step.restype = ctypes.c_int32
    lib.opw_llama_decode_step.argtypes = [ctypes.c_void_p, ctypes.c_int32, ctypes.c_char_p, ctypes.c_int]
    lib.opw_llama_destroy_session.argtypes = [ctypes.c_void_p]
    lib.opw_llama_free.argtypes = [ctypes.c_void_p]
    err = ctypes.create_string_buffer(512)
    m = lib.opw_llama_load(pack_path.encode(), err, 512)
    if not m:
        return {"unavailable": err.value.decode(errors="replace")}
    out = {"library": "oracle/_ref/libopworks_llama_ref.so (reference sources, unchanged, nvcc sm_100a)",
           "weights": "fp32 pack as loaded by the reference"}
    try:
        rng = np.random.default_rng(5)
        prompt = rng.integers(0, 128256, 128).astype(np.int32)
        s = lib.opw_llama_create_session(m, 128 + c2_steps + 8, err, 512)
        arr = (ctypes.c_int32 * len(prompt))(*prompt.tolist())
        t = time.perf_counter()
        tok = lib.opw_llama_prefill(s, arr, len(prompt), err, 512)
        ttft = time.perf_counter() - t
        t = time.perf_counter()
        for _ in range(c2_steps):
            tok = lib.opw_llama_decode_step(s, tok, err, 512)
        dec = time.perf_counter() - t
        lib.opw_llama_destroy_session(s)
        out["c2"] = {"prompt": 128, "ttft_ms": round(ttft * 1e3, 2), "decode_steps": c2_steps,
                     "decode_tok_s": round(c2_steps / dec, 1), "timing": "host wall clock per call (blocking ABI)"}
        sess, toks = [], []
        for i in range(c3_sessions):
            ids = np.random.default_rng(60 + i).integers(0, 128256, CTX).astype(np.int32)
            si = lib.opw_llama_create_session(m, CTX + c3_steps + 8, err, 512)
            a = (ctypes.c_int32 * CTX)(*ids.tolist())
            toks.append(lib.opw_llama_prefill(si, a, CTX, err, 512))
            sess.append(si)
        t = time.perf_counter()
        for _ in range(c3_steps):
            for i, si in enumerate(sess):
                toks[i] = lib.opw_llama_decode_step(si, toks[i], err, 512)
        dt = time.perf_counter() - t
        for si in sess:
            lib.opw_llama_destroy_session(si)
        out["c3"] = {"value": round(c3_sessions * c3_steps / dt, 1), "unit": UNIT,
                     "sample": f"{c3_sessions} sessions prefilled to {CTX}, {c3_steps} round-robin greedy decode "
                               "steps each (device sampling excluded: the reference samples on the host)"}
        # C4: one 8192-token prefill (create_session(8192), the reference's cap)
        ids8 = np.random.default_rng(8).integers(0, 128256, 8192).astype(np.int32)
        s8 = lib.opw_llama_create_session(m, 8192, err, 512)
        if s8:
            a8 = (ctypes.c_int32 * 8192)(*ids8.tolist())
            t = time.perf_counter()
            ok = lib.opw_llama_prefill(s8, a8, 8192, err, 512) >= 0
            dt8 = time.perf_counter() - t
            lib.opw_llama_destroy_session(s8)
            if ok:
                out["c4"] = {"tokens": 8192, "ms": round(dt8 * 1e3, 1), "tok_s": round(8192 / dt8, 1)}
    finally:
        lib.opw_llama_free(m)
    return out


# ------------------------------------------------- CPU arm (oracle port)


def _oracle_model(pack_path):
    import oracle
    from opworks_b200 import pack

    manifest, tensors = pack.read_pack(pack_path)
    return oracle.Llama(manifest["config"], tensors), manifest


def cpu_decode_steps(pack_path, batch, steps, warmup, ctx=CTX):
    """Batched decode steps of the C++ oracle: `batch` sequences at context
    `ctx` whose KV cache holds seeded random values (the cost of a decode step
    does not depend on the cached values). Returns (seconds per step, threads)."""
    import oracle

    m, _ = _oracle_model(pack_path)
    cap = ctx + warmup + steps + 1
    rng = np.random.default_rng(11)
    shape = (batch, m.L, m.kvh, cap, m.D)
    kc = rng.standard_normal(shape, dtype=np.float32)
    vc = rng.standard_normal(shape, dtype=np.float32)
    ids = rng.integers(0, m.V, batch).astype(np.int32)
    times = []
    for i in range(warmup + steps):
        pos = np.full(batch, ctx + i, np.int32)
        t = time.perf_counter()
        logits = m.decode_batch(ids, pos, kc, vc)
        if i >= warmup:
            times.append(time.perf_counter() - t)
        ids = logits.argmax(axis=1).astype(np.int32)
    return float(np.mean(times)), oracle.lib().orc_num_threads()


CPU_STEP_BUDGET_S = 1.5  # one CPU sample step: a batched decode step of at most this long


def cpu_sample_batch(pack_path):
    """Sequences per CPU sample step: all 32 of C3 unless one 32-sequence step
    (probed once) takes longer than CPU_STEP_BUDGET_S, then proportionally
    fewer. Returns (batch, probe seconds of the full step)."""
    probe, _ = cpu_decode_steps(pack_path, BATCH, 1, warmup=0)
    batch = BATCH if probe <= CPU_STEP_BUDGET_S else max(1, int(BATCH * CPU_STEP_BUDGET_S / probe))
    return batch, probe


def cpu_measure(pack_path, steps, warmup):
    """The one CPU measurement method of this file (the cpu_baseline leg and
    the --impl reference arm): `steps` timed batched decode steps of the
    oracle after `warmup` untimed ones, each step the sample of
    cpu_sample_batch at context 2048; value = sequences per step / seconds per
    step (tok/s)."""
    import oracle

    # every host thread this process may use: torchrun sets OMP_NUM_THREADS=1
    # for its ranks, and rank 0 runs this alone
    oracle.lib().orc_set_threads(len(os.sched_getaffinity(0)))
    batch, probe = cpu_sample_batch(pack_path)
    sec, threads = cpu_decode_steps(pack_path, batch, steps, warmup=warmup)
    return {"value": round(batch / sec, 3), "unit": UNIT, "cores": threads, "kind": "port",
            "sample": f"{steps} timed decode steps (after {warmup} untimed) of {batch} sequences at context {CTX}, "
                      f"random KV; C++/OpenMP restatement of the reference math; one 32-sequence step took "
                      f"{probe:.2f} s", "batch": batch, "sec_per_step": sec}


def cpu_extras(pack_path):
    """The CPU numbers reported beside the C3 one, on the host
    cores (the C++/OpenMP oracle, double accumulation): C1 operators timed in
    full; C2 = a 128-token prefill timed in full and 8 greedy decode steps
    (per token); C4 (8192-token prefill) extrapolated from the measured
    per-token projection cost and the measured causal-attention cost at 1024
    tokens scaled by (8192 / 1024)^2, labelled as such."""
    import oracle

    rng = np.random.default_rng(1)

    def timed(fn, reps=1):
        best = float("inf")
        for _ in range(reps):
            t = time.perf_counter()
            fn()
            best = min(best, time.perf_counter() - t)
        return best

    x = (rng.standard_normal((4096, 1024)) * 4).astype(np.float32)
    ln = rng.standard_normal((4096, 2048)).astype(np.float32)
    g, b = rng.uniform(0.5, 1.5, 2048).astype(np.float32), (rng.standard_normal(2048) * 0.1).astype(np.float32)
    A = (rng.standard_normal((1024, 2048)) / 2048 ** 0.5).astype(np.float32)
    B = (rng.standard_normal((2048, 1024)) / 2048 ** 0.5).astype(np.float32)
    s24 = rng.uniform(-1, 1, 1 << 24).astype(np.float32)
    c1 = {"softmax_4096x1024_ms": round(timed(lambda: oracle.softmax(x), 3) * 1e3, 2),
          "layer_norm_4096x2048_ms": round(timed(lambda: oracle.layer_norm(ln, g, b), 3) * 1e3, 2),
          "mat_mul_relu_1024x2048x1024_ms": round(timed(lambda: oracle.mat_mul(A, B, epilogue=1), 2) * 1e3, 2),
          "sum_2e24_ms": round(timed(lambda: oracle.reduce_sum(s24), 3) * 1e3, 2)}
    m, _ = _oracle_model(pack_path)
    prompt = np.random.default_rng(5).integers(0, m.V, 128).astype(np.int32)
    kc, vc = m.new_cache(128 + 9)
    t = time.perf_counter()
    logits = m.forward(prompt, 0, kc, vc)
    prefill_s = time.perf_counter() - t
    tok = oracle.argmax(logits)
    t = time.perf_counter()
    for k in range(8):
        tok = oracle.argmax(m.forward([tok], 128 + k, kc, vc))
    decode_s = (time.perf_counter() - t) / 8
    q = rng.standard_normal((1024, m.qh, m.D)).astype(np.float32)
    kv = rng.standard_normal((1024, m.kvh, m.D)).astype(np.float32)
    attn1k = timed(lambda: oracle.attention(q, kv, kv))
    per_tok = prefill_s / 128  # attention is < 1% of a 128-token prefill
    c4_s = per_tok * 8192 + attn1k * 64 * m.L
    return {"threads": oracle.lib().orc_num_threads(), "c1": c1,
            "c2": {"prefill_128_ms": round(prefill_s * 1e3, 1), "ttft_tok_s": round(128 / prefill_s, 1),
                   "decode_tok_s": round(1 / decode_s, 2), "decode_steps": 8},
            "c4_extrapolated": {"ms": round(c4_s * 1e3), "tok_s": round(8192 / c4_s, 1),
                                "method": "128-token prefill cost per token x 8192 + 1024-token causal attention "
                                          "x 64 x layers (extrapolated, not run)"}}


def cpu_baseline(pack_path, steps=6):
    out = cpu_measure(pack_path, steps, warmup=1)
    out.pop("batch")
    out["sec_per_step"] = round(out["sec_per_step"], 3)
    return out


def run_reference(args):
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    if rank != 0:
        return
    from opworks_b200 import pack

    pack_path = pack.ensure_random_llama_pack()
    K, W = args.steps, args.warmup
    # the same sample step as the cpu_baseline leg of our arm (cpu_measure)
    m = cpu_measure(pack_path, K, W)
    batch, sec, threads, value = m["batch"], m["sec_per_step"], m["cores"], m["value"]
    line = {
        "metric": METRIC, "value": round(value, 3), "unit": UNIT, "n_gpus": world, "steps": K, "warmup": W,
        "ms_per_step": round(sec * 1e3, 2), "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
        "dtype": "fp32", "impl": "reference",
        "data": "synthetic: random-init weights N(0,0.02), random token ids, random KV values",
        "config": {"workload": "C3 batched decode step on the host cores (reference algorithm restated in C++ / "
                               "OpenMP; OpWorks has no CPU path of its own)", "global_batch": batch,
                   "seq_len": CTX, "parallelism": "host threads"},
        "cpu_baseline": {"value": round(value, 3), "unit": UNIT, "cores": threads, "kind": "port",
                         "sample": m["sample"]},
        "e2e": {"value": round(value, 3), "unit": UNIT, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def c5_serve(model, args, rank, world, device_id):
    """Config C5 on an already loaded model: 256 requests (prompt lengths
    U[256, 1024], 256 sampled tokens each, T=0.7 top-p 0.9) split over the
    ranks by the deterministic LPT partition (opworks_b200/serving.py); every
    rank serves its share with continuous batching on its GPU, no collective
    on the data path. Timed on the device (CUDA events on each engine stream,
    max over ranks); returns (on every rank) the strong-scaling record: total
    generated tokens / that time, plus each rank's busy time."""
    import torch
    import torch.distributed as dist

    from opworks_b200 import serving
    from opworks_b200.llama import LlamaBatch

    reqs = serving.c5_requests()
    eng = LlamaBatch(model, args.c5_max_batch, 1024 + 256 + 16, "fast", prefill_rows=1024)
    stream = torch.cuda.ExternalStream(eng.stream())
    # warm-up: module loads and the decode graphs of every batch size used
    warm = [serving.Request(10_000 + i, list(range(300)), 2, 0.7, 0.9, i) for i in range(args.c5_max_batch)]
    serving.Server(eng, args.c5_max_batch).run(warm)
    for n in range(1, args.c5_max_batch + 1):
        eng.decode(list(range(n)), [0] * n, temperature=0.7, top_p=0.9)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    t0 = time.perf_counter()
    a.record(stream)
    server = serving.Server(eng, args.c5_max_batch)
    out = serving.serve_partitioned(reqs, rank, world, lambda: server, gather=False)
    b.record(stream)
    torch.cuda.synchronize()
    wall = time.perf_counter() - t0
    ms = a.elapsed_time(b)
    gen = sum(len(v) for v in out.values())
    my = [ms, float(gen), float(server.prefill_tokens)]
    busy = [my]
    if world > 1:
        t = torch.tensor(my, dtype=torch.float64, device=device_id)
        allt = [torch.zeros_like(t) for _ in range(world)]
        dist.all_gather(allt, t)
        busy = [x.tolist() for x in allt]
        w = torch.tensor([wall], dtype=torch.float64, device=device_id)
        dist.all_reduce(w, op=dist.ReduceOp.MAX)
        wall = float(w.item())
    eng.close()
    ms_max = max(r[0] for r in busy)
    gen = int(sum(r[1] for r in busy))
    pre = int(sum(r[2] for r in busy))
    return {"metric": "C5 serving: generated tok/s (256 requests, prompts U[256,1024], 256 new tokens)",
            "value": round(gen / (ms_max / 1e3), 1), "unit": UNIT, "n_gpus": world, "scaling": "strong",
            "ms": round(ms_max, 1), "wall_s": round(wall, 2), "generated_tokens": gen, "prefill_tokens": pre,
            "requests": len(reqs), "rank_busy_ms": [round(r[0], 1) for r in busy],
            "rank_generated_tokens": [int(r[1]) for r in busy],
            "config": {"max_batch_per_gpu": args.c5_max_batch,
                       "parallelism": f"request-partitioned x{world} (LPT by prompt + new tokens, no collective)",
                       "sampling": "T=0.7 top-p 0.9 on the device"}}


def run_c5(args):
    """`--workload c5`: the C5 serving run alone (c5_serve) as the line."""
    import torch
    import torch.distributed as dist

    from opworks_b200 import pack
    from opworks_b200.llama import Model

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=torch.device("cuda", local))
    if rank == 0:
        pack.ensure_random_llama_pack()
    if world > 1:
        dist.barrier()
    pack_path = pack.ensure_random_llama_pack()
    model = Model(pack_path, weight_sets=1, device=local)
    line = c5_serve(model, args, rank, world, torch.device("cuda", local))
    if rank == 0:
        line.update({"higher_is_better": True, "dtype": "f16",
                     "data": "synthetic: random-init weights, uniform random prompt ids"})
        print(json.dumps(line), flush=True)
    model.close()
    if world > 1:
        dist.destroy_process_group()


def main():
    global BATCH, CTX
    args = parse()
    BATCH, CTX = args.batch, args.ctx
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "c5":
        run_c5(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
