"""The tensor-parallel control path on CPU, with two gloo ranks: each rank
takes its shard from the library's own plan (opw_llama_tp_shard in
libopworks_llama.so, the function the engine slices its weights with; no GPU
call), runs a tiny Llama forward over its query / KV heads and MLP columns
(oracle ops on the sliced fused matrices, in the engine's layouts: QKV =
[q; k; v] rows, gate/up rows interleaved), and sums the o and down partial
products with a gloo all-reduce, as the engine does with NCCL or peer stores
after those two projections. Prefill logits and three greedy decode steps
(each rank keeping the KV cache of its own heads only) must equal the
unsharded oracle forward; every rank must end with the same logits.
"""

import ctypes
import os
import socket

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LLAMA_LIB = os.path.join(ROOT, "opworks_b200", "lib", "libopworks_llama.so")


def shard_plan(cfg, rank, world):
    lib = ctypes.CDLL(LLAMA_LIB)
    fn = lib.opw_llama_tp_shard
    fn.argtypes = [ctypes.POINTER(ctypes.c_int32), ctypes.c_int, ctypes.c_int, ctypes.POINTER(ctypes.c_int64),
                   ctypes.c_char_p, ctypes.c_int]
    fn.restype = ctypes.c_int
    c5 = np.array([cfg["hidden_size"], cfg["intermediate_size"], cfg["num_attention_heads"],
                   cfg["num_key_value_heads"], cfg["head_dim"]], np.int32)
    out = np.zeros(12, np.int64)
    err = ctypes.create_string_buffer(256)
    rc = fn(c5.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), rank, world,
            out.ctypes.data_as(ctypes.POINTER(ctypes.c_int64)), err, 256)
    if rc != 0:
        raise ValueError(err.value.decode())
    keys = ["q_heads", "kv_heads", "inter", "q_row0", "k_row0", "v_row0", "q_rows", "kv_rows", "o_col0", "gu_row0",
            "gu_rows", "down_col0"]
    return dict(zip(keys, (int(v) for v in out)))


class RankModel:
    """One rank's shard of the tiny Llama, numpy + oracle ops."""

    def __init__(self, cfg, w, plan):
        import oracle

        self.o = oracle
        self.cfg, self.p = cfg, plan
        self.L, self.H, self.D = cfg["num_hidden_layers"], cfg["hidden_size"], cfg["head_dim"]
        self.eps = cfg["rms_norm_eps"]
        self.inv = oracle.rope_inv_freq(self.D, cfg["rope_theta"], cfg.get("rope_scaling"))
        self.w = w
        self.layers = []
        p = plan
        for i in range(self.L):
            g = lambda n: np.asarray(w[f"model.layers.{i}.{n}"], np.float32)  # noqa: E731
            qkv = np.concatenate([g("self_attn.q_proj.weight"), g("self_attn.k_proj.weight"),
                                  g("self_attn.v_proj.weight")])
            gate, up = g("mlp.gate_proj.weight"), g("mlp.up_proj.weight")
            gu = np.empty((2 * gate.shape[0], gate.shape[1]), np.float32)
            gu[0::2], gu[1::2] = gate, up
            self.layers.append({
                "in_norm": g("input_layernorm.weight"), "post_norm": g("post_attention_layernorm.weight"),
                "q": qkv[p["q_row0"]:p["q_row0"] + p["q_rows"]],
                "k": qkv[p["k_row0"]:p["k_row0"] + p["kv_rows"]],
                "v": qkv[p["v_row0"]:p["v_row0"] + p["kv_rows"]],
                "o": np.ascontiguousarray(g("self_attn.o_proj.weight")[:, p["o_col0"]:p["o_col0"] + p["q_rows"]]),
                "gu": gu[p["gu_row0"]:p["gu_row0"] + p["gu_rows"]],
                "down": np.ascontiguousarray(
                    g("mlp.down_proj.weight")[:, p["down_col0"]:p["down_col0"] + p["inter"]]),
            })
        self.k_cache = [np.zeros((0, p["kv_heads"], self.D), np.float32) for _ in range(self.L)]
        self.v_cache = [np.zeros((0, p["kv_heads"], self.D), np.float32) for _ in range(self.L)]

    def forward(self, ids, pos, allreduce):
        o, p, D = self.o, self.p, self.D
        x = np.asarray(self.w["model.embed_tokens.weight"], np.float32)[np.asarray(ids)].copy()
        n = x.shape[0]
        for l, lw in enumerate(self.layers):
            h = o.rms_norm(x, lw["in_norm"], self.eps)
            q = o.rope(o.linear(h, lw["q"]), self.inv, p["q_heads"], D, pos)
            k = o.rope(o.linear(h, lw["k"]), self.inv, p["kv_heads"], D, pos)
            v = o.linear(h, lw["v"])
            self.k_cache[l] = np.concatenate([self.k_cache[l], k.reshape(n, p["kv_heads"], D)])
            self.v_cache[l] = np.concatenate([self.v_cache[l], v.reshape(n, p["kv_heads"], D)])
            att = o.attention(q.reshape(n, p["q_heads"], D), self.k_cache[l], self.v_cache[l]).reshape(n, -1)
            x = x + allreduce(o.linear(att, lw["o"]))
            h = o.rms_norm(x, lw["post_norm"], self.eps)
            gu = o.linear(h, lw["gu"])
            act = o.swiglu(gu[:, 0::2], gu[:, 1::2])
            x = x + allreduce(o.linear(act, lw["down"]))
        h = o.rms_norm(x[-1:], np.asarray(self.w["model.norm.weight"], np.float32), self.eps)
        return o.linear(h, np.asarray(self.w["model.embed_tokens.weight"], np.float32))[0]


def _worker(rank, world, port, q):
    import sys

    sys.path.insert(0, ROOT)
    sys.path.insert(0, os.path.join(ROOT, "tests", "golden"))
    import torch
    import torch.distributed as dist

    import inputs
    import oracle

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        cfg, w = inputs.TINY_CFG, inputs.tiny_weights()
        m = RankModel(cfg, w, shard_plan(cfg, rank, world))

        def allreduce(a):
            t = torch.from_numpy(np.ascontiguousarray(a, np.float32))
            dist.all_reduce(t)
            return t.numpy()

        prompt = inputs.TINY_PROMPT
        got = [m.forward(prompt, 0, allreduce)]
        toks = [oracle.argmax(got[-1])]
        for k in range(3):
            got.append(m.forward([toks[-1]], len(prompt) + k, allreduce))
            toks.append(oracle.argmax(got[-1]))
        # every rank holds the same logits
        t = torch.from_numpy(np.stack(got))
        mx, mn = t.clone(), t.clone()
        dist.all_reduce(mx, op=dist.ReduceOp.MAX)
        dist.all_reduce(mn, op=dist.ReduceOp.MIN)
        spread = float((mx - mn).abs().max())
        if rank == 0:
            full = oracle.Llama(cfg, w)
            kc, vc = full.new_cache(len(prompt) + 8)
            want = [full.forward(prompt, 0, kc, vc)]
            for k in range(3):
                want.append(full.forward([toks[k]], len(prompt) + k, kc, vc))
            err = max(float(np.max(np.abs(a - b))) for a, b in zip(got, want))
            q.put((err, spread, toks, [oracle.argmax(x) for x in want]))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_plan_covers_every_row_once():
    if not os.path.exists(LLAMA_LIB):
        pytest.skip("libopworks_llama.so not built")
    import inputs

    cfg = dict(inputs.TINY_CFG)
    for world in (1, 2):
        plans = [shard_plan(cfg, r, world) for r in range(world)]
        H, I, D = cfg["hidden_size"], cfg["intermediate_size"], cfg["head_dim"]
        qh, kvh = cfg["num_attention_heads"], cfg["num_key_value_heads"]
        rows = sorted(r for p in plans for a, n in ((p["q_row0"], p["q_rows"]), (p["k_row0"], p["kv_rows"]),
                                                     (p["v_row0"], p["kv_rows"])) for r in range(a, a + n))
        assert rows == list(range((qh + 2 * kvh) * D))
        assert sorted(c for p in plans for c in range(p["o_col0"], p["o_col0"] + p["q_rows"])) == list(range(qh * D))
        assert sorted(r for p in plans for r in range(p["gu_row0"], p["gu_row0"] + p["gu_rows"])) == list(range(2 * I))
        assert sorted(c for p in plans for c in range(p["down_col0"], p["down_col0"] + p["inter"])) == list(range(I))
    with pytest.raises(ValueError):
        shard_plan(cfg, 0, 3)  # 2 KV heads do not split 3 ways


@pytest.mark.timeout(240)
def test_two_gloo_ranks_tensor_parallel_forward_equals_full_model():
    if not os.path.exists(LLAMA_LIB):
        pytest.skip("libopworks_llama.so not built")
    import torch.multiprocessing as mp

    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(200)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    err, spread, toks, want_toks = q.get(timeout=5)
    assert spread == 0.0, spread
    assert err <= 1e-4, err
    assert toks == want_toks
