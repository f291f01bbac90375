"""Seeded inputs shared by the golden-vector generator (make_golden.py, run
where the reference tree is mounted) and the tests that replay them. Only
numpy is used so the tests regenerate bit-identical inputs anywhere."""

from __future__ import annotations

import numpy as np

H, I, QH, KVH, D, V = 2048, 8192, 32, 8, 64, 128256
ROPE_SCALING = {"factor": 32.0, "low_freq_factor": 1.0, "high_freq_factor": 4.0,
                "original_max_position_embeddings": 8192, "rope_type": "llama3"}
THETA = 500000.0
EPS = 1e-5


def op_inputs():
    rng = np.random.default_rng(20261201)
    f = lambda *s: rng.standard_normal(s, dtype=np.float32)
    x = {}
    x["rms.x"] = f(5, H) * np.float32(3)
    x["rms.w"] = f(H) * np.float32(0.5) + np.float32(1)
    x["lin.x"] = f(3, H)
    x["lin.w"] = f(512, H) / np.float32(np.sqrt(H))
    x["gemv.x"] = f(1, H)
    x["gemv.w"] = f(I, H) / np.float32(np.sqrt(H))
    x["rope.q"] = f(17, QH * D)
    x["rope.k"] = f(17, KVH * D)
    x["rope.pos0"] = np.int32(29)
    x["attn.q"] = f(37, QH, D)
    x["attn.k"] = f(37, KVH, D)
    x["attn.v"] = f(37, KVH, D)
    x["attn.qd"] = f(1, QH, D)
    x["swiglu.g"] = f(4, I)
    x["swiglu.u"] = f(4, I)
    x["argmax.x"] = f(V)
    return x


TINY_CFG = {
    "num_hidden_layers": 2, "hidden_size": 512, "intermediate_size": 1024, "num_attention_heads": 8,
    "num_key_value_heads": 2, "head_dim": 64, "vocab_size": 2048, "rms_norm_eps": 1e-5, "rope_theta": THETA,
    "rope_scaling": dict(ROPE_SCALING), "tie_word_embeddings": True,
}
TINY_PROMPT = [5, 17, 1999, 0, 42, 1024, 7, 7, 300, 1500, 2047, 64]
TINY_STEPS = 8


def tiny_weights(cfg=TINY_CFG, seed=7):
    """HF-named fp32 weights: projections N(0, 0.02) (embedding N(0, 1) so the
    tiny model has well separated logits), norm gains 1 + 0.1 N(0, 1)."""
    rng = np.random.default_rng(seed)
    Hs, Is = cfg["hidden_size"], cfg["intermediate_size"]
    qw, kw = cfg["num_attention_heads"] * cfg["head_dim"], cfg["num_key_value_heads"] * cfg["head_dim"]
    g = lambda *s: rng.standard_normal(s, dtype=np.float32)
    w = {"model.embed_tokens.weight": g(cfg["vocab_size"], Hs), "model.norm.weight": 1 + np.float32(0.1) * g(Hs)}
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        w[p + "input_layernorm.weight"] = 1 + np.float32(0.1) * g(Hs)
        w[p + "self_attn.q_proj.weight"] = np.float32(0.05) * g(qw, Hs)
        w[p + "self_attn.k_proj.weight"] = np.float32(0.05) * g(kw, Hs)
        w[p + "self_attn.v_proj.weight"] = np.float32(0.05) * g(kw, Hs)
        w[p + "self_attn.o_proj.weight"] = np.float32(0.05) * g(Hs, qw)
        w[p + "post_attention_layernorm.weight"] = 1 + np.float32(0.1) * g(Hs)
        w[p + "mlp.gate_proj.weight"] = np.float32(0.05) * g(Is, Hs)
        w[p + "mlp.up_proj.weight"] = np.float32(0.05) * g(Is, Hs)
        w[p + "mlp.down_proj.weight"] = np.float32(0.05) * g(Hs, Is)
    return w


SAMPLER_CASES = [  # (vocab, logit scale, temperature, top_p, seed)
    (4096, 3.0, 0.7, 0.9, 11),
    (4096, 3.0, 1.0, 1.0, 12),
    (4096, 1.0, 0.7, 0.5, 13),
    (128256, 1.0, 0.7, 0.9, 14),
]
SAMPLER_DRAWS = 16


def sampler_logits(vocab, scale, seed):
    rng = np.random.default_rng(1000 + seed)
    return rng.standard_normal(vocab, dtype=np.float32) * np.float32(scale)
