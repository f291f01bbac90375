"""Generates tests/golden/*.npz from the REFERENCE's own code (run where the
reference tree is mounted; the outputs are committed, the tree is not needed
afterwards):

* ops_golden.npz     reference math of scripts/llama/export_reference.py:32-88
                     (rms_norm, llama3_inv_freq, apply_rope, causal_attention,
                     silu_mul) + torch matmul/argmax on tests/golden/inputs.py
* tiny_llama.npz     transformers LlamaForCausalLM (fp32, eager attention, TF32
                     off) on the tiny config/weights of inputs.py: per-layer
                     hidden states, last logits, greedy continuation
* sampler_golden.npz the reference host sampler LlamaGenerator._sample
                     (examples/llama/generate.py:83-109) with a seeded
                     numpy Generator, logits served by a stand-in for the C ABI

Usage: python tests/golden/make_golden.py [<reference root>]
(default: OPWORKS_REFERENCE, else a `reference` directory beside the repository)
"""

from __future__ import annotations

import ctypes
import importlib.util
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)
import inputs  # noqa: E402


def _load(path, name):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    sys.path.insert(0, os.path.dirname(path))
    spec.loader.exec_module(mod)
    sys.path.pop(0)
    return mod


def ops_golden(ref):
    er = _load(os.path.join(ref, "scripts/llama/export_reference.py"), "ref_export_reference")
    x = inputs.op_inputs()
    t = {k: torch.from_numpy(np.asarray(v)) for k, v in x.items() if isinstance(v, np.ndarray)}
    out = {}
    out["rms.out"] = er.rms_norm(t["rms.x"], t["rms.w"], inputs.EPS).numpy()
    inv = er.llama3_inv_freq(inputs.D, inputs.THETA, inputs.ROPE_SCALING)
    out["rope.inv_freq"] = inv.numpy()
    pos = torch.arange(17) + int(x["rope.pos0"])
    out["rope.q_out"] = er.apply_rope(t["rope.q"], pos, inv).numpy()
    out["rope.k_out"] = er.apply_rope(t["rope.k"], pos, inv).numpy()
    out["attn.out"] = er.causal_attention(t["attn.q"], t["attn.k"], t["attn.v"], inputs.KVH).numpy()
    out["attn.out_decode"] = er.causal_attention(t["attn.qd"], t["attn.k"], t["attn.v"], inputs.KVH).numpy()
    out["swiglu.out"] = er.silu_mul(t["swiglu.g"], t["swiglu.u"]).numpy()
    torch.backends.cuda.matmul.allow_tf32 = False
    out["lin.out"] = (t["lin.x"].double() @ t["lin.w"].double().T).float().numpy()
    out["gemv.out"] = (t["gemv.x"].double() @ t["gemv.w"].double().T).float().numpy()
    out["argmax.out"] = np.array([int(torch.argmax(t["argmax.x"]))], np.int32)
    np.savez_compressed(os.path.join(HERE, "ops_golden.npz"), **out)


def tiny_llama_golden():
    from transformers import LlamaConfig, LlamaForCausalLM

    torch.set_float32_matmul_precision("highest")
    c = inputs.TINY_CFG
    cfg = LlamaConfig(vocab_size=c["vocab_size"], hidden_size=c["hidden_size"],
                      intermediate_size=c["intermediate_size"], num_hidden_layers=c["num_hidden_layers"],
                      num_attention_heads=c["num_attention_heads"], num_key_value_heads=c["num_key_value_heads"],
                      head_dim=c["head_dim"], rms_norm_eps=c["rms_norm_eps"], rope_theta=c["rope_theta"],
                      rope_scaling=dict(c["rope_scaling"]), tie_word_embeddings=True,
                      max_position_embeddings=131072, attn_implementation="eager")
    model = LlamaForCausalLM(cfg).float().eval()
    w = inputs.tiny_weights()
    sd = {k: torch.from_numpy(v) for k, v in w.items()}
    sd["lm_head.weight"] = sd["model.embed_tokens.weight"]
    missing, unexpected = model.load_state_dict(sd, strict=False)
    assert not unexpected, unexpected
    assert all("rotary" in m for m in missing), missing
    ids = torch.tensor([inputs.TINY_PROMPT])
    with torch.no_grad():
        pre = {}
        hook = model.model.norm.register_forward_pre_hook(lambda m, a: pre.setdefault("x", a[0].detach()))
        out = model(input_ids=ids, output_hidden_states=True, use_cache=False)
        hook.remove()
        hs = out.hidden_states  # embed, layer1.., last is final-normed in transformers 5
        L = c["num_hidden_layers"]
        hidden = [hs[i][0].float().numpy() for i in range(L)] + [pre["x"][0].float().numpy()]
        gen = model.generate(input_ids=ids, max_new_tokens=inputs.TINY_STEPS, do_sample=False, num_beams=1,
                             pad_token_id=0)[0].tolist()
    np.savez_compressed(os.path.join(HERE, "tiny_llama.npz"), hidden=np.stack(hidden),
                        logits=out.logits[0, -1].float().numpy(),
                        greedy=np.array(gen[len(inputs.TINY_PROMPT):], np.int32))


def sampler_golden(ref):
    gen_mod = _load(os.path.join(ref, "examples/llama/generate.py"), "ref_generate")

    class _FakeLib:
        def __init__(self, logits):
            self.logits = logits

        def opw_llama_last_logits(self, session, out, n, err, err_len):
            ctypes.memmove(out, self.logits.ctypes.data, 4 * n)
            return 0

    class _FakeApi:
        def __init__(self, logits):
            self.lib = _FakeLib(logits)
            self.err = ctypes.create_string_buffer(8)

        def check(self, rc, what):
            return rc

    out = {}
    for vocab, scale, temp, top_p, seed in inputs.SAMPLER_CASES:
        logits = inputs.sampler_logits(vocab, scale, seed)
        g = object.__new__(gen_mod.LlamaGenerator)
        g._api = _FakeApi(logits)
        g._session = None
        g._vocab = vocab
        g._logits = (ctypes.c_float * vocab)()
        rng = np.random.default_rng(seed)
        toks = [g._sample(rng, temp, top_p) for _ in range(inputs.SAMPLER_DRAWS)]
        out[f"case{seed}"] = np.array(toks, np.int32)
    np.savez_compressed(os.path.join(HERE, "sampler_golden.npz"), **out)


if __name__ == "__main__":
    sys.path.insert(0, os.path.join(HERE, "..", "..", "oracle"))
    import build_ref  # noqa: E402

    ref = build_ref.reference_root(sys.argv[1] if len(sys.argv) > 1 else None)
    if ref is None:
        sys.exit("reference tree not found: pass its path or set OPWORKS_REFERENCE")
    ops_golden(ref)
    tiny_llama_golden()
    sampler_golden(ref)
    print("golden vectors written to", HERE)
