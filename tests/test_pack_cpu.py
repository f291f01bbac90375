"""OPWPACK1 packs (opworks_b200/pack.py; format of OpWorks
scripts/llama/pack_format.py:1-87 and include/runtime/pack_reader.cuh:25-92):
write/read round trip, 64-byte tensor alignment, aliases, the HF tensor order,
and the bf16-grid rounding used by random-init packs."""

import json
import struct

import numpy as np
import torch

from opworks_b200 import pack


def test_round_trip_alignment_and_alias(tmp_path):
    rng = np.random.default_rng(3)
    arrays = {"a": rng.standard_normal((3, 5)).astype(np.float32), "b": rng.standard_normal(7).astype(np.float32)}
    path = str(tmp_path / "t.pack")
    pack.write_pack(path, [(k, v.shape) for k, v in arrays.items()], lambda n, s: arrays[n],
                    extra={"config": {"x": 1}}, aliases={"c": "a"})
    with open(path, "rb") as f:
        assert f.read(8) == b"OPWPACK1"
        (n,) = struct.unpack("<Q", f.read(8))
        manifest = json.loads(f.read(n))
    assert manifest["format_version"] == 1 and manifest["dtype"] == "float32"
    assert all(t["offset"] % 64 == 0 for t in manifest["tensors"].values())
    m2, t2 = pack.read_pack(path)
    assert m2["config"] == {"x": 1}
    for k, v in arrays.items():
        np.testing.assert_array_equal(t2[k], v)
    np.testing.assert_array_equal(t2["c"], arrays["a"])


def test_bf16_pack_stores_raw_bits(tmp_path):
    x = np.array([1.0, -2.5, 3.140625], np.float32)
    bits = (x.view(np.uint32) >> 16).astype(np.uint16)
    path = str(tmp_path / "b.pack")
    pack.write_pack(path, [("w", x.shape)], lambda n, s: bits, dtype="bfloat16")
    m, t = pack.read_pack(path)
    assert m["dtype"] == "bfloat16"
    np.testing.assert_array_equal(t["w"], bits)


def test_bf16_grid_rounding_matches_torch():
    x = np.random.default_rng(1).standard_normal(10000).astype(np.float32) * 0.02
    ours = pack.round_to_bf16_grid(x)
    want = torch.from_numpy(x).to(torch.bfloat16).float().numpy()
    np.testing.assert_array_equal(ours, want)


def test_llama_tensor_order_and_count():
    specs = pack.llama_tensor_specs(pack.LLAMA_3_2_1B)
    names = [s[0] for s in specs]
    assert names[:2] == ["model.embed_tokens.weight", "model.norm.weight"]
    assert len(names) == 2 + 9 * 16
    params = sum(int(np.prod(s[1])) for s in specs)
    assert params == 1_235_814_400  # tied LM head: the embedding once


def test_tiny_random_pack(tmp_path):
    cfg = dict(pack.LLAMA_3_2_1B, num_hidden_layers=1, hidden_size=64, intermediate_size=128,
               num_attention_heads=4, num_key_value_heads=2, head_dim=16, vocab_size=100)
    path = pack.random_llama_pack(str(tmp_path / "r.pack"), cfg, seed=5)
    m, t = pack.read_pack(path)
    assert m["config"]["hidden_size"] == 64
    assert m["eos_token_ids"] == pack.LLAMA_EOS
    w = np.asarray(t["model.layers.0.self_attn.q_proj.weight"])
    np.testing.assert_array_equal(w, pack.round_to_bf16_grid(w))
    np.testing.assert_array_equal(np.asarray(t["model.layers.0.input_layernorm.weight"]), np.ones(64, np.float32))
    np.testing.assert_array_equal(np.asarray(t["lm_head.weight"]), np.asarray(t["model.embed_tokens.weight"]))
