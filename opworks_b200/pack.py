"""OPWPACK1 tensor packs: the weight format ``opw_llama_load`` reads.

Layout (same bytes as OpWorks scripts/llama/pack_format.py:1-87 and
include/runtime/pack_reader.cuh:25-92):

    [8B "OPWPACK1"][u64 LE json_len][json manifest][blob]

The manifest holds ``format_version`` 1, ``dtype`` (float32 / bfloat16),
``tensors`` {name: {offset, shape}} with offsets relative to the blob start and
64-byte aligned, optional ``aliases``, and the model ``config`` and
``eos_token_ids`` the runtime reads. This writer streams tensors to disk one at
a time, so a 4.9 GB Llama-3.2-1B pack never sits in memory.
"""

from __future__ import annotations

import json
import os
import struct

import numpy as np

MAGIC = b"OPWPACK1"
ALIGN = 64

# Llama-3.2-1B architecture (HF config.json values used by the reference).
LLAMA_3_2_1B = {
    "num_hidden_layers": 16,
    "hidden_size": 2048,
    "intermediate_size": 8192,
    "num_attention_heads": 32,
    "num_key_value_heads": 8,
    "head_dim": 64,
    "vocab_size": 128256,
    "rms_norm_eps": 1e-5,
    "rope_theta": 500000.0,
    "rope_scaling": {
        "rope_type": "llama3",
        "factor": 32.0,
        "low_freq_factor": 1.0,
        "high_freq_factor": 4.0,
        "original_max_position_embeddings": 8192,
    },
    "tie_word_embeddings": True,
}
LLAMA_EOS = [128001, 128008, 128009]


def _align(n: int) -> int:
    return (n + ALIGN - 1) // ALIGN * ALIGN


def llama_tensor_specs(cfg):
    """(name, shape, kind) in the HF order the reference uploads them
    (include/runtime/weights.cuh:71-85); kind is 'norm' or 'proj'."""
    H, I = cfg["hidden_size"], cfg["intermediate_size"]
    D = cfg.get("head_dim") or H // cfg["num_attention_heads"]
    qw, kw = cfg["num_attention_heads"] * D, cfg["num_key_value_heads"] * D
    specs = [("model.embed_tokens.weight", (cfg["vocab_size"], H), "proj"), ("model.norm.weight", (H,), "norm")]
    for i in range(cfg["num_hidden_layers"]):
        p = f"model.layers.{i}."
        specs += [
            (p + "input_layernorm.weight", (H,), "norm"),
            (p + "self_attn.q_proj.weight", (qw, H), "proj"),
            (p + "self_attn.k_proj.weight", (kw, H), "proj"),
            (p + "self_attn.v_proj.weight", (kw, H), "proj"),
            (p + "self_attn.o_proj.weight", (H, qw), "proj"),
            (p + "post_attention_layernorm.weight", (H,), "norm"),
            (p + "mlp.gate_proj.weight", (I, H), "proj"),
            (p + "mlp.up_proj.weight", (I, H), "proj"),
            (p + "mlp.down_proj.weight", (H, I), "proj"),
        ]
    return specs


def write_pack(path, specs, produce, extra=None, aliases=None, dtype="float32"):
    """Stream a pack: specs = [(name, shape)], produce(name, shape) -> array."""
    if dtype not in ("float32", "bfloat16"):
        raise ValueError(f"unsupported pack dtype {dtype}")
    esize = 4 if dtype == "float32" else 2
    manifest = {"format_version": 1, "dtype": dtype, "tensors": {}}
    offset = 0
    for name, shape in specs:
        n = int(np.prod(shape))
        manifest["tensors"][name] = {"offset": offset, "shape": list(shape)}
        offset = _align(offset + n * esize)
    if aliases:
        manifest["aliases"] = dict(aliases)
    if extra:
        manifest.update(extra)
    js = json.dumps(manifest, sort_keys=True).encode("utf-8")
    tmp = path + ".tmp"
    with open(tmp, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<Q", len(js)))
        f.write(js)
        pos = 0
        for name, shape in specs:
            arr = np.asarray(produce(name, shape))
            if dtype == "float32":
                data = np.ascontiguousarray(arr, dtype="<f4").tobytes()
            else:
                data = np.ascontiguousarray(arr, dtype="<u2").tobytes()  # raw bf16 bits
            f.write(data)
            pos += len(data)
            pad = _align(pos) - pos
            f.write(b"\x00" * pad)
            pos += pad
    os.replace(tmp, path)
    return path


def round_to_bf16_grid(a):
    """fp32 values rounded (nearest-even) to the bf16 grid, kept as fp32."""
    u = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    r = (u + np.uint32(0x7FFF) + ((u >> np.uint32(16)) & np.uint32(1))) & np.uint32(0xFFFF0000)
    return r.view(np.float32)


def bf16_bits(a):
    """fp32 values rounded (nearest-even) to bf16, as raw uint16 bits."""
    return (round_to_bf16_grid(a).view(np.uint32) >> np.uint32(16)).astype(np.uint16)


def random_llama_pack(path, cfg=None, seed=1234, std=0.02, norm_value=1.0, eos=None, bf16_grid=True,
                      dtype="float32"):
    """Random-init Llama pack: projections/embedding ~ N(0, std) drawn from
    numpy default_rng(seed) in HF order, RMSNorm gains = norm_value (the HF
    init), lm_head.weight aliased to the embedding (tied). With bf16_grid the
    fp32 values are rounded to the bf16 grid, so the bf16 copy the fast path
    makes at load is exact and the fp32 and bf16 paths run the same model."""
    cfg = dict(cfg or LLAMA_3_2_1B)
    rng = np.random.default_rng(seed)
    specs = llama_tensor_specs(cfg)

    def produce(name, shape):
        if name.endswith("norm.weight"):
            a = np.full(shape, norm_value, np.float32)
        else:
            a = rng.standard_normal(shape, dtype=np.float32)
            a *= np.float32(std)
            if bf16_grid:
                a = round_to_bf16_grid(a)
        return bf16_bits(a) if dtype == "bfloat16" else a

    extra = {"config": cfg, "eos_token_ids": list(eos if eos is not None else LLAMA_EOS),
             "meta": {"init": "random", "seed": seed, "std": std, "norm_value": norm_value,
                      "bf16_grid": bool(bf16_grid)}}
    return write_pack(path, [(n, s) for n, s, _ in specs], produce, extra=extra,
                      aliases={"lm_head.weight": "model.embed_tokens.weight"}, dtype=dtype)


def read_pack(path, mmap=True):
    """(manifest, {name: ndarray}); float32 packs map to float32 arrays,
    bfloat16 packs to uint16 arrays of raw bits."""
    with open(path, "rb") as f:
        if f.read(8) != MAGIC:
            raise ValueError(f"{path}: bad magic")
        (n,) = struct.unpack("<Q", f.read(8))
        manifest = json.loads(f.read(n))
    base = 16 + n
    dt = np.dtype("<f4") if manifest["dtype"] == "float32" else np.dtype("<u2")
    raw = np.memmap(path, dtype=np.uint8, mode="r") if mmap else np.fromfile(path, dtype=np.uint8)
    out = {}
    for name, meta in manifest["tensors"].items():
        cnt = int(np.prod(meta["shape"]))
        start = base + meta["offset"]
        out[name] = raw[start:start + cnt * dt.itemsize].view(dt).reshape(meta["shape"])
    for alias, target in manifest.get("aliases", {}).items():
        out[alias] = out[target]
    return manifest, out


def default_pack_dir():
    return os.environ.get("OPWORKS_PACK_DIR", "/tmp/opworks_packs")


def ensure_random_llama_pack(cfg=None, seed=1234, name=None, bf16_grid=False, dtype="float32"):
    """Path of a cached random-init pack, generating it on first use. By
    default the weights keep every fp32 bit of the N(0, 0.02) draw (the fast
    path's 16-bit copy is then a rounding of them); bf16_grid=True rounds them
    to the bf16 grid first. dtype="bfloat16" writes a bf16 pack of the same
    draw (each weight rounded to nearest even)."""
    cfg = cfg or LLAMA_3_2_1B
    d = default_pack_dir()
    os.makedirs(d, exist_ok=True)
    grid = "bf16pack" if dtype == "bfloat16" else ("bf16grid" if bf16_grid else "fp32")
    tag = name or f"llama_L{cfg['num_hidden_layers']}_H{cfg['hidden_size']}_V{cfg['vocab_size']}_s{seed}_{grid}"
    path = os.path.join(d, tag + ".pack")
    if not os.path.exists(path):
        random_llama_pack(path, cfg, seed, bf16_grid=bf16_grid, dtype=dtype)
    return path
