"""A tiny Kimi-K3-format checkpoint for the loader tests: safetensors shards (an 8-byte
little-endian header length, the JSON header padded to 8 bytes, then the tensors),
``config.json`` with the ``text_config`` fields the manifest reads, and
``model.safetensors.index.json``. Layer 0 is dense, layer 1 is a latent MoE whose MXFP4
experts store each ``weight_scale`` right after its ``weight_packed`` (the layout the
reference's one-read pair relies on) unless ``scale_first`` puts it before.
"""
from __future__ import annotations

import json
import struct
from pathlib import Path

import numpy as np

TINY = dict(hidden_size=256, num_hidden_layers=2, num_experts=8, num_experts_per_token=2,
            num_shared_experts=1, routed_expert_hidden_size=128, moe_intermediate_size=128,
            intermediate_size=256, first_k_dense_replace=1, vocab_size=512, rms_norm_eps=1e-5,
            routed_scaling_factor=2.5, moe_renormalize=True, activation_situ_beta=4.0,
            activation_situ_linear_beta=25.0,
            quantization_config={"config_groups": {"group_0": {"weights": {"group_size": 32}}}},
            linear_attn_config={"full_attn_layers": [2], "kda_layers": [1]})
PREFIX = "language_model.model.layers."


def _bf16_bits(a: np.ndarray) -> np.ndarray:
    u = a.astype(np.float32).view(np.uint32)
    return ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)


def save_safetensors(path: Path, tensors: list) -> None:
    """tensors: [(name, array, dtype string)] in file order."""
    header, blobs, off = {}, [], 0
    for name, arr, dt in tensors:
        b = np.ascontiguousarray(arr).tobytes()
        header[name] = {"dtype": dt, "shape": list(arr.shape), "data_offsets": [off, off + len(b)]}
        blobs.append(b)
        off += len(b)
    js = json.dumps(header).encode()
    js += b" " * (-len(js) % 8)
    with Path(path).open("wb") as fh:
        fh.write(struct.pack("<Q", len(js)))
        fh.write(js)
        for b in blobs:
            fh.write(b)


def make_tiny_k3(out: Path, seed: int = 0, scale_first: bool = False, **dims) -> dict:
    """Writes the checkpoint; returns {name: (array, dtype)} of every tensor written.
    ``dims`` overrides TINY's sizes (e.g. 256-wide experts for the tiled kernels)."""
    out = Path(out)
    out.mkdir(parents=True, exist_ok=True)
    rng = np.random.default_rng(seed)
    c = {**TINY, **dims}
    H, Lt, I, E = c["hidden_size"], c["routed_expert_hidden_size"], c["moe_intermediate_size"], c["num_experts"]

    def bf(*shape, s=0.05):
        return _bf16_bits(rng.standard_normal(shape) * s)

    def mx(rows, cols):
        return (rng.integers(0, 256, (rows, cols // 2), dtype=np.uint8),
                rng.integers(120, 131, (rows, cols // 32), dtype=np.uint8))

    shards, allt = {}, {}
    p0 = PREFIX + "0."
    shards["model-00001-of-00003.safetensors"] = [
        (p0 + "input_layernorm.weight", bf(H, s=1.0), "BF16"),
        (p0 + "mlp.gate_proj.weight", bf(c["intermediate_size"], H), "BF16"),
        (p0 + "mlp.up_proj.weight", bf(c["intermediate_size"], H), "BF16"),
        (p0 + "mlp.down_proj.weight", bf(H, c["intermediate_size"]), "BF16"),
        (p0 + "self_attn.A_log", rng.standard_normal(16).astype(np.float32), "F32"),
    ]
    m = PREFIX + "1.block_sparse_moe."
    t = [(PREFIX + "1.post_attention_layernorm.weight", bf(H, s=1.0), "BF16"),
         (m + "gate.weight", bf(E, H, s=0.02), "BF16"),
         (m + "gate.e_score_correction_bias", (rng.standard_normal(E) * 0.1).astype(np.float32), "F32"),
         (m + "routed_expert_down_proj.weight", bf(Lt, H, s=H ** -0.5), "BF16"),
         (m + "routed_expert_up_proj.weight", bf(H, Lt, s=Lt ** -0.5), "BF16"),
         (m + "routed_expert_norm.weight", _bf16_bits(1.0 + 0.1 * rng.standard_normal(Lt)), "BF16"),
         (m + "shared_experts.gate_proj.weight", bf(I, H, s=H ** -0.5), "BF16"),
         (m + "shared_experts.up_proj.weight", bf(I, H, s=H ** -0.5), "BF16"),
         (m + "shared_experts.down_proj.weight", bf(H, I, s=I ** -0.5), "BF16")]
    for e in range(E):
        for w, (rows, cols) in (("w1", (I, Lt)), ("w3", (I, Lt)), ("w2", (Lt, I))):
            pk, sc = mx(rows, cols)
            pair = [(f"{m}experts.{e}.{w}.weight_packed", pk, "U8"), (f"{m}experts.{e}.{w}.weight_scale", sc, "U8")]
            t += pair[::-1] if scale_first else pair
    shards["model-00002-of-00003.safetensors"] = t
    shards["model-00003-of-00003.safetensors"] = [
        ("language_model.model.embed_tokens.weight", bf(c["vocab_size"], H), "BF16"),
        ("language_model.lm_head.weight", bf(c["vocab_size"], H), "BF16"),
        ("language_model.model.norm.weight", bf(H, s=1.0), "BF16"),
    ]
    weight_map = {}
    for fn, tensors in shards.items():
        save_safetensors(out / fn, tensors)
        for name, arr, dt in tensors:
            weight_map[name] = fn
            allt[name] = (arr, dt)
    (out / "model.safetensors.index.json").write_text(json.dumps({"metadata": {"total_size": 0},
                                                                   "weight_map": weight_map}))
    (out / "config.json").write_text(json.dumps({"model_type": "kimi_k3", "text_config": c}, indent=1))
    return allt
