"""Load the committed golden fixtures and regenerate their seeded inputs.

Shared by the CPU oracle tests and the GPU parity tests; reads only files under
``tests/golden`` (never the reference checkout).
"""
from __future__ import annotations

import json
from pathlib import Path

import numpy as np

import inputs as I
from oracle import mxfp4_oracle as O

GOLDEN = Path(__file__).resolve().parent / "golden"


def load(name: str) -> dict:
    with np.load(GOLDEN / f"{name}.npz", allow_pickle=False) as z:
        return {k: z[k] for k in z.files}


def config0():
    g = load("config0")
    d = I.config0_inputs(seed=int(g["seed"]))
    assert I.digest(d["x_bf16"], *d["w1"], *d["w3"], *d["w2"]) == str(g["digest"]), "input regen drift"
    return d, g


def moe_case(name: str):
    """(inputs dict, golden dict, oracle MoESpec, experts source, shared dict) for a
    BASELINE-semantics MoE fixture."""
    g = load(name)
    M, H, I_, E = (int(g[k]) for k in ("M", "H", "I", "E"))
    d = I.moe_inputs(int(g["seed"]), M, H, I_, E, shared=True, bias_std=float(g["bias_std"]))
    flat = [a for tr in d["experts"] for pair in tr for a in pair] + [a for pair in d["shared"] for a in pair]
    assert I.digest(d["x_bf16"], d["gate_bf16"], d["bias"], *flat) == str(g["digest"]), "input regen drift"
    spec = O.MoESpec(num_experts=E, top_k=int(g["k"]), routed_scaling_factor=float(g["scale"]),
                     renormalize=True, activation="silu")
    src = lambda e, w: d["experts"][e][{"w1": 0, "w3": 1, "w2": 2}[w]]  # noqa: E731
    sh = {"kind": "mxfp4", "w1": d["shared"][0], "w3": d["shared"][1], "w2": d["shared"][2]}
    return d, g, spec, src, sh


def latent_case():
    g = load("moe_latent")
    M, H, L, I_, E, S = (int(g[k]) for k in ("M", "H", "L", "I", "E", "S"))
    d = I.latent_moe_inputs(int(g["seed"]), M, H, L, I_, E, S)
    keys = ("x_bf16", "gate_bf16", "bias", "down_bf16", "up_bf16", "norm_bf16",
            "sh_gate_bf16", "sh_up_bf16", "sh_down_bf16")
    flat = [a for tr in d["experts"] for pair in tr for a in pair]
    assert I.digest(*[d[q] for q in keys], *flat) == str(g["digest"]), "input regen drift"
    spec = O.MoESpec(num_experts=E, top_k=int(g["k"]), routed_scaling_factor=1.0, renormalize=True,
                     activation="situ", situ_beta=4.0, situ_linear_beta=25.0, rms_norm_eps=1e-5)
    src = lambda e, w: d["experts"][e][{"w1": 0, "w3": 1, "w2": 2}[w]]  # noqa: E731
    latent = {"down": I.as_f32(d["down_bf16"]), "up": I.as_f32(d["up_bf16"]),
              "norm": I.as_f32(d["norm_bf16"])}
    shared = {"kind": "dense", "gate": I.as_f32(d["sh_gate_bf16"]), "up": I.as_f32(d["sh_up_bf16"]),
              "down": I.as_f32(d["sh_down_bf16"])}
    return d, g, spec, src, latent, shared


def mini_k3_case():
    g = load("mini_k3")
    meta = json.loads(str(g["meta"]))
    t = {k[2:]: v for k, v in g.items() if k.startswith("t.")}
    E = int(meta["num_experts"])
    experts = [tuple((t[f"e{e}.{w}.packed"], t[f"e{e}.{w}.scales"]) for w in ("w1", "w3", "w2"))
               for e in range(E)]
    spec = O.MoESpec(num_experts=E, top_k=int(meta["num_experts_per_token"]),
                     routed_scaling_factor=float(meta["routed_scaling_factor"]),
                     renormalize=bool(meta["moe_renormalize"]), activation="situ",
                     situ_beta=float(meta["activation_situ_beta"]),
                     situ_linear_beta=float(meta["activation_situ_linear_beta"]),
                     rms_norm_eps=float(meta["rms_norm_eps"]))
    src = lambda e, w: experts[e][{"w1": 0, "w3": 1, "w2": 2}[w]]  # noqa: E731
    f = lambda k: I.as_f32(t[k]) if t[k].dtype == np.uint16 else t[k].astype(np.float32)  # noqa: E731
    latent = {"down": f("routed_expert_down_proj.weight"), "up": f("routed_expert_up_proj.weight"),
              "norm": f("routed_expert_norm.weight")}
    shared = {"kind": "dense", "gate": f("shared_experts.gate_proj.weight"),
              "up": f("shared_experts.up_proj.weight"), "down": f("shared_experts.down_proj.weight")}
    gate = t["gate.weight"]
    bias = t["gate.e_score_correction_bias"].astype(np.float32)
    return g, meta, spec, src, latent, shared, gate, bias, experts


def index_sets_match(idx_got, idx_want_sorted, corrected_ref, k, tie_tol=1e-6):
    """Compare top-k index SETS per row (order-free, like ``tests/test_moe_mlx.py:70-75``).
    Rows whose k-th/(k+1)-th corrected-score gap is below ``tie_tol`` are near-ties that
    two fp32 implementations may order differently; they are returned separately.
    Returns (n_mismatch_outside_ties, n_ties)."""
    got = np.sort(np.asarray(idx_got), axis=-1)
    want = np.asarray(idx_want_sorted)
    gap = O.topk_gap(corrected_ref, k)
    ties = gap < tie_tol
    bad = ~np.all(got == want, axis=-1) & ~ties
    return int(bad.sum()), int(ties.sum())


def canon_weights(idx, w):
    o = np.argsort(np.asarray(idx), axis=-1)
    return np.take_along_axis(np.asarray(w), o, axis=-1)
