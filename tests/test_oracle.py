"""Pin the CPU oracle to the reference's own outputs (golden fixtures), on CPU.

Mirrors the reference's checkpoint-free gates: ``tests/test_mxfp4_mlx.py:33-61`` (codec
KATs), ``tests/test_mxfp4_kernel.py:42-54`` (fused matvec vs fp64),
``tools/make_synthetic_k3.py:255-268`` (encoder), and ``tests/test_moe_mlx.py:70-124``
(router exactness, weights 1e-5, block agreement) on synthetic weights.
"""
import numpy as np
import pytest

import goldens as G
import inputs as I
from oracle import mxfp4_oracle as O


def test_all_codes_exact():
    g = G.load("codec_kat")
    got = O.decode_mxfp4(g["all256_packed"], g["all256_scales"])
    assert np.array_equal(got, g["all256_decoded"])
    # the third-party decoder the reference was proven against (compressed-tensors)
    assert np.array_equal(got, g["all256_ct"])


def test_all_scale_bytes_exact():
    g = G.load("codec_kat")
    with np.errstate(over="ignore"):
        got = O.decode_mxfp4(g["scales_packed"], g["scales_bytes"])
    assert np.array_equal(got, g["scales_decoded"])          # incl. byte 0 (2**-127) and 255 (inf)
    assert np.array_equal(O.decode_scale(g["scale_bytes_1_254"]), g["scale_values_1_254"])


def test_scale_range_guard():
    O.assert_scales_representable(np.array([2, 127, 252], np.uint8))
    for bad in (0, 1, 253, 255):
        with pytest.raises(ValueError):
            O.assert_scales_representable(np.array([127, bad], np.uint8))


@pytest.mark.parametrize("M", [1, 2, 4])
def test_fused_order_matvec_vs_fp64(M):
    g = G.load("matvec_kat")
    got = O.matvec_fused(g[f"x{M}"], g["packed"], g["scales"])
    assert O.rel_max(got, g[f"want{M}"]) < 1e-6
    assert O.rel_max(O.matvec_fp64(g[f"x{M}"], g["packed"], g["scales"]), g[f"want{M}"]) < 1e-12


def test_encoder_matches_reference_packer():
    g = G.load("encoder")
    for k in ("a", "b"):
        p, s = O.encode_mxfp4(g[k])
        assert np.array_equal(p, g[f"{k}_packed"]) and np.array_equal(s, g[f"{k}_scales"])
        p2, s2 = O.encode_mxfp4(O.decode_mxfp4(p, s))          # idempotent on its own output
        assert np.array_equal(p, p2) and np.array_equal(s, s2)


def test_config0_expert_forward():
    d, g = G.config0()
    x = I.as_f32(d["x_bf16"])
    W = [O.decode_mxfp4(*d[w]) for w in ("w1", "w3", "w2")]
    y = O.expert_forward(x, *W, act="silu")
    assert O.rel_l2(y, g["y"]) < 1e-5
    y64 = O.expert_forward(x, *W, act="silu", precision="fp64")
    assert O.rel_l2(g["y"], y64) < 1e-5                       # the reference itself vs fp64


@pytest.mark.parametrize("name", ["moe_small_m1", "moe_small_m5", "moe_small_m8"])
def test_moe_block_matches_reference(name):
    d, g, spec, src, sh = G.moe_case(name)
    x = I.as_f32(d["x_bf16"])
    y, r = O.moe_forward(x, spec, I.as_f32(d["gate_bf16"]), d["bias"], src, shared=sh)
    bad, ties = G.index_sets_match(r.expert_indices, g["idx_sorted"], g["corrected"], spec.top_k)
    assert bad == 0 and ties == 0
    assert np.abs(G.canon_weights(r.expert_indices, r.expert_weights) - g["w_canon"]).max() <= 1e-5
    assert np.abs(r.raw_scores - g["raw"]).max() <= 1e-5
    assert O.rel_l2(y, g["y"]) < 1e-5


def test_latent_moe_matches_reference():
    d, g, spec, src, latent, shared = G.latent_case()
    y, r = O.moe_forward(I.as_f32(d["x_bf16"]), spec, I.as_f32(d["gate_bf16"]), d["bias"], src,
                         shared=shared, latent=latent)
    bad, ties = G.index_sets_match(r.expert_indices, g["idx_sorted"], g["corrected"], spec.top_k)
    assert bad == 0 and ties == 0
    assert O.rel_l2(y, g["y"]) < 1e-5


def test_mini_k3_layer_matches_reference():
    g, meta, spec, src, latent, shared, gate, bias, _ = G.mini_k3_case()
    y, r = O.moe_forward(I.as_f32(g["x_bf16"]), spec, I.as_f32(gate), bias, src,
                         shared=shared, latent=latent)
    bad, ties = G.index_sets_match(r.expert_indices, g["idx_sorted"], g["corrected"], spec.top_k)
    assert bad == 0 and ties == 0
    assert O.rel_l2(y, g["y"]) < 1e-5


@pytest.mark.parametrize("case", ["small", "none", "k3"])
def test_attn_res_moe_input_matches_reference(case):
    """The decoder layer's MoE input, rmsnorm(apply_attn_res(...)), against the reference's
    own torch oracle (``k3ref/layers.py:83-96``) on regenerated inputs (digest-checked)."""
    g = G.load("attn_res")
    c = {k: int(g[f"{case}_{k}"]) for k in ("seed", "N", "B", "H")}
    d = I.attnres_inputs(**c)
    assert I.digest(d["prefix_sum"], d["block_residual"], d["proj_bf16"], d["res_norm_bf16"],
                    d["post_norm_bf16"]) == str(g[f"{case}_digest"]), "input regen drift"
    x = O.attn_res(d["prefix_sum"], d["block_residual"], I.as_f32(d["proj_bf16"]), I.as_f32(d["res_norm_bf16"]),
                   d["eps"])
    y = O.moe_input(d["prefix_sum"], d["block_residual"], I.as_f32(d["proj_bf16"]), I.as_f32(d["res_norm_bf16"]),
                    I.as_f32(d["post_norm_bf16"]), d["eps"])
    assert O.rel_l2(x, g[f"{case}_attn"]) < 1e-6
    assert O.rel_l2(y, g[f"{case}_y"]) < 1e-6
