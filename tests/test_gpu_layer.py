"""The caller step around the MoE (``k3_attn_res_norm``, ``layer.MoEBlock``) on the GPU.

The MoE input rmsnorm(apply_attn_res(prefix_sum, block_residual)) against the reference's
own torch oracle outputs (``tests/golden/attn_res.npz``, ``k3ref/layers.py:83-96``) and
the oracle restatement; then the whole MoE half of a decoder layer (``layer.py:119-126``)
on the reference's latent golden layer against the oracle.
"""
import numpy as np
import pytest
import torch

import goldens as G
import inputs as I
from oracle import mxfp4_oracle as O

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("case", ["small", "none", "k3"])
def test_attn_res_norm_matches_reference(k3, case):
    from kimi_k3_mlx_macmini_b200 import layer
    g = G.load("attn_res")
    c = {k: int(g[f"{case}_{k}"]) for k in ("seed", "N", "B", "H")}
    d = I.attnres_inputs(**c)
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    br = cu(d["block_residual"]) if c["B"] else None
    y = layer.attn_res_norm(cu(d["prefix_sum"]), br, cu(I.as_f32(d["proj_bf16"])), cu(I.as_f32(d["res_norm_bf16"])),
                            cu(I.as_f32(d["post_norm_bf16"])), d["eps"])
    torch.cuda.synchronize()
    assert O.rel_l2(y.cpu().numpy(), g[f"{case}_y"]) < 2e-6
    yb = layer.attn_res_norm(cu(d["prefix_sum"]), br, cu(I.as_f32(d["proj_bf16"])), cu(I.as_f32(d["res_norm_bf16"])),
                             cu(I.as_f32(d["post_norm_bf16"])), d["eps"], out_dtype=torch.bfloat16)
    assert O.rel_l2(yb.float().cpu().numpy(), g[f"{case}_y"]) < 4e-3


def test_moe_block_matches_oracle(k3):
    """prefix_sum + moe(rmsnorm(attn_res(prefix_sum, block_residual))) on the reference's
    latent golden layer (situ, latent down/up/norm, dense shared experts)."""
    from kimi_k3_mlx_macmini_b200 import layer
    d, g, spec, src, latent, shared = G.latent_case()
    E, H = spec.num_experts, d["x_bf16"].shape[1]
    cfg = k3.MoEConfig(hidden_size=H, num_experts=E, num_experts_per_token=spec.top_k,
                       moe_intermediate_size=d["experts"][0][0][0].shape[0],
                       routed_expert_hidden_size=latent["down"].shape[0], routed_scaling_factor=1.0,
                       situ_beta=4.0, situ_linear_beta=25.0, activation="situ")
    cu = lambda a: torch.from_numpy(np.ascontiguousarray(a)).cuda()  # noqa: E731
    w = {"gate.weight": cu(d["gate_bf16"]).view(torch.bfloat16), "gate.e_score_correction_bias": cu(d["bias"]),
         "routed_expert_down_proj.weight": cu(latent["down"]), "routed_expert_up_proj.weight": cu(latent["up"]),
         "routed_expert_norm.weight": cu(latent["norm"]),
         "shared_experts.gate_proj.weight": cu(shared["gate"]), "shared_experts.up_proj.weight": cu(shared["up"]),
         "shared_experts.down_proj.weight": cu(shared["down"])}
    moe = k3.LatentMoE(cfg, 1, w, lambda L_, e, wh: d["experts"][int(e)][("w1", "w3", "w2").index(wh)])
    rng = np.random.default_rng(17)
    M, B = 3, 2
    ps = rng.standard_normal((M, H)).astype(np.float32)
    br = rng.standard_normal((M, B, H)).astype(np.float32)
    norms = {"post_attention_layernorm.weight": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32),
             "mlp_res_proj.weight": (0.05 * rng.standard_normal((1, H))).astype(np.float32),
             "mlp_res_norm.weight": (1 + 0.1 * rng.standard_normal(H)).astype(np.float32)}
    blk = layer.MoEBlock(cfg, moe, norms)
    out, r = blk(cu(ps), cu(br))
    x = O.moe_input(ps, br, norms["mlp_res_proj.weight"], norms["mlp_res_norm.weight"],
                    norms["post_attention_layernorm.weight"], 1e-5)
    y, rr = O.moe_forward(x, spec, I.as_f32(d["gate_bf16"]), d["bias"], src, shared=shared, latent=latent)
    want = ps + y
    bad, _ = G.index_sets_match(r.expert_indices.cpu().numpy(), np.sort(rr.expert_indices, -1),
                                rr.corrected_scores, spec.top_k)
    assert bad == 0
    assert O.rel_l2(out.cpu().numpy(), want) < 1e-5
