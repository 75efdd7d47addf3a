"""Seeded synthetic MoE layers with BASELINE.json's shapes and value distributions,
generated directly in HBM (there is no checkpoint; random-init weights of the stated
architecture stand in for it):

* E2M1 codes uniform over all 16 values, packed two per byte (low nibble = even
  element), E8M0 scale bytes uniform in [120, 130];
* router weight bf16 ~ N(0, 0.02), correction bias 0; x bf16 ~ N(0, 1);
* Kimi-K3 layers (``k3_layer``) add the latent projections and the bf16 shared expert,
  bf16 ~ N(0, 1/fan_in), and an RMSNorm weight bf16 ~ 1 + N(0, 0.1).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

from .moe import SHARED, LatentMoE, MoEConfig


def random_mxfp4(gen: torch.Generator, rows: int, cols: int, device, scale_lo: int = 120,
                 scale_hi: int = 130):
    packed = torch.randint(0, 256, (rows, cols // 2), generator=gen, device=device, dtype=torch.uint8)
    scales = torch.randint(scale_lo, scale_hi + 1, (rows, cols // 32), generator=gen, device=device,
                           dtype=torch.uint8)
    return packed, scales


def bf16_normal(gen: torch.Generator, shape, std: float, device) -> torch.Tensor:
    return (torch.randn(shape, generator=gen, device=device, dtype=torch.float32) * std).to(torch.bfloat16)


@dataclass
class SyntheticLayer:
    """Router weights plus lazily generated experts: expert e's three projections come
    from a generator seeded with (seed, e), so any subset (one rank's share of an
    expert-parallel layer) is generated alone and identically."""
    cfg: MoEConfig
    gate: torch.Tensor            # bf16 [E, H]
    bias: torch.Tensor            # f32 [E]
    seed: int
    device: str
    with_shared: bool
    dense: Optional[dict] = None  # Kimi-K3: latent projections, norm, bf16 shared expert

    def expert(self, e):
        """(w1, w3, w2), each (packed, scales), of routed expert e or SHARED; experts act
        on the latent width (the hidden width when there is no latent wrapper)."""
        c = self.cfg
        H, I = c.routed_expert_hidden_size, c.moe_intermediate_size
        idx = c.num_experts if e == SHARED else int(e)
        gen = torch.Generator(device=self.device)
        gen.manual_seed(self.seed * 1_000_003 + 7 + idx)
        return (random_mxfp4(gen, I, H, self.device), random_mxfp4(gen, I, H, self.device),
                random_mxfp4(gen, H, I, self.device))

    def source(self, layer: int, e, which: str):
        key = (e if e == SHARED else int(e))
        if getattr(self, "_cached_key", None) != key:           # the pool asks w1, w3, w2 in turn
            self._cached = self.expert(e)
            self._cached_key = key
        return self._cached[("w1", "w3", "w2").index(which)]

    def moe(self, device="cuda") -> LatentMoE:
        w = {"gate.weight": self.gate, "gate.e_score_correction_bias": self.bias, **(self.dense or {})}
        return LatentMoE(self.cfg, 0, w, self.source, fused=True, device=device)

    def nbytes_expert(self) -> int:
        c = self.cfg
        H, I = c.routed_expert_hidden_size, c.moe_intermediate_size
        return 3 * (I * H // 2 + I * H // 32)


def baseline_layer(seed: int = 0, E: int = 384, H: int = 7168, I: int = 2048, top_k: int = 8,
                   scale: float = 2.5, shared: bool = True, device="cuda") -> SyntheticLayer:
    """BASELINE configs[2]/[3]: 384 routed + 1 shared MXFP4 expert, hidden 7168,
    intermediate 2048, sigmoid top-8, renormalised weights x 2.5."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    cfg = MoEConfig(hidden_size=H, num_experts=E, num_experts_per_token=top_k,
                    moe_intermediate_size=I, routed_expert_hidden_size=H,
                    routed_scaling_factor=scale, moe_renormalize=True,
                    num_shared_experts=1 if shared else 0, activation="silu")
    gate = bf16_normal(gen, (E, H), 0.02, device)
    bias = torch.zeros(E, dtype=torch.float32, device=device)
    return SyntheticLayer(cfg, gate, bias, seed, device, shared)


def k3_layer(seed: int = 0, E: int = 896, H: int = 7168, L: int = 3584, I: int = 3072, I_shared: int = 3072,
             top_k: int = 16, scale: float = 2.5, device="cuda") -> SyntheticLayer:
    """A Kimi-K3 MoE layer (``air_llm/models/kimi_k3/moe.py:1-12``): 896 routed MXFP4
    experts, top-16, acting in a 3584-wide latent space (w1/w3: 3584 -> 3072, w2: 3072 ->
    3584) between bf16 ``routed_expert_down_proj`` [3584, 7168] and ``routed_expert_up_proj``
    [7168, 3584] with an RMSNorm, plus one bf16 shared expert [2 x 3072, 7168] on the
    original hidden; situ activation."""
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    cfg = MoEConfig(hidden_size=H, num_experts=E, num_experts_per_token=top_k,
                    moe_intermediate_size=I, routed_expert_hidden_size=L,
                    routed_scaling_factor=scale, moe_renormalize=True,
                    num_shared_experts=1, activation="situ")
    gate = bf16_normal(gen, (E, H), 0.02, device)
    bias = torch.zeros(E, dtype=torch.float32, device=device)
    norm = (1.0 + 0.1 * torch.randn(L, generator=gen, device=device)).to(torch.bfloat16).float()
    dense = {"routed_expert_down_proj.weight": bf16_normal(gen, (L, H), H ** -0.5, device),
             "routed_expert_up_proj.weight": bf16_normal(gen, (H, L), L ** -0.5, device),
             "routed_expert_norm.weight": norm,
             "shared_experts.gate_proj.weight": bf16_normal(gen, (I_shared, H), H ** -0.5, device),
             "shared_experts.up_proj.weight": bf16_normal(gen, (I_shared, H), H ** -0.5, device),
             "shared_experts.down_proj.weight": bf16_normal(gen, (H, I_shared), I_shared ** -0.5, device)}
    return SyntheticLayer(cfg, gate, bias, seed, device, False, dense)


def tokens(seed: int, M: int, H: int, device="cuda") -> torch.Tensor:
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    return bf16_normal(gen, (M, H), 1.0, device)
