"""The caller step around the MoE in a Kimi-K3 decoder layer.

``DecoderLayer.__call__`` (``air_llm/models/kimi_k3/layer.py:111-126``) feeds its MoE with

    x = rmsnorm(apply_attn_res(prefix_sum, block_residual, mlp_res_proj, mlp_res_norm),
                post_attention_layernorm)
    x, router = mlp(x, return_router=True)
    prefix_sum = prefix_sum + x

where ``apply_attn_res`` (``ops.py:61-74``) is a softmax attention over the layer
block's residual checkpoints plus the running sum. ``attn_res_norm`` is that input in one
library launch (``k3_attn_res_norm``); ``MoEBlock`` is the whole MoE half of the layer.
"""
from __future__ import annotations

from typing import Optional

import torch

from . import _lib as L

NORM_KEYS = ("post_attention_layernorm.weight", "mlp_res_proj.weight", "mlp_res_norm.weight")


def attn_res_norm(prefix_sum: torch.Tensor, block_residual: Optional[torch.Tensor], res_proj: torch.Tensor,
                  res_norm: torch.Tensor, post_norm: torch.Tensor, eps: float,
                  out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """rmsnorm(apply_attn_res(prefix_sum [N, H], block_residual [N, B, H]), post_norm)
    (``layer.py:120-121``); B may be 0 (``block_residual`` None or empty)."""
    L.require_cuda(prefix_sum, "prefix_sum")
    ps = prefix_sum.reshape(-1, prefix_sum.shape[-1]).float().contiguous()
    N, H = ps.shape
    nb = 0 if block_residual is None else block_residual.shape[1]
    br = None if nb == 0 else block_residual.float().contiguous()
    f32 = lambda t: t.reshape(-1).float().contiguous()  # noqa: E731
    proj, rn, pn = f32(res_proj), f32(res_norm), f32(post_norm)
    if proj.numel() != H or rn.numel() != H or pn.numel() != H:
        raise ValueError("attn_res_norm: the weights must have the hidden size")
    out = torch.empty((N, H), dtype=out_dtype, device=ps.device)
    L.check(L.load_library().k3_attn_res_norm(ps.data_ptr(), None if br is None else br.data_ptr(), nb, N, H,
                                              proj.data_ptr(), rn.data_ptr(), pn.data_ptr(), float(eps),
                                              out.data_ptr(), L.dtype_code(out), L.stream_of(ps)),
            "k3_attn_res_norm")
    return out.reshape(*prefix_sum.shape[:-1], H)


class MoEBlock:
    """The MoE half of ``DecoderLayer.__call__`` (``layer.py:119-126``) over a
    ``LatentMoE``: returns (new prefix_sum, RouterResult)."""

    def __init__(self, cfg, mlp, norms: dict, device="cuda"):
        self.cfg, self.mlp = cfg, mlp
        dev = torch.device(device)
        self.post_norm, self.res_proj, self.res_norm = (torch.as_tensor(norms[k]).to(dev).float().contiguous()
                                                        for k in NORM_KEYS)

    def __call__(self, prefix_sum: torch.Tensor, block_residual: Optional[torch.Tensor]):
        x = attn_res_norm(prefix_sum, block_residual, self.res_proj, self.res_norm, self.post_norm,
                          float(self.cfg.rms_norm_eps))
        y, router = self.mlp(x, return_router=True)
        return prefix_sum.float() + y, router


__all__ = ["attn_res_norm", "MoEBlock", "NORM_KEYS"]
