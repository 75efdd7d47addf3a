"""B200-native (sm_100a) MXFP4 quantized-expert path of sjdthree/kimi-k3-mlx-macmini.

Python mirrors of the reference interfaces over the ``libk3b200.so`` C ABI
(``include/k3b200.h``):

* ``mxfp4``: ``mxfp4_matvec_fused``, ``expert_projection``, ``decode_mxfp4``,
  ``decode_scale``, ``assert_scales_representable``, ``mxfp4_matvec``;
* ``moe``: ``LatentMoE``, ``RouterResult``, ``MoEConfig``.
"""
from .mxfp4 import (assert_scales_representable, decode_mxfp4, decode_mxfp4_mlx,  # noqa: F401
                    decode_scale, expert_projection, mxfp4_matvec, mxfp4_matvec_fused)
from .moe import LatentMoE, MoEConfig, RouterResult  # noqa: F401

__all__ = ["mxfp4_matvec_fused", "expert_projection", "decode_mxfp4", "decode_mxfp4_mlx",
           "decode_scale", "assert_scales_representable", "mxfp4_matvec", "LatentMoE",
           "MoEConfig", "RouterResult"]
