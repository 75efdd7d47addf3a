"""Streamed-expert decode (BASELINE configs[4] semantics): routed experts copied from a
pinned host store into staging slots on a side stream must give the resident layer's
output."""
import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O

pytestmark = pytest.mark.gpu


def test_streamed_layer_matches_resident(k3):
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.moe import SHARED
    from kimi_k3_mlx_macmini_b200.stream import HostExpertStore, StreamedMoE
    lay = synthetic.baseline_layer(seed=21, E=16, H=1024, I=512, top_k=4)
    store = HostExpertStore(16, lay.expert)
    w = {"gate.weight": lay.gate, "gate.e_score_correction_bias": lay.bias}
    sm = StreamedMoE(lay.cfg, 0, w, store, lambda: lay.expert(SHARED))
    ref_layer = lay.moe()
    for seed in (1, 2, 3):                              # staging slots are reused call to call
        x = synthetic.tokens(seed, 1, 1024)
        y = sm(x)
        ref = ref_layer(x)
        assert O.rel_l2(y.cpu().numpy(), ref.float().cpu().numpy()) < 1e-6
