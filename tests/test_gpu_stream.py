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


def test_streamed_layer_from_checkpoint_files(k3, tmp_path):
    """The disk tier: routed experts read from checkpoint shards on every call (one pread
    per contiguous run of an expert's six tensors, copy, re-layout on the GPU) give the
    same output, bit for bit, as the pinned-host tier over the same expert bytes."""
    import ckpt_util
    from kimi_k3_mlx_macmini_b200 import loader, synthetic
    from kimi_k3_mlx_macmini_b200.stream import DiskExpertStore, HostExpertStore, StreamedMoE
    H, E = 512, 8                                       # the pairs kernels want H, I % 512 == 0
    arrays = ckpt_util.make_tiny_k3(tmp_path / "ck", seed=5, hidden_size=H, routed_expert_hidden_size=H,
                                    moe_intermediate_size=H)
    loader.build_manifest(tmp_path / "ck", tmp_path / "m.jsonl.gz")
    src = loader.TensorSource(tmp_path / "m.jsonl.gz")
    p = "language_model.model.layers.1.block_sparse_moe."

    def expert(e):
        return tuple(tuple(torch.from_numpy(arrays[f"{p}experts.{e}.{w}.{k}"][0].copy()).cuda()
                           for k in ("weight_packed", "weight_scale")) for w in ("w1", "w3", "w2"))
    cfg = k3.MoEConfig(hidden_size=H, num_experts=E, num_experts_per_token=2, moe_intermediate_size=H,
                       routed_expert_hidden_size=H, routed_scaling_factor=2.5, activation="silu")
    w = {"gate.weight": torch.from_numpy(arrays[p + "gate.weight"][0].copy()).cuda().view(torch.bfloat16),
         "gate.e_score_correction_bias": torch.from_numpy(arrays[p + "gate.e_score_correction_bias"][0].copy()).cuda()}
    shared = lambda: expert(E - 1)  # noqa: E731 -- any MXFP4 triple of the right shape
    disk = StreamedMoE(cfg, 1, w, DiskExpertStore(src, 1, E), shared)
    host = StreamedMoE(cfg, 1, w, HostExpertStore(E, expert), shared)
    for seed in (1, 2, 3):
        x = synthetic.tokens(seed, 1, H)
        assert torch.equal(disk(x), host(x))
    per_expert = 3 * (H * H // 2 + H * H // 32)
    assert disk.store.bytes_read % per_expert == 0 and disk.store.bytes_read >= 3 * per_expert
