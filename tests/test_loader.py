"""Checkpoint reads (``loader.py``, ``csrc/k3_io.cu``) on a tiny Kimi-K3-format checkpoint.

CPU: the manifest equals the one the reference's own builder wrote for the same
checkpoint (``tests/golden/manifest_tiny.json``, ``tools/k3_manifest.py:97-156``); whole
tensors, rows, row blocks and expert projections read by the library's pread reader are
byte-identical to the arrays written; the one-read and two-read expert paths; errors.
GPU: reads straight into HBM, and a latent MoE layer built from the checkpoint equals the
same layer built from the arrays in memory.
"""
import gzip
import json
from pathlib import Path

import numpy as np
import pytest
import torch

import ckpt_util

GOLDEN = Path(__file__).resolve().parent / "golden" / "manifest_tiny.json"
P1 = "language_model.model.layers.1.block_sparse_moe."


@pytest.fixture(scope="module")
def ckpt(tmp_path_factory):
    d = tmp_path_factory.mktemp("k3ckpt")
    arrays = ckpt_util.make_tiny_k3(d / "ck", seed=0)
    from kimi_k3_mlx_macmini_b200 import loader
    loader.build_manifest(d / "ck", d / "manifest.jsonl.gz")
    return d, arrays


def _np(t):
    t = t.cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.uint16).numpy()
    return t.numpy()


def test_manifest_matches_reference_builder(ckpt):
    from kimi_k3_mlx_macmini_b200 import loader
    d, _ = ckpt
    g = json.loads(GOLDEN.read_text())
    meta, recs = loader.manifest_records(d / "ck")
    meta.pop("checkpoint")
    assert meta == g["meta"]
    assert recs == g["records"]
    # the written file round-trips through load_manifest
    m2, by_name = loader.load_manifest(d / "manifest.jsonl.gz")
    assert len(by_name) == len(recs) and m2["checkpoint"] == str((d / "ck").resolve())
    with gzip.open(d / "manifest.jsonl.gz", "rt") as fh:
        assert json.loads(fh.readline())["__meta__"] is True


def test_tensor_reads_are_byte_exact(ckpt):
    from kimi_k3_mlx_macmini_b200 import loader
    d, arrays = ckpt
    src = loader.TensorSource(d / "manifest.jsonl.gz")
    for name in (P1 + "gate.weight", P1 + "gate.e_score_correction_bias", "language_model.model.layers.0.self_attn.A_log",
                 P1 + "experts.5.w2.weight_packed"):
        t, dt = src.raw(name)
        assert dt == arrays[name][1]
        assert np.array_equal(_np(t), arrays[name][0])
    emb = arrays["language_model.model.embed_tokens.weight"][0]
    rows = src.rows("language_model.model.embed_tokens.weight", [3, 0, 511, 3])
    assert np.array_equal(_np(rows), emb[[3, 0, 511, 3]])
    blk = src.row_block("language_model.lm_head.weight", 100, 37)
    assert np.array_equal(_np(blk), arrays["language_model.lm_head.weight"][0][100:137])
    assert src.bytes_read > 0


@pytest.mark.parametrize("scale_first", [False, True])
def test_expert_source_one_or_two_reads(tmp_path, scale_first):
    """Adjacent packed + scale (one read) and the reverse order (two reads) give the
    same arrays; the counters add the projection's bytes."""
    from kimi_k3_mlx_macmini_b200 import loader
    arrays = ckpt_util.make_tiny_k3(tmp_path / "ck", seed=3, scale_first=scale_first)
    loader.build_manifest(tmp_path / "ck", tmp_path / "m.jsonl.gz")
    src = loader.TensorSource(tmp_path / "m.jsonl.gz")
    for e in (0, 7):
        for which in ("w1", "w3", "w2"):
            pk, sc = src.expert_source(1, e, which)
            assert np.array_equal(pk.numpy(), arrays[f"{P1}experts.{e}.{which}.weight_packed"][0])
            assert np.array_equal(sc.numpy(), arrays[f"{P1}experts.{e}.{which}.weight_scale"][0])
    assert src.experts_loaded == 6
    assert src.expert_bytes == 6 * (128 * 64 + 128 * 4)


def test_read_ranges_merges_and_splits(tmp_path):
    """Many ranges, adjacent and not, into one buffer; a range larger than a read task
    (8 MiB) is split across threads."""
    from kimi_k3_mlx_macmini_b200 import loader
    rng = np.random.default_rng(1)
    data = rng.integers(0, 256, 20 << 20, dtype=np.uint8)
    f = tmp_path / "blob.bin"
    f.write_bytes(data.tobytes())
    out = np.zeros(20 << 20, np.uint8)
    base = out.ctypes.data
    ranges = [(0, 1000, base), (1000, 24, base + 1000), (5000, 17, base + 5000), (4096, 904, base + 4096),
              (1 << 20, 18 << 20, base + (1 << 20))]
    got = loader.read_ranges(f, ranges, threads=4)
    assert got == sum(r[1] for r in ranges)
    for off, n, _ in ranges:
        assert np.array_equal(out[off:off + n], data[off:off + n])
    assert not out[1024:4096].any()                    # untouched gap stays zero


def test_read_errors(tmp_path, ckpt):
    from kimi_k3_mlx_macmini_b200 import loader
    d, _ = ckpt
    buf = np.zeros(16, np.uint8)
    with pytest.raises(OSError):
        loader.read_ranges(tmp_path / "missing.bin", [(0, 16, buf.ctypes.data)])
    f = tmp_path / "small.bin"
    f.write_bytes(b"x" * 10)
    with pytest.raises(ValueError):                     # past the end of the file
        loader.read_ranges(f, [(4, 16, buf.ctypes.data)])
    with pytest.raises(FileNotFoundError):
        loader.TensorSource(tmp_path / "no_manifest.jsonl.gz")
    src = loader.TensorSource(d / "manifest.jsonl.gz")
    with pytest.raises(KeyError):
        src.expert_source(1, 99, "w1")
    # a projection whose scale bytes leave 2..252 is refused, as the reference refuses it
    bad = tmp_path / "bad"
    ckpt_util.make_tiny_k3(bad, seed=0)
    _, recs = loader.manifest_records(bad)
    r = next(x for x in recs if x["name"] == P1 + "experts.2.w3.weight_scale")
    with (bad / r["file"]).open("r+b") as fh:
        fh.seek(r["offset"] + 5)
        fh.write(bytes([255]))
    loader.build_manifest(bad, tmp_path / "bad.jsonl.gz")
    with pytest.raises(ValueError, match="scale range"):
        loader.TensorSource(tmp_path / "bad.jsonl.gz").expert_source(1, 2, "w3")


@pytest.mark.gpu
def test_reads_to_device(ckpt):
    from kimi_k3_mlx_macmini_b200 import loader
    d, arrays = ckpt
    src = loader.TensorSource(d / "manifest.jsonl.gz")
    st = loader.pinned_empty(16 << 10)                  # two 8 KiB halves: many round trips
    for name in (P1 + "shared_experts.down_proj.weight", "language_model.lm_head.weight",
                 P1 + "gate.e_score_correction_bias"):
        t = src.tensor(name, staging=st)
        assert t.is_cuda and np.array_equal(_np(t), arrays[name][0])
    w = src.moe_weights(1)
    assert set(w) == set(loader.MOE_KEYS)
    assert np.array_equal(_np(w["gate.weight"]), arrays[P1 + "gate.weight"][0])


@pytest.mark.gpu
def test_latent_layer_from_checkpoint(k3, ckpt):
    """LatentMoE built from the manifest (dense weights read into HBM, experts through
    expert_source) equals the layer built from the written arrays, bit for bit."""
    from kimi_k3_mlx_macmini_b200 import loader
    d, arrays = ckpt
    c = ckpt_util.TINY
    cfg = k3.MoEConfig(hidden_size=c["hidden_size"], num_experts=c["num_experts"],
                       num_experts_per_token=c["num_experts_per_token"],
                       moe_intermediate_size=c["moe_intermediate_size"],
                       routed_expert_hidden_size=c["routed_expert_hidden_size"],
                       routed_scaling_factor=c["routed_scaling_factor"], activation="situ")
    src = loader.TensorSource(d / "manifest.jsonl.gz")
    moe_disk = k3.LatentMoE(cfg, 1, src.moe_weights(1), src.expert_source)

    def mem(k):
        a, dt = arrays[P1 + k]
        t = torch.from_numpy(a.copy()).cuda()
        return t.view(torch.bfloat16) if dt == "BF16" else t

    def mem_src(layer, e, which):
        return tuple(torch.from_numpy(arrays[f"{P1}experts.{e}.{which}.{k}"][0].copy())
                     for k in ("weight_packed", "weight_scale"))
    moe_mem = k3.LatentMoE(cfg, 1, {k: mem(k) for k in loader.MOE_KEYS}, mem_src)
    x = (torch.randn((5, c["hidden_size"]), device="cuda") * 0.5).to(torch.bfloat16)
    y1, r1 = moe_disk(x, return_router=True)
    y2, r2 = moe_mem(x, return_router=True)
    assert torch.equal(r1.expert_indices, r2.expert_indices)
    assert torch.equal(y1, y2)
