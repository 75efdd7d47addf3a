"""Generate the golden fixtures in this folder FROM THE REFERENCE'S OWN CODE.

    python tests/golden/make_golden.py --ref /path/to/kimi-k3-mlx-macmini

Runs in a container where the reference checkout is importable (its ``k3ref`` torch/CPU
oracle, ``tools/make_synthetic_k3.py`` and the third-party ``compressed_tensors``
decoder it was validated against). The GPU box never runs this script: the tests read
only the committed ``*.npz`` outputs. Large inputs are not stored; they are regenerated
from seeds by ``inputs.py`` and checked against the stored sha256 digest.

What each fixture pins (reference file:line):
  codec_kat.npz    all 256 bytes / 16 codes at scale 127 and 0x22 x all 256 scale bytes,
                   decoded by ``k3ref/weights.py:29-37`` and by compressed_tensors
                   ``unpack_fp4_from_uint8`` (``archive/p0/p0_3_mxfp4.py:44-72``)
  matvec_kat.npz   the synthetic fused-kernel gate of ``tests/test_mxfp4_kernel.py:42-54``
                   (rng(0), N=128, K=256, scales [100,140), M=1,2,4, fp64 expected)
  encoder.npz      ``tools/make_synthetic_k3.py:87-110`` encode_mxfp4 outputs
  config0.npz      one expert FFN through ``k3ref`` LatentMoE.expert_forward
  moe_*.npz        whole MoE blocks through ``k3ref`` LatentMoE.route / __call__
  mini_k3.npz      layer 1 of the reference's own synthetic mini-K3 checkpoint
                   (``tools/make_synthetic_k3.py:152-252``, seed 0) through ``k3ref``
"""
from __future__ import annotations

import argparse
import contextlib
import json
import struct
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import inputs as I  # noqa: E402


def _import_reference(ref: Path):
    sys.path.insert(0, str(ref))
    sys.path.insert(0, str(ref / "tools"))
    import torch  # noqa: F401
    import k3ref.layers as L
    import k3ref.weights as W
    import make_synthetic_k3 as MS
    return L, W, MS


def _cfg(L, *, H, E, k, I_, latent, scale, renorm=True, beta=4.0, lbeta=25.0):
    return L.K3Config(hidden_size=H, num_hidden_layers=2, rms_norm_eps=1e-5,
                      num_attention_heads=1, num_key_value_heads=1, q_lora_rank=1,
                      kv_lora_rank=1, qk_nope_head_dim=1, qk_rope_head_dim=1, v_head_dim=1,
                      mla_use_output_gate=False, num_experts=E, num_experts_per_token=k,
                      num_shared_experts=1, moe_intermediate_size=I_,
                      routed_expert_hidden_size=latent, routed_scaling_factor=scale,
                      moe_renormalize=renorm, first_k_dense_replace=1, intermediate_size=I_,
                      attn_res_block_size=2, situ_beta=beta, situ_linear_beta=lbeta,
                      kda_num_heads=1, kda_head_dim=1, kda_conv_size=4,
                      kda_gate_lower_bound=-5.0)


class FakeStore:
    """Stands in for ``k3ref.weights.WeightStore``: ``get`` returns fp32 tensors by name,
    ``expert`` decodes MXFP4 with the reference decoder (``weights.py:117-122``)."""

    def __init__(self, W, tensors: dict, experts: list):
        import torch
        self._t, self._e, self._W, self._torch = tensors, experts, W, torch

    def get(self, name):
        key = name.split("block_sparse_moe.")[-1]
        return self._torch.from_numpy(np.ascontiguousarray(self._t[key], dtype=np.float32))

    def expert(self, layer, e, w):
        p, s = self._e[e][{"w1": 0, "w3": 1, "w2": 2}[w]]
        return self._torch.from_numpy(self._W.decode_mxfp4(np.ascontiguousarray(p), np.ascontiguousarray(s)))


@contextlib.contextmanager
def baseline_substitutions(L):
    """BASELINE.json's layer: SiLU-and-mul instead of situ, and no latent rmsnorm.
    (The identity down/up projections are passed as weights.)"""
    import torch.nn.functional as F
    saved = L.situ, L.rmsnorm

    def silu_and_mul(gate_up, beta, linear_beta):
        d = gate_up.shape[-1] // 2
        return F.silu(gate_up[..., :d].float()) * gate_up[..., d:].float()

    L.situ = silu_and_mul
    L.rmsnorm = lambda x, w, eps: x
    try:
        yield
    finally:
        L.situ, L.rmsnorm = saved


def _router_arrays(r):
    idx = r.expert_indices.numpy()
    o = np.argsort(idx, axis=-1)
    return {"idx_sorted": np.sort(idx, axis=-1).astype(np.int32),
            "w_canon": np.take_along_axis(r.expert_weights.numpy(), o, axis=-1).astype(np.float32),
            "raw": r.raw_scores.numpy().astype(np.float32),
            "corrected": r.corrected_scores.numpy().astype(np.float32)}


def make_codec(L, W, out):
    from compressed_tensors.compressors.nvfp4.helpers import unpack_fp4_from_uint8
    import torch
    p256 = np.arange(256, dtype=np.uint8).reshape(16, 16)
    s127 = np.full((16, 1), 127, dtype=np.uint8)
    ps = np.full((256, 16), 0x22, dtype=np.uint8)
    sall = np.arange(256, dtype=np.uint8).reshape(256, 1)
    ct = unpack_fp4_from_uint8(torch.from_numpy(p256.copy()), 16, 32, dtype=torch.float32).numpy()
    e = np.arange(1, 255)
    np.savez_compressed(out / "codec_kat.npz",
                        all256_packed=p256, all256_scales=s127,
                        all256_decoded=W.decode_mxfp4(p256, s127), all256_ct=ct.astype(np.float32),
                        scales_packed=ps, scales_bytes=sall,
                        scales_decoded=W.decode_mxfp4(ps, sall),
                        scale_bytes_1_254=e.astype(np.uint8),
                        scale_values_1_254=np.ldexp(np.ones(254, np.float32), e - 127).astype(np.float32))


def make_matvec(W, out):
    rng = np.random.default_rng(0)
    N, K = 128, 256
    packed = rng.integers(0, 256, size=(N, K // 2), dtype=np.uint8)
    scales = rng.integers(100, 140, size=(N, K // 32), dtype=np.uint8)
    Wd = W.decode_mxfp4(packed, scales)
    d = {"packed": packed, "scales": scales}
    for M in (1, 2, 4):
        x = rng.standard_normal((M, K)).astype(np.float32)
        d[f"x{M}"] = x
        d[f"want{M}"] = x.astype(np.float64) @ Wd.T.astype(np.float64)
    np.savez_compressed(out / "matvec_kat.npz", **d)


def make_encoder(MS, out):
    rng = np.random.default_rng(3)
    a = (rng.standard_normal((64, 96)) * 0.05).astype(np.float32)     # selftest input
    rng = np.random.default_rng(5)
    b = (rng.standard_normal((32, 256)) * 10.0 ** rng.uniform(-3, 3, size=(32, 1))).astype(np.float32)
    b[3] = 0.0                                                       # all-zero row
    b[7, :32] = 0.0                                                  # all-zero group
    pa, sa = MS.encode_mxfp4(a)
    pb, sb = MS.encode_mxfp4(b)
    np.savez_compressed(out / "encoder.npz", a=a, a_packed=pa, a_scales=sa,
                        b=b, b_packed=pb, b_scales=sb)


def make_config0(L, W, out):
    import torch
    d = I.config0_inputs(seed=0)
    H, I_ = 1024, 512
    cfg = _cfg(L, H=H, E=1, k=1, I_=I_, latent=H, scale=1.0)
    tensors = {k: np.zeros((1, 1), np.float32) for k in
               ("gate.weight", "gate.e_score_correction_bias", "routed_expert_down_proj.weight",
                "routed_expert_up_proj.weight", "routed_expert_norm.weight",
                "shared_experts.gate_proj.weight", "shared_experts.up_proj.weight",
                "shared_experts.down_proj.weight")}
    ws = FakeStore(W, tensors, [(d["w1"], d["w3"], d["w2"])])
    with baseline_substitutions(L):
        moe = L.LatentMoE(cfg, 1, ws)
        x = torch.from_numpy(I.as_f32(d["x_bf16"]))
        y = moe.expert_forward(x, 0).numpy()
    np.savez_compressed(out / "config0.npz", seed=0, digest=I.digest(d["x_bf16"], *d["w1"], *d["w3"], *d["w2"]),
                        y=y.astype(np.float32))


def make_moe(L, W, out, name, *, seed, M, H, I_, E, k, scale, bias_std):
    import torch
    d = I.moe_inputs(seed, M, H, I_, E, shared=True, bias_std=bias_std)
    sh = d["shared"]
    tensors = {
        "gate.weight": I.as_f32(d["gate_bf16"]),
        "gate.e_score_correction_bias": d["bias"],
        "routed_expert_down_proj.weight": np.eye(H, dtype=np.float32),
        "routed_expert_up_proj.weight": np.eye(H, dtype=np.float32),
        "routed_expert_norm.weight": np.ones(H, np.float32),
        "shared_experts.gate_proj.weight": W.decode_mxfp4(*sh[0]),
        "shared_experts.up_proj.weight": W.decode_mxfp4(*sh[1]),
        "shared_experts.down_proj.weight": W.decode_mxfp4(*sh[2]),
    }
    cfg = _cfg(L, H=H, E=E, k=k, I_=I_, latent=H, scale=scale)
    ws = FakeStore(W, tensors, d["experts"])
    flat = [a for tr in d["experts"] for pair in tr for a in pair] + [a for pair in sh for a in pair]
    with baseline_substitutions(L):
        moe = L.LatentMoE(cfg, 1, ws)
        x = torch.from_numpy(I.as_f32(d["x_bf16"])).reshape(1, M, H)
        y, r = moe(x, return_router=True)
    np.savez_compressed(out / f"{name}.npz", seed=seed, M=M, H=H, I=I_, E=E, k=k, scale=scale,
                        bias_std=bias_std,
                        digest=I.digest(d["x_bf16"], d["gate_bf16"], d["bias"], *flat),
                        y=y.reshape(M, H).numpy().astype(np.float32), **_router_arrays(r))


def make_latent(L, W, out, *, seed=11, M=3, H=256, Lt=128, I_=128, E=16, k=4, S=128):
    import torch
    d = I.latent_moe_inputs(seed, M, H, Lt, I_, E, S)
    tensors = {
        "gate.weight": I.as_f32(d["gate_bf16"]),
        "gate.e_score_correction_bias": d["bias"],
        "routed_expert_down_proj.weight": I.as_f32(d["down_bf16"]),
        "routed_expert_up_proj.weight": I.as_f32(d["up_bf16"]),
        "routed_expert_norm.weight": I.as_f32(d["norm_bf16"]),
        "shared_experts.gate_proj.weight": I.as_f32(d["sh_gate_bf16"]),
        "shared_experts.up_proj.weight": I.as_f32(d["sh_up_bf16"]),
        "shared_experts.down_proj.weight": I.as_f32(d["sh_down_bf16"]),
    }
    cfg = _cfg(L, H=H, E=E, k=k, I_=I_, latent=Lt, scale=1.0)
    ws = FakeStore(W, tensors, d["experts"])
    moe = L.LatentMoE(cfg, 1, ws)
    x = torch.from_numpy(I.as_f32(d["x_bf16"])).reshape(1, M, H)
    y, r = moe(x, return_router=True)
    flat = [a for tr in d["experts"] for pair in tr for a in pair]
    keys = ("x_bf16", "gate_bf16", "bias", "down_bf16", "up_bf16", "norm_bf16",
            "sh_gate_bf16", "sh_up_bf16", "sh_down_bf16")
    np.savez_compressed(out / "moe_latent.npz", seed=seed, M=M, H=H, L=Lt, I=I_, E=E, k=k, S=S,
                        digest=I.digest(*[d[q] for q in keys], *flat),
                        y=y.reshape(M, H).numpy().astype(np.float32), **_router_arrays(r))


def _read_safetensors(path: Path) -> dict:
    raw = path.read_bytes()
    n = struct.unpack("<Q", raw[:8])[0]
    hdr = json.loads(raw[8:8 + n])
    dt = {"BF16": np.uint16, "F32": np.float32, "U8": np.uint8}
    out = {}
    for name, t in hdr.items():
        if name == "__metadata__":
            continue
        s, e = t["data_offsets"]
        out[name] = (np.frombuffer(raw[8 + n + s:8 + n + e], dtype=dt[t["dtype"]]).reshape(t["shape"]),
                     t["dtype"])
    return out


def make_mini_k3(L, W, MS, out, layer=1):
    import torch
    with tempfile.TemporaryDirectory() as tmp:
        MS.build(Path(tmp), seed=0)
        cfg_json = json.loads((Path(tmp) / "config.json").read_text())["text_config"]
        nl = cfg_json["num_hidden_layers"]
        ts = _read_safetensors(Path(tmp) / f"model-{layer + 1:05d}-of-{nl + 1:05d}.safetensors")
    pre = f"language_model.model.layers.{layer}.block_sparse_moe."
    E = cfg_json["num_experts"]
    tensors, store = {}, {}
    for name, (a, dtype) in ts.items():
        if not name.startswith(pre) or ".experts." in name:
            continue
        key = name[len(pre):]
        store[key] = a
        tensors[key] = I.as_f32(a) if dtype == "BF16" else a.astype(np.float32)
    experts = []
    for e in range(E):
        trip = []
        for w in ("w1", "w3", "w2"):
            p = ts[f"{pre}experts.{e}.{w}.weight_packed"][0]
            s = ts[f"{pre}experts.{e}.{w}.weight_scale"][0]
            store[f"e{e}.{w}.packed"], store[f"e{e}.{w}.scales"] = p, s
            trip.append((p, s))
        experts.append(tuple(trip))
    c = cfg_json
    cfg = _cfg(L, H=c["hidden_size"], E=E, k=c["num_experts_per_token"], I_=c["moe_intermediate_size"],
               latent=c["routed_expert_hidden_size"], scale=c["routed_scaling_factor"],
               renorm=c["moe_renormalize"], beta=c["activation_situ_beta"],
               lbeta=c["activation_situ_linear_beta"])
    moe = L.LatentMoE(cfg, layer, FakeStore(W, tensors, experts))
    rng = np.random.default_rng(7)
    M = 4
    xb = I.bf16_normal(rng, (M, c["hidden_size"]))
    y, r = moe(torch.from_numpy(I.as_f32(xb)).reshape(1, M, -1), return_router=True)
    meta = {k: c[k] for k in ("hidden_size", "num_experts", "num_experts_per_token",
                              "moe_intermediate_size", "routed_expert_hidden_size",
                              "routed_scaling_factor", "moe_renormalize", "activation_situ_beta",
                              "activation_situ_linear_beta", "rms_norm_eps")}
    np.savez_compressed(out / "mini_k3.npz", meta=json.dumps(meta), x_bf16=xb,
                        y=y.reshape(M, -1).numpy().astype(np.float32), **_router_arrays(r),
                        **{"t." + k: v for k, v in store.items()})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, required=True, help="reference checkout (read-only)")
    a = ap.parse_args()
    L, W, MS = _import_reference(a.ref)
    make_codec(L, W, HERE)
    make_matvec(W, HERE)
    make_encoder(MS, HERE)
    make_config0(L, W, HERE)
    make_moe(L, W, HERE, "moe_small_m1", seed=1, M=1, H=256, I_=128, E=16, k=4, scale=2.5, bias_std=0.0)
    make_moe(L, W, HERE, "moe_small_m5", seed=2, M=5, H=256, I_=128, E=16, k=4, scale=2.5, bias_std=0.05)
    make_moe(L, W, HERE, "moe_small_m8", seed=3, M=8, H=512, I_=256, E=32, k=8, scale=2.5, bias_std=0.0)
    make_latent(L, W, HERE)
    make_mini_k3(L, W, MS, HERE)
    for f in sorted(HERE.glob("*.npz")):
        print(f"{f.name:20s} {f.stat().st_size / 1024:8.1f} KiB")


if __name__ == "__main__":
    main()
