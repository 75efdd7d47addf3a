"""Golden fixtures for the MoE input of a Kimi-K3 decoder layer, FROM THE REFERENCE'S
OWN CODE: ``x = rmsnorm(apply_attn_res(prefix_sum, block_residual, mlp_res_proj,
mlp_res_norm), post_attention_layernorm)`` (``k3ref/layers.py:83-96,321-322``, mirroring
``air_llm/models/kimi_k3/layer.py:120-121`` and ``ops.py:61-74``).

    python tests/golden/make_attnres_golden.py --ref /path/to/reference

Inputs are regenerated from seeds by ``inputs.attnres_inputs`` (numpy PCG64) and checked
by digest; the fixture stores the seeds, the digest and the reference's outputs.
"""
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE))
import inputs as I  # noqa: E402

CASES = {"small": dict(seed=3, N=5, B=3, H=512), "none": dict(seed=4, N=2, B=0, H=512),
         "k3": dict(seed=5, N=3, B=8, H=7168)}


def main(ref: str) -> None:
    sys.path.insert(0, ref)
    import torch
    import k3ref.layers as L
    out = {}
    for name, c in CASES.items():
        d = I.attnres_inputs(**c)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        x = L.apply_attn_res(t(d["prefix_sum"]), t(d["block_residual"]), t(I.as_f32(d["proj_bf16"])),
                             t(I.as_f32(d["res_norm_bf16"])), d["eps"])
        y = L.rmsnorm(x, t(I.as_f32(d["post_norm_bf16"])), d["eps"])
        out[f"{name}_digest"] = I.digest(d["prefix_sum"], d["block_residual"], d["proj_bf16"], d["res_norm_bf16"],
                                         d["post_norm_bf16"])
        out[f"{name}_attn"] = x.numpy().astype(np.float32)
        out[f"{name}_y"] = y.numpy().astype(np.float32)
        for k, v in c.items():
            out[f"{name}_{k}"] = v
    np.savez_compressed(HERE / "attn_res.npz", **out)
    print("wrote", HERE / "attn_res.npz")


if __name__ == "__main__":
    import argparse
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", type=Path, required=True, help="reference checkout (read-only)")
    main(str(ap.parse_args().ref))
