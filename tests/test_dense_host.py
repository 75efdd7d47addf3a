"""Host-side pieces of the dense path (``dense.py``) that run without a GPU: the GEMM
helper's fp32 result for shapes the tensor-core GEMM does not take, rmsnorm and the gate/up activations against numpy
(``ops.py:11-28``), and the dispatch between the library matvec and the GEMM path."""
import numpy as np
import torch

from oracle import mxfp4_oracle as O


def test_mm_f32_and_norm_and_activation():
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import dense as D
    g = torch.Generator().manual_seed(0)
    x = torch.randn((12, 96), generator=g)
    w = (torch.randn((40, 96), generator=g) * 0.1).to(torch.bfloat16)
    want = x.double().numpy() @ w.double().numpy().T
    assert O.rel_l2(D._mm_f32(x, w).numpy(), want) < 1e-6
    nw = 1.0 + 0.1 * torch.randn(96, generator=g)
    assert O.rel_l2(D._rmsnorm(x, nw, 1e-5).numpy(), O.rmsnorm(x.numpy(), nw.numpy(), 1e-5)) < 1e-6
    gg, uu = torch.randn((5, 7), generator=g) * 3, torch.randn((5, 7), generator=g) * 3
    for kind, act, lb in ((L.K3_ACT_SILU, "silu", None), (L.K3_ACT_SITU, "situ", 25.0), (L.K3_ACT_SITU, "situ", None)):
        got = D._activation(kind, gg, uu, 4.0, -1.0 if lb is None else lb).numpy()
        assert O.rel_l2(got, O.activation(gg.numpy(), uu.numpy(), act, 4.0, lb)) < 1e-6


def test_device_weight_and_dispatch():
    from kimi_k3_mlx_macmini_b200 import dense as D
    w = torch.randn((64, 32)).to(torch.bfloat16).float()           # bf16-representable fp32
    assert D.device_weight(w, "cpu").dtype == torch.bfloat16
    assert D.device_weight(torch.randn((64, 32)), "cpu").dtype == torch.float32   # not representable
    wb = torch.zeros((64, 32), dtype=torch.bfloat16)
    assert D._native_ok([(wb, torch.zeros((8, 32)), None, 0.0)])
    assert not D._native_ok([(wb, torch.zeros((9, 32)), None, 0.0)])             # > 8 tokens: GEMM path
    assert not D._native_ok([(wb[:, :20], torch.zeros((2, 20)), None, 0.0)])      # K % 8 != 0
    assert not D._native_ok([(wb.float(), torch.zeros((2, 32)), None, 0.0)])      # fp32 weights
    assert D._native_ok([(wb, torch.zeros((2, 64)), None, 0.0, True)])            # act_input segment


def test_dense_seg_struct_matches_header():
    """The ctypes mirror of k3_dense_seg carries every field of the header's struct, in
    order, ending with act_input (ABI 3)."""
    import re
    from pathlib import Path
    from kimi_k3_mlx_macmini_b200 import _lib as L
    hdr = (Path(__file__).resolve().parents[1] / "include" / "k3b200.h").read_text()
    body = re.search(r"typedef struct k3_dense_seg \{(.*?)\} k3_dense_seg;", hdr, re.S).group(1)
    names = re.findall(r"(\w+);", body)
    assert names == [f[0] for f in L.K3DenseSeg._fields_]
    assert names[-1] == "act_input"
