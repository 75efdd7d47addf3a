"""The fused decode router's top-k (``route_fused_kernel``) on rows with exact ties.

Gate rows (and score-correction biases) repeat with period D, so every score occurs about
E/D times and the k-th largest corrected score is usually shared by several experts. The
reference selects with an argpartition of the corrected scores and gathers the weights
from the raw scores (``air_llm/models/kimi_k3/moe.py:65-76``); this library fixes the
choice among equal scores to the lowest index, the order of k rounds of argmax on
(corrected desc, index asc), and returns the k experts in that order. The expected
selection is built from the scores of the separate router entry point (``k3_moe_route``);
equal gate rows give equal scores in either kernel, and a row whose boundary gap between
distinct scores is within float rounding is skipped.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

H, I_ = 1024, 512


def _tied_moe(E, k, D, seed):
    from kimi_k3_mlx_macmini_b200 import synthetic
    lay = synthetic.baseline_layer(seed=seed, E=E, H=H, I=I_, top_k=k, scale=2.5)
    rep = torch.arange(E, device="cuda") % D
    lay.gate = lay.gate[rep].contiguous()
    g = torch.Generator(device="cuda").manual_seed(seed + 1)
    lay.bias = (torch.rand(D, generator=g, device="cuda") * 0.1)[rep].contiguous()
    moe = lay.moe()
    assert moe.fused and moe.tiled
    return moe


def _expected(cor, raw, k, scale, tol=1e-5):
    """Per token: the k experts by (corrected desc, index asc) and their weights, or None
    where two distinct scores among the top k + 1 groups are within float rounding."""
    out = []
    E = cor.shape[1]
    for c, r in zip(cor, raw):
        order = np.lexsort((np.arange(E), -c))
        vals = np.unique(c[order[:k]])
        nxt = c[order][c[order] < vals.min()]
        levels = np.concatenate([vals, nxt[:1]])
        if len(levels) > 1 and np.min(np.diff(np.sort(levels))) < tol * np.abs(levels).max():
            out.append(None)
            continue
        sel = order[:k]
        w = (r[sel] / (r[sel].sum() + 1e-20) if k > 1 else r[sel]) * scale    # no renorm at k = 1
        out.append((sel, w))
    return out


@pytest.mark.parametrize("E,k,M,D", [
    (96, 6, 3, 11),      # 3 keys per lane
    (384, 8, 8, 37),     # the BASELINE router width
    (640, 16, 5, 41),
    (896, 16, 1, 53),    # the Kimi-K3 router width
    (896, 16, 8, 29),
    (1024, 16, 4, 61),   # the widest router the kernels take
    (520, 1, 2, 19),     # k = 1 in the counting form
])
def test_fused_topk_lowest_index_on_ties(k3, E, k, M, D):
    moe = _tied_moe(E, k, D, seed=E + M)
    checked = 0
    for trial in range(3):
        g = torch.Generator(device="cuda").manual_seed(1000 * trial + E + M)
        x = torch.randn((M, H), generator=g, device="cuda").to(torch.bfloat16)
        _, idx, w = moe._fused_decode(x)
        r = moe.route(x)
        cor, raw = r.corrected_scores.cpu().numpy(), r.raw_scores.cpu().numpy()
        for e in range(E):                      # equal gate rows score equally
            assert np.array_equal(cor[:, e], cor[:, e % D])
        exp = _expected(cor, raw, k, 2.5)
        got_i, got_w = idx.cpu().numpy(), w.cpu().numpy()
        for t in range(M):
            if exp[t] is None:
                continue
            sel, ww = exp[t]
            assert np.array_equal(got_i[t], sel), f"token {t}: {got_i[t]} vs {sel}"
            np.testing.assert_allclose(got_w[t], ww, rtol=1e-5, atol=1e-7)
            checked += 1
    assert checked >= 2 * M


@pytest.mark.parametrize("E,k", [(384, 8), (896, 16)])
def test_fused_topk_nan_row_gives_distinct_valid_experts(k3, E, k):
    """A row of NaN scores (NaN input) has no top-k: the router flags the call invalid and
    still hands the expert kernels k distinct in-range experts (NaN ranks below every
    number, lowest index first), in the register and the counting form alike."""
    M = 2
    moe = _tied_moe(E, k, E, seed=5)
    x = torch.randn((M, H), device="cuda").to(torch.bfloat16)
    x[1] = float("nan")
    _, idx, _ = moe._fused_decode(x)
    got = idx.cpu().numpy()
    assert ((got >= 0) & (got < E)).all()
    assert len(set(got[1].tolist())) == k
    assert got[1].tolist() == list(range(k))
