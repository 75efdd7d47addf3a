"""Dense bf16 matvecs (``k3_dense_matvec``, ``k3_lm_head_argmax``) and the Kimi-K3 layer
built on them, on the GPU through the C ABI.

The reference computes the latent projections, the bf16 shared expert and the lm_head
logits in fp32 over bf16 weights (``air_llm/models/kimi_k3/moe.py:105-107,116,128-130``,
``model.py:111-133``); the checks compare with the same math in fp64 on the host.
fp32 accumulation over K <= 7168 terms stays within ~1e-6 relative of fp64.
"""
import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O

pytestmark = pytest.mark.gpu

F32_REL_L2 = 2e-6              # fp32 products and sums vs fp64
NORTH_STAR_REL_L2 = 1e-3       # layer outputs within rel-L2 1e-3


def _w(gen, n, k):
    return (torch.randn((n, k), generator=gen, device="cuda") * k ** -0.5).to(torch.bfloat16)


def _x(gen, m, k, dtype=torch.float32):
    return torch.randn((m, k), generator=gen, device="cuda").to(dtype)


def _h64(t):
    return t.detach().double().cpu().numpy()


def _rms64(x, w, eps):
    return w * (x / np.sqrt((x * x).mean(-1, keepdims=True) + eps))


@pytest.mark.parametrize("M,N,K", [(1, 3584, 7168), (8, 3584, 7168), (3, 100, 264), (5, 7168, 3584),
                                   (2, 64, 256), (4, 1000, 8), (8, 70, 1032), (1, 1, 16)])
def test_dense_sum_matches_fp64(k3, M, N, K):
    """One segment, row blocks straddling CTAs, ragged N and K (K % 256 != 0), M padded."""
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(M * 1000 + N + K)
    w, x = _w(gen, N, K), _x(gen, M, K)
    y = D.matvec([(w, x, None, 0.0)], N)
    torch.cuda.synchronize()
    assert y.shape == (M, N) and y.dtype == torch.float32
    assert O.rel_l2(_h64(y), _h64(x) @ _h64(w).T) < F32_REL_L2


def test_dense_bf16_input_and_output(k3):
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(3)
    w, x = _w(gen, 2048, 7168), _x(gen, 6, 7168, torch.bfloat16)
    want = _h64(x) @ _h64(w).T
    assert O.rel_l2(_h64(D.matvec([(w, x, None, 0.0)], 2048)), want) < F32_REL_L2
    yb = D.matvec([(w, x, None, 0.0)], 2048, out_dtype=torch.bfloat16)
    assert yb.dtype == torch.bfloat16
    assert O.rel_l2(_h64(yb), want) < 4e-3                        # bf16 output rounding


@pytest.mark.parametrize("M,xdt", [(1, torch.float32), (5, torch.bfloat16), (8, torch.float32)])
def test_dense_act_input_segment(k3, M, xdt):
    """A segment marked act_input reads act(gate, up) from [gate | up] rows (row stride
    above 2K): the bf16 shared expert's down projection fed straight from the front
    matvec's output, next to a plain segment. The activation is fp32 on the device, so
    the bound is twice the plain fp32 one."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(40 + M)
    K, N, ld = 3072, 1536, 2 * 3072 + 512
    base = (torch.randn((M, ld), generator=gen, device="cuda") * 2.0).to(xdt)
    gu = base[:, 512:512 + 2 * K]
    w, w2, x2 = _w(gen, N, K), _w(gen, N, 640), _x(gen, M, 640)
    for act, name, lb in ((L.K3_ACT_SITU, "situ", 25.0), (L.K3_ACT_SITU, "situ", None), (L.K3_ACT_SILU, "silu", None)):
        y = D.matvec([(w2, x2, None, 0.0), (w, gu, None, 0.0, True)], N, activation=act, situ_beta=4.0,
                     situ_linear_beta=-1.0 if lb is None else lb)
        a = O.activation(_h64(gu[:, :K]), _h64(gu[:, K:]), name, 4.0, lb)
        want = _h64(x2) @ _h64(w2).T + a @ _h64(w).T
        assert O.rel_l2(_h64(y), want) < 2 * F32_REL_L2, name


def test_dense_act_input_checks(k3):
    from kimi_k3_mlx_macmini_b200 import dense as D
    w = torch.zeros((64, 256), dtype=torch.bfloat16, device="cuda")
    x = torch.zeros((1, 400), device="cuda")                      # row shorter than 2K
    with pytest.raises(ValueError, match="ldx must be >= 2K"):
        D.matvec([(w, x, None, 0.0, True)], 64)
    with pytest.raises(ValueError, match="exclude each other"):
        D.matvec([(w, torch.zeros((1, 512), device="cuda"), torch.ones(256, device="cuda"), 1e-5, True)], 64)


def test_dense_two_segments_with_rmsnorm(k3):
    """rmsnorm(y) @ up.T + a @ sh_down.T in one call (the K3 layer's last matvec)."""
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    M, N, K0, K1 = 4, 7168, 3584, 3072
    up, sd = _w(gen, N, K0), _w(gen, N, K1)
    y_lat, a = _x(gen, M, K0) * 3.0, _x(gen, M, K1)
    nw = (1.0 + 0.1 * torch.randn(K0, generator=gen, device="cuda")).float()
    out = D.matvec([(up, y_lat, nw, 1e-5), (sd, a, None, 0.0)], N)
    want = _rms64(_h64(y_lat), _h64(nw), 1e-5) @ _h64(up).T + _h64(a) @ _h64(sd).T
    assert O.rel_l2(_h64(out), want) < F32_REL_L2


@pytest.mark.parametrize("act,lbeta", [("silu", None), ("situ", 25.0), ("situ", None)])
def test_dense_gate_up_activation(k3, act, lbeta):
    """act(x Wg^T, x Wu^T) of the bf16 shared expert (ops.situ, ops.py:17-28)."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(5)
    M, N, K = 8, 3072, 7168
    wg, wu, x = _w(gen, N, K), _w(gen, N, K), _x(gen, M, K, torch.bfloat16)
    kind = L.K3_ACT_SILU if act == "silu" else L.K3_ACT_SITU
    y = D.matvec([(wg, x, None, 0.0), (wu, x, None, 0.0)], N, combine=L.K3_DENSE_ACT, activation=kind,
                 situ_beta=4.0, situ_linear_beta=-1.0 if lbeta is None else lbeta)
    g, u = _h64(x) @ _h64(wg).T, _h64(x) @ _h64(wu).T
    want = O.activation(g, u, act, 4.0, lbeta)
    assert O.rel_l2(_h64(y), want) < 1e-5


def test_dense_repeatable(k3):
    """The split-k partial sums are added in a fixed order: bitwise equal across calls."""
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(9)
    w, x = _w(gen, 3584, 7168), _x(gen, 8, 7168)
    a = D.matvec([(w, x, None, 0.0)], 3584)
    for _ in range(3):
        assert torch.equal(D.matvec([(w, x, None, 0.0)], 3584), a)


def test_dense_status_stays_ok(k3):
    """No bounded wait gives up on ordinary calls (the status word stays K3_OK), for
    SUM, ACT and the lm_head argmax, through the C ABI with explicit workspaces."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    gen = torch.Generator(device="cuda")
    gen.manual_seed(12)
    M, N, K = 8, 3584, 7168
    w, w2, x = _w(gen, N, K), _w(gen, N, K), _x(gen, M, K)
    out = torch.empty((M, N), device="cuda")
    for comb in (L.K3_DENSE_SUM, L.K3_DENSE_ACT):
        ws = L.workspace(x.device, lib.k3_dense_workspace(M, N, 2, K, K))
        arr = (L.K3DenseSeg * 2)(L.K3DenseSeg(w.data_ptr(), K, K, x.data_ptr(), L.K3_F32, K, None, 0.0),
                                 L.K3DenseSeg(w2.data_ptr(), K, K, x.data_ptr(), L.K3_F32, K, None, 0.0))
        for _ in range(3):
            L.check(lib.k3_dense_matvec(arr, 2, M, N, comb, L.K3_ACT_SILU, 4.0, -1.0, out.data_ptr(), L.K3_F32, N,
                                        ws.data_ptr(), ws.numel(), L.stream_of(x)), "k3_dense_matvec")
        assert lib.k3_dense_status(ws.data_ptr(), L.stream_of(x)) == L.K3_OK
    idx = torch.empty(1, dtype=torch.int32, device="cuda")
    val = torch.empty(1, device="cuda")
    ws = L.workspace(x.device, lib.k3_lm_head_workspace(K, N))
    L.check(lib.k3_lm_head_argmax(x.data_ptr(), L.K3_F32, K, w.data_ptr(), N, idx.data_ptr(), val.data_ptr(), None,
                                  ws.data_ptr(), ws.numel(), L.stream_of(x)), "k3_lm_head_argmax")
    assert lib.k3_dense_status(ws.data_ptr(), L.stream_of(x)) == L.K3_OK


def test_dense_rejects_bad_arguments(k3):
    """Shape errors come back as K3_ERR_INVALID from the host checks (no launch)."""
    import ctypes
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    w = torch.zeros((64, 24), dtype=torch.bfloat16, device="cuda")
    x = torch.zeros((2, 24), device="cuda")
    out = torch.zeros((2, 64), device="cuda")
    ws = L.workspace(x.device, lib.k3_dense_workspace(2, 64, 2, 24, 24))
    seg = L.K3DenseSeg(w.data_ptr(), 24, 20, x.data_ptr(), L.K3_F32, 24, None, 0.0)   # K % 8 != 0
    arr = (L.K3DenseSeg * 2)(seg, seg)
    call = lambda n, comb: lib.k3_dense_matvec(arr, n, 2, 64, comb, 0, 4.0, -1.0, out.data_ptr(),  # noqa: E731
                                               L.K3_F32, 64, ws.data_ptr(), ws.numel(), L.stream_of(x))
    assert call(1, L.K3_DENSE_SUM) == L.K3_ERR_INVALID
    arr[0].K = arr[1].K = 24
    assert call(1, L.K3_DENSE_ACT) == L.K3_ERR_INVALID          # ACT needs (gate, up)
    assert lib.k3_dense_matvec(arr, 1, 9, 64, 0, 0, 4.0, -1.0, out.data_ptr(), L.K3_F32, 64, ws.data_ptr(),
                               ws.numel(), L.stream_of(x)) == L.K3_ERR_UNSUPPORTED      # M > 8
    assert lib.k3_dense_matvec(arr, 1, 2, 64, 0, 0, 4.0, -1.0, out.data_ptr(), L.K3_F32, 64, ws.data_ptr(),
                               ctypes.c_size_t(16), L.stream_of(x)) == L.K3_ERR_WORKSPACE
    assert call(2, L.K3_DENSE_SUM) == L.K3_OK
    torch.cuda.synchronize()


def test_lm_head_argmax(k3):
    """Streamed argmax over a ragged vocabulary (V % 64 != 0); logits vs fp64; the
    lowest index wins a tie, like the reference's first-occurrence argmax over chunks."""
    from kimi_k3_mlx_macmini_b200 import dense as D
    gen = torch.Generator(device="cuda")
    gen.manual_seed(21)
    V, H = 50001, 1024
    w = _w(gen, V, H)
    h = _x(gen, 1, H)
    i, v, nbytes, logits = D.lm_head_argmax(h, w, return_logits=True)
    want = (_h64(w) @ _h64(h)[0])
    assert O.rel_l2(_h64(logits), want) < F32_REL_L2
    assert i == int(np.argmax(_h64(logits))) and v == float(logits[i])
    assert abs(want[i] - want.max()) <= 1e-5 * abs(want.max())
    assert nbytes == V * H * 2
    # plant the same row twice in one row block (same summation order): the lower index
    # wins; the planted logit beats every other block's
    w[777] = w[781] = (h[0] * 4.0).to(torch.bfloat16)
    i2, v2, _ = D.lm_head_argmax(h, w)
    assert i2 == 777 and v2 > v


@pytest.fixture(scope="module")
def k3_layer(k3):
    from kimi_k3_mlx_macmini_b200 import synthetic
    lay = synthetic.k3_layer(seed=77)
    return lay, lay.moe()


def _k3_oracle(lay, x_bf16):
    """The whole K3 layer in the oracle (reference order, ``k3ref/layers.py:241-261``)."""
    c = lay.cfg
    h = lambda t: t.float().cpu().numpy()  # noqa: E731
    d = {k: h(v) for k, v in lay.dense.items()}
    spec = O.MoESpec(num_experts=c.num_experts, top_k=c.num_experts_per_token,
                     routed_scaling_factor=c.routed_scaling_factor, renormalize=True, activation="situ",
                     situ_beta=c.situ_beta, situ_linear_beta=c.situ_linear_beta, rms_norm_eps=c.rms_norm_eps)
    cache = {}

    def src(e, which):
        if e not in cache:
            cache.clear()
            cache[e] = [(p.cpu().numpy(), s.cpu().numpy()) for p, s in lay.expert(e)]
        return cache[e][("w1", "w3", "w2").index(which)]
    latent = {"down": d["routed_expert_down_proj.weight"], "up": d["routed_expert_up_proj.weight"],
              "norm": d["routed_expert_norm.weight"]}
    shared = {"kind": "dense", "gate": d["shared_experts.gate_proj.weight"],
              "up": d["shared_experts.up_proj.weight"], "down": d["shared_experts.down_proj.weight"]}
    return O.moe_forward(h(x_bf16), spec, h(lay.gate), h(lay.bias), src, shared=shared, latent=latent)


def test_k3_layer_decode_matches_oracle(k3, k3_layer):
    """A Kimi-K3 layer at full size (896 experts, top-16, latent 3584/3072, bf16 shared
    expert 2 x 3072 x 7168), 2 decode tokens: router index sets exact, output vs oracle."""
    from kimi_k3_mlx_macmini_b200 import synthetic
    import goldens as G
    lay, moe = k3_layer
    assert moe.latent and moe.dense_shared and moe.tiled
    x = synthetic.tokens(404, 2, 7168)
    y, r = moe(x, return_router=True)
    torch.cuda.synchronize()
    want, rr = _k3_oracle(lay, x)
    bad, _ = G.index_sets_match(r.expert_indices.cpu().numpy(), np.sort(rr.expert_indices, -1),
                                rr.corrected_scores, 16)
    assert bad == 0
    assert O.rel_l2(y.cpu().numpy(), want) < NORTH_STAR_REL_L2


def test_k3_layer_prefill_agrees_with_decode(k3, k3_layer):
    """40 tokens (the cuBLAS split-bf16 dense path and the prefill expert kernels) against
    the same tokens 8 at a time (the streaming matvecs and the decode kernels)."""
    from kimi_k3_mlx_macmini_b200 import synthetic
    _, moe = k3_layer
    x = synthetic.tokens(405, 40, 7168)
    y = moe(x)
    yd = torch.cat([moe(x[m:m + 8]) for m in range(0, 40, 8)])
    torch.cuda.synchronize()
    assert O.rel_l2(y.cpu().numpy(), yd.cpu().numpy()) < 5e-4


# ---------------------------------------------------- dense GEMM (more than 8 tokens)

def _gemm_call(x, w, out, accumulate, ldo=None):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    M, K = x.shape
    N = w.shape[0]
    ws = L.workspace(x.device, lib.k3_dense_gemm_workspace(M, K))
    L.check(lib.k3_dense_gemm(x.data_ptr(), L.dtype_code(x), x.stride(0), M, K, w.data_ptr(), w.stride(0), N,
                              out.data_ptr(), out.stride(0) if ldo is None else ldo, int(accumulate), ws.data_ptr(),
                              ws.numel(), L.stream_of(x)), "k3_dense_gemm")


@pytest.mark.parametrize("M,K,N,xdt", [
    (40, 3584, 7168, torch.float32),     # Kimi-K3 latent up above 8 tokens
    (200, 7168, 3584, torch.float32),    # latent down, ragged token tiles (200 = 2 x 96 + 8)
    (97, 1024, 300, torch.bfloat16),     # ragged rows of W (300 = 2 x 128 + 44), bf16 x exact
])
def test_dense_gemm_against_fp64(k3, M, K, N, xdt):
    """k3_dense_gemm (tcgen05 kind::f16): fp32 x as bf16 hi + lo pieces keeps ~16 bits of
    every input (bar 2e-5 relative L2); bf16 x is exact in fp32 accumulation (2e-6)."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(M + K + N)
    x = (torch.randn((M, K), generator=gen, device="cuda") * 2.0).to(xdt)
    w = (torch.randn((N, K), generator=gen, device="cuda") * K ** -0.5).to(torch.bfloat16)
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    _gemm_call(x, w, out, False)
    want = x.double().cpu().numpy() @ w.double().cpu().numpy().T
    err = O.rel_l2(out.cpu().numpy(), want)
    assert err < (2e-5 if xdt == torch.float32 else 2e-6), err
    again = torch.empty_like(out)
    _gemm_call(x, w, again, False)
    assert torch.equal(out, again)                         # fixed k order: bitwise repeatable


def test_dense_gemm_accumulates_into_strided_output(k3):
    """Two segments into one output (row stride above N), views with row strides above K."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(11)
    base_x = torch.randn((33, 1024 + 64), generator=gen, device="cuda")
    x0 = base_x[:, :1024]                                   # row stride 1088
    x1 = torch.randn((33, 512), generator=gen, device="cuda")
    w0 = (torch.randn((130, 1024), generator=gen, device="cuda") * 0.03).to(torch.bfloat16)
    w1 = (torch.randn((130, 512), generator=gen, device="cuda") * 0.04).to(torch.bfloat16)
    big = torch.full((33, 160), 7.0, device="cuda")
    out = big[:, :130]                                      # row stride 160
    _gemm_call(x0, w0, out, False)
    _gemm_call(x1, w1, out, True)
    want = (x0.double().cpu().numpy() @ w0.double().cpu().numpy().T
            + x1.double().cpu().numpy() @ w1.double().cpu().numpy().T)
    assert O.rel_l2(out.cpu().numpy(), want) < 2e-5
    assert torch.all(big[:, 130:] == 7.0)                   # untouched beyond N


def test_dense_gemm_rejects_bad_shapes(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    x = torch.zeros((4, 96), device="cuda")
    w = torch.zeros((8, 96), dtype=torch.bfloat16, device="cuda")
    out = torch.zeros((4, 8), device="cuda")
    ws = torch.zeros(1 << 16, dtype=torch.uint8, device="cuda")
    rc = lib.k3_dense_gemm(x.data_ptr(), L.K3_F32, 96, 4, 96, w.data_ptr(), 96, 8, out.data_ptr(), 8, 0,
                           ws.data_ptr(), ws.numel(), None)
    assert rc == L.K3_ERR_UNSUPPORTED and b"multiple of 64" in lib.k3_last_error()
