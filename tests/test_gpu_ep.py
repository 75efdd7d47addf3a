"""Expert-parallel local computation on the GPU: ``k3_moe_pairs_decode`` against the C
oracle (more than 8 tokens in one call, an expert split into several 8-pair items,
skipped candidates), and the full expert-parallel layer (decode and prefill) on up to 4
GPUs when the box has them."""
import os
import socket

import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O

pytestmark = pytest.mark.gpu

H, I, E = 1024, 512, 16


def _small_layer(seed=5, top_k=4):
    from kimi_k3_mlx_macmini_b200 import synthetic
    return synthetic.baseline_layer(seed=seed, E=E, H=H, I=I, top_k=top_k)


def _params(pool, cfg, num_experts):
    import ctypes
    from kimi_k3_mlx_macmini_b200 import _lib as L
    return L.K3MoEParams(hidden=pool.hidden, inter=pool.inter, num_experts=num_experts,
                         top_k=cfg.num_experts_per_token, renormalize=1,
                         routed_scaling_factor=float(cfg.routed_scaling_factor), has_shared=1,
                         activation=L.K3_ACT_SILU, situ_beta=4.0, situ_linear_beta=-1.0,
                         experts=pool.table.data_ptr(), pool=ctypes.pointer(pool.desc))


def test_pairs_decode_matches_oracle(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.moe import SHARED, ExpertPool
    lay = _small_layer()
    pool = ExpertPool(0, E, lay.source, "cuda", with_shared=True)
    params = _params(pool, lay.cfg, E)
    T = 12
    x = synthetic.tokens(77, T, H)
    rng = np.random.default_rng(3)
    slot = rng.integers(-1, E + 1, size=40).astype(np.int32)     # E = the shared slot
    slot[:10] = 3                                                # 10 pairs on one expert: 2 items
    tok = rng.integers(0, T, size=40).astype(np.int32)
    w = rng.uniform(0.1, 1.0, size=40).astype(np.float32)
    lib = L.load_library()
    y = torch.empty((T, H), dtype=torch.float32, device="cuda")
    ws = L.workspace(torch.device("cuda"), lib.k3_moe_pairs_workspace(params, T, 40))
    ts = [torch.from_numpy(a).cuda() for a in (slot, tok, w)]
    L.check(lib.k3_moe_pairs_decode(params, x.data_ptr(), L.K3_BF16, T, ts[0].data_ptr(), ts[1].data_ptr(),
                                    ts[2].data_ptr(), 40, y.data_ptr(), L.K3_F32, ws.data_ptr(), ws.numel(),
                                    L.stream_of(x)), "k3_moe_pairs_decode")
    xf = x.float().cpu().numpy()
    h = lambda t: t.cpu().numpy()  # noqa: E731
    ref = np.zeros((T, H), np.float64)
    for i in np.argsort(slot, kind="stable"):
        if slot[i] < 0:
            continue
        e = SHARED if slot[i] == E else int(slot[i])
        (p1, s1), (p3, s3), (p2, s2) = lay.expert(e)
        xt = xf[tok[i]:tok[i] + 1]
        g = O.matvec_fused(xt, h(p1), h(s1))
        u = O.matvec_fused(xt, h(p3), h(s3))
        ref[tok[i]] += O.matvec_fused(O.silu(g) * u, h(p2), h(s2))[0].astype(np.float64) * w[i]
    got = y.cpu().numpy()
    assert O.rel_l2(got, ref) < 1e-5
    untouched = np.setdiff1d(np.arange(T), tok[slot >= 0])
    assert np.all(got[untouched] == 0)


@pytest.mark.parametrize("T", [12, 300])
def test_ep_local_matches_explicit_pairs(k3, T):
    """k3_moe_ep_local (pairs taken on the device from the gathered routing, experts
    offset by expert_lo, the shared expert on a token range) equals the explicit-pair
    calls on the same candidates: the decode kernels at T=12, the prefill kernels at
    T=300 (more than 1024 candidates)."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.moe import SHARED, ExpertPool
    lay = _small_layer(seed=13)
    lo, E_loc, k = 4, 8, 4
    pool = ExpertPool(0, E_loc, lambda la, e, which: lay.source(la, e if e == SHARED else lo + int(e), which),
                      "cuda", with_shared=True)
    params = _params(pool, lay.cfg, E_loc)
    x = synthetic.tokens(31 + T, T, H)
    rng = np.random.default_rng(T)
    idx = np.stack([rng.choice(E, k, replace=False) for _ in range(T)]).astype(np.int32)
    w = rng.uniform(0.1, 1.0, size=(T, k)).astype(np.float32)
    routing = np.concatenate([idx, w.view(np.int32)], axis=1)
    t0, ns = 2, T - 5
    lib = L.load_library()
    dev = torch.device("cuda")
    r_all = torch.from_numpy(routing).cuda()
    y1 = torch.empty((T, H), dtype=torch.float32, device=dev)
    ws = L.workspace(dev, lib.k3_moe_ep_local_workspace(params, T, ns))
    L.check(lib.k3_moe_ep_local(params, x.data_ptr(), L.K3_BF16, T, r_all.data_ptr(),
                                r_all[:, k:].view(torch.float32).data_ptr(), 2 * k, lo, t0, ns, y1.data_ptr(),
                                L.K3_F32, ws.data_ptr(), ws.numel(), L.stream_of(x)), "k3_moe_ep_local")
    e_loc = idx.reshape(-1) - lo
    slot = np.where((e_loc >= 0) & (e_loc < E_loc), e_loc, -1).astype(np.int32)
    tok = np.repeat(np.arange(T, dtype=np.int32), k)
    wv = w.reshape(-1)
    slot = np.concatenate([slot, np.full(ns, E_loc, np.int32)])
    tok = np.concatenate([tok, np.arange(t0, t0 + ns, dtype=np.int32)])
    wv = np.concatenate([wv, np.ones(ns, np.float32)])
    ts = [torch.from_numpy(np.ascontiguousarray(a)).cuda() for a in (slot, tok, wv)]
    y2 = torch.empty((T, H), dtype=torch.float32, device=dev)
    n = slot.size
    fn, wsfn = ((lib.k3_moe_pairs_decode, lib.k3_moe_pairs_workspace) if n <= 1024 else
                (lib.k3_moe_pairs_prefill, lib.k3_moe_pairs_prefill_workspace))
    ws2 = L.workspace(dev, wsfn(params, T, n))
    L.check(fn(params, x.data_ptr(), L.K3_BF16, T, ts[0].data_ptr(), ts[1].data_ptr(), ts[2].data_ptr(), n,
               y2.data_ptr(), L.K3_F32, ws2.data_ptr(), ws2.numel(), L.stream_of(x)), "explicit pairs")
    a, b = y1.cpu().numpy(), y2.cpu().numpy()
    assert O.rel_l2(a, b) < 1e-6
    assert np.abs(b).sum() > 0


def _ep_worker(rank, world, port, q, T=6):
    import torch.distributed as dist
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    os.environ["NCCL_NVLS_ENABLE"] = "0"
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, device_id=torch.device("cuda", rank))
    ep = None
    try:
        from kimi_k3_mlx_macmini_b200 import synthetic
        from kimi_k3_mlx_macmini_b200.ep import ExpertParallelMoE
        lay = _small_layer(seed=9, top_k=4)
        w = {"gate.weight": lay.gate, "gate.e_score_correction_bias": lay.bias}
        ep = ExpertParallelMoE(lay.cfg, 0, w, lay.source)
        x = synthetic.tokens(500 + rank, T, H)
        y = ep(x)                             # captures the step, then replays it
        x2 = synthetic.tokens(900 + rank, T, H)
        y2 = ep(x2)                           # replay on new tokens
        assert ep.graph_error is None, ep.graph_error
        ref = lay.moe()(x)                    # the whole layer on this GPU
        ref2 = lay.moe()(x2)
        err = max(O.rel_l2(y.cpu().numpy(), ref.float().cpu().numpy()),
                  O.rel_l2(y2.cpu().numpy(), ref2.float().cpu().numpy()))
        q.put((rank, err))
    finally:
        if ep is not None:
            ep.release_graphs()               # graphs holding NCCL calls go before the group
        dist.destroy_process_group()


def _run_ep(world, T):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q, T)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=300) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    return res


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_decode():
    """Every GPU of the box (up to 4) as one expert-parallel layer, 6 tokens per rank."""
    world = min(4, torch.cuda.device_count())
    for rank, err in _run_ep(world, 6).items():
        assert err < 1e-5, (rank, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_expert_parallel_prefill():
    """300 tokens per rank: the local experts run on the prefill kernels
    (k3_moe_pairs_prefill); the single-GPU reference runs the prefill path too, so the
    two agree to the unordered fp32 adds into y."""
    world = min(4, torch.cuda.device_count())
    for rank, err in _run_ep(world, 300).items():
        assert err < 1e-5, (rank, err)
