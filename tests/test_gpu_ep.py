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


def _ep_worker(rank, world, port, q, T=6, exchange="auto"):
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
        ep = ExpertParallelMoE(lay.cfg, 0, w, lay.source, exchange=exchange)
        x = synthetic.tokens(500 + rank, T, H)
        y = ep(x)                             # captures the step, then replays it
        x2 = synthetic.tokens(900 + rank, T, H)
        y2 = ep(x2)                           # replay on new tokens
        assert ep.graph_error is None, ep.graph_error
        if exchange in ("p2p", "auto") and T <= 8:
            assert ep.p2p is not None, ep.p2p_error       # one GPU per rank: the peer-memory step
        if ep.p2p is not None:
            assert ep.p2p.status.tolist() == [0, 0]
        ref = lay.moe()(x)                    # the whole layer on this GPU
        ref2 = lay.moe()(x2)
        err = max(O.rel_l2(y.cpu().numpy(), ref.float().cpu().numpy()),
                  O.rel_l2(y2.cpu().numpy(), ref2.float().cpu().numpy()))
        q.put((rank, err))
    finally:
        if ep is not None:
            ep.release_graphs()               # graphs holding NCCL calls go before the group
        dist.destroy_process_group()


def _run_ep(world, T, exchange="auto"):
    import torch.multiprocessing as mp
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        port = s.getsockname()[1]
    procs = [ctx.Process(target=_ep_worker, args=(r, world, port, q, T, exchange)) for r in range(world)]
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


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("exchange,T", [("p2p", 8), ("gather", 6)])
def test_expert_parallel_decode_exchanges(exchange, T):
    """The decode step with its all-gather and reduce-scatter as kernels over NVLink peer
    memory (exchange="p2p", also the default at decode) and as NCCL collectives
    ("gather"), both captured and replayed."""
    world = min(4, torch.cuda.device_count())
    for rank, err in _run_ep(world, T, exchange).items():
        assert err < 1e-5, (rank, err)


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.parametrize("T", [6, 300])
def test_expert_parallel_all_to_all(T):
    """The counted all-to-all exchange (exchange="a2a") at decode size (tokens that reach
    only some ranks; decode kernels) and at prefill size (prefill kernels)."""
    world = min(4, torch.cuda.device_count())
    for rank, err in _run_ep(world, T, "a2a").items():
        assert err < 1e-5, (rank, err)


# ---------------------------------------------------------------- counted all-to-all


@pytest.mark.parametrize("M,W,rank", [(1, 1, 0), (7, 2, 1), (2500, 8, 3), (1030, 32, 31)])
def test_a2a_plan_kernel_matches_host(k3, M, W, rank):
    """k3_ep_a2a_plan against the host restatement (ep.a2a_plan): counts, offsets, send
    rows (destination-major, tokens ascending) and each token's row per destination;
    routing rows wider than top_k (ids then weight bits) as the layer packs them."""
    from kimi_k3_mlx_macmini_b200.ep import a2a_plan, a2a_plan_dev
    k, E_all = 8, 384
    E_loc = E_all // W
    rng = np.random.default_rng(M + W)
    ids = rng.integers(0, E_all, size=(M, k)).astype(np.int32)
    wbits = rng.integers(0, 2**31, size=(M, k)).astype(np.int32)
    routing = torch.from_numpy(np.concatenate([ids, wbits], axis=1)).cuda()
    meta, rows, slot, st = a2a_plan_dev(routing, k, E_loc, W, rank)
    counts, rows_h, slot_h = a2a_plan(torch.from_numpy(ids), rank, W, E_loc)
    torch.cuda.synchronize()
    assert meta[:W].tolist() == counts
    assert meta[W:].tolist() == [int(v) for v in np.concatenate([[0], np.cumsum(counts)[:-1]])]
    S = sum(counts)
    assert torch.equal(rows[:S].cpu(), rows_h)
    assert torch.equal(slot.cpu(), slot_h)
    assert st.tolist() == [0, 0, 0, 0]


def test_a2a_plan_flags_bad_expert_id(k3):
    from kimi_k3_mlx_macmini_b200.ep import a2a_plan_dev
    routing = torch.tensor([[0, 3], [400, 1]], dtype=torch.int32, device="cuda")
    meta, rows, slot, st = a2a_plan_dev(routing, 2, 2, 2, 0)
    torch.cuda.synchronize()
    assert st[0].item() == 1                                      # K3_ERR_INVALID
    assert meta[:2].tolist() == [2, 1]                            # the bad id is skipped


@pytest.mark.parametrize("out_dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("with_base_own", [False, True])
def test_gather_rows_and_combine_exact(k3, out_dtype, with_base_own):
    """Packing copies rows bit for bit (16-byte and 4-byte word paths, into a fresh or a
    given buffer); the combine is the fp32 sum base + destinations in ascending order (the
    own rank's row from ``own``), bit-exact against the same adds."""
    from kimi_k3_mlx_macmini_b200.ep import a2a_combine_dev, gather_rows_dev
    g = torch.Generator(device="cuda").manual_seed(5)
    src = torch.randn((300, 7168), device="cuda", generator=g).to(torch.bfloat16)
    narrow = torch.randint(-2**31, 2**31 - 1, (300, 9), dtype=torch.int32, device="cuda")   # 36-byte rows
    rows = torch.randint(0, 300, (517,), dtype=torch.int32, device="cuda")
    st = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert torch.equal(gather_rows_dev(src, rows, 517, st), src[rows.long()])
    assert torch.equal(gather_rows_dev(narrow, rows, 517, st[1:]), narrow[rows.long()])
    out = torch.zeros((600, 7168), dtype=torch.bfloat16, device="cuda")
    gather_rows_dev(src, rows[100:300], 200, st, out=out[50:250])
    assert torch.equal(out[50:250], src[rows[100:300].long()]) and not out[:50].any() and not out[250:].any()
    M, W, H, rank = 100, 8, 7168, 3
    part = torch.randn((640, H), device="cuda", generator=g)
    slot = torch.randint(-1, 640, (M, W), dtype=torch.int32, device="cuda")
    base = own = None
    ref = torch.zeros((M, H), dtype=torch.float32, device="cuda")
    if with_base_own:
        base = torch.randn((M, H), device="cuda", generator=g)
        own = torch.randn((M, H), device="cuda", generator=g)
        slot[:, rank] = torch.arange(M, dtype=torch.int32, device="cuda")   # the own rank holds every token
        ref += base
    y = a2a_combine_dev(part, slot, st[2:], out_dtype, base=base, own=own, rank=rank)
    for d in range(W):
        s = slot[:, d].long()
        rowsd = own if (with_base_own and d == rank) else part[s.clamp(min=0)]
        ref += torch.where((s >= 0)[:, None], rowsd, torch.zeros((), device="cuda"))
    assert torch.equal(y, ref.to(out_dtype))
    torch.cuda.synchronize()
    assert st.tolist() == [0, 0, 0]


@pytest.mark.parametrize("M", [6, 120])
def test_a2a_step_emulated_on_one_gpu(k3, M):
    """The counted all-to-all data flow of ``ExpertParallelMoE._forward_a2a`` for 4 ranks
    on one GPU: the device plan and packing per rank (own segment not packed), the
    collectives replaced by the equivalent slicing, the shared expert over each rank's own
    tokens, ``k3_moe_ep_local`` per rank over its own pool (M = 6: decode kernels; M = 120:
    > 1024 candidates, prefill kernels), the reverse exchange without the own rows, and
    the ordered combine. Each rank's result must equal the whole layer on its tokens."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic
    from kimi_k3_mlx_macmini_b200.ep import a2a_combine_dev, a2a_plan_dev, gather_rows_dev
    from kimi_k3_mlx_macmini_b200.moe import MAX_DECODE_TOKENS, SHARED, ExpertPool
    lay = _small_layer(seed=9, top_k=4)
    W, k = 4, lay.cfg.num_experts_per_token
    E_loc = E // W
    full = lay.moe()
    lib = L.load_library()
    dev = torch.device("cuda")
    xs = [synthetic.tokens(700 + r, M, H) for r in range(W)]
    routing, plans, sends = [], [], []
    for r in range(W):
        rr = full.route(xs[r])
        pk = torch.cat([rr.expert_indices.to(torch.int32), rr.expert_weights.float().view(torch.int32)], 1)
        routing.append(pk.contiguous())
        meta, rows, slot, st = a2a_plan_dev(routing[r], k, E_loc, W, r)
        cnt, offs = meta[:W].tolist(), meta[W:].tolist()
        plans.append((cnt, offs, slot, st))
        S = sum(cnt)
        xsend = torch.zeros((S, H), dtype=torch.bfloat16, device=dev)
        rsend = torch.zeros((S, 2 * k), dtype=torch.int32, device=dev)
        for lo, hi in ((0, offs[r]), (offs[r] + cnt[r], S)):
            if hi > lo:
                gather_rows_dev(xs[r], rows[lo:hi], hi - lo, st[1:], out=xsend[lo:hi])
                gather_rows_dev(routing[r], rows[lo:hi], hi - lo, st[2:], out=rsend[lo:hi])
        sends.append((xsend, rsend))
    pools, y_part, y_shared = [], [], []
    for d in range(W):
        segs = [(plans[s][1][d], plans[s][0][d]) for s in range(W)]           # (offset, count) from rank s
        x_recv = torch.cat([xs[d] if s == d else sends[s][0][o:o + n] for s, (o, n) in enumerate(segs)]).contiguous()
        r_recv = torch.cat([routing[d] if s == d else sends[s][1][o:o + n]
                            for s, (o, n) in enumerate(segs)]).contiguous()
        lo = d * E_loc
        pool = ExpertPool(0, E_loc, lambda lay_, e, which, lo=lo: lay.source(lay_, e if e == SHARED else lo + int(e),
                                                                              which),
                          "cuda", with_shared=True)
        params = _params(pool, lay.cfg, E_loc)
        pools.append(pool)
        R = x_recv.shape[0]
        y = torch.empty((R, H), dtype=torch.float32, device=dev)
        ws = L.workspace(dev, lib.k3_moe_ep_local_workspace(params, R, 0))
        L.check(lib.k3_moe_ep_local(params, x_recv.data_ptr(), L.K3_BF16, R, r_recv.data_ptr(),
                                    r_recv.data_ptr() + 4 * k, 2 * k, lo, 0, 0, y.data_ptr(), L.K3_F32,
                                    ws.data_ptr(), ws.numel(), L.stream_of(x_recv)), "k3_moe_ep_local")
        # the shared expert over this rank's own tokens (slot E_loc of its pool)
        ys = torch.empty((M, H), dtype=torch.float32, device=dev)
        cand = [torch.full((M,), E_loc, dtype=torch.int32, device=dev), torch.arange(M, dtype=torch.int32, device=dev),
                torch.ones(M, dtype=torch.float32, device=dev)]
        args = (params, xs[d].data_ptr(), L.K3_BF16, M, cand[0].data_ptr(), cand[1].data_ptr(), cand[2].data_ptr(), M,
                ys.data_ptr(), L.K3_F32)
        if M > MAX_DECODE_TOKENS:                  # as the one-GPU layer (and ExpertParallelMoE) runs it
            ws2 = L.workspace(dev, lib.k3_moe_pairs_prefill_workspace(params, M, M))
            L.check(lib.k3_moe_pairs_prefill(*args, ws2.data_ptr(), ws2.numel(), L.stream_of(ys)), "pairs_prefill")
        else:
            ws2 = L.workspace(dev, lib.k3_moe_pairs_workspace(params, M, M))
            L.check(lib.k3_moe_pairs_decode(*args, ws2.data_ptr(), ws2.numel(), L.stream_of(ys)), "pairs_decode")
        torch.cuda.synchronize()
        y_part.append((y, [n for _, n in segs]))
        y_shared.append(ys)
    for s in range(W):
        cnt, offs, slot, st = plans[s]
        y_back = torch.zeros((sum(cnt), H), dtype=torch.float32, device=dev)
        for d in range(W):
            if d == s:
                continue
            y, cnts = y_part[d]
            o = sum(cnts[:s])
            y_back[offs[d]:offs[d] + cnt[d]] = y[o:o + cnts[s]]
        ys_own, cnts_own = y_part[s]
        o = sum(cnts_own[:s])
        y = a2a_combine_dev(y_back, slot, st[3:], base=y_shared[s], own=ys_own[o:o + M], rank=s)
        ref = full(xs[s]).float()
        torch.cuda.synchronize()
        assert st.tolist() == [0, 0, 0, 0]
        assert O.rel_l2(y.cpu().numpy(), ref.cpu().numpy()) < 1e-5, s
