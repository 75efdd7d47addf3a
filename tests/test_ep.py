"""Expert parallelism: the collective logic of ``kimi_k3_mlx_macmini_b200.ep`` on CPU
``gloo`` ranks (world size 2), with the oracle as router and local expert computation.
Each rank keeps its own tokens; the combined result must equal the single-process
oracle of the whole layer (``moe_forward``, i.e. ``k3ref/layers.py:241-261`` with the
BASELINE substitutions)."""
import os
import socket

import numpy as np
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import mxfp4_oracle as O

E, H, I, K, M, SCALE = 8, 64, 32, 2, 3, 2.5


def _layer(seed=11):
    rng = np.random.default_rng(seed)
    gate = (rng.standard_normal((E, H)) * 0.2).astype(np.float32)
    bias = (rng.standard_normal(E) * 0.01).astype(np.float32)
    experts = {e: {w: O.random_mxfp4(rng, *((I, H) if w != "w2" else (H, I))) for w in ("w1", "w3", "w2")}
               for e in list(range(E)) + ["shared"]}
    return gate, bias, experts


def _worker(rank, world, port, out_q, exchange="gather"):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from kimi_k3_mlx_macmini_b200.ep import ep_forward
        gate, bias, experts = _layer()
        rng = np.random.default_rng(100 + rank)
        x = rng.standard_normal((M, H)).astype(np.float32)
        E_loc = E // world
        dec = {e: {w: O.decode_mxfp4(*experts[e][w]) for w in ("w1", "w3", "w2")} for e in experts}

        def route_fn(xt):
            r = O.route(xt.numpy(), gate, bias, K, True, SCALE)
            return torch.from_numpy(r.expert_indices.astype(np.int32)), torch.from_numpy(r.expert_weights)

        def local_fn(x_all, slot, tok, w):
            y = np.zeros((x_all.shape[0], H), np.float32)
            order = np.argsort(slot.numpy(), kind="stable")          # ascending slot, shared last
            for i in order:
                s = int(slot[i])
                if s < 0:
                    continue
                e = "shared" if s == E_loc else rank * E_loc + s
                t = int(tok[i])
                out = O.expert_forward(x_all[t:t + 1].numpy(), dec[e]["w1"], dec[e]["w3"], dec[e]["w2"])
                y[t] += (out[0] * float(w[i])).astype(np.float32)
            return torch.from_numpy(y)

        y = ep_forward(torch.from_numpy(x), route_fn, local_fn, num_experts=E, with_shared=True,
                       exchange=exchange)
        ref, _ = O.moe_forward(x, O.MoESpec(E, K, SCALE, True, "silu"), gate, bias,
                               lambda e, w: experts[e][w],
                               shared={"kind": "mxfp4", **{w: experts["shared"][w] for w in ("w1", "w3", "w2")}})
        out_q.put((rank, O.rel_l2(y.numpy(), ref)))
    finally:
        dist.destroy_process_group()


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _run(world, exchange):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q, exchange)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert set(res) == set(range(world))
    for rank, err in res.items():
        assert err < 1e-5, (rank, err)


def test_ep_forward_gloo_two_ranks():
    _run(2, "gather")


def test_ep_forward_a2a_gloo_two_ranks():
    """The counted all-to-all exchange (send plan, row counts, tokens and routing out,
    partial rows back, ordered per-token sum) on gloo ranks."""
    _run(2, "a2a")


def test_ep_forward_a2a_gloo_four_ranks():
    """Four ranks of two experts each: tokens reach some ranks and not others, so the
    split sizes differ per pair of ranks."""
    _run(4, "a2a")


def test_a2a_plan_layout():
    from kimi_k3_mlx_macmini_b200.ep import a2a_plan
    # 4 tokens, top-2 of 8 experts over 4 ranks (2 each); this is rank 1
    idx = torch.tensor([[0, 1], [2, 7], [6, 3], [5, 4]], dtype=torch.int32)
    counts, rows, slot = a2a_plan(idx, rank=1, world=4, experts_per_rank=2)
    # rank 0: token 0; rank 1 (own): all tokens; rank 2: tokens 3; rank 3: tokens 1, 2
    assert counts == [1, 4, 1, 2]
    assert rows.tolist() == [0, 0, 1, 2, 3, 3, 1, 2]
    assert slot.tolist() == [[0, 1, -1, -1], [-1, 2, -1, 6], [-1, 3, -1, 7], [-1, 4, 5, -1]]
    # an expert id outside the layer is skipped (the device plan also flags the call)
    counts, rows, slot = a2a_plan(torch.tensor([[9, -1]], dtype=torch.int32), rank=0, world=4,
                                  experts_per_rank=2)
    assert counts == [1, 0, 0, 0] and rows.tolist() == [0] and slot.tolist() == [[0, -1, -1, -1]]


def test_pair_candidates_layout():
    from kimi_k3_mlx_macmini_b200.ep import pair_candidates
    idx = torch.tensor([[0, 5], [3, 4], [7, 1]], dtype=torch.int32)     # 3 gathered tokens, k = 2
    w = torch.arange(6, dtype=torch.float32).reshape(3, 2)
    slot, tok, wt = pair_candidates(idx, w, rank=1, world=2, num_experts=8, with_shared=True, M=1)
    # rank 1 owns experts 4..7 (slots 0..3) and the shared expert at slot 4 for its own token 1
    assert slot.tolist() == [-1, 1, -1, 0, 3, -1, 4]
    assert tok.tolist() == [0, 0, 1, 1, 2, 2, 1]
    assert wt.tolist() == [0, 1, 2, 3, 4, 5, 1]


def test_a2a_plan_properties():
    """For random routings: every (token, destination) that needs a row gets exactly one,
    rows are destination-major with tokens ascending, the own destination holds every
    token, and tok_slot points back at the rows."""
    from kimi_k3_mlx_macmini_b200.ep import a2a_plan
    rng = np.random.default_rng(17)
    for trial in range(20):
        W = int(rng.choice([1, 2, 3, 4, 8]))
        E_loc = int(rng.integers(1, 6))
        M = int(rng.integers(1, 40))
        k = int(rng.integers(1, min(4, W * E_loc) + 1))
        rank = int(rng.integers(0, W))
        idx = np.stack([rng.choice(W * E_loc, size=k, replace=False) for _ in range(M)]).astype(np.int32)
        counts, rows, slot = a2a_plan(torch.from_numpy(idx), rank, W, E_loc)
        need = np.zeros((M, W), bool)
        for t in range(M):
            need[t, idx[t] // E_loc] = True
            need[t, rank] = True
        assert counts == need.sum(0).tolist()
        rows, slot = rows.numpy(), slot.numpy()
        off = np.concatenate([[0], np.cumsum(counts)])
        for d in range(W):
            seg = rows[off[d]:off[d + 1]]
            assert seg.tolist() == np.flatnonzero(need[:, d]).tolist()        # ascending tokens
            for i, t in enumerate(seg):
                assert slot[t, d] == off[d] + i
        assert ((slot >= 0) == need).all()


def _leaver(rank, world, port, out_q):
    """Rank 1 leaves before the step; rank 0's step must end with an error (the peer is
    gone or the short process-group timeout runs out), not wait for good."""
    import datetime
    import time
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=5))
    if rank == 1:
        out_q.put((rank, "left"))
        return                                              # exits without joining the step
    from kimi_k3_mlx_macmini_b200.ep import ep_forward
    time.sleep(0.5)
    x = torch.zeros((M, H))
    t0 = time.time()
    try:
        ep_forward(x, lambda xt: (torch.zeros((M, K), dtype=torch.int32), torch.ones((M, K))),
                   lambda xa, s, t, w: torch.zeros((xa.shape[0], H)), num_experts=E, with_shared=True,
                   exchange="a2a")
        out_q.put((rank, "no error"))
    except Exception as exc:                                # noqa: BLE001 -- the outcome under test
        out_q.put((rank, f"error after {time.time() - t0:.1f}s: {type(exc).__name__}"))


def test_step_fails_fast_when_a_rank_leaves():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_leaver, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = dict(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert res[1] == "left"
    assert res[0].startswith("error after"), res[0]
    assert float(res[0].split()[2].rstrip("s:")) < 30.0, res[0]
