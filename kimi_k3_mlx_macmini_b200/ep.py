"""Expert-parallel MoE layer at decode (BASELINE configs[2] at 2/4/8 GPUs).

One process per GPU. Rank r owns routed experts [r*E/W, (r+1)*E/W) and a copy of the
shared expert; the router is replicated. Every rank brings M tokens. A step:

1. route: each rank runs the router on its own M tokens (top-k ids and weights);
2. dispatch: ``all_gather`` of the tokens (bf16 [W*M, H]) and of their routing (one
   [M, 2k] int32 block: expert ids, then the weights' bits) -- at decode M is at most 8,
   so broadcasting every token to every rank is smaller than a counted all-to-all and
   needs no host synchronisation;
3. local experts: every rank runs its experts over the (token, expert) pairs that route
   to them, plus the shared expert for its own tokens (``k3_moe_ep_local``: the pairs
   are taken from the gathered routing on the device), producing one f32 partial row per
   gathered token (zero for tokens that touch none of its experts);
4. combine: ``reduce_scatter`` (sum) returns to each rank the total of its own M rows.

At prefill (thousands of tokens per rank) the same steps run with the local expert
computation on the grouped-GEMM kernels (``k3_moe_pairs_prefill``).

All transfers have fixed sizes, so a step captures into one CUDA graph with its NCCL
collectives. Compared with W replicas of the whole layer, each rank streams only the
experts its share is routed to by all W*M tokens, once.

The reference has no multi-device path (``air_llm/models/kimi_k3/moe.py:110-132`` runs
every expert of one process); the per-token result equals its ``LatentMoE.__call__`` up
to the order in which the ranks' partial sums are added.
"""
from __future__ import annotations

import ctypes
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from .moe import SHARED, ExpertPool, LatentMoE

PAIRS_DECODE_MAX = 1024      # candidates one k3_moe_pairs_decode call takes

RouteFn = Callable[[torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]
LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _is_nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


def pair_candidates(idx_all: torch.Tensor, w_all: torch.Tensor, rank: int, world: int,
                    num_experts: int, with_shared: bool, M: int):
    """(slot, token row, weight) candidates of rank ``rank``: every routed pair of the W*M
    gathered tokens, with slot = expert - first local expert when the expert is local and
    -1 otherwise, then the shared expert (slot E/W) for this rank's own M tokens."""
    E_loc = num_experts // world
    lo = rank * E_loc
    k = idx_all.shape[1]
    T = idx_all.shape[0]
    dev = idx_all.device
    local = (idx_all >= lo) & (idx_all < lo + E_loc)
    slot = torch.where(local, idx_all - lo, torch.full_like(idx_all, -1)).reshape(-1).to(torch.int32)
    tok = torch.arange(T, device=dev, dtype=torch.int32).repeat_interleave(k)
    w = w_all.reshape(-1).to(torch.float32)
    if with_shared:
        own = torch.arange(rank * M, rank * M + M, device=dev, dtype=torch.int32)
        slot = torch.cat([slot, torch.full((M,), E_loc, device=dev, dtype=torch.int32)])
        tok = torch.cat([tok, own])
        w = torch.cat([w, torch.ones(M, device=dev, dtype=torch.float32)])
    return slot.contiguous(), tok.contiguous(), w.contiguous()


def ep_forward(x: torch.Tensor, route_fn: RouteFn, local_fn: LocalFn, *, group=None,
               num_experts: int, with_shared: bool) -> torch.Tensor:
    """One expert-parallel step for this rank's tokens x [M, H]; returns y [M, H] f32.
    ``route_fn(x) -> (idx [M, k] int32, w [M, k] f32)``; ``local_fn(x_all, slot, tok, w)
    -> [W*M, H] f32`` computes this rank's experts over the candidate pairs."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    M, H = x.shape
    idx, w = route_fn(x)
    idx = idx.to(torch.int32).contiguous()
    w = w.to(torch.float32).contiguous()
    nccl = _is_nccl(group)
    if nccl:
        x_all = torch.empty((W * M, H), dtype=x.dtype, device=x.device)
        idx_all = torch.empty((W * M, idx.shape[1]), dtype=idx.dtype, device=x.device)
        w_all = torch.empty((W * M, w.shape[1]), dtype=w.dtype, device=x.device)
        dist.all_gather_into_tensor(x_all, x.contiguous(), group=group)
        dist.all_gather_into_tensor(idx_all, idx, group=group)
        dist.all_gather_into_tensor(w_all, w, group=group)
    else:
        parts = [[torch.empty_like(t) for _ in range(W)] for t in (x, idx, w)]
        for lst, t in zip(parts, (x.contiguous(), idx, w)):
            dist.all_gather(lst, t, group=group)
        x_all, idx_all, w_all = (torch.cat(lst) for lst in parts)
    slot, tok, wt = pair_candidates(idx_all, w_all, r, W, num_experts, with_shared, M)
    y_part = local_fn(x_all, slot, tok, wt)
    if nccl:
        y = torch.empty((M, H), dtype=torch.float32, device=x.device)
        dist.reduce_scatter_tensor(y, y_part.contiguous(), group=group)
        return y
    dist.all_reduce(y_part, group=group)
    return y_part[r * M:(r + 1) * M].clone()


class ExpertParallelMoE:
    """This rank's share of an expert-parallel MoE layer on its GPU; ``__call__(x)`` is
    ``LatentMoE.__call__`` (``moe.py:110-132``) for this rank's tokens, computed jointly
    by all ranks of ``group`` (every rank calls with the same M)."""

    def __init__(self, cfg, layer: int, w: dict, expert_source: Callable, group=None,
                 device=None, graphs: bool = True):
        self.cfg, self.group = cfg, group
        # On NCCL, a step (router, collectives, local experts: ~15 launches) is captured
        # into a CUDA graph per token count at its first call and replayed afterwards, so a
        # decode loop is not bound by the host's launch rate.
        self.graphs = graphs
        self._steps: dict = {}
        self.graph_error: Optional[str] = None
        self.W = dist.get_world_size(group)
        self.r = dist.get_rank(group)
        E = cfg.num_experts
        if E % self.W:
            raise ValueError(f"{E} experts do not split over {self.W} ranks")
        self.E_loc = E // self.W
        self.lo = self.r * self.E_loc
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        # the router is replicated; its expert pool is never built
        self.router = LatentMoE(cfg, layer, w, expert_source, fused=True, device=self.device)
        if self.router.latent or self.router.dense_shared:
            raise NotImplementedError("expert parallelism covers the BASELINE layer (no latent "
                                      "wrapper, MXFP4 shared expert)")
        self.with_shared = self.router.mxfp4_shared
        lo = self.lo
        self.pool = ExpertPool(layer, self.E_loc,
                               lambda lay, e, which: expert_source(lay, e if e == SHARED else lo + int(e), which),
                               self.device, with_shared=self.with_shared)
        if self.pool.scales_tc is None:
            raise NotImplementedError("expert parallelism needs the block-scaled pool (H, I multiples of 512)")
        c = cfg
        lb = getattr(c, "situ_linear_beta", None)
        self.params = L.K3MoEParams(
            hidden=self.pool.hidden, inter=self.pool.inter, num_experts=self.E_loc,
            top_k=c.num_experts_per_token, renormalize=int(bool(c.moe_renormalize)),
            routed_scaling_factor=float(c.routed_scaling_factor), has_shared=int(self.with_shared),
            activation=L.K3_ACT_SITU if self.router.act == "situ" else L.K3_ACT_SILU,
            situ_beta=float(getattr(c, "situ_beta", 4.0)),
            situ_linear_beta=-1.0 if lb is None else float(lb),
            experts=self.pool.table.data_ptr(), pool=ctypes.pointer(self.pool.desc))

    def _route(self, x: torch.Tensor):
        rr = self.router.route(x)
        return rr.expert_indices, rr.expert_weights

    def _local(self, x_all: torch.Tensor, slot: torch.Tensor, tok: torch.Tensor,
               w: torch.Tensor) -> torch.Tensor:
        """This rank's experts over the candidate pairs: the decode kernels for up to
        ``PAIRS_DECODE_MAX`` candidates, the grouped-GEMM prefill kernels beyond."""
        lib = L.load_library()
        T, H = x_all.shape
        n = slot.numel()
        y = torch.empty((T, H), dtype=torch.float32, device=x_all.device)
        if n > PAIRS_DECODE_MAX:
            ws = L.workspace(x_all.device, lib.k3_moe_pairs_prefill_workspace(self.params, T, n))
            L.check(lib.k3_moe_pairs_prefill(self.params, x_all.data_ptr(), L.dtype_code(x_all), T,
                                             slot.data_ptr(), tok.data_ptr(), w.data_ptr(), n,
                                             y.data_ptr(), L.K3_F32, ws.data_ptr(), ws.numel(),
                                             L.stream_of(x_all)), "k3_moe_pairs_prefill")
            return y
        ws = L.workspace(x_all.device, lib.k3_moe_pairs_workspace(self.params, T, n))
        L.check(lib.k3_moe_pairs_decode(self.params, x_all.data_ptr(), L.dtype_code(x_all), T,
                                        slot.data_ptr(), tok.data_ptr(), w.data_ptr(), n,
                                        y.data_ptr(), L.K3_F32, ws.data_ptr(), ws.numel(),
                                        L.stream_of(x_all)), "k3_moe_pairs_decode")
        return y

    def _forward_nccl(self, flat: torch.Tensor) -> torch.Tensor:
        """One step with two all_gathers issued as one NCCL group (tokens; routing packed
        as [M][2k] int32: expert ids, then the weights' bits) and the local experts taken
        straight from the gathered routing on the device (``k3_moe_ep_local``)."""
        lib = L.load_library()
        c = self.cfg
        M, H = flat.shape
        k, E, W = c.num_experts_per_token, c.num_experts, self.W
        dev = flat.device
        idx = torch.empty((M, k), dtype=torch.int32, device=dev)
        w = torch.empty((M, k), dtype=torch.float32, device=dev)
        r = self.router
        ws = L.workspace(dev, lib.k3_moe_route_workspace(M, E))
        L.check(lib.k3_moe_route(flat.data_ptr(), L.dtype_code(flat), M, H, r.gate_w.data_ptr(),
                                 None if r.gate_b is None else r.gate_b.data_ptr(), E, k,
                                 int(bool(c.moe_renormalize)), float(c.routed_scaling_factor),
                                 idx.data_ptr(), w.data_ptr(), None, None, ws.data_ptr(), ws.numel(),
                                 L.stream_of(flat)), "k3_moe_route")
        routing = torch.cat([idx, w.view(torch.int32)], dim=1)
        x_all = torch.empty((W * M, H), dtype=flat.dtype, device=dev)
        r_all = torch.empty((W * M, 2 * k), dtype=torch.int32, device=dev)
        # both gathers in one NCCL group: one collective launch per step instead of two
        with dist._coalescing_manager(group=self.group, device=dev):
            dist.all_gather_into_tensor(x_all, flat, group=self.group)
            dist.all_gather_into_tensor(r_all, routing, group=self.group)
        y_part = torch.empty((W * M, H), dtype=torch.float32, device=dev)
        w_all = r_all[:, k:].view(torch.float32)
        shared_n = M if self.with_shared else 0
        ws2 = L.workspace(dev, lib.k3_moe_ep_local_workspace(self.params, W * M, shared_n))
        L.check(lib.k3_moe_ep_local(self.params, x_all.data_ptr(), L.dtype_code(x_all), W * M, r_all.data_ptr(),
                                    w_all.data_ptr(), 2 * k, self.lo, self.r * M, shared_n, y_part.data_ptr(),
                                    L.K3_F32, ws2.data_ptr(), ws2.numel(), L.stream_of(x_all)), "k3_moe_ep_local")
        y = torch.empty((M, H), dtype=torch.float32, device=dev)
        dist.reduce_scatter_tensor(y, y_part, group=self.group)
        return y

    def _replay(self, flat: torch.Tensor) -> torch.Tensor:
        """The step as a CUDA graph: captured once per (tokens, dtype) -- every rank at the
        same call, since all ranks call with the same M -- over static input and output
        buffers; each call copies x in, replays, and returns a copy of the output."""
        key = (flat.shape[0], flat.dtype)
        ent = self._steps.get(key)
        if ent is None:
            cur = torch.cuda.current_stream(flat.device)
            side = torch.cuda.Stream(flat.device)
            sx = flat.clone()
            side.wait_stream(cur)
            with torch.cuda.stream(side):
                self._forward_nccl(sx)               # warm-up: workspaces exist before capture
            cur.wait_stream(side)
            torch.cuda.synchronize(flat.device)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=side):
                sy = self._forward_nccl(sx)
            ent = (g, sx, sy)
            self._steps[key] = ent
        g, sx, sy = ent
        sx.copy_(flat)
        g.replay()
        return sy.clone()

    def release_graphs(self) -> None:
        """Drop the captured steps (before the process group is destroyed)."""
        self._steps.clear()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        L.require_cuda(x, "x")
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        if flat.dtype not in (torch.float32, torch.bfloat16):
            flat = flat.float()
        flat = flat.contiguous()
        if _is_nccl(self.group):
            if self.graphs and self.graph_error is None and not torch.cuda.is_current_stream_capturing():
                try:
                    return self._replay(flat).reshape(shape)
                except Exception as exc:              # noqa: BLE001 -- kept, then launched eagerly
                    torch.cuda.synchronize(flat.device)
                    self.graph_error = f"{type(exc).__name__}: {str(exc).splitlines()[0][:200] if str(exc) else ''}"
                    self._steps.clear()
            return self._forward_nccl(flat).reshape(shape)
        y = ep_forward(flat, self._route, self._local, group=self.group,
                       num_experts=self.cfg.num_experts, with_shared=self.with_shared)
        return y.reshape(shape)

    def pairs_decode(self, x_all: torch.Tensor, slot: torch.Tensor, tok: torch.Tensor,
                     w: torch.Tensor) -> torch.Tensor:
        """The local expert computation alone (for tests and diagnostics)."""
        return self._local(x_all, slot, tok, w)


__all__ = ["ExpertParallelMoE", "ep_forward", "pair_candidates"]
