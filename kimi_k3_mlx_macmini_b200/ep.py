"""Expert-parallel MoE layer (BASELINE configs[2] and [3] at 2/4/8 GPUs).

One process per GPU. Rank r owns routed experts [r*E/W, (r+1)*E/W) and a copy of the
shared expert; the router is replicated. Every rank brings M tokens. A step:

1. route: each rank runs the router on its own M tokens (top-k ids and weights);
2. dispatch: an all-gather of the tokens (bf16 [W*M, H]) and of their routing (one
   [M, 2k] int32 block: expert ids, then the weights' bits) -- at decode M is at most 8,
   so broadcasting every token to every rank is smaller than a counted all-to-all and
   needs no host synchronisation;
3. local experts: every rank runs its experts over the (token, expert) pairs that route
   to them, plus the shared expert for its own tokens (``k3_moe_ep_local``: the pairs
   are taken from the gathered routing on the device), producing one f32 partial row per
   gathered token (zero for tokens that touch none of its experts);
4. combine: a reduce-scatter (sum) returns to each rank the total of its own M rows.

At decode (up to MAX_DECODE_TOKENS tokens per rank) the all-gather and the reduce-scatter
are two kernels over NVLink peer memory by default (``P2PExchange``: IPC-mapped buffers,
flags with bounded waits); above that, or where peer memory is unavailable, they are the
NCCL collectives (``exchange="gather"`` forces those). All transfers have fixed sizes, so
a step captures into one CUDA graph. Compared with W replicas of the whole layer, each
rank streams only the experts its share is routed to by all W*M tokens, once.

The counted all-to-all exchange (``exchange="a2a"``) sends a token once to each rank
that owns one of its experts (and to its own rank, for the shared expert), not to every
rank, and returns only the partial rows of those tokens:

1. route, then ``k3_ep_a2a_plan`` builds the send plan on the device (rows per
   destination, tokens ascending; each token's row per destination);
2. the row counts go through one ``all_to_all_single`` and to the host (the split sizes
   of the next collectives: one host synchronisation per step, so the step is launched
   eagerly); meanwhile the shared expert runs over the own tokens;
3. ``k3_ep_gather_rows`` packs the tokens and routing rows bound for other ranks; two
   ``all_to_all`` deliver them (the own tokens go straight from the input), so the
   receive buffer is [rows from rank 0][rows from rank 1]..., the own segment holding all
   own tokens in order;
4. ``k3_moe_ep_local`` runs this rank's routed experts over the received rows;
5. the reverse ``all_to_all`` returns each partial row to its token's rank (the own rows
   stay), and ``k3_ep_a2a_combine`` sums a token's shared-expert row and its rows in
   ascending rank order.

With top-8 of 384 experts over 8 ranks a token reaches ~4.6 other ranks instead of 7, so
the exchange moves ~0.66 of the gather's token bytes and of the reduce-scatter's fp32
bytes. Measured at prefill (T = 4096 per GPU, BASELINE layer) it is not faster on B200
over NVSwitch: 4.36 against 4.09 ms per step at N = 2 and 6.09 against 5.99 ms at N = 8
(the packing, the ordered combine, a second GEMM launch set for the shared expert and
the host synchronisation cost about what the smaller transfers save). ``exchange="auto"``
(the default) therefore runs the gather step at every size; ``"a2a"`` selects the
all-to-all.

The reference has no multi-device path (``air_llm/models/kimi_k3/moe.py:110-132`` runs
every expert of one process); the per-token result equals its ``LatentMoE.__call__`` up
to the order in which the ranks' partial sums are added.
"""
from __future__ import annotations

import ctypes
import hashlib
from typing import Callable, Optional, Tuple

import torch
import torch.distributed as dist

from . import _lib as L
from .moe import MAX_DECODE_TOKENS, SHARED, ExpertPool, LatentMoE

PAIRS_DECODE_MAX = 1024      # candidates one k3_moe_pairs_decode call takes

RouteFn = Callable[[torch.Tensor], Tuple[torch.Tensor, torch.Tensor]]
LocalFn = Callable[[torch.Tensor, torch.Tensor, torch.Tensor, torch.Tensor], torch.Tensor]


def _is_nccl(group) -> bool:
    return dist.get_backend(group) == "nccl"


def pair_candidates(idx_all: torch.Tensor, w_all: torch.Tensor, rank: int, world: int,
                    num_experts: int, with_shared: bool, M: int, own_t0: Optional[int] = None):
    """(slot, token row, weight) candidates of rank ``rank``: every routed pair of the
    gathered (or received) token rows, with slot = expert - first local expert when the
    expert is local and -1 otherwise, then the shared expert (slot E/W) for this rank's own
    M token rows, which start at row ``own_t0`` (default rank * M: the gathered layout)."""
    E_loc = num_experts // world
    if own_t0 is None:
        own_t0 = rank * M
    lo = rank * E_loc
    k = idx_all.shape[1]
    T = idx_all.shape[0]
    dev = idx_all.device
    local = (idx_all >= lo) & (idx_all < lo + E_loc)
    slot = torch.where(local, idx_all - lo, torch.full_like(idx_all, -1)).reshape(-1).to(torch.int32)
    tok = torch.arange(T, device=dev, dtype=torch.int32).repeat_interleave(k)
    w = w_all.reshape(-1).to(torch.float32)
    if with_shared:
        own = torch.arange(own_t0, own_t0 + M, device=dev, dtype=torch.int32)
        slot = torch.cat([slot, torch.full((M,), E_loc, device=dev, dtype=torch.int32)])
        tok = torch.cat([tok, own])
        w = torch.cat([w, torch.ones(M, device=dev, dtype=torch.float32)])
    return slot.contiguous(), tok.contiguous(), w.contiguous()


def a2a_plan(idx: torch.Tensor, rank: int, world: int, experts_per_rank: int):
    """The send plan of the counted all-to-all (what ``k3_ep_a2a_plan`` computes on the
    device), from this rank's routing idx [M, k]: per destination d the rows of the tokens
    that have an expert on rank d, or that are this rank's own (d == rank), ascending.
    Returns (counts: list of W ints, rows: int32 [sum(counts)] destination-major,
    tok_slot: int32 [M, W], the send row of (t, d) or -1)."""
    M = idx.shape[0]
    dev = idx.device
    ids = idx.long()
    valid = (ids >= 0) & (ids < experts_per_rank * world)
    dest = torch.where(valid, ids // experts_per_rank, torch.full_like(ids, rank))   # invalid ids: skipped
    mask = torch.zeros((M, world), dtype=torch.bool, device=dev)
    mask.scatter_(1, dest, True)
    mask[:, rank] = True
    counts = mask.sum(0).tolist()
    dt = mask.t().nonzero()                                   # (d, t), d-major, t ascending
    rows = dt[:, 1].to(torch.int32).contiguous()
    tok_slot = torch.full((M, world), -1, dtype=torch.int32, device=dev)
    tok_slot[dt[:, 1], dt[:, 0]] = torch.arange(dt.shape[0], dtype=torch.int32, device=dev)
    return counts, rows, tok_slot


def a2a_plan_dev(routing: torch.Tensor, k: int, experts_per_rank: int, world: int, rank: int):
    """``k3_ep_a2a_plan`` on this rank's routing rows (device, int32 [M, >= k], expert ids
    first). Returns (meta int64 [2W]: send counts then their exclusive prefix, rows int32
    [M*W]: the send rows' tokens, destination-major, tok_slot int32 [M, W], status int32
    [4]: the status words of the plan, the two packings and the combine)."""
    lib = L.load_library()
    M = routing.shape[0]
    dev = routing.device
    meta = torch.empty(2 * world, dtype=torch.int64, device=dev)
    rows = torch.empty(M * world, dtype=torch.int32, device=dev)
    tok_slot = torch.empty((M, world), dtype=torch.int32, device=dev)
    status = torch.zeros(4, dtype=torch.int32, device=dev)
    L.check(lib.k3_ep_a2a_plan(routing.data_ptr(), routing.stride(0), M, k, experts_per_rank, world, rank,
                               meta.data_ptr(), meta[world:].data_ptr(), rows.data_ptr(), tok_slot.data_ptr(),
                               status.data_ptr(), L.stream_of(routing)), "k3_ep_a2a_plan")
    return meta, rows, tok_slot, status


def gather_rows_dev(src: torch.Tensor, rows: torch.Tensor, n: int, status: torch.Tensor,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """``k3_ep_gather_rows``: src[rows[:n]] for a row-major device tensor src, into
    ``out`` (contiguous, n rows) when given; a bad row index sets status[0] (a device
    word)."""
    lib = L.load_library()
    dst = torch.empty((n,) + tuple(src.shape[1:]), dtype=src.dtype, device=src.device) if out is None else out
    row_bytes = src[0].numel() * src.element_size()
    L.check(lib.k3_ep_gather_rows(src.data_ptr(), src.shape[0], row_bytes, rows.data_ptr(), n, dst.data_ptr(),
                                  status.data_ptr(), L.stream_of(src)), "k3_ep_gather_rows")
    return dst


def a2a_combine_dev(part: torch.Tensor, tok_slot: torch.Tensor, status: torch.Tensor,
                    dtype: torch.dtype = torch.float32, base: Optional[torch.Tensor] = None,
                    own: Optional[torch.Tensor] = None, rank: int = 0) -> torch.Tensor:
    """``k3_ep_a2a_combine``: y[t] = base[t] + sum over d ascending of (own[t] when d ==
    rank and own is given, else part[tok_slot[t, d]]), fp32 rows [., H]; a bad slot sets
    status[0]."""
    lib = L.load_library()
    M, W = tok_slot.shape
    H = part.shape[1]
    y = torch.empty((M, H), dtype=dtype, device=part.device)
    L.check(lib.k3_ep_a2a_combine(None if base is None else base.data_ptr(), None if own is None else own.data_ptr(),
                                  rank, part.data_ptr(), part.shape[0], tok_slot.data_ptr(), M, W, H, y.data_ptr(),
                                  L.dtype_code(y), status.data_ptr(), L.stream_of(part)), "k3_ep_a2a_combine")
    return y


def _ep_forward_a2a(x, idx, w, local_fn, group, num_experts, with_shared):
    """The counted all-to-all step on any backend (torch ops for the plan, packing and
    combine; ``ExpertParallelMoE`` runs the same data flow on its CUDA kernels)."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    M, H = x.shape
    k = idx.shape[1]
    E_loc = num_experts // W
    counts, rows, tok_slot = a2a_plan(idx, r, W, E_loc)
    cnt = torch.tensor(counts, dtype=torch.int64)
    rcnt = torch.empty_like(cnt)
    dist.all_to_all_single(rcnt, cnt, group=group)
    recv = rcnt.tolist()
    routing = torch.cat([idx, w.view(torch.int32)], dim=1)
    x_recv = torch.empty((sum(recv), H), dtype=x.dtype)
    r_recv = torch.empty((sum(recv), 2 * k), dtype=torch.int32)
    dist.all_to_all_single(x_recv, x[rows.long()].contiguous(), recv, counts, group=group)
    dist.all_to_all_single(r_recv, routing[rows.long()].contiguous(), recv, counts, group=group)
    own_t0 = sum(recv[:r])
    slot, tok, wt = pair_candidates(r_recv[:, :k], r_recv[:, k:].view(torch.float32), r, W, num_experts,
                                    with_shared, M, own_t0=own_t0)
    y_part = local_fn(x_recv, slot, tok, wt).to(torch.float32).contiguous()
    y_back = torch.empty((sum(counts), H), dtype=torch.float32)
    dist.all_to_all_single(y_back, y_part, counts, recv, group=group)
    y = torch.zeros((M, H), dtype=torch.float32)
    for d in range(W):                                         # ascending rank: a fixed order
        sel = tok_slot[:, d] >= 0
        y[sel] += y_back[tok_slot[sel, d].long()]
    return y


def ep_forward(x: torch.Tensor, route_fn: RouteFn, local_fn: LocalFn, *, group=None,
               num_experts: int, with_shared: bool, exchange: str = "gather") -> torch.Tensor:
    """One expert-parallel step for this rank's tokens x [M, H]; returns y [M, H] f32.
    ``route_fn(x) -> (idx [M, k] int32, w [M, k] f32)``; ``local_fn(x_rows, slot, tok, w)
    -> [rows, H] f32`` computes this rank's experts over the candidate pairs of the
    gathered (``exchange="gather"``) or received (``"a2a"``, host tensors) token rows."""
    W = dist.get_world_size(group)
    r = dist.get_rank(group)
    M, H = x.shape
    idx, w = route_fn(x)
    idx = idx.to(torch.int32).contiguous()
    w = w.to(torch.float32).contiguous()
    if exchange == "a2a":
        return _ep_forward_a2a(x.contiguous(), idx, w, local_fn, group, num_experts, with_shared)
    if exchange != "gather":
        raise ValueError(f"exchange must be 'gather' or 'a2a', not {exchange!r}")
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


class P2PUnavailable(RuntimeError):
    """Peer-memory exchange not possible for this group (ranks sharing a GPU, no CUDA IPC
    between the ranks' GPUs, ...); every rank of the group raises it together."""


class P2PExchange:
    """Exchange buffers of an expert-parallel group over NVLink peer memory (CUDA IPC):
    a decode step's all-gather of the tokens and routing and its reduce-scatter of the
    partial rows as ``k3_p2p_*`` kernels that store straight into the peers' buffers,
    instead of NCCL collectives. Built collectively (every rank of ``group`` at once):
    each rank allocates its buffer, exports its IPC handle, receives every peer's (one
    NCCL all_gather) and maps them; the ranks agree on the outcome (one all_reduce), so
    either all use it or all raise ``P2PUnavailable``. The kernels wait on flags that
    other ranks set, so the group needs one GPU per rank: ranks that share a GPU make it
    unavailable. Capacities are per rank and call."""

    def __init__(self, group, device: torch.device, gather_bytes: int, gather2_bytes: int, reduce_bytes: int):
        lib = L.load_library()
        self.group = group
        self.W, self.r = dist.get_world_size(group), dist.get_rank(group)
        self.caps = (int(gather_bytes), int(gather2_bytes), int(reduce_bytes))
        self._opened = []
        nbytes = int(lib.k3_p2p_buffer_bytes(self.W, *self.caps))
        if nbytes == 0:
            raise ValueError("k3_p2p_buffer_bytes: bad world size or capacities")
        self._buf = torch.zeros(nbytes + 256, dtype=torch.uint8, device=device)
        skew = (-self._buf.data_ptr()) % 256
        self.own = self._buf[skew:skew + nbytes]
        offs = (ctypes.c_int64 * 4)()
        L.check(lib.k3_p2p_area_offsets(self.W, *self.caps, offs), "k3_p2p_area_offsets")
        self.offsets = list(offs)
        torch.cuda.synchronize(device)                       # zeroed before any peer maps it
        why = ""
        handle = (ctypes.c_uint8 * 64)()
        ioff = ctypes.c_int64()
        if lib.k3_p2p_export(self.own.data_ptr(), handle, ctypes.byref(ioff)) != 0:
            why = f"rank {self.r}: k3_p2p_export: {L.last_error()}"
        uuid = str(torch.cuda.get_device_properties(device).uuid).encode()
        gpu_id = int.from_bytes(hashlib.sha1(uuid).digest()[:7], "little")
        rec = (list(bytes(handle)) + list(int(ioff.value).to_bytes(8, "little", signed=True))
               + list(gpu_id.to_bytes(8, "little")))
        allh = torch.empty((self.W, len(rec)), dtype=torch.uint8, device=device)
        dist.all_gather_into_tensor(allh, torch.tensor(rec, dtype=torch.uint8, device=device), group=group)
        allh = allh.cpu()
        gpus = [int.from_bytes(bytes(allh[s, 72:80].tolist()), "little") for s in range(self.W)]
        if not why and len(set(gpus)) != self.W:
            why = "two ranks share a GPU"
        bases = []
        if not why:
            for s in range(self.W):
                if s == self.r:
                    bases.append(self.own.data_ptr())
                    continue
                h = (ctypes.c_uint8 * 64)(*allh[s, :64].tolist())
                o = int.from_bytes(bytes(allh[s, 64:72].tolist()), "little", signed=True)
                ptr = ctypes.c_void_p()
                if lib.k3_p2p_open(h, o, ctypes.byref(ptr)) != 0:
                    why = f"rank {self.r}: k3_p2p_open of rank {s}'s buffer: {L.last_error()}"
                    break
                self._opened.append((ptr.value, o))
                bases.append(ptr.value)
        ok = torch.tensor([0 if why else 1], dtype=torch.int32, device=device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            self.close()
            raise P2PUnavailable(why or "another rank could not map the exchange buffers")
        self.desc = L.K3P2PGroup(world=self.W, rank=self.r, gather_bytes=self.caps[0],
                                 gather2_bytes=self.caps[1], reduce_bytes=self.caps[2],
                                 base=(ctypes.c_void_p * 32)(*bases))
        # status words of the all-gather and the reduce-scatter (K3_ERR_TIMEOUT after a wait
        # gave up: the group is then out of step and must be rebuilt)
        self.status = torch.zeros(2, dtype=torch.int32, device=device)
        dist.barrier(group=group)                            # every buffer mapped everywhere

    def area(self, i: int) -> int:
        """Device address of this rank's gather area 0, gather area 1 or reduce area."""
        return self.own.data_ptr() + self.offsets[i]

    def allgather(self, src: torch.Tensor, src2: torch.Tensor) -> None:
        lib = L.load_library()
        L.check(lib.k3_p2p_allgather(ctypes.byref(self.desc), src.data_ptr(), src.numel() * src.element_size(),
                                     src2.data_ptr(), src2.numel() * src2.element_size(), 3,
                                     self.status.data_ptr(), L.stream_of(src)), "k3_p2p_allgather")

    def reduce_scatter(self, src: torch.Tensor, out: torch.Tensor) -> None:
        lib = L.load_library()
        L.check(lib.k3_p2p_reduce_scatter(ctypes.byref(self.desc), src.data_ptr(), out.numel(), out.data_ptr(), 3,
                                          self.status[1:].data_ptr(), L.stream_of(src)), "k3_p2p_reduce_scatter")

    def close(self) -> None:
        """Unmaps the peers' buffers (after this rank's work on the device is done; the
        own buffer lives until the object goes)."""
        if not self._opened:
            return
        torch.cuda.synchronize(self.own.device)
        lib = L.load_library()
        for ptr, o in self._opened:
            lib.k3_p2p_close(ptr, o)
        self._opened = []


class _CollTimer:
    def __init__(self, owner, name: str):
        self.owner, self.name, self.ev = owner, name, None

    def __enter__(self):
        if self.owner.collective_timing and not torch.cuda.is_current_stream_capturing():
            self.ev = (torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True))
            self.ev[0].record()
        return self

    def __exit__(self, *exc):
        if self.ev is not None:
            self.ev[1].record()
            self.owner._coll_events.append((self.name, *self.ev))
        return False


class ExpertParallelMoE:
    """This rank's share of an expert-parallel MoE layer on its GPU; ``__call__(x)`` is
    ``LatentMoE.__call__`` (``moe.py:110-132``) for this rank's tokens, computed jointly
    by all ranks of ``group`` (every rank calls with the same M)."""

    def __init__(self, cfg, layer: int, w: dict, expert_source: Callable, group=None,
                 device=None, graphs: bool = True, exchange: str = "auto"):
        if exchange not in ("auto", "gather", "a2a", "p2p"):
            raise ValueError(f"exchange must be 'auto', 'gather', 'a2a' or 'p2p', not {exchange!r}")
        # "gather": NCCL all_gather + reduce_scatter (fixed sizes, captured as a CUDA
        # graph); "a2a": the counted NCCL all-to-all (one host synchronisation per step,
        # launched eagerly); "p2p": the gather step's two exchanges as kernels over NVLink
        # peer memory up to MAX_DECODE_TOKENS tokens per rank (one GPU per rank, CUDA IPC
        # between them; otherwise, and above that size, the NCCL gather step); "auto": as
        # "p2p" -- the fastest measured at decode, and the gather step at prefill.
        self.exchange = exchange
        self.cfg, self.group = cfg, group
        # On NCCL, a step (router, collectives, local experts: ~15 launches) is captured
        # into a CUDA graph per token count at its first call and replayed afterwards, so a
        # decode loop is not bound by the host's launch rate.
        self.graphs = graphs
        self._steps: dict = {}
        self.graph_error: Optional[str] = None
        # set by a profiling caller: CUDA events around each collective of eagerly launched
        # steps (never inside a captured graph), summed by collective_ms()
        self.collective_timing = False
        self._coll_events: list = []
        self.p2p: Optional[P2PExchange] = None
        self.p2p_error: Optional[str] = None             # why the peer-memory exchange is off
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

    def _coll(self, name: str):
        """Context for one collective: with ``collective_timing`` set (and not capturing),
        events on the launching stream before and after it -- the collective's exposed
        time on that stream, waits for slower ranks included."""
        return _CollTimer(self, name)

    def collective_ms(self) -> dict:
        """{collective: total ms} of the timed collectives since the last call (waits for
        their events)."""
        out: dict = {}
        for name, e0, e1 in self._coll_events:
            e1.synchronize()
            out[name] = out.get(name, 0.0) + e0.elapsed_time(e1)
        self._coll_events = []
        return out

    def uses_a2a(self, M: int) -> bool:
        """Whether a call with M tokens per rank runs the counted all-to-all step."""
        return self.exchange == "a2a" and _is_nccl(self.group)

    def capturable(self, M: int) -> bool:
        """Whether a call with M tokens per rank can be captured into a CUDA graph (the
        all-to-all step reads its split sizes on the host)."""
        return not self.uses_a2a(M)

    def _route_packed(self, flat: torch.Tensor) -> torch.Tensor:
        """The router on this rank's tokens; routing packed as [M][2k] int32 (expert ids,
        then the weights' bits)."""
        lib = L.load_library()
        c = self.cfg
        M, H = flat.shape
        k, E = c.num_experts_per_token, c.num_experts
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
        return torch.cat([idx, w.view(torch.int32)], dim=1)

    def _forward_a2a(self, flat: torch.Tensor) -> torch.Tensor:
        """One step with the counted all-to-all exchange (module docstring, steps 1-5), on
        two streams: the shared expert over the own tokens runs on the caller's stream
        while the host waits for the row counts and while the tokens travel; the packing,
        the exchanges and the routed local experts run on a side stream. A rank's own rows
        do not travel back: the combine reads them from the local partial rows."""
        lib = L.load_library()
        k, W, r = self.cfg.num_experts_per_token, self.W, self.r
        M, H = flat.shape
        dev = flat.device
        main = torch.cuda.current_stream(dev)
        side = self._side_stream(dev)
        routing = self._route_packed(flat)
        meta, rows, tok_slot, status = a2a_plan_dev(routing, k, self.E_loc, W, r)
        rcnt = torch.empty(W, dtype=torch.int64, device=dev)
        with self._coll("a2a_counts"):
            dist.all_to_all_single(rcnt, meta[:W], group=self.group)
        host = self._pinned_counts(W)
        host.copy_(torch.cat([meta[:W], rcnt, status[:1].to(torch.int64)]), non_blocking=True)
        ready = torch.cuda.Event()
        ready.record(main)
        y_shared = None
        if self.with_shared:                                   # overlaps the host's wait below
            y_shared = self._shared_part(flat)
        ready.synchronize()                                    # the step's one host synchronisation
        counts = host.tolist()
        send, recv = counts[:W], counts[W:2 * W]
        if counts[2 * W]:
            raise ValueError("k3_ep_a2a_plan: the routing holds an expert id outside the layer")
        S, R = sum(send), sum(recv)
        soff = [sum(send[:d]) for d in range(W)]
        roff = [sum(recv[:d]) for d in range(W)]
        side.wait_event(ready)
        with torch.cuda.stream(side):
            x_send = torch.empty((S, H), dtype=flat.dtype, device=dev)
            r_send = torch.empty((S, 2 * k), dtype=torch.int32, device=dev)
            # the send buffers keep the plan's layout; the own segment is not packed (the own
            # tokens go from flat / routing straight into the receive buffers)
            for lo, hi in ((0, soff[r]), (soff[r] + send[r], S)):
                if hi > lo:
                    gather_rows_dev(flat, rows[lo:hi], hi - lo, status[1:], out=x_send[lo:hi])
                    gather_rows_dev(routing, rows[lo:hi], hi - lo, status[2:], out=r_send[lo:hi])
            x_recv = torch.empty((R, H), dtype=flat.dtype, device=dev)
            r_recv = torch.empty((R, 2 * k), dtype=torch.int32, device=dev)
            ins_x = [flat if d == r else x_send[soff[d]:soff[d] + send[d]] for d in range(W)]
            ins_r = [routing if d == r else r_send[soff[d]:soff[d] + send[d]] for d in range(W)]
            with self._coll("a2a_dispatch"):
                dist.all_to_all([x_recv[roff[d]:roff[d] + recv[d]] for d in range(W)], ins_x, group=self.group)
                dist.all_to_all([r_recv[roff[d]:roff[d] + recv[d]] for d in range(W)], ins_r, group=self.group)
            y_part = torch.empty((R, H), dtype=torch.float32, device=dev)
            ws = L.workspace(dev, lib.k3_moe_ep_local_workspace(self.params, R, 0))
            L.check(lib.k3_moe_ep_local(self.params, x_recv.data_ptr(), L.dtype_code(x_recv), R, r_recv.data_ptr(),
                                        r_recv.data_ptr() + 4 * k, 2 * k, self.lo, 0, 0, y_part.data_ptr(), L.K3_F32,
                                        ws.data_ptr(), ws.numel(), L.stream_of(x_recv)), "k3_moe_ep_local")
            # the own rows do not travel back: zero-size slots for this rank
            y_back = torch.empty((S, H), dtype=torch.float32, device=dev)
            none = y_part[:0]
            with self._coll("a2a_combine"):
                dist.all_to_all([none if d == r else y_back[soff[d]:soff[d] + send[d]] for d in range(W)],
                                [none if d == r else y_part[roff[d]:roff[d] + recv[d]] for d in range(W)],
                                group=self.group)
        main.wait_stream(side)
        for t in (y_part, y_back):                             # read below on the caller's stream
            t.record_stream(main)
        y = a2a_combine_dev(y_back, tok_slot, status[3:], base=y_shared, own=y_part[roff[r]:roff[r] + M], rank=r)
        # the status words of the packing and the combine (non-zero only for a plan that
        # points outside its buffers); read by the tests, not per step
        self.last_a2a_status = status
        return y

    def _side_stream(self, dev: torch.device) -> torch.cuda.Stream:
        st = getattr(self, "_side", None)
        if st is None:
            st = self._side = torch.cuda.Stream(dev)
        return st

    def _pinned_counts(self, W: int) -> torch.Tensor:
        buf = getattr(self, "_counts_host", None)
        if buf is None:
            buf = self._counts_host = torch.empty(2 * W + 1, dtype=torch.int64).pin_memory()
        return buf

    def _shared_part(self, flat: torch.Tensor) -> torch.Tensor:
        """The shared expert over this rank's M own tokens (slot E/W of the pool, weight 1),
        fp32 [M, H]: on the prefill kernels above MAX_DECODE_TOKENS tokens and on the decode
        kernels up to it, as the one-GPU layer runs it."""
        lib = L.load_library()
        M, H = flat.shape
        dev = flat.device
        cache = self.__dict__.setdefault("_shared_cand", {})
        c = cache.get(M)
        if c is None:
            c = cache[M] = (torch.full((M,), self.E_loc, dtype=torch.int32, device=dev),
                            torch.arange(M, dtype=torch.int32, device=dev),
                            torch.ones(M, dtype=torch.float32, device=dev))
        y = torch.empty((M, H), dtype=torch.float32, device=dev)
        args = (flat.data_ptr(), L.dtype_code(flat), M, c[0].data_ptr(), c[1].data_ptr(), c[2].data_ptr(), M,
                y.data_ptr(), L.K3_F32)
        if M > MAX_DECODE_TOKENS:
            ws = L.workspace(dev, lib.k3_moe_pairs_prefill_workspace(self.params, M, M))
            L.check(lib.k3_moe_pairs_prefill(self.params, *args, ws.data_ptr(), ws.numel(), L.stream_of(flat)),
                    "k3_moe_pairs_prefill")
        else:
            ws = L.workspace(dev, lib.k3_moe_pairs_workspace(self.params, M, M))
            L.check(lib.k3_moe_pairs_decode(self.params, *args, ws.data_ptr(), ws.numel(), L.stream_of(flat)),
                    "k3_moe_pairs_decode")
        return y

    def _forward_nccl(self, flat: torch.Tensor) -> torch.Tensor:
        """One step with two all_gathers issued as one NCCL group (tokens; routing packed
        as [M][2k] int32: expert ids, then the weights' bits) and the local experts taken
        straight from the gathered routing on the device (``k3_moe_ep_local``)."""
        lib = L.load_library()
        c = self.cfg
        M, H = flat.shape
        k, W = c.num_experts_per_token, self.W
        dev = flat.device
        routing = self._route_packed(flat)
        p2p = self._p2p_for(flat)
        if p2p is not None:
            # both gathers as one peer-memory kernel: rows land in this rank's gather areas
            with self._coll("p2p_allgather"):
                p2p.allgather(flat, routing)
            x_ptr, r_ptr = p2p.area(0), p2p.area(1)
        else:
            x_all = torch.empty((W * M, H), dtype=flat.dtype, device=dev)
            r_all = torch.empty((W * M, 2 * k), dtype=torch.int32, device=dev)
            # both gathers in one NCCL group: one collective launch per step instead of two
            with self._coll("all_gather"), dist._coalescing_manager(group=self.group, device=dev):
                dist.all_gather_into_tensor(x_all, flat, group=self.group)
                dist.all_gather_into_tensor(r_all, routing, group=self.group)
            x_ptr, r_ptr = x_all.data_ptr(), r_all.data_ptr()
        y_part = torch.empty((W * M, H), dtype=torch.float32, device=dev)
        shared_n = M if self.with_shared else 0
        ws2 = L.workspace(dev, lib.k3_moe_ep_local_workspace(self.params, W * M, shared_n))
        L.check(lib.k3_moe_ep_local(self.params, x_ptr, L.dtype_code(flat), W * M, r_ptr, r_ptr + 4 * k, 2 * k,
                                    self.lo, self.r * M, shared_n, y_part.data_ptr(), L.K3_F32, ws2.data_ptr(),
                                    ws2.numel(), L.stream_of(flat)), "k3_moe_ep_local")
        y = torch.empty((M, H), dtype=torch.float32, device=dev)
        if p2p is not None:
            with self._coll("p2p_reduce_scatter"):
                p2p.reduce_scatter(y_part, y)
        else:
            with self._coll("reduce_scatter"):
                dist.reduce_scatter_tensor(y, y_part, group=self.group)
        return y

    def _p2p_for(self, flat: torch.Tensor) -> Optional[P2PExchange]:
        """The peer-memory exchange for a step over this rank's tokens ``flat`` [M, H],
        built at its first use (collectively: every rank calls with the same M and dtype),
        or None for the NCCL step (too many tokens, or rows whose sizes are not multiples
        of 16 bytes, as the exchange kernels copy 16-byte words)."""
        M, H = flat.shape
        dev = flat.device
        k = self.cfg.num_experts_per_token
        if self.exchange not in ("p2p", "auto") or M > MAX_DECODE_TOKENS or not _is_nccl(self.group):
            return None
        if (M * H * flat.element_size()) % 16 or (M * 2 * k * 4) % 16:
            return None
        if self.p2p is None and self.p2p_error is None:
            H = self.pool.hidden
            try:
                self.p2p = P2PExchange(self.group, dev, MAX_DECODE_TOKENS * H * 4, MAX_DECODE_TOKENS * 2 * k * 4,
                                       MAX_DECODE_TOKENS * H * 4)
            except P2PUnavailable as exc:                    # every rank: the NCCL step instead
                self.p2p_error = str(exc)
        return self.p2p

    def exchange_used(self, M: int) -> str:
        """The exchange a call with M bf16 tokens per rank runs: "a2a", "p2p" or "gather"."""
        if self.uses_a2a(M):
            return "a2a"
        k = self.cfg.num_experts_per_token
        fits = M <= MAX_DECODE_TOKENS and (M * 2 * k * 4) % 16 == 0
        return "p2p" if (self.p2p is not None and fits) else "gather"

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
        """Drop the captured steps and unmap the peers' exchange buffers (before the
        process group is destroyed)."""
        self._steps.clear()
        if self.p2p is not None:
            self.p2p.close()
            self.p2p = None

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        L.require_cuda(x, "x")
        shape = x.shape
        flat = x.reshape(-1, shape[-1])
        if flat.dtype not in (torch.float32, torch.bfloat16):
            flat = flat.float()
        flat = flat.contiguous()
        if self.uses_a2a(flat.shape[0]):
            if torch.cuda.is_current_stream_capturing():
                raise RuntimeError("the all-to-all step reads its split sizes on the host and cannot be "
                                   "captured; use exchange='gather' for a capturable layer")
            return self._forward_a2a(flat).reshape(shape)
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


__all__ = ["ExpertParallelMoE", "P2PExchange", "P2PUnavailable", "a2a_combine_dev", "a2a_plan", "a2a_plan_dev", "ep_forward",
           "gather_rows_dev", "pair_candidates"]
