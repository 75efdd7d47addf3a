"""Streamed-expert decode: the routed experts live in pinned host
memory and only the ones a token routes to are copied to HBM.

The reference streams experts from SSD on every use (``air_llm/models/kimi_k3/
loader.py:229-266``, one contiguous read of packed + scales per projection) and runs
them through the Metal kernel. Here the host tier is pinned memory holding every expert
already in the block-scaled kernels' layout (contiguous 128-row x 128-byte tiles of the
E2M1 codes and the re-laid E8M0 scale chunks, ``k3_mxfp4_tiles`` /
``k3_mxfp4_scales_tc``), so a copy lands ready to use. Per layer:

1. the router (weights resident in HBM) picks the token's experts; their ids come back to
   the host (one small device->host read: copies need host addresses);
2. a side stream copies each routed expert's six arrays (tiles and scales of w1, w3, w2)
   into a staging slot with ``cudaMemcpyAsync`` (one call per array) and records an event
   per expert;
3. meanwhile the compute stream runs the shared expert (resident, staging slot S);
4. the compute stream runs each routed expert (``k3_moe_pairs_decode`` over its staging
   slot) once that expert's event fires, so the copies of later experts overlap the
   compute of earlier ones, then adds the shared output last, like ``moe.py:131``.
"""
from __future__ import annotations

import ctypes
from typing import Callable

import torch

from . import _lib as L
from .moe import SHARED, LatentMoE
from .mxfp4 import packed_tiles, scales_tc

WHICH = ("w1", "w3", "w2")


def _relaid(trip):
    """((tiles, tc) for w1, w3, w2) of one expert given its device (packed, scales) pairs."""
    return [(packed_tiles(p)[0], scales_tc(s)[0]) for p, s in trip]


class HostExpertStore:
    """Every routed expert of a layer in pinned host memory, in the block-scaled layout:
    ``tiles[w]`` [E, rows/128, cols/256, 128, 128] and ``tc[w]`` [E, rows/128, cols/128,
    512] per projection w (uint8)."""

    def __init__(self, num_experts: int, expert: Callable, device="cuda"):
        self.E = num_experts
        self.tiles, self.tc = {}, {}
        for e in range(num_experts):
            for w, (t, s) in zip(WHICH, _relaid(expert(e))):
                if e == 0:
                    self.tiles[w] = torch.empty((num_experts, *t.shape), dtype=torch.uint8, pin_memory=True)
                    self.tc[w] = torch.empty((num_experts, *s.shape), dtype=torch.uint8, pin_memory=True)
                self.tiles[w][e].copy_(t)
                self.tc[w][e].copy_(s)
        torch.cuda.synchronize(device)

    def nbytes_expert(self) -> int:
        return sum(self.tiles[w][0].numel() + self.tc[w][0].numel() for w in WHICH)


class DiskExpertStore:
    """The routed experts of one layer read from the checkpoint on every use: the
    reference's SSD tier (``air_llm/models/kimi_k3/loader.py:229-266``). An expert's six
    tensors (packed + scale of w1, w3, w2) are read with as few ``pread`` calls as their
    manifest records allow (one per run of contiguous tensors: one for the whole expert
    when the shard stores them back to back) into a pinned host slot, copied to a device
    slot, and re-laid there into the block-scaled layout (``k3_mxfp4_tiles`` /
    ``k3_mxfp4_scales_tc``) straight into the streaming slot the kernels read."""

    def __init__(self, src, layer: int, num_experts: int, device="cuda"):
        self.src, self.layer, self.E = src, layer, num_experts
        self.device = torch.device(device)
        self.plan = [self._expert_plan(e) for e in range(num_experts)]
        self.bytes_read = 0
        self.host = self.dev = None
        self.host_free = []

    def _expert_plan(self, e: int):
        """(reads [(path, file offset, nbytes, host offset)], host bytes, device bytes,
        parts {(which, kind): (host offset, device offset, nbytes, shape)}) of expert e:
        the host slot mirrors the file runs, the device slot puts every tensor at a
        256-byte boundary for the re-layout kernels."""
        recs = []
        for w in WHICH:
            for name in self.src.expert_names(self.layer, e, w):
                path, off, r = self.src._locate(name)
                recs.append((path, off, r, w, name.rsplit(".", 1)[1]))
        recs.sort(key=lambda t: (str(t[0]), t[1]))
        reads, parts, pos, dpos = [], {}, 0, 0
        for path, off, r, w, kind in recs:
            n = r["nbytes"]
            if reads and reads[-1][0] == path and reads[-1][1] + reads[-1][2] == off:
                reads[-1] = (path, reads[-1][1], reads[-1][2] + n, reads[-1][3])
            else:
                reads.append((path, off, n, pos))
            parts[(w, kind)] = (pos, dpos, n, tuple(r["shape"]))
            pos += n
            dpos += (n + 255) // 256 * 256
        return reads, pos, dpos, parts

    def nbytes_expert(self) -> int:
        return max(p[1] for p in self.plan)

    def bind(self, slots: int) -> None:
        if self.host is None or self.host.shape[0] < slots:
            self.host = torch.empty((slots, max(p[1] for p in self.plan)), dtype=torch.uint8, pin_memory=True)
            self.dev = torch.empty((slots, max(p[2] for p in self.plan)), dtype=torch.uint8, device=self.device)
            self.host_free = [None] * slots

    def stage_one(self, moe: "StreamedMoE", j: int, e: int, stream: torch.cuda.Stream) -> None:
        """Reads expert e (blocking pread on this thread) and queues its copy and re-layout
        into streaming slot j on ``stream``; moe.events[j] fires when it is ready."""
        from .loader import read_ranges
        self.bind(moe.S)
        if self.host_free[j] is not None:
            self.host_free[j].synchronize()                  # the slot's previous copies are done
        reads, _, _, parts = self.plan[e]
        base = self.host[j].data_ptr()
        by_file = {}
        for path, off, n, pos in reads:
            by_file.setdefault(path, []).append((off, n, base + pos))
        for path, rr in by_file.items():
            self.bytes_read += read_ranges(path, rr, self.src.threads)
        lib = L.load_library()
        with torch.cuda.stream(stream):
            for hp, dp, n, _ in parts.values():
                self.dev[j, dp:dp + n].copy_(self.host[j, hp:hp + n], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(stream)
            self.host_free[j] = ev
            for w in WHICH:
                (_, dpk, _, (rows, half)), (_, dsc, _, _) = parts[(w, "weight_packed")], parts[(w, "weight_scale")]
                L.check(lib.k3_mxfp4_tiles(self.dev[j].data_ptr() + dpk, rows, 2 * half, 1,
                                           moe.tiles[w][j].data_ptr(), stream.cuda_stream), "k3_mxfp4_tiles")
                L.check(lib.k3_mxfp4_scales_tc(self.dev[j].data_ptr() + dsc, rows, 2 * half, 1,
                                               moe.tc[w][j].data_ptr(), stream.cuda_stream), "k3_mxfp4_scales_tc")
            moe.events[j].record(stream)


class StreamedMoE:
    """One MoE layer (BASELINE semantics: MXFP4 routed experts in ``store``, resident
    MXFP4 shared expert) whose routed experts are copied to HBM on demand."""

    def __init__(self, cfg, layer: int, w: dict, store, shared: Callable, device="cuda"):
        self.cfg, self.store = cfg, store
        self.device = torch.device(device)
        self.router = LatentMoE(cfg, layer, w, lambda *a: None, fused=True, device=self.device)
        self.S = cfg.num_experts_per_token                   # staging slots (M = 1 decode)
        sh = _relaid(shared())                               # the shared expert, resident
        self.tiles, self.tc = {}, {}
        for w_, (t, s) in zip(WHICH, sh):
            self.tiles[w_] = torch.empty((self.S + 1, *t.shape), dtype=torch.uint8, device=self.device)
            self.tc[w_] = torch.empty((self.S + 1, *s.shape), dtype=torch.uint8, device=self.device)
            self.tiles[w_][self.S].copy_(t)
            self.tc[w_][self.S].copy_(s)
        H, I = cfg.hidden_size, cfg.moe_intermediate_size
        self.desc = L.K3ExpertPool(num_slots=self.S + 1,
                                   w1_scales_tc=self.tc["w1"].data_ptr(), w3_scales_tc=self.tc["w3"].data_ptr(),
                                   w2_scales_tc=self.tc["w2"].data_ptr(), w1_tiles=self.tiles["w1"].data_ptr(),
                                   w3_tiles=self.tiles["w3"].data_ptr(), w2_tiles=self.tiles["w2"].data_ptr())
        self.params = L.K3MoEParams(
            hidden=H, inter=I, num_experts=self.S, top_k=cfg.num_experts_per_token,
            renormalize=int(bool(cfg.moe_renormalize)), routed_scaling_factor=float(cfg.routed_scaling_factor),
            has_shared=1, activation=L.K3_ACT_SILU, situ_beta=4.0, situ_linear_beta=-1.0,
            experts=None, pool=ctypes.pointer(self.desc))
        self.copy_stream = torch.cuda.Stream(self.device)
        self.events = [torch.cuda.Event() for _ in range(self.S)]

    def _pairs(self, x, slot, tok, w):
        lib = L.load_library()
        T, H = x.shape
        y = torch.empty((T, H), dtype=torch.float32, device=x.device)
        ws = L.workspace(x.device, lib.k3_moe_pairs_workspace(self.params, T, slot.numel()))
        L.check(lib.k3_moe_pairs_decode(self.params, x.data_ptr(), L.dtype_code(x), T, slot.data_ptr(),
                                        tok.data_ptr(), w.data_ptr(), slot.numel(), y.data_ptr(), L.K3_F32,
                                        ws.data_ptr(), ws.numel(), L.stream_of(x)), "k3_moe_pairs_decode")
        return y

    def stage(self, experts):
        """Copy the given experts into staging slots 0.. on the side stream (one event each)."""
        cur = torch.cuda.current_stream(self.device)
        self.copy_stream.wait_stream(cur)                    # slots are free once earlier compute ran
        with torch.cuda.stream(self.copy_stream):
            for j, e in enumerate(experts):
                for w_ in WHICH:
                    self.tiles[w_][j].copy_(self.store.tiles[w_][e], non_blocking=True)
                    self.tc[w_][j].copy_(self.store.tc[w_][e], non_blocking=True)
                self.events[j].record(self.copy_stream)

    def __call__(self, x: torch.Tensor, stage: bool = True) -> torch.Tensor:
        """y = routed experts (streamed) + shared expert, for M tokens routing to at most
        ``top_k`` distinct experts in total (M = 1 decode). ``stage=False`` skips the
        copies (the routed experts must already sit in slots 0.. in ascending id order).

        Each routed expert runs as soon as its own copy has landed (one pairs call per
        expert, waiting on that expert's event), so only the last expert's compute trails
        the copies; the outputs are summed in ascending expert order and the shared
        expert's output is added last, the order of ``moe.py:120-131``."""
        flat = x.reshape(-1, x.shape[-1])
        M = flat.shape[0]
        dev = flat.device
        rr = self.router.route(flat)
        ids = rr.expert_indices.cpu()                        # host addresses need the ids
        experts = sorted(set(ids.reshape(-1).tolist()))
        if len(experts) > self.S:
            raise NotImplementedError(f"{len(experts)} distinct experts exceed the {self.S} staging slots")
        # a disk store reads expert j+1 on the host while the GPU runs expert j
        lazy = stage and hasattr(self.store, "stage_one")
        if lazy:
            self.copy_stream.wait_stream(torch.cuda.current_stream(self.device))
        elif stage:
            self.stage(experts)
        else:
            for j in range(len(experts)):
                self.events[j].record(torch.cuda.current_stream(self.device))
        # pairs grouped by expert (tokens ascending within an expert), uploaded once
        k = ids.shape[1]
        flat_ids = ids.reshape(-1).tolist()
        order = sorted(range(len(flat_ids)), key=lambda p: (flat_ids[p], p))
        slot_of = {e: j for j, e in enumerate(experts)}
        host = torch.tensor([[slot_of[flat_ids[p]], p // k, p] for p in order], dtype=torch.int32)
        dev_idx = host.to(dev, non_blocking=False)
        slot = dev_idx[:, 0].contiguous()
        tok = dev_idx[:, 1].contiguous()
        wts = rr.expert_weights.reshape(-1).float()[dev_idx[:, 2].long()].contiguous()
        own = torch.arange(M, dtype=torch.int32, device=dev)
        y_sh = self._pairs(flat, torch.full((M,), self.S, dtype=torch.int32, device=dev), own,
                           torch.ones(M, dtype=torch.float32, device=dev))
        cur = torch.cuda.current_stream(self.device)
        y, start = None, 0
        counts = [sum(1 for e in flat_ids if e == ex) for ex in experts]
        for j, n in enumerate(counts):
            if lazy:
                self.store.stage_one(self, j, experts[j], self.copy_stream)
            cur.wait_event(self.events[j])
            y_j = self._pairs(flat, slot[start:start + n], tok[start:start + n], wts[start:start + n])
            y = y_j if y is None else y + y_j
            start += n
        return (y + y_sh).reshape(x.shape[:-1] + (y.shape[-1],))


__all__ = ["HostExpertStore", "DiskExpertStore", "StreamedMoE", "SHARED"]
