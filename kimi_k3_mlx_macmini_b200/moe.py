"""Router + MoE block on the B200 -- the drop-in for ``air_llm/models/kimi_k3/moe.py``.

``LatentMoE(cfg, layer, w, expert_source, fused=True)`` keeps the reference's
constructor, methods (``route``, ``expert_forward``, ``shared_forward``, ``__call__``)
and semantics (``moe.py:40-132``; oracle ``k3ref/layers.py:188-261``):

* router: sigmoid scores, correction bias for SELECTION only, weights gathered from the
  raw scores, renormalised by sum + 1e-20, times ``routed_scaling_factor``;
* routed experts visited in ascending id order, ``y[tok] += out * w[tok, slot]``;
* with the latent wrapper (``routed_expert_down_proj``/``up_proj``/``norm`` in ``w``):
  hidden -> latent before the experts, rmsnorm + latent -> hidden after;
* shared experts act on the ORIGINAL hidden: dense when ``w`` holds
  ``shared_experts.*`` weights (Kimi-K3), MXFP4 when ``expert_source(layer, "shared",
  which)`` provides them (the BASELINE layer), absent otherwise.

The expert weights returned by ``expert_source`` are uploaded once into HBM (the
reference streams them per call from SSD; on a B200 the whole layer fits) and bound
into a device pointer table that the fused kernels index. Activation: ``cfg.activation``
("situ" for Kimi-K3 -- the default -- or "silu" for SwiGLU).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass
from typing import Callable, Optional

import numpy as np
import torch

from . import _lib as L
from . import dense as D
from .mxfp4 import decode_mxfp4, mxfp4_matvec_fused, packed_tiles, scale_minmax, scales_tc

SHARED = "shared"
WHICH = ("w1", "w3", "w2")
MAX_DECODE_TOKENS = 8


@dataclass
class MoEConfig:
    """The MoE fields of ``K3Config`` (``air_llm/models/kimi_k3/config.py:11-41``) plus the
    activation choice; any object with these attributes works."""
    hidden_size: int
    num_experts: int
    num_experts_per_token: int
    moe_intermediate_size: int
    routed_expert_hidden_size: int
    routed_scaling_factor: float = 1.0
    moe_renormalize: bool = True
    situ_beta: float = 4.0
    situ_linear_beta: Optional[float] = 25.0
    rms_norm_eps: float = 1e-5
    num_shared_experts: int = 1
    activation: str = "situ"


@dataclass
class RouterResult:
    """``moe.py:32-37``."""
    expert_indices: torch.Tensor    # [N, top_k] int64, descending corrected score
    expert_weights: torch.Tensor    # [N, top_k] fp32
    raw_scores: torch.Tensor        # [N, num_experts] sigmoid(logits)
    corrected_scores: torch.Tensor  # raw + e_score_correction_bias


def _as_device_u8(a, device) -> torch.Tensor:
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    if not isinstance(a, torch.Tensor):
        a = torch.as_tensor(np.asarray(a))
    if a.dtype != torch.uint8:
        raise ValueError(f"MXFP4 tensors must be uint8, got {a.dtype}")
    return a.to(device, non_blocking=False).contiguous()


def _as_device(a, device, dtype=None) -> torch.Tensor:
    if isinstance(a, np.ndarray):
        a = torch.from_numpy(np.ascontiguousarray(a))
    a = torch.as_tensor(a)
    return a.to(device=device, dtype=dtype or a.dtype).contiguous()


class ExpertPool:
    """HBM-resident MXFP4 expert weights of one layer.

    Each projection kind lives in one contiguous pool -- w1/w3 packed ``[slots][I][H/2]``
    and scales ``[slots][I][H/32]``, w2 packed ``[slots][H][I/2]`` and scales
    ``[slots][H][I/32]`` -- with slot e = expert e and slot E = the shared expert. The
    pools feed the TMA kernels (``k3_expert_pool``); a device pointer table
    (``k3_expert_ptrs[slots]``) into the same memory feeds the generic kernels.

    ``expert_source(layer, e, which) -> (packed, scales)`` is called once per projection
    (the reference calls it on every use, ``moe.py:86``). Scale ranges are checked at
    upload like ``loader.py:246-247``.
    """

    def __init__(self, layer: int, num_experts: int, expert_source: Callable, device,
                 with_shared: bool, check_scales: bool = True, block_scaled: bool = True):
        self.layer, self.E, self.device = layer, num_experts, torch.device(device)
        self.with_shared = with_shared
        ids = list(range(num_experts)) + ([SHARED] if with_shared else [])
        self.slots = len(ids)
        self.pools = None
        for i, e in enumerate(ids):
            trip = [expert_source(layer, e, which) for which in WHICH]
            if self.pools is None:
                self.pools = [(torch.empty((self.slots, *np.shape(pk)), dtype=torch.uint8, device=self.device),
                               torch.empty((self.slots, *np.shape(sc)), dtype=torch.uint8, device=self.device))
                              for pk, sc in trip]
            for (pp, sp), (pk, sc) in zip(self.pools, trip):
                if tuple(np.shape(pk)) != tuple(pp.shape[1:]) or tuple(np.shape(sc)) != tuple(sp.shape[1:]):
                    raise ValueError(f"expert {e}: projection shape {tuple(np.shape(pk))} differs from expert 0")
                pp[i].copy_(_as_device_u8(pk, self.device))
                sp[i].copy_(_as_device_u8(sc, self.device))
        if check_scales:
            lo, hi = 255, 0
            for _, sp in self.pools:
                a, b = scale_minmax(sp)
                lo, hi = min(lo, a), max(hi, b)
            if lo < 2 or hi > 252:
                raise ValueError(f"Unsupported MXFP4 scale range {lo}..{hi}; require 2..252 "
                                 "to avoid Metal subnormal flushing, overflow, and E8M0 NaN")
        self.tensors = [tuple((pp[i], sp[i]) for pp, sp in self.pools) for i in range(self.slots)]
        table = torch.tensor([[t.data_ptr() for pair in trip for t in pair] for trip in self.tensors],
                             dtype=torch.int64)
        self.table = table.to(self.device)
        (w1p, w1s), (w3p, w3s), (w2p, w2s) = self.pools
        # scales re-laid once for the block-scaled tensor-core path (when the shapes allow)
        self.scales_tc = self.tiles = None
        if block_scaled and all(sp.shape[1] % 128 == 0 and (sp.shape[2] * 32) % 256 == 0
                                for _, sp in self.pools):
            self.scales_tc = [scales_tc(sp) for _, sp in self.pools]
            self.tiles = [packed_tiles(pp) for pp, _ in self.pools]
        tc = [t.data_ptr() for t in self.scales_tc] if self.scales_tc is not None else [None] * 3
        tl = [t.data_ptr() for t in self.tiles] if self.tiles is not None else [None] * 3
        self.desc = L.K3ExpertPool(w1_packed=w1p.data_ptr(), w1_scales=w1s.data_ptr(),
                                   w3_packed=w3p.data_ptr(), w3_scales=w3s.data_ptr(),
                                   w2_packed=w2p.data_ptr(), w2_scales=w2s.data_ptr(),
                                   num_slots=self.slots, w1_scales_tc=tc[0], w3_scales_tc=tc[1],
                                   w2_scales_tc=tc[2], w1_tiles=tl[0], w3_tiles=tl[1], w2_tiles=tl[2])
        self.desc_f16 = L.K3ExpertPool(w1_packed=w1p.data_ptr(), w1_scales=w1s.data_ptr(),
                                       w3_packed=w3p.data_ptr(), w3_scales=w3s.data_ptr(),
                                       w2_packed=w2p.data_ptr(), w2_scales=w2s.data_ptr(),
                                       num_slots=self.slots)
        self.inter, self.hidden = w1p.shape[1], w1p.shape[2] * 2

    def get(self, e, which: str):
        i = self.E if e == SHARED else int(e)
        return self.tensors[i][WHICH.index(which)]

    def nbytes(self) -> int:
        extra = [t for group in (self.scales_tc, self.tiles) if group is not None for t in group]
        return sum(pp.numel() + sp.numel() for pp, sp in self.pools) + sum(t.numel() for t in extra)


class LatentMoE:
    """Drop-in for ``air_llm.models.kimi_k3.moe.LatentMoE`` on CUDA tensors."""

    def __init__(self, cfg, layer: int, w: dict, expert_source: Callable, fused: bool = True,
                 device=None):
        self.cfg, self.L, self.src, self.fused = cfg, layer, expert_source, fused
        self.device = torch.device(device) if device is not None else torch.device("cuda")
        self.act = getattr(cfg, "activation", "situ")
        if self.act not in ("silu", "situ"):
            raise ValueError(f"unknown activation {self.act!r}")
        gw = _as_device(w["gate.weight"], self.device)
        self.gate_w = gw.to(torch.bfloat16).contiguous()       # stored bf16 on disk
        if gw.dtype == torch.float32 and not torch.equal(self.gate_w.float(), gw):
            raise ValueError("gate.weight is not bf16-representable; the router reads bf16 weights")
        b = w.get("gate.e_score_correction_bias")
        self.gate_b = None if b is None else _as_device(b, self.device, torch.float32)
        # dense weights stay bf16 (the checkpoint dtype) for the streaming matvecs
        self.latent = "routed_expert_down_proj.weight" in w
        if self.latent:
            self.down = D.device_weight(w["routed_expert_down_proj.weight"], self.device)
            self.up = D.device_weight(w["routed_expert_up_proj.weight"], self.device)
            self.norm_w = _as_device(w["routed_expert_norm.weight"], self.device, torch.float32)
        self.dense_shared = "shared_experts.gate_proj.weight" in w
        if self.dense_shared:
            self.sh_gate = D.device_weight(w["shared_experts.gate_proj.weight"], self.device)
            self.sh_up = D.device_weight(w["shared_experts.up_proj.weight"], self.device)
            self.sh_down = D.device_weight(w["shared_experts.down_proj.weight"], self.device)
        # the three bf16 projections of the hidden state -- latent down, shared gate, shared
        # up -- in one [L + 2 I_shared][H] matrix (the old names are row views of it), so a
        # decode step streams them in one launch
        self.front = None
        if self.latent and self.dense_shared:
            parts = [self.down, self.sh_gate, self.sh_up]
            if all(t.dtype == torch.bfloat16 for t in parts) and len({t.shape[1] for t in parts}) == 1:
                self.front = torch.cat(parts, 0).contiguous()
                n0, n1 = self.down.shape[0], self.down.shape[0] + self.sh_gate.shape[0]
                self.down, self.sh_gate, self.sh_up = self.front[:n0], self.front[n0:n1], self.front[n1:]
        self.mxfp4_shared = (not self.dense_shared) and getattr(cfg, "num_shared_experts", 0) > 0
        self._pool: Optional[ExpertPool] = None
        # the contiguous pools feed the TMA kernels; False forces the pointer-table kernels
        self.use_pool = True
        # block-scaled (kind::mxf4) tensor-core kernels when the pool carries re-laid
        # scales; False runs the f16 tensor-core kernels over the same pool
        self.block_scaled = True

    # ------------------------------------------------------------------ plumbing
    @property
    def pool(self) -> ExpertPool:
        if self._pool is None:
            self._pool = ExpertPool(self.L, self.cfg.num_experts, self.src, self.device,
                                    with_shared=self.mxfp4_shared)
        return self._pool

    @property
    def tiled(self) -> bool:
        """True when the fused decode kernels tile this layer (H, I multiples of 128,
        <= 1024 experts, top-k <= 16); otherwise experts run one by one through
        ``mxfp4_matvec_fused`` (still on the GPU)."""
        c, p = self.cfg, self.pool
        return (p.hidden % 128 == 0 and p.inter % 128 == 0 and c.num_experts <= 1024
                and c.num_experts_per_token <= 16)

    def _params(self, *, num_experts=None, top_k=None, has_shared=None) -> L.K3MoEParams:
        """The call's k3_moe_params, built once per variant (a decode call is short enough
        that rebuilding the ctypes struct every time shows in its host time)."""
        key = (num_experts, top_k, has_shared, self.block_scaled, self.use_pool)
        cache = self.__dict__.setdefault("_pcache", {})
        hit = cache.get(key)
        if hit is None:
            hit = cache[key] = self._make_params(num_experts=num_experts, top_k=top_k, has_shared=has_shared)
        return hit

    def _make_params(self, *, num_experts=None, top_k=None, has_shared=None) -> L.K3MoEParams:
        c, pool = self.cfg, self.pool
        lb = getattr(c, "situ_linear_beta", None)
        return L.K3MoEParams(
            hidden=pool.hidden, inter=pool.inter,
            num_experts=self.cfg.num_experts if num_experts is None else num_experts,
            top_k=c.num_experts_per_token if top_k is None else top_k,
            renormalize=int(bool(c.moe_renormalize)),
            routed_scaling_factor=float(c.routed_scaling_factor),
            has_shared=int(self.mxfp4_shared if has_shared is None else has_shared),
            activation=L.K3_ACT_SITU if self.act == "situ" else L.K3_ACT_SILU,
            situ_beta=float(getattr(c, "situ_beta", 4.0)),
            situ_linear_beta=-1.0 if lb is None else float(lb),
            experts=pool.table.data_ptr(),
            pool=(ctypes.pointer(pool.desc if self.block_scaled else pool.desc_f16)
                  if self.use_pool else None))

    @property
    def prefill_ok(self) -> bool:
        """True when calls of more than 8 tokens run on the block-scaled grouped GEMMs
        (``k3_moe_prefill``): the pool carries tiles and re-laid scales, H and I are
        multiples of 256."""
        p = self.pool
        return (self.use_pool and self.block_scaled and p.tiles is not None and p.scales_tc is not None
                and p.hidden % 256 == 0 and p.inter % 256 == 0 and self.cfg.num_experts <= 1024
                and self.cfg.num_experts_per_token <= 32)

    def _experts_decode(self, h: torch.Tensor, idx: torch.Tensor, w: torch.Tensor,
                        params: L.K3MoEParams) -> torch.Tensor:
        """y[t] = sum_slot w[t,slot] * expert_{idx[t,slot]}(h[t]) (+ MXFP4 shared), fp32."""
        lib = L.load_library()
        out = torch.empty((h.shape[0], self.pool.hidden), dtype=torch.float32, device=h.device)
        if h.shape[0] > MAX_DECODE_TOKENS and self.prefill_ok:
            hc = h.contiguous()
            ic = idx.to(torch.int32).contiguous()
            wc = w.to(torch.float32).contiguous()
            ws = L.workspace(h.device, lib.k3_moe_prefill_workspace(params, hc.shape[0]))
            L.check(lib.k3_moe_experts_prefill(params, hc.data_ptr(), L.dtype_code(hc), hc.shape[0],
                                               ic.data_ptr(), wc.data_ptr(), out.data_ptr(), L.K3_F32,
                                               ws.data_ptr(), ws.numel(), L.stream_of(hc)),
                    "k3_moe_experts_prefill")
            return out
        for m0 in range(0, h.shape[0], MAX_DECODE_TOKENS):
            hc = h[m0:m0 + MAX_DECODE_TOKENS].contiguous()
            ic = idx[m0:m0 + MAX_DECODE_TOKENS].to(torch.int32).contiguous()
            wc = w[m0:m0 + MAX_DECODE_TOKENS].to(torch.float32).contiguous()
            M = hc.shape[0]
            need = lib.k3_moe_decode_workspace(params, M)
            L.check(0 if need else L.K3_ERR_INVALID, "k3_moe_decode_workspace")
            ws = L.workspace(h.device, need)
            oc = out[m0:m0 + M]
            L.check(lib.k3_moe_experts_decode(params, hc.data_ptr(), L.dtype_code(hc), M,
                                              ic.data_ptr(), wc.data_ptr(), oc.data_ptr(), L.K3_F32,
                                              ws.data_ptr(), ws.numel(), L.stream_of(hc)),
                    "k3_moe_experts_decode")
        return out

    def _activation(self, g: torch.Tensor, u: torch.Tensor) -> torch.Tensor:
        if self.act == "silu":
            return torch.nn.functional.silu(g) * u
        c = self.cfg
        beta, lb = float(c.situ_beta), getattr(c, "situ_linear_beta", None)
        a = beta * torch.tanh(g / beta) * torch.sigmoid(g)
        if lb is not None:
            u = lb * torch.tanh(u / lb)
        return a * u

    # -------------------------------------------------------------------- routing
    def route(self, x: torch.Tensor) -> RouterResult:
        """``moe.py:65-76`` on the device (``k3_moe_route``)."""
        L.require_cuda(x, "x")
        c = self.cfg
        flat = x.reshape(-1, x.shape[-1])
        if flat.dtype not in (torch.float32, torch.bfloat16):
            flat = flat.float()
        flat = flat.contiguous()
        N, E, k = flat.shape[0], c.num_experts, c.num_experts_per_token
        dev = flat.device
        idx = torch.empty((N, k), dtype=torch.int32, device=dev)
        w = torch.empty((N, k), dtype=torch.float32, device=dev)
        raw = torch.empty((N, E), dtype=torch.float32, device=dev)
        cor = torch.empty((N, E), dtype=torch.float32, device=dev)
        lib = L.load_library()
        ws = L.workspace(dev, lib.k3_moe_route_workspace(N, E))
        L.check(lib.k3_moe_route(flat.data_ptr(), L.dtype_code(flat), N, flat.shape[1],
                                 self.gate_w.data_ptr(),
                                 None if self.gate_b is None else self.gate_b.data_ptr(), E, k,
                                 int(bool(c.moe_renormalize)), float(c.routed_scaling_factor),
                                 idx.data_ptr(), w.data_ptr(), raw.data_ptr(), cor.data_ptr(),
                                 ws.data_ptr(), ws.numel(), L.stream_of(flat)), "k3_moe_route")
        return RouterResult(idx.long(), w, raw, cor)

    # -------------------------------------------------------------------- experts
    def _proj(self, h: torch.Tensor, e, which: str) -> torch.Tensor:
        """``moe.py:79-88``: h @ W.T for one MXFP4 projection."""
        p, s = self.pool.get(e, which)
        if self.fused:
            return mxfp4_matvec_fused(h, p, s)
        return h.float() @ decode_mxfp4(p, s, out_dtype=torch.bfloat16).float().T

    def expert_forward(self, h: torch.Tensor, e: int) -> torch.Tensor:
        """One routed expert, unweighted (``moe.py:90-103``): act(h W1^T, h W3^T) W2^T."""
        L.require_cuda(h, "h")
        if not self.fused or not self.tiled:
            return self._proj(self._activation(self._proj(h, e, "w1"), self._proj(h, e, "w3")), e, "w2")
        h2 = h.reshape(-1, h.shape[-1])
        if h2.dtype not in (torch.float32, torch.bfloat16):
            h2 = h2.float()
        M = h2.shape[0]
        if self._ffn_ok(M):
            # the expert's FFN alone: no routing plan, three launches
            lib = L.load_library()
            h2 = h2.contiguous()
            params = self._params(top_k=1, has_shared=0)
            y = torch.empty((M, self.pool.hidden), dtype=torch.float32, device=h.device)
            ws = L.workspace(h.device, lib.k3_moe_expert_forward_workspace(params, M))
            L.check(lib.k3_moe_expert_forward(params, h2.data_ptr(), L.dtype_code(h2), M, int(e), y.data_ptr(),
                                              L.K3_F32, ws.data_ptr(), ws.numel(), L.stream_of(h2)),
                    "k3_moe_expert_forward")
            return y.reshape(*h.shape[:-1], y.shape[-1])
        idx = torch.full((M, 1), int(e), dtype=torch.int32, device=h.device)
        w = torch.ones((M, 1), dtype=torch.float32, device=h.device)
        y = self._experts_decode(h2, idx, w, self._params(top_k=1, has_shared=0))
        return y.reshape(*h.shape[:-1], y.shape[-1])

    def _ffn_ok(self, M: int) -> bool:
        """True when ``expert_forward`` of M tokens runs ``k3_moe_expert_forward``: at most
        8 tokens on the block-scaled pool, H and I multiples of 512."""
        p = self.pool
        return (M <= MAX_DECODE_TOKENS and self.use_pool and self.block_scaled and p.scales_tc is not None
                and p.hidden % 512 == 0 and p.inter % 512 == 0)

    def _act_args(self):
        c = self.cfg
        lb = getattr(c, "situ_linear_beta", None)
        return dict(activation=L.K3_ACT_SITU if self.act == "situ" else L.K3_ACT_SILU,
                    situ_beta=float(getattr(c, "situ_beta", 4.0)),
                    situ_linear_beta=-1.0 if lb is None else float(lb))

    def _dense_shared_act(self, flat: torch.Tensor) -> torch.Tensor:
        """act(x W_gate^T, x W_up^T) of the bf16 shared expert, fp32 [M][I_shared]."""
        return D.matvec([(self.sh_gate, flat, None, 0.0), (self.sh_up, flat, None, 0.0)],
                        self.sh_gate.shape[0], combine=L.K3_DENSE_ACT, **self._act_args())

    def shared_forward(self, x: torch.Tensor) -> torch.Tensor:
        """Shared experts on the original hidden (``moe.py:105-107``)."""
        if self.dense_shared:
            flat = x.reshape(-1, x.shape[-1])
            a = self._dense_shared_act(flat)
            y = D.matvec([(self.sh_down, a, None, 0.0)], self.sh_down.shape[0])
            return y.reshape(*x.shape[:-1], y.shape[-1])
        if not self.mxfp4_shared:
            return torch.zeros((*x.shape[:-1], self.cfg.hidden_size), dtype=torch.float32,
                               device=x.device)
        if not self.tiled:
            xf = x.float()
            return self._proj(self._activation(self._proj(xf, SHARED, "w1"),
                                               self._proj(xf, SHARED, "w3")), SHARED, "w2")
        x2 = x.reshape(-1, x.shape[-1])
        if x2.dtype not in (torch.float32, torch.bfloat16):
            x2 = x2.float()
        M = x2.shape[0]
        E = self.cfg.num_experts
        idx = torch.full((M, 1), E, dtype=torch.int32, device=x.device)
        w = torch.ones((M, 1), dtype=torch.float32, device=x.device)
        y = self._experts_decode(x2, idx, w, self._params(num_experts=E + 1, top_k=1, has_shared=0))
        return y.reshape(*x.shape[:-1], y.shape[-1])

    # -------------------------------------------------------------------- forward
    def _fused_decode(self, flat: torch.Tensor):
        """route + routed experts + MXFP4 shared expert in one library call per <= 8 tokens."""
        lib = L.load_library()
        params = self._params()
        k = self.cfg.num_experts_per_token
        T, dev = flat.shape[0], flat.device
        y = torch.empty((T, self.pool.hidden), dtype=torch.float32, device=dev)
        idx = torch.empty((T, k), dtype=torch.int32, device=dev)
        w = torch.empty((T, k), dtype=torch.float32, device=dev)
        stream = L.stream_of(flat)
        wsz = self.__dict__.setdefault("_wsz", {})
        xdt, xsz = L.dtype_code(flat), flat.element_size()
        gb = None if self.gate_b is None else self.gate_b.data_ptr()
        for m0 in range(0, T, MAX_DECODE_TOKENS):
            M = min(MAX_DECODE_TOKENS, T - m0)
            need = wsz.get(M)
            if need is None:
                need = wsz[M] = lib.k3_moe_decode_workspace(params, M)
            ws = L.workspace(dev, need, stream)
            H = flat.shape[1]
            L.check(lib.k3_moe_decode(params, flat.data_ptr() + m0 * H * xsz, xdt, M, self.gate_w.data_ptr(), gb,
                                      y.data_ptr() + m0 * y.shape[1] * 4, L.K3_F32, idx.data_ptr() + m0 * k * 4,
                                      w.data_ptr() + m0 * k * 4, ws.data_ptr(), ws.numel(), stream),
                    "k3_moe_decode")
        return y, idx, w

    def _fused_prefill(self, flat: torch.Tensor):
        """route + routed experts + MXFP4 shared expert for any number of tokens in one
        library call (``k3_moe_prefill``: router GEMM, grouped block-scaled GEMMs)."""
        lib = L.load_library()
        params = self._params()
        T, k = flat.shape[0], self.cfg.num_experts_per_token
        y = torch.empty((T, self.pool.hidden), dtype=torch.float32, device=flat.device)
        idx = torch.empty((T, k), dtype=torch.int32, device=flat.device)
        w = torch.empty((T, k), dtype=torch.float32, device=flat.device)
        ws = L.workspace(flat.device, lib.k3_moe_prefill_workspace(params, T))
        L.check(lib.k3_moe_prefill(params, flat.data_ptr(), L.dtype_code(flat), T, self.gate_w.data_ptr(),
                                   None if self.gate_b is None else self.gate_b.data_ptr(), y.data_ptr(),
                                   L.K3_F32, idx.data_ptr(), w.data_ptr(), ws.data_ptr(), ws.numel(),
                                   L.stream_of(flat)), "k3_moe_prefill")
        return y, idx, w

    def _latent_fused_ok(self, flat: torch.Tensor) -> bool:
        return (self.latent and self.fused and self.tiled and self.use_pool and self.block_scaled
                and flat.shape[0] <= MAX_DECODE_TOKENS and self.pool.scales_tc is not None
                and flat.shape[1] % 512 == 0)

    def _fused_latent_decode(self, flat: torch.Tensor, h: torch.Tensor, return_router: bool):
        """Routed experts of a latent MoE for <= 8 tokens in one library call
        (``k3_moe_decode_latent``): route on the hidden state ``flat``, experts on the
        latent ``h``. Returns (y_latent fp32, RouterResult or None)."""
        lib = L.load_library()
        params = self._params(has_shared=0)       # a shared expert acts on the hidden state
        M, k, E = flat.shape[0], self.cfg.num_experts_per_token, self.cfg.num_experts
        dev = flat.device
        y = torch.empty((M, self.pool.hidden), dtype=torch.float32, device=dev)
        idx = torch.empty((M, k), dtype=torch.int32, device=dev)
        w = torch.empty((M, k), dtype=torch.float32, device=dev)
        logits = torch.empty((M, E), dtype=torch.float32, device=dev) if return_router else None
        hc = h.contiguous()
        ws = L.workspace(dev, lib.k3_moe_decode_latent_workspace(params, M, flat.shape[1]))
        L.check(lib.k3_moe_decode_latent(params, flat.data_ptr(), L.dtype_code(flat), flat.shape[1],
                                         hc.data_ptr(), L.dtype_code(hc), M, self.gate_w.data_ptr(),
                                         None if self.gate_b is None else self.gate_b.data_ptr(),
                                         y.data_ptr(), L.K3_F32, idx.data_ptr(), w.data_ptr(),
                                         None if logits is None else logits.data_ptr(), ws.data_ptr(),
                                         ws.numel(), L.stream_of(flat)), "k3_moe_decode_latent")
        r = None
        if return_router:
            raw = torch.sigmoid(logits)
            cor = raw if self.gate_b is None else raw + self.gate_b
            r = RouterResult(idx.long(), w, raw, cor)
        return y, r

    def __call__(self, x: torch.Tensor, return_router: bool = False):
        """``moe.py:110-132``: returns y shaped like x (fp32), and the RouterResult if asked."""
        L.require_cuda(x, "x")
        orig = x.shape
        flat = x.reshape(-1, orig[-1])
        if flat.dtype not in (torch.float32, torch.bfloat16):
            flat = flat.float()
        flat = flat.contiguous()
        if (not self.latent and not self.dense_shared and not return_router and self.fused
                and self.tiled):
            if flat.shape[0] > MAX_DECODE_TOKENS and self.prefill_ok:
                y, _, _ = self._fused_prefill(flat)
                return y.reshape(*orig[:-1], y.shape[-1])
            y, _, _ = self._fused_decode(flat)
            return y.reshape(*orig[:-1], y.shape[-1])
        gu = None                        # [gate | up] of the bf16 shared expert, when fused
        if self._latent_fused_ok(flat):
            # latent decode: hidden -> latent matvec (with the shared expert's gate and up
            # rows when they share its matrix), then one fused router launch (routing on
            # the hidden state, E2M1 pieces of the latent) and the block-scaled experts
            if self.front is not None:
                hf = D.matvec([(self.front, flat, None, 0.0)], self.front.shape[0])
                h, gu = hf[:, :self.down.shape[0]], hf[:, self.down.shape[0]:]
            else:
                h = D.matvec([(self.down, flat, None, 0.0)], self.down.shape[0])
            y, r = self._fused_latent_decode(flat, h, return_router)
        else:
            r = self.route(flat)
            h = flat if not self.latent else D.matvec([(self.down, flat, None, 0.0)], self.down.shape[0])
            if self.fused and self.tiled:
                y = self._experts_decode(h.contiguous(), r.expert_indices, r.expert_weights,
                                         self._params(has_shared=0))
            else:
                y = torch.zeros((flat.shape[0], h.shape[1]), dtype=torch.float32, device=x.device)
                for e in sorted(set(r.expert_indices.reshape(-1).tolist())):
                    tok, slot = (r.expert_indices == e).nonzero(as_tuple=True)
                    y.index_add_(0, tok, self.expert_forward(h[tok].float(), e)
                                 * r.expert_weights[tok, slot, None])
        if self.latent:
            # rmsnorm(y) @ up.T (+ the bf16 shared expert's down projection) in one matvec
            segs = [(self.up, y, self.norm_w, float(self.cfg.rms_norm_eps))]
            if self.dense_shared and gu is not None:
                segs.append((self.sh_down, gu, None, 0.0, True))         # act(gate, up) staged in
            elif self.dense_shared:
                segs.append((self.sh_down, self._dense_shared_act(flat), None, 0.0))
            y = D.matvec(segs, self.up.shape[0], **self._act_args())
            if not self.dense_shared:
                y = y + self.shared_forward(flat)
        else:
            y = y + self.shared_forward(flat)
        y = y.reshape(*orig[:-1], y.shape[-1])
        return (y, r) if return_router else y
