"""numpy restatement of the reference's MXFP4 expert path (test infrastructure only).

Every function names the reference lines it restates. The reference's own CPU oracle
is ``k3ref`` (torch, fp32); this module restates its arithmetic in numpy so the
checks do not depend on torch's CPU kernels, and adds an fp64 mode that serves as
the "true value" against which both fp32 implementations are measured.

MXFP4 format (reference ``air_llm/models/kimi_k3/mxfp4.py:3-12``):
  * nibble order: low nibble = even element 2i, high nibble = odd element 2i+1;
  * code: bit 3 = sign, bits 0-2 index the E2M1 magnitudes [0,.5,1,1.5,2,3,4,6];
  * scale: one E8M0 byte per 32 contiguous input elements, value 2**(byte-127).
"""
from __future__ import annotations

import ctypes
import os
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Optional

import numpy as np

E2M1 = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0], dtype=np.float32)
GROUP = 32


# ----------------------------------------------------------------------------- codec

def decode_mxfp4(packed: np.ndarray, scales: np.ndarray, group_size: int = GROUP) -> np.ndarray:
    """packed u8 [R, C/2], scales u8 [R, C/group] -> float32 [R, C].

    Restates ``k3ref/weights.py:29-37`` and ``air_llm/models/kimi_k3/mxfp4.py:26-36``
    (``decode_mxfp4_reference``): interleave nibbles (low = even), look up the E2M1
    magnitude, apply the sign bit, multiply by ``ldexp(1, byte-127)``.
    """
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    R, half = packed.shape
    codes = np.empty((R, half * 2), dtype=np.uint8)
    codes[:, 0::2] = packed & 0x0F
    codes[:, 1::2] = (packed >> 4) & 0x0F
    mag = E2M1[codes & 0x07]
    vals = np.where((codes & 0x08) != 0, -mag, mag)
    scale = np.ldexp(np.ones(scales.shape, dtype=np.float32), scales.astype(np.int32) - 127)
    return (vals * np.repeat(scale, group_size, axis=1)).astype(np.float32)


def decode_scale(scales: np.ndarray) -> np.ndarray:
    """E8M0 byte -> float32 by placing the byte in the exponent field.

    Restates ``mxfp4.py:41-55`` (``decode_scale_mlx``): ``(byte << 23).view(f32)``. Exact
    for bytes 1..254; byte 0 gives +0.0 here (the Metal path flushes 2**-127 to zero) and
    byte 255 gives +inf.
    """
    return (np.asarray(scales, dtype=np.uint32) << 23).view(np.float32)


def assert_scales_representable(scales) -> None:
    """Restates ``mxfp4.py:58-65``: scale bytes must lie in 2..252."""
    s = np.asarray(scales)
    lo, hi = int(s.min()), int(s.max())
    if lo < 2 or hi > 252:
        raise ValueError(f"Unsupported MXFP4 scale range {lo}..{hi}; require 2..252 "
                         "to avoid Metal subnormal flushing, overflow, and E8M0 NaN")


def encode_mxfp4(x: np.ndarray, group: int = GROUP):
    """float [R, C] -> (packed u8 [R, C/2], scales u8 [R, C/group]).

    Restates the reference packer ``tools/make_synthetic_k3.py:87-110``: per group,
    exponent e = floor(log2(amax)) - 2 (so the group max lands in [4, 8)), byte =
    clip(e+127, 1, 254), nearest E2M1 magnitude (first index on a tie), low nibble =
    even element.
    """
    R, C = x.shape
    if C % group:
        raise ValueError(f"C={C} is not a multiple of the group size {group}")
    g = np.asarray(x, dtype=np.float32).reshape(R, C // group, group)
    amax = np.abs(g).max(axis=-1)
    with np.errstate(divide="ignore"):
        e = np.floor(np.log2(np.where(amax > 0, amax, 1.0))).astype(np.int32) - 2
    byte = np.clip(e + 127, 1, 254).astype(np.uint8)
    scale = np.ldexp(np.ones_like(byte, dtype=np.float32), byte.astype(np.int32) - 127)
    q = g / scale[..., None]
    sign = np.signbit(q)
    idx = np.abs(np.abs(q)[..., None] - E2M1).argmin(axis=-1).astype(np.uint8)
    codes = (idx | (sign.astype(np.uint8) << 3)).reshape(R, C)
    packed = (codes[:, 0::2] | (codes[:, 1::2] << 4)).astype(np.uint8)
    return packed, byte


def random_mxfp4(rng: np.random.Generator, rows: int, cols: int, scale_lo: int = 120,
                 scale_hi: int = 130):
    """Synthetic MXFP4 tensor: nibbles uniform over the 16 codes, scale bytes uniform in
    [scale_lo, scale_hi] (both inclusive) -- the value distribution BASELINE.json names
    for every config. Returns (packed [rows, cols/2], scales [rows, cols/32])."""
    packed = rng.integers(0, 256, size=(rows, cols // 2), dtype=np.uint8)
    scales = rng.integers(scale_lo, scale_hi + 1, size=(rows, cols // GROUP), dtype=np.uint8)
    return packed, scales


# ------------------------------------------------------------------------------ bf16

def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """float32 -> bf16 bit pattern, round-to-nearest-even (``make_synthetic_k3.py:124-128``)."""
    u = np.asarray(a, dtype=np.float32).view(np.uint32)
    rounded = ((u >> 16) & 1) + 0x7FFF
    return ((u + rounded) >> 16).astype(np.uint16)


def bf16_bits_to_f32(b: np.ndarray) -> np.ndarray:
    """bf16 bit pattern -> float32 (``k3ref/weights.py:40-41``)."""
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ------------------------------------------------------------------------- matvecs

def matvec_fp64(x: np.ndarray, packed: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp64 ``x @ W.T`` on the exactly decoded weights: the yardstick of the reference's
    kernel gate (``tests/test_mxfp4_kernel.py:42-54``)."""
    W = decode_mxfp4(packed, scales).astype(np.float64)
    return np.asarray(x, dtype=np.float64) @ W.T


_LIB = None


def _lib():
    """Load the C restatement (``_build/libk3oracle.so``), building it if absent."""
    global _LIB
    if _LIB is None:
        here = Path(__file__).resolve().parent
        so = here / "_build" / "libk3oracle.so"
        if not so.exists():
            from . import build as _b
            _b.build()
        lib = ctypes.CDLL(str(so))
        lib.k3o_mxfp4_matvec.argtypes = [
            ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64, ctypes.c_void_p, ctypes.c_void_p,
            ctypes.c_int64, ctypes.c_void_p, ctypes.c_int]
        lib.k3o_mxfp4_matvec.restype = ctypes.c_int
        lib.k3o_num_threads.restype = ctypes.c_int
        _LIB = lib
    return _LIB


def matvec_fused(x: np.ndarray, packed: np.ndarray, scales: np.ndarray,
                 threads: int = 0) -> np.ndarray:
    """The reference's fused kernel order, in C: per output, sequential fp32 ``fma`` over
    k pairs with the scale built by ``byte << 23`` (``mxfp4_matvec.py:29-63``).

    x [M, K] any float (cast to fp32 like ``mxfp4_matvec.py:81-82``), packed [N, K/2],
    scales [N, K/32] -> fp32 [M, N]. ``threads`` = 0 uses every host core.
    """
    x = np.ascontiguousarray(x, dtype=np.float32)
    packed = np.ascontiguousarray(packed, dtype=np.uint8)
    scales = np.ascontiguousarray(scales, dtype=np.uint8)
    M, K = x.shape
    N = packed.shape[0]
    if packed.shape[1] * 2 != K:
        raise ValueError(f"K mismatch: x has {K}, packed implies {packed.shape[1] * 2}")
    out = np.empty((M, N), dtype=np.float32)
    rc = _lib().k3o_mxfp4_matvec(x.ctypes.data, M, K, packed.ctypes.data, scales.ctypes.data,
                                 N, out.ctypes.data, int(threads))
    if rc != 0:
        raise ValueError(f"k3o_mxfp4_matvec failed ({rc})")
    return out


def oracle_threads() -> int:
    """Number of OpenMP threads the C restatement uses by default."""
    return int(_lib().k3o_num_threads())


def oracle_isa() -> str:
    """The instruction-set level of the C restatement's clone that runs on this host."""
    return f"x86-64-v{int(_lib().k3o_isa_level())}"


# ----------------------------------------------------------------------- activations

def silu(x):
    """``ops.py:42-43``: x * sigmoid(x)."""
    x = np.asarray(x)
    with np.errstate(over="ignore"):          # exp(-x) -> inf gives the exact limit -0
        return x / (1.0 + np.exp(-x))


def situ_and_mul(g, u, beta: float, linear_beta: Optional[float]):
    """``k3ref/layers.py:53-60`` / ``ops.py:17-28``:
    beta*tanh(g/beta)*sigmoid(g) * linear_beta*tanh(u/linear_beta)."""
    with np.errstate(over="ignore"):
        a = beta * np.tanh(g / beta) * (1.0 / (1.0 + np.exp(-g)))
    if linear_beta is not None:
        u = linear_beta * np.tanh(u / linear_beta)
    return a * u


def rmsnorm(x, w, eps: float):
    """``k3ref/layers.py:46-49`` / ``ops.py:11-14`` (KimiRMSNorm), fp32."""
    xf = np.asarray(x, dtype=np.float32)
    r = 1.0 / np.sqrt((xf * xf).mean(-1, keepdims=True) + np.float32(eps))
    return (np.asarray(w, dtype=np.float32) * (xf * r.astype(np.float32))).astype(np.float32)


def attn_res(prefix_sum, block_residual, proj_w, norm_w, eps: float):
    """``apply_attn_res`` (``air_llm/models/kimi_k3/ops.py:61-74``, ``k3ref/layers.py:83-96``):
    a softmax over the block checkpoints plus the running sum, each scored by its
    RMS-normalised dot with norm_w * proj_w; returns the probability-weighted sum.
    prefix_sum [N, H], block_residual [N, B, H], proj_w [1, H] or [H], norm_w [H]."""
    v = np.concatenate([np.asarray(block_residual, np.float32).reshape(len(prefix_sum), -1, prefix_sum.shape[-1]),
                        np.asarray(prefix_sum, np.float32)[:, None, :]], axis=1)
    k = v / np.sqrt((v * v).mean(-1, keepdims=True) + eps)
    sw = np.asarray(norm_w, np.float32) * np.asarray(proj_w, np.float32).reshape(-1)
    s = (k * sw).sum(-1)
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return (p[..., None] * v).sum(1).astype(np.float32)


def moe_input(prefix_sum, block_residual, res_proj, res_norm, post_norm, eps: float):
    """The MoE input of a decoder layer: rmsnorm(attn_res(...), post_attention_layernorm)
    (``air_llm/models/kimi_k3/layer.py:120-121``)."""
    return rmsnorm(attn_res(prefix_sum, block_residual, res_proj, res_norm, eps), post_norm, eps)


def activation(g, u, act: str, situ_beta: float = 4.0, situ_linear_beta: Optional[float] = 25.0):
    if act == "silu":
        return silu(g) * u
    if act == "situ":
        return situ_and_mul(g, u, situ_beta, situ_linear_beta)
    raise ValueError(f"unknown activation {act!r}")


# ---------------------------------------------------------------------------- router

@dataclass
class RouterResult:
    """``k3ref/layers.py:190-195`` / ``moe.py:32-37``."""
    expert_indices: np.ndarray   # [T, k] int64
    expert_weights: np.ndarray   # [T, k] float32
    raw_scores: np.ndarray       # [T, E] sigmoid(logits)
    corrected_scores: np.ndarray  # raw + e_score_correction_bias


def route(x, gate_w, gate_b, top_k: int, renormalize: bool, scale: float,
          precision: str = "fp32") -> RouterResult:
    """``k3ref/layers.py:214-224`` (KimiMoEGate:703): scores = sigmoid(x_f32 @ W_g^T),
    corrected = scores + bias, idx = top-k(corrected) (selection only), w = scores[idx],
    renormalised by sum + 1e-20 when k > 1, times routed_scaling_factor.

    Indices are returned in descending corrected-score order (ties: lower index first);
    the reference's ``torch.topk(sorted=False)`` order is unspecified, so callers compare
    index SETS per row, as ``tests/test_moe_mlx.py:70-75`` does.
    """
    dt = np.float64 if precision == "fp64" else np.float32
    flat = np.asarray(x, dtype=np.float32).reshape(-1, np.shape(x)[-1]).astype(dt)
    W = np.asarray(gate_w, dtype=np.float32).astype(dt)
    logits = flat @ W.T
    with np.errstate(over="ignore"):
        scores = (1.0 / (1.0 + np.exp(-logits))).astype(dt)
    bias = np.zeros(W.shape[0], dt) if gate_b is None else np.asarray(gate_b, dtype=np.float32).astype(dt)
    corrected = scores + bias[None, :]
    E = W.shape[0]
    # stable descending order: sort by (-value, index)
    order = np.lexsort((np.broadcast_to(np.arange(E), corrected.shape), -corrected), axis=-1)
    idx = order[:, :top_k]
    w = np.take_along_axis(scores, idx, axis=-1)
    if top_k > 1 and renormalize:
        w = w / (w.sum(axis=-1, keepdims=True) + 1e-20)
    return RouterResult(idx.astype(np.int64), (w * scale).astype(np.float32),
                        scores.astype(np.float32), corrected.astype(np.float32))


def topk_gap(corrected: np.ndarray, top_k: int) -> np.ndarray:
    """Per row, corrected[k-th largest] - corrected[(k+1)-th largest]: how far the
    selection boundary is from a tie. Rows whose gap is below the fp32 rounding of the
    logits cannot have a reproducible top-k across two fp32 implementations."""
    s = -np.sort(-np.asarray(corrected, dtype=np.float64), axis=-1)
    if s.shape[-1] <= top_k:
        return np.full(s.shape[0], np.inf)
    return s[:, top_k - 1] - s[:, top_k]


# ---------------------------------------------------------------------------- experts

ExpertSource = Callable[[int, str], tuple]


class DecodedExperts:
    """Memoised decode of (packed, scales) pairs: ``WeightStore.expert`` (``k3ref/
    weights.py:117-122``) with a cache so a parity test decodes each projection once."""

    def __init__(self, source: ExpertSource):
        self.source = source
        self._cache: dict = {}

    def __call__(self, e: int, which: str) -> np.ndarray:
        key = (e, which)
        if key not in self._cache:
            p, s = self.source(e, which)
            self._cache[key] = decode_mxfp4(p, s)
        return self._cache[key]


def expert_forward(h, w1, w3, w2, act: str = "silu", situ_beta: float = 4.0,
                   situ_linear_beta: Optional[float] = 25.0, precision: str = "fp32"):
    """``k3ref/layers.py:226-234``: act(h @ w1^T, h @ w3^T) @ w2^T, fp32 (or fp64)."""
    dt = np.float64 if precision == "fp64" else np.float32
    h = np.asarray(h, dtype=np.float32).astype(dt)
    g = h @ np.asarray(w1, dt).T
    u = h @ np.asarray(w3, dt).T
    a = activation(g, u, act, situ_beta, situ_linear_beta).astype(dt)
    return a @ np.asarray(w2, dt).T


@dataclass
class MoESpec:
    """The MoE fields of ``K3Config`` (``air_llm/models/kimi_k3/config.py:11-41``) that the
    expert path reads, plus which latent/shared variant applies."""
    num_experts: int
    top_k: int
    routed_scaling_factor: float = 1.0
    renormalize: bool = True
    activation: str = "silu"          # "silu" or "situ" (Kimi-K3)
    situ_beta: float = 4.0
    situ_linear_beta: Optional[float] = 25.0
    rms_norm_eps: float = 1e-5


def moe_forward(x, spec: MoESpec, gate_w, gate_b, experts: ExpertSource,
                shared: Optional[dict] = None, latent: Optional[dict] = None,
                precision: str = "fp32"):
    """``k3ref/layers.py:241-261`` (LatentMoE.__call__), with the variant choices explicit.

    * ``latent`` None: experts act on the hidden state directly;
      otherwise ``{"down": [L,H], "up": [H,L], "norm": [L]}`` applies
      hidden->latent, then rmsnorm and latent->hidden around the routed sum
      (``k3ref/layers.py:248,258-259``).
    * ``shared`` None: no shared expert; ``{"kind": "mxfp4", "w1": (p, s), "w3": ..., "w2":
      ...}`` for an MXFP4 shared expert (BASELINE); ``{"kind": "dense", "gate": ..., "up":
      ..., "down": ...}`` for the reference's bf16 dense shared experts
      (``k3ref/layers.py:236-239``). The shared expert acts on the ORIGINAL hidden.
    * Routed experts are visited in ascending id order and accumulated with
      ``y[tok] += out * w[tok, slot]`` (``k3ref/layers.py:252-256``).
    Returns (y float32 shaped like x, RouterResult).
    """
    dt = np.float64 if precision == "fp64" else np.float32
    x = np.asarray(x, dtype=np.float32)
    orig = x.shape
    flat = x.reshape(-1, orig[-1])
    r = route(flat, gate_w, gate_b, spec.top_k, spec.renormalize,
              spec.routed_scaling_factor, precision)
    dec = DecodedExperts(experts)
    h = flat.astype(dt) if latent is None else flat.astype(dt) @ np.asarray(latent["down"], dt).T
    y = np.zeros((flat.shape[0], h.shape[1]), dtype=dt)
    idx = r.expert_indices
    for e in sorted(set(idx.reshape(-1).tolist())):
        tok, slot = np.nonzero(idx == e)
        out = expert_forward(h[tok], dec(e, "w1"), dec(e, "w3"), dec(e, "w2"), spec.activation,
                             spec.situ_beta, spec.situ_linear_beta, precision)
        np.add.at(y, tok, out * r.expert_weights[tok, slot][:, None].astype(dt))
    if latent is not None:
        y = rmsnorm(y.astype(np.float32), latent["norm"], spec.rms_norm_eps).astype(dt)
        y = y @ np.asarray(latent["up"], dt).T
    if shared is not None:
        xs = flat.astype(dt)
        if shared["kind"] == "mxfp4":
            w1 = decode_mxfp4(*shared["w1"])
            w3 = decode_mxfp4(*shared["w3"])
            w2 = decode_mxfp4(*shared["w2"])
        else:
            w1, w3, w2 = shared["gate"], shared["up"], shared["down"]
        y = y + expert_forward(xs, w1, w3, w2, spec.activation, spec.situ_beta,
                               spec.situ_linear_beta, precision)
    return y.astype(np.float32).reshape(orig[:-1] + (y.shape[-1],)), r


def rel_l2(a, b) -> float:
    """||a-b|| / ||b|| in fp64."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    den = np.linalg.norm(b)
    return float(np.linalg.norm(a - b) / (den if den > 0 else 1.0))


def rel_max(a, b) -> float:
    """max|a-b| / max|b|: the reference kernel gate's measure (``test_mxfp4_kernel.py:52``)."""
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.abs(a - b).max() / max(np.abs(b).max(), 1e-30))
