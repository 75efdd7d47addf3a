"""Dense bf16 matvecs of the Kimi-K3 layer around the MXFP4 experts.

The reference computes these in fp32 over bf16 checkpoint weights:

* the latent projections ``h = flat @ down.T`` and ``rmsnorm(y) @ up.T``
  (``air_llm/models/kimi_k3/moe.py:116,128-129``, ``ops.rmsnorm`` at ``ops.py:11-14``);
* the bf16 shared expert ``situ(x @ sh_gate.T, x @ sh_up.T) @ sh_down.T``
  (``moe.py:105-107``);
* the streamed lm_head argmax ``KimiK3.logits`` (``model.py:111-133``).

Up to 8 tokens run on the library's HBM-streaming matvec (``k3_dense_matvec``,
``k3_lm_head_argmax``): every weight byte read once, fp32 products and sums, fused
rmsnorm on the input and fused activation on the gate/up pair. More tokens make these
plain GEMMs, which run on cuBLAS bf16 tensor cores with the fp32 input split into two
bf16 pieces (hi + lo, about 16 bits of the input kept) and fp32 outputs.
"""
from __future__ import annotations

from typing import Optional, Sequence, Tuple

import torch

from . import _lib as L

MAX_DENSE_TOKENS = 8

# (weight bf16 [N][K], input [M][K], rmsnorm weight or None, eps[, act_input]); with
# act_input true the input is [M][2K] = [gate | up] and the segment reads act(gate, up)
Seg = Tuple


def device_weight(t, device) -> torch.Tensor:
    """Checkpoint weight on the device: bf16 when every value is bf16-representable (the
    checkpoint's own dtype), else fp32 (those run on the fp32 GEMM path only)."""
    t = t if isinstance(t, torch.Tensor) else torch.as_tensor(t)
    t = t.to(device)
    if t.dtype == torch.bfloat16:
        return t.contiguous()
    b = t.to(torch.bfloat16)
    if torch.equal(b.float(), t.float()):
        return b.contiguous()
    return t.float().contiguous()


def _native_ok(segs: Sequence[Seg]) -> bool:
    for w, x, *_ in segs:
        if (w.dtype != torch.bfloat16 or w.dim() != 2 or w.stride(1) != 1 or w.shape[1] % 8
                or w.stride(0) % 8 or w.data_ptr() % 16 or x.shape[0] > MAX_DENSE_TOKENS):
            return False
    return True


def _rmsnorm(x: torch.Tensor, norm_w: torch.Tensor, eps: float) -> torch.Tensor:
    xf = x.float()
    return norm_w * (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps))


def _gemm(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 out [M][N] (+)= x [M][K] . W [N][K]^T on this library's tcgen05 GEMM
    (``k3_dense_gemm``): bf16 W, fp32 x as bf16 hi + lo pieces; ``out`` given: accumulate
    into it."""
    xc = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
    if xc.stride(-1) != 1:
        xc = xc.contiguous()
    M, K = xc.shape
    N = w.shape[0]
    acc = out is not None
    if out is None:
        out = torch.empty((M, N), dtype=torch.float32, device=x.device)
    lib = L.load_library()
    ws = L.workspace(x.device, lib.k3_dense_gemm_workspace(M, K))
    L.check(lib.k3_dense_gemm(xc.data_ptr(), L.dtype_code(xc), xc.stride(0), M, K, w.data_ptr(), w.stride(0), N,
                              out.data_ptr(), out.stride(0), int(acc), ws.data_ptr(), ws.numel(), L.stream_of(xc)),
            "k3_dense_gemm")
    return out


def _gemm_ok(x: torch.Tensor, w: torch.Tensor) -> bool:
    return (w.is_cuda and x.is_cuda and w.dtype == torch.bfloat16 and w.dim() == 2 and w.stride(1) == 1 and w.shape[1] % 64 == 0
            and w.stride(0) % 8 == 0 and w.data_ptr() % 16 == 0 and x.shape[-1] == w.shape[1])


def _mm_f32(x: torch.Tensor, w: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """fp32 x [M][K] times bf16 W [N][K]^T in fp32 (added into ``out`` when given): the
    library's tcgen05 GEMM for bf16 weights whose K is a multiple of 64; other shapes (the
    reference's tiny test models) multiply in fp32 on the GPU."""
    if _gemm_ok(x, w):
        return _gemm(x, w, out)
    y = x.float() @ w.float().t()
    return y if out is None else out.add_(y)


def _activation(kind: int, g: torch.Tensor, u: torch.Tensor, beta: float, lbeta: float) -> torch.Tensor:
    if kind == L.K3_ACT_SILU:
        return torch.nn.functional.silu(g) * u
    a = beta * torch.tanh(g / beta) * torch.sigmoid(g)
    if lbeta > 0:
        u = lbeta * torch.tanh(u / lbeta)
    return a * u


def matvec(segs: Sequence[Seg], N: int, combine: int = L.K3_DENSE_SUM, activation: int = L.K3_ACT_SITU,
           situ_beta: float = 4.0, situ_linear_beta: float = -1.0,
           out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """out [M][N] = sum_s X_s W_s^T (``K3_DENSE_SUM``) or act(X W_0^T, X W_1^T)
    (``K3_DENSE_ACT``: two segments over the first segment's X). A segment with a norm
    weight uses rmsnorm(X) instead of X; one marked act_input uses act(X[:, :K], X[:, K:2K])."""
    x0 = segs[0][1]
    L.require_cuda(x0, "x")
    M = x0.shape[0]
    dev = x0.device
    if _native_ok(segs):
        lib = L.load_library()
        arr = (L.K3DenseSeg * len(segs))()
        keep = []
        for i, sg in enumerate(segs):
            w, x, nw, eps = sg[:4]
            act_in = bool(sg[4]) if len(sg) > 4 else False
            xc = x if x.dtype in (torch.float32, torch.bfloat16) else x.float()
            xc = xc if xc.stride(-1) == 1 and xc.stride(0) >= xc.shape[1] else xc.contiguous()
            nwc = None if nw is None else nw.float().contiguous()
            keep += [xc, nwc]
            arr[i] = L.K3DenseSeg(w.data_ptr(), w.stride(0), w.shape[1], xc.data_ptr(), L.dtype_code(xc),
                                  xc.stride(0), None if nwc is None else nwc.data_ptr(), float(eps),
                                  int(act_in))
        out = torch.empty((M, N), dtype=out_dtype, device=dev)
        K1 = segs[1][0].shape[1] if len(segs) > 1 else 0
        ws = L.workspace(dev, lib.k3_dense_workspace(M, N, len(segs), segs[0][0].shape[1], K1))
        L.check(lib.k3_dense_matvec(arr, len(segs), M, N, combine, activation, float(situ_beta),
                                    float(situ_linear_beta), out.data_ptr(), L.dtype_code(out), N,
                                    ws.data_ptr(), ws.numel(), L.stream_of(x0)), "k3_dense_matvec")
        return out
    # more than 8 tokens: GEMMs on the tensor cores (k3_dense_gemm); summed segments
    # accumulate into one output in segment order
    def seg_input(sg):
        w, x, nw, eps = sg[:4]
        if len(sg) > 4 and sg[4]:
            K = w.shape[1]
            x = _activation(activation, x[:, :K].float(), x[:, K:2 * K].float(), situ_beta, situ_linear_beta)
        return x if nw is None else _rmsnorm(x, nw, eps)

    if combine == L.K3_DENSE_ACT:
        g, u = (_mm_f32(seg_input(sg), sg[0]) for sg in segs[:2])
        y = _activation(activation, g, u, situ_beta, situ_linear_beta)
    else:
        y = None
        for sg in segs:
            y = _mm_f32(seg_input(sg), sg[0], y)
    return y.to(out_dtype)


def lm_head_argmax(h: torch.Tensor, w: torch.Tensor, return_logits: bool = False):
    """``KimiK3.logits`` (``model.py:111-133``) for the last position: (argmax id, max
    logit, bytes streamed) of h [H] . W[n] over the vocabulary W bf16 [V][H]; with
    ``return_logits`` also the fp32 logits [V]. Device scalars are read back once."""
    L.require_cuda(h, "h")
    v = h.reshape(-1, h.shape[-1])[-1]
    v = v if v.dtype in (torch.float32, torch.bfloat16) else v.float()
    v = v.contiguous()
    if w.dtype != torch.bfloat16 or w.stride(1) != 1 or w.stride(0) != w.shape[1]:
        raise ValueError("lm_head weight must be contiguous bf16 [V][H]")
    V, H = w.shape
    if v.shape[0] != H:
        raise ValueError(f"hidden size {v.shape[0]} != lm_head columns {H}")
    lib = L.load_library()
    idx = torch.empty(1, dtype=torch.int32, device=v.device)
    val = torch.empty(1, dtype=torch.float32, device=v.device)
    logits = torch.empty(V, dtype=torch.float32, device=v.device) if return_logits else None
    ws = L.workspace(v.device, lib.k3_lm_head_workspace(H, V))
    L.check(lib.k3_lm_head_argmax(v.data_ptr(), L.dtype_code(v), H, w.data_ptr(), V, idx.data_ptr(),
                                  val.data_ptr(), None if logits is None else logits.data_ptr(),
                                  ws.data_ptr(), ws.numel(), L.stream_of(v)), "k3_lm_head_argmax")
    out = (int(idx.item()), float(val.item()), V * H * 2)
    return (*out, logits) if return_logits else out


__all__ = ["MAX_DENSE_TOKENS", "device_weight", "matvec", "lm_head_argmax"]
