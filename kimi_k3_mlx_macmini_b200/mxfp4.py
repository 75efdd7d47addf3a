"""MXFP4 codec and fused matvec on the B200 -- the drop-in for
``air_llm/models/kimi_k3/mxfp4.py`` and ``air_llm/kernels/metal/mxfp4_matvec.py``.

Same names, argument meaning and errors as the reference:

* ``mxfp4_matvec_fused(x, packed, scales)`` -> fp32 [M, N]; ValueError on K mismatch
  (``mxfp4_matvec.py:75-96``).
* ``expert_projection(x, packed, scales)`` accepts 1-D or 2-D x (``:99-105``).
* ``decode_mxfp4(packed, scales, group_size, out_dtype)`` (``mxfp4.py:68-81``; named
  ``decode_mxfp4_mlx`` in the reference, exported here under both names).
* ``decode_scale(scales)`` (``mxfp4.py:41-55``), ``assert_scales_representable`` (``:58-65``).
* ``mxfp4_matvec(x, packed, scales)`` -- the unfused path: dequantise to bf16, then a
  bf16 GEMM with fp32 output (``mxfp4.py:84-92``).

All tensors live on a CUDA device; the work is enqueued on the current stream.
"""
from __future__ import annotations

import torch

from . import _lib as L

GROUP = 32


def _u8(t: torch.Tensor, name: str) -> torch.Tensor:
    L.require_cuda(t, name)
    if t.dtype != torch.uint8:
        raise ValueError(f"{name} must be uint8, got {t.dtype}")
    return t.contiguous()


def mxfp4_matvec_fused(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                       out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """y = x @ W.T with W given by (packed [N, K/2], scales [N, K/32]); x [M, K] any of
    f32/bf16 (other float types are cast to fp32, as the reference casts to fp32); fp32
    accumulation; out [M, N] in ``out_dtype`` (fp32 by default, like the reference)."""
    L.require_cuda(x, "x")
    packed, scales = _u8(packed, "packed"), _u8(scales, "scales")
    if x.dim() != 2:
        raise ValueError(f"x must be [M, K], got {tuple(x.shape)}")
    M, K = x.shape
    N = packed.shape[0]
    if packed.shape[1] * 2 != K:
        raise ValueError(f"K mismatch: x has {K}, packed implies {packed.shape[1] * 2}")
    if scales.shape != (N, K // GROUP):
        raise ValueError(f"scales must be [{N}, {K // GROUP}], got {tuple(scales.shape)}")
    if x.dtype not in (torch.float32, torch.bfloat16):
        x = x.float()
    x = x.contiguous()
    out = torch.empty((M, N), dtype=out_dtype, device=x.device)
    if M == 0 or N == 0:
        return out
    lib = L.load_library()
    need = lib.k3_mxfp4_matvec_workspace(M, K, N)
    ws = L.workspace(x.device, need)
    L.check(lib.k3_mxfp4_matvec(x.data_ptr(), L.dtype_code(x), M, K, packed.data_ptr(),
                                scales.data_ptr(), N, out.data_ptr(), L.dtype_code(out),
                                ws.data_ptr(), ws.numel(), L.stream_of(x)), "k3_mxfp4_matvec")
    return out


def expert_projection(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """``mxfp4_matvec.py:99-105``: 1-D x gives a 1-D result."""
    squeeze = x.dim() == 1
    y = mxfp4_matvec_fused(x.reshape(1, -1) if squeeze else x, packed, scales)
    return y.reshape(-1) if squeeze else y


def decode_mxfp4(packed: torch.Tensor, scales: torch.Tensor, group_size: int = GROUP,
                 out_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """packed [R, C/2], scales [R, C/32] -> [R, C] fp32 or bf16, bit-exact."""
    packed, scales = _u8(packed, "packed"), _u8(scales, "scales")
    if group_size != GROUP:
        raise ValueError("group_size must be 32")
    R, half = packed.shape
    C = half * 2
    if C % GROUP or scales.shape != (R, C // GROUP):
        raise ValueError(f"scales must be [{R}, {C // GROUP}], got {tuple(scales.shape)}")
    if out_dtype not in (torch.float32, torch.bfloat16):
        raise ValueError("out_dtype must be float32 or bfloat16")
    out = torch.empty((R, C), dtype=out_dtype, device=packed.device)
    lib = L.load_library()
    L.check(lib.k3_mxfp4_dequant(packed.data_ptr(), scales.data_ptr(), R, C, GROUP, out.data_ptr(),
                                 L.dtype_code(out), L.stream_of(packed)), "k3_mxfp4_dequant")
    return out


decode_mxfp4_mlx = decode_mxfp4          # the reference's name for the device decoder


def decode_scale(scales: torch.Tensor) -> torch.Tensor:
    """E8M0 byte -> fp32 2**(b-127) by placing the byte in the exponent field
    (``mxfp4.py:41-55``): exact for 1..254."""
    L.require_cuda(scales, "scales")
    return (scales.to(torch.int32) << 23).view(torch.float32)


def scale_minmax(scales: torch.Tensor) -> tuple[int, int]:
    """(min, max) scale byte, reduced on the device (one small host read)."""
    scales = _u8(scales, "scales")
    mm = torch.empty(2, dtype=torch.int32, device=scales.device)
    lib = L.load_library()
    L.check(lib.k3_mxfp4_scale_minmax(scales.data_ptr(), scales.numel(), mm.data_ptr(),
                                      L.stream_of(scales)), "k3_mxfp4_scale_minmax")
    lo, hi = mm.tolist()
    return int(lo), int(hi)


def scales_tc(scales: torch.Tensor) -> torch.Tensor:
    """E8M0 scales ``[..., rows, cols/32]`` re-laid for the block-scaled tensor-core path:
    ``[batch, rows/128, cols/128, 512]`` chunks (``k3_mxfp4_scales_tc``)."""
    scales = _u8(scales, "scales")
    if scales.dim() < 2:
        raise ValueError("scales must be at least 2-D [rows, cols/32]")
    rows, g = scales.shape[-2], scales.shape[-1]
    batch = scales.numel() // max(1, rows * g)
    out = torch.empty((batch, rows // 128, (g * 32) // 128, 512), dtype=torch.uint8, device=scales.device)
    lib = L.load_library()
    L.check(lib.k3_mxfp4_scales_tc(scales.data_ptr(), rows, g * 32, batch, out.data_ptr(),
                                   L.stream_of(scales)), "k3_mxfp4_scales_tc")
    return out


def packed_tiles(packed: torch.Tensor) -> torch.Tensor:
    """Packed E2M1 codes ``[..., rows, cols/2]`` re-laid into contiguous 128-row x 128-byte
    tiles ``[batch, rows/128, cols/256, 128, 128]`` (``k3_mxfp4_tiles``)."""
    packed = _u8(packed, "packed")
    if packed.dim() < 2:
        raise ValueError("packed must be at least 2-D [rows, cols/2]")
    rows, half = packed.shape[-2], packed.shape[-1]
    batch = packed.numel() // max(1, rows * half)
    out = torch.empty((batch, rows // 128, (half * 2) // 256, 128, 128), dtype=torch.uint8,
                      device=packed.device)
    lib = L.load_library()
    L.check(lib.k3_mxfp4_tiles(packed.data_ptr(), rows, half * 2, batch, out.data_ptr(),
                               L.stream_of(packed)), "k3_mxfp4_tiles")
    return out


def assert_scales_representable(scales: torch.Tensor) -> None:
    """``mxfp4.py:58-65``: scale bytes must lie in 2..252."""
    lo, hi = scale_minmax(scales)
    if lo < 2 or hi > 252:
        raise ValueError(f"Unsupported MXFP4 scale range {lo}..{hi}; require 2..252 "
                         "to avoid Metal subnormal flushing, overflow, and E8M0 NaN")


def mxfp4_matvec(x: torch.Tensor, packed: torch.Tensor, scales: torch.Tensor,
                 group_size: int = GROUP, accum_dtype: torch.dtype = torch.float32) -> torch.Tensor:
    """Unfused path (``mxfp4.py:84-92``): decode to bf16 (lossless), bf16 GEMM, fp32 out."""
    w = decode_mxfp4(packed, scales, group_size, out_dtype=torch.bfloat16)
    return (x.to(torch.bfloat16) @ w.T).to(accum_dtype)
