"""ctypes binding of ``libk3b200.so`` (declared in ``include/k3b200.h``).

The library is the only compute path: if it is missing or no CUDA device is present,
every call raises. PyTorch supplies device memory, the current stream and dtype tags.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

import torch

LIB_PATH = Path(__file__).resolve().with_name("libk3b200.so")

K3_OK, K3_ERR_INVALID, K3_ERR_UNSUPPORTED, K3_ERR_CUDA, K3_ERR_WORKSPACE, K3_ERR_TIMEOUT, K3_ERR_IO = range(7)
K3_F32, K3_BF16, K3_F16 = 0, 1, 2
K3_ACT_SILU, K3_ACT_SITU = 0, 1
K3_DENSE_SUM, K3_DENSE_ACT = 0, 1
PROF_KINDS = ("router", "topk", "gateup", "down", "matvec", "other", "dense")

_DTYPE = {torch.float32: K3_F32, torch.bfloat16: K3_BF16, torch.float16: K3_F16}

_vp, _i64, _i32, _f32, _sz = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int, ctypes.c_float, ctypes.c_size_t


class K3ExpertPtrs(ctypes.Structure):
    _fields_ = [(n, ctypes.c_void_p) for n in ("w1_packed", "w1_scales", "w3_packed", "w3_scales",
                                               "w2_packed", "w2_scales")]


class K3ExpertPool(ctypes.Structure):
    _fields_ = ([(n, ctypes.c_void_p) for n in ("w1_packed", "w1_scales", "w3_packed", "w3_scales",
                                                "w2_packed", "w2_scales")] + [("num_slots", ctypes.c_int64)]
                + [(n, ctypes.c_void_p) for n in ("w1_scales_tc", "w3_scales_tc", "w2_scales_tc",
                                                  "w1_tiles", "w3_tiles", "w2_tiles")])


class K3MoEParams(ctypes.Structure):
    _fields_ = [("hidden", ctypes.c_int64), ("inter", ctypes.c_int64),
                ("num_experts", ctypes.c_int64), ("top_k", ctypes.c_int32),
                ("renormalize", ctypes.c_int32), ("routed_scaling_factor", ctypes.c_float),
                ("has_shared", ctypes.c_int32), ("activation", ctypes.c_int32),
                ("situ_beta", ctypes.c_float), ("situ_linear_beta", ctypes.c_float),
                ("experts", ctypes.c_void_p), ("pool", ctypes.POINTER(K3ExpertPool))]


class K3DenseSeg(ctypes.Structure):
    _fields_ = [("w", ctypes.c_void_p), ("ldw", ctypes.c_int64), ("K", ctypes.c_int64),
                ("x", ctypes.c_void_p), ("x_dtype", ctypes.c_int32), ("ldx", ctypes.c_int64),
                ("norm_w", ctypes.c_void_p), ("eps", ctypes.c_float), ("act_input", ctypes.c_int32)]


class K3P2PGroup(ctypes.Structure):
    _fields_ = [("world", ctypes.c_int32), ("rank", ctypes.c_int32), ("gather_bytes", ctypes.c_int64),
                ("gather2_bytes", ctypes.c_int64), ("reduce_bytes", ctypes.c_int64),
                ("base", ctypes.c_void_p * 32)]


# name -> (restype, argtypes); mirrors include/k3b200.h
SIGNATURES = {
    "k3_abi_version": (_i32, []),
    "k3_last_error": (ctypes.c_char_p, []),
    "k3_device_sms": (_i32, []),
    "k3_profile_enable": (_i32, [_i32]),
    "k3_profile_collect": (_i32, [_vp, _vp, _i32]),
    "k3_mxfp4_dequant": (_i32, [_vp, _vp, _i64, _i64, _i32, _vp, _i32, _vp]),
    "k3_mxfp4_scale_minmax": (_i32, [_vp, _i64, _vp, _vp]),
    "k3_mxfp4_scales_tc": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "k3_mxfp4_tiles": (_i32, [_vp, _i64, _i64, _i64, _vp, _vp]),
    "k3_moe_pairs_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64, _i64]),
    "k3_moe_pairs_decode": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp, _i64, _vp,
                                   _i32, _vp, _sz, _vp]),
    "k3_mxfp4_matvec_workspace": (_sz, [_i64, _i64, _i64]),
    "k3_mxfp4_matvec": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp, _sz, _vp]),
    "k3_mxfp4_matvec_noalloc": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _vp, _i32, _vp]),
    "k3_moe_route_workspace": (_sz, [_i64, _i64]),
    "k3_moe_route": (_i32, [_vp, _i32, _i64, _i64, _vp, _vp, _i64, _i32, _i32, _f32, _vp, _vp,
                            _vp, _vp, _vp, _sz, _vp]),
    "k3_moe_decode_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64]),
    "k3_moe_decode": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp, _i32,
                             _vp, _vp, _vp, _sz, _vp]),
    "k3_moe_experts_decode": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp,
                                     _i32, _vp, _sz, _vp]),
    "k3_moe_expert_forward_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64]),
    "k3_moe_expert_forward": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _i64, _vp, _i32, _vp,
                                     _sz, _vp]),
    "k3_moe_prefill_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64]),
    "k3_moe_prefill": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp, _i32,
                              _vp, _vp, _vp, _sz, _vp]),
    "k3_moe_experts_prefill": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp,
                                      _i32, _vp, _sz, _vp]),
    "k3_moe_pairs_prefill_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64, _i64]),
    "k3_moe_pairs_prefill": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _vp, _i64,
                                    _vp, _i32, _vp, _sz, _vp]),
    "k3_moe_prefill_status": (_i32, [_vp, _vp]),
    "k3_moe_decode_latent_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64, _i64]),
    "k3_moe_decode_latent": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _i32, _i64, _vp, _vp, _vp,
                                    _i32, _vp, _vp, _vp, _vp, _sz, _vp]),
    "k3_dense_workspace": (_sz, [_i64, _i64, _i32, _i64, _i64]),
    "k3_dense_matvec": (_i32, [ctypes.POINTER(K3DenseSeg), _i32, _i64, _i64, _i32, _i32, _f32, _f32, _vp, _i32,
                               _i64, _vp, _sz, _vp]),
    "k3_lm_head_workspace": (_sz, [_i64, _i64]),
    "k3_dense_status": (_i32, [_vp, _vp]),
    "k3_attn_res_norm": (_i32, [_vp, _vp, _i64, _i64, _i64, _vp, _vp, _vp, _f32, _vp, _i32, _vp]),
    "k3_file_read_ranges": (_i32, [ctypes.c_char_p, _vp, _vp, _i32, _vp, _i32, _vp]),
    "k3_file_read_to_device": (_i32, [ctypes.c_char_p, _vp, _vp, _i32, _vp, _vp, _sz, _i32, _vp]),
    "k3_lm_head_argmax": (_i32, [_vp, _i32, _i64, _vp, _i64, _vp, _vp, _vp, _vp, _sz, _vp]),
    "k3_moe_ep_local_workspace": (_sz, [ctypes.POINTER(K3MoEParams), _i64, _i64]),
    "k3_wait_selftest": (_i32, [_i64, _i32, _vp, _vp]),
    "k3_dense_gemm_workspace": (_sz, [_i64, _i64]),
    "k3_dense_gemm": (_i32, [_vp, _i32, _i64, _i64, _i64, _vp, _i64, _i64, _vp, _i64, _i32, _vp, _sz, _vp]),
    "k3_moe_ep_local": (_i32, [ctypes.POINTER(K3MoEParams), _vp, _i32, _i64, _vp, _vp, _i64, _i32, _i32, _i32,
                               _vp, _i32, _vp, _sz, _vp]),
    "k3_p2p_buffer_bytes": (_sz, [_i32, _i64, _i64, _i64]),
    "k3_p2p_area_offsets": (_i32, [_i32, _i64, _i64, _i64, _vp]),
    "k3_p2p_export": (_i32, [_vp, _vp, _vp]),
    "k3_p2p_open": (_i32, [_vp, _i64, _vp]),
    "k3_p2p_close": (_i32, [_vp, _i64]),
    "k3_p2p_allgather": (_i32, [ctypes.POINTER(K3P2PGroup), _vp, _i64, _vp, _i64, _i32, _vp, _vp]),
    "k3_p2p_reduce_scatter": (_i32, [ctypes.POINTER(K3P2PGroup), _vp, _i64, _vp, _i32, _vp, _vp]),
    "k3_ep_a2a_plan": (_i32, [_vp, _i64, _i64, _i32, _i32, _i32, _i32, _vp, _vp, _vp, _vp, _vp, _vp]),
    "k3_ep_gather_rows": (_i32, [_vp, _i64, _i64, _vp, _i64, _vp, _vp, _vp]),
    "k3_ep_a2a_combine": (_i32, [_vp, _vp, _i32, _vp, _i64, _vp, _i64, _i32, _i64, _vp, _i32, _vp, _vp]),
}

_lib = None
_lock = threading.Lock()


def load_library(path: Path = LIB_PATH):
    """Load the shared library and bind every declared symbol (no GPU needed)."""
    global _lib
    if _lib is not None:                # every call of the layer comes here: no lock once loaded
        return _lib
    with _lock:
        if _lib is None:
            if not path.exists():
                raise ImportError(f"{path} is missing: build it with "
                                  "`python -m kimi_k3_mlx_macmini_b200.build` (needs nvcc)")
            lib = ctypes.CDLL(str(path))
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


class K3Error(RuntimeError):
    """A CUDA or workspace failure reported by the library."""


def last_error() -> str:
    """The calling thread's last library error message."""
    return (load_library().k3_last_error() or b"").decode(errors="replace")


def check(rc: int, what: str) -> None:
    if rc == K3_OK:
        return
    msg = (load_library().k3_last_error() or b"").decode(errors="replace")
    if rc == K3_ERR_INVALID:
        raise ValueError(f"{what}: {msg}")
    if rc == K3_ERR_UNSUPPORTED:
        raise NotImplementedError(f"{what}: {msg}")
    if rc == K3_ERR_IO:
        raise OSError(f"{what}: {msg}")
    raise K3Error(f"{what} failed ({rc}): {msg}")


def require_cuda(t: torch.Tensor, name: str) -> None:
    if not isinstance(t, torch.Tensor) or not t.is_cuda:
        raise ValueError(f"{name} must be a CUDA tensor (this path has no CPU fallback)")


def dtype_code(t: torch.Tensor) -> int:
    try:
        return _DTYPE[t.dtype]
    except KeyError:
        raise ValueError(f"unsupported dtype {t.dtype}") from None


def stream_of(t: torch.Tensor) -> int:
    return torch.cuda.current_stream(t.device).cuda_stream


_ws: dict = {}


def workspace(device: torch.device, nbytes: int, stream: int = None) -> torch.Tensor:
    """Per-(device, stream) scratch buffer, grown on demand (stream-ordered reuse);
    ``stream`` is the current stream's handle when the caller already has it."""
    key = (device.index, torch.cuda.current_stream(device).cuda_stream if stream is None else stream)
    buf = _ws.get(key)
    if buf is None or buf.numel() < nbytes:
        buf = torch.empty(max(int(nbytes), 256), dtype=torch.uint8, device=device)
        _ws[key] = buf
    return buf


def profile_enable(on: bool) -> None:
    load_library().k3_profile_enable(1 if on else 0)


def profile_collect() -> dict:
    """{kind: (total_ms, launches)} since the previous collect (waits for the events)."""
    n = len(PROF_KINDS)
    ms = (ctypes.c_double * n)()
    cnt = (ctypes.c_int64 * n)()
    check(load_library().k3_profile_collect(ms, cnt, n), "k3_profile_collect")
    return {k: (float(ms[i]), int(cnt[i])) for i, k in enumerate(PROF_KINDS)}
