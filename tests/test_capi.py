"""The C-ABI library loads and exports every symbol ``include/k3b200.h`` declares, and
argument validation answers before any CUDA call (no GPU needed)."""
import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def header_symbols():
    text = (ROOT / "include" / "k3b200.h").read_text()
    return sorted(set(re.findall(r"K3_API\s+[\w\s\*]+?\b(k3_\w+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from kimi_k3_mlx_macmini_b200 import build
    build.build()
    from kimi_k3_mlx_macmini_b200 import _lib as L
    return L.load_library()


def test_header_declares_entry_points():
    syms = header_symbols()
    assert "k3_mxfp4_matvec" in syms and "k3_moe_decode" in syms and len(syms) >= 12


def test_library_exports_every_declared_symbol(lib):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    for name in header_symbols():
        assert hasattr(lib, name), f"{name} not exported"
        assert name in L.SIGNATURES, f"{name} has no ctypes signature"


def test_version_and_error_string(lib):
    assert lib.k3_abi_version() == 3
    assert isinstance(lib.k3_last_error(), bytes)


def test_null_and_shape_errors_before_cuda(lib):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    rc = lib.k3_mxfp4_matvec(None, L.K3_F32, 1, 64, None, None, 4, None, L.K3_F32, None, 0, None)
    assert rc == L.K3_ERR_INVALID and b"NULL" in lib.k3_last_error()
    # non-NULL placeholders are never dereferenced: validation fails first
    fake = ctypes.c_void_p(16)
    assert lib.k3_mxfp4_matvec(fake, L.K3_F32, 1, 48, fake, fake, 4, fake, L.K3_F32, None, 0,
                               None) == L.K3_ERR_INVALID
    assert b"multiple of 32" in lib.k3_last_error()
    assert lib.k3_mxfp4_matvec(fake, 7, 1, 64, fake, fake, 4, fake, L.K3_F32, None, 0, None) == L.K3_ERR_INVALID
    assert lib.k3_mxfp4_dequant(fake, fake, 4, 64, 16, fake, L.K3_F32, None) == L.K3_ERR_UNSUPPORTED
    assert lib.k3_moe_route(fake, L.K3_F32, 1, 64, fake, None, 2000, 8, 1, 1.0, fake, fake, None,
                            None, None, 0, None) == L.K3_ERR_UNSUPPORTED


def test_moe_params_validation(lib):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    p = L.K3MoEParams(hidden=7168, inter=2048, num_experts=384, top_k=8, renormalize=1,
                      routed_scaling_factor=2.5, has_shared=1, activation=L.K3_ACT_SILU,
                      situ_beta=4.0, situ_linear_beta=25.0, experts=None)
    assert lib.k3_moe_decode_workspace(p, 1) == 0          # NULL table rejected
    p.experts = 16
    assert lib.k3_moe_decode_workspace(p, 9) == 0          # decode takes <= 8 tokens
    p.hidden = 7000
    assert lib.k3_moe_decode_workspace(p, 1) == 0          # hidden % 128
    assert b"hidden" in lib.k3_last_error()


def test_python_layer_refuses_cpu_tensors():
    import numpy as np
    import torch
    from kimi_k3_mlx_macmini_b200 import mxfp4_matvec_fused
    with pytest.raises(ValueError, match="CUDA"):
        mxfp4_matvec_fused(torch.zeros(1, 64), torch.zeros(4, 32, dtype=torch.uint8),
                           torch.zeros(4, 2, dtype=torch.uint8))


def test_exchange_layouts_and_validation(lib):
    """The expert-parallel exchange entry points: the peer-memory buffer layout (a 1 KB
    header, then world slots per area, each slot 16-byte aligned) and argument checks that
    answer before any CUDA call."""
    import ctypes as C
    from kimi_k3_mlx_macmini_b200 import _lib as L
    for W, g0, g1, rb in ((2, 114688, 512, 229376), (8, 229376, 1024, 229376), (3, 100, 36, 20)):
        offs = (C.c_int64 * 4)()
        assert lib.k3_p2p_area_offsets(W, g0, g1, rb, offs) == 0
        r16 = lambda v: (v + 15) // 16 * 16  # noqa: E731
        assert list(offs) == [1024, 1024 + W * r16(g0), 1024 + W * (r16(g0) + r16(g1)),
                              1024 + W * (r16(g0) + r16(g1) + r16(rb))]
        assert lib.k3_p2p_buffer_bytes(W, g0, g1, rb) == offs[3]
    assert lib.k3_p2p_buffer_bytes(0, 16, 16, 16) == 0 and lib.k3_p2p_buffer_bytes(33, 16, 16, 16) == 0
    g = L.K3P2PGroup(world=2, rank=2, gather_bytes=64, gather2_bytes=64, reduce_bytes=64,
                     base=(C.c_void_p * 32)(256, 512))
    fake = C.c_void_p(256)
    assert lib.k3_p2p_allgather(C.byref(g), fake, 16, fake, 16, 3, fake, None) == L.K3_ERR_INVALID   # rank >= world
    g.rank = 0
    assert lib.k3_p2p_allgather(C.byref(g), fake, 80, fake, 16, 3, fake, None) == L.K3_ERR_INVALID   # > capacity
    assert lib.k3_p2p_allgather(C.byref(g), fake, 24, fake, 16, 3, fake, None) == L.K3_ERR_INVALID   # not 16-multiple
    assert lib.k3_p2p_reduce_scatter(C.byref(g), fake, 6, fake, 3, fake, None) == L.K3_ERR_INVALID   # n % 4
    assert lib.k3_ep_a2a_plan(fake, 8, 4, 8, 48, 33, 0, fake, fake, fake, fake, fake, None) == L.K3_ERR_UNSUPPORTED
    assert lib.k3_ep_a2a_plan(fake, 4, 4, 8, 48, 8, 0, fake, fake, fake, fake, fake, None) == L.K3_ERR_INVALID
    assert lib.k3_ep_gather_rows(fake, 4, 6, fake, 4, fake, fake, None) == L.K3_ERR_INVALID          # row bytes % 4
    assert lib.k3_ep_a2a_combine(None, None, 0, fake, 4, fake, 4, 2, 6, fake, L.K3_F32, fake, None) == L.K3_ERR_INVALID
