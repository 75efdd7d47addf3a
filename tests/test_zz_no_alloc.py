"""k3_mxfp4_matvec_noalloc -- the fused MXFP4 matvec for callers that cannot allocate.

Some hosts of this path can hand it only their own input and output buffers: an FFI
binding of the three-argument ``mxfp4_matvec_fused`` inside a runtime whose device
memory belongs to another allocator cannot call cudaMalloc (the memory would go behind
that allocator's back or not exist, and cudaMalloc/cudaFree synchronise the device).
The no-alloc entry point serves them from one 4 MiB device array built into the
library. These GPU tests call it through the C ABI and check it against the workspace
entry point ``k3_mxfp4_matvec``, on two calls in a row, and check that a shape needing
more scratch than the array is refused with a clear error.

The file is named to be collected last, so a run that stops at the first failure has
already run every other test; it also passes alone in a fresh process.
"""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

REL_L2_TOL = 1e-5          # the fp32-output tolerance of the parity tests


@pytest.fixture(scope="module")
def lib():
    if not torch.cuda.is_available():
        pytest.fail("GPU tests need a CUDA device")
    from kimi_k3_mlx_macmini_b200 import build
    build.build()
    from kimi_k3_mlx_macmini_b200 import _lib as L
    return L


def _inputs(gen, M, K, N, xdt):
    x = torch.randn((M, K), generator=gen, device="cuda", dtype=torch.float32).to(xdt)
    packed = torch.randint(0, 256, (N, K // 2), generator=gen, device="cuda", dtype=torch.uint8)
    scales = torch.randint(120, 131, (N, K // 32), generator=gen, device="cuda", dtype=torch.uint8)
    return x, packed, scales


def _with_workspace(L, x, packed, scales, N):
    lib = L.load_library()
    M, K = x.shape
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    ws = torch.empty(lib.k3_mxfp4_matvec_workspace(M, K, N), dtype=torch.uint8, device="cuda")
    L.check(lib.k3_mxfp4_matvec(x.data_ptr(), L.dtype_code(x), M, K, packed.data_ptr(),
                                scales.data_ptr(), N, out.data_ptr(), L.K3_F32, ws.data_ptr(),
                                ws.numel(), L.stream_of(x)), "k3_mxfp4_matvec")
    return out


def _no_alloc(L, x, packed, scales, N):
    lib = L.load_library()
    M, K = x.shape
    out = torch.empty((M, N), dtype=torch.float32, device="cuda")
    L.check(lib.k3_mxfp4_matvec_noalloc(x.data_ptr(), L.dtype_code(x), M, K, packed.data_ptr(),
                                        scales.data_ptr(), N, out.data_ptr(), L.K3_F32,
                                        L.stream_of(x)), "k3_mxfp4_matvec_noalloc")
    return out


@pytest.mark.parametrize("M,K,N,xdt", [
    (8, 7168, 2048, torch.bfloat16),     # BASELINE gate/up projection, decode batch
    (3, 2048, 7168, torch.float32),      # BASELINE down projection, fp32 activations
    (11, 256, 128, torch.float32),       # more than 8 tokens: chunked launches
])
def test_no_alloc_matches_workspace_entry_point(lib, M, K, N, xdt):
    gen = torch.Generator(device="cuda")
    gen.manual_seed(M * 7919 + K + N)
    for call in range(2):                                # two calls in a row, fresh inputs
        x, packed, scales = _inputs(gen, M, K, N, xdt)
        want = _with_workspace(lib, x, packed, scales, N)
        got = _no_alloc(lib, x, packed, scales, N)
        torch.cuda.synchronize()
        rel = float(torch.linalg.vector_norm((got - want).double()) /
                    torch.linalg.vector_norm(want.double()))
        assert rel < REL_L2_TOL, f"call {call}: rel-L2 {rel:.3e}"


def test_no_alloc_refuses_shapes_beyond_its_scratch(lib):
    L = lib.load_library()
    M, K = 8, 7168
    N = next(n for n in (2048, 7168, 14336, 28672, 57344, 114688)
             if L.k3_mxfp4_matvec_workspace(M, K, n) > 4 << 20)
    tiny = torch.zeros(64, dtype=torch.uint8, device="cuda")   # never read: refused first
    rc = L.k3_mxfp4_matvec_noalloc(tiny.data_ptr(), lib.K3_F32, M, K, tiny.data_ptr(),
                                   tiny.data_ptr(), N, tiny.data_ptr(), lib.K3_F32,
                                   lib.stream_of(tiny))
    assert rc == lib.K3_ERR_INVALID
    assert b"no-alloc limit" in L.k3_last_error()
