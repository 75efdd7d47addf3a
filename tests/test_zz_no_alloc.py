"""k3_mxfp4_matvec_noalloc -- the fused MXFP4 matvec for callers that cannot allocate.

Some hosts of this path can hand it only their own input and output buffers: an FFI
binding of the three-argument ``mxfp4_matvec_fused`` inside a runtime whose device
memory belongs to another allocator cannot call cudaMalloc (the memory would go behind
that allocator's back or not exist, and cudaMalloc/cudaFree synchronise the device).
The no-alloc entry point serves them from one 4 MiB device array built into the
library. These GPU tests call it through the C ABI and check it against the workspace
entry point ``k3_mxfp4_matvec`` bit for bit, on two calls in a row and on consecutive
calls of different shapes, against the CPU oracle at the BASELINE gate/up shape, and that
a shape needing more scratch than the array is refused with a clear error.

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


def _with_workspace(L, x, packed, scales, N, odt=torch.float32):
    lib = L.load_library()
    M, K = x.shape
    out = torch.empty((M, N), dtype=odt, device="cuda")
    ws = torch.empty(lib.k3_mxfp4_matvec_workspace(M, K, N), dtype=torch.uint8, device="cuda")
    L.check(lib.k3_mxfp4_matvec(x.data_ptr(), L.dtype_code(x), M, K, packed.data_ptr(),
                                scales.data_ptr(), N, out.data_ptr(), L.dtype_code(out), ws.data_ptr(),
                                ws.numel(), L.stream_of(x)), "k3_mxfp4_matvec")
    return out


def _no_alloc(L, x, packed, scales, N, odt=torch.float32):
    lib = L.load_library()
    M, K = x.shape
    out = torch.empty((M, N), dtype=odt, device="cuda")
    L.check(lib.k3_mxfp4_matvec_noalloc(x.data_ptr(), L.dtype_code(x), M, K, packed.data_ptr(),
                                        scales.data_ptr(), N, out.data_ptr(), L.dtype_code(out),
                                        L.stream_of(x)), "k3_mxfp4_matvec_noalloc")
    return out


def _rel(got, want):
    return float(torch.linalg.vector_norm((got.double() - want.double())) / torch.linalg.vector_norm(want.double()))


@pytest.mark.parametrize("M,K,N,xdt,odt", [
    (8, 7168, 2048, torch.bfloat16, torch.float32),    # BASELINE gate/up projection, decode batch
    (1, 7168, 2048, torch.bfloat16, torch.bfloat16),   # one token, bf16 result
    (3, 2048, 7168, torch.float32, torch.float32),     # BASELINE down projection, fp32 activations
    (11, 256, 128, torch.float32, torch.float32),      # more than 8 tokens: chunked launches
])
def test_no_alloc_matches_workspace_entry_point(lib, M, K, N, xdt, odt):
    """Both entry points run the same kernels, whose split-k partial sums are added in a
    fixed order, so the results are identical bit for bit -- a leftover of an earlier
    call's scratch would show as a difference."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(M * 7919 + K + N)
    for call in range(2):                                # two calls in a row, fresh inputs
        x, packed, scales = _inputs(gen, M, K, N, xdt)
        want = _with_workspace(lib, x, packed, scales, N, odt)
        got = _no_alloc(lib, x, packed, scales, N, odt)
        torch.cuda.synchronize()
        assert _rel(got, want) < REL_L2_TOL, f"call {call}"
        assert torch.equal(got, want), f"call {call}: not bitwise equal"


def test_no_alloc_consecutive_calls_on_different_shapes(lib):
    """Calls that leave different plans, counters and partial sums in the shared scratch
    (a tall down-projection shape, then the gate/up shape, then a small one) each match
    the workspace entry point bit for bit."""
    gen = torch.Generator(device="cuda")
    gen.manual_seed(99)
    for M, K, N, xdt in [(8, 2048, 7168, torch.float32), (5, 7168, 2048, torch.bfloat16),
                         (2, 512, 256, torch.bfloat16), (8, 7168, 2048, torch.float32)]:
        x, packed, scales = _inputs(gen, M, K, N, xdt)
        got = _no_alloc(lib, x, packed, scales, N)
        want = _with_workspace(lib, x, packed, scales, N)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (M, K, N)


def test_no_alloc_matches_oracle_at_baseline_shape(lib):
    """The BASELINE gate/up projection (7168 -> 2048) at M = 8 against the C restatement
    of the reference's fused-kernel loop (``mxfp4_matvec.py:29-63``) and fp64."""
    from oracle import mxfp4_oracle as O
    rng = np.random.default_rng(2048)
    p, s = O.random_mxfp4(rng, 2048, 7168)
    xb = O.f32_to_bf16_bits(rng.standard_normal((8, 7168)).astype(np.float32))
    xf = O.bf16_bits_to_f32(xb)
    x = torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16)
    got = _no_alloc(lib, x, torch.from_numpy(p).cuda(), torch.from_numpy(s).cuda(), 2048).cpu().numpy()
    assert O.rel_l2(got, O.matvec_fused(xf, p, s)) < REL_L2_TOL
    assert O.rel_l2(got, O.matvec_fp64(xf, p, s)) < REL_L2_TOL


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
