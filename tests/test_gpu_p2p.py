"""Exchanges over peer memory (``k3_p2p_allgather`` / ``k3_p2p_reduce_scatter``).

On one GPU the ranks are emulated with one buffer each: every rank's put phase (mode 1)
runs first, then every rank's wait phase (mode 2), so no launch waits on another one.
Results are bit-exact: the gathers copy bytes, the reduce-scatter adds the ranks' chunks
in rank order, as the reference sum below does. A wait on a flag that no rank sets gives
up after its bound and reports K3_ERR_TIMEOUT. The same kernels between processes on 2
GPUs run inside ``ExpertParallelMoE(exchange="p2p")`` in ``tests/test_gpu_ep.py``."""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu


def _groups(W, caps):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    nbytes = int(lib.k3_p2p_buffer_bytes(W, *caps))
    offs = (ctypes.c_int64 * 4)()
    L.check(lib.k3_p2p_area_offsets(W, *caps, offs), "k3_p2p_area_offsets")
    bufs = [torch.zeros(nbytes + 256, dtype=torch.uint8, device="cuda") for _ in range(W)]
    views = [b[(-b.data_ptr()) % 256:][:nbytes] for b in bufs]
    bases = [v.data_ptr() for v in views]
    descs = [L.K3P2PGroup(world=W, rank=r, gather_bytes=caps[0], gather2_bytes=caps[1], reduce_bytes=caps[2],
                          base=(ctypes.c_void_p * 32)(*bases)) for r in range(W)]
    torch.cuda.synchronize()
    return views, list(offs), descs


@pytest.mark.parametrize("W", [2, 3, 8])
def test_p2p_allgather_and_reduce_scatter_emulated(k3, W):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    M, H, k = 8, 7168, 8
    caps = (M * H * 4, M * 2 * k * 4, M * H * 4)
    views, offs, descs = _groups(W, caps)
    st = torch.zeros((W, 2), dtype=torch.int32, device="cuda")
    g = torch.Generator(device="cuda").manual_seed(W)
    for step in range(3):                                  # epochs advance without a reset
        Ms = M - step                                      # a different size per step
        xs = [torch.randn((Ms, H), device="cuda", generator=g).to(torch.bfloat16) for _ in range(W)]
        rs = [torch.randint(-2**31, 2**31 - 1, (Ms, 2 * k), dtype=torch.int32, device="cuda", generator=g)
              for _ in range(W)]
        parts = [torch.randn((W * Ms, H), device="cuda", generator=g) for _ in range(W)]
        outs = [torch.empty((Ms, H), device="cuda") for _ in range(W)]
        for mode in (1, 2):
            for r in range(W):
                L.check(lib.k3_p2p_allgather(ctypes.byref(descs[r]), xs[r].data_ptr(), xs[r].numel() * 2,
                                             rs[r].data_ptr(), rs[r].numel() * 4, mode, st[r].data_ptr(),
                                             L.stream_of(xs[r])), "k3_p2p_allgather")
        for mode in (1, 2):
            for r in range(W):
                L.check(lib.k3_p2p_reduce_scatter(ctypes.byref(descs[r]), parts[r].data_ptr(), Ms * H,
                                                  outs[r].data_ptr(), mode, st[r, 1:].data_ptr(),
                                                  L.stream_of(parts[r])), "k3_p2p_reduce_scatter")
        torch.cuda.synchronize()
        assert not st.any(), st
        want_x = torch.cat(xs).view(torch.uint8).reshape(-1)
        want_r = torch.cat(rs).view(torch.uint8).reshape(-1)
        for r in range(W):
            got_x = views[r][offs[0]:offs[0] + want_x.numel()]
            got_r = views[r][offs[1]:offs[1] + want_r.numel()]
            assert torch.equal(got_x, want_x), (step, r)
            assert torch.equal(got_r, want_r), (step, r)
            ref = torch.zeros((Ms, H), device="cuda")
            for s in range(W):
                ref += parts[s][r * Ms:(r + 1) * Ms]
            assert torch.equal(outs[r], ref), (step, r)


def test_p2p_wait_gives_up(k3):
    """Rank 0 of a 2-rank group publishes and waits; rank 1 never puts: the wait ends at
    its bound with K3_ERR_TIMEOUT, and the kernel returns (its own slot is written)."""
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    H = 1024
    caps = (H * 2, 64, H * 4)
    views, offs, descs = _groups(2, caps)
    st = torch.zeros(2, dtype=torch.int32, device="cuda")
    x = torch.randn((1, H), device="cuda").to(torch.bfloat16)
    r = torch.zeros((1, 16), dtype=torch.int32, device="cuda")
    L.check(lib.k3_p2p_allgather(ctypes.byref(descs[0]), x.data_ptr(), H * 2, r.data_ptr(), 64, 3, st.data_ptr(),
                                 L.stream_of(x)), "k3_p2p_allgather")
    torch.cuda.synchronize()
    assert st[0].item() == 5                                  # K3_ERR_TIMEOUT
    assert torch.equal(views[0][offs[0]:offs[0] + H * 2], x.view(torch.uint8).reshape(-1))
    # and the reduce-scatter's wait likewise
    part = torch.randn((2, H), device="cuda")
    out = torch.empty(H, device="cuda")
    L.check(lib.k3_p2p_reduce_scatter(ctypes.byref(descs[0]), part.data_ptr(), H, out.data_ptr(), 3,
                                      st[1:].data_ptr(), L.stream_of(part)), "k3_p2p_reduce_scatter")
    torch.cuda.synchronize()
    assert st[1].item() == 5


def test_p2p_export_and_open_reject_bad_arguments(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    h = (ctypes.c_uint8 * 64)()
    o = ctypes.c_int64()
    assert lib.k3_p2p_export(None, h, ctypes.byref(o)) == 1
    p = ctypes.c_void_p()
    assert lib.k3_p2p_open(None, 0, ctypes.byref(p)) == 1
    desc = L.K3P2PGroup(world=2, rank=0, gather_bytes=64, gather2_bytes=64, reduce_bytes=64,
                        base=(ctypes.c_void_p * 32)())
    st = torch.zeros(1, dtype=torch.int32, device="cuda")
    assert lib.k3_p2p_allgather(ctypes.byref(desc), None, 0, None, 0, 3, st.data_ptr(), None) == 1   # NULL bases
