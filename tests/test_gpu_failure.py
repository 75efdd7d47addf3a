"""Failure detection on the device, without a GPU fault.

Every pipelined kernel of the library waits on mbarriers with a time limit; a wait that
runs out writes K3_ERR_TIMEOUT into the call's status word and returns, so the kernel
ends and the context stays usable. ``k3_wait_selftest`` runs that same wait against a
barrier nothing arrives at (the failure made harmlessly, on purpose), and against one that
completes or is aborted. The reference's guards for the same situations are host-side
(``air_llm/models/kimi_k3/model.py:211-216``, ``loader.py:246-247``).
"""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _selftest(k3, limit_ns, mode):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    res = torch.full((3,), -1, dtype=torch.int32, device="cuda")
    L.check(L.load_library().k3_wait_selftest(limit_ns, mode, res.data_ptr(), L.stream_of(res)),
            "k3_wait_selftest")
    torch.cuda.synchronize()
    return res.tolist()


def test_wait_runs_out_and_reports_timeout(k3):
    status, ok, waited = _selftest(k3, 20_000_000, 0)          # 20 ms limit, nothing arrives
    from kimi_k3_mlx_macmini_b200 import _lib as L
    assert status == L.K3_ERR_TIMEOUT and ok == 0
    assert 20_000_000 <= waited < 2_000_000_000                 # gave up after its limit, not never


def test_wait_succeeds_when_the_barrier_completes(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    status, ok, _ = _selftest(k3, 1_000_000_000, 1)
    assert status == L.K3_OK and ok == 1


def test_wait_gives_up_on_abort_without_timeout(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    status, ok, waited = _selftest(k3, 1_000_000_000, 2)
    assert status == L.K3_OK and ok == 0 and waited < 1_000_000_000


def test_context_usable_after_a_timeout(k3):
    """After a wait ran out, the next library calls run and are correct."""
    import numpy as np
    from oracle import mxfp4_oracle as O
    from kimi_k3_mlx_macmini_b200 import _lib as L
    assert _selftest(k3, 5_000_000, 0)[0] == L.K3_ERR_TIMEOUT
    rng = np.random.default_rng(5)
    p, s = O.random_mxfp4(rng, 256, 512)
    x = rng.standard_normal((2, 512)).astype(np.float32)
    got = k3.mxfp4_matvec_fused(torch.from_numpy(x).cuda(), torch.from_numpy(p).cuda(),
                                torch.from_numpy(s).cuda()).cpu().numpy()
    assert O.rel_l2(got, O.matvec_fp64(x, p, s)) < 1e-5


def test_selftest_rejects_bad_arguments(k3):
    from kimi_k3_mlx_macmini_b200 import _lib as L
    lib = L.load_library()
    res = torch.zeros(3, dtype=torch.int32, device="cuda")
    assert lib.k3_wait_selftest(10, 0, res.data_ptr(), None) == L.K3_ERR_INVALID
    assert lib.k3_wait_selftest(10_000_000, 3, res.data_ptr(), None) == L.K3_ERR_INVALID
    assert lib.k3_wait_selftest(10_000_000, 0, None, None) == L.K3_ERR_INVALID
