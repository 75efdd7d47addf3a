"""One process driving two GPUs: every kernel that needs more than 48 KB of dynamic shared
memory gets its attribute set in each device's context, not once per process. Plain local
launches on each device (no peer memory). Runs when the box has 2 GPUs or more."""
import numpy as np
import pytest
import torch

from oracle import mxfp4_oracle as O

pytestmark = pytest.mark.gpu


def _two_devices():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")


def test_matvec_and_decode_on_two_devices_in_one_process(k3):
    _two_devices()
    from kimi_k3_mlx_macmini_b200 import _lib as L
    from kimi_k3_mlx_macmini_b200 import synthetic
    lib = L.load_library()
    rng = np.random.default_rng(12)
    p, s = O.random_mxfp4(rng, 2048, 7168)
    x = rng.standard_normal((8, 7168)).astype(np.float32)
    want = O.matvec_fp64(x, p, s)
    for dev in (0, 1, 0, 1):                      # alternate: each context set up once, reused
        with torch.cuda.device(dev):
            xd, pd, sd = (torch.from_numpy(a).to(f"cuda:{dev}") for a in (x, p, s))
            y = k3.mxfp4_matvec_fused(xd, pd, sd)
            out = torch.empty((8, 2048), dtype=torch.float32, device=f"cuda:{dev}")
            L.check(lib.k3_mxfp4_matvec_noalloc(xd.data_ptr(), L.K3_F32, 8, 7168, pd.data_ptr(), sd.data_ptr(),
                                                2048, out.data_ptr(), L.K3_F32, L.stream_of(xd)),
                    "k3_mxfp4_matvec_noalloc")
            torch.cuda.synchronize(dev)
            assert O.rel_l2(y.cpu().numpy(), want) < 1e-5
            assert torch.equal(out, y)
    # the block-scaled decode kernels (largest shared-memory rings) on each device
    outs = []
    for dev in (0, 1):
        with torch.cuda.device(dev):
            lay = synthetic.baseline_layer(seed=17, E=16, H=1024, I=512, top_k=4, device=f"cuda:{dev}")
            moe = lay.moe(device=f"cuda:{dev}")
            xt = synthetic.tokens(5, 8, 1024, device=f"cuda:{dev}")
            outs.append(moe(xt).cpu())
            del moe, lay
    assert torch.equal(outs[0], outs[1])
