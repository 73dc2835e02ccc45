"""The full-resolution transformer half on the independent-lane kernel
(`trans32_mp_kernel`, SCB_OPT_TRANS32_LANES = 1) against the oracle: single
ConvTransBlocks of the two full-resolution stages (down1, up1) at W and SW, odd
window counts (a pair with one window), several images and the cyclic-shift mask at
the image edges (tests/cuda_ops.rs:130-158), and the whole network against the
golden fixtures."""
import numpy as np
import pytest

from test_kernels_gpu import STAGES, close
from test_forward_gpu import check_parity

pytestmark = pytest.mark.gpu


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


@pytest.mark.parametrize("stage,index,n,H,W", [
    (0, 0, 1, 16, 16), (0, 1, 2, 16, 24), (0, 1, 1, 8, 24), (6, 3, 1, 24, 16), (6, 2, 3, 8, 8), (0, 1, 1, 72, 64),
    (0, 3, 1, 136, 200),
])
def test_block_lanes(be3, weights3, oracle, scb, stage, index, n, H, W):
    torch = _torch()
    c = 64
    rng = np.random.default_rng(stage * 10 + index + H)
    x = (rng.standard_normal((n, H, W, c)) * 0.5).astype(np.float32)
    first = 1 if stage >= 4 else 0
    prefix = f"m_{STAGES[stage]}.{first + index}"
    want = np.stack([oracle.conv_trans_block(x[i], weights3.tensors, prefix, index % 2 == 1) for i in range(n)])
    tx = torch.from_numpy(x).cuda()
    ty = torch.empty_like(tx)
    be3.set_option(scb.backend.SCB_OPT_TRANS32_LANES, 1)
    try:
        rc = be3.lib.scb_probe_block(be3.ctx, stage, index, tx.data_ptr(), n, H, W, ty.data_ptr())
    finally:
        be3.set_option(scb.backend.SCB_OPT_TRANS32_LANES, 0)
    assert rc == 0, be3.lib.scb_last_error(be3.ctx)
    r = close(f"lanes block {prefix} {n}x{H}x{W}", want, ty.cpu().numpy(), 1e-3)
    print(f"lanes block {prefix} {n}x{H}x{W}: rel err {r:.2e}")


@pytest.mark.parametrize("stem", ["color_64x64", "color_80x64", "color_72x40", "gray_64x64", "color_128x128"])
def test_forward_lanes_matches_golden(stem, goldens, oracle, scb, be1, be3):
    _torch()
    g = goldens[stem]
    be = be3 if g["c"] == 3 else be1
    be.set_option(scb.backend.SCB_OPT_TRANS32_LANES, 1)
    try:
        got = scb.run(be, g["x"][0], g["c"], g["h"], g["w"], be.weights)
        again = scb.run(be, g["x"][0], g["c"], g["h"], g["w"], be.weights)
    finally:
        be.set_option(scb.backend.SCB_OPT_TRANS32_LANES, 0)
    assert np.array_equal(got, again), "repeats differ"
    check_parity(oracle, f"lanes {stem}", g["y"][0], got)
