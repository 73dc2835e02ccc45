"""The torch restatement of the oracle (`oracle/scunet_torch.py`) pinned on CPU: it
must reproduce the committed goldens (upstream torch outputs) and the numpy oracle
before the full-size GPU parity tests use it as their reference."""
import numpy as np
import pytest


@pytest.fixture(scope="module")
def toracle():
    import scunet_torch
    return scunet_torch


@pytest.mark.parametrize("stem", ["color_64x64", "color_80x64", "color_72x40", "gray_64x64", "color_128x128"])
def test_torch_oracle_matches_golden(stem, goldens, toracle, scb):
    g = goldens[stem]
    w = scb.weights.seeded(g["c"], 0)
    y = toracle.forward(g["x"], w).numpy()
    d = np.abs(y - g["y"]).max()
    assert d < 1e-5, f"{stem}: torch oracle vs upstream-torch golden {d:.3e}"


def test_torch_oracle_matches_numpy_oracle_batched(toracle, oracle, scb):
    """Two images in one call (the window/mask bookkeeping over a batch), a width that
    pads (100 -> 128) and both window kinds at every level."""
    x = np.stack([scb.synth.noisy_image(s, 3, 64, 100, 25 / 255) for s in (5, 6)]).astype(np.float32) / 255
    w = scb.weights.seeded(3, 0)
    want = oracle.forward(x, w)
    got = toracle.forward(x, w).numpy()
    d = np.abs(want - got).max()
    assert d < 1e-5, f"torch oracle vs numpy oracle {d:.3e}"
