"""A checkpoint loaded from a file runs on the GPU: seeded weights written as the
reference's converter writes them (`tools/convert.py:227-236` metadata; the byte
identity is checked on CPU in test_checkpoint.py), read back through
`Weights.load` (`src/weights.rs:101-280`: metadata, arch, names, shapes), uploaded
by scb_create and run. The output must be bit-identical to the same weights
uploaded from memory, and match the golden fixture at the acceptance bar."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_loaded_checkpoint_forward(scb, oracle, goldens, weights3, be3, tmp_path):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    p = tmp_path / "scunet-color-seeded.safetensors"
    weights3.save(p)
    loaded = scb.Weights.load(p)
    g = goldens["color_80x64"]
    be = scb.B200(loaded)
    try:
        got = be.forward_host(g["x"])
    finally:
        be.close()
    mem = be3.forward_host(g["x"])
    assert np.array_equal(got, mem), "loaded weights give a different output than the same weights in memory"
    r = oracle.parity_report(g["y"], got)
    print(f"loaded checkpoint vs golden color_80x64: {r}")
    assert r["max_abs"] <= 2e-3 and r["frac_level_gt1"] == 0
