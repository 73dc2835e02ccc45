"""The oracle against the committed goldens, and the reference's own known-answer
tests for the attention semantics, restated on the oracle (CPU only)."""
import json

import numpy as np
import pytest

from conftest import GOLDEN


def test_weights_generator_matches_manifest(scb):
    import hashlib
    man = json.loads((GOLDEN / "manifest.json").read_text())
    for in_nc in (1, 3):
        w = scb.weights.seeded(in_nc, man["weights_seed"])
        h = hashlib.sha256()
        for k in sorted(w):
            h.update(k.encode())
            h.update(np.ascontiguousarray(w[k], "<f4").tobytes())
        assert h.hexdigest() == man["weights"][str(in_nc)]["sha256"], "seeded weights drifted"


@pytest.mark.parametrize("stem", ["color_64x64", "color_80x64", "color_72x40", "gray_64x64", "color_128x128"])
def test_oracle_matches_golden(stem, goldens, oracle, scb):
    g = goldens[stem]
    w = scb.weights.seeded(g["c"], 0)
    y = oracle.forward(g["x"], w)
    d = np.abs(y - g["y"]).max()
    assert d < 1e-5, f"{stem}: oracle vs upstream-torch golden {d:.3e}"


def test_golden_manifest_records_reference_agreement():
    man = json.loads((GOLDEN / "manifest.json").read_text())
    for stem, c in man["cases"].items():
        assert c["max_abs_reference_py_vs_torch"] < 1e-5, stem
        assert c["max_abs_oracle_vs_reference_py"] < 1e-5, stem


def test_attention_uniform_softmax(oracle):
    """k = 0 -> uniform softmax -> each output is the mean of v over its window
    (tests/cuda_ops.rs:365-403)."""
    nw, t = 4, 32
    qkv = np.zeros((nw, 64, 3 * t), np.float32)
    qkv[..., :t] = 1.0
    tok = np.arange(nw * 64).reshape(nw, 64)
    qkv[..., 2 * t] = (tok % 17).astype(np.float32)
    qkv[..., 2 * t + 1:] = 2.0
    o = oracle.attention_core(qkv, np.zeros((1, 15, 15), np.float32), 2, 2, False)
    want0 = (tok % 17).mean(axis=1)
    assert np.allclose(o[..., 0], want0[:, None], atol=1e-5)
    assert np.allclose(o[..., 1:], 2.0, atol=1e-5)


def test_attention_known_softmax(oracle):
    """q = e0, k_t = e_(t mod 32): logit = 1 iff t % 32 == 0 (tests/cuda_ops.rs:409-450)."""
    t = 32
    qkv = np.zeros((1, 64, 3 * t), np.float32)
    for k in range(64):
        qkv[0, k, 0] = 1.0
        qkv[0, k, t + (k % t)] = 1.0
        qkv[0, k, 2 * t] = 3.0
        qkv[0, k, 2 * t + 1] = 1.0
    o = oracle.attention_core(qkv, np.zeros((1, 15, 15), np.float32), 1, 1, False)
    e = np.where(np.arange(64) % t == 0, np.exp(t ** -0.5), 1.0)
    p = e / e.sum()
    assert np.allclose(o[0, :, 0], 3.0 * p.sum(), atol=1e-5)
    assert np.allclose(o[0, :, 1], p.sum(), atol=1e-5)


@pytest.mark.parametrize("h,w,shift", [(8, 8, 0), (16, 16, 4), (32, 24, 4), (24, 32, 0)])
def test_window_index_map(oracle, h, w, shift):
    """Gather/scatter is a permutation and matches the reference pix map
    ((wh*8+i+shift) % h, (ww*8+j+shift) % w) (tests/cuda_ops.rs:322-359)."""
    c = 3
    x = np.random.default_rng(0).standard_normal((h, w, c)).astype(np.float32)
    tok = oracle.window_tokens(x, shift)
    nww = w // 8
    for wi in range(tok.shape[0]):
        wh, ww = divmod(wi, nww)
        for t in range(64):
            i, j = divmod(t, 8)
            assert np.array_equal(tok[wi, t], x[(wh * 8 + i + shift) % h, (ww * 8 + j + shift) % w])
    assert np.array_equal(oracle.window_untokens(tok, h, w, shift), x)


def test_mask_never_masks_a_whole_row(oracle):
    """The SW mask compares the same axis on both sides of each edge and always
    leaves the diagonal, so no softmax row is empty (cuda/scunet.cu:11-15, 119-147)."""
    m = oracle.sw_mask(3, 3)
    assert not m[:, np.arange(64), np.arange(64)].any()
    assert m[0].sum() == 0                     # interior window
    assert m[8].sum() == 2 * 64 * 32 - 32 * 32  # corner: row and column edges


def test_plan_geometry(scb):
    """`tests/parity.rs:130-141`: padded geometry and the min-size refusal."""
    P = scb.Plan
    assert (P.new(80, 64).hp, P.new(80, 64).wp) == (128, 64)
    assert (P.new(1080, 1920).hp, P.new(1080, 1920).wp) == (1088, 1920)
    assert P.new(64, 64).windows(3) == (1, 1)
    scb.plan.check_min_size(1, 1)
    with pytest.raises(ValueError):
        scb.plan.check_min_size(0, 64)
    x = np.arange(2 * 3 * 5, dtype=np.float32).reshape(2, 3, 5)
    p = scb.plan.pad_replicate(x, 2, 3, 5, 64, 64)
    assert p.shape == (2, 64, 64) and p[1, 63, 63] == x[1, 2, 4] and p[0, 10, 2] == x[0, 2, 2]
    assert np.array_equal(scb.plan.crop(p, 2, 3, 5, 64, 64), x)


def test_flop_count(scb):
    assert scb.weights.flops_per_pixel(3) == 2403072
    assert scb.weights.flops_per_pixel(1) == 2398464


def test_safetensors_round_trip(scb, tmp_path):
    w = scb.Weights.seeded(1, 3)
    p = tmp_path / "m.safetensors"
    w.save(p)
    w2 = scb.Weights.load(p)
    assert w2.in_nc == 1 and w2.config == (4,) * 7
    for k in w.tensors:
        assert np.array_equal(w.tensors[k], w2.tensors[k])


def test_weights_validation(scb):
    t = dict(scb.weights.seeded(3, 0))
    t["m_body.2.conv1_1.weight"] = np.zeros((512, 512, 1, 2), np.float32)
    with pytest.raises(ValueError, match="m_body.2.conv1_1.weight"):
        scb.Weights(t)
    del t["m_body.2.conv1_1.weight"]
    with pytest.raises(ValueError, match="missing"):
        scb.Weights(t)
