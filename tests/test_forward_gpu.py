"""End to end on the device: the golden fixtures (upstream torch FP32 on seeded
weights), batched vs single, and bit-identical repeats (the reference's race
detector, tests/cuda_ops.rs:217-251)."""
import re

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3       # north-star bar on the [0,1] output before quantisation
LEVEL_FRAC = 0.999   # >= 99.9 % of values within 1 8-bit level


def _gpu():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def check_parity(oracle, what, want, got):
    rep = oracle.parity_report(want, got)
    print(f"{what}: {rep}")
    assert rep["max_abs"] <= MAX_ABS, f"{what}: {rep}"
    assert 1.0 - rep["frac_level_gt1"] >= LEVEL_FRAC, f"{what}: {rep}"
    return rep


@pytest.mark.parametrize("stem", ["color_64x64", "color_80x64", "color_72x40", "gray_64x64", "color_128x128"])
def test_forward_matches_golden(stem, goldens, oracle, scb, be1, be3):
    _gpu()
    g = goldens[stem]
    be = be3 if g["c"] == 3 else be1
    wt = be.weights
    got = scb.run(be, g["x"][0], g["c"], g["h"], g["w"], wt)
    check_parity(oracle, stem, g["y"][0], got)


def test_forward_unfused_transformer_matches_golden(goldens, oracle, scb, be3):
    """The separate-launch transformer path (SCB_OPT_FUSE_TRANS = 0) end to end."""
    _gpu()
    g = goldens["color_80x64"]
    be3.set_option(scb.backend.SCB_OPT_FUSE_TRANS, 0)
    try:
        got = scb.run(be3, g["x"][0], 3, g["h"], g["w"], be3.weights)
    finally:
        be3.set_option(scb.backend.SCB_OPT_FUSE_TRANS, 1)
    check_parity(oracle, "unfused 80x64", g["y"][0], got)


@pytest.mark.parametrize("stem", ["color_80x64", "color_128x128"])
def test_forward_fp32_residual_matches_golden(goldens, oracle, scb, be3, stem):
    """The residual stream kept in fp32 (SCB_OPT_RESIDUAL32 = 1), the reference's
    precision, end to end; the default keeps it in fp16."""
    _gpu()
    g = goldens[stem]
    be3.set_option(scb.backend.SCB_OPT_RESIDUAL32, 1)
    try:
        got = scb.run(be3, g["x"][0], 3, g["h"], g["w"], be3.weights)
    finally:
        be3.set_option(scb.backend.SCB_OPT_RESIDUAL32, 0)
    check_parity(oracle, f"fp32 residual {stem}", g["y"][0], got)


def test_forward_host_batched_uint8(scb, oracle, be3, weights3):
    """uint8 in, the pad/crop fused on the device, two different images in one
    call; each must match the oracle."""
    _gpu()
    x = np.concatenate([scb.synth.noisy_image(s, 3, 72, 136, 25 / 255)[None] for s in (1, 2)])
    y = be3.forward_host(x)
    want = oracle.forward(x.astype(np.float32) / 255.0, weights3.tensors)
    for i in range(2):
        check_parity(oracle, f"batched {i}", want[i], y[i])


def test_uint8_output_matches_quantised_f32(scb, oracle, be3):
    """The fused uint8 output path quantises exactly like src/image.rs:60-63."""
    _gpu()
    x = scb.synth.noisy_image(9, 3, 100, 72, 15 / 255)[None]
    y32 = be3.forward_host(x)
    y8 = be3.forward_host(x, out_u8=True)
    assert y8.dtype == np.uint8
    assert np.array_equal(y8.astype(np.int32), oracle.quantise(y32))


def test_gray_batched(scb, oracle, be1, weights1):
    """Grayscale (config 3's model) with a batch of 3 uint8 images."""
    _gpu()
    x = np.concatenate([scb.synth.noisy_image(20 + s, 1, 64, 128, 50 / 255)[None] for s in range(3)])
    y = be1.forward_host(x)
    want = oracle.forward(x.astype(np.float32) / 255.0, weights1.tensors)
    for i in range(3):
        check_parity(oracle, f"gray batched {i}", want[i], y[i])


def test_repeats_are_bit_identical(scb, be3):
    _gpu()
    x = scb.synth.noisy_image(5, 3, 256, 192, 25 / 255)[None]
    first = be3.forward_host(x)
    for r in range(5):
        again = be3.forward_host(x)
        assert np.array_equal(first, again), f"run {r + 1} differs: max {np.abs(first - again).max():.3e}"


def test_footprint_and_release(scb, be3):
    _gpu()
    be3.forward_host(scb.synth.noisy_image(3, 3, 64, 64, 0.1)[None])
    wb, sb = be3.footprint()
    assert wb > 30e6 and sb > 0
    be3.release_scratch()
    assert be3.footprint()[1] == 0


@pytest.mark.parametrize("stem,h,w", [("c64", 256, 192), ("c64b", 72, 136), ("c64c", 200, 328)])
def test_block_boundary_kernel_is_bit_identical(scb, be3, stem, h, w):
    """The block-boundary kernel (block i's conv1_2 and block i+1's conv1_1 in one
    launch, SCB_OPT_FUSE_PAIR = 1, the default) computes the same fp16 values as the
    two separate GEMM launches: the whole forward is bit-identical either way."""
    _gpu()
    x = scb.synth.noisy_image(len(stem) + h, 3, h, w, 25 / 255)[None]
    fused = be3.forward_host(x)
    n_fused = be3.last_launch_count()
    be3.set_option(scb.backend.SCB_OPT_FUSE_PAIR, 0)
    try:
        sep = be3.forward_host(x)
        n_sep = be3.last_launch_count()
    finally:
        be3.set_option(scb.backend.SCB_OPT_FUSE_PAIR, 1)
    assert n_sep - n_fused == 12, (n_sep, n_fused)  # 3 boundaries x 4 stages at 64 / 128 channels
    assert np.array_equal(fused, sep), f"max |diff| {np.abs(fused - sep).max():.3e}"


def test_paired_slab_epilogue_is_bit_identical(scb, be3):
    """The flat GEMMs' 64-column epilogue rounds (SCB_OPT_GEMM_PAIRS = 1, the default:
    qkv and the LayerNorm-fused conv1_1 at 1/4 and 1/8 resolution, among others) store
    the same fp16 / fp32 values as the 32-column slab loop: the forward is bit-identical,
    and the paired variants are the ones that ran."""
    _gpu()
    x = scb.synth.noisy_image(91, 3, 136, 200, 25 / 255)[None]
    be3.set_profiling(True)
    try:
        paired = be3.forward_host(x)
        k_on = be3.profile_kernels()
        be3.set_option(scb.backend.SCB_OPT_GEMM_PAIRS, 0)
        try:
            slabs = be3.forward_host(x)
            k_off = be3.profile_kernels()
        finally:
            be3.set_option(scb.backend.SCB_OPT_GEMM_PAIRS, 1)
    finally:
        be3.set_profiling(False)
    paired_name = re.compile(r"gemm_tc_kernel<\d+, \d+, \d+, 1, 1>")  # <BN, BK, geometry, TMA, paired>
    assert any(paired_name.fullmatch(k) for k in k_on) and not any(paired_name.fullmatch(k) for k in k_off)
    assert len(k_on) == len(k_off)
    assert np.array_equal(paired, slabs), f"max |diff| {np.abs(paired - slabs).max():.3e}"
