"""Parity at the benchmark configurations' full sizes, through the C ABI.

The reference is `oracle/scunet_torch.py` (the oracle restated in torch, pinned on
CPU to the numpy oracle and the goldens) run on the same B200 in strict FP32 (TF32
off). The bar is the acceptance criterion: max |diff| <= 2e-3 on the [0,1] output
and at most one 8-bit level of difference on >= 99.9 % of the values.

* config 4: 32 frames spread over the 256-frame batch (frame k of batch seed 4000
  is `synth.frame_at(4000, k)`, k = 0, 8, ..., 248), in the bench's 4-frame calls;
* config 3: all 64 gray 1024x1024 images, in 16-image calls;
* config 2: the 512x512 image;
* config 5: 8192^2 is too large for any FP32 oracle (~200 GB of activations); its
  banded path (8 bands, the 8-GPU split, run in lockstep on one GPU) is checked
  against the library's own whole-image forward of the same image, which the
  oracle checks at every other size.
Each test prints the worst max |diff| and the worst fraction of values more than one
8-bit level off over its images."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3          # north star: max |diff| on the [0,1] output
MAX_FRAC_GT1 = 1e-3     # north star: <= 1 level off on >= 99.9 % of values


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def _b200(be, scb, torch, x_u8):
    n, c, h, w = x_u8.shape
    xd = torch.from_numpy(x_u8).cuda()
    y = torch.empty((n, c, h, w), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    be.forward_dev(xd.data_ptr(), scb.SCB_U8, n, c, h, w, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    return y.cpu().numpy()


def _check(name, want, got, oracle):
    r = oracle.parity_report(want, got)
    print(f"{name}: {r}")
    assert r["max_abs"] <= MAX_ABS, f"{name}: max |diff| {r['max_abs']:.3e}"
    assert r["frac_level_gt1"] <= MAX_FRAC_GT1, f"{name}: {100 * r['frac_level_gt1']:.3f} % of values > 1 level"
    return r


def _batched(name, scb, be, weights, oracle, x, per_call):
    """Every image of x through the library (per_call images per call) and through
    the strict-FP32 torch oracle one image at a time; each image must meet the bar."""
    torch = _torch()
    import scunet_torch
    worst = {"max_abs": 0.0, "frac_level_gt1": 0.0}
    for i0 in range(0, x.shape[0], per_call):
        got = _b200(be, scb, torch, x[i0:i0 + per_call])
        for j in range(got.shape[0]):
            xi = x[i0 + j:i0 + j + 1].astype(np.float32) / 255
            with torch.no_grad():
                want = scunet_torch.forward(xi, weights.tensors, device="cuda").cpu().numpy()
            r = _check(f"{name}, image {i0 + j}", want, got[j:j + 1], oracle)
            for k in worst:
                worst[k] = max(worst[k], r[k])
    print(f"{name}: worst over {x.shape[0]} images: max |diff| {worst['max_abs']:.3e}, "
          f"values > 1 level off {100 * worst['frac_level_gt1']:.4f} %")
    be.release_scratch()


def test_config4_frames(scb, be3, weights3, oracle):
    """32 1920x1080 frames spread over the 256-frame batch, 4 per call (padded to
    1088 rows on the device)."""
    x = np.stack([scb.synth.frame_at(4000, k) for k in range(0, 256, 8)])
    _batched("config 4, 1920x1080", scb, be3, weights3, oracle, x, 4)


def test_config3_gray(scb, be1, weights1, oracle):
    """All 64 1024x1024 gray images of the batch (sigma drawn per image from
    {15, 25, 50}/255), 16 per call."""
    x = scb.synth.gray_batch(3001, 64)
    _batched("config 3, 1024x1024 gray", scb, be1, weights1, oracle, x, 16)


def test_config2_512(scb, be3, weights3, oracle):
    torch = _torch()
    import scunet_torch
    x = scb.synth.config_input(2)
    got = _b200(be3, scb, torch, x)
    want = scunet_torch.forward(x.astype(np.float32) / 255, weights3.tensors, device="cuda").cpu().numpy()
    _check("config 2, 512x512", want, got, oracle)


def test_config5_bands_at_8192(scb, be3):
    """Config 5 at its own size: one 8192x8192 image as 8 row bands of 1024 rows (the
    8-GPU split) in lockstep, against the whole-image forward of the same image
    (78 GB of scratch; released before the bands allocate theirs)."""
    torch = _torch()
    S = 8192
    x = scb.synth.noisy_image_device(1005, 3, S, S, 25 / 255, device="cuda")
    whole = torch.empty((1, 3, S, S), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    be3.release_scratch()
    be3.forward_dev(x.data_ptr(), scb.SCB_U8, 1, 3, S, S, whole.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    be3.release_scratch()
    bands = torch.full_like(whole, float("nan"))
    be3.forward_bands(8, x.data_ptr(), scb.SCB_U8, 3, S, S, bands.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    be3.release_scratch()
    assert bool(torch.isfinite(bands).all()), "some output rows were not written"
    d = (bands - whole).abs()
    dmax = float(d.max())
    rows = d.amax(dim=(0, 1, 3))
    print(f"8192x8192 in 8 bands: max |bands - whole| {dmax:.3e}; rows with any difference: "
          f"{int((rows > 0).sum())} of {S}")
    assert dmax <= 1e-4


def test_config5_bands_at_4096(scb, be3):
    """The banded schedule (4 lockstep bands) against the whole-image forward of the
    same 4096x4096 image; any difference would come from band geometry."""
    torch = _torch()
    x = scb.synth.noisy_image_device(1005, 3, 4096, 4096, 25 / 255, device="cuda")
    whole = torch.empty((1, 3, 4096, 4096), dtype=torch.float32, device="cuda")
    bands = torch.full_like(whole, float("nan"))
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    be3.forward_dev(x.data_ptr(), scb.SCB_U8, 1, 3, 4096, 4096, whole.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    be3.release_scratch()
    be3.forward_bands(4, x.data_ptr(), scb.SCB_U8, 3, 4096, 4096, bands.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    assert bool(torch.isfinite(bands).all()), "some output rows were not written"
    d = float((bands - whole).abs().max())
    print(f"4096x4096 in 4 bands: max |bands - whole| {d:.3e}")
    be3.release_scratch()  # ~30 GB of band arenas
    _, scratch = be3.footprint()
    assert scratch == 0, f"{scratch} bytes of scratch still held after release_scratch"
    assert d <= 1e-4


def test_speed_vs_torch_fp32_cuda(scb, be3, weights3):
    """The speed proxy for the reference's own CUDA path: the same network in torch
    CUDA FP32 (TF32 off) on the same B200, one 1920x1080 frame (padded to 1088 rows),
    inputs resident on the device, CUDA-event timed after warm-up. The reference
    reports its CUDA path 1.1-1.25x slower than upstream torch CUDA
    (`docs/TECH_NOTES.md:65-69`), so this ratio understates the speed-up over it."""
    torch = _torch()
    import scunet_torch
    import torch.nn.functional as F
    x = scb.synth.frames(4001, 1, 1080, 1920)
    xd = torch.from_numpy(x).cuda()
    y = torch.empty((1, 3, 1080, 1920), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()

    def ours():
        be3.forward_dev(xd.data_ptr(), scb.SCB_U8, 1, 3, 1080, 1920, y.data_ptr(), scb.SCB_F32, s.cuda_stream)

    scunet_torch.strict_fp32()
    wt = {k: torch.as_tensor(v, dtype=torch.float32).cuda().contiguous() for k, v in weights3.tensors.items()}
    xp = F.pad(xd.float().div_(255), (0, 0, 0, 8), mode="replicate")

    def proxy():
        with torch.no_grad():
            scunet_torch.forward_padded(xp, wt)

    def time_ms(fn, stream, warm, reps):
        with torch.cuda.stream(stream):
            for _ in range(warm):
                fn()
            torch.cuda.synchronize()
            t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            t0.record(stream)
            for _ in range(reps):
                fn()
            t1.record(stream)
        torch.cuda.synchronize()
        return t0.elapsed_time(t1) / reps

    ms_ours = time_ms(ours, s, 3, 10)
    ms_proxy = time_ms(proxy, torch.cuda.current_stream(), 1, 3)
    ratio = ms_proxy / ms_ours
    print(f"1920x1080 frame: this library {ms_ours:.2f} ms, torch CUDA FP32 {ms_proxy:.1f} ms, "
          f"ratio {ratio:.1f}x (x1.1-1.25 against the reference CUDA path: "
          f"{1.1 * ratio:.1f}-{1.25 * ratio:.1f}x)")
    assert ratio > 1.0
