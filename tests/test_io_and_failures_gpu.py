"""The network's two ends on their own, and the failure paths, on the GPU through
the C ABI.

* m_head (`scb_probe_head`): the replicate pad of `src/plan.rs:67-82`, fused as a
  clamped read, then the 3x3 conv c -> 64 (zero pad 1, no bias); uint8 and float32
  inputs, colour and gray, widths and heights that are not multiples of 64.
* m_tail (`scb_probe_tail`): the 3x3 conv 64 -> c and the crop of
  `src/plan.rs:85-94`, float32 and uint8 outputs (the quantisation of
  `src/image.rs:60-63`).
  Each is checked twice: against a float64 convolution of the very fp16 operands
  the tensor cores read (1e-5 of scale: only accumulation order differs), and
  against the oracle's own pad / conv3x3 / crop on the float32 data at the
  acceptance bar (2e-3).
* Failure paths, in forms that fault nothing: a bounded device wait that runs out
  (SCB_EDEVICE, the context still usable afterwards), the admission refusal before
  any allocation (SCB_ENOMEM), and the memory and profile reports
  (`Backend::mem_report` / `profile_report`, `src/backend.rs:33-44`).
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

BAR = 2e-3


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def _f16(a):
    return np.asarray(a, np.float32).astype(np.float16).astype(np.float64)


def _conv3x3_f64(x_hwc, w):
    """x [h][w][ci] float64, w [co][ci][3][3] float64 -> [h][w][co], zero pad 1."""
    h, wd, _ = x_hwc.shape
    xp = np.pad(x_hwc, ((1, 1), (1, 1), (0, 0)))
    acc = np.zeros((h, wd, w.shape[0]))
    for ky in range(3):
        for kx in range(3):
            acc += xp[ky:ky + h, kx:kx + wd] @ w[:, :, ky, kx].T
    return acc


def _scaled_max(want, got):
    return float(np.abs(np.asarray(want, np.float64) - got).max() / max(np.abs(want).max(), 1e-6))


@pytest.mark.parametrize("in_nc,n,h,w,u8", [(3, 2, 72, 136, True), (3, 1, 64, 64, False), (1, 2, 100, 70, True),
                                           (3, 1, 130, 200, False), (1, 1, 1, 1, False)])
def test_head_probe(scb, oracle, be3, be1, in_nc, n, h, w, u8):
    torch = _torch()
    be = be3 if in_nc == 3 else be1
    hp, wp = -(-h // 64) * 64, -(-w // 64) * 64
    rng = np.random.default_rng(100 * in_nc + h + w)
    if u8:
        x = rng.integers(0, 256, (n, in_nc, h, w), dtype=np.uint8)
        xf = x.astype(np.float32) / np.float32(255)
    else:
        xf = x = rng.random((n, in_nc, h, w), dtype=np.float32)
    xd = torch.from_numpy(x).cuda()
    x1 = torch.full((n, hp, wp, 64), float("nan"), dtype=torch.float32, device="cuda")
    x16 = torch.full((n, hp, wp, 64), float("nan"), dtype=torch.float16, device="cuda")
    rc = be.lib.scb_probe_head(be.ctx, xd.data_ptr(), scb.SCB_U8 if u8 else scb.SCB_F32, n, in_nc, h, w,
                               x1.data_ptr(), x16.data_ptr())
    assert rc == 0, be.lib.scb_last_error(be.ctx).decode()
    got32, got16 = x1.cpu().numpy(), x16.float().cpu().numpy()
    assert np.isfinite(got32).all() and np.isfinite(got16).all(), "head left pixels unwritten"
    wh = be.weights.tensors["m_head.0.weight"]
    for i in range(n):
        padded = scb.plan.pad_replicate(xf[i], in_nc, h, w, hp, wp).transpose(1, 2, 0)   # [hp][wp][c]
        exact = _conv3x3_f64(_f16(padded), _f16(wh))
        assert _scaled_max(exact, got32[i]) <= 1e-5, f"image {i}: x1 vs the fp16-operand conv"
        assert _scaled_max(exact, got16[i]) <= 1e-3, f"image {i}: fp16 shadow"
        want = oracle.conv3x3(np.ascontiguousarray(padded), wh)                          # the oracle, fp32
        d = float(np.abs(want - got32[i]).max())
        assert d <= BAR, f"image {i}: |head - oracle| {d:.2e}"


@pytest.mark.parametrize("in_nc,n,h,w", [(3, 2, 72, 136), (3, 1, 64, 64), (1, 2, 100, 70), (3, 1, 130, 250),
                                         (1, 1, 1, 1)])
def test_tail_probe(scb, oracle, be3, be1, in_nc, n, h, w):
    torch = _torch()
    be = be3 if in_nc == 3 else be1
    hp, wp = -(-h // 64) * 64, -(-w // 64) * 64
    rng = np.random.default_rng(7 * in_nc + h * w)
    s = (rng.standard_normal((n, hp, wp, 64)) * 0.5).astype(np.float16)  # (y + x1), the tail's operand
    sd = torch.from_numpy(s).cuda()
    y32 = torch.full((n, in_nc, h, w), float("nan"), dtype=torch.float32, device="cuda")
    y8 = torch.zeros((n, in_nc, h, w), dtype=torch.uint8, device="cuda")
    for y, dt in ((y32, scb.SCB_F32), (y8, scb.SCB_U8)):
        rc = be.lib.scb_probe_tail(be.ctx, sd.data_ptr(), n, in_nc, h, w, y.data_ptr(), dt)
        assert rc == 0, be.lib.scb_last_error(be.ctx).decode()
    got = y32.cpu().numpy()
    assert np.isfinite(got).all(), "tail left output values unwritten"
    wt = be.weights.tensors["m_tail.0.weight"]
    for i in range(n):
        exact = _conv3x3_f64(s[i].astype(np.float64), _f16(wt)).transpose(2, 0, 1)
        exact = scb.plan.crop(exact, in_nc, h, w, hp, wp)
        assert _scaled_max(exact, got[i]) <= 1e-5, f"image {i}: tail vs the fp16-operand conv"
        want = scb.plan.crop(oracle.conv3x3(s[i].astype(np.float32), wt).transpose(2, 0, 1), in_nc, h, w, hp, wp)
        d = float(np.abs(want - got[i]).max())
        assert d <= BAR, f"image {i}: |tail - oracle| {d:.2e}"
    # uint8 output: the quantisation of src/image.rs:60-63 applied to the f32 output
    # (one level apart at most where v*255 + 0.5 lands on an integer: fma rounding)
    lv = np.abs(y8.cpu().numpy().astype(np.int32) - oracle.quantise(got))
    assert lv.max() <= 1 and (lv > 0).mean() <= 1e-4


def test_wait_timeout_reports_edevice_and_context_survives(scb, be3):
    """A bounded wait that nothing completes: the kernel gives up after 2 ms, the call
    returns SCB_EDEVICE with the message a forward would give, the error word is
    cleared, and the next forward on the same context works."""
    torch = _torch()
    import time
    t = time.perf_counter()
    rc = be3.lib.scb_probe_wait_timeout(be3.ctx, 2000)
    dt = time.perf_counter() - t
    assert rc == -5, rc
    assert "bounded wait" in be3.lib.scb_last_error(be3.ctx).decode()
    assert dt < 5.0
    assert be3.lib.scb_probe_wait_timeout(be3.ctx, 0) == -1  # limits are range-checked
    x = scb.synth.noisy_image(3, 3, 64, 64, 0.1)[None]
    y = be3.forward_host(x)
    assert np.isfinite(y).all()
    assert torch.cuda.is_available()


def test_admission_refuses_before_allocating(scb, be3):
    """A batch whose arena cannot fit in device memory is refused on the host with the
    memguard message, before cudaMalloc (`memguard::check_cuda`,
    src/memguard.rs:262-285); nothing is launched and the context stays usable."""
    torch = _torch()
    n, h, w = 100, 2048, 2048                     # ~490 GB of scratch, > any B200
    assert scb.need_bytes(n, 3, h, w) > 2 * torch.cuda.get_device_properties(0).total_memory
    xd = torch.zeros((n, 3, h, w), dtype=torch.uint8, device="cuda")      # real buffers of the
    yd = torch.zeros((n, 3, h, w), dtype=torch.uint8, device="cuda")      # requested size
    be3.release_scratch()
    import ctypes
    need, avail = ctypes.c_size_t(0), ctypes.c_size_t(0)
    assert be3.lib.scb_check_admission(be3.ctx, 1, 64, 64, ctypes.byref(need), ctypes.byref(avail)) == 0
    assert 0 < need.value < avail.value
    rc = be3.lib.scb_check_admission(be3.ctx, n, h, w, ctypes.byref(need), ctypes.byref(avail))
    assert rc == -4 and need.value == scb.need_bytes(n, 3, h, w) and need.value > avail.value
    rc = be3.lib.scb_forward_dev(be3.ctx, xd.data_ptr(), scb.SCB_U8, n, 3, h, w, yd.data_ptr(), scb.SCB_U8, None)
    msg = be3.lib.scb_last_error(be3.ctx).decode()
    assert rc == -4 and "needs" in msg and "GiB free" in msg, (rc, msg)
    assert be3.footprint()[1] == 0, "an arena was allocated for a refused request"
    del xd, yd
    y = be3.forward_host(scb.synth.noisy_image(4, 3, 64, 64, 0.1)[None])
    assert np.isfinite(y).all()


def test_mem_and_profile_report(scb, weights3):
    """mem_report's high-water covers the largest arena held at once, survives
    release_scratch, and `fixed` is the no-allocation array reserved by scb_create;
    profile_report lists the op classes of a profiled forward."""
    torch = _torch()
    be = scb.B200(weights3)
    try:
        m0 = be.mem_report()
        wb, _ = be.footprint()
        assert m0["live"] == wb and m0["high_water"] == wb and m0["fixed"] == 14 << 20
        x = scb.synth.noisy_image(1, 3, 256, 256, 0.1)[None]
        be.forward_host(x)
        m1 = be.mem_report()
        assert m1["live"] == sum(be.footprint()) and m1["high_water"] >= m1["live"] > wb
        be.release_scratch()
        m2 = be.mem_report()
        assert m2["live"] == wb and m2["high_water"] == m1["high_water"]
        assert be.profile_report() == ""
        be.set_profiling(True)
        be.forward_host(x)
        rep = be.profile_report()
        print(rep)
        for cls in ("conv1x1", "conv3x3", "trans_fused", "head", "tail"):
            assert cls in rep, cls
        assert "device time per op class" in rep
    finally:
        be.close()
    assert torch.cuda.is_available()
