"""The no-allocation forward, scb_forward_dev_noalloc, against scb_forward_dev.

scb_forward_dev_noalloc serves callers that cannot allocate device memory when
they call - a server that reserves all of its device memory at start-up and must
not have a request stall or fail inside cudaMalloc, or a host whose own allocator
owns the GPU's memory. Its scratch is a fixed 14 MiB array inside the library, so
it takes padded batches of at most 8192 pixels. This test calls it twice in a row
through the C ABI, on two different images and geometries inside that limit, and
checks each output against the allocating entry point's output for the same
input; then it checks that a request over the limit is refused with a message.

A second test creates a fresh context and makes the no-allocation forward its
first GPU work: the device's free memory must not change across that call (the
context reserved the array and loaded the device code when it was created), and
its output must match a later allocating forward.

This file is named to be collected last, so a run that stops at the first
failure has already run every other test.
"""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu

MAX_ABS = 2e-3  # the parity bar the other forward tests use


def test_noalloc_forward_matches_forward_dev(scb, weights3):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    be = scb.B200(weights3)
    try:
        stream = torch.cuda.Stream()
        sp = stream.cuda_stream
        for call, (n, h, w) in enumerate([(1, 64, 100), (2, 64, 64)]):
            x = np.concatenate([scb.synth.noisy_image(40 + 5 * call + k, 3, h, w, 25 / 255)[None] for k in range(n)])
            xd = torch.from_numpy(x).cuda()
            y_ref = torch.empty((n, 3, h, w), dtype=torch.float32, device="cuda")
            y_na = torch.full((n, 3, h, w), float("nan"), dtype=torch.float32, device="cuda")
            torch.cuda.synchronize()
            be.forward_dev(xd.data_ptr(), scb.SCB_U8, n, 3, h, w, y_ref.data_ptr(), scb.SCB_F32, sp)
            rc = be.lib.scb_forward_dev_noalloc(be.ctx, xd.data_ptr(), scb.SCB_U8, n, 3, h, w, y_na.data_ptr(),
                                                scb.SCB_F32, sp)
            assert rc == 0, be.lib.scb_last_error(be.ctx).decode()
            stream.synchronize()
            want, got = y_ref.cpu().numpy(), y_na.cpu().numpy()
            assert np.isfinite(got).all(), f"call {call}: output not fully written"
            d = float(np.abs(want - got).max())
            print(f"call {call} ({n} x {h}x{w}): max |noalloc - forward_dev| = {d:.3e}")
            assert d <= MAX_ABS, f"call {call}: max |diff| {d:.3e}"

        # over the limit: refused with a message, nothing launched
        xd = torch.zeros((1, 3, 72, 100), dtype=torch.uint8, device="cuda")
        yd = torch.zeros((1, 3, 72, 100), dtype=torch.float32, device="cuda")
        rc = be.lib.scb_forward_dev_noalloc(be.ctx, xd.data_ptr(), scb.SCB_U8, 1, 3, 72, 100, yd.data_ptr(),
                                            scb.SCB_F32, sp)
        assert rc == -1 and "8192" in be.lib.scb_last_error(be.ctx).decode()
    finally:
        be.close()


def test_noalloc_first_call_on_fresh_context_allocates_nothing(scb, weights3):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    be = scb.B200(weights3)
    try:
        n, h, w = 1, 64, 128
        x = scb.synth.noisy_image(77, 3, h, w, 25 / 255)[None]
        xd = torch.from_numpy(x).cuda()
        y_na = torch.full((n, 3, h, w), float("nan"), dtype=torch.float32, device="cuda")
        y_ref = torch.empty((n, 3, h, w), dtype=torch.float32, device="cuda")
        stream = torch.cuda.Stream()
        sp = stream.cuda_stream
        torch.cuda.synchronize()
        free0, _ = torch.cuda.mem_get_info()
        rc = be.lib.scb_forward_dev_noalloc(be.ctx, xd.data_ptr(), scb.SCB_U8, n, 3, h, w, y_na.data_ptr(),
                                            scb.SCB_F32, sp)
        assert rc == 0, be.lib.scb_last_error(be.ctx).decode()
        stream.synchronize()
        free1, _ = torch.cuda.mem_get_info()
        assert free1 == free0, f"the first no-allocation call changed free device memory by {free0 - free1} bytes"
        assert be.footprint()[1] == 0 and be.mem_report()["fixed"] == 14 << 20
        be.forward_dev(xd.data_ptr(), scb.SCB_U8, n, 3, h, w, y_ref.data_ptr(), scb.SCB_F32, sp)
        stream.synchronize()
        got, want = y_na.cpu().numpy(), y_ref.cpu().numpy()
        assert np.isfinite(got).all()
        d = float(np.abs(want - got).max())
        print(f"fresh context: max |noalloc - forward_dev| = {d:.3e}")
        assert d <= MAX_ABS
    finally:
        be.close()
