"""One image in row bands (the 8192x8192 configuration's split) against the
whole-image forward.

The banded schedule (halo rows, per-block boundary exchange, shifted windows that
straddle band edges, the image-edge wrap handled by the global window mask) must
reproduce scb_forward_dev on the same image. On one GPU all bands run in lockstep
with device-to-device halo copies; with two or more GPUs the same bands run one per
process with NCCL send/recv."""
import multiprocessing as mp
import os

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-4  # same kernels on the same pixels; only tile grouping differs


def _torch():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    return torch


def _whole(be, scb, torch, x):
    c, h, w = x.shape[1:]
    xd = torch.from_numpy(x).cuda()
    y = torch.empty((1, c, h, w), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    be.forward_dev(xd.data_ptr(), scb.SCB_U8, 1, c, h, w, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    return y.cpu().numpy()


@pytest.mark.parametrize("fused", [1, 0])
@pytest.mark.parametrize("h,w,nbands", [(256, 192, 2), (256, 192, 4), (200, 136, 3), (512, 128, 8)])
def test_virtual_bands_match_whole_image(scb, be3, h, w, nbands, fused):
    torch = _torch()
    if not fused and nbands not in (2, 3):
        pytest.skip("one geometry per split is enough for the separate-launch path")
    be3.set_option(scb.backend.SCB_OPT_FUSE_TRANS, fused)
    try:
        x = scb.synth.noisy_image(60 + nbands, 3, h, w, 25 / 255)[None]
        want = _whole(be3, scb, torch, x)
        xd = torch.from_numpy(x).cuda()
        y = torch.full((1, 3, h, w), float("nan"), dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        torch.cuda.synchronize()
        be3.forward_bands(nbands, xd.data_ptr(), scb.SCB_U8, 3, h, w, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
        s.synchronize()
        got = y.cpu().numpy()
    finally:
        be3.set_option(scb.backend.SCB_OPT_FUSE_TRANS, 1)
    assert np.isfinite(got).all(), "some output rows were not written"
    d = np.abs(got - want)
    print(f"{h}x{w} in {nbands} bands (fused {fused}): max |bands - whole| {d.max():.3e}")
    assert d.max() <= TOL, f"max {d.max():.3e} at row {np.unravel_index(d.argmax(), d.shape)[2]}"


def test_single_rank_band_group(scb, be3):
    """scb_band_init with one rank: the NCCL path with the whole image as one band."""
    torch = _torch()
    x = scb.synth.noisy_image(70, 3, 128, 192, 25 / 255)[None]
    want = _whole(be3, scb, torch, x)
    be = scb.B200(be3.weights)
    try:
        be.band_init(scb.band_unique_id(), 0, 1)
        xd = torch.from_numpy(x).cuda()
        y = torch.full((1, 3, 128, 192), float("nan"), dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        torch.cuda.synchronize()
        be.forward_band(xd.data_ptr(), scb.SCB_U8, 3, 128, 192, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
        s.synchronize()
        got = y.cpu().numpy()
    finally:
        be.close()
    assert np.abs(got - want).max() <= TOL


def _band_worker(rank, nranks, uid, x, q):
    import importlib
    import sys
    import torch
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    scb = importlib.import_module("scunet-rs_b200")
    torch.cuda.set_device(rank)
    be = scb.B200(scb.Weights.seeded(3, 0), device=rank)
    be.band_init(uid, rank, nranks)
    c, h, w = x.shape[1:]
    # Only the input rows the band reads hold the image; the others hold its negative,
    # which must not reach this rank's output.
    lo, hi = scb.shard.band_input_rows(h, -(-h // 64) * 64, rank, nranks)
    xs = 255 - x
    xs[:, :, lo:hi] = x[:, :, lo:hi]
    xd = torch.from_numpy(xs).cuda()
    y = torch.full((1, c, h, w), float("nan"), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    be.forward_band(xd.data_ptr(), scb.SCB_U8, c, h, w, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    r0, rows = scb.shard.band_rows(-(-h // 64) * 64, rank, nranks)
    q.put((rank, r0, y.cpu().numpy()[:, :, r0:min(r0 + rows, h)]))
    be.close()


def test_two_gpu_bands_over_nccl(scb, be3):
    """Two processes, one GPU and one band each, halo rows over NCCL; each rank's
    input holds the image only on the rows `shard.band_input_rows` names."""
    torch = _torch()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    x = scb.synth.noisy_image(71, 3, 320, 256, 25 / 255)[None]
    want = _whole(be3, scb, torch, x)
    uid = scb.band_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_band_worker, args=(r, 2, uid, x, q)) for r in range(2)]
    for p in procs:
        p.start()
    parts = [q.get(timeout=300) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    got = np.full_like(want, np.nan)
    for _, r0, part in parts:
        got[:, :, r0:r0 + part.shape[2]] = part
    d = np.abs(got - want)
    print(f"2-GPU bands: max |bands - whole| {np.nanmax(d):.3e}")
    assert np.isfinite(got).all() and d.max() <= TOL


def _full_size_worker(rank, nranks, uid, S, q):
    """One rank of the 8192^2 check: the whole-image forward of the image on this
    rank's own GPU, then this rank's band over NCCL, compared on the device."""
    import importlib
    import sys
    import torch
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    scb = importlib.import_module("scunet-rs_b200")
    torch.cuda.set_device(rank)
    be = None
    try:
        be = scb.B200(scb.Weights.seeded(3, 0), device=rank)
        x = scb.synth.noisy_image_device(1005, 3, S, S, 25 / 255, device="cuda")
        whole = torch.empty((1, 3, S, S), dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        torch.cuda.synchronize()
        be.forward_dev(x.data_ptr(), scb.SCB_U8, 1, 3, S, S, whole.data_ptr(), scb.SCB_F32, s.cuda_stream)
        s.synchronize()
        be.release_scratch()
        be.band_init(uid, rank, nranks)
        y = torch.full_like(whole, float("nan"))
        be.forward_band(x.data_ptr(), scb.SCB_U8, 3, S, S, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
        be.band_sync(600000, s.cuda_stream)
        r0, rows = scb.shard.band_rows(S, rank, nranks)
        band, ref = y[:, :, r0:r0 + rows], whole[:, :, r0:r0 + rows]
        q.put((rank, bool(torch.isfinite(band).all()), float((band - ref).abs().max())))
    except Exception as e:  # reported, not raised: the parent reads the queue
        q.put((rank, False, repr(e)))
    finally:
        if be is not None:
            be.close()


def test_two_gpu_bands_at_8192(scb):
    """Config 5 at its own size over two GPUs and NCCL: each rank's band of the
    8192x8192 image equals the whole-image forward's rows (both ranks also run the
    whole image on their own GPU, 78 GB of scratch, released before the bands)."""
    torch = _torch()
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    uid = scb.band_unique_id()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_full_size_worker, args=(r, 2, uid, 8192, q)) for r in range(2)]
    for p in procs:
        p.start()
    try:
        res = sorted(q.get(timeout=600) for _ in procs)
    finally:
        for p in procs:
            p.join(timeout=120)
            if p.is_alive():
                p.kill()
    for rank, finite, d in res:
        print(f"8192^2, 2 GPUs, rank {rank}: max |band - whole| {d}")
        assert finite and isinstance(d, float) and d <= TOL, (rank, finite, d)


def test_band_sync_deadline_aborts_group(scb, be3):
    """scb_band_sync's deadline on one GPU: a one-rank band group (no peer, so no NCCL
    kernel ever waits), a forward of a 2048x2048 image, and a wait with a 0 ms
    deadline that the forward cannot meet. The call returns SCB_ECUDA naming the
    deadline, the group is aborted (the next banded forward refuses until scb_band_init
    runs again), the forward itself completes, and a re-initialised group works.
    The other failure - a peer rank that dies while its memory is mapped by this
    one - is not run on a GPU (see the design notes); its host logic is tested on CPU."""
    torch = _torch()
    x = scb.synth.noisy_image_device(72, 3, 2048, 2048, 25 / 255, device="cuda")
    be = scb.B200(be3.weights)
    try:
        be.band_init(scb.band_unique_id(), 0, 1)
        y = torch.empty((1, 3, 2048, 2048), dtype=torch.float32, device="cuda")
        s = torch.cuda.Stream()
        torch.cuda.synchronize()
        be.forward_band(x.data_ptr(), scb.SCB_U8, 3, 2048, 2048, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
        rc = be.lib.scb_band_sync(be.ctx, s.cuda_stream, 0)
        msg = be.lib.scb_last_error(be.ctx).decode()
        s.synchronize()
        assert rc == -3 and "did not finish within 0 ms" in msg and "aborted" in msg, (rc, msg)
        rc = be.lib.scb_forward_band(be.ctx, x.data_ptr(), scb.SCB_U8, 3, 2048, 2048, y.data_ptr(), scb.SCB_F32,
                                     s.cuda_stream)
        assert rc == -1, "a banded forward ran on an aborted group"
        be.band_init(scb.band_unique_id(), 0, 1)
        be.forward_band(x.data_ptr(), scb.SCB_U8, 3, 2048, 2048, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
        be.band_sync(120000, s.cuda_stream)
        assert bool(torch.isfinite(y).all())
    finally:
        be.close()
