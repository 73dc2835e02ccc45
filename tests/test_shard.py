"""Host logic of the multi-GPU paths on CPU: frame and row-band partitions, and the
max-over-ranks reduction the bench times with, over a 2-rank gloo group."""
import multiprocessing as mp
import os
import socket

import pytest


def test_frame_slices_cover_batch(scb):
    for n, world in [(256, 8), (64, 3), (16, 16), (5, 2)]:
        sl = [scb.shard.frame_slice(n, r, world) for r in range(world)]
        assert sl[0][0] == 0 and sl[-1][1] == n
        assert all(a[1] == b[0] for a, b in zip(sl, sl[1:]))
        assert max(b - a for a, b in sl) - min(b - a for a, b in sl) <= 1


def test_band_rows_cover_image(scb):
    for hp, world in [(8192, 8), (1088, 3), (256, 4), (64, 1)]:
        bands = [scb.shard.band_rows(hp, r, world) for r in range(world)]
        assert bands[0][0] == 0 and sum(r for _, r in bands) == hp
        assert all(r % 64 == 0 and r > 0 for _, r in bands)
    with pytest.raises(ValueError):
        scb.shard.band_rows(128, 0, 3)


def test_band_input_rows_are_the_rows_the_head_reads(scb):
    """The input rows a band reads, against the head conv's read pattern written out:
    rows y - 1, y, y + 1 of every band row y inside the padded image, clamped to
    h - 1 by the replicate pad (io_kernels.cuh, head_tc_kernel's im2col)."""
    for h, world in [(8192, 8), (1080, 3), (1000, 2), (65, 2), (130, 3), (1, 1), (64, 1)]:
        hp = -(-h // 64) * 64
        for r in range(world):
            r0, rows = scb.shard.band_rows(hp, r, world)
            read = {min(yy, h - 1) for y in range(r0, r0 + rows) for yy in (y - 1, y, y + 1) if 0 <= yy < hp}
            lo, hi = scb.shard.band_input_rows(h, hp, r, world)
            assert (lo, hi) == (min(read), max(read) + 1), (h, world, r)
            assert read == set(range(lo, hi))
    with pytest.raises(ValueError):
        scb.shard.band_input_rows(100, 64, 0, 1)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _gloo_worker(rank, world, port, q):
    import importlib
    import sys
    import torch.distributed as dist
    sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
    scb = importlib.import_module("scunet-rs_b200")
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    lo, hi = scb.shard.frame_slice(256, rank, world)
    t = scb.shard.max_over_ranks(float(10 + rank))
    q.put((rank, lo, hi, t))
    dist.destroy_process_group()


def test_max_over_ranks_gloo(scb):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    ps = [ctx.Process(target=_gloo_worker, args=(r, world, port, q)) for r in range(world)]
    for p in ps:
        p.start()
    out = sorted(q.get(timeout=120) for _ in ps)
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert [o[3] for o in out] == [11.0, 11.0]          # every rank sees the max
    assert out[0][1:3] == (0, 128) and out[1][1:3] == (128, 256)
