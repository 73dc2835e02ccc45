"""How work is divided over ranks (host logic of the multi-GPU paths).

Batch sharding (configs 3-4): frame i of a batch goes to rank i * world // n ... as
contiguous, near-equal slices; no collective touches the data. Row bands (config
5): the padded image's 64-row blocks go to ranks as contiguous near-equal runs -
the same rule the library's band planner uses (scb_forward_band), so a caller
knows which output rows each rank writes.
"""
from __future__ import annotations


def frame_slice(n_frames, rank, world):
    """[lo, hi) of the frames this rank processes."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} of {world}")
    return n_frames * rank // world, n_frames * (rank + 1) // world


def band_rows(hp, rank, world):
    """(R0, rows): the padded-image rows of this rank's band (hp a multiple of 64)."""
    nblk = hp // 64
    if hp % 64 or nblk < world or not 0 <= rank < world:
        raise ValueError(f"{hp} padded rows cannot be split into {world} bands of 64-row blocks")
    b0, b1 = rank * nblk // world, (rank + 1) * nblk // world
    return 64 * b0, 64 * (b1 - b0)


def band_input_rows(h, hp, rank, world):
    """[lo, hi) of the input image's h rows that this rank's band reads. The head's
    3x3 conv of band rows [R0, R0 + rows) reads one row above and one below, and a
    padded row at or past h reads row h - 1 (the replicate pad), so a caller holding
    the image on the host copies only these rows to the rank's GPU."""
    if h < 1 or hp < h:
        raise ValueError(f"image of {h} rows, padded to {hp}")
    r0, rows = band_rows(hp, rank, world)
    lo = min(max(r0 - 1, 0), h - 1)
    return lo, max(lo + 1, min(r0 + rows + 1, h))


def max_over_ranks(value, group=None):
    """The largest value over the ranks of the default (or given) process group;
    the value itself when torch.distributed is not initialised."""
    import torch
    import torch.distributed as dist
    if not dist.is_available() or not dist.is_initialized():
        return value
    dev = "cuda" if dist.get_backend(group) == "nccl" else "cpu"
    t = torch.tensor([float(value)], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
