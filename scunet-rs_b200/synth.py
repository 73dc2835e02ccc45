"""Seeded synthetic inputs for the five benchmark configurations.

The reference ships no generator (its benchmark plane is a golden-ratio sequence,
`tools/bench_torch.py:37-43`; its tests use `sin(sin(i*a)*0.7+0.3a)`,
`tests/cuda_ops.rs:36-38`). These stand in for real photographs with the shapes,
value ranges and noise models the configurations name: a smooth clean field (8
low-frequency sinusoids plus 16 constant rectangles per channel, normalised to
[0,1]) plus Gaussian noise, clipped and quantised to uint8 - the form the CLI
feeds the network after `image::read` (`src/image.rs:17-42`).
"""
from __future__ import annotations

import numpy as np


def smooth_field(rng, c, h, w):
    """[c][h][w] float64 in [0, 1]. Each sinusoid sin(2 pi (fy y/h + fx x/w) + ph) is
    evaluated separably, sin(a + b) = sin a cos b + cos a sin b, as two outer products."""
    ya = 2 * np.pi * np.arange(h, dtype=np.float64) / h
    xa = 2 * np.pi * np.arange(w, dtype=np.float64) / w
    out = np.empty((c, h, w))
    for ch in range(c):
        f = np.zeros((h, w))
        for _ in range(8):
            fy, fx = rng.uniform(0.0, 4.0, 2)
            ph = rng.uniform(0.0, 2 * np.pi)
            amp = rng.uniform(0.2, 1.0)
            a = fy * ya + ph
            b = fx * xa
            f += np.multiply.outer(amp * np.sin(a), np.cos(b))
            f += np.multiply.outer(amp * np.cos(a), np.sin(b))
        for _ in range(16):
            y0, x0 = int(rng.integers(0, h)), int(rng.integers(0, w))
            rh, rw = int(rng.integers(2, max(3, h // 4))), int(rng.integers(2, max(3, w // 4)))
            f[y0:y0 + rh, x0:x0 + rw] = rng.uniform(f.min(), f.max())
        lo, hi = f.min(), f.max()
        out[ch] = (f - lo) / (hi - lo + 1e-12)
    return out


def noisy_image_device(seed, c, h, w, sigma, device="cuda"):
    """Config 5 on the GPU: the same construction as `noisy_image` (smooth field +
    N(0, sigma), clipped, quantised) computed with torch on `device`, for sizes
    where the host generator would dominate a benchmark run. Deterministic for a
    seed on a given device type (its random stream is torch's, not numpy's)."""
    import torch
    rng = np.random.default_rng(seed)
    gen = torch.Generator(device=device)
    gen.manual_seed(seed)
    ya = 2 * np.pi * torch.arange(h, device=device, dtype=torch.float32) / h
    xa = 2 * np.pi * torch.arange(w, device=device, dtype=torch.float32) / w
    out = torch.empty((c, h, w), device=device, dtype=torch.float32)
    for ch in range(c):
        f = torch.zeros((h, w), device=device, dtype=torch.float32)
        for _ in range(8):
            fy, fx = rng.uniform(0.0, 4.0, 2)
            ph = rng.uniform(0.0, 2 * np.pi)
            amp = rng.uniform(0.2, 1.0)
            a = fy * ya + ph
            b = fx * xa
            f += amp * (torch.outer(torch.sin(a), torch.cos(b)) + torch.outer(torch.cos(a), torch.sin(b)))
        for _ in range(16):
            y0, x0 = int(rng.integers(0, h)), int(rng.integers(0, w))
            rh, rw = int(rng.integers(2, max(3, h // 4))), int(rng.integers(2, max(3, w // 4)))
            f[y0:y0 + rh, x0:x0 + rw] = float(rng.uniform(float(f.min()), float(f.max())))
        out[ch] = (f - f.min()) / (f.max() - f.min() + 1e-12)
    out += torch.randn(out.shape, generator=gen, device=device) * sigma
    return torch.floor(out.clamp(0.0, 1.0) * 255.0 + 0.5).to(torch.uint8)[None]


def quantise(x):
    """float [0,1] -> uint8, `clamp(v,0,1)*255 + 0.5` truncated (`src/image.rs:60-63`)."""
    return np.floor(np.clip(x, 0.0, 1.0) * 255.0 + 0.5).astype(np.uint8)


def noisy_image(seed, c, h, w, sigma):
    """Config 1/2/5: smooth field + N(0, sigma) (sigma on the [0,1] scale) -> uint8."""
    rng = np.random.default_rng(seed)
    clean = smooth_field(rng, c, h, w)
    return quantise(clean + rng.normal(0.0, sigma, clean.shape))


def gray_batch(seed, n, h=1024, w=1024):
    """Config 3: n gray images, sigma drawn per image from {15, 25, 50}/255."""
    rng = np.random.default_rng(seed)
    out = np.empty((n, 1, h, w), np.uint8)
    for i in range(n):
        sigma = rng.choice([15.0, 25.0, 50.0]) / 255.0
        clean = smooth_field(rng, 1, h, w)
        out[i] = quantise(clean + rng.normal(0.0, sigma, clean.shape))
    return out


def frame(rng, h=1080, w=1920):
    """Config 4 frame: sigma(x) = 5/255 + 20/255 * luma, plus 2x2-block-correlated
    N(0, 5/255)."""
    clean = smooth_field(rng, 3, h, w)
    luma = 0.299 * clean[0] + 0.587 * clean[1] + 0.114 * clean[2]
    sig = 5.0 / 255.0 + 20.0 / 255.0 * luma
    white = rng.normal(0.0, 1.0, clean.shape) * sig[None]
    blk = rng.normal(0.0, 5.0 / 255.0, (3, (h + 1) // 2, (w + 1) // 2))
    blk = np.repeat(np.repeat(blk, 2, axis=1), 2, axis=2)[:, :h, :w]
    return quantise(clean + white + blk)


def frames(seed, n, h=1080, w=1920, distinct=None):
    """Config 4: n frames [n][3][h][w] uint8. With `distinct`, only that many frames
    are generated and the batch cycles through them (the generator is CPU work that
    does not belong to the measured path)."""
    rng = np.random.default_rng(seed)
    k = n if distinct is None else min(n, distinct)
    base = [frame(rng, h, w) for _ in range(k)]
    return np.stack([base[i % k] for i in range(n)])


def frame_at(seed, k, h=1080, w=1920):
    """Frame k of the config-4 batch with seed `seed`, generated on its own (its
    random stream is seeded with (seed, k)), so a test can take any subset of the
    256 frames without generating the ones before it."""
    return frame(np.random.default_rng([seed, k]), h, w)


CONFIGS = {
    1: dict(name="color 64x64", c=3, h=64, w=64, n=1, sigma=25.0 / 255.0),
    2: dict(name="color 512x512", c=3, h=512, w=512, n=1, sigma=15.0 / 255.0),
    3: dict(name="gray 1024x1024 x64", c=1, h=1024, w=1024, n=64),
    4: dict(name="color 1920x1080 x256", c=3, h=1080, w=1920, n=256),
    5: dict(name="color 8192x8192", c=3, h=8192, w=8192, n=1, sigma=25.0 / 255.0),
}


def config_input(cfg, seed=None, distinct=None):
    """uint8 [n][c][h][w] for configuration `cfg` (1..5)."""
    d = CONFIGS[cfg]
    seed = 1000 + cfg if seed is None else seed
    if cfg in (1, 2, 5):
        return noisy_image(seed, d["c"], d["h"], d["w"], d["sigma"])[None]
    if cfg == 3:
        return gray_batch(seed, d["n"] if distinct is None else distinct, d["h"], d["w"])
    return frames(seed, d["n"], d["h"], d["w"], distinct=distinct)
