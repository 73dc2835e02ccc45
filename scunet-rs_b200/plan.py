"""Padded geometry of one forward pass: the host mirror of `src/plan.rs`.

SCUNet replicate-pads the input to the next multiple of 64 (window 8 times the
three stride-2 stages), runs one whole-plane pass and crops (`src/plan.rs:1-22`).
Padding by replication (edge clamp) makes one padded pass exact at any size, so
there is no tile loop anywhere on this path.
"""
from __future__ import annotations

from dataclasses import dataclass

import numpy as np

PAD_TO = 64  # `src/plan.rs:40`


@dataclass(frozen=True)
class Plan:
    """`Plan` (`src/plan.rs:26-58`)."""
    h: int
    w: int
    hp: int
    wp: int
    win: int = 8

    @classmethod
    def new(cls, h, w, win=8):
        return cls(h, w, -(-h // PAD_TO) * PAD_TO, -(-w // PAD_TO) * PAD_TO, win)

    def plane(self):
        return self.hp * self.wp

    def windows(self, dn):
        return ((self.hp >> dn) // self.win, (self.wp >> dn) // self.win)


def check_min_size(h, w, win=8):
    """`check_min_size` (`src/plan.rs:105-118`): the 1/8 body needs one window."""
    hp = -(-h // PAD_TO) * PAD_TO
    wp = -(-w // PAD_TO) * PAD_TO
    if hp < 8 * win or wp < 8 * win:
        raise ValueError(f"{h}x{w} pads to {hp}x{wp}, but the 1/8-resolution body needs at "
                         f"least {win}x{win} pixels there")
    if h <= 0 or w <= 0:
        raise ValueError(f"{h}x{w}: empty image")


def pad_replicate(x, c, h, w, hp, wp):
    """`pad_replicate` (`src/plan.rs:67-82`): [c][h][w] -> [c][hp][wp], edge clamp on
    the bottom and right."""
    x = np.asarray(x, np.float32).reshape(c, h, w)
    return np.pad(x, ((0, 0), (0, hp - h), (0, wp - w)), mode="edge")


def crop(y, c, h, w, hp, wp):
    """`crop` (`src/plan.rs:85-94`)."""
    return np.ascontiguousarray(np.asarray(y).reshape(c, hp, wp)[:, :h, :w])
