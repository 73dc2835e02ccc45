"""SCUNet checkpoints: the tensor table, seeded initialisation and safetensors I/O.

The tensor names and shapes are the ones the reference validates in
`src/weights.rs:204-280` (scunet-rs) and that upstream `SCUNet.__init__` creates
(`tools/network_scunet.py:181-237`). The safetensors `__metadata__` keys are the
ones `tools/convert.py:227-236` writes and `src/weights.rs:117-164` reads back.

Seeded weights follow upstream torch's default initialisation *distributions*
(not its random stream), which is the initialisation the benchmark configs name:

* Conv2d / Linear / ConvTranspose2d weights: kaiming-uniform with a = sqrt(5), i.e.
  U(-1/sqrt(fan_in), 1/sqrt(fan_in)); fan_in is `weight.shape[1] * kh * kw`, which for
  a ConvTranspose2d (`[c_in][c_out][kh][kw]`) is `c_out * kh * kw`, as torch computes it.
* biases: U(-1/sqrt(fan_in), 1/sqrt(fan_in)).
* relative-position tables: normal(0, 0.02) clamped to +-2 sigma, the
  `trunc_normal_` of `tools/timm_shim.py:33-36`.
* LayerNorm: gamma = 1, beta = 0.

The generator is numpy's PCG64 (`default_rng(seed)`) walked in one fixed order
(`tensor_table`), so the same seed gives the same bytes on every machine.
"""
from __future__ import annotations

import json
import struct
from collections import OrderedDict

import numpy as np

DIM = 64
HEAD_DIM = 32
WINDOW = 8
CONFIG = (4, 4, 4, 4, 4, 4, 4)
STAGES = ("down1", "down2", "down3", "body", "up3", "up2", "up1")
# Channel count of each stage's plane, as a multiple of `dim` (upstream
# `tools/network_scunet.py:194-225`: 64, 128, 256, 512, 256, 128, 64).
STAGE_MULT = {"down1": 1, "down2": 2, "down3": 4, "body": 8, "up3": 4, "up2": 2, "up1": 1}
VARIANTS = {
    "color-15": 3, "color-25": 3, "color-50": 3, "color-real-psnr": 3, "color-real-gan": 3,
    "gray-15": 1, "gray-25": 1, "gray-50": 1,
}


def block_prefixes(stage, count=4):
    """The ConvTransBlock prefixes of one stage. Up stages hold their transposed
    conv at index 0, so their blocks are 1..count (`tools/network_scunet.py:213-225`)."""
    first = 1 if stage.startswith("up") else 0
    return [f"m_{stage}.{first + i}" for i in range(count)]


def block_table(prefix, c):
    """Tensors of one ConvTransBlock whose plane has `c` channels (c/2 conv, c/2 trans)."""
    t = c // 2
    heads = t // HEAD_DIM
    tb = prefix + ".trans_block"
    return [
        (tb + ".ln1.weight", (t,), "ln_w"),
        (tb + ".ln1.bias", (t,), "ln_b"),
        (tb + ".msa.relative_position_params", (heads, 2 * WINDOW - 1, 2 * WINDOW - 1), "relpos"),
        (tb + ".msa.embedding_layer.weight", (3 * t, t), "w"),
        (tb + ".msa.embedding_layer.bias", (3 * t,), ("b", t)),
        (tb + ".msa.linear.weight", (t, t), "w"),
        (tb + ".msa.linear.bias", (t,), ("b", t)),
        (tb + ".ln2.weight", (t,), "ln_w"),
        (tb + ".ln2.bias", (t,), "ln_b"),
        (tb + ".mlp.0.weight", (4 * t, t), "w"),
        (tb + ".mlp.0.bias", (4 * t,), ("b", t)),
        (tb + ".mlp.2.weight", (t, 4 * t), "w"),
        (tb + ".mlp.2.bias", (t,), ("b", 4 * t)),
        (prefix + ".conv1_1.weight", (c, c, 1, 1), "w"),
        (prefix + ".conv1_1.bias", (c,), ("b", c)),
        (prefix + ".conv1_2.weight", (c, c, 1, 1), "w"),
        (prefix + ".conv1_2.bias", (c,), ("b", c)),
        (prefix + ".conv_block.0.weight", (t, t, 3, 3), "w"),
        (prefix + ".conv_block.2.weight", (t, t, 3, 3), "w"),
    ]


def tensor_table(in_nc=3, dim=DIM, config=CONFIG):
    """Every tensor of the network as (name, shape, init), in a fixed order."""
    tab = [("m_head.0.weight", (dim, in_nc, 3, 3), "w")]
    for si, stage in enumerate(STAGES):
        c = dim * STAGE_MULT[stage]
        if stage.startswith("up"):
            # ConvTranspose2d(2c, c, 2, 2): weight [c_in][c_out][2][2].
            tab.append((f"m_{stage}.0.weight", (2 * c, c, 2, 2), "wT"))
        for p in block_prefixes(stage, config[si]):
            tab.extend(block_table(p, c))
        if stage.startswith("down"):
            tab.append((f"m_{stage}.{config[si]}.weight", (2 * c, c, 2, 2), "w"))
    tab.append(("m_tail.0.weight", (in_nc, dim, 3, 3), "w"))
    return tab


def seeded(in_nc=3, seed=0, dim=DIM, config=CONFIG):
    """A full seeded weight set {name: float32 array} (see module docstring)."""
    rng = np.random.default_rng(seed)
    out = OrderedDict()
    for name, shape, kind in tensor_table(in_nc, dim, config):
        if kind == "w":
            fan_in = int(np.prod(shape[1:]))
            bound = 1.0 / np.sqrt(fan_in)
            a = rng.uniform(-bound, bound, shape)
        elif kind == "wT":
            fan_in = int(shape[1] * np.prod(shape[2:]))
            bound = 1.0 / np.sqrt(fan_in)
            a = rng.uniform(-bound, bound, shape)
        elif isinstance(kind, tuple):  # bias, with the fan_in of its layer
            bound = 1.0 / np.sqrt(kind[1])
            a = rng.uniform(-bound, bound, shape)
        elif kind == "relpos":
            a = np.clip(rng.normal(0.0, 0.02, shape), -0.04, 0.04)
        elif kind == "ln_w":
            a = np.ones(shape)
        elif kind == "ln_b":
            a = np.zeros(shape)
        else:
            raise ValueError(kind)
        out[name] = np.ascontiguousarray(a, dtype=np.float32)
    return out


def metadata(in_nc=3, variant=None, dim=DIM, config=CONFIG):
    """The `__metadata__` map `tools/convert.py:227-236` writes."""
    if variant is None:
        variant = f"in{in_nc}-seeded"
    return {
        "format": "pt", "arch": "scunet", "variant": variant, "in_nc": str(in_nc),
        "dim": str(dim), "config": ",".join(str(v) for v in config),
        "head_dim": str(HEAD_DIM), "window_size": str(WINDOW),
    }


def save_safetensors(path, tensors, meta):
    """Write {name: f32 array} with `meta` as `__metadata__` (8-byte aligned data)."""
    header, offset, blobs = {}, 0, []
    for name in sorted(tensors):
        arr = np.ascontiguousarray(tensors[name], dtype="<f4")
        n = arr.nbytes
        header[name] = {"dtype": "F32", "shape": list(arr.shape), "data_offsets": [offset, offset + n]}
        blobs.append((offset, arr.tobytes()))
        offset += (n + 7) & ~7
    header["__metadata__"] = dict(meta)
    hj = json.dumps(header, separators=(",", ":")).encode()
    hj += b" " * ((-(8 + len(hj))) & 7)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hj)))
        f.write(hj)
        pos = 0
        for off, raw in blobs:
            if pos < off:
                f.write(b"\0" * (off - pos))
                pos = off
            f.write(raw)
            pos += len(raw)


def load_safetensors(path):
    """Read a safetensors file -> ({name: f32 array}, metadata). F32/F16/BF16 inputs
    are widened to float32 (the checkpoints the reference ships are F32)."""
    with open(path, "rb") as f:
        n = struct.unpack("<Q", f.read(8))[0]
        header = json.loads(f.read(n))
        blob = f.read()
    meta = header.pop("__metadata__", {})
    out = OrderedDict()
    for name, info in header.items():
        a, b = info["data_offsets"]
        dt = info["dtype"]
        raw = blob[a:b]
        if dt == "F32":
            arr = np.frombuffer(raw, "<f4")
        elif dt == "F16":
            arr = np.frombuffer(raw, "<f2").astype(np.float32)
        elif dt == "BF16":
            arr = (np.frombuffer(raw, "<u2").astype(np.uint32) << 16).view(np.float32)
        else:
            raise ValueError(f"{path}: {name}: unsupported dtype {dt}")
        out[name] = np.ascontiguousarray(arr.reshape(info["shape"]), dtype=np.float32)
    return out, meta


class Weights:
    """A validated weight set: the Python side of the reference's `Weights`
    (`src/weights.rs:84-200`). Architecture scalars come from the metadata (or the
    caller) and every tensor's shape is checked against the table, so a checkpoint
    of the wrong family fails here naming the tensor."""

    def __init__(self, tensors, in_nc=None, dim=DIM, config=CONFIG, head_dim=HEAD_DIM,
                 window=WINDOW, variant=None):
        if in_nc is None:
            in_nc = int(tensors["m_head.0.weight"].shape[1])
        if head_dim != HEAD_DIM or window != WINDOW:
            raise ValueError(f"head_dim {head_dim} / window {window}: only 32 / 8 exist")
        if in_nc not in (1, 3):
            raise ValueError(f"in_nc {in_nc}: SCUNet is 1 or 3")
        self.in_nc, self.dim, self.config = in_nc, dim, tuple(config)
        self.head_dim, self.window, self.variant = head_dim, window, variant
        want = {n: s for n, s, _ in tensor_table(in_nc, dim, self.config)}
        for n, s in want.items():
            if n not in tensors:
                raise ValueError(f"missing tensor {n}")
            if tuple(tensors[n].shape) != tuple(s):
                raise ValueError(f"{n}: shape {tuple(tensors[n].shape)}, expected {tuple(s)}")
        self.tensors = OrderedDict((n, np.ascontiguousarray(tensors[n], dtype=np.float32)) for n in want)

    @classmethod
    def seeded(cls, in_nc=3, seed=0):
        return cls(seeded(in_nc, seed), in_nc=in_nc, variant=f"in{in_nc}-seeded")

    @classmethod
    def load(cls, path):
        """`Weights::load` (`src/weights.rs:101-185`): metadata first, then shapes."""
        tensors, meta = load_safetensors(path)
        for k in ("arch", "variant", "in_nc", "dim", "config", "head_dim", "window_size"):
            if k not in meta:
                raise ValueError(f"{path}: no `{k}` in __metadata__")
        if meta["arch"] != "scunet":
            raise ValueError(f"{path}: arch `{meta['arch']}` is not scunet")
        cfg = tuple(int(v) for v in meta["config"].split(","))
        if len(cfg) != 7:
            raise ValueError(f"{path}: config has {len(cfg)} entries, want 7")
        return cls(tensors, in_nc=int(meta["in_nc"]), dim=int(meta["dim"]), config=cfg,
                   head_dim=int(meta["head_dim"]), window=int(meta["window_size"]),
                   variant=meta["variant"])

    def t(self, name):
        return self.tensors[name]

    def save(self, path):
        save_safetensors(path, self.tensors, metadata(self.in_nc, self.variant, self.dim, self.config))

    def nbytes(self):
        return sum(a.nbytes for a in self.tensors.values())


def flops_per_pixel(in_nc=3, dim=DIM):
    """Algorithmic FLOPs per padded full-resolution pixel (2 per multiply-add).

    Counts every conv, linear and the two attention products (QK^T and PV over the
    64 keys of a window) once; m_head is counted once (the reference recomputes
    it, which is not algorithmic work). 2,403,072 for colour, 2,398,464 for gray."""
    mac = 0.0
    for stage in STAGES:
        c = dim * STAGE_MULT[stage]
        px = 1.0 / (STAGE_MULT[stage] ** 2)          # stage pixels per full-res pixel
        t = c // 2
        per_block = 2 * c * c + 2 * 9 * t * t + (3 + 1 + 4 + 4) * t * t + 2 * 64 * t
        mac += 4 * per_block * px
        if stage.startswith("down"):
            mac += (2 * c) * c * 4 * px / 4            # 2x2 s2: out px = px/4, K = 4c, N = 2c
        if stage.startswith("up"):
            mac += (2 * c) * c * 4 * (px / 4)          # convT: in px = px/4, K = 2c, N = 4c
    mac += 9 * in_nc * dim * 2                        # m_head + m_tail
    return 2.0 * mac
