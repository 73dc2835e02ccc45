"""Generate the committed golden fixtures and pin the oracle to the reference.

Run in a container that has the reference checked out (it is not needed anywhere
else, and nothing at test or bench time reads it):

    python tests/golden/make_golden.py --reference <path to scunet-rs>

For each case it builds the seeded weights (`scunet-rs_b200/weights.py`), a seeded
uint8 input (`scunet-rs_b200/synth.py`), and runs three implementations of the
same forward pass on CPU in float32:

1. the upstream torch module the reference vendors (`tools/network_scunet.py`),
   built with `input_resolution=256` so that no stage loses its shifted windows
   (the trap `tools/compare.py:86-98` records);
2. the reference's own numpy SCUNet (`tools/reference.py`), given the same weights;
3. this repository's oracle (`oracle/scunet_np.py`).

The fixture's expected output is (1); the manifest records the max |diff| of (2)
and (3) against it, and a digest of the weights so a drifting generator is caught.
Fixtures use the reference's SCUF v1 container (`src/fixture.rs:1-75`,
`tools/make_fixture.py:1-20`): magic, version, h, w, c, win, variant, input f32
NCHW, output f32 NCHW.
"""
from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import struct
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT / "scunet-rs_b200"))
sys.path.insert(0, str(ROOT / "oracle"))
import weights as W  # noqa: E402
import synth  # noqa: E402
import scunet_np  # noqa: E402

# (file stem, in_nc, h, w, seed, sigma): the two reference fixture geometries
# (80x64 pads rows, 64x64 does not; `tools/reference.py:378-393`) plus a case that
# pads both axes, a grayscale case and one with several windows at every stage.
CASES = [
    ("color_64x64", 3, 64, 64, 11, 25 / 255),
    ("color_80x64", 3, 80, 64, 12, 25 / 255),
    ("color_72x40", 3, 72, 40, 13, 15 / 255),
    ("gray_64x64", 1, 64, 64, 14, 50 / 255),
    ("color_128x128", 3, 128, 128, 15, 15 / 255),
]
WEIGHT_SEED = 0


def weights_digest(w):
    h = hashlib.sha256()
    for k in sorted(w):
        h.update(k.encode())
        h.update(np.ascontiguousarray(w[k], "<f4").tobytes())
    return h.hexdigest()


def write_scuf(path, x, y, variant, win=8):
    _, c, h, w = x.shape
    v = variant.encode()
    with open(path, "wb") as f:
        f.write(b"SCUF")
        f.write(struct.pack("<IIIIII", 1, h, w, c, win, len(v)))
        f.write(v)
        f.write(np.ascontiguousarray(x, "<f4").tobytes())
        f.write(np.ascontiguousarray(y, "<f4").tobytes())


def load_module(name, path):
    spec = importlib.util.spec_from_file_location(name, path)
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="root of the scunet-rs checkout")
    args = ap.parse_args()
    ref = Path(args.reference)
    sys.path.insert(0, str(ref / "tools"))
    import torch
    torch.set_num_threads(8)
    ns = load_module("network_scunet", ref / "tools" / "network_scunet.py")
    rp = load_module("reference_np", ref / "tools" / "reference.py")

    manifest = {"weights_seed": WEIGHT_SEED, "cases": {}, "weights": {}}
    for in_nc in (1, 3):
        wt = W.seeded(in_nc, WEIGHT_SEED)
        manifest["weights"][str(in_nc)] = {"sha256": weights_digest(wt),
                                           "sum": float(sum(float(a.astype(np.float64).sum()) for a in wt.values()))}
    for stem, in_nc, h, w, seed, sigma in CASES:
        wt = W.seeded(in_nc, WEIGHT_SEED)
        x = synth.noisy_image(seed, in_nc, h, w, sigma).astype(np.float32)[None] / 255.0
        net = ns.SCUNet(in_nc=in_nc, config=[4] * 7, dim=64, input_resolution=256).eval()
        sd = net.state_dict()
        assert set(sd) == set(wt), sorted(set(sd) ^ set(wt))
        with torch.no_grad():
            for k, v in sd.items():
                assert tuple(v.shape) == wt[k].shape, (k, v.shape, wt[k].shape)
                v.copy_(torch.from_numpy(wt[k]))
            t0 = time.time()
            y_t = net(torch.from_numpy(x)).numpy()
            t_torch = time.time() - t0
        meta = W.metadata(in_nc)
        y_r = rp.SCUNet(dict(wt), meta).forward(x.copy())
        t0 = time.time()
        y_o = scunet_np.forward(x, wt)
        t_or = time.time() - t0
        d_ref = float(np.abs(y_r - y_t).max())
        d_or = float(np.abs(y_o - y_t).max())
        d_or_ref = float(np.abs(y_o - y_r).max())
        print(f"{stem}: torch {t_torch:.2f}s oracle {t_or:.2f}s | max|ref.py - torch| {d_ref:.3e} "
              f"max|oracle - torch| {d_or:.3e} max|oracle - ref.py| {d_or_ref:.3e}")
        assert d_ref < 1e-4 and d_or < 1e-4 and d_or_ref < 1e-4, stem
        write_scuf(HERE / f"{stem}.scuf", x, y_t, f"in{in_nc}-seeded-{WEIGHT_SEED}")
        manifest["cases"][stem] = {
            "in_nc": in_nc, "h": h, "w": w, "input_seed": seed, "sigma": sigma,
            "max_abs_reference_py_vs_torch": d_ref, "max_abs_oracle_vs_torch": d_or,
            "max_abs_oracle_vs_reference_py": d_or_ref,
            "out_min": float(y_t.min()), "out_max": float(y_t.max()),
        }
    (HERE / "manifest.json").write_text(json.dumps(manifest, indent=1) + "\n")
    print("wrote", HERE / "manifest.json")


if __name__ == "__main__":
    main()
