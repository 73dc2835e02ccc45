"""Pin this repository's checkpoint writer to the reference's converter.

Run where the reference is checked out (nothing at test time reads it):

    python tests/golden/make_checkpoint_pin.py --reference <path to scunet-rs>

It writes the seeded colour weights (`scunet-rs_b200/weights.py`, seed 0) as a
torch `.pth` state_dict the way upstream SCUNet saves one - each
`relative_position_params` a non-contiguous view over a `[15][15][heads]` storage,
as `WMSA.__init__` builds it (`tools/network_scunet.py:46-47`) - under the
published file name `scunet_color_15.pth`, converts it with the reference's own
`tools/convert.py`, and records the SHA-256 of the resulting `.safetensors` file in
`checkpoint_pin.json`, after checking that

* `Weights.load` of that file gives tensors bit-identical to the seeded ones, and
* `Weights.save` of the seeded weights (variant `color-15`) writes the identical
  bytes.

`tests/test_checkpoint.py` then re-checks the second point against the recorded
digest without the reference: the writer here and the reference's converter
produce the same file.
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import subprocess
import sys
import tempfile
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
sys.path.insert(0, str(ROOT))

SEED, IN_NC, VARIANT, PTH_NAME = 0, 3, "color-15", "scunet_color_15.pth"


def sha256(path):
    return hashlib.sha256(Path(path).read_bytes()).hexdigest()


def save_pth(tensors, path):
    """torch.save of a state_dict whose rel-pos tables are views, like upstream's."""
    import torch
    sd = {}
    for name, a in tensors.items():
        t = torch.from_numpy(np.ascontiguousarray(a))
        if name.endswith("relative_position_params"):
            # storage [15][15][heads], exposed as [heads][15][15]
            store = torch.from_numpy(np.ascontiguousarray(a.transpose(1, 2, 0)))
            t = store.permute(2, 0, 1)
            assert a.shape[0] == 1 or not t.is_contiguous()
        sd[name] = t
    torch.save(sd, path)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path to the scunet-rs checkout")
    a = ap.parse_args()
    import importlib
    scb = importlib.import_module("scunet-rs_b200")
    conv = Path(a.reference) / "tools" / "convert.py"
    w = scb.Weights.seeded(IN_NC, SEED)
    with tempfile.TemporaryDirectory() as d:
        pth = Path(d) / PTH_NAME
        ref_out = Path(d) / "ref.safetensors"
        ours = Path(d) / "ours.safetensors"
        save_pth(w.tensors, pth)
        r = subprocess.run([sys.executable, str(conv), str(pth), str(ref_out)], capture_output=True, text=True)
        if r.returncode:
            raise SystemExit(f"convert.py failed:\n{r.stdout}\n{r.stderr}")
        loaded = scb.Weights.load(ref_out)
        assert loaded.variant == VARIANT and loaded.in_nc == IN_NC
        for k, v in w.tensors.items():
            assert np.array_equal(v, loaded.tensors[k]), k
        scb.Weights(w.tensors, in_nc=IN_NC, variant=VARIANT).save(ours)
        assert sha256(ours) == sha256(ref_out), "Weights.save differs from tools/convert.py"
        pin = {"reference_tool": "tools/convert.py", "weights": f"Weights.seeded({IN_NC}, {SEED})",
               "pth_name": PTH_NAME, "variant": VARIANT, "bytes": os.path.getsize(ref_out),
               "sha256": sha256(ref_out), "convert_stdout": r.stdout.strip()}
    (HERE / "checkpoint_pin.json").write_text(json.dumps(pin, indent=1) + "\n")
    print(json.dumps(pin, indent=1))


if __name__ == "__main__":
    main()
