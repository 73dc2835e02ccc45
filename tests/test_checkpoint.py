"""Checkpoint files: the writer here produces, byte for byte, the `.safetensors` the
reference's own converter (`tools/convert.py:200-260`) writes for the same weights,
so `Weights.load` (`src/weights.rs:101-185`) reads exactly what a reference user
has. The digest was recorded by `tests/golden/make_checkpoint_pin.py`, which ran
the reference's converter on a torch `.pth` of the same seeded weights (rel-pos
tables as non-contiguous views, as upstream saves them)."""
import hashlib
import json

import numpy as np

from conftest import GOLDEN


def test_writer_matches_reference_converter(scb, tmp_path):
    pin = json.loads((GOLDEN / "checkpoint_pin.json").read_text())
    w = scb.Weights.seeded(3, 0)
    p = tmp_path / "m.safetensors"
    scb.Weights(w.tensors, in_nc=3, variant=pin["variant"]).save(p)
    raw = p.read_bytes()
    assert len(raw) == pin["bytes"]
    assert hashlib.sha256(raw).hexdigest() == pin["sha256"]
    back = scb.Weights.load(p)
    assert back.variant == pin["variant"] and back.in_nc == 3 and back.config == (4,) * 7
    for k, v in w.tensors.items():
        assert np.array_equal(v, back.tensors[k]), k
