"""Shared fixtures. GPU tests are marked `gpu`; everything else runs on CPU."""
import importlib
import struct
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden"
sys.path.insert(0, str(ROOT))
sys.path.insert(0, str(ROOT / "oracle"))


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a B200 and the built library")


@pytest.fixture(scope="session")
def scb():
    return importlib.import_module("scunet-rs_b200")


@pytest.fixture(scope="session")
def oracle():
    import scunet_np
    return scunet_np


def load_scuf(path):
    """SCUF v1 (`src/fixture.rs:36-75`): magic, version, h, w, c, win, variant, in, out."""
    b = Path(path).read_bytes()
    assert b[:4] == b"SCUF", path
    ver, h, w, c, win, vlen = struct.unpack("<IIIIII", b[4:28])
    assert ver == 1
    variant = b[28:28 + vlen].decode()
    off = 28 + vlen
    n = h * w * c
    assert len(b) == off + 8 * n, "truncated fixture"
    x = np.frombuffer(b, "<f4", n, off).reshape(1, c, h, w)
    y = np.frombuffer(b, "<f4", n, off + 4 * n).reshape(1, c, h, w)
    return dict(h=h, w=w, c=c, win=win, variant=variant, x=x.copy(), y=y.copy())


@pytest.fixture(scope="session")
def goldens():
    return {p.stem: load_scuf(p) for p in sorted(GOLDEN.glob("*.scuf"))}


@pytest.fixture(scope="session")
def weights3(scb):
    return scb.Weights.seeded(3, 0)


@pytest.fixture(scope="session")
def weights1(scb):
    return scb.Weights.seeded(1, 0)


@pytest.fixture(scope="session")
def be3(scb, weights3):
    be = scb.B200(weights3)
    yield be
    be.close()


@pytest.fixture(scope="session")
def be1(scb, weights1):
    be = scb.B200(weights1)
    yield be
    be.close()
