"""The C ABI on CPU: the library loads, exports every symbol the header declares,
and its host-side validation (weight names/shapes, geometry, admission arithmetic)
answers without a GPU."""
import ctypes
import re

import numpy as np
import pytest

from conftest import ROOT


def header_symbols():
    text = (ROOT / "include" / "scunet_b200.h").read_text()
    return sorted(set(re.findall(r"\b(scb_[a-z0-9_]+)\s*\(", text)))


def test_header_and_library_agree(scb):
    lib = scb.load_library()
    declared = header_symbols()
    assert len(declared) >= 15
    missing = [s for s in declared if not hasattr(lib, s)]
    assert not missing, missing
    assert sorted(scb.SYMBOLS) == declared


def _tensor_array(scb, tensors):
    arr = (scb.backend.ScbTensor * len(tensors))()
    keep = []
    for k, (name, a) in enumerate(tensors.items()):
        a = np.ascontiguousarray(a, np.float32)
        keep.append((name.encode(), a))
        arr[k].name = keep[-1][0]
        arr[k].data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
        arr[k].ndim = a.ndim
        for d in range(4):
            arr[k].shape[d] = a.shape[d] if d < a.ndim else 0
    return arr, keep


def _create(scb, tensors, in_nc=3, dim=64):
    lib = scb.load_library()
    arr, keep = _tensor_array(scb, tensors)
    ctx = ctypes.c_void_p()
    cfg = (ctypes.c_int * 7)(*([4] * 7))
    rc = lib.scb_create(arr, len(tensors), in_nc, dim, 32, 8, cfg, 0, ctypes.byref(ctx))
    return rc, lib.scb_last_error(None).decode(), ctx


def test_create_rejects_missing_tensor(scb):
    t = dict(scb.weights.seeded(3, 0))
    del t["m_up2.3.trans_block.mlp.0.bias"]
    rc, msg, ctx = _create(scb, t)
    assert rc == -2 and "m_up2.3.trans_block.mlp.0.bias" in msg and not ctx.value


def test_create_rejects_bad_shape(scb):
    t = dict(scb.weights.seeded(3, 0))
    t["m_down2.1.trans_block.msa.relative_position_params"] = np.zeros((1, 15, 15), np.float32)
    rc, msg, _ = _create(scb, t)
    assert rc == -2 and "relative_position_params" in msg and "dim 0" in msg


def test_create_rejects_bad_arch(scb):
    t = dict(scb.weights.seeded(3, 0))
    rc, msg, _ = _create(scb, t, in_nc=2)
    assert rc == -1 and "in_nc" in msg
    rc, msg, _ = _create(scb, t, dim=96)
    assert rc == -1 and "dim 64" in msg


def test_create_without_device_fails_loudly(scb):
    """No CPU fallback: with valid weights and no usable B200 the call fails with the
    CUDA runtime's reason (on a GPU box this test is skipped)."""
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a GPU is present")
    except Exception:
        pass
    rc, msg, ctx = _create(scb, dict(scb.weights.seeded(3, 0)))
    assert rc == -3 and msg and not ctx.value


def test_need_bytes(scb):
    a = scb.need_bytes(1, 3, 1088, 1920)
    b = scb.need_bytes(2, 3, 1088, 1920)
    assert 1.0e3 < a / (1088 * 1920) < 1.4e3      # ~1.16 KB per padded pixel (default options)
    assert abs(b - 2 * a) < 64 * 1024
    with pytest.raises(Exception):
        scb.need_bytes(1, 3, 100, 64)             # not padded


def test_null_context_calls_are_errors(scb):
    lib = scb.load_library()
    assert lib.scb_forward(None, None, 3, 64, 64, None) == -1
    assert lib.scb_forward_dev(None, None, 0, 1, 3, 64, 64, None, 0, None) == -1
    lib.scb_destroy(None)
    lib.scb_release_scratch(None)
    assert lib.scb_last_launch_count(None) == 0
