"""scunet_b200: the SCUNet forward pass on B200 (sm_100a) behind a C ABI.

Import by path (the directory name is not a Python identifier):

    import importlib, sys; sys.path.insert(0, REPO)
    scb = importlib.import_module("scunet-rs_b200")

Modules:
  backend  - the `Backend`-shaped host mirror over `libscunet_b200.so` (ctypes)
  plan     - padded geometry: Plan, pad_replicate, crop, check_min_size
  weights  - tensor table, seeded initialisation, safetensors I/O
  synth    - seeded synthetic inputs for the benchmark configurations
  build    - nvcc build of the library
"""
from . import plan, weights, synth, build, shard  # noqa: F401
from .backend import (B200, BackendError, run, load_library, need_bytes, band_unique_id, SYMBOLS, SCB_F32,  # noqa: F401
                      SCB_U8)
from .plan import Plan  # noqa: F401
from .weights import Weights  # noqa: F401
