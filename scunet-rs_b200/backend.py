"""Host-side mirror of the reference's `Backend` boundary over the C ABI.

`B200` is the device backend behind `include/scunet_b200.h`, shaped like the
reference's `trait Backend` (scunet-rs `src/backend.rs:19-56`): `name()`,
`forward(x, plan)` on an already padded `[c][hp][wp]` plane, `footprint()`,
`release_scratch()`. `run()` is `backend::run` (`src/backend.rs:63-105`): size
check, admission against free device memory, replicate pad, forward, length check,
crop. Errors are `BackendError` carrying the library's message (the reference's
`Result<_, String>`).

There is no CPU fallback: constructing `B200` without the built library, or on a
machine without a B200, raises.
"""
from __future__ import annotations

import ctypes
from pathlib import Path

import numpy as np

from . import plan as _plan

HERE = Path(__file__).resolve().parent
LIB_PATH = HERE / "libscunet_b200.so"

SCB_F32, SCB_U8 = 0, 1
SYMBOLS = [
    "scb_create", "scb_forward", "scb_forward_dev", "scb_forward_host", "scb_need_bytes", "scb_footprint",
    "scb_release_scratch", "scb_last_error", "scb_destroy", "scb_probe_gemm", "scb_probe_conv3x3",
    "scb_probe_down2", "scb_probe_up2", "scb_probe_attention", "scb_probe_block", "scb_last_launch_count",
    "scb_set_profiling", "scb_profile_read", "scb_set_option", "scb_forward_dev_noalloc",
    "scb_forward_bands", "scb_band_unique_id", "scb_band_init", "scb_forward_band", "scb_profile_bytes", "scb_probe_mlp",
    "scb_band_sync", "scb_probe_head", "scb_probe_tail", "scb_probe_wait_timeout", "scb_mem_report",
    "scb_profile_report", "scb_check_admission", "scb_profile_kernels",
]
SCB_OPT_FUSE_TRANS = 1
SCB_OPT_RESIDUAL32 = 2
SCB_OPT_HOST_CHUNK = 3
SCB_OPT_TRANS32_LANES = 4
SCB_OPT_FUSE_PAIR = 5
SCB_OPT_GEMM_PAIRS = 6
SCB_OPT_CONV3_TWIN = 7
OP_CLASSES = ["head", "tail", "conv1x1", "conv3x3", "qkv", "attention", "proj", "mlp0", "mlp2", "down", "up",
              "trans_fused", "halo", "mlp"]


class BackendError(RuntimeError):
    pass


class ScbTensor(ctypes.Structure):
    _fields_ = [("name", ctypes.c_char_p), ("data", ctypes.POINTER(ctypes.c_float)), ("ndim", ctypes.c_int),
                ("shape", ctypes.c_int64 * 4)]


_lib = None


def load_library(path=None):
    """dlopen the C-ABI library and declare every entry point's signature."""
    global _lib
    if _lib is not None and path is None:
        return _lib
    p = Path(path) if path else LIB_PATH
    if not p.exists():
        raise BackendError(f"{p} is not built (python scunet-rs_b200/build.py)")
    lib = ctypes.CDLL(str(p))
    vp, i, sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_size_t
    fp = ctypes.POINTER(ctypes.c_float)
    lib.scb_create.argtypes = [ctypes.POINTER(ScbTensor), i, i, i, i, i, ctypes.POINTER(ctypes.c_int), i,
                               ctypes.POINTER(vp)]
    lib.scb_forward.argtypes = [vp, fp, i, i, i, fp]
    lib.scb_forward_dev.argtypes = [vp, vp, i, i, i, i, i, vp, i, vp]
    lib.scb_forward_host.argtypes = [vp, vp, i, i, i, i, i, vp, i]
    lib.scb_forward_dev_noalloc.argtypes = [vp, vp, i, i, i, i, i, vp, i, vp]
    lib.scb_forward_bands.argtypes = [vp, i, vp, i, i, i, i, vp, i, vp]
    lib.scb_band_unique_id.argtypes = [vp]
    lib.scb_band_init.argtypes = [vp, vp, i, i]
    lib.scb_forward_band.argtypes = [vp, vp, i, i, i, i, vp, i, vp]
    lib.scb_profile_bytes.argtypes = [vp, ctypes.POINTER(ctypes.c_double), i]
    lib.scb_band_sync.argtypes = [vp, vp, i]
    lib.scb_probe_head.argtypes = [vp, vp, i, i, i, i, i, vp, vp]
    lib.scb_probe_tail.argtypes = [vp, vp, i, i, i, i, vp, i]
    lib.scb_probe_wait_timeout.argtypes = [vp, i]
    lib.scb_mem_report.argtypes = [vp, ctypes.POINTER(sz), ctypes.POINTER(sz), ctypes.POINTER(sz)]
    lib.scb_profile_report.argtypes = [vp, ctypes.c_char_p, sz]
    lib.scb_profile_kernels.argtypes = [vp, ctypes.c_char_p, sz]
    lib.scb_check_admission.argtypes = [vp, i, i, i, ctypes.POINTER(sz), ctypes.POINTER(sz)]
    lib.scb_probe_mlp.argtypes = [vp, i, i, vp, vp, i]
    lib.scb_need_bytes.argtypes = [i, i, i, i, ctypes.POINTER(sz)]
    lib.scb_footprint.argtypes = [vp, ctypes.POINTER(sz), ctypes.POINTER(sz)]
    lib.scb_footprint.restype = None
    lib.scb_release_scratch.argtypes = [vp]
    lib.scb_release_scratch.restype = None
    lib.scb_last_error.argtypes = [vp]
    lib.scb_last_error.restype = ctypes.c_char_p
    lib.scb_destroy.argtypes = [vp]
    lib.scb_destroy.restype = None
    lib.scb_last_launch_count.argtypes = [vp]
    lib.scb_probe_gemm.argtypes = [vp, vp, i, i, vp, i, vp, i, vp, vp, vp]
    lib.scb_probe_conv3x3.argtypes = [vp, vp, i, i, i, i, vp, i, i, vp, vp]
    lib.scb_probe_down2.argtypes = [vp, vp, i, i, i, i, vp, i, vp, vp]
    lib.scb_probe_up2.argtypes = [vp, vp, i, i, i, i, vp, i, vp, vp]
    lib.scb_probe_attention.argtypes = [vp, vp, i, i, i, i, i, vp, vp]
    lib.scb_probe_block.argtypes = [vp, i, i, vp, i, i, i, vp]
    lib.scb_set_profiling.argtypes = [vp, i]
    lib.scb_set_option.argtypes = [vp, i, i]
    lib.scb_profile_read.argtypes = [vp, ctypes.POINTER(ctypes.c_int), ctypes.POINTER(ctypes.c_double),
                                     ctypes.POINTER(ctypes.c_float), i]
    if path is None:
        _lib = lib
    return lib


def band_unique_id():
    """A fresh 128-byte NCCL unique id for scb_band_init (rank 0 makes it)."""
    lib = load_library()
    buf = ctypes.create_string_buffer(128)
    if lib.scb_band_unique_id(buf) != 0:
        raise BackendError(f"scb_band_unique_id: {lib.scb_last_error(None).decode()}")
    return buf.raw


def need_bytes(n, in_nc, hp, wp):
    """`memguard::device_need` (`src/memguard.rs:66-74`) for the B200 arena."""
    lib = load_library()
    out = ctypes.c_size_t(0)
    if lib.scb_need_bytes(n, in_nc, hp, wp, ctypes.byref(out)) != 0:
        raise BackendError(f"no arena for {n} x {hp}x{wp}")
    return out.value


class B200:
    """The B200 device backend (`impl Backend`, `src/backend.rs:19-56`)."""

    def __init__(self, weights, device=0):
        self.lib = load_library()
        self.weights = weights
        self.in_nc = weights.in_nc
        self.device = device
        names, self._keep = [], []
        arr = (ScbTensor * len(weights.tensors))()
        for k, (name, a) in enumerate(weights.tensors.items()):
            a = np.ascontiguousarray(a, np.float32)
            self._keep.append(a)
            nm = name.encode()
            names.append(nm)
            arr[k].name = nm
            arr[k].data = a.ctypes.data_as(ctypes.POINTER(ctypes.c_float))
            arr[k].ndim = a.ndim
            for d in range(4):
                arr[k].shape[d] = a.shape[d] if d < a.ndim else 0
        cfg = (ctypes.c_int * 7)(*weights.config)
        ctx = ctypes.c_void_p()
        rc = self.lib.scb_create(arr, len(weights.tensors), weights.in_nc, weights.dim, weights.head_dim,
                                 weights.window, cfg, device, ctypes.byref(ctx))
        self._names = names
        if rc != 0:
            raise BackendError(f"scb_create: {self.lib.scb_last_error(None).decode()}")
        self.ctx = ctx
        self._keep = None  # weights are on the device now
        self.options = {}  # the SCB_OPT_* values set on this context

    # -- the trait ------------------------------------------------------------
    def name(self):
        return "b200"

    def _check(self, rc, what):
        if rc != 0:
            raise BackendError(f"{what}: {self.lib.scb_last_error(self.ctx).decode()}")

    def forward(self, x, plan):
        """`Backend::forward`: padded [c][hp][wp] float32 -> same shape (host arrays)."""
        x = np.ascontiguousarray(x, np.float32).reshape(self.in_nc, plan.hp, plan.wp)
        y = np.empty_like(x)
        fp = ctypes.POINTER(ctypes.c_float)
        self._check(self.lib.scb_forward(self.ctx, x.ctypes.data_as(fp), self.in_nc, plan.hp, plan.wp,
                                         y.ctypes.data_as(fp)), "scb_forward")
        return y

    def footprint(self):
        w, s = ctypes.c_size_t(0), ctypes.c_size_t(0)
        self.lib.scb_footprint(self.ctx, ctypes.byref(w), ctypes.byref(s))
        return w.value, s.value

    def release_scratch(self):
        self.lib.scb_release_scratch(self.ctx)

    def mem_report(self):
        """`Backend::mem_report` (`src/backend.rs:33-44`) as numbers: {high_water, live,
        fixed} device bytes (fixed = the no-allocation array, held since creation)."""
        hw, live, fixed = ctypes.c_size_t(0), ctypes.c_size_t(0), ctypes.c_size_t(0)
        self._check(self.lib.scb_mem_report(self.ctx, ctypes.byref(hw), ctypes.byref(live), ctypes.byref(fixed)),
                    "scb_mem_report")
        return {"high_water": hw.value, "live": live.value, "fixed": fixed.value}

    def profile_report(self):
        """`Backend::profile_report` (`src/backend.rs:33-38`): the last profiled
        forward's device time per op class as text ("" when profiling is off)."""
        n = self.lib.scb_profile_report(self.ctx, None, 0)
        if n <= 0:
            return ""
        buf = ctypes.create_string_buffer(n + 1)
        self.lib.scb_profile_report(self.ctx, buf, n + 1)
        return buf.value.decode()

    # -- batched paths ----------------------------------------------------------
    def forward_host(self, x, out_u8=False):
        """[n][c][h][w] uint8 or float32 host array -> [n][c][h][w] float32 (or uint8
        quantised as the CLI writes PNGs, src/image.rs:60-63); pad and crop fused on
        the device."""
        x = np.ascontiguousarray(x)
        n, c, h, w = x.shape
        xd = SCB_U8 if x.dtype == np.uint8 else SCB_F32
        if xd == SCB_F32:
            x = x.astype(np.float32, copy=False)
        y = np.empty((n, c, h, w), np.uint8 if out_u8 else np.float32)
        self._check(self.lib.scb_forward_host(self.ctx, x.ctypes.data, xd, n, c, h, w, y.ctypes.data,
                                              SCB_U8 if out_u8 else SCB_F32), "scb_forward_host")
        return y

    def forward_dev(self, x_ptr, x_dtype, n, c, h, w, y_ptr, y_dtype, stream=0):
        """Device pointers (e.g. torch tensors' data_ptr()); asynchronous."""
        self._check(self.lib.scb_forward_dev(self.ctx, x_ptr, x_dtype, n, c, h, w, y_ptr, y_dtype, stream or None),
                    "scb_forward_dev")

    def forward_dev_noalloc(self, x_ptr, x_dtype, n, c, h, w, y_ptr, y_dtype, stream=0):
        """Like forward_dev, with the library's fixed device scratch instead of an
        allocation (padded batch of at most 8192 pixels)."""
        self._check(self.lib.scb_forward_dev_noalloc(self.ctx, x_ptr, x_dtype, n, c, h, w, y_ptr, y_dtype,
                                                     stream or None), "scb_forward_dev_noalloc")

    # -- one large image in row bands (config 5) ---------------------------------
    def forward_bands(self, nbands, x_ptr, x_dtype, c, h, w, y_ptr, y_dtype, stream=0):
        """All bands on this GPU in lockstep (device pointers, one image)."""
        self._check(self.lib.scb_forward_bands(self.ctx, nbands, x_ptr, x_dtype, c, h, w, y_ptr, y_dtype,
                                               stream or None), "scb_forward_bands")

    def band_init(self, uid, rank, nranks):
        """Join a band group (collective over the ranks); `uid` from band_unique_id()."""
        buf = ctypes.create_string_buffer(bytes(uid), 128)
        self._check(self.lib.scb_band_init(self.ctx, buf, rank, nranks), "scb_band_init")

    def forward_band(self, x_ptr, x_dtype, c, h, w, y_ptr, y_dtype, stream=0):
        """This rank's band of the full image x; writes its rows of y."""
        self._check(self.lib.scb_forward_band(self.ctx, x_ptr, x_dtype, c, h, w, y_ptr, y_dtype, stream or None),
                    "scb_forward_band")

    def band_sync(self, timeout_ms, stream=0):
        """Wait for the banded forward on `stream` with a deadline; a failed peer or
        the deadline aborts the band group and raises."""
        self._check(self.lib.scb_band_sync(self.ctx, stream or None, int(timeout_ms)), "scb_band_sync")

    def set_option(self, option, value):
        self._check(self.lib.scb_set_option(self.ctx, option, int(value)), "scb_set_option")
        self.options[option] = int(value)

    def set_profiling(self, on):
        self._check(self.lib.scb_set_profiling(self.ctx, int(bool(on))), "scb_set_profiling")

    def profile(self, max_ops=4096):
        """[(class, flops, bytes, ms)] for every launch of the last profiled forward:
        algorithmic FLOPs and HBM bytes, device time."""
        tags = (ctypes.c_int * max_ops)()
        flops = (ctypes.c_double * max_ops)()
        nbytes = (ctypes.c_double * max_ops)()
        ms = (ctypes.c_float * max_ops)()
        n = self.lib.scb_profile_read(self.ctx, tags, flops, ms, max_ops)
        self.lib.scb_profile_bytes(self.ctx, nbytes, max_ops)
        return [(OP_CLASSES[tags[k]], flops[k], nbytes[k], ms[k]) for k in range(n)]

    def profile_kernels(self):
        """The kernel each launch of the last profiled forward ran (profiler names)."""
        n = self.lib.scb_profile_kernels(self.ctx, None, 0)
        buf = ctypes.create_string_buffer(max(n, 0) + 1)
        self.lib.scb_profile_kernels(self.ctx, buf, n + 1)
        return buf.value.decode().splitlines()

    def last_launch_count(self):
        return self.lib.scb_last_launch_count(self.ctx)

    def close(self):
        if getattr(self, "ctx", None):
            self.lib.scb_destroy(self.ctx)
            self.ctx = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def run(be, x, c, h, w, wt):
    """`backend::run` (`src/backend.rs:63-105`): min-size check, admission, replicate
    pad, forward, length check, crop. x is [c][h][w] float32 in [0,1]."""
    p = _plan.Plan.new(h, w, wt.window)
    _plan.check_min_size(h, w, wt.window)
    if be.name() == "b200":
        check_b200(be, p)
    padded = _plan.pad_replicate(x, c, h, w, p.hp, p.wp)
    y = be.forward(padded, p)
    if y.size != c * p.plane():
        raise BackendError(f"{be.name()}: the backend returned {y.size} floats for a {p.hp}x{p.wp} plane of {c} "
                           f"channels")
    return _plan.crop(y, c, h, w, p.hp, p.wp)


def check_b200(be, p, n=1):
    """`memguard::check_cuda` (`src/memguard.rs:262-285`) through the library's own
    admission (`scb_check_admission`): refuse before allocating when the arena would
    not fit in free device memory; fail open when the free figure cannot be read."""
    need, avail = ctypes.c_size_t(0), ctypes.c_size_t(0)
    rc = be.lib.scb_check_admission(be.ctx, n, p.hp, p.wp, ctypes.byref(need), ctypes.byref(avail))
    if rc != 0:
        raise BackendError(f"{p.h}x{p.w}: {be.lib.scb_last_error(be.ctx).decode()}")
