"""Window attention against the reference's own CUDA kernel.

`sc_window_attn_r64` (scunet-rs `cuda/scunet.cu:618-625`, launched as
`src/cuda.rs:795-800` does) is built from the reference's source by `oracle/Makefile`
into `oracle/_ref/`. On the same fp16-representable q/k/v and the same rel-pos table
it must agree with the numpy oracle (FP32 vs FP32) and with this library's
window_attn_kernel (fp16 operands and P, fp32 accumulation), for W and SW windows,
1 to 8 heads, and a window offset w0 that places the SW mask."""
import ctypes
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

REF_LIB = Path(__file__).resolve().parent.parent / "oracle" / "_ref" / "libscunet_ref.so"


def _ref():
    if not REF_LIB.exists():
        pytest.skip("reference kernels not built (make -C oracle REF=<scunet-rs checkout>)")
    lib = ctypes.CDLL(str(REF_LIB))
    vp, i = ctypes.c_void_p, ctypes.c_int
    lib.ref_window_attn_r64.argtypes = [vp, vp, vp, i, i, i, i, i, i, i, vp]
    return lib


def _close(want, got, tol):
    scale = max(float(np.abs(want).max()), 1e-6)
    d = float(np.abs(want - got).max())
    return d / scale, d <= tol * scale


@pytest.mark.parametrize("H,W,t,shift", [(32, 48, 128, 0), (32, 48, 128, 4), (24, 40, 64, 4), (16, 16, 256, 4),
                                         (8, 64, 32, 4)])
def test_attention_vs_reference_kernel(be3, oracle, H, W, t, shift):
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = _ref()
    rng = np.random.default_rng(H * W + t + shift)
    heads = t // 32
    qkv = rng.standard_normal((H, W, 3 * t)).astype(np.float16)
    rp = (rng.standard_normal((heads, 15, 15)) * 0.5).astype(np.float32)
    tok = oracle.window_tokens(qkv.astype(np.float32), shift)          # [nw][64][3t]
    nw = tok.shape[0]
    want = oracle.window_untokens(oracle.attention_core(tok, rp, H // 8, W // 8, shift > 0), H, W, shift)

    # the reference's kernel, FP32 in and out, tokens in window order
    tt = torch.from_numpy(np.ascontiguousarray(tok.reshape(nw * 64, 3 * t))).cuda()
    trp = torch.from_numpy(rp).cuda()
    tout = torch.empty((nw * 64, t), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    torch.cuda.synchronize()
    rc = lib.ref_window_attn_r64(tt.data_ptr(), trp.data_ptr(), tout.data_ptr(), nw, W // 8, H, W, heads, shift, 0,
                                 s.cuda_stream)
    assert rc == 0, f"reference launch failed ({rc})"
    s.synchronize()
    ref = oracle.window_untokens(tout.cpu().numpy().reshape(nw, 64, t), H, W, shift)

    # this library's kernel, fp16 in and out, pixel order (the cyclic shift read in place)
    tq = torch.from_numpy(qkv[None]).cuda()
    out = torch.empty((1, H, W, t), dtype=torch.float16, device="cuda")
    rc = be3.lib.scb_probe_attention(be3.ctx, tq.data_ptr(), 1, H, W, t, shift, trp.data_ptr(), out.data_ptr())
    assert rc == 0, be3.lib.scb_last_error(be3.ctx)
    got = out[0].float().cpu().numpy()

    r1, ok1 = _close(want, ref, 1e-4)
    r2, ok2 = _close(ref, got, 4e-3)
    print(f"attention {H}x{W} t{t} s{shift}: reference kernel vs oracle {r1:.2e}, B200 vs reference kernel {r2:.2e}")
    assert ok1, f"reference kernel vs numpy oracle: {r1:.3e} of scale"
    assert ok2, f"B200 kernel vs reference kernel: {r2:.3e} of scale"


def test_attention_speed_vs_reference_kernel(scb, be3):
    """Device time of the window attention at the config-4 geometries the forward
    runs it on (quarter and eighth resolution of a 1920x1088 frame, W and SW): this
    library's kernel inside a profiled forward vs the reference's kernel on the same
    windows (FP32 qkv, its native format), CUDA events on one stream."""
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no GPU")
    lib = _ref()
    x = torch.from_numpy(scb.synth.frames(4000, 1, 1080, 1920)).cuda()
    y = torch.empty((1, 3, 1080, 1920), dtype=torch.float32, device="cuda")
    s = torch.cuda.Stream()
    be3.forward_dev(x.data_ptr(), scb.SCB_U8, 1, 3, 1080, 1920, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    be3.set_profiling(True)
    be3.forward_dev(x.data_ptr(), scb.SCB_U8, 1, 3, 1080, 1920, y.data_ptr(), scb.SCB_F32, s.cuda_stream)
    s.synchronize()
    prof = be3.profile()
    be3.set_profiling(False)
    att = [ms for name, _, _, ms in prof if name == "attention"]
    assert len(att) == 12, "8 quarter-resolution + 4 eighth-resolution attention launches expected"
    mine = {128: sorted(att[:4] + att[8:12])[4], 256: sorted(att[4:8])[2]}  # medians by width
    rows = []
    for t, (H, W) in ((128, (272, 480)), (256, (136, 240))):
        heads, nw = t // 32, (H // 8) * (W // 8)
        qkv = torch.randn((nw * 64, 3 * t), device="cuda")
        rp = torch.randn((heads, 15, 15), device="cuda") * 0.02
        out = torch.empty((nw * 64, t), device="cuda")
        with torch.cuda.stream(s):
            for _ in range(3):
                lib.ref_window_attn_r64(qkv.data_ptr(), rp.data_ptr(), out.data_ptr(), nw, W // 8, H, W, heads, 4, 0,
                                        s.cuda_stream)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            for _ in range(10):
                lib.ref_window_attn_r64(qkv.data_ptr(), rp.data_ptr(), out.data_ptr(), nw, W // 8, H, W, heads, 4, 0,
                                        s.cuda_stream)
            e1.record(s)
        s.synchronize()
        ref_ms = e0.elapsed_time(e1) / 10
        rows.append((t, H, W, mine[t], ref_ms))
        print(f"attention {H}x{W} t={t}: B200 kernel {mine[t] * 1e3:.1f} us, reference kernel {ref_ms * 1e3:.1f} us "
              f"({ref_ms / mine[t]:.1f}x)")
    for t, H, W, m, r in rows:
        assert m < r, f"t={t}: this kernel ({m:.3f} ms) is not faster than the reference's ({r:.3f} ms)"
