"""CPU oracle: a float32 numpy restatement of the SCUNet forward pass.

TEST INFRASTRUCTURE ONLY. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import this module, and
only as the checker or the timed CPU baseline. The product path (the CUDA library
behind `include/scunet_b200.h`) never calls it.

What it restates (scunet-rs, paths relative to that project):
* the reference's own numpy SCUNet, `tools/reference.py:73-349`;
* the upstream torch module it is held to, `tools/network_scunet.py:25-259`;
* the Rust CPU twin, `src/cpu.rs` (same stage order, `forward_dump` `:1175-1321`).

It is written channels-last ([h][w][c] per image) so that every convolution and
linear is a plain matmul over pixels; the arithmetic is the reference's.

Parity pinning: `tests/golden/make_golden.py` runs this file, the reference's own
`tools/reference.py` and the upstream torch module on the same seeded weights and
inputs, and records their agreement in `tests/golden/manifest.json`;
`tests/test_oracle.py` re-checks this file against the committed fixtures.
"""
from __future__ import annotations

import numpy as np

try:  # exact-erf GELU; scipy is in the image, math.erf is the slow fallback
    from scipy.special import erf as _erf
except Exception:  # pragma: no cover
    import math
    _erf = np.vectorize(math.erf, otypes=[np.float64])

F32 = np.float32
WIN = 8
HEAD_DIM = 32


# ---------------------------------------------------------------------------
# primitives, [h][w][c]
# ---------------------------------------------------------------------------

def conv3x3(x, w):
    """3x3, stride 1, ZERO pad 1, no bias (`src/cpu.rs:66-137`,
    `tools/reference.py:73-97`). x [h][w][ci], w [co][ci][3][3] -> [h][w][co]."""
    h, wd, _ = x.shape
    xp = np.pad(x, ((1, 1), (1, 1), (0, 0)))
    acc = np.zeros((h, wd, w.shape[0]), F32)
    for ky in range(3):          # accumulation order ky, kx, ci
        for kx in range(3):
            acc += xp[ky:ky + h, kx:kx + wd] @ w[:, :, ky, kx].T
    return acc


def conv1x1(x, w, b):
    """1x1 with bias (`src/cpu.rs:175-217`). w [co][ci][1][1]."""
    return x @ w[:, :, 0, 0].T + b


def conv2x2s2(x, w):
    """`m_down*.4`: 2x2 stride 2, no pad, no bias (`src/cpu.rs:141-170`).
    w [co][ci][2][2] -> [h/2][w/2][co]."""
    acc = None
    for dy in range(2):
        for dx in range(2):
            t = x[dy::2, dx::2] @ w[:, :, dy, dx].T
            acc = t if acc is None else acc + t
    return acc


def conv_t2x2(x, w):
    """`m_up*.0`: ConvTranspose2d(2, stride 2), no tap flip (`src/cpu.rs:232-263`,
    `tools/reference.py:100-117`). w [ci][co][2][2] -> [2h][2w][co]."""
    h, wd, _ = x.shape
    out = np.empty((2 * h, 2 * wd, w.shape[1]), F32)
    for dy in range(2):
        for dx in range(2):
            out[dy::2, dx::2] = x @ w[:, :, dy, dx]
    return out


def layer_norm(x, g, b, eps=1e-5):
    """LayerNorm over the last axis, biased variance (`src/cpu.rs:338-357`)."""
    mu = x.mean(axis=-1, keepdims=True, dtype=F32)
    var = ((x - mu) ** 2).mean(axis=-1, keepdims=True, dtype=F32)
    return ((x - mu) / np.sqrt(var + F32(eps)) * g + b).astype(F32)


def gelu(x):
    """Exact-erf GELU (`tools/reference.py:127-137`)."""
    return (0.5 * x * (1.0 + _erf(x.astype(np.float64) / np.sqrt(2.0)))).astype(F32)


def relpos_bias(rp):
    """[heads][15][15] -> [heads][64][64]: entry (p, q) = rp[h][py-qy+7][px-qx+7]
    (`tools/network_scunet.py:104-108`, `src/cpu.rs:532-546`)."""
    idx = np.arange(WIN * WIN)
    py, px = idx // WIN, idx % WIN
    dy = py[:, None] - py[None, :] + WIN - 1
    dx = px[:, None] - px[None, :] + WIN - 1
    return rp[:, dy, dx]


def sw_mask(nwh, nww):
    """[nwh*nww][64][64] bool, True = masked (`tools/network_scunet.py:49-67`).

    On the last window ROW a query and a key are masked when they sit on different
    sides of row 4 of the window; on the last window COLUMN, on different sides of
    column 4. Each edge compares the same axis on both sides."""
    s = WIN - WIN // 2
    idx = np.arange(WIN * WIN)
    r, c = idx // WIN, idx % WIN
    row_hit = (r[:, None] < s) != (r[None, :] < s)
    col_hit = (c[:, None] < s) != (c[None, :] < s)
    m = np.zeros((nwh, nww, WIN * WIN, WIN * WIN), bool)
    m[-1, :] |= row_hit
    m[:, -1] |= col_hit
    return m.reshape(nwh * nww, WIN * WIN, WIN * WIN)


def window_tokens(x, shift):
    """[h][w][c] -> [nw][64][c]: token (i, j) of window (wh, ww) is pixel
    ((wh*8+i+shift) mod h, (ww*8+j+shift) mod w) - torch.roll by -shift then windows
    (`tools/network_scunet.py:77-84`)."""
    h, w, c = x.shape
    if shift:
        x = np.roll(x, (-shift, -shift), axis=(0, 1))
    t = x.reshape(h // WIN, WIN, w // WIN, WIN, c).transpose(0, 2, 1, 3, 4)
    return np.ascontiguousarray(t.reshape(-1, WIN * WIN, c))


def window_untokens(t, h, w, shift):
    """Inverse of `window_tokens` (`tools/network_scunet.py:99-101`)."""
    c = t.shape[-1]
    x = t.reshape(h // WIN, w // WIN, WIN, WIN, c).transpose(0, 2, 1, 3, 4).reshape(h, w, c)
    if shift:
        x = np.roll(x, (shift, shift), axis=(0, 1))
    return np.ascontiguousarray(x)


def attention_core(qkv, rp, nwh, nww, shifted):
    """The kernel-level op: qkv [nw][64][3t] (q | k | v column blocks, heads
    contiguous inside each, `cuda/scunet.cu:159-168`) -> o [nw][64][t].
    sim = q.k^T * hd^-1/2 + bias; SW mask -> -inf; softmax over keys; P.v
    (`tools/network_scunet.py:85-97`)."""
    nw, n, c3 = qkv.shape
    t = c3 // 3
    heads = t // HEAD_DIM
    q = qkv[..., :t].reshape(nw, n, heads, HEAD_DIM).transpose(2, 0, 1, 3)
    k = qkv[..., t:2 * t].reshape(nw, n, heads, HEAD_DIM).transpose(2, 0, 1, 3)
    v = qkv[..., 2 * t:].reshape(nw, n, heads, HEAD_DIM).transpose(2, 0, 1, 3)
    sim = (q @ k.transpose(0, 1, 3, 2)) * F32(HEAD_DIM ** -0.5)
    sim = sim + relpos_bias(rp)[:, None]
    if shifted:
        sim = np.where(sw_mask(nwh, nww)[None], F32(-np.inf), sim)
    sim = sim - sim.max(axis=-1, keepdims=True)
    e = np.exp(sim)
    p = (e / e.sum(axis=-1, keepdims=True)).astype(F32)
    o = p @ v                                          # [heads][nw][64][hd]
    return np.ascontiguousarray(o.transpose(1, 2, 0, 3).reshape(nw, n, t))


def wmsa(x, w, pre, shifted):
    """Window MSA on an LN'd [h][w][t] plane (`tools/network_scunet.py:69-102`)."""
    h, wd, t = x.shape
    s = WIN // 2 if shifted else 0
    tok = window_tokens(x, s)
    qkv = tok @ w[pre + ".embedding_layer.weight"].T + w[pre + ".embedding_layer.bias"]
    o = attention_core(qkv, w[pre + ".relative_position_params"], h // WIN, wd // WIN, shifted)
    o = o @ w[pre + ".linear.weight"].T + w[pre + ".linear.bias"]
    return window_untokens(o, h, wd, s)


def trans_block(x, w, pre, shifted):
    """Swin block (`tools/network_scunet.py:134-137`): two pre-LN residuals."""
    x = x + wmsa(layer_norm(x, w[pre + ".ln1.weight"], w[pre + ".ln1.bias"]), w, pre + ".msa", shifted)
    hdn = layer_norm(x, w[pre + ".ln2.weight"], w[pre + ".ln2.bias"])
    hdn = gelu(hdn @ w[pre + ".mlp.0.weight"].T + w[pre + ".mlp.0.bias"])
    return x + (hdn @ w[pre + ".mlp.2.weight"].T + w[pre + ".mlp.2.bias"])


def conv_trans_block(x, w, pre, shifted):
    """ConvTransBlock (`tools/network_scunet.py:167-176`, `src/cpu.rs:869-953`):
    y = conv1_1(x); conv half (first c/2) = conv3x3(relu(conv3x3(y_c))) + y_c;
    trans half = Swin block; out = x + conv1_2(concat(conv, trans))."""
    c = x.shape[-1]
    cc = c // 2
    y = conv1x1(x, w[pre + ".conv1_1.weight"], w[pre + ".conv1_1.bias"])
    yc, yt = y[..., :cc], y[..., cc:]
    hc = np.maximum(conv3x3(yc, w[pre + ".conv_block.0.weight"]), 0)
    hc = conv3x3(hc, w[pre + ".conv_block.2.weight"]) + yc
    ht = trans_block(yt, w, pre + ".trans_block", shifted)
    return x + conv1x1(np.concatenate([hc, ht], axis=-1), w[pre + ".conv1_2.weight"], w[pre + ".conv1_2.bias"])


def _stage_blocks(x, w, stage, count):
    """Blocks of one stage; block i is shifted iff i is odd, in EVERY stage
    (`tools/network_scunet.py:194-225`; up stages too, `tools/reference.py:337-349`)."""
    first = 1 if stage.startswith("up") else 0
    for i in range(count):
        x = conv_trans_block(x, w, f"m_{stage}.{first + i}", bool(i % 2))
    return x


def forward_padded(x, w, config=(4,) * 7):
    """[hp][wp][in_nc] (already padded) -> same. `SCUNet.forward`
    (`tools/network_scunet.py:240-259`): skips are added BEFORE each up conv."""
    x1 = conv3x3(x, w["m_head.0.weight"])
    x2 = conv2x2s2(_stage_blocks(x1, w, "down1", config[0]), w[f"m_down1.{config[0]}.weight"])
    x3 = conv2x2s2(_stage_blocks(x2, w, "down2", config[1]), w[f"m_down2.{config[1]}.weight"])
    x4 = conv2x2s2(_stage_blocks(x3, w, "down3", config[2]), w[f"m_down3.{config[2]}.weight"])
    b = _stage_blocks(x4, w, "body", config[3])
    y = _stage_blocks(conv_t2x2(b + x4, w["m_up3.0.weight"]), w, "up3", config[4])
    y = _stage_blocks(conv_t2x2(y + x3, w["m_up2.0.weight"]), w, "up2", config[5])
    y = _stage_blocks(conv_t2x2(y + x2, w["m_up1.0.weight"]), w, "up1", config[6])
    return conv3x3(y + x1, w["m_tail.0.weight"])


def forward(x_nchw, w, config=(4,) * 7):
    """[n][c][h][w] float32 in [0,1] -> [n][c][h][w]: replicate-pad to 64, run, crop
    (`src/backend.rs:63-105`, `src/plan.rs:67-94`)."""
    x_nchw = np.asarray(x_nchw, F32)
    n, c, h, wd = x_nchw.shape
    hp, wp = -(-h // 64) * 64, -(-wd // 64) * 64
    w = {k: np.asarray(v, F32) for k, v in w.items()}
    out = np.empty_like(x_nchw)
    for i in range(n):
        xi = np.pad(x_nchw[i], ((0, 0), (0, hp - h), (0, wp - wd)), mode="edge")
        yi = forward_padded(np.ascontiguousarray(xi.transpose(1, 2, 0)), w, config)
        out[i] = yi.transpose(2, 0, 1)[:, :h, :wd]
    return out


def quantise(y):
    """[0,1] float -> 8-bit level, `clamp(v,0,1)*255+0.5` truncated (`src/image.rs:60-63`)."""
    return np.floor(np.clip(y, 0.0, 1.0) * 255.0 + 0.5).astype(np.int32)


def parity_report(want, got):
    """The two parity numbers the acceptance bar uses: max |diff| on the [0,1]
    output, and the fraction of values whose 8-bit level differs by more than 1."""
    want = np.asarray(want, np.float64)
    got = np.asarray(got, np.float64)
    d = np.abs(want - got)
    lv = np.abs(quantise(want) - quantise(got))
    return {"max_abs": float(d.max()), "mean_abs": float(d.mean()),
            "frac_level_gt1": float((lv > 1).mean()), "frac_level_ne": float((lv > 0).mean())}
