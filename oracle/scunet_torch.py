"""Fast oracle: the numpy oracle (`scunet_np.py`) restated in torch float32.

TEST INFRASTRUCTURE ONLY. Only `tests/`, `__graft_entry__.smoke()` and the
`cpu_baseline` / `--impl reference` legs of `bench.py` may import this module, and
only as the checker or the timed CPU baseline. The product path (the CUDA library
behind `include/scunet_b200.h`) never calls it.

Same algorithm, same citations (scunet-rs paths), laid out channels-first so that
convolutions are `torch.nn.functional` calls; it runs on the CPU (all host threads:
the timed CPU baseline) or on a GPU in strict FP32 (TF32 switched off for matmul and
cuDNN), which is the only oracle fast enough for the full-size configurations (one
1920x1080 frame, 1024x1024 gray images). `tests/test_oracle_torch.py` pins it to the
numpy oracle and to the committed golden fixtures before anything relies on it.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

WIN = 8
HEAD_DIM = 32


def strict_fp32():
    """No TF32 anywhere: the oracle is the reference's FP32 arithmetic."""
    torch.backends.cuda.matmul.allow_tf32 = False
    torch.backends.cudnn.allow_tf32 = False
    torch.set_float32_matmul_precision("highest")


def conv3x3(x, w):
    """3x3, stride 1, ZERO pad 1, no bias (`src/cpu.rs:66-137`). x [n][ci][h][w]."""
    return F.conv2d(x, w, padding=1)


def conv1x1(x, w, b):
    """1x1 with bias (`src/cpu.rs:175-217`)."""
    return F.conv2d(x, w, b)


def conv2x2s2(x, w):
    """`m_down*.4`: 2x2 stride 2, no pad, no bias (`src/cpu.rs:141-170`)."""
    return F.conv2d(x, w, stride=2)


def conv_t2x2(x, w):
    """`m_up*.0`: ConvTranspose2d(2, stride 2), w [ci][co][2][2] (`src/cpu.rs:232-263`)."""
    return F.conv_transpose2d(x, w, stride=2)


def layer_norm(x, g, b, eps=1e-5):
    """LayerNorm over the last axis, biased variance (`src/cpu.rs:338-357`)."""
    return F.layer_norm(x, (x.shape[-1],), g, b, eps)


def gelu(x):
    """Exact-erf GELU (`tools/reference.py:127-137`)."""
    return F.gelu(x)


def relpos_bias(rp):
    """[heads][15][15] -> [heads][64][64], entry (p, q) = rp[h][py-qy+7][px-qx+7]
    (`tools/network_scunet.py:104-108`)."""
    idx = torch.arange(WIN * WIN, device=rp.device)
    py, px = idx // WIN, idx % WIN
    return rp[:, py[:, None] - py[None, :] + WIN - 1, px[:, None] - px[None, :] + WIN - 1]


def sw_mask(nwh, nww, device):
    """[nwh*nww][64][64] bool, True = masked: last window row splits rows at 4, last
    window column splits columns at 4 (`tools/network_scunet.py:49-67`)."""
    s = WIN - WIN // 2
    idx = torch.arange(WIN * WIN, device=device)
    r, c = idx // WIN, idx % WIN
    m = torch.zeros(nwh, nww, WIN * WIN, WIN * WIN, dtype=torch.bool, device=device)
    m[-1, :] |= (r[:, None] < s) != (r[None, :] < s)
    m[:, -1] |= (c[:, None] < s) != (c[None, :] < s)
    return m.reshape(nwh * nww, WIN * WIN, WIN * WIN)


def window_tokens(x, shift):
    """[n][h][w][c] -> [n*nw][64][c]; token (i, j) of window (wh, ww) is pixel
    ((wh*8+i+shift) mod h, (ww*8+j+shift) mod w) (`tools/network_scunet.py:77-84`)."""
    n, h, w, c = x.shape
    if shift:
        x = torch.roll(x, (-shift, -shift), dims=(1, 2))
    t = x.reshape(n, h // WIN, WIN, w // WIN, WIN, c).permute(0, 1, 3, 2, 4, 5)
    return t.reshape(-1, WIN * WIN, c)


def window_untokens(t, n, h, w, shift):
    """Inverse of `window_tokens` (`tools/network_scunet.py:99-101`)."""
    c = t.shape[-1]
    x = t.reshape(n, h // WIN, w // WIN, WIN, WIN, c).permute(0, 1, 3, 2, 4, 5).reshape(n, h, w, c)
    if shift:
        x = torch.roll(x, (shift, shift), dims=(1, 2))
    return x


def attention_core(qkv, rp, nwh, nww, shifted):
    """qkv [n*nw][64][3t] (q | k | v column blocks, heads contiguous inside each,
    `cuda/scunet.cu:159-168`) -> [n*nw][64][t] (`tools/network_scunet.py:85-97`)."""
    nw, n, c3 = qkv.shape
    t = c3 // 3
    heads = t // HEAD_DIM
    q, k, v = (qkv[..., i * t:(i + 1) * t].reshape(nw, n, heads, HEAD_DIM).transpose(1, 2) for i in range(3))
    sim = (q @ k.transpose(-1, -2)) * HEAD_DIM ** -0.5 + relpos_bias(rp)[None]
    if shifted:
        m = sw_mask(nwh, nww, qkv.device).repeat(nw // (nwh * nww), 1, 1)
        sim = sim.masked_fill(m[:, None], float("-inf"))
    p = torch.softmax(sim, dim=-1)
    return (p @ v).transpose(1, 2).reshape(nw, n, t)


def wmsa(x, w, pre, shifted):
    """Window MSA on an LN'd [n][h][w][t] plane (`tools/network_scunet.py:69-102`)."""
    n, h, wd, t = x.shape
    s = WIN // 2 if shifted else 0
    tok = window_tokens(x, s)
    qkv = F.linear(tok, w[pre + ".embedding_layer.weight"], w[pre + ".embedding_layer.bias"])
    o = attention_core(qkv, w[pre + ".relative_position_params"], h // WIN, wd // WIN, shifted)
    o = F.linear(o, w[pre + ".linear.weight"], w[pre + ".linear.bias"])
    return window_untokens(o, n, h, wd, s)


def trans_block(x, w, pre, shifted):
    """Swin block on [n][h][w][t] (`tools/network_scunet.py:134-137`)."""
    x = x + wmsa(layer_norm(x, w[pre + ".ln1.weight"], w[pre + ".ln1.bias"]), w, pre + ".msa", shifted)
    hdn = gelu(F.linear(layer_norm(x, w[pre + ".ln2.weight"], w[pre + ".ln2.bias"]), w[pre + ".mlp.0.weight"],
                        w[pre + ".mlp.0.bias"]))
    return x + F.linear(hdn, w[pre + ".mlp.2.weight"], w[pre + ".mlp.2.bias"])


def conv_trans_block(x, w, pre, shifted):
    """ConvTransBlock on [n][c][h][w] (`tools/network_scunet.py:167-176`): conv half
    first in the concat."""
    cc = x.shape[1] // 2
    y = conv1x1(x, w[pre + ".conv1_1.weight"], w[pre + ".conv1_1.bias"])
    yc, yt = y[:, :cc], y[:, cc:]
    hc = conv3x3(torch.relu(conv3x3(yc, w[pre + ".conv_block.0.weight"])), w[pre + ".conv_block.2.weight"]) + yc
    ht = trans_block(yt.permute(0, 2, 3, 1), w, pre + ".trans_block", shifted).permute(0, 3, 1, 2)
    return x + conv1x1(torch.cat([hc, ht], 1), w[pre + ".conv1_2.weight"], w[pre + ".conv1_2.bias"])


def _stage_blocks(x, w, stage, count):
    """Block i is shifted iff i is odd, in every stage, up stages included
    (`tools/network_scunet.py:194-225`, `tools/reference.py:337-349`)."""
    first = 1 if stage.startswith("up") else 0
    for i in range(count):
        x = conv_trans_block(x, w, f"m_{stage}.{first + i}", bool(i % 2))
    return x


def forward_padded(x, w, config=(4,) * 7):
    """[n][in_nc][hp][wp] (padded) -> same (`tools/network_scunet.py:240-259`): skips
    are added BEFORE each up conv."""
    x1 = conv3x3(x, w["m_head.0.weight"])
    x2 = conv2x2s2(_stage_blocks(x1, w, "down1", config[0]), w[f"m_down1.{config[0]}.weight"])
    x3 = conv2x2s2(_stage_blocks(x2, w, "down2", config[1]), w[f"m_down2.{config[1]}.weight"])
    x4 = conv2x2s2(_stage_blocks(x3, w, "down3", config[2]), w[f"m_down3.{config[2]}.weight"])
    b = _stage_blocks(x4, w, "body", config[3])
    y = _stage_blocks(conv_t2x2(b + x4, w["m_up3.0.weight"]), w, "up3", config[4])
    y = _stage_blocks(conv_t2x2(y + x3, w["m_up2.0.weight"]), w, "up2", config[5])
    y = _stage_blocks(conv_t2x2(y + x2, w["m_up1.0.weight"]), w, "up1", config[6])
    return conv3x3(y + x1, w["m_tail.0.weight"])


@torch.no_grad()
def forward(x_nchw, w, config=(4,) * 7, device="cpu"):
    """[n][c][h][w] float in [0,1] (numpy or torch) -> torch [n][c][h][w] float32 on
    `device`: replicate-pad to 64, run, crop (`src/backend.rs:63-105`,
    `src/plan.rs:67-94`). `w`: name -> array."""
    strict_fp32()
    x = torch.as_tensor(x_nchw, dtype=torch.float32).to(device)
    n, c, h, wd = x.shape
    hp, wp = -(-h // 64) * 64, -(-wd // 64) * 64
    wt = {k: torch.as_tensor(v, dtype=torch.float32).to(device).contiguous() for k, v in w.items()}
    xp = F.pad(x, (0, wp - wd, 0, hp - h), mode="replicate") if (hp, wp) != (h, wd) else x
    return forward_padded(xp, wt, config)[:, :, :h, :wd]
