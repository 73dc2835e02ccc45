// 8x8 window multi-head self-attention, W and SW, on tcgen05 (the trans half of the
// quarter- and eighth-resolution blocks, whose transformer runs as separate launches).
//
// Semantics are upstream `WMSA.forward` (tools/network_scunet.py:69-102) and the
// reference kernel `sc_window_attn_r64` (cuda/scunet.cu:461-625), for head_dim 32:
//   token (i, j) of window (wh, ww) is pixel ((wh*8+i+s) mod H, (ww*8+j+s) mod W),
//   s = 4 for SW blocks, 0 for W (the cyclic roll, read in place - no gather pass);
//   S = q.k^T * 32^-1/2 + rp[h][qi-ki+7][qj-kj+7];
//   SW only: on the last window row a query and key on different sides of window
//   row 4 are masked, on the last window column likewise for column 4
//   (tools/network_scunet.py:49-67, cuda/scunet.cu:137-147);
//   softmax over the 64 keys, O = P.v.
//
// Persistent CTAs of 256 threads walk pairs of windows (128 tokens, one UMMA M
// tile), two threads per token row (warps w and w + 4 share TMEM lane quarter w % 4
// and split each row's channels and keys in halves). Per head:
//   q, k  -> smem [128 x 32] fp16 K-major (64B swizzle)            (UMMA A and B)
//   v^T   -> smem [V_0 | V_1]^T [64 x 64 keys] (128B swizzle)       (UMMA B)
//   S = Q K^T       : M=128 N=128 K=32 into TMEM columns 0..127 (both windows' keys;
//                     a row reads only its own window's 64)
//   softmax         : scores in base 2 (table pre-multiplied by log2 e), the mask only
//                     on the image's last window row / column; unnormalised exp()
//                     as fp16 to P' [128 tokens x 64 keys] - each row's own keys
//   O' = P' [V_0|V_1]: M=128 N=64 K=64 into TMEM columns 128..191; a token of window
//                     s reads columns 32 s .. 32 s + 31, the product with its own V
//   out = O / rowsum: fp16 to the output plane at the token's pixel.
// The next head's q, k, v (or the next pair's first head) are loaded into registers
// while the current head computes, so no head waits a DRAM round trip.
#pragma once
#include "ptx.cuh"

namespace scb {

struct AttnGeom {
  WinGeom win;
  int t;           // channels of the trans half (heads * 32)
  int heads;
  long qkv_ld;     // elements per pixel row of qkv (3t)
  long out_ld;     // elements per pixel row of out
};

constexpr int ATT_Q = 0;
constexpr int ATT_K = 8192;
constexpr int ATT_V = 16384;              // [V_0 | V_1]^T: 2 x [32 rows x 128 B]
constexpr int ATT_P = 24576;              // P' [128 rows x 128 B]
constexpr int ATT_BIAS = ATT_P + 16384;   // heads x 225 floats (<= 8 heads), times log2(e)
constexpr int ATT_RED = ATT_BIAS + 8 * 225 * 4;  // 2 areas x [2 halves x 128 rows] float2
constexpr int ATT_BAR = ATT_RED + 4096;
constexpr int ATT_SMEM = ATT_BAR + 64 + 1024;
constexpr int ATT_CTAS = 2;               // per SM (TMEM: 256 columns each)

__global__ void __launch_bounds__(256, ATT_CTAS)
window_attn_kernel(const __half* __restrict__ qkv, __half* __restrict__ out, const float* __restrict__ rp,
                   const AttnGeom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* bias = reinterpret_cast<float*>(sm + ATT_BIAS);
  float2* red = reinterpret_cast<float2*>(sm + ATT_RED);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + ATT_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane, hf = warp >> 2;
  const int slot = row >> 6, tok = row & 63;
  const int qi = tok >> 3, qj = tok & 7;

  for (int i = tid; i < g.heads * 225; i += blockDim.x) bias[i] = rp[i] * 1.4426950408889634f;
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 256);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const uint32_t sb = smem_u32(sm);
  uint32_t phase = 0;
  constexpr float kScaleLog2e = 0.17677669529663687f * 1.4426950408889634f;  // 32^-1/2 log2(e)
  uint32_t mrow = 0, mcol = 0;  // this token's mask over its thread's 32 keys (bit j: key hf*32 + j)
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int kt = hf * 32 + j;
    mrow |= (uint32_t)((qi < 4) != ((kt >> 3) < 4)) << j;
    mcol |= (uint32_t)((qj < 4) != ((kt & 7) < 4)) << j;
  }
  const long n_pairs = (g.win.n_windows + 1) / 2;
  auto locate = [&](long pr, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * pr + slot;
    lr = lc = st = false;
    if (pr >= n_pairs || win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
  // this thread's 16 channels of q, k and v of head h at pixel pix
  auto load_head = [&](long pix, int h, uint4* d) {
#pragma unroll
    for (int m = 0; m < 3; ++m)
#pragma unroll
      for (int c = 0; c < 2; ++c)
        d[2 * m + c] = pix >= 0 ? __ldg(reinterpret_cast<const uint4*>(qkv + pix * g.qkv_ld + m * g.t + h * 32 +
                                                                       hf * 16) + c)
                                : make_uint4(0, 0, 0, 0);
  };
  auto sync_mma = [&]() {
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  auto wait_mma = [&]() {
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);  // bounded; a timeout is reported, never hangs
    phase ^= 1;
    tc_fence_after();
  };

  long pair = blockIdx.x;
  bool lr, lc, st;
  long pix = locate(pair, lr, lc, st);
  uint4 nx[6];
  load_head(pix, 0, nx);

  for (; pair < n_pairs; pair += gridDim.x) {
    const bool last_row = lr, last_col = lc, store = st;
    const long pix_c = pix;
    for (int h = 0; h < g.heads; ++h) {
      uint4 cur[6];
#pragma unroll
      for (int m = 0; m < 6; ++m) cur[m] = nx[m];
      if (h + 1 < g.heads) {
        load_head(pix_c, h + 1, nx);
      } else {  // the next pair's first head
        pix = locate(pair + gridDim.x, lr, lc, st);
        load_head(pix, 0, nx);
      }
      // ---- q, k -> Q, K (16-byte chunks 2 hf, 2 hf + 1 of 64-byte rows); v -> V^T ----
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        *reinterpret_cast<uint4*>(sm + ATT_Q + swz_off(row, 2 * hf + c, 64)) = cur[c];
        *reinterpret_cast<uint4*>(sm + ATT_K + swz_off(row, 2 * hf + c, 64)) = cur[2 + c];
      }
      {
        const __half* vh = reinterpret_cast<const __half*>(&cur[4]);
        uint8_t* vb = sm + ATT_V + slot * 4096;
#pragma unroll
        for (int d = 0; d < 16; ++d)
          *reinterpret_cast<__half*>(vb + swz_off(hf * 16 + d, tok >> 3, 128) + (tok & 7) * 2) = vh[d];
      }
      sync_mma();
      if (tid == 0) {
        constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_f16(tmem, make_sdesc(sb + ATT_Q + k * 32, 64, SW_64B), make_sdesc(sb + ATT_K + k * 32, 64, SW_64B),
                   id, k);
        umma_commit(bar);
      }
      wait_mma();

      // ---- softmax over the row's 64 in-window keys (32 per thread) -> P' ----
      float s[32];
      tmem_ld16x2(trow + slot * 64 + hf * 32, s, trow + slot * 64 + hf * 32 + 16, s + 16);
      const float* bh = bias + h * 225 + (qi + 7) * 15 + (qj + 7);  // bias(key) = bh[-(15 ki + kj)]
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int kt = hf * 32 + j;
        s[j] = fmaf(s[j], kScaleLog2e, bh[-((kt >> 3) * 15 + (kt & 7))]);
      }
      if (last_row || last_col) {  // warp-uniform: the warp's tokens share a window
        const uint32_t m = (last_row ? mrow : 0u) | (last_col ? mcol : 0u);
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = (m >> j) & 1u ? -INFINITY : s[j];
      }
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) mx = fmaxf(mx, s[j]);
      red[hf * 128 + row].x = mx;
      __syncthreads();
      mx = fmaxf(mx, red[(hf ^ 1) * 128 + row].x);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float e = ex2_approx(s[j] - mx);
        s[j] = e;
        sum += e;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(sm + ATT_P + swz_off(row, hf * 4 + c, 128)) =
            make_uint4(pack_half2(s[8 * c], s[8 * c + 1]), pack_half2(s[8 * c + 2], s[8 * c + 3]),
                       pack_half2(s[8 * c + 4], s[8 * c + 5]), pack_half2(s[8 * c + 6], s[8 * c + 7]));
      red[256 + hf * 128 + row].x = sum;  // second exchange area: no barrier needed before this write
      sync_mma();
      sum += red[256 + (hf ^ 1) * 128 + row].x;
      if (tid == 0) {  // O' = P' [V_0 | V_1] -> TMEM [128, 192)
        constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem + 128, make_sdesc(sb + ATT_P + k * 32, 128, SW_128B),
                   make_sdesc(sb + ATT_V + k * 32, 128, SW_128B), id, k);
        umma_commit(bar);
      }
      wait_mma();
      float o[16];
      tmem_ld16(trow + 128 + slot * 32 + hf * 16, o);  // this token's window's half of O'
      const float inv = 1.f / sum;
      if (pix_c >= 0 && store) {
        uint4* dst = reinterpret_cast<uint4*>(out + pix_c * g.out_ld + h * 32 + hf * 16);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          dst[c] = make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv), pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                              pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                              pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
      }
      tc_fence_before();
      __syncthreads();  // Q, K, V^T, P' and the TMEM accumulators are reused by the next head
      tc_fence_after();
    }
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 256);
}

}  // namespace scb
