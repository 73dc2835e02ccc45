// 8x8 window multi-head self-attention, W and SW, on tcgen05.
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
// One CTA = 128 threads = one PAIR of windows (128 tokens, thread = token row),
// looping over heads. Per head:
//   q, k  -> smem [128 x 32] fp16 K-major (64B swizzle)            (UMMA A and B)
//   v^T   -> smem [32 x 128] fp16 K-major (128B swizzle, 2 K blocks) (UMMA B)
//   S = Q K^T            : one M=128 N=128 K=32 UMMA chain into TMEM columns 0..127
//   softmax              : thread t reads its row's 64 in-window scores from TMEM,
//                          writes unnormalised exp() as fp16 to P (the other
//                          window's 64 keys stay zero, so the full K=128 product
//                          below only sums in-window keys)
//   O = P V              : M=128 N=32 K=128 UMMA chain into TMEM columns 0..31
//   out = O / rowsum     : fp16 to the output plane at the token's pixel.
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
constexpr int ATT_V = 16384;             // 2 blocks x [32 rows x 128 B]
constexpr int ATT_P = 24576;             // 2 blocks x [128 rows x 128 B]
constexpr int ATT_BIAS = ATT_P + 32768;  // heads x 225 floats (<= 8 heads)
constexpr int ATT_BAR = ATT_BIAS + 8 * 225 * 4;
constexpr int ATT_SMEM = ATT_BAR + 64 + 1024;

__global__ void __launch_bounds__(128)
window_attn_kernel(const __half* __restrict__ qkv, __half* __restrict__ out, const float* __restrict__ rp,
                   const AttnGeom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* bias = reinterpret_cast<float*>(sm + ATT_BIAS);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + ATT_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);

  const int tid = threadIdx.x, warp = tid >> 5;
  const int slot = tid >> 6, tok = tid & 63;
  const long win = 2L * blockIdx.x + slot;
  const bool valid = win < g.win.n_windows;
  const int qi = tok >> 3, qj = tok & 7;
  long pix = 0;
  bool last_row = false, last_col = false, store = false;
  if (valid) pix = win_token_pixel(g.win, win, qi, qj, last_row, last_col, store);

  for (int i = tid; i < g.heads * 225; i += 128) bias[i] = rp[i];
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 128);
  // P rows of the other window's keys are zero for every head: write them once.
  {
    uint8_t* pz = sm + ATT_P + (slot ^ 1) * 16384;
#pragma unroll
    for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(pz + swz_off(tid, c, 128)) = make_uint4(0, 0, 0, 0);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t s_base = smem_u32(sm);
  uint32_t phase = 0;
  constexpr float kScale = 0.17677669529663687f;  // 32^-1/2
  constexpr float kLog2e = 1.4426950408889634f;

  for (int h = 0; h < g.heads; ++h) {
    // ---- stage q, k, v^T for this head ----
    uint4 qv[4], kv[4], vv[4];
    if (valid) {
      const uint4* src = reinterpret_cast<const uint4*>(qkv + pix * g.qkv_ld + h * 32);
      const uint4* srk = reinterpret_cast<const uint4*>(qkv + pix * g.qkv_ld + g.t + h * 32);
      const uint4* srv = reinterpret_cast<const uint4*>(qkv + pix * g.qkv_ld + 2 * g.t + h * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        qv[c] = __ldg(src + c);
        kv[c] = __ldg(srk + c);
        vv[c] = __ldg(srv + c);
      }
    } else {
#pragma unroll
      for (int c = 0; c < 4; ++c) qv[c] = kv[c] = vv[c] = make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      *reinterpret_cast<uint4*>(sm + ATT_Q + swz_off(tid, c, 64)) = qv[c];
      *reinterpret_cast<uint4*>(sm + ATT_K + swz_off(tid, c, 64)) = kv[c];
    }
    {
      // v^T: row d (head channel), K index = key token tid (block tid/64).
      uint8_t* vb = sm + ATT_V + slot * 4096;
      const uint32_t kk = tid & 63;
      const __half* vh = reinterpret_cast<const __half*>(vv);
#pragma unroll
      for (int d = 0; d < 32; ++d)
        *reinterpret_cast<__half*>(vb + swz_off(d, kk >> 3, 128) + (kk & 7) * 2) = vh[d];
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t idS = make_idesc_f16(128, 128);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(s_base + ATT_Q + k * 32, 64, SW_64B), make_sdesc(s_base + ATT_K + k * 32, 64, SW_64B),
                 idS, k);
      umma_commit(bar);
    }
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);  // bounded; a timeout is reported, never hangs
    phase ^= 1;
    tc_fence_after();

    // ---- softmax over the 64 in-window keys of this row ----
    float s[64];
#pragma unroll
    for (int c = 0; c < 4; ++c) tmem_ld16(trow + slot * 64 + c * 16, s + c * 16);
    const float* bh = bias + h * 225;
    float mx = -INFINITY;
#pragma unroll
    for (int kt = 0; kt < 64; ++kt) {
      const int ki = kt >> 3, kj = kt & 7;
      float v = s[kt] * kScale + bh[(qi - ki + 7) * 15 + (qj - kj + 7)];
      const bool masked = (last_row && ((qi < 4) != (ki < 4))) || (last_col && ((qj < 4) != (kj < 4)));
      v = masked ? -INFINITY : v;
      s[kt] = v;
      mx = fmaxf(mx, v);
    }
    float sum = 0.f;
#pragma unroll
    for (int kt = 0; kt < 64; ++kt) {
      const float e = ex2_approx((s[kt] - mx) * kLog2e);
      s[kt] = e;
      sum += e;
    }
    {
      uint8_t* pr = sm + ATT_P + slot * 16384;
#pragma unroll
      for (int c = 0; c < 8; ++c)
        *reinterpret_cast<uint4*>(pr + swz_off(tid, c, 128)) =
            make_uint4(pack_half2(s[8 * c], s[8 * c + 1]), pack_half2(s[8 * c + 2], s[8 * c + 3]),
                       pack_half2(s[8 * c + 4], s[8 * c + 5]), pack_half2(s[8 * c + 6], s[8 * c + 7]));
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t idO = make_idesc_f16(128, 32);
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tmem, make_sdesc(s_base + ATT_P + kb * 16384 + k * 32, 128, SW_128B),
                   make_sdesc(s_base + ATT_V + kb * 4096 + k * 32, 128, SW_128B), idO, (kb | k) != 0);
      umma_commit(bar);
    }
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);  // bounded; a timeout is reported, never hangs
    phase ^= 1;
    tc_fence_after();
    float o[32];
    tmem_ld16(trow, o);
    tmem_ld16(trow + 16, o + 16);
    const float inv = 1.f / sum;
    if (valid && store) {
      uint4* dst = reinterpret_cast<uint4*>(out + pix * g.out_ld + h * 32);
#pragma unroll
      for (int c = 0; c < 4; ++c)
        dst[c] = make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv), pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                            pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv), pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
    }
    tc_fence_before();
    __syncthreads();  // smem q/k/v/P of this head are free for the next
    tc_fence_after();
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace scb
