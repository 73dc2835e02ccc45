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
// Persistent CTAs of 128 threads (four per SM, 128 TMEM columns each) walk pairs of
// windows (128 tokens, one UMMA M tile), one thread per token row; a CTA keeps one
// head. Per pair:
//   q, k  -> smem [128 x 32] fp16 K-major (64B swizzle)            (UMMA A and B)
//   v     -> smem [V_0 | V_1] MN-major [64 keys x 64] (128B swizzle) + a ones atom
//   S = Q K^T       : M=128 N=128 K=32 into TMEM columns 0..127 (both windows' keys;
//                     a row reads only its own window's 64)
//   softmax         : scores in base 2 (bias table pre-multiplied by log2 e, fp16),
//                     the mask only on the image's last window row / column;
//                     2^(s - max) as packed fp16 (ex2.approx.f16x2) to P' in TMEM
//                     columns 0..31 - each row's own keys
//   O' | rowsum = P' [V_0 | V_1 | 1]: M=128 N=80 K=64 into TMEM columns 32..111; a
//                     token of window s reads columns 32 + 32 s .. + 31 and the row
//                     sum of the fp16 P' it was multiplied with at column 96
//   out = O / rowsum: fp16 to the output plane at the token's pixel.
// The next pair's v is copied (cp.async) into a second operand buffer while the
// current pair computes, and its q and k into the single Q and K buffers as soon as
// this pair's S has been computed from them, so no pair waits a DRAM round trip; one
// Q / K buffer instead of two keeps a CTA's shared memory small enough for four CTAs
// per SM (three measured slower). Global loads and stores go four lanes per token
// (a token's 64 bytes of one head in one 16-byte chunk per lane, eight tokens per
// instruction, the pixel of each token passed by shuffle, the output staged through
// shared memory): with one lane per token every instruction touched 32 different
// rows, and the load/store unit's per-row work, not DRAM, set the kernel's pace.
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

// Layout per CTA (4 CTAs per SM, 128 TMEM columns each). A CTA keeps one head h for
// its whole life, so its relative-position bias table is built once. The v rows of
// the next pair are copied by cp.async straight into the other of two V buffers while
// the current pair computes; its q and k rows into the one Q / K buffer once this
// pair's S is done.
constexpr int ATT_Q = 0;                  // [128 x 64 B] SW64
constexpr int ATT_K = 8192;               // [128 x 64 B] SW64
constexpr int ATT_V = 16384;              // 2 x V, MN-major: [64 keys x 128 B] = [V_0 | V_1]
constexpr int ATT_ONES = 32768;           // [64 keys x 128 B]: N element 64 = 1 (the row sums)
constexpr int ATT_BIAS = ATT_ONES + 8192; // fp16 [64 query positions][64 keys], log2 units, chunk-swizzled
constexpr int ATT_BAR = ATT_BIAS + 8192;
constexpr int ATT_SMEM = ATT_BAR + 64 + 1024;
constexpr int ATT_CTAS = 4;               // per SM
constexpr int ATT_THREADS = 128;          // one per token row of a window pair

__global__ void __launch_bounds__(ATT_THREADS, ATT_CTAS)
window_attn_kernel(const __half* __restrict__ qkv, __half* __restrict__ out, const float* __restrict__ rp,
                   const AttnGeom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + ATT_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = warp * 32 + lane;  // TMEM lane = token row of the pair
  const int slot = row >> 6, tok = row & 63;
  const int qi = tok >> 3, qj = tok & 7;
  // CTA c works on head c % heads, pairs c / heads, c / heads + G, ... (G = CTAs per head)
  const int h = (int)(blockIdx.x % g.heads);
  const long p0 = blockIdx.x / g.heads, pstride = gridDim.x / g.heads;

  {
    // B_h(query m, key k) = rp[h][(mi - ki + 7) * 15 + (mj - kj + 7)] log2(e), fp16, the
    // 16-byte chunks of row m XOR-swizzled by m % 8
    __half* tb = reinterpret_cast<__half*>(sm + ATT_BIAS);
    for (int i = tid; i < 64 * 64; i += blockDim.x) {
      const int m = i >> 6, k = i & 63, c = k >> 3;
      const float v = rp[h * 225 + ((m >> 3) - (k >> 3) + 7) * 15 + ((m & 7) - (k & 7) + 7)] * 1.4426950408889634f;
      tb[m * 64 + ((c ^ (m & 7)) << 3) + (k & 7)] = __float2half_rn(v);
    }
    // the ones atom of the V operand: N element 64 = 1 for every key (the row sums)
    for (int i = tid; i < 64 * 8; i += blockDim.x)
      *reinterpret_cast<uint4*>(sm + ATT_ONES + swz_off(i >> 3, i & 7, 128)) =
          make_uint4((i & 7) == 0 ? 0x3C00u : 0u, 0u, 0u, 0u);
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, 128);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t sb = smem_u32(sm);
  uint32_t phase = 0;
  constexpr float kScaleLog2e = 0.17677669529663687f * 1.4426950408889634f;  // 32^-1/2 log2(e)
  const long n_pairs = (g.win.n_windows + 1) / 2;

  auto locate = [&](long pr, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * pr + slot;
    lr = lc = st = false;
    if (pr >= n_pairs || win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
  // The v (q, k) rows of head h of the warp's 32 tokens -> V rows tok, N elements
  // [32 slot, +32), of V buffer b (the Q and K rows); zeros past the last window. Lane
  // l copies 16-byte chunk l % 4 of the tokens of rows l / 4 + 8 k (k < 4), whose
  // pixel it takes from that row's lane (`pix`: the pixel of this lane's own row), so
  // one copy instruction covers eight whole 64-byte rows instead of one chunk of 32.
  // One cp.async group each.
  auto fetch_v = [&](long pix, int b) {
    const int c = lane & 3;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int sl = (lane >> 2) + 8 * k, rr = warp * 32 + sl;
      const long pk = __shfl_sync(0xffffffffu, pix, sl);
      const __half* src = pk >= 0 ? qkv + pk * g.qkv_ld + h * 32 : qkv;
      cp_async16(sm + ATT_V + b * 8192 + swz_off(rr & 63, 4 * (rr >> 6) + c, 128), src + 2 * g.t + 8 * c, pk >= 0);
    }
    cp_async_commit();
  };
  auto fetch_qk = [&](long pix) {
    const int c = lane & 3;
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int sl = (lane >> 2) + 8 * k, rr = warp * 32 + sl;
      const long pk = __shfl_sync(0xffffffffu, pix, sl);
      const __half* src = pk >= 0 ? qkv + pk * g.qkv_ld + h * 32 : qkv;
      cp_async16(sm + ATT_Q + swz_off(rr, c, 64), src + 8 * c, pk >= 0);
      cp_async16(sm + ATT_K + swz_off(rr, c, 64), src + g.t + 8 * c, pk >= 0);
    }
    cp_async_commit();
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

  long pair = p0;
  bool lr, lc, st;
  long pix = locate(pair, lr, lc, st);
  fetch_v(pix, 0);
  fetch_qk(pix);
  for (int u = 0; pair < n_pairs; pair += pstride, ++u) {
    const int b = u & 1;
    const bool last_row = lr, last_col = lc, store = st;
    const long pix_c = pix;
    // the next pair's v streams into V buffer b ^ 1 (its last reader, the P.V UMMA of
    // pair u - 1, has completed) while this pair computes
    pix = locate(pair + pstride, lr, lc, st);
    fetch_v(pix, b ^ 1);
    cp_async_wait_1();  // this thread's rows of pair u have landed (all but the group above)
    sync_mma();
    if (tid == 0) {  // S = Q K^T -> TMEM [0, 128)
      constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(sb + ATT_Q + k * 32, 64, SW_64B), make_sdesc(sb + ATT_K + k * 32, 64, SW_64B), id,
                 k);
      umma_commit(bar);
    }
    wait_mma();
    // S has read Q and K: the next pair's q and k stream in while this pair finishes
    fetch_qk(pix);

    // ---- softmax over the row's 64 in-window keys -> P' (TMEM [0, 32), fp16) ----
    {
      float s[64];
      tmem_ld16x2(trow + slot * 64, s, trow + slot * 64 + 16, s + 16);
      tmem_ld16x2(trow + slot * 64 + 32, s + 32, trow + slot * 64 + 48, s + 48);
      const uint8_t* rb = sm + ATT_BIAS + tok * 128;
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const uint4 u = *reinterpret_cast<const uint4*>(rb + ((c ^ (tok & 7)) << 4));
        const __half2* hb = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 r = __ffma2_rn(make_float2(s[8 * c + 2 * e], s[8 * c + 2 * e + 1]),
                                      make_float2(kScaleLog2e, kScaleLog2e), __half22float2(hb[e]));
          s[8 * c + 2 * e] = r.x;
          s[8 * c + 2 * e + 1] = r.y;
        }
      }
      if (last_row || last_col) {  // warp-uniform: the warp's tokens share a window
        const bool qtop = qi < 4, qleft = qj < 4;
#pragma unroll
        for (int j = 0; j < 64; ++j) {
          const bool m = (last_row && (qtop != ((j >> 3) < 4))) || (last_col && (qleft != ((j & 7) < 4)));
          s[j] = m ? -INFINITY : s[j];
        }
      }
      const float mx = row_max<64>(s);
      // P' = 2^(s - max) as packed fp16, the precision the P.V operand has anyway; the
      // row sum comes from the same fp16 values (the ones column of V)
      uint32_t p[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float2 d = __fadd2_rn(make_float2(s[2 * j], s[2 * j + 1]), make_float2(-mx, -mx));
        p[j] = ex2_approx_h2(pack_half2(d.x, d.y));
      }
      tmem_st32u(trow, p);
      tmem_wait_st();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {  // O' | rowsum = P' [V_0 | V_1 | 1] -> TMEM [32, 112)
      constexpr uint32_t id = make_idesc_f16_bmn(128, 80);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16_ts(tmem + 32, tmem + 8 * k,
                    make_sdesc_lbo_sbo(sb + ATT_V + b * 8192 + 2048 * k, ATT_ONES - ATT_V - b * 8192, 1024, SW_128B),
                    id, k);
      umma_commit(bar);
    }
    wait_mma();
    {
      float o[32];
      tmem_ld16x2(trow + 32 + slot * 32, o, trow + 48 + slot * 32, o + 16);  // this token's window's half of O'
      const float inv = __fdividef(1.f, tmem_ld1(trow + 96));
      // the row's 64 output bytes -> the current V tile (its P.V has completed) as
      // staging, then each lane stores chunk l % 4 of rows l / 4 + 8 k: one store
      // instruction writes eight whole 64-byte rows
      uint8_t* stg = sm + ATT_V + b * 8192;
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(stg + row * 64 + 16 * (c ^ (row & 3))) =
            make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv), pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                       pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                       pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
      __syncwarp();
      const long mine = (pix_c >= 0 && store) ? pix_c : -1;
      const int c = lane & 3;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int sl = (lane >> 2) + 8 * k, rr = warp * 32 + sl;
        const long pk = __shfl_sync(0xffffffffu, mine, sl);
        const uint4 v = *reinterpret_cast<const uint4*>(stg + rr * 64 + 16 * (c ^ (rr & 3)));
        if (pk >= 0) *reinterpret_cast<uint4*>(out + pk * g.out_ld + h * 32 + 8 * c) = v;
      }
    }
    tc_fence_before();
    __syncthreads();  // Q, K, V, P' and the TMEM accumulators are reused by the next pair
    tc_fence_after();
  }
  cp_async_wait_all();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 128);
}

}  // namespace scb
