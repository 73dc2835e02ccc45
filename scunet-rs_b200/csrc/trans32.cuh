// The transformer half of a full-resolution ConvTransBlock (trans width T = 32, one
// head) in one kernel per launch; the common structure and semantics are described
// in trans.cuh. This kernel is laid out so that three CTAs fit on an SM:
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136)
//
// Layout and schedule:
//  * TMEM: 128 columns. Each accumulator is read out before the next MMA that
//    overwrites it is issued, so qkv [0, 96), S [0, 128), O' [0, 64) and proj [0, 32)
//    share columns; the MLP output accumulates on top of proj (cols 0-31) and the
//    hidden chunk lives in cols 64-127.
//  * P.V without zero padding: P' [128 tokens x 64 keys] holds each token's own
//    window's keys, and one MMA computes O' = P' . [V_0 | V_1] (N = 64); a token of
//    window s reads columns [32 s, 32 s + 32) of O', the product with its own V.
//  * Shared memory: one 24 KB region holds, in turn, LN1 | Q | K, then P', then O,
//    then LN2 | hidden chunk. With the resident weights (24 KB), V^T (8 KB) and the
//    parameters and an 8 KB y_t staging buffer that is ~72 KB per CTA.
//  * The hidden layer runs in two 64-wide chunks; the second chunk's mlp0 MMA is
//    issued with the first chunk's mlp2 MMA, so the MLP costs three MMA round trips.
//  * Scores carry log2(e): the relative-position table is staged pre-multiplied and
//    q.k is scaled by 32^-1/2 log2(e), so the softmax exponent is one subtraction.
//    The shifted-window mask is only evaluated for windows on the image's last
//    window row or column (a warp's 32 tokens share one window).
//
// x1 = y_t + O.Wproj^T + b_proj is written back into the proj accumulator's TMEM
// columns, the mlp2 MMAs accumulate GELU(hid).W2^T onto it in fp32, and z = acc + b_2.
// y_t reaches shared memory by per-thread cp.async: the next pair's copy is issued
// once this pair has read it for the last time (x1), so its latency hides behind the
// MLP and no register holds it across the softmax.
#pragma once
#include "trans.cuh"

namespace scb {

struct Trans32Layout {
  static constexpr int T = 32;
  static constexpr int W_QKV = 0;                    // [96 x 64 B], SW64
  static constexpr int W_PROJ = W_QKV + 96 * 64;     // [32 x 64 B]
  static constexpr int W_0 = W_PROJ + 32 * 64;       // [128 x 64 B]
  static constexpr int W_2 = W_0 + 128 * 64;         // 2 K-blocks of [32 x 128 B], SW128
  static constexpr int R = W_2 + 2 * 32 * 128;       // the reused 24 KB region (1024-aligned)
  static constexpr int R_A1 = R, R_Q = R + 8192, R_K = R + 16384;
  static constexpr int R_P = R;                      // P' [128 x 128 B], SW128
  static constexpr int R_O = R;
  static constexpr int R_H = R + 8192;               // hidden chunk [128 x 128 B]
  static constexpr int VT = R + 24576;               // [V_0 | V_1]^T: 2 x [32 x 128 B]
  static constexpr int PAR = VT + 8192;
  static constexpr int P_BQKV = 0, P_BPROJ = 3 * T, P_B0 = 4 * T, P_B2 = 8 * T, P_L1G = 9 * T, P_L1B = 10 * T,
                       P_L2G = 11 * T, P_L2B = 12 * T, P_RP = 13 * T, P_N = 13 * T + 225;
  static constexpr int RED = (PAR + P_N * 4 + 15) & ~15;  // 2 x [2 halves x 128 rows] float2
  static constexpr int YB = RED + 2 * 256 * 8;       // y_t: 2 x [256 threads x 16 B], thread-private
  static constexpr int BAR = YB + 2 * 256 * 16;
  static constexpr int SMEM = BAR + 64 + 1024;
  static constexpr int TMEM_COLS = 128;
  static constexpr int C_HID = 64;
  static constexpr int CTAS = 3;
};

__global__ void __launch_bounds__(256, Trans32Layout::CTAS) trans32_kernel(const TransGeom g) {
  using L = Trans32Layout;
  constexpr int T = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* par = reinterpret_cast<float*>(sm + L::PAR);
  float2* red = reinterpret_cast<float2*>(sm + L::RED);
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // two threads per token row: warps w and w + 4 share TMEM lane quarter w % 4 and
  // take the halves hf = 0, 1 of every row's columns
  const int row = (warp & 3) * 32 + lane, hf = warp >> 2;

  stage_kmajor(sm + L::W_QKV, g.wqkv, 3 * T, T, T);
  stage_kmajor(sm + L::W_PROJ, g.wproj, T, T, T);
  stage_kmajor(sm + L::W_0, g.w0, 4 * T, T, T);
  stage_kmajor(sm + L::W_2, g.w2, T, 4 * T, 64);
  for (int i = tid; i < L::P_N; i += blockDim.x) {
    float v;
    if (i < L::P_BPROJ) v = g.bqkv[i];
    else if (i < L::P_B0) v = g.bproj[i - L::P_BPROJ];
    else if (i < L::P_B2) v = g.b0[i - L::P_B0];
    else if (i < L::P_L1G) v = g.b2[i - L::P_B2];
    else if (i < L::P_L1B) v = g.ln1g[i - L::P_L1G];
    else if (i < L::P_L2G) v = g.ln1b[i - L::P_L1B];
    else if (i < L::P_L2B) v = g.ln2g[i - L::P_L2G];
    else if (i < L::P_RP) v = g.ln2b[i - L::P_L2B];
    else v = g.rp[i - L::P_RP] * 1.4426950408889634f;  // log2(e): scores are kept in base 2
    par[i] = v;
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, L::TMEM_COLS);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const uint32_t sb = smem_u32(sm);
  uint32_t phase = 0;

  const int slot = row >> 6, tok = row & 63;
  const int qi = tok >> 3, qj = tok & 7;
  const long n_pairs = (g.win.n_windows + 1) / 2;
  constexpr float kScaleLog2e = 0.17677669529663687f * 1.4426950408889634f;  // 32^-1/2 log2(e)

  auto locate = [&](long pr, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * pr + slot;
    lr = lc = st = false;
    if (pr >= n_pairs || win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
  auto sync_mma = [&]() {  // operands written and TMEM reads finished, by every thread
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
  };
  auto wait_mma = [&]() {
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);
    phase ^= 1;
    tc_fence_after();
  };
  auto pair_sum = [&](float a, float b) -> float2 {
    red[hf * 128 + row] = make_float2(a, b);
    __syncthreads();
    const float2 o = red[(hf ^ 1) * 128 + row];
    return make_float2(a + o.x, b + o.y);
  };
  // this thread's 16 channels of a T-wide row -> 16-byte chunks 2 hf, 2 hf + 1 of a
  // 64-byte swizzled row
  auto put16 = [&](uint32_t off, const float* o) {
#pragma unroll
    for (int c = 0; c < 2; ++c)
      *reinterpret_cast<uint4*>(sm + off + swz_off(row, 2 * hf + c, 64)) =
          make_uint4(pack_half2(o[8 * c], o[8 * c + 1]), pack_half2(o[8 * c + 2], o[8 * c + 3]),
                     pack_half2(o[8 * c + 4], o[8 * c + 5]), pack_half2(o[8 * c + 6], o[8 * c + 7]));
  };
  auto layer_norm16 = [&](const float* x, int pg, int pb, float* o) {
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      s1 += x[k];
      s2 += x[k] * x[k];
    }
    const float2 st = pair_sum(s1, s2);
    const float mu = st.x * (1.f / T);
    const float rstd = rsqrtf(fmaxf(st.y * (1.f / T) - mu * mu, 0.f) + 1e-5f);
    const float4* g4 = reinterpret_cast<const float4*>(par + pg + hf * 16);
    const float4* b4 = reinterpret_cast<const float4*>(par + pb + hf * 16);
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 gg = g4[q], bb = b4[q];
      o[4 * q] = (x[4 * q] - mu) * rstd * gg.x + bb.x;
      o[4 * q + 1] = (x[4 * q + 1] - mu) * rstd * gg.y + bb.y;
      o[4 * q + 2] = (x[4 * q + 2] - mu) * rstd * gg.z + bb.z;
      o[4 * q + 3] = (x[4 * q + 3] - mu) * rstd * gg.w + bb.w;
    }
  };
  auto unpack16 = [](const uint4* src, float* dst) {
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&src[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        dst[8 * c + 2 * j] = f.x;
        dst[8 * c + 2 * j + 1] = f.y;
      }
    }
  };
  // this thread's 16 channels of the token's y_t row, fetched asynchronously into
  // its private 32 bytes of YB (zeros past the image) and read back where used
  auto fetch_y = [&](long pix) {
    const __half* src = pix >= 0 ? g.y + pix * T + hf * 16 : g.y;
#pragma unroll
    for (int c = 0; c < 2; ++c) cp_async16(sm + L::YB + c * 4096 + tid * 16, src + 8 * c, pix >= 0);
    cp_async_commit();
  };
  auto read_y = [&](float* yt) {
    uint4 u[2];
#pragma unroll
    for (int c = 0; c < 2; ++c) u[c] = *reinterpret_cast<const uint4*>(sm + L::YB + c * 4096 + tid * 16);
    unpack16(u, yt);
  };

  long pair = blockIdx.x;
  bool last_row, last_col, store;
  long pix = locate(pair, last_row, last_col, store);
  fetch_y(pix);

  for (; pair < n_pairs; pair += gridDim.x) {
    cp_async_wait_all();

    // ---- LN1 -> A1; qkv = A1 . Wqkv^T -> TMEM [0, 96) ----
    {
      float yt[16], o[16];
      read_y(yt);
      layer_norm16(yt, L::P_L1G, L::P_L1B, o);
      put16(L::R_A1, o);
    }
    sync_mma();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 3 * T);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(sb + L::R_A1 + k * 32, 64, SW_64B), make_sdesc(sb + L::W_QKV + k * 32, 64, SW_64B),
                 id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- q, k -> Q, K; v -> V^T; S = Q K^T -> TMEM [0, 128) ----
    {
      float q[16], k[16];
      tmem_ld16x2(trow + hf * 16, q, trow + T + hf * 16, k);
      const float4* bq4 = reinterpret_cast<const float4*>(par + L::P_BQKV + hf * 16);
      const float4* bk4 = reinterpret_cast<const float4*>(par + L::P_BQKV + T + hf * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 bq = bq4[j], bk = bk4[j];
        q[4 * j] += bq.x; q[4 * j + 1] += bq.y; q[4 * j + 2] += bq.z; q[4 * j + 3] += bq.w;
        k[4 * j] += bk.x; k[4 * j + 1] += bk.y; k[4 * j + 2] += bk.z; k[4 * j + 3] += bk.w;
      }
      put16(L::R_Q, q);
      put16(L::R_K, k);
    }
    {
      float v[16];
      tmem_ld16(trow + 2 * T + hf * 16, v);
      const float4* bv4 = reinterpret_cast<const float4*>(par + L::P_BQKV + 2 * T + hf * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 bv = bv4[j];
        v[4 * j] += bv.x; v[4 * j + 1] += bv.y; v[4 * j + 2] += bv.z; v[4 * j + 3] += bv.w;
      }
      uint8_t* vb = sm + L::VT + slot * 4096;
#pragma unroll
      for (int d = 0; d < 16; ++d)
        *reinterpret_cast<__half*>(vb + swz_off(hf * 16 + d, tok >> 3, 128) + (tok & 7) * 2) = __float2half_rn(v[d]);
    }
    sync_mma();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(sb + L::R_Q + k * 32, 64, SW_64B), make_sdesc(sb + L::R_K + k * 32, 64, SW_64B), id,
                 k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- softmax over the row's 64 in-window keys (32 per thread) -> P' ----
    float sum;
    {
      float s[32];
      tmem_ld16x2(trow + slot * 64 + hf * 32, s, trow + slot * 64 + hf * 32 + 16, s + 16);
      const float* bh = par + L::P_RP + (qi + 7) * 15 + (qj + 7);  // bias(key) = bh[-(15 ki + kj)]
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int kt = hf * 32 + j;
        s[j] = fmaf(s[j], kScaleLog2e, bh[-((kt >> 3) * 15 + (kt & 7))]);
      }
      if (last_row || last_col) {  // warp-uniform: the warp's tokens share a window
        // the cyclic shift put tokens from opposite image edges into windows of the
        // last window row / column; a token attends only to keys from its own side
        // (cuda/scunet.cu:137-147). Key hf*32 + j sits in window row 4 hf + j / 8
        // (top half iff hf = 0) and column j % 8.
        const bool rmask = last_row && ((qi < 4) != (hf == 0));
        const bool qleft = qj < 4;
#pragma unroll
        for (int j = 0; j < 32; ++j) s[j] = (rmask || (last_col && (qleft != ((j & 7) < 4)))) ? -INFINITY : s[j];
      }
#pragma unroll
      for (int j = 0; j < 32; ++j) mx = fmaxf(mx, s[j]);
      red[hf * 128 + row].x = mx;
      __syncthreads();
      mx = fmaxf(mx, red[(hf ^ 1) * 128 + row].x);
      sum = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float e = ex2_approx(s[j] - mx);
        s[j] = e;
        sum += e;
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(sm + L::R_P + swz_off(row, hf * 4 + c, 128)) =
            make_uint4(pack_half2(s[8 * c], s[8 * c + 1]), pack_half2(s[8 * c + 2], s[8 * c + 3]),
                       pack_half2(s[8 * c + 4], s[8 * c + 5]), pack_half2(s[8 * c + 6], s[8 * c + 7]));
      red[256 + hf * 128 + row].x = sum;  // second exchange slot: no barrier needed before this write
    }
    sync_mma();
    sum += red[256 + (hf ^ 1) * 128 + row].x;
    if (tid == 0) {  // O' = P' . [V_0 | V_1]  -> TMEM [0, 64)
      constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16(tmem, make_sdesc(sb + L::R_P + k * 32, 128, SW_128B), make_sdesc(sb + L::VT + k * 32, 128, SW_128B),
                 id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- O / sum -> O; proj = O . Wproj^T -> TMEM [0, 32) ----
    {
      float o[16];
      tmem_ld16(trow + slot * 32 + hf * 16, o);  // this token's window's half of O'
      const float inv = 1.f / sum;
#pragma unroll
      for (int j = 0; j < 16; ++j) o[j] *= inv;
      put16(L::R_O, o);
    }
    sync_mma();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(sb + L::R_O + k * 32, 64, SW_64B), make_sdesc(sb + L::W_PROJ + k * 32, 64, SW_64B),
                 id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- x1 = proj + y_t + b_proj, back into TMEM [0, 32) where mlp2 accumulates
    //      onto it; LN2 -> A1; hid_0 = A1 . W0[0:64]^T -> TMEM [64, 128) ----
    bool lr_n, lc_n, st_n;
    long pix_n;
    {
      float x1[16], o[16], yt[16];
      tmem_ld16(trow + hf * 16, x1);
      read_y(yt);
      const float4* bp4 = reinterpret_cast<const float4*>(par + L::P_BPROJ + hf * 16);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const float4 b = bp4[q];
        x1[4 * q] += yt[4 * q] + b.x;
        x1[4 * q + 1] += yt[4 * q + 1] + b.y;
        x1[4 * q + 2] += yt[4 * q + 2] + b.z;
        x1[4 * q + 3] += yt[4 * q + 3] + b.w;
      }
      tmem_st16(trow + hf * 16, x1);
      layer_norm16(x1, L::P_L2G, L::P_L2B, o);
      put16(L::R_A1, o);
      tmem_wait_st();
      // the next pair's y_t is fetched while this pair's MLP runs (YB is free now)
      pix_n = locate(pair + gridDim.x, lr_n, lc_n, st_n);
      fetch_y(pix_n);
    }
    sync_mma();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem + L::C_HID, make_sdesc(sb + L::R_A1 + k * 32, 64, SW_64B),
                 make_sdesc(sb + L::W_0 + k * 32, 64, SW_64B), id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- MLP: two 64-wide hidden chunks; mlp2 accumulates onto proj in [0, 32) ----
#pragma unroll 1
    for (int j = 0; j < 2; ++j) {
      {
        float hv[32];
        tmem_ld16x2(trow + L::C_HID + hf * 32, hv, trow + L::C_HID + hf * 32 + 16, hv + 16);
        const float4* b4 = reinterpret_cast<const float4*>(par + L::P_B0 + j * 64 + hf * 32);
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b = b4[q];
          __half2 a0 = __floats2half2_rn(hv[4 * q] + b.x, hv[4 * q + 1] + b.y);
          __half2 a1 = __floats2half2_rn(hv[4 * q + 2] + b.z, hv[4 * q + 3] + b.w);
          a0 = gelu_tanh_h2(a0);
          a1 = gelu_tanh_h2(a1);
          pk[2 * q] = *reinterpret_cast<uint32_t*>(&a0);
          pk[2 * q + 1] = *reinterpret_cast<uint32_t*>(&a1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(sm + L::R_H + swz_off(row, hf * 4 + q, 128)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      sync_mma();
      if (tid == 0) {
        {
          constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem, make_sdesc(sb + L::R_H + k * 32, 128, SW_128B),
                     make_sdesc(sb + L::W_2 + j * T * 128 + k * 32, 128, SW_128B), id, 1);
        }
        if (j == 0) {  // the second chunk's hidden layer, behind the first chunk's output
          constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
          for (int k = 0; k < 2; ++k)
            umma_f16(tmem + L::C_HID, make_sdesc(sb + L::R_A1 + k * 32, 64, SW_64B),
                     make_sdesc(sb + L::W_0 + 64 * 64 + k * 32, 64, SW_64B), id, k);
        }
        umma_commit(bar);
      }
      wait_mma();
    }

    // ---- z = acc + b_2 (acc = x1 + mlp2) -> Z[:, 32:64) ----
    {
      float m[16];
      tmem_ld16(trow + hf * 16, m);
      if (pix >= 0 && store) {
        const float4* b24 = reinterpret_cast<const float4*>(par + L::P_B2 + hf * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float4 b2 = b24[q];
          m[4 * q] += b2.x;
          m[4 * q + 1] += b2.y;
          m[4 * q + 2] += b2.z;
          m[4 * q + 3] += b2.w;
        }
        uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T + hf * 16);
#pragma unroll
        for (int c = 0; c < 2; ++c)
          dst[c] = make_uint4(pack_half2(m[8 * c], m[8 * c + 1]), pack_half2(m[8 * c + 2], m[8 * c + 3]),
                              pack_half2(m[8 * c + 4], m[8 * c + 5]), pack_half2(m[8 * c + 6], m[8 * c + 7]));
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and shared memory are reused by the next pair
    tc_fence_after();
    pix = pix_n;
    last_row = lr_n;
    last_col = lc_n;
    store = st_n;
  }
  cp_async_wait_all();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace scb
