// The transformer half of a half-resolution ConvTransBlock (trans width T = 64, two
// heads of 32) in one kernel per launch (common structure and semantics: trans.cuh),
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136)
//
// organised as TWO independent pair pipelines per CTA. The block's weights (96 KB
// fp16) fill most of an SM's shared memory, so only one CTA fits; one pipeline per
// CTA leaves the SM idle whenever its MMA round trip is in flight. Here warps 0-7
// and 8-15 each walk their own pairs of 8x8 windows with their own named barrier,
// mbarrier, MMA-issuing thread, 256 TMEM columns and 52 KB of shared memory, and
// share the resident weights: while one pipeline waits on the tensor core the other
// runs its CUDA-core work.
//
// Per pipeline: accumulators are read out before
// the MMA that overwrites them is issued (qkv [0, 192) -> S [0, 128), O'_0 [128, 192),
// O'_1 [192, 256) -> proj/acc [0, 64), hidden [64, 128)); one 32 KB region holds in
// turn LN1, Q|K of both heads, P'_0 | P'_1, O | P'_1, LN2 | hidden chunk; P'_h . [V_0 |
// V_1] replaces the zero-padded P.V; scores carry log2(e); the SW mask is evaluated
// only on edge windows; GELU is the packed fp16 tanh form; the hidden layer runs in
// four 64-wide chunks, each chunk's mlp0 MMA issued behind the previous chunk's mlp2.
#pragma once
#include "trans.cuh"

namespace scb {

struct Trans64Layout {
  static constexpr int T = 64;
  static constexpr int W_QKV = 0;                    // [192 x 128 B], SW128
  static constexpr int W_PROJ = W_QKV + 192 * 128;   // [64 x 128 B]
  static constexpr int W_0 = W_PROJ + 64 * 128;      // [256 x 128 B]
  static constexpr int W_2 = W_0 + 256 * 128;        // 4 K-blocks of [64 x 128 B]
  static constexpr int PIPE = W_2 + 4 * 64 * 128;    // two pipeline areas (1024-aligned)
  static constexpr int PIPE_BYTES = 53248;
  // within a pipeline area
  static constexpr int R = 0;                        // 32 KB reused region
  static constexpr int VT = 32768;                   // 2 heads x [V_0 | V_1]^T [64 x 128 B]
  static constexpr int RED = VT + 16384;             // 2 slots x [2 halves x 128 rows] float2
  static constexpr int PAR = PIPE + 2 * PIPE_BYTES;
  static constexpr int P_BQKV = 0, P_BPROJ = 3 * T, P_B0 = 4 * T, P_B2 = 8 * T, P_L1G = 9 * T, P_L1B = 10 * T,
                       P_L2G = 11 * T, P_L2B = 12 * T, P_RP = 13 * T, P_N = 13 * T + 2 * 225;
  static constexpr int BAR = (PAR + P_N * 4 + 15) & ~15;
  static constexpr int SMEM = BAR + 64 + 1024;
  static constexpr int TMEM_COLS = 512;              // 256 per pipeline
};

__device__ __forceinline__ void pipe_sync(int id) { asm volatile("bar.sync %0, 256;" ::"r"(id) : "memory"); }

__global__ void __launch_bounds__(512, 1) trans64_kernel(const TransGeom g) {
  using L = Trans64Layout;
  constexpr int T = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* par = reinterpret_cast<float*>(sm + L::PAR);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 2);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int pp = warp >> 3;                 // pipeline
  const int ptid = tid & 255, pwarp = warp & 7;
  // two threads per token row: pipeline warps w and w + 4 share TMEM lane quarter
  // w % 4 (= warp % 4) and take the halves hf = 0, 1 of every row's columns
  const int row = (pwarp & 3) * 32 + lane, hf = pwarp >> 2;
  uint8_t* pa = sm + L::PIPE + pp * L::PIPE_BYTES;
  float2* red = reinterpret_cast<float2*>(pa + L::RED);
  uint64_t* bar = bars + pp;

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
    mbar_init(bars, 1);
    mbar_init(bars + 1, 1);
    mbar_fence_init();
  }
  if (warp == 0) tmem_alloc(tmem_slot, L::TMEM_COLS);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tp = *tmem_slot + 256u * pp;  // this pipeline's columns
  const uint32_t trow = tp + ((uint32_t)((pwarp & 3) * 32) << 16);
  const uint32_t sb = smem_u32(sm);
  const uint32_t pb = smem_u32(pa);
  uint32_t phase = 0;
  const bool issuer = ptid == 0;

  const int slot = row >> 6, tok = row & 63;
  const int qi = tok >> 3, qj = tok & 7;
  const long n_pairs = (g.win.n_windows + 1) / 2;
  constexpr float kScaleLog2e = 0.17677669529663687f * 1.4426950408889634f;  // 32^-1/2 log2(e)
  uint32_t mrow = 0, mcol = 0;  // shifted-window mask over this thread's 32 keys
#pragma unroll
  for (int j = 0; j < 32; ++j) {
    const int kt = hf * 32 + j;
    mrow |= (uint32_t)((qi < 4) != ((kt >> 3) < 4)) << j;
    mcol |= (uint32_t)((qj < 4) != ((kt & 7) < 4)) << j;
  }

  auto locate = [&](long pr, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * pr + slot;
    lr = lc = st = false;
    if (pr >= n_pairs || win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
  auto sync_mma = [&]() {  // this pipeline's operands written and TMEM reads finished
    fence_proxy_async_smem();
    tc_fence_before();
    pipe_sync(1 + pp);
    tc_fence_after();
  };
  auto wait_mma = [&]() {
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);
    phase ^= 1;
    tc_fence_after();
  };
  // this thread's 32 channels of a 64-wide row -> 16-byte chunks 4 hf .. 4 hf + 3 of a
  // 128-byte swizzled row
  auto put32 = [&](uint32_t off, const float* o) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(pa + off + swz_off(row, 4 * hf + c, 128)) =
          make_uint4(pack_half2(o[8 * c], o[8 * c + 1]), pack_half2(o[8 * c + 2], o[8 * c + 3]),
                     pack_half2(o[8 * c + 4], o[8 * c + 5]), pack_half2(o[8 * c + 6], o[8 * c + 7]));
  };
  // LayerNorm of a row from this thread's 32 values (x) and its partner's, in place
  auto layer_norm32 = [&](float* x, int pg, int pbeta) {
    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < 32; ++k) {
      s1 += x[k];
      s2 += x[k] * x[k];
    }
    red[hf * 128 + row] = make_float2(s1, s2);
    pipe_sync(1 + pp);
    const float2 o = red[(hf ^ 1) * 128 + row];
    const float mu = (s1 + o.x) * (1.f / T);
    const float rstd = rsqrtf(fmaxf((s2 + o.y) * (1.f / T) - mu * mu, 0.f) + 1e-5f);
    const float4* g4 = reinterpret_cast<const float4*>(par + pg + hf * 32);
    const float4* b4 = reinterpret_cast<const float4*>(par + pbeta + hf * 32);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      const float4 gg = g4[q], bb = b4[q];
      x[4 * q] = (x[4 * q] - mu) * rstd * gg.x + bb.x;
      x[4 * q + 1] = (x[4 * q + 1] - mu) * rstd * gg.y + bb.y;
      x[4 * q + 2] = (x[4 * q + 2] - mu) * rstd * gg.z + bb.z;
      x[4 * q + 3] = (x[4 * q + 3] - mu) * rstd * gg.w + bb.w;
    }
  };
  auto unpack32 = [](const uint4* src, float* dst) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&src[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        dst[8 * c + 2 * j] = f.x;
        dst[8 * c + 2 * j + 1] = f.y;
      }
    }
  };
  // bias-added q, k (16 channels each) of head h -> Q_h, K_h; v -> V_h^T
  auto stage_qkv = [&](int h) {
    {
      float q[16], k[16];
      tmem_ld16x2(trow + h * 32 + hf * 16, q, trow + T + h * 32 + hf * 16, k);
      const float4* bq4 = reinterpret_cast<const float4*>(par + L::P_BQKV + h * 32 + hf * 16);
      const float4* bk4 = reinterpret_cast<const float4*>(par + L::P_BQKV + T + h * 32 + hf * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 bq = bq4[j], bk = bk4[j];
        q[4 * j] += bq.x; q[4 * j + 1] += bq.y; q[4 * j + 2] += bq.z; q[4 * j + 3] += bq.w;
        k[4 * j] += bk.x; k[4 * j + 1] += bk.y; k[4 * j + 2] += bk.z; k[4 * j + 3] += bk.w;
      }
      uint8_t* qs = pa + L::R + h * 16384;
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        *reinterpret_cast<uint4*>(qs + swz_off(row, 2 * hf + c, 64)) =
            make_uint4(pack_half2(q[8 * c], q[8 * c + 1]), pack_half2(q[8 * c + 2], q[8 * c + 3]),
                       pack_half2(q[8 * c + 4], q[8 * c + 5]), pack_half2(q[8 * c + 6], q[8 * c + 7]));
        *reinterpret_cast<uint4*>(qs + 8192 + swz_off(row, 2 * hf + c, 64)) =
            make_uint4(pack_half2(k[8 * c], k[8 * c + 1]), pack_half2(k[8 * c + 2], k[8 * c + 3]),
                       pack_half2(k[8 * c + 4], k[8 * c + 5]), pack_half2(k[8 * c + 6], k[8 * c + 7]));
      }
    }
    {
      float v[16];
      tmem_ld16(trow + 2 * T + h * 32 + hf * 16, v);
      const float4* bv4 = reinterpret_cast<const float4*>(par + L::P_BQKV + 2 * T + h * 32 + hf * 16);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float4 bv = bv4[j];
        v[4 * j] += bv.x; v[4 * j + 1] += bv.y; v[4 * j + 2] += bv.z; v[4 * j + 3] += bv.w;
      }
      uint8_t* vb = pa + L::VT + h * 8192;
#pragma unroll
      for (int d = 0; d < 16; ++d)
        *reinterpret_cast<__half*>(vb + swz_off(slot * 32 + hf * 16 + d, tok >> 3, 128) + (tok & 7) * 2) =
            __float2half_rn(v[d]);
    }
  };
  // softmax of head h's scores (TMEM [0, 128)) over the row's 64 in-window keys ->
  // P'_h at region offset 16 KB h; returns this thread's partial sum
  auto softmax = [&](int h, bool last_row, bool last_col) -> float {
    float s[32];
    tmem_ld16x2(trow + slot * 64 + hf * 32, s, trow + slot * 64 + hf * 32 + 16, s + 16);
    const float* bh = par + L::P_RP + h * 225 + (qi + 7) * 15 + (qj + 7);
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
    float* rm = reinterpret_cast<float*>(red);  // slot 0: head h's max in component h
    rm[2 * (hf * 128 + row) + h] = mx;
    pipe_sync(1 + pp);
    mx = fmaxf(mx, rm[2 * ((hf ^ 1) * 128 + row) + h]);
    float sum = 0.f;
#pragma unroll
    for (int j = 0; j < 32; ++j) {
      const float e = ex2_approx(s[j] - mx);
      s[j] = e;
      sum += e;
    }
    uint8_t* pr = pa + L::R + h * 16384;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(pr + swz_off(row, hf * 4 + c, 128)) =
          make_uint4(pack_half2(s[8 * c], s[8 * c + 1]), pack_half2(s[8 * c + 2], s[8 * c + 3]),
                     pack_half2(s[8 * c + 4], s[8 * c + 5]), pack_half2(s[8 * c + 6], s[8 * c + 7]));
    rm[2 * (256 + hf * 128 + row) + h] = sum;  // slot 1: head h's sum in component h
    return sum;
  };
  // O'_h (TMEM [128 + 64 h, ...)) / sum -> head h's channels of O (region offset 0)
  auto put_o = [&](int h, float inv) {
    float o[16];
    tmem_ld16(trow + 128 + 64 * h + slot * 32 + hf * 16, o);
#pragma unroll
    for (int c = 0; c < 2; ++c)
      *reinterpret_cast<uint4*>(pa + L::R + swz_off(row, 4 * h + 2 * hf + c, 128)) =
          make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv), pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                     pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                     pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
  };
  auto mma_pv = [&](int h) {  // O'_h = P'_h . [V_0 | V_1]_h -> TMEM [128 + 64 h, +64)
    constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_f16(tp + 128 + 64 * h, make_sdesc(pb + L::R + h * 16384 + k * 32, 128, SW_128B),
               make_sdesc(pb + L::VT + h * 8192 + k * 32, 128, SW_128B), id, k);
  };
  auto mma_s = [&](int h) {  // S = Q_h K_h^T -> TMEM [0, 128)
    constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
    for (int k = 0; k < 2; ++k)
      umma_f16(tp, make_sdesc(pb + L::R + h * 16384 + k * 32, 64, SW_64B),
               make_sdesc(pb + L::R + h * 16384 + 8192 + k * 32, 64, SW_64B), id, k);
  };
  auto mma_hid = [&](int j) {  // hid_j = LN2 . W0[64 j : 64 j + 64]^T -> TMEM [64, 128)
    constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
    for (int k = 0; k < 4; ++k)
      umma_f16(tp + 64, make_sdesc(pb + L::R + k * 32, 128, SW_128B),
               make_sdesc(sb + L::W_0 + j * 64 * 128 + k * 32, 128, SW_128B), id, k);
  };
  auto load_y = [&](long pix, uint4* dst) {
#pragma unroll
    for (int c = 0; c < 4; ++c)
      dst[c] = pix >= 0 ? __ldg(reinterpret_cast<const uint4*>(g.y + pix * T + hf * 32) + c)
                        : make_uint4(0, 0, 0, 0);
  };

  long pair = 2L * blockIdx.x + pp;
  const long stride = 2L * gridDim.x;
  bool lr_n, lc_n, st_n;
  long pix_n = locate(pair, lr_n, lc_n, st_n);

  for (; pair < n_pairs; pair += stride) {
    const long pix = pix_n;
    const bool last_row = lr_n, last_col = lc_n, store = st_n;
    uint4 ycur[4];  // y_t stays packed (fp16 data)
    load_y(pix, ycur);
    pix_n = locate(pair + stride, lr_n, lc_n, st_n);
    if (pix_n >= 0) prefetch_l2(g.y + pix_n * T + hf * 32);

    // ---- LN1 -> A1; qkv -> TMEM [0, 192) ----
    {
      float a[32];
      unpack32(ycur, a);
      layer_norm32(a, L::P_L1G, L::P_L1B);
      put32(L::R, a);
    }
    sync_mma();
    if (issuer) {
      constexpr uint32_t id = make_idesc_f16(128, 3 * T);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16(tp, make_sdesc(pb + L::R + k * 32, 128, SW_128B), make_sdesc(sb + L::W_QKV + k * 32, 128, SW_128B),
                 id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- Q, K, V^T of both heads (TMEM qkv is then free); S_0 ----
    stage_qkv(0);
    stage_qkv(1);
    sync_mma();
    if (issuer) {
      mma_s(0);
      umma_commit(bar);
    }
    wait_mma();

    // ---- head 0 softmax -> P'_0; O'_0 = P'_0 [V]_0 and S_1 together ----
    const float sum0p = softmax(0, last_row, last_col);
    sync_mma();
    const float inv0 = 1.f / (sum0p + reinterpret_cast<const float*>(red)[2 * (256 + (hf ^ 1) * 128 + row)]);
    if (issuer) {
      mma_pv(0);
      mma_s(1);
      umma_commit(bar);
    }
    wait_mma();

    // ---- head 1 softmax -> P'_1; head 0's O -> O; O'_1 ----
    const float sum1p = softmax(1, last_row, last_col);
    put_o(0, inv0);
    sync_mma();
    const float inv1 = 1.f / (sum1p + reinterpret_cast<const float*>(red)[2 * (256 + (hf ^ 1) * 128 + row) + 1]);
    if (issuer) {
      mma_pv(1);
      umma_commit(bar);
    }
    wait_mma();

    // ---- head 1's O; proj = O . Wproj^T -> TMEM [0, 64) ----
    put_o(1, inv1);
    sync_mma();
    if (issuer) {
      constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16(tp, make_sdesc(pb + L::R + k * 32, 128, SW_128B), make_sdesc(sb + L::W_PROJ + k * 32, 128, SW_128B),
                 id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- x1 = proj + y_t + b_proj, back into TMEM [0, 64) where mlp2 accumulates
    //      onto it; LN2 -> A1; hid_0 ----
    {
      float x1[32], yt[32];
      tmem_ld16x2(trow + hf * 32, x1, trow + hf * 32 + 16, x1 + 16);
      unpack32(ycur, yt);
      const float4* bp4 = reinterpret_cast<const float4*>(par + L::P_BPROJ + hf * 32);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float4 b = bp4[q];
        x1[4 * q] += yt[4 * q] + b.x;
        x1[4 * q + 1] += yt[4 * q + 1] + b.y;
        x1[4 * q + 2] += yt[4 * q + 2] + b.z;
        x1[4 * q + 3] += yt[4 * q + 3] + b.w;
      }
      tmem_st16(trow + hf * 32, x1);
      tmem_st16(trow + hf * 32 + 16, x1 + 16);
      layer_norm32(x1, L::P_L2G, L::P_L2B);
      put32(L::R, x1);
      tmem_wait_st();
    }
    sync_mma();
    if (issuer) {
      mma_hid(0);
      umma_commit(bar);
    }
    wait_mma();

    // ---- MLP: four 64-wide hidden chunks; mlp2 accumulates onto proj in [0, 64) ----
#pragma unroll 1
    for (int j = 0; j < 4; ++j) {
      {
        float hv[32];
        tmem_ld16x2(trow + 64 + hf * 32, hv, trow + 64 + hf * 32 + 16, hv + 16);
        const float4* b4 = reinterpret_cast<const float4*>(par + L::P_B0 + j * 64 + hf * 32);
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b = b4[q];
          __half2 a0 = gelu_tanh_h2(__floats2half2_rn(hv[4 * q] + b.x, hv[4 * q + 1] + b.y));
          __half2 a1 = gelu_tanh_h2(__floats2half2_rn(hv[4 * q + 2] + b.z, hv[4 * q + 3] + b.w));
          pk[2 * q] = *reinterpret_cast<uint32_t*>(&a0);
          pk[2 * q + 1] = *reinterpret_cast<uint32_t*>(&a1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(pa + L::R + 16384 + swz_off(row, hf * 4 + q, 128)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      sync_mma();
      if (issuer) {
        constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16(tp, make_sdesc(pb + L::R + 16384 + k * 32, 128, SW_128B),
                   make_sdesc(sb + L::W_2 + j * T * 128 + k * 32, 128, SW_128B), id, 1);
        if (j < 3) mma_hid(j + 1);  // the next chunk's hidden layer, behind this chunk's output
        umma_commit(bar);
      }
      wait_mma();
    }

    // ---- z = acc + b_2 (acc = x1 + mlp2) -> Z[:, 64:128) ----
    {
      float m[32];
      tmem_ld16x2(trow + hf * 32, m, trow + hf * 32 + 16, m + 16);
      if (pix >= 0 && store) {
        const float4* b24 = reinterpret_cast<const float4*>(par + L::P_B2 + hf * 32);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b2 = b24[q];
          m[4 * q] += b2.x;
          m[4 * q + 1] += b2.y;
          m[4 * q + 2] += b2.z;
          m[4 * q + 3] += b2.w;
        }
        uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T + hf * 32);
#pragma unroll
        for (int c = 0; c < 4; ++c)
          dst[c] = make_uint4(pack_half2(m[8 * c], m[8 * c + 1]), pack_half2(m[8 * c + 2], m[8 * c + 3]),
                              pack_half2(m[8 * c + 4], m[8 * c + 5]), pack_half2(m[8 * c + 6], m[8 * c + 7]));
      }
    }
    tc_fence_before();
    pipe_sync(1 + pp);  // TMEM and shared memory are reused by the next pair
    tc_fence_after();
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(*tmem_slot, L::TMEM_COLS);
}

}  // namespace scb
