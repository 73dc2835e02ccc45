// The whole transformer half of a ConvTransBlock in one kernel, for the two
// widest stages (trans width T = 32 at full resolution, T = 64 at 1/2):
//
//   x  = y_t                                   (fp16 plane, columns [T, 2T) of Y)
//   x1 = x + proj(WMSA(LN1(x)))                (tools/network_scunet.py:134-135)
//   z  = x1 + mlp2(GELU(mlp0(LN2(x1))))        (tools/network_scunet.py:128-136)
//   -> columns [T, 2T) of Z (fp16), the conv1_2 operand.
//
// WMSA semantics are those of window_attn_kernel (attn.cuh): cyclic shift read in
// place, rel-pos bias, SW mask on the last window row/column, softmax, P.V.
//
// One CTA (256 threads, two per token row) walks pairs of 8x8 windows (128
// tokens) persistently. Every GEMM of the block runs on tcgen05 with its
// accumulator in TMEM and its operands in shared memory:
//
//   qkv   [128 x 3T] = LN1 [128 x T]  . Wqkv^T       (one UMMA chain, N = 3T)
//   S_h   [128 x 128] = Q_h . K_h^T                  (both windows at once; the
//         off-window half of each row is never read and P is zero there)
//   O_h   [128 x 32]  = P_h . V_h
//   proj  [128 x T]   = O . Wproj^T
//   hid_j [128 x 128] = LN2 . W0[j]^T                (hidden in 128-wide chunks)
//   mlp   [128 x T]  += GELU(hid_j) . W2[:, j]^T
//
// The weights of the block (24 KB at T = 32, 96 KB at T = 64, fp16) stay in
// shared memory for the CTA's lifetime; the next pair's tokens are prefetched
// into registers while the current pair computes. HBM traffic is one read of y_t
// and one write of z_t per token.
#pragma once
#include "ptx.cuh"

namespace scb {

struct TransGeom {
  WinGeom win;
  const __half* y;    // Y plane, pixel stride 2T, trans half at column T
  __half* z;          // Z plane, pixel stride 2T, output at column T
  const __half* wqkv; // [3T][T]
  const __half* wproj;// [T][T]
  const __half* w0;   // [4T][T]
  const __half* w2;   // [T][4T]
  const float *bqkv, *bproj, *b0, *b2, *ln1g, *ln1b, *ln2g, *ln2b, *rp;
};

template <int T>
struct TransLayout {
  static constexpr int HEADS = T / 32;
  static constexpr int RB = T * 2;  // bytes of a T-wide fp16 row (64 or 128 = the swizzle span)
  static constexpr uint32_t SWZ = (T == 32) ? SW_64B : SW_128B;
  static constexpr int W_QKV = 0;
  static constexpr int W_PROJ = W_QKV + 3 * T * RB;
  static constexpr int W_0 = W_PROJ + T * RB;
  static constexpr int W_2 = W_0 + 4 * T * RB;          // (4T/64) K-blocks of [T rows x 128 B]
  static constexpr int A1 = W_2 + 4 * T * 2 * T;         // LN1 out, then LN2 out
  static constexpr int QS = A1 + 128 * RB;
  static constexpr int KS = QS + 128 * 64;
  static constexpr int VT = KS + 128 * 64;               // 2 x [32 x 128 B]
  static constexpr int PS = VT + 2 * 32 * 128;           // 2 x [128 x 128 B]; also the MLP hidden chunk
  static constexpr int OS = PS + 2 * 128 * 128;
  static constexpr int PAR = OS + 128 * RB;              // fp32 parameters
  static constexpr int P_BQKV = 0, P_BPROJ = 3 * T, P_B0 = 4 * T, P_B2 = 8 * T, P_L1G = 9 * T, P_L1B = 10 * T,
                       P_L2G = 11 * T, P_L2B = 12 * T, P_RP = 13 * T, P_N = 13 * T + HEADS * 225;
  static constexpr int RED = (PAR + P_N * 4 + 15) & ~15;  // 2 x [2 halves x 128 rows] float2
  static constexpr int BAR = RED + 2 * 256 * 8;
  static constexpr int SMEM = BAR + 64 + 1024;
  // TMEM columns
  static constexpr int C_QKV = 0, C_O = 3 * T, C_S = 4 * T, C_PROJ = 0, C_MLP2 = T, C_HID = 4 * T;
  static constexpr int TMEM_COLS = (T == 32) ? 256 : 512;
  static constexpr int CTAS = (T == 32) ? 2 : 1;
};

// Copy a row-major fp16 [R][K] matrix into K-major swizzled tiles: K split into
// blocks of `kblk` elements (kblk*2 = row bytes = swizzle span), block b at
// dst + b * R * kblk * 2.
__device__ __forceinline__ void stage_kmajor(uint8_t* dst, const __half* src, int R, int K, int kblk) {
  const int rb = kblk * 2, cpr = K / 8, cpb = kblk / 8;
  for (int idx = threadIdx.x; idx < R * cpr; idx += blockDim.x) {
    const int r = idx / cpr, j = idx - r * cpr;
    const int b = j / cpb, jj = j - b * cpb;
    *reinterpret_cast<uint4*>(dst + b * R * rb + swz_off(r, jj, rb)) =
        __ldg(reinterpret_cast<const uint4*>(src + (long)r * K + j * 8));
  }
}

__device__ __forceinline__ float gelu_f(float x) { return gelu_as(x); }

template <int T>
__global__ void __launch_bounds__(256, TransLayout<T>::CTAS) trans_fused_kernel(const TransGeom g) {
  using L = TransLayout<T>;
  // Two threads per token row: warps w and w + 4 share TMEM lane quarter w % 4 and
  // split every row's columns in halves (hf = 0, 1); row statistics (LayerNorm
  // moments, softmax max and sum) are combined through `red`.
  constexpr int HALF = T / 2;           // columns of a T-wide row per thread
  constexpr int NCH = HALF / 8;         // 16-byte chunks per half row
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  float* par = reinterpret_cast<float*>(sm + L::PAR);
  float2* red = reinterpret_cast<float2*>(sm + L::RED);  // [2 halves][128 rows]
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane, hf = warp >> 2;

  // ---- once per CTA: weights and parameters into shared memory ----
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
    else v = g.rp[i - L::P_RP];
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
  constexpr float kScale = 0.17677669529663687f;  // 32^-1/2
  constexpr float kLog2e = 1.4426950408889634f;

  // token -> pixel of pair `pr` (or -1 when the window does not exist); `st`:
  // whether this token's output is stored (band halo rows are not)
  auto locate = [&](long pr, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * pr + slot;
    lr = lc = st = false;
    if (pr >= n_pairs || win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
  auto sync_mma = [&]() {  // all threads: operands written, TMEM reads finished
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
  // combine a per-half pair of partial sums with the partner thread
  auto pair_sum = [&](float a, float b) -> float2 {
    red[hf * 128 + row] = make_float2(a, b);
    __syncthreads();
    const float2 o = red[(hf ^ 1) * 128 + row];
    return make_float2(a + o.x, b + o.y);
  };
  auto load_half = [&](long pix, uint4* dst) {
#pragma unroll
    for (int c = 0; c < NCH; ++c)
      dst[c] = pix >= 0 ? __ldg(reinterpret_cast<const uint4*>(g.y + pix * (2 * T) + T + hf * HALF) + c)
                        : make_uint4(0, 0, 0, 0);
  };

  long pair = blockIdx.x;
  bool lr_n, lc_n, st_n;
  long pix_n = locate(pair, lr_n, lc_n, st_n);
  uint4 nx[NCH];
  load_half(pix_n, nx);

  for (; pair < n_pairs; pair += gridDim.x) {
    const long pix = pix_n;
    const bool last_row = lr_n, last_col = lc_n, store = st_n;
    uint4 cur[NCH];
#pragma unroll
    for (int c = 0; c < NCH; ++c) cur[c] = nx[c];
    pix_n = locate(pair + gridDim.x, lr_n, lc_n, st_n);
    load_half(pix_n, nx);

    float yt[HALF];  // this thread's half of y_t (the first residual)
#pragma unroll
    for (int c = 0; c < NCH; ++c) {
      const __half2* h2 = reinterpret_cast<const __half2*>(&cur[c]);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h2[j]);
        yt[8 * c + 2 * j] = f.x;
        yt[8 * c + 2 * j + 1] = f.y;
      }
    }

    // ---- LN1 -> A1 (this thread's half of the row) ----
    {
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int k = 0; k < HALF; ++k) {
        s1 += yt[k];
        s2 += yt[k] * yt[k];
      }
      const float2 st = pair_sum(s1, s2);
      const float mu = st.x * (1.f / T);
      const float rstd = rsqrtf(fmaxf(st.y * (1.f / T) - mu * mu, 0.f) + 1e-5f);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float o[8];
        const int k0 = hf * HALF + 8 * c;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (yt[8 * c + j] - mu) * rstd * par[L::P_L1G + k0 + j] + par[L::P_L1B + k0 + j];
        *reinterpret_cast<uint4*>(sm + L::A1 + swz_off(row, hf * NCH + c, L::RB)) =
            make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
      }
      // the other window's key half of P must read as zero in every P.V product
      uint8_t* pz = sm + L::PS + (slot ^ 1) * 16384;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(pz + swz_off(row, hf * 4 + c, 128)) = make_uint4(0, 0, 0, 0);
    }
    sync_mma();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 3 * T);
#pragma unroll
      for (int k = 0; k < T / 16; ++k)
        umma_f16(tmem + L::C_QKV, make_sdesc(sb + L::A1 + k * 32, L::RB, L::SWZ),
                 make_sdesc(sb + L::W_QKV + k * 32, L::RB, L::SWZ), id, k);
      umma_commit(bar);
    }
    wait_mma();

    // ---- window attention, head by head ----
    for (int h = 0; h < L::HEADS; ++h) {
      {
        // this thread's 16 of the head's 32 channels of q, k, v
        float q[16], k[16], v[16];
        const int c0 = h * 32 + hf * 16;
        tmem_ld16x3(trow + L::C_QKV + c0, q, trow + L::C_QKV + T + c0, k, trow + L::C_QKV + 2 * T + c0, v);
        const float4* bq4 = reinterpret_cast<const float4*>(par + L::P_BQKV + c0);
        const float4* bk4 = reinterpret_cast<const float4*>(par + L::P_BQKV + T + c0);
        const float4* bv4 = reinterpret_cast<const float4*>(par + L::P_BQKV + 2 * T + c0);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float4 bq = bq4[j], bk = bk4[j], bv = bv4[j];
          q[4 * j] += bq.x; q[4 * j + 1] += bq.y; q[4 * j + 2] += bq.z; q[4 * j + 3] += bq.w;
          k[4 * j] += bk.x; k[4 * j + 1] += bk.y; k[4 * j + 2] += bk.z; k[4 * j + 3] += bk.w;
          v[4 * j] += bv.x; v[4 * j + 1] += bv.y; v[4 * j + 2] += bv.z; v[4 * j + 3] += bv.w;
        }
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float a[8], b[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            a[j] = q[8 * c + j];
            b[j] = k[8 * c + j];
          }
          *reinterpret_cast<uint4*>(sm + L::QS + swz_off(row, 2 * hf + c, 64)) =
              make_uint4(pack_half2(a[0], a[1]), pack_half2(a[2], a[3]), pack_half2(a[4], a[5]), pack_half2(a[6], a[7]));
          *reinterpret_cast<uint4*>(sm + L::KS + swz_off(row, 2 * hf + c, 64)) =
              make_uint4(pack_half2(b[0], b[1]), pack_half2(b[2], b[3]), pack_half2(b[4], b[5]), pack_half2(b[6], b[7]));
        }
        uint8_t* vb = sm + L::VT + slot * 4096;
        const uint32_t kk = row & 63;
#pragma unroll
        for (int d = 0; d < 16; ++d)
          *reinterpret_cast<__half*>(vb + swz_off(hf * 16 + d, kk >> 3, 128) + (kk & 7) * 2) = __float2half_rn(v[d]);
      }
      sync_mma();
      if (tid == 0) {
        constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
        for (int k = 0; k < 2; ++k)
          umma_f16(tmem + L::C_S, make_sdesc(sb + L::QS + k * 32, 64, SW_64B), make_sdesc(sb + L::KS + k * 32, 64, SW_64B),
                   id, k);
        umma_commit(bar);
      }
      wait_mma();
      // this thread's 32 of the row's 64 in-window keys
      float s[32];
      tmem_ld16x2(trow + L::C_S + slot * 64 + hf * 32, s, trow + L::C_S + slot * 64 + hf * 32 + 16, s + 16);
      const float* bh = par + L::P_RP + h * 225;
      float mx = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int kt = hf * 32 + j;
        const int ki = kt >> 3, kj = kt & 7;
        float v = s[j] * kScale + bh[(qi - ki + 7) * 15 + (qj - kj + 7)];
        const bool masked = (last_row && ((qi < 4) != (ki < 4))) || (last_col && ((qj < 4) != (kj < 4)));
        v = masked ? -INFINITY : v;
        s[j] = v;
        mx = fmaxf(mx, v);
      }
      red[hf * 128 + row].x = mx;
      __syncthreads();
      mx = fmaxf(mx, red[(hf ^ 1) * 128 + row].x);
      float sum = 0.f;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const float e = ex2_approx((s[j] - mx) * kLog2e);
        s[j] = e;
        sum += e;
      }
      {
        uint8_t* pr = sm + L::PS + slot * 16384;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(pr + swz_off(row, hf * 4 + c, 128)) =
              make_uint4(pack_half2(s[8 * c], s[8 * c + 1]), pack_half2(s[8 * c + 2], s[8 * c + 3]),
                         pack_half2(s[8 * c + 4], s[8 * c + 5]), pack_half2(s[8 * c + 6], s[8 * c + 7]));
      }
      red[256 + hf * 128 + row].x = sum;  // second exchange slot: no barrier needed before this write
      sync_mma();
      sum += red[256 + (hf ^ 1) * 128 + row].x;
      if (tid == 0) {
        constexpr uint32_t id = make_idesc_f16(128, 32);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + L::C_O + h * 32, make_sdesc(sb + L::PS + kb * 16384 + k * 32, 128, SW_128B),
                     make_sdesc(sb + L::VT + kb * 4096 + k * 32, 128, SW_128B), id, (kb | k) != 0);
        umma_commit(bar);
      }
      wait_mma();
      {
        float o[16];
        tmem_ld16(trow + L::C_O + h * 32 + hf * 16, o);
        const float inv = 1.f / sum;
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          // head h occupies 16-byte chunks [4h, 4h + 4) of the T-wide O row
          *reinterpret_cast<uint4*>(sm + L::OS + swz_off(row, 4 * h + 2 * hf + c, L::RB)) =
              make_uint4(pack_half2(o[8 * c] * inv, o[8 * c + 1] * inv), pack_half2(o[8 * c + 2] * inv, o[8 * c + 3] * inv),
                         pack_half2(o[8 * c + 4] * inv, o[8 * c + 5] * inv),
                         pack_half2(o[8 * c + 6] * inv, o[8 * c + 7] * inv));
        }
      }
      sync_mma();  // Q/K/V^T/P free for the next head; O complete after the last
    }

    // ---- proj + residual -> x1, LN2 -> A1 ----
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
      for (int k = 0; k < T / 16; ++k)
        umma_f16(tmem + L::C_PROJ, make_sdesc(sb + L::OS + k * 32, L::RB, L::SWZ),
                 make_sdesc(sb + L::W_PROJ + k * 32, L::RB, L::SWZ), id, k);
      umma_commit(bar);
    }
    wait_mma();
    float x1[HALF];
    {
      if (HALF == 32)
        tmem_ld16x2(trow + L::C_PROJ + hf * HALF, x1, trow + L::C_PROJ + hf * HALF + 16, x1 + 16);
      else
        tmem_ld16(trow + L::C_PROJ + hf * HALF, x1);
      float s1 = 0.f, s2 = 0.f;
#pragma unroll
      for (int k = 0; k < HALF; ++k) {
        x1[k] += yt[k] + par[L::P_BPROJ + hf * HALF + k];
        s1 += x1[k];
        s2 += x1[k] * x1[k];
      }
      const float2 st = pair_sum(s1, s2);
      const float mu = st.x * (1.f / T);
      const float rstd = rsqrtf(fmaxf(st.y * (1.f / T) - mu * mu, 0.f) + 1e-5f);
#pragma unroll
      for (int c = 0; c < NCH; ++c) {
        float o[8];
        const int k0 = hf * HALF + 8 * c;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = (x1[8 * c + j] - mu) * rstd * par[L::P_L2G + k0 + j] + par[L::P_L2B + k0 + j];
        *reinterpret_cast<uint4*>(sm + L::A1 + swz_off(row, hf * NCH + c, L::RB)) =
            make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
      }
    }
    sync_mma();

    // ---- MLP in 128-wide hidden chunks; thread half hf fills K block hf ----
    for (int j = 0; j < (4 * T) / 128; ++j) {
      if (tid == 0) {
        constexpr uint32_t id = make_idesc_f16(128, 128);
#pragma unroll
        for (int k = 0; k < T / 16; ++k)
          umma_f16(tmem + L::C_HID, make_sdesc(sb + L::A1 + k * 32, L::RB, L::SWZ),
                   make_sdesc(sb + L::W_0 + j * 128 * L::RB + k * 32, L::RB, L::SWZ), id, k);
        umma_commit(bar);
      }
      wait_mma();
      uint8_t* hb = sm + L::PS + hf * 16384;
#pragma unroll 1
      for (int c = 0; c < 64; c += 32) {
        float hv[32];
        tmem_ld16x2(trow + L::C_HID + hf * 64 + c, hv, trow + L::C_HID + hf * 64 + c + 16, hv + 16);
        const float4* b4 = reinterpret_cast<const float4*>(par + L::P_B0 + j * 128 + hf * 64 + c);
        uint32_t pk[16];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 b = b4[q];
          __half2 a0 = __floats2half2_rn(hv[4 * q] + b.x, hv[4 * q + 1] + b.y);
          __half2 a1 = __floats2half2_rn(hv[4 * q + 2] + b.z, hv[4 * q + 3] + b.w);
          a0 = gelu_as_h2(a0);
          a1 = gelu_as_h2(a1);
          pk[2 * q] = *reinterpret_cast<uint32_t*>(&a0);
          pk[2 * q + 1] = *reinterpret_cast<uint32_t*>(&a1);
        }
#pragma unroll
        for (int q = 0; q < 4; ++q)
          *reinterpret_cast<uint4*>(hb + swz_off(row, (c >> 3) + q, 128)) =
              make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
      }
      sync_mma();
      if (tid == 0) {
        constexpr uint32_t id = make_idesc_f16(128, T);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + L::C_MLP2, make_sdesc(sb + L::PS + kb * 16384 + k * 32, 128, SW_128B),
                     make_sdesc(sb + L::W_2 + (2 * j + kb) * T * 128 + k * 32, 128, SW_128B), id,
                     (j | kb | k) != 0);
        umma_commit(bar);
      }
      wait_mma();  // the hidden chunk buffer is free again
    }

    // ---- z = x1 + mlp + b2 -> Z[:, T:2T) (this thread's half) ----
    {
      float m[HALF];
      if (HALF == 32)
        tmem_ld16x2(trow + L::C_MLP2 + hf * HALF, m, trow + L::C_MLP2 + hf * HALF + 16, m + 16);
      else
        tmem_ld16(trow + L::C_MLP2 + hf * HALF, m);
      if (pix >= 0 && store) {
        uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T + hf * HALF);
#pragma unroll
        for (int c = 0; c < NCH; ++c) {
          float o[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) o[q] = x1[8 * c + q] + m[8 * c + q] + par[L::P_B2 + hf * HALF + 8 * c + q];
          dst[c] = make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
        }
      }
    }
    tc_fence_before();
    __syncthreads();  // TMEM and smem are reused by the next pair
    tc_fence_after();
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace scb
