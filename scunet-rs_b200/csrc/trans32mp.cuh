// The transformer half of a full-resolution ConvTransBlock (trans width T = 32, one
// head) with independent pair lanes: one CTA per SM keeps the block's weights in
// shared memory once and runs LANES = 4 lanes of 128 threads, each of which takes a
// window pair (two 8x8 windows = 128 tokens = one UMMA M tile) through the whole
// half on its own, one thread per token row:
//
//   y_t row (global -> shared by cp.async, a pair ahead) -> LN1 -> A1 (TMEM)
//   -> [qkv = A1.Wqkv'^T + b] -> Q, K (shared, K-major), V (shared, MN-major)
//   -> [S = Q.K^T] -> + rel-pos bias, mask, P' = 2^(s - max) (TMEM)
//   -> [O' | rowsum = P'.[V0 | V1 | 1]] -> O = O'/rowsum (TMEM) -> [x1 = O.Wp^T + b]
//   -> x1 += y_t (written back to TMEM as the MLP accumulator's start value)
//   -> LN2 -> A2 (shared) -> [h0 = A2.W0'_0^T + b0'_0] -> 2 GELU(h0) -> H0 (TMEM)
//   -> [z += H0.(W2_0/2)^T ; h1 = A2.W0'_1^T + b0'_1] -> H1 -> [z += H1.(W2_1/2)^T]
//   -> z + b2 -> Z
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136; WMSA as tools/network_scunet.py:69-102)
//
// A lane waits for each of its seven UMMA groups per pair; while it waits, the
// other three lanes of the SM run their CUDA-core work (LayerNorms, softmax, GELU),
// so the tensor cores' round trips hide behind one another instead of forming one
// chain. Every row's work stays in its own thread (no cross-thread reductions), and
// lanes share nothing but the read-only weights, so the only synchronisation is a
// lane's own named barrier before each UMMA issue and its own mbarrier after.
//
// A lane owns 128 TMEM columns, reused across the pair's phases (columns):
//   qkv [0, 96) with A1 [112, 128); S [0, 128); P' [0, 32) with O' and the row sums
//   [32, 112) and O [112, 128); x1 / z [0, 32); hidden chunk 0 [32, 96) -> H0
//   [32, 64); hidden chunk 1 [64, 128) -> H1 [64, 96).
// Numerics as trans32ws.cuh: LayerNorm affine maps and the attention scale folded
// into the weights on the host, biases of qkv, proj and mlp0 through a ones K step
// (fp16 high part + remainder), softmax in base 2 on fp16 differences, row sums from
// the same fp16 P' (a ones column of the MN-major V operand), the GELU's 1/2 folded
// into W2 (exact). Every wait is bounded and gives up on a CTA-wide abort flag.
#pragma once
#include "trans32ws.cuh"

namespace scb {

struct T32M {
  static constexpr int T = 32;
  static constexpr int LANES = 4;
  // read-only tiles shared by the lanes (offsets from the 1024-aligned base)
  static constexpr int W_QKV = 0;                  // [96 x 64 B]  SW64 Wqkv' (LN1 gamma, q scale folded)
  static constexpr int B_QKV = W_QKV + 96 * 64;    // [96 x 64 B]  bias hi/lo in K elements 0, 1
  static constexpr int W_PROJ = B_QKV + 96 * 64;   // [32 x 64 B]
  static constexpr int B_PROJ = W_PROJ + 32 * 64;  // [32 x 64 B]
  static constexpr int W_0 = B_PROJ + 32 * 64;     // [128 x 64 B] W0' (LN2 gamma folded)
  static constexpr int B_0 = W_0 + 128 * 64;       // [128 x 64 B]
  static constexpr int W_2 = B_0 + 128 * 64;       // 2 K blocks of [32 x 128 B] SW128: W2 / 2
  static constexpr int ONES = W_2 + 2 * 32 * 128;  // [128 x 64 B] K elements 0, 1 = 1
  static constexpr int RPB = ONES + 128 * 64;      // rel-pos bias, log2 units, fp32 [64][64], chunk-swizzled
  static constexpr int B2F = RPB + 64 * 64 * 4;    // mlp2 bias, 32 floats
  // per lane: Q (A of S; later A2, A of mlp0), keys, V (MN-major B of P.V), the y_t rows
  static constexpr int LANE0 = B2F + 1024;
  static constexpr int L_Q = 0, L_K = 8192, L_V = 16384, L_Y = 24576, L_BYTES = 32768;
  // the ones atom of the P.V operand (N element 64 = 1), shared: each lane's
  // descriptor reaches it through its own atom stride
  static constexpr int V_ONE = LANE0 + LANES * L_BYTES;
  static constexpr int BAR = V_ONE + 8192;
  static constexpr int SMEM = BAR + 256 + 1024;  // + alignment slack
  static constexpr int THREADS = 128 * LANES;
  static constexpr uint32_t COLS = 128;          // TMEM columns per lane
};

__global__ void __launch_bounds__(T32M::THREADS, 1) trans32_mp_kernel(const TransGeom g) {
  using L = T32M;
  constexpr int T = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);  // [LANES] UMMA done, [LANES] drain
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + 2 * L::LANES);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* status = misc + 2;  // [LANES][2]

  const int tid = threadIdx.x, warp = tid >> 5;
  const int lane_id = tid >> 7;               // which pair lane
  const int row = tid & 127;                   // token row of the pair = TMEM lane
  const int slot = row >> 6, tok = row & 63, qi = tok >> 3, qj = tok & 7;

  // ---- resident tiles ----
  stage_kmajor(sm + L::W_QKV, g.wqkv_f, 3 * T, T, T);
  stage_kmajor(sm + L::W_PROJ, g.wproj, T, T, T);
  stage_kmajor(sm + L::W_0, g.w0_f, 4 * T, T, T);
  for (int idx = tid; idx < T * (4 * T / 8); idx += blockDim.x) {  // W2 / 2 (exact in fp16)
    const int r = idx >> 4, j = idx & 15, blk = j >> 3;
    uint4 u = __ldg(reinterpret_cast<const uint4*>(g.w2 + (long)r * 4 * T + j * 8));
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __hmul2(h[e], __float2half2_rn(0.5f));
    *reinterpret_cast<uint4*>(sm + L::W_2 + blk * T * 128 + swz_off(r, j & 7, 128)) = u;
  }
  if (tid < T) reinterpret_cast<float*>(sm + L::B2F)[tid] = g.b2[tid];
  {
    // SW64 side tiles: bias hi/lo (qkv 96, proj 32, mlp0 128 rows) and the ones tile
    constexpr int R_BQ = 0, R_BP = 96, R_B0 = 128, R_ONE = 256, R_END = 384;
    for (int i = tid; i < R_END * 4; i += blockDim.x) {
      const int r = i >> 2, c = i & 3;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      uint8_t* base;
      int rr;
      if (r < R_BP) {
        base = sm + L::B_QKV, rr = r - R_BQ;
        if (c == 0) v.x = bias_hilo(g.bqkv_f[rr]);
      } else if (r < R_B0) {
        base = sm + L::B_PROJ, rr = r - R_BP;
        if (c == 0) v.x = bias_hilo(g.bproj[rr]);
      } else if (r < R_ONE) {
        base = sm + L::B_0, rr = r - R_B0;
        if (c == 0) v.x = bias_hilo(g.b0_f[rr]);
      } else {
        base = sm + L::ONES, rr = r - R_ONE;
        if (c == 0) v.x = 0x3C003C00u;
      }
      *reinterpret_cast<uint4*>(base + swz_off(rr, c, 64)) = v;
    }
    // the shared ones atom of P.V's B operand: key row k, N element 0 = 1
    for (int i = tid; i < 64 * 8; i += blockDim.x) {
      const int k = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(sm + L::V_ONE + swz_off(k, c, 128)) = make_uint4(c == 0 ? 0x3C00u : 0u, 0u, 0u, 0u);
    }
    // rel-pos bias B(query m, key k) = rp[(mi - ki + 7) * 15 + (mj - kj + 7)] log2(e); the 16-byte
    // chunks of row m are XOR-swizzled by m % 8 within each 128-byte half (conflict-free float4 reads)
    float* rpb = reinterpret_cast<float*>(sm + L::RPB);
    for (int i = tid; i < 64 * 64; i += blockDim.x) {
      const int m = i >> 6, k = i & 63, c = k >> 2;
      const float v = g.rp[((m >> 3) - (k >> 3) + 7) * 15 + ((m & 7) - (k & 7) + 7)] * 1.4426950408889634f;
      rpb[m * 64 + (((c & 8) | ((c ^ m) & 7)) << 2) + (k & 3)] = v;
    }
  }
  if (tid == 0) {
    for (int i = 0; i < 2 * L::LANES; ++i) mbar_init(bars + i, 1);
    mbar_fence_init();
    *abort_flag = 0u;
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tbase = *tmem_slot + (uint32_t)lane_id * L::COLS;           // this lane's columns
  const uint32_t trow = tbase + ((uint32_t)((warp & 3) * 32) << 16);         // + this warp's TMEM lanes
  const uint32_t sb = smem_u32(sm);
  uint8_t* lsm = sm + L::LANE0 + lane_id * L::L_BYTES;
  const uint32_t lsb = sb + L::LANE0 + lane_id * L::L_BYTES;
  uint64_t* done = bars + lane_id;
  GroupSync gs{1 + lane_id, 128, row == 0, status + 2 * lane_id, abort_flag, 0u};
  uint32_t phase = 0;
  // one UMMA round trip: every thread's operand writes are fenced, the leader issues
  // `issue()` and commits, and the lane waits for completion
  auto round = [&](auto issue) -> bool {
    tc_fence_before();
    gs.sync();
    if (gs.leader) {
      tc_fence_after();
      issue();
      umma_commit(done);
    }
    const bool ok = gs.wait(done, phase, SCB_ERR_WAIT_ATTN);
    phase ^= 1u;
    tc_fence_after();
    return ok;
  };
  auto d64 = [&](uint32_t a) { return make_sdesc(a, 64, SW_64B); };
  auto d128 = [&](uint32_t a) { return make_sdesc(a, 128, SW_128B); };
  constexpr uint32_t ID_QKV = make_idesc_f16(128, 3 * T), ID_S = make_idesc_f16(128, 128),
                     ID_PV = make_idesc_f16_bmn(128, 80), ID_T = make_idesc_f16(128, T),
                     ID_H = make_idesc_f16(128, 64);
  auto pack8 = [](const float* f) -> uint4 {
    return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
  };

  const long n_pairs = (g.win.n_windows + 1) / 2;
  const long first = (long)blockIdx.x * L::LANES + lane_id;
  const long step = (long)gridDim.x * L::LANES;
  WinCursor cur;
  cur.init(g.win, 2 * first + slot);
  // this row's y_t (32 fp16) into the lane's Y tile, a pair ahead (zeros past the
  // last window); only this thread reads its row back
  auto load_y = [&]() {
    bool lr, lc, st;
    const long pix = cur.pixel(g.win, qi, qj, lr, lc, st);
    const __half* src = pix >= 0 ? g.y + pix * T : g.y;
#pragma unroll
    for (int c = 0; c < 4; ++c) cp_async16(lsm + L::L_Y + swz_off(row, c, 64), src + 8 * c, pix >= 0);
    cp_async_commit();
  };
  // y_t as 32 floats from the Y tile
  auto read_y = [&](float* x) {
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const uint4 u = *reinterpret_cast<const uint4*>(lsm + L::L_Y + swz_off(row, c, 64));
      const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 f = __half22float2(h[j]);
        x[8 * c + 2 * j] = f.x;
        x[8 * c + 2 * j + 1] = f.y;
      }
    }
  };
  if (first < n_pairs) load_y();

  for (long p = first; p < n_pairs; p += step) {
    bool last_row, last_col, st;
    const long pix = cur.pixel(g.win, qi, qj, last_row, last_col, st);
    // ---- LN1 -> A1 ----
    float x[32];
    cp_async_wait_all();
    read_y(x);
    {
      float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        s0 += x[j];
        s1 += x[j + 1];
        q0 = fmaf(x[j], x[j], q0);
        q1 = fmaf(x[j + 1], x[j + 1], q1);
      }
      const float mu = (s0 + s1) * (1.f / T);
      const float rstd = rsqrtf(fmaxf((q0 + q1) * (1.f / T) - mu * mu, 0.f) + 1e-5f);
      const float nmr = -mu * rstd;
      uint32_t a[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) a[j] = pack_half2(fmaf(x[2 * j], rstd, nmr), fmaf(x[2 * j + 1], rstd, nmr));
      tmem_st16u(trow + 112, a);
      tmem_wait_st();
    }
    // ---- [qkv] ----
    if (!round([&] {
          umma_f16_ts(tbase, tbase + 112, d64(sb + L::W_QKV), ID_QKV, 0);
          umma_f16_ts(tbase, tbase + 120, d64(sb + L::W_QKV + 32), ID_QKV, 1);
          umma_f16(tbase, d64(sb + L::ONES), d64(sb + L::B_QKV), ID_QKV, 1);
        }))
      break;
    {
      float v[32];
      tmem_ld16x2(trow, v, trow + 16, v + 16);  // q
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(lsm + L::L_Q + swz_off(row, c, 64)) = pack8(v + 8 * c);
      tmem_ld16x2(trow + 32, v, trow + 48, v + 16);  // k
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(lsm + L::L_K + swz_off(row, c, 64)) = pack8(v + 8 * c);
      tmem_ld16x2(trow + 64, v, trow + 80, v + 16);  // v: key row tok, N elements 32 slot .. + 31
#pragma unroll
      for (int c = 0; c < 4; ++c)
        *reinterpret_cast<uint4*>(lsm + L::L_V + swz_off(tok, 4 * slot + c, 128)) = pack8(v + 8 * c);
    }
    fence_proxy_async_smem();
    // ---- [S] ----
    if (!round([&] {
          umma_f16(tbase, d64(lsb + L::L_Q), d64(lsb + L::L_K), ID_S, 0);
          umma_f16(tbase, d64(lsb + L::L_Q + 32), d64(lsb + L::L_K + 32), ID_S, 1);
        }))
      break;
    {
      float s[64];  // the keys of this row's own window
      {
        uint32_t r[64];
        tmem_ld16_issue(trow + 64 * slot, r);
        tmem_ld16_issue(trow + 64 * slot + 16, r + 16);
        tmem_ld16_issue(trow + 64 * slot + 32, r + 32);
        tmem_ld16_issue(trow + 64 * slot + 48, r + 48);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) tmem_fence16(r + 16 * j);
#pragma unroll
        for (int j = 0; j < 64; ++j) s[j] = __uint_as_float(r[j]);
      }
      const float* rb = reinterpret_cast<const float*>(sm + L::RPB) + tok * 64;
#pragma unroll
      for (int c = 0; c < 16; ++c) {
        const float4 bb = *reinterpret_cast<const float4*>(rb + (((c & 8) | ((c ^ tok) & 7)) << 2));
        s[4 * c] += bb.x;
        s[4 * c + 1] += bb.y;
        s[4 * c + 2] += bb.z;
        s[4 * c + 3] += bb.w;
      }
      if (last_row || last_col) {  // warp-uniform: a warp's 32 tokens share one window
        // the cyclic shift put tokens from opposite image edges into the last window
        // row / column; a token attends only to keys from its own side
        // (cuda/scunet.cu:137-147). Key j sits at window row j / 8, column j % 8.
        const bool qtop = qi < 4, qleft = qj < 4;
#pragma unroll
        for (int j = 0; j < 64; ++j)
          s[j] = ((last_row && (qtop != ((j >> 3) < 4))) || (last_col && (qleft != ((j & 7) < 4)))) ? -INFINITY : s[j];
      }
      float m0 = s[0], m1 = s[1], m2 = s[2], m3 = s[3];
#pragma unroll
      for (int j = 4; j < 64; j += 4) {
        m0 = fmaxf(m0, s[j]);
        m1 = fmaxf(m1, s[j + 1]);
        m2 = fmaxf(m2, s[j + 2]);
        m3 = fmaxf(m3, s[j + 3]);
      }
      const float mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
      // P' = 2^(s - max) as packed fp16, the precision the P.V operand has anyway
      uint32_t pp[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) pp[j] = ex2_approx_h2(pack_half2(s[2 * j] - mx, s[2 * j + 1] - mx));
      tmem_st16u(trow, pp);
      tmem_st16u(trow + 16, pp + 16);
      tmem_wait_st();
    }
    // ---- [O' | rowsum] ----
    if (!round([&] {
          const uint32_t vb = lsb + L::L_V;
          const uint32_t lbo = (uint32_t)(L::V_ONE - (L::LANE0 + lane_id * L::L_BYTES + L::L_V));
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K step k = keys 16k .. 16k + 15
            umma_f16_ts(tbase + 32, tbase + 8 * k, make_sdesc_lbo_sbo(vb + 2048 * k, lbo, 1024, SW_128B), ID_PV, k);
        }))
      break;
    {
      float o[32];
      tmem_ld16x2(trow + 32 + 32 * slot, o, trow + 48 + 32 * slot, o + 16);  // own window's half
      const float inv = __fdividef(1.f, tmem_ld1(trow + 96));
      uint32_t po[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) po[j] = pack_half2(o[2 * j] * inv, o[2 * j + 1] * inv);
      tmem_st16u(trow + 112, po);
      tmem_wait_st();
    }
    // ---- [x1 = O.Wp^T + b] ----
    if (!round([&] {
          umma_f16_ts(tbase, tbase + 112, d64(sb + L::W_PROJ), ID_T, 0);
          umma_f16_ts(tbase, tbase + 120, d64(sb + L::W_PROJ + 32), ID_T, 1);
          umma_f16(tbase, d64(sb + L::ONES), d64(sb + L::B_PROJ), ID_T, 1);
        }))
      break;
    {
      // x1 = acc + y_t, back into TMEM (the MLP accumulator starts from it); LN2 -> A2
      read_y(x);
      {
        float acc[32];
        tmem_ld16x2(trow, acc, trow + 16, acc + 16);
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] += acc[j];
      }
      tmem_st16(trow, x);
      tmem_st16(trow + 16, x + 16);
      float s0 = 0.f, s1 = 0.f, q0 = 0.f, q1 = 0.f;
#pragma unroll
      for (int j = 0; j < 32; j += 2) {
        s0 += x[j];
        s1 += x[j + 1];
        q0 = fmaf(x[j], x[j], q0);
        q1 = fmaf(x[j + 1], x[j + 1], q1);
      }
      const float mu = (s0 + s1) * (1.f / T);
      const float rstd = rsqrtf(fmaxf((q0 + q1) * (1.f / T) - mu * mu, 0.f) + 1e-5f);
      const float nmr = -mu * rstd;
      float a[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) a[j] = fmaf(x[j], rstd, nmr);
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(lsm + L::L_Q + swz_off(row, c, 64)) = pack8(a + 8 * c);
      tmem_wait_st();
    }
    fence_proxy_async_smem();
    // the next pair's y_t, in flight during the MLP
    cur.advance(g.win, (int)(2 * step));
    if (p + step < n_pairs) load_y();
    // ---- [h0] ----
    if (!round([&] {
          umma_f16(tbase + 32, d64(lsb + L::L_Q), d64(sb + L::W_0), ID_H, 0);
          umma_f16(tbase + 32, d64(lsb + L::L_Q + 32), d64(sb + L::W_0 + 32), ID_H, 1);
          umma_f16(tbase + 32, d64(sb + L::ONES), d64(sb + L::B_0), ID_H, 1);
        }))
      break;
    // 2 GELU(hidden chunk) over 64 columns at `src` -> 32 packed fp16 columns at
    // `dst` (this thread's row), 32 columns at a time: the packed half of each step
    // lands below the columns the next step reads (dst <= src)
    auto gelu_chunk = [&](uint32_t src, uint32_t dst) {
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t r[32];
        tmem_ld16_issue(trow + src + 32 * hh, r);
        tmem_ld16_issue(trow + src + 32 * hh + 16, r + 16);
        tmem_wait_ld();
        tmem_fence16(r);
        tmem_fence16(r + 16);
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          __half2 h = __floats2half2_rn(__uint_as_float(r[2 * j]), __uint_as_float(r[2 * j + 1]));
          h = gelu2_tanh_h2(h);
          pk[j] = *reinterpret_cast<uint32_t*>(&h);
        }
        tmem_st16u(trow + dst + 16 * hh, pk);
      }
      tmem_wait_st();
    };
    gelu_chunk(32, 32);
    // ---- [z += H0.(W2_0/2)^T ; h1] ----
    if (!round([&] {
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16_ts(tbase, tbase + 32 + 8 * k, d128(sb + L::W_2 + 32 * k), ID_T, 1);
          umma_f16(tbase + 64, d64(lsb + L::L_Q), d64(sb + L::W_0 + 64 * 64), ID_H, 0);
          umma_f16(tbase + 64, d64(lsb + L::L_Q + 32), d64(sb + L::W_0 + 64 * 64 + 32), ID_H, 1);
          umma_f16(tbase + 64, d64(sb + L::ONES), d64(sb + L::B_0 + 64 * 64), ID_H, 1);
        }))
      break;
    gelu_chunk(64, 64);
    // ---- [z += H1.(W2_1/2)^T] ----
    if (!round([&] {
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(tbase, tbase + 64 + 8 * k, d128(sb + L::W_2 + T * 128 + 32 * k), ID_T, 1);
        }))
      break;
    {
      float z[32];
      tmem_ld16x2(trow, z, trow + 16, z + 16);
      if (pix >= 0 && st) {
        const float4* b24 = reinterpret_cast<const float4*>(sm + L::B2F);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 bb = b24[q];
          z[4 * q] += bb.x;
          z[4 * q + 1] += bb.y;
          z[4 * q + 2] += bb.z;
          z[4 * q + 3] += bb.w;
        }
        uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T);
#pragma unroll
        for (int c = 0; c < 4; ++c) dst[c] = pack8(z + 8 * c);
      }
    }
  }
  // nothing of this lane may be in flight when the TMEM is released
  if (gs.leader) {
    umma_commit(bars + L::LANES + lane_id);
    mbar_wait(bars + L::LANES + lane_id, 0, SCB_ERR_WAIT_ATTN);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(*tmem_slot, 512);
}

}  // namespace scb
