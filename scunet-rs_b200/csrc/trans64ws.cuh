// The transformer half of a half-resolution ConvTransBlock (trans width T = 64, two
// heads of 32), warp-specialised like trans32ws.cuh (whose helpers it uses): one
// 512-thread CTA per SM streams pairs of 8x8 windows (128 tokens, one UMMA M tile)
// through four warp groups working on different pairs ([..] = a UMMA):
//
//   G1 (4 warps, one thread per token row): y_t row by cp.async (a pair ahead) ->
//      LN1 -> A1 -> [qkv = A1.Wqkv'^T + b] -> Q (TMEM), K and V of both heads
//      (shared memory) -> [S_h = Q_h.K_h^T], h = 0, 1
//   G2 (4 warps, one thread per row, the two heads in turn): + rel-pos bias, mask,
//      max, P'_h = 2^(s - max) -> [O'_h | rowsum_h = P'_h.[V0 | V1 | 1]_h]
//   G3 (4 warps, one thread per row): O = O'/rowsum -> [x1 = O.Wproj^T + b_proj];
//      x1 += y_t (re-read from L2) written back to TMEM; LN2(x1) -> A2 ->
//      [hid_c = A2.W0'_c^T + b0'_c] for four 64-wide hidden chunks c, two TMEM
//      buffers, each refilled as soon as its chunk's mlp2 K steps have completed;
//      z = acc + b2 -> Z
//   G4 (4 warps, one thread per row, a chunk's 64 columns in two halves): per chunk,
//      2 GELU(hid_c) -> H_c (over the chunk's own columns) -> [acc += H_c.(W2_c/2)^T]
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136; WMSA as tools/network_scunet.py:69-102)
//
// Differences from the T = 32 kernel, all forced by the 512 TMEM columns: the
// attention stage of a pair (qkv, S of both heads, P', O', O) uses one 256-column
// score buffer, so a pair's qkv waits until the previous pair's proj has read its O;
// there is one x1 / z accumulator (64 columns), so a pair's proj follows the previous
// pair's z; y_t enters x1 on the CUDA cores (the G3 threads read their rows from a
// shared-memory copy staged during the previous pair's MLP, not from a y_t operand tile
// of an identity UMMA); the rel-pos bias table is fp16. Numerics as trans32ws.cuh: LayerNorm
// affine maps and the attention scale folded into the weights on the host, biases
// of qkv, proj and mlp0 through a ones K step (fp16 high + remainder), softmax row
// sums from the fp16 P' via a ones column of the MN-major V operand, the GELU's 1/2
// folded into W2 (exact).
#pragma once
#include "trans32ws.cuh"

namespace scb {

struct T64 {
  static constexpr int T = 64;
  // resident shared-memory tiles (offsets from the 1024-aligned base)
  static constexpr int W_QKV = 0;                    // [192 x 128 B] SW128, Wqkv' (LN1 gamma, q scale folded)
  static constexpr int B_QKV = W_QKV + 192 * 128;    // [192 x 64 B] SW64, bias hi/lo in K elements 0, 1
  static constexpr int W_PROJ = B_QKV + 192 * 64;    // [64 x 128 B] SW128
  static constexpr int B_PROJ = W_PROJ + 64 * 128;   // [64 x 64 B] SW64
  static constexpr int W_0 = B_PROJ + 64 * 64;       // [256 x 128 B] SW128, W0' (LN2 gamma folded)
  static constexpr int B_0 = W_0 + 256 * 128;        // [256 x 64 B] SW64
  static constexpr int W_2 = B_0 + 256 * 64;         // 4 K blocks of [64 x 128 B] SW128: W2 / 2
  static constexpr int ONES = W_2 + 4 * 64 * 128;    // [128 x 64 B] SW64, K elements 0, 1 = 1
  // rel-pos bias in log2 units, fp16 [2 heads][64 query positions][64 keys]; the
  // 16-byte chunks of a row are XOR-swizzled by the query position
  static constexpr int RPB = ONES + 128 * 64;
  static constexpr int Y = RPB + 2 * 64 * 64 * 2;    // [128 x 128 B] y_t rows (LN1 input)
  static constexpr int K = Y + 128 * 128;            // 2 heads x [128 x 64 B] SW64
  // V as the MN-major B operand of P.V: per head an atom [64 keys x 128 B] holding
  // [V_0 | V_1] of the head, and one shared atom whose first N element is 1
  static constexpr int V = K + 2 * 8192;             // V_0, V_1, ones atom (8 KB each)
  static constexpr int B2F = V + 3 * 8192;           // mlp2 bias, 64 floats
  static constexpr int YS = B2F + 256;               // [128 x 128 B] y_t rows of the next x1 (G3)
  static constexpr int BAR = YS + 128 * 128;
  static constexpr int SMEM = BAR + 256 + 1024;      // + alignment slack
  // TMEM columns (packed fp16 A operands: 8 columns per K step of 16)
  static constexpr uint32_t C_SB = 0;     // score buffer [0, 256): qkv acc [0, 192), A1 [192, 224);
                                          // then S_h [128 h, +128), P'_h [128 h, +32),
                                          // O'_h [128 h + 32, +64) + rowsum at 128 h + 96, O_h [128 h + 112, +16)
  static constexpr uint32_t SB_A1 = 192;
  static constexpr uint32_t C_Q = 256;    // Q_h at 256 + 16 h
  static constexpr uint32_t C_A2 = 288;   // LN2 output (32)
  static constexpr uint32_t C_ACC = 320;  // x1, then z (64)
  static constexpr uint32_t C_HID = 384;  // two 64-column hidden chunk buffers; 2 GELU overwrites the first 32
  static constexpr int G1_WARPS = 4, G2_WARPS = 4, G3_WARPS = 4, G4_WARPS = 4;
  static constexpr int THREADS = 32 * (G1_WARPS + G2_WARPS + G3_WARPS + G4_WARPS);
};

__global__ void __launch_bounds__(T64::THREADS, 1) trans64_ws_kernel(const TransGeom g) {
  using L = T64;
  constexpr int T = 64;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* bar_qkv = bars + 0;
  uint64_t* bar_s = bars + 1;
  uint64_t* bar_o = bars + 2;
  uint64_t* x1_done = bars + 3;
  uint64_t* so_free = bars + 4;   // the score buffer's O read by a completed proj (128 arrivals)
  uint64_t* bar_hid = bars + 5;   // [2] per hidden buffer: mlp0 committed
  uint64_t* bar_out = bars + 7;   // [2] per hidden buffer: its mlp2 K steps committed
  uint64_t* drain = bars + 9;     // [4] one per issuing group
  constexpr int NBAR = 13;
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + NBAR);
  static_assert(13 * 8 + 10 * 4 <= 256, "barrier region");
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* status = misc + 2;  // [4][2]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane;  // TMEM lane = token row of the pair
  const int slot = row >> 6, tok = row & 63, qi = tok >> 3, qj = tok & 7;

  // ---- resident tiles ----
  stage_kmajor(sm + L::W_QKV, g.wqkv_f, 3 * T, T, T);
  stage_kmajor(sm + L::W_PROJ, g.wproj, T, T, T);
  stage_kmajor(sm + L::W_0, g.w0_f, 4 * T, T, T);
  // W2 / 2 (exact in fp16): the GELU below returns 2 GELU(x)
  for (int idx = tid; idx < T * (4 * T / 8); idx += blockDim.x) {
    const int r = idx >> 5, j = idx & 31, blk = j >> 3;
    uint4 u = __ldg(reinterpret_cast<const uint4*>(g.w2 + (long)r * 4 * T + j * 8));
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __hmul2(h[e], __float2half2_rn(0.5f));
    *reinterpret_cast<uint4*>(sm + L::W_2 + blk * T * 128 + swz_off(r, j & 7, 128)) = u;
  }
  if (tid < T) reinterpret_cast<float*>(sm + L::B2F)[tid] = g.b2[tid];
  {
    // SW64 side tiles: bias hi/lo (qkv 192, proj 64, mlp0 256 rows), ones
    constexpr int R_BQ = 0, R_BP = 192, R_B0 = 256, R_ONE = 512, R_END = 640;
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
    // the ones atom of the V operand (64 key rows: N element 64 = 1)
    for (int i = tid; i < 64 * 8; i += blockDim.x) {
      const int q = i >> 3, c = i & 7;
      *reinterpret_cast<uint4*>(sm + L::V + 2 * 8192 + swz_off(q, c, 128)) =
          make_uint4(c == 0 ? 0x3C00u : 0u, 0u, 0u, 0u);
    }
    // rel-pos bias B_h(query m, key k) = rp[h][(mi - ki + 7) * 15 + (mj - kj + 7)] log2(e), fp16
    __half* rpb = reinterpret_cast<__half*>(sm + L::RPB);
    for (int i = tid; i < 2 * 64 * 64; i += blockDim.x) {
      const int h = i >> 12, m = (i >> 6) & 63, k = i & 63, c = k >> 3;
      const float v = g.rp[h * 225 + ((m >> 3) - (k >> 3) + 7) * 15 + ((m & 7) - (k & 7) + 7)] * 1.4426950408889634f;
      rpb[(h * 64 + m) * 64 + ((c ^ (m & 7)) << 3) + (k & 7)] = __float2half_rn(v);
    }
  }
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bars + i, i == 4 ? 128u : 1u);
    mbar_fence_init();
    *abort_flag = 0u;
  }
  if (warp == 0) tmem_alloc(tmem_slot, 512);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)((warp & 3) * 32) << 16);
  const uint32_t sb = smem_u32(sm);

  const long n_pairs = (g.win.n_windows + 1) / 2;
  const long first = blockIdx.x;
  const int n_local = first < n_pairs ? (int)((n_pairs - 1 - first) / gridDim.x + 1) : 0;
  const int win_step = 2 * (int)gridDim.x;
  auto pack8 = [](const float* f) -> uint4 {
    return make_uint4(pack_half2(f[0], f[1]), pack_half2(f[2], f[3]), pack_half2(f[4], f[5]), pack_half2(f[6], f[7]));
  };
  auto unpack8 = [](uint4 u, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 p = __half22float2(h[j]);
      f[2 * j] = p.x;
      f[2 * j + 1] = p.y;
    }
  };
  constexpr uint32_t ID_QKV = make_idesc_f16(128, 3 * T), ID_S = make_idesc_f16(128, 128),
                     ID_PV = make_idesc_f16_bmn(128, 80), ID_T = make_idesc_f16(128, T),
                     ID_H64 = make_idesc_f16(128, 64);
  auto d64 = [&](int off) { return make_sdesc(sb + off, 64, SW_64B); };
  auto d128 = [&](int off) { return make_sdesc(sb + off, 128, SW_128B); };

  if (warp < L::G1_WARPS) {
    // ====== G1: y_t -> LN1 -> [qkv] -> Q (TMEM), K, V (smem) -> [S_0, S_1] ======
    GroupSync gs{1, 32 * L::G1_WARPS, tid == 0, status, abort_flag, 0u};
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    // the y_t rows of the warp's 32 tokens at the pair the cursor stands at, lane l
    // copying 16-byte chunk l % 8 of rows l / 8 + 4 k (pixel by shuffle from the row's
    // lane): one copy instruction covers four whole 128-byte rows
    auto fetch = [&]() {
      bool lr, lc, st;
      const long pix = cur.pixel(g.win, qi, qj, lr, lc, st);
      const int c = lane & 7;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int sl = (lane >> 3) + 4 * k;
        const long pk = __shfl_sync(0xffffffffu, pix, sl);
        const __half* src = pk >= 0 ? g.y + pk * T : g.y;
        cp_async16(sm + L::Y + swz_off((warp & 3) * 32 + sl, c, 128), src + 8 * c, pk >= 0);
      }
      cp_async_commit();
    };
    if (n_local > 0) fetch();
    for (int li = 0; li < n_local; ++li) {
      cp_async_wait_all();  // this thread's copies of pair li have landed,
      __syncwarp();         // and those of the other lanes, which hold this row's chunks
      uint32_t a[32];
      {
        float x[64];
#pragma unroll
        for (int c = 0; c < 8; ++c) unpack8(*reinterpret_cast<const uint4*>(sm + L::Y + swz_off(row, c, 128)), x + 8 * c);
        ln_pack_f32x2<T>(x, a);
      }
      if (li + 1 < n_local) {  // the warp's rows were read: fetch the next pair's
        __syncwarp();
        cur.advance(g.win, win_step);
        fetch();
      }
      // the score buffer held pair li - 1 until its proj read O
      if (li >= 1 && !gs.wait(so_free, (li - 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      tmem_st32u(trow + L::C_SB + L::SB_A1, a);
      tmem_wait_st();
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k)
          umma_f16_ts(tmem + L::C_SB, tmem + L::C_SB + L::SB_A1 + 8 * k, d128(L::W_QKV + 32 * k), ID_QKV, k);
        umma_f16(tmem + L::C_SB, d64(L::ONES), d64(L::B_QKV), ID_QKV, 1);
        umma_commit(bar_qkv);
      }
      if (!gs.wait(bar_qkv, li & 1, SCB_ERR_WAIT_ATTN)) break;
      // Q, K of pair li - 1 are operands of its S UMMAs (its V was freed with the
      // score buffer)
      if (li >= 1 && !gs.wait(bar_s, (li - 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      {
        float q[64];
        tmem_ld16x2(trow + L::C_SB, q, trow + L::C_SB + 16, q + 16);
        tmem_ld16x2(trow + L::C_SB + 32, q + 32, trow + L::C_SB + 48, q + 48);
        uint32_t pq[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) pq[j] = pack_half2(q[2 * j], q[2 * j + 1]);
        tmem_st32u(trow + L::C_Q, pq);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float k[32];
        tmem_ld16x2(trow + L::C_SB + 64 + 32 * h, k, trow + L::C_SB + 80 + 32 * h, k + 16);
        uint8_t* kb = sm + L::K + h * 8192;
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(kb + swz_off(row, c, 64)) = pack8(k + 8 * c);
      }
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        float v[32];
        tmem_ld16x2(trow + L::C_SB + 128 + 32 * h, v, trow + L::C_SB + 144 + 32 * h, v + 16);
        // V_h, MN-major: key row tok, N elements 32 slot .. 32 slot + 31
        uint8_t* vb = sm + L::V + h * 8192;
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(vb + swz_off(tok, 4 * slot + c, 128)) = pack8(v + 8 * c);
      }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          umma_f16_ts(tmem + L::C_SB + 128 * h, tmem + L::C_Q + 16 * h, d64(L::K + h * 8192), ID_S, 0);
          umma_f16_ts(tmem + L::C_SB + 128 * h, tmem + L::C_Q + 16 * h + 8, d64(L::K + h * 8192 + 32), ID_S, 1);
        }
        umma_commit(bar_s);
      }
    }
    cp_async_wait_all();
    if (gs.leader) {
      umma_commit(drain + 0);
      mbar_wait(drain + 0, 0, SCB_ERR_WAIT_ATTN);
    }
  } else if (warp < L::G1_WARPS + L::G2_WARPS) {
    // ====== G2 (one thread per row, heads in turn): softmax_h -> P'_h -> [O'_h, rowsum_h] ======
    GroupSync gs{2, 32 * L::G2_WARPS, tid == 32 * (L::G1_WARPS + 1), status + 2, abort_flag, 0u};
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    for (int li = 0; li < n_local; ++li, cur.advance(g.win, win_step)) {
      if (!gs.wait(bar_s, li & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      bool last_row, last_col, st;
      (void)cur.pixel(g.win, qi, qj, last_row, last_col, st);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const uint32_t hb = L::C_SB + 128 * h;
        float s[64];  // the row's 64 in-window keys of head h
        tmem_ld16x2(trow + hb + slot * 64, s, trow + hb + slot * 64 + 16, s + 16);
        tmem_ld16x2(trow + hb + slot * 64 + 32, s + 32, trow + hb + slot * 64 + 48, s + 48);
        {
          const uint8_t* rb = sm + L::RPB + (h * 64 + tok) * 128;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            float bb[8];
            unpack8(*reinterpret_cast<const uint4*>(rb + ((c ^ (tok & 7)) << 4)), bb);
#pragma unroll
            for (int e = 0; e < 8; e += 2) {
              const float2 v = __fadd2_rn(make_float2(s[8 * c + e], s[8 * c + e + 1]), make_float2(bb[e], bb[e + 1]));
              s[8 * c + e] = v.x;
              s[8 * c + e + 1] = v.y;
            }
          }
        }
        if (last_row || last_col) {  // warp-uniform: a warp's 32 tokens share one window
          // the cyclic shift put tokens from opposite image edges into the last window
          // row / column; a token attends only to keys from its own side
          // (cuda/scunet.cu:137-147)
          const bool qtop = qi < 4, qleft = qj < 4;
#pragma unroll
          for (int j = 0; j < 64; ++j) {
            const bool m = (last_row && (qtop != ((j >> 3) < 4))) || (last_col && (qleft != ((j & 7) < 4)));
            s[j] = m ? -INFINITY : s[j];
          }
        }
        const float mx = row_max<64>(s);
        // P'_h = 2^(s - max) as packed fp16 over this row's own S columns (read above)
        uint32_t p[32];
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const float2 d = __fadd2_rn(make_float2(s[2 * j], s[2 * j + 1]), make_float2(-mx, -mx));
          p[j] = ex2_approx_h2(pack_half2(d.x, d.y));
        }
        tmem_st32u(trow + hb, p);
      }
      tmem_wait_st();
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const uint32_t vb = sb + L::V + hh * 8192;
          const uint32_t lbo = 2 * 8192 - hh * 8192;  // V_hh atom -> ones atom
#pragma unroll
          for (int k = 0; k < 4; ++k)  // K step k = keys 16k .. 16k + 15 = two 8-row groups
            umma_f16_ts(tmem + L::C_SB + 128 * hh + 32, tmem + L::C_SB + 128 * hh + 8 * k,
                        make_sdesc_lbo_sbo(vb + 2048 * k, lbo, 1024, SW_128B), ID_PV, k);
        }
        umma_commit(bar_o);
      }
    }
    if (gs.leader) {
      umma_commit(drain + 1);
      mbar_wait(drain + 1, 0, SCB_ERR_WAIT_ATTN);
    }
  } else if (warp < L::G1_WARPS + L::G2_WARPS + L::G3_WARPS) {
    // ====== G3 (one thread per row): O -> [x1]; x1 += y_t; LN2 -> A2 -> [hid_c];
    //        z out ======
    GroupSync gs{3, 32 * L::G3_WARPS, tid == 32 * (L::G1_WARPS + L::G2_WARPS + 2), status + 4, abort_flag, 0u};
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    // O'_h / rowsum_h of pair li -> O_h (TMEM) -> [acc = O.Wproj^T + b_proj]; the
    // accumulator's previous z has been written out
    auto normproj = [&](int li) -> bool {
      if (!gs.wait(bar_o, li & 1, SCB_ERR_WAIT_ATTN)) return false;
      tc_fence_after();
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const uint32_t hb = L::C_SB + 128 * h;
        float o[32];
        tmem_ld16x2(trow + hb + 32 + slot * 32, o, trow + hb + 48 + slot * 32, o + 16);  // own window's half
        const float inv = __fdividef(1.f, tmem_ld1(trow + hb + 96));
        uint32_t po[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float2 v = __fmul2_rn(make_float2(o[2 * j], o[2 * j + 1]), make_float2(inv, inv));
          po[j] = pack_half2(v.x, v.y);
        }
        tmem_st16u(trow + hb + 112, po);
      }
      tmem_wait_st();
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        const uint32_t d = tmem + L::C_ACC;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // K steps 0, 1: O_0 at [112, 128); 2, 3: O_1 at [240, 256)
          umma_f16_ts(d, tmem + L::C_SB + 128 * (k >> 1) + 112 + 8 * (k & 1), d128(L::W_PROJ + 32 * k), ID_T, k);
        umma_f16(d, d64(L::ONES), d64(L::B_PROJ), ID_T, 1);
        umma_commit(x1_done);
      }
      return true;
    };
    auto ln2 = [&](int li) -> bool {  // x1 = acc + y_t (back into TMEM) -> LN2 -> A2; cursor at pair li
      uint4 yreg[8];  // this row's y_t (fp16, packed; staged during the previous pair's MLP)
      cp_async_wait_all();
      __syncwarp();  // the warp's lanes copied this row's chunks
#pragma unroll
      for (int c = 0; c < 8; ++c) yreg[c] = *reinterpret_cast<const uint4*>(sm + L::YS + swz_off(row, c, 128));
      __syncwarp();  // read before the next pair's rows are staged
      if (!gs.wait(x1_done, li & 1, SCB_ERR_WAIT_ATTN)) return false;
      tc_fence_after();
      float x[64];
      tmem_ld16x2(trow + L::C_ACC, x, trow + L::C_ACC + 16, x + 16);
      tmem_ld16x2(trow + L::C_ACC + 32, x + 32, trow + L::C_ACC + 48, x + 48);
      tc_fence_before();
      mbar_arrive(so_free);  // O read by the completed proj: the score buffer is free
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        float yy[8];
        unpack8(yreg[c], yy);
#pragma unroll
        for (int e = 0; e < 8; e += 2) {
          const float2 v = __fadd2_rn(make_float2(x[8 * c + e], x[8 * c + e + 1]), make_float2(yy[e], yy[e + 1]));
          x[8 * c + e] = v.x;
          x[8 * c + e + 1] = v.y;
        }
      }
      tmem_st16(trow + L::C_ACC, x);
      tmem_st16(trow + L::C_ACC + 16, x + 16);
      tmem_st16(trow + L::C_ACC + 32, x + 32);
      tmem_st16(trow + L::C_ACC + 48, x + 48);
      uint32_t a[32];
      ln_pack_f32x2<T>(x, a);
      tmem_st32u(trow + L::C_A2, a);
      tmem_wait_st();
      tc_fence_before();
      return true;
    };
    auto issue_mlp0 = [&](int c) {  // hidden chunk c -> buffer c & 1
      tc_fence_after();
      const uint32_t d = tmem + L::C_HID + (c & 1) * 64;
#pragma unroll
      for (int k = 0; k < 4; ++k)
        umma_f16_ts(d, tmem + L::C_A2 + 8 * k, d128(L::W_0 + c * 64 * 128 + 32 * k), ID_H64, k);
      umma_f16(d, d64(L::ONES), d64(L::B_0 + c * 64 * 64), ID_H64, 1);
      umma_commit(bar_hid + (c & 1));
    };
    // the y_t rows of the warp's 32 tokens at the pair cursor `cs` stands at -> YS, lane
    // l copying 16-byte chunk l % 8 of rows l / 8 + 4 k (pixel by shuffle from the row's
    // lane): four whole 128-byte rows per copy instruction, and ln2 reads its row from
    // shared memory instead of waiting on 32 scattered global loads
    auto stage_y = [&](WinCursor& cs) {
      bool lr, lc, st;
      const long pix = cs.pixel(g.win, qi, qj, lr, lc, st);
      const int c = lane & 7;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const int sl = (lane >> 3) + 4 * k;
        const long pk = __shfl_sync(0xffffffffu, pix, sl);
        const __half* src = pk >= 0 ? g.y + pk * T : g.y;
        cp_async16(sm + L::YS + swz_off((warp & 3) * 32 + sl, c, 128), src + 8 * c, pk >= 0);
      }
      cp_async_commit();
    };
    if (n_local > 0) stage_y(cur);
    bool ok = n_local > 0 && normproj(0) && ln2(0);
    if (ok) {
      gs.sync();
      if (gs.leader) {
        issue_mlp0(0);
        issue_mlp0(1);
      }
    }
    WinCursor nxt = cur;  // one pair ahead: whose y_t is fetched during this pair's MLP
    for (int li = 0; ok && li < n_local; ++li) {
      bool fine = true;
      if (li + 1 < n_local) {  // stage the next pair's y_t rows for its ln2
        nxt.advance(g.win, win_step);
        stage_y(nxt);
      }
      // chunk c of pair li lives in buffer c & 1; its mlp2 completing frees the
      // buffer for chunk c + 2 (buffer b's u-th use: u = 2 li + c / 2)
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int u = 2 * li + (c >> 1);
        if (!gs.wait(bar_out + (c & 1), u & 1, SCB_ERR_WAIT_ATTN)) {
          fine = false;
          break;
        }
        if (c + 2 < 4 && gs.leader) issue_mlp0(c + 2);
      }
      if (!fine) break;
      // z of pair li is final
      tc_fence_after();
      {
        float z[64];
        tmem_ld16x2(trow + L::C_ACC, z, trow + L::C_ACC + 16, z + 16);
        tmem_ld16x2(trow + L::C_ACC + 32, z + 32, trow + L::C_ACC + 48, z + 48);
        tc_fence_before();
        bool lr, lc, st;
        const long pix = cur.pixel(g.win, qi, qj, lr, lc, st);
        if (pix >= 0 && st) {
          const float4* b24 = reinterpret_cast<const float4*>(sm + L::B2F);
#pragma unroll
          for (int q = 0; q < 16; ++q) {
            const float4 bb = b24[q];
            const float2 lo = __fadd2_rn(make_float2(z[4 * q], z[4 * q + 1]), make_float2(bb.x, bb.y));
            const float2 hi = __fadd2_rn(make_float2(z[4 * q + 2], z[4 * q + 3]), make_float2(bb.z, bb.w));
            z[4 * q] = lo.x;
            z[4 * q + 1] = lo.y;
            z[4 * q + 2] = hi.x;
            z[4 * q + 3] = hi.y;
          }
          uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T);
#pragma unroll
          for (int c = 0; c < 8; ++c) dst[c] = pack8(z + 8 * c);
        }
      }
      if (li + 1 < n_local) {
        cur.advance(g.win, win_step);
        // the accumulator's z was read (above, before the barrier in normproj); A2 of
        // pair li was read by its last mlp0, complete before that chunk's mlp2
        if (!normproj(li + 1) || !ln2(li + 1)) break;
        gs.sync();
        if (gs.leader) {
          issue_mlp0(0);
          issue_mlp0(1);
        }
      }
    }
    if (gs.leader) {
      umma_commit(drain + 2);
      mbar_wait(drain + 2, 0, SCB_ERR_WAIT_ATTN);
    }
  } else {
    // ====== G4 (one thread per row): per hidden chunk, 2 GELU -> H -> [acc += H.(W2/2)^T] ======
    GroupSync gs{4, 32 * L::G4_WARPS, tid == 32 * (L::G1_WARPS + L::G2_WARPS + L::G3_WARPS + 3), status + 6,
                 abort_flag, 0u};
    for (int li = 0; li < n_local; ++li) {
      bool ok = true;
#pragma unroll 1
      for (int c = 0; c < 4; ++c) {
        const int b = c & 1, u = 2 * li + (c >> 1);
        if (!gs.wait(bar_hid + b, u & 1, SCB_ERR_WAIT_ATTN)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t col = L::C_HID + b * 64;
        // the row's 64 hidden columns of chunk c in two halves hf; the packed result of
        // a half goes to its first 16 columns (hidden 32 hf + 2j, + 1 at column 32 hf + j)
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          float hv[32];
          tmem_ld16x2(trow + col + 32 * hf, hv, trow + col + 32 * hf + 16, hv + 16);
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __half2 a = __floats2half2_rn(hv[2 * j], hv[2 * j + 1]);
            a = gelu2_tanh_h2(a);
            pk[j] = *reinterpret_cast<uint32_t*>(&a);
          }
          tmem_st16u(trow + col + 32 * hf, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        gs.sync();
        if (gs.leader) {
          tc_fence_after();
          // K step k = hidden 64 c + 16 k .. + 16, packed at column 32 (k / 2) + 8 (k % 2)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(tmem + L::C_ACC, tmem + col + 32 * (k >> 1) + 8 * (k & 1),
                        d128(L::W_2 + c * 64 * 128 + 32 * k), ID_T, 1);
          umma_commit(bar_out + b);
        }
      }
      if (!ok) break;
    }
    if (gs.leader) {
      umma_commit(drain + 3);
      mbar_wait(drain + 3, 0, SCB_ERR_WAIT_ATTN);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace scb
