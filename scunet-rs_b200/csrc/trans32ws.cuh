// The transformer half of a full-resolution ConvTransBlock (trans width T = 32, one
// head), warp-specialised: one CTA per SM streams pairs of 8x8 windows (128 tokens,
// one UMMA M tile) through three warp groups that work on different pairs at the
// same time, each issuing the UMMAs its own output feeds:
//
//   G1 (warps 0-3, one thread per token row): y_t rows by cp.async (two pairs
//      ahead) -> LN1 -> A1 -> [qkv = A1.Wqkv'^T + b] -> Q, K rows and V^T columns
//      -> [S = Q.K^T + E.F^T]
//   G2 (warps 4-7, one thread per row): softmax of its window's 64 scores -> P'
//      -> [O' = P'.[V0|V1], rowsum = P'.1] -> O = O'/rowsum
//      -> [x1 = O.Wproj^T + y_t.I + b_proj]
//   G3 (warps 8-15, two threads per row, one per column half): LN2(x1) -> A2
//      -> [hid = A2.W0'^T + b0'] -> GELU -> H -> [acc = x1 + H.W2^T + b2] -> z
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136; WMSA as tools/network_scunet.py:69-102)
//
// Everything that is linear in a UMMA operand runs on the tensor cores:
//  * biases: every A operand gets one extra K step from a resident "ones" tile
//    (K elements 0 and 1 = 1) whose B partner holds the bias split into an fp16
//    high part and an fp16 remainder, so the bias reaches fp32 accumulation intact;
//  * the LayerNorm affine maps are folded into the next weights on the host
//    (W' = W diag(gamma), b' = b + W beta): the kernels store (x - mu) rstd only;
//  * the attention scale 32^-1/2 and log2(e) are folded into the q rows of Wqkv';
//  * the relative-position bias is E.F^T: E is the one-hot [128 x 64] of each query
//    token's position in its window, F[key][m] = B(m, key) log2(e) (fp16), so S
//    arrives in TMEM with the bias added and in base 2;
//  * the softmax denominator is the row sum of the fp16 P' that the P.V product
//    uses, from one N = 16 UMMA against a row of ones;
//  * x1 = y_t + ...: the proj UMMA adds y_t through an identity B operand.
// The CUDA cores keep only LN statistics, the softmax max/exp2, GELU and the fp16
// packing. The shifted-window mask (cuda/scunet.cu:137-147) is applied in
// registers on the image's last window row/column only.
//
// Hand-offs between groups are mbarriers (UMMA commits, or thread arrivals for
// "TMEM read, columns free"); inside a group, one leader thread waits on the
// mbarrier and a named barrier releases the others. Every wait is bounded: a wait
// that times out records an error code and raises a CTA-wide abort flag, every
// other wait gives up as soon as it sees the flag, and each issuing thread drains
// its UMMAs before the CTA frees its TMEM and exits.
#pragma once
#include "trans.cuh"

namespace scb {

struct T32 {
  static constexpr int T = 32;
  // resident tiles (offsets from the 1024-aligned base); SW64 tiles have 64-byte
  // rows, SW128 tiles 128-byte rows
  static constexpr int W_QKV = 0;                  // [96 x 64 B]  Wqkv' (LN1 gamma, q scale folded)
  static constexpr int B_QKV = W_QKV + 96 * 64;    // [96 x 64 B]  bias hi/lo in K elements 0, 1
  static constexpr int W_PROJ = B_QKV + 96 * 64;   // [32 x 64 B]
  static constexpr int B_PROJ = W_PROJ + 32 * 64;  // [32 x 64 B]
  static constexpr int IDENT = B_PROJ + 32 * 64;   // [32 x 64 B]  identity (x1 += y_t)
  static constexpr int W_0 = IDENT + 32 * 64;      // [128 x 64 B] W0' (LN2 gamma folded)
  static constexpr int B_0 = W_0 + 128 * 64;       // [128 x 64 B]
  static constexpr int W_2 = B_0 + 128 * 64;       // 2 K blocks of [32 x 128 B], SW128
  static constexpr int B_2 = W_2 + 2 * 32 * 128;   // [32 x 64 B]
  static constexpr int ONES = B_2 + 32 * 64;       // [128 x 64 B] K elements 0, 1 = 1
  static constexpr int E1H = ONES + 128 * 64;      // [128 x 128 B] one-hot query position, SW128
  static constexpr int FB = E1H + 128 * 128;       // [128 x 128 B] rel-pos bias, key x query position
  static constexpr int ONES_B = FB + 128 * 128;    // [16 x 128 B] row 0 = 1 (softmax row sums)
  // pipeline buffers
  static constexpr int Y = ONES_B + 16 * 128;      // 3 x [128 x 64 B] y_t rows (A of the identity step)
  static constexpr int A1 = Y + 3 * 8192;          // [128 x 64 B] LN1 output
  static constexpr int Q = A1 + 8192;              // [128 x 64 B]
  static constexpr int K = Q + 8192;               // [128 x 64 B]
  static constexpr int VT = K + 8192;              // [64 x 128 B] rows (window, d), K = key, SW128
  static constexpr int P = VT + 8192;              // [128 x 128 B] P' (own window's 64 keys), SW128
  static constexpr int O = P + 16384;              // [128 x 64 B]
  static constexpr int A2 = O + 8192;              // [128 x 64 B] LN2 output
  static constexpr int H = A2 + 8192;              // 2 K blocks of [128 x 128 B] GELU(hidden), SW128
  static constexpr int BAR = H + 32768;
  static constexpr int SMEM = BAR + 256 + 1024;    // + alignment slack
  // TMEM columns
  static constexpr uint32_t C_QKV = 0, C_S = 128, C_OP = 128, C_SUM = 192, C_ACC = 256, C_HID = 384;
  static constexpr int THREADS = 512;
};

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// One 32x32b column: thread t of the warp gets row (lane base + t), column `taddr`.
// Waits for the load itself (one value: nothing to overlap it with).
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  tmem_wait_ld();
  asm volatile("" : "+r"(r));
  return __uint_as_float(r);
}

__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// Bounded mbarrier wait that also gives up when another group raised `abort_flag`;
// a timeout records `code` and raises the flag.
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                    unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    __nanosleep(32);  // a spinning leader would take issue slots from its SMSP's other warps
    if ((i & 63u) == 63u) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > 1000000000ull) {
        record_error(code);
        *abort_flag = 1u;
        return false;
      }
    }
  }
}

// A warp group's view of a wait: the leader polls, a named barrier releases the
// group, and every thread reads the same verdict (two alternating status slots, so
// the leader can post the next verdict while slow threads still read this one).
struct GroupSync {
  int id, n;
  bool leader;
  volatile uint32_t* status;  // 2 words
  volatile uint32_t* abort_flag;
  uint32_t seq;

  __device__ __forceinline__ bool wait(uint64_t* bar, uint32_t parity, unsigned code) {
    if (leader) status[seq & 1] = mbar_wait_abortable(bar, parity, abort_flag, code) ? 1u : 0u;
    named_bar(id, n);
    const bool ok = status[seq & 1] != 0;
    ++seq;
    if (ok) mbar_try_wait(bar, parity);  // this thread's own acquire of the completed phase
    return ok;
  }
  __device__ __forceinline__ void sync() { named_bar(id, n); }
};

__device__ __forceinline__ void set_half(uint4& v, int e, uint16_t h) {
  uint32_t* w = reinterpret_cast<uint32_t*>(&v);
  w[e >> 1] |= (uint32_t)h << ((e & 1) * 16);
}

__device__ __forceinline__ uint16_t half_bits(float f) { return __half_as_ushort(__float2half_rn(f)); }

// bias b as the fp16 pair (hi, lo) with hi + lo = b to ~2^-22 relative
__device__ __forceinline__ uint32_t bias_hilo(float b) {
  const __half hi = __float2half_rn(b);
  const float lo = b - __half2float(hi);
  return (uint32_t)__half_as_ushort(hi) | ((uint32_t)half_bits(lo) << 16);
}

__global__ void __launch_bounds__(T32::THREADS, 1) trans32_ws_kernel(const TransGeom g) {
  using L = T32;
  constexpr int T = 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::BAR);
  uint64_t* bar_qkv = bars + 0;
  uint64_t* bar_s = bars + 1;
  uint64_t* bar_o = bars + 2;
  uint64_t* bar_hid = bars + 3;
  uint64_t* bar_out = bars + 4;
  uint64_t* x1_done = bars + 5;   // [2], per x1 accumulator buffer
  uint64_t* so_free = bars + 7;   // G2 has read O' and the row sums (128 arrivals)
  uint64_t* acc_free = bars + 8;  // [2] G3 has read z (256 arrivals)
  uint64_t* drain = bars + 10;    // [3] one per issuing group
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + 13);
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* status = misc + 2;  // [3][2]

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane;  // TMEM lane = token row of the pair
  const int slot = row >> 6, tok = row & 63, qi = tok >> 3, qj = tok & 7;

  // ---- resident tiles ----
  stage_kmajor(sm + L::W_QKV, g.wqkv_f, 3 * T, T, T);
  stage_kmajor(sm + L::W_PROJ, g.wproj, T, T, T);
  stage_kmajor(sm + L::W_0, g.w0_f, 4 * T, T, T);
  stage_kmajor(sm + L::W_2, g.w2, T, 4 * T, 64);
  {
    // SW64 side tiles: bias hi/lo (qkv 96, proj 32, mlp0 128, mlp2 32 rows), ones, identity
    constexpr int R_BQ = 0, R_BP = 96, R_B0 = 128, R_B2 = 256, R_ONE = 288, R_ID = 416, R_END = 448;
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
      } else if (r < R_B2) {
        base = sm + L::B_0, rr = r - R_B0;
        if (c == 0) v.x = bias_hilo(g.b0_f[rr]);
      } else if (r < R_ONE) {
        base = sm + L::B_2, rr = r - R_B2;
        if (c == 0) v.x = bias_hilo(g.b2[rr]);
      } else if (r < R_ID) {
        base = sm + L::ONES, rr = r - R_ONE;
        if (c == 0) v.x = 0x3C003C00u;
      } else {
        base = sm + L::IDENT, rr = r - R_ID;
        if (c == (rr >> 3)) set_half(v, rr & 7, 0x3C00);
      }
      *reinterpret_cast<uint4*>(base + swz_off(rr, c, 64)) = v;
    }
    // SW128 tiles: one-hot query position (128 rows), rel-pos bias (128 key rows), row sums
    for (int i = tid; i < (128 + 128 + 16) * 8; i += blockDim.x) {
      const int r = i >> 3, c = i & 7;
      uint4 v = make_uint4(0u, 0u, 0u, 0u);
      uint8_t* base;
      int rr;
      if (r < 128) {
        base = sm + L::E1H, rr = r;
        const int m = rr & 63;
        if (c == (m >> 3)) set_half(v, m & 7, 0x3C00);
      } else if (r < 256) {
        base = sm + L::FB, rr = r - 128;
        const int kp = rr & 63, ki = kp >> 3, kj = kp & 7;
        // query position m = (c, e): B(m, key) = rp[(mi - ki + 7) * 15 + (mj - kj + 7)]
        const float* rp = g.rp + (c - ki + 7) * 15 + (7 - kj);
#pragma unroll
        for (int e = 0; e < 8; ++e) set_half(v, e, half_bits(rp[e] * 1.4426950408889634f));
      } else {
        base = sm + L::ONES_B, rr = r - 256;
        if (rr == 0) v = make_uint4(0x3C003C00u, 0x3C003C00u, 0x3C003C00u, 0x3C003C00u);
      }
      *reinterpret_cast<uint4*>(base + swz_off(rr, c, 128)) = v;
    }
  }
  if (tid == 0) {
    for (int i = 0; i < 13; ++i) {
      const uint32_t cnt = (bars + i == so_free) ? 128u : ((bars + i == acc_free || bars + i == acc_free + 1) ? 256u : 1u);
      mbar_init(bars + i, cnt);
    }
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
  auto locate = [&](int li, bool& lr, bool& lc, bool& st) -> long {
    const long win = 2 * (first + (long)li * gridDim.x) + slot;
    lr = lc = st = false;
    if (win >= g.win.n_windows) return -1;
    return win_token_pixel(g.win, win, qi, qj, lr, lc, st);
  };
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
                     ID_PV = make_idesc_f16(128, 64), ID_SUM = make_idesc_f16(128, 16),
                     ID_T = make_idesc_f16(128, T), ID_HID = make_idesc_f16(128, 4 * T);
  auto d64 = [&](int off) { return make_sdesc(sb + off, 64, SW_64B); };
  auto d128 = [&](int off) { return make_sdesc(sb + off, 128, SW_128B); };

  if (warp < 4) {
    // ======================= G1: y_t -> LN1 -> qkv -> Q, K, V^T -> S =======================
    GroupSync gs{1, 128, tid == 0, status, abort_flag, 0u};
    auto fetch = [&](int li) {
      bool lr, lc, st;
      const long pix = locate(li, lr, lc, st);
      uint8_t* dst = sm + L::Y + (li % 3) * 8192;
      const __half* src = pix >= 0 ? g.y + pix * T : g.y;
#pragma unroll
      for (int c = 0; c < 4; ++c) cp_async16(dst + swz_off(row, c, 64), src + 8 * c, pix >= 0);
    };
    if (n_local > 0) fetch(0);
    cp_async_commit();
    for (int li = 0; li < n_local; ++li) {
      if (li + 1 < n_local) {
        // buffer (li + 1) % 3 last held pair li - 2's y_t, an operand of its proj UMMA
        if (li >= 2 && !gs.wait(x1_done + ((li - 2) & 1), ((li - 2) >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
        fetch(li + 1);
      }
      cp_async_commit();
      cp_async_wait_1();  // this thread's row of pair li has landed
      {
        const uint8_t* yb = sm + L::Y + (li % 3) * 8192;
        float x[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) unpack8(*reinterpret_cast<const uint4*>(yb + swz_off(row, c, 64)), x + 8 * c);
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
#pragma unroll
        for (int j = 0; j < 32; ++j) x[j] = fmaf(x[j], rstd, nmr);
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(sm + L::A1 + swz_off(row, c, 64)) = pack8(x + 8 * c);
      }
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        umma_f16(tmem + L::C_QKV, d64(L::A1), d64(L::W_QKV), ID_QKV, 0);
        umma_f16(tmem + L::C_QKV, d64(L::A1 + 32), d64(L::W_QKV + 32), ID_QKV, 1);
        umma_f16(tmem + L::C_QKV, d64(L::ONES), d64(L::B_QKV), ID_QKV, 1);
        umma_commit(bar_qkv);
      }
      if (!gs.wait(bar_qkv, li & 1, SCB_ERR_WAIT_ATTN)) break;
      // Q, K, V^T of pair li - 1 are free once its P.V product has completed
      if (li >= 1 && !gs.wait(bar_o, (li - 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      {
        float q[32];
        tmem_ld16x2(trow + L::C_QKV, q, trow + L::C_QKV + 16, q + 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(sm + L::Q + swz_off(row, c, 64)) = pack8(q + 8 * c);
      }
      {
        float k[32];
        tmem_ld16x2(trow + L::C_QKV + 32, k, trow + L::C_QKV + 48, k + 16);
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(sm + L::K + swz_off(row, c, 64)) = pack8(k + 8 * c);
      }
      {
        float v[32];
        tmem_ld16x2(trow + L::C_QKV + 64, v, trow + L::C_QKV + 80, v + 16);
        // V^T: row (window slot, d), key = this token
        uint8_t* vb = sm + L::VT + slot * 32 * 128 + (tok & 7) * 2;
        const int kc = tok >> 3;
#pragma unroll
        for (int d = 0; d < 32; ++d)
          *reinterpret_cast<__half*>(vb + d * 128 + (((kc ^ d) & 7) << 4)) = __float2half_rn(v[d]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        // S reuses the columns of pair li - 1's O' and row sums: G2 must have read them
        const bool ok = li == 0 || mbar_wait_abortable(so_free, (li - 1) & 1, abort_flag, SCB_ERR_WAIT_ATTN);
        if (ok) {
          tc_fence_after();
          umma_f16(tmem + L::C_S, d64(L::Q), d64(L::K), ID_S, 0);
          umma_f16(tmem + L::C_S, d64(L::Q + 32), d64(L::K + 32), ID_S, 1);
#pragma unroll
          for (int k = 0; k < 4; ++k) umma_f16(tmem + L::C_S, d128(L::E1H + 32 * k), d128(L::FB + 32 * k), ID_S, 1);
          umma_commit(bar_s);
        }
      }
    }
    cp_async_wait_all();
    if (gs.leader) {
      umma_commit(drain + 0);
      mbar_wait(drain + 0, 0, SCB_ERR_WAIT_ATTN);
    }
  } else if (warp < 8) {
    // ======================= G2: softmax -> P' -> O'/rowsum -> O -> x1 =======================
    GroupSync gs{2, 128, tid == 160, status + 2, abort_flag, 0u};  // leaders sit on different SMSPs
    for (int li = 0; li < n_local; ++li) {
      if (!gs.wait(bar_s, li & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      bool last_row, last_col, st;
      (void)locate(li, last_row, last_col, st);
      {
        float s[64];
        tmem_ld16x2(trow + L::C_S + slot * 64, s, trow + L::C_S + slot * 64 + 16, s + 16);
        tmem_ld16x2(trow + L::C_S + slot * 64 + 32, s + 32, trow + L::C_S + slot * 64 + 48, s + 48);
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
        float m0 = s[0], m1 = s[1], m2 = s[2], m3 = s[3];
#pragma unroll
        for (int j = 4; j < 64; j += 4) {
          m0 = fmaxf(m0, s[j]);
          m1 = fmaxf(m1, s[j + 1]);
          m2 = fmaxf(m2, s[j + 2]);
          m3 = fmaxf(m3, s[j + 3]);
        }
        const float mx = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3));
#pragma unroll
        for (int j = 0; j < 64; ++j) s[j] = ex2_approx(s[j] - mx);
#pragma unroll
        for (int c = 0; c < 8; ++c) *reinterpret_cast<uint4*>(sm + L::P + swz_off(row, c, 128)) = pack8(s + 8 * c);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tmem + L::C_OP, d128(L::P + 32 * k), d128(L::VT + 32 * k), ID_PV, k);
#pragma unroll
        for (int k = 0; k < 4; ++k) umma_f16(tmem + L::C_SUM, d128(L::P + 32 * k), d128(L::ONES_B + 32 * k), ID_SUM, k);
        umma_commit(bar_o);
      }
      if (!gs.wait(bar_o, li & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      float o[32];
      tmem_ld16x2(trow + L::C_OP + slot * 32, o, trow + L::C_OP + slot * 32 + 16, o + 16);  // own window's half
      const float sum = tmem_ld1(trow + L::C_SUM);
      tc_fence_before();
      mbar_arrive(so_free);
      const float inv = __fdividef(1.f, sum);
#pragma unroll
      for (int j = 0; j < 32; ++j) o[j] *= inv;
      // O of pair li - 1 is an operand of its proj UMMA
      if (li >= 1 && !gs.wait(x1_done + ((li - 1) & 1), ((li - 1) >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
#pragma unroll
      for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(sm + L::O + swz_off(row, c, 64)) = pack8(o + 8 * c);
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        const int b = li & 1;
        // accumulator b last held pair li - 2's z: G3 must have read it
        const bool ok = li < 2 || mbar_wait_abortable(acc_free + b, ((li - 2) >> 1) & 1, abort_flag, SCB_ERR_WAIT_ATTN);
        if (ok) {
          tc_fence_after();
          const uint32_t d = tmem + L::C_ACC + b * T;
          const int yb = L::Y + (li % 3) * 8192;
          umma_f16(d, d64(L::O), d64(L::W_PROJ), ID_T, 0);
          umma_f16(d, d64(L::O + 32), d64(L::W_PROJ + 32), ID_T, 1);
          umma_f16(d, d64(yb), d64(L::IDENT), ID_T, 1);
          umma_f16(d, d64(yb + 32), d64(L::IDENT + 32), ID_T, 1);
          umma_f16(d, d64(L::ONES), d64(L::B_PROJ), ID_T, 1);
          umma_commit(x1_done + b);
        }
      }
    }
    if (gs.leader) {
      umma_commit(drain + 1);
      mbar_wait(drain + 1, 0, SCB_ERR_WAIT_ATTN);
    }
  } else {
    // ======================= G3: LN2 -> hidden -> GELU -> mlp2 -> z =======================
    GroupSync gs{3, 256, tid == 320, status + 4, abort_flag, 0u};
    const int hf = (warp - 8) >> 2;  // column half of the row this thread owns
    for (int li = 0; li < n_local; ++li) {
      const int b = li & 1;
      const uint32_t acc = L::C_ACC + b * T;
      if (!gs.wait(x1_done + b, (li >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      {
        float x[32];
        tmem_ld16x2(trow + acc, x, trow + acc + 16, x + 16);
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
        float a[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) a[j] = fmaf(hf ? x[16 + j] : x[j], rstd, nmr);  // no runtime index: x stays in registers
#pragma unroll
        for (int c = 0; c < 2; ++c)
          *reinterpret_cast<uint4*>(sm + L::A2 + swz_off(row, 2 * hf + c, 64)) = pack8(a + 8 * c);
      }
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        umma_f16(tmem + L::C_HID, d64(L::A2), d64(L::W_0), ID_HID, 0);
        umma_f16(tmem + L::C_HID, d64(L::A2 + 32), d64(L::W_0 + 32), ID_HID, 1);
        umma_f16(tmem + L::C_HID, d64(L::ONES), d64(L::B_0), ID_HID, 1);
        umma_commit(bar_hid);
      }
      if (!gs.wait(bar_hid, li & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float hv[32];
        const uint32_t col = trow + L::C_HID + hf * 64 + h2 * 32;
        tmem_ld16x2(col, hv, col + 16, hv + 16);
        uint32_t pk[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          __half2 a = __floats2half2_rn(hv[2 * j], hv[2 * j + 1]);
          a = gelu_tanh_h2(a);
          pk[j] = *reinterpret_cast<uint32_t*>(&a);
        }
        uint8_t* hb = sm + L::H + hf * 16384;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(hb + swz_off(row, h2 * 4 + c, 128)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      tc_fence_before();
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        const uint32_t d = tmem + acc;
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(d, d128(L::H + kb * 16384 + 32 * k), d128(L::W_2 + kb * 4096 + 32 * k), ID_T, 1);
        umma_f16(d, d64(L::ONES), d64(L::B_2), ID_T, 1);
        umma_commit(bar_out);
      }
      if (!gs.wait(bar_out, li & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      float z[16];
      tmem_ld16(trow + acc + hf * 16, z);
      tc_fence_before();
      mbar_arrive(acc_free + b);
      bool lr, lc, st;
      const long pix = locate(li, lr, lc, st);
      if (pix >= 0 && st) {
        uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T + hf * 16);
        dst[0] = pack8(z);
        dst[1] = pack8(z + 8);
      }
    }
    if (gs.leader) {
      umma_commit(drain + 2);
      mbar_wait(drain + 2, 0, SCB_ERR_WAIT_ATTN);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == 0) tmem_dealloc(tmem, 512);
}

}  // namespace scb
