// The transformer half of a full-resolution ConvTransBlock (trans width T = 32, one
// head), warp-specialised: one CTA per SM streams pairs of 8x8 windows (128 tokens,
// one UMMA M tile) through four warp groups that work on different pairs at the
// same time, each issuing the UMMAs its own output feeds ([..] = a UMMA):
//
//   G1 (4 warps, one thread per token row): y_t rows by cp.async (a pair ahead)
//      -> LN1 -> A1 -> [qkv = A1.Wqkv'^T + b] -> Q (TMEM), K rows and V rows
//      (shared memory) -> [S = Q.K^T]
//   G2 (8 warps, two threads per row, 32 keys each): + rel-pos bias, mask, max
//      (exchanged through shared memory), P' = 2^(s - max)
//      -> [O' | rowsum = P'.[V0 | V1 | 1]]
//   G3 (4 warps, one thread per row): O = O' / rowsum -> [x1 = O.Wproj^T + y_t.I +
//      b_proj] -> LN2(x1) -> A2 -> [hid = A2.W0'^T + b0'] for the next pair while G4
//      works on this one, in two 64-column chunks with their own TMEM buffers;
//      z = acc + b2 -> Z
//   G4 (4 warps, one thread per row, the chunk's 64 columns in two halves): per
//      chunk, 2 GELU(hid) -> H -> [acc += H.(W2/2)^T] (8 warps, two threads per row,
//      measured 2.5 % slower: the SM's issue slots are shared by all groups)
//
//   x  = y_t;  x1 = x + proj(WMSA(LN1(x)));  z = x1 + mlp2(GELU(mlp0(LN2(x1))))
//   (tools/network_scunet.py:128-136; WMSA as tools/network_scunet.py:69-102)
//
// Operands the threads produce (A1, Q, P', O, A2, H) are written to tensor memory
// with tcgen05.st as packed fp16 and read by the UMMAs as their A operand, so a
// UMMA reads only its B operand from shared memory. Measured on B200: an M = 128,
// K = 16 UMMA with A in shared memory costs ~32 + N/4 cycles of shared-memory
// bandwidth (2.5x its tensor time at N = 32); one issuing thread sustains one UMMA
// per ~50 cycles, so the groups issue their own UMMAs.
//
// Work moved onto the tensor cores:
//  * biases (qkv, proj, mlp0): one extra K step from a resident "ones" tile (K
//    elements 0 and 1 = 1) whose B partner holds the bias split into an fp16 high
//    part and an fp16 remainder, so the bias reaches fp32 accumulation intact;
//  * the LayerNorm affine maps are folded into the next weights on the host
//    (W' = W diag(gamma), b' = b + W beta): the kernel stores (x - mu) rstd only;
//  * the attention scale 32^-1/2 and log2(e) are folded into the q rows of Wqkv';
//  * the softmax denominator is the row sum of the fp16 P' that P.V uses: the
//    MN-major V operand carries a ones column (N = 80);
//  * x1 = y_t + ...: the proj UMMA adds y_t through an identity B operand;
//  * the GELU's factor 1/2 is folded into W2 (exact in fp16).
// The shifted-window mask (cuda/scunet.cu:137-147) is applied in registers on the
// image's last window row/column only.
//
// Hand-offs between groups are mbarriers (UMMA commits, or thread arrivals for
// "TMEM read, columns free"); inside a group, one leader thread waits on the
// mbarrier (sleeping in hardware) and a named barrier releases the others. Every
// wait is bounded: a wait that times out records an error code and raises a
// CTA-wide abort flag, every other wait gives up as soon as it sees the flag, and
// each issuing thread drains its UMMAs before the CTA frees its TMEM and exits.
#pragma once
#include "trans.cuh"

namespace scb {

struct T32 {
  static constexpr int T = 32;
  // resident shared-memory tiles (offsets from the 1024-aligned base); SW64 tiles
  // have 64-byte rows, SW128 tiles 128-byte rows
  static constexpr int W_QKV = 0;                  // [96 x 64 B]  Wqkv' (LN1 gamma, q scale folded)
  static constexpr int B_QKV = W_QKV + 96 * 64;    // [96 x 64 B]  bias hi/lo in K elements 0, 1
  static constexpr int W_PROJ = B_QKV + 96 * 64;   // [32 x 64 B]
  static constexpr int B_PROJ = W_PROJ + 32 * 64;  // [32 x 64 B]
  static constexpr int IDENT = B_PROJ + 32 * 64;   // [32 x 64 B]  identity (x1 += y_t)
  static constexpr int W_0 = IDENT + 32 * 64;      // [128 x 64 B] W0' (LN2 gamma folded)
  static constexpr int B_0 = W_0 + 128 * 64;       // [128 x 64 B]
  static constexpr int W_2 = B_0 + 128 * 64;       // 2 K blocks of [32 x 128 B], SW128: W2 / 2
  static constexpr int ONES = W_2 + 2 * 32 * 128;  // [128 x 64 B] K elements 0, 1 = 1
  // relative-position bias in log2 units, fp32 [64 query positions][64 keys]; the
  // 16-byte chunks of row q are XOR-swizzled by q % 8 within each 128-byte half
  static constexpr int RPB = ONES + 128 * 64;
  // pipeline buffers (B operands and the y_t rows)
  static constexpr int Y = RPB + 64 * 64 * 4;      // 3 x [128 x 64 B] y_t rows (A of the identity step)
  static constexpr int K = Y + 3 * 8192;           // 2 x [128 x 64 B] keys
  // V as the MN-major B operand of P.V (N = (window, d) contiguous per key): per
  // buffer an atom [64 keys x 128 B] holding [V_0 | V_1] and an atom whose first N
  // element is 1 (N = 64: the softmax row sums)
  static constexpr int V = K + 2 * 8192;
  static constexpr int V_BYTES = 2 * 8192;
  static constexpr int B2F = V + 2 * V_BYTES;      // mlp2 bias, 32 floats
  static constexpr int RED = B2F + 128;            // [2 halves x 128 rows] softmax partial maxima
  static constexpr int BAR = RED + 1024;
  static constexpr int SMEM = BAR + 256 + 1024;    // + alignment slack
  // TMEM columns. UMMA A operands written by the threads (tcgen05.st) are packed
  // fp16 pairs, 8 columns per K step of 16. Pair i uses score buffer SB(i & 1):
  // its qkv accumulator [0, 96), then S [0, 128), then P' [0, 32) (A of P.V) with
  // O' [32, 96) and the row sums at 96 (N = 80).
  static constexpr uint32_t C_SB = 0;     // 2 x 128
  static constexpr uint32_t C_A1 = 256;   // LN1 output, A of qkv (16)
  static constexpr uint32_t C_Q = 272;    // Q, A of S (16)
  static constexpr uint32_t C_A2 = 288;   // LN2 output, A of mlp0 (16)
  static constexpr uint32_t C_O = 304;    // O / rowsum, A of proj (16)
  static constexpr uint32_t C_ACC = 320;  // 2 x 32: x1, then x1 + mlp2 (z)
  static constexpr uint32_t C_HID = 384;  // hidden accumulator (128); GELU(hidden) (A of
                                          // mlp2) overwrites the first 32 of each half
  static constexpr int G1_WARPS = 4, G2_WARPS = 8, G3_WARPS = 4, G4_WARPS = 4;
  static constexpr int THREADS = 32 * (G1_WARPS + G2_WARPS + G3_WARPS + G4_WARPS);
};

__device__ __forceinline__ void named_bar(int id, int n) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}


// Bounded mbarrier wait that also gives up when another group raised `abort_flag`;
// a timeout records `code` and raises the flag. (Polling without the suspend hint
// before sleeping was measured: the leader resumes ~100 cycles sooner per round trip,
// but the polling takes issue slots from the working warps of the SM, and the
// full-resolution and half-resolution kernels got 3-40 % slower.)
__device__ __forceinline__ bool mbar_wait_abortable(uint64_t* bar, uint32_t parity, volatile uint32_t* abort_flag,
                                                    unsigned code) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (;;) {
    // sleeps in hardware (no issue slots taken from the SMSP's other warps) until
    // the phase completes or ~20 us pass
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (*abort_flag) return false;
    if (globaltimer() - t0 > 1000000000ull) {
      record_error(code);
      *abort_flag = 1u;
      return false;
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
  // Barriers that complete once per pair come in pairs indexed by the pair's parity
  // wherever a waiter could otherwise see the barrier two phases ahead of it.
  uint64_t* bar_qkv = bars + 0;
  uint64_t* bar_s = bars + 1;     // [2] per score buffer: S committed
  uint64_t* bar_o = bars + 3;     // [2] per score buffer: P.V committed
  uint64_t* x1_done = bars + 5;   // [2] per x1 accumulator buffer: proj committed
  uint64_t* so_free = bars + 7;   // [2] per score buffer: G3 has read O' and the row sums (128 arrivals)
  uint64_t* bar_hid = bars + 9;   // [2] per hidden chunk: mlp0 committed
  uint64_t* bar_out = bars + 11;  // [2] per hidden chunk: its mlp2 K steps committed
  uint64_t* drain = bars + 13;    // [4] one per issuing group
  constexpr int NBAR = 17;
  uint32_t* misc = reinterpret_cast<uint32_t*>(bars + NBAR);
  static_assert(17 * 8 + 10 * 4 <= 256, "barrier region");
  uint32_t* tmem_slot = misc;
  volatile uint32_t* abort_flag = misc + 1;
  volatile uint32_t* status = misc + 2;  // [4][2]
  float* red = reinterpret_cast<float*>(sm + L::RED);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int row = (warp & 3) * 32 + lane;  // TMEM lane = token row of the pair
  const int slot = row >> 6, tok = row & 63, qi = tok >> 3, qj = tok & 7;

  // ---- resident tiles ----
  stage_kmajor(sm + L::W_QKV, g.wqkv_f, 3 * T, T, T);
  stage_kmajor(sm + L::W_PROJ, g.wproj, T, T, T);
  stage_kmajor(sm + L::W_0, g.w0_f, 4 * T, T, T);
  // W2 / 2 (exact in fp16): the GELU below returns 2 GELU(x)
  for (int idx = tid; idx < T * (4 * T / 8); idx += blockDim.x) {
    const int r = idx >> 4, j = idx & 15, blk = j >> 3;
    uint4 u = __ldg(reinterpret_cast<const uint4*>(g.w2 + (long)r * 4 * T + j * 8));
    __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
    for (int e = 0; e < 4; ++e) h[e] = __hmul2(h[e], __float2half2_rn(0.5f));
    *reinterpret_cast<uint4*>(sm + L::W_2 + blk * T * 128 + swz_off(r, j & 7, 128)) = u;
  }
  if (tid < T) reinterpret_cast<float*>(sm + L::B2F)[tid] = g.b2[tid];
  {
    // SW64 side tiles: bias hi/lo (qkv 96, proj 32, mlp0 128 rows), ones, identity
    constexpr int R_BQ = 0, R_BP = 96, R_B0 = 128, R_ONE = 256, R_ID = 384, R_END = 416;
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
      } else if (r < R_ID) {
        base = sm + L::ONES, rr = r - R_ONE;
        if (c == 0) v.x = 0x3C003C00u;
      } else {
        base = sm + L::IDENT, rr = r - R_ID;
        if (c == (rr >> 3)) set_half(v, rr & 7, 0x3C00);
      }
      *reinterpret_cast<uint4*>(base + swz_off(rr, c, 64)) = v;
    }
    // the ones atoms of both V buffers (64 key rows each: N element 64 = 1)
    for (int i = tid; i < 128 * 8; i += blockDim.x) {
      const int q = i >> 3, c = i & 7;  // buffer q / 64, key row q % 64
      *reinterpret_cast<uint4*>(sm + L::V + (q >> 6) * L::V_BYTES + 8192 + swz_off(q & 63, c, 128)) =
          make_uint4(c == 0 ? 0x3C00u : 0u, 0u, 0u, 0u);
    }
    // rel-pos bias B(query m, key k) = rp[(mi - ki + 7) * 15 + (mj - kj + 7)] log2(e)
    float* rpb = reinterpret_cast<float*>(sm + L::RPB);
    for (int i = tid; i < 64 * 64; i += blockDim.x) {
      const int m = i >> 6, k = i & 63, c = k >> 2;
      const float v = g.rp[((m >> 3) - (k >> 3) + 7) * 15 + ((m & 7) - (k & 7) + 7)] * 1.4426950408889634f;
      rpb[m * 64 + (((c & 8) | ((c ^ m) & 7)) << 2) + (k & 3)] = v;
    }
  }
  if (tid == 0) {
    for (int i = 0; i < NBAR; ++i) mbar_init(bars + i, (i == 7 || i == 8) ? 128u : 1u);
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
  const int win_step = 2 * (int)gridDim.x;  // a thread's window advances by this per pair
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
                     ID_HID = make_idesc_f16(128, 4 * T);
  auto d64 = [&](int off) { return make_sdesc(sb + off, 64, SW_64B); };
  auto d128 = [&](int off) { return make_sdesc(sb + off, 128, SW_128B); };

  if (warp < L::G1_WARPS) {
    // ====== G1: y_t -> LN1 -> [qkv] -> Q (TMEM), K, V^T (smem) -> [S] ======
    GroupSync gs{1, 32 * L::G1_WARPS, tid == 0, status, abort_flag, 0u};
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    // the cursor stands at pair li: the y_t rows of the warp's 32 tokens, lane l copying
    // 16-byte chunk l % 4 of rows l / 4 + 8 k (pixel by shuffle from the row's lane), so
    // that one copy instruction covers eight whole 64-byte rows
    auto fetch = [&](int li) {
      bool lr, lc, st;
      const long pix = cur.pixel(g.win, qi, qj, lr, lc, st);
      uint8_t* dst = sm + L::Y + (li % 3) * 8192;
      const int c = lane & 3;
#pragma unroll
      for (int k = 0; k < 4; ++k) {
        const int sl = (lane >> 2) + 8 * k;
        const long pk = __shfl_sync(0xffffffffu, pix, sl);
        const __half* src = pk >= 0 ? g.y + pk * T : g.y;
        cp_async16(dst + swz_off((warp & 3) * 32 + sl, c, 64), src + 8 * c, pk >= 0);
      }
    };
    if (n_local > 0) fetch(0);
    cp_async_commit();
    for (int li = 0; li < n_local; ++li) {
      const uint32_t sbuf = L::C_SB + (li & 1) * 128;
      if (li + 1 < n_local) {
        // buffer (li + 1) % 3 last held pair li - 2's y_t, an operand of its proj UMMA
        if (li >= 2 && !gs.wait(x1_done + ((li - 2) & 1), ((li - 2) >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
        cur.advance(g.win, win_step);
        fetch(li + 1);
      }
      cp_async_commit();
      cp_async_wait_1();  // this thread's copies of pair li have landed,
      __syncwarp();       // and those of the other lanes, which hold this row's chunks
      {
        const uint8_t* yb = sm + L::Y + (li % 3) * 8192;
        float x[32];
#pragma unroll
        for (int c = 0; c < 4; ++c) unpack8(*reinterpret_cast<const uint4*>(yb + swz_off(row, c, 64)), x + 8 * c);
        uint32_t a[16];
        ln_pack_f32x2<T>(x, a);
        tmem_st16u(trow + L::C_A1, a);  // (pair li - 1's qkv UMMA has completed)
        tmem_wait_st();
      }
      fence_proxy_async_smem();  // the y_t rows (cp.async) are read by proj's identity step
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        // score buffer li & 1 held pair li - 2 until G2 read its O' (after its P.V)
        const bool ok = li < 2 || mbar_wait_abortable(so_free + (li & 1), ((li - 2) >> 1) & 1, abort_flag,
                                                        SCB_ERR_WAIT_ATTN);
        if (ok) {
          tc_fence_after();
          umma_f16_ts(tmem + sbuf, tmem + L::C_A1, d64(L::W_QKV), ID_QKV, 0);
          umma_f16_ts(tmem + sbuf, tmem + L::C_A1 + 8, d64(L::W_QKV + 32), ID_QKV, 1);
          umma_f16(tmem + sbuf, d64(L::ONES), d64(L::B_QKV), ID_QKV, 1);
          umma_commit(bar_qkv);
        }
      }
      if (!gs.wait(bar_qkv, li & 1, SCB_ERR_WAIT_ATTN)) break;
      // Q of pair li - 1 is an operand of its S UMMA (K and V^T buffers li & 1 were
      // freed with score buffer li & 1)
      if (li >= 1 && !gs.wait(bar_s + ((li - 1) & 1), ((li - 1) >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      {
        float q[32];
        tmem_ld16x2(trow + sbuf, q, trow + sbuf + 16, q + 16);
        uint32_t pq[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) pq[j] = pack_half2(q[2 * j], q[2 * j + 1]);
        tmem_st16u(trow + L::C_Q, pq);
      }
      {
        float k[32];
        tmem_ld16x2(trow + sbuf + 32, k, trow + sbuf + 48, k + 16);
        uint8_t* kb = sm + L::K + (li & 1) * 8192;
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(kb + swz_off(row, c, 64)) = pack8(k + 8 * c);
      }
      {
        float v[32];
        tmem_ld16x2(trow + sbuf + 64, v, trow + sbuf + 80, v + 16);
        // V, MN-major: key row tok, N elements 32 slot .. 32 slot + 31
        uint8_t* vb = sm + L::V + (li & 1) * L::V_BYTES;
#pragma unroll
        for (int c = 0; c < 4; ++c) *reinterpret_cast<uint4*>(vb + swz_off(tok, 4 * slot + c, 128)) = pack8(v + 8 * c);
      }
      tmem_wait_st();
      tc_fence_before();
      fence_proxy_async_smem();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        const int kb = L::K + (li & 1) * 8192;
        umma_f16_ts(tmem + sbuf, tmem + L::C_Q, d64(kb), ID_S, 0);
        umma_f16_ts(tmem + sbuf, tmem + L::C_Q + 8, d64(kb + 32), ID_S, 1);
        umma_commit(bar_s + (li & 1));
      }
    }
    cp_async_wait_all();
    if (gs.leader) {
      umma_commit(drain + 0);
      mbar_wait(drain + 0, 0, SCB_ERR_WAIT_ATTN);
    }
  } else if (warp < L::G1_WARPS + L::G2_WARPS) {
    // ====== G2 (two threads per row, 32 keys each): softmax -> P' -> [O', rowsum] ======
    GroupSync gs{2, 32 * L::G2_WARPS, tid == 160, status + 2, abort_flag, 0u};  // leaders sit on different SMSPs
    const int hf = (warp - L::G1_WARPS) >> 2;
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    for (int li = 0; li < n_local; ++li, cur.advance(g.win, win_step)) {
      const uint32_t sbuf = L::C_SB + (li & 1) * 128;
      if (!gs.wait(bar_s + (li & 1), (li >> 1) & 1, SCB_ERR_WAIT_ATTN)) break;
      tc_fence_after();
      bool last_row, last_col, st;
      (void)cur.pixel(g.win, qi, qj, last_row, last_col, st);
      {
        float s[32];  // keys 32 hf .. 32 hf + 31 of the row's own window
        tmem_ld16x2(trow + sbuf + slot * 64 + hf * 32, s, trow + sbuf + slot * 64 + hf * 32 + 16, s + 16);
        {
          const float* rb = reinterpret_cast<const float*>(sm + L::RPB) + tok * 64;
#pragma unroll
          for (int c = 0; c < 8; ++c) {
            const float4 bb = *reinterpret_cast<const float4*>(rb + ((hf * 8 + ((c ^ tok) & 7)) << 2));
            const float2 lo = __fadd2_rn(make_float2(s[4 * c], s[4 * c + 1]), make_float2(bb.x, bb.y));
            const float2 hi = __fadd2_rn(make_float2(s[4 * c + 2], s[4 * c + 3]), make_float2(bb.z, bb.w));
            s[4 * c] = lo.x;
            s[4 * c + 1] = lo.y;
            s[4 * c + 2] = hi.x;
            s[4 * c + 3] = hi.y;
          }
        }
        if (last_row || last_col) {  // warp-uniform: a warp's 32 tokens share one window
          // the cyclic shift put tokens from opposite image edges into the last window
          // row / column; a token attends only to keys from its own side
          // (cuda/scunet.cu:137-147). Key 32 hf + j sits in window row 4 hf + j / 8.
          const bool rmask = last_row && ((qi < 4) != (hf == 0));
          const bool qleft = qj < 4;
#pragma unroll
          for (int j = 0; j < 32; ++j) s[j] = (rmask || (last_col && (qleft != ((j & 7) < 4)))) ? -INFINITY : s[j];
        }
        float mx = row_max<32>(s);
        red[hf * 128 + row] = mx;
        tmem_wait_ld();
        tc_fence_before();
        gs.sync();  // both halves of the row have read S (P' overwrites it) and posted their maxima
        tc_fence_after();
        mx = fmaxf(mx, red[(hf ^ 1) * 128 + row]);
        // P' = 2^(s - max) as packed fp16, the precision the P.V operand has anyway;
        // the row sum comes from the same fp16 values (the ones row of V^T)
        uint32_t p[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const float2 d = __fadd2_rn(make_float2(s[2 * j], s[2 * j + 1]), make_float2(-mx, -mx));
          p[j] = ex2_approx_h2(pack_half2(d.x, d.y));
        }
        tmem_st16u(trow + sbuf + hf * 16, p);
        tmem_wait_st();
      }
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        const uint32_t vb = sb + L::V + (li & 1) * L::V_BYTES;
#pragma unroll
        for (int k = 0; k < 4; ++k)  // K step k = keys 16k .. 16k + 15 = two 8-row groups
          umma_f16_ts(tmem + sbuf + 32, tmem + sbuf + 8 * k, make_sdesc_lbo_sbo(vb + 2048 * k, 8192, 1024, SW_128B),
                      ID_PV, k);
        umma_commit(bar_o + (li & 1));
      }
    }
    if (gs.leader) {
      umma_commit(drain + 1);
      mbar_wait(drain + 1, 0, SCB_ERR_WAIT_ATTN);
    }
  } else if (warp < L::G1_WARPS + L::G2_WARPS + L::G3_WARPS) {
    // ====== G3 (one thread per row): O = O'/rowsum -> [x1]; LN2(x1) -> A2 -> [hidden];
    //        z out ======
    // It runs a pair ahead of G4: proj and LN2 of pair li + 1 while G4 applies GELU to pair
    // li; the hidden layer is two 64-column chunks with their own buffers, and mlp0
    // of chunk c of pair li + 1 is issued as soon as mlp2's K steps of chunk c of
    // pair li (the last reader of that buffer) have completed, so the GELU warps
    // find the next chunk computed while they work on the current one.
    GroupSync gs{3, 32 * L::G3_WARPS, tid == 32 * (L::G1_WARPS + L::G2_WARPS + 2), status + 4, abort_flag, 0u};
    WinCursor cur;
    cur.init(g.win, 2 * first + slot);
    auto ln2 = [&](int li) -> bool {  // x1 of pair li -> A2 (TMEM)
      const int b = li & 1;
      if (!gs.wait(x1_done + b, (li >> 1) & 1, SCB_ERR_WAIT_ATTN)) return false;
      tc_fence_after();
      float x[32];
      tmem_ld16x2(trow + L::C_ACC + b * T, x, trow + L::C_ACC + b * T + 16, x + 16);
      uint32_t a[16];
      ln_pack_f32x2<T>(x, a);
      tmem_st16u(trow + L::C_A2, a);
      tmem_wait_st();
      tc_fence_before();
      return true;
    };
    constexpr uint32_t ID_H64 = make_idesc_f16(128, 64);
    auto issue_mlp0 = [&](int c) {  // hidden columns [64 c, 64 c + 64) -> buffer c
      tc_fence_after();
      const uint32_t d = tmem + L::C_HID + c * 64;
      umma_f16_ts(d, tmem + L::C_A2, d64(L::W_0 + c * 64 * 64), ID_H64, 0);
      umma_f16_ts(d, tmem + L::C_A2 + 8, d64(L::W_0 + c * 64 * 64 + 32), ID_H64, 1);
      umma_f16(d, d64(L::ONES), d64(L::B_0 + c * 64 * 64), ID_H64, 1);
      umma_commit(bar_hid + c);
    };
    // O' / rowsum of pair li -> O (TMEM) -> [x1 = O.Wproj^T + y_t.I + b_proj]. The O
    // columns were last read by pair li - 1's proj, which ln2(li - 1) waited for; the
    // accumulator li & 1 last held pair li - 2's z, which this group has read.
    auto normproj = [&](int li) -> bool {
      const int b = li & 1;
      const uint32_t sbuf = L::C_SB + b * 128;
      if (!gs.wait(bar_o + b, (li >> 1) & 1, SCB_ERR_WAIT_ATTN)) return false;
      tc_fence_after();
      float o[32];
      tmem_ld16x2(trow + sbuf + 32 + slot * 32, o, trow + sbuf + 48 + slot * 32, o + 16);  // own window's half
      const float inv = __fdividef(1.f, tmem_ld1(trow + sbuf + 32 + 64));
      tc_fence_before();
      mbar_arrive(so_free + b);  // score buffer b may take pair li + 2's qkv
      uint32_t po[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const float2 v = __fmul2_rn(make_float2(o[2 * j], o[2 * j + 1]), make_float2(inv, inv));
        po[j] = pack_half2(v.x, v.y);
      }
      tmem_st16u(trow + L::C_O, po);
      tmem_wait_st();
      tc_fence_before();
      gs.sync();
      if (gs.leader) {
        tc_fence_after();
        const uint32_t d = tmem + L::C_ACC + b * T;
        const int yb = L::Y + (li % 3) * 8192;
        umma_f16_ts(d, tmem + L::C_O, d64(L::W_PROJ), ID_T, 0);
        umma_f16_ts(d, tmem + L::C_O + 8, d64(L::W_PROJ + 32), ID_T, 1);
        umma_f16(d, d64(yb), d64(L::IDENT), ID_T, 1);
        umma_f16(d, d64(yb + 32), d64(L::IDENT + 32), ID_T, 1);
        umma_f16(d, d64(L::ONES), d64(L::B_PROJ), ID_T, 1);
        umma_commit(x1_done + b);
      }
      return true;
    };
    bool ok = n_local > 0 && normproj(0) && ln2(0);
    if (ok) {
      gs.sync();
      if (gs.leader) {
        issue_mlp0(0);
        issue_mlp0(1);
      }
    }
    for (int li = 0; ok && li < n_local; ++li, cur.advance(g.win, win_step)) {
      const bool more = li + 1 < n_local;
      if (more) {
        // A2 of pair li is read by both of its mlp0 chunks (one issuer: chunk 1's
        // commit covers chunk 0)
        if (!normproj(li + 1) || !gs.wait(bar_hid + 1, li & 1, SCB_ERR_WAIT_ATTN) || !ln2(li + 1)) break;
      }
      if (!gs.wait(bar_out + 0, li & 1, SCB_ERR_WAIT_ATTN)) break;
      if (more && gs.leader) issue_mlp0(0);
      // chunk 1's mlp2 has completed: z is final
      if (!gs.wait(bar_out + 1, li & 1, SCB_ERR_WAIT_ATTN)) break;
      if (more && gs.leader) issue_mlp0(1);
      tc_fence_after();
      const int b = li & 1;
      float z[32];
      tmem_ld16x2(trow + L::C_ACC + b * T, z, trow + L::C_ACC + b * T + 16, z + 16);
      tc_fence_before();
      bool lr, lc, st;
      const long pix = cur.pixel(g.win, qi, qj, lr, lc, st);
      {
        const float4* b24 = reinterpret_cast<const float4*>(sm + L::B2F);
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const float4 bb = b24[q];
          const float2 lo = __fadd2_rn(make_float2(z[4 * q], z[4 * q + 1]), make_float2(bb.x, bb.y));
          const float2 hi = __fadd2_rn(make_float2(z[4 * q + 2], z[4 * q + 3]), make_float2(bb.z, bb.w));
          z[4 * q] = lo.x;
          z[4 * q + 1] = lo.y;
          z[4 * q + 2] = hi.x;
          z[4 * q + 3] = hi.y;
        }
        if (pix >= 0 && st) {
          uint4* dst = reinterpret_cast<uint4*>(g.z + pix * (2 * T) + T);
#pragma unroll
          for (int c = 0; c < 4; ++c) dst[c] = pack8(z + 8 * c);
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
      for (int c = 0; c < 2 && ok; ++c) {
        if (!gs.wait(bar_hid + c, li & 1, SCB_ERR_WAIT_ATTN)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // the row's 64 hidden columns of chunk c in two halves hf; the packed result
        // of a half (A of mlp2) goes to its first 16 columns, after they have been read
#pragma unroll
        for (int hf = 0; hf < 2; ++hf) {
          const uint32_t col = L::C_HID + c * 64 + hf * 32;
          float hv[32];
          tmem_ld16x2(trow + col, hv, trow + col + 16, hv + 16);
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            __half2 a = __floats2half2_rn(hv[2 * j], hv[2 * j + 1]);
            a = gelu2_tanh_h2(a);
            pk[j] = *reinterpret_cast<uint32_t*>(&a);
          }
          tmem_st16u(trow + col, pk);
        }
        tmem_wait_st();
        tc_fence_before();
        gs.sync();
        if (gs.leader) {
          tc_fence_after();
          const uint32_t d = tmem + L::C_ACC + (li & 1) * T;
          // K steps of chunk c: hidden [64 c + 16 k, + 16) sits at H columns
          // C_HID + 64 c + 32 (k / 2) + 8 (k % 2)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16_ts(d, tmem + L::C_HID + c * 64 + (k >> 1) * 32 + (k & 1) * 8,
                        d128(L::W_2 + c * 4096 + 32 * k), ID_T, 1);
          umma_commit(bar_out + c);
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
