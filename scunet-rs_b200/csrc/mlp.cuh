// The MLP of a transformer half at 1/4 and 1/8 resolution (trans width T = 128,
// 256), where the transformer runs as separate launches, in ONE kernel:
//
//   z = x1 + mlp2(GELU(mlp0(a)))      a = LN2(x1)   (tools/network_scunet.py:128-136)
//
// The 4T-wide hidden layer never leaves the SM. Persistent CTAs take tiles of 128
// tokens; per tile the hidden layer is produced in 128-wide chunks j:
//
//   H_j   [128 x 128] = a . W0[128 j : 128 j + 128]^T      (UMMA, TMEM, two buffers)
//   Hs_j  = GELU(H_j + b0_j) in fp16                      (epilogue warps -> smem)
//   acc   [128 x T]  += Hs_j . W2[:, 128 j : 128 j + 128]^T (UMMA, TMEM)
//
// Warp 0 streams the tile's a (once) and the weights' 64-wide K blocks through a
// ring of shared-memory stages with TMA; warp 1 issues the UMMAs, H_{j+1} before
// acc += Hs_j, so the tensor pipe computes the next chunk while the 16 epilogue warps
// evaluate GELU of this one (four warps per TMEM lane quarter, each a quarter of the
// columns; 8 warps measured 4 % slower at T = 128) and finally write z = acc + b2 + x1
// in place over x1.
// HBM traffic per token: a (2T bytes) in, x1 (2T) in, z (2T) out; the weights
// (16 T^2 bytes) stream from L2.
#pragma once
#include "ptx.cuh"

namespace scb {

struct MlpGeom {
  int M;                 // tokens (rows of a)
  int m_tiles;
  __half* z;             // x1 in, z out: z[p * z_ld + col]
  long z_ld;
  const float* b0;       // [4T]
  const float* b2;       // [T]
};

template <int T>
struct MlpLayout {
  static constexpr int NCH = 4 * T / 128;                  // hidden chunks
  static constexpr int KB = T / 64;                        // 64-wide K blocks of a / of W0
  static constexpr int A_BYTES = KB * 128 * 128;           // [128 x T] fp16, K blocks of [128 x 128 B]
  static constexpr int STAGE = (T > 128 ? T : 128) * 128;  // one K block of W0 [128 x 64] or W2 [T x 64]
  static constexpr int STAGES = T == 128 ? 4 : 3;
  static constexpr int HS_BYTES = 2 * 128 * 128;           // one GELU chunk: 2 K blocks of [128 x 128 B]
  static constexpr int A_OFF = 0;
  static constexpr int RING = A_OFF + A_BYTES;
  static constexpr int HS = RING + STAGES * STAGE;          // two chunk buffers
  // T = 128: the tile's x1 rows [128 x 256 B], staged by coalesced copies at the tile's
  // start (at T = 256 there is no room: x1 is loaded straight into registers)
  static constexpr bool X1_STAGED = T == 128;
  static constexpr int X1S = HS + 2 * HS_BYTES;
  static constexpr int BAR = X1S + (X1_STAGED ? 128 * T * 2 : 0);
  static constexpr int SMEM = BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;                     // H: [0, 128) and [128, 256); acc: [256, 256 + T)
};

constexpr int MLP_EPI_WARPS = 16;
constexpr int MLP_THREADS = 64 + 32 * MLP_EPI_WARPS;  // producer, UMMA issuer, epilogue warps

template <int T>
__global__ void __launch_bounds__(MLP_THREADS, 1)
mlp_fused_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmW0,
                 const __grid_constant__ CUtensorMap tmW2, const MlpGeom g) {
  using L = MlpLayout<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::BAR);  // [STAGES]
  uint64_t* empty = full + L::STAGES;                         // [STAGES]
  uint64_t* a_full = empty + L::STAGES;
  uint64_t* a_empty = a_full + 1;
  uint64_t* h_full = a_empty + 1;     // [2] H_j in TMEM
  uint64_t* h_empty = h_full + 2;     // [2] H buffer read out by the epilogue
  uint64_t* hs_full = h_empty + 2;    // [2] Hs_j in smem
  uint64_t* hs_empty = hs_full + 2;   // [2] Hs buffer consumed by its UMMAs
  uint64_t* acc_full = hs_empty + 2;
  uint64_t* acc_empty = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 1);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < L::STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(a_full, 1);
    mbar_init(a_empty, 1);
    for (int b = 0; b < 2; ++b) {
      mbar_init(&h_full[b], 1);
      mbar_init(&h_empty[b], 32 * MLP_EPI_WARPS);
      mbar_init(&hs_full[b], 32 * MLP_EPI_WARPS);
      mbar_init(&hs_empty[b], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(acc_empty, 32 * MLP_EPI_WARPS);
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmW0);
    tma_prefetch_desc(&tmW2);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sb = smem_u32(sm);

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0, t = 0;
      bool ok = true;
      auto stage_in = [&](const CUtensorMap* m, int x, int y, int bytes) -> bool {
        const uint32_t s = it % L::STAGES, ph = (it / L::STAGES) & 1;
        ++it;
        if (!mbar_wait(&empty[s], ph ^ 1, SCB_ERR_WAIT_EMPTY)) return false;
        mbar_arrive_expect_tx(&full[s], bytes);
        tma_load_2d(sm + L::RING + s * L::STAGE, m, &full[s], x, y);
        return true;
      };
      for (int tile = blockIdx.x; tile < g.m_tiles && ok; tile += gridDim.x, ++t) {
        if (!mbar_wait(a_empty, (t & 1) ^ 1, SCB_ERR_WAIT_EMPTY)) break;
        mbar_arrive_expect_tx(a_full, L::A_BYTES);
        for (int kb = 0; kb < L::KB; ++kb) tma_load_2d(sm + L::A_OFF + kb * 16384, &tmA, a_full, kb * 64, tile * 128);
        // the UMMA warp's order: W0_0, W0_1, W2_0, W0_2, W2_1, ..., W0_{N-1}, W2_{N-2}, W2_{N-1}
        for (int j = 0; j <= L::NCH && ok; ++j) {
          if (j < L::NCH)
            for (int kb = 0; kb < L::KB && ok; ++kb) ok = stage_in(&tmW0, kb * 64, j * 128, 128 * 128);
          if (j >= 1)
            for (int kb = 0; kb < 2 && ok; ++kb) ok = stage_in(&tmW2, (j - 1) * 128 + kb * 64, 0, T * 128);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, t = 0, hc = 0;  // ring position, tiles, hidden chunks issued (over all tiles)
      bool ok = true;
      constexpr uint32_t id_h = make_idesc_f16(128, 128);
      constexpr uint32_t id_o = make_idesc_f16(128, T);
      auto next_stage = [&](uint32_t& s) -> bool {
        s = it % L::STAGES;
        const uint32_t ph = (it / L::STAGES) & 1;
        ++it;
        if (!mbar_wait(&full[s], ph, SCB_ERR_WAIT_FULL)) return false;
        tc_fence_after();
        return true;
      };
      for (int tile = blockIdx.x; tile < g.m_tiles && ok; tile += gridDim.x, ++t) {
        if (!mbar_wait(a_full, t & 1, SCB_ERR_WAIT_FULL)) break;
        tc_fence_after();
        for (int j = 0; j <= L::NCH && ok; ++j) {
          if (j < L::NCH) {  // H_j = a . W0_j^T into H buffer (hc + j) & 1
            const uint32_t c = hc + j, b = c & 1;
            if (!mbar_wait(&h_empty[b], ((c >> 1) & 1) ^ 1, SCB_ERR_WAIT_ACC_FREE)) { ok = false; break; }
            tc_fence_after();
            for (int kb = 0; kb < L::KB && ok; ++kb) {
              uint32_t s;
              if (!(ok = next_stage(s))) break;
              const uint32_t wa = sb + L::RING + s * L::STAGE, aa = sb + L::A_OFF + kb * 16384;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tmem + 128 * b, make_sdesc(aa + k * 32, 128, SW_128B), make_sdesc(wa + k * 32, 128, SW_128B),
                         id_h, (kb | k) != 0);
              umma_commit(&empty[s]);
            }
            umma_commit(&h_full[b]);
            if (j == L::NCH - 1) umma_commit(a_empty);  // the tile's a is no longer read
          }
          if (j >= 1) {  // acc += Hs_{j-1} . W2_{j-1}^T
            const uint32_t c = hc + j - 1, b = c & 1;
            if (j == 1 && !mbar_wait(acc_empty, (t & 1) ^ 1, SCB_ERR_WAIT_ACC_FREE)) { ok = false; break; }
            if (!mbar_wait(&hs_full[b], (c >> 1) & 1, SCB_ERR_WAIT_ACC)) { ok = false; break; }
            tc_fence_after();
            for (int kb = 0; kb < 2 && ok; ++kb) {
              uint32_t s;
              if (!(ok = next_stage(s))) break;
              const uint32_t wa = sb + L::RING + s * L::STAGE, ha = sb + L::HS + b * L::HS_BYTES + kb * 16384;
#pragma unroll
              for (int k = 0; k < 4; ++k)
                umma_f16(tmem + 256, make_sdesc(ha + k * 32, 128, SW_128B), make_sdesc(wa + k * 32, 128, SW_128B),
                         id_o, (j > 1 || kb > 0 || k > 0));
              umma_commit(&empty[s]);
            }
            umma_commit(&hs_empty[b]);
          }
        }
        hc += L::NCH;
        umma_commit(acc_full);
      }
    }
  } else {
    // ---------------- epilogue: warps 2.., thread = (token row, column share) ----------------
    const int q = warp & 3;            // TMEM lane quarter of this warp
    const int hf = (warp - 2) >> 2;    // which share of the columns
    constexpr int NSH = MLP_EPI_WARPS / 4, HC = 128 / NSH, ZC = T / NSH;  // shares; columns per share
    const int r = q * 32 + lane;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    uint32_t t = 0, hc = 0;
    bool ok = true;  // a timed-out wait (error recorded) ends the loops; the final barrier still runs
    for (int tile = blockIdx.x; tile < g.m_tiles && ok; tile += gridDim.x, ++t) {
      if (L::X1_STAGED) {
        // this warp's share of the tile's x1 (rows 32 q .. + 31, 16-byte chunks 4 hf .. + 3
        // of each 256-byte row) -> X1S, lane l copying chunk 4 hf + l % 4 of rows l / 4 + 8 k:
        // eight rows per copy instruction instead of 32 scattered ones; chunks XOR-swizzled
        // by row % 8
        const int ch = 4 * hf + (lane & 3);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const int rr = q * 32 + (lane >> 2) + 8 * k;
          const long pr = (long)tile * 128 + rr;
          const __half* src = pr < g.M ? g.z + pr * g.z_ld + 8 * ch : g.z;
          cp_async16(sm + L::X1S + rr * 256 + 16 * (ch ^ (rr & 7)), src, pr < g.M);
        }
        cp_async_commit();
      }
      for (int j = 0; j < L::NCH && ok; ++j) {
        const uint32_t c = hc + j, b = c & 1, ph = (c >> 1) & 1;
        // H_j in TMEM, and the Hs buffer's previous chunk consumed by its UMMAs
        ok = mbar_wait(&h_full[b], ph, SCB_ERR_WAIT_ACC) && mbar_wait(&hs_empty[b], ph ^ 1, SCB_ERR_WAIT_ACC_FREE);
        if (!ok) break;
        tc_fence_after();
        uint8_t* hs = sm + L::HS + b * L::HS_BYTES;
#pragma unroll 1
        for (int cc = HC * hf; cc < HC * hf + HC; cc += 32) {
          float v[32];
          tmem_ld16x2(trow + 128 * b + cc, v, trow + 128 * b + cc + 16, v + 16);
          const float4* b4 = reinterpret_cast<const float4*>(g.b0 + j * 128 + cc);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const float4 bb = __ldg(b4 + i);
            const float2 h0 = __fadd2_rn(make_float2(v[4 * i], v[4 * i + 1]), make_float2(bb.x, bb.y));
            const float2 h1 = __fadd2_rn(make_float2(v[4 * i + 2], v[4 * i + 3]), make_float2(bb.z, bb.w));
            __half2 a0 = gelu_tanh_h2(__floats2half2_rn(h0.x, h0.y));
            __half2 a1 = gelu_tanh_h2(__floats2half2_rn(h1.x, h1.y));
            pk[2 * i] = *reinterpret_cast<uint32_t*>(&a0);
            pk[2 * i + 1] = *reinterpret_cast<uint32_t*>(&a1);
          }
          // columns cc .. cc + 31 = 16-byte chunks (cc % 64) / 8 .. + 3 of K block cc / 64
          uint8_t* blk = hs + (cc >> 6) * 16384;
#pragma unroll
          for (int i = 0; i < 4; ++i)
            *reinterpret_cast<uint4*>(blk + swz_off(r, ((cc & 63) >> 3) + i, 128)) =
                make_uint4(pk[4 * i], pk[4 * i + 1], pk[4 * i + 2], pk[4 * i + 3]);
        }
        tc_fence_before();
        mbar_arrive(&h_empty[b]);    // the H TMEM buffer may be overwritten
        fence_proxy_async_smem();
        mbar_arrive(&hs_full[b]);    // Hs_j is the next UMMA's operand
      }
      hc += L::NCH;
      // ---- z = acc + b2 + x1, in place ----
      // this thread's x1 columns are loaded before the wait for the accumulator, so
      // their latency overlaps the last chunk's UMMAs
      if (!ok) break;
      const long p = (long)tile * 128 + r;
      uint4 xv[ZC / 8];
      if (L::X1_STAGED) {
        cp_async_wait_all();
        __syncwarp();  // the warp's lanes copied this row's chunks
#pragma unroll
        for (int i = 0; i < ZC / 8; ++i)
          xv[i] = *reinterpret_cast<const uint4*>(sm + L::X1S + r * 256 + 16 * ((4 * hf + i) ^ (r & 7)));
        __syncwarp();  // read before the next tile's rows are staged
      } else if (p < g.M) {
        const uint4* zp = reinterpret_cast<const uint4*>(g.z + p * g.z_ld + hf * ZC);
#pragma unroll
        for (int i = 0; i < ZC / 8; ++i) xv[i] = zp[i];
      }
      if (!(ok = mbar_wait(acc_full, t & 1, SCB_ERR_WAIT_ACC))) break;
      tc_fence_after();
#pragma unroll
      for (int cc = hf * ZC; cc < (hf + 1) * ZC; cc += 32) {
        float v[32];
        tmem_ld16x2(trow + 256 + cc, v, trow + 256 + cc + 16, v + 16);
        if (p < g.M) {
          uint4* zp = reinterpret_cast<uint4*>(g.z + p * g.z_ld + cc);
          const float4* b4 = reinterpret_cast<const float4*>(g.b2 + cc);
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            const uint4 u = xv[(cc - hf * ZC) / 8 + i];
            const __half2* hp = reinterpret_cast<const __half2*>(&u);
            const float4 ba = __ldg(b4 + 2 * i), bb = __ldg(b4 + 2 * i + 1);
            const float bs[8] = {ba.x, ba.y, ba.z, ba.w, bb.x, bb.y, bb.z, bb.w};
            float o[8];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float2 t = __fadd2_rn(make_float2(v[8 * i + 2 * e], v[8 * i + 2 * e + 1]),
                                          make_float2(bs[2 * e], bs[2 * e + 1]));
              const float2 r = __fadd2_rn(t, __half22float2(hp[e]));
              o[2 * e] = r.x;
              o[2 * e + 1] = r.y;
            }
            zp[i] = make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]),
                               pack_half2(o[6], o[7]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(acc_empty);
    }
  }
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem, L::TMEM_COLS);
}

}  // namespace scb
