// A block boundary inside a stage as one kernel: block i's conv1_2 and block i+1's
// conv1_1 (tools/network_scunet.py:167-176; src/cuda.rs:1077, 1140):
//
//   x'  = x + Z.W12^T + b12           (conv1_2 of block i, the residual stream update)
//   Y   = x'.W11^T + b11              (conv1_1 of block i+1, split into its conv half
//                                      Y_c and its trans half Y_t)
//
// per 128-pixel tile of the C-channel NHWC plane. x' leaves the SM twice from one
// on-chip copy: as the tile's store to the residual plane xs (the next conv1_2's
// residual and the down conv's input) and as the A operand of the second UMMA chain,
// so conv1_1 does not read xs back from HBM.
//
// Warp roles (192 threads): warp 0 TMA producer (per tile C/64 k-blocks of Z, then
// C/64 k-blocks of x, one [128 x 64] fp16 box each); warp 1 TMEM allocator and UMMA
// issuer; warps 2-5 the two epilogues (thread = pixel row of the tile). The
// residual x enters the first accumulator as extra UMMA k blocks against a 64 x 64
// identity (exact: fp16 x 1 summed in fp32). The issuer runs G1(t+1) before G2(t)
// and the epilogue E1(t+1) (x' of the next tile) before E2(t) (Y of this tile), so
// the second chain of a tile overlaps the first epilogue of the next; two TMEM
// accumulator pairs (4 C columns) let the tiles overlap.
//
// Numerics are those of the separate launches: x' is stored in fp16 and conv1_1 reads
// exactly those fp16 values; both biases are added in fp32 before rounding.
#pragma once
#include "gemm.cuh"

namespace scb {

struct PairGeom {
  int M;        // pixels (rows of the flat GEMMs)
  int tiles;    // ceil(M / 128)
  int stages;   // TMA ring depth (runtime)
  const float* b12;  // [C]
  const float* b11;  // [C]
};

template <int C>
struct PairSmem {
  static constexpr int KB = C / 64;                 // k blocks of 64 channels
  static constexpr int WBLK = C * 128;              // one k block of a weight: [C rows x 128 B]
  static constexpr int W12 = 0;                     // KB blocks, SW128
  static constexpr int W11 = W12 + KB * WBLK;
  static constexpr int IDENT = W11 + KB * WBLK;     // [64 x 128 B] SW128 identity
  static constexpr int XP = IDENT + 64 * 128;       // 2 buffers of KB x [128 x 128 B]: x' as an A operand
  static constexpr int XP_BYTES = KB * 16384;
  static constexpr int YS = XP + 2 * XP_BYTES;      // C / 32 slabs of [128 x 64 B] SW64: the Y staging
  static constexpr int STAGE0 = YS + (C / 32) * 8192;
  static constexpr int STAGE_BYTES = 16384;         // [128 x 128 B] SW128
  __host__ __device__ static constexpr int bar_off(int stages) { return STAGE0 + stages * STAGE_BYTES; }
  __host__ __device__ static constexpr int smem(int stages) { return bar_off(stages) + 256 + 1024; }
  static constexpr int TMEM_COLS = 4 * C;           // two (acc1, acc2) pairs of C columns
};

template <int C>
__global__ void __launch_bounds__(192, 1)
conv_pair_kernel(const __grid_constant__ CUtensorMap mZ, const __grid_constant__ CUtensorMap mX,
                 const __grid_constant__ CUtensorMap mYc, const __grid_constant__ CUtensorMap mYt,
                 const __half* __restrict__ w12, const __half* __restrict__ w11, const PairGeom g) {
  using L = PairSmem<C>;
  constexpr int KB = L::KB;
  constexpr uint32_t ID_C = make_idesc_f16(128, C), ID_64 = make_idesc_f16(128, 64);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const int S = g.stages;
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + L::bar_off(S));
  uint64_t* empty = full + S;
  uint64_t* acc1_full = empty + S;       // [2]
  uint64_t* acc1_empty = acc1_full + 2;  // [2], 128 arrivals
  uint64_t* xp_full = acc1_empty + 2;    // [2]
  uint64_t* acc2_full = xp_full + 2;     // [2]
  uint64_t* acc2_empty = acc2_full + 2;  // [2], 128 arrivals
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc2_empty + 2);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // resident weights ([C][C] fp16, row = output channel, K contiguous) as KB
  // K-major SW128 blocks, and the identity of the residual k blocks
  for (int idx = threadIdx.x; idx < C * (C / 8); idx += blockDim.x) {
    const int r = idx / (C / 8), j = idx % (C / 8);
    const int blk = j >> 3, ch = j & 7;
    *reinterpret_cast<uint4*>(sm + L::W12 + blk * L::WBLK + swz_off(r, ch, 128)) =
        __ldg(reinterpret_cast<const uint4*>(w12 + (long)r * C + j * 8));
    *reinterpret_cast<uint4*>(sm + L::W11 + blk * L::WBLK + swz_off(r, ch, 128)) =
        __ldg(reinterpret_cast<const uint4*>(w11 + (long)r * C + j * 8));
  }
  for (int idx = threadIdx.x; idx < 64 * 8; idx += blockDim.x) {
    const int n = idx >> 3, ch = idx & 7;
    uint32_t w[4] = {0u, 0u, 0u, 0u};
    const int k = n - ch * 8;  // position of the one inside this 8-element chunk, if any
    if (k >= 0 && k < 8) w[k >> 1] = (k & 1) ? 0x3C000000u : 0x00003C00u;
    *reinterpret_cast<uint4*>(sm + L::IDENT + swz_off(n, ch, 128)) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < S; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc1_full[b], 1);
      mbar_init(&acc1_empty[b], 128);
      mbar_init(&xp_full[b], 1);
      mbar_init(&acc2_full[b], 1);
      mbar_init(&acc2_empty[b], 128);
    }
    mbar_fence_init();
    tma_prefetch_desc(&mZ);
    tma_prefetch_desc(&mX);
    tma_prefetch_desc(&mYc);
    tma_prefetch_desc(&mYt);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sb = smem_u32(sm);
  const int n_local = (int)blockIdx.x < g.tiles ? (g.tiles - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
  auto tile_of = [&](int t) { return (int)blockIdx.x + t * (int)gridDim.x; };

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int t = 0; t < n_local && ok; ++t) {
        const int row0 = tile_of(t) * 128;
        for (int j = 0; j < 2 * KB; ++j, ++it) {
          const uint32_t s = it % S, ph = (it / S) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, SCB_ERR_WAIT_EMPTY)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&full[s], L::STAGE_BYTES);
          tma_load_2d(sm + L::STAGE0 + s * L::STAGE_BYTES, j < KB ? &mZ : &mX, &full[s], (j % KB) * 64, row0);
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer: G1(0), then G1(t + 1) before G2(t) ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      auto g1 = [&](int t) {
        const int b = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&acc1_empty[b], ph ^ 1, SCB_ERR_WAIT_ACC_FREE)) return false;
        tc_fence_after();
        const uint32_t d = tmem + b * 2 * C;
        for (int j = 0; j < 2 * KB; ++j, ++it) {
          const uint32_t s = it % S, sph = (it / S) & 1;
          if (!mbar_wait(&full[s], sph, SCB_ERR_WAIT_FULL)) return false;
          tc_fence_after();
          const uint32_t sa = sb + L::STAGE0 + s * L::STAGE_BYTES;
          if (j < KB) {  // Z k block j against W12's k block j
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(d, make_sdesc(sa + 32 * k, 128, SW_128B),
                       make_sdesc(sb + L::W12 + j * L::WBLK + 32 * k, 128, SW_128B), ID_C, (j | k) != 0);
          } else {  // the residual's channels [64 jj, + 64) into accumulator columns [64 jj, + 64)
            const int jj = j - KB;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              umma_f16(d + 64 * jj, make_sdesc(sa + 32 * k, 128, SW_128B),
                       make_sdesc(sb + L::IDENT + 32 * k, 128, SW_128B), ID_64, 1);
          }
          umma_commit(&empty[s]);
        }
        umma_commit(&acc1_full[b]);
        return true;
      };
      auto g2 = [&](int t) {
        const int b = t & 1;
        const uint32_t ph = (t >> 1) & 1;
        if (!mbar_wait(&xp_full[b], ph, SCB_ERR_WAIT_ACC) || !mbar_wait(&acc2_empty[b], ph ^ 1, SCB_ERR_WAIT_ACC_FREE))
          return false;
        tc_fence_after();
        const uint32_t d = tmem + b * 2 * C + C;
        const uint32_t xa = sb + L::XP + b * L::XP_BYTES;
        for (int j = 0; j < KB; ++j)
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(d, make_sdesc(xa + j * 16384 + 32 * k, 128, SW_128B),
                     make_sdesc(sb + L::W11 + j * L::WBLK + 32 * k, 128, SW_128B), ID_C, (j | k) != 0);
        umma_commit(&acc2_full[b]);
        return true;
      };
      if (n_local > 0) ok = g1(0);
      for (int t = 0; t < n_local && ok; ++t) {
        if (t + 1 < n_local && !g1(t + 1)) break;
        ok = g2(t);
      }
    }
  } else {
    // ---------------- epilogues: warps 2..5, thread = pixel row ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const bool elected = warp == 2 && lane == 0;
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16);
    // E1(t): x' = acc1 + b12 -> fp16 into XP[b] (the A operand of G2(t)) -> TMA store to xs
    auto e1 = [&](int t) {
      const int b = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      if (!mbar_wait(&acc1_full[b], ph, SCB_ERR_WAIT_ACC)) return false;
      tc_fence_after();
      // XP[b] was last stored by E1(t - 2); at most two groups have been committed
      // since (x'(t - 1), Y(t - 2)), so waiting down to two pending ones covers it
      if (elected) bulk_wait_group_read<2>();
      epi_bar();
      uint8_t* xp = sm + L::XP + b * L::XP_BYTES;
#pragma unroll 1
      for (int c = 0; c < C; c += 32) {
        float v[32];
        tmem_ld16x2(trow + b * 2 * C + c, v, trow + b * 2 * C + c + 16, v + 16);
        const float4* b4 = reinterpret_cast<const float4*>(g.b12 + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 bb = __ldg(b4 + j);
          add4_f32x2(v + 4 * j, bb);
        }
        uint8_t* blk = xp + (c >> 6) * 16384;
#pragma unroll
        for (int h = 0; h < 4; ++h)
          *reinterpret_cast<uint4*>(blk + swz_off(r, ((c & 63) >> 3) + h, 128)) =
              make_uint4(pack_half2(v[8 * h], v[8 * h + 1]), pack_half2(v[8 * h + 2], v[8 * h + 3]),
                         pack_half2(v[8 * h + 4], v[8 * h + 5]), pack_half2(v[8 * h + 6], v[8 * h + 7]));
      }
      tc_fence_before();
      mbar_arrive(&acc1_empty[b]);
      fence_proxy_async_smem();
      epi_bar();
      if (elected) {
        mbar_arrive(&xp_full[b]);
        for (int j = 0; j < KB; ++j) tma_store_2d(&mX, xp + j * 16384, 64 * j, tile_of(t) * 128);
        bulk_commit_group();
      }
      return true;
    };
    // E2(t): Y = acc2 + b11 -> fp16 -> the conv half to Y_c, the trans half to Y_t
    auto e2 = [&](int t) {
      const int b = t & 1;
      const uint32_t ph = (t >> 1) & 1;
      if (!mbar_wait(&acc2_full[b], ph, SCB_ERR_WAIT_ACC)) return false;
      tc_fence_after();
      // the Y staging was last stored by E2(t - 1); only x'(t + 1), when there is one,
      // has been committed since
      if (elected) {
        if (t + 1 < n_local)
          bulk_wait_group_read<1>();
        else
          bulk_wait_group_read<0>();
      }
      epi_bar();
#pragma unroll 1
      for (int c = 0; c < C; c += 32) {
        float v[32];
        tmem_ld16x2(trow + b * 2 * C + C + c, v, trow + b * 2 * C + C + c + 16, v + 16);
        const float4* b4 = reinterpret_cast<const float4*>(g.b11 + c);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float4 bb = __ldg(b4 + j);
          add4_f32x2(v + 4 * j, bb);
        }
        uint8_t* slab = sm + L::YS + (c >> 5) * 8192;
#pragma unroll
        for (int h = 0; h < 4; ++h)
          *reinterpret_cast<uint4*>(slab + swz_off(r, h, 64)) =
              make_uint4(pack_half2(v[8 * h], v[8 * h + 1]), pack_half2(v[8 * h + 2], v[8 * h + 3]),
                         pack_half2(v[8 * h + 4], v[8 * h + 5]), pack_half2(v[8 * h + 6], v[8 * h + 7]));
      }
      tc_fence_before();
      mbar_arrive(&acc2_empty[b]);
      fence_proxy_async_smem();
      epi_bar();
      if (elected) {
        const int row0 = tile_of(t) * 128;
        for (int c = 0; c < C; c += 32) {
          if (c < C / 2)
            tma_store_2d(&mYc, sm + L::YS + (c >> 5) * 8192, c, row0);
          else
            tma_store_2d(&mYt, sm + L::YS + (c >> 5) * 8192, c - C / 2, row0);
        }
        bulk_commit_group();
      }
      return true;
    };
    bool ok = n_local == 0 || e1(0);
    for (int t = 0; t < n_local && ok; ++t) {
      if (t + 1 < n_local && !e1(t + 1)) break;
      ok = e2(t);
    }
    if (elected) bulk_wait_group<0>();
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

}  // namespace scb
