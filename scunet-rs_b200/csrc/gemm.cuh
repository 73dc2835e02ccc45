// The tensor-core workhorse: D[M x N] = A[M x K] * B[N x K]^T on tcgen05 with the
// accumulator in TMEM, A and B fp16 K-major tiles landed by TMA (128B/64B
// swizzle), fp32 accumulate, and a fused epilogue (bias, ReLU/GELU, fp16/fp32
// residual, fp32 skip add, LayerNorm of a column range, fp16/fp32 stores).
//
// One kernel covers every channel-mixing op of the network; only how A's tiles
// are addressed (GEO_*) and where the epilogue stores a row differ:
//
//   GEO_FLAT  1x1 convs and linears: row m = pixel m of an NHWC plane.
//   GEO_CONV3 3x3 / stride 1 / zero pad 1 conv as an implicit GEMM: an M tile is a
//             TH x TW block of output pixels of one image; the K loop walks the 9
//             taps (ky, kx) x channel chunks, each tap a TMA box of the NHWC input
//             at offset (y+ky-1, x+kx-1). Out-of-range boxes are zero-filled by the
//             TMA unit, which IS the zero padding.
//   GEO_DOWN2 2x2 / stride 2 conv: the input viewed as 5-D (C, dx, W/2, dy, rows/2);
//             tap (dy, dx) of a TH x TW output block is one TMA box.
//   GEO_UP2   2x2 / stride 2 transposed conv: a plain GEMM over input pixels with
//             N ordered (dy, dx, c_out); each N tile lies in one output quadrant
//             (dy, dx) and goes to output pixels (2y+dy, 2x+dx) (pixel shuffle).
//             With the TMA epilogue the M tiles are TW x TH input pixels (A: a
//             3-D box) and an output slab is one box of a 5-D view of the output
//             (channel, dx, x, dy, row); the direct epilogue takes 128
//             consecutive input pixels and scatters per thread.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM allocator and
// UMMA issuer (one elected lane), warps 2..5 = epilogue (thread = accumulator row).
// The grid is persistent; tiles are strided over CTAs and the two TMEM
// accumulator buffers let tile i's epilogue overlap tile i+1's main loop. The
// pipeline depth (stages) is a runtime value so the host can trade stages for
// epilogue staging space.
//
// Two epilogues:
//   TMAEPI = true : asynchronous. The epilogue works in 32-column slabs. An fp16
//                   residual without an activation enters the accumulator as
//                   extra UMMA k blocks (GemmGeom::res_kb); other residual slabs
//                   (fp32/skip) are TMA-loaded into swizzled smem one slab ahead
//                   (the first before the accumulator wait); outputs are written to
//                   swizzled smem staging and leave through TMA bulk tensor stores,
//                   double-buffered. Every global byte moves in full lines through
//                   the TMA unit. PAIRS = true (flat GEMMs without residual slabs):
//                   two slabs per round, one in each staging buffer, so a tile pays
//                   half the rounds of barriers, proxy fences and store issues that
//                   bound these epilogues (measured: the level-2 qkv linear 154 ->
//                   118 us per 4-frame launch).
//   TMAEPI = false: per-thread vector loads/stores, for the variants without a TMA
//                   one (and the LayerNorm of non-flat GEMMs).
#pragma once
#include <cuda.h>
#include "ptx.cuh"

namespace scb {

enum Geo : int { GEO_FLAT = 0, GEO_CONV3 = 1, GEO_DOWN2 = 2, GEO_UP2 = 3, GEO_CONV3X = 4, GEO_CONV3W = 5 };

// GEO_CONV3X: the 3x3 conv with 8-row x 16-column output tiles and one TMA box per
// column shift kx: the box covers the tile's 10 input rows (halo included), and the
// three row taps ky are 16-row views into it (UMMA descriptors at +16*ky rows). A
// tile reads 3 x 160 instead of 9 x 128 input pixel-rows.
//
// GEO_CONV3W: the 3x3 conv with 16-row x 8-column output tiles and ONE TMA box per
// channel chunk: the box covers the tile's 18 x 10 input pixels (halo rows and
// columns), and each of the nine taps (ky, kx) is a view into it: output row m =
// (r, c) of the tile reads box pixel (r + ky, c + kx), i.e. the operand's 8-row
// groups (one tile row each) start at box row 10 (r + ky) + kx and lie 10 box rows
// apart. The box is 20 rows high (two unused) so that it holds a whole number of
// 8-row swizzle atoms. A tile reads 200 input pixel-rows instead of 480 (CONV3X)
// or 1152 (CONV3).
__host__ __device__ constexpr bool is_conv3(int geo) {
  return geo == GEO_CONV3 || geo == GEO_CONV3X || geo == GEO_CONV3W;
}
constexpr int kConv3wTW = 8, kConv3wTH = 16, kConv3wBoxRows = kConv3wTH + 4;
enum Act : int { ACT_NONE = 0, ACT_RELU = 1, ACT_GELU = 2 };

struct GemmGeom {
  int M;            // rows of A (FLAT/UP2: pixels; CONV3/DOWN2: output pixels, for bounds)
  int n_total;      // N
  int num_kb;       // K / BK
  int kb_per_tap;   // CONV3/DOWN2: channel chunks per tap
  int m_tiles, n_tiles;
  // CONV3: per-image stored plane H x W, output rows [row0, row0 + rows_out) of it
  // (the whole plane, or a row band between halo rows); DOWN2: stacked output rows
  // H (= n*Ho) x W (= Wo)
  int H, W, TH, TW, tiles_x, tiles_y;
  int row0, rows_out;
  // UP2: input width and c_out
  int up_w, up_cout;
  int stages;       // pipeline depth (runtime)
  // 1: all of B (every k block of the op's single N tile) is loaded into shared
  // memory once per CTA and stays there; the pipeline stages then carry A only
  int b_res;
  // flat GEMMs and 3x3 convs with an fp16 residual (TMA epilogue, no activation):
  // > 0 = the residual enters the accumulator on the tensor cores as res_kb =
  // BN / BK more k blocks per tile: k block j is A = the tile's residual columns
  // [n0 + j BK, + BK) (EpiMaps::resA), added into accumulator columns
  // [j BK, + BK) by UMMAs of N = 32 against slices of a 32 x 32 identity B (built
  // in shared memory). Exact: fp16 x 1 summed in fp32.
  int res_kb;
  // GEO_CONV3X, 128-wide, one N tile: 1 = two M tiles per pipeline stage (the CTA's
  // tiles i and i + grid, one A box each) share the stage's B, halving the weight
  // bytes each tile pulls through shared memory, the bound of these convs
  int twin;
};

struct GemmEpi {
  const float* bias;    // [N] or null
  int act;              // Act
  const __half* res16;  // residual, fp16, element (pixel, col) at res16[p*res16_ld + col]
  long res16_ld;
  const float* res32;   // residual, fp32
  long res32_ld;
  const float* skip32;  // if set, the fp16 store holds (v + skip) and the fp32 store v
  long skip_ld;
  __half* out16;
  long out16_ld;
  // if set, GEMM columns [out16_split, N) go to out16b[p*out16b_ld + (col - out16_split)]
  // instead (two planes, e.g. the conv and the trans half of conv1_1's output)
  __half* out16b;
  long out16b_ld;
  int out16_split;
  float* out32;
  long out32_ld;
  // LayerNorm over global columns [ln_lo, ln_lo + ln_n) of the final value v,
  // written as fp16 to ln_out[p*ln_ld + (col - ln_lo)].
  const float* ln_g;
  const float* ln_b;
  __half* ln_out;
  long ln_ld;
  int ln_lo, ln_n;
  // TMA epilogue: staging offsets (bytes within one buffer) of each stream's
  // [128 x 32-column] slab; -1 = stream absent. st_ln: the LayerNorm output slab
  // (GEO_FLAT, no activation, fp16 residual at most).
  int st_res16, st_res32, st_skip, st_out16, st_out32, st_ln;
  int st_res_bytes, st_out_bytes;  // bytes of one buffer of all residual / output slabs
  int st_ident_bytes;              // the residual k blocks' 32 x 32 identity B (fp16), first in staging
  int res_bufs;                    // residual buffers (2..4): slabs are requested res_bufs - 1 ahead
};

// Tensor maps of the epilogue streams (TMA epilogue only); box = 32 columns x the
// M tile's pixel block.
struct EpiMaps {
  CUtensorMap res16, res32, skip, out16, out32, lnout, out16b;
  CUtensorMap resA;  // the residual as an A operand: box = BK channels x the tile's pixels
};


// One 16-column chunk of a row's residual inputs, loaded ahead of use.
struct ResChunk {
  uint4 r16[2];
  float4 r32[4];
  float4 sk[4];
};

__device__ __forceinline__ void load_res(const GemmEpi& e, long p, int oc, ResChunk& rc) {
  if (e.res16) {
    const uint4* src = reinterpret_cast<const uint4*>(e.res16 + p * e.res16_ld + oc);
    rc.r16[0] = __ldg(src);
    rc.r16[1] = __ldg(src + 1);
  }
  if (e.res32) {
    const float4* src = reinterpret_cast<const float4*>(e.res32 + p * e.res32_ld + oc);
#pragma unroll
    for (int h = 0; h < 4; ++h) rc.r32[h] = __ldg(src + h);
  }
  if (e.skip32) {
    const float4* src = reinterpret_cast<const float4*>(e.skip32 + p * e.skip_ld + oc);
#pragma unroll
    for (int h = 0; h < 4; ++h) rc.sk[h] = __ldg(src + h);
  }
}

// smem: [stages x (A tile | B tile)] [barriers, tmem slot: 1 KB] [TMA-epilogue staging]
template <int BN, int BK, int GEO = GEO_FLAT>
struct GemmSmem {
  // CONV3X: 10 input rows x 16 columns; CONV3W: 20 x 10
  static constexpr int A_ROWS = GEO == GEO_CONV3X ? 160 : GEO == GEO_CONV3W ? kConv3wBoxRows * (kConv3wTW + 2) : 128;
  // CONV3X: the three ky taps of one kx; CONV3W: all nine taps
  static constexpr int B_TAPS = GEO == GEO_CONV3X ? 3 : GEO == GEO_CONV3W ? 9 : 1;
  static constexpr int A_TX = A_ROWS * BK * 2;                    // bytes one A box delivers
  static constexpr int A_BYTES = (A_TX + 1023) / 1024 * 1024;      // its slot: stages stay 1024-aligned
  static constexpr int B_BYTES = B_TAPS * BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  // layout: stages (A, or A + B, or A0 + A1 + B for twin tiles) | resident B (num_kb x
  // B_BYTES, when b_res) | barriers | staging
  __host__ __device__ static constexpr int stage_bytes(bool b_res, bool twin = false) {
    return b_res ? A_BYTES : twin ? 2 * A_BYTES + B_BYTES : STAGE_BYTES;
  }
  // TMEM accumulator buffers: four for narrow tiles (so the loads and MMAs of the next
  // tiles run ahead while the epilogue drains one) and for the 128-wide 3x3 convs (two
  // twin tiles in flight), two otherwise
  static constexpr int NACC = (BN <= 64 || (GEO == GEO_CONV3X && BN == 128)) ? 4 : 2;
  static constexpr int TMEM_COLS = (NACC * BN <= 32) ? 32 : (NACC * BN <= 64) ? 64 : (NACC * BN <= 128) ? 128
                                   : (NACC * BN <= 256) ? 256 : 512;
  __host__ __device__ static constexpr int bres_off(int stages, bool b_res, bool twin = false) {
    return stages * stage_bytes(b_res, twin);
  }
  __host__ __device__ static constexpr int bar_off(int stages, bool b_res, int num_kb, bool twin = false) {
    return bres_off(stages, b_res, twin) + (b_res ? num_kb * B_BYTES : 0);
  }
  __host__ __device__ static constexpr int staging_off(int stages, bool b_res, int num_kb, bool twin = false) {
    return bar_off(stages, b_res, num_kb, twin) + 1024;
  }
};

// Where accumulator row `r` of M tile `mt` lives: returns the output pixel index
// (or -1 when the row is outside the plane) for a given N-tile base `n0`, and the
// output column of the tile's first column.
template <int GEO>
__device__ __forceinline__ long row_pixel(const GemmGeom& g, int mt, int r, int n0, int& col0) {
  col0 = n0;
  if (GEO == GEO_FLAT) {
    const long p = (long)mt * 128 + r;
    return p < g.M ? p : -1;
  } else if (is_conv3(GEO)) {
    const int per_img = g.tiles_y * g.tiles_x;
    const int img = mt / per_img;
    const int rem = mt - img * per_img;
    const int ty = rem / g.tiles_x, tx = rem - ty * g.tiles_x;
    const int y = g.row0 + ty * g.TH + r / g.TW, x = tx * g.TW + r % g.TW;
    if (x >= g.W || y >= g.row0 + g.rows_out) return -1;
    return ((long)img * g.H + y) * g.W + x;
  } else if (GEO == GEO_DOWN2) {
    const int ty = mt / g.tiles_x, tx = mt - ty * g.tiles_x;
    const int y = ty * g.TH + r / g.TW, x = tx * g.TW + r % g.TW;
    if (x >= g.W || y >= g.H) return -1;
    return (long)y * g.W + x;
  } else {  // GEO_UP2: flat tiles of 128 input pixels, or TW x TH tiles when g.TW > 0
    long R;
    int x;
    if (g.TW > 0) {
      const int ty = mt / g.tiles_x;
      R = (long)ty * g.TH + r / g.TW;
      x = (mt - ty * g.tiles_x) * g.TW + r % g.TW;
      if (x >= g.up_w || R >= g.H) return -1;
    } else {
      const long p = (long)mt * 128 + r;
      if (p >= g.M) return -1;
      R = p / g.up_w;
      x = (int)(p - R * g.up_w);
    }
    const int d = n0 / g.up_cout;
    col0 = n0 - d * g.up_cout;
    return (2 * R + (d >> 1)) * (2L * g.up_w) + 2 * x + (d & 1);
  }
}

// Spatial origin of M tile `mt`: (img, y0, x0) for CONV3, (y0, x0) for DOWN2.
template <int GEO>
__device__ __forceinline__ void tile_origin(const GemmGeom& g, int mt, int& img, int& y0, int& x0) {
  img = 0;
  y0 = 0;
  x0 = 0;
  if (is_conv3(GEO)) {
    const int per_img = g.tiles_y * g.tiles_x;
    img = mt / per_img;
    const int rem = mt - img * per_img;
    const int ty = rem / g.tiles_x;
    y0 = g.row0 + ty * g.TH;
    x0 = (rem - ty * g.tiles_x) * g.TW;
  } else if (GEO == GEO_DOWN2 || (GEO == GEO_UP2 && g.TW > 0)) {
    const int ty = mt / g.tiles_x;
    y0 = ty * g.TH;
    x0 = (mt - ty * g.tiles_x) * g.TW;
  }
}

// TMA load / store of one epilogue slab at column `col` of the tile's pixel block.
template <int GEO>
__device__ __forceinline__ void epi_slab_load(void* dst, const CUtensorMap* m, uint64_t* bar, int col, int mt,
                                              const GemmGeom& g) {
  int img, y0, x0;
  tile_origin<GEO>(g, mt, img, y0, x0);
  if (is_conv3(GEO)) {
    tma_load_4d(dst, m, bar, col, x0, y0, img);
  } else if (GEO == GEO_DOWN2) {
    tma_load_3d(dst, m, bar, col, x0, y0);
  } else if (GEO == GEO_UP2) {  // the output quadrant (dy, dx) of GEMM column col
    const int d = col / g.up_cout;
    tma_load_5d(dst, m, bar, col - d * g.up_cout, d & 1, x0, d >> 1, y0);
  } else {
    tma_load_2d(dst, m, bar, col, mt * 128);
  }
}

template <int GEO>
__device__ __forceinline__ void epi_slab_store(const CUtensorMap* m, const void* src, int col, int mt,
                                               const GemmGeom& g) {
  int img, y0, x0;
  tile_origin<GEO>(g, mt, img, y0, x0);
  if (is_conv3(GEO)) {
    tma_store_4d(m, src, col, x0, y0, img);
  } else if (GEO == GEO_DOWN2) {
    tma_store_3d(m, src, col, x0, y0);
  } else if (GEO == GEO_UP2) {  // the output quadrant (dy, dx) of GEMM column col
    const int d = col / g.up_cout;
    tma_store_5d(m, src, col - d * g.up_cout, d & 1, x0, d >> 1, y0);
  } else {
    tma_store_2d(m, src, col, mt * 128);
  }
}

// Named barrier over the four epilogue warps only.
__device__ __forceinline__ void epi_bar() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

template <int BN, int BK, int GEO, bool TMAEPI, bool PAIRS = false>
__global__ void __launch_bounds__(192, 2)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, const GemmGeom g,
               const GemmEpi e, const __grid_constant__ EpiMaps em) {
  using L = GemmSmem<BN, BK, GEO>;
  static_assert(BN % 16 == 0 && BN >= 16 && BN <= 256, "UMMA N for M=128");
  static_assert(BK == 64 || BK == 32, "BK is one 128B or 64B swizzle row of fp16");
  static_assert(!TMAEPI || BN % 32 == 0, "TMA epilogue works in 32-column slabs");
  static_assert(!PAIRS || (TMAEPI && BN % 64 == 0), "paired slabs: TMA epilogue, 64-column rounds");
  constexpr uint32_t ROWB = BK * 2;
  constexpr uint32_t SWZ = (BK == 64) ? SW_128B : SW_64B;
  constexpr uint32_t IDESC = make_idesc_f16(128, BN);
  const int STAGES = g.stages;
  const bool b_res = g.b_res != 0;
  // (compiled for the 128-wide conv only: at 64 channels two tiles per stage measured 15 %
  // slower - one CTA per SM instead of two)
  const bool twin = GEO == GEO_CONV3X && BN == 128 && g.twin != 0 && !b_res && g.n_tiles == 1;
  const int SBYTES = L::stage_bytes(b_res, twin);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* bres = smem + L::bres_off(STAGES, b_res, twin);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::bar_off(STAGES, b_res, g.num_kb, twin));
  uint64_t* empty = full + STAGES;
  uint64_t* acc_full = empty + STAGES;
  uint64_t* acc_empty = acc_full + L::NACC;
  uint64_t* res_full = acc_empty + L::NACC;
  uint64_t* bres_full = res_full + 4;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bres_full + 1);
  uint8_t* staging = smem + L::staging_off(STAGES, b_res, g.num_kb, twin);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int total_tiles = g.m_tiles * g.n_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int a = 0; a < L::NACC; ++a) {
      mbar_init(&acc_full[a], 1);
      mbar_init(&acc_empty[a], 128);
    }
    for (int b = 0; b < 4; ++b) mbar_init(&res_full[b], 1);
    mbar_init(bres_full, 1);
    mbar_fence_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  constexpr bool RES_MMA = TMAEPI && (GEO == GEO_FLAT || is_conv3(GEO));
  if (RES_MMA && g.res_kb > 0) {
    // the 32 x 32 identity B of the residual k blocks: K-major 64-byte rows,
    // 64B-swizzled like a TMA-loaded tile
    for (int idx = threadIdx.x; idx < 32 * 4; idx += blockDim.x) {
      const int n = idx >> 2, c = idx & 3;
      uint32_t w[4] = {0u, 0u, 0u, 0u};
      const int k = n - c * 8;  // position of the one inside this chunk, if any
      if (k >= 0 && k < 8) w[k >> 1] = (k & 1) ? 0x3C000000u : 0x00003C00u;
      *reinterpret_cast<uint4*>(staging + swz_off(n, c, 64)) = make_uint4(w[0], w[1], w[2], w[3]);
    }
    fence_proxy_async_smem();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      // B's B_TAPS boxes of k block kb (N tile n0) -> dst
      auto load_b = [&](uint8_t* dst, uint64_t* bar, int kb, int n0) {
        if (GEO == GEO_CONV3X) {
          const int kx = kb % 3, ch = kb / 3;
          const int cin = g.kb_per_tap * BK;
#pragma unroll
          for (int ky = 0; ky < 3; ++ky)
            tma_load_2d(dst + ky * (BN * BK * 2), &tmB, bar, (ky * 3 + kx) * cin + ch * BK, n0);
        } else if (GEO == GEO_CONV3W) {
          const int cin = g.kb_per_tap * BK;
#pragma unroll
          for (int tap = 0; tap < 9; ++tap) tma_load_2d(dst + tap * (BN * BK * 2), &tmB, bar, tap * cin + kb * BK, n0);
        } else {
          tma_load_2d(dst, &tmB, bar, kb * BK, n0);
        }
      };
      if (b_res && (int)blockIdx.x < total_tiles) {
        mbar_arrive_expect_tx(bres_full, g.num_kb * L::B_BYTES);
        for (int kb = 0; kb < g.num_kb; ++kb) load_b(bres + kb * L::B_BYTES, bres_full, kb, 0);
      }
      const int tstep = twin ? 2 : 1;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += tstep * gridDim.x) {
        const int mt = tile / g.n_tiles, nt = tile - mt * g.n_tiles;
        const int n0 = nt * BN;
        int img, y0, x0;
        tile_origin<GEO>(g, mt, img, y0, x0);
        // twin tiles: the CTA's next tile (one N tile, so mt1 = tile1) shares this one's stages
        const int tile1 = tile + (int)gridDim.x;
        const bool has1 = twin && tile1 < total_tiles;
        int img1 = 0, y1 = 0, x1 = 0;
        if (has1) tile_origin<GEO>(g, tile1, img1, y1, x1);
        for (int kb = 0; kb < g.num_kb; ++kb, ++it) {
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, SCB_ERR_WAIT_EMPTY)) { ok = false; break; }
          uint8_t* sa = smem + s * SBYTES;
          mbar_arrive_expect_tx(&full[s], b_res ? L::A_TX : (has1 ? 2 : 1) * L::A_TX + L::B_BYTES);
          if (GEO == GEO_UP2 && g.TW > 0) {
            tma_load_3d(sa, &tmA, &full[s], kb * BK, x0, y0);
          } else if (GEO == GEO_FLAT || GEO == GEO_UP2) {
            tma_load_2d(sa, &tmA, &full[s], kb * BK, mt * 128);
          } else if (GEO == GEO_CONV3) {
            const int tap = kb / g.kb_per_tap, ch = kb - tap * g.kb_per_tap;
            const int ky = tap / 3, kx = tap - ky * 3;
            tma_load_4d(sa, &tmA, &full[s], ch * BK, x0 + kx - 1, y0 + ky - 1, img);
          } else if (GEO == GEO_CONV3X) {
            // k block = (channel chunk, kx): one 10 x 16 box, three weight taps
            const int kx = kb % 3, ch = kb / 3;
            tma_load_4d(sa, &tmA, &full[s], ch * BK, x0 + kx - 1, y0 - 1, img);
            if (has1) tma_load_4d(sa + L::A_BYTES, &tmA, &full[s], ch * BK, x1 + kx - 1, y1 - 1, img1);
          } else if (GEO == GEO_CONV3W) {
            // k block = channel chunk: one 20 x 10 box, all nine weight taps
            tma_load_4d(sa, &tmA, &full[s], kb * BK, x0 - 1, y0 - 1, img);
          } else {  // GEO_DOWN2
            const int tap = kb / g.kb_per_tap, ch = kb - tap * g.kb_per_tap;
            tma_load_5d(sa, &tmA, &full[s], ch * BK, tap & 1, x0, tap >> 1, y0);
          }
          if (!b_res) load_b(sa + (twin ? 2 : 1) * L::A_BYTES, &full[s], kb, n0);
        }
        if (RES_MMA) {
          for (int j = 0; j < g.res_kb && ok; ++j, ++it) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&empty[s], ph ^ 1, SCB_ERR_WAIT_EMPTY)) { ok = false; break; }
            mbar_arrive_expect_tx(&full[s], (has1 ? 2 : 1) * 128 * BK * 2);
            if (GEO == GEO_FLAT)
              tma_load_2d(smem + s * SBYTES, &em.resA, &full[s], n0 + j * BK, mt * 128);
            else
              tma_load_4d(smem + s * SBYTES, &em.resA, &full[s], n0 + j * BK, x0, y0, img);
            if (has1) tma_load_4d(smem + s * SBYTES + L::A_BYTES, &em.resA, &full[s], n0 + j * BK, x1, y1, img1);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- UMMA issuer ----------------
    if (lane == 0) {
      uint32_t it = 0, t = 0;
      bool ok = true;
      if (b_res && (int)blockIdx.x < total_tiles) {
        ok = mbar_wait(bres_full, 0, SCB_ERR_WAIT_FULL);
        tc_fence_after();
      }
      const int tstep = twin ? 2 : 1;
      for (int tile = blockIdx.x; tile < total_tiles && ok; tile += tstep * gridDim.x, t += tstep) {
        // twin tiles: this tile and the CTA's next one, accumulators t and t + 1
        const bool has1 = twin && tile + (int)gridDim.x < total_tiles;
        const uint32_t a = t % L::NACC, aph = (t / L::NACC) & 1;
        const uint32_t a1 = (t + 1) % L::NACC, aph1 = ((t + 1) / L::NACC) & 1;
        if (!mbar_wait(&acc_empty[a], aph ^ 1, SCB_ERR_WAIT_ACC_FREE)) break;
        if (has1 && !mbar_wait(&acc_empty[a1], aph1 ^ 1, SCB_ERR_WAIT_ACC_FREE)) break;
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + a * BN, d_tmem1 = tmem_base + a1 * BN;
        for (int kb = 0; kb < g.num_kb; ++kb, ++it) {
          const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
          if (!mbar_wait(&full[s], ph, SCB_ERR_WAIT_FULL)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = smem_u32(smem + s * SBYTES);
          const uint32_t sb = b_res ? smem_u32(bres + kb * L::B_BYTES) : sa + (twin ? 2 : 1) * L::A_BYTES;
          if (GEO == GEO_CONV3X && has1) {  // twin tiles: each B view feeds both tiles' UMMAs
#pragma unroll
            for (int ky = 0; ky < 3; ++ky)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k) {
                const uint64_t bdesc = make_sdesc(sb + ky * (BN * BK * 2) + k * 32, ROWB, SWZ);
                umma_f16(d_tmem, make_sdesc(sa + ky * 16 * ROWB + k * 32, ROWB, SWZ), bdesc, IDESC, (kb | ky | k) != 0);
                umma_f16(d_tmem1, make_sdesc(sa + L::A_BYTES + ky * 16 * ROWB + k * 32, ROWB, SWZ), bdesc, IDESC,
                         (kb | ky | k) != 0);
              }
          } else if (GEO == GEO_CONV3X) {
#pragma unroll
            for (int ky = 0; ky < 3; ++ky)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                umma_f16(d_tmem, make_sdesc(sa + ky * 16 * ROWB + k * 32, ROWB, SWZ),
                         make_sdesc(sb + ky * (BN * BK * 2) + k * 32, ROWB, SWZ), IDESC, (kb | ky | k) != 0);
          } else if (GEO == GEO_CONV3W) {
            constexpr uint32_t BW = kConv3wTW + 2;  // box row pitch in pixels
#pragma unroll
            for (int tap = 0; tap < 9; ++tap)
#pragma unroll
              for (int k = 0; k < BK / 16; ++k)
                umma_f16(d_tmem,
                         make_sdesc_sbo(sa + ((tap / 3) * BW + tap % 3) * ROWB + k * 32, BW * ROWB, SWZ),
                         make_sdesc(sb + tap * (BN * BK * 2) + k * 32, ROWB, SWZ), IDESC, (kb | tap | k) != 0);
          } else {
#pragma unroll
            for (int k = 0; k < BK / 16; ++k) {
              umma_f16(d_tmem, make_sdesc(sa + k * 32, ROWB, SWZ), make_sdesc(sb + k * 32, ROWB, SWZ), IDESC,
                       (kb | k) != 0);
            }
          }
          umma_commit(&empty[s]);
        }
        if (RES_MMA) {
          // accumulator columns j BK + 32 h + n += A channels 32 h + 16 q + k' (k' < 16)
          // against identity rows n, columns 16 q + k': a one where n = 16 q + k'
          constexpr uint32_t IDESC_R = make_idesc_f16(128, 32);
          const uint32_t si = smem_u32(staging);
          for (int j = 0; j < g.res_kb && ok; ++j, ++it) {
            const uint32_t s = it % STAGES, ph = (it / STAGES) & 1;
            if (!mbar_wait(&full[s], ph, SCB_ERR_WAIT_FULL)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_u32(smem + s * SBYTES);
#pragma unroll
            for (int h = 0; h < BK / 32; ++h)
#pragma unroll
              for (int q = 0; q < 2; ++q)
                umma_f16(d_tmem + j * BK + h * 32, make_sdesc(sa + (2 * h + q) * 32, ROWB, SWZ),
                         make_sdesc(si + q * 32, 64, SW_64B), IDESC_R, 1);
            if (has1) {
#pragma unroll
              for (int h = 0; h < BK / 32; ++h)
#pragma unroll
                for (int q = 0; q < 2; ++q)
                  umma_f16(d_tmem1 + j * BK + h * 32, make_sdesc(sa + L::A_BYTES + (2 * h + q) * 32, ROWB, SWZ),
                           make_sdesc(si + q * 32, 64, SW_64B), IDESC_R, 1);
            }
            umma_commit(&empty[s]);
          }
        }
        umma_commit(&acc_full[a]);
        if (has1) umma_commit(&acc_full[a1]);
      }
    }
  } else if (TMAEPI) {
    // ---------------- asynchronous (TMA) epilogue: warps 2..5 ----------------
    const int q = warp & 3;
    const int r = q * 32 + lane;
    const bool elected = (warp == 2 && lane == 0);
    const bool has_res = e.st_res16 >= 0 || e.st_res32 >= 0 || e.st_skip >= 0;
    uint32_t t = 0, rs = 0, os = 0;  // tiles, residual slabs consumed, output slabs stored
    const uint32_t NRES = (uint32_t)e.res_bufs;
    uint8_t* res_stage = staging + e.st_ident_bytes;
    uint8_t* out_stage = res_stage + NRES * e.st_res_bytes;
    auto issue_res = [&](int mt, int col, uint32_t idx) {
      const uint32_t b = idx % NRES;
      uint8_t* base = res_stage + b * e.st_res_bytes;
      mbar_arrive_expect_tx(&res_full[b], e.st_res_bytes);
      if (e.st_res16 >= 0) epi_slab_load<GEO>(base + e.st_res16, &em.res16, &res_full[b], col, mt, g);
      if (e.st_res32 >= 0) epi_slab_load<GEO>(base + e.st_res32, &em.res32, &res_full[b], col, mt, g);
      if (e.st_skip >= 0) epi_slab_load<GEO>(base + e.st_skip, &em.skip, &res_full[b], col, mt, g);
    };
    // Residual slabs are requested NRES - 1 slabs ahead, across tile boundaries:
    // slab j of this CTA is 32-column slab j % (BN / 32) of its tile j / (BN / 32),
    // so the first slabs of a tile never wait a full DRAM round trip.
    constexpr uint32_t SPT = BN >= 32 ? BN / 32 : 1;  // slabs per tile
    auto issue_slab = [&](uint32_t j) {
      const int tile = (int)blockIdx.x + (int)(j / SPT) * (int)gridDim.x;
      if (tile >= total_tiles) return;
      const int mt = tile / g.n_tiles;
      issue_res(mt, (tile - mt * g.n_tiles) * BN + (int)(j % SPT) * 32, j);
    };
    if (has_res && elected)
      for (uint32_t j = 0; j + 1 < NRES; ++j) issue_slab(j);
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++t) {
      const int mt = tile / g.n_tiles, nt = tile - mt * g.n_tiles;
      const int n0 = nt * BN;
      const uint32_t a = t % L::NACC, aph = (t / L::NACC) & 1;
      if (!mbar_wait(&acc_full[a], aph, SCB_ERR_WAIT_ACC)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + a * BN;
      // LayerNorm statistics of this row over the tile's LN columns, from the
      // accumulator (+ bias + fp16 residual, re-read from global memory here), with
      // a shifted sum of squares
      const bool do_ln = e.st_ln >= 0 && e.ln_lo >= n0 && e.ln_lo < n0 + BN;
      float ln_mean = 0.f, ln_rstd = 0.f;
      if (GEO == GEO_FLAT && do_ln) {
        const long p = (long)mt * 128 + r;
        float shift = 0.f, s1 = 0.f, s2 = 0.f;
#pragma unroll 1
        for (int c = e.ln_lo - n0; c < e.ln_lo - n0 + e.ln_n; c += 32) {
          float v[32];
          tmem_ld16x2(tbase + c, v, tbase + c + 16, v + 16);
          if (e.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(e.bias + n0 + c);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 bb = __ldg(b4 + j);
              add4_f32x2(v + 4 * j, bb);
            }
          }
          if (e.res16 && g.res_kb == 0 && p < g.M) {  // (else already in the accumulator)
            const uint4* src = reinterpret_cast<const uint4*>(e.res16 + p * e.res16_ld + n0 + c);
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              const uint4 u = __ldg(src + h);
              const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(hp[i]);
                add2_f32x2(v + 8 * h + 2 * i, f.x, f.y);
              }
            }
          }
          if (c == e.ln_lo - n0) shift = v[0];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float d = v[j] - shift;
            s1 += d;
            s2 += d * d;
          }
        }
        const float inv_n = 1.f / (float)e.ln_n;
        const float md = s1 * inv_n;
        ln_mean = shift + md;
        ln_rstd = rsqrtf(fmaxf(s2 * inv_n - md * md, 0.f) + 1e-5f);
      }
      if constexpr (PAIRS) {
        // Two 32-column slabs per round, one in each staging buffer: half the barrier,
        // fence and store rounds of the slab loop below (no residual slabs here: the
        // host picks this form only without them)
#pragma unroll 1
        for (int c = 0; c < BN; c += 64, os += 2) {
          float v[64];
          {
            uint32_t rr[4][16];
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) tmem_ld16_issue(tbase + c + 16 * q4, rr[q4]);
            tmem_wait_ld();
#pragma unroll
            for (int q4 = 0; q4 < 4; ++q4) {
              tmem_fence16(rr[q4]);
              u32_to_f32_16(rr[q4], v + 16 * q4);
            }
          }
          const int n = n0 + c;
          if (e.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(e.bias + n);
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const float4 bb = __ldg(b4 + j);
              add4_f32x2(v + 4 * j, bb);
            }
          }
          if (e.act == ACT_RELU) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] = fmaxf(v[j], 0.f);
          } else if (e.act == ACT_GELU) {
#pragma unroll
            for (int j = 0; j < 64; j += 2) {
              const __half2 gv = gelu_tanh_h2(__floats2half2_rn(v[j], v[j + 1]));
              const float2 f = __half22float2(gv);
              v[j] = f.x;
              v[j + 1] = f.y;
            }
          }
          // both staging buffers were last read by the previous round's stores
          if (elected) bulk_wait_group_read<0>();
          epi_bar();
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            uint8_t* ob = out_stage + hh * e.st_out_bytes;
            const float* vh = v + 32 * hh;
            const int nh = n + 32 * hh;
            if (e.st_out32 >= 0) {
#pragma unroll
              for (int j = 0; j < 8; ++j)
                *reinterpret_cast<float4*>(ob + e.st_out32 + swz_off(r, j, 128)) =
                    make_float4(vh[4 * j], vh[4 * j + 1], vh[4 * j + 2], vh[4 * j + 3]);
            }
            if (do_ln && nh >= e.ln_lo && nh < e.ln_lo + e.ln_n) {
              const float* lg = e.ln_g + (nh - e.ln_lo);
              const float* lb = e.ln_b + (nh - e.ln_lo);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float o[8];
#pragma unroll
                for (int i = 0; i < 8; ++i)
                  o[i] = (vh[8 * j + i] - ln_mean) * ln_rstd * __ldg(lg + 8 * j + i) + __ldg(lb + 8 * j + i);
                *reinterpret_cast<uint4*>(ob + e.st_ln + swz_off(r, j, 64)) =
                    make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]),
                               pack_half2(o[6], o[7]));
              }
            }
            if (e.st_out16 >= 0) {
#pragma unroll
              for (int j = 0; j < 4; ++j)
                *reinterpret_cast<uint4*>(ob + e.st_out16 + swz_off(r, j, 64)) =
                    make_uint4(pack_half2(vh[8 * j], vh[8 * j + 1]), pack_half2(vh[8 * j + 2], vh[8 * j + 3]),
                               pack_half2(vh[8 * j + 4], vh[8 * j + 5]), pack_half2(vh[8 * j + 6], vh[8 * j + 7]));
            }
          }
          fence_proxy_async_smem();
          epi_bar();  // both halves staged
          if (elected) {
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const uint8_t* ob = out_stage + hh * e.st_out_bytes;
              const int nh = n + 32 * hh;
              if (e.st_out32 >= 0) epi_slab_store<GEO>(&em.out32, ob + e.st_out32, nh, mt, g);
              if (e.st_out16 >= 0) {
                if (e.out16b && nh >= e.out16_split)
                  epi_slab_store<GEO>(&em.out16b, ob + e.st_out16, nh - e.out16_split, mt, g);
                else
                  epi_slab_store<GEO>(&em.out16, ob + e.st_out16, nh, mt, g);
              }
              if (do_ln && nh >= e.ln_lo && nh < e.ln_lo + e.ln_n)
                epi_slab_store<GEO>(&em.lnout, ob + e.st_ln, nh - e.ln_lo, mt, g);
            }
            bulk_commit_group();
          }
        }
      } else {
#pragma unroll 1
      for (int c = 0; c < BN; c += 32, ++os) {
        // buffer (rs + NRES - 1) % NRES held slab rs - 1, which every thread finished
        // reading before the previous slab's second barrier
        if (has_res && elected) issue_slab(rs + NRES - 1);
        float v[32];
        tmem_ld16x2(tbase + c, v, tbase + c + 16, v + 16);
        const int n = n0 + c;
        if (e.bias) {  // 32 columns of bias as eight 16-byte loads (n is a multiple of 32)
          const float4* b4 = reinterpret_cast<const float4*>(e.bias + n);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 bb = __ldg(b4 + j);
            add4_f32x2(v + 4 * j, bb);
          }
        }
        if (e.act == ACT_RELU) {
#pragma unroll
          for (int j = 0; j < 32; ++j) v[j] = fmaxf(v[j], 0.f);
        } else if (e.act == ACT_GELU) {
          // the GELU output is an fp16 operand: evaluate it in packed half2
#pragma unroll
          for (int j = 0; j < 32; j += 2) {
            const __half2 gv = gelu_tanh_h2(__floats2half2_rn(v[j], v[j + 1]));
            const float2 f = __half22float2(gv);
            v[j] = f.x;
            v[j + 1] = f.y;
          }
        }
        float sk[32];
        if (has_res) {
          const uint32_t b = rs % NRES;
          mbar_wait(&res_full[b], (rs / NRES) & 1, SCB_ERR_WAIT_ACC);
          const uint8_t* base = res_stage + b * e.st_res_bytes;
          if (e.st_res16 >= 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const uint4 u = *reinterpret_cast<const uint4*>(base + e.st_res16 + swz_off(r, j, 64));
              const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const float2 f = __half22float2(hp[i]);
                add2_f32x2(v + 8 * j + 2 * i, f.x, f.y);
              }
            }
          }
          if (e.st_res32 >= 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 f = *reinterpret_cast<const float4*>(base + e.st_res32 + swz_off(r, j, 128));
              add4_f32x2(v + 4 * j, f);
            }
          }
          if (e.st_skip >= 0) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 f = *reinterpret_cast<const float4*>(base + e.st_skip + swz_off(r, j, 128));
              sk[4 * j] = f.x; sk[4 * j + 1] = f.y; sk[4 * j + 2] = f.z; sk[4 * j + 3] = f.w;
            }
          }
          ++rs;
        }
        // Output staging buffer (os & 1): the store that last used it (two slabs
        // ago) must have finished reading it before the threads refill it.
        if (elected) bulk_wait_group_read<1>();
        epi_bar();
        uint8_t* ob = out_stage + (os & 1) * e.st_out_bytes;
        if (e.st_out32 >= 0) {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            *reinterpret_cast<float4*>(ob + e.st_out32 + swz_off(r, j, 128)) =
                make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]);
        }
        const bool ln_slab = do_ln && n >= e.ln_lo && n < e.ln_lo + e.ln_n;
        if (ln_slab) {
          const float* lg = e.ln_g + (n - e.ln_lo);
          const float* lb = e.ln_b + (n - e.ln_lo);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float o[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) o[i] = (v[8 * j + i] - ln_mean) * ln_rstd * __ldg(lg + 8 * j + i) + __ldg(lb + 8 * j + i);
            *reinterpret_cast<uint4*>(ob + e.st_ln + swz_off(r, j, 64)) =
                make_uint4(pack_half2(o[0], o[1]), pack_half2(o[2], o[3]), pack_half2(o[4], o[5]), pack_half2(o[6], o[7]));
          }
        }
        if (e.st_out16 >= 0) {
          if (e.st_skip >= 0) {
#pragma unroll
            for (int j = 0; j < 32; j += 2) add2_f32x2(v + j, sk[j], sk[j + 1]);
          }
#pragma unroll
          for (int j = 0; j < 4; ++j)
            *reinterpret_cast<uint4*>(ob + e.st_out16 + swz_off(r, j, 64)) =
                make_uint4(pack_half2(v[8 * j], v[8 * j + 1]), pack_half2(v[8 * j + 2], v[8 * j + 3]),
                           pack_half2(v[8 * j + 4], v[8 * j + 5]), pack_half2(v[8 * j + 6], v[8 * j + 7]));
        }
        fence_proxy_async_smem();
        epi_bar();  // staging complete; also every thread is done with this slab's residuals
        if (elected) {
          if (e.st_out32 >= 0) epi_slab_store<GEO>(&em.out32, ob + e.st_out32, n, mt, g);
          if (e.st_out16 >= 0) {
            if (e.out16b && n >= e.out16_split)
              epi_slab_store<GEO>(&em.out16b, ob + e.st_out16, n - e.out16_split, mt, g);
            else
              epi_slab_store<GEO>(&em.out16, ob + e.st_out16, n, mt, g);
          }
          if (ln_slab) epi_slab_store<GEO>(&em.lnout, ob + e.st_ln, n - e.ln_lo, mt, g);
          bulk_commit_group();
        }
      }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
    if (elected) bulk_wait_group<0>();
  } else {
    // ---------------- direct epilogue: warps 2..5, thread = accumulator row ----------------
    // Residual loads are software-pipelined one 16-column chunk ahead, and the
    // first chunk's loads are issued before waiting for the accumulator.
    const int q = warp & 3;
    const int r = q * 32 + lane;
    uint32_t t = 0;
    for (int tile = blockIdx.x; tile < total_tiles; tile += gridDim.x, ++t) {
      const int mt = tile / g.n_tiles, nt = tile - mt * g.n_tiles;
      const int n0 = nt * BN;
      const uint32_t a = t % L::NACC, aph = (t / L::NACC) & 1;
      int col0;
      const long p = row_pixel<GEO>(g, mt, r, n0, col0);
      ResChunk cur, nxt;
      if (p >= 0) load_res(e, p, col0, cur);
      if (!mbar_wait(&acc_full[a], aph, SCB_ERR_WAIT_ACC)) break;
      tc_fence_after();
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + a * BN;
      const bool do_ln = e.ln_out != nullptr && e.ln_lo >= n0 && e.ln_lo < n0 + BN;
      float ln_sum = 0.f, ln_sq = 0.f, ln_shift = 0.f;
#pragma unroll 1
      for (int c = 0; c < BN; c += 16) {
        if (p >= 0 && c + 16 < BN) load_res(e, p, col0 + c + 16, nxt);
        float v[16];
        tmem_ld16(tbase + c, v);
        const int n = n0 + c;       // global GEMM column
        const int oc = col0 + c;    // output column
        if (e.bias) {  // n is a multiple of 16
          const float4* b4 = reinterpret_cast<const float4*>(e.bias + n);
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            const float4 bb = __ldg(b4 + j);
            add4_f32x2(v + 4 * j, bb);
          }
        }
        if (e.act == ACT_RELU) {
#pragma unroll
          for (int j = 0; j < 16; ++j) v[j] = fmaxf(v[j], 0.f);
        } else if (e.act == ACT_GELU) {
          // the GELU output is an fp16 operand: evaluate it in packed half2
#pragma unroll
          for (int j = 0; j < 16; j += 2) {
            const float2 f = __half22float2(gelu_tanh_h2(__floats2half2_rn(v[j], v[j + 1])));
            v[j] = f.x;
            v[j + 1] = f.y;
          }
        }
        if (p >= 0) {
          if (e.res16) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
              const __half2* hp = reinterpret_cast<const __half2*>(&cur.r16[h]);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                float2 f = __half22float2(hp[j]);
                v[h * 8 + 2 * j] += f.x;
                v[h * 8 + 2 * j + 1] += f.y;
              }
            }
          }
          if (e.res32) {
#pragma unroll
            for (int h = 0; h < 4; ++h) {
              v[4 * h] += cur.r32[h].x; v[4 * h + 1] += cur.r32[h].y;
              v[4 * h + 2] += cur.r32[h].z; v[4 * h + 3] += cur.r32[h].w;
            }
          }
          if (e.out32) {
            float4* dst = reinterpret_cast<float4*>(e.out32 + p * e.out32_ld + oc);
#pragma unroll
            for (int h = 0; h < 4; ++h) dst[h] = make_float4(v[4 * h], v[4 * h + 1], v[4 * h + 2], v[4 * h + 3]);
          }
          if (e.out16) {
            float s[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) s[j] = v[j];
            if (e.skip32) {
#pragma unroll
              for (int h = 0; h < 4; ++h) {
                s[4 * h] += cur.sk[h].x; s[4 * h + 1] += cur.sk[h].y;
                s[4 * h + 2] += cur.sk[h].z; s[4 * h + 3] += cur.sk[h].w;
              }
            }
            uint4* dst = (e.out16b && oc >= e.out16_split)
                             ? reinterpret_cast<uint4*>(e.out16b + p * e.out16b_ld + (oc - e.out16_split))
                             : reinterpret_cast<uint4*>(e.out16 + p * e.out16_ld + oc);
#pragma unroll
            for (int h = 0; h < 2; ++h)
              dst[h] = make_uint4(pack_half2(s[8 * h], s[8 * h + 1]), pack_half2(s[8 * h + 2], s[8 * h + 3]),
                                  pack_half2(s[8 * h + 4], s[8 * h + 5]), pack_half2(s[8 * h + 6], s[8 * h + 7]));
          }
        }
        if (do_ln && n >= e.ln_lo && n < e.ln_lo + e.ln_n) {
          if (n == e.ln_lo) ln_shift = v[0];
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const float d = v[j] - ln_shift;
            ln_sum += d;
            ln_sq += d * d;
          }
        }
        cur = nxt;
      }
      if (do_ln) {
        // Second pass over the LN columns: recompute v exactly as above and normalise.
        const float inv_n = 1.f / (float)e.ln_n;
        const float md = ln_sum * inv_n;
        const float var = fmaxf(ln_sq * inv_n - md * md, 0.f);
        const float mean = ln_shift + md;
        const float rstd = rsqrtf(var + 1e-5f);
#pragma unroll 1
        for (int c = e.ln_lo - n0; c < e.ln_lo - n0 + e.ln_n; c += 16) {
          float v[16];
          tmem_ld16(tbase + c, v);
          const int n = n0 + c;
          const int oc = col0 + c;
          if (e.bias) {
            const float4* b4 = reinterpret_cast<const float4*>(e.bias + n);
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float4 bb = __ldg(b4 + j);
              add4_f32x2(v + 4 * j, bb);
            }
          }
          if (p >= 0) {
            if (e.res16) {
              const uint4* src = reinterpret_cast<const uint4*>(e.res16 + p * e.res16_ld + oc);
#pragma unroll
              for (int h = 0; h < 2; ++h) {
                uint4 u = __ldg(src + h);
                const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                  float2 f = __half22float2(hp[j]);
                  v[h * 8 + 2 * j] += f.x;
                  v[h * 8 + 2 * j + 1] += f.y;
                }
              }
            }
            float o[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int k = n + j - e.ln_lo;
              o[j] = (v[j] - mean) * rstd * __ldg(e.ln_g + k) + __ldg(e.ln_b + k);
            }
            uint4* dst = reinterpret_cast<uint4*>(e.ln_out + p * e.ln_ld + (n - e.ln_lo));
#pragma unroll
            for (int h = 0; h < 2; ++h)
              dst[h] = make_uint4(pack_half2(o[8 * h], o[8 * h + 1]), pack_half2(o[8 * h + 2], o[8 * h + 3]),
                                  pack_half2(o[8 * h + 4], o[8 * h + 5]), pack_half2(o[8 * h + 6], o[8 * h + 7]));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&acc_empty[a]);
    }
  }

  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, L::TMEM_COLS);
  }
}

}  // namespace scb
