// The input end of the network:
//
//   head: uint8 or f32 NCHW image [n][c][h][w] -> replicate pad to [hp][wp]
//         (src/plan.rs:67-82, fused: the pad is a clamped read) -> m_head 3x3 conv
//         c -> 64, zero pad 1, no bias (tools/network_scunet.py:191) -> the x1 skip
//         (fp32 NHWC) and its fp16 shadow (the next GEMM's A operand).
//
//   tail: the (y + x1) fp16 shadow (NHWC, 64 channels) -> m_tail 3x3 conv 64 -> c,
//         zero pad 1, no bias (tools/network_scunet.py:195) -> crop to h x w
//         (src/backend.rs:98-105) -> f32 or uint8 NCHW.
#pragma once
#include "ptx.cuh"

namespace scb {

struct HeadGeom {
  int n, c, h, w, hp, wp;
  int in_u8;  // 1: uint8 input scaled by 1/255; 0: f32 in [0,1]
  int row0;   // image row of output row 0 (a row band starts below 0)
  int rows;   // output rows per image (hp for the whole image)
};

// m_head on tcgen05: each 128-pixel tile's im2col rows (27 taps, zero-padded to
// K = 32, order ci, ky, kx) are built by the threads straight into a 64B-swizzled
// K-major smem tile, then D[128 x 64] = A . Wh^T is one UMMA chain into TMEM. The
// epilogue stages x1 (f32) and its fp16 shadow in 128B-swizzled smem and sends them
// with three TMA tensor stores per tile (whole 128-byte pixel rows, coalesced); rows
// past the last pixel are clipped by the tensor maps. The replicate pad is the
// clamped read; the conv's own zero pad is the bounds test.
constexpr int HEAD_ST = 8192 + 4096;               // staging: 2 f32 slabs + 1 fp16 slab of [128 x 128 B]
constexpr int HEAD_BAR = HEAD_ST + 3 * 16384;
constexpr int HEAD_SMEM = HEAD_BAR + 64 + 1024;

__global__ void __launch_bounds__(128)
head_tc_kernel(const void* __restrict__ x, const __half* __restrict__ wk /*[64][32] K-major*/,
               const __grid_constant__ CUtensorMap m32, const __grid_constant__ CUtensorMap m16, const HeadGeom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bar = reinterpret_cast<uint64_t*>(sm + HEAD_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bar + 1);
  uint8_t* st = sm + HEAD_ST;
  const int tid = threadIdx.x, warp = tid >> 5;
  for (int idx = tid; idx < 64 * 4; idx += 128) {
    const int r = idx >> 2, j = idx & 3;
    *reinterpret_cast<uint4*>(sm + 8192 + swz_off(r, j, 64)) = __ldg(reinterpret_cast<const uint4*>(wk + r * 32 + j * 8));
  }
  if (tid == 0) {
    mbar_init(bar, 1);
    mbar_fence_init();
    tma_prefetch_desc(&m32);
    tma_prefetch_desc(&m16);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 64);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
  const uint32_t sb = smem_u32(sm);
  uint32_t phase = 0;
  const long npx = (long)g.n * g.rows * g.wp;
  const long tiles = (npx + 127) / 128;
  // The 27 input taps of this thread's pixel of `tile`, as the raw bits loaded (a
  // uint8 value or an f32 bit pattern; 0 outside the image = the conv's zero pad):
  // the next tile's loads are issued before this tile's MMA wait and epilogue and
  // converted only when they are written to shared memory, so their latency is
  // hidden behind that work.
  auto gather = [&](long tile, uint32_t* raw) {
    const long p = tile * 128 + tid;
#pragma unroll
    for (int k = 0; k < 27; ++k) raw[k] = 0u;
    if (tile >= tiles || p >= npx) return;
    const int img = (int)(p / ((long)g.rows * g.wp));
    const int rem = (int)(p - (long)img * g.rows * g.wp);
    const int y = g.row0 + rem / g.wp, xx = rem % g.wp;
#pragma unroll
    for (int ci = 0; ci < 3; ++ci) {
      if (ci < g.c) {
#pragma unroll
        for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const int yy = y + ky - 1, xq = xx + kx - 1;
            if (yy >= 0 && yy < g.hp && xq >= 0 && xq < g.wp) {
              const int sy = min(yy, g.h - 1), sx = min(xq, g.w - 1);
              const long off = (((long)img * g.c + ci) * g.h + sy) * g.w + sx;
              raw[(ci * 3 + ky) * 3 + kx] = g.in_u8 ? (uint32_t)__ldg(reinterpret_cast<const uint8_t*>(x) + off)
                                                    : __ldg(reinterpret_cast<const uint32_t*>(x) + off);
            }
          }
        }
      }
    }
  };
  uint32_t raw[27];
  gather(blockIdx.x, raw);
  for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    float in[32];
#pragma unroll
    for (int k = 0; k < 27; ++k) in[k] = g.in_u8 ? (float)raw[k] * (1.0f / 255.0f) : __uint_as_float(raw[k]);
#pragma unroll
    for (int k = 27; k < 32; ++k) in[k] = 0.f;
#pragma unroll
    for (int c = 0; c < 4; ++c)
      *reinterpret_cast<uint4*>(sm + swz_off(tid, c, 64)) =
          make_uint4(pack_half2(in[8 * c], in[8 * c + 1]), pack_half2(in[8 * c + 2], in[8 * c + 3]),
                     pack_half2(in[8 * c + 4], in[8 * c + 5]), pack_half2(in[8 * c + 6], in[8 * c + 7]));
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (tid == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 64);
#pragma unroll
      for (int k = 0; k < 2; ++k)
        umma_f16(tmem, make_sdesc(sb + k * 32, 64, SW_64B), make_sdesc(sb + 8192 + k * 32, 64, SW_64B), id, k);
      umma_commit(bar);
    }
    gather(tile + gridDim.x, raw);
    mbar_wait(bar, phase, SCB_ERR_WAIT_ATTN);
    phase ^= 1;
    tc_fence_after();
    // the previous tile's stores must have finished reading the staging buffers
    if (tid == 0) bulk_wait_group_read<0>();
    __syncthreads();
#pragma unroll
    for (int c = 0; c < 64; c += 16) {
      float v[16];
      tmem_ld16(trow + c, v);
      // f32 slab c / 32, 16-byte chunks (c % 32) / 4 .. + 3; fp16 slab, chunks c / 8, c / 8 + 1
      uint8_t* s32 = st + (c >> 5) * 16384;
#pragma unroll
      for (int h4 = 0; h4 < 4; ++h4)
        *reinterpret_cast<float4*>(s32 + swz_off(tid, ((c & 31) >> 2) + h4, 128)) =
            make_float4(v[4 * h4], v[4 * h4 + 1], v[4 * h4 + 2], v[4 * h4 + 3]);
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2)
        *reinterpret_cast<uint4*>(st + 2 * 16384 + swz_off(tid, (c >> 3) + h2, 128)) =
            make_uint4(pack_half2(v[8 * h2], v[8 * h2 + 1]), pack_half2(v[8 * h2 + 2], v[8 * h2 + 3]),
                       pack_half2(v[8 * h2 + 4], v[8 * h2 + 5]), pack_half2(v[8 * h2 + 6], v[8 * h2 + 7]));
    }
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();  // staging complete; the A tile and TMEM are free for the next tile
    tc_fence_after();
    if (tid == 0) {
      tma_store_2d(&m32, st, 0, (int)(tile * 128));
      tma_store_2d(&m32, st + 16384, 32, (int)(tile * 128));
      tma_store_2d(&m16, st + 2 * 16384, 0, (int)(tile * 128));
      bulk_commit_group();
    }
  }
  if (tid == 0) bulk_wait_group<0>();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 64);
}

// m_tail with the tensor cores doing the channel sums and the CUDA cores the
// spatial ones. For every input pixel p one UMMA chain (K = 64 channels, N = 32)
// gives P[p][3 * tap + co] = sum_ci x[p][ci] * Wt[co][ci][tap] for all nine taps and
// output channels at once (27 of the 32 columns); output pixel (y, x) is then
// sum_(ky,kx) P[(y + ky - 1, x + kx - 1)][3 * (3 ky + kx) + co]. Four UMMAs of
// 128 x 32 x 16 per 128 input pixels instead of 36 of 128 x 16 x 16 for the 3x3
// implicit GEMM with N = 16, and each input pixel crosses shared memory once.
//
// A work unit is a strip of TAIL_COLS output columns x up to TAIL_ROWS output rows
// of one image. Its input rows (one more above and below; the strip's 128 input
// columns start one left of it) stream through a TMA stage ring; the TMA zero fill
// outside the stored plane is the conv's zero padding. Warp 4 issues the loads,
// warp 5 the UMMAs into a ring of TAIL_NB 32-column TMEM buffers, warps 0-3 (one
// thread per TMEM lane = input column) move each row's P through a shared row
// buffer, and thread j then adds the three horizontal neighbours j, j + 1, j + 2 of
// that row into three rolling output rows (ky = 2, 1, 0) and stores the finished
// one, coalesced along x.
struct TailGeom {
  int n, H, W;         // stored plane: n images of H rows x W columns, 64 channels
  int row0, rows_out;  // output rows [row0, row0 + rows_out) of each image's H
  int c;               // output channels (1 or 3)
  int h, w;            // crop
  int row_off;         // image row of stored row y is y + row_off
  int u8;              // 1: uint8 output, clamp(v, 0, 1) * 255 + 0.5 truncated (src/image.rs:60-63); 0: f32
  int strips, chunks;  // work units per image
};
constexpr int TAIL_COLS = 126, TAIL_ROWS = 32, TAIL_STAGES = 4, TAIL_NB = 4;
constexpr int TAIL_THREADS = 192;
constexpr int TAIL_PSTRIDE = 27;                        // floats per pixel in the P row buffer (odd)
constexpr int TAIL_B = TAIL_STAGES * 16384;             // stages: [128 px x 128 B], 128B-swizzled
constexpr int TAIL_P = TAIL_B + 32 * 128;               // B: [32 x 128 B], 128B-swizzled K-major
constexpr int TAIL_BAR = TAIL_P + 2 * 128 * TAIL_PSTRIDE * 4;
constexpr int TAIL_SMEM = TAIL_BAR + 256 + 1024;

__global__ void __launch_bounds__(TAIL_THREADS, 2)
tail_tc_kernel(const __grid_constant__ CUtensorMap tmx, const __half* __restrict__ wt /*[32][64] K-major*/,
               void* __restrict__ out, const TailGeom g) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(sm + TAIL_BAR);
  uint64_t* empty = full + TAIL_STAGES;
  uint64_t* mma_done = empty + TAIL_STAGES;
  uint64_t* tmem_free = mma_done + TAIL_NB;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tmem_free + TAIL_NB);
  float* prow = reinterpret_cast<float*>(sm + TAIL_P);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  for (int idx = tid; idx < 32 * 8; idx += TAIL_THREADS) {
    const int r = idx >> 3, j = idx & 7;
    *reinterpret_cast<uint4*>(sm + TAIL_B + swz_off(r, j, 128)) = __ldg(reinterpret_cast<const uint4*>(wt + r * 64 + j * 8));
  }
  if (tid == 0) {
    for (int s = 0; s < TAIL_STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < TAIL_NB; ++b) {
      mbar_init(&mma_done[b], 1);
      mbar_init(&tmem_free[b], 128);
    }
    mbar_fence_init();
    tma_prefetch_desc(&tmx);
  }
  if (warp == 0) tmem_alloc(tmem_slot, 32 * TAIL_NB);
  fence_proxy_async_smem();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int per_img = g.strips * g.chunks;
  const int units = g.n * per_img;
  // unit u: image, first output column, output rows [r0, r1) of the stored plane
  auto unit = [&](int u, int& img, int& x0, int& r0, int& r1) {
    img = u / per_img;
    const int rem = u - img * per_img, ch = rem / g.strips;
    x0 = (rem - ch * g.strips) * TAIL_COLS;
    r0 = g.row0 + ch * TAIL_ROWS;
    r1 = min(r0 + TAIL_ROWS, g.row0 + g.rows_out);
  };
  if (warp == 4) {
    // ---------------- TMA producer: one 128-column input row per stage ----------------
    if (lane == 0) {
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int img, x0, r0, r1;
        unit(u, img, x0, r0, r1);
        for (int ir = r0 - 1; ir <= r1; ++ir, ++it) {
          const uint32_t s = it % TAIL_STAGES, ph = (it / TAIL_STAGES) & 1;
          if (!mbar_wait(&empty[s], ph ^ 1, SCB_ERR_WAIT_EMPTY)) { ok = false; break; }
          mbar_arrive_expect_tx(&full[s], 16384);
          tma_load_4d(sm + s * 16384, &tmx, &full[s], 0, x0 - 1, ir, img);
        }
      }
    }
  } else if (warp == 5) {
    // ---------------- UMMA issuer: P of one input row into a TMEM buffer ----------------
    if (lane == 0) {
      constexpr uint32_t id = make_idesc_f16(128, 32);
      const uint32_t sbw = smem_u32(sm + TAIL_B);
      uint32_t it = 0;
      bool ok = true;
      for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
        int img, x0, r0, r1;
        unit(u, img, x0, r0, r1);
        for (int ir = r0 - 1; ir <= r1; ++ir, ++it) {
          const uint32_t s = it % TAIL_STAGES, ph = (it / TAIL_STAGES) & 1;
          const uint32_t b = it % TAIL_NB, bph = (it / TAIL_NB) & 1;
          if (!mbar_wait(&tmem_free[b], bph ^ 1, SCB_ERR_WAIT_ACC_FREE) || !mbar_wait(&full[s], ph, SCB_ERR_WAIT_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sa = smem_u32(sm + s * 16384);
#pragma unroll
          for (int k = 0; k < 4; ++k)
            umma_f16(tmem + b * 32, make_sdesc(sa + k * 32, 128, SW_128B), make_sdesc(sbw + k * 32, 128, SW_128B), id, k);
          umma_commit(&empty[s]);
          umma_commit(&mma_done[b]);
        }
      }
    }
  } else {
    // ---------------- spatial sum: thread j = TMEM lane j = input column x0 - 1 + j ----------------
    const int j = tid;
    const uint32_t trow = tmem + ((uint32_t)(warp * 32) << 16);
    uint32_t it = 0, pb = 0;
    bool ok = true;
    for (int u = blockIdx.x; u < units && ok; u += gridDim.x) {
      int img, x0, r0, r1;
      unit(u, img, x0, r0, r1);
      float a0[3] = {0.f, 0.f, 0.f}, a1[3] = {0.f, 0.f, 0.f}, a2[3] = {0.f, 0.f, 0.f};  // rows ir - 1, ir, ir + 1
      const int x = x0 + j;
      const bool col_ok = j < TAIL_COLS && x < g.w;
      for (int ir = r0 - 1; ir <= r1; ++ir, ++it) {
        const uint32_t b = it % TAIL_NB, bph = (it / TAIL_NB) & 1;
        if (!mbar_wait(&mma_done[b], bph, SCB_ERR_WAIT_ACC)) { ok = false; break; }
        tc_fence_after();
        float v[32];
        tmem_ld16x2(trow + b * 32, v, trow + b * 32 + 16, v + 16);
        tc_fence_before();
        mbar_arrive(&tmem_free[b]);
        float* P = prow + pb * (128 * TAIL_PSTRIDE);
#pragma unroll
        for (int k = 0; k < 27; ++k) P[j * TAIL_PSTRIDE + k] = v[k];
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (j < TAIL_COLS) {
#pragma unroll
          for (int kx = 0; kx < 3; ++kx) {
            const float* q = P + (j + kx) * TAIL_PSTRIDE;
#pragma unroll
            for (int co = 0; co < 3; ++co) {
              a0[co] += q[3 * (6 + kx) + co];
              a1[co] += q[3 * (3 + kx) + co];
              a2[co] += q[3 * kx + co];
            }
          }
        }
        // output row ir - 1 has all three of its input rows
        const int y = ir - 1 + g.row_off;
        if (ir - 1 >= r0 && col_ok && y >= 0 && y < g.h) {
          for (int co = 0; co < g.c; ++co) {
            const long o = (((long)img * g.c + co) * g.h + y) * g.w + x;
            if (g.u8)
              reinterpret_cast<uint8_t*>(out)[o] = (uint8_t)(int)(fminf(fmaxf(a0[co], 0.f), 1.f) * 255.f + 0.5f);
            else
              reinterpret_cast<float*>(out)[o] = a0[co];
          }
        }
#pragma unroll
        for (int co = 0; co < 3; ++co) {
          a0[co] = a1[co];
          a1[co] = a2[co];
          a2[co] = 0.f;
        }
        pb ^= 1;
      }
    }
  }
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, 32 * TAIL_NB);
}

}  // namespace scb
