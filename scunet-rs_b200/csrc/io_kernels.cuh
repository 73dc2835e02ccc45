// The input end of the network:
//
//   head: uint8 or f32 NCHW image [n][c][h][w] -> replicate pad to [hp][wp]
//         (src/plan.rs:67-82, fused: the pad is a clamped read) -> m_head 3x3 conv
//         c -> 64, zero pad 1, no bias (tools/network_scunet.py:191) -> the x1 skip
//         (fp32 NHWC) and its fp16 shadow (the next GEMM's A operand).
//
// The output end (m_tail 3x3 conv 64 -> c, crop, f32 or uint8 NCHW) is the 3x3
// implicit GEMM of gemm.cuh with N = 16 and its crop-to-NCHW epilogue.
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
  for (long tile = blockIdx.x; tile < tiles; tile += gridDim.x) {
    const long p = tile * 128 + tid;
    float in[32];
#pragma unroll
    for (int k = 0; k < 32; ++k) in[k] = 0.f;
    if (p < npx) {
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
                in[(ci * 3 + ky) * 3 + kx] = g.in_u8 ? (float)reinterpret_cast<const uint8_t*>(x)[off] * (1.0f / 255.0f)
                                                     : reinterpret_cast<const float*>(x)[off];
              }
            }
          }
        }
      }
    }
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

}  // namespace scb
