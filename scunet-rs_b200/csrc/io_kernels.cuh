// The two ends of the network, where the channel count is 1 or 3 and tensor cores
// have nothing to chew on:
//
//   head: uint8 or f32 NCHW image [n][c][h][w] -> replicate pad to [hp][wp]
//         (src/plan.rs:67-82, fused: the pad is a clamped read) -> m_head 3x3 conv
//         c -> 64, zero pad 1, no bias (tools/network_scunet.py:191) -> the x1 skip
//         (fp32 NHWC) and its fp16 shadow (the next GEMM's A operand).
//   tail: fp16 NHWC (y + x1, already summed by the last up1 block's epilogue) ->
//         m_tail 3x3 conv 64 -> c -> crop to [h][w] (src/plan.rs:85-94) -> f32 NCHW,
//         or uint8 with the CLI's quantisation clamp(v,0,1)*255+0.5 truncated
//         (src/image.rs:60-63).
#pragma once
#include "ptx.cuh"

namespace scb {

struct HeadGeom {
  int n, c, h, w, hp, wp;
  int in_u8;  // 1: uint8 input scaled by 1/255; 0: f32 in [0,1]
};

// One thread per (pixel, 16-channel group): 4 threads per pixel.
__global__ void __launch_bounds__(256)
head_conv_kernel(const void* __restrict__ x, const float* __restrict__ wt /*[64][c][3][3]*/,
                 float* __restrict__ out32, __half* __restrict__ out16, const HeadGeom g) {
  __shared__ float sw[64 * 27];
  for (int i = threadIdx.x; i < 64 * g.c * 9; i += blockDim.x) sw[i] = wt[i];
  __syncthreads();
  const long gid = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long npx = (long)g.n * g.hp * g.wp;
  if (gid >= npx * 4) return;
  const long p = gid >> 2;
  const int grp = (int)(gid & 3);
  const int img = (int)(p / ((long)g.hp * g.wp));
  const int rem = (int)(p - (long)img * g.hp * g.wp);
  const int y = rem / g.wp, xx = rem - y * g.wp;
  float in[27];
#pragma unroll
  for (int ci = 0; ci < 3; ++ci) {
#pragma unroll
    for (int ky = 0; ky < 3; ++ky) {
#pragma unroll
      for (int kx = 0; kx < 3; ++kx) {
        const int yy = y + ky - 1, xq = xx + kx - 1;
        float v = 0.f;
        if (ci < g.c && yy >= 0 && yy < g.hp && xq >= 0 && xq < g.wp) {
          const int sy = min(yy, g.h - 1), sx = min(xq, g.w - 1);  // replicate pad
          const long off = (((long)img * g.c + ci) * g.h + sy) * g.w + sx;
          v = g.in_u8 ? (float)reinterpret_cast<const uint8_t*>(x)[off] * (1.0f / 255.0f)
                      : reinterpret_cast<const float*>(x)[off];
        }
        in[(ci * 3 + ky) * 3 + kx] = v;
      }
    }
  }
  float acc[16];
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const float* wr = sw + (grp * 16 + j) * g.c * 9;
    float a = 0.f;
    for (int k = 0; k < g.c * 9; ++k) a = fmaf(wr[k], in[k], a);  // order ci, ky, kx
    acc[j] = a;
  }
  float4* d32 = reinterpret_cast<float4*>(out32 + p * 64 + grp * 16);
#pragma unroll
  for (int h4 = 0; h4 < 4; ++h4) d32[h4] = make_float4(acc[4 * h4], acc[4 * h4 + 1], acc[4 * h4 + 2], acc[4 * h4 + 3]);
  uint4* d16 = reinterpret_cast<uint4*>(out16 + p * 64 + grp * 16);
#pragma unroll
  for (int h2 = 0; h2 < 2; ++h2)
    d16[h2] = make_uint4(pack_half2(acc[8 * h2], acc[8 * h2 + 1]), pack_half2(acc[8 * h2 + 2], acc[8 * h2 + 3]),
                         pack_half2(acc[8 * h2 + 4], acc[8 * h2 + 5]), pack_half2(acc[8 * h2 + 6], acc[8 * h2 + 7]));
}

struct TailGeom {
  int n, c, h, w, hp, wp;
  int out_u8;
};

// One thread per output pixel (all c outputs); weights [c][64][3][3] in smem.
__global__ void __launch_bounds__(128)
tail_conv_kernel(const __half* __restrict__ yin, const float* __restrict__ wt, void* __restrict__ out,
                 const TailGeom g) {
  __shared__ float sw[3 * 64 * 9];
  for (int i = threadIdx.x; i < g.c * 64 * 9; i += blockDim.x) {
    // repack [co][ci][ky][kx] -> [co][ky][kx][ci]
    const int co = i / 576, r = i - co * 576, ci = r / 9, t = r - ci * 9;
    sw[co * 576 + t * 64 + ci] = wt[i];
  }
  __syncthreads();
  const long p = (long)blockIdx.x * blockDim.x + threadIdx.x;
  const long npx = (long)g.n * g.h * g.w;
  if (p >= npx) return;
  const int img = (int)(p / ((long)g.h * g.w));
  const int rem = (int)(p - (long)img * g.h * g.w);
  const int y = rem / g.w, xx = rem - y * g.w;
  float acc[3] = {0.f, 0.f, 0.f};
  for (int ky = 0; ky < 3; ++ky) {
    const int yy = y + ky - 1;
    if (yy < 0 || yy >= g.hp) continue;
    for (int kx = 0; kx < 3; ++kx) {
      const int xq = xx + kx - 1;
      if (xq < 0 || xq >= g.wp) continue;
      const uint4* src = reinterpret_cast<const uint4*>(yin + (((long)img * g.hp + yy) * g.wp + xq) * 64);
      const int t = ky * 3 + kx;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        uint4 u = __ldg(src + q);
        const __half2* hp = reinterpret_cast<const __half2*>(&u);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const float2 f = __half22float2(hp[j]);
          const int ci = q * 8 + 2 * j;
#pragma unroll
          for (int co = 0; co < 3; ++co) {
            if (co < g.c) {
              acc[co] = fmaf(sw[co * 576 + t * 64 + ci], f.x, acc[co]);
              acc[co] = fmaf(sw[co * 576 + t * 64 + ci + 1], f.y, acc[co]);
            }
          }
        }
      }
    }
  }
  for (int co = 0; co < g.c; ++co) {
    const long off = (((long)img * g.c + co) * g.h + y) * g.w + xx;
    if (g.out_u8) {
      const float v = fminf(fmaxf(acc[co], 0.f), 1.f) * 255.f + 0.5f;
      reinterpret_cast<uint8_t*>(out)[off] = (uint8_t)(int)v;
    } else {
      reinterpret_cast<float*>(out)[off] = acc[co];
    }
  }
}

}  // namespace scb
