// Shared pieces of the fused transformer-half kernels (trans32ws.cuh for trans width
// T = 32 at full resolution, trans64ws.cuh for T = 64 at half resolution). Each runs
// the whole transformer half of a ConvTransBlock on pairs of 8x8 windows (128
// tokens, one UMMA M tile):
//
//   x  = y_t                                   (fp16 plane Y_t, T channels)
//   x1 = x + proj(WMSA(LN1(x)))                (tools/network_scunet.py:134-135)
//   z  = x1 + mlp2(GELU(mlp0(LN2(x1))))        (tools/network_scunet.py:128-136)
//   -> columns [T, 2T) of Z (fp16), the conv1_2 operand.
//
// WMSA semantics are those of window_attn_kernel (attn.cuh): cyclic shift read in
// place, rel-pos bias, SW mask on the last window row/column, softmax, P.V. Every
// GEMM of the block runs on tcgen05 with its accumulator in TMEM and its operands
// in shared memory; the block's weights stay in shared memory for the CTA's
// lifetime, so HBM traffic is one read of y_t and one write of z_t per token.
#pragma once
#include "ptx.cuh"

namespace scb {

struct TransGeom {
  WinGeom win;
  const __half* y;    // Y_t plane (conv1_1's trans half), pixel stride T
  __half* z;          // Z plane, pixel stride 2T, output at column T
  const __half* wqkv; // [3T][T]
  const __half* wproj;// [T][T]
  const __half* w0;   // [4T][T]
  const __half* w2;   // [T][4T]
  const float *bqkv, *bproj, *b0, *b2, *ln1g, *ln1b, *ln2g, *ln2b, *rp;
  // LayerNorm affine maps folded into the following linear (W diag(gamma),
  // b + W beta; the q rows of wqkv_f/bqkv_f also carry 32^-1/2 log2(e)): used by
  // the warp-specialised T = 32 kernel, which stores (x - mu) rstd only
  const __half *wqkv_f, *w0_f;
  const float *bqkv_f, *b0_f;
};

// LayerNorm of N fp32 values (no affine map: the kernels fold it into the next
// weights) as packed fp16 pairs (x - mu) rstd, in fp32x2 arithmetic (half the FP32
// instructions; the same sums and roundings as two scalar accumulators of the even and
// odd elements).
template <int N>
__device__ __forceinline__ void ln_pack_f32x2(const float* x, uint32_t* a) {
  float2 s = make_float2(0.f, 0.f), q = make_float2(0.f, 0.f);
#pragma unroll
  for (int j = 0; j < N; j += 2) {
    const float2 v = make_float2(x[j], x[j + 1]);
    s = __fadd2_rn(s, v);
    q = __ffma2_rn(v, v, q);
  }
  const float mu = (s.x + s.y) * (1.f / N);
  const float rstd = rsqrtf(fmaxf((q.x + q.y) * (1.f / N) - mu * mu, 0.f) + 1e-5f);
  const float2 r2 = make_float2(rstd, rstd), n2 = make_float2(-mu * rstd, -mu * rstd);
#pragma unroll
  for (int j = 0; j < N / 2; ++j) {
    const float2 o = __ffma2_rn(make_float2(x[2 * j], x[2 * j + 1]), r2, n2);
    a[j] = pack_half2(o.x, o.y);
  }
}

// Copy a row-major fp16 [R][K] matrix into K-major swizzled tiles: K split into
// blocks of `kblk` elements (kblk*2 = row bytes = swizzle span), block b at
// dst + b * R * kblk * 2.
__device__ __forceinline__ void stage_kmajor(uint8_t* dst, const __half* src, int R, int K, int kblk) {
  const int rb = kblk * 2, cpr = K / 8, cpb = kblk / 8;
  for (int idx = threadIdx.x; idx < R * cpr; idx += blockDim.x) {
    const int r = idx / cpr, j = idx - r * cpr;
    const int b = j / cpb, jj = j - b * cpb;
    *reinterpret_cast<uint4*>(dst + b * R * rb + swz_off(r, jj, rb)) =
        __ldg(reinterpret_cast<const uint4*>(src + (long)r * K + j * 8));
  }
}

}  // namespace scb
