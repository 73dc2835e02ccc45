// Host launchers for the reference's own CUDA kernels (scunet-rs cuda/scunet.cu),
// compiled from that file where it lies (oracle/Makefile) into oracle/_ref/.
//
// TEST INFRASTRUCTURE ONLY. The reference's window attention kernel is a second
// oracle and the timing comparison arm for window_attn_kernel: only tests/ and the
// attention comparison in bench.py load the library this file builds. Nothing in the
// product (include/scunet_b200.h) calls it.
#include <cuda_runtime.h>

#include "scunet.cu"  // the reference's kernels, found through -I <reference>/cuda

extern "C" {

// sc_window_attn_r64 with the launch the reference's walker uses for 8x8 windows and
// 32-wide heads (src/cuda.rs:795-800): one block of 2n threads per (window, head),
// k, v and the cross-thread exchange in 3 n hd floats of shared memory.
// qkv [nw*64][3c] float32, tokens in window order (q | k | v column blocks);
// rp [heads][15][15]; out [nw*64][c]; w0 = global index of window 0 (SW mask).
int ref_window_attn_r64(const float* qkv, const float* rp, float* out, int nw, int nww, int hp, int wp,
                        int heads, int shift, int w0, void* stream) {
  const int n = 64, win = 8, hd = 32;
  if (nw <= 0 || heads <= 0 || heads > SC_MAX_HEADS || nww <= 0 || hp % win || wp % win) return 1;
  sc_window_attn_r64<<<dim3(nw, heads), 2 * n, 3 * n * hd * sizeof(float), static_cast<cudaStream_t>(stream)>>>(
      qkv, rp, out, nw, n, nww, win, hp, wp, heads, hd, shift, w0);
  return (int)cudaGetLastError();
}

}  // extern "C"
