/*
 * scunet_b200 — B200 (sm_100a) SCUNet forward pass behind a C ABI.
 *
 * This is the device side of the reference's `Backend` trait
 * (scunet-rs src/backend.rs:19-56) for the CUDA backend that `Cuda::new` /
 * `Cuda::forward` (src/cuda.rs:192-241, 1606-1848) implement today. A Rust
 * `impl Backend for B200` (or any other host) binds these symbols; nothing here
 * takes a torch, Rust or C++ type: plain pointers, sizes and status codes.
 *
 * Conventions
 *  - Every function returning int returns 0 on success and a negative SCB_E*
 *    code on failure; the message is then available from scb_last_error().
 *    Nothing here aborts the process (the reference panics on a device OOM,
 *    src/cuda.rs:346-360, and on a missing weight, src/weights.rs:309-314).
 *  - One context owns one device's weights, streams and scratch arena. A context
 *    is used by one host thread at a time (the reference serialises on a mutex,
 *    tests/device_lock.rs:7-14). Independent contexts on different devices run
 *    concurrently (batch sharding: one context per GPU).
 *  - Images are NCHW float32 in [0,1] (or uint8 where stated). The network's
 *    arithmetic is fp16 tensor-core operands with fp32 accumulation; the four
 *    U-Net skips are stored in fp32 and every other intermediate, including by
 *    default the residual stream inside a stage, in fp16 (SCB_OPT_RESIDUAL32 keeps
 *    that stream in fp32, the reference's precision).
 */
#ifndef SCUNET_B200_H
#define SCUNET_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct scb_ctx scb_ctx;

/* One named weight tensor, C-order float32, as `Weights::t(name)` hands it out
 * (src/weights.rs:312-314). Names and shapes: src/weights.rs:207-263. */
typedef struct {
  const char* name;
  const float* data;
  int ndim;
  int64_t shape[4];
} scb_tensor;

enum {
  SCB_OK = 0,
  SCB_EINVAL = -1,    /* bad argument, shape or geometry */
  SCB_ENOWEIGHT = -2, /* a required tensor is missing */
  SCB_ECUDA = -3,     /* CUDA runtime / driver error */
  SCB_ENOMEM = -4,    /* device allocation refused (admission, scb_need_bytes) */
  SCB_EDEVICE = -5    /* a kernel reported a failure through the device error word */
};

enum { SCB_F32 = 0, SCB_U8 = 1 };

/* Validate, repack (fp16 K-major tiles) and upload every weight once.
 * Replaces `Cuda::new(&Weights)` (src/cuda.rs:192-241). `config` is the seven
 * per-stage block counts ([4]*7 for every published checkpoint); dim 64,
 * head_dim 32, window 8 are the only supported values (src/weights.rs:204-280).
 * On failure *out is NULL and the message is in scb_last_error(NULL). */
int scb_create(const scb_tensor* tensors, int n_tensors, int in_nc, int dim, int head_dim, int window,
               const int config[7], int device, scb_ctx** out);

/* `Backend::forward` (src/backend.rs:19-25; src/cuda.rs:1606-1848): x is the
 * already replicate-padded [c][hp][wp] float32 host plane (hp, wp multiples of
 * 64), y receives the same shape. Synchronous. */
int scb_forward(scb_ctx* ctx, const float* x_nchw, int c, int hp, int wp, float* y_nchw);

/* Batched device-pointer forward with the pad and crop fused
 * (`backend::run`, src/backend.rs:63-105, for n images at once): x is
 * [n][c][h][w] (x_dtype SCB_U8 or SCB_F32) and y is [n][c][h][w] (y_dtype
 * SCB_F32, or SCB_U8 quantised as clamp(v,0,1)*255+0.5 truncated,
 * src/image.rs:60-63). Both are device pointers. Asynchronous on `stream`
 * (a cudaStream_t; NULL = the context's own stream). */
int scb_forward_dev(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y, int y_dtype,
                    void* stream);

/* scb_forward_dev for callers that cannot allocate device memory when they call:
 * a server that reserves all device memory at start-up and must not have a
 * request fail or stall on cudaMalloc (which can fail under fragmentation and
 * synchronises the device), or a host whose own allocator owns the GPU's memory.
 * This entry point has no counterpart in the reference. It allocates nothing:
 * its scratch is a 14 MiB array inside the library's device image. scb_create
 * reserves it: it looks the array's device address up (cudaGetSymbolAddress),
 * which loads the library's device code on that GPU together with the array, so
 * a later call here loads and allocates nothing; the GPU then holds the 14 MiB
 * until the process exits (scb_mem_report's `fixed`). Limit: the padded batch
 * (n * ceil(h/64)*64 * ceil(w/64)*64) may hold at most 8192 pixels, e.g. one
 * 64x128 or two 64x64 images; larger requests fail with SCB_EINVAL and a
 * message. Every call, from every context on a device, shares the one array and
 * overwrites it (nothing in it needs to start at zero), so calls whose GPU work
 * overlaps race: run them on one stream or order them with events. Same inputs,
 * outputs and asynchrony as scb_forward_dev; the context's weights must already
 * be on the device (scb_create allocates them). */
int scb_forward_dev_noalloc(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y,
                            int y_dtype, void* stream);

/* Same as scb_forward_dev with host pointers: copies in, runs, copies out,
 * synchronises (the end-to-end call a host application makes). The batch runs as
 * a pipeline of chunks of images (SCB_OPT_HOST_CHUNK images each; by default as
 * many as make up four 1920x1088 frames): while chunk k computes, chunk k + 1 is
 * copied in and chunk k - 1 out on two copy streams, so with pinned host buffers
 * the copies hide behind the compute. */
int scb_forward_host(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y, int y_dtype);

/* ---- one large image split into row bands (an image too large to run whole) ----
 * The padded image's 64-row blocks are divided into contiguous row bands. Each band
 * runs the whole network on its rows, stored with 4 halo rows above and below at
 * every level; after every block's conv1_1 (and before the tail conv) the bands
 * swap their 4 boundary rows, which covers the 3x3 conv pair and the shifted
 * windows that straddle band edges. The shifted-window mask uses the window's row
 * in the whole image, so the image's top and bottom bands need no wrap-around
 * exchange. 2x2 down/up convs never cross a 64-aligned band edge. Output equals
 * scb_forward_dev's on the same image (the same ops on the same pixels). */

/* All `nbands` bands of one image on this context's GPU, run in lockstep with
 * device-to-device halo copies (validates the banded schedule on one GPU).
 * x, y: device [1][c][h][w]. Asynchronous on `stream`. */
int scb_forward_bands(scb_ctx* ctx, int nbands, const void* x, int x_dtype, int c, int h, int w, void* y,
                      int y_dtype, void* stream);

/* Multi-GPU bands, one process and context per GPU: rank 0 creates a 128-byte
 * NCCL unique id, every rank passes it to scb_band_init (collective), then every
 * rank calls scb_forward_band with the FULL image x (device, on its own GPU); it
 * computes its band and writes that band's rows of y (device [1][c][h][w] on its
 * own GPU). Halo rows travel with NCCL send/recv over NVLink on the compute
 * stream. scb_band_init with nranks = 1 runs the whole image as one band.
 * Of x, scb_forward_band reads only the input rows [lo, hi) of its band
 * [R0, R0 + rows): lo = min(max(R0 - 1, 0), h - 1), hi = max(lo + 1, min(R0 + rows
 * + 1, h)) (the head's 3x3 conv reads one row above and below; padded rows at or
 * past h read row h - 1), so a caller holding the image on the host copies only
 * those rows to each rank; the other rows of x may hold anything. */
int scb_band_unique_id(void* id_out);
int scb_band_init(scb_ctx* ctx, const void* id, int rank, int nranks);
int scb_forward_band(scb_ctx* ctx, const void* x, int x_dtype, int c, int h, int w, void* y, int y_dtype,
                     void* stream);

/* Wait for a banded forward on `stream` (NULL = the context's own) with a deadline.
 * NCCL's send/recv kernels wait for the peer without a bound, so a rank whose peer
 * died would otherwise hang in cudaStreamSynchronize. This polls the stream and the
 * band group's asynchronous NCCL error every 0.2 ms; when a peer fails or
 * `timeout_ms` passes it aborts the group (ncclCommAbort, which stops this GPU's
 * NCCL kernels) and returns SCB_ECUDA; the next banded forward then needs a new
 * scb_band_init. No counterpart in the reference (single GPU). */
int scb_band_sync(scb_ctx* ctx, void* stream, int timeout_ms);

/* Device bytes a forward of n images of hp x wp needs beyond the weights
 * (`memguard::device_need`, src/memguard.rs:66-74). Pure arithmetic, for the
 * default options (SCB_OPT_FUSE_TRANS on, SCB_OPT_RESIDUAL32 off); a context whose
 * options differ allocates what its own options need. */
int scb_need_bytes(int n, int in_nc, int hp, int wp, size_t* bytes);

/* `memguard::check_cuda` (src/memguard.rs:262-285) for this context: would a forward
 * of n images of hp x wp (multiples of 64) fit now? *need = the scratch arena this
 * context's options need; *avail = free device memory plus the arena the context
 * holds (the next forward frees or reuses it). SCB_OK when it fits, SCB_ENOMEM with
 * the message when it does not; fails open (SCB_OK, *avail = 0) when free memory
 * cannot be read. The forwards apply the same test before they allocate. */
int scb_check_admission(scb_ctx* ctx, int n, int hp, int wp, size_t* need, size_t* avail);

/* `Backend::footprint` (src/backend.rs:27-31): device bytes held now - the weights,
 * and the scratch arenas scb_release_scratch frees. The fixed no-allocation array
 * is not scratch in that sense (nothing frees it); scb_mem_report gives it. */
void scb_footprint(const scb_ctx* ctx, size_t* weights_bytes, size_t* scratch_bytes);

/* `Backend::mem_report` (src/backend.rs:33-44; `Cuda::mem_report`,
 * src/cuda.rs:395-424) as numbers: the most device memory the context has held at
 * once (weights + scratch arenas; the number that decides whether a size fits),
 * what it holds now, and the fixed 14 MiB no-allocation array its GPU holds since
 * scb_create. Any pointer may be NULL. */
int scb_mem_report(const scb_ctx* ctx, size_t* high_water, size_t* live, size_t* fixed);

/* `Backend::release_scratch` (src/backend.rs:46-55): drop the arena. */
void scb_release_scratch(scb_ctx* ctx);

/* Message of the last failure on ctx (or of the last failed scb_create when ctx
 * is NULL); "" when the last call succeeded. */
const char* scb_last_error(const scb_ctx* ctx);

void scb_destroy(scb_ctx* ctx);

/* ---- single-op probes: the device ops one at a time on caller-owned device
 * buffers, for parity tests (the reference's `op_probe`, `linear_probe`,
 * `attention_kernel_probe` and `block_dump`, src/cuda.rs:1246-1468). All
 * pointers are device pointers; activations are NHWC (pixel-major). ---- */

/* out[m][n] = act(sum_k a[m][k] * b[n][k] + bias[n]) (+ res16[m][n]); fp16 a, b,
 * res16, out16; fp32 bias, out32 (either output may be NULL). act 0/1/2 =
 * none/ReLU/GELU-erf. K, N multiples of 32 / 16. */
int scb_probe_gemm(scb_ctx* ctx, const void* a16, int M, int K, const void* b16, int N, const float* bias, int act,
                   const void* res16, void* out16, float* out32);

/* 3x3 stride-1 zero-pad-1 conv, no bias: x16 [n][H][W][cin] -> [n][H][W][cout];
 * w16 [cout][ky][kx][cin]. act as above; res16 added after act when non-NULL. */
int scb_probe_conv3x3(scb_ctx* ctx, const void* x16, int n, int H, int W, int cin, const void* w16, int cout,
                      int act, const void* res16, void* out16);

/* 2x2 stride-2 conv: x16 [n][H][W][cin] -> out32/out16 [n][H/2][W/2][cout];
 * w16 [cout][dy][dx][cin]. */
int scb_probe_down2(scb_ctx* ctx, const void* x16, int n, int H, int W, int cin, const void* w16, int cout,
                    float* out32, void* out16);

/* 2x2 stride-2 transposed conv: x16 [n][h][w][cin] -> [n][2h][2w][cout];
 * w16 [(dy, dx, cout)][cin]. */
int scb_probe_up2(scb_ctx* ctx, const void* x16, int n, int h, int w, int cin, const void* w16, int cout,
                  float* out32, void* out16);

/* Window attention: qkv16 [n][H][W][3t] (q | k | v column blocks) ->
 * out16 [n][H][W][t]; rp float32 [t/32][15][15]; shift 0 (W) or 4 (SW). */
int scb_probe_attention(scb_ctx* ctx, const void* qkv16, int n, int H, int W, int t, int shift, const float* rp,
                        void* out16);

/* The fused MLP of block (stage, index) of a 1/4 or 1/8 resolution stage (trans
 * width t = 128 or 256): a16 [tokens][t] fp16 (the LN2 output) in; z16 [tokens][t]
 * holds x1 and receives z = x1 + mlp2(GELU(mlp0(a))) (tools/network_scunet.py:128-136). */
int scb_probe_mlp(scb_ctx* ctx, int stage, int index, const void* a16, void* z16, int tokens);

/* One ConvTransBlock with the context's weights: `stage` 0..6 (down1, down2,
 * down3, body, up3, up2, up1), `index` 0..3 within the stage; x32 [n][H][W][c]
 * float32 is read and y32 written (may alias). shift follows the block index
 * (odd = SW), as the reference walker does (src/cuda.rs:1702, 1775, 1811-1817). */
int scb_probe_block(scb_ctx* ctx, int stage, int index, const float* x32, int n, int H, int W, float* y32);

/* m_head alone: x [n][c][h][w] (x_dtype SCB_U8 or SCB_F32, device) -> the replicate-
 * padded 3x3 conv c -> 64 as x1_32 float32 and x1_16 fp16, both [n][hp][wp][64]
 * (NHWC, hp and wp the multiples of 64 above h and w). */
int scb_probe_head(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, float* x1_32, void* x1_16);

/* m_tail alone: s16 fp16 [n][hp][wp][64] -> the 3x3 conv 64 -> c cropped to h x w,
 * y [n][c][h][w] as float32 or uint8 (quantised as scb_forward_dev does). */
int scb_probe_tail(scb_ctx* ctx, const void* s16, int n, int c, int h, int w, void* y, int y_dtype);

/* The failure path of every kernel's bounded waits, on purpose and without a fault:
 * one warp waits up to `limit_us` (1 .. 1e6) on an mbarrier nothing completes, gives
 * up, records the failure in the device error word and returns; this returns
 * SCB_EDEVICE with the message the forwards give, and the context stays usable. */
int scb_probe_wait_timeout(scb_ctx* ctx, int limit_us);

/* Number of kernel launches the last forward issued (for launch accounting). */
int scb_last_launch_count(const scb_ctx* ctx);

/* Execution options. SCB_OPT_FUSE_TRANS (default 1): run the transformer half of
 * the blocks whose trans width is 32 or 64 (full and half resolution) as one fused
 * kernel; 0 runs it as separate qkv / attention / proj / mlp launches (the
 * reference's op sequence, src/cuda.rs:1104-1131). Takes effect at the next forward. */
/* SCB_OPT_RESIDUAL32 (default 0): keep the residual stream inside a stage in fp32
 * (the reference's precision) with an fp16 copy as the next GEMM's operand; 0 keeps
 * it in fp16 only, which is that operand already (the four U-Net skips stay fp32
 * either way). Measured cost of fp16: max |diff| vs the FP32 reference 1.0e-3 ->
 * 1.2e-3 at 256x256, inside the 2e-3 acceptance bar; it saves 6 of the 16 bytes per
 * channel a block moves through its 1x1 convs. */
/* SCB_OPT_HOST_CHUNK (default 0 = automatic): images per compute call of
 * scb_forward_host's pipeline. */
/* SCB_OPT_TRANS32_LANES: the full-resolution transformer half (trans width 32) on the
 * kernel with independent pair lanes (1) or on the warp-specialised one (0). */
/* SCB_OPT_FUSE_PAIR (default 1): at 64 and 128 channels, run each block boundary
 * inside a stage (block i's conv1_2 and block i + 1's conv1_1) as one kernel, so
 * conv1_1 reads the updated residual stream from the chip instead of from HBM; 0 runs
 * them as two GEMM launches (the reference's op sequence). Needs the fp16 residual
 * stream and the fused transformer halves; ignored otherwise. */
/* SCB_OPT_GEMM_PAIRS (default 1): the 1x1 convs and linears whose epilogue has no
 * residual to stream in write their output tile in 64-column rounds (two 32-column
 * slabs per barrier / store round); 0 keeps 32-column rounds. Same results. */
/* SCB_OPT_CONV3_TWIN (default 1): the 128-channel 3x3 convs (1/4 resolution) load each
 * weight stage once for two pixel tiles, halving the weight bytes through shared
 * memory, which bounds them; 0 loads it per tile. Same results. */
enum { SCB_OPT_FUSE_TRANS = 1, SCB_OPT_RESIDUAL32 = 2, SCB_OPT_HOST_CHUNK = 3, SCB_OPT_TRANS32_LANES = 4,
       SCB_OPT_FUSE_PAIR = 5, SCB_OPT_GEMM_PAIRS = 6, SCB_OPT_CONV3_TWIN = 7 };
int scb_set_option(scb_ctx* ctx, int option, int value);

/* Per-launch device timing (the reference's SCUNET_PROFILE, src/cuda.rs:106-135,
 * 263-273): while on, every launch of a forward is bracketed by CUDA events on the
 * launch stream. */
int scb_set_profiling(scb_ctx* ctx, int on);

/* For the last profiled forward: per launch, its op class (0 head, 1 tail,
 * 2 conv1x1, 3 conv3x3, 4 qkv, 5 attention, 6 proj, 7 mlp0, 8 mlp2, 9 down,
 * 10 up, 11 fused transformer half, 12 band halo exchange or edge-halo clear, 13 fused MLP of a
 * separate-launch transformer half), its algorithmic FLOPs and its device time in ms (waits for the
 * events). Returns the number of entries written (<= max). */
int scb_profile_read(scb_ctx* ctx, int* tags, double* flops, float* ms, int max);

/* For the same launches: algorithmic HBM bytes (every operand read once, every
 * result written once, weights included), the numerator of a memory roofline. No
 * counterpart in the reference, whose profile reports times only. */
int scb_profile_bytes(const scb_ctx* ctx, double* bytes, int max);

/* For the same launches: the kernel each one ran, as profilers name it (e.g.
 * "gemm_tc_kernel<64, 64, 0, 1>"), one per line, so a per-kernel profiler capture
 * can be matched to the op list. Writes at most cap - 1 bytes and a NUL (buf may be
 * NULL to size it); returns the full length. */
int scb_profile_kernels(const scb_ctx* ctx, char* buf, size_t cap);

/* `Backend::profile_report` (src/backend.rs:33-38; `Cuda::profile_report`,
 * src/cuda.rs:1875-1886): the last profiled forward's device time per op class,
 * most expensive first, as text (one line per class: ms, share, launches, achieved
 * TFLOP/s, class). Writes at most cap - 1 bytes and a NUL into buf (buf may be NULL
 * to size it); returns the full length. Empty when profiling is off. */
int scb_profile_report(scb_ctx* ctx, char* buf, size_t cap);

#ifdef __cplusplus
}
#endif

#endif /* SCUNET_B200_H */
