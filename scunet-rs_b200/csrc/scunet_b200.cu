// scunet_b200: the C-ABI (include/scunet_b200.h), weight repack, the per-geometry
// arena and op plan, and the U-Net walker that replaces `Cuda::forward`
// (scunet-rs src/cuda.rs:1606-1848) with the same stage order:
//
//   x1 = head(pad(x))                                   (tools/network_scunet.py:247)
//   x2 = down1(x1), x3 = down2(x2), x4 = down3(x3)      4 blocks + 2x2 s2 conv each
//   b  = body(x4)                                       4 blocks
//   y  = up3(b + x4), up2(y + x3), up1(y + x2)          2x2 transposed conv + 4 blocks
//   out = crop(tail(y + x1))
//
// Activations live in HBM as NHWC: the residual stream and the four U-Net skips in
// fp32, every other intermediate in fp16 (it is only ever a tensor-core operand).
// Each GEMM epilogue that produces the residual stream also writes its fp16
// "shadow" - the A operand of the next GEMM - and the last block of body/up3/up2/
// up1 writes the shadow of (x + skip) directly, which is the skip add that
// upstream performs before each up conv and before the tail.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>  // types only: the functions are resolved with dlopen at run time

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <ctime>
#include <map>
#include <string>
#include <vector>

#include "../../include/scunet_b200.h"
#include "attn.cuh"
#include "host_logic.h"
#include "gemm.cuh"
#include "io_kernels.cuh"
#include "trans.cuh"
#include "trans32ws.cuh"
#include "trans32mp.cuh"
#include "trans64ws.cuh"
#include "mlp.cuh"
#include "convpair.cuh"

using namespace scb;

// Scratch for scb_forward_dev_noalloc, for callers that cannot allocate device
// memory at call time. It is a fixed array in the library's device image: the
// device code is loaded (and these 14 MiB reserved) on a GPU when scb_create looks
// the array up, and the GPU holds it until the process exits. Its size covers the
// scratch plan of any batch whose padded pixels (n * hp * wp) total at most
// kNoAllocMaxPixels (1704 bytes per padded pixel plus 1 KiB alignment per buffer).
// Host code only ever takes its address with cudaGetSymbolAddress.
static constexpr long kNoAllocMaxPixels = 8192;
static constexpr size_t kNoAllocBytes = 14u << 20;
// scb_forward_host: padded pixels per compute call when SCB_OPT_HOST_CHUNK is 0
// (four 1920x1088 frames).
static constexpr long kHostChunkPixels = 4L * 1088 * 1920;
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocBytes];

namespace {

thread_local std::string g_create_error;

// --------------------------------------------------------------------------
// Tensor maps (driver entry point fetched through the runtime, so the library
// links no libcuda and loads on a machine without a driver).
// --------------------------------------------------------------------------
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn(std::string& err) {
  static EncodeTiledFn fn = nullptr;
  if (fn) return fn;
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || !p) {
    err = "cuTensorMapEncodeTiled is not available from the driver";
    return nullptr;
  }
  fn = reinterpret_cast<EncodeTiledFn>(p);
  return fn;
}

// Encode a tiled tensor map. es = element bytes (2: fp16, 4: fp32); swizzle_bytes
// = 128, 64 or 0 and must equal box[0] * es when non-zero.
bool encode_map(CUtensorMap* m, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                const uint32_t* box, int es, int swizzle_bytes, std::string& err) {
  EncodeTiledFn fn = encode_fn(err);
  if (!fn) return false;
  cuuint64_t d[5], s[4];
  cuuint32_t b[5], el[5];
  for (int i = 0; i < rank; ++i) {
    d[i] = dims[i];
    b[i] = box[i];
    el[i] = 1;
    if (i < rank - 1) s[i] = strides[i];
  }
  const CUtensorMapSwizzle swz = swizzle_bytes == 128  ? CU_TENSOR_MAP_SWIZZLE_128B
                                 : swizzle_bytes == 64 ? CU_TENSOR_MAP_SWIZZLE_64B
                                                       : CU_TENSOR_MAP_SWIZZLE_NONE;
  CUresult r = fn(m, es == 2 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT32, rank,
                  const_cast<void*>(base), d, s, b, el, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    char buf[256];
    snprintf(buf, sizeof buf, "cuTensorMapEncodeTiled failed (%d), rank %d, dims %llu x %llu", (int)r, rank,
             (unsigned long long)dims[0], (unsigned long long)dims[1]);
    err = buf;
    return false;
  }
  return true;
}

// --------------------------------------------------------------------------
// GEMM op: tiles, maps, dispatch over the compiled (BN, BK, GEO, epilogue) variants
// --------------------------------------------------------------------------
constexpr int kSmemPerSm = 227 * 1024;

struct GemmOp {
  int geo = GEO_FLAT, bn = 64, bk = 64;
  bool tma_epi = false;
  bool pairs = false;  // TMA epilogue in 64-column rounds (flat GEMMs without residual slabs)
  bool twin = false;   // 3x3 conv (GEO_CONV3X): two pixel tiles per pipeline stage share its B
  CUtensorMap ta, tb;
  GemmGeom g{};
  GemmEpi e{};
  EpiMaps em;
};

// Pipeline depth and CTAs per SM for one op: GEMMs whose two accumulators fit in
// half of TMEM (BN <= 128) try for two CTAs per SM (more epilogue warps in
// flight); stages fill what shared memory is left after the epilogue staging and,
// when B is resident (`bres_bytes` > 0), after the whole of B.
void plan_launch(int bn, int a_bytes, int b_bytes, int staging_bytes, int bres_bytes, int max_ctas, int& stages,
                 int& ctas, int& smem) {
  const int stage_bytes = bres_bytes ? a_bytes : a_bytes + b_bytes;
  ctas = std::min(bn <= 128 ? 2 : 1, max_ctas);  // max_ctas: what the kernel's TMEM columns allow
  for (;;) {
    const int budget = kSmemPerSm / ctas - 1024 /*reserved*/ - 1024 /*align*/ - 1024 /*barriers*/ - staging_bytes -
                       bres_bytes;
    stages = std::min(8, budget / stage_bytes);
    if (stages >= 2 || ctas == 1) break;
    ctas = 1;
  }
  stages = std::max(stages, 2);
  smem = stages * stage_bytes + bres_bytes + 1024 + staging_bytes + 1024;
}

// B stays resident in shared memory when the op has one N tile and all of its k
// blocks take at most this much (the 3x3 convs and 1x1 convs of the wide levels).
constexpr int kMaxResidentB = 40 * 1024;

// Residual slab buffers of the TMA epilogue. Four (three slabs of lookahead) were
// measured slower than two: the extra staging costs the 1x1 convs pipeline stages.
// The 3x3 convs measured the same with two to six.
constexpr int kResBufs = 2;

// An fp16 residual of a flat GEMM or 3x3 conv (TMA epilogue, no activation) is added on
// the tensor cores as extra k blocks against an identity B, not in the epilogue.
#ifndef SCB_RESIDUAL_MMA
#define SCB_RESIDUAL_MMA 1
#endif
constexpr bool kResidualMma = SCB_RESIDUAL_MMA != 0;

template <int BN, int BK, int GEO, bool TMAEPI, bool PAIRS = false>
cudaError_t launch_t(const GemmOp& op, int sms, cudaStream_t st) {
  using L = GemmSmem<BN, BK, GEO>;
  auto kfn = gemm_tc_kernel<BN, BK, GEO, TMAEPI, PAIRS>;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kfn, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemPerSm);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  GemmEpi e = op.e;
  e.res_bufs = e.st_res_bytes ? kResBufs : 2;
  const int staging = TMAEPI ? e.st_ident_bytes + e.res_bufs * e.st_res_bytes + 2 * e.st_out_bytes : 0;
  GemmGeom g = op.g;
  const int bres_bytes = g.num_kb * L::B_BYTES;
  g.b_res = g.n_tiles == 1 && bres_bytes <= kMaxResidentB;
  g.twin = op.twin && GEO == GEO_CONV3X && BN == 128 && g.n_tiles == 1 && !g.b_res;
  int stages, ctas, smem;
  // twin tiles: each stage holds two A boxes and one B
  plan_launch(BN, g.twin ? 2 * L::A_BYTES : L::A_BYTES, L::B_BYTES, staging, g.b_res ? bres_bytes : 0,
              512 / L::TMEM_COLS, stages, ctas, smem);
  g.stages = stages;
  const int tiles = g.m_tiles * g.n_tiles;
  const int grid = std::max(1, std::min(tiles, sms * ctas));
  kfn<<<grid, 192, smem, st>>>(op.ta, op.tb, g, e, op.em);
  return cudaGetLastError();
}

#define SCB_GEMM_CASE(BN, BK, GEO)                                                     \
  if (op.bn == BN && op.bk == BK && op.geo == GEO && !op.tma_epi)                      \
    return launch_t<BN, BK, GEO, false>(op, sms, st);
#define SCB_GEMM_TCASE(BN, BK, GEO)                                                    \
  if (op.bn == BN && op.bk == BK && op.geo == GEO && op.tma_epi && !op.pairs)          \
    return launch_t<BN, BK, GEO, true>(op, sms, st);
#define SCB_GEMM_PCASE(BN, BK, GEO)                                                    \
  if (op.bn == BN && op.bk == BK && op.geo == GEO && op.tma_epi && op.pairs)           \
    return launch_t<BN, BK, GEO, true, true>(op, sms, st);

// Every compiled GEMM variant: T = with the TMA epilogue, D = direct epilogue, P = TMA
// epilogue in paired slabs (flat GEMMs whose tile is a multiple of 64 columns).
#define SCB_GEMM_VARIANTS(T, D, P)                                                                           \
  P(64, 64, GEO_FLAT) P(128, 64, GEO_FLAT) P(192, 64, GEO_FLAT) P(256, 64, GEO_FLAT) P(128, 32, GEO_FLAT)   \
  T(64, 64, GEO_FLAT) T(128, 64, GEO_FLAT) T(192, 64, GEO_FLAT) T(256, 64, GEO_FLAT) T(128, 32, GEO_FLAT)   \
  T(32, 32, GEO_CONV3X) T(32, 32, GEO_CONV3W) T(64, 64, GEO_CONV3X) T(128, 64, GEO_CONV3X)                  \
  T(256, 64, GEO_CONV3) T(128, 64, GEO_DOWN2) T(256, 64, GEO_DOWN2) T(64, 64, GEO_UP2) T(128, 64, GEO_UP2)  \
  T(256, 64, GEO_UP2)                                                                                       \
  D(32, 32, GEO_FLAT) D(32, 64, GEO_FLAT) D(64, 64, GEO_FLAT) D(96, 32, GEO_FLAT) D(128, 32, GEO_FLAT)      \
  D(128, 64, GEO_FLAT) D(192, 64, GEO_FLAT) D(256, 64, GEO_FLAT) D(64, 64, GEO_UP2) D(128, 64, GEO_UP2)     \
  D(256, 64, GEO_UP2) D(32, 32, GEO_CONV3) D(64, 64, GEO_CONV3) D(128, 64, GEO_CONV3) D(256, 64, GEO_CONV3) \
  D(128, 64, GEO_DOWN2) D(256, 64, GEO_DOWN2)

cudaError_t launch_gemm(const GemmOp& op, int sms, cudaStream_t st) {
  SCB_GEMM_VARIANTS(SCB_GEMM_TCASE, SCB_GEMM_CASE, SCB_GEMM_PCASE)
  return cudaErrorInvalidConfiguration;
}

bool tma_epi_supported(int geo, int bn, int bk) {
  static const int tab[][3] = {{64, 64, GEO_FLAT},   {128, 64, GEO_FLAT},  {192, 64, GEO_FLAT},  {256, 64, GEO_FLAT},
                               {128, 32, GEO_FLAT},  {32, 32, GEO_CONV3X}, {32, 32, GEO_CONV3W}, {64, 64, GEO_CONV3X}, {128, 64, GEO_CONV3X}, {256, 64, GEO_CONV3},
                               {128, 64, GEO_DOWN2}, {256, 64, GEO_DOWN2}, {64, 64, GEO_UP2},    {128, 64, GEO_UP2},
                               {256, 64, GEO_UP2}};
  for (auto& r : tab)
    if (r[0] == bn && r[1] == bk && r[2] == geo) return true;
  return false;
}

bool gemm_supported(int geo, int bn, int bk) {
  static const int tab[][3] = {{32, 32, GEO_FLAT},   {32, 64, GEO_FLAT},   {64, 64, GEO_FLAT},   {96, 32, GEO_FLAT},
                               {128, 32, GEO_FLAT},  {128, 64, GEO_FLAT},  {192, 64, GEO_FLAT},  {256, 64, GEO_FLAT},
                               {64, 64, GEO_UP2},    {128, 64, GEO_UP2},   {256, 64, GEO_UP2},   {32, 32, GEO_CONV3},
                               {64, 64, GEO_CONV3},  {128, 64, GEO_CONV3}, {256, 64, GEO_CONV3}, {128, 64, GEO_DOWN2},
                               {256, 64, GEO_DOWN2}};
  for (auto& r : tab)
    if (r[0] == bn && r[1] == bk && r[2] == geo) return true;
  return false;
}

// Tile width of a 1x1 (flat) GEMM: at most 128 columns, so that the tile's two TMEM
// accumulators (2 BN columns) leave room for a second CTA on the SM: these GEMMs are
// memory-bound with short K, and one CTA per SM leaves only four epilogue warps to
// drain the accumulators. `min_bn` widens it where a LayerNorm epilogue needs its
// whole row range inside one tile.
int pick_bn_flat(int N, int min_bn) {
  int bn = (N == 32 || N == 64 || N == 96 || N == 128) ? N : (N % 128 == 0) ? 128 : (N % 64 == 0) ? 64 : 32;
  while (bn < min_bn && N % (2 * bn) == 0 && 2 * bn <= 256) bn *= 2;
  return bn;
}

int pick_bn(int N) {
  if (N <= 256 && (N == 32 || N == 64 || N == 96 || N == 128 || N == 192 || N == 256)) return N;
  if (N % 256 == 0) return 256;
  if (N % 192 == 0) return 192;
  if (N % 128 == 0) return 128;
  if (N % 64 == 0) return 64;
  return 32;
}

// Output-block tile for the spatial GEMMs: TW x TH = 128 pixels, TW the widest
// power of two <= 128 that divides W (16 with edge masking otherwise).
void pick_tile(int W, int& TW, int& TH) {
  TW = 16;
  for (int c : {128, 64, 32, 16})
    if (W % c == 0) {
      TW = c;
      break;
    }
  TH = 128 / TW;
}

struct Maker {
  std::string* err;
  bool pairs_enabled = true;  // SCB_OPT_GEMM_PAIRS
  bool twin_enabled = true;   // SCB_OPT_CONV3_TWIN
  bool ok = true;

  bool mapB(GemmOp& op, const __half* w, int N, int K) {
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)N};
    const uint64_t str[1] = {(uint64_t)K * 2};
    const uint32_t box[2] = {(uint32_t)op.bk, (uint32_t)op.bn};
    return encode_map(&op.tb, w, 2, dims, str, box, 2, op.bk * 2, *err);
  }

  // Plain GEMM over M rows of an fp16 [M][lda] matrix (first K columns).
  // `bk32`: 32-wide K blocks where the tile is 128 columns wide (half the
  // pipeline-stage bytes, for epilogues whose staging leaves little shared memory).
  bool flat(GemmOp& op, const __half* a, long M, int K, long lda, const __half* w, int N, int geo = GEO_FLAT,
            int min_bn = 0, bool bk32 = false) {
    op.geo = geo;
    op.bn = geo == GEO_UP2 ? std::min(pick_bn(N), op.g.up_cout) : pick_bn_flat(N, min_bn);
    op.bk = (K % 64 == 0 && !(bk32 && op.bn == 128)) ? 64 : 32;
    if (!gemm_supported(op.geo, op.bn, op.bk) || K % 32 || N % op.bn) {
      *err = "no GEMM variant for N=" + std::to_string(N) + " K=" + std::to_string(K);
      return false;
    }
    const uint64_t dims[2] = {(uint64_t)K, (uint64_t)M};
    const uint64_t str[1] = {(uint64_t)lda * 2};
    const uint32_t box[2] = {(uint32_t)op.bk, 128};
    if (!encode_map(&op.ta, a, 2, dims, str, box, 2, op.bk * 2, *err)) return false;
    if (!mapB(op, w, N, K)) return false;
    op.g.M = (int)M;
    op.g.n_total = N;
    op.g.num_kb = K / op.bk;
    op.g.kb_per_tap = op.g.num_kb;
    op.g.m_tiles = (int)((M + 127) / 128);
    op.g.n_tiles = N / op.bn;
    return true;
  }

  // 3x3 implicit GEMM over n images of H x W, input channels [0, cin) of an fp16
  // NHWC buffer whose pixel stride is pix_ld elements.
  // `kx_boxes`: use a schedule with fewer, larger input boxes: GEO_CONV3W (16 x 8
  // tiles, one box per channel chunk) where compiled, else GEO_CONV3X (8 x 16
  // tiles, one box per column shift); both only with the TMA epilogue.
  // Output rows [row0, row0 + rows_out) of each image's H stored rows (default:
  // all of them); rows outside are read as input (halo) but never written.
  bool conv3(GemmOp& op, const __half* x, int n, int H, int W, int cin, long pix_ld, const __half* w, int cout,
             bool kx_boxes = true, int row0 = 0, int rows_out = -1) {
    if (rows_out < 0) rows_out = H - row0;
    op.bk = (cin % 64 == 0) ? 64 : 32;
    op.bn = cout;
    op.geo = !kx_boxes                                                 ? GEO_CONV3
             : tma_epi_supported(GEO_CONV3W, op.bn, op.bk)              ? GEO_CONV3W
             : tma_epi_supported(GEO_CONV3X, op.bn, op.bk)              ? GEO_CONV3X
                                                                         : GEO_CONV3;
    if ((op.geo == GEO_CONV3 && !gemm_supported(op.geo, op.bn, op.bk)) || cin % 32) {
      *err = "no conv3x3 variant for cin=" + std::to_string(cin) + " cout=" + std::to_string(cout);
      return false;
    }
    int TW, TH;
    if (op.geo == GEO_CONV3X) {
      TW = 16;
      TH = 8;
    } else if (op.geo == GEO_CONV3W) {
      TW = kConv3wTW;
      TH = kConv3wTH;
    } else {
      pick_tile(W, TW, TH);
    }
    const int box_rows = op.geo == GEO_CONV3X ? TH + 2 : op.geo == GEO_CONV3W ? kConv3wBoxRows : TH;
    const int box_cols = op.geo == GEO_CONV3W ? TW + 2 : TW;
    const uint64_t dims[4] = {(uint64_t)cin, (uint64_t)W, (uint64_t)H, (uint64_t)n};
    const uint64_t str[3] = {(uint64_t)pix_ld * 2, (uint64_t)W * pix_ld * 2, (uint64_t)H * W * pix_ld * 2};
    const uint32_t box[4] = {(uint32_t)op.bk, (uint32_t)box_cols, (uint32_t)box_rows, 1};
    if (!encode_map(&op.ta, x, 4, dims, str, box, 2, op.bk * 2, *err)) return false;
    if (!mapB(op, w, cout, 9 * cin)) return false;
    op.g.M = n * H * W;
    op.g.n_total = cout;
    op.g.kb_per_tap = cin / op.bk;
    op.g.num_kb = op.geo == GEO_CONV3X ? 3 * op.g.kb_per_tap
                  : op.geo == GEO_CONV3W ? op.g.kb_per_tap
                                         : 9 * op.g.kb_per_tap;
    op.g.row0 = row0;
    op.g.rows_out = rows_out;
    op.g.H = H;
    op.g.W = W;
    op.g.TH = TH;
    op.g.TW = TW;
    op.g.tiles_x = (W + TW - 1) / TW;
    op.g.tiles_y = (rows_out + TH - 1) / TH;
    op.g.m_tiles = n * op.g.tiles_y * op.g.tiles_x;
    op.g.n_tiles = 1;
    op.twin = op.geo == GEO_CONV3X && op.bn == 128 && twin_enabled;
    return true;
  }

  // 2x2 stride-2 conv of an fp16 NHWC [n*H][W][cin] plane (contiguous).
  bool down2(GemmOp& op, const __half* x, int n, int H, int W, int cin, const __half* w, int cout) {
    op.geo = GEO_DOWN2;
    op.bk = 64;
    op.bn = pick_bn(cout);
    if (!gemm_supported(op.geo, op.bn, op.bk) || cin % 64) {
      *err = "no down-conv variant for cin=" + std::to_string(cin);
      return false;
    }
    const int Ho = H / 2, Wo = W / 2, rows = n * Ho;
    int TW, TH;
    pick_tile(Wo, TW, TH);
    const uint64_t dims[5] = {(uint64_t)cin, 2, (uint64_t)Wo, 2, (uint64_t)rows};
    const uint64_t str[4] = {(uint64_t)cin * 2, (uint64_t)cin * 4, (uint64_t)W * cin * 2, (uint64_t)W * cin * 4};
    const uint32_t box[5] = {(uint32_t)op.bk, 1, (uint32_t)TW, 1, (uint32_t)TH};
    if (!encode_map(&op.ta, x, 5, dims, str, box, 2, op.bk * 2, *err)) return false;
    if (!mapB(op, w, cout, 4 * cin)) return false;
    op.g.M = rows * Wo;
    op.g.n_total = cout;
    op.g.kb_per_tap = cin / op.bk;
    op.g.num_kb = 4 * op.g.kb_per_tap;
    op.g.H = rows;
    op.g.W = Wo;
    op.g.TH = TH;
    op.g.TW = TW;
    op.g.tiles_x = (Wo + TW - 1) / TW;
    op.g.tiles_y = (rows + TH - 1) / TH;
    op.g.m_tiles = op.g.tiles_y * op.g.tiles_x;
    op.g.n_tiles = cout / op.bn;
    return true;
  }

  // One epilogue stream's map: `cols` columns starting at `base` (element stride
  // `ld` between pixels), boxed as 32 columns x the M tile's pixel block.
  bool stream_map(const GemmOp& op, CUtensorMap* m, const void* base, long ld, int cols, int es) {
    const uint32_t sw = 32 * es;
    const GemmGeom& g = op.g;
    if (op.geo == GEO_FLAT) {
      const uint64_t dims[2] = {(uint64_t)cols, (uint64_t)g.M};
      const uint64_t str[1] = {(uint64_t)ld * es};
      const uint32_t box[2] = {32, 128};
      return encode_map(m, base, 2, dims, str, box, es, sw, *err);
    } else if (is_conv3(op.geo)) {
      // rows past the op's output range are clipped on store and read as zero
      const uint64_t n = (uint64_t)g.M / ((uint64_t)g.H * g.W);
      const uint64_t dims[4] = {(uint64_t)cols, (uint64_t)g.W, (uint64_t)(g.row0 + g.rows_out), n};
      const uint64_t str[3] = {(uint64_t)ld * es, (uint64_t)g.W * ld * es, (uint64_t)g.H * g.W * ld * es};
      const uint32_t box[4] = {32, (uint32_t)g.TW, (uint32_t)g.TH, 1};
      return encode_map(m, base, 4, dims, str, box, es, sw, *err);
    } else if (op.geo == GEO_UP2) {
      // output pixel (2R + dy, 2x + dx) of input pixel (R, x) as (channel, dx, x, dy, R)
      const uint64_t cw = (uint64_t)ld * es;
      const uint64_t dims[5] = {(uint64_t)g.up_cout, 2, (uint64_t)g.W, 2, (uint64_t)g.H};
      const uint64_t str[4] = {cw, 2 * cw, 2 * (uint64_t)g.W * cw, 4 * (uint64_t)g.W * cw};
      const uint32_t box[5] = {32, 1, (uint32_t)g.TW, 1, (uint32_t)g.TH};
      (void)cols;
      return encode_map(m, base, 5, dims, str, box, es, sw, *err);
    } else {  // GEO_DOWN2
      const uint64_t dims[3] = {(uint64_t)cols, (uint64_t)g.W, (uint64_t)g.H};
      const uint64_t str[2] = {(uint64_t)ld * es, (uint64_t)g.W * ld * es};
      const uint32_t box[3] = {32, (uint32_t)g.TW, (uint32_t)g.TH};
      return encode_map(m, base, 3, dims, str, box, es, sw, *err);
    }
  }

  // After the epilogue pointers are set: pick the TMA epilogue when this op can use
  // it (a LayerNorm only on a flat GEMM, an up conv only with its 2-D tiles, a
  // compiled variant) and build its stream maps and staging layout.
  bool finish_epi(GemmOp& op) {
    GemmEpi& e = op.e;
    e.st_res16 = e.st_res32 = e.st_skip = e.st_out16 = e.st_out32 = e.st_ln = -1;
    e.st_res_bytes = e.st_out_bytes = e.st_ident_bytes = 0;
    op.g.res_kb = 0;
    op.tma_epi = false;
    if (e.out16b && (e.out16_split % 32 || e.out16_split <= 0 || e.out16_split >= op.g.n_total)) {
      *err = "a split fp16 output must split at a multiple of 32 columns";
      return false;
    }
    if (e.ln_out && (e.ln_lo % op.bn) + e.ln_n > op.bn) {
      *err = "LayerNorm columns [" + std::to_string(e.ln_lo) + ", +" + std::to_string(e.ln_n) + ") span two " +
             std::to_string(op.bn) + "-column tiles";
      return false;
    }
    // the TMA epilogue's LayerNorm: flat GEMMs without activation, fp16 residual at most
    const bool ln_tma = !e.ln_out || (op.geo == GEO_FLAT && e.act == ACT_NONE && !e.res32 && !e.skip32);
    if (!ln_tma || (op.geo == GEO_UP2 && op.g.TW == 0) || !tma_epi_supported(op.geo, op.bn, op.bk))
      return true;
    const int N = op.g.n_total;
    int off = 0;
    if (e.res16 && kResidualMma && (is_conv3(op.geo) || op.geo == GEO_FLAT) && !e.res32 && !e.skip32 &&
        e.act == ACT_NONE) {
      // the residual as extra k blocks on the tensor cores (A = its pixels, B = I);
      // not under an activation, which the epilogue applies before the residual
      const GemmGeom& g = op.g;
      const uint32_t sw = op.bk * 2;
      if (op.geo == GEO_FLAT) {
        const uint64_t dims[2] = {(uint64_t)N, (uint64_t)g.M};
        const uint64_t str[1] = {(uint64_t)e.res16_ld * 2};
        const uint32_t box[2] = {(uint32_t)op.bk, 128};
        if (!encode_map(&op.em.resA, e.res16, 2, dims, str, box, 2, sw, *err)) return false;
      } else {
        const uint64_t n = (uint64_t)g.M / ((uint64_t)g.H * g.W);
        const uint64_t dims[4] = {(uint64_t)N, (uint64_t)g.W, (uint64_t)(g.row0 + g.rows_out), n};
        const uint64_t str[3] = {(uint64_t)e.res16_ld * 2, (uint64_t)g.W * e.res16_ld * 2,
                                 (uint64_t)g.H * g.W * e.res16_ld * 2};
        const uint32_t box[4] = {(uint32_t)op.bk, (uint32_t)g.TW, (uint32_t)g.TH, 1};
        if (!encode_map(&op.em.resA, e.res16, 4, dims, str, box, 2, sw, *err)) return false;
      }
      op.g.res_kb = op.bn / op.bk;
      e.st_ident_bytes = 2048;
    } else if (e.res16) {
      if (!stream_map(op, &op.em.res16, e.res16, e.res16_ld, N, 2)) return false;
      e.st_res16 = off;
      off += 128 * 64;
    }
    if (e.res32) {
      if (!stream_map(op, &op.em.res32, e.res32, e.res32_ld, N, 4)) return false;
      e.st_res32 = off;
      off += 128 * 128;
    }
    if (e.skip32) {
      if (!stream_map(op, &op.em.skip, e.skip32, e.skip_ld, N, 4)) return false;
      e.st_skip = off;
      off += 128 * 128;
    }
    e.st_res_bytes = off;
    off = 0;
    if (e.out32) {
      if (!stream_map(op, &op.em.out32, e.out32, e.out32_ld, N, 4)) return false;
      e.st_out32 = off;
      off += 128 * 128;
    }
    if (e.out16) {
      if (!stream_map(op, &op.em.out16, e.out16, e.out16_ld, e.out16b ? e.out16_split : N, 2)) return false;
      if (e.out16b && !stream_map(op, &op.em.out16b, e.out16b, e.out16b_ld, N - e.out16_split, 2)) return false;
      e.st_out16 = off;
      off += 128 * 64;
    }
    if (e.ln_out) {
      if (!stream_map(op, &op.em.lnout, e.ln_out, e.ln_ld, e.ln_n, 2)) return false;
      e.st_ln = off;
      off += 128 * 64;
    }
    e.st_out_bytes = off;
    op.tma_epi = true;
    op.pairs = op.geo == GEO_FLAT && op.bn % 64 == 0 && e.st_res_bytes == 0 && pairs_enabled;
    return true;
  }

  bool up2(GemmOp& op, const __half* x, int n, int h, int w, int cin, const __half* wt, int cout) {
    op.g.up_w = w;
    op.g.up_cout = cout;
    if (!flat(op, x, (long)n * h * w, cin, cin, wt, 4 * cout, GEO_UP2)) return false;
    if (tma_epi_supported(GEO_UP2, op.bn, op.bk)) {
      // TW x TH tiles of input pixels over the stacked rows, for the TMA epilogue
      int TW, TH;
      pick_tile(w, TW, TH);
      const int rows = n * h;
      const uint64_t dims[3] = {(uint64_t)cin, (uint64_t)w, (uint64_t)rows};
      const uint64_t str[2] = {(uint64_t)cin * 2, (uint64_t)w * cin * 2};
      const uint32_t box[3] = {(uint32_t)op.bk, (uint32_t)TW, (uint32_t)TH};
      if (!encode_map(&op.ta, x, 3, dims, str, box, 2, op.bk * 2, *err)) return false;
      op.g.W = w;
      op.g.H = rows;
      op.g.TW = TW;
      op.g.TH = TH;
      op.g.tiles_x = (w + TW - 1) / TW;
      op.g.tiles_y = (rows + TH - 1) / TH;
      op.g.m_tiles = op.g.tiles_x * op.g.tiles_y;
    }
    return true;
  }
};

// --------------------------------------------------------------------------
// Weights on the device
// --------------------------------------------------------------------------
struct BlockW {
  int c = 0;
  __half *w11, *w12, *wc0, *wc2, *wqkv, *wproj, *w0, *w2;
  float *b11, *b12, *bqkv, *bproj, *b0, *b2, *ln1g, *ln1b, *ln2g, *ln2b, *rp;
  // LayerNorm-folded copies for the fused transformer kernels (null where t > 64)
  __half *wqkv_f = nullptr, *w0_f = nullptr;
  float *bqkv_f = nullptr, *b0_f = nullptr;
};

const char* kStageName[7] = {"down1", "down2", "down3", "body", "up3", "up2", "up1"};
const int kStageLevel[7] = {0, 1, 2, 3, 2, 1, 0};

// Op classes for profiling (scb_profile_read): the reference's per-op budget
// classes (docs/TECH_NOTES.md:346-367).
enum OpTag : int {
  TAG_HEAD = 0, TAG_TAIL = 1, TAG_CONV1X1 = 2, TAG_CONV3X3 = 3, TAG_QKV = 4, TAG_ATTN = 5, TAG_PROJ = 6,
  TAG_MLP0 = 7, TAG_MLP2 = 8, TAG_DOWN = 9, TAG_UP = 10, TAG_TRANS = 11, TAG_HALO = 12, TAG_MLP = 13
};

struct Op {
  enum Kind { GEMM, ATTN, HEAD, TAIL, TRANS, XCHG, ZERO, MLP, PAIR } kind;
  // XCHG (row bands): swap kHalo boundary rows of a stored plane with the
  // neighbouring bands; xchg_base is the plane, xchg_row the bytes of one row
  char* xchg_base = nullptr;
  size_t xchg_row = 0;
  int xchg_row0 = 0, xchg_rows = 0;  // the band's working rows in the plane
  // ZERO: clear zero_bytes at zero_ptr (an edge band's halo rows, which the conv's
  // zero padding reads)
  char* zero_ptr = nullptr;
  size_t zero_bytes = 0;
  TransGeom trans{};
  int trans_t = 0;
  bool trans_lanes = false;  // t = 32: the independent-lane kernel instead of the warp-specialised one
  int tag = 0;
  double flops = 0;  // algorithmic FLOPs of this launch (2 per multiply-add)
  GemmOp gemm;
  AttnGeom attn{};
  const __half* attn_in = nullptr;
  __half* attn_out = nullptr;
  const float* attn_rp = nullptr;
  // MLP: the fused mlp0 + GELU + mlp2 of a t = 128 / 256 transformer half
  int mlp_t = 0;
  MlpGeom mlp{};
  CUtensorMap mlp_a, mlp_w0, mlp_w2;
  // HEAD: the x1 (f32) and shadow (fp16) planes as TMA store maps
  CUtensorMap head_m32, head_m16;
  // TAIL: the (y + x1) shadow as a TMA load map (one 128-pixel row segment per box)
  CUtensorMap tail_map;
  TailGeom tail{};
  // PAIR: conv1_2 of a block and conv1_1 of the next in one kernel (convpair.cuh): Z
  // and the residual plane as [64 x 128] SW128 boxes, the two Y planes as [32 x 128]
  // SW64 store boxes
  int pair_c = 0;
  CUtensorMap pair_mz, pair_mx, pair_myc, pair_myt;
  const __half *pair_w12 = nullptr, *pair_w11 = nullptr;
  PairGeom pair{};
};

// A row band of one image (config 5): full-resolution rows [R0, R0 + rows) of the
// padded image, stored with kHalo extra rows above and below at every level.
constexpr int kHalo = 4;

struct Band {
  int rank = 0, nranks = 1;
  int R0 = 0, rows = 0;      // full-resolution band rows
  bool top = true, bottom = true;  // the band touches the image top / bottom
};

struct Arena {
  int n = 0, hp = 0, wp = 0;
  bool banded = false;
  Band band;
  char* base = nullptr;
  size_t bytes = 0;
  float* skip[4] = {};
  __half* xs[4] = {};
  float* xw = nullptr;
  __half *y = nullptr, *yt = nullptr;  // conv1_1 output: conv half, trans half (two planes)
  __half *hc = nullptr, *z = nullptr, *a = nullptr, *o = nullptr, *qh = nullptr;
  std::vector<Op> ops;     // head .. tail
};

// Stored pixels of the level-l plane: the whole image, or a band with its halo rows.
size_t plane_px(int n, int hp, int wp, const Band* band, int l) {
  if (band) return (size_t)((band->rows >> l) + 2 * kHalo) * (size_t)(wp >> l);
  return (size_t)n * (hp >> l) * (wp >> l);
}

// What the plan needs besides the geometry: the fp32 residual plane only with
// SCB_OPT_RESIDUAL32, the separate-launch transformer buffers (LN output, attention
// output, qkv / MLP hidden) only at the levels that do not run a fused kernel.
struct ArenaOpts {
  bool residual32 = false;
  bool fuse_trans = true;
};

size_t arena_layout(int n, int in_nc, int hp, int wp, Arena* A, const Band* band = nullptr,
                    ArenaOpts opt = ArenaOpts{}) {
  size_t off = 0;
  auto take = [&](size_t bytes) {
    size_t o = off;
    off += (bytes + 1023) & ~size_t(1023);
    return o;
  };
  // wmax: the largest (stored pixels x 64-channel units) over levels; umax: the same
  // over the levels whose transformer half runs as separate launches
  size_t px[4], wmax = 0, umax = 0;
  for (int l = 0; l < 4; ++l) {
    px[l] = plane_px(n, hp, wp, band, l);
    wmax = std::max(wmax, px[l] << l);
    if (!opt.fuse_trans || l >= 2) umax = std::max(umax, px[l] << l);
  }
  size_t o_skip[4], o_xs[4];
  for (int l = 0; l < 4; ++l) o_skip[l] = take((px[l] << l) * 256);
  for (int l = 0; l < 4; ++l) o_xs[l] = take((px[l] << l) * 128);
  size_t o_xw = take(opt.residual32 ? wmax * 256 : 0), o_y = take(wmax * 64), o_yt = take(wmax * 64),
         o_hc = take(wmax * 64),
         o_z = take(wmax * 128), o_a = take(umax * 64), o_o = take(umax * 64), o_qh = take(umax * 256);
  if (A) {
    char* b = A->base;
    for (int s = 0; s < 4; ++s) {
      A->skip[s] = reinterpret_cast<float*>(b + o_skip[s]);
      A->xs[s] = reinterpret_cast<__half*>(b + o_xs[s]);
    }
    A->xw = reinterpret_cast<float*>(b + o_xw);
    A->y = reinterpret_cast<__half*>(b + o_y);
    A->yt = reinterpret_cast<__half*>(b + o_yt);
    A->hc = reinterpret_cast<__half*>(b + o_hc);
    A->z = reinterpret_cast<__half*>(b + o_z);
    A->a = reinterpret_cast<__half*>(b + o_a);
    A->o = reinterpret_cast<__half*>(b + o_o);
    A->qh = reinterpret_cast<__half*>(b + o_qh);
  }
  return off;
}

// The stored plane of one level and the rows the ops work on.
struct Region {
  int n = 1;         // images
  int H = 0, W = 0;  // stored rows per image, columns
  int row0 = 0;      // first working row (kHalo for a band)
  int rows = 0;      // working rows per image
  bool banded = false;
  int grow0 = 0;     // image row of working row 0 (band)
  int H_image = 0;   // rows of the whole padded image at this level
  bool top = true, bottom = true;
  long px() const { return (long)n * rows * W; }  // working pixels
  long off(int ch) const { return (long)row0 * W * ch; }  // element offset of working row 0 (n == 1 when banded)
};

// The level-l region of arena A (the whole batch, or A's band).
Region region_of(const Arena& A, int l) {
  Region R;
  R.W = A.wp >> l;
  R.H_image = A.hp >> l;
  if (!A.banded) {
    R.n = A.n;
    R.H = A.hp >> l;
    R.row0 = 0;
    R.rows = R.H;
  } else {
    R.n = 1;
    R.banded = true;
    R.rows = A.band.rows >> l;
    R.row0 = kHalo;
    R.H = R.rows + 2 * kHalo;
    R.grow0 = A.band.R0 >> l;
    R.top = A.band.top;
    R.bottom = A.band.bottom;
  }
  return R;
}

}  // namespace

struct scb_ctx {
  int device = 0, in_nc = 3, dim = 64, sms = 148;
  int config[7] = {4, 4, 4, 4, 4, 4, 4};
  cudaStream_t stream = nullptr;
  std::string err;
  char* wblob = nullptr;
  size_t wbytes = 0;
  std::vector<BlockW> blocks[7];
  __half* wdown[3] = {};
  __half* wup[3] = {};
  __half* whead16 = nullptr;  // [64][32]: K = (ci, ky, kx) zero-padded to 32
  __half* wtail16 = nullptr;  // [32][64]: row 3 * tap + co, K = ci (unused rows zero)
  Arena arena;
  int last_launches = 0;
  bool fuse_trans = true;  // SCB_OPT_FUSE_TRANS
  bool residual32 = false; // SCB_OPT_RESIDUAL32
  bool trans32_lanes = false;  // SCB_OPT_TRANS32_LANES
  bool fuse_pair = true;       // SCB_OPT_FUSE_PAIR
  bool gemm_pairs = true;      // SCB_OPT_GEMM_PAIRS
  bool conv3_twin = true;      // SCB_OPT_CONV3_TWIN
  // scb_forward_dev_noalloc: the device address of g_noalloc_scratch on this
  // context's device (looked up by scb_create, which loads the device code and
  // with it the array) and the plan laid out in it.
  void* noalloc_base = nullptr;
  Arena noalloc;
  // device bytes this context has held: weights + scratch arenas now, and the
  // most it held at once (`Cuda::mem_report`'s high-water, src/cuda.rs:395-424)
  size_t high_water = 0;
  // scb_forward_host: a copy stream each way, two staging slots each way
  // ([in0 | in1 | out0 | out1], `io_slot` bytes each) and the events that order
  // them against the compute stream; images per compute call (SCB_OPT_HOST_CHUNK,
  // 0 = as many as fit kHostChunkPixels)
  cudaStream_t h2d = nullptr, d2h = nullptr;
  char* io = nullptr;
  size_t io_bytes = 0, io_slot = 0;
  cudaEvent_t ev_in[2] = {}, ev_comp[2] = {}, ev_out[2] = {};
  int host_chunk = 0;
  // row bands (config 5): one band per rank over NCCL, or all bands of one image
  // on this GPU (virtual bands, in lockstep)
  ncclComm_t nccl = nullptr;
  int band_rank = 0, band_nranks = 1;
  bool band_ready = false;  // scb_band_init has run and the group has not been aborted
  Arena band_arena;
  std::vector<Arena> vbands;
  // SCUNET_PROFILE equivalent (src/cuda.rs:106-135): events around every launch
  bool profiling = false;
  std::vector<cudaEvent_t> events;
  std::vector<int> prof_tags;
  std::vector<double> prof_flops;
  std::vector<double> prof_bytes;
  std::string prof_kernels;  // the kernel of each launch, one name per line
  std::vector<float> prof_ms;
};

ArenaOpts arena_opts(const scb_ctx* ctx) {
  ArenaOpts o;
  o.residual32 = ctx->residual32;
  o.fuse_trans = ctx->fuse_trans;
  return o;
}

namespace {

int fail(scb_ctx* ctx, int code, const std::string& msg) {
  if (ctx)
    ctx->err = msg;
  else
    g_create_error = msg;
  return code;
}

int cuda_fail(scb_ctx* ctx, cudaError_t e, const char* what) {
  return fail(ctx, SCB_ECUDA, std::string(what) + ": " + cudaGetErrorString(e));
}

#define CKC(ctx, x, what)                           \
  do {                                              \
    cudaError_t _e = (x);                           \
    if (_e != cudaSuccess) return cuda_fail(ctx, _e, what); \
  } while (0)

// Device bytes the context holds now (weights and every scratch arena it owns;
// the fixed no-allocation array is reported on its own).
size_t live_bytes(const scb_ctx* ctx) {
  size_t s = ctx->wbytes + ctx->arena.bytes + ctx->band_arena.bytes + ctx->io_bytes;
  for (const Arena& A : ctx->vbands) s += A.bytes;
  return s;
}

// Record the high-water after an allocation.
void note_mem(scb_ctx* ctx) { ctx->high_water = std::max(ctx->high_water, live_bytes(ctx)); }

// Host-side weight table lookup with shape check.
struct Table {
  std::map<std::string, const scb_tensor*> by_name;
  std::string err;
  const float* get(const std::string& name, std::initializer_list<int64_t> shape) {
    auto it = by_name.find(name);
    if (it == by_name.end()) {
      err = "missing tensor " + name;
      return nullptr;
    }
    const scb_tensor* t = it->second;
    if ((size_t)t->ndim != shape.size()) {
      err = name + ": rank " + std::to_string(t->ndim) + ", expected " + std::to_string(shape.size());
      return nullptr;
    }
    int i = 0;
    for (int64_t s : shape) {
      if (t->shape[i] != s) {
        err = name + ": dim " + std::to_string(i) + " is " + std::to_string(t->shape[i]) + ", expected " +
              std::to_string(s);
        return nullptr;
      }
      ++i;
    }
    if (!t->data) {
      err = name + ": null data";
      return nullptr;
    }
    return t->data;
  }
};

// Host staging for the weight blob: appends converted arrays, 256-byte aligned.
struct Blob {
  std::vector<char> host;
  size_t put(const void* p, size_t bytes) {
    size_t off = (host.size() + 255) & ~size_t(255);
    host.resize(off + bytes);
    memcpy(host.data() + off, p, bytes);
    return off;
  }
  size_t half(const std::vector<float>& v) {
    std::vector<__half> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = __float2half_rn(v[i]);
    return put(h.data(), h.size() * 2);
  }
  size_t f32(const float* p, size_t n) { return put(p, n * 4); }
};

cudaError_t launch_attn(const Op& op, cudaStream_t st) {
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(window_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, ATT_SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  int dev_sms = 148;
  cudaDeviceGetAttribute(&dev_sms, cudaDevAttrMultiProcessorCount, dev);
  // CTA c takes head c % heads: the grid is a multiple of the head count
  const long pairs = (op.attn.win.n_windows + 1) / 2;
  const long per_head = std::max(1L, std::min(pairs, (long)dev_sms * ATT_CTAS / op.attn.heads));
  const unsigned grid = (unsigned)(per_head * op.attn.heads);
  window_attn_kernel<<<grid, ATT_THREADS, ATT_SMEM, st>>>(op.attn_in, op.attn_out, op.attn_rp, op.attn);
  return cudaGetLastError();
}

cudaError_t launch_head(scb_ctx* ctx, const void* x, const HeadGeom& g, const Op& op, cudaStream_t st);
cudaError_t launch_tail(scb_ctx* ctx, void* y, const TailGeom& g, const Op& op, cudaStream_t st);

cudaError_t launch_trans32(const Op& op, int sms, cudaStream_t st) {
  using L = T32;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(trans32_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const long pairs = (op.trans.win.n_windows + 1) / 2;
  const int grid = (int)std::max(1L, std::min(pairs, (long)sms));  // one CTA per SM, persistent over pairs
  trans32_ws_kernel<<<grid, L::THREADS, L::SMEM, st>>>(op.trans);
  return cudaGetLastError();
}

cudaError_t launch_trans64(const Op& op, int sms, cudaStream_t st) {
  using L = T64;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(trans64_ws_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const long pairs = (op.trans.win.n_windows + 1) / 2;
  const int grid = (int)std::max(1L, std::min(pairs, (long)sms));  // one CTA per SM, persistent over pairs
  trans64_ws_kernel<<<grid, L::THREADS, L::SMEM, st>>>(op.trans);
  return cudaGetLastError();
}

template <int T>
cudaError_t launch_mlp_t(const Op& op, int sms, cudaStream_t st) {
  using L = MlpLayout<T>;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(mlp_fused_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const int grid = std::max(1, std::min(op.mlp.m_tiles, sms));
  mlp_fused_kernel<T><<<grid, MLP_THREADS, L::SMEM, st>>>(op.mlp_a, op.mlp_w0, op.mlp_w2, op.mlp);
  return cudaGetLastError();
}

cudaError_t launch_mlp(const Op& op, int sms, cudaStream_t st) {
  if (op.mlp_t == 128) return launch_mlp_t<128>(op, sms, st);
  if (op.mlp_t == 256) return launch_mlp_t<256>(op, sms, st);
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_trans32mp(const Op& op, int sms, cudaStream_t st) {
  using L = T32M;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(trans32_mp_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const long pairs = (op.trans.win.n_windows + 1) / 2;
  const long ctas = (pairs + L::LANES - 1) / L::LANES;
  const int grid = (int)std::max(1L, std::min(ctas, (long)sms));  // one CTA per SM, persistent over pairs
  trans32_mp_kernel<<<grid, L::THREADS, L::SMEM, st>>>(op.trans);
  return cudaGetLastError();
}

// TMA ring depth and CTAs per SM of the block-boundary kernel: at 64 channels two
// CTAs per SM (eight epilogue warps) with a two-stage ring each; at 128 channels the
// resident weights and staging leave room for one CTA with three stages.
template <int C>
cudaError_t launch_pair_t(const Op& op, int sms, cudaStream_t st) {
  using L = PairSmem<C>;
  constexpr int stages = C == 64 ? 2 : 3, ctas = C == 64 ? 2 : 1;
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(conv_pair_kernel<C>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         L::smem(stages));
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  PairGeom g = op.pair;
  g.stages = stages;
  const int grid = std::max(1, std::min(g.tiles, sms * ctas));
  conv_pair_kernel<C><<<grid, 192, L::smem(stages), st>>>(op.pair_mz, op.pair_mx, op.pair_myc, op.pair_myt,
                                                             op.pair_w12, op.pair_w11, g);
  return cudaGetLastError();
}

cudaError_t launch_pair(const Op& op, int sms, cudaStream_t st) {
  if (op.pair_c == 64) return launch_pair_t<64>(op, sms, st);
  if (op.pair_c == 128) return launch_pair_t<128>(op, sms, st);
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_trans(const Op& op, int sms, cudaStream_t st) {
  if (op.trans_t == 32) return op.trans_lanes ? launch_trans32mp(op, sms, st) : launch_trans32(op, sms, st);
  if (op.trans_t == 64) return launch_trans64(op, sms, st);
  return cudaErrorInvalidConfiguration;
}

cudaError_t launch_head(scb_ctx* ctx, const void* x, const HeadGeom& g, const Op& op, cudaStream_t st) {
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(head_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, HEAD_SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const long tiles = ((long)g.n * g.rows * g.wp + 127) / 128;
  const int grid = (int)std::max(1L, std::min(tiles, (long)ctx->sms * 3));
  head_tc_kernel<<<grid, 128, HEAD_SMEM, st>>>(x, ctx->whead16, op.head_m32, op.head_m16, g);
  return cudaGetLastError();
}

cudaError_t launch_tail(scb_ctx* ctx, void* y, const TailGeom& g, const Op& op, cudaStream_t st) {
  static bool attr_set[16] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 16 && !attr_set[dev]) {
    cudaError_t e = cudaFuncSetAttribute(tail_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, TAIL_SMEM);
    if (e != cudaSuccess) return e;
    attr_set[dev] = true;
  }
  const long units = (long)g.n * g.strips * g.chunks;
  const int grid = (int)std::max(1L, std::min(units, (long)ctx->sms * 2));
  tail_tc_kernel<<<grid, TAIL_THREADS, TAIL_SMEM, st>>>(op.tail_map, ctx->wtail16, y, g);
  return cudaGetLastError();
}

// Run the ops of the arena's plan on `st`, with the image pointers of this call.
// The image of one forward call.
struct Io {
  const void* x;
  int x_u8;
  void* y;
  int y_u8;
  int c, h, w;
};

// Halo exchange of one XCHG op between bands. `nb` bands of this process (one, for
// a rank of a NCCL group; all of them for virtual bands on one GPU).
int exchange_nccl(scb_ctx* ctx, Arena& A, const Op& op, cudaStream_t st);

int exchange_local(scb_ctx* ctx, std::vector<Arena>& bands, size_t k, cudaStream_t st) {
  // every band copies its kHalo first/last working rows into its neighbours' halo
  for (size_t b = 0; b < bands.size(); ++b) {
    const Op& op = bands[b].ops[k];
    const size_t bytes = (size_t)kHalo * op.xchg_row;
    if (b > 0) {
      const Op& up = bands[b - 1].ops[k];
      CKC(ctx, cudaMemcpyAsync(up.xchg_base + (size_t)(up.xchg_row0 + up.xchg_rows) * up.xchg_row,
                               op.xchg_base + (size_t)op.xchg_row0 * op.xchg_row, bytes, cudaMemcpyDeviceToDevice, st),
          "halo copy");
    }
    if (b + 1 < bands.size()) {
      const Op& dn = bands[b + 1].ops[k];
      CKC(ctx, cudaMemcpyAsync(dn.xchg_base + (size_t)(dn.xchg_row0 - kHalo) * dn.xchg_row,
                               op.xchg_base + (size_t)(op.xchg_row0 + op.xchg_rows - kHalo) * op.xchg_row, bytes,
                               cudaMemcpyDeviceToDevice, st),
          "halo copy");
    }
  }
  return SCB_OK;
}

// NCCL, loaded at run time so the library needs it only for multi-GPU bands.
struct NcclApi {
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  // the band watchdog (scb_band_sync): a peer's failure, and tearing the group down
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
};

const NcclApi* nccl_api(std::string& err) {
  static NcclApi api;
  static bool loaded = false, tried = false;
  if (!tried) {
    tried = true;
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (h) {
      api.GetUniqueId = reinterpret_cast<decltype(api.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
      api.CommInitRank = reinterpret_cast<decltype(api.CommInitRank)>(dlsym(h, "ncclCommInitRank"));
      api.CommDestroy = reinterpret_cast<decltype(api.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
      api.Send = reinterpret_cast<decltype(api.Send)>(dlsym(h, "ncclSend"));
      api.Recv = reinterpret_cast<decltype(api.Recv)>(dlsym(h, "ncclRecv"));
      api.GroupStart = reinterpret_cast<decltype(api.GroupStart)>(dlsym(h, "ncclGroupStart"));
      api.GroupEnd = reinterpret_cast<decltype(api.GroupEnd)>(dlsym(h, "ncclGroupEnd"));
      api.GetErrorString = reinterpret_cast<decltype(api.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
      api.CommGetAsyncError =
          reinterpret_cast<decltype(api.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
      api.CommAbort = reinterpret_cast<decltype(api.CommAbort)>(dlsym(h, "ncclCommAbort"));
      loaded = api.GetUniqueId && api.CommInitRank && api.CommDestroy && api.Send && api.Recv && api.GroupStart &&
               api.GroupEnd && api.GetErrorString && api.CommGetAsyncError && api.CommAbort;
    }
  }
  if (!loaded) {
    err = "libnccl.so.2 could not be loaded (needed for multi-GPU row bands)";
    return nullptr;
  }
  return &api;
}

// Launch one op of arena A's plan.
cudaError_t exec_op(scb_ctx* ctx, Arena& A, const Op& op, const Io& io, cudaStream_t st) {
  switch (op.kind) {
    case Op::HEAD: {
      const Region R = region_of(A, 0);
      HeadGeom g{R.n, io.c, io.h, io.w, A.hp, A.wp, io.x_u8, R.grow0, R.rows};
      return launch_head(ctx, io.x, g, op, st);
    }
    case Op::TAIL: {
      TailGeom g = op.tail;
      g.c = io.c;
      g.h = io.h;
      g.w = io.w;
      g.u8 = io.y_u8;
      return launch_tail(ctx, io.y, g, op, st);
    }
    case Op::GEMM:
      return launch_gemm(op.gemm, ctx->sms, st);
    case Op::ATTN:
      return launch_attn(op, st);
    case Op::TRANS:
      return launch_trans(op, ctx->sms, st);
    case Op::MLP:
      return launch_mlp(op, ctx->sms, st);
    case Op::PAIR:
      return launch_pair(op, ctx->sms, st);
    case Op::XCHG:
      return cudaSuccess;  // handled by the caller (it needs the other bands)
    case Op::ZERO:
      return op.zero_bytes ? cudaMemsetAsync(op.zero_ptr, 0, op.zero_bytes, st) : cudaSuccess;
  }
  return cudaErrorInvalidValue;
}

// Algorithmic HBM bytes of one launch - every operand read once, every result
// written once, weights included: the numerator of its memory roofline.
double op_bytes(const Arena& A, const Op& op, const Io& io) {
  switch (op.kind) {
    case Op::TAIL: {  // the shadow in, the crop out, the weights
      const TailGeom& g = op.tail;
      return (double)g.n * g.rows_out * g.W * 64 * 2 + 32.0 * 64 * 2 + (double)A.n * io.h * io.w * io.c * (io.y_u8 ? 1 : 4);
    }
    case Op::GEMM: {
      const GemmOp& o = op.gemm;
      const GemmGeom& g = o.g;
      const GemmEpi& e = o.e;
      double px = g.M, px_in = g.M;  // GEMM rows (output pixels; UP2: input pixels), pixels read
      if (is_conv3(o.geo)) {
        px = (double)g.M / g.H * g.rows_out;
        px_in = px;
      } else if (o.geo == GEO_DOWN2) {
        px_in = 4.0 * g.M;
      }
      const double cin = (double)g.kb_per_tap * o.bk;
      const double taps = is_conv3(o.geo) ? 9 : o.geo == GEO_DOWN2 ? 4 : 1;
      const double n_cols = g.n_total;
      double per_elem = 0;
      if (e.out16) per_elem += 2;
      if (e.out32) per_elem += 4;
      if (e.res16) per_elem += 2;
      if (e.res32) per_elem += 4;
      if (e.skip32) per_elem += 4;
      double b = px_in * cin * 2 + n_cols * cin * taps * 2 + px * n_cols * per_elem;
      if (e.ln_out) b += px * e.ln_n * 2;
      return b;
    }
    case Op::TRANS: {
      const double t = op.trans_t, tokens = 64.0 * op.trans.win.n_windows;
      return tokens * t * 2 * 2 + 12.0 * t * t * 2;
    }
    case Op::ATTN:
      return 64.0 * op.attn.win.n_windows * (3.0 * op.attn.t + op.attn.t) * 2;
    case Op::MLP:  // a in, x1 in, z out; both weight matrices
      return (double)op.mlp.M * op.mlp_t * 2 * 3 + 16.0 * op.mlp_t * op.mlp_t;
    case Op::PAIR:  // Z and x in, x' and Y out; both weight matrices
      return (double)op.pair.M * op.pair_c * 2 * 4 + 4.0 * op.pair_c * op.pair_c;
    case Op::HEAD: {
      const Region R = region_of(A, 0);
      return (double)R.px() * (io.c * (io.x_u8 ? 1 : 4) + 64 * (4 + 2));
    }
    case Op::XCHG:
      return 4.0 * kHalo * op.xchg_row;  // up to two halos sent and two received
    case Op::ZERO:
      return (double)op.zero_bytes;
  }
  return 0;
}

// The kernel a launch of `op` runs, as profilers print it.
std::string op_kernel_name(const Op& op) {
  switch (op.kind) {
    case Op::GEMM: {
      const GemmOp& g = op.gemm;
      return "gemm_tc_kernel<" + std::to_string(g.bn) + ", " + std::to_string(g.bk) + ", " + std::to_string(g.geo) +
             ", " + (g.tma_epi ? "1" : "0") + (g.pairs ? ", 1" : "") + ">";
    }
    case Op::ATTN: return "window_attn_kernel";
    case Op::HEAD: return "head_tc_kernel";
    case Op::TAIL: return "tail_tc_kernel";
    case Op::TRANS:
      return op.trans_t == 64 ? "trans64_ws_kernel" : op.trans_lanes ? "trans32_mp_kernel" : "trans32_ws_kernel";
    case Op::MLP: return "mlp_fused_kernel<" + std::to_string(op.mlp_t) + ">";
    case Op::PAIR: return "conv_pair_kernel<" + std::to_string(op.pair_c) + ">";
    case Op::XCHG: return "(halo exchange)";
    case Op::ZERO: return "(memset)";
  }
  return "?";
}

int run_ops(scb_ctx* ctx, Arena& A, const void* x, int x_u8, void* y, int y_u8, int c, int h, int w,
            cudaStream_t st, bool allow_profile = true) {
  // (a banded arena here is one rank of a NCCL band group)
  int launches = 0;
  const bool profiling = ctx->profiling && allow_profile;
  const Io io{x, x_u8, y, y_u8, c, h, w};
  if (profiling) {
    while (ctx->events.size() < A.ops.size() + 1) {
      cudaEvent_t ev;
      CKC(ctx, cudaEventCreate(&ev), "cudaEventCreate");
      ctx->events.push_back(ev);
    }
    CKC(ctx, cudaEventRecord(ctx->events[0], st), "cudaEventRecord");
  }
  for (const Op& op : A.ops) {
    if (op.kind == Op::XCHG) {
      const int r = exchange_nccl(ctx, A, op, st);
      if (r) return r;
    } else {
      const cudaError_t e = exec_op(ctx, A, op, io, st);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "kernel launch");
    }
    ++launches;
    if (profiling) CKC(ctx, cudaEventRecord(ctx->events[launches], st), "cudaEventRecord");
  }
  ctx->last_launches = launches;
  if (profiling) {
    ctx->prof_tags.clear();
    ctx->prof_flops.clear();
    ctx->prof_bytes.clear();
    ctx->prof_kernels.clear();
    for (const Op& op : A.ops) {
      ctx->prof_tags.push_back(op.tag);
      ctx->prof_flops.push_back(op.flops);
      ctx->prof_bytes.push_back(op_bytes(A, op, io));
      ctx->prof_kernels += op_kernel_name(op);
      ctx->prof_kernels += '\n';
    }
    ctx->prof_ms.assign(A.ops.size(), -1.f);  // filled by scb_profile_read after a sync
  }
  return SCB_OK;
}

Op xchg_op(void* plane, const Region& R, int ch, int elem_bytes) {
  Op x{};
  x.kind = Op::XCHG;
  x.tag = TAG_HALO;
  x.xchg_base = static_cast<char*>(plane);
  x.xchg_row = (size_t)R.W * ch * elem_bytes;
  x.xchg_row0 = R.row0;
  x.xchg_rows = R.rows;
  return x;
}

// Window placement of a block's attention over region R.
WinGeom win_geom(const Region& R, bool shifted) {
  WinGeom g{};
  g.H = R.H;
  g.W = R.W;
  g.shift = shifted ? 4 : 0;
  g.nwc = R.W / 8;
  g.nwr_global = R.H_image / 8;
  if (!R.banded) {
    g.wrap = 1;
    g.row_base = 0;
    g.nwr = R.H / 8;
    g.gwr0 = 0;
    g.store_lo = 0;
    g.store_hi = R.H;
  } else {
    // W: the band's own windows. SW: one more window row; the first starts 4 rows
    // above the band, the last ends 4 rows below it (both in the halo).
    g.wrap = 0;
    g.row_base = shifted ? R.row0 - 4 : R.row0;
    g.nwr = R.rows / 8 + (shifted ? 1 : 0);
    g.gwr0 = ((R.grow0 / 8 - (shifted ? 1 : 0)) % g.nwr_global + g.nwr_global) % g.nwr_global;
    g.store_lo = R.row0;
    g.store_hi = R.row0 + R.rows;
  }
  g.n_windows = (long)R.n * g.nwr * g.nwc;
  return g;
}

// The ops of one ConvTransBlock over region R of a level with c channels.
//   xin (fp32, its fp16 shadow already in xs) -> xout (fp32, may alias xin; may be
//   null when `skip` is given: then only the fp16 shadow of (x + skip) is written).
// Plane pointers are the stored planes; FLAT ops address the working rows.
// The fused MLP of a t = 128 / 256 transformer half over P tokens: a = LN2(x1) [P][t]
// (ld t) in, x1 in and z = x1 + mlp2(GELU(mlp0(a))) out at z[p * z_ld + col].
bool mlp_op(Op& mo, const BlockW& bw, const __half* a, __half* z, long z_ld, long P, std::string& err) {
  const int t = bw.c / 2;
  if (t != 128 && t != 256) {
    err = "the fused MLP is built for trans widths 128 and 256";
    return false;
  }
  mo.kind = Op::MLP;
  mo.tag = TAG_MLP;
  mo.mlp_t = t;
  mo.flops = 2.0 * 2.0 * P * t * 4 * t;
  mo.mlp.M = (int)P;
  mo.mlp.m_tiles = (int)((P + 127) / 128);
  mo.mlp.z = z;
  mo.mlp.z_ld = z_ld;
  mo.mlp.b0 = bw.b0;
  mo.mlp.b2 = bw.b2;
  const uint64_t da[2] = {(uint64_t)t, (uint64_t)P}, sa[1] = {(uint64_t)t * 2};
  const uint64_t d0[2] = {(uint64_t)t, (uint64_t)(4 * t)}, s0[1] = {(uint64_t)t * 2};
  const uint64_t d2[2] = {(uint64_t)(4 * t), (uint64_t)t}, s2[1] = {(uint64_t)(4 * t) * 2};
  const uint32_t ba[2] = {64, 128}, b2b[2] = {64, (uint32_t)t};
  return encode_map(&mo.mlp_a, a, 2, da, sa, ba, 2, 128, err) &&
         encode_map(&mo.mlp_w0, bw.w0, 2, d0, s0, ba, 2, 128, err) &&
         encode_map(&mo.mlp_w2, bw.w2, 2, d2, s2, b2b, 2, 128, err);
}

// `next`: the following block of the same stage, whose conv1_1 then runs in this
// block's conv1_2 kernel (one PAIR op); `conv11_done`: this block's conv1_1 already
// ran that way in the previous block's op.
bool block_ops(scb_ctx* ctx, std::vector<Op>& ops, const BlockW& bw, const Arena& A, const Region& R,
               const float* xin, float* xout, __half* xs, const float* skip, bool shifted, std::string& err,
               const BlockW* next = nullptr, bool conv11_done = false) {
  const int c = bw.c, t = c / 2, cc = c / 2, heads = t / 32;
  const int n = R.n, H = R.H, W = R.W;
  const long P = R.px();
  const bool fused = ctx->fuse_trans && (t == 32 || t == 64);
  Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
  Op op{};
  op.kind = Op::GEMM;
  // 1. y = conv1_1(x) + b  -> Y (fp16, both halves); LN1 of the trans half -> A
  if (!conv11_done) {
    GemmOp g{};
    if (!mk.flat(g, xs + R.off(c), P, c, c, bw.w11, c, GEO_FLAT, fused ? 0 : t)) return false;
    g.e.bias = bw.b11;
    // the conv half and the trans half to separate planes: their readers (the 3x3
    // pair, the transformer) then read whole contiguous pixel rows
    g.e.out16 = A.y + R.off(cc);
    g.e.out16_ld = cc;
    g.e.out16b = A.yt + R.off(t);
    g.e.out16b_ld = t;
    g.e.out16_split = cc;
    if (!fused) {  // the fused transformer kernel normalises its own input
      g.e.ln_g = bw.ln1g;
      g.e.ln_b = bw.ln1b;
      g.e.ln_out = A.a + R.off(t);
      g.e.ln_ld = t;
      g.e.ln_lo = cc;
      g.e.ln_n = t;
    }
    if (!mk.finish_epi(g)) return false;
    op.gemm = g;
    op.tag = TAG_CONV1X1;
    op.flops = 2.0 * P * c * c;
    ops.push_back(op);
  }
  if (R.banded) {
    // the one exchange of the block: Y's boundary rows (3x3 pair and SW windows),
    // and for the separate-launch transformer path also LN1's
    ops.push_back(xchg_op(A.y, R, cc, 2));
    ops.push_back(xchg_op(A.yt, R, t, 2));
    if (!fused) ops.push_back(xchg_op(A.a, R, t, 2));
  }
  // 2. h = relu(conv3x3(y_c)), on the working rows plus one halo row on each side
  //    that has a neighbour (conv 3 reads it); the image's own edges stay zero
  {
    const int lo = R.banded && !R.top ? R.row0 - 1 : R.row0;
    const int hi = R.banded && !R.bottom ? R.row0 + R.rows + 1 : R.row0 + R.rows;
    GemmOp g{};
    if (!mk.conv3(g, A.y, n, H, W, cc, cc, bw.wc0, cc, true, lo, hi - lo)) return false;
    g.e.act = ACT_RELU;
    g.e.out16 = A.hc;
    g.e.out16_ld = cc;
    if (!mk.finish_epi(g)) return false;
    op.gemm = g;
    op.tag = TAG_CONV3X3;
    op.flops = 2.0 * n * (hi - lo) * W * 9 * cc * cc;
    ops.push_back(op);
  }
  // 3. z[:, :cc] = conv3x3(h) + y_c
  {
    GemmOp g{};
    if (!mk.conv3(g, A.hc, n, H, W, cc, cc, bw.wc2, cc, true, R.row0, R.rows)) return false;
    g.e.res16 = A.y;
    g.e.res16_ld = cc;
    g.e.out16 = A.z;
    g.e.out16_ld = c;
    if (!mk.finish_epi(g)) return false;
    op.gemm = g;
    op.tag = TAG_CONV3X3;
    op.flops = 2.0 * P * 9 * cc * cc;
    ops.push_back(op);
  }
  const WinGeom wg = win_geom(R, shifted);
  if (fused) {
    // 4-8. the whole transformer half in one kernel
    Op tr{};
    tr.kind = Op::TRANS;
    tr.trans_t = t;
    tr.trans_lanes = t == 32 && ctx->trans32_lanes;
    tr.tag = TAG_TRANS;
    tr.flops = 2.0 * P * (3.0 * t * t + 2.0 * 64 * t + t * t + 8.0 * t * t);
    TransGeom& tg = tr.trans;
    tg.win = wg;
    tg.y = A.yt;
    tg.z = A.z;
    tg.wqkv = bw.wqkv; tg.wproj = bw.wproj; tg.w0 = bw.w0; tg.w2 = bw.w2;
    tg.bqkv = bw.bqkv; tg.bproj = bw.bproj; tg.b0 = bw.b0; tg.b2 = bw.b2;
    tg.ln1g = bw.ln1g; tg.ln1b = bw.ln1b; tg.ln2g = bw.ln2g; tg.ln2b = bw.ln2b; tg.rp = bw.rp;
    tg.wqkv_f = bw.wqkv_f; tg.w0_f = bw.w0_f; tg.bqkv_f = bw.bqkv_f; tg.b0_f = bw.b0_f;
    ops.push_back(tr);
  } else {
    // 4. qkv = LN1(y_t) W^T + b; a band needs it on its halo rows too (SW windows)
    {
      const long Pq = R.banded ? (long)n * H * W : P;
      const long oq = R.banded ? 0 : R.off(t);
      GemmOp g{};
      if (!mk.flat(g, A.a + oq, Pq, t, t, bw.wqkv, 3 * t)) return false;
      g.e.bias = bw.bqkv;
      g.e.out16 = A.qh + (R.banded ? 0 : R.off(3 * t));
      g.e.out16_ld = 3 * t;
      if (!mk.finish_epi(g)) return false;
      op.gemm = g;
      op.tag = TAG_QKV;
      op.flops = 2.0 * Pq * t * 3 * t;
      ops.push_back(op);
    }
    // 5. window attention
    {
      Op at{};
      at.kind = Op::ATTN;
      at.attn = AttnGeom{wg, t, heads, 3L * t, (long)t};
      at.attn_in = A.qh;
      at.attn_out = A.o;
      at.attn_rp = bw.rp;
      at.tag = TAG_ATTN;
      at.flops = 2.0 * 2.0 * P * 64 * t;
      ops.push_back(at);
    }
    // 6. x1t = o Wp^T + b + y_t -> z[:, cc:]; LN2(x1t) -> A
    {
      GemmOp g{};
      if (!mk.flat(g, A.o + R.off(t), P, t, t, bw.wproj, t, GEO_FLAT, t, true)) return false;
      g.e.bias = bw.bproj;
      g.e.res16 = A.yt + R.off(t);
      g.e.res16_ld = t;
      g.e.out16 = A.z + R.off(c) + cc;
      g.e.out16_ld = c;
      g.e.ln_g = bw.ln2g;
      g.e.ln_b = bw.ln2b;
      g.e.ln_out = A.a + R.off(t);
      g.e.ln_ld = t;
      g.e.ln_lo = 0;
      g.e.ln_n = t;
      if (!mk.finish_epi(g)) return false;
      op.gemm = g;
      op.tag = TAG_PROJ;
      op.flops = 2.0 * P * t * t;
      ops.push_back(op);
    }
    if (t == 128 || t == 256) {
      // 7-8. z[:, cc:] = x1t + mlp2(GELU(mlp0(LN2(x1t)))) in one kernel: the 4t-wide
      //      hidden layer stays on chip (mlp.cuh)
      Op mo{};
      if (!mlp_op(mo, bw, A.a + R.off(t), A.z + R.off(c) + cc, c, P, err)) return false;
      ops.push_back(mo);
    } else {
      // 7. hid = gelu(LN2 W0^T + b0)
      {
        GemmOp g{};
        if (!mk.flat(g, A.a + R.off(t), P, t, t, bw.w0, 4 * t)) return false;
        g.e.bias = bw.b0;
        g.e.act = ACT_GELU;
        g.e.out16 = A.qh + R.off(4 * t);
        g.e.out16_ld = 4 * t;
        if (!mk.finish_epi(g)) return false;
        op.gemm = g;
        op.tag = TAG_MLP0;
        op.flops = 2.0 * P * t * 4 * t;
        ops.push_back(op);
      }
      // 8. z[:, cc:] = hid W2^T + b2 + x1t
      {
        GemmOp g{};
        if (!mk.flat(g, A.qh + R.off(4 * t), P, 4 * t, 4 * t, bw.w2, t)) return false;
        g.e.bias = bw.b2;
        g.e.res16 = A.z + R.off(c) + cc;
        g.e.res16_ld = c;
        g.e.out16 = A.z + R.off(c) + cc;
        g.e.out16_ld = c;
        if (!mk.finish_epi(g)) return false;
        op.gemm = g;
        op.tag = TAG_MLP2;
        op.flops = 2.0 * P * t * 4 * t;
        ops.push_back(op);
      }
    }
  }
  // 9. x = x + conv1_2(z) + b and its fp16 copy (or that of x + skip). The residual
  //    x is `xin` (fp32) when given, else the fp16 plane xs itself, updated in place
  //    (every tile reads its residual slab before storing that slab); fp32 x is
  //    written only when `xout` is given.
  if (next) {
    // x' = x + conv1_2(z) + b12 -> xs, and the next block's Y = conv1_1(x') + b11
    if ((c != 64 && c != 128) || xin || xout || skip || next->c != c) {
      err = "a block boundary kernel needs 64 or 128 channels and the fp16 residual stream";
      return false;
    }
    Op po{};
    po.kind = Op::PAIR;
    po.tag = TAG_CONV1X1;
    po.flops = 2.0 * 2.0 * P * c * c;
    po.pair_c = c;
    po.pair_w12 = bw.w12;
    po.pair_w11 = next->w11;
    po.pair.M = (int)P;
    po.pair.tiles = (int)((P + 127) / 128);
    po.pair.b12 = bw.b12;
    po.pair.b11 = next->b11;
    const uint64_t dz[2] = {(uint64_t)c, (uint64_t)P}, sz[1] = {(uint64_t)c * 2};
    const uint64_t dy[2] = {(uint64_t)cc, (uint64_t)P}, sy[1] = {(uint64_t)cc * 2};
    const uint32_t bz[2] = {64, 128}, by[2] = {32, 128};
    if (!encode_map(&po.pair_mz, A.z + R.off(c), 2, dz, sz, bz, 2, 128, err) ||
        !encode_map(&po.pair_mx, xs + R.off(c), 2, dz, sz, bz, 2, 128, err) ||
        !encode_map(&po.pair_myc, A.y + R.off(cc), 2, dy, sy, by, 2, 64, err) ||
        !encode_map(&po.pair_myt, A.yt + R.off(t), 2, dy, sy, by, 2, 64, err))
      return false;
    ops.push_back(po);
  } else {
    GemmOp g{};
    if (!mk.flat(g, A.z + R.off(c), P, c, c, bw.w12, c)) return false;
    g.e.bias = bw.b12;
    if (xin) {
      g.e.res32 = xin + R.off(c);
      g.e.res32_ld = c;
    } else {
      g.e.res16 = xs + R.off(c);
      g.e.res16_ld = c;
    }
    g.e.out32 = xout ? xout + R.off(c) : nullptr;
    g.e.out32_ld = c;
    g.e.out16 = xs + R.off(c);
    g.e.out16_ld = c;
    g.e.skip32 = skip ? skip + R.off(c) : nullptr;
    g.e.skip_ld = c;
    if (!mk.finish_epi(g)) return false;
    op.gemm = g;
    op.tag = TAG_CONV1X1;
    op.flops = 2.0 * P * c * c;
    ops.push_back(op);
  }
  (void)ctx;
  return true;
}

int build_plan(scb_ctx* ctx, Arena& A) {
  std::string err;
  std::vector<Op>& ops = A.ops;
  ops.clear();
  const Region R0 = region_of(A, 0);
  const double P0 = (double)R0.px();
  Op head{};
  head.kind = Op::HEAD;
  head.tag = TAG_HEAD;
  head.flops = 2.0 * P0 * 9 * ctx->in_nc * 64;
  {
    const uint64_t d[2] = {64, (uint64_t)P0}, s32[1] = {256}, s16[1] = {128};
    const uint32_t b32[2] = {32, 128}, b16[2] = {64, 128};
    if (!encode_map(&head.head_m32, A.skip[0] + R0.off(64), 2, d, s32, b32, 4, 128, err) ||
        !encode_map(&head.head_m16, A.xs[0] + R0.off(64), 2, d, s16, b16, 2, 128, err))
      return fail(ctx, SCB_EINVAL, err);
  }
  ops.push_back(head);
  for (int s = 0; s < 7; ++s) {
    const int lvl = kStageLevel[s];
    const int c = 64 << lvl;
    const bool up = s >= 4;
    const Region R = region_of(A, lvl);
    if (R.banded) {
      // Y and Hc are shared by all levels; at an image edge their halo rows must read
      // as zero (conv zero padding) although other levels wrote that memory
      // (every band gets the same ops - lockstep execution pairs them by index - and
      // the interior sides clear nothing)
      // (the trans half's halo rows are only read by masked shifted-window keys, but
      // they must be finite: a zero attention weight times NaN is NaN)
      const size_t rb = (size_t)R.W * (c / 2) * 2;  // one row of Y_c, Y_t or Hc
      for (int side = 0; side < 2; ++side) {
        const bool edge = side == 0 ? R.top : R.bottom;
        const int r = side == 0 ? 0 : R.row0 + R.rows;
        for (__half* plane : {A.y, A.yt, A.hc}) {
          Op zp{};
          zp.kind = Op::ZERO;
          zp.tag = TAG_HALO;
          zp.zero_ptr = reinterpret_cast<char*>(plane) + r * rb;
          zp.zero_bytes = edge ? kHalo * rb : 0;
          ops.push_back(zp);
        }
      }
    }
    if (up) {
      // m_up{k}.0 : transposed conv from level lvl+1 (shadow already holds x + skip)
      const Region Rn = region_of(A, lvl + 1);
      Op op{};
      op.kind = Op::GEMM;
      Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
      GemmOp g{};
      if (!mk.up2(g, A.xs[lvl + 1] + Rn.off(2 * c), Rn.n, Rn.rows, Rn.W, 2 * c, ctx->wup[s - 4], c))
        return fail(ctx, SCB_EINVAL, err);
      g.e.out32 = ctx->residual32 ? A.xw + R.off(c) : nullptr;
      g.e.out32_ld = c;
      g.e.out16 = A.xs[lvl] + R.off(c);
      g.e.out16_ld = c;
      if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
      op.gemm = g;
      op.tag = TAG_UP;
      op.flops = 2.0 * Rn.px() * (2 * c) * (4 * c);
      ops.push_back(op);
    }
    const int nb = ctx->config[s];
    bool prev_pair = false;
    for (int i = 0; i < nb; ++i) {
      // the residual stream: fp16 in xs (default; a down stage's first block reads the
      // skip plane's fp16 shadow, which the head / down conv wrote into xs), or fp32
      // in xw with xs its copy (SCB_OPT_RESIDUAL32; a down stage then starts from the
      // fp32 skip plane itself)
      const float* xin = !ctx->residual32 ? nullptr : (!up && i == 0) ? A.skip[lvl] : A.xw;
      const bool last = i == nb - 1;
      const float* skip = nullptr;
      float* xout = ctx->residual32 ? A.xw : nullptr;
      if (last && s >= 3) {  // body, up3, up2, up1: the fp16 plane holds x + skip
        skip = A.skip[lvl];
        xout = nullptr;
      }
      // a boundary between two blocks of the stage at 64 or 128 channels runs as one
      // kernel (this block's conv1_2 with the next block's conv1_1), when the residual
      // stream is fp16 and the next block's transformer half normalises its own input
      const bool pair = ctx->fuse_pair && !ctx->residual32 && ctx->fuse_trans && !skip && i + 1 < nb &&
                        (c == 64 || c == 128);
      if (!block_ops(ctx, ops, ctx->blocks[s][i], A, R, xin, xout, A.xs[lvl], skip, (i % 2) == 1, err,
                     pair ? &ctx->blocks[s][i + 1] : nullptr, prev_pair))
        return fail(ctx, SCB_EINVAL, err);
      prev_pair = pair;
    }
    if (s < 3) {
      // m_down{k}.4 : 2x2 stride-2 conv -> the next level's skip (fp32) + shadow
      const Region Rn = region_of(A, lvl + 1);
      Op op{};
      op.kind = Op::GEMM;
      Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
      GemmOp g{};
      if (!mk.down2(g, A.xs[lvl] + R.off(c), R.n, R.rows, R.W, c, ctx->wdown[s], 2 * c))
        return fail(ctx, SCB_EINVAL, err);
      g.e.out32 = A.skip[lvl + 1] + Rn.off(2 * c);
      g.e.out32_ld = 2 * c;
      g.e.out16 = A.xs[lvl + 1] + Rn.off(2 * c);
      g.e.out16_ld = 2 * c;
      if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
      op.gemm = g;
      op.tag = TAG_DOWN;
      op.flops = 2.0 * Rn.px() * (4 * c) * (2 * c);
      ops.push_back(op);
    }
  }
  if (R0.banded) ops.push_back(xchg_op(A.xs[0], R0, 64, 2));  // the tail conv's halo row
  Op tail{};
  tail.kind = Op::TAIL;
  {
    const uint64_t dims[4] = {64, (uint64_t)R0.W, (uint64_t)R0.H, (uint64_t)R0.n};
    const uint64_t str[3] = {64 * 2, (uint64_t)R0.W * 64 * 2, (uint64_t)R0.H * R0.W * 64 * 2};
    const uint32_t box[4] = {64, 128, 1, 1};
    if (!encode_map(&tail.tail_map, A.xs[0], 4, dims, str, box, 2, 128, err)) return fail(ctx, SCB_EINVAL, err);
    TailGeom& tg = tail.tail;
    tg.n = R0.n;
    tg.H = R0.H;
    tg.W = R0.W;
    tg.row0 = R0.row0;
    tg.rows_out = R0.rows;
    tg.row_off = R0.grow0 - R0.row0;
    tg.strips = (R0.W + TAIL_COLS - 1) / TAIL_COLS;
    tg.chunks = (R0.rows + TAIL_ROWS - 1) / TAIL_ROWS;
  }
  tail.tag = TAG_TAIL;
  tail.flops = 2.0 * P0 * 9 * 64 * ctx->in_nc;
  ops.push_back(tail);
  return SCB_OK;
}

int ensure_arena(scb_ctx* ctx, int n, int hp, int wp) {
  Arena& A = ctx->arena;
  if (A.base && A.n == n && A.hp == hp && A.wp == wp) return SCB_OK;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  const size_t need = arena_layout(n, ctx->in_nc, hp, wp, nullptr, nullptr, arena_opts(ctx));
  if (A.base && A.bytes < need) {
    cudaFree(A.base);
    A.base = nullptr;
    A.bytes = 0;
  }
  if (!A.base) {
    // admission before allocating (`memguard::check_cuda`, src/memguard.rs:262-285):
    // refuse what cannot fit; if free memory cannot be read, let cudaMalloc decide
    size_t free_b = 0, total_b = 0;
    const bool query_ok = cudaMemGetInfo(&free_b, &total_b) == cudaSuccess;
    if (!query_ok) cudaGetLastError();  // not sticky: clear it
    if (admit_arena(need, query_ok, free_b) == Admit::refuse)
      return fail(ctx, SCB_ENOMEM, admit_message(n, hp, wp, need, free_b));
    cudaError_t e = cudaMalloc(&A.base, need);
    if (e != cudaSuccess) {
      A.base = nullptr;
      cudaGetLastError();
      return fail(ctx, SCB_ENOMEM, std::string("arena allocation refused: ") + cudaGetErrorString(e));
    }
    A.bytes = need;
    note_mem(ctx);
  }
  A.n = n;
  A.hp = hp;
  A.wp = wp;
  arena_layout(n, ctx->in_nc, hp, wp, &A, nullptr, arena_opts(ctx));
  return build_plan(ctx, A);
}

int exchange_nccl(scb_ctx* ctx, Arena& A, const Op& op, cudaStream_t st) {
  if (!A.banded || A.band.nranks == 1) return SCB_OK;
  std::string err;
  const NcclApi* nc = nccl_api(err);
  if (!nc || !ctx->nccl) return fail(ctx, SCB_EINVAL, err.empty() ? "band group not initialised" : err);
  const size_t bytes = (size_t)kHalo * op.xchg_row;
  char* first = op.xchg_base + (size_t)op.xchg_row0 * op.xchg_row;                      // first working rows
  char* last = op.xchg_base + (size_t)(op.xchg_row0 + op.xchg_rows - kHalo) * op.xchg_row;  // last working rows
  char* halo_top = op.xchg_base + (size_t)(op.xchg_row0 - kHalo) * op.xchg_row;
  char* halo_bot = op.xchg_base + (size_t)(op.xchg_row0 + op.xchg_rows) * op.xchg_row;
  const int r = A.band.rank;
  ncclResult_t e = nc->GroupStart();
  if (e == ncclSuccess && !A.band.top) {
    e = nc->Send(first, bytes, ncclUint8, r - 1, ctx->nccl, st);
    if (e == ncclSuccess) e = nc->Recv(halo_top, bytes, ncclUint8, r - 1, ctx->nccl, st);
  }
  if (e == ncclSuccess && !A.band.bottom) {
    e = nc->Send(last, bytes, ncclUint8, r + 1, ctx->nccl, st);
    if (e == ncclSuccess) e = nc->Recv(halo_bot, bytes, ncclUint8, r + 1, ctx->nccl, st);
  }
  const ncclResult_t e2 = nc->GroupEnd();
  if (e == ncclSuccess) e = e2;
  if (e != ncclSuccess) return fail(ctx, SCB_ECUDA, std::string("halo exchange: ") + nc->GetErrorString(e));
  return SCB_OK;
}

// Rank `rank` of `nranks` gets a contiguous run of the padded image's 64-row blocks.
bool band_of(int hp, int rank, int nranks, Band& b, std::string& err) {
  const int nblk = hp / 64;
  if (nranks < 1 || rank < 0 || rank >= nranks) {
    err = "band rank out of range";
    return false;
  }
  if (nblk < nranks) {
    err = "the padded image has " + std::to_string(nblk) + " 64-row blocks, fewer than the " +
          std::to_string(nranks) + " bands asked for";
    return false;
  }
  const int b0 = (int)((long)rank * nblk / nranks), b1 = (int)((long)(rank + 1) * nblk / nranks);
  b.rank = rank;
  b.nranks = nranks;
  b.R0 = 64 * b0;
  b.rows = 64 * (b1 - b0);
  b.top = rank == 0;
  b.bottom = rank == nranks - 1;
  return true;
}

// Allocate (zeroed: edge halo rows must read as zero) and plan one band's arena.
int ensure_band_arena(scb_ctx* ctx, Arena& A, const Band& band, int hp, int wp) {
  if (A.base && A.banded && A.hp == hp && A.wp == wp && A.band.R0 == band.R0 && A.band.rows == band.rows &&
      A.band.nranks == band.nranks && !A.ops.empty())
    return SCB_OK;
  const size_t need = arena_layout(1, ctx->in_nc, hp, wp, nullptr, &band, arena_opts(ctx));
  if (A.base && A.bytes < need) {
    cudaFree(A.base);
    A.base = nullptr;
    A.bytes = 0;
  }
  if (!A.base) {
    cudaError_t e = cudaMalloc(&A.base, need);
    if (e != cudaSuccess) {
      A.base = nullptr;
      cudaGetLastError();
      return fail(ctx, SCB_ENOMEM, std::string("band arena allocation refused: ") + cudaGetErrorString(e));
    }
    A.bytes = need;
    note_mem(ctx);
  }
  CKC(ctx, cudaMemset(A.base, 0, A.bytes), "band arena clear");
  CKC(ctx, cudaDeviceSynchronize(), "band arena clear");
  A.n = 1;
  A.hp = hp;
  A.wp = wp;
  A.banded = true;
  A.band = band;
  arena_layout(1, ctx->in_nc, hp, wp, &A, &band, arena_opts(ctx));
  return build_plan(ctx, A);
}

void free_arena(Arena& A) {
  if (A.base) cudaFree(A.base);
  A = Arena{};
}

// One warp waits, with a limit of `limit_ns`, on an mbarrier that nothing ever
// arrives on: the bounded wait runs out, records SCB_ERR_WAIT_PROBE in the device
// error word and returns. It exercises the path every kernel takes when a
// handshake is lost, without a fault: the kernel holds no TMEM and issues no copies.
__global__ void wait_probe_kernel(unsigned long long limit_ns) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    mbar_fence_init();
  }
  __syncwarp();
  if (threadIdx.x == 0) mbar_wait_limit(&bar, 0, SCB_ERR_WAIT_PROBE, limit_ns);
  __syncwarp();
}

// Load every kernel of the library on the current device now. With lazy module
// loading (the CUDA 12 default) a kernel's code is otherwise uploaded, into newly
// allocated device memory, at its first launch; scb_create calls this so that no
// later call - scb_forward_dev_noalloc's first one included - loads or allocates
// anything for code. Querying a kernel's attributes loads it.
cudaError_t preload_kernels() {
  cudaFuncAttributes fa;
  cudaError_t e = cudaSuccess;
#define SCB_PRELOAD_T(BN, BK, GEO) \
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, gemm_tc_kernel<BN, BK, GEO, true>);
#define SCB_PRELOAD_D(BN, BK, GEO) \
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, gemm_tc_kernel<BN, BK, GEO, false>);
#define SCB_PRELOAD_P(BN, BK, GEO) \
  if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, gemm_tc_kernel<BN, BK, GEO, true, true>);
  SCB_GEMM_VARIANTS(SCB_PRELOAD_T, SCB_PRELOAD_D, SCB_PRELOAD_P)
#undef SCB_PRELOAD_T
#undef SCB_PRELOAD_D
#undef SCB_PRELOAD_P
  const void* others[] = {(const void*)window_attn_kernel,     (const void*)trans32_ws_kernel,
                          (const void*)trans64_ws_kernel,      (const void*)mlp_fused_kernel<128>,
                          (const void*)mlp_fused_kernel<256>,  (const void*)head_tc_kernel,
                          (const void*)tail_tc_kernel,         (const void*)wait_probe_kernel,
                          (const void*)trans32_mp_kernel,      (const void*)conv_pair_kernel<64>,
                          (const void*)conv_pair_kernel<128>};
  for (const void* f : others)
    if (e == cudaSuccess) e = cudaFuncGetAttributes(&fa, f);
  return e;
}

int check_device_error(scb_ctx* ctx) {
  unsigned v = 0;
  CKC(ctx, cudaMemcpyFromSymbol(&v, scb::g_device_error, sizeof v), "read device error word");
  if (v) {
    unsigned z = 0;
    cudaMemcpyToSymbol(scb::g_device_error, &z, sizeof z);
    return fail(ctx, SCB_EDEVICE, "a kernel gave up on a bounded wait (device error code " + std::to_string(v) + ")");
  }
  return SCB_OK;
}

bool geom_ok(scb_ctx* ctx, int n, int c, int h, int w) {
  if (n <= 0 || h <= 0 || w <= 0) {
    fail(ctx, SCB_EINVAL, "empty image");
    return false;
  }
  if (c != ctx->in_nc) {
    fail(ctx, SCB_EINVAL, "the image has " + std::to_string(c) + " channels, the weights take " + std::to_string(ctx->in_nc));
    return false;
  }
  return true;
}

}  // namespace

// ============================================================================
// C ABI
// ============================================================================
extern "C" {

int scb_create(const scb_tensor* tensors, int n_tensors, int in_nc, int dim, int head_dim, int window,
               const int config[7], int device, scb_ctx** out) {
  if (!out) return fail(nullptr, SCB_EINVAL, "out is NULL");
  *out = nullptr;
  if (in_nc != 1 && in_nc != 3) return fail(nullptr, SCB_EINVAL, "in_nc must be 1 or 3");
  if (dim != 64 || head_dim != 32 || window != 8)
    return fail(nullptr, SCB_EINVAL, "only dim 64, head_dim 32, window 8 exist (src/weights.rs:204-280)");
  if (!tensors || n_tensors <= 0) return fail(nullptr, SCB_ENOWEIGHT, "no tensors");
  int cfg[7];
  for (int i = 0; i < 7; ++i) {
    cfg[i] = config ? config[i] : 4;
    if (cfg[i] < 1 || cfg[i] > 16) return fail(nullptr, SCB_EINVAL, "config entries must be 1..16");
  }
  Table tab;
  for (int i = 0; i < n_tensors; ++i) {
    if (!tensors[i].name) return fail(nullptr, SCB_EINVAL, "tensor with NULL name");
    tab.by_name[tensors[i].name] = &tensors[i];
  }
  Blob blob;
  struct Pending {
    size_t w11, w12, wc0, wc2, wqkv, wproj, w0, w2, b11, b12, bqkv, bproj, b0, b2, l1g, l1b, l2g, l2b, rp;
    size_t wqkv_f, w0_f, bqkv_f, b0_f;
    int c;
  };
  std::vector<Pending> pend[7];
  size_t o_down[3], o_up[3], o_head16, o_tail16;

  auto need = [&](const std::string& nm, std::initializer_list<int64_t> sh) -> const float* {
    const float* p = tab.get(nm, sh);
    return p;
  };
  // m_head / m_tail: fp16 K-major tiles for their tensor-core kernels
  const float* p = need("m_head.0.weight", {dim, in_nc, 3, 3});
  if (!p) return fail(nullptr, SCB_ENOWEIGHT, tab.err);
  p = need("m_tail.0.weight", {in_nc, dim, 3, 3});
  if (!p) return fail(nullptr, SCB_ENOWEIGHT, tab.err);
  {
    // m_tail as the tail kernel's B operand: row 3 * tap + co, K = ci (rows 27..31
    // and those of absent output channels zero)
    std::vector<float> t16((size_t)32 * dim, 0.f);
    for (int co = 0; co < in_nc; ++co)
      for (int ci = 0; ci < dim; ++ci)
        for (int k = 0; k < 9; ++k) t16[((size_t)3 * k + co) * dim + ci] = p[((size_t)co * dim + ci) * 9 + k];
    o_tail16 = blob.half(t16);
    const float* hw = tab.get("m_head.0.weight", {dim, in_nc, 3, 3});
    std::vector<float> h16((size_t)dim * 32, 0.f);
    for (int co = 0; co < dim; ++co)
      for (int k = 0; k < in_nc * 9; ++k) h16[(size_t)co * 32 + k] = hw[(size_t)co * in_nc * 9 + k];
    o_head16 = blob.half(h16);
  }

  for (int s = 0; s < 7; ++s) {
    const int c = dim << kStageLevel[s], t = c / 2, heads = t / 32;
    const int first = s >= 4 ? 1 : 0;
    for (int i = 0; i < cfg[s]; ++i) {
      const std::string pre = std::string("m_") + kStageName[s] + "." + std::to_string(first + i);
      const std::string tb = pre + ".trans_block";
      Pending pd{};
      pd.c = c;
      auto half_of = [&](const std::string& nm, std::initializer_list<int64_t> sh, size_t& off) {
        const float* q = need(nm, sh);
        if (!q) return false;
        size_t cnt = 1;
        for (auto d : sh) cnt *= (size_t)d;
        off = blob.half(std::vector<float>(q, q + cnt));
        return true;
      };
      auto f32_of = [&](const std::string& nm, std::initializer_list<int64_t> sh, size_t& off) {
        const float* q = need(nm, sh);
        if (!q) return false;
        size_t cnt = 1;
        for (auto d : sh) cnt *= (size_t)d;
        off = blob.f32(q, cnt);
        return true;
      };
      // 3x3 conv weights: [co][ci][ky][kx] -> [co][ky][kx][ci]
      auto conv3_of = [&](const std::string& nm, size_t& off) {
        const float* q = need(nm, {t, t, 3, 3});
        if (!q) return false;
        std::vector<float> r((size_t)t * t * 9);
        for (int co = 0; co < t; ++co)
          for (int ci = 0; ci < t; ++ci)
            for (int k = 0; k < 9; ++k) r[((size_t)co * 9 + k) * t + ci] = q[((size_t)co * t + ci) * 9 + k];
        off = blob.half(r);
        return true;
      };
      bool ok = half_of(pre + ".conv1_1.weight", {c, c, 1, 1}, pd.w11) && f32_of(pre + ".conv1_1.bias", {c}, pd.b11) &&
                half_of(pre + ".conv1_2.weight", {c, c, 1, 1}, pd.w12) && f32_of(pre + ".conv1_2.bias", {c}, pd.b12) &&
                conv3_of(pre + ".conv_block.0.weight", pd.wc0) && conv3_of(pre + ".conv_block.2.weight", pd.wc2) &&
                f32_of(tb + ".ln1.weight", {t}, pd.l1g) && f32_of(tb + ".ln1.bias", {t}, pd.l1b) &&
                f32_of(tb + ".ln2.weight", {t}, pd.l2g) && f32_of(tb + ".ln2.bias", {t}, pd.l2b) &&
                half_of(tb + ".msa.embedding_layer.weight", {3 * t, t}, pd.wqkv) &&
                f32_of(tb + ".msa.embedding_layer.bias", {3 * t}, pd.bqkv) &&
                half_of(tb + ".msa.linear.weight", {t, t}, pd.wproj) && f32_of(tb + ".msa.linear.bias", {t}, pd.bproj) &&
                f32_of(tb + ".msa.relative_position_params", {heads, 15, 15}, pd.rp) &&
                half_of(tb + ".mlp.0.weight", {4 * t, t}, pd.w0) && f32_of(tb + ".mlp.0.bias", {4 * t}, pd.b0) &&
                half_of(tb + ".mlp.2.weight", {t, 4 * t}, pd.w2) && f32_of(tb + ".mlp.2.bias", {t}, pd.b2);
      if (!ok) return fail(nullptr, SCB_ENOWEIGHT, tab.err);
      if (t <= 64) {
        // LN1 -> qkv and LN2 -> mlp0 with the LayerNorm affine folded into the
        // linear: W (gamma x_hat + beta) + b = (W diag gamma) x_hat + (b + W beta),
        // computed from the fp32 tensors; the q rows also take the attention scale
        // 32^-1/2 (tools/network_scunet.py:73) and log2(e) (softmax in base 2)
        const float qs = 0.17677669529663687f * 1.4426950408889634f;
        auto fold = [&](const std::string& wn, const std::string& bn, const std::string& gn, const std::string& be,
                        int rows, int qrows, size_t& ow, size_t& ob) {
          const float* W = tab.get(wn, {rows, t});
          const float* B = tab.get(bn, {rows});
          const float* G = tab.get(gn, {t});
          const float* Be = tab.get(be, {t});
          std::vector<float> w((size_t)rows * t), b(rows);
          for (int o = 0; o < rows; ++o) {
            const float sc = o < qrows ? qs : 1.f;
            double acc = B[o];
            for (int i = 0; i < t; ++i) {
              w[(size_t)o * t + i] = W[(size_t)o * t + i] * G[i] * sc;
              acc += (double)W[(size_t)o * t + i] * Be[i];
            }
            b[o] = (float)(acc * sc);
          }
          ow = blob.half(w);
          ob = blob.f32(b.data(), b.size());
        };
        fold(tb + ".msa.embedding_layer.weight", tb + ".msa.embedding_layer.bias", tb + ".ln1.weight",
             tb + ".ln1.bias", 3 * t, t, pd.wqkv_f, pd.bqkv_f);
        fold(tb + ".mlp.0.weight", tb + ".mlp.0.bias", tb + ".ln2.weight", tb + ".ln2.bias", 4 * t, 0, pd.w0_f,
             pd.b0_f);
      }
      pend[s].push_back(pd);
    }
    if (s < 3) {  // m_down{k}.{cfg}: [2c][c][2][2] -> [co][dy][dx][ci]
      const std::string nm = std::string("m_") + kStageName[s] + "." + std::to_string(cfg[s]) + ".weight";
      const float* q = need(nm, {2 * c, c, 2, 2});
      if (!q) return fail(nullptr, SCB_ENOWEIGHT, tab.err);
      std::vector<float> r((size_t)2 * c * c * 4);
      for (int co = 0; co < 2 * c; ++co)
        for (int ci = 0; ci < c; ++ci)
          for (int k = 0; k < 4; ++k) r[((size_t)co * 4 + k) * c + ci] = q[((size_t)co * c + ci) * 4 + k];
      o_down[s] = blob.half(r);
    }
    if (s >= 4) {  // m_up{k}.0: [ci=2c][co=c][2][2] -> [(dy,dx,co)][ci]
      const std::string nm = std::string("m_") + kStageName[s] + ".0.weight";
      const float* q = need(nm, {2 * c, c, 2, 2});
      if (!q) return fail(nullptr, SCB_ENOWEIGHT, tab.err);
      std::vector<float> r((size_t)2 * c * c * 4);
      for (int ci = 0; ci < 2 * c; ++ci)
        for (int co = 0; co < c; ++co)
          for (int k = 0; k < 4; ++k) r[((size_t)k * c + co) * (2 * c) + ci] = q[((size_t)ci * c + co) * 4 + k];
      o_up[s - 4] = blob.half(r);
    }
  }

  scb_ctx* ctx = new scb_ctx();
  ctx->device = device;
  ctx->in_nc = in_nc;
  ctx->dim = dim;
  memcpy(ctx->config, cfg, sizeof cfg);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) {
    delete ctx;
    return fail(nullptr, SCB_ECUDA, std::string("cudaSetDevice: ") + cudaGetErrorString(e));
  }
  int major = 0, minor = 0;
  cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, device);
  cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, device);
  if (major != 10) {
    delete ctx;
    return fail(nullptr, SCB_ECUDA, "this library is built for sm_100a (B200); device has compute capability " +
                                        std::to_string(major) + "." + std::to_string(minor));
  }
  cudaDeviceGetAttribute(&ctx->sms, cudaDevAttrMultiProcessorCount, device);
  e = cudaStreamCreateWithFlags(&ctx->stream, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->h2d, cudaStreamNonBlocking);
  if (e == cudaSuccess) e = cudaStreamCreateWithFlags(&ctx->d2h, cudaStreamNonBlocking);
  for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
    e = cudaEventCreateWithFlags(&ctx->ev_in[b], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_comp[b], cudaEventDisableTiming);
    if (e == cudaSuccess) e = cudaEventCreateWithFlags(&ctx->ev_out[b], cudaEventDisableTiming);
  }
  if (e == cudaSuccess) e = cudaMalloc(&ctx->wblob, blob.host.size());
  if (e == cudaSuccess) e = cudaMemcpy(ctx->wblob, blob.host.data(), blob.host.size(), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    std::string m = std::string("weight upload: ") + cudaGetErrorString(e);
    scb_destroy(ctx);
    return fail(nullptr, SCB_ECUDA, m);
  }
  ctx->wbytes = blob.host.size();
  note_mem(ctx);
  // Load the device code on this GPU now, and with it the no-allocation scratch
  // array, so that scb_forward_dev_noalloc never loads a module (or allocates) when
  // it is called: looking up a __device__ symbol loads the module that holds it.
  e = cudaGetSymbolAddress(&ctx->noalloc_base, g_noalloc_scratch);
  if (e == cudaSuccess && ctx->noalloc_base) e = preload_kernels();
  if (e != cudaSuccess || !ctx->noalloc_base) {
    std::string m = std::string("loading the device code: ") + cudaGetErrorString(e);
    scb_destroy(ctx);
    return fail(nullptr, SCB_ECUDA, m);
  }
  char* b = ctx->wblob;
  auto H16 = [&](size_t o) { return reinterpret_cast<__half*>(b + o); };
  auto F = [&](size_t o) { return reinterpret_cast<float*>(b + o); };
  ctx->whead16 = H16(o_head16);
  ctx->wtail16 = H16(o_tail16);
  for (int s = 0; s < 3; ++s) ctx->wdown[s] = H16(o_down[s]);
  for (int s = 0; s < 3; ++s) ctx->wup[s] = H16(o_up[s]);
  for (int s = 0; s < 7; ++s)
    for (auto& pd : pend[s]) {
      BlockW bw;
      bw.c = pd.c;
      bw.w11 = H16(pd.w11); bw.w12 = H16(pd.w12); bw.wc0 = H16(pd.wc0); bw.wc2 = H16(pd.wc2);
      bw.wqkv = H16(pd.wqkv); bw.wproj = H16(pd.wproj); bw.w0 = H16(pd.w0); bw.w2 = H16(pd.w2);
      bw.b11 = F(pd.b11); bw.b12 = F(pd.b12); bw.bqkv = F(pd.bqkv); bw.bproj = F(pd.bproj);
      bw.b0 = F(pd.b0); bw.b2 = F(pd.b2); bw.ln1g = F(pd.l1g); bw.ln1b = F(pd.l1b);
      bw.ln2g = F(pd.l2g); bw.ln2b = F(pd.l2b); bw.rp = F(pd.rp);
      if (pd.c / 2 <= 64) {
        bw.wqkv_f = H16(pd.wqkv_f); bw.w0_f = H16(pd.w0_f); bw.bqkv_f = F(pd.bqkv_f); bw.b0_f = F(pd.b0_f);
      }
      ctx->blocks[s].push_back(bw);
    }
  g_create_error.clear();
  *out = ctx;
  return SCB_OK;
}

int scb_forward_dev(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y, int y_dtype,
                    void* stream) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !y) return fail(ctx, SCB_EINVAL, "NULL image pointer");
  if (!geom_ok(ctx, n, c, h, w)) return SCB_EINVAL;
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  int r = ensure_arena(ctx, n, hp, wp);
  if (r) return r;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  r = run_ops(ctx, ctx->arena, x, x_dtype == SCB_U8, y, y_dtype == SCB_U8, c, h, w, st);
  if (r) return r;
  ctx->err.clear();
  return SCB_OK;
}

int scb_forward_dev_noalloc(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y,
                            int y_dtype, void* stream) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !y) return fail(ctx, SCB_EINVAL, "NULL image pointer");
  if (!geom_ok(ctx, n, c, h, w)) return SCB_EINVAL;
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  if ((long)n * hp * wp > kNoAllocMaxPixels) {
    char buf[256];
    snprintf(buf, sizeof buf,
             "%d image(s) of %dx%d pad to %ld pixels; the no-allocation forward takes at most %ld padded pixels "
             "(one 64x128 or two 64x64 images) - use scb_forward_dev for larger batches",
             n, h, w, (long)n * hp * wp, kNoAllocMaxPixels);
    return fail(ctx, SCB_EINVAL, buf);
  }
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if (!ctx->noalloc_base) return fail(ctx, SCB_EINVAL, "the no-allocation scratch was not reserved by scb_create");
  Arena& A = ctx->noalloc;
  if (!(A.n == n && A.hp == hp && A.wp == wp && !A.ops.empty())) {
    const size_t need = arena_layout(n, ctx->in_nc, hp, wp, nullptr, nullptr, arena_opts(ctx));
    if (need > kNoAllocBytes) return fail(ctx, SCB_EINVAL, "no-allocation scratch is too small for this geometry");
    A = Arena{};
    A.base = static_cast<char*>(ctx->noalloc_base);
    A.bytes = kNoAllocBytes;
    A.n = n;
    A.hp = hp;
    A.wp = wp;
    arena_layout(n, ctx->in_nc, hp, wp, &A, nullptr, arena_opts(ctx));
    int r = build_plan(ctx, A);
    if (r) {
      A.ops.clear();
      return r;
    }
  }
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  int r = run_ops(ctx, A, x, x_dtype == SCB_U8, y, y_dtype == SCB_U8, c, h, w, st, /*allow_profile=*/false);
  if (r) return r;
  ctx->err.clear();
  return SCB_OK;
}

// The host-pointer forward runs the batch as a pipeline of chunks of images: the
// copy in of chunk k + 1 and the copy out of chunk k - 1 (each on its own stream,
// so both copy engines work) overlap the compute of chunk k. Two staging slots each
// way; events keep a slot from being overwritten while a copy or the forward still
// reads it.
int forward_host_pipelined(scb_ctx* ctx, const char* x, int x_u8, int n, int c, int h, int w, char* y, int y_u8) {
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  const int chunk = std::min(n, ctx->host_chunk > 0 ? ctx->host_chunk
                                                    : (int)std::max(1L, kHostChunkPixels / ((long)hp * wp)));
  const size_t img_in = (size_t)c * h * w * (x_u8 ? 1 : 4), img_out = (size_t)c * h * w * (y_u8 ? 1 : 4);
  const size_t slot = ((size_t)chunk * c * h * w * 4 + 1023) & ~size_t(1023);
  if (ctx->io_bytes < 4 * slot) {
    if (ctx->io) cudaFree(ctx->io);
    ctx->io = nullptr;
    ctx->io_bytes = 0;
    if (cudaMalloc(&ctx->io, 4 * slot) != cudaSuccess) {
      cudaGetLastError();
      ctx->io = nullptr;
      return fail(ctx, SCB_ENOMEM, "host staging allocation refused");
    }
    ctx->io_bytes = 4 * slot;
    note_mem(ctx);
  }
  ctx->io_slot = slot;
  cudaStream_t cs = ctx->stream;
  for (int i0 = 0, k = 0; i0 < n; i0 += chunk, ++k) {
    const int b = k & 1, m = std::min(chunk, n - i0);
    int r = ensure_arena(ctx, m, hp, wp);
    if (r) return r;
    char* in = ctx->io + b * slot;
    char* out = ctx->io + (2 + b) * slot;
    if (k >= 2) CKC(ctx, cudaStreamWaitEvent(ctx->h2d, ctx->ev_comp[b], 0), "wait");  // chunk k-2 read `in`
    CKC(ctx, cudaMemcpyAsync(in, x + i0 * img_in, m * img_in, cudaMemcpyHostToDevice, ctx->h2d), "H2D");
    CKC(ctx, cudaEventRecord(ctx->ev_in[b], ctx->h2d), "event");
    CKC(ctx, cudaStreamWaitEvent(cs, ctx->ev_in[b], 0), "wait");
    if (k >= 2) CKC(ctx, cudaStreamWaitEvent(cs, ctx->ev_out[b], 0), "wait");  // chunk k-2's `out` copied
    r = run_ops(ctx, ctx->arena, in, x_u8, out, y_u8, c, h, w, cs);
    if (r) return r;
    CKC(ctx, cudaEventRecord(ctx->ev_comp[b], cs), "event");
    CKC(ctx, cudaStreamWaitEvent(ctx->d2h, ctx->ev_comp[b], 0), "wait");
    CKC(ctx, cudaMemcpyAsync(y + i0 * img_out, out, m * img_out, cudaMemcpyDeviceToHost, ctx->d2h), "D2H");
    CKC(ctx, cudaEventRecord(ctx->ev_out[b], ctx->d2h), "event");
  }
  return SCB_OK;
}

int scb_forward_host(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, void* y, int y_dtype) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !y) return fail(ctx, SCB_EINVAL, "NULL image pointer");
  if (!geom_ok(ctx, n, c, h, w)) return SCB_EINVAL;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  int r = forward_host_pipelined(ctx, static_cast<const char*>(x), x_dtype == SCB_U8, n, c, h, w,
                                 static_cast<char*>(y), y_dtype == SCB_U8);
  // whatever happened, nothing of this call may still be running when it returns
  const cudaError_t e1 = cudaStreamSynchronize(ctx->h2d), e2 = cudaStreamSynchronize(ctx->stream),
                    e3 = cudaStreamSynchronize(ctx->d2h);
  if (r) return r;
  CKC(ctx, e1, "copy in");
  CKC(ctx, e2, "forward");
  CKC(ctx, e3, "copy out");
  r = check_device_error(ctx);
  if (r) return r;
  ctx->err.clear();
  return SCB_OK;
}

int scb_forward(scb_ctx* ctx, const float* x_nchw, int c, int hp, int wp, float* y_nchw) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (hp % 64 || wp % 64) return fail(ctx, SCB_EINVAL, "scb_forward takes a plane already padded to a multiple of 64");
  return scb_forward_host(ctx, x_nchw, SCB_F32, 1, c, hp, wp, y_nchw, SCB_F32);
}

int scb_forward_bands(scb_ctx* ctx, int nbands, const void* x, int x_dtype, int c, int h, int w, void* y,
                      int y_dtype, void* stream) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !y) return fail(ctx, SCB_EINVAL, "NULL image pointer");
  if (!geom_ok(ctx, 1, c, h, w)) return SCB_EINVAL;
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  if ((int)ctx->vbands.size() != nbands) {
    for (Arena& A : ctx->vbands) free_arena(A);
    ctx->vbands.assign(std::max(nbands, 0), Arena{});
  }
  std::string err;
  for (int b = 0; b < nbands; ++b) {
    Band band;
    if (!band_of(hp, b, nbands, band, err)) return fail(ctx, SCB_EINVAL, err);
    const int r = ensure_band_arena(ctx, ctx->vbands[b], band, hp, wp);
    if (r) return r;
  }
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  const Io io{x, x_dtype == SCB_U8, y, y_dtype == SCB_U8, c, h, w};
  const size_t nops = ctx->vbands[0].ops.size();
  for (const Arena& A : ctx->vbands)
    if (A.ops.size() != nops) return fail(ctx, SCB_EINVAL, "band plans differ in length");
  int launches = 0;
  for (size_t k = 0; k < nops; ++k) {  // lockstep: op k of every band before op k + 1
    if (ctx->vbands[0].ops[k].kind == Op::XCHG) {
      const int r = exchange_local(ctx, ctx->vbands, k, st);
      if (r) return r;
      continue;
    }
    for (Arena& A : ctx->vbands) {
      const cudaError_t e = exec_op(ctx, A, A.ops[k], io, st);
      if (e != cudaSuccess) return cuda_fail(ctx, e, "kernel launch");
      ++launches;
    }
  }
  ctx->last_launches = launches;
  ctx->err.clear();
  return SCB_OK;
}

int scb_band_unique_id(void* id_out) {
  if (!id_out) return fail(nullptr, SCB_EINVAL, "id_out is NULL");
  std::string err;
  const NcclApi* nc = nccl_api(err);
  if (!nc) return fail(nullptr, SCB_EINVAL, err);
  ncclUniqueId id;
  const ncclResult_t e = nc->GetUniqueId(&id);
  if (e != ncclSuccess) return fail(nullptr, SCB_ECUDA, std::string("ncclGetUniqueId: ") + nc->GetErrorString(e));
  memcpy(id_out, &id, sizeof id);
  return SCB_OK;
}

int scb_band_init(scb_ctx* ctx, const void* id, int rank, int nranks) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!id || rank < 0 || nranks < 1 || rank >= nranks) return fail(ctx, SCB_EINVAL, "band rank / id");
  std::string err;
  const NcclApi* nc = nccl_api(err);
  if (!nc) return fail(ctx, SCB_EINVAL, err);
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  ctx->band_ready = false;
  if (ctx->nccl) {
    nc->CommDestroy(ctx->nccl);
    ctx->nccl = nullptr;
  }
  ncclUniqueId uid;
  memcpy(&uid, id, sizeof uid);
  const ncclResult_t e = nc->CommInitRank(&ctx->nccl, nranks, uid, rank);
  if (e != ncclSuccess) {
    ctx->nccl = nullptr;
    return fail(ctx, SCB_ECUDA, std::string("ncclCommInitRank: ") + nc->GetErrorString(e));
  }
  ctx->band_rank = rank;
  ctx->band_nranks = nranks;
  ctx->band_ready = true;
  free_arena(ctx->band_arena);
  ctx->err.clear();
  return SCB_OK;
}

int scb_forward_band(scb_ctx* ctx, const void* x, int x_dtype, int c, int h, int w, void* y, int y_dtype,
                     void* stream) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !y) return fail(ctx, SCB_EINVAL, "NULL image pointer");
  if (!geom_ok(ctx, 1, c, h, w)) return SCB_EINVAL;
  if (!ctx->band_ready || (ctx->band_nranks > 1 && !ctx->nccl))
    return fail(ctx, SCB_EINVAL, "no band group: scb_band_init has not run, or the group was aborted");
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  std::string err;
  Band band;
  if (!band_of(hp, ctx->band_rank, ctx->band_nranks, band, err)) return fail(ctx, SCB_EINVAL, err);
  int r = ensure_band_arena(ctx, ctx->band_arena, band, hp, wp);
  if (r) return r;
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  r = run_ops(ctx, ctx->band_arena, x, x_dtype == SCB_U8, y, y_dtype == SCB_U8, c, h, w, st);
  if (r) return r;
  ctx->err.clear();
  return SCB_OK;
}

int scb_band_sync(scb_ctx* ctx, void* stream, int timeout_ms) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (timeout_ms < 0) return fail(ctx, SCB_EINVAL, "timeout_ms must be >= 0");
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  cudaStream_t st = stream ? static_cast<cudaStream_t>(stream) : ctx->stream;
  std::string err;
  const NcclApi* nc = ctx->nccl ? nccl_api(err) : nullptr;
  cudaError_t serr = cudaSuccess;
  ncclResult_t aerr = ncclSuccess;
  auto query = [&]() {
    const cudaError_t q = cudaStreamQuery(st);
    if (q == cudaSuccess) return 0;
    if (q == cudaErrorNotReady) return 1;
    serr = q;
    return -1;
  };
  auto async_err = [&]() {
    if (!nc) return 0;
    ncclResult_t a = ncclSuccess;
    if (nc->CommGetAsyncError(ctx->nccl, &a) != ncclSuccess) a = ncclSystemError;
    if (a == ncclInProgress) return 0;
    aerr = a;
    return a == ncclSuccess ? 0 : 1;
  };
  auto now = []() {
    timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
  };
  auto nap = []() {
    timespec ts{0, 200000};  // 0.2 ms
    nanosleep(&ts, nullptr);
  };
  const Watch w = watch_until(query, async_err, now, nap, timeout_ms / 1000.0);
  if (w == Watch::done) {
    const int r = check_device_error(ctx);
    if (r) return r;
    ctx->err.clear();
    return SCB_OK;
  }
  if (w == Watch::stream_error) return cuda_fail(ctx, serr, "banded forward");
  // a peer failed or the exchange did not finish in time: abort the group so that
  // NCCL's kernels on this GPU stop waiting for the peer; the context needs a new
  // scb_band_init before the next banded forward
  std::string why = w == Watch::peer_error
                        ? std::string("a band peer failed: ") + (nc ? nc->GetErrorString(aerr) : "?")
                        : "the banded forward did not finish within " + std::to_string(timeout_ms) + " ms";
  if (nc && ctx->nccl) {
    nc->CommAbort(ctx->nccl);
    ctx->nccl = nullptr;
  }
  ctx->band_ready = false;
  return fail(ctx, SCB_ECUDA, why + "; the band group was aborted (call scb_band_init again)");
}

int scb_need_bytes(int n, int in_nc, int hp, int wp, size_t* bytes) {
  if (!bytes || n <= 0 || hp <= 0 || wp <= 0 || hp % 64 || wp % 64 || (in_nc != 1 && in_nc != 3)) return SCB_EINVAL;
  *bytes = arena_layout(n, in_nc, hp, wp, nullptr);
  return SCB_OK;
}

int scb_check_admission(scb_ctx* ctx, int n, int hp, int wp, size_t* need, size_t* avail) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (n <= 0 || hp <= 0 || wp <= 0 || hp % 64 || wp % 64) return fail(ctx, SCB_EINVAL, "geometry must be padded to 64");
  const size_t nb = arena_layout(n, ctx->in_nc, hp, wp, nullptr, nullptr, arena_opts(ctx));
  if (need) *need = nb;
  if (avail) *avail = 0;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  size_t free_b = 0, total_b = 0;
  const bool query_ok = cudaMemGetInfo(&free_b, &total_b) == cudaSuccess;
  if (!query_ok) cudaGetLastError();
  // the arena this context holds now is freed or reused by the next forward
  const size_t have = free_b + ctx->arena.bytes;
  if (avail) *avail = query_ok ? have : 0;
  if (admit_arena(nb, query_ok, have) == Admit::refuse) return fail(ctx, SCB_ENOMEM, admit_message(n, hp, wp, nb, have));
  ctx->err.clear();
  return SCB_OK;
}

void scb_footprint(const scb_ctx* ctx, size_t* weights_bytes, size_t* scratch_bytes) {
  if (weights_bytes) *weights_bytes = ctx ? ctx->wbytes : 0;
  if (scratch_bytes) {
    size_t s = 0;
    if (ctx) {
      s = ctx->arena.bytes + ctx->band_arena.bytes + ctx->io_bytes;
      for (const Arena& A : ctx->vbands) s += A.bytes;
    }
    *scratch_bytes = s;
  }
}

void scb_release_scratch(scb_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  if (ctx->h2d) cudaStreamSynchronize(ctx->h2d);
  if (ctx->d2h) cudaStreamSynchronize(ctx->d2h);
  free_arena(ctx->arena);
  free_arena(ctx->band_arena);
  for (Arena& A : ctx->vbands) free_arena(A);
  ctx->vbands.clear();
  if (ctx->io) cudaFree(ctx->io);
  ctx->io = nullptr;
  ctx->io_bytes = 0;
}

int scb_set_option(scb_ctx* ctx, int option, int value) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (option == SCB_OPT_FUSE_TRANS || option == SCB_OPT_RESIDUAL32) {
    (option == SCB_OPT_FUSE_TRANS ? ctx->fuse_trans : ctx->residual32) = value != 0;
    ctx->arena.ops.clear();
    ctx->arena.n = 0;  // re-plan on the next forward
    ctx->noalloc.ops.clear();
    ctx->noalloc.n = 0;
    ctx->band_arena.ops.clear();
    for (Arena& A : ctx->vbands) A.ops.clear();
    return SCB_OK;
  }
  if (option == SCB_OPT_TRANS32_LANES || option == SCB_OPT_FUSE_PAIR || option == SCB_OPT_GEMM_PAIRS) {
    (option == SCB_OPT_TRANS32_LANES ? ctx->trans32_lanes
     : option == SCB_OPT_FUSE_PAIR   ? ctx->fuse_pair
                                     : ctx->gemm_pairs) = value != 0;
    ctx->arena.ops.clear();
    ctx->arena.n = 0;
    ctx->noalloc.ops.clear();
    ctx->noalloc.n = 0;
    ctx->band_arena.ops.clear();
    for (Arena& A : ctx->vbands) A.ops.clear();
    return SCB_OK;
  }
  if (option == SCB_OPT_CONV3_TWIN) {
    ctx->conv3_twin = value != 0;
    ctx->arena.ops.clear();
    ctx->arena.n = 0;
    ctx->noalloc.ops.clear();
    ctx->noalloc.n = 0;
    ctx->band_arena.ops.clear();
    for (Arena& A : ctx->vbands) A.ops.clear();
    return SCB_OK;
  }
  if (option == SCB_OPT_HOST_CHUNK) {
    if (value < 0) return fail(ctx, SCB_EINVAL, "SCB_OPT_HOST_CHUNK must be >= 0");
    ctx->host_chunk = value;
    return SCB_OK;
  }
  return fail(ctx, SCB_EINVAL, "unknown option " + std::to_string(option));
}

int scb_set_profiling(scb_ctx* ctx, int on) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  ctx->profiling = on != 0;
  return SCB_OK;
}

int scb_profile_read(scb_ctx* ctx, int* tags, double* flops, float* ms, int max) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!ctx->profiling || ctx->prof_tags.empty()) return 0;
  const int n = (int)std::min<size_t>(ctx->prof_tags.size(), (size_t)std::max(max, 0));
  for (int i = 0; i < n; ++i) {
    float t = -1.f;
    if (cudaEventSynchronize(ctx->events[i + 1]) == cudaSuccess) cudaEventElapsedTime(&t, ctx->events[i], ctx->events[i + 1]);
    if (tags) tags[i] = ctx->prof_tags[i];
    if (flops) flops[i] = ctx->prof_flops[i];
    if (ms) ms[i] = t;
  }
  return n;
}

int scb_profile_bytes(const scb_ctx* ctx, double* bytes, int max) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!ctx->profiling || ctx->prof_bytes.empty()) return 0;
  const int n = (int)std::min<size_t>(ctx->prof_bytes.size(), (size_t)std::max(max, 0));
  for (int i = 0; i < n && bytes; ++i) bytes[i] = ctx->prof_bytes[i];
  return n;
}

int scb_profile_kernels(const scb_ctx* ctx, char* buf, size_t cap) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  const std::string& s = ctx->profiling ? ctx->prof_kernels : std::string();
  if (buf && cap) {
    const size_t m = std::min(cap - 1, s.size());
    memcpy(buf, s.data(), m);
    buf[m] = 0;
  }
  return (int)s.size();
}

const char* scb_last_error(const scb_ctx* ctx) { return ctx ? ctx->err.c_str() : g_create_error.c_str(); }

int scb_last_launch_count(const scb_ctx* ctx) { return ctx ? ctx->last_launches : 0; }

void scb_destroy(scb_ctx* ctx) {
  if (!ctx) return;
  cudaSetDevice(ctx->device);
  if (ctx->stream) cudaStreamSynchronize(ctx->stream);
  scb_release_scratch(ctx);
  free_arena(ctx->band_arena);
  for (Arena& A : ctx->vbands) free_arena(A);
  if (ctx->nccl) {
    std::string err;
    if (const NcclApi* nc = nccl_api(err)) nc->CommDestroy(ctx->nccl);
  }
  for (cudaEvent_t ev : ctx->events) cudaEventDestroy(ev);
  for (int b = 0; b < 2; ++b)
    for (cudaEvent_t ev : {ctx->ev_in[b], ctx->ev_comp[b], ctx->ev_out[b]})
      if (ev) cudaEventDestroy(ev);
  if (ctx->wblob) cudaFree(ctx->wblob);
  if (ctx->stream) cudaStreamDestroy(ctx->stream);
  if (ctx->h2d) cudaStreamDestroy(ctx->h2d);
  if (ctx->d2h) cudaStreamDestroy(ctx->d2h);
  delete ctx;
}

// ---------------------------------------------------------------------------- probes
static int probe_finish(scb_ctx* ctx, cudaError_t e) {
  if (e != cudaSuccess) return cuda_fail(ctx, e, "probe launch");
  CKC(ctx, cudaStreamSynchronize(ctx->stream), "probe");
  int r = check_device_error(ctx);
  if (r) return r;
  ctx->err.clear();
  return SCB_OK;
}

int scb_probe_gemm(scb_ctx* ctx, const void* a16, int M, int K, const void* b16, int N, const float* bias, int act,
                   const void* res16, void* out16, float* out32) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  std::string err;
  Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
  GemmOp g{};
  if (!mk.flat(g, static_cast<const __half*>(a16), M, K, K, static_cast<const __half*>(b16), N))
    return fail(ctx, SCB_EINVAL, err);
  if (reinterpret_cast<uintptr_t>(bias) % 16)
    return fail(ctx, SCB_EINVAL, "bias must be 16-byte aligned (the epilogue reads it as float4)");
  g.e.bias = bias;
  g.e.act = act;
  g.e.res16 = static_cast<const __half*>(res16);
  g.e.res16_ld = N;
  g.e.out16 = static_cast<__half*>(out16);
  g.e.out16_ld = N;
  g.e.out32 = out32;
  g.e.out32_ld = N;
  if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
  return probe_finish(ctx, launch_gemm(g, ctx->sms, ctx->stream));
}

int scb_probe_conv3x3(scb_ctx* ctx, const void* x16, int n, int H, int W, int cin, const void* w16, int cout, int act,
                      const void* res16, void* out16) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  std::string err;
  Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
  GemmOp g{};
  if (!mk.conv3(g, static_cast<const __half*>(x16), n, H, W, cin, cin, static_cast<const __half*>(w16), cout))
    return fail(ctx, SCB_EINVAL, err);
  g.e.act = act;
  g.e.res16 = static_cast<const __half*>(res16);
  g.e.res16_ld = cout;
  g.e.out16 = static_cast<__half*>(out16);
  g.e.out16_ld = cout;
  if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
  return probe_finish(ctx, launch_gemm(g, ctx->sms, ctx->stream));
}

int scb_probe_down2(scb_ctx* ctx, const void* x16, int n, int H, int W, int cin, const void* w16, int cout,
                    float* out32, void* out16) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  std::string err;
  Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
  GemmOp g{};
  if (!mk.down2(g, static_cast<const __half*>(x16), n, H, W, cin, static_cast<const __half*>(w16), cout))
    return fail(ctx, SCB_EINVAL, err);
  g.e.out32 = out32;
  g.e.out32_ld = cout;
  g.e.out16 = static_cast<__half*>(out16);
  g.e.out16_ld = cout;
  if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
  return probe_finish(ctx, launch_gemm(g, ctx->sms, ctx->stream));
}

int scb_probe_up2(scb_ctx* ctx, const void* x16, int n, int h, int w, int cin, const void* w16, int cout,
                  float* out32, void* out16) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  std::string err;
  Maker mk{&err, ctx->gemm_pairs, ctx->conv3_twin};
  GemmOp g{};
  if (!mk.up2(g, static_cast<const __half*>(x16), n, h, w, cin, static_cast<const __half*>(w16), cout))
    return fail(ctx, SCB_EINVAL, err);
  g.e.out32 = out32;
  g.e.out32_ld = cout;
  g.e.out16 = static_cast<__half*>(out16);
  g.e.out16_ld = cout;
  if (!mk.finish_epi(g)) return fail(ctx, SCB_EINVAL, err);
  return probe_finish(ctx, launch_gemm(g, ctx->sms, ctx->stream));
}

int scb_probe_mlp(scb_ctx* ctx, int stage, int index, const void* a16, void* z16, int tokens) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (stage < 0 || stage > 6 || index < 0 || index >= ctx->config[stage] || tokens <= 0)
    return fail(ctx, SCB_EINVAL, "block index / token count");
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  const BlockW& bw = ctx->blocks[stage][index];
  std::string err;
  Op mo{};
  if (!mlp_op(mo, bw, static_cast<const __half*>(a16), static_cast<__half*>(z16), bw.c / 2, tokens, err))
    return fail(ctx, SCB_EINVAL, err);
  return probe_finish(ctx, launch_mlp(mo, ctx->sms, ctx->stream));
}

int scb_probe_attention(scb_ctx* ctx, const void* qkv16, int n, int H, int W, int t, int shift, const float* rp,
                        void* out16) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (t % 32 || t / 32 > 8 || H % 8 || W % 8 || (shift != 0 && shift != 4)) return fail(ctx, SCB_EINVAL, "attention geometry");
  Op op{};
  op.kind = Op::ATTN;
  Region R;
  R.n = n;
  R.H = R.rows = R.H_image = H;
  R.W = W;
  op.attn = AttnGeom{win_geom(R, shift != 0), t, t / 32, 3L * t, (long)t};
  op.attn_in = static_cast<const __half*>(qkv16);
  op.attn_out = static_cast<__half*>(out16);
  op.attn_rp = rp;
  return probe_finish(ctx, launch_attn(op, ctx->stream));
}

int scb_probe_block(scb_ctx* ctx, int stage, int index, const float* x32, int n, int H, int W, float* y32) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (stage < 0 || stage > 6 || index < 0 || index >= ctx->config[stage]) return fail(ctx, SCB_EINVAL, "block index");
  if (H % 8 || W % 8 || n <= 0) return fail(ctx, SCB_EINVAL, "block plane must be a multiple of 8");
  const BlockW& bw = ctx->blocks[stage][index];
  const int c = bw.c;
  // A private arena sized as a full-resolution plane of n*H*W pixels is more than enough.
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  Arena tmp;
  const long P = (long)n * H * W;
  const size_t bytes = (size_t)P * (c * 2 /*xs*/ + c * 2 /*y, yt*/ + c /*hc*/ + c * 2 /*z*/ + c /*a*/ + c /*o*/ + c * 4 /*qh*/) + 16 * 1024;
  char* base = nullptr;
  CKC(ctx, cudaMalloc(&base, bytes), "probe scratch");
  size_t off = 0;
  auto take = [&](size_t b) {
    char* p = base + off;
    off += (b + 1023) & ~size_t(1023);
    return p;
  };
  __half* xs = reinterpret_cast<__half*>(take((size_t)P * c * 2));
  tmp.y = reinterpret_cast<__half*>(take((size_t)P * c));
  tmp.yt = reinterpret_cast<__half*>(take((size_t)P * c));
  tmp.hc = reinterpret_cast<__half*>(take((size_t)P * c));
  tmp.z = reinterpret_cast<__half*>(take((size_t)P * c * 2));
  tmp.a = reinterpret_cast<__half*>(take((size_t)P * c));
  tmp.o = reinterpret_cast<__half*>(take((size_t)P * c));
  tmp.qh = reinterpret_cast<__half*>(take((size_t)P * c * 4));
  // shadow of x: a one-off conversion on the device
  std::vector<float> hx((size_t)P * c);
  cudaError_t e = cudaMemcpy(hx.data(), x32, hx.size() * 4, cudaMemcpyDeviceToHost);
  std::vector<__half> hs(hx.size());
  for (size_t i = 0; i < hx.size(); ++i) hs[i] = __float2half_rn(hx[i]);
  if (e == cudaSuccess) e = cudaMemcpy(xs, hs.data(), hs.size() * 2, cudaMemcpyHostToDevice);
  if (e != cudaSuccess) {
    cudaFree(base);
    return cuda_fail(ctx, e, "probe staging");
  }
  std::vector<Op> ops;
  std::string err;
  Region R;
  R.n = n;
  R.H = R.rows = R.H_image = H;
  R.W = W;
  if (!block_ops(ctx, ops, bw, tmp, R, x32, y32, xs, nullptr, (index % 2) == 1, err)) {
    cudaFree(base);
    return fail(ctx, SCB_EINVAL, err);
  }
  int r = SCB_OK;
  for (const Op& op : ops) {
    switch (op.kind) {
      case Op::GEMM: e = launch_gemm(op.gemm, ctx->sms, ctx->stream); break;
      case Op::TRANS: e = launch_trans(op, ctx->sms, ctx->stream); break;
      case Op::ATTN: e = launch_attn(op, ctx->stream); break;
      case Op::MLP: e = launch_mlp(op, ctx->sms, ctx->stream); break;
      case Op::PAIR: e = launch_pair(op, ctx->sms, ctx->stream); break;
      default: e = cudaErrorInvalidValue;  // a block builds none of the other kinds
    }
    if (e != cudaSuccess) break;
  }
  r = probe_finish(ctx, e);
  cudaFree(base);
  return r;
}

int scb_probe_head(scb_ctx* ctx, const void* x, int x_dtype, int n, int c, int h, int w, float* x1_32, void* x1_16) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!x || !x1_32 || !x1_16) return fail(ctx, SCB_EINVAL, "NULL pointer");
  if (!geom_ok(ctx, n, c, h, w)) return SCB_EINVAL;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  const double P = (double)n * hp * wp;
  Op head{};
  std::string err;
  const uint64_t d[2] = {64, (uint64_t)P}, s32[1] = {256}, s16[1] = {128};
  const uint32_t b32[2] = {32, 128}, b16[2] = {64, 128};
  if (!encode_map(&head.head_m32, x1_32, 2, d, s32, b32, 4, 128, err) ||
      !encode_map(&head.head_m16, x1_16, 2, d, s16, b16, 2, 128, err))
    return fail(ctx, SCB_EINVAL, err);
  const HeadGeom g{n, c, h, w, hp, wp, x_dtype == SCB_U8, 0, hp};
  return probe_finish(ctx, launch_head(ctx, x, g, head, ctx->stream));
}

int scb_probe_tail(scb_ctx* ctx, const void* s16, int n, int c, int h, int w, void* y, int y_dtype) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (!s16 || !y) return fail(ctx, SCB_EINVAL, "NULL pointer");
  if (!geom_ok(ctx, n, c, h, w)) return SCB_EINVAL;
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  const int hp = (h + 63) / 64 * 64, wp = (w + 63) / 64 * 64;
  Op tail{};
  std::string err;
  const uint64_t dims[4] = {64, (uint64_t)wp, (uint64_t)hp, (uint64_t)n};
  const uint64_t str[3] = {64 * 2, (uint64_t)wp * 64 * 2, (uint64_t)hp * wp * 64 * 2};
  const uint32_t box[4] = {64, 128, 1, 1};
  if (!encode_map(&tail.tail_map, s16, 4, dims, str, box, 2, 128, err)) return fail(ctx, SCB_EINVAL, err);
  TailGeom g{};
  g.n = n;
  g.H = hp;
  g.W = wp;
  g.row0 = 0;
  g.rows_out = hp;
  g.row_off = 0;
  g.strips = (wp + TAIL_COLS - 1) / TAIL_COLS;
  g.chunks = (hp + TAIL_ROWS - 1) / TAIL_ROWS;
  g.c = c;
  g.h = h;
  g.w = w;
  g.u8 = y_dtype == SCB_U8;
  return probe_finish(ctx, launch_tail(ctx, y, g, tail, ctx->stream));
}

int scb_probe_wait_timeout(scb_ctx* ctx, int limit_us) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (limit_us < 1 || limit_us > 1000000) return fail(ctx, SCB_EINVAL, "limit_us must be 1 .. 1000000");
  CKC(ctx, cudaSetDevice(ctx->device), "cudaSetDevice");
  wait_probe_kernel<<<1, 32, 0, ctx->stream>>>(1000ull * (unsigned long long)limit_us);
  return probe_finish(ctx, cudaGetLastError());
}

int scb_mem_report(const scb_ctx* ctx, size_t* high_water, size_t* live, size_t* fixed) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  if (high_water) *high_water = ctx->high_water;
  if (live) *live = live_bytes(ctx);
  if (fixed) *fixed = ctx->noalloc_base ? kNoAllocBytes : 0;
  return SCB_OK;
}

int scb_profile_report(scb_ctx* ctx, char* buf, size_t cap) {
  if (!ctx) return fail(nullptr, SCB_EINVAL, "ctx is NULL");
  static const char* kClass[] = {"head", "tail", "conv1x1", "conv3x3", "qkv", "attention", "proj", "mlp0",
                                 "mlp2", "down", "up", "trans_fused", "halo", "mlp_fused"};
  const int n = (int)ctx->prof_tags.size();
  std::vector<int> tags(n);
  std::vector<double> fl(n);
  std::vector<float> ms(n);
  const int got = ctx->profiling ? scb_profile_read(ctx, tags.data(), fl.data(), ms.data(), n) : 0;
  // per class: launches, device ms, algorithmic FLOPs; most expensive first
  struct Row { int launches = 0; double ms = 0, flops = 0; };
  std::vector<Row> rows(14);
  double total = 0;
  for (int i = 0; i < got; ++i) {
    if (tags[i] < 0 || tags[i] >= 14 || ms[i] < 0) continue;
    rows[tags[i]].launches++;
    rows[tags[i]].ms += ms[i];
    rows[tags[i]].flops += fl[i];
    total += ms[i];
  }
  std::vector<int> order;
  for (int k = 0; k < 14; ++k)
    if (rows[k].launches) order.push_back(k);
  std::sort(order.begin(), order.end(), [&](int a, int b) { return rows[a].ms > rows[b].ms; });
  std::string out;
  if (got > 0) {
    char line[160];
    snprintf(line, sizeof line, "  ---- device time per op class (total %.2f ms, %d launches) ----\n", total, got);
    out += line;
    for (int k : order) {
      snprintf(line, sizeof line, "  %9.3f ms  %5.1f %%  %6d launches  %8.1f TFLOP/s  %s\n", rows[k].ms,
               total > 0 ? 100.0 * rows[k].ms / total : 0.0, rows[k].launches,
               rows[k].ms > 0 ? rows[k].flops / (rows[k].ms * 1e-3) / 1e12 : 0.0, kClass[k]);
      out += line;
    }
  }
  if (buf && cap) {
    const size_t m = std::min(cap - 1, out.size());
    memcpy(buf, out.data(), m);
    buf[m] = 0;
  }
  return (int)out.size();
}

}  // extern "C"
