// Thin inline-PTX layer for sm_100a: mbarriers, TMA tensor loads, tcgen05
// (TMEM allocation, UMMA issue/commit, TMEM loads) and the shared-memory matrix
// descriptors the UMMA reads its operands through.
//
// Every wait here is BOUNDED: a wait that has not completed after ~1 s of
// %globaltimer records a code in the device error word and returns false, so a
// kernel that loses a handshake ends with an error the host reads, never a hang.
#pragma once
#include <cstdint>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

namespace scb {

// Device-wide error word: 0 = ok; otherwise the first failure's code (see
// SCB_ERR_* below). Read and cleared by the host after every forward. The library
// is one translation unit, so this header is included exactly once.
__device__ unsigned int g_device_error = 0;

enum : unsigned {
  SCB_ERR_WAIT_FULL = 1,   // MMA waited for a TMA stage that never landed
  SCB_ERR_WAIT_EMPTY = 2,  // producer waited for a stage the MMA never released
  SCB_ERR_WAIT_ACC = 3,    // epilogue waited for an accumulator never committed
  SCB_ERR_WAIT_ACC_FREE = 4,
  SCB_ERR_WAIT_ATTN = 5,
  SCB_ERR_WAIT_PROBE = 6,  // scb_probe_wait_timeout: a wait nothing completes, by design
};

__device__ __forceinline__ void record_error(unsigned code) {
  atomicCAS(&g_device_error, 0u, code);
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or about `ns` nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete; false (and the error word set to
// `code`) after `limit_ns` of %globaltimer.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t* bar, uint32_t parity, unsigned code, uint64_t limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255u) == 255u) {
      if (globaltimer() - t0 > limit_ns) {
        record_error(code);
        return false;
      }
      __nanosleep(64);
    }
  }
}

// The kernels' waits: ~1 s, far beyond any legitimate stall.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned code) {
  return mbar_wait_limit(bar, parity, code, 1000000000ull);
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor): every load in this library fills its own CTA only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* tmap) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void* dst, const void* tmap, uint64_t* bar, int c0, int c1, int c2,
                                            int c3, int c4) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6, "
      "%7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(tmap), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
      : "memory");
}

// TMA bulk tensor stores (smem -> global), tracked by bulk async-groups of the
// issuing thread. Stores never start at a negative coordinate here; elements past
// the tensor's extent are clipped by the TMA unit.
__device__ __forceinline__ void tma_store_2d(const void* tmap, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}
__device__ __forceinline__ void tma_store_3d(const void* tmap, const void* src, int c0, int c1, int c2) {
  asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2)
               : "memory");
}
__device__ __forceinline__ void tma_store_4d(const void* tmap, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void tma_store_5d(const void* tmap, const void* src, int c0, int c1, int c2, int c3,
                                             int c4) {
  asm volatile("cp.async.bulk.tensor.5d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5, %6}], [%1];" ::"l"(tmap),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// At most N of this thread's committed store groups may still be READING smem.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// At most N of this thread's committed store groups may still be in flight.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Generic-proxy smem writes -> visible to the async proxy (UMMA / TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: TMEM allocation, UMMA, commit, TMEM -> registers
// ---------------------------------------------------------------------------
// Executed by one whole warp. Writes the TMEM base address to *dst_smem.
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (fp16 inputs, fp32 accumulate).
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// The same with A read from tensor memory: `a_tmem` addresses a [128 lanes x K]
// operand whose 32-bit columns each hold two fp16 K elements (lower K in the low
// half); one K step of 16 spans 8 columns. Only B is read from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every UMMA this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// 32 lanes x 32 bit, 16 consecutive columns: thread t of the warp gets row
// (lane base + t), columns [col, col + 16). The _issue form only starts the load:
// several loads can be in flight before one tmem_wait_ld(); tmem_fence16 then ties
// the registers to the wait so no use is scheduled above it.
__device__ __forceinline__ void tmem_ld16_issue(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// The store counterpart: thread t writes row (lane base + t), columns [col, col + 16).
// tmem_wait_st() before anything (an MMA, after a barrier) reads the columns.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])), "r"(__float_as_uint(v[3])),
      "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])), "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])),
      "r"(__float_as_uint(v[8])), "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])),
      "r"(__float_as_uint(v[11])), "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])),
      "r"(__float_as_uint(v[14])), "r"(__float_as_uint(v[15]))
      : "memory");
}
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Raw 32-bit stores of 8 / 16 / 32 consecutive columns of this thread's row.
__device__ __forceinline__ void tmem_st8u(uint32_t taddr, const uint32_t* r) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
               "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
               : "memory");
}
__device__ __forceinline__ void tmem_st16u(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st32u(uint32_t taddr, const uint32_t* r) {
  tmem_st16u(taddr, r);
  tmem_st16u(taddr + 16, r + 16);
}

__device__ __forceinline__ void tmem_fence16(uint32_t* r) {
#pragma unroll
  for (int i = 0; i < 16; ++i) asm volatile("" : "+r"(r[i]));
}

__device__ __forceinline__ void u32_to_f32_16(const uint32_t* r, float* v) {
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// One 32x32b column: thread t of the warp gets row (lane base + t), column `taddr`.
// Waits for the load itself (one value: nothing to overlap it with).
__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r) : "r"(taddr));
  tmem_wait_ld();
  asm volatile("" : "+r"(r));
  return __uint_as_float(r);
}

// One 16-column load, waited for immediately.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float* v) {
  uint32_t r[16];
  tmem_ld16_issue(taddr, r);
  tmem_wait_ld();
  tmem_fence16(r);
  u32_to_f32_16(r, v);
}

// Two / three / four 16-column loads in flight, one wait.
__device__ __forceinline__ void tmem_ld16x2(uint32_t a0, float* v0, uint32_t a1, float* v1) {
  uint32_t r0[16], r1[16];
  tmem_ld16_issue(a0, r0);
  tmem_ld16_issue(a1, r1);
  tmem_wait_ld();
  tmem_fence16(r0);
  tmem_fence16(r1);
  u32_to_f32_16(r0, v0);
  u32_to_f32_16(r1, v1);
}

__device__ __forceinline__ void tmem_ld16x3(uint32_t a0, float* v0, uint32_t a1, float* v1, uint32_t a2, float* v2) {
  uint32_t r0[16], r1[16], r2[16];
  tmem_ld16_issue(a0, r0);
  tmem_ld16_issue(a1, r1);
  tmem_ld16_issue(a2, r2);
  tmem_wait_ld();
  tmem_fence16(r0);
  tmem_fence16(r1);
  tmem_fence16(r2);
  u32_to_f32_16(r0, v0);
  u32_to_f32_16(r1, v1);
  u32_to_f32_16(r2, v2);
}

// ---------------------------------------------------------------------------
// Descriptors
// ---------------------------------------------------------------------------
// Swizzle modes of the K-major canonical layouts this library uses.
enum SwizzleMode : uint32_t { SW_NONE = 0, SW_128B = 2, SW_64B = 4, SW_32B = 6 };

// Shared-memory matrix descriptor (sm100 format): K-major operand whose rows are
// `row_bytes` long (= the swizzle span) and whose 8-row groups are 8*row_bytes apart.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t row_bytes, uint32_t swz) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);              // start address
  d |= (uint64_t)1u << 16;                               // LBO (unused for swizzled K-major) = 16 B
  d |= (uint64_t)(((8u * row_bytes) >> 4) & 0x3FFFu) << 32;  // SBO: 8-row group stride
  d |= (uint64_t)1u << 46;                               // descriptor version (sm100)
  d |= (uint64_t)swz << 61;                              // layout type
  return d;
}

// The same with an explicit 8-row group stride (bytes): an operand whose rows are
// gathered from a larger swizzled tile, groups `sbo` apart.
__device__ __forceinline__ uint64_t make_sdesc_sbo(uint32_t saddr, uint32_t sbo, uint32_t swz) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)1u << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)swz << 61;
  return d;
}

// The general form: leading-dimension and stride byte offsets given explicitly. For
// an MN-major SW128 operand, LBO is the stride between 64-element MN atoms and SBO
// the stride between groups of 8 K rows (128-byte rows, swizzled within 1 KB).
__device__ __forceinline__ uint64_t make_sdesc_lbo_sbo(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swz) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)swz << 61;
  return d;
}

// Instruction descriptor, kind::f16: A = B = fp16, D = fp32, both K-major.
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N) {
  return (1u << 4)                       // D format: f32
         | (0u << 7) | (0u << 10)        // A, B format: f16
         | (0u << 15) | (0u << 16)       // A, B K-major
         | ((uint32_t)(N >> 3) << 17)    // N / 8
         | ((uint32_t)(M >> 4) << 24);   // M / 16
}

// The same with B read MN-major (N contiguous in shared memory).
__host__ __device__ constexpr uint32_t make_idesc_f16_bmn(int M, int N) { return make_idesc_f16(M, N) | (1u << 16); }

// Byte offset of 16-byte chunk `chunk` of row `row` inside a K-major tile whose
// rows are `row_bytes` (= swizzle span: 128, 64 or 32) long, with the tile base
// aligned to 8*row_bytes. Matches the TMA SWIZZLE_{128,64,32}B patterns.
__device__ __forceinline__ uint32_t swz_off(uint32_t row, uint32_t chunk, uint32_t row_bytes) {
  const uint32_t mask = row_bytes / 16 - 1;                 // 7, 3, 1
  const uint32_t phase = (row_bytes == 128) ? (row & 7) : (row_bytes == 64 ? ((row >> 1) & 3) : ((row >> 2) & 1));
  return row * row_bytes + (((chunk ^ phase) & mask) << 4);
}

// 16-byte asynchronous global -> shared copy by this thread (bypassing L1); when
// `valid` is false nothing is read and the 16 bytes are zero-filled. Completion is
// per thread: cp_async_wait_all() makes this thread's copies visible to itself.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all() { asm volatile("cp.async.wait_all;" ::: "memory"); }
// All but this thread's most recent committed group have landed.
__device__ __forceinline__ void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

__device__ __forceinline__ __half2 tanh_approx_h2(__half2 x) {
  uint32_t y;
  asm("tanh.approx.f16x2 %0, %1;" : "=r"(y) : "r"(*reinterpret_cast<const uint32_t*>(&x)));
  return *reinterpret_cast<const __half2*>(&y);
}

// GELU on two fp16 values in the tanh form of Hendrycks & Gimpel,
//   GELU(x) ~= x/2 (1 + tanh(x (a + b x^2))),
// with a, b refitted (minimax over the real line) to the exact-erf GELU of
// nn.GELU() (tools/network_scunet.py:130): a = 0.80015708, b = 0.03470089, max
// |error| 2.7e-4 (the textbook a = sqrt(2/pi), b = 0.044715 a gives 4.7e-4). Used
// where the result is stored as fp16 (the MLP hidden layer); six packed operations
// and one tanh.approx.f16x2 per two values. Large |x| saturates: x^2 -> inf gives
// tanh -> +-1 and GELU -> x or 0.
// 2 GELU(x) = x (1 + tanh(x (a + b x^2))), the form above without its factor 1/2
// (callers fold the 1/2 into the next linear map, exactly, in fp16): five packed
// operations and one tanh.approx.f16x2 per two values.
__device__ __forceinline__ __half2 gelu2_tanh_h2(__half2 x) {
  const __half2 x2 = __hmul2(x, x);
  const __half2 p = __hfma2(__float2half2_rn(0.03470089f), x2, __float2half2_rn(0.80015708f));
  const __half2 t = tanh_approx_h2(__hmul2(x, p));
  return __hfma2(x, t, x);
}

__device__ __forceinline__ __half2 gelu_tanh_h2(__half2 x) {
  const __half2 x2 = __hmul2(x, x);
  const __half2 p = __hfma2(__float2half2_rn(0.03470089f), x2, __float2half2_rn(0.80015708f));
  const __half2 t = tanh_approx_h2(__hmul2(x, p));
  const __half2 hx = __hmul2(__float2half2_rn(0.5f), x);
  return __hfma2(hx, t, hx);
}

// 2^x, hardware approximation (relative error ~2^-22, far below the fp16 rounding
// every consumer of these values applies).
// 2^x on two fp16 values (one MUFU operation for both).
__device__ __forceinline__ uint32_t ex2_approx_h2(uint32_t x) {
  uint32_t y;
  asm("ex2.approx.f16x2 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Where the tokens of 8x8 (shifted) windows live in a stored plane. Token (i, j)
// of window (wr, wc) is pixel (row, (8 wc + j + shift) mod W) with
//   wrap = 1 (the whole image): row = (8 wr + i + shift) mod H - the cyclic roll
//            of tools/network_scunet.py:77, read in place;
//   wrap = 0 (a row band stored with halo rows): row = row_base + 8 wr + i; the
//            band's first and last shifted window rows reach into the halo rows.
// The SW mask needs the window's row in the WHOLE image (gwr0 + wr) mod nwr_global:
// only the image's last window row/column is masked (cuda/scunet.cu:137-147).
struct WinGeom {
  int H, W;                 // stored rows and columns per image
  int shift;                // 0 (W) or 4 (SW)
  int nwr, nwc;             // window rows handled per image, window columns
  long n_windows;           // images * nwr * nwc
  int wrap, row_base;
  int gwr0, nwr_global;
  int store_lo, store_hi;   // stored rows whose outputs are written
};

__device__ __forceinline__ long win_token_pixel(const WinGeom& g, long win, int qi, int qj, bool& last_row,
                                                bool& last_col, bool& store) {
  // 32-bit index arithmetic: a plane that fits in device memory holds far fewer than
  // 2^31 windows; every wrapped coordinate is below twice its period, so one
  // conditional subtraction replaces the modulo
  const unsigned per_img = (unsigned)(g.nwr * g.nwc);
  const unsigned w = (unsigned)win;
  const unsigned img = w / per_img;
  const unsigned wrem = w - img * per_img;
  const int wr = (int)(wrem / (unsigned)g.nwc), wc = (int)wrem - wr * g.nwc;
  int y;
  if (g.wrap) {
    y = wr * 8 + qi + g.shift;
    if (y >= g.H) y -= g.H;
  } else {
    y = g.row_base + wr * 8 + qi;
  }
  int x = wc * 8 + qj + g.shift;
  if (x >= g.W) x -= g.W;
  int gwr = g.gwr0 + wr;
  if (gwr >= g.nwr_global) gwr -= g.nwr_global;
  last_row = g.shift && gwr == g.nwr_global - 1;
  last_col = g.shift && wc == g.nwc - 1;
  store = y >= g.store_lo && y < g.store_hi;
  return ((long)img * g.H + y) * g.W + x;
}

// A thread's window within a persistent loop whose window index grows by a fixed
// step: the image / window-row / window-column split is carried from one pair to
// the next instead of being divided out again (win_token_pixel's arithmetic).
struct WinCursor {
  long win;
  int img, wr, wc;
  __device__ __forceinline__ void init(const WinGeom& g, long w) {
    win = w;
    const unsigned per_img = (unsigned)(g.nwr * g.nwc);
    const unsigned uw = (unsigned)w;
    img = (int)(uw / per_img);
    const unsigned rem = uw - (unsigned)img * per_img;
    wr = (int)(rem / (unsigned)g.nwc);
    wc = (int)rem - wr * g.nwc;
  }
  // step < nwc * nwr is not required: each loop runs step / nwc + 1 times at most
  __device__ __forceinline__ void advance(const WinGeom& g, int step) {
    win += step;
    wc += step;
    while (wc >= g.nwc) {
      wc -= g.nwc;
      if (++wr == g.nwr) {
        wr = 0;
        ++img;
      }
    }
  }
  // the token's pixel, or -1 past the last window; flags as win_token_pixel
  __device__ __forceinline__ long pixel(const WinGeom& g, int qi, int qj, bool& last_row, bool& last_col,
                                        bool& store) const {
    last_row = last_col = store = false;
    if (win >= g.n_windows) return -1;
    int y;
    if (g.wrap) {
      y = wr * 8 + qi + g.shift;
      if (y >= g.H) y -= g.H;
    } else {
      y = g.row_base + wr * 8 + qi;
    }
    int x = wc * 8 + qj + g.shift;
    if (x >= g.W) x -= g.W;
    int gwr = g.gwr0 + wr;
    if (gwr >= g.nwr_global) gwr -= g.nwr_global;
    last_row = g.shift && gwr == g.nwr_global - 1;
    last_col = g.shift && wc == g.nwc - 1;
    store = y >= g.store_lo && y < g.store_hi;
    return ((long)img * g.H + y) * g.W + x;
  }
};

// v[0..1] += (a, b) / v[0..3] += b as fp32x2 adds (Blackwell's paired FP32 pipe: half
// the instructions, the same roundings as scalar adds).
__device__ __forceinline__ void add2_f32x2(float* v, float a, float b) {
  const float2 r = __fadd2_rn(make_float2(v[0], v[1]), make_float2(a, b));
  v[0] = r.x;
  v[1] = r.y;
}
__device__ __forceinline__ void add4_f32x2(float* v, float4 b) {
  add2_f32x2(v, b.x, b.y);
  add2_f32x2(v + 2, b.z, b.w);
}

// max(a, b, c) in one instruction (the three-input form of max.f32, sm_100).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// The maximum of N >= 4 values (N even) with three-input maxes: N/2 instructions
// instead of N - 1, two independent chains.
template <int N>
__device__ __forceinline__ float row_max(const float* s) {
  static_assert(N >= 4 && N % 2 == 0, "row_max: N even, at least 4");
  float m0 = s[0], m1 = s[1];
  int j = 2;
#pragma unroll
  for (; j + 3 < N; j += 4) {
    m0 = fmax3(m0, s[j], s[j + 1]);
    m1 = fmax3(m1, s[j + 2], s[j + 3]);
  }
  if (j < N) m0 = fmax3(m0, s[j], s[j + 1]);
  return fmaxf(m0, m1);
}

__device__ __forceinline__ uint32_t pack_half2(float a, float b) {
  __half2 h = __floats2half2_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

}  // namespace scb
