// sm100.cuh - thin inline-PTX wrappers for the Blackwell (sm_100a) features the kernels use:
// mbarriers with bounded waits, TMA tile loads, TMEM allocation, tcgen05 MMA / commit / load,
// and the shared-memory and instruction descriptors of tcgen05.mma kind::f16.
//
// Every wait is bounded (kWaitTimeoutNs of %globaltimer time). A wait that expires returns
// false; the caller then records a failure bit in the caller-provided status word and unwinds,
// so a broken pipeline ends the kernel with an error the host can read instead of hanging.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace dv3 {

constexpr uint64_t kWaitTimeoutNs = 2000000000ull;  // 2 s; a healthy wait lasts microseconds

// Failure bits written to status[0].
constexpr uint32_t kErrProducerWait = 1u << 0;
constexpr uint32_t kErrMmaWait = 1u << 1;
constexpr uint32_t kErrEpilogueWait = 1u << 2;
constexpr uint32_t kErrAttentionWait = 1u << 3;
constexpr uint32_t kErrSelfTestWait = 1u << 4;   // the bounded-wait self-test's expired wait
constexpr uint32_t kErrSelfTestAbort = 1u << 5;  // the self-test's second role unwound on abort

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report(uint32_t *status, uint32_t bit) {
  if (status) atomicOr(status, bit);
}

// Programmatic dependent launch. A kernel launched with programmatic stream serialization may
// start while the kernel before it on the stream is still running: it does its set-up (barrier
// init, TMEM allocation, staging of weights), then pdl_wait() blocks until that kernel has
// completed and its writes are visible, before any read of activations or any global write.
// pdl_trigger() lets the next kernel start its own set-up once every CTA of this one has issued
// it. Both are no-ops for a kernel launched without the attribute.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile(
      "{\n\t.reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint32_t addr, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(addr), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking: has the phase with the given parity completed?
__device__ __forceinline__ bool mbar_test(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait until the phase with the given parity has completed. Returns false if the wait expired
// (after `timeout_ns` of %globaltimer time) or another role raised `abort`.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, volatile int *abort,
                                          uint64_t timeout_ns = kWaitTimeoutNs) {
  const uint32_t addr = smem_u32(bar);
  if (mbar_try_wait(addr, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
#pragma unroll 1
    for (int i = 0; i < 16; ++i)
      if (mbar_try_wait(addr, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > timeout_ns) return false;
  }
}

// Bounded wait that ignores the abort flag: used while unwinding, to let copies and MMAs already
// in flight land before the CTA releases its shared memory and TMEM.
__device__ __forceinline__ bool mbar_drain(uint64_t *bar, uint32_t parity) {
  volatile int never = 0;
  return mbar_wait(bar, parity, &never);
}

// ---------------------------------------------------------------------------------------------
// TMA (bulk tensor copies global -> shared, completion counted on an mbarrier)
// ---------------------------------------------------------------------------------------------
// This CTA's share of an L2 prefetch of [p, p + bytes) (16-byte aligned, a multiple of 16
// bytes): 64 KB pieces dealt round-robin over the grid, each one cp.async.bulk.prefetch.L2 with
// no shared memory and nothing to wait for. Used for weights of a later kernel, which no kernel
// writes.
__device__ __forceinline__ void l2_prefetch_share(const void *p, size_t bytes) {
  constexpr size_t kPiece = 65536;
  for (size_t off = blockIdx.x * kPiece; off < bytes; off += gridDim.x * kPiece) {
    const uint32_t n = static_cast<uint32_t>(bytes - off < kPiece ? bytes - off : kPiece);
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(
                     reinterpret_cast<uint64_t>(static_cast<const uint8_t *>(p) + off)),
                 "r"(n)
                 : "memory");
  }
}

// Drop this CTA's share (thread t of nt) of a dead buffer from L2 without writing it back
// (discard.global.L2: afterwards the lines read as indeterminate until written again), so that
// an intermediate no kernel reads any more neither costs a DRAM write-back nor holds L2 space.
// [p, p + bytes) is whole 128-byte lines. Only for a buffer whose readers have completed (after
// griddepcontrol.wait) and that this kernel does not write.
__device__ __forceinline__ void l2_discard_share(const void *p, size_t bytes, int t, int nt) {
  const size_t lines = bytes >> 7;
  for (size_t i = static_cast<size_t>(blockIdx.x) * nt + t; i < lines;
       i += static_cast<size_t>(gridDim.x) * nt)
    asm volatile("discard.global.L2 [%0], 128;" ::"l"(
                     reinterpret_cast<uint64_t>(static_cast<const uint8_t *>(p) + (i << 7)))
                 : "memory");
}

__device__ __forceinline__ void tma_prefetch_map(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Load the box at element coordinates (x = innermost, y = row) into shared memory. x times
// the element size must be a multiple of 16 bytes.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 3D box at (x, y, z): x innermost (x times the element size a multiple of 16 bytes).
__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int32_t x, int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
__device__ __forceinline__ void tma_store_3d(const CUtensorMap *map, const void *src, int32_t x,
                                             int32_t y, int32_t z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
      : "memory");
}

// Store a box from shared memory to global memory at element coordinates (x, y); the box's
// rows past the tensor's extent are not written. Completion is tracked per thread in bulk
// groups (bulk_commit / bulk_wait_*).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's bulk groups are incomplete (writes done).
template <int N>
__device__ __forceinline__ void bulk_wait() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Make this thread's generic-proxy shared-memory writes visible to the async proxy (TMA and
// the tensor cores read shared memory through it).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------------
// TMEM and tcgen05
// ---------------------------------------------------------------------------------------------
// Whole-warp operations. `ncols` is a power of two >= 32; the TMEM address lands in *dst.
__device__ __forceinline__ void tmem_alloc(uint32_t *dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], f16 inputs, f32 accumulate. One thread issues.
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc]: A (M rows in TMEM lanes, 2 f16 per 32-bit column along K)
// is read from tensor memory. One thread issues.
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05.mma this thread issued so far has completed.
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

#define DV3_R32(r)                                                                               \
  "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]),           \
      "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]),   \
      "+r"(r[14]), "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]),             \
      "+r"(r[20]), "+r"(r[21]), "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]),             \
      "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]), "+r"(r[30]), "+r"(r[31])

// tcgen05.wait::ld that also takes the loaded registers as read-write operands: the compiler
// sees the values as produced by the wait, so no use of them can be scheduled before it.
__device__ __forceinline__ void tmem_wait_ld(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : DV3_R32(r)::"memory");
}

// Orders a second batch of loaded registers after a preceding tmem_wait_ld (volatile asm
// statements keep their order).
__device__ __forceinline__ void tmem_regs_ready(uint32_t (&r)[32]) {
  asm volatile("" : DV3_R32(r));
}

// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane taddr.lane + i.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
      "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]),
      "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]),
      "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]),
      "r"(r[30]), "r"(r[31])
      : "memory");
}

// 32 lanes x 16 (or 8) consecutive 32-bit columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_regs_ready16(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]),
                 "+r"(r[6]), "+r"(r[7]), "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]),
                 "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]));
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7])
      : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// Barrier over the `nthreads` threads (a multiple of 32) that use named barrier `id` (1..15).
__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Load 32 columns and wait for them.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t (&r)[32]) {
  tmem_ld32(taddr, r);
  tmem_wait_ld(r);
}

// Load two 32-column chunks with one wait.
__device__ __forceinline__ void tmem_load32x2(uint32_t ta, uint32_t (&a)[32], uint32_t tb,
                                              uint32_t (&b)[32]) {
  tmem_ld32(ta, a);
  tmem_ld32(tb, b);
  tmem_wait_ld(a);
  tmem_regs_ready(b);
}

// Shared-memory matrix descriptor for a tile stored with the 128-byte swizzle: rows of 128
// bytes, 8-row groups 1024 bytes apart (the stride byte offset), 1024-byte aligned groups.
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused by swizzled
// K-major tiles; 1), stride byte offset >> 4 [32,46), descriptor version 1 [46,48),
// layout type 2 = 128-byte swizzle [61,64).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// The same for a K-major tile of 32-byte rows (16 f16 columns, one MMA's K) stored with the
// 32-byte swizzle (the layout TMA writes for a 16-column box with CU_TENSOR_MAP_SWIZZLE_32B):
// 8-row groups 256 bytes apart, 256-byte aligned groups, layout type 6 = 32-byte swizzle.
__device__ __forceinline__ uint64_t sw32_desc(uint32_t smem_addr) {
  return static_cast<uint64_t>((smem_addr >> 4) & 0x3FFFu) | (1ull << 16) |
         (static_cast<uint64_t>(256 >> 4) << 32) | (1ull << 46) | (6ull << 61);
}

// Instruction descriptor of tcgen05.mma kind::f16 with f16 A and B and an f32 accumulator:
// D format f32 (1) at [4,6), A/B format f16 (0) at [7,10) / [10,13), A major [15], B major [16]
// (0 = K-major, 1 = MN-major), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t idesc_f16_f32(uint32_t m, uint32_t n, bool b_mn_major) {
  return (1u << 4) | (b_mn_major ? (1u << 16) : 0u) | ((n >> 3) << 17) | ((m >> 4) << 24);
}

// ---------------------------------------------------------------------------------------------
// small numeric helpers
// ---------------------------------------------------------------------------------------------
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t *>(&h);
}

// Hardware base-2 exponential approximation (one MUFU operation; subnormal results flush to 0).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Hardware tanh approximation (one MUFU operation).
__device__ __forceinline__ float tanh_approx(float x) {
  float y;
  asm("tanh.approx.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// silu(a) = a * sigmoid(a) = h + h * tanh(h) with h = a / 2.
__device__ __forceinline__ float silu(float a) {
  const float h = 0.5f * a;
  return fmaf(h, tanh_approx(h), h);
}

// The folded LayerNorm's aux row of a token row with statistics (mean, rstd): 16 f16 values
// (-mean_hi, -mean_lo, -mean_hi, r_hi, r_lo, r_hi, 0, ...) with r = 1 / rstd, each *_lo the f16
// of what the f16 *_hi leaves over; the tensor cores multiply it with the weight aux (s_hi,
// s_hi, s_lo, c_hi, c_hi, c_lo, 0, ...) into -mean s + r c. 32 bytes at dst (16-byte aligned).
__device__ __forceinline__ void store_row_aux(__half *dst, float mean, float rstd) {
  const float r = 1.0f / rstd;
  const __half mh = __float2half_rn(-mean), rh = __float2half_rn(r);
  const __half ml = __float2half_rn(-mean - __half2float(mh));
  const __half rl = __float2half_rn(r - __half2float(rh));
  auto pk = [](__half a, __half b) {
    return static_cast<uint32_t>(__half_as_ushort(a)) |
           (static_cast<uint32_t>(__half_as_ushort(b)) << 16);
  };
  uint4 *d = reinterpret_cast<uint4 *>(dst);
  d[0] = make_uint4(pk(mh, ml), pk(mh, rh), pk(rl, rh), 0u);
  d[1] = make_uint4(0u, 0u, 0u, 0u);
}

__device__ __forceinline__ float2 unpack_half2(uint32_t v) {
  __half2 h = *reinterpret_cast<__half2 *>(&v);
  return __half22float2(h);
}

}  // namespace dv3
