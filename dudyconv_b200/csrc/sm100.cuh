// sm100.cuh -- thin inline-PTX wrappers for the Blackwell (sm_100a) features the
// tensor-core kernels use: mbarriers, TMA (cp.async.bulk.tensor), tcgen05 MMA with
// TMEM accumulators, and the shared-memory matrix / instruction descriptors.
//
// Every wait is bounded: a wait that does not complete within kWaitLimitNs sets the
// kernel's error word and returns false, so a lost arrival ends the kernel with an
// error status instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace dudy {
namespace sm100 {

// error codes written to the device error word
enum : int { kErrNone = 0, kErrWaitTimeout = 1 };
// wait sites of the bounded-wait self-test (dudy_selftest_wait_timeout)
constexpr int kSelftestSite = 901;
// wait sites of the peer-memory grad_mix exchange (xrank.cu): kXrankSite + peer rank
constexpr int kXrankSite = 950;

constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The device error record err[0..3]: the first timeout stores its wait-site id in err[0]
// (nonzero), and the block, thread and loop counter of that wait in err[1..3].
__device__ __forceinline__ void record_timeout(int *err, int site, int aux) {
  if (atomicCAS(err, 0, site) == 0) {
    err[1] = (int)blockIdx.x;
    err[2] = (int)threadIdx.x;
    err[3] = aux;
    __threadfence();
  }
}

// The polling loop of mbar_wait_limit, kept out of line: the kernels wait at many sites,
// and inlining the loop (timer reads, abort checks, error record) at each of them would
// multiply the code every warp role runs, at the cost of instruction-cache misses.
static __device__ __noinline__ bool mbar_wait_slow(uint64_t *bar, uint32_t parity, int *err,
                                            volatile int *abort, uint64_t limit_ns, int site,
                                            int aux) {
  const uint64_t t0 = global_ns();
  uint32_t spins = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++spins & 63u) == 0) {
      if (*abort) return false;
      if (global_ns() - t0 > limit_ns) {
        record_timeout(err, site, aux);
        *abort = 1;
        return false;
      }
    }
  }
  return true;
}

// Wait until the phase with `parity` has completed. Returns false (and records a
// timeout in the error record and *abort) if it does not complete within `limit_ns`,
// or if another role of the CTA has already aborted. One inline poll, then the loop.
__device__ __forceinline__ bool mbar_wait_limit(uint64_t *bar, uint32_t parity, int *err,
                                                volatile int *abort, uint64_t limit_ns,
                                                int site, int aux) {
  if (mbar_try_wait(bar, parity)) return true;
  return mbar_wait_slow(bar, parity, err, abort, limit_ns, site, aux);
}

// mbar_wait_limit with the kernels' limit (kWaitLimitNs).
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, int *err,
                                          volatile int *abort, int site = kErrWaitTimeout,
                                          int aux = 0) {
  return mbar_wait_limit(bar, parity, err, abort, kWaitLimitNs, site, aux);
}

// Warp-uniform bounded wait: every lane polls, and the warp proceeds only if all lanes
// saw the phase complete, so warp-collective instructions that follow (tcgen05.ld) run
// converged even when the wait times out.
__device__ __forceinline__ bool mbar_wait_warp(uint64_t *bar, uint32_t parity, int *err,
                                               volatile int *abort, int site = kErrWaitTimeout,
                                               int aux = 0) {
  const bool ok = mbar_wait(bar, parity, err, abort, site, aux);
  return __all_sync(0xffffffffu, ok) != 0;
}

// ---------------------------------------------------------------------------------------
// TMA (tiled tensor copies, global -> shared, completion on an mbarrier)
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// shared -> global tiled store (bulk async-group completion; out-of-range elements of the
// box are not written). Coordinates must be non-negative.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap *map, const void *src, int x,
                                             int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
          reinterpret_cast<uint64_t>(map)),
      "r"(x), "r"(y), "r"(smem_u32(src))
      : "memory");
}

__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// this thread's committed bulk stores have finished reading their shared-memory source
__device__ __forceinline__ void bulk_wait_group_read0() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}

// this thread's committed bulk stores have completed
__device__ __forceinline__ void bulk_wait_group0() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

// bring a tensor tile into L2 (no shared-memory destination, no completion tracking)
__device__ __forceinline__ void tma_prefetch_2d(const CUtensorMap *map, int x, int y) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y)
               : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap *map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// make this thread's generic-proxy shared-memory writes visible to the async proxy
// (tensor core operand reads)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------------------------------
// tcgen05: TMEM allocation, MMA, commit, loads
// ---------------------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
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

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (fp16/bf16 inputs, fp32 accumulate)
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16. A is M x K in TMEM: lane m holds row m,
// K elements packed two 16-bit values per 32-bit column (K = 16 -> 8 columns).
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                            uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers; thread i writes lane (base+i).
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// wait until this thread's earlier tcgen05.st have completed
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// arrive on `bar` once every previously issued tcgen05.mma of this thread has completed
__device__ __forceinline__ void umma_commit(uint64_t *bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp receives lane (base+i).
// The load and its wait are one asm statement, so no use of the destination registers
// can be scheduled before the data has arrived.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "{\n tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n"
      " tcgen05.wait::ld.sync.aligned;\n}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 32 consecutive 32-bit columns (raw bits), load and wait in one statement.
__device__ __forceinline__ void tmem_ld32_raw(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "{\n tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      " tcgen05.wait::ld.sync.aligned;\n}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]),
        "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]),
        "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// ---------------------------------------------------------------------------------------
// descriptors
// ---------------------------------------------------------------------------------------
// shared-memory layout (swizzle) codes of the tcgen05 matrix descriptor, bits [61,64)
enum : uint32_t { kSwNone = 0, kSw128 = 2, kSw64 = 4, kSw32 = 6 };

// Matrix descriptor: start address, leading / stride byte offsets (16-byte units),
// version 1 (bits [46,48)), base offset 0, layout code. Addresses are shared-window.
__device__ __forceinline__ uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes,
                                               uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;
  d |= (uint64_t)(layout & 7u) << 61;
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
//   is_bf16: operand format (0 = fp16, 1 = bf16, same for A and B)
//   a_mn / b_mn: 1 if that operand is MN-major in shared memory, 0 if K-major
__host__ __device__ constexpr uint32_t make_idesc_f16(int M, int N, int is_bf16, int a_mn,
                                                      int b_mn) {
  return (1u << 4)                              // D format: f32
         | ((uint32_t)is_bf16 << 7)             // A format
         | ((uint32_t)is_bf16 << 10)            // B format
         | ((uint32_t)a_mn << 15)               // A major
         | ((uint32_t)b_mn << 16)               // B major
         | ((uint32_t)(N >> 3) << 17)           // N / 8
         | ((uint32_t)(M >> 4) << 24);          // M / 16
}

// byte offset of 16-byte chunk `c` (0..7) of 128-byte row `r` in a SWIZZLE_128B tile
__device__ __forceinline__ uint32_t sw128_off(uint32_t r, uint32_t c) {
  return r * 128u + ((c ^ (r & 7u)) << 4);
}

}  // namespace sm100
}  // namespace dudy
