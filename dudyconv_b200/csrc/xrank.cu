// xrank.cu -- the data-parallel grad_mix exchange, fused into the backward's last kernel.
//
// With the batch sharded over ranks (one GPU each), every rank's backward ends with
// per-CTA fp32 partial sums of grad_mix [D,N] in its workspace, and the data-parallel
// step needs the sum over ranks. Instead of reducing locally, casting, and running a
// separate all-reduce (a cast kernel, the collective's kernel, a copy back), one kernel
// does it all over peer memory:
//   1. a block sums its 256 grad_mix elements over the local partials in a fixed order
//      (as the single-GPU reduction does) and stores each fp32 value, together with the
//      call counter `epoch`, as one 64-bit word {epoch:value} into this rank's exchange
//      buffer (slot `epoch % 4`), a warp's lanes on consecutive words;
//   2. it reads the words of the call it sums from every other rank's buffer through the
//      peer mappings (NVLink), polling each word (bounded) until it carries that call's
//      counter; one thread row per rank, so the ranks' reads are in flight together, and
//      a warp's lanes on consecutive words, so each word crosses NVLink once;
//   3. it adds every rank's values in rank order 0..world-1 and writes the sum, rounded
//      once to the output type. Every rank performs the same fp32 additions in the same
//      order, so all ranks hold bitwise-identical results.
// Synchronous mode sums the call itself (step 2 waits for the slowest rank). Deferred mode
// sums the previous call instead, whose words every peer published one call earlier, so
// nothing waits in practice and its reads are issued before the local sum; the last
// call's sum comes from a finish launch (mode 2). The flag travels in the same naturally
// aligned 64-bit word as the value, so a reader that sees the flag sees the value: no
// fences and no separate flag array (the flag-in-data scheme of low-latency all-reduce
// protocols). Plain loads and stores only (no TMA, no switch-side reduction).
// Slot reuse: a rank rewrites slot s four calls after it wrote it. Peers read it at the
// latest in their call after the one that wrote it (deferred mode), and a rank knows that
// call of every peer has completed once it has read the peers' words of the call after
// that one, which it does before its next publication; four slots cover that lag in both
// modes, so no further barrier is needed. A wait that runs out (a peer that never arrives)
// records its site in the device error record and that block writes nothing, instead of
// hanging.
#include "common.cuh"
#include "sm100.cuh"

namespace dudy {

namespace {

constexpr int kSlice = 256;  // grad_mix elements per block (64 x 4 lanes)

__device__ __forceinline__ unsigned long long ld_volatile_u64(const unsigned long long *p) {
  unsigned long long v;
  asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_volatile_u64(unsigned long long *p, unsigned long long v) {
  asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}

// four consecutive elements [e, e+4) of a row of `n` floats; 16-byte loads when rows are
// 16-byte aligned (VEC), element loads (zero past the end) otherwise
template <bool VEC>
__device__ __forceinline__ float4 load4(const float *row, int64_t e, int64_t n) {
  if (VEC) return __ldg(reinterpret_cast<const float4 *>(row + e));
  float v[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) v[i] = e + i < n ? __ldg(row + e + i) : 0.f;
  return make_float4(v[0], v[1], v[2], v[3]);
}

// Rank r's words of call `ep` for the block's elements tx + 64 i, i = 0..3 (a warp's lanes
// read consecutive words: each load instruction covers 256 contiguous bytes, so a word
// crosses NVLink once): fetch4_issue loads them (past the end: a word that already carries
// `ep`), fetch4_finish polls each until it carries `ep` (bounded) and returns the values;
// false after a wait ran out (recorded in the error record). Work placed between the two
// overlaps the loads' latency.
__device__ __forceinline__ void fetch4_issue(const unsigned long long *src, int64_t g0, int64_t DN,
                                             uint32_t ep, unsigned long long (&w)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i)
    w[i] = g0 + 64 * i < DN ? ld_volatile_u64(src + 64 * i) : ((unsigned long long)ep << 32);
}

__device__ __forceinline__ bool fetch4_finish(const unsigned long long *src, uint32_t ep, int r,
                                              int *err, unsigned long long (&w)[4],
                                              float (&out)[4]) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if ((uint32_t)(w[i] >> 32) == ep) continue;
    const uint64_t t0 = sm100::global_ns();
    while ((uint32_t)((w[i] = ld_volatile_u64(src + 64 * i)) >> 32) != ep) {
      if (sm100::global_ns() - t0 > sm100::kWaitLimitNs) {
        sm100::record_timeout(err, sm100::kXrankSite + r, (int)ep);
        return false;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) out[i] = __uint_as_float((uint32_t)w[i]);
  return true;
}

// Block = 64 x 16 threads over the 256 grad_mix elements [b0, b0 + 256). All 16 rows sum the
// local partials for elements 4 tx .. 4 tx + 3 (row ty takes partials ty, ty + 16, ...);
// rows 0-3 then finish element tx + 64 ty (the 16 row sums in order) and publish its word;
// row ty < world fetches rank ty's words of the summed call for elements tx + 64 i, so the
// ranks' fetches are in flight together (in deferred mode issued before the local sum);
// row 0 adds the ranks in order 0..world-1 for elements 4 tx .. 4 tx + 3.
template <typename T, bool VEC>
__global__ void __launch_bounds__(1024)
fdc_mix_reduce_xrank_kernel(const float *__restrict__ part, T *__restrict__ out, int64_t DN,
                            int nparts, XRank x, int *err) {
  __shared__ float4 red[16][64];
  __shared__ float4 got[DUDY_MAX_PEERS][64];  // [rank][element / 4]
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int64_t b0 = (int64_t)blockIdx.x * 256;
  const int64_t e = b0 + 4 * tx;  // this column's four elements in the local sum
  const uint32_t sum_epoch = x.mode == 1 ? x.epoch - 1u : x.epoch;
  const int64_t slot = (int64_t)(sum_epoch & 3u) * DN;
  // the fetching row of rank ty (in synchronous mode this rank's own values come from the
  // local sum instead)
  const bool fetch = ty < x.world && b0 + tx < DN && sum_epoch != 0u &&
                     !(x.mode == 0 && ty == x.rank);
  const unsigned long long *src =
      reinterpret_cast<const unsigned long long *>(x.bufs[ty < x.world ? ty : 0]) + slot + b0 + tx;
  bool fail = false;
  float g[4] = {0.f, 0.f, 0.f, 0.f};
  unsigned long long w[4];
  // deferred: the previous call's words (this rank's were written by its previous call,
  // which completed before this kernel's predecessors started), in flight during the sum
  if (x.mode == 1 && fetch) fetch4_issue(src, b0 + tx, DN, sum_epoch, w);
  pdl_wait();  // the partials are written by the kernel launched just before
  if (tx == 0 && ty == 0) pdl_trigger();
  // ---- 1. local fixed-order sum of this block's slice
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e < DN) {
    int p = ty;
    for (; p + 48 < nparts; p += 64) {
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = load4<VEC>(part + (int64_t)(p + 16 * j) * DN, e, DN);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
      }
    }
    for (; p < nparts; p += 16) {
      const float4 v = load4<VEC>(part + (int64_t)p * DN, e, DN);
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  red[ty][tx] = acc;
  if (x.mode == 1 && fetch) fail = !fetch4_finish(src, sum_epoch, ty, err, w, g);
  __syncthreads();
  float *gotf = reinterpret_cast<float *>(got);
  // ---- 2a. element tx + 64 ty: the 16 row sums in order, published as an {epoch:value} word
  const int el = tx + 64 * ty;
  if (ty < 4 && b0 + el < DN && x.mode != 2) {
    const float *rf = reinterpret_cast<const float *>(red);
    float v = rf[el];
#pragma unroll
    for (int r = 1; r < 16; ++r) v += rf[r * 256 + el];
    unsigned long long *own =
        reinterpret_cast<unsigned long long *>(x.bufs[x.rank]) + (int64_t)(x.epoch & 3u) * DN + b0 + el;
    st_volatile_u64(own, ((unsigned long long)x.epoch << 32) | __float_as_uint(v));
    if (x.mode == 1)
      stf(out + b0 + el, v);       // deferred: grad_mix gets this rank's own sum
    else
      gotf[x.rank * 256 + el] = v;  // synchronous: this rank's values for the sum below
  }
  // ---- 2b. the other ranks' words of this call (synchronous mode, finish)
  if (x.mode != 1 && fetch) {
    fetch4_issue(src, b0 + tx, DN, sum_epoch, w);
    fail = !fetch4_finish(src, sum_epoch, ty, err, w, g);
  }
  if (fetch) {
#pragma unroll
    for (int i = 0; i < 4; ++i) gotf[ty * 256 + tx + 64 * i] = g[i];
  }
  // a block with a wait that ran out writes nothing
  if (__syncthreads_or(fail) || sum_epoch == 0u || ty != 0 || e >= DN) return;
  // ---- 3. ranks in order 0..world-1, rounded once
  T *dst = x.mode == 1 ? reinterpret_cast<T *>(x.prev_out) : out;
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < x.world; ++r) {
    const float4 v = got[r][tx];
    sum[0] += v.x; sum[1] += v.y; sum[2] += v.z; sum[3] += v.w;
  }
#pragma unroll
  for (int i = 0; i < 4; ++i)
    if (e + i < DN) stf(dst + e + i, sum[i]);
}

template <typename T>
cudaError_t launch_xrank(const float *part, int nparts, T *out, int64_t DN, const XRank &x,
                         int *err, cudaStream_t st) {
  const dim3 grid((unsigned)cdiv(DN, kSlice)), block(64, 16);
  const bool vec = DN % 4 == 0 && (reinterpret_cast<uintptr_t>(part) & 15u) == 0;
  return vec ? launch_pdl(fdc_mix_reduce_xrank_kernel<T, true>, grid, block, 0, st, part, out,
                          DN, nparts, x, err)
             : launch_pdl(fdc_mix_reduce_xrank_kernel<T, false>, grid, block, 0, st, part, out,
                          DN, nparts, x, err);
}

}  // namespace

size_t xrank_buffer_bytes(int64_t DN) {
  // four slots of DN 64-bit {epoch:value} words
  return (size_t)(4 * DN) * sizeof(unsigned long long);
}

int xrank_reduce_launch(const float *part, int nparts, void *grad_mix, int64_t DN, int dtype,
                        const XRank &x, int *err, cudaStream_t st) {
  cudaError_t e;
  switch (dtype) {
    case DUDY_DTYPE_F32: e = launch_xrank(part, nparts, (float *)grad_mix, DN, x, err, st); break;
    case DUDY_DTYPE_F16: e = launch_xrank(part, nparts, (__half *)grad_mix, DN, x, err, st); break;
    default: e = launch_xrank(part, nparts, (__nv_bfloat16 *)grad_mix, DN, x, err, st);
  }
  if (e != cudaSuccess) return check_launch("fdc_mix_reduce_xrank_kernel");
  return DUDY_OK;
}

}  // namespace dudy
