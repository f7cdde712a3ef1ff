// xrank.cu -- the data-parallel grad_mix exchange, fused into the backward's last kernel.
//
// With the batch sharded over ranks (one GPU each), every rank's backward ends with
// per-CTA fp32 partial sums of grad_mix [D,N] in its workspace, and the data-parallel
// step needs the sum over ranks. Instead of reducing locally, casting, and running a
// separate all-reduce (a cast kernel, the collective's kernel, a copy back), one kernel
// does it all over peer memory:
//   1. each thread sums its 4 grad_mix elements over the local partials in a fixed order
//      (as the single-GPU reduction does) and stores each fp32 value, together with the
//      call counter `epoch`, as one 64-bit word {epoch:value} into this rank's exchange
//      buffer (slot `epoch % 4`);
//   2. it reads the words of the call it sums from every other rank's buffer through the
//      peer mappings (NVLink), polling each word (bounded) until it carries that call's
//      counter;
//   3. it adds every rank's values in rank order 0..world-1 and writes the sum, rounded
//      once to the output type. Every rank performs the same fp32 additions in the same
//      order, so all ranks hold bitwise-identical results.
// Synchronous mode sums the call itself (step 2 waits for the slowest rank). Deferred mode
// sums the previous call instead, whose words every peer published one call earlier, so
// nothing waits in practice and the exchange adds only its loads to the step; the last
// call's sum comes from a finish launch (mode 2). The flag travels in the same naturally
// aligned 64-bit word as the value, so a reader that sees the flag sees the value: no
// fences and no separate flag array (the flag-in-data scheme of low-latency all-reduce
// protocols). Plain loads and stores only (no TMA, no switch-side reduction).
// Slot reuse: a rank rewrites slot s four calls after it wrote it. Peers read it at the
// latest in their call after the one that wrote it (deferred mode), and a rank knows that
// call of every peer has completed once it has read the peers' words of the call after
// that one, which it does before its next publication; four slots cover that lag in both
// modes, so no further barrier is needed. A wait that runs out (a peer that never arrives)
// records its site in the device error record and that thread writes nothing, instead of
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

template <typename T, bool VEC>
__global__ void __launch_bounds__(1024)
fdc_mix_reduce_xrank_kernel(const float *__restrict__ part, T *__restrict__ out, int64_t DN,
                            int nparts, XRank x, int *err) {
  __shared__ float4 red[16][64];
  const int tx = threadIdx.x, ty = threadIdx.y;
  pdl_wait();  // the partials are written by the kernel launched just before
  if (tx == 0 && ty == 0) pdl_trigger();
  const int64_t e = ((int64_t)blockIdx.x * 64 + tx) * 4;
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
  __syncthreads();
  if (ty != 0 || e >= DN) return;
  float mine[4] = {0.f, 0.f, 0.f, 0.f};
  if (x.mode != 2) {
    float4 m4 = red[0][tx];
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      m4.x += red[r][tx].x; m4.y += red[r][tx].y; m4.z += red[r][tx].z; m4.w += red[r][tx].w;
    }
    mine[0] = m4.x; mine[1] = m4.y; mine[2] = m4.z; mine[3] = m4.w;
    // ---- 2a. publish {epoch:value} words
    const unsigned long long tag = (unsigned long long)x.epoch << 32;
    unsigned long long *own =
        reinterpret_cast<unsigned long long *>(x.bufs[x.rank]) + (int64_t)(x.epoch & 3u) * DN + e;
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (e + i < DN) st_volatile_u64(own + i, tag | __float_as_uint(mine[i]));
    if (x.mode == 1) {
      // deferred: grad_mix gets this rank's own sum
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (e + i < DN) stf(out + e + i, mine[i]);
    }
  }
  // ---- 2b. gather the summed call's words from every rank (own values from registers
  // when the call is this one)
  const uint32_t sum_epoch = x.mode == 1 ? x.epoch - 1u : x.epoch;
  if (sum_epoch == 0u) return;  // deferred mode, first call: nothing before it
  T *dst = x.mode == 1 ? reinterpret_cast<T *>(x.prev_out) : out;
  const int64_t slot = (int64_t)(sum_epoch & 3u) * DN;
  float sum[4] = {0.f, 0.f, 0.f, 0.f};
  for (int r = 0; r < x.world; ++r) {
    float v[4];
    if (r == x.rank && sum_epoch == x.epoch && x.mode == 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = mine[i];
    } else {
      const unsigned long long *src =
          reinterpret_cast<const unsigned long long *>(x.bufs[r]) + slot + e;
      unsigned long long w[4];
#pragma unroll
      for (int i = 0; i < 4; ++i)
        w[i] = e + i < DN ? ld_volatile_u64(src + i) : ((unsigned long long)sum_epoch << 32);
      bool ok = true;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        if ((uint32_t)(w[i] >> 32) == sum_epoch) continue;
        const uint64_t t0 = sm100::global_ns();
        while ((uint32_t)((w[i] = ld_volatile_u64(src + i)) >> 32) != sum_epoch) {
          if (sm100::global_ns() - t0 > sm100::kWaitLimitNs) {
            sm100::record_timeout(err, sm100::kXrankSite + r, (int)sum_epoch);
            ok = false;
            break;
          }
        }
        if (!ok) break;
      }
      if (!ok) return;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __uint_as_float((uint32_t)w[i]);
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) sum[i] += v[i];
  }
  // ---- 3. round once
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
