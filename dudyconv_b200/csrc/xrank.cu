// xrank.cu -- the data-parallel grad_mix exchange, fused into the backward's last kernel.
//
// With the batch sharded over ranks (one GPU each), every rank's backward ends with
// per-CTA fp32 partial sums of grad_mix [D,N] in its workspace, and the data-parallel
// step needs the sum over ranks. Instead of reducing locally, casting, and running a
// separate all-reduce (a cast kernel, the collective's kernel, a copy back), one kernel
// does it all over peer memory:
//   1. each block sums its 256-element slice of the local partials in a fixed order
//      (as the single-GPU reduction does) and stores the fp32 slice into this rank's
//      exchange buffer (half `epoch & 1` of a double buffer);
//   2. it publishes the slice with a release store of `epoch` into its flag, then
//      waits (bounded) until every other rank's flag for the same slice reaches `epoch`
//      (acquire loads through the peers' mappings, i.e. over NVLink);
//   3. it reads every rank's slice in rank order 0..world-1 and writes the sum, rounded
//      once to the output type, into grad_mix. Every rank performs the same fp32 additions
//      in the same order, so all ranks hold bitwise-identical results.
// Plain loads and stores only (no TMA, no switch-side reduction). A rank reuses a buffer half two
// calls later; by then every peer has published the call in between, which it does only
// after finishing its reads of this half, so the double buffer needs no further barrier.
// A wait that runs out (a peer that never arrives) records its site in the device error
// record and the block writes nothing, instead of hanging.
#include "common.cuh"
#include "sm100.cuh"

namespace dudy {

namespace {

constexpr int kSlice = 256;  // grad_mix elements per block (64 x 4 lanes)

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t *p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void st_release_sys(uint32_t *p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
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
  __shared__ int go_on;
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
  // exchange buffer: two halves of DNp = DN rounded up to 4 floats, then the flags
  const int64_t DNp = (DN + 3) & ~int64_t(3);
  const int64_t half = (int64_t)(x.epoch & 1u) * DNp;
  float4 mine = make_float4(0.f, 0.f, 0.f, 0.f);
  if (ty == 0 && e < DN) {
    mine = red[0][tx];
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      mine.x += red[r][tx].x; mine.y += red[r][tx].y; mine.z += red[r][tx].z;
      mine.w += red[r][tx].w;
    }
    *reinterpret_cast<float4 *>(x.bufs[x.rank] + half + e) = mine;
  }
  __syncthreads();
  // ---- 2. publish this slice, wait for every peer's
  if (tx == 0 && ty == 0) {
    // the barrier above orders every thread's slice store before this release store (the
    // release is cumulative over the writes this thread has observed through the barrier)
    st_release_sys(reinterpret_cast<uint32_t *>(x.bufs[x.rank] + 2 * DNp) + blockIdx.x, x.epoch);
    int ok = 1;
    for (int r = 0; r < x.world && ok; ++r) {
      if (r == x.rank) continue;
      const uint32_t *f = reinterpret_cast<const uint32_t *>(x.bufs[r] + 2 * DNp) + blockIdx.x;
      if ((int32_t)(ld_acquire_sys(f) - x.epoch) >= 0) continue;
      const uint64_t t0 = sm100::global_ns();
      while ((int32_t)(ld_acquire_sys(f) - x.epoch) < 0) {
        if (sm100::global_ns() - t0 > sm100::kWaitLimitNs) {
          sm100::record_timeout(err, sm100::kXrankSite + r, (int)x.epoch);
          ok = 0;
          break;
        }
      }
    }
    go_on = ok;
  }
  __syncthreads();
  if (!go_on) return;
  // ---- 3. sum over ranks in rank order, round once
  if (ty == 0 && e < DN) {
    float4 s = make_float4(0.f, 0.f, 0.f, 0.f);
    for (int r = 0; r < x.world; ++r) {
      const float4 v =
          r == x.rank ? mine : __ldcv(reinterpret_cast<const float4 *>(x.bufs[r] + half + e));
      s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
    }
    const float o[4] = {s.x, s.y, s.z, s.w};
#pragma unroll
    for (int i = 0; i < 4; ++i)
      if (e + i < DN) stf(out + e + i, o[i]);
  }
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
  // two fp32 halves (each rounded up to 4 floats) plus one 32-bit flag per block
  const int64_t DNp = (DN + 3) & ~int64_t(3);
  return (size_t)(2 * DNp) * sizeof(float) + (size_t)cdiv(DN, kSlice) * sizeof(uint32_t);
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
