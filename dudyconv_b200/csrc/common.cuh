// common.cuh -- element-type traits, shape structs and error plumbing shared by the
// dudyconv_b200 kernels. Everything here is internal to libdudyconv_b200.so.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

#include "../../include/dudyconv_b200.h"

namespace dudy {

// ---------------------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------------------
template <typename T>
struct Elem;

template <>
struct Elem<float> {
  static __device__ __forceinline__ float to_f(float v) { return v; }
  static __device__ __forceinline__ float from_f(float v) { return v; }
};

template <>
struct Elem<__half> {
  static __device__ __forceinline__ float to_f(__half v) { return __half2float(v); }
  static __device__ __forceinline__ __half from_f(float v) { return __float2half_rn(v); }
};

template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float to_f(__nv_bfloat16 v) { return __bfloat162float(v); }
  static __device__ __forceinline__ __nv_bfloat16 from_f(float v) {
    return __float2bfloat16_rn(v);
  }
};

template <typename T>
__device__ __forceinline__ float ldf(const T *p) {
  return Elem<T>::to_f(*p);
}

template <typename T>
__device__ __forceinline__ void stf(T *p, float v) {
  *p = Elem<T>::from_f(v);
}

template <typename T>
struct IsBf16 {
  static constexpr int value = 0;
};
template <>
struct IsBf16<__nv_bfloat16> {
  static constexpr int value = 1;
};

inline size_t dtype_size(int dtype) { return dtype == DUDY_DTYPE_F32 ? 4 : 2; }

// ---------------------------------------------------------------------------------------
// shapes
// ---------------------------------------------------------------------------------------
struct FdcShape {
  int64_t B, D, L, T, N, K, off, dil;
  // first and one-past-last h positions that receive gradient: [off-(K-1)*dil, off+T)
  int64_t gh_lo() const {
    int64_t lo = off - (K - 1) * dil;
    return lo < 0 ? 0 : lo;
  }
  int64_t gh_hi() const { return off + T; }
};

// Peer-memory exchange of the data-parallel grad_mix sum (xrank.cu): every rank's
// exchange buffer as mapped in this process, this rank, the number of ranks and the call
// counter (identical on every rank).
// mode 0 (synchronous): publish this call's sums (counter `epoch`) and write the sum over
// ranks of this call into grad_mix; mode 1 (deferred): publish, write this rank's own sum
// into grad_mix and the sum over ranks of the previous call (epoch - 1, if any) into
// `prev_out`; mode 2 (finish): publish nothing, write the sum over ranks of call `epoch`.
struct XRank {
  float *bufs[DUDY_MAX_PEERS];
  int rank, world;
  uint32_t epoch;
  int mode;
  void *prev_out;
};
size_t xrank_buffer_bytes(int64_t DN);
int xrank_reduce_launch(const float *part, int nparts, void *grad_mix, int64_t DN, int dtype,
                        const XRank &x, int *err, cudaStream_t st);

struct FscmShape {
  int64_t B, D, L, C, S, off, T, dil;
  bool has_bias;
  int64_t halo() const { return dil * (S - 1); }
};

// ---------------------------------------------------------------------------------------
// error plumbing: a thread-local message, read back through dudy_last_error()
// ---------------------------------------------------------------------------------------
void set_error(const std::string &msg);
void clear_error();

// Launch-error check: returns DUDY_ERR_CUDA with a message, else DUDY_OK.
int check_launch(const char *what);

inline int64_t cdiv(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Launch with programmatic dependent launch: the kernel may start while the previous
// kernel of the stream finishes, so its prologue (barrier setup, TMEM allocation, tensor
// map prefetch) overlaps that kernel's tail. Kernels launched this way call pdl_wait()
// before their first global-memory access and pdl_trigger() once every CTA has started.
// launch_pdl with the grid's CTAs grouped in clusters of `cluster_x` consecutive blocks
// (co-scheduled on one GPC). The kernels use no cluster shared memory; CTAs of a cluster
// work on the same tile, so their reads of shared inputs reach L2 at the same time.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl_cluster(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                               cudaStream_t st, unsigned cluster_x, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster_x > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = cluster_x;
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t st, Args... args) {
  return launch_pdl_cluster(kern, grid, block, smem, st, 1, args...);
}


// Device side of launch_pdl: wait until the previous kernel of the stream has completed
// and its writes are visible (a no-op without a programmatic launch).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Allow the next kernel of the stream to begin launching.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// cudaFuncSetAttribute(kern, MaxDynamicSharedMemorySize, bytes) on the current device,
// skipped when an earlier call already set at least `bytes` there (the attribute persists
// and setting it costs host time on every launch of the small-chunk call path)
cudaError_t set_smem_once(const void *kern, int bytes);

// number of SMs of the current device (cached per device)
int sm_count();
// compute capability major*10+minor of the current device (cached per device)
int device_cc();

}  // namespace dudy
