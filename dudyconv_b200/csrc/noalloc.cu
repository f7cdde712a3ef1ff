// noalloc.cu -- dudy_fdc_backward_noalloc: the dynamic-conv backward for callers that
// cannot allocate device memory at call time.
//
// Who needs it: hosts whose device memory is fixed up front (a serving process that
// reserves its whole budget at start-up and forbids later allocation), code running in
// a context where cudaMalloc is not allowed or would implicitly synchronize the device,
// and foreign-function callers that have no allocator to pass a workspace from. For
// them the scratch that dudy_fdc_backward takes as a caller workspace (the per-CTA fp32
// partial sums of grad_mix) lives in a fixed device array of this library instead.
//
// The array is a file-scope static __device__ object of DUDY_NOALLOC_SCRATCH_BYTES;
// every GPU that loads the library holds it until the process exits. In host code its
// name is only a host-side stand-in, not a device address, so the device address is
// looked up per device (cudaGetSymbolAddress, with that device current) the first time
// this entry point runs there, and passed to the kernels from then on. Only a successful
// lookup is kept: a failed one (for example a first call made during stream capture, or
// with an earlier error pending) is retried on the next call. A cudaDeviceReset destroys
// the array with the context, so a process that resets a device must not call this entry
// point on it again.
#include <mutex>
#include <string>

#include "common.cuh"

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[DUDY_NOALLOC_SCRATCH_BYTES];

constexpr int kMaxDevices = 64;
void *g_scratch_ptr[kMaxDevices];
std::mutex g_scratch_mu;

// Device address of the scratch array on the current device (nullptr on failure, with
// the reason in the thread's error message).
void *scratch_for_current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
    dudy::set_error("dudy_fdc_backward_noalloc: no usable current CUDA device");
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_ptr[dev]) {
    void *p = nullptr;
    const cudaError_t rc = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (rc != cudaSuccess) {
      dudy::set_error(std::string("dudy_fdc_backward_noalloc: cudaGetSymbolAddress failed: ") +
                      cudaGetErrorString(rc));
      return nullptr;
    }
    g_scratch_ptr[dev] = p;
  }
  return g_scratch_ptr[dev];
}

}  // namespace

extern "C" int dudy_fdc_backward_noalloc(const void *go, const void *h, const void *kc,
                                         const void *mix, void *grad_h, void *grad_kc,
                                         void *grad_mix, int64_t B, int64_t D, int64_t L,
                                         int64_t T, int64_t N, int64_t K, int64_t off,
                                         int64_t dilation, int dtype, int plan,
                                         void *stream) {
  dudy::clear_error();
  const size_t need =
      dudy_fdc_backward_workspace_size(B, D, L, T, N, K, off, dilation, dtype, plan);
  if (need > (size_t)DUDY_NOALLOC_SCRATCH_BYTES) {
    dudy::set_error("dudy_fdc_backward_noalloc: these shapes need " + std::to_string(need) +
                    " bytes of scratch, more than the fixed " +
                    std::to_string((size_t)DUDY_NOALLOC_SCRATCH_BYTES) +
                    " bytes; use dudy_fdc_backward with a caller workspace");
    return DUDY_ERR_WORKSPACE;
  }
  void *scratch = scratch_for_current_device();
  if (!scratch) return DUDY_ERR_CUDA;
  // Every partial the kernels read is written earlier in the same call, so nothing in
  // the array has to start at zero.
  return dudy_fdc_backward(go, h, kc, mix, grad_h, grad_kc, grad_mix, scratch,
                           (size_t)DUDY_NOALLOC_SCRATCH_BYTES, B, D, L, T, N, K, off, dilation,
                           dtype, plan, stream);
}
