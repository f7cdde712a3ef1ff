// capi.cu -- the extern "C" boundary of libdudyconv_b200.so (declared in
// include/dudyconv_b200.h): argument validation with the reference's rules and
// messages, plan selection, and dispatch to the CUDA-core or tcgen05 kernels.
#include <cudaTypedefs.h>

#include <mutex>
#include <string>

#include "common.cuh"
#include "sm100.cuh"
#include "tma_host.h"

namespace dudy {

// ---- kernels implemented elsewhere -----------------------------------------------------
int fdc_simt_forward(const void *h, const void *kc, const void *mix, void *out,
                     const FdcShape &s, int dtype, cudaStream_t st);
int fdc_simt_grad_h(const void *go, const void *kc, const void *mix, void *grad_h,
                    const FdcShape &s, int dtype, cudaStream_t st);
int fdc_simt_grad_kc_mix(const void *go, const void *h, const void *mix, const void *kc,
                         void *grad_kc, void *grad_mix, void *ws, const FdcShape &s, int dtype,
                         const XRank *xr, int *err, cudaStream_t st);
size_t fdc_simt_bwd_workspace(const FdcShape &s);
namespace tc {
bool conv_supported(bool gh, const FdcShape &s, int dtype);
int conv_launch(bool gh, const void *kc, const void *mix, const void *fac, void *y,
                const FdcShape &s, int dtype, bool dep_late, int *err, cudaStream_t st);
bool bk_supported(const FdcShape &s, int dtype);
size_t bk_workspace(const FdcShape &s);
int bk_launch(const void *go, const void *h, const void *kc, const void *mix, void *grad_kc,
              void *grad_mix, void *ws, const FdcShape &s, int dtype, bool dep_late, int *err,
              const XRank *xr, cudaStream_t st);
}  // namespace tc
bool fscm_shapes_fit(const FscmShape &s, int64_t tile_t);
size_t fscm_bwd_workspace(const FscmShape &s, int64_t tile_t);
int check_phi_approx(float *max_abs_err);
int fscm_forward_impl(const void *x, const void *w, const void *bias, const void *mw,
                      const void *mb, void *out, const FscmShape &s, int dtype, cudaStream_t st);
int fscm_backward_impl(const void *go, const void *x, const void *w, const void *bias,
                       const void *mw, void *gx, void *gw, void *gb, void *gmw, void *gmb,
                       void *ws, const FscmShape &s, int64_t tile_t, int dtype, cudaStream_t st);

// ---- error plumbing ---------------------------------------------------------------------
namespace {
thread_local std::string g_last_error;
constexpr int kMaxDevices = 64;
int g_sm_count[kMaxDevices];
int g_cc[kMaxDevices];
int *g_err_word[kMaxDevices];
std::once_flag g_dev_once[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}
}  // namespace

// device-side error record, one per device: [0] site id of the first bounded wait that
// timed out (0 = none), [1] block, [2] thread, [3] loop counter of that wait
__device__ int g_device_error_word[4];

void set_error(const std::string &msg) { g_last_error = msg; }
void clear_error() { g_last_error.clear(); }

int check_launch(const char *what) {
  const cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) return DUDY_OK;
  set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return DUDY_ERR_CUDA;
}

static void init_device(int dev) {
  std::call_once(g_dev_once[dev], [dev] {
    cudaDeviceGetAttribute(&g_sm_count[dev], cudaDevAttrMultiProcessorCount, dev);
    int maj = 0, mnr = 0;
    cudaDeviceGetAttribute(&maj, cudaDevAttrComputeCapabilityMajor, dev);
    cudaDeviceGetAttribute(&mnr, cudaDevAttrComputeCapabilityMinor, dev);
    g_cc[dev] = maj * 10 + mnr;
    void *p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error_word) == cudaSuccess) g_err_word[dev] = (int *)p;
  });
}

cudaError_t set_smem_once(const void *kern, int bytes) {
  struct Entry {
    const void *kern;
    int dev, bytes;
  };
  static std::mutex mu;
  static Entry table[64];
  static int used = 0;
  const int dev = current_device();
  std::lock_guard<std::mutex> lock(mu);
  for (int i = 0; i < used; ++i)
    if (table[i].kern == kern && table[i].dev == dev && table[i].bytes >= bytes) return cudaSuccess;
  const cudaError_t e =
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  for (int i = 0; i < used; ++i)
    if (table[i].kern == kern && table[i].dev == dev) {
      table[i].bytes = bytes;
      return cudaSuccess;
    }
  if (used < 64) table[used++] = Entry{kern, dev, bytes};
  return cudaSuccess;
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  init_device(dev);
  return g_sm_count[dev] > 0 ? g_sm_count[dev] : 148;
}

int device_cc() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 0;
  init_device(dev);
  return g_cc[dev];
}

static int *device_err_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  init_device(dev);
  return g_err_word[dev];
}

// ---- TMA maps ------------------------------------------------------------------------------
// Driver-API calls need a current context on the calling thread. Threads that only ever
// touched CUDA through another runtime instance (e.g. torch's autograd worker threads)
// may have none; cudaSetDevice makes the device's primary context current.
static void ensure_context() {
  thread_local int ready_dev = -1;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return;
  if (dev != ready_dev && cudaSetDevice(dev) == cudaSuccess) ready_dev = dev;
}

bool make_tmap_2d(CUtensorMap *map, const void *base, bool bf16, uint64_t dim0, uint64_t dim1,
                  uint64_t row_stride_bytes, uint32_t box0, uint32_t box1, int swizzle_bytes) {
  ensure_context();
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
            cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  });
  if (!encode) {
    set_error("cuTensorMapEncodeTiled is not available from the driver");
    return false;
  }
  cuuint64_t dims[2] = {dim0, dim1};
  cuuint64_t strides[1] = {row_stride_bytes};
  cuuint32_t box[2] = {box0, box1};
  cuuint32_t estr[2] = {1, 1};
  CUtensorMapSwizzle sw = CU_TENSOR_MAP_SWIZZLE_NONE;
  if (swizzle_bytes == 32) sw = CU_TENSOR_MAP_SWIZZLE_32B;
  if (swizzle_bytes == 64) sw = CU_TENSOR_MAP_SWIZZLE_64B;
  if (swizzle_bytes == 128) sw = CU_TENSOR_MAP_SWIZZLE_128B;
  const CUresult r = encode(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                            2, const_cast<void *>(base), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return false;
  }
  return true;
}

}  // namespace dudy

using dudy::FdcShape;
using dudy::FscmShape;

namespace {

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

bool dtype_ok(int dtype) {
  return dtype == DUDY_DTYPE_F32 || dtype == DUDY_DTYPE_F16 || dtype == DUDY_DTYPE_BF16;
}

// The reference's checks (cuda_ops/fused_dynamic_conv.py:108-186 and
// fused_dynamic_conv_kernel.cu:390-452), with its messages.
int validate_fdc(const FdcShape &s, int dtype) {
  if (s.dil <= 0) return dudy::set_error("dilation must be positive."), DUDY_ERR_INVALID;
  if (s.T <= 0) return dudy::set_error("T must be positive."), DUDY_ERR_INVALID;
  if (s.K <= 0) return dudy::set_error("K must be positive."), DUDY_ERR_INVALID;
  if (s.B <= 0 || s.D <= 0 || s.N <= 0 || s.L <= 0)
    return dudy::set_error("B, D, N and L must be positive."), DUDY_ERR_INVALID;
  if (s.off < 0) return dudy::set_error("t_offset must be non-negative."), DUDY_ERR_INVALID;
  if (s.off + s.T > s.L)
    return dudy::set_error("t_offset + T must be <= L, got t_offset=" + std::to_string(s.off) +
                           ", T=" + std::to_string(s.T) + ", L=" + std::to_string(s.L) + "."),
           DUDY_ERR_INVALID;
  if (!dtype_ok(dtype)) return dudy::set_error("Unsupported dtype."), DUDY_ERR_INVALID;
  if (s.B * s.D * s.L >= ((int64_t)1 << 31) || s.B * s.K * s.N * s.T >= ((int64_t)1 << 31))
    return dudy::set_error("tensor too large (more than 2^31 elements)."), DUDY_ERR_INVALID;
  return DUDY_OK;
}

int device_ok() {
  if (dudy::device_cc() != 100) {
    dudy::set_error("current CUDA device is not an sm_100 (B200-class) GPU; this library is "
                    "built for sm_100a only");
    return DUDY_ERR_DEVICE;
  }
  return DUDY_OK;
}

bool tc_fwd_ok(const void *h, const void *kc, const void *mix, const FdcShape &s, int dtype) {
  return aligned16(h) && aligned16(kc) && aligned16(mix) &&
         dudy::tc::conv_supported(false, s, dtype);
}

bool tc_bwd_ok(const void *go, const void *h, const void *kc, const void *mix,
               const FdcShape &s, int dtype) {
  return aligned16(go) && aligned16(h) && aligned16(kc) && aligned16(mix) &&
         dudy::tc::conv_supported(true, s, dtype) && dudy::tc::bk_supported(s, dtype);
}

FdcShape fdc_shape(int64_t B, int64_t D, int64_t L, int64_t T, int64_t N, int64_t K,
                   int64_t off, int64_t dil) {
  return FdcShape{B, D, L, T, N, K, off, dil};
}

}  // namespace

extern "C" {

const char *dudy_version(void) { return "dudyconv_b200 0.1.0 (sm_100a)"; }

const char *dudy_last_error(void) { return dudy::g_last_error.c_str(); }

const char *dudy_fdc_plan_name(int plan) {
  switch (plan) {
    case -1: return "not_cached";
    case DUDY_FDC_PLAN_SIMT: return "simt_generic";
    case DUDY_FDC_PLAN_TC: return "tcgen05_tmem";
    default: return "unknown_plan";
  }
}

int dudy_fdc_plan_available(int plan, const void *h, const void *kc, const void *mix,
                            int64_t B, int64_t D, int64_t L, int64_t T, int64_t N, int64_t K,
                            int64_t off, int64_t dilation, int dtype) {
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (validate_fdc(s, dtype)) return 0;
  if (plan == DUDY_FDC_PLAN_SIMT) return 1;
  if (plan == DUDY_FDC_PLAN_TC)
    return tc_fwd_ok(h, kc, mix, s, dtype) && tc_bwd_ok(h, h, kc, mix, s, dtype) ? 1 : 0;
  return 0;
}

int dudy_fdc_default_plan(const void *h, const void *kc, const void *mix, int64_t B, int64_t D,
                          int64_t L, int64_t T, int64_t N, int64_t K, int64_t off,
                          int64_t dilation, int dtype) {
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (validate_fdc(s, dtype)) return -1;
  return tc_fwd_ok(h, kc, mix, s, dtype) ? DUDY_FDC_PLAN_TC : DUDY_FDC_PLAN_SIMT;
}

int dudy_fdc_forward(const void *h, const void *kc, const void *mix, void *out, int64_t B,
                     int64_t D, int64_t L, int64_t T, int64_t N, int64_t K, int64_t off,
                     int64_t dilation, int dtype, int plan, void *stream) {
  dudy::clear_error();
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (int rc = validate_fdc(s, dtype)) return rc;
  if (!h || !kc || !mix || !out) return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool tc_ok = tc_fwd_ok(h, kc, mix, s, dtype);
  if (plan == DUDY_PLAN_AUTO) plan = tc_ok ? DUDY_FDC_PLAN_TC : DUDY_FDC_PLAN_SIMT;
  if (plan == DUDY_FDC_PLAN_TC) {
    if (!tc_ok) return dudy::set_error("plan tcgen05_tmem is not available for these shapes"), DUDY_ERR_UNSUPPORTED;
    return dudy::tc::conv_launch(false, kc, mix, h, out, s, dtype, false, dudy::device_err_word(),
                                 st);
  }
  if (plan == DUDY_FDC_PLAN_SIMT) return dudy::fdc_simt_forward(h, kc, mix, out, s, dtype, st);
  dudy::set_error("unknown forward plan id " + std::to_string(plan));
  return DUDY_ERR_UNSUPPORTED;
}

size_t dudy_fdc_backward_workspace_size(int64_t B, int64_t D, int64_t L, int64_t T, int64_t N,
                                        int64_t K, int64_t off, int64_t dilation, int dtype,
                                        int plan) {
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (validate_fdc(s, dtype)) return 0;
  size_t ws = dudy::fdc_simt_bwd_workspace(s);
  if ((plan == DUDY_PLAN_AUTO || plan == DUDY_FDC_PLAN_TC) &&
      dudy::tc::bk_supported(s, dtype)) {
    const size_t t = dudy::tc::bk_workspace(s);
    if (t > ws) ws = t;
  }
  return (ws + 255) & ~size_t(255);
}

// ---- backward: grad_h part and grad_kc/grad_mix part ---------------------------------
// Zeroes bytes [0, head) and [tail, row) of every row of y (row a multiple of 16 and y
// 16-byte aligned; head and tail multiples of 2): 16-byte stores, 2-byte stores at the
// unaligned ends. Programmatic launch: it waits for the previous kernel of the stream, then
// lets the next one start; the tensor-core grad_h kernel that follows writes the positions
// in between (at most re-writing zeros next to them) and waits for this kernel before exiting.
__global__ void gh_fill_kernel(char *y, int64_t rows, int64_t row, int64_t head, int64_t tail) {
  dudy::pdl_wait();
  if (threadIdx.x == 0) dudy::pdl_trigger();
  const int64_t head16 = head & ~int64_t(15), tail16 = (tail + 15) & ~int64_t(15);
  const int64_t hc = head16 / 16, tc = tail16 < row ? (row - tail16) / 16 : 0;
  const int64_t per_row = hc + tc + 1;  // + one thread for the unaligned ends
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < rows * per_row;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / per_row, c = i % per_row;
    char *p = y + r * row;
    if (c < hc) {
      *reinterpret_cast<uint4 *>(p + c * 16) = make_uint4(0, 0, 0, 0);
    } else if (c < hc + tc) {
      *reinterpret_cast<uint4 *>(p + tail16 + (c - hc) * 16) = make_uint4(0, 0, 0, 0);
    } else {
      for (int64_t b = head16; b < head; b += 2) *reinterpret_cast<uint16_t *>(p + b) = 0;
      for (int64_t b = tail; b < tail16 && b < row; b += 2)
        *reinterpret_cast<uint16_t *>(p + b) = 0;
    }
  }
}

static int fdc_grad_h_impl(const void *go, const void *kc, const void *mix, void *grad_h,
                           const FdcShape &s, int dtype, bool tc, cudaStream_t st) {
  const size_t es = dudy::dtype_size(dtype);
  const int64_t lo = s.gh_lo(), hi = s.gh_hi();
  if (tc && aligned16(grad_h)) {
    // zero fill beside the tensor-core kernel (chunked calls: most of the full-length
    // grad_h is zero); rows are L * es bytes, a multiple of 16 on this plan
    const int64_t head = lo * (int64_t)es, tail = hi * (int64_t)es;
    const int64_t row = s.L * (int64_t)es;
    const bool fill = head > 0 || tail < row;
    if (fill) {
      const int64_t per_row =
          (head & ~int64_t(15)) / 16 + (row - ((tail + 15) & ~int64_t(15))) / 16 + 1;
      int64_t blocks = dudy::cdiv(s.B * s.D * per_row, 256);
      const int64_t cap = 4 * (int64_t)dudy::sm_count();
      if (blocks > cap) blocks = cap;
      if (dudy::launch_pdl(gh_fill_kernel, dim3((unsigned)blocks), dim3(256), 0, st,
                           (char *)grad_h, s.B * s.D, row, head, tail) != cudaSuccess)
        return dudy::check_launch("gh_fill_kernel");
    }
    return dudy::tc::conv_launch(true, kc, mix, go, grad_h, s, dtype, fill,
                                 dudy::device_err_word(), st);
  }
  if (lo > 0 && cudaMemset2DAsync(grad_h, s.L * es, 0, lo * es, s.B * s.D, st) != cudaSuccess)
    return dudy::check_launch("cudaMemset2DAsync(grad_h head)");
  if (hi < s.L && cudaMemset2DAsync((char *)grad_h + hi * es, s.L * es, 0, (s.L - hi) * es,
                                    s.B * s.D, st) != cudaSuccess)
    return dudy::check_launch("cudaMemset2DAsync(grad_h tail)");
  if (tc)
    return dudy::tc::conv_launch(true, kc, mix, go, grad_h, s, dtype, false,
                                 dudy::device_err_word(), st);
  return dudy::fdc_simt_grad_h(go, kc, mix, grad_h, s, dtype, st);
}

static int resolve_bwd_plan(int plan, bool tc_ok) {
  if (plan == DUDY_PLAN_AUTO) return tc_ok ? DUDY_FDC_PLAN_TC : DUDY_FDC_PLAN_SIMT;
  if (plan == DUDY_FDC_PLAN_SIMT) return plan;
  if (plan == DUDY_FDC_PLAN_TC) {
    if (!tc_ok) {
      dudy::set_error("plan tcgen05_tmem is not available for these shapes");
      return -2;
    }
    return plan;
  }
  dudy::set_error("unknown backward plan id " + std::to_string(plan));
  return -2;
}

int dudy_fdc_backward_grad_h(const void *go, const void *kc, const void *mix, void *grad_h,
                             int64_t B, int64_t D, int64_t L, int64_t T, int64_t N, int64_t K,
                             int64_t off, int64_t dilation, int dtype, int plan, void *stream) {
  dudy::clear_error();
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (int rc = validate_fdc(s, dtype)) return rc;
  if (!go || !kc || !mix || !grad_h) return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  const bool tc_ok = aligned16(go) && aligned16(kc) && aligned16(mix) &&
                     dudy::tc::conv_supported(true, s, dtype);
  plan = resolve_bwd_plan(plan, tc_ok);
  if (plan < 0) return DUDY_ERR_UNSUPPORTED;
  return fdc_grad_h_impl(go, kc, mix, grad_h, s, dtype, plan == DUDY_FDC_PLAN_TC,
                         reinterpret_cast<cudaStream_t>(stream));
}

// dep_late: called by dudy_fdc_backward right after its grad_h kernel (see bk_launch)
static int fdc_grad_kc_mix_entry(const void *go, const void *h, const void *kc, const void *mix,
                                 void *grad_kc, void *grad_mix, void *workspace,
                                 size_t workspace_bytes, int64_t B, int64_t D, int64_t L,
                                 int64_t T, int64_t N, int64_t K, int64_t off, int64_t dilation,
                                 int dtype, int plan, bool dep_late, const dudy::XRank *xr,
                                 void *stream) {
  dudy::clear_error();
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (int rc = validate_fdc(s, dtype)) return rc;
  if (!go || !h || !kc || !mix || !grad_kc || !grad_mix)
    return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  const bool tc_ok = aligned16(go) && aligned16(h) && aligned16(kc) && aligned16(mix) &&
                     dudy::tc::bk_supported(s, dtype);
  plan = resolve_bwd_plan(plan, tc_ok);
  if (plan < 0) return DUDY_ERR_UNSUPPORTED;
  const size_t need = dudy_fdc_backward_workspace_size(B, D, L, T, N, K, off, dilation, dtype, plan);
  if (workspace_bytes < need || (need > 0 && !workspace)) {
    dudy::set_error("workspace too small: need " + std::to_string(need) + " bytes, got " +
                    std::to_string(workspace_bytes));
    return DUDY_ERR_WORKSPACE;
  }
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  if (plan == DUDY_FDC_PLAN_TC)
    return dudy::tc::bk_launch(go, h, kc, mix, grad_kc, grad_mix, workspace, s, dtype,
                               dep_late, dudy::device_err_word(), xr, st);
  return dudy::fdc_simt_grad_kc_mix(go, h, mix, kc, grad_kc, grad_mix, workspace, s, dtype, xr,
                                    dudy::device_err_word(), st);
}

int dudy_fdc_backward_grad_kc_mix(const void *go, const void *h, const void *kc, const void *mix,
                                  void *grad_kc, void *grad_mix, void *workspace,
                                  size_t workspace_bytes, int64_t B, int64_t D, int64_t L,
                                  int64_t T, int64_t N, int64_t K, int64_t off, int64_t dilation,
                                  int dtype, int plan, void *stream) {
  return fdc_grad_kc_mix_entry(go, h, kc, mix, grad_kc, grad_mix, workspace, workspace_bytes, B,
                               D, L, T, N, K, off, dilation, dtype, plan, false, nullptr, stream);
}

static int fdc_backward_impl(const void *go, const void *h, const void *kc, const void *mix,
                             void *grad_h, void *grad_kc, void *grad_mix, void *workspace,
                             size_t workspace_bytes, int64_t B, int64_t D, int64_t L, int64_t T,
                             int64_t N, int64_t K, int64_t off, int64_t dilation, int dtype,
                             int plan, const dudy::XRank *xr, void *stream);

int dudy_fdc_backward(const void *go, const void *h, const void *kc, const void *mix,
                      void *grad_h, void *grad_kc, void *grad_mix, void *workspace,
                      size_t workspace_bytes, int64_t B, int64_t D, int64_t L, int64_t T,
                      int64_t N, int64_t K, int64_t off, int64_t dilation, int dtype, int plan,
                      void *stream) {
  return fdc_backward_impl(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, workspace_bytes,
                           B, D, L, T, N, K, off, dilation, dtype, plan, nullptr, stream);
}

size_t dudy_fdc_exchange_bytes(int64_t D, int64_t N) {
  if (D <= 0 || N <= 0) return 0;
  return (dudy::xrank_buffer_bytes(D * N) + 255) & ~size_t(255);
}

// The exchange descriptor as the kernels take it (mode: see dudy::XRank).
static int xrank_of(const DudyPeerExchange *xchg, int mode, void *prev_out, dudy::XRank *xr,
                    const char *who) {
  if (!xchg || xchg->world < 1 || xchg->world > DUDY_MAX_PEERS || xchg->rank < 0 ||
      xchg->rank >= xchg->world || xchg->epoch == 0)
    return dudy::set_error(std::string(who) + ": bad exchange descriptor (rank, world, epoch)"),
           DUDY_ERR_INVALID;
  *xr = dudy::XRank{};
  for (int r = 0; r < xchg->world; ++r) {
    if (!xchg->bufs[r] || !aligned16(xchg->bufs[r]))
      return dudy::set_error(std::string(who) + ": exchange buffer pointers must be non-null "
                             "and 16-byte aligned"),
             DUDY_ERR_INVALID;
    xr->bufs[r] = (float *)xchg->bufs[r];
  }
  xr->rank = xchg->rank;
  xr->world = xchg->world;
  xr->epoch = xchg->epoch;
  xr->mode = mode;
  xr->prev_out = prev_out;
  return DUDY_OK;
}

int dudy_fdc_backward_dp(const void *go, const void *h, const void *kc, const void *mix,
                         void *grad_h, void *grad_kc, void *grad_mix, void *workspace,
                         size_t workspace_bytes, const DudyPeerExchange *xchg, int64_t B,
                         int64_t D, int64_t L, int64_t T, int64_t N, int64_t K, int64_t off,
                         int64_t dilation, int dtype, int plan, void *stream) {
  dudy::clear_error();
  dudy::XRank xr;
  if (int rc = xrank_of(xchg, 0, nullptr, &xr, "dudy_fdc_backward_dp")) return rc;
  return fdc_backward_impl(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, workspace_bytes,
                           B, D, L, T, N, K, off, dilation, dtype, plan,
                           xchg->world > 1 ? &xr : nullptr, stream);
}

int dudy_fdc_backward_dp_deferred(const void *go, const void *h, const void *kc, const void *mix,
                                  void *grad_h, void *grad_kc, void *grad_mix,
                                  void *grad_mix_prev, void *workspace, size_t workspace_bytes,
                                  const DudyPeerExchange *xchg, int64_t B, int64_t D, int64_t L,
                                  int64_t T, int64_t N, int64_t K, int64_t off, int64_t dilation,
                                  int dtype, int plan, void *stream) {
  dudy::clear_error();
  dudy::XRank xr;
  if (int rc = xrank_of(xchg, 1, grad_mix_prev, &xr, "dudy_fdc_backward_dp_deferred")) return rc;
  if (xchg->epoch > 1 && !grad_mix_prev)
    return dudy::set_error("dudy_fdc_backward_dp_deferred: grad_mix_prev is null"),
           DUDY_ERR_INVALID;
  return fdc_backward_impl(go, h, kc, mix, grad_h, grad_kc, grad_mix, workspace, workspace_bytes,
                           B, D, L, T, N, K, off, dilation, dtype, plan, &xr, stream);
}

int dudy_fdc_exchange_finish(const DudyPeerExchange *xchg, void *grad_mix, int64_t D, int64_t N,
                             int dtype, void *stream) {
  dudy::clear_error();
  dudy::XRank xr;
  if (int rc = xrank_of(xchg, 2, nullptr, &xr, "dudy_fdc_exchange_finish")) return rc;
  if (!grad_mix || D <= 0 || N <= 0 || !dtype_ok(dtype))
    return dudy::set_error("dudy_fdc_exchange_finish: bad arguments"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  return dudy::xrank_reduce_launch(nullptr, 0, grad_mix, D * N, dtype, xr,
                                   dudy::device_err_word(), reinterpret_cast<cudaStream_t>(stream));
}

static int fdc_backward_impl(const void *go, const void *h, const void *kc, const void *mix,
                             void *grad_h, void *grad_kc, void *grad_mix, void *workspace,
                             size_t workspace_bytes, int64_t B, int64_t D, int64_t L, int64_t T,
                             int64_t N, int64_t K, int64_t off, int64_t dilation, int dtype,
                             int plan, const dudy::XRank *xr, void *stream) {
  dudy::clear_error();
  const FdcShape s = fdc_shape(B, D, L, T, N, K, off, dilation);
  if (int rc = validate_fdc(s, dtype)) return rc;
  if (!go || !h || !kc || !mix || !grad_h || !grad_kc || !grad_mix)
    return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  // one plan for the whole backward: tcgen05 only when both halves can use it
  plan = resolve_bwd_plan(plan, tc_bwd_ok(go, h, kc, mix, s, dtype));
  if (plan < 0) return DUDY_ERR_UNSUPPORTED;
  // grad_h first; the grad_kc/grad_mix kernel reads none of its output, so on the tcgen05
  // plan it starts on each SM as soon as the grad_h kernel leaves it (dep_late)
  if (int rc = dudy_fdc_backward_grad_h(go, kc, mix, grad_h, B, D, L, T, N, K, off, dilation,
                                        dtype, plan, stream))
    return rc;
  return fdc_grad_kc_mix_entry(go, h, kc, mix, grad_kc, grad_mix, workspace, workspace_bytes, B,
                               D, L, T, N, K, off, dilation, dtype, plan,
                               plan == DUDY_FDC_PLAN_TC, xr, stream);
}

// Reads (and optionally clears) the device error word of the current device. A nonzero
// value means a bounded wait inside a tensor-core kernel timed out (the kernel returned
// early and its outputs are not valid). Synchronizes the device.
int dudy_device_error(int reset) {
  int info[4];
  return dudy_device_error_info(info, reset);
}

int dudy_device_error_info(int *info4, int reset) {
  int *p = dudy::device_err_word();
  if (!p || !info4) return -1;
  if (cudaMemcpy(info4, p, 4 * sizeof(int), cudaMemcpyDeviceToHost) != cudaSuccess) return -1;
  if (reset && info4[0]) {
    const int z[4] = {0, 0, 0, 0};
    cudaMemcpy(p, z, sizeof(z), cudaMemcpyHostToDevice);
  }
  return info4[0];
}

// ---- self-test of the bounded waits ---------------------------------------------------
// One CTA of two warps, as the tensor-core kernels are organised: warp 1 owns a TMEM
// allocation; warp 0 waits (bounded by `limit_ns`) on an mbarrier that nothing arrives at,
// so the wait gives up, records its site in the device error record and raises the CTA's
// abort flag; warp 1, waiting on another barrier with the kernels' normal limit, sees the
// abort flag and returns; the CTA then frees its TMEM and exits. g_selftest_result gets
// each warp's wait result (1 = completed, 0 = gave up).
__device__ int g_selftest_result[2];

__global__ void wait_timeout_selftest_kernel(int *err, unsigned long long limit_ns) {
  using namespace dudy::sm100;
  __shared__ __align__(8) uint64_t bars[2];
  __shared__ uint32_t tmem_hold;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5;
  if (threadIdx.x == 0) {
    mbar_init(&bars[0], 1);
    mbar_init(&bars[1], 1);
    abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(&tmem_hold, 32);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  bool ok;
  if (warp == 0)
    ok = mbar_wait_limit(&bars[0], 0, err, &abort_flag, limit_ns, kSelftestSite, 7);
  else
    ok = mbar_wait_limit(&bars[1], 0, err, &abort_flag, kWaitLimitNs, kSelftestSite + 1, 8);
  ok = __all_sync(0xffffffffu, ok);
  if ((threadIdx.x & 31) == 0) g_selftest_result[warp] = ok ? 1 : 0;
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_hold, 32);
  }
}

// ---- fused source conv ------------------------------------------------------------------
static int validate_fscm(const FscmShape &s, int dtype) {
  if (s.B <= 0) return dudy::set_error("B must be positive."), DUDY_ERR_INVALID;
  if (s.D <= 0) return dudy::set_error("D must be positive."), DUDY_ERR_INVALID;
  if (s.L <= 0) return dudy::set_error("L must be positive."), DUDY_ERR_INVALID;
  if (s.C <= 0) return dudy::set_error("C must be positive."), DUDY_ERR_INVALID;
  if (s.S <= 0) return dudy::set_error("S must be positive."), DUDY_ERR_INVALID;
  if (s.off < 0) return dudy::set_error("off must be non-negative."), DUDY_ERR_INVALID;
  if (s.T <= 0) return dudy::set_error("T must be positive."), DUDY_ERR_INVALID;
  if (s.off + s.T > s.L)
    return dudy::set_error("off + T must be <= L, got off=" + std::to_string(s.off) + ", T=" +
                           std::to_string(s.T) + ", L=" + std::to_string(s.L) + "."),
           DUDY_ERR_INVALID;
  if (s.dil <= 0) return dudy::set_error("dilation must be positive."), DUDY_ERR_INVALID;
  if (!dtype_ok(dtype)) return dudy::set_error("Unsupported dtype."), DUDY_ERR_INVALID;
  if (s.B * s.D * s.L >= ((int64_t)1 << 31) || s.dil * (s.S - 1) >= ((int64_t)1 << 24))
    return dudy::set_error("tensor too large."), DUDY_ERR_INVALID;
  return DUDY_OK;
}

int dudy_fscm_forward_plan_legal(int plan, int64_t D, int64_t C, int64_t S, int64_t off,
                                 int64_t dilation) {
  // fused_source_conv_mixed_forward.cu:309-365
  const bool nb = off >= dilation * (S - 1);
  switch (plan) {
    case 0: return 1;
    case 1: return C == 8 && S == 3;
    case 2: return C == 32 && S == 3;
    case 3: return D == 256 && C == 16 && S == 3;
    case 100: return nb;
    case 101: return nb && C == 8 && S == 3;
    case 102: return nb && C == 32 && S == 3;
    case 103: return nb && D == 256 && C == 16 && S == 3;
    default: return 0;
  }
}

int dudy_fscm_forward_default_plan(int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                                   int64_t off, int64_t T, int64_t dilation) {
  // fused_source_conv_mixed_forward.cu:596-662: specialised shapes first, NoBoundary when
  // no tap can reach before index 0
  (void)B; (void)L; (void)T;
  const int nb = off >= dilation * (S - 1) ? 100 : 0;
  if (D == 256 && C == 16 && S == 3) return 3 + nb;
  if (C == 8 && S == 3) return 1 + nb;
  if (C == 32 && S == 3) return 2 + nb;
  return 0 + nb;
}

int dudy_fscm_forward(const void *x, const void *weight, const void *bias, const void *mix_w,
                      const void *mix_b, void *out, int64_t B, int64_t D, int64_t L, int64_t C,
                      int64_t S, int64_t off, int64_t T, int64_t dilation, int dtype, int plan,
                      void *stream) {
  dudy::clear_error();
  const FscmShape s{B, D, L, C, S, off, T, dilation, bias != nullptr};
  if (int rc = validate_fscm(s, dtype)) return rc;
  if (!x || !weight || !mix_w || !mix_b || !out)
    return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (plan != DUDY_PLAN_AUTO && !dudy_fscm_forward_plan_legal(plan, D, C, S, off, dilation)) {
    dudy::set_error("fused_source_conv_mixed_forward_plan: illegal plan " + std::to_string(plan) +
                    " for D=" + std::to_string(D) + ", C=" + std::to_string(C) + ", S=" +
                    std::to_string(S) + ", off=" + std::to_string(off) + ", dilation=" +
                    std::to_string(dilation));
    return DUDY_ERR_UNSUPPORTED;
  }
  if (!dudy::fscm_shapes_fit(s, 0))
    return dudy::set_error("source conv halo too large for shared memory"), DUDY_ERR_UNSUPPORTED;
  if (int rc = device_ok()) return rc;
  return dudy::fscm_forward_impl(x, weight, bias, mix_w, mix_b, out, s, dtype,
                                 reinterpret_cast<cudaStream_t>(stream));
}

int dudy_fscm_backward_plan_legal(int plan, int64_t C, int64_t S, int64_t tile_t) {
  // fused_source_conv_mixed_backward.cu:358-393 (C <= 64 and S <= 8 for the reduce plans)
  switch (plan) {
    case 0: return 1;
    case 1:
    case 2: return tile_t > 0 && C <= 64 && S <= 8;
    default: return 0;
  }
}

int dudy_fscm_backward_default_plan(int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                                    int64_t off, int64_t T, int64_t dilation) {
  // fused_source_conv_mixed_backward.cu:672-730
  (void)off;
  if (!(C <= 64 && S <= 8)) return 0;
  if (T <= 32 || B * D * T < 8192) return 0;
  if ((T + dilation * (S - 1)) * 2 >= L && C <= 32 && S <= 4) return 2;
  return 1;
}

size_t dudy_fscm_backward_workspace_size(int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                                         int64_t off, int64_t T, int64_t dilation, int dtype,
                                         int plan, int64_t tile_t) {
  const FscmShape s{B, D, L, C, S, off, T, dilation, true};
  if (validate_fscm(s, dtype)) return 0;
  const int64_t tt = (plan == 1 || plan == 2) ? tile_t : 0;
  return (dudy::fscm_bwd_workspace(s, tt) + 255) & ~size_t(255);
}

int dudy_fscm_backward(const void *go, const void *x, const void *weight, const void *bias,
                       const void *mix_w, const void *mix_b, void *grad_x, void *grad_w,
                       void *grad_bias, void *grad_mix_w, void *grad_mix_b, void *workspace,
                       size_t workspace_bytes, int64_t B, int64_t D, int64_t L, int64_t C,
                       int64_t S, int64_t off, int64_t T, int64_t dilation, int dtype, int plan,
                       int64_t tile_t, void *stream) {
  dudy::clear_error();
  (void)mix_b;
  const FscmShape s{B, D, L, C, S, off, T, dilation, bias != nullptr};
  if (int rc = validate_fscm(s, dtype)) return rc;
  if (!go || !x || !weight || !mix_w || !grad_x || !grad_w || !grad_mix_w || !grad_mix_b ||
      (bias && !grad_bias))
    return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  if (plan != DUDY_PLAN_AUTO && !dudy_fscm_backward_plan_legal(plan, C, S, tile_t)) {
    dudy::set_error("fused_source_conv_mixed_backward_plan: illegal plan=" + std::to_string(plan) +
                    ", tile_t=" + std::to_string(tile_t));
    return DUDY_ERR_UNSUPPORTED;
  }
  const int64_t tt = (plan == 1 || plan == 2) ? tile_t : 0;
  if (!dudy::fscm_shapes_fit(s, tt))
    return dudy::set_error("source conv halo too large for shared memory"), DUDY_ERR_UNSUPPORTED;
  const size_t need = dudy_fscm_backward_workspace_size(B, D, L, C, S, off, T, dilation, dtype,
                                                        plan, tile_t);
  if (workspace_bytes < need || !workspace) {
    dudy::set_error("workspace too small: need " + std::to_string(need) + " bytes, got " +
                    std::to_string(workspace_bytes));
    return DUDY_ERR_WORKSPACE;
  }
  if (int rc = device_ok()) return rc;
  return dudy::fscm_backward_impl(go, x, weight, bias, mix_w, grad_x, grad_w, grad_bias,
                                  grad_mix_w, grad_mix_b, workspace, s, tt, dtype,
                                  reinterpret_cast<cudaStream_t>(stream));
}

int dudy_selftest_wait_timeout(int limit_us, int *results2) {
  dudy::clear_error();
  if (!results2 || limit_us <= 0 || limit_us > 1000000)
    return dudy::set_error("dudy_selftest_wait_timeout: limit_us must be in (0, 1e6]"),
           DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  int *err = dudy::device_err_word();
  if (!err) return dudy::set_error("device error record not available"), DUDY_ERR_CUDA;
  const int init[2] = {-1, -1};
  if (cudaMemcpyToSymbol(g_selftest_result, init, sizeof(init)) != cudaSuccess)
    return dudy::check_launch("cudaMemcpyToSymbol(selftest result)");
  wait_timeout_selftest_kernel<<<1, 64>>>(err, (unsigned long long)limit_us * 1000ull);
  if (int rc = dudy::check_launch("wait_timeout_selftest_kernel")) return rc;
  if (cudaMemcpyFromSymbol(results2, g_selftest_result, sizeof(init)) != cudaSuccess)
    return dudy::check_launch("wait_timeout_selftest_kernel");
  return DUDY_OK;
}

int dudy_check_phi_approx(float *max_abs_err) {
  dudy::clear_error();
  if (!max_abs_err) return dudy::set_error("null pointer"), DUDY_ERR_INVALID;
  if (int rc = device_ok()) return rc;
  return dudy::check_phi_approx(max_abs_err);
}

}  // extern "C"
