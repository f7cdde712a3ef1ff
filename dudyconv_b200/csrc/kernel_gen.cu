// kernel_gen.cu -- the tail of the reference's kernel generator in one pass each way.
//
// Forward (StreamingKernelGenConv1d._logits_to_kernel, backbone_dil_unshared.py:1821-1900:
// reshape logits [B, N*K, T] to [B,N,K,T], softmax over K, flip K so that kk = 0 is the
// current token, permute to [B,K,N,T] and make it contiguous):
//     kc[b,kk,n,t] = y[b,n,K-1-kk,t],   y[b,n,:,t] = softmax_k(logits[b, n*K + k, t])
// Backward (autograd of the same: softmax backward after undoing the flip and permute):
//     grad_logits[b, n*K + k, t] = y_k * (g_k - sum_j y_j g_j),
//     y_k = kc[b,K-1-k,n,t],  g_k = grad_kc[b,K-1-k,n,t]
// PyTorch runs this as three kernels forward (softmax, flip copy, permute copy) and three
// backward, each a full read and write of the [B,K,N,T] tensor; here each direction is one
// read of its inputs and one write of its output. Arithmetic is fp32 (softmax with the
// maximum subtracted, exact division), rounded once to the tensor type, as PyTorch's
// softmax does for 16-bit inputs.
//
// Thread = (b, n, 8 consecutive tokens): 16-byte loads of K logit rows and 16-byte stores
// of K kc rows (consecutive threads take consecutive token groups: coalesced), when T is
// a multiple of 8 and the tensors are 16-byte aligned; otherwise one token per thread.
#include "common.cuh"

namespace dudy {
namespace {

constexpr int kKMax = 16;  // taps held in registers; larger K loops over memory

template <typename T>
__device__ __forceinline__ void load8(const T *p, float (&v)[8]) {
  const uint4 q = *reinterpret_cast<const uint4 *>(p);
  const T *e = reinterpret_cast<const T *>(&q);
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = Elem<T>::to_f(e[i]);
}

template <>
__device__ __forceinline__ void load8<float>(const float *p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4 *>(p);
  const float4 b = *reinterpret_cast<const float4 *>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <typename T>
__device__ __forceinline__ void store8(T *p, const float (&v)[8]) {
  uint4 q;
  T *e = reinterpret_cast<T *>(&q);
#pragma unroll
  for (int i = 0; i < 8; ++i) e[i] = Elem<T>::from_f(v[i]);
  *reinterpret_cast<uint4 *>(p) = q;
}

template <>
__device__ __forceinline__ void store8<float>(float *p, const float (&v)[8]) {
  *reinterpret_cast<float4 *>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4 *>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}

// ---- forward -------------------------------------------------------------------------
template <typename T, int KC>
__global__ void __launch_bounds__(256)
logits_to_kc_vec8_kernel(const T *__restrict__ logits, T *__restrict__ kc, int64_t B, int N,
                         int K, int64_t T8) {
  const int kdim = KC > 0 ? KC : K;
  const int64_t total = B * N * T8;
  const int64_t Tn = T8 * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = (i % T8) * 8;
    const int64_t bn = i / T8;
    const int n = (int)(bn % N);
    const int64_t b = bn / N;
    const T *src = logits + ((b * N + n) * kdim) * Tn + t;
    T *dst = kc + (b * kdim * N + n) * Tn + t;
    if (KC > 0) {
      float x[KC > 0 ? KC : 1][8];
#pragma unroll
      for (int k = 0; k < KC; ++k) load8(src + k * Tn, x[k]);
      float m[8], s[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) m[j] = x[0][j];
#pragma unroll
      for (int k = 1; k < KC; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], x[k][j]);
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = 0.f;
#pragma unroll
      for (int k = 0; k < KC; ++k)
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          x[k][j] = expf(x[k][j] - m[j]);
          s[j] += x[k][j];
        }
#pragma unroll
      for (int k = 0; k < KC; ++k) {
        float y[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = x[k][j] / s[j];
        // tap kk = K-1-k
        store8(dst + (int64_t)(KC - 1 - k) * N * Tn, y);
      }
    } else {
      // any K: max, then sum, then write (the K rows stay in L1 between the passes)
      float m[8], s[8], v[8];
      load8(src, m);
      for (int k = 1; k < kdim; ++k) {
        load8(src + k * Tn, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) m[j] = fmaxf(m[j], v[j]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) s[j] = 0.f;
      for (int k = 0; k < kdim; ++k) {
        load8(src + k * Tn, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) s[j] += expf(v[j] - m[j]);
      }
      for (int k = 0; k < kdim; ++k) {
        load8(src + k * Tn, v);
#pragma unroll
        for (int j = 0; j < 8; ++j) v[j] = expf(v[j] - m[j]) / s[j];
        store8(dst + (int64_t)(kdim - 1 - k) * N * Tn, v);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
logits_to_kc_scalar_kernel(const T *__restrict__ logits, T *__restrict__ kc, int64_t B, int N,
                           int K, int64_t Tn) {
  const int64_t total = B * N * Tn;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i % Tn;
    const int64_t bn = i / Tn;
    const int n = (int)(bn % N);
    const int64_t b = bn / N;
    const T *src = logits + ((b * N + n) * K) * Tn + t;
    T *dst = kc + (b * K * N + n) * Tn + t;
    float m = ldf(src);
    for (int k = 1; k < K; ++k) m = fmaxf(m, ldf(src + k * Tn));
    float s = 0.f;
    for (int k = 0; k < K; ++k) s += expf(ldf(src + k * Tn) - m);
    for (int k = 0; k < K; ++k)
      stf(dst + (int64_t)(K - 1 - k) * N * Tn, expf(ldf(src + k * Tn) - m) / s);
  }
}

// ---- backward ------------------------------------------------------------------------
template <typename T, int KC>
__global__ void __launch_bounds__(256)
logits_to_kc_bwd_vec8_kernel(const T *__restrict__ kc, const T *__restrict__ gkc,
                             T *__restrict__ glogits, int64_t B, int N, int K, int64_t T8) {
  const int kdim = KC > 0 ? KC : K;
  const int64_t total = B * N * T8;
  const int64_t Tn = T8 * 8;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = (i % T8) * 8;
    const int64_t bn = i / T8;
    const int n = (int)(bn % N);
    const int64_t b = bn / N;
    const int64_t kc_off = (b * kdim * N + n) * Tn + t;  // tap kk at + kk * N * Tn
    T *dst = glogits + ((b * N + n) * kdim) * Tn + t;    // logit row k at + k * Tn
    float dot[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) dot[j] = 0.f;
    if (KC > 0) {
      float y[KC > 0 ? KC : 1][8], g[KC > 0 ? KC : 1][8];
#pragma unroll
      for (int kk = 0; kk < KC; ++kk) {
        load8(kc + kc_off + (int64_t)kk * N * Tn, y[kk]);
        load8(gkc + kc_off + (int64_t)kk * N * Tn, g[kk]);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot[j] += y[kk][j] * g[kk][j];
      }
#pragma unroll
      for (int kk = 0; kk < KC; ++kk) {
        float o[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = y[kk][j] * (g[kk][j] - dot[j]);
        store8(dst + (int64_t)(KC - 1 - kk) * Tn, o);
      }
    } else {
      float y[8], g[8];
      for (int kk = 0; kk < kdim; ++kk) {
        load8(kc + kc_off + (int64_t)kk * N * Tn, y);
        load8(gkc + kc_off + (int64_t)kk * N * Tn, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) dot[j] += y[j] * g[j];
      }
      for (int kk = 0; kk < kdim; ++kk) {
        load8(kc + kc_off + (int64_t)kk * N * Tn, y);
        load8(gkc + kc_off + (int64_t)kk * N * Tn, g);
#pragma unroll
        for (int j = 0; j < 8; ++j) y[j] = y[j] * (g[j] - dot[j]);
        store8(dst + (int64_t)(kdim - 1 - kk) * Tn, y);
      }
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256)
logits_to_kc_bwd_scalar_kernel(const T *__restrict__ kc, const T *__restrict__ gkc,
                               T *__restrict__ glogits, int64_t B, int N, int K, int64_t Tn) {
  const int64_t total = B * N * Tn;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
       i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = i % Tn;
    const int64_t bn = i / Tn;
    const int n = (int)(bn % N);
    const int64_t b = bn / N;
    const int64_t kc_off = (b * K * N + n) * Tn + t;
    T *dst = glogits + ((b * N + n) * K) * Tn + t;
    float dot = 0.f;
    for (int kk = 0; kk < K; ++kk)
      dot += ldf(kc + kc_off + (int64_t)kk * N * Tn) * ldf(gkc + kc_off + (int64_t)kk * N * Tn);
    for (int kk = 0; kk < K; ++kk) {
      const float y = ldf(kc + kc_off + (int64_t)kk * N * Tn);
      const float g = ldf(gkc + kc_off + (int64_t)kk * N * Tn);
      stf(dst + (int64_t)(K - 1 - kk) * Tn, y * (g - dot));
    }
  }
}

bool al16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

unsigned grid_for(int64_t work) {
  int64_t g = cdiv(work, 256);
  const int64_t cap = 8 * (int64_t)sm_count();
  return (unsigned)(g < 1 ? 1 : (g > cap ? cap : g));
}

template <typename T>
int fwd_launch(const void *logits, void *kc, int64_t B, int64_t N, int64_t K, int64_t Tn,
               cudaStream_t st) {
  const T *x = (const T *)logits;
  T *y = (T *)kc;
  if (Tn % 8 == 0 && al16(logits) && al16(kc)) {
    const int64_t T8 = Tn / 8;
    const unsigned g = grid_for(B * N * T8);
    switch (K) {
      case 1: logits_to_kc_vec8_kernel<T, 1><<<g, 256, 0, st>>>(x, y, B, (int)N, 1, T8); break;
      case 2: logits_to_kc_vec8_kernel<T, 2><<<g, 256, 0, st>>>(x, y, B, (int)N, 2, T8); break;
      case 3: logits_to_kc_vec8_kernel<T, 3><<<g, 256, 0, st>>>(x, y, B, (int)N, 3, T8); break;
      case 4: logits_to_kc_vec8_kernel<T, 4><<<g, 256, 0, st>>>(x, y, B, (int)N, 4, T8); break;
      case 5: logits_to_kc_vec8_kernel<T, 5><<<g, 256, 0, st>>>(x, y, B, (int)N, 5, T8); break;
      default: logits_to_kc_vec8_kernel<T, 0><<<g, 256, 0, st>>>(x, y, B, (int)N, (int)K, T8);
    }
  } else {
    logits_to_kc_scalar_kernel<T><<<grid_for(B * N * Tn), 256, 0, st>>>(x, y, B, (int)N, (int)K,
                                                                        Tn);
  }
  return check_launch("logits_to_kc_kernel");
}

template <typename T>
int bwd_launch(const void *kc, const void *gkc, void *glogits, int64_t B, int64_t N, int64_t K,
               int64_t Tn, cudaStream_t st) {
  const T *y = (const T *)kc;
  const T *g = (const T *)gkc;
  T *o = (T *)glogits;
  if (Tn % 8 == 0 && al16(kc) && al16(gkc) && al16(glogits)) {
    const int64_t T8 = Tn / 8;
    const unsigned gr = grid_for(B * N * T8);
    switch (K) {
      case 1: logits_to_kc_bwd_vec8_kernel<T, 1><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, 1, T8); break;
      case 2: logits_to_kc_bwd_vec8_kernel<T, 2><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, 2, T8); break;
      case 3: logits_to_kc_bwd_vec8_kernel<T, 3><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, 3, T8); break;
      case 4: logits_to_kc_bwd_vec8_kernel<T, 4><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, 4, T8); break;
      case 5: logits_to_kc_bwd_vec8_kernel<T, 5><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, 5, T8); break;
      default:
        logits_to_kc_bwd_vec8_kernel<T, 0><<<gr, 256, 0, st>>>(y, g, o, B, (int)N, (int)K, T8);
    }
  } else {
    logits_to_kc_bwd_scalar_kernel<T><<<grid_for(B * N * Tn), 256, 0, st>>>(y, g, o, B, (int)N,
                                                                            (int)K, Tn);
  }
  return check_launch("logits_to_kc_bwd_kernel");
}

int validate(int64_t B, int64_t N, int64_t K, int64_t Tn, int dtype) {
  if (B <= 0 || N <= 0 || K <= 0 || Tn <= 0)
    return set_error("B, N, K and T must be positive."), DUDY_ERR_INVALID;
  if (dtype != DUDY_DTYPE_F32 && dtype != DUDY_DTYPE_F16 && dtype != DUDY_DTYPE_BF16)
    return set_error("Unsupported dtype."), DUDY_ERR_INVALID;
  if (B * N * K * Tn >= ((int64_t)1 << 40))
    return set_error("tensor too large."), DUDY_ERR_INVALID;
  return DUDY_OK;
}

}  // namespace
}  // namespace dudy

extern "C" int dudy_logits_to_kernel(const void *logits, void *kc, int64_t B, int64_t N,
                                     int64_t K, int64_t T, int dtype, void *stream) {
  dudy::clear_error();
  if (int rc = dudy::validate(B, N, K, T, dtype)) return rc;
  if (!logits || !kc) return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DUDY_DTYPE_F32: return dudy::fwd_launch<float>(logits, kc, B, N, K, T, st);
    case DUDY_DTYPE_F16: return dudy::fwd_launch<__half>(logits, kc, B, N, K, T, st);
    default: return dudy::fwd_launch<__nv_bfloat16>(logits, kc, B, N, K, T, st);
  }
}

extern "C" int dudy_logits_to_kernel_backward(const void *kc, const void *grad_kc,
                                              void *grad_logits, int64_t B, int64_t N,
                                              int64_t K, int64_t T, int dtype, void *stream) {
  dudy::clear_error();
  if (int rc = dudy::validate(B, N, K, T, dtype)) return rc;
  if (!kc || !grad_kc || !grad_logits)
    return dudy::set_error("null tensor pointer"), DUDY_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case DUDY_DTYPE_F32: return dudy::bwd_launch<float>(kc, grad_kc, grad_logits, B, N, K, T, st);
    case DUDY_DTYPE_F16: return dudy::bwd_launch<__half>(kc, grad_kc, grad_logits, B, N, K, T, st);
    default: return dudy::bwd_launch<__nv_bfloat16>(kc, grad_kc, grad_logits, B, N, K, T, st);
  }
}
