// fdc_simt.cu -- CUDA-core kernels for the fused dynamic causal convolution.
//
// These cover every shape the reference accepts (any D, N, K, dilation, offset, T, L)
// and are the fp32 production path (fp32 FMA keeps the rel-1e-5 fp32 contract).
// fp16/bf16 at the hot shapes go to the tcgen05 kernels in fdc_tc.cu instead.
//
// Semantics follow the reference's generic forward (cuda_ops/
// fused_dynamic_conv_forward_direct_exec.cu:26-75) and its autograd backward
// (test_fused_dynamic_conv_against_reference.py:91-189); the kernels are this
// library's own register-tiled designs:
//   forward   block = (64 t) x (32 d) x b, thread = 4 t x 2 d, W_kk built in registers
//             from smem tiles of kc and mix, then multiplied by the shifted h.
//   grad_h    same tiling over h positions s; the tap shift moves to kc and go.
//   grad_kc   block = (64 t) x (32 n) x (b,kk); G = go * shifted h built in smem.
//   grad_mix  split-K over (b, kk, t): per-split fp32 partials in the caller's
//             workspace, then a fixed-order reduction (deterministic).
#include "common.cuh"

namespace dudy {
namespace {

constexpr int kTT = 64;   // tokens per block
constexpr int kTD = 32;   // channels per block
constexpr int kNC = 16;   // contraction chunk

// -----------------------------------------------------------------------------------
// forward / grad_h share one kernel body:
//   FWD : y[b,d,s]  = sum_kk h[b,d,off+s-kk*dil] * W_kk[b,d,s]           s in [0,T)
//   GH  : y[b,d,s]  = sum_kk go[b,d,s-off+kk*dil] * W_kk[b,d,s-off+kk*dil] s in [s_lo,s_hi)
// -----------------------------------------------------------------------------------
template <typename T, bool GH>
__global__ void __launch_bounds__(256)
fdc_conv_simt_kernel(const T *__restrict__ src,   // FWD: h [B,D,L];  GH: go [B,D,T]
                     const T *__restrict__ kc, const T *__restrict__ mix,
                     T *__restrict__ y,            // FWD: out [B,D,T]; GH: grad_h [B,D,L]
                     int D, int L, int Tn, int N, int K, int off, int dil, int s_lo,
                     int s_hi) {
  __shared__ float Ms[kNC][kTD + 1];
  __shared__ __align__(16) float Ks[kNC][kTT];
  const int b = blockIdx.z;
  const int d0 = blockIdx.y * kTD;
  const int s0 = s_lo + blockIdx.x * kTT;
  const int tid = threadIdx.x;
  const int tx = tid & 15, ty = tid >> 4;

  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  const int64_t kc_b = (int64_t)b * K * N * Tn;
  for (int kk = 0; kk < K; ++kk) {
    // token index t that feeds output position s: FWD t = s, GH t = s - off + kk*dil
    const int tshift = GH ? (kk * dil - off) : 0;
    float w[2][4];
#pragma unroll
    for (int i = 0; i < 2; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) w[i][j] = 0.f;

    for (int n0 = 0; n0 < N; n0 += kNC) {
      for (int i = tid; i < kNC * kTD; i += 256) {
        const int n = i % kNC, dd = i / kNC;
        const int d = d0 + dd, nn = n0 + n;
        Ms[n][dd] = (d < D && nn < N) ? ldf(mix + (int64_t)d * N + nn) : 0.f;
      }
      for (int i = tid; i < kNC * kTT; i += 256) {
        const int n = i / kTT, ss = i % kTT;
        const int t = s0 + ss + tshift, nn = n0 + n;
        Ks[n][ss] = (nn < N && t >= 0 && t < Tn)
                        ? ldf(kc + kc_b + ((int64_t)kk * N + nn) * Tn + t)
                        : 0.f;
      }
      __syncthreads();
      const int nlim = min(kNC, N - n0);
      for (int n = 0; n < nlim; ++n) {
        const float m0 = Ms[n][ty * 2], m1 = Ms[n][ty * 2 + 1];
        const float4 kv = *reinterpret_cast<const float4 *>(&Ks[n][tx * 4]);
        const float k[4] = {kv.x, kv.y, kv.z, kv.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          w[0][j] = fmaf(m0, k[j], w[0][j]);
          w[1][j] = fmaf(m1, k[j], w[1][j]);
        }
      }
      __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int d = d0 + ty * 2 + i;
      if (d >= D) continue;
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int s = s0 + tx * 4 + j;
        if (s >= s_hi) continue;
        if (GH) {
          const int t = s + tshift;
          if (t >= 0 && t < Tn) acc[i][j] += w[i][j] * ldf(src + ((int64_t)b * D + d) * Tn + t);
        } else {
          const int hs = off + s - kk * dil;
          if (hs >= 0) acc[i][j] += w[i][j] * ldf(src + ((int64_t)b * D + d) * L + hs);
        }
      }
    }
  }
  const int ylen = GH ? L : Tn;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int d = d0 + ty * 2 + i;
    if (d >= D) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int s = s0 + tx * 4 + j;
      if (s < s_hi) stf(y + ((int64_t)b * D + d) * ylen + s, acc[i][j]);
    }
  }
}

// -----------------------------------------------------------------------------------
// grad_kc[b,kk,n,t] = sum_d mix[d,n] * go[b,d,t] * h[b,d,off+t-kk*dil]
// block = (64 t) x (32 n) x (b*K + kk); thread = 4 t x 2 n
// -----------------------------------------------------------------------------------
template <typename T>
__global__ void __launch_bounds__(256)
fdc_grad_kc_simt_kernel(const T *__restrict__ go, const T *__restrict__ h,
                        const T *__restrict__ mix, T *__restrict__ grad_kc, int D, int L,
                        int Tn, int N, int K, int off, int dil) {
  __shared__ float Ms[kNC][kTD + 1];                // mix[d][n] chunk, n fastest
  __shared__ __align__(16) float Gs[kNC][kTT];      // G[d][t] chunk
  const int bk = blockIdx.z;
  const int b = bk / K, kk = bk % K;
  const int n0 = blockIdx.y * kTD;
  const int t0 = blockIdx.x * kTT;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float acc[2][4];
#pragma unroll
  for (int i = 0; i < 2; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  for (int dc = 0; dc < D; dc += kNC) {
    for (int i = tid; i < kNC * kTD; i += 256) {
      const int nn = i % kTD, d = i / kTD;
      Ms[d][nn] = (dc + d < D && n0 + nn < N) ? ldf(mix + (int64_t)(dc + d) * N + n0 + nn) : 0.f;
    }
    for (int i = tid; i < kNC * kTT; i += 256) {
      const int d = i / kTT, tt = i % kTT;
      const int t = t0 + tt, hs = off + t - kk * dil;
      float g = 0.f;
      if (dc + d < D && t < Tn && hs >= 0) {
        const int64_t row = (int64_t)b * D + dc + d;
        g = ldf(go + row * Tn + t) * ldf(h + row * L + hs);
      }
      Gs[d][tt] = g;
    }
    __syncthreads();
    const int dlim = min(kNC, D - dc);
    for (int d = 0; d < dlim; ++d) {
      const float m0 = Ms[d][ty * 2], m1 = Ms[d][ty * 2 + 1];
      const float4 gv = *reinterpret_cast<const float4 *>(&Gs[d][tx * 4]);
      const float g[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[0][j] = fmaf(m0, g[j], acc[0][j]);
        acc[1][j] = fmaf(m1, g[j], acc[1][j]);
      }
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int n = n0 + ty * 2 + i;
    if (n >= N) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int t = t0 + tx * 4 + j;
      if (t < Tn) stf(grad_kc + (((int64_t)b * K + kk) * N + n) * Tn + t, acc[i][j]);
    }
  }
}

// -----------------------------------------------------------------------------------
// grad_mix partials: part[split][d][n] = sum over this split's (b,kk,t-chunk) range of
// G_kk[b,d,t] * kc[b,kk,n,t].   block = (64 n) x (64 d) x split, thread = 4 d x 4 n
// -----------------------------------------------------------------------------------
constexpr int kMixT = 16;

template <typename T>
__global__ void __launch_bounds__(256)
fdc_grad_mix_partial_kernel(const T *__restrict__ go, const T *__restrict__ h,
                            const T *__restrict__ kc, float *__restrict__ part, int D,
                            int L, int Tn, int N, int K, int off, int dil,
                            int64_t chunks_total, int64_t chunks_per_split) {
  __shared__ float Gs[kMixT][64 + 1];  // [t][d]
  __shared__ float Ks[kMixT][64 + 1];  // [t][n]
  const int n0 = blockIdx.x * 64, d0 = blockIdx.y * 64;
  const int split = blockIdx.z;
  const int tid = threadIdx.x, tx = tid & 15, ty = tid >> 4;
  float acc[4][4];
#pragma unroll
  for (int i = 0; i < 4; ++i)
#pragma unroll
    for (int j = 0; j < 4; ++j) acc[i][j] = 0.f;

  const int64_t tch = (Tn + kMixT - 1) / kMixT;
  const int64_t c_begin = (int64_t)split * chunks_per_split;
  const int64_t c_end = min(chunks_total, c_begin + chunks_per_split);
  for (int64_t c = c_begin; c < c_end; ++c) {
    const int64_t bk = c / tch;
    const int t0 = (int)(c % tch) * kMixT;
    const int b = (int)(bk / K), kk = (int)(bk % K);
    for (int i = tid; i < kMixT * 64; i += 256) {
      const int tt = i % kMixT, dd = i / kMixT;
      const int t = t0 + tt, d = d0 + dd, hs = off + t - kk * dil;
      float g = 0.f;
      if (d < D && t < Tn && hs >= 0) {
        const int64_t row = (int64_t)b * D + d;
        g = ldf(go + row * Tn + t) * ldf(h + row * L + hs);
      }
      Gs[tt][dd] = g;
      const int n = n0 + dd;
      Ks[tt][dd] = (n < N && t < Tn) ? ldf(kc + (((int64_t)b * K + kk) * N + n) * Tn + t) : 0.f;
    }
    __syncthreads();
#pragma unroll 4
    for (int tt = 0; tt < kMixT; ++tt) {
      float g[4], k[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) g[i] = Gs[tt][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) k[j] = Ks[tt][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(g[i], k[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = d0 + ty * 4 + i;
    if (d >= D) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int n = n0 + tx * 4 + j;
      if (n < N) part[((int64_t)split * D + d) * N + n] = acc[i][j];
    }
  }
}

template <typename T>
__global__ void fdc_grad_mix_reduce_kernel(const float *__restrict__ part, T *__restrict__ out,
                                           int64_t DN, int splits) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= DN) return;
  float s = 0.f;
  for (int k = 0; k < splits; ++k) s += part[(int64_t)k * DN + i];
  stf(out + i, s);
}

int grad_mix_splits(const FdcShape &s) {
  const int64_t tiles = cdiv(s.D, 64) * cdiv(s.N, 64);
  const int64_t chunks = s.B * s.K * cdiv(s.T, kMixT);
  int64_t want = cdiv(4 * (int64_t)sm_count(), tiles);
  if (want > chunks) want = chunks;
  if (want < 1) want = 1;
  if (want > 1024) want = 1024;
  return (int)want;
}

template <typename T>
int fwd_impl(const void *h, const void *kc, const void *mix, void *out, const FdcShape &s,
             cudaStream_t st) {
  dim3 grid((unsigned)cdiv(s.T, kTT), (unsigned)cdiv(s.D, kTD), (unsigned)s.B);
  fdc_conv_simt_kernel<T, false><<<grid, 256, 0, st>>>(
      (const T *)h, (const T *)kc, (const T *)mix, (T *)out, (int)s.D, (int)s.L, (int)s.T,
      (int)s.N, (int)s.K, (int)s.off, (int)s.dil, 0, (int)s.T);
  return check_launch("fdc_conv_simt_kernel<fwd>");
}

template <typename T>
int grad_h_impl(const void *go, const void *kc, const void *mix, void *grad_h, const FdcShape &s,
                cudaStream_t st) {
  // positions outside [gh_lo, gh_hi) are zero-filled by the caller
  const int64_t lo = s.gh_lo(), hi = s.gh_hi();
  dim3 grid((unsigned)cdiv(hi - lo, kTT), (unsigned)cdiv(s.D, kTD), (unsigned)s.B);
  fdc_conv_simt_kernel<T, true><<<grid, 256, 0, st>>>(
      (const T *)go, (const T *)kc, (const T *)mix, (T *)grad_h, (int)s.D, (int)s.L, (int)s.T,
      (int)s.N, (int)s.K, (int)s.off, (int)s.dil, (int)lo, (int)hi);
  return check_launch("fdc_conv_simt_kernel<grad_h>");
}

template <typename T>
int grad_kc_mix_impl(const void *go, const void *h, const void *mix, const void *kc,
                     void *grad_kc, void *grad_mix, void *ws, const FdcShape &s, int dtype,
                     const XRank *xr, int *err, cudaStream_t st) {
  {
    dim3 grid((unsigned)cdiv(s.T, kTT), (unsigned)cdiv(s.N, kTD), (unsigned)(s.B * s.K));
    fdc_grad_kc_simt_kernel<T><<<grid, 256, 0, st>>>(
        (const T *)go, (const T *)h, (const T *)mix, (T *)grad_kc, (int)s.D, (int)s.L,
        (int)s.T, (int)s.N, (int)s.K, (int)s.off, (int)s.dil);
    if (int rc = check_launch("fdc_grad_kc_simt_kernel")) return rc;
  }
  const int splits = grad_mix_splits(s);
  const int64_t chunks = s.B * s.K * cdiv(s.T, kMixT);
  const int64_t per = cdiv(chunks, splits);
  dim3 grid((unsigned)cdiv(s.N, 64), (unsigned)cdiv(s.D, 64), (unsigned)splits);
  fdc_grad_mix_partial_kernel<T><<<grid, 256, 0, st>>>(
      (const T *)go, (const T *)h, (const T *)kc, (float *)ws, (int)s.D, (int)s.L, (int)s.T,
      (int)s.N, (int)s.K, (int)s.off, (int)s.dil, chunks, per);
  if (int rc = check_launch("fdc_grad_mix_partial_kernel")) return rc;
  const int64_t DN = s.D * s.N;
  if (xr) return xrank_reduce_launch((const float *)ws, splits, grad_mix, DN, dtype, *xr, err, st);
  fdc_grad_mix_reduce_kernel<T><<<(unsigned)cdiv(DN, 256), 256, 0, st>>>(
      (const float *)ws, (T *)grad_mix, DN, splits);
  return check_launch("fdc_grad_mix_reduce_kernel");
}

}  // namespace

size_t fdc_simt_bwd_workspace(const FdcShape &s) {
  return (size_t)grad_mix_splits(s) * (size_t)(s.D * s.N) * sizeof(float);
}

int fdc_simt_forward(const void *h, const void *kc, const void *mix, void *out,
                     const FdcShape &s, int dtype, cudaStream_t st) {
  switch (dtype) {
    case DUDY_DTYPE_F32: return fwd_impl<float>(h, kc, mix, out, s, st);
    case DUDY_DTYPE_F16: return fwd_impl<__half>(h, kc, mix, out, s, st);
    default: return fwd_impl<__nv_bfloat16>(h, kc, mix, out, s, st);
  }
}

int fdc_simt_grad_h(const void *go, const void *kc, const void *mix, void *grad_h,
                    const FdcShape &s, int dtype, cudaStream_t st) {
  switch (dtype) {
    case DUDY_DTYPE_F32: return grad_h_impl<float>(go, kc, mix, grad_h, s, st);
    case DUDY_DTYPE_F16: return grad_h_impl<__half>(go, kc, mix, grad_h, s, st);
    default: return grad_h_impl<__nv_bfloat16>(go, kc, mix, grad_h, s, st);
  }
}

int fdc_simt_grad_kc_mix(const void *go, const void *h, const void *mix, const void *kc,
                         void *grad_kc, void *grad_mix, void *ws, const FdcShape &s, int dtype,
                         const XRank *xr, int *err, cudaStream_t st) {
  switch (dtype) {
    case DUDY_DTYPE_F32:
      return grad_kc_mix_impl<float>(go, h, mix, kc, grad_kc, grad_mix, ws, s, dtype, xr, err, st);
    case DUDY_DTYPE_F16:
      return grad_kc_mix_impl<__half>(go, h, mix, kc, grad_kc, grad_mix, ws, s, dtype, xr, err, st);
    default:
      return grad_kc_mix_impl<__nv_bfloat16>(go, h, mix, kc, grad_kc, grad_mix, ws, s, dtype, xr,
                                             err, st);
  }
}

}  // namespace dudy
