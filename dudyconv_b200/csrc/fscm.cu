// fscm.cu -- fused source conv: depthwise causal conv (S taps at one dilation) per
// source channel c, + bias, exact-erf GELU, static per-(d,c) mix + per-d bias.
//
// Semantics: cuda_ops/fused_source_conv_mixed_plans.h:7-44 and the reference formula
// test_fused_source_conv_mixed.py:111-255 (tap j = S-1 is the current token).
//
// Design (this library's own):
//   forward  one block per (b, d, 1024-token tile); the d's parameters sit in shared
//            memory, the x tile plus its causal halo is staged once in shared memory,
//            each thread produces 4 tokens.
//   backward gather form, no atomics on global memory. One block per (b, d, tile of
//            TT output positions s). It recomputes z over the TT + halo tokens that
//            feed the tile, folds sum_c gz*w[c,j] into per-tap shared rows, gathers
//            grad_x, and writes fp32 parameter partials (owned tokens only) that a
//            second kernel reduces in a fixed order (deterministic).
#include "common.cuh"

namespace dudy {
namespace {

constexpr float kInvSqrt2 = 0.70710678118654752f;
constexpr float kInvSqrt2Pi = 0.39894228040143268f;

__device__ __forceinline__ float gelu_erf(float z) { return 0.5f * z * (1.f + erff(z * kInvSqrt2)); }

__device__ __forceinline__ void gelu_and_grad(float z, float &g, float &gp) {
  const float cdf = 0.5f * (1.f + erff(z * kInvSqrt2));
  g = z * cdf;
  gp = cdf + z * expf(-0.5f * z * z) * kInvSqrt2Pi;
}

constexpr int kFwdTile = 1024;  // tokens per forward block (256 threads x 4)
constexpr int kMaxSReg = 8;     // taps held in registers

template <typename T>
__global__ void __launch_bounds__(256)
fscm_fwd_kernel(const T *__restrict__ x, const T *__restrict__ w, const T *__restrict__ bias,
                const T *__restrict__ mw, const T *__restrict__ mb, T *__restrict__ out, int D,
                int L, int C, int S, int off, int Tn, int dil, int xs_len) {
  extern __shared__ float sm[];
  float *w_s = sm;                // [C][S]
  float *b_s = w_s + C * S;       // [C]
  float *m_s = b_s + C;           // [C]
  float *x_s = m_s + C;           // [xs_len] x[off + t0 - H + i]
  const int d = blockIdx.y, b = blockIdx.z;
  const int t0 = blockIdx.x * kFwdTile;
  const int H = dil * (S - 1);
  for (int i = threadIdx.x; i < C * S; i += blockDim.x) w_s[i] = ldf(w + (int64_t)d * C * S + i);
  for (int i = threadIdx.x; i < C; i += blockDim.x) {
    b_s[i] = bias ? ldf(bias + (int64_t)d * C + i) : 0.f;
    m_s[i] = ldf(mw + (int64_t)d * C + i);
  }
  const int64_t row = ((int64_t)b * D + d) * L;
  const int xbase = off + t0 - H;
  for (int i = threadIdx.x; i < xs_len; i += blockDim.x) {
    const int p = xbase + i;
    x_s[i] = (p >= 0 && p < L) ? ldf(x + row + p) : 0.f;
  }
  __syncthreads();
  const float mbias = ldf(mb + d);
  for (int k = 0; k < kFwdTile / 256; ++k) {
    const int tl = k * 256 + threadIdx.x;
    const int t = t0 + tl;
    if (t >= Tn) break;
    float acc = mbias;
    if (S <= kMaxSReg) {
      float xv[kMaxSReg];
#pragma unroll
      for (int j = 0; j < kMaxSReg; ++j) xv[j] = j < S ? x_s[tl + j * dil] : 0.f;
      for (int c = 0; c < C; ++c) {
        float z = b_s[c];
#pragma unroll
        for (int j = 0; j < kMaxSReg; ++j)
          if (j < S) z = fmaf(xv[j], w_s[c * S + j], z);
        acc = fmaf(gelu_erf(z), m_s[c], acc);
      }
    } else {
      for (int c = 0; c < C; ++c) {
        float z = b_s[c];
        for (int j = 0; j < S; ++j) z = fmaf(x_s[tl + j * dil], w_s[c * S + j], z);
        acc = fmaf(gelu_erf(z), m_s[c], acc);
      }
    }
    stf(out + ((int64_t)b * D + d) * Tn + t, acc);
  }
}

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
// parameter-partial layout per (d, block): [gb C][gmw C][gw C*S][gmb 1]
__host__ __device__ inline int fscm_np(int C, int S) { return C * (S + 2) + 1; }

template <typename T>
__global__ void __launch_bounds__(256)
fscm_bwd_kernel(const T *__restrict__ go, const T *__restrict__ x, const T *__restrict__ w,
                const T *__restrict__ bias, const T *__restrict__ mw, T *__restrict__ gx,
                float *__restrict__ part, int B, int D, int L, int C, int S, int off, int Tn,
                int dil, int TT, int ntiles) {
  extern __shared__ float sm[];
  const int H = dil * (S - 1);
  const int NP = fscm_np(C, S);
  float *w_s = sm;                 // [C][S]
  float *b_s = w_s + C * S;        // [C]
  float *m_s = b_s + C;            // [C]
  float *acc_s = m_s + C;          // [NP] block partials
  float *P_s = acc_s + NP;         // [S][TT] per-tap folded gz
  float *x_s = P_s + S * TT;       // [TT + 2H] x[off + t_lo - H + i]
  float *g_s = x_s + TT + 2 * H;   // [TT + H]  go[t_lo + i]

  const int tile = blockIdx.x, d = blockIdx.y, b = blockIdx.z;
  const int tid = threadIdx.x;
  for (int i = tid; i < C * S; i += blockDim.x) w_s[i] = ldf(w + (int64_t)d * C * S + i);
  for (int i = tid; i < C; i += blockDim.x) {
    b_s[i] = bias ? ldf(bias + (int64_t)d * C + i) : 0.f;
    m_s[i] = ldf(mw + (int64_t)d * C + i);
  }
  for (int i = tid; i < NP; i += blockDim.x) acc_s[i] = 0.f;
  for (int i = tid; i < S * TT; i += blockDim.x) P_s[i] = 0.f;
  // tokens t in [t_lo, t_lo + TT + H) feed this tile; tokens [own_lo, own_lo+TT) are owned
  const int own_lo = tile * TT;
  const int t_lo = own_lo - H;
  const int64_t xrow = ((int64_t)b * D + d) * L;
  const int64_t grow = ((int64_t)b * D + d) * Tn;
  for (int i = tid; i < TT + 2 * H; i += blockDim.x) {
    const int p = off + t_lo - H + i;
    x_s[i] = (p >= 0 && p < L) ? ldf(x + xrow + p) : 0.f;
  }
  for (int i = tid; i < TT + H; i += blockDim.x) {
    const int t = t_lo + i;
    g_s[i] = (t >= 0 && t < Tn) ? ldf(go + grow + t) : 0.f;
  }
  __syncthreads();

  const int lane = tid & 31;
  for (int c = 0; c < C; ++c) {
    float lb = 0.f, lm = 0.f, lg = 0.f;
    float lw[kMaxSReg];
#pragma unroll
    for (int j = 0; j < kMaxSReg; ++j) lw[j] = 0.f;
    for (int i = tid; i < TT + H; i += blockDim.x) {
      const int t = t_lo + i;
      if (t < 0 || t >= Tn) continue;
      // x_s index of x[off + t - dil*(S-1-j)] is i + H - dil*(S-1-j) = i + dil*j
      float z = b_s[c];
      for (int j = 0; j < S; ++j) z = fmaf(x_s[i + dil * j], w_s[c * S + j], z);
      float g, gp;
      gelu_and_grad(z, g, gp);
      const float gov = g_s[i];
      const float q = gov * m_s[c] * gp;
      if (t >= own_lo) {  // owned token (t < own_lo + TT always holds here)
        lb += q;
        lm = fmaf(gov, g, lm);
        if (c == 0) lg += gov;
        if (S <= kMaxSReg) {
#pragma unroll
          for (int j = 0; j < kMaxSReg; ++j)
            if (j < S) lw[j] = fmaf(q, x_s[i + dil * j], lw[j]);
        } else {
          for (int j = 0; j < S; ++j)
            atomicAdd(&acc_s[2 * C + c * S + j], q * x_s[i + dil * j]);
        }
      }
      // fold into per-tap rows: tap j of output u reads token own_lo + u - dil*j
      for (int j = 0; j < S; ++j) {
        const int u = t - own_lo + dil * j;
        if (u >= 0 && u < TT) P_s[j * TT + u] = fmaf(q, w_s[c * S + j], P_s[j * TT + u]);
      }
    }
    // block reduction of this c's partials: warp shuffle, then shared atomics
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      lb += __shfl_xor_sync(0xffffffffu, lb, o);
      lm += __shfl_xor_sync(0xffffffffu, lm, o);
      if (c == 0) lg += __shfl_xor_sync(0xffffffffu, lg, o);
    }
    if (S <= kMaxSReg) {
#pragma unroll
      for (int j = 0; j < kMaxSReg; ++j) {
        if (j >= S) break;
        float v = lw[j];
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (lane == 0) atomicAdd(&acc_s[2 * C + c * S + j], v);
      }
    }
    if (lane == 0) {
      atomicAdd(&acc_s[c], lb);
      atomicAdd(&acc_s[C + c], lm);
      if (c == 0) atomicAdd(&acc_s[NP - 1], lg);
    }
  }
  __syncthreads();
  // grad_x for s = off - H + own_lo + u
  const int s_hi = off + Tn;
  for (int u = tid; u < TT; u += blockDim.x) {
    const int s = off - H + own_lo + u;
    if (s < 0 || s >= s_hi) continue;
    float v = 0.f;
    for (int j = 0; j < S; ++j) v += P_s[j * TT + u];
    stf(gx + xrow + s, v);
  }
  // parameter partials: part[d][b*ntiles + tile][NP]
  float *dst = part + ((int64_t)d * B * ntiles + (int64_t)b * ntiles + tile) * NP;
  for (int i = tid; i < NP; i += blockDim.x) dst[i] = acc_s[i];
}

template <typename T>
__global__ void fscm_param_reduce_kernel(const float *__restrict__ part, T *__restrict__ gw,
                                         T *__restrict__ gb, T *__restrict__ gmw,
                                         T *__restrict__ gmb, int D, int C, int S, int nblk) {
  const int NP = fscm_np(C, S);
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)D * NP) return;
  const int d = (int)(i / NP), p = (int)(i % NP);
  const float *src = part + (int64_t)d * nblk * NP + p;
  float s = 0.f;
  for (int k = 0; k < nblk; ++k) s += src[(int64_t)k * NP];
  if (p < C) {
    if (gb) stf(gb + (int64_t)d * C + p, s);
  } else if (p < 2 * C) {
    stf(gmw + (int64_t)d * C + (p - C), s);
  } else if (p < 2 * C + C * S) {
    stf(gw + (int64_t)d * C * S + (p - 2 * C), s);
  } else {
    stf(gmb + d, s);
  }
}

size_t fwd_smem(const FscmShape &s) {
  return (size_t)(s.C * s.S + 2 * s.C + kFwdTile + s.halo()) * sizeof(float);
}

int bwd_tile(const FscmShape &s, int64_t tile_t) {
  int64_t tt = tile_t > 0 ? tile_t : 256;
  if (tt > 1024) tt = 1024;
  if (tt < 32) tt = 32;
  return (int)tt;
}

size_t bwd_smem(const FscmShape &s, int TT) {
  const int64_t H = s.halo();
  return (size_t)(s.C * s.S + 2 * s.C + fscm_np((int)s.C, (int)s.S) + s.S * TT + TT + 2 * H +
                  TT + H) *
         sizeof(float);
}

template <typename T>
int fwd_impl(const void *x, const void *w, const void *bias, const void *mw, const void *mb,
             void *out, const FscmShape &s, cudaStream_t st) {
  const size_t smem = fwd_smem(s);
  auto kern = fscm_fwd_kernel<T>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fscm_fwd_kernel)");
  dim3 grid((unsigned)cdiv(s.T, kFwdTile), (unsigned)s.D, (unsigned)s.B);
  kern<<<grid, 256, smem, st>>>((const T *)x, (const T *)w, s.has_bias ? (const T *)bias : nullptr,
                                (const T *)mw, (const T *)mb, (T *)out, (int)s.D, (int)s.L,
                                (int)s.C, (int)s.S, (int)s.off, (int)s.T, (int)s.dil,
                                (int)(kFwdTile + s.halo()));
  return check_launch("fscm_fwd_kernel");
}

template <typename T>
int bwd_impl(const void *go, const void *x, const void *w, const void *bias, const void *mw,
             void *gx, void *gw, void *gb, void *gmw, void *gmb, void *ws, const FscmShape &s,
             int64_t tile_t, cudaStream_t st) {
  const size_t es = sizeof(T);
  const int TT = bwd_tile(s, tile_t);
  const int64_t H = s.halo();
  const int ntiles = (int)cdiv(s.T + H, TT);
  const int64_t lo = s.off - H < 0 ? 0 : s.off - H, hi = s.off + s.T;
  if (lo > 0 && cudaMemset2DAsync(gx, s.L * es, 0, lo * es, s.B * s.D, st) != cudaSuccess)
    return check_launch("cudaMemset2DAsync(grad_x head)");
  if (hi < s.L && cudaMemset2DAsync((char *)gx + hi * es, s.L * es, 0, (s.L - hi) * es,
                                    s.B * s.D, st) != cudaSuccess)
    return check_launch("cudaMemset2DAsync(grad_x tail)");
  const size_t smem = bwd_smem(s, TT);
  auto kern = fscm_bwd_kernel<T>;
  if (smem > 48 * 1024 &&
      cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fscm_bwd_kernel)");
  dim3 grid((unsigned)ntiles, (unsigned)s.D, (unsigned)s.B);
  kern<<<grid, 256, smem, st>>>((const T *)go, (const T *)x, (const T *)w,
                                s.has_bias ? (const T *)bias : nullptr, (const T *)mw, (T *)gx,
                                (float *)ws, (int)s.B, (int)s.D, (int)s.L, (int)s.C, (int)s.S,
                                (int)s.off, (int)s.T, (int)s.dil, TT, ntiles);
  if (int rc = check_launch("fscm_bwd_kernel")) return rc;
  const int64_t n = s.D * fscm_np((int)s.C, (int)s.S);
  fscm_param_reduce_kernel<T><<<(unsigned)cdiv(n, 256), 256, 0, st>>>(
      (const float *)ws, (T *)gw, s.has_bias ? (T *)gb : nullptr, (T *)gmw, (T *)gmb, (int)s.D,
      (int)s.C, (int)s.S, (int)(s.B * ntiles));
  return check_launch("fscm_param_reduce_kernel");
}

}  // namespace

// shared-memory bound for the staged kernels (227 KB opt-in per block on sm_100)
constexpr size_t kMaxSmem = 227 * 1024;

bool fscm_shapes_fit(const FscmShape &s, int64_t tile_t) {
  return fwd_smem(s) <= kMaxSmem && bwd_smem(s, bwd_tile(s, tile_t)) <= kMaxSmem;
}

size_t fscm_bwd_workspace(const FscmShape &s, int64_t tile_t) {
  const int TT = bwd_tile(s, tile_t);
  const int64_t ntiles = cdiv(s.T + s.halo(), TT);
  return (size_t)(s.D * s.B * ntiles) * fscm_np((int)s.C, (int)s.S) * sizeof(float);
}

int fscm_forward_impl(const void *x, const void *w, const void *bias, const void *mw,
                      const void *mb, void *out, const FscmShape &s, int dtype,
                      cudaStream_t st) {
  switch (dtype) {
    case DUDY_DTYPE_F32: return fwd_impl<float>(x, w, bias, mw, mb, out, s, st);
    case DUDY_DTYPE_F16: return fwd_impl<__half>(x, w, bias, mw, mb, out, s, st);
    default: return fwd_impl<__nv_bfloat16>(x, w, bias, mw, mb, out, s, st);
  }
}

int fscm_backward_impl(const void *go, const void *x, const void *w, const void *bias,
                       const void *mw, void *gx, void *gw, void *gb, void *gmw, void *gmb,
                       void *ws, const FscmShape &s, int64_t tile_t, int dtype,
                       cudaStream_t st) {
  switch (dtype) {
    case DUDY_DTYPE_F32:
      return bwd_impl<float>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, tile_t, st);
    case DUDY_DTYPE_F16:
      return bwd_impl<__half>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, tile_t, st);
    default:
      return bwd_impl<__nv_bfloat16>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, tile_t,
                                     st);
  }
}

}  // namespace dudy
