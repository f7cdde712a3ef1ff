// fscm.cu -- fused source conv: depthwise causal conv (S taps at one dilation) per
// source channel c, + bias, exact-erf GELU, static per-(d,c) mix + per-d bias.
//
//   z[b,d,c,t] = bias[d,c] + sum_j x[b,d, off+t-dil*(S-1-j)] * w[d,c,j]
//   out[b,d,t] = mix_b[d] + sum_c GELU_erf(z[b,d,c,t]) * mix_w[d,c]
//
// Semantics: cuda_ops/fused_source_conv_mixed_plans.h:7-44 and the reference formula
// test_fused_source_conv_mixed.py:111-255 (tap j = S-1 is the current token).
//
// Design (this library's own). The op is bound by the FP32/SFU work of C erf-GELUs per
// (token, channel) at the model's C = 16, and by HBM at small C. One block per
// (b, d, 2048-token span), 256 threads, thread k of the block owns the 8 tokens
// span + k, span + 256 + k, ... (interleaved, so the staged-row reads are
// bank-conflict free and the global loads/stores coalesce). The x row of the span plus
// its causal halo is staged once in shared memory as fp32; each thread keeps its 8 x S
// tap values in registers and loops over the C channels, so each x element is read
// from shared memory S times per block, not C x S times.
//
//   forward  out for the span.
//   backward gather form, no atomics. The tokens [0, T) split into equal tiles of at
//            most 2048, each computed once by one block; per token it folds
//            q_c * w[c,j] over c into S per-tap sums, which are gathered into grad_x
//            through shared memory. A grad_x position within halo = dil*(S-1) of a tile
//            boundary takes taps from both tiles: each block writes its part to a
//            boundary scratch and the reduce kernel adds the two parts. (Where a tile
//            would hold fewer than halo tokens, tiles of owned positions recompute the
//            halo tokens after them instead.) Parameter gradients of a block's tokens
//            are reduced per warp with shuffles, then across warps and blocks in a fixed
//            order (deterministic).
#include <string.h>

#include "common.cuh"

namespace dudy {
namespace {

constexpr float kInvSqrt2 = 0.70710678118654752f;
constexpr float kInvSqrt2Pi = 0.39894228040143268f;
constexpr float kNegHalfLog2e = -0.72134752044448170f;  // -log2(e) / 2

// Single-instruction approximations (PTX rcp.approx.ftz.f32 and ex2.approx.ftz.f32), used
// for 16-bit tensors only: exp(-z^2 / 2) = 2^(-log2(e) z^2 / 2). Subnormal inputs and
// results flush to zero, which only moves values far below the 16-bit output grids.
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

// Standard normal CDF Phi(z) = (1 + erf(z / sqrt 2)) / 2 and its tail
// h(z) = Phi(-|z|) = (1 - erf(|z| / sqrt 2)) / 2, so that Phi(z) = (z >= 0 ? 1 - h : h) and
// GELU(z) = z Phi(z) = max(z, 0) - |z| h.
//  * fp32 tensors: erff and expf.
//  * fp16 / bf16 tensors (results rounded to 16 bits): h from two approximations of
//    Abramowitz & Stegun, Handbook of Mathematical Functions:
//      forward  eq. 7.1.28  1 - erf x = (1 + a1 x + ... + a6 x^6)^-16,          |err| <= 3e-7
//               (one reciprocal, four squarings, no exponential; x = |z| / sqrt 2 and the
//               factor 1/2 folded into the coefficients);
//      backward eq. 26.2.16  h(z) = phi(z) (a1 t + a2 t^2 + a3 t^3), t = 1 / (1 + p |z|),
//               phi(z) = exp(-z^2 / 2) / sqrt(2 pi),                          |err| < 1e-5
//               (phi(z) is also the factor of GELU'(z) = Phi(z) + z phi(z), taken as
//               2^(log2(e) (-z^2/2) + log2 phi(0))). The three-term form is far below the
//               16-bit output grids (the backward's results are rounded to 16 bits and its
//               parameter sums see the error as a relative 1e-5) and saves two packed
//               multiply-adds per token pair against the five-term eq. 26.2.17 (7.5e-8):
//               350.7 against 361.3 us at C = 16 on B200.
//    The tail is evaluated directly, so Phi keeps its relative accuracy for z < 0.
//    Max absolute error in fp32 arithmetic: Phi about 1e-6 (forward), GELU' about 1e-5
//    (backward) (tests/test_gpu_fscm.py checks both against erff / expf on the GPU).
// 7.1.28: a_k / 2^(k/2), k = 1..6
constexpr float kA28_1 = 0.049867347f, kA28_2 = 0.021141006f, kA28_3 = 0.0032776264f,
                kA28_4 = 3.8003574e-05f, kA28_5 = 4.8890637e-05f, kA28_6 = 5.3829749e-06f;
// 26.2.16: p and a_k, k = 1..3; log2 of 1 / sqrt(2 pi)
constexpr float kP26 = 0.33267f;
constexpr float kA26_1 = 0.4361836f, kA26_2 = -0.1201676f, kA26_3 = 0.9372980f;
constexpr float kLog2InvSqrt2Pi = -1.32574809f;

// r16 = (1 + a1 x + ... + a6 x^6)^-16 = 2 h(z) from 7.1.28, given az = |z|
__device__ __forceinline__ float r16_as7128(float az) {
  float p = fmaf(kA28_6, az, kA28_5);
  p = fmaf(p, az, kA28_4);
  p = fmaf(p, az, kA28_3);
  p = fmaf(p, az, kA28_2);
  p = fmaf(p, az, kA28_1);
  p = fmaf(p, az, 1.f);
  const float r = rcp_approx(p);  // p >= 1
  const float r2 = r * r, r4 = r2 * r2, r8 = r4 * r4;
  return r8 * r8;
}

// phi(z) = exp(-z^2 / 2) / sqrt(2 pi), single-instruction exponential
__device__ __forceinline__ float npdf_approx(float z) {
  return ex2_approx(fmaf(kNegHalfLog2e * z, z, kLog2InvSqrt2Pi));
}

// h(z) from 26.2.16, given az = |z| and pz = phi(z)
__device__ __forceinline__ float tail_as26216(float az, float pz) {
  const float t = rcp_approx(fmaf(kP26, az, 1.f));
  const float q = fmaf(fmaf(kA26_3, t, kA26_2), t, kA26_1);
  return (q * t) * pz;
}

__device__ __forceinline__ float phi_from_tail(float z, float h) { return z >= 0.f ? 1.f - h : h; }

// GELU(z) and GELU'(z) for the backward pass
template <typename T>
__device__ __forceinline__ void gelu_and_grad(float z, float &g, float &gp) {
  if constexpr (sizeof(T) == 2) {
    const float pz = npdf_approx(z);
    const float cdf = phi_from_tail(z, tail_as26216(fabsf(z), pz));
    g = z * cdf;
    gp = fmaf(z, pz, cdf);
  } else {
    const float e = expf(-0.5f * z * z);
    const float cdf = 0.5f * (1.f + erff(z * kInvSqrt2));
    g = z * cdf;
    gp = fmaf(z * e, kInvSqrt2Pi, cdf);
  }
}

// GELU(z) for the forward pass (fp32 tensors; the 16-bit forward uses the packed form)
__device__ __forceinline__ float gelu_fp32(float z) {
  return z * (0.5f * (1.f + erff(z * kInvSqrt2)));
}

// Packed-fp32 versions for two tokens at once (sm_100 FFMA2 / FMUL2 / FADD2 issue two
// IEEE fp32 operations per instruction, saving issue slots); used for 16-bit tensors.
// Same operations and rounding per lane as the scalar forms above.
__device__ __forceinline__ float2 bc2(float a) { return make_float2(a, a); }
__device__ __forceinline__ float2 abs2(float2 z) { return make_float2(fabsf(z.x), fabsf(z.y)); }

__device__ __forceinline__ float2 r16_as7128(float2 az) {
  float2 p = __ffma2_rn(bc2(kA28_6), az, bc2(kA28_5));
  p = __ffma2_rn(p, az, bc2(kA28_4));
  p = __ffma2_rn(p, az, bc2(kA28_3));
  p = __ffma2_rn(p, az, bc2(kA28_2));
  p = __ffma2_rn(p, az, bc2(kA28_1));
  p = __ffma2_rn(p, az, bc2(1.f));
  const float2 r = make_float2(rcp_approx(p.x), rcp_approx(p.y));
  const float2 r2 = __fmul2_rn(r, r), r4 = __fmul2_rn(r2, r2), r8 = __fmul2_rn(r4, r4);
  return __fmul2_rn(r8, r8);
}

__device__ __forceinline__ float2 tail_as26216(float2 az, float2 pz) {
  const float2 d = __ffma2_rn(bc2(kP26), az, bc2(1.f));
  const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  const float2 q = __ffma2_rn(__ffma2_rn(bc2(kA26_3), t, bc2(kA26_2)), t, bc2(kA26_1));
  return __fmul2_rn(__fmul2_rn(q, t), pz);
}

constexpr int kThreads = 256;
constexpr int kTok = 8;                    // tokens per thread
constexpr int kSpan = kThreads * kTok;     // tokens per block
constexpr int kMaxS = 8;                   // taps held in registers
constexpr int kMaxHalo = 1024;             // dil * (S - 1) limit of the staged design

// dst[i] = row[start + i] as fp32 for i < n (0 outside [0, len)); block-cooperative.
template <typename T>
__device__ __forceinline__ void stage_row(const T *__restrict__ row, int len, int start, int n,
                                          float *__restrict__ dst) {
  for (int i = threadIdx.x; i < n; i += kThreads) {
    const int p = start + i;
    dst[i] = (p >= 0 && p < len) ? ldf(row + p) : 0.f;
  }
}

// CT / ST: compile-time C and S (0 = runtime value). Launch bounds: the 16-bit C = 16
// instantiation with one block as the stated minimum (80 registers instead of 64) measured
// 156 -> 153 us on B200 (B=16 T=4096 D=256 S=3 fp16); the others state no minimum (0), which
// keeps the compiler's own register choice (C = 3: 60 registers; at most 64 measured slower).
template <typename T, int CT, int ST>
__global__ void __launch_bounds__(kThreads, sizeof(T) == 2 && CT == 16 ? 1 : 0)
fscm_fwd_kernel(const T *__restrict__ x, const T *__restrict__ w, const T *__restrict__ bias,
                const T *__restrict__ mw, const T *__restrict__ mb, T *__restrict__ out, int D,
                int L, int C_, int S_, int off, int Tn, int dil, int TT) {
  const int C = CT ? CT : C_, S = ST ? ST : S_;
  extern __shared__ float sm[];
  float *w_s = sm;                // [C][S]
  float *b_s = w_s + C * S;       // [C]
  float *m_s = b_s + C;           // [C]
  float *x_s = m_s + C;           // [kSpan + H]: x[off + t0 - H + i]
  const int d = blockIdx.y, b = blockIdx.z;
  // TT <= kSpan tokens per block, the tiles of a row of equal size (no idle span)
  const int t0 = blockIdx.x * TT;
  const int active = min(TT, Tn - t0);
  const int H = dil * (S - 1);
  for (int i = threadIdx.x; i < C * S; i += kThreads) w_s[i] = ldf(w + (int64_t)d * C * S + i);
  for (int i = threadIdx.x; i < C; i += kThreads) {
    b_s[i] = bias ? ldf(bias + (int64_t)d * C + i) : 0.f;
    m_s[i] = ldf(mw + (int64_t)d * C + i);
  }
  const int64_t row = ((int64_t)b * D + d) * L;
  // the whole span is staged (zero past the tile) and computed: a skip inside the token
  // loop stops the compiler from interleaving the 8 independent GELU chains (measured
  // 18% slower); only the stores are masked
  stage_row(x + row, L, off + t0 - H, kSpan + H, x_s);
  __syncthreads();
  const int k = threadIdx.x;
  // token t0 + i*256 + k reads tap j at x_s[i*256 + k + j*dil]
  float xv[kMaxS][kTok];
#pragma unroll
  for (int j = 0; j < kMaxS; ++j)
#pragma unroll
    for (int i = 0; i < kTok; ++i) xv[j][i] = j < S ? x_s[i * kThreads + k + j * dil] : 0.f;
  const float mbias = ldf(mb + d);
  float acc[kTok];
#pragma unroll
  for (int i = 0; i < kTok; ++i) acc[i] = mbias;
  if constexpr (sizeof(T) == 2) {
    // tokens (2p, 2p+1) of the thread in one packed register pair
    float2 acc2[kTok / 2];
#pragma unroll
    for (int p = 0; p < kTok / 2; ++p) acc2[p] = bc2(mbias);
#pragma unroll(CT ? CT : 1)
    for (int c = 0; c < C; ++c) {
      // GELU(z) m = max(z, 0) m - |z| (2h) (m / 2)
      const float2 b2 = bc2(b_s[c]), m2 = bc2(m_s[c]), nmh2 = bc2(-0.5f * m_s[c]);
      float2 w2[kMaxS];
#pragma unroll
      for (int j = 0; j < kMaxS; ++j) w2[j] = bc2(j < S ? w_s[c * S + j] : 0.f);
#pragma unroll
      for (int p = 0; p < kTok / 2; ++p) {
        float2 z = b2;
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) z = __ffma2_rn(make_float2(xv[j][2 * p], xv[j][2 * p + 1]), w2[j], z);
        const float2 az = abs2(z);
        const float2 r16 = r16_as7128(az);
        acc2[p] = __ffma2_rn(make_float2(fmaxf(z.x, 0.f), fmaxf(z.y, 0.f)), m2, acc2[p]);
        acc2[p] = __ffma2_rn(__fmul2_rn(az, r16), nmh2, acc2[p]);
      }
    }
#pragma unroll
    for (int p = 0; p < kTok / 2; ++p) {
      acc[2 * p] = acc2[p].x;
      acc[2 * p + 1] = acc2[p].y;
    }
  } else {
#pragma unroll(CT ? CT : 1)
    for (int c = 0; c < C; ++c) {
      const float bc = b_s[c], mc = m_s[c];
      float wc[kMaxS];
#pragma unroll
      for (int j = 0; j < kMaxS; ++j) wc[j] = j < S ? w_s[c * S + j] : 0.f;
#pragma unroll
      for (int i = 0; i < kTok; ++i) {
        float z = bc;
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) z = fmaf(xv[j][i], wc[j], z);
        acc[i] = fmaf(gelu_fp32(z), mc, acc[i]);
      }
    }
  }
  T *orow = out + ((int64_t)b * D + d) * Tn;
#pragma unroll
  for (int i = 0; i < kTok; ++i) {
    const int r = i * kThreads + k;
    if (r < active) stf(orow + t0 + r, acc[i]);
  }
}

// ---------------------------------------------------------------------------------------
// backward
// ---------------------------------------------------------------------------------------
// parameter-partial layout per (d, block): [gb C][gmw C][gw C*S][gmb 1]
__host__ __device__ inline int fscm_np(int C, int S) { return C * (S + 2) + 1; }

// Parameter partials of one channel: sums over groups of 2^gsh lanes (gsh in [2, 5]); the
// first lane of each group writes the group's row (8 warps x 32 >> gsh rows of NP).
// Fewer shuffle levels than a full warp tree; the host picks the smallest gsh whose rows
// fit in shared memory.
__device__ __forceinline__ void put_partials(float *wp_s, int NP, int C, int S, int c, int lane,
                                             int wid, int gsh, float lb, float lm,
                                             float (&lw)[kMaxS]) {
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    if (o < (1 << gsh)) {
      lb += __shfl_xor_sync(0xffffffffu, lb, o);
      lm += __shfl_xor_sync(0xffffffffu, lm, o);
#pragma unroll
      for (int j = 0; j < kMaxS; ++j)
        if (j < S) lw[j] += __shfl_xor_sync(0xffffffffu, lw[j], o);
    }
  }
  if ((lane & ((1 << gsh) - 1)) == 0) {
    float *wp = wp_s + ((wid << (5 - gsh)) + (lane >> gsh)) * NP;
    wp[c] = lb;
    wp[C + c] = lm;
#pragma unroll
    for (int j = 0; j < kMaxS; ++j)
      if (j < S) wp[2 * C + c * S + j] = lw[j];
  }
}

// Backward tilings.
//  * split (preferred): the tokens [0, T) in ntiles equal tiles of TT <= kSpan tokens. A block
//    owns its tokens' parameter gradients and writes grad_x where all taps' tokens are its
//    own; for the H positions on each side of a tile boundary it writes its part of the sum
//    to a boundary scratch, and the reduce kernel adds the two sides (fixed order). Each
//    token is computed once. Needs every tile to hold at least H tokens.
//  * recompute: the position range [-H, T) in equal tiles of TT owned positions, each block
//    recomputing the TT + H <= kSpan tokens that feed them (H tokens computed twice per
//    boundary); for halos too large for the split tiling.
__host__ __device__ inline int bwd_split_ntiles(int T) { return (T + kSpan - 1) / kSpan; }
__host__ __device__ inline int bwd_split_tt(int T) {
  const int n = bwd_split_ntiles(T);
  return (T + n - 1) / n;
}
__host__ __device__ inline bool bwd_split_ok(int T, int H) {
  const int n = bwd_split_ntiles(T), tt = bwd_split_tt(T);
  return T - (n - 1) * tt >= H;  // the last (shortest) tile holds at least H tokens
}
__host__ __device__ inline int bwd_ntiles_of(int T, int H) {
  if (bwd_split_ok(T, H)) return bwd_split_ntiles(T);
  return (T + H + kSpan - H - 1) / (kSpan - H);
}
__host__ __device__ inline int bwd_tt_of(int T, int H) {
  if (bwd_split_ok(T, H)) return bwd_split_tt(T);
  const int n = bwd_ntiles_of(T, H);
  return (T + H + n - 1) / n;
}

// Launch bounds (measured on B200, B=16 T=4096 D=256 S=3 fp16): C = 3 capped at 4 blocks
// per SM (64 registers, a few spills): 171 -> 163 us; the other 16-bit instantiations with
// one block as the stated minimum, which lets the compiler choose more registers (C = 16:
// 128 instead of 116, still 2 blocks per SM): 459 -> 436 us. fp32 keeps 3 blocks (80
// registers), as without a stated minimum.
template <typename T, int CT, int ST, bool SPLIT>
__global__ void __launch_bounds__(kThreads, sizeof(T) == 2 ? (CT == 3 ? 4 : 1) : (CT ? 3 : 1))
fscm_bwd_kernel(const T *__restrict__ go, const T *__restrict__ x, const T *__restrict__ w,
                const T *__restrict__ bias, const T *__restrict__ mw, T *__restrict__ gx,
                float *__restrict__ part, float *__restrict__ bnd, int B, int D, int L,
                int C_, int S_, int off, int Tn, int dil, int ntiles, int TT, int gsh_) {
  constexpr bool split = SPLIT;
  const int C = CT ? CT : C_, S = ST ? ST : S_;
  const int gsh = CT ? 2 : gsh_;  // lanes per parameter-partial row: 2^gsh
  extern __shared__ float sm[];
  const int H = dil * (S - 1);
  const int tile = blockIdx.x, d = blockIdx.y, b = blockIdx.z;
  // split tiling: tokens [u0, u0 + span) with span = TT (shorter last tile), all owned
  // (tokens past the end have go = 0, so they add nothing to the parameter sums);
  // recompute tiling: owned tokens [u0, u0 + TT) plus the H after them
  const int u0 = split ? tile * TT : -H + tile * TT;
  const int span = split ? min(TT, Tn - u0) : TT + H;  // tokens computed (<= kSpan)
  const int own_n = split ? span : TT;
  const int NP = fscm_np(C, S);
  float *w_s = sm;                    // [C][S]
  float *b_s = w_s + C * S;           // [C]
  float *m_s = b_s + C;               // [C]
  float *wp_s = m_s + C;              // [kThreads >> gsh][NP] lane-group parameter partials
  float *x_s = wp_s + (kThreads >> gsh) * NP;  // [kSpan + H]: x[off + u0 - H + i]
  float *P_s = x_s + kSpan + H;       // [S][kSpan]: sum_c q_c * w[c,j] at token u0 + i

  const int k = threadIdx.x, lane = k & 31, wid = k >> 5;
  for (int i = k; i < C * S; i += kThreads) w_s[i] = ldf(w + (int64_t)d * C * S + i);
  for (int i = k; i < C; i += kThreads) {
    b_s[i] = bias ? ldf(bias + (int64_t)d * C + i) : 0.f;
    m_s[i] = ldf(mw + (int64_t)d * C + i);
  }
  const int64_t xrow = ((int64_t)b * D + d) * L;
  const int64_t grow = ((int64_t)b * D + d) * Tn;
  stage_row(x + xrow, L, off + u0 - H, span + H, x_s);
  __syncthreads();

  float xv[kMaxS][kTok], gv[kTok], P[kMaxS][kTok];
  unsigned owned = 0u;  // per token: parameter grads owned by this block
#pragma unroll
  for (int i = 0; i < kTok; ++i) {
    const int r = i * kThreads + k;
    const int t = u0 + r;
    const bool valid = r < span && t >= 0 && t < Tn;
    gv[i] = valid ? ldf(go + grow + t) : 0.f;
    if (valid && r < own_n) owned |= 1u << i;
#pragma unroll
    for (int j = 0; j < kMaxS; ++j) {
      xv[j][i] = (j < S && valid) ? x_s[r + j * dil] : 0.f;
      P[j][i] = 0.f;
    }
  }
  float lg = 0.f;  // grad of mix_b: sum of go over owned tokens
#pragma unroll
  for (int i = 0; i < kTok; ++i)
    if (SPLIT || (owned >> i & 1u)) lg += gv[i];

  // packed pairs pay off where the channel loop is long; at small C (fully unrolled) the
  // extra registers cost occupancy and the scalar form is faster (measured on B200)
  if constexpr (sizeof(T) == 2 && !(CT > 0 && CT <= 4)) {
    // tokens (2p, 2p+1) in packed register pairs; the ownership mask enters as a 0/1
    // factor (exact), so the owned-token sums need no branch
    float2 own2[kTok / 2], gvo2[kTok / 2];
#pragma unroll
    for (int p = 0; p < kTok / 2; ++p) {
      own2[p] = make_float2((owned >> (2 * p)) & 1u ? 1.f : 0.f, (owned >> (2 * p + 1)) & 1u ? 1.f : 0.f);
      gvo2[p] = SPLIT ? make_float2(gv[2 * p], gv[2 * p + 1])
                      : __fmul2_rn(make_float2(gv[2 * p], gv[2 * p + 1]), own2[p]);
    }
#pragma unroll(CT <= 4 ? (CT ? CT : 1) : 1)
    for (int c = 0; c < C; ++c) {
      const float2 b2 = bc2(b_s[c]), m2 = bc2(m_s[c]);
      float2 w2[kMaxS];
#pragma unroll
      for (int j = 0; j < kMaxS; ++j) w2[j] = bc2(j < S ? w_s[c * S + j] : 0.f);
      float2 lb2 = bc2(0.f), lm2 = bc2(0.f), lw2[kMaxS];
#pragma unroll
      for (int j = 0; j < kMaxS; ++j) lw2[j] = bc2(0.f);
#pragma unroll
      for (int p = 0; p < kTok / 2; ++p) {
        if (2 * p * kThreads >= span) continue;  // block-uniform: slices past the tile
        float2 xp[kMaxS];
#pragma unroll
        for (int j = 0; j < kMaxS; ++j) xp[j] = make_float2(xv[j][2 * p], xv[j][2 * p + 1]);
        float2 z = b2;
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) z = __ffma2_rn(xp[j], w2[j], z);
        const float2 arg = __ffma2_rn(__fmul2_rn(bc2(kNegHalfLog2e), z), z, bc2(kLog2InvSqrt2Pi));
        const float2 pz = make_float2(ex2_approx(arg.x), ex2_approx(arg.y));  // phi(z)
        const float2 h = tail_as26216(abs2(z), pz);
        const float2 cdf = make_float2(phi_from_tail(z.x, h.x), phi_from_tail(z.y, h.y));
        const float2 g = __fmul2_rn(z, cdf);
        const float2 gp = __ffma2_rn(z, pz, cdf);
        const float2 gv2 = make_float2(gv[2 * p], gv[2 * p + 1]);
        const float2 q = __fmul2_rn(__fmul2_rn(gv2, m2), gp);
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) {
            const float2 pj = __ffma2_rn(q, w2[j], make_float2(P[j][2 * p], P[j][2 * p + 1]));
            P[j][2 * p] = pj.x;
            P[j][2 * p + 1] = pj.y;
          }
        const float2 qo = SPLIT ? q : __fmul2_rn(q, own2[p]);
        lb2 = __fadd2_rn(lb2, qo);
        lm2 = __ffma2_rn(gvo2[p], g, lm2);
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) lw2[j] = __ffma2_rn(qo, xp[j], lw2[j]);
      }
      float lb = lb2.x + lb2.y, lm = lm2.x + lm2.y, lw[kMaxS];
#pragma unroll
      for (int j = 0; j < kMaxS; ++j) lw[j] = lw2[j].x + lw2[j].y;
      put_partials(wp_s, NP, C, S, c, lane, wid, gsh, lb, lm, lw);
    }
  } else {
// a fully unrolled C = 16 body overflows the instruction cache (ncu: no_instruction
  // was the top stall); small C unrolls
#pragma unroll(CT <= 4 ? (CT ? CT : 1) : 1)
  for (int c = 0; c < C; ++c) {
    const float bc = b_s[c], mc = m_s[c];
    float wc[kMaxS];
#pragma unroll
    for (int j = 0; j < kMaxS; ++j) wc[j] = j < S ? w_s[c * S + j] : 0.f;
    float lb = 0.f, lm = 0.f, lw[kMaxS];
#pragma unroll
    for (int j = 0; j < kMaxS; ++j) lw[j] = 0.f;
#pragma unroll
    for (int i = 0; i < kTok; ++i) {
      if (i * kThreads >= span) continue;  // block-uniform: slice past the tile
      float z = bc;
#pragma unroll
      for (int j = 0; j < kMaxS; ++j)
        if (j < S) z = fmaf(xv[j][i], wc[j], z);
      float g, gp;
      gelu_and_grad<T>(z, g, gp);
      const float q = gv[i] * mc * gp;   // d out / d z (zero where go is zero)
#pragma unroll
      for (int j = 0; j < kMaxS; ++j)
        if (j < S) P[j][i] = fmaf(q, wc[j], P[j][i]);
      if (SPLIT || (owned >> i & 1u)) {
        lb += q;
        lm = fmaf(gv[i], g, lm);
#pragma unroll
        for (int j = 0; j < kMaxS; ++j)
          if (j < S) lw[j] = fmaf(q, xv[j][i], lw[j]);
      }
    }
    put_partials(wp_s, NP, C, S, c, lane, wid, gsh, lb, lm, lw);
  }
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1)
    if (o < (1 << gsh)) lg += __shfl_xor_sync(0xffffffffu, lg, o);
  if ((lane & ((1 << gsh) - 1)) == 0) wp_s[((wid << (5 - gsh)) + (lane >> gsh)) * NP + NP - 1] = lg;
#pragma unroll
  for (int j = 0; j < kMaxS; ++j)
    if (j < S)
#pragma unroll
      for (int i = 0; i < kTok; ++i)
        if (i * kThreads + k < span) P_s[j * kSpan + i * kThreads + k] = P[j][i];
  __syncthreads();
  // grad_x at position off + u: token u + dil*(S-1-j) read x there at tap j. Recompute
  // tiling: the owned positions r in [0, TT), all taps inside. Split tiling: r in [-H, span);
  // positions within H of either end of the tile get part of their sum from the
  // neighbouring tile and go to the boundary scratch [head H | tail H] of this block.
  const int rlo = split ? -H : 0, rhi = split ? span : TT;
  float *bb = split ? bnd + (((int64_t)b * D + d) * ntiles + tile) * 2 * H : nullptr;
  for (int r = rlo + k; r < rhi; r += kThreads) {
    float v = 0.f;
    for (int j = 0; j < S; ++j) {
      const int rr = r + dil * (S - 1 - j);
      if (rr >= 0 && rr < span) v += P_s[j * kSpan + rr];
    }
    if (split && r < 0) {
      bb[r + H] = v;
      continue;
    }
    if (split && r >= span - H) {
      bb[H + r - (span - H)] = v;
      continue;
    }
    const int u = u0 + r;
    const int s = off + u;
    if (s < 0 || u >= Tn) continue;
    stf(gx + xrow + s, v);
  }
  // block partial: lane-group rows summed in a fixed order
  float *dst = part + ((int64_t)d * B * ntiles + (int64_t)b * ntiles + tile) * NP;
  // four interleaved accumulators (rows q = 4i + a), so the shared-memory loads are not
  // one dependent chain
  const int rows = kThreads >> gsh;  // a multiple of 4
  for (int p = k; p < NP; p += kThreads) {
    float v[4] = {0.f, 0.f, 0.f, 0.f};
    for (int q = 0; q < rows; q += 4) {
#pragma unroll
      for (int a = 0; a < 4; ++a) v[a] += wp_s[(q + a) * NP + p];
    }
    dst[p] = (v[0] + v[1]) + (v[2] + v[3]);
  }
}

// Block = 32 x 8 threads over 32 consecutive (d, p) entries: row y sums the block partials
// k = y, y + 8, ... of its entry (independent loads in flight across rows), then row 0 adds
// the 8 row sums in order (fixed order: deterministic).
// Blocks past the parameter entries finish the split tiling's grad_x positions at tile
// boundaries (one thread per position): boundary e of a row takes the tail part of tile
// e - 1 plus the head part of tile e (fixed order); the row's first boundary is tile 0's
// head alone, its last the last tile's tail alone.
struct FscmBoundary {
  const float *bnd;  // [B*D][ntiles][head H | tail H]
  int nblocks;       // blocks of this kind (0: no split tiling)
  int64_t L;
  int off, Tn, H, TT, ntiles, rows;  // rows = B * D
};

template <typename T>
__global__ void __launch_bounds__(256)
fscm_param_reduce_kernel(const float *__restrict__ part, T *__restrict__ gw,
                         T *__restrict__ gb, T *__restrict__ gmw,
                         T *__restrict__ gmb, int D, int C, int S, int nblk, T *__restrict__ gx,
                         FscmBoundary fb) {
  __shared__ float rs[8][33];
  const int NP = fscm_np(C, S);
  const int tx = threadIdx.x, ty = threadIdx.y;
  const int pblocks = (int)gridDim.x - fb.nblocks;
  if ((int)blockIdx.x >= pblocks) {
    const int64_t q = (int64_t)(blockIdx.x - pblocks) * 256 + ty * 32 + tx;
    const int per_row = (fb.ntiles + 1) * fb.H;
    if (q >= (int64_t)fb.rows * per_row) return;
    const int row = (int)(q / per_row), rem = (int)(q % per_row);
    const int e = rem / fb.H, h = rem % fb.H;
    const int u = e * fb.TT - fb.H + h;  // e * TT: first token of tile e (or T for the last)
    const float *rb = fb.bnd + (int64_t)row * fb.ntiles * 2 * fb.H;
    float v = 0.f;
    if (e > 0) v += rb[(int64_t)(e - 1) * 2 * fb.H + fb.H + h];  // tail of tile e - 1
    if (e < fb.ntiles) v += rb[(int64_t)e * 2 * fb.H + h];       // head of tile e
    const int64_t sp = (int64_t)fb.off + (e == fb.ntiles ? fb.Tn - fb.H + h : u);
    if (sp >= 0 && sp < fb.L) stf(gx + (int64_t)row * fb.L + sp, v);
    return;
  }
  const int64_t i = (int64_t)blockIdx.x * 32 + tx;
  const bool in = i < (int64_t)D * NP;
  const int d = in ? (int)(i / NP) : 0, p = in ? (int)(i % NP) : 0;
  float v = 0.f;
  if (in) {
    const float *src = part + (int64_t)d * nblk * NP + p;
    for (int k = ty; k < nblk; k += 8) v += src[(int64_t)k * NP];
  }
  rs[ty][tx] = v;
  __syncthreads();
  if (ty != 0 || !in) return;
  float s = rs[0][tx];
#pragma unroll
  for (int y = 1; y < 8; ++y) s += rs[y][tx];
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
  return (size_t)(s.C * s.S + 2 * s.C + kSpan + s.halo()) * sizeof(float);
}

// shared-memory bound for the staged kernels (227 KB opt-in per block on sm_100)
constexpr size_t kMaxSmem = 227 * 1024;

size_t bwd_smem_g(const FscmShape &s, int gsh) {
  const int64_t H = s.halo();
  return (size_t)(s.C * s.S + 2 * s.C + (kThreads >> gsh) * fscm_np((int)s.C, (int)s.S) +
                  kSpan + H + s.S * kSpan) *
         sizeof(float);
}

// lanes per partial row = 2^gsh: the smallest group (fewest shuffles) whose rows fit;
// the kernels specialised on C use groups of 4 lanes
int bwd_gsh(const FscmShape &s) {
  for (int g = 2; g < 5; ++g)
    if (bwd_smem_g(s, g) <= kMaxSmem) return g;
  return 5;
}

size_t bwd_smem(const FscmShape &s) { return bwd_smem_g(s, bwd_gsh(s)); }

int64_t bwd_ntiles(const FscmShape &s) { return bwd_ntiles_of((int)s.T, (int)s.halo()); }

// workspace: block parameter partials [D][B*ntiles][NP], then (split tiling) the boundary
// scratch [B*D][ntiles][2H]
size_t bwd_part_bytes(const FscmShape &s) {
  return (size_t)(s.D * s.B * bwd_ntiles(s)) * fscm_np((int)s.C, (int)s.S) * sizeof(float);
}
size_t bwd_bnd_bytes(const FscmShape &s) {
  if (!bwd_split_ok((int)s.T, (int)s.halo())) return 0;
  return (size_t)(s.B * s.D * bwd_ntiles(s) * 2 * s.halo()) * sizeof(float);
}


template <typename T, int CT, int ST>
int fwd_launch(const void *x, const void *w, const void *bias, const void *mw, const void *mb,
               void *out, const FscmShape &s, cudaStream_t st) {
  const size_t smem = fwd_smem(s);
  auto kern = fscm_fwd_kernel<T, CT, ST>;
  if (smem > 48 * 1024 &&
      set_smem_once((const void *)kern, (int)smem) !=
          cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fscm_fwd_kernel)");
  const int nt = (int)cdiv(s.T, kSpan);
  const int TT = (int)cdiv(s.T, nt);
  dim3 grid((unsigned)nt, (unsigned)s.D, (unsigned)s.B);
  kern<<<grid, kThreads, smem, st>>>((const T *)x, (const T *)w,
                                     s.has_bias ? (const T *)bias : nullptr, (const T *)mw,
                                     (const T *)mb, (T *)out, (int)s.D, (int)s.L, (int)s.C,
                                     (int)s.S, (int)s.off, (int)s.T, (int)s.dil, TT);
  return check_launch("fscm_fwd_kernel");
}

template <typename T>
int fwd_impl(const void *x, const void *w, const void *bias, const void *mw, const void *mb,
             void *out, const FscmShape &s, cudaStream_t st) {
  if (s.S == 3 && s.C == 16) return fwd_launch<T, 16, 3>(x, w, bias, mw, mb, out, s, st);
  if (s.S == 3 && s.C == 3) return fwd_launch<T, 3, 3>(x, w, bias, mw, mb, out, s, st);
  return fwd_launch<T, 0, 0>(x, w, bias, mw, mb, out, s, st);
}

template <typename T, int CT, int ST>
int bwd_launch(const void *go, const void *x, const void *w, const void *bias, const void *mw,
               void *gx, float *ws, const FscmShape &s, int ntiles, cudaStream_t st) {
  const int gsh = bwd_gsh(s);
  if (CT && gsh != 2) return DUDY_ERR_UNSUPPORTED;  // the C-specialised kernels fix gsh = 2
  const size_t smem = bwd_smem_g(s, gsh);
  const bool split = bwd_split_ok((int)s.T, (int)s.halo());
  auto kern = split ? fscm_bwd_kernel<T, CT, ST, true> : fscm_bwd_kernel<T, CT, ST, false>;
  if (smem > 48 * 1024 &&
      set_smem_once((const void *)kern, (int)smem) !=
          cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fscm_bwd_kernel)");
  dim3 grid((unsigned)ntiles, (unsigned)s.D, (unsigned)s.B);
  float *bnd = reinterpret_cast<float *>(reinterpret_cast<char *>(ws) + bwd_part_bytes(s));
  kern<<<grid, kThreads, smem, st>>>((const T *)go, (const T *)x, (const T *)w,
                                     s.has_bias ? (const T *)bias : nullptr, (const T *)mw,
                                     (T *)gx, ws, bnd, (int)s.B, (int)s.D, (int)s.L, (int)s.C,
                                     (int)s.S, (int)s.off, (int)s.T, (int)s.dil, ntiles,
                                     bwd_tt_of((int)s.T, (int)s.halo()), gsh);
  return check_launch("fscm_bwd_kernel");
}

template <typename T>
int bwd_impl(const void *go, const void *x, const void *w, const void *bias, const void *mw,
             void *gx, void *gw, void *gb, void *gmw, void *gmb, void *ws, const FscmShape &s,
             cudaStream_t st) {
  const size_t es = sizeof(T);
  const int64_t H = s.halo();
  const int ntiles = (int)bwd_ntiles(s);
  const int64_t lo = s.off - H < 0 ? 0 : s.off - H, hi = s.off + s.T;
  if (lo > 0 && cudaMemset2DAsync(gx, s.L * es, 0, lo * es, s.B * s.D, st) != cudaSuccess)
    return check_launch("cudaMemset2DAsync(grad_x head)");
  if (hi < s.L && cudaMemset2DAsync((char *)gx + hi * es, s.L * es, 0, (s.L - hi) * es,
                                    s.B * s.D, st) != cudaSuccess)
    return check_launch("cudaMemset2DAsync(grad_x tail)");
  int rc;
  if (s.S == 3 && s.C == 16)
    rc = bwd_launch<T, 16, 3>(go, x, w, bias, mw, gx, (float *)ws, s, ntiles, st);
  else if (s.S == 3 && s.C == 3)
    rc = bwd_launch<T, 3, 3>(go, x, w, bias, mw, gx, (float *)ws, s, ntiles, st);
  else
    rc = bwd_launch<T, 0, 0>(go, x, w, bias, mw, gx, (float *)ws, s, ntiles, st);
  if (rc) return rc;
  const int64_t n = s.D * fscm_np((int)s.C, (int)s.S);
  FscmBoundary fb{};
  if (bwd_split_ok((int)s.T, (int)H) && H > 0) {
    fb.bnd = reinterpret_cast<const float *>(reinterpret_cast<const char *>(ws) + bwd_part_bytes(s));
    fb.L = s.L;
    fb.off = (int)s.off;
    fb.Tn = (int)s.T;
    fb.H = (int)H;
    fb.TT = bwd_tt_of((int)s.T, (int)H);
    fb.ntiles = ntiles;
    fb.rows = (int)(s.B * s.D);
    fb.nblocks = (int)cdiv(s.B * s.D * (ntiles + 1) * H, 256);
  }
  fscm_param_reduce_kernel<T><<<(unsigned)(cdiv(n, 32) + fb.nblocks), dim3(32, 8), 0, st>>>(
      (const float *)ws, (T *)gw, s.has_bias ? (T *)gb : nullptr, (T *)gmw, (T *)gmb, (int)s.D,
      (int)s.C, (int)s.S, (int)(s.B * ntiles), (T *)gx, fb);
  return check_launch("fscm_param_reduce_kernel");
}

// Self-check of the 16-bit path's approximations against CUDA's erff / expf over n points
// of [lo, hi]: max of |Phi_A&S7.1.28(z) - Phi_erff(z)| and |GELU'_16bit(z) - GELU'_fp32(z)|
// (the latter adds the ex2.approx Gaussian); result as the bits of a non-negative float.
__device__ unsigned g_phi_check_max_bits;  // the self-check's result word (no allocation)

__global__ void phi_check_kernel(int n, float lo, float hi) {
  unsigned *max_bits = &g_phi_check_max_bits;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
    const float z = lo + (hi - lo) * ((float)i / (float)(n - 1));
    float g16, gp16, g32, gp32;
    gelu_and_grad<__half>(z, g16, gp16);
    gelu_and_grad<float>(z, g32, gp32);
    const float ref = 0.5f * (1.f + erff(z * kInvSqrt2));
    const float fwd = phi_from_tail(z, 0.5f * r16_as7128(fabsf(z)));
    const float bwd = phi_from_tail(z, tail_as26216(fabsf(z), npdf_approx(z)));
    const float e = fmaxf(fmaxf(fabsf(fwd - ref), fabsf(bwd - ref)), fabsf(gp16 - gp32));
    atomicMax(max_bits, __float_as_uint(e));
  }
}

}  // namespace

int check_phi_approx(float *max_abs_err) {
  const unsigned zero = 0;
  if (cudaMemcpyToSymbol(g_phi_check_max_bits, &zero, sizeof(zero)) != cudaSuccess)
    return check_launch("cudaMemcpyToSymbol(phi check word)");
  phi_check_kernel<<<296, 256>>>(1 << 22, -12.f, 12.f);
  if (int rc = check_launch("phi_check_kernel")) return rc;
  unsigned h = 0;
  if (cudaMemcpyFromSymbol(&h, g_phi_check_max_bits, sizeof(h)) != cudaSuccess)
    return check_launch("phi_check_kernel");
  uint32_t bits = h;
  float v;
  memcpy(&v, &bits, sizeof(v));
  *max_abs_err = v;
  return DUDY_OK;
}

// tile_t (the reference backward plan's token tile) is accepted for interface parity; this
// design's tile is fixed by its 2048-token span.
bool fscm_shapes_fit(const FscmShape &s, int64_t tile_t) {
  (void)tile_t;
  return s.S <= kMaxS && s.halo() <= kMaxHalo && fwd_smem(s) <= kMaxSmem &&
         bwd_smem(s) <= kMaxSmem;
}

size_t fscm_bwd_workspace(const FscmShape &s, int64_t tile_t) {
  (void)tile_t;
  return bwd_part_bytes(s) + bwd_bnd_bytes(s);
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
  (void)tile_t;
  switch (dtype) {
    case DUDY_DTYPE_F32:
      return bwd_impl<float>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, st);
    case DUDY_DTYPE_F16:
      return bwd_impl<__half>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, st);
    default:
      return bwd_impl<__nv_bfloat16>(go, x, w, bias, mw, gx, gw, gb, gmw, gmb, ws, s, st);
  }
}

}  // namespace dudy
