/*
 * dudyconv_b200.h -- C ABI of the B200 (sm_100a) fused dynamic causal convolution
 * and fused source conv library (libdudyconv_b200.so).
 *
 * Plain pointers and sizes only: no torch types cross this boundary. Every
 * tensor is a dense, row-major (C-contiguous) device buffer of `dtype`
 * elements, laid out as named below. All work is enqueued on `stream`
 * (a cudaStream_t passed as void*; NULL = legacy default stream) of the
 * current CUDA device. No compute call allocates device memory: scratch is the
 * caller's `workspace`, sized by the *_workspace_size query, except for
 * dudy_fdc_backward_noalloc, whose scratch is a fixed array inside the library.
 *
 * Every compute entry point returns a status (DUDY_OK = 0). On failure,
 * dudy_last_error() gives a message (per host thread). Status mapping mirrors
 * the reference's error behaviour: a shape/argument error is raised there as
 * RuntimeError via TORCH_CHECK (fused_dynamic_conv_kernel.cu:390-452), and the
 * torch binding in this package converts DUDY_ERR_INVALID the same way.
 *
 * Reference interfaces replaced (adjfangjiawei/DUDyConv, cuda_ops/):
 *   dudy_fdc_forward   <- fused_dynamic_conv_forward_chunk_cuda
 *                         (fused_dynamic_conv_kernel.cu:920-942, bound as
 *                         cuda_ops_ext.forward_chunk, fused_dynamic_conv.cpp:59-61)
 *   dudy_fdc_backward  <- fused_dynamic_conv_backward_chunk_cuda
 *                         (fused_dynamic_conv_kernel.cu:944-1024, bound as
 *                         cuda_ops_ext.backward_chunk, fused_dynamic_conv.cpp:79-82)
 *   dudy_fscm_forward  <- fused_source_conv_mixed_forward_cuda / _plan_cuda
 *                         (fused_source_conv_mixed_forward.cu:828-997, bound as
 *                         torch.ops.fused_source_conv_mixed.forward[_plan],
 *                         fused_source_conv_mixed_ops.cpp:354-378)
 *   dudy_fscm_backward <- fused_source_conv_mixed_backward_cuda / _plan_cuda
 *                         (fused_source_conv_mixed_backward.cu:736-1055, bound as
 *                         torch.ops.fused_source_conv_mixed.backward[_plan],
 *                         fused_source_conv_mixed_ops.cpp:404-430)
 */
#ifndef DUDYCONV_B200_H_
#define DUDYCONV_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DUDY_API __attribute__((visibility("default")))
#else
#define DUDY_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- element types (the reference accepts fp32 / fp16 / bf16, all tensors equal;
 *      cuda_ops/fused_dynamic_conv.py:170-186) ---- */
#define DUDY_DTYPE_F32 0
#define DUDY_DTYPE_F16 1
#define DUDY_DTYPE_BF16 2

/* ---- status codes ---- */
#define DUDY_OK 0
#define DUDY_ERR_INVALID 1     /* shape / argument check failed (reference: RuntimeError) */
#define DUDY_ERR_UNSUPPORTED 2 /* explicit plan is not legal for these shapes            */
#define DUDY_ERR_CUDA 3        /* a CUDA runtime / driver call or launch failed           */
#define DUDY_ERR_WORKSPACE 4   /* workspace missing or smaller than the size query says   */
#define DUDY_ERR_DEVICE 5      /* current device is not an sm_100 (B200-class) GPU        */

/* ---- dynamic-conv plans (the reference's plan ids are autotune bookkeeping; these are
 *      this library's own, stable ids) ---- */
#define DUDY_PLAN_AUTO (-1)
#define DUDY_FDC_PLAN_SIMT 100   /* CUDA-core kernels: any shape, the fp32 path            */
#define DUDY_FDC_PLAN_TC 200     /* tcgen05/TMEM + TMA kernels: fp16/bf16, D%128==0
                                    (backward: D in {128,256}), N in {16,32,64,128},
                                    (K-1)*dil <= 121, T%8==0, L%8==0, 16B-aligned tensors */

/* Human-readable name of a dynamic-conv plan id ("not_cached" for -1). Never NULL. */
DUDY_API const char *dudy_fdc_plan_name(int plan);

/* Message of the last failed call on this host thread ("" if none). Never NULL. */
DUDY_API const char *dudy_last_error(void);

/* Library version string. */
DUDY_API const char *dudy_version(void);

/* Device error word of the current device: nonzero means a bounded wait inside a
 * tensor-core kernel gave up (that call's outputs are invalid; the kernel returned
 * instead of hanging). Synchronizes the device. reset != 0 clears the word.
 * Returns -1 if the word cannot be read. No counterpart in the reference (its kernels
 * have no device-side waits). */
DUDY_API int dudy_device_error(int reset);

/* As dudy_device_error, and copies the device error record into info4[0..3]:
 * [0] id of the wait site that timed out first (0 = none), [1] block index, [2] thread
 * index, [3] loop counter of that wait. */
DUDY_API int dudy_device_error_info(int *info4, int reset);

/* ========================================================================================
 * Fused dynamic causal convolution
 *
 *   h    [B, D, L]     kc [B, K, N, T]     mix [D, N]      out [B, D, T]
 *   out[b,d,t] = sum_{kk<K} sum_{n<N} h[b,d, off+t-kk*dil] * kc[b,kk,n,t] * mix[d,n]
 *   (terms with off+t-kk*dil < 0 are zero; requires off >= 0, dil >= 1, off+T <= L)
 * ======================================================================================== */

/* Plan that DUDY_PLAN_AUTO resolves to for these shapes and pointers (pointers are
 * only inspected for alignment). Returns a plan id, or -1 on invalid arguments. */
DUDY_API int dudy_fdc_default_plan(const void *h, const void *kc, const void *mix,
                          int64_t B, int64_t D, int64_t L, int64_t T, int64_t N,
                          int64_t K, int64_t off, int64_t dilation, int dtype);

/* 1 if `plan` can run these shapes/pointers, else 0. */
DUDY_API int dudy_fdc_plan_available(int plan, const void *h, const void *kc, const void *mix,
                            int64_t B, int64_t D, int64_t L, int64_t T, int64_t N,
                            int64_t K, int64_t off, int64_t dilation, int dtype);

/* out[B,D,T] <- forward. plan: DUDY_PLAN_AUTO or an available plan id. */
DUDY_API int dudy_fdc_forward(const void *h, const void *kc, const void *mix, void *out,
                     int64_t B, int64_t D, int64_t L, int64_t T, int64_t N, int64_t K,
                     int64_t off, int64_t dilation, int dtype, int plan, void *stream);

/* Bytes of workspace dudy_fdc_backward needs for these shapes and plan. */
DUDY_API size_t dudy_fdc_backward_workspace_size(int64_t B, int64_t D, int64_t L, int64_t T,
                                        int64_t N, int64_t K, int64_t off,
                                        int64_t dilation, int dtype, int plan);

/* Backward of the forward above, for upstream gradient go[B,D,T]:
 *   grad_h   [B,D,L]   (written in full: zero outside [off-(K-1)*dil, off+T))
 *   grad_kc  [B,K,N,T]
 *   grad_mix [D,N]     (reduced over batch, taps and time in fp32, then cast)
 * `workspace` must hold dudy_fdc_backward_workspace_size(...) bytes (256-byte aligned).
 * All three outputs are overwritten (not accumulated). */
DUDY_API int dudy_fdc_backward(const void *go, const void *h, const void *kc, const void *mix,
                      void *grad_h, void *grad_kc, void *grad_mix,
                      void *workspace, size_t workspace_bytes,
                      int64_t B, int64_t D, int64_t L, int64_t T, int64_t N, int64_t K,
                      int64_t off, int64_t dilation, int dtype, int plan, void *stream);

/* The two halves of dudy_fdc_backward, for callers that need only some gradients
 * (e.g. h does not require grad). Together they equal dudy_fdc_backward. No single
 * counterpart in the reference, whose backward always returns all three
 * (fused_dynamic_conv_kernel.cu:944-1024).
 *   dudy_fdc_backward_grad_h      : grad_h [B,D,L] only (no workspace).
 *   dudy_fdc_backward_grad_kc_mix : grad_kc [B,K,N,T] and grad_mix [D,N]; workspace as
 *                                   for dudy_fdc_backward. */
DUDY_API int dudy_fdc_backward_grad_h(const void *go, const void *kc, const void *mix,
                                      void *grad_h, int64_t B, int64_t D, int64_t L,
                                      int64_t T, int64_t N, int64_t K, int64_t off,
                                      int64_t dilation, int dtype, int plan, void *stream);
DUDY_API int dudy_fdc_backward_grad_kc_mix(const void *go, const void *h, const void *kc,
                                           const void *mix, void *grad_kc, void *grad_mix,
                                           void *workspace, size_t workspace_bytes,
                                           int64_t B, int64_t D, int64_t L, int64_t T,
                                           int64_t N, int64_t K, int64_t off,
                                           int64_t dilation, int dtype, int plan,
                                           void *stream);

/* The backward above without a caller workspace, for callers that cannot allocate device
 * memory when they call (a process whose device memory is fixed at start-up, code where
 * cudaMalloc is not allowed or would synchronize the device, or a foreign-function caller
 * with no allocator to hand a workspace from). No counterpart in the reference (its
 * backward allocates its scratch with torch::empty on every call).
 * The scratch is a fixed array of DUDY_NOALLOC_SCRATCH_BYTES inside the library, held by
 * every GPU that loads it until process exit; shapes whose scratch need
 * (dudy_fdc_backward_workspace_size) exceeds it are rejected with DUDY_ERR_WORKSPACE.
 * The first call on a device looks up the array's device address (cudaGetSymbolAddress),
 * so make that first call before any stream capture (a failed lookup is retried on the
 * next call; after a cudaDeviceReset the array is gone). All calls share the one array
 * and nothing in it needs to start at zero (every partial is written before it is read
 * within a call): calls that can overlap on the GPU (different streams without ordering)
 * race; calls on one stream are ordered. */
#define DUDY_NOALLOC_SCRATCH_BYTES (20u * 1024u * 1024u)
DUDY_API int dudy_fdc_backward_noalloc(const void *go, const void *h, const void *kc,
                                       const void *mix, void *grad_h, void *grad_kc,
                                       void *grad_mix, int64_t B, int64_t D, int64_t L,
                                       int64_t T, int64_t N, int64_t K, int64_t off,
                                       int64_t dilation, int dtype, int plan, void *stream);

/* ---- data-parallel backward with the grad_mix sum over ranks in the same call ----
 * For a batch sharded over ranks (one GPU each): the backward of this rank's sequences,
 * with grad_mix summed over all ranks by the backward's last kernel itself, over peer
 * memory (plain loads and stores through NVLink mappings): each rank publishes its fp32
 * sum in its exchange buffer as 64-bit {call counter : value} words, reads the others'
 * (polling, bounded, until a word carries the current counter) and adds them in rank order,
 * so every rank ends with bitwise-identical grad_mix, rounded once to `dtype`. grad_h and
 * grad_kc are this rank's. Replaces dudy_fdc_backward followed by an all-reduce of
 * grad_mix (no counterpart in the reference, which has no distributed code).
 *   xchg->bufs[r] : rank r's exchange buffer of dudy_fdc_exchange_bytes(D, N) bytes, as
 *                   mapped in this process (own buffer at bufs[rank]); 16-byte aligned;
 *                   zero-filled before the first call, and the same on every rank.
 *   xchg->epoch   : call counter, 1 for the first call and +1 per call, equal on all ranks.
 * Every rank must make the same sequence of calls, each on its own GPU (ranks that wait
 * for each other must run at the same time: never two ranks on one GPU). A peer that does
 * not arrive within the wait limit leaves grad_mix unwritten and sets the device error
 * record (site 950 + its rank; dudy_device_error_info). world = 1 is the plain backward. */
#define DUDY_MAX_PEERS 8
typedef struct DudyPeerExchange {
  void *bufs[DUDY_MAX_PEERS];
  int rank, world;
  uint32_t epoch;
} DudyPeerExchange;
DUDY_API size_t dudy_fdc_exchange_bytes(int64_t D, int64_t N);
/* Deferred form, for training loops that overlap the exchange with the next step (as
 * data-parallel training overlaps its gradient exchange with later compute): the call's last
 * kernel publishes this call's sums (counter xchg->epoch), writes this rank's own grad_mix
 * into `grad_mix`, and writes the sum over ranks of the PREVIOUS call (epoch - 1) into
 * `grad_mix_prev` (not touched on the first call, epoch 1). The previous call's words were
 * published by every rank one call earlier, so no wait is on the critical path in practice.
 * dudy_fdc_exchange_finish writes the sum over ranks of call xchg->epoch (the last one) into
 * `grad_mix` (waits, bounded, for every rank's words of that call). Same descriptor and
 * buffers as dudy_fdc_backward_dp; one counter sequence per buffer set. */
DUDY_API int dudy_fdc_backward_dp_deferred(const void *go, const void *h, const void *kc,
                                           const void *mix, void *grad_h, void *grad_kc,
                                           void *grad_mix, void *grad_mix_prev,
                                           void *workspace, size_t workspace_bytes,
                                           const DudyPeerExchange *xchg, int64_t B, int64_t D,
                                           int64_t L, int64_t T, int64_t N, int64_t K,
                                           int64_t off, int64_t dilation, int dtype, int plan,
                                           void *stream);
DUDY_API int dudy_fdc_exchange_finish(const DudyPeerExchange *xchg, void *grad_mix, int64_t D,
                                      int64_t N, int dtype, void *stream);
DUDY_API int dudy_fdc_backward_dp(const void *go, const void *h, const void *kc, const void *mix,
                                  void *grad_h, void *grad_kc, void *grad_mix, void *workspace,
                                  size_t workspace_bytes, const DudyPeerExchange *xchg,
                                  int64_t B, int64_t D, int64_t L, int64_t T, int64_t N,
                                  int64_t K, int64_t off, int64_t dilation, int dtype, int plan,
                                  void *stream);

/* ---- the kernel generator's tail, fused (one pass each way) ----
 * Replaces the reshape -> softmax over K -> flip(K) -> permute -> contiguous sequence of
 * StreamingKernelGenConv1d._logits_to_kernel (backbone_dil_unshared.py:1821-1900), which
 * produces the op's kernel_chunk from the kernel generator's logits:
 *   logits [B, N*K, T]  ->  kc [B, K, N, T],
 *   kc[b,kk,n,t] = softmax_k(logits[b, n*K+k, t]) evaluated at k = K-1-kk
 * (fp32 arithmetic, one rounding). The backward takes that kc (the forward's output) and
 * grad_kc [B,K,N,T] and writes grad_logits [B, N*K, T] (softmax backward in fp32). */
DUDY_API int dudy_logits_to_kernel(const void *logits, void *kc, int64_t B, int64_t N,
                                   int64_t K, int64_t T, int dtype, void *stream);
DUDY_API int dudy_logits_to_kernel_backward(const void *kc, const void *grad_kc,
                                            void *grad_logits, int64_t B, int64_t N,
                                            int64_t K, int64_t T, int dtype, void *stream);

/* ========================================================================================
 * Fused source conv (depthwise causal conv -> bias -> exact GELU -> static mix)
 *
 *   x [B,D,L]  weight [D,C,S]  bias [D,C] or NULL  mix_w [D,C]  mix_b [D]  out [B,D,T]
 *   z[b,d,c,t]  = bias[d,c] + sum_{j<S} x[b,d, off+t-dil*(S-1-j)] * weight[d,c,j]
 *   out[b,d,t]  = mix_b[d] + sum_{c<C} GELU_erf(z[b,d,c,t]) * mix_w[d,c]
 *
 * Plan ids are the reference's (cuda_ops/fused_source_conv_mixed.py:12-25):
 *   forward : 0 Generic, 1 C8S3, 2 C32S3, 3 D256C16S3, +100 for the NoBoundary variants
 *             (legal when off >= dil*(S-1)); -1 = heuristic.
 *   backward: 0 Atomic, 1 PerDReduce, 2 GatherX (tile_t in {>0}); -1 = heuristic.
 * Every legal plan runs this library's kernels; plans select tiling, not semantics.
 * ======================================================================================== */

/* 1 if the forward plan is legal for the shapes (reference legality rules,
 * fused_source_conv_mixed_forward.cu:309-365), else 0. */
DUDY_API int dudy_fscm_forward_plan_legal(int plan, int64_t D, int64_t C, int64_t S,
                                 int64_t off, int64_t dilation);

/* The reference heuristic's forward plan choice for these shapes. */
DUDY_API int dudy_fscm_forward_default_plan(int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                                   int64_t off, int64_t T, int64_t dilation);

DUDY_API int dudy_fscm_forward(const void *x, const void *weight, const void *bias,
                      const void *mix_w, const void *mix_b, void *out,
                      int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                      int64_t off, int64_t T, int64_t dilation, int dtype, int plan,
                      void *stream);

/* 1 if the backward plan/tile is legal (fused_source_conv_mixed_backward.cu:358-393). */
DUDY_API int dudy_fscm_backward_plan_legal(int plan, int64_t C, int64_t S, int64_t tile_t);

/* The reference heuristic's backward plan (fused_source_conv_mixed_backward.cu:672-730). */
DUDY_API int dudy_fscm_backward_default_plan(int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                                    int64_t off, int64_t T, int64_t dilation);

DUDY_API size_t dudy_fscm_backward_workspace_size(int64_t B, int64_t D, int64_t L, int64_t C,
                                         int64_t S, int64_t off, int64_t T,
                                         int64_t dilation, int dtype, int plan,
                                         int64_t tile_t);

/* Backward for upstream gradient go[B,D,T]; writes grad_x [B,D,L] (full, zero outside
 * the receptive range), grad_w [D,C,S], grad_bias [D,C] (ignored if bias == NULL),
 * grad_mix_w [D,C], grad_mix_b [D]. Parameter gradients are reduced in fp32,
 * deterministically, then cast. */
DUDY_API int dudy_fscm_backward(const void *go, const void *x, const void *weight, const void *bias,
                       const void *mix_w, const void *mix_b,
                       void *grad_x, void *grad_w, void *grad_bias, void *grad_mix_w,
                       void *grad_mix_b, void *workspace, size_t workspace_bytes,
                       int64_t B, int64_t D, int64_t L, int64_t C, int64_t S,
                       int64_t off, int64_t T, int64_t dilation, int dtype, int plan,
                       int64_t tile_t, void *stream);

/* Self-test of the bounded waits (no reference counterpart: its kernels have no
 * device-side waits). Runs one CTA built like the tensor-core kernels (one warp holding a
 * TMEM allocation) in which one warp waits, with a limit of `limit_us` microseconds
 * (0 < limit_us <= 1e6), on an mbarrier that nothing arrives at: the wait gives up,
 * records wait site 901 (block 0, thread 0, counter 7) in the device error record and
 * raises the CTA's abort flag; the other warp's wait (normal limit) sees the flag and
 * returns; the CTA frees its TMEM and exits. results2[i] = 1 if warp i's wait completed,
 * 0 if it gave up. Synchronous (legacy default stream); nothing is allocated. Read the
 * record with dudy_device_error_info and clear it before further use. */
DUDY_API int dudy_selftest_wait_timeout(int limit_us, int *results2);

/* Self-check (no reference counterpart): the source conv's fp16/bf16 kernels evaluate the
 * normal CDF with Abramowitz & Stegun approximations (7.1.28 in the forward, 26.2.16 in
 * the backward) and the Gaussian in GELU' with a single-instruction base-2 exponential. This runs both against CUDA's erff /
 * expf on 4M points of [-12, 12] on the current device (synchronous, on the legacy default
 * stream; its result word is a library variable, nothing is allocated) and
 * stores the largest absolute difference of Phi or of GELU'. */
DUDY_API int dudy_check_phi_approx(float *max_abs_err);

#ifdef __cplusplus
}
#endif

#endif /* DUDYCONV_B200_H_ */
