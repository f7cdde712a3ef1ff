// torch_ext.cpp -- the torch-facing binding of libdudyconv_b200, built as the Python
// module `cuda_ops_ext`.
//
// It exposes the same surface the reference's Python layer binds to:
//   * pybind functions of `cuda_ops_ext` (reference cuda_ops/fused_dynamic_conv.cpp:58-101):
//     forward_chunk, forward_chunk_warmup, forward_chunk_cached_plan,
//     forward_chunk_clear_warmup_cache, forward_plan_name, backward_chunk,
//     backward_chunk_warmup, backward_chunk_cached_plan, backward_chunk_clear_warmup_cache,
//     backward_plan_name -- same argument names and defaults;
//   * TORCH_LIBRARY(fused_source_conv_mixed) with the 14 schemas of the reference
//     (cuda_ops/fused_source_conv_mixed_ops.cpp:354-505).
// Tensors are checked here (CUDA, dtype, shape; reference messages), outputs are
// allocated with the caching allocator, and all compute goes through the C ABI on the
// current stream. A nonzero C-ABI status becomes a RuntimeError (TORCH_CHECK).
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <string>
#include <tuple>
#include <vector>

#include "dudyconv_b200.h"

namespace {

int dtype_code(const torch::Tensor &t) {
  switch (t.scalar_type()) {
    case at::ScalarType::Float: return DUDY_DTYPE_F32;
    case at::ScalarType::Half: return DUDY_DTYPE_F16;
    case at::ScalarType::BFloat16: return DUDY_DTYPE_BF16;
    default: TORCH_CHECK(false, "Unsupported dtype: ", t.scalar_type(), ".");
  }
  return -1;
}

void check_status(int rc, const char *what) {
  TORCH_CHECK(rc == DUDY_OK, what, ": ", dudy_last_error(), " (status ", rc, ")");
}

bool debug_path() {
  static const bool on = std::getenv("DUDY_DEBUG_PATH") != nullptr ||
                         std::getenv("FDC_DEBUG_PATH") != nullptr;
  return on;
}

void *stream_ptr() { return reinterpret_cast<void *>(at::cuda::getCurrentCUDAStream().stream()); }

// ---------------------------------------------------------------------------------------
// dynamic conv
// ---------------------------------------------------------------------------------------
struct FdcDims {
  int64_t B, D, L, T, N, K;
};

// checks of the reference (cuda_ops/fused_dynamic_conv.py:108-186)
FdcDims check_fdc(const torch::Tensor &h, const torch::Tensor &kc, const torch::Tensor &mix,
                  int64_t off, int64_t dilation) {
  TORCH_CHECK(dilation > 0, "dilation must be positive.");
  TORCH_CHECK(h.is_cuda(), "h_full must be CUDA tensor.");
  TORCH_CHECK(kc.is_cuda(), "kernel_chunk must be CUDA tensor.");
  TORCH_CHECK(mix.is_cuda(), "kernel_mix must be CUDA tensor.");
  TORCH_CHECK(h.dim() == 3, "h_full must be [B,D,L], got ", h.sizes(), ".");
  TORCH_CHECK(kc.dim() == 4, "kernel_chunk must be [B,K,N,T], got ", kc.sizes(), ".");
  TORCH_CHECK(mix.dim() == 2, "kernel_mix must be [D,N], got ", mix.sizes(), ".");
  FdcDims d{h.size(0), h.size(1), h.size(2), kc.size(3), kc.size(2), kc.size(1)};
  TORCH_CHECK(kc.size(0) == d.B, "B mismatch: h_full=", d.B, ", kernel_chunk=", kc.size(0), ".");
  TORCH_CHECK(mix.size(0) == d.D, "D mismatch: h_full=", d.D, ", kernel_mix=", mix.size(0), ".");
  TORCH_CHECK(mix.size(1) == d.N, "N mismatch: kernel_chunk=", d.N, ", kernel_mix=", mix.size(1), ".");
  TORCH_CHECK(d.T > 0, "T must be positive.");
  TORCH_CHECK(d.K > 0, "K must be positive.");
  TORCH_CHECK(off >= 0, "t_offset must be non-negative.");
  TORCH_CHECK(off + d.T <= d.L, "t_offset + T must be <= L, got t_offset=", off, ", T=", d.T,
              ", L=", d.L, ".");
  dtype_code(h);
  TORCH_CHECK(kc.scalar_type() == h.scalar_type(), "kernel_chunk dtype must equal h_full dtype.");
  TORCH_CHECK(mix.scalar_type() == h.scalar_type(), "kernel_mix dtype must equal h_full dtype.");
  TORCH_CHECK(kc.device() == h.device() && mix.device() == h.device(),
              "all tensors must be on the same device.");
  TORCH_CHECK(h.is_contiguous() && kc.is_contiguous() && mix.is_contiguous(),
              "h, kc and mix must be contiguous.");
  return d;
}

void check_go(const torch::Tensor &go, const torch::Tensor &h, const FdcDims &d) {
  TORCH_CHECK(go.is_cuda(), "grad_out must be CUDA tensor.");
  TORCH_CHECK(go.dim() == 3, "grad_out must be [B,D,T], got ", go.sizes(), ".");
  TORCH_CHECK(go.size(0) == d.B, "grad_out B mismatch: grad_out=", go.size(0), ", h_full=", d.B, ".");
  TORCH_CHECK(go.size(1) == d.D, "grad_out D mismatch: grad_out=", go.size(1), ", h_full=", d.D, ".");
  TORCH_CHECK(go.size(2) == d.T, "grad_out T mismatch: grad_out=", go.size(2),
              ", kernel_chunk T=", d.T, ".");
  TORCH_CHECK(go.scalar_type() == h.scalar_type(), "grad_out dtype must equal h_full dtype.");
  TORCH_CHECK(go.device() == h.device(), "grad_out must be on the device of h.");
  TORCH_CHECK(go.is_contiguous(), "grad_out must be contiguous.");
}

using PlanKey = std::tuple<int, int, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                           int64_t>;
std::mutex g_mu;
std::map<PlanKey, int> g_fwd_cache, g_bwd_cache;

PlanKey make_key(const torch::Tensor &h, int64_t N, int64_t K, int64_t T, int64_t off,
                 int64_t dil) {
  return PlanKey{h.get_device(), dtype_code(h), h.size(0), h.size(1), h.size(2), T, N, K, off, dil};
}

int cached(std::map<PlanKey, int> &m, const PlanKey &k) {
  std::lock_guard<std::mutex> lk(g_mu);
  auto it = m.find(k);
  return it == m.end() ? -1 : it->second;
}

torch::Tensor fwd_run(const torch::Tensor &h, const torch::Tensor &kc, const torch::Tensor &mix,
                      const FdcDims &d, int64_t off, int64_t dil, int plan) {
  auto out = torch::empty({d.B, d.D, d.T}, h.options());
  const int rc = dudy_fdc_forward(h.data_ptr(), kc.data_ptr(), mix.data_ptr(), out.data_ptr(),
                                  d.B, d.D, d.L, d.T, d.N, d.K, off, dil, dtype_code(h), plan,
                                  stream_ptr());
  check_status(rc, "fused_dynamic_conv forward");
  return out;
}

std::vector<torch::Tensor> bwd_run(const torch::Tensor &go, const torch::Tensor &h,
                                   const torch::Tensor &kc, const torch::Tensor &mix,
                                   const FdcDims &d, int64_t off, int64_t dil, int plan) {
  auto gh = torch::empty_like(h);
  auto gk = torch::empty_like(kc);
  auto gm = torch::empty_like(mix);
  const int dt = dtype_code(h);
  const size_t ws_bytes =
      dudy_fdc_backward_workspace_size(d.B, d.D, d.L, d.T, d.N, d.K, off, dil, dt, plan);
  auto ws = torch::empty({(int64_t)std::max<size_t>(ws_bytes, 256)},
                         h.options().dtype(torch::kUInt8));
  const int rc = dudy_fdc_backward(go.data_ptr(), h.data_ptr(), kc.data_ptr(), mix.data_ptr(),
                                   gh.data_ptr(), gk.data_ptr(), gm.data_ptr(), ws.data_ptr(),
                                   (size_t)ws.numel(), d.B, d.D, d.L, d.T, d.N, d.K, off, dil, dt,
                                   plan, stream_ptr());
  check_status(rc, "fused_dynamic_conv backward");
  return {gh, gk, gm};
}

std::vector<int> candidate_plans(const torch::Tensor &h, const torch::Tensor &kc,
                                 const torch::Tensor &mix, const FdcDims &d, int64_t off,
                                 int64_t dil) {
  std::vector<int> c;
  const int dt = dtype_code(h);
  if (dudy_fdc_plan_available(DUDY_FDC_PLAN_TC, h.data_ptr(), kc.data_ptr(), mix.data_ptr(), d.B,
                              d.D, d.L, d.T, d.N, d.K, off, dil, dt))
    c.push_back(DUDY_FDC_PLAN_TC);
  c.push_back(DUDY_FDC_PLAN_SIMT);
  return c;
}

template <typename F>
float median_ms(F &&fn, int64_t repeat) {
  auto stream = at::cuda::getCurrentCUDAStream();
  fn();  // dry run
  std::vector<float> ms;
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  for (int64_t i = 0; i < repeat; ++i) {
    cudaEventRecord(a, stream.stream());
    fn();
    cudaEventRecord(b, stream.stream());
    cudaEventSynchronize(b);
    float t = 0.f;
    cudaEventElapsedTime(&t, a, b);
    ms.push_back(t);
  }
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  std::sort(ms.begin(), ms.end());
  return ms[ms.size() / 2];
}

torch::Tensor forward_chunk(torch::Tensor h, torch::Tensor kc, torch::Tensor mix, int64_t off,
                            int64_t dilation) {
  const FdcDims d = check_fdc(h, kc, mix, off, dilation);
  const c10::cuda::CUDAGuard guard(h.device());
  const int plan = cached(g_fwd_cache, make_key(h, d.N, d.K, d.T, off, dilation));
  if (debug_path())
    TORCH_WARN("[dudyconv] forward plan ", plan < 0 ? "auto" : dudy_fdc_plan_name(plan), " -> ",
               dudy_fdc_plan_name(dudy_fdc_default_plan(h.data_ptr(), kc.data_ptr(),
                                                        mix.data_ptr(), d.B, d.D, d.L, d.T, d.N,
                                                        d.K, off, dilation, dtype_code(h))));
  return fwd_run(h, kc, mix, d, off, dilation, plan);
}

int64_t forward_chunk_warmup(torch::Tensor h, torch::Tensor kc, torch::Tensor mix, int64_t off,
                             int64_t dilation, int64_t repeat) {
  TORCH_CHECK(repeat > 0, "repeat must be positive.");
  const FdcDims d = check_fdc(h, kc, mix, off, dilation);
  const c10::cuda::CUDAGuard guard(h.device());
  int best = -1;
  float best_ms = 1e30f;
  for (int p : candidate_plans(h, kc, mix, d, off, dilation)) {
    const float ms = median_ms([&] { fwd_run(h, kc, mix, d, off, dilation, p); }, repeat);
    if (debug_path()) TORCH_WARN("[dudyconv] forward warmup ", dudy_fdc_plan_name(p), ": ", ms, " ms");
    if (ms < best_ms) {
      best_ms = ms;
      best = p;
    }
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_fwd_cache[make_key(h, d.N, d.K, d.T, off, dilation)] = best;
  return best;
}

int64_t forward_chunk_cached_plan(torch::Tensor h, torch::Tensor kc, torch::Tensor mix,
                                  int64_t off, int64_t dilation) {
  const FdcDims d = check_fdc(h, kc, mix, off, dilation);
  return cached(g_fwd_cache, make_key(h, d.N, d.K, d.T, off, dilation));
}

void forward_chunk_clear_warmup_cache() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_fwd_cache.clear();
}

std::string plan_name(int64_t plan_id) { return dudy_fdc_plan_name((int)plan_id); }

std::vector<torch::Tensor> backward_chunk(torch::Tensor go, torch::Tensor h, torch::Tensor kc,
                                          torch::Tensor mix, int64_t off, int64_t dilation) {
  const FdcDims d = check_fdc(h, kc, mix, off, dilation);
  check_go(go, h, d);
  const c10::cuda::CUDAGuard guard(h.device());
  const int plan = cached(g_bwd_cache, make_key(h, d.N, d.K, d.T, off, dilation));
  if (debug_path())
    TORCH_WARN("[dudyconv] backward plan ", plan < 0 ? "auto" : dudy_fdc_plan_name(plan));
  return bwd_run(go, h, kc, mix, d, off, dilation, plan);
}

int64_t backward_chunk_warmup(torch::Tensor go, torch::Tensor h, torch::Tensor kc,
                              torch::Tensor mix, int64_t off, int64_t dilation, int64_t repeat) {
  TORCH_CHECK(repeat > 0, "repeat must be positive.");
  const FdcDims d = check_fdc(h, kc, mix, off, dilation);
  check_go(go, h, d);
  const c10::cuda::CUDAGuard guard(h.device());
  int best = -1;
  float best_ms = 1e30f;
  for (int p : candidate_plans(h, kc, mix, d, off, dilation)) {
    const float ms = median_ms([&] { bwd_run(go, h, kc, mix, d, off, dilation, p); }, repeat);
    if (debug_path()) TORCH_WARN("[dudyconv] backward warmup ", dudy_fdc_plan_name(p), ": ", ms, " ms");
    if (ms < best_ms) {
      best_ms = ms;
      best = p;
    }
  }
  std::lock_guard<std::mutex> lk(g_mu);
  g_bwd_cache[make_key(h, d.N, d.K, d.T, off, dilation)] = best;
  return best;
}

int64_t backward_chunk_cached_plan(torch::Tensor h, torch::Tensor kc, int64_t off,
                                   int64_t dilation) {
  TORCH_CHECK(h.dim() == 3 && kc.dim() == 4, "h must be [B,D,L] and kc [B,K,N,T].");
  return cached(g_bwd_cache, make_key(h, kc.size(2), kc.size(1), kc.size(3), off, dilation));
}

void backward_chunk_clear_warmup_cache() {
  std::lock_guard<std::mutex> lk(g_mu);
  g_bwd_cache.clear();
}

// ---------------------------------------------------------------------------------------
// fused source conv (schemas of cuda_ops/fused_source_conv_mixed_ops.cpp:354-505)
// ---------------------------------------------------------------------------------------
struct FscmDims {
  int64_t B, D, L, C, S;
  bool has_bias;
};

FscmDims check_fscm(const torch::Tensor &x, const torch::Tensor &w, const torch::Tensor &bias,
                    const torch::Tensor &mw, const torch::Tensor &mb, int64_t off, int64_t T,
                    int64_t dil) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda() && mw.is_cuda() && mb.is_cuda(),
              "fused_source_conv_mixed: tensors must be CUDA tensors.");
  TORCH_CHECK(x.dim() == 3, "x_norm must be [B,D,L], got ", x.sizes(), ".");
  TORCH_CHECK(w.dim() == 3, "weight must be [D,C,S], got ", w.sizes(), ".");
  TORCH_CHECK(mw.dim() == 2, "mix_weight must be [D,C], got ", mw.sizes(), ".");
  TORCH_CHECK(mb.dim() == 1, "mix_bias must be [D], got ", mb.sizes(), ".");
  FscmDims d{x.size(0), x.size(1), x.size(2), w.size(1), w.size(2),
             bias.defined() && bias.numel() > 0};
  TORCH_CHECK(w.size(0) == d.D, "weight D mismatch: weight=", w.size(0), ", x_norm=", d.D, ".");
  TORCH_CHECK(mw.size(0) == d.D && mw.size(1) == d.C, "mix_weight must be [D,C].");
  TORCH_CHECK(mb.size(0) == d.D, "mix_bias D mismatch: mix_bias=", mb.size(0), ", x_norm=", d.D, ".");
  if (d.has_bias) {
    TORCH_CHECK(bias.is_cuda(), "bias must be CUDA tensor when provided.");
    TORCH_CHECK(bias.dim() == 2 && bias.size(0) == d.D && bias.size(1) == d.C,
                "bias must be [D,C], got ", bias.sizes(), ".");
    TORCH_CHECK(bias.scalar_type() == x.scalar_type(), "bias dtype must equal x_norm dtype.");
    TORCH_CHECK(bias.is_contiguous(), "bias must be contiguous.");
  }
  dtype_code(x);
  TORCH_CHECK(w.scalar_type() == x.scalar_type(), "weight dtype must equal x_norm dtype.");
  TORCH_CHECK(mw.scalar_type() == x.scalar_type(), "mix_weight dtype must equal x_norm dtype.");
  TORCH_CHECK(mb.scalar_type() == x.scalar_type(), "mix_bias dtype must equal x_norm dtype.");
  TORCH_CHECK(off >= 0, "off must be non-negative.");
  TORCH_CHECK(T > 0, "T must be positive.");
  TORCH_CHECK(off + T <= d.L, "off + T must be <= L, got off=", off, ", T=", T, ", L=", d.L, ".");
  TORCH_CHECK(dil > 0, "dilation must be positive.");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous() && mw.is_contiguous() && mb.is_contiguous(),
              "fused_source_conv_mixed: tensors must be contiguous.");
  return d;
}

torch::Tensor fscm_fwd(const torch::Tensor &x, const torch::Tensor &w, const torch::Tensor &bias,
                       const torch::Tensor &mw, const torch::Tensor &mb, int64_t off, int64_t T,
                       int64_t dil, int64_t plan) {
  const FscmDims d = check_fscm(x, w, bias, mw, mb, off, T, dil);
  const c10::cuda::CUDAGuard guard(x.device());
  auto out = torch::empty({d.B, d.D, T}, x.options());
  const int rc = dudy_fscm_forward(x.data_ptr(), w.data_ptr(), d.has_bias ? bias.data_ptr() : nullptr,
                                   mw.data_ptr(), mb.data_ptr(), out.data_ptr(), d.B, d.D, d.L, d.C,
                                   d.S, off, T, dil, dtype_code(x), (int)plan, stream_ptr());
  check_status(rc, "fused_source_conv_mixed forward");
  return out;
}

std::vector<torch::Tensor> fscm_bwd(const torch::Tensor &go, const torch::Tensor &x,
                                    const torch::Tensor &w, const torch::Tensor &bias,
                                    const torch::Tensor &mw, const torch::Tensor &mb, int64_t off,
                                    int64_t T, int64_t dil, int64_t plan, int64_t tile_t) {
  const FscmDims d = check_fscm(x, w, bias, mw, mb, off, T, dil);
  TORCH_CHECK(go.is_cuda() && go.dim() == 3, "grad_out must be [B,D,T], got ", go.sizes(), ".");
  TORCH_CHECK(go.size(0) == d.B && go.size(1) == d.D && go.size(2) == T,
              "grad_out must be [B,D,T], got ", go.sizes(), ".");
  TORCH_CHECK(go.scalar_type() == x.scalar_type(), "grad_out dtype must equal x_norm dtype.");
  TORCH_CHECK(go.is_contiguous(), "grad_out must be contiguous.");
  const c10::cuda::CUDAGuard guard(x.device());
  auto gx = torch::empty_like(x);
  auto gw = torch::empty_like(w);
  auto gb = d.has_bias ? torch::empty_like(bias) : torch::empty({0}, x.options());
  auto gmw = torch::empty_like(mw);
  auto gmb = torch::empty_like(mb);
  const int dt = dtype_code(x);
  const size_t ws_bytes = dudy_fscm_backward_workspace_size(d.B, d.D, d.L, d.C, d.S, off, T, dil,
                                                            dt, (int)plan, tile_t);
  auto ws = torch::empty({(int64_t)std::max<size_t>(ws_bytes, 256)}, x.options().dtype(torch::kUInt8));
  const int rc = dudy_fscm_backward(
      go.data_ptr(), x.data_ptr(), w.data_ptr(), d.has_bias ? bias.data_ptr() : nullptr,
      mw.data_ptr(), mb.data_ptr(), gx.data_ptr(), gw.data_ptr(),
      d.has_bias ? gb.data_ptr() : nullptr, gmw.data_ptr(), gmb.data_ptr(), ws.data_ptr(),
      (size_t)ws.numel(), d.B, d.D, d.L, d.C, d.S, off, T, dil, dt, (int)plan, tile_t,
      stream_ptr());
  check_status(rc, "fused_source_conv_mixed backward");
  return {gx, gw, gb, gmw, gmb};
}

torch::Tensor fscm_forward_op(torch::Tensor x, torch::Tensor w, torch::Tensor bias,
                              torch::Tensor mw, torch::Tensor mb, int64_t off, int64_t T,
                              int64_t dil) {
  return fscm_fwd(x, w, bias, mw, mb, off, T, dil, DUDY_PLAN_AUTO);
}

torch::Tensor fscm_forward_plan_op(torch::Tensor x, torch::Tensor w, torch::Tensor bias,
                                   torch::Tensor mw, torch::Tensor mb, int64_t off, int64_t T,
                                   int64_t dil, int64_t plan) {
  TORCH_CHECK(dudy_fscm_forward_plan_legal((int)plan, x.size(1), w.size(1), w.size(2), off, dil),
              "fused_source_conv_mixed_forward_plan_cuda: illegal plan=", plan);
  return fscm_fwd(x, w, bias, mw, mb, off, T, dil, plan);
}

torch::Tensor fscm_forward_cached_plan_op(torch::Tensor x, torch::Tensor w, torch::Tensor bias,
                                          torch::Tensor mw, torch::Tensor mb, int64_t off,
                                          int64_t T, int64_t dil, int64_t cached_plan) {
  return fscm_forward_plan_op(x, w, bias, mw, mb, off, T, dil, cached_plan);
}

template <typename F>
float avg_ms(F &&fn, int64_t warmup_iters, int64_t bench_iters) {
  auto stream = at::cuda::getCurrentCUDAStream();
  for (int64_t i = 0; i < warmup_iters; ++i) fn();
  cudaEvent_t a, b;
  cudaEventCreate(&a);
  cudaEventCreate(&b);
  cudaEventRecord(a, stream.stream());
  for (int64_t i = 0; i < bench_iters; ++i) fn();
  cudaEventRecord(b, stream.stream());
  cudaEventSynchronize(b);
  float t = 0.f;
  cudaEventElapsedTime(&t, a, b);
  cudaEventDestroy(a);
  cudaEventDestroy(b);
  return t / (float)bench_iters;
}

int64_t fscm_forward_warmup_op(torch::Tensor x, torch::Tensor w, torch::Tensor bias,
                               torch::Tensor mw, torch::Tensor mb, int64_t off, int64_t T,
                               int64_t dil, int64_t warmup_iters, int64_t bench_iters) {
  TORCH_CHECK(warmup_iters >= 0, "fused_source_conv_mixed_forward_warmup_cuda: warmup_iters must be >= 0.");
  TORCH_CHECK(bench_iters > 0, "fused_source_conv_mixed_forward_warmup_cuda: bench_iters must be > 0.");
  check_fscm(x, w, bias, mw, mb, off, T, dil);
  const int64_t D = x.size(1), C = w.size(1), S = w.size(2);
  // candidate order of the reference (fused_source_conv_mixed_forward.cu:367-437)
  const int order[8] = {103, 101, 102, 100, 3, 1, 2, 0};
  int64_t best = -1;
  float best_ms = 1e30f;
  for (int p : order) {
    if (!dudy_fscm_forward_plan_legal(p, D, C, S, off, dil)) continue;
    const float ms = avg_ms([&] { fscm_fwd(x, w, bias, mw, mb, off, T, dil, p); }, warmup_iters, bench_iters);
    if (ms < best_ms) {
      best_ms = ms;
      best = p;
    }
  }
  return best;
}

std::vector<torch::Tensor> fscm_backward_op(torch::Tensor go, torch::Tensor x, torch::Tensor w,
                                            torch::Tensor bias, torch::Tensor mw, torch::Tensor mb,
                                            int64_t off, int64_t T, int64_t dil) {
  const int64_t tile = std::min<int64_t>(64, T);
  const int plan = dudy_fscm_backward_default_plan(x.size(0), x.size(1), x.size(2), w.size(1),
                                                   w.size(2), off, T, dil);
  return fscm_bwd(go, x, w, bias, mw, mb, off, T, dil, plan, plan == 0 ? 0 : tile);
}

std::vector<torch::Tensor> fscm_backward_plan_op(torch::Tensor go, torch::Tensor x,
                                                 torch::Tensor w, torch::Tensor bias,
                                                 torch::Tensor mw, torch::Tensor mb, int64_t off,
                                                 int64_t T, int64_t dil, int64_t plan,
                                                 int64_t tile_t) {
  TORCH_CHECK(dudy_fscm_backward_plan_legal((int)plan, w.size(1), w.size(2), tile_t),
              "fused_source_conv_mixed_backward_plan_cuda: illegal plan=", plan, ", tile_t=", tile_t);
  return fscm_bwd(go, x, w, bias, mw, mb, off, T, dil, plan, tile_t);
}

int64_t pack_plan(int64_t plan, int64_t tile_t) {
  const uint64_t p = (uint64_t)(uint32_t)plan, t = (uint64_t)(uint32_t)tile_t;
  return (int64_t)(p | (t << 32));
}
int64_t unpack_plan(int64_t packed) { return (int64_t)((uint64_t)packed & 0xffffffffull); }
int64_t unpack_tile(int64_t packed) { return (int64_t)(((uint64_t)packed >> 32) & 0xffffffffull); }

std::vector<torch::Tensor> fscm_backward_cached_plan_op(torch::Tensor go, torch::Tensor x,
                                                        torch::Tensor w, torch::Tensor bias,
                                                        torch::Tensor mw, torch::Tensor mb,
                                                        int64_t off, int64_t T, int64_t dil,
                                                        int64_t cached_plan) {
  const int64_t plan = unpack_plan(cached_plan);
  const int64_t tile = plan == 0 ? 0 : unpack_tile(cached_plan);
  return fscm_backward_plan_op(go, x, w, bias, mw, mb, off, T, dil, plan, tile);
}

int64_t fscm_backward_warmup_op(torch::Tensor go, torch::Tensor x, torch::Tensor w,
                                torch::Tensor bias, torch::Tensor mw, torch::Tensor mb,
                                int64_t off, int64_t T, int64_t dil, int64_t warmup_iters,
                                int64_t bench_iters) {
  TORCH_CHECK(warmup_iters >= 0, "fused_source_conv_mixed_backward_warmup_cuda: warmup_iters must be >= 0.");
  TORCH_CHECK(bench_iters > 0, "fused_source_conv_mixed_backward_warmup_cuda: bench_iters must be > 0.");
  check_fscm(x, w, bias, mw, mb, off, T, dil);
  const int64_t C = w.size(1), S = w.size(2);
  // candidates of the reference (fused_source_conv_mixed_backward.cu:395-466)
  std::vector<std::pair<int, int64_t>> cands{{0, 0}};
  if (C <= 64 && S <= 8) {
    for (int64_t t : {64, 128, 256}) {
      const int64_t tt = (t > T) ? T : t;
      cands.push_back({1, tt});
      cands.push_back({2, tt});
    }
  }
  int best = 0;
  int64_t best_tile = 0;
  float best_ms = 1e30f;
  for (auto &c : cands) {
    const float ms = avg_ms([&] { fscm_bwd(go, x, w, bias, mw, mb, off, T, dil, c.first, c.second); },
                            warmup_iters, bench_iters);
    if (ms < best_ms) {
      best_ms = ms;
      best = c.first;
      best_tile = c.second;
    }
  }
  return pack_plan(best, best == 0 ? 0 : best_tile);
}

std::vector<torch::Tensor> fscm_backward_atomic_op(torch::Tensor go, torch::Tensor x,
                                                   torch::Tensor w, torch::Tensor bias,
                                                   torch::Tensor mw, torch::Tensor mb, int64_t off,
                                                   int64_t T, int64_t dil) {
  return fscm_bwd(go, x, w, bias, mw, mb, off, T, dil, 0, 0);
}

std::vector<torch::Tensor> fscm_backward_per_d_reduce_op(torch::Tensor go, torch::Tensor x,
                                                         torch::Tensor w, torch::Tensor bias,
                                                         torch::Tensor mw, torch::Tensor mb,
                                                         int64_t off, int64_t T, int64_t dil,
                                                         int64_t tile_t) {
  return fscm_backward_plan_op(go, x, w, bias, mw, mb, off, T, dil, 1, tile_t);
}

std::vector<torch::Tensor> fscm_backward_gather_x_op(torch::Tensor go, torch::Tensor x,
                                                     torch::Tensor w, torch::Tensor bias,
                                                     torch::Tensor mw, torch::Tensor mb,
                                                     int64_t off, int64_t T, int64_t dil,
                                                     int64_t tile_t) {
  return fscm_backward_plan_op(go, x, w, bias, mw, mb, off, T, dil, 2, tile_t);
}

// ---------------------------------------------------------------------------------------
// kernel generator tail: logits [B, N*K, T] -> kernel_chunk [B, K, N, T] (softmax over K,
// flip), and its backward; no counterpart in the reference's binding (the reference runs
// StreamingKernelGenConv1d._logits_to_kernel in PyTorch, backbone_dil_unshared.py:1821-1900)
// ---------------------------------------------------------------------------------------
torch::Tensor logits_to_kernel(torch::Tensor logits, int64_t num_kernels, int64_t kernel_size) {
  TORCH_CHECK(logits.is_cuda(), "logits must be CUDA tensor.");
  TORCH_CHECK(logits.dim() == 3, "logits must be [B,N*K,T], got ", logits.sizes(), ".");
  TORCH_CHECK(num_kernels > 0 && kernel_size > 0, "num_kernels and kernel_size must be positive.");
  TORCH_CHECK(logits.size(1) == num_kernels * kernel_size, "logits channels must be N*K=",
              num_kernels * kernel_size, ", got ", logits.size(1), ".");
  TORCH_CHECK(logits.is_contiguous(), "logits must be contiguous.");
  const c10::cuda::CUDAGuard guard(logits.device());
  const int64_t B = logits.size(0), T = logits.size(2);
  auto kc = torch::empty({B, kernel_size, num_kernels, T}, logits.options());
  check_status(dudy_logits_to_kernel(logits.data_ptr(), kc.data_ptr(), B, num_kernels,
                                     kernel_size, T, dtype_code(logits), stream_ptr()),
               "logits_to_kernel");
  return kc;
}

torch::Tensor logits_to_kernel_backward(torch::Tensor kc, torch::Tensor grad_kc) {
  TORCH_CHECK(kc.is_cuda() && grad_kc.is_cuda(), "kc and grad_kc must be CUDA tensors.");
  TORCH_CHECK(kc.dim() == 4 && grad_kc.sizes() == kc.sizes(),
              "kc and grad_kc must both be [B,K,N,T].");
  TORCH_CHECK(grad_kc.scalar_type() == kc.scalar_type(), "grad_kc dtype must equal kc dtype.");
  TORCH_CHECK(kc.is_contiguous() && grad_kc.is_contiguous(), "kc and grad_kc must be contiguous.");
  const c10::cuda::CUDAGuard guard(kc.device());
  const int64_t B = kc.size(0), K = kc.size(1), N = kc.size(2), T = kc.size(3);
  auto gl = torch::empty({B, N * K, T}, kc.options());
  check_status(dudy_logits_to_kernel_backward(kc.data_ptr(), grad_kc.data_ptr(), gl.data_ptr(),
                                              B, N, K, T, dtype_code(kc), stream_ptr()),
               "logits_to_kernel_backward");
  return gl;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "dudyconv_b200: B200 (sm_100a) fused dynamic conv / fused source conv";
  m.def("forward_chunk", &forward_chunk, "Fused dynamic convolution forward chunk",
        py::arg("h"), py::arg("kc"), py::arg("mix"), py::arg("off"), py::arg("dilation"));
  m.def("forward_chunk_warmup", &forward_chunk_warmup, "Forward plan warmup / autotune",
        py::arg("h"), py::arg("kc"), py::arg("mix"), py::arg("off"), py::arg("dilation"),
        py::arg("repeat") = 3);
  m.def("forward_chunk_cached_plan", &forward_chunk_cached_plan, "Cached forward plan (-1 if none)",
        py::arg("h"), py::arg("kc"), py::arg("mix"), py::arg("off"), py::arg("dilation"));
  m.def("forward_chunk_clear_warmup_cache", &forward_chunk_clear_warmup_cache,
        "Clear the forward plan cache");
  m.def("forward_plan_name", &plan_name, "Forward plan name", py::arg("plan_id"));
  m.def("backward_chunk", &backward_chunk, "Fused dynamic convolution backward chunk",
        py::arg("go"), py::arg("h"), py::arg("kc"), py::arg("mix"), py::arg("off"),
        py::arg("dilation"));
  m.def("backward_chunk_warmup", &backward_chunk_warmup, "Backward plan warmup / autotune",
        py::arg("go"), py::arg("h"), py::arg("kc"), py::arg("mix"), py::arg("off"),
        py::arg("dilation"), py::arg("repeat") = 3);
  m.def("backward_chunk_cached_plan", &backward_chunk_cached_plan,
        "Cached backward plan (-1 if none)", py::arg("h"), py::arg("kc"), py::arg("off"),
        py::arg("dilation"));
  m.def("backward_chunk_clear_warmup_cache", &backward_chunk_clear_warmup_cache,
        "Clear the backward plan cache");
  m.def("backward_plan_name", &plan_name, "Backward plan name", py::arg("plan_id"));
  m.def("library_version", [] { return std::string(dudy_version()); });
  m.def("device_error", [](bool reset) { return dudy_device_error(reset ? 1 : 0); },
        py::arg("reset") = false);
  m.def("logits_to_kernel", &logits_to_kernel,
        "Kernel generator tail: softmax over K, flip, [B,N*K,T] -> [B,K,N,T]",
        py::arg("logits"), py::arg("num_kernels"), py::arg("kernel_size"));
  m.def("logits_to_kernel_backward", &logits_to_kernel_backward,
        "Backward of logits_to_kernel from its output kc and grad_kc", py::arg("kc"),
        py::arg("grad_kc"));
}

TORCH_LIBRARY(fused_source_conv_mixed, m) {
  m.def("forward(Tensor x_norm, Tensor weight, Tensor bias, Tensor mix_weight, Tensor mix_bias, "
        "int off, int T, int dilation) -> Tensor");
  m.def("forward_plan(Tensor x_norm, Tensor weight, Tensor bias, Tensor mix_weight, "
        "Tensor mix_bias, int off, int T, int dilation, int plan) -> Tensor");
  m.def("forward_cached_plan(Tensor x_norm, Tensor weight, Tensor bias, Tensor mix_weight, "
        "Tensor mix_bias, int off, int T, int dilation, int cached_plan) -> Tensor");
  m.def("forward_warmup(Tensor x_norm, Tensor weight, Tensor bias, Tensor mix_weight, "
        "Tensor mix_bias, int off, int T, int dilation, int warmup_iters, int bench_iters) -> int");
  m.def("backward(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, Tensor mix_weight, "
        "Tensor mix_bias, int off, int T, int dilation) -> Tensor[]");
  m.def("backward_plan(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation, int plan, int tile_t) "
        "-> Tensor[]");
  m.def("backward_cached_plan(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation, int cached_plan) "
        "-> Tensor[]");
  m.def("backward_warmup(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation, int warmup_iters, "
        "int bench_iters) -> int");
  m.def("backward_pack_cached_plan(int plan, int tile_t) -> int");
  m.def("backward_cached_plan_get_plan(int cached_plan) -> int");
  m.def("backward_cached_plan_get_tile_t(int cached_plan) -> int");
  m.def("backward_atomic(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation) -> Tensor[]");
  m.def("backward_per_d_reduce(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation, int tile_t) -> Tensor[]");
  m.def("backward_gather_x(Tensor grad_out, Tensor x_norm, Tensor weight, Tensor bias, "
        "Tensor mix_weight, Tensor mix_bias, int off, int T, int dilation, int tile_t) -> Tensor[]");
}

TORCH_LIBRARY_IMPL(fused_source_conv_mixed, CUDA, m) {
  m.impl("forward", TORCH_FN(fscm_forward_op));
  m.impl("forward_plan", TORCH_FN(fscm_forward_plan_op));
  m.impl("forward_cached_plan", TORCH_FN(fscm_forward_cached_plan_op));
  m.impl("forward_warmup", TORCH_FN(fscm_forward_warmup_op));
  m.impl("backward", TORCH_FN(fscm_backward_op));
  m.impl("backward_plan", TORCH_FN(fscm_backward_plan_op));
  m.impl("backward_cached_plan", TORCH_FN(fscm_backward_cached_plan_op));
  m.impl("backward_warmup", TORCH_FN(fscm_backward_warmup_op));
  m.impl("backward_atomic", TORCH_FN(fscm_backward_atomic_op));
  m.impl("backward_per_d_reduce", TORCH_FN(fscm_backward_per_d_reduce_op));
  m.impl("backward_gather_x", TORCH_FN(fscm_backward_gather_x_op));
}

TORCH_LIBRARY_IMPL(fused_source_conv_mixed, CompositeExplicitAutograd, m) {
  m.impl("backward_pack_cached_plan", TORCH_FN(pack_plan));
  m.impl("backward_cached_plan_get_plan", TORCH_FN(unpack_plan));
  m.impl("backward_cached_plan_get_tile_t", TORCH_FN(unpack_tile));
}
