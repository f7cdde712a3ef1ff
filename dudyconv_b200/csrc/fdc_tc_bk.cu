// fdc_tc_bk.cu -- tcgen05/TMEM kernel for grad_kc and grad_mix of the dynamic conv.
//
//   G_kk[b,d,t]          = go[b,d,t] * h[b,d, off+t-kk*dil]        (built in smem)
//   grad_kc[b,kk,n,t]    = sum_d G_kk[b,d,t] * mix[d,n]            (per item, per tap)
//   grad_mix[d,n]        = sum_{b,kk,t} G_kk[b,d,t] * kc[b,kk,n,t] (TMEM-resident over
//                                                                    the CTA's items)
// (autograd of test_fused_dynamic_conv_against_reference.py:91-189; the reference
// materialises G in HBM and runs cuBLAS, cuda_ops/
// fused_dynamic_conv_backward_n_k3_d256_gemm_fp16_template.cuh:122-320.)
//
// Work item = (b, 128-token tile, tap kk). Per channel half h (128 channels) one G
// slot (128 ch x 128 tok, SWIZZLE_128B, rows = channel) and one G_lo slot of the same
// shape cycle through:
//   TMA producer: go[half h] tile -> G slot (same shape and swizzle as G);
//   8 builder warps: the exact products go * shifted h as two 16-bit terms
//   (split_mul8): G_hi over go in the G slot, G_lo into the G_lo slot; h fetched with
//   16-byte loads of two aligned chunks per output chunk (the causal shift is a funnel
//   shift), all of a thread's loads issued before the first use;
//   MMA warp (each contraction once with G_hi and once with G_lo, same accumulator, so
//   it sums the exact products in fp32):
//     grad_kc : acc_kc[128 tok x N]  += G^T (MN-major) * mix[half h]  (MN-major)
//     grad_mix: acc_gm[h][128 ch x N] += G (K-major)  * kc_kk (K-major)
//   acc_kc drains per tap through 4 epilogue warps (lane = token, coalesced stores);
//   acc_gm stays in TMEM until the CTA's last item, then goes out as an fp32 partial
//   that a fixed-order reduction kernel sums (deterministic grad_mix).
//
// Warp roles (512 threads): 0 TMA producer (mix once, kc per tap, L2 prefetch of the
// next item's go / h), 1 MMA issuer (+TMEM owner), 2 go-tile producer, 3 idle,
// 4-7 grad_kc epilogue, 8-15 G builders.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tile_util.cuh"

namespace dudy {
namespace tc {

using namespace sm100;

namespace bk {

constexpr int kTile = 128;
constexpr int kThreads = 512;
constexpr int kEpiWarp0 = 4, kNumEpiWarps = 4;
constexpr int kBuildWarp0 = 8, kNumBuildWarps = 8;
constexpr int kKcStages = 2, kGStages = 2;
constexpr uint32_t kGBytes = 2 * 128 * 128;  // one (tap, half) unit: 128 ch x 128 tok fp16
constexpr size_t kSmemBudget = 232448;

struct Args {
  const void *go;   // [B,D,T]
  const void *h;    // [B,D,L]
  void *grad_kc;    // [B,K,N,T]
  float *part;      // [gridDim.x][D][N] fp32 grad_mix partials
  int B, D, L, T, K, off, dil;
  int ntile;
  int dep_late;     // 1: wait for the previous kernel of the stream only before exiting
  int *err;
};

struct Layout {
  uint32_t mix, kc, g, glo, bar, total;
};

__host__ __device__ inline Layout layout(int D, int N) {
  Layout s;
  uint32_t o = 0;
  s.mix = o;
  o += D * N * 2;
  o = (o + 1023) & ~1023u;
  s.kc = o;
  o += kKcStages * N * 256;
  s.g = o;
  o += kGStages * kGBytes;
  s.glo = o;
  o += kGStages * kGBytes;
  s.bar = o;
  o += 256;
  s.total = o;
  return s;
}

__host__ __device__ inline int tmem_cols(int D, int N) {
  const int need = 2 * N + (D / 128) * N;
  int c = 32;
  while (c < need) c <<= 1;
  return c;
}

// mix as the MN-major B operand of grad_kc: rows = channels (the K dim), N contiguous
template <int NB>
struct MixMN {
  static constexpr int kRowBytes = NB >= 64 ? 128 : NB * 2;
  static constexpr uint32_t kLayout = NB >= 64 ? kSw128 : (NB == 32 ? kSw64 : kSw32);
  static constexpr int kBoxN = NB >= 64 ? 64 : NB;
  static constexpr int kBlocks = NB >= 64 ? NB / 64 : 1;
  // 16-channel k-step `row16` (counted from channel 0)
  __device__ static uint64_t desc(uint32_t base, int D, int row16) {
    const uint32_t lbo = (uint32_t)D * kRowBytes;  // stride between 64-wide basis blocks
    return make_sdesc(base + (uint32_t)row16 * 16u * kRowBytes, lbo, 8 * kRowBytes, kLayout);
  }
};

}  // namespace bk

// Teardown wait (ignores the abort flag); a timeout is recorded in the error word.
__device__ __forceinline__ bool bk_drain(uint64_t *bar, uint32_t parity, int *err,
                                         int site = 90) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      record_timeout(err, site, (int)parity);
      return false;
    }
  }
  return true;
}

template <typename T, int NB>
__global__ void __launch_bounds__(bk::kThreads, 1)
fdc_tc_bk_kernel(const __grid_constant__ CUtensorMap tm_kc,
                 const __grid_constant__ CUtensorMap tm_mix,
                 const __grid_constant__ CUtensorMap tm_go,
                 const __grid_constant__ CUtensorMap tm_h,
                 const __grid_constant__ CUtensorMap tm_go_tile, const bk::Args a) {
  using namespace bk;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array itself, so that the compiler keeps
  // every pointer below in the shared window (32-bit LDS/STS addressing, not generic)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const Layout Ly = layout(a.D, NB);
  uint8_t *mix_s = smem + Ly.mix;
  uint8_t *kc_s = smem + Ly.kc;
  uint8_t *g_s = smem + Ly.g;
  uint8_t *glo_s = smem + Ly.glo;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Ly.bar);
  uint64_t *kc_full = bars;        // [2]
  uint64_t *kc_empty = bars + 2;   // [2]
  uint64_t *g_full = bars + 4;     // [kGStages <= 3]
  uint64_t *g_empty = bars + 7;    // [kGStages <= 3]
  uint64_t *gk_full = bars + 10;   // [2]
  uint64_t *gk_empty = bars + 12;  // [2]
  uint64_t *mix_full = bars + 14;
  uint64_t *gm_done = bars + 15;
  uint32_t *tmem_hold = reinterpret_cast<uint32_t *>(bars + 16);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 17);
  volatile int *group_go = reinterpret_cast<volatile int *>(bars + 18);
  uint64_t *go_full = bars + 19;   // [kGStages <= 3] go tile landed in the G slot

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HD = a.D / 128;
  // work item = (b, 128-token tile, tap), tap fastest: the CTAs that run the three taps of
  // one tile at the same time share its go / h reads through L2
  const int items = a.B * a.ntile * a.K;
  constexpr uint32_t kKcStageBytes = NB * 256;
  const int ncols = tmem_cols(a.D, NB);

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kc_full[i], 1);
      mbar_init(&kc_empty[i], 1);
      mbar_init(&gk_full[i], 1);
      mbar_init(&gk_empty[i], kNumEpiWarps);
    }
    for (int i = 0; i < kGStages; ++i) {
      mbar_init(&g_full[i], 1);
      mbar_init(&g_empty[i], 1);
      mbar_init(&go_full[i], 1);
    }
    mbar_init(mix_full, 1);
    mbar_init(gm_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_hold, ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_hold;
  // inputs may come from the previous kernel of the stream (programmatic launch); with
  // dep_late (as in fdc_tc_bk_n128_kernel) the kernel starts at once and waits for the
  // previous kernel only before it exits
  if (!a.dep_late) pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();
  const uint32_t gk_col0 = 0, gm_col0 = 2 * NB;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tensormap(&tm_kc);
      prefetch_tensormap(&tm_mix);
      using MM = MixMN<NB>;
      mbar_arrive_expect_tx(mix_full, a.D * NB * 2);
      for (int blk = 0; blk < MM::kBlocks; ++blk)
        for (int hh = 0; hh < HD; ++hh)
          tma_load_2d(mix_s + (blk * a.D + hh * 128) * MM::kRowBytes, &tm_mix, mix_full,
                      blk * 64, hh * 128);
      int q = 0;
      int last_par[kKcStages] = {-1, -1};
      bool ok = true;
      // L2 prefetch of the go / h tiles of the CTA's next item
      auto prefetch_item = [&](int it2) {
        if (it2 >= items) return;
        const int b2 = it2 / (a.ntile * a.K), t2 = ((it2 / a.K) % a.ntile) * kTile;
        const int hx = (a.off + t2 - (a.K - 1) * a.dil) & ~7;
        for (int hh = 0; hh < HD; ++hh) {
          tma_prefetch_2d(&tm_go, t2, b2 * a.D + hh * 128);
          tma_prefetch_2d(&tm_h, hx, b2 * a.D + hh * 128);
        }
      };
      prefetch_tensormap(&tm_go);
      prefetch_tensormap(&tm_h);
      prefetch_item(blockIdx.x);
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
        const int b = it / (a.ntile * a.K);
        const int t0 = ((it / a.K) % a.ntile) * kTile;
        const int kk = it % a.K;
        prefetch_item(it + gridDim.x);
        const int st = q % kKcStages;
        if (!mbar_wait(&kc_empty[st], ((q / kKcStages) & 1) ^ 1, a.err, abort_flag, 60, q)) { ok = false; break; }
        uint8_t *dst = kc_s + st * kKcStageBytes;
        mbar_arrive_expect_tx(&kc_full[st], kKcStageBytes);
        const int row = (b * a.K + kk) * NB;
        tma_load_2d(dst, &tm_kc, &kc_full[st], t0, row);
        tma_load_2d(dst + NB * 128, &tm_kc, &kc_full[st], t0 + 64, row);
        last_par[st] = (q / kKcStages) & 1;
      }
      for (int st = 0; st < kKcStages; ++st)
        if (last_par[st] >= 0) bk_drain(&kc_full[st], last_par[st], a.err);
      bk_drain(mix_full, 0, a.err);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ go-tile producer
    // Fills the G slots with the go half-tile each (tap, half) unit starts from; kept
    // apart from the kc ring so neither queue waits behind the other.
    if (lane == 0) {
      prefetch_tensormap(&tm_go_tile);
      int gu = 0, last_go_par[kGStages];
      for (int i = 0; i < kGStages; ++i) last_go_par[i] = -1;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int b = it / (a.ntile * a.K);
        const int t0 = ((it / a.K) % a.ntile) * kTile;
        for (int hh = 0; hh < HD; ++hh, ++gu) {
          const int gs = gu % kGStages;
          if (!mbar_wait(&g_empty[gs], ((gu / kGStages) & 1) ^ 1, a.err, abort_flag, 61, gu)) { ok = false; break; }
          uint8_t *gdst = g_s + gs * kGBytes;
          mbar_arrive_expect_tx(&go_full[gs], kGBytes);
          tma_load_2d(gdst, &tm_go_tile, &go_full[gs], t0, b * a.D + hh * 128);
          tma_load_2d(gdst + 16384, &tm_go_tile, &go_full[gs], t0 + 64, b * a.D + hh * 128);
          last_go_par[gs] = (gu / kGStages) & 1;
        }
      }
      for (int gs = 0; gs < kGStages; ++gs)
        if (last_go_par[gs] >= 0) bk_drain(&go_full[gs], last_go_par[gs], a.err, 91);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      using MM = MixMN<NB>;
      constexpr uint32_t idesc_kc = make_idesc_f16(128, NB, IsBf16<T>::value, 1, 1);
      constexpr uint32_t idesc_gm = make_idesc_f16(128, NB, IsBf16<T>::value, 0, 0);
      const uint32_t mix_base = smem_u32(mix_s), kc_base = smem_u32(kc_s), g_base = smem_u32(g_s);
      const uint32_t l_base = smem_u32(glo_s);
      bool ok = mbar_wait(mix_full, 0, a.err, abort_flag, 70, 0);
      bool first_gm[2] = {true, true};
      int q = 0, gu = 0;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
        {
          const int st = q % kKcStages, slot = q & 1;
          if (!mbar_wait(&kc_full[st], (q / kKcStages) & 1, a.err, abort_flag, 71, q) ||
              !mbar_wait(&gk_empty[slot], ((q >> 1) & 1) ^ 1, a.err, abort_flag, 72, q)) {
            ok = false;
            break;
          }
          const uint32_t kcb = kc_base + st * kKcStageBytes;
          for (int hh = 0; hh < HD; ++hh, ++gu) {
            const int gs = gu % kGStages;
            if (!mbar_wait(&g_full[gs], (gu / kGStages) & 1, a.err, abort_flag, 73, gu)) { ok = false; break; }
            tc_fence_after();
            const uint32_t gb = g_base + gs * kGBytes;  // G_hi
            const uint32_t lb = l_base + gs * kGBytes;  // G_lo
            // grad_kc: M = tokens, K = channels of this half
#pragma unroll
            for (int ks = 0; ks < 16; ++ks) {
              const uint64_t ad = make_sdesc((ks < 8 ? gb : lb) + (ks & 7) * 2048, 16384, 1024, kSw128);
              const uint64_t bd = MM::desc(mix_base, a.D, hh * 8 + (ks & 7));
              umma_f16(tmem + gk_col0 + slot * NB, ad, bd, idesc_kc, (hh > 0 || ks > 0) ? 1u : 0u);
            }
            // grad_mix: M = channels of this half, K = tokens
#pragma unroll
            for (int ks = 0; ks < 16; ++ks) {
              const int k8 = ks & 7;
              const uint64_t ad = make_sdesc((ks < 8 ? gb : lb) + (k8 >> 2) * 16384 + (k8 & 3) * 32,
                                             16, 1024, kSw128);
              const uint64_t bd = make_sdesc(kcb + (k8 >> 2) * (NB * 128) + (k8 & 3) * 32, 16, 1024, kSw128);
              umma_f16(tmem + gm_col0 + hh * NB, ad, bd, idesc_gm,
                       (first_gm[hh] && ks == 0) ? 0u : 1u);
            }
            first_gm[hh] = false;
            umma_commit(&g_empty[gs]);
          }
          if (!ok) break;
          umma_commit(&kc_empty[st]);
          umma_commit(&gk_full[slot]);
        }
      }
      umma_commit(gm_done);
      bk_drain(gm_done, 0, a.err);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kNumEpiWarps) {
    // ------------------------------------------------------------ grad_kc epilogue
    const int qd = warp & 3;
    const int tl = qd * 32 + lane;
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    T *gkc = reinterpret_cast<T *>(a.grad_kc);
    int q = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
      const int b = it / (a.ntile * a.K);
      const int t = ((it / a.K) % a.ntile) * kTile + tl;
      const int kk = it % a.K;
      {
        const int slot = q & 1;
        if (!mbar_wait_warp(&gk_full[slot], (q >> 1) & 1, a.err, abort_flag, 80, q)) { ok = false; break; }
        tc_fence_after();
        T *dst = gkc + ((size_t)(b * a.K + kk) * NB) * a.T + t;
#pragma unroll
        for (int c = 0; c < NB / 16; ++c) {
          float v[16];
          tmem_ld16(lane_addr + gk_col0 + slot * NB + c * 16, v);
          if (t < a.T) {
#pragma unroll
            for (int i = 0; i < 16; ++i) dst[(size_t)(c * 16 + i) * a.T] = Elem<T>::from_f(v[i]);
          }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&gk_empty[slot]);
      }
    }
    // grad_mix partial of this CTA: TMEM lane = channel within the half. A CTA without work
    // items (the grid is even and at least 2, so a one-item shape has one) never wrote its
    // grad_mix accumulator and contributes zeros.
    const bool gm_ok = bk_drain(gm_done, 0, a.err) && !*abort_flag;
    if (__all_sync(0xffffffffu, gm_ok)) {
      tc_fence_after();
      const bool any = (int)blockIdx.x < items;
      for (int hh = 0; hh < HD; ++hh) {
        float *dst = a.part + ((size_t)blockIdx.x * a.D + hh * 128 + tl) * NB;
#pragma unroll
        for (int c = 0; c < NB / 16; ++c) {
          float v[16];
          tmem_ld16(lane_addr + gm_col0 + hh * NB + c * 16, v);
#pragma unroll
          for (int i = 0; i < 16; i += 4)
            *reinterpret_cast<float4 *>(dst + c * 16 + i) =
                any ? make_float4(v[i], v[i + 1], v[i + 2], v[i + 3])
                    : make_float4(0.f, 0.f, 0.f, 0.f);
        }
      }
    }
  } else if (warp >= kBuildWarp0 && warp < kBuildWarp0 + kNumBuildWarps) {
    // ------------------------------------------------------------ G builders
    // G slot holds go (TMA); each thread turns its 8 chunks into G = go * h(shifted) in
    // place. All h loads of a thread are issued before the first use.
    const int bid = threadIdx.x - kBuildWarp0 * 32;  // 0..255
    const T *hp = reinterpret_cast<const T *>(a.h);
    constexpr int kPer = 128 * 16 / 256;  // chunks per thread per unit
    int gu = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const int b = it / (a.ntile * a.K);
      const int t0 = ((it / a.K) % a.ntile) * kTile;
      const int kk = it % a.K;
      {
        const int sh = (a.off - kk * a.dil) & 7;
        for (int hh = 0; hh < HD; ++hh, ++gu) {
          const int gs = gu % kGStages;
          // issue this unit's h loads before waiting for the go tile
          uint4 q0[kPer], q1[kPer];
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int idx = bid + 256 * i;
            const int r = idx >> 4, j = (idx >> 3) & 1, c = idx & 7;
            const int t = t0 + j * 64 + c * 8;
            const T *hrow = hp + ((size_t)b * a.D + hh * 128 + r) * a.L;
            const int pa = a.off + t - kk * a.dil - sh;
            q0[i] = make_uint4(0, 0, 0, 0);
            q1[i] = make_uint4(0, 0, 0, 0);
            if (t < a.T && pa >= 0 && pa + 8 <= a.L)
              q0[i] = __ldg(reinterpret_cast<const uint4 *>(hrow + pa));
            if (t < a.T && sh != 0 && pa + 8 >= 0 && pa + 16 <= a.L)
              q1[i] = __ldg(reinterpret_cast<const uint4 *>(hrow + pa + 8));
          }
          // one thread waits; the decision is broadcast through shared memory so the
          // whole group takes the same branch at the named barriers
          if (bid == 0)
            *group_go = (mbar_wait(&go_full[gs], (gu / kGStages) & 1, a.err, abort_flag, 85, gu) &&
                         !*abort_flag) ? 1 : 0;
          asm volatile("bar.sync 2, 256;" ::: "memory");
          if (!*group_go) { ok = false; break; }
          uint8_t *slot = g_s + gs * kGBytes;
          uint8_t *lslot = glo_s + gs * kGBytes;
#pragma unroll
          for (int i = 0; i < kPer; ++i) {
            const int idx = bid + 256 * i;
            const int r = idx >> 4, j = (idx >> 3) & 1, c = idx & 7;
            const uint32_t o = j * 16384 + sw128_off(r, c);
            uint4 *gp = reinterpret_cast<uint4 *>(slot + o);
            uint4 hi, lo;
            split_mul8<T>(*gp, shift8(q0[i], q1[i], sh), hi, lo);
            *gp = hi;
            *reinterpret_cast<uint4 *>(lslot + o) = lo;
          }
          fence_proxy_async_smem();
          asm volatile("bar.sync 2, 256;" ::: "memory");
          if (bid == 0) mbar_arrive(&g_full[gs]);
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, ncols);
  }
  if (a.dep_late) pdl_wait();
}

// grad_mix = sum over the CTAs' fp32 partials, in a fixed order (deterministic).
// Block = 64 x 16 threads over 256 consecutive elements: thread (x, y) sums partials
// y, y+16, ... of elements 4x..4x+3 with float4 loads, then row 0 adds the 16 row sums
// in order. Many independent 16-byte loads in flight keep this L2-bandwidth bound.
template <typename T>
__global__ void __launch_bounds__(1024)
fdc_tc_mix_reduce_kernel(const float *__restrict__ part, T *__restrict__ out, int64_t DN,
                         int nparts) {
  __shared__ float4 red[16][64];
  const int tx = threadIdx.x, ty = threadIdx.y;
  pdl_wait();  // the partials are written by the kernel launched just before
  if (tx == 0 && ty == 0) pdl_trigger();
  const int64_t e = ((int64_t)blockIdx.x * 64 + tx) * 4;
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  if (e < DN) {
    int p = ty;
    for (; p + 48 < nparts; p += 64) {
      float4 v[4];
#pragma unroll
      for (int j = 0; j < 4; ++j)
        v[j] = __ldg(reinterpret_cast<const float4 *>(part + (int64_t)(p + 16 * j) * DN + e));
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc.x += v[j].x; acc.y += v[j].y; acc.z += v[j].z; acc.w += v[j].w;
      }
    }
    for (; p < nparts; p += 16) {
      const float4 v = __ldg(reinterpret_cast<const float4 *>(part + (int64_t)p * DN + e));
      acc.x += v.x; acc.y += v.y; acc.z += v.z; acc.w += v.w;
    }
  }
  red[ty][tx] = acc;
  __syncthreads();
  if (ty == 0 && e < DN) {
    float4 s = red[0][tx];
#pragma unroll
    for (int r = 1; r < 16; ++r) {
      s.x += red[r][tx].x; s.y += red[r][tx].y; s.z += red[r][tx].z; s.w += red[r][tx].w;
    }
    stf(out + e, s.x);
    stf(out + e + 1, s.y);
    stf(out + e + 2, s.z);
    stf(out + e + 3, s.w);
  }
}

}  // namespace tc
}  // namespace dudy

// =====================================================================================
// host launcher
// =====================================================================================
#include "tma_host.h"

namespace dudy {
namespace tc {

namespace {

struct BkMaps {
  CUtensorMap kc, mix, go, h, go_tile;
};

template <typename T, int NB>
int launch_bk(const BkMaps &m, const bk::Args &a, int grid, size_t smem, cudaStream_t st) {
  auto kern = fdc_tc_bk_kernel<T, NB>;
  if (set_smem_once((const void *)kern, (int)smem) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fdc_tc_bk_kernel)");
  if (launch_pdl(kern, dim3(grid), dim3(bk::kThreads), smem, st, m.kc, m.mix, m.go, m.h,
                 m.go_tile, a) != cudaSuccess)
    return check_launch("fdc_tc_bk_kernel");
  return DUDY_OK;
}

template <typename T>
int bk_dispatch(int N, const BkMaps &m, const bk::Args &a, int grid, size_t smem,
                cudaStream_t st) {
  switch (N) {
    case 16: return launch_bk<T, 16>(m, a, grid, smem, st);
    case 32: return launch_bk<T, 32>(m, a, grid, smem, st);
    case 64: return launch_bk<T, 64>(m, a, grid, smem, st);
    default:  // N = 128 runs fdc_tc_bk_n128_kernel (bk_launch dispatches it first)
      set_error("fdc_tc_bk_kernel: unsupported basis size");
      return DUDY_ERR_UNSUPPORTED;
  }
}

int bk_grid(const FdcShape &s) {
  const int64_t items = s.B * cdiv(s.T, bk::kTile) * s.K;
  int g = sm_count();
  if (g > items) g = (int)items;
  g &= ~1;  // the N = 128 kernel launches clusters of 2
  return g < 2 ? 2 : g;
}

}  // namespace

bool bk128_supported(const FdcShape &s, int dtype);

bool bk_supported(const FdcShape &s, int dtype) {
  if (bk128_supported(s, dtype)) return true;
  if (dtype != DUDY_DTYPE_F16 && dtype != DUDY_DTYPE_BF16) return false;
  if (!(s.D == 128 || s.D == 256)) return false;
  if (!(s.N == 16 || s.N == 32 || s.N == 64 || s.N == 128)) return false;
  if (s.T % 8 != 0 || s.L % 8 != 0) return false;
  if (bk::tmem_cols((int)s.D, (int)s.N) > 512) return false;
  return bk::layout((int)s.D, (int)s.N).total + 1024 <= bk::kSmemBudget;
}

size_t bk_workspace(const FdcShape &s) {
  return (size_t)bk_grid(s) * (size_t)(s.D * s.N) * sizeof(float);
}

int bk128_launch(const void *go, const void *h, const void *kc, const void *mix, void *grad_kc,
                 float *part, const FdcShape &s, int dtype, int grid, bool dep_late, int *err,
                 cudaStream_t st);

static int bk_reduce(const void *ws, void *grad_mix, const FdcShape &s, bool bf16, int nparts,
                     const XRank *xr, int *err, cudaStream_t st) {
  const int64_t DN = s.D * s.N;
  if (xr)
    return xrank_reduce_launch((const float *)ws, nparts, grad_mix, DN,
                               bf16 ? DUDY_DTYPE_BF16 : DUDY_DTYPE_F16, *xr, err, st);
  const dim3 grid((unsigned)cdiv(DN, 256)), block(64, 16);
  const cudaError_t e =
      bf16 ? launch_pdl(fdc_tc_mix_reduce_kernel<__nv_bfloat16>, grid, block, 0, st,
                        (const float *)ws, (__nv_bfloat16 *)grad_mix, DN, nparts)
           : launch_pdl(fdc_tc_mix_reduce_kernel<__half>, grid, block, 0, st, (const float *)ws,
                        (__half *)grad_mix, DN, nparts);
  if (e != cudaSuccess) return check_launch("fdc_tc_mix_reduce_kernel");
  return DUDY_OK;
}

// dep_late: the kernel launched just before on this stream belongs to the same backward
// call and reads nothing this one writes; its inputs were complete before it started (it
// waited for its own predecessor before triggering), so this kernel need not wait for it
// to start, only before it exits.
int bk_launch(const void *go, const void *h, const void *kc, const void *mix, void *grad_kc,
              void *grad_mix, void *ws, const FdcShape &s, int dtype, bool dep_late, int *err,
              const XRank *xr, cudaStream_t st) {
  const bool bf16 = dtype == DUDY_DTYPE_BF16;
  if (bk128_supported(s, dtype)) {
    const int grid = bk_grid(s);
    const int rc =
        bk128_launch(go, h, kc, mix, grad_kc, (float *)ws, s, dtype, grid, dep_late, err, st);
    return rc ? rc : bk_reduce(ws, grad_mix, s, bf16, grid, xr, err, st);
  }
  const int N = (int)s.N, D = (int)s.D, T = (int)s.T, K = (int)s.K;
  bk::Args a{};
  a.go = go;
  a.h = h;
  a.grad_kc = grad_kc;
  a.part = (float *)ws;
  a.B = (int)s.B; a.D = D; a.L = (int)s.L; a.T = T; a.K = K;
  a.off = (int)s.off; a.dil = (int)s.dil;
  a.ntile = (int)cdiv(T, bk::kTile);
  a.dep_late = dep_late ? 1 : 0;
  a.err = err;
  const int grid = bk_grid(s);
  const size_t smem = bk::layout(D, N).total + 1024;
  BkMaps m;
  const int mix_box = N >= 64 ? 64 : N;
  const int mix_sw = N >= 64 ? 128 : 2 * N;
  const int hH = (K - 1) * (int)s.dil;
  const uint32_t hbox = (uint32_t)((bk::kTile + hH + 7 + 7) & ~7);
  if (!make_tmap_2d(&m.kc, kc, bf16, (uint64_t)T, (uint64_t)(s.B * K * N), (uint64_t)T * 2, 64,
                    (uint32_t)N, 128) ||
      !make_tmap_2d(&m.mix, mix, bf16, (uint64_t)N, (uint64_t)D, (uint64_t)N * 2,
                    (uint32_t)mix_box, 128u, mix_sw) ||
      !make_tmap_2d(&m.go, go, bf16, (uint64_t)T, (uint64_t)(s.B * D), (uint64_t)T * 2,
                    (uint32_t)bk::kTile, 128u, 0) ||
      !make_tmap_2d(&m.h, h, bf16, (uint64_t)s.L, (uint64_t)(s.B * D), (uint64_t)s.L * 2,
                    hbox > 256 ? 256u : hbox, 128u, 0) ||
      !make_tmap_2d(&m.go_tile, go, bf16, (uint64_t)T, (uint64_t)(s.B * D), (uint64_t)T * 2, 64,
                    128u, 128))
    return DUDY_ERR_CUDA;
  int rc = bf16 ? bk_dispatch<__nv_bfloat16>(N, m, a, grid, smem, st)
                : bk_dispatch<__half>(N, m, a, grid, smem, st);
  return rc ? rc : bk_reduce(ws, grad_mix, s, bf16, grid, xr, err, st);
}

}  // namespace tc
}  // namespace dudy
