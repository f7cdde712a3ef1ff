// fdc_tc_conv2.cu -- tcgen05/TMEM kernel for the dynamic-conv forward and for grad_h when
// D is 128 or 256: one CTA per work item covers every channel, so each kc tile crosses
// from L2 into shared memory once (the per-half kernel in fdc_tc_conv.cu reads it once per
// 128-channel half; on B200 the L2 -> SM path is barely faster than HBM, so that second
// read costs nearly as much as a DRAM read).
//
//   forward : out[b,d,u]    = sum_kk W_kk[d,u]        * h[b,d, off+u-kk*dil]
//             (reference: cuda_ops/fused_dynamic_conv_forward_direct_exec.cu:26-75)
//   grad_h  : gh[b,d,off+u] = sum_kk W_kk[d,u+kk*dil] * go[b,d, u+kk*dil]
//             (autograd of test_fused_dynamic_conv_against_reference.py:91-189)
//   with W_kk[d,v] = sum_n mix[d,n] * kc[b,kk,n,v] computed on the tensor cores.
//
// Work item = (b, 120-token output tile). The CTA runs the channel halves of an item one
// after the other; per half hh and tap kk one MMA chain
//     W^T[128 ch x 128 tok] (TMEM) = mix_hh[128 ch x N] (A, resident in TMEM)
//                                    * kc_kk[N x 128 tok] (B, MN-major SWIZZLE_128B, TMA)
// so the item's K kc tiles stay in shared memory until the last half has used them.
// TMEM lane = channel, column = token. The kc tile starts at the 8-aligned token at or
// before the tap's first token, so grad_h's causal shift (kk*dil) becomes a per-tap column
// offset sh < 8 that the epilogue applies when it reads TMEM; 120 + 7 < 128 keeps every
// needed column inside the tile.
//
// Epilogue: 16 warps; warp (quadrant qd, range g) owns channels 32*qd.. of the current
// half and output tokens [32g, 32g+32) of the tile (the last range has 24). It keeps the
// sum over taps in registers, reads its factor row (h or go) from the staged window with
// 16-byte loads, rounds the sum into a staging tile and one thread TMA-stores the tile.
//
// Warp roles (608 threads): 0 TMA producer (lane 0: kc stages, lane 1: factor windows),
// 1 MMA issuer (+TMEM owner), 2-17 epilogue (+ mix into TMEM at start), 18 output TMA
// stores. Every wait is bounded.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tile_util.cuh"

namespace dudy {
namespace tc {

using namespace sm100;

namespace cv2 {

constexpr int kTileOut = 120;                 // output tokens per item
constexpr int kTileMma = 128;                 // tokens per MMA tile (TMEM columns)
constexpr int kEpiWarp0 = 2, kNumEpiWarps = 16;
constexpr int kStoreWarp = kEpiWarp0 + kNumEpiWarps;  // issues the output TMA stores
constexpr int kThreads = 32 * (kStoreWarp + 1);
constexpr int kWSlots = 3;                    // W slots of 128 TMEM columns after the mix
constexpr uint32_t kWCol0 = 128;
constexpr int kMaxKcStages = 8, kMaxFacStages = 4;
constexpr size_t kSmemBudget = 232448;
constexpr uint32_t kOutPitch = kTileOut * 2;  // staged output rows: 240 bytes

struct Args {
  const void *mix;  // [D,N]
  int B, D, L, T, N, K, off, dil;
  int u_first;      // token coordinate of tile 0 (grad_h: off + u_first is 8-aligned)
  int ntile;
  int kc_stages, fac_stages, fac_w;
  int split;        // 1: a work item is (b, tile, half); 0: (b, tile) with every half
  int dep_late;     // 1: wait for the previous kernel of the stream only before exiting
  int *err;
};

// Work item `it` -> batch, first output token and the range of channel halves it covers.
struct Item {
  int b, u0, h_lo, h_hi;
};

// Work items run from the end of the batch to its start: the kernels next to this one on
// the stream (the forward before it, the grad_kc/grad_mix kernel after it) sweep the batch
// forwards, so each finds the tiles the other touched last still in L2.
__device__ __forceinline__ Item item_of(const Args &a, int it, int HD) {
  Item x;
  it = a.B * a.ntile * (a.split ? HD : 1) - 1 - it;
  if (a.split) {
    x.b = it / (a.ntile * HD);
    x.u0 = a.u_first + ((it / HD) % a.ntile) * kTileOut;
    x.h_lo = it % HD;
    x.h_hi = x.h_lo + 1;
  } else {
    x.b = it / a.ntile;
    x.u0 = a.u_first + (it % a.ntile) * kTileOut;
    x.h_lo = 0;
    x.h_hi = HD;
  }
  return x;
}

struct Layout {
  uint32_t kc, fac, stg, bar, total;
};

__host__ __device__ inline Layout layout(int N, int kc_stages, int fac_stages, int fac_w) {
  Layout s;
  s.kc = 0;
  s.fac = (uint32_t)kc_stages * (uint32_t)N * 256u;
  s.stg = s.fac + (uint32_t)fac_stages * 128u * (uint32_t)fac_w * 2u;
  s.bar = s.stg + 128u * kOutPitch;
  s.total = s.bar + 512;
  return s;
}

}  // namespace cv2

__device__ __forceinline__ bool cv2_drain(uint64_t *bar, uint32_t parity, int *err, int site) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      record_timeout(err, site, (int)parity);
      return false;
    }
  }
  return true;
}

// 32 lanes x 8 consecutive 32-bit TMEM columns, load and wait in one statement
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, float (&v)[8]) {
  uint32_t r[8];
  asm volatile(
      "{\n tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
      " tcgen05.wait::ld.sync.aligned;\n}"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 8; ++i) v[i] = __uint_as_float(r[i]);
}

// acc[0..8) += W[c0 + sh + i] * f[i], W read from the 16 TMEM columns [c0, c0 + 16)
// (c0 8-aligned, sh warp-uniform in 0..7)
template <typename T>
__device__ __forceinline__ void fma_piece(float *acc, uint32_t taddr, int sh, uint4 f8) {
  float w[16];
  {
    float lo[8], hi[8];
    tmem_ld8(taddr, lo);
    if (sh != 0) {
      tmem_ld8(taddr + 8, hi);
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) hi[i] = 0.f;
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      w[i] = lo[i];
      w[i + 8] = hi[i];
    }
  }
  const T *f = reinterpret_cast<const T *>(&f8);
#define DUDY_FMA_CASE(S)                                                       \
  case S:                                                                      \
    _Pragma("unroll") for (int i = 0; i < 8; ++i) acc[i] =                     \
        fmaf(w[i + S], Elem<T>::to_f(f[i]), acc[i]);                           \
    break;
  switch (sh) {
    DUDY_FMA_CASE(0)
    DUDY_FMA_CASE(1)
    DUDY_FMA_CASE(2)
    DUDY_FMA_CASE(3)
    DUDY_FMA_CASE(4)
    DUDY_FMA_CASE(5)
    DUDY_FMA_CASE(6)
    default:
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = fmaf(w[i + 7], Elem<T>::to_f(f[i]), acc[i]);
      break;
  }
#undef DUDY_FMA_CASE
}

// acc[0..16) += W[c0 + sh + i] * f[i]; W read from TMEM columns [c0, c0 + 16) and, when
// sh > 0, [c0 + 16, c0 + 24)
template <typename T>
__device__ __forceinline__ void fma_piece16(float *acc, uint32_t taddr, int sh, uint4 fa,
                                            uint4 fb) {
  float w[24];
  {
    float v[16];
    tmem_ld16(taddr, v);
#pragma unroll
    for (int i = 0; i < 16; ++i) w[i] = v[i];
  }
  if (sh != 0) {
    float v[8];
    tmem_ld8(taddr + 16, v);
#pragma unroll
    for (int i = 0; i < 8; ++i) w[16 + i] = v[i];
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) w[16 + i] = 0.f;
  }
  const T *f = reinterpret_cast<const T *>(&fa);
  const T *f2 = reinterpret_cast<const T *>(&fb);
#define DUDY_FMA16_CASE(S)                                                                 \
  case S:                                                                                  \
    _Pragma("unroll") for (int i = 0; i < 8; ++i) {                                        \
      acc[i] = fmaf(w[i + S], Elem<T>::to_f(f[i]), acc[i]);                               \
      acc[8 + i] = fmaf(w[8 + i + S], Elem<T>::to_f(f2[i]), acc[8 + i]);                  \
    }                                                                                      \
    break;
  switch (sh) {
    DUDY_FMA16_CASE(0)
    DUDY_FMA16_CASE(1)
    DUDY_FMA16_CASE(2)
    DUDY_FMA16_CASE(3)
    DUDY_FMA16_CASE(4)
    DUDY_FMA16_CASE(5)
    DUDY_FMA16_CASE(6)
    default:
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        acc[i] = fmaf(w[i + 7], Elem<T>::to_f(f[i]), acc[i]);
        acc[8 + i] = fmaf(w[15 + i], Elem<T>::to_f(f2[i]), acc[8 + i]);
      }
      break;
  }
#undef DUDY_FMA16_CASE
}

template <typename T, int NB, bool GH>
__global__ void __launch_bounds__(cv2::kThreads, 1)
fdc_tc_conv2_kernel(const __grid_constant__ CUtensorMap tm_kc,
                    const __grid_constant__ CUtensorMap tm_fac,
                    const __grid_constant__ CUtensorMap tm_y, const cv2::Args a) {
  using namespace cv2;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array itself, so that the compiler keeps
  // every pointer below in the shared window (32-bit LDS/STS addressing, not generic)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const Layout Ly = layout(NB, a.kc_stages, a.fac_stages, a.fac_w);
  uint8_t *kc_s = smem + Ly.kc;
  uint8_t *fac_s = smem + Ly.fac;
  uint8_t *stg_s = smem + Ly.stg;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + Ly.bar);
  uint64_t *kc_full = bars;          // [8]
  uint64_t *kc_empty = bars + 8;     // [8]
  uint64_t *fac_full = bars + 16;    // [4]
  uint64_t *fac_empty = bars + 20;   // [4]
  uint64_t *w_full = bars + 24;      // [3]
  uint64_t *w_empty = bars + 27;     // [3]
  uint64_t *mix_ready = bars + 30;
  uint64_t *mma_done = bars + 31;
  uint32_t *tmem_hold = reinterpret_cast<uint32_t *>(bars + 32);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 33);
  uint64_t *stg_full = bars + 34;    // the 16 epilogue warps wrote the staging tile
  uint64_t *stg_empty = bars + 35;   // its TMA store has read it

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HD = a.D / 128;
  const int items = a.B * a.ntile * (a.split ? HD : 1);
  const int S = a.kc_stages, F = a.fac_stages;
  constexpr uint32_t kKcStageBytes = NB * 256;
  const uint32_t fac_bytes = 128u * (uint32_t)a.fac_w * 2u;
  const int hH = (a.K - 1) * a.dil;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kMaxKcStages; ++i) {
      mbar_init(&kc_full[i], 1);
      mbar_init(&kc_empty[i], 1);
    }
    for (int i = 0; i < kMaxFacStages; ++i) {
      mbar_init(&fac_full[i], 1);
      mbar_init(&fac_empty[i], kNumEpiWarps);
    }
    mbar_init(stg_full, kNumEpiWarps);
    mbar_init(stg_empty, 1);
    for (int i = 0; i < kWSlots; ++i) {
      mbar_init(&w_full[i], 1);
      mbar_init(&w_empty[i], kNumEpiWarps);
    }
    mbar_init(mix_ready, 4 * HD);
    mbar_init(mma_done, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_hold, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_hold;
  // inputs may come from the previous kernel of the stream (programmatic launch); with
  // dep_late that kernel is the grad_h zero fill, which writes a disjoint part of y and
  // triggered after its own wait: start at once and wait for it only before exiting
  if (!a.dep_late) pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == 0) {
    if (lane == 0) {
      // ---------------------------------------------------------- kc-stage producer
      prefetch_tensormap(&tm_kc);
      int q = 0, last_par[kMaxKcStages];
      for (int i = 0; i < kMaxKcStages; ++i) last_par[i] = -1;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const Item I = item_of(a, it, HD);
        const int b = I.b, u0 = I.u0;
        for (int kk = 0; kk < a.K; ++kk, ++q) {
          const int st = q % S;
          if (!mbar_wait(&kc_empty[st], ((q / S) & 1) ^ 1, a.err, abort_flag, 110, q)) { ok = false; break; }
          const int tx = GH ? u0 + kk * a.dil : u0;
          const int x0 = tx - (tx & 7);
          uint8_t *dst = kc_s + st * kKcStageBytes;
          const int row = (b * a.K + kk) * NB;
          mbar_arrive_expect_tx(&kc_full[st], kKcStageBytes);
          tma_load_2d(dst, &tm_kc, &kc_full[st], x0, row);
          tma_load_2d(dst + NB * 128, &tm_kc, &kc_full[st], x0 + 64, row);
          last_par[st] = (q / S) & 1;
        }
      }
      for (int st = 0; st < S; ++st)
        if (last_par[st] >= 0) cv2_drain(&kc_full[st], last_par[st], a.err, 150);
    } else if (lane == 1) {
      // ---------------------------------------------------------- factor-window producer
      // One window per (item, half): h[off+u0-hH ..] (forward) or go[u0 ..] (grad_h),
      // 8-aligned start, fac_w tokens, 128 channel rows.
      prefetch_tensormap(&tm_fac);
      int f = 0, last_par[kMaxFacStages] = {-1, -1, -1, -1};
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const Item I = item_of(a, it, HD);
        const int b = I.b, u0 = I.u0;
        const int fs0 = GH ? u0 : a.off + u0 - hH;
        const int fx = fs0 - (fs0 & 7);
        for (int hh = I.h_lo; hh < I.h_hi; ++hh, ++f) {
          const int fs = f % F;
          if (!mbar_wait(&fac_empty[fs], ((f / F) & 1) ^ 1, a.err, abort_flag, 111, f)) { ok = false; break; }
          mbar_arrive_expect_tx(&fac_full[fs], fac_bytes);
          tma_load_2d(fac_s + fs * fac_bytes, &tm_fac, &fac_full[fs], fx, b * a.D + hh * 128);
          last_par[fs] = (f / F) & 1;
        }
      }
      for (int fs = 0; fs < F; ++fs)
        if (last_par[fs] >= 0) cv2_drain(&fac_full[fs], last_par[fs], a.err, 151);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(128, kTileMma, IsBf16<T>::value, 0, 1);
      const uint32_t kc_base = smem_u32(kc_s);
      bool ok = mbar_wait(mix_ready, 0, a.err, abort_flag, 120, 0);
      tc_fence_after();
      int q0 = 0, w = 0;   // q0: (item, tap) counter of the item's first tap
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, q0 += a.K) {
        const Item I = item_of(a, it, HD);
        for (int hh = I.h_lo; hh < I.h_hi && ok; ++hh) {
          for (int kk = 0; kk < a.K; ++kk, ++w) {
            const int q = q0 + kk;
            const int st = q % S;
            if (hh == I.h_lo && !mbar_wait(&kc_full[st], (q / S) & 1, a.err, abort_flag, 121, q)) { ok = false; break; }
            const int slot = w % kWSlots;
            if (!mbar_wait(&w_empty[slot], ((w / kWSlots) & 1) ^ 1, a.err, abort_flag, 122, w)) { ok = false; break; }
            tc_fence_after();
            const uint32_t bbase = kc_base + st * kKcStageBytes;
#pragma unroll
            for (int ks = 0; ks < NB / 16; ++ks)
              umma_f16_ts(tmem + kWCol0 + slot * 128, tmem + hh * 64 + ks * 8,
                          make_sdesc(bbase + ks * 2048, NB * 128, 1024, kSw128), idesc,
                          ks > 0 ? 1u : 0u);
            umma_commit(&w_full[slot]);
            // the last half is the kc tile's last reader
            if (hh == I.h_hi - 1) umma_commit(&kc_empty[st]);
          }
        }
      }
      umma_commit(mma_done);
      cv2_drain(mma_done, 0, a.err, 152);
    }
  } else if (warp == kStoreWarp) {
    // ------------------------------------------------------------ output stores
    // One TMA store per (item, half) staging use, once the 16 epilogue warps have written
    // the tile; the tile is handed back after the store has read it.
    if (lane == 0) {
      prefetch_tensormap(&tm_y);
      int f = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const Item I = item_of(a, it, HD);
        for (int hh = I.h_lo; hh < I.h_hi; ++hh, ++f) {
          if (!mbar_wait(stg_full, f & 1, a.err, abort_flag, 140, f)) { ok = false; break; }
          tma_store_2d(&tm_y, stg_s, GH ? a.off + I.u0 : I.u0, I.b * a.D + hh * 128);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(stg_empty);
        }
      }
      bulk_wait_group0();
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int e = warp - kEpiWarp0;         // 0..15
    const int qd = warp & 3;                // TMEM lane quadrant
    const int g = e >> 2;                   // token range [32g, 32g + 32)
    const int r = qd * 32 + lane;           // channel within the half = TMEM lane
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    const bool last_range = g == 3;         // 24 tokens: [96, 120)
    // mix rows into TMEM: warp (qd, g < HD) writes half g's row 32*qd + lane into lane r,
    // columns 64*g .. (pairs of basis entries)
    if (g < HD) {
      const uint4 *mrow = reinterpret_cast<const uint4 *>(
          reinterpret_cast<const T *>(a.mix) + (size_t)(g * 128 + r) * NB);
#pragma unroll
      for (int c0 = 0; c0 < NB / 2; c0 += 16) {
        uint32_t v[16];
        if (NB / 2 - c0 >= 16) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 m = __ldg(mrow + c0 / 4 + k);
            v[4 * k] = m.x; v[4 * k + 1] = m.y; v[4 * k + 2] = m.z; v[4 * k + 3] = m.w;
          }
          tmem_st16(lane_addr + g * 64 + c0, v);
        }
      }
      if (NB / 2 < 16) {
        // NB = 16: 8 packed columns; the other 8 of the 16-column store are zero and lie
        // in the unused part of this half's 64 mix columns
        uint32_t v[16];
#pragma unroll
        for (int k = 0; k < 2; ++k) {
          const uint4 m = __ldg(mrow + k);
          v[4 * k] = m.x; v[4 * k + 1] = m.y; v[4 * k + 2] = m.z; v[4 * k + 3] = m.w;
        }
#pragma unroll
        for (int k = 8; k < 16; ++k) v[k] = 0u;
        tmem_st16(lane_addr + g * 64, v);
      }
      tmem_wait_st();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(mix_ready);
    }
    // Every handoff is an mbarrier, so the 16 warps never wait for one another: a warp
    // releases the factor window after its last tap, waits only until the staging tile's
    // previous store has read it, writes its part and arrives on stg_full.
    int f = 0, w = 0;
    bool ok = true;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
      const Item I = item_of(a, it, HD);
      const int u0 = I.u0;
      const int fs0 = GH ? u0 : a.off + u0 - hH;
      // window column of output token 32g for tap 0 (forward: of h[off + u0 + 32g];
      // grad_h: of go[u0 + 32g])
      const int fbase = (fs0 & 7) + (GH ? 0 : hH) + 32 * g;
      for (int hh = I.h_lo; hh < I.h_hi && ok; ++hh, ++f) {
        const int fs = f % F;
        if (!mbar_wait_warp(&fac_full[fs], (f / F) & 1, a.err, abort_flag, 130, f)) { ok = false; break; }
        const uint8_t *frow = fac_s + fs * fac_bytes + (size_t)r * a.fac_w * 2;
        float acc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) acc[i] = 0.f;
        for (int kk = 0; kk < a.K; ++kk, ++w) {
          const int slot = w % kWSlots;
          if (!mbar_wait_warp(&w_full[slot], (w / kWSlots) & 1, a.err, abort_flag, 131, w)) { ok = false; break; }
          tc_fence_after();
          const int sh = GH ? ((u0 + kk * a.dil) & 7) : 0;   // TMEM column shift
          const int fcol = fbase + (GH ? kk * a.dil : -kk * a.dil);
          const uint32_t wcol = lane_addr + kWCol0 + slot * 128 + 32 * g;
#pragma unroll
          for (int p = 0; p < 2; ++p) {
            const int c = fcol + 16 * p;
            const int ca = c & ~7;
            const uint4 f0 = *reinterpret_cast<const uint4 *>(frow + ca * 2);
            const uint4 f1 = *reinterpret_cast<const uint4 *>(frow + ca * 2 + 16);
            const uint4 f2 = *reinterpret_cast<const uint4 *>(frow + ca * 2 + 32);
            const uint4 fa = shift8(f0, f1, c & 7), fb = shift8(f1, f2, c & 7);
            if (p == 1 && last_range) {
              // tokens [112, 120): columns [112 + sh, 120 + sh) lie in [112, 128)
              fma_piece<T>(acc + 16, wcol + 16, sh, fa);
            } else {
              fma_piece16<T>(acc + 16 * p, wcol + 16 * p, sh, fa, fb);
            }
          }
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(&w_empty[slot]);
        }
        if (!ok) break;
        __syncwarp();
        if (lane == 0) mbar_arrive(&fac_empty[fs]);
        // staging use f: the store of use f - 1 must have read the tile
        if (!mbar_wait_warp(stg_empty, (f & 1) ^ 1, a.err, abort_flag, 132, f)) { ok = false; break; }
        uint8_t *orow = stg_s + (size_t)r * kOutPitch + 64 * g;
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          if (!(last_range && c == 3))
            *reinterpret_cast<uint4 *>(orow + 16 * c) = make_uint4(
                pack2<T>(acc[8 * c], acc[8 * c + 1]), pack2<T>(acc[8 * c + 2], acc[8 * c + 3]),
                pack2<T>(acc[8 * c + 4], acc[8 * c + 5]), pack2<T>(acc[8 * c + 6], acc[8 * c + 7]));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(stg_full);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (a.dep_late) pdl_wait();
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

// kSplit = true would make a work item (b, tile, half): deeper rings, but each kc tile
// crosses L2 -> SM once per half. Measured slower on B200 (forward 38.4 vs 35.7 us at
// B=16 T=4096 D=256 N=128), so an item covers every half.
constexpr bool kSplit = false;

struct Conv2Plan {
  bool ok;
  int kc_stages, fac_stages, fac_w;
  size_t smem;
};

// Factor window width: the epilogue reads up to column hH + 142 of a window (largest tap
// offset hH + 7, plus 119 tokens, plus the 16-byte read-ahead of the shift), rounded to a
// multiple of 8 with an odd number of 16-byte chunks per row (row pitch = odd * 16 bytes
// keeps the row-per-lane 16-byte reads conflict free). kc stages: at least K, since the
// second half re-reads every tap of the item.
Conv2Plan plan_conv2(int N, int K, int hH, bool split) {
  Conv2Plan p{false, 0, 0, 0, 0};
  int w = (hH + 143 + 7) & ~7;
  if (((w / 8) & 1) == 0) w += 8;
  if (w > 256) return p;  // TMA box limit
  p.fac_w = w;
  const size_t budget = cv2::kSmemBudget - 1024;
  for (int F = 3; F >= 2 && !p.ok; --F)
    for (int S = cv2::kMaxKcStages; S >= (split ? 2 : K) && S >= 2; --S)
      if (cv2::layout(N, S, F, w).total <= budget) {
        p.ok = true;
        p.kc_stages = S;
        p.fac_stages = F;
        break;
      }
  if (p.ok) p.smem = cv2::layout(N, p.kc_stages, p.fac_stages, w).total + 1024;
  return p;
}

template <typename T, bool GH>
int conv2_dispatch(int N, const CUtensorMap &tkc, const CUtensorMap &tfac, const CUtensorMap &ty,
                   const cv2::Args &a, int grid, size_t smem, cudaStream_t st) {
  auto run = [&](auto kern) {
    if (set_smem_once((const void *)kern, (int)smem) !=
        cudaSuccess)
      return check_launch("cudaFuncSetAttribute(fdc_tc_conv2_kernel)");
    if (launch_pdl(kern, dim3(grid), dim3(cv2::kThreads), smem, st, tkc, tfac, ty, a) !=
        cudaSuccess)
      return check_launch("fdc_tc_conv2_kernel");
    return (int)DUDY_OK;
  };
  switch (N) {
    case 16: return run(fdc_tc_conv2_kernel<T, 16, GH>);
    case 32: return run(fdc_tc_conv2_kernel<T, 32, GH>);
    case 64: return run(fdc_tc_conv2_kernel<T, 64, GH>);
    default: return run(fdc_tc_conv2_kernel<T, 128, GH>);
  }
}

}  // namespace

bool conv2_supported(bool gh, const FdcShape &s, int dtype) {
  (void)gh;
  if (dtype != DUDY_DTYPE_F16 && dtype != DUDY_DTYPE_BF16) return false;
  if (!(s.D == 128 || s.D == 256)) return false;
  if (!(s.N == 16 || s.N == 32 || s.N == 64 || s.N == 128)) return false;
  if (s.T % 8 != 0 || s.L % 8 != 0) return false;
  if (s.K < 1) return false;
  if (s.B * s.D > (int64_t)1 << 31 || s.L > (int64_t)1 << 30) return false;
  return plan_conv2((int)s.N, (int)s.K, (int)((s.K - 1) * s.dil), kSplit).ok;
}

// forward: fac = h, y = out [B,D,T].  grad_h: fac = go, y = grad_h [B,D,L]; the tiles cover
// positions [floor8(max(0, off - hH)), off + T) (the caller zeroes the rest).
int conv2_launch(bool gh, const void *kc, const void *mix, const void *fac, void *y,
                 const FdcShape &s, int dtype, bool dep_late, int *err, cudaStream_t st) {
  const int N = (int)s.N, D = (int)s.D, T = (int)s.T, L = (int)s.L, K = (int)s.K;
  const int hH = (K - 1) * (int)s.dil;
  const bool split = kSplit;
  const Conv2Plan p = plan_conv2(N, K, hH, split);
  if (!p.ok) {
    set_error("tcgen05 conv: shared-memory plan does not fit");
    return DUDY_ERR_UNSUPPORTED;
  }
  const bool bf16 = dtype == DUDY_DTYPE_BF16;
  cv2::Args a{};
  a.mix = mix;
  a.B = (int)s.B; a.D = D; a.L = L; a.T = T; a.N = N; a.K = K;
  a.off = (int)s.off; a.dil = (int)s.dil;
  a.kc_stages = p.kc_stages; a.fac_stages = p.fac_stages; a.fac_w = p.fac_w;
  a.split = split ? 1 : 0;
  a.dep_late = dep_late ? 1 : 0;
  a.err = err;
  if (gh) {
    const int s_lo = (int)s.gh_lo();
    const int s0 = s_lo & ~7;
    a.u_first = s0 - (int)s.off;
    a.ntile = (int)cdiv((int64_t)s.off + T - s0, cv2::kTileOut);
  } else {
    a.u_first = 0;
    a.ntile = (int)cdiv(T, cv2::kTileOut);
  }
  const int64_t items = s.B * (int64_t)a.ntile * (split ? D / 128 : 1);
  int grid = sm_count();
  if (grid > items) grid = (int)items;
  if (grid < 1) grid = 1;
  CUtensorMap tkc, tfac, ty;
  const uint64_t ylen = gh ? (uint64_t)L : (uint64_t)T;
  const uint64_t flen = gh ? (uint64_t)T : (uint64_t)L;
  if (!make_tmap_2d(&tkc, kc, bf16, (uint64_t)T, (uint64_t)(s.B * K * N), (uint64_t)T * 2, 64,
                    (uint32_t)N, 128) ||
      !make_tmap_2d(&tfac, fac, bf16, flen, (uint64_t)(s.B * D), flen * 2, (uint32_t)p.fac_w,
                    128u, 0) ||
      !make_tmap_2d(&ty, y, bf16, ylen, (uint64_t)(s.B * D), ylen * 2, (uint32_t)cv2::kTileOut,
                    128u, 0))
    return DUDY_ERR_CUDA;
  if (bf16)
    return gh ? conv2_dispatch<__nv_bfloat16, true>(N, tkc, tfac, ty, a, grid, p.smem, st)
              : conv2_dispatch<__nv_bfloat16, false>(N, tkc, tfac, ty, a, grid, p.smem, st);
  return gh ? conv2_dispatch<__half, true>(N, tkc, tfac, ty, a, grid, p.smem, st)
            : conv2_dispatch<__half, false>(N, tkc, tfac, ty, a, grid, p.smem, st);
}

}  // namespace tc
}  // namespace dudy
