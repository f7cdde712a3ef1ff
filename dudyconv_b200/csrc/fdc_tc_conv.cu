// fdc_tc_conv.cu -- tcgen05/TMEM kernel for the dynamic-conv forward and for grad_h.
//
// Both are "per-token kernel, then depthwise causal apply" with the per-token kernel
// W_kk[t, d] = sum_n kc[b,kk,n,t] * mix[d,n] computed on the tensor cores and never
// written to memory:
//
//   forward : out[b,d,u]      = sum_kk W_kk[u, d]        * h[b,d, off+u-kk*dil]
//             (reference: cuda_ops/fused_dynamic_conv_forward_direct_exec.cu:26-75)
//   grad_h  : gh[b,d,off+u]   = sum_kk W_kk[u+kk*dil, d] * go[b,d, u+kk*dil]
//             (autograd of test_fused_dynamic_conv_against_reference.py:91-189)
//
// Work item = (b, 128-token tile); each CTA owns one 128-channel half of D, so it keeps
// only its half of mix resident. Per tap kk one MMA chain
//     acc[128 tok x 128 ch] = A_kk[128 tok x N] * mix_half[128 ch x N]^T
// with M = tokens (TMEM lane = token), N_mma = channels, K = N (basis size).
//   A_kk  : kc tile, MN-major (tokens contiguous), SWIZZLE_128B, staged by TMA.
//           For grad_h the tile starts kk*dil tokens later; when that start is not a
//           multiple of 8 tokens (TMA needs 16-byte aligned x), TMA loads the aligned
//           tile plus an 8-token side box and four shifter warps shift it in place.
//   B     : mix half, K-major (basis contiguous), resident for the whole kernel.
//   fac   : h (forward) or go (grad_h) tile [128 ch x (128 + halo)] staged by TMA; the
//           epilogue reads it at a per-tap column offset (lane = token, so every warp
//           read is 32 consecutive elements of one row: bank-conflict free).
// TMEM holds 4 accumulator slots of 128 columns (one per tap in flight); the epilogue
// (16 warps, 32 channels each) keeps the running sum over taps in registers.
//
// Warp roles: 0 kc-stage producer (TMA), 1 MMA issuer (+TMEM owner), 2 factor-tile
// producer (TMA), 3 idle, 4-19 epilogue, 20-23 in-place shifters (grad_h only). Every
// mbarrier wait is bounded.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tile_util.cuh"

namespace dudy {
namespace tc {

using namespace sm100;

constexpr int kTile = 128;     // tokens per item (MMA M)
constexpr int kHalf = 128;     // channels per CTA (MMA N)
constexpr int kEpiWarp0 = 4, kNumEpiWarps = 16;   // 4 per TMEM lane quadrant
constexpr int kEpiCols = 128 / (kNumEpiWarps / 4);  // channels per epilogue warp
constexpr int kShiftWarp0 = kEpiWarp0 + kNumEpiWarps, kNumShiftWarps = 4;
// forward: producer, MMA, 2 idle, epilogue; grad_h adds the 4 kc-stage filler warps
template <bool GH>
struct ConvThreads {
  static constexpr int value = 32 * (kShiftWarp0 + (GH ? kNumShiftWarps : 0));
};
constexpr int kSlots = 4;      // TMEM accumulator slots (128 columns each)
constexpr int kMaxKcStages = 4, kMaxFacStages = 2;
constexpr size_t kSmemBudget = 232448;  // 227 KB opt-in

struct ConvArgs {
  const void *kc;   // [B,K,N,T]
  void *y;          // forward: out [B,D,T]; grad_h: grad_h [B,D,L]
  int B, D, L, T, N, K, off, dil;
  int u_first;      // first tile start (multiple of 8; may be negative for grad_h)
  int u_lo, u_hi;   // output positions written, in token coordinates
  int ntile;        // tiles per sequence
  int kc_stages, fac_stages, fac_w;
  int fac_x0;       // forward: floor8(off - (K-1)*dil); grad_h: 0 (tile start)
  int dep_late;     // 1: wait for the previous kernel of the stream only before exiting
  int *err;
};

struct SmemLayout {
  uint32_t mix, kc, side, fac, bar, total;
};

// grad_h side box: the 8 tokens after a shifted tap's aligned 128-token tile, one 16-byte
// row per basis entry (no swizzle)
__host__ __device__ inline uint32_t side_bytes(int N) { return 16u * N; }

__host__ __device__ inline SmemLayout smem_layout(int N, int kc_stages, int fac_stages,
                                                  int fac_w, bool gh) {
  SmemLayout s;
  uint32_t o = 0;
  s.mix = o;
  o += kHalf * N * 2;
  o = (o + 1023) & ~1023u;
  s.kc = o;
  o += kc_stages * (N * 256);
  s.side = o;
  o += gh ? kc_stages * side_bytes(N) : 0u;
  s.fac = o;
  o += fac_stages * (kHalf * fac_w * 2);
  o = (o + 15) & ~15u;
  s.bar = o;
  o += 256;
  s.total = o;
  return s;
}

template <int NB>
struct MixLayout {
  // K-major B operand: rows = channels, NB basis entries per row
  static constexpr int kRowBytes = NB >= 64 ? 128 : NB * 2;
  static constexpr uint32_t kLayout = NB >= 64 ? kSw128 : (NB == 32 ? kSw64 : kSw32);
  static constexpr int kBoxN = NB >= 64 ? 64 : NB;
  static constexpr int kBlocks = NB >= 64 ? NB / 64 : 1;
  static constexpr uint32_t kBlockBytes = kHalf * kRowBytes;
  __device__ static uint64_t desc(uint32_t base, int ks) {
    // ks-th group of 16 basis entries
    const uint32_t blk = NB >= 64 ? (uint32_t)(ks >> 2) : 0u;
    const uint32_t in = NB >= 64 ? (uint32_t)(ks & 3) * 32u : (uint32_t)ks * 32u;
    return make_sdesc(base + blk * kBlockBytes + in, 16, 8 * kRowBytes, kLayout);
  }
};

// Teardown wait (ignores the abort flag: copies in flight must land before exit);
// a timeout is still recorded in the error word.
__device__ __forceinline__ bool mbar_wait_drain(uint64_t *bar, uint32_t parity, int *err,
                                                int site = 50) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      record_timeout(err, site, (int)parity);
      return false;
    }
  }
  return true;
}

// FW: factor-tile row pitch in elements when known at compile time (0: a.fac_w), so the
// epilogue's per-channel row offsets are immediates
template <typename T, int NB, bool GH, int FW>
__global__ void __launch_bounds__(ConvThreads<GH>::value, 1)
fdc_tc_conv_kernel(const __grid_constant__ CUtensorMap tm_kc,
                   const __grid_constant__ CUtensorMap tm_mix,
                   const __grid_constant__ CUtensorMap tm_fac,
                   const __grid_constant__ CUtensorMap tm_kc_side, const ConvArgs a) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array itself, so that the compiler keeps
  // every pointer below in the shared window (32-bit LDS/STS addressing, not generic)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const SmemLayout L = smem_layout(NB, a.kc_stages, a.fac_stages, a.fac_w, GH);
  uint8_t *mix_s = smem + L.mix;
  uint8_t *kc_s = smem + L.kc;
  uint8_t *side_s = smem + L.side;
  uint8_t *fac_s = smem + L.fac;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + L.bar);
  uint64_t *kc_full = bars;                       // [4]
  uint64_t *kc_empty = bars + 4;                  // [4]
  uint64_t *fac_full = bars + 8;                  // [2]
  uint64_t *fac_empty = bars + 10;                // [2]
  uint64_t *acc_full = bars + 12;                 // [4]
  uint64_t *acc_empty = bars + 16;                // [4]
  uint64_t *mix_full = bars + 20;
  uint64_t *mma_done = bars + 21;
  uint32_t *tmem_hold = reinterpret_cast<uint32_t *>(bars + 22);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 23);
  volatile int *group_go = reinterpret_cast<volatile int *>(bars + 24);
  uint64_t *raw_full = bars + 25;                 // [4] grad_h: unshifted tile landed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int halves = a.D / kHalf;
  const int half = blockIdx.x % halves;
  const int cta_in_half = blockIdx.x / halves;
  const int ctas_per_half = gridDim.x / halves;
  const int items = a.B * a.ntile;
  const int S = a.kc_stages, F = a.fac_stages;
  constexpr uint32_t kKcStageBytes = NB * 256;
  const int fw = FW ? FW : a.fac_w;
  const uint32_t fac_stage_bytes = kHalf * fw * 2;
  const int hH = (a.K - 1) * a.dil;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(&kc_full[i], 1);
      mbar_init(&kc_empty[i], 1);
      mbar_init(&acc_full[i], 1);
      mbar_init(&acc_empty[i], kNumEpiWarps);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&fac_full[i], 1);
      mbar_init(&fac_empty[i], kNumEpiWarps);
    }
    mbar_init(mix_full, 1);
    mbar_init(mma_done, 1);
    for (int i = 0; i < 4; ++i) mbar_init(&raw_full[i], 1);
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
    // ------------------------------------------------------------ kc-stage producer
    // The only filler of the kc ring (parity waits need one filler per ring). grad_h taps
    // whose start is not 8-aligned load the aligned tile and an 8-token side box and
    // complete raw_full; the shifter warps then shift in place and complete kc_full.
    if (lane == 0) {
      prefetch_tensormap(&tm_kc);
      prefetch_tensormap(&tm_mix);
      if (GH) prefetch_tensormap(&tm_kc_side);
      using ML = MixLayout<NB>;
      mbar_arrive_expect_tx(mix_full, kHalf * NB * 2);
#pragma unroll
      for (int blk = 0; blk < ML::kBlocks; ++blk)
        tma_load_2d(mix_s + blk * ML::kBlockBytes, &tm_mix, mix_full, blk * 64, half * kHalf);
      int q = 0;
      int uses[4] = {0, 0, 0, 0}, raws[4] = {0, 0, 0, 0};
      bool last_raw[4] = {false, false, false, false};
      bool ok = true;
      for (int it = cta_in_half; it < items && ok; it += ctas_per_half) {
        const int b = it / a.ntile;
        const int u0 = a.u_first + (it % a.ntile) * kTile;
        for (int kk = 0; kk < a.K; ++kk, ++q) {
          const int tx = GH ? u0 + kk * a.dil : u0;
          const int st = q % S;
          if (!mbar_wait(&kc_empty[st], ((q / S) & 1) ^ 1, a.err, abort_flag, 10, q)) { ok = false; break; }
          uint8_t *dst = kc_s + st * kKcStageBytes;
          const int row = (b * a.K + kk) * NB;
          if (GH && (tx & 7) != 0) {
            const int x0 = tx & ~7;
            mbar_arrive_expect_tx(&raw_full[st], kKcStageBytes + side_bytes(NB));
            tma_load_2d(dst, &tm_kc, &raw_full[st], x0, row);
            tma_load_2d(dst + NB * 128, &tm_kc, &raw_full[st], x0 + 64, row);
            tma_load_2d(side_s + st * side_bytes(NB), &tm_kc_side, &raw_full[st], x0 + 128, row);
            ++raws[st];
            last_raw[st] = true;
          } else {
            mbar_arrive_expect_tx(&kc_full[st], kKcStageBytes);
            tma_load_2d(dst, &tm_kc, &kc_full[st], tx, row);
            tma_load_2d(dst + NB * 128, &tm_kc, &kc_full[st], tx + 64, row);
            last_raw[st] = false;
          }
          ++uses[st];
        }
      }
      // drain: the last copy into each stage must land before the CTA may exit
      for (int st = 0; st < S; ++st) {
        if (uses[st] == 0) continue;
        if (last_raw[st])
          mbar_wait_drain(&raw_full[st], (raws[st] - 1) & 1, a.err, 51);
        else
          mbar_wait_drain(&kc_full[st], (uses[st] - 1) & 1, a.err, 51);
      }
      mbar_wait_drain(mix_full, 0, a.err, 54);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ factor-tile producer
    // h (forward) or go (grad_h) tile of each item, decoupled from the kc ring so the
    // epilogue's next factor tile is never queued behind kc stage waits.
    if (lane == 0) {
      prefetch_tensormap(&tm_fac);
      int f = 0, last_par[2] = {-1, -1};
      for (int it = cta_in_half; it < items; it += ctas_per_half, ++f) {
        const int b = it / a.ntile;
        const int u0 = a.u_first + (it % a.ntile) * kTile;
        const int fs = f % F;
        if (!mbar_wait(&fac_empty[fs], ((f / F) & 1) ^ 1, a.err, abort_flag, 11, f)) break;
        mbar_arrive_expect_tx(&fac_full[fs], fac_stage_bytes);
        const int fx = GH ? u0 : a.fac_x0 + u0;
        tma_load_2d(fac_s + fs * fac_stage_bytes, &tm_fac, &fac_full[fs], fx,
                    b * a.D + half * kHalf);
        last_par[fs] = (f / F) & 1;
      }
      for (int fs = 0; fs < F; ++fs)
        if (last_par[fs] >= 0) mbar_wait_drain(&fac_full[fs], last_par[fs], a.err, 52);
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      using ML = MixLayout<NB>;
      constexpr uint32_t idesc = make_idesc_f16(kTile, kHalf, IsBf16<T>::value, 1, 0);
      const uint32_t mix_base = smem_u32(mix_s);
      const uint32_t kc_base = smem_u32(kc_s);
      bool ok = mbar_wait(mix_full, 0, a.err, abort_flag, 20, 0);
      int q = 0;
      for (int it = cta_in_half; it < items && ok; it += ctas_per_half) {
        for (int kk = 0; kk < a.K; ++kk, ++q) {
          const int st = q % S, slot = q % kSlots;
          if (!mbar_wait(&kc_full[st], (q / S) & 1, a.err, abort_flag, 21, q) ||
              !mbar_wait(&acc_empty[slot], ((q / kSlots) & 1) ^ 1, a.err, abort_flag, 22, q)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t abase = kc_base + st * kKcStageBytes;
#pragma unroll
          for (int ks = 0; ks < NB / 16; ++ks) {
            const uint64_t ad = make_sdesc(abase + ks * 2048, NB * 128, 1024, kSw128);
            const uint64_t bd = ML::desc(mix_base, ks);
            umma_f16(tmem + slot * 128, ad, bd, idesc, ks > 0 ? 1u : 0u);
          }
          umma_commit(&kc_empty[st]);
          umma_commit(&acc_full[slot]);
        }
      }
      // all issued MMAs complete before teardown
      umma_commit(mma_done);
      mbar_wait_drain(mma_done, 0, a.err, 55);
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int qd = warp & 3;                     // TMEM lane quadrant
    const int grp = (warp - kEpiWarp0) >> 2;     // channel group: [kEpiCols*grp, +kEpiCols)
    const int tl = qd * 32 + lane;               // token within the tile
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    int q = 0, f = 0;
    bool ok = true;
    for (int it = cta_in_half; it < items && ok; it += ctas_per_half, ++f) {
      const int b = it / a.ntile;
      const int u0 = a.u_first + (it % a.ntile) * kTile;
      const int u = u0 + tl;
      const int fs = f % F;
      if (!mbar_wait_warp(&fac_full[fs], (f / F) & 1, a.err, abort_flag, 30, f)) { ok = false; break; }
      const T *fac_row0 = reinterpret_cast<const T *>(fac_s + fs * fac_stage_bytes) +
                          grp * kEpiCols * fw;
      float acc[kEpiCols];
#pragma unroll
      for (int i = 0; i < kEpiCols; ++i) acc[i] = 0.f;
      for (int kk = 0; kk < a.K; ++kk, ++q) {
        const int slot = q % kSlots;
        if (!mbar_wait_warp(&acc_full[slot], (q / kSlots) & 1, a.err, abort_flag, 31, q)) { ok = false; break; }
        tc_fence_after();
        // column of this lane's factor value for tap kk
        const int col = GH ? tl + kk * a.dil : (a.off + u0 - hH) - (a.fac_x0 + u0) + (a.K - 1 - kk) * a.dil + tl;
        const T *fp = fac_row0 + col;
#pragma unroll
        for (int c = 0; c < kEpiCols / 16; ++c) {
          // shared-memory factor loads first, so their latency overlaps the TMEM load
          T fv[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) fv[i] = fp[(c * 16 + i) * fw];
          float v[16];
          tmem_ld16(lane_addr + slot * 128 + grp * kEpiCols + c * 16, v);
#pragma unroll
          for (int i = 0; i < 16; ++i)
            acc[c * 16 + i] = fmaf(v[i], Elem<T>::to_f(fv[i]), acc[c * 16 + i]);
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&acc_empty[slot]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&fac_empty[fs]);
      if (!ok) break;
      if (u >= a.u_lo && u < a.u_hi) {
        const int dbase = half * kHalf + grp * kEpiCols;
        T *yp;
        if (GH)
          yp = reinterpret_cast<T *>(a.y) + ((size_t)b * a.D + dbase) * a.L + (a.off + u);
        else
          yp = reinterpret_cast<T *>(a.y) + ((size_t)b * a.D + dbase) * a.T + u;
        const size_t ystride = GH ? (size_t)a.L : (size_t)a.T;
#pragma unroll
        for (int i = 0; i < kEpiCols; ++i) yp[(size_t)i * ystride] = Elem<T>::from_f(acc[i]);
      }
    }
  } else if (GH && warp >= kShiftWarp0 && warp < kShiftWarp0 + kNumShiftWarps) {
    // ------------------------------------------------------------ in-place shifters
    // (grad_h) A shifted tap's stage holds the aligned tile starting sh = tx & 7 tokens
    // early and the side buffer the 8 tokens after it. Thread n shifts row n left by sh
    // tokens in increasing chunk order (each 16-byte chunk is read before the chunk before
    // it is overwritten), then kc_full releases the stage to the MMA.
    const int n = threadIdx.x - kShiftWarp0 * 32;  // row (basis entry), 0..127
    const bool active = n < NB;
    int q = 0;
    int raws[4] = {0, 0, 0, 0};
    bool ok = true;
    for (int it = cta_in_half; it < items && ok; it += ctas_per_half) {
      const int u0 = a.u_first + (it % a.ntile) * kTile;
      for (int kk = 0; kk < a.K; ++kk, ++q) {
        const int tx = u0 + kk * a.dil;
        if ((tx & 7) == 0) continue;
        const int st = q % S;
        // one thread waits; the decision is broadcast through shared memory so the whole
        // group takes the same branch at the named barriers
        if (n == 0)
          *group_go = (mbar_wait(&raw_full[st], raws[st] & 1, a.err, abort_flag, 41, q) &&
                       !*abort_flag) ? 1 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (!*group_go) { ok = false; break; }
        ++raws[st];
        if (active) {
          uint8_t *tile = kc_s + st * kKcStageBytes;
          const uint4 *side = reinterpret_cast<const uint4 *>(side_s + st * side_bytes(NB));
          const int sh = tx & 7;
          // two phases of 8 chunks; a phase issues all its loads (its 8 chunks' right
          // neighbours included) before its first store
          uint4 w[9];
#pragma unroll
          for (int p = 0; p < 2; ++p) {
#pragma unroll
            for (int j = (p == 0 ? 0 : 1); j < 9; ++j) {
              const int cn = 8 * p + j;
              w[j] = cn < 16 ? *reinterpret_cast<const uint4 *>(tile + (cn >> 3) * (NB * 128) +
                                                               sw128_off(n, cn & 7))
                             : side[n];
            }
#pragma unroll
            for (int j = 0; j < 8; ++j)
              *reinterpret_cast<uint4 *>(tile + p * (NB * 128) + sw128_off(n, j)) =
                  shift8(w[j], w[j + 1], sh);
            w[0] = w[8];
          }
        }
        fence_proxy_async_smem();
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (n == 0) mbar_arrive(&kc_full[st]);
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

inline int floor8(int v) { return v & ~7; }
inline int round8(int v) { return (v + 7) & ~7; }

struct ConvPlan {
  int fac_w, kc_stages, fac_stages;
  size_t smem;
  bool ok;
};

ConvPlan plan_conv(bool gh, int N, int K, int dil) {
  ConvPlan p{};
  const int hH = (K - 1) * dil;
  p.fac_w = gh ? round8(kTile + hH) : round8(kTile + hH + 7);
  p.ok = false;
  if (p.fac_w > 256) return p;
  for (int fac = kMaxFacStages; fac >= 1 && !p.ok; --fac) {
    for (int ks = kMaxKcStages; ks >= 2; --ks) {
      const SmemLayout L = smem_layout(N, ks, fac, p.fac_w, gh);
      if (L.total + 1024 <= kSmemBudget) {
        p.kc_stages = ks;
        p.fac_stages = fac;
        p.smem = L.total + 1024;
        p.ok = true;
        break;
      }
    }
  }
  return p;
}

template <typename T, int NB, bool GH, int FW>
int launch_conv(const CUtensorMap &tkc, const CUtensorMap &tmix, const CUtensorMap &tfac,
                const CUtensorMap &tside, const ConvArgs &a, int grid, size_t smem,
                cudaStream_t st) {
  auto kern = fdc_tc_conv_kernel<T, NB, GH, FW>;
  if (set_smem_once((const void *)kern, (int)smem) !=
      cudaSuccess)
    return check_launch("cudaFuncSetAttribute(fdc_tc_conv_kernel)");
  // the CTAs of one work item (one per channel half) form a cluster, so both read each
  // kc tile from L2 at about the same time
  const unsigned halves = (unsigned)(a.D / kHalf);
  if (launch_pdl_cluster(kern, dim3(grid), dim3(ConvThreads<GH>::value), smem, st,
                         halves <= 2 ? halves : 1u, tkc, tmix, tfac, tside, a) != cudaSuccess)
    return check_launch(GH ? "fdc_tc_conv_kernel<grad_h>" : "fdc_tc_conv_kernel<forward>");
  return DUDY_OK;
}

template <typename T, bool GH, int FW>
int dispatch_n(int N, const CUtensorMap &tkc, const CUtensorMap &tmix, const CUtensorMap &tfac,
               const CUtensorMap &tside, const ConvArgs &a, int grid, size_t smem,
               cudaStream_t st) {
  switch (N) {
    case 16: return launch_conv<T, 16, GH, FW>(tkc, tmix, tfac, tside, a, grid, smem, st);
    case 32: return launch_conv<T, 32, GH, FW>(tkc, tmix, tfac, tside, a, grid, smem, st);
    case 64: return launch_conv<T, 64, GH, FW>(tkc, tmix, tfac, tside, a, grid, smem, st);
    default: return launch_conv<T, 128, GH, FW>(tkc, tmix, tfac, tside, a, grid, smem, st);
  }
}

// the forward's factor pitch for (K-1)*dil in [2, 9] (K = 3 up to dilation 4) is 144
constexpr int kFwdPitch = 144;

template <typename T>
int dispatch_fw(bool gh, int N, const CUtensorMap &tkc, const CUtensorMap &tmix,
                const CUtensorMap &tfac, const CUtensorMap &tside, const ConvArgs &a, int grid,
                size_t smem, cudaStream_t st) {
  if (gh) return dispatch_n<T, true, 0>(N, tkc, tmix, tfac, tside, a, grid, smem, st);
  if (a.fac_w == kFwdPitch)
    return dispatch_n<T, false, kFwdPitch>(N, tkc, tmix, tfac, tside, a, grid, smem, st);
  return dispatch_n<T, false, 0>(N, tkc, tmix, tfac, tside, a, grid, smem, st);
}

}  // namespace

bool conv2_supported(bool gh, const FdcShape &s, int dtype);
int conv2_launch(bool gh, const void *kc, const void *mix, const void *fac, void *y,
                 const FdcShape &s, int dtype, bool dep_late, int *err, cudaStream_t st);

bool conv_supported(bool gh, const FdcShape &s, int dtype) {
  if (gh && conv2_supported(gh, s, dtype)) return true;
  if (dtype != DUDY_DTYPE_F16 && dtype != DUDY_DTYPE_BF16) return false;
  if (s.D % kHalf != 0 || s.D <= 0) return false;
  if (!(s.N == 16 || s.N == 32 || s.N == 64 || s.N == 128)) return false;
  if (s.T % 8 != 0 || s.L % 8 != 0) return false;
  if (s.K < 1 || (s.K - 1) * s.dil > 1024) return false;
  if (s.B * s.D > (int64_t)1 << 31 || s.L > (int64_t)1 << 30) return false;
  return plan_conv(gh, (int)s.N, (int)s.K, (int)s.dil).ok;
}

// forward: fac = h, y = out.   grad_h: fac = go, y = grad_h (only [u_lo, T) + off written)
// dep_late: the kernel launched just before is the grad_h zero fill (see capi.cu)
int conv_launch(bool gh, const void *kc, const void *mix, const void *fac, void *y,
                const FdcShape &s, int dtype, bool dep_late, int *err, cudaStream_t st) {
  // grad_h with a tap whose start is not 8-token aligned: the all-channel kernel applies
  // the shift as a TMEM column offset instead of shifting kc tiles in shared memory
  // (B=16 T=4096 D=256 N=128 dil=1: 39 vs 42 us). Without shifted taps, and for the
  // forward, this per-half kernel measured faster (forward 31.6 vs 35.7 us).
  bool shifted = false;
  for (int kk = 1; kk < (int)s.K; ++kk) shifted |= ((kk * s.dil) & 7) != 0;
  const ConvPlan p = plan_conv(gh, (int)s.N, (int)s.K, (int)s.dil);
  if (gh && (shifted || !p.ok) && conv2_supported(gh, s, dtype))
    return conv2_launch(gh, kc, mix, fac, y, s, dtype, dep_late, err, st);
  if (!p.ok) {
    set_error("tcgen05 conv: shared-memory plan does not fit");
    return DUDY_ERR_UNSUPPORTED;
  }
  const bool bf16 = dtype == DUDY_DTYPE_BF16;
  const int N = (int)s.N, D = (int)s.D, T = (int)s.T, L = (int)s.L, K = (int)s.K;
  const int hH = (K - 1) * (int)s.dil;
  ConvArgs a{};
  a.kc = kc;
  a.y = y;
  a.B = (int)s.B; a.D = D; a.L = L; a.T = T; a.N = N; a.K = K;
  a.off = (int)s.off; a.dil = (int)s.dil;
  a.kc_stages = p.kc_stages; a.fac_stages = p.fac_stages; a.fac_w = p.fac_w;
  a.dep_late = dep_late ? 1 : 0;
  a.err = err;
  if (gh) {
    a.u_lo = -hH > -(int)s.off ? -hH : -(int)s.off;
    a.u_first = floor8(a.u_lo);
    a.u_hi = T;
    a.fac_x0 = 0;
  } else {
    a.u_lo = 0;
    a.u_first = 0;
    a.u_hi = T;
    a.fac_x0 = floor8((int)s.off - hH);
  }
  a.ntile = (int)cdiv(a.u_hi - a.u_first, kTile);
  const int halves = D / kHalf;
  const int64_t items = s.B * (int64_t)a.ntile;
  int per_half = sm_count() / halves;
  if (per_half < 1) per_half = 1;
  if (per_half > items) per_half = (int)items;
  const int grid = per_half * halves;

  CUtensorMap tkc, tmix, tfac, tside;
  const int mix_box = N >= 64 ? 64 : N;
  const int mix_sw = N >= 64 ? 128 : 2 * N;
  if (!make_tmap_2d(&tkc, kc, bf16, (uint64_t)T, (uint64_t)(s.B * K * N), (uint64_t)T * 2, 64,
                    (uint32_t)N, 128) ||
      !make_tmap_2d(&tmix, mix, bf16, (uint64_t)N, (uint64_t)D, (uint64_t)N * 2,
                    (uint32_t)mix_box, (uint32_t)kHalf, mix_sw) ||
      !make_tmap_2d(&tfac, fac, bf16, gh ? (uint64_t)T : (uint64_t)L, (uint64_t)(s.B * D),
                    (gh ? (uint64_t)T : (uint64_t)L) * 2, (uint32_t)p.fac_w, (uint32_t)kHalf, 0) ||
      !make_tmap_2d(&tside, kc, bf16, (uint64_t)T, (uint64_t)(s.B * K * N), (uint64_t)T * 2, 8,
                    (uint32_t)N, 0))
    return DUDY_ERR_CUDA;
  if (bf16)
    return dispatch_fw<__nv_bfloat16>(gh, N, tkc, tmix, tfac, tside, a, grid, p.smem, st);
  return dispatch_fw<__half>(gh, N, tkc, tmix, tfac, tside, a, grid, p.smem, st);
}

}  // namespace tc
}  // namespace dudy
