// fdc_tc_bk_n128.cu -- grad_kc / grad_mix kernel for a 128-entry basis (N = 128), with
// kernel_mix resident in tensor memory.
//
//   G_kk[b,d,t]       = go[b,d,t] * h[b,d, off+t-kk*dil]       (built in shared memory)
//   grad_kc[b,kk,n,t] = sum_d mix[d,n] * G_kk[b,d,t]
//   grad_mix[d,n]     = sum_{b,kk,t} G_kk[b,d,t] * kc[b,kk,n,t]
// (autograd of test_fused_dynamic_conv_against_reference.py:91-189; the reference
// materialises G in HBM and runs cuBLAS, cuda_ops/
// fused_dynamic_conv_backward_n_k3_d256_gemm_fp16_template.cuh:122-320.)
//
// Differences from the general kernel (fdc_tc_bk.cu), possible because N = 128 fills the
// 128 TMEM lanes:
//  * mix^T [128 n x D ch] lives in TMEM and is the A operand of grad_kc
//    (tcgen05.mma with A in tensor memory), so no shared memory holds mix;
//  * grad_kc is accumulated transposed, acc[n x 128 tok] (TMEM lane = basis entry): an
//    epilogue thread owns 128 consecutive tokens of one grad_kc row, rounds them into a
//    swizzled staging tile and TMA stores it (row-scattered 16-byte stores from the
//    threads would queue in the load/store unit ahead of the builders' shared-memory
//    traffic);
//  * the shared memory mix used to take holds a ring of h windows brought in by TMA
//    (136 tokens: the 128-token tile plus the 8 tokens a causal shift can reach), so the
//    G builders read h from shared memory instead of waiting on global loads.
//
// Work item = (b, 128-token tile, tap kk), tap fastest. Per item and 128-channel half (one
// "unit"): a go tile (TMA, SWIZZLE_128B) lands in a G slot, the h window in an h stage,
// 8 builder warps form the exact products G = go * shifted h as two 16-bit terms
// G = G_hi + G_lo (split_mul8): G_hi replaces go in the G slot, G_lo goes into the h stage
// once every builder has read its h chunks (a 256-thread barrier), and the MMA warp issues
//     grad_mix[half] (TMEM, M = ch) += G_hi (K-major) * kc_kk + G_lo * kc_kk
//     acc          (TMEM, M = n)  += mix^T[:, half] (TMEM) * G_hi (MN-major) + ... * G_lo
// so the contraction sees the exact products (fp32 accumulation only); the G slot and the
// h stage are released together by the MMA commit.
// acc drains once per item through 4 epilogue warps; grad_mix stays in TMEM until the
// CTA's last item and leaves as an fp32 partial for the fixed-order reduction.
//
// Warp roles (512 threads): 0 kc producer (+ mix staging load, L2 prefetch), 1 MMA issuer
// (+TMEM owner), 2 go / h producer, 3 grad_kc TMA stores, 4-7 epilogue (+ mix^T into TMEM
// at start), 8-15 G builders. Every hand-off is an mbarrier and every wait is bounded.
#include <cuda.h>

#include "common.cuh"
#include "sm100.cuh"
#include "tile_util.cuh"

namespace dudy {
namespace tc {

using namespace sm100;

namespace bk128 {

constexpr int kTile = 128;
constexpr int kN = 128;
constexpr int kThreads = 512;
constexpr int kEpiWarp0 = 4, kNumEpiWarps = 4;
constexpr int kBuildWarp0 = 8, kNumBuildWarps = 8;
constexpr int kKcStages = 2, kGStages = 2;  // the h ring has kGStages stages too
constexpr uint32_t kKcBytes = kN * kTile * 2;
constexpr uint32_t kGBytes = 128 * kTile * 2;
constexpr int kHW = 136;                          // h window: tile + 8 shift tokens
constexpr uint32_t kHPitch = kHW * 2;             // 272-byte rows (unswizzled)
constexpr uint32_t kHBytes = 128 * kHPitch;
constexpr uint32_t kOffKc = 0;
constexpr uint32_t kOffG = kOffKc + kKcStages * kKcBytes;
constexpr uint32_t kOffH = kOffG + kGStages * kGBytes;
constexpr uint32_t kStgBytes = kN * 64 * 2;          // grad_kc store staging: 64 tokens
constexpr uint32_t kOffStg = kOffH + kGStages * kHBytes;
constexpr uint32_t kOffBar = kOffStg + kStgBytes;
constexpr uint32_t kSmemBytes = kOffBar + 256;
// TMEM columns: mix^T (D/2 packed columns), grad_kc accumulator, grad_mix per half
constexpr uint32_t kMixCol = 0, kAccCol = 128, kGmCol = 256;

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

}  // namespace bk128

__device__ __forceinline__ bool bk128_drain(uint64_t *bar, uint32_t parity, int *err, int site) {
  const uint64_t t0 = global_ns();
  while (!mbar_try_wait(bar, parity)) {
    if (global_ns() - t0 > kWaitLimitNs) {
      record_timeout(err, site, (int)parity);
      return false;
    }
  }
  return true;
}

// Named barrier 2 over the 256 builder threads, returning the AND of their `ok` flags (the
// same value in every thread).
__device__ __forceinline__ bool builders_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n .reg .pred p, q;\n setp.ne.u32 p, %1, 0;\n"
      " barrier.red.and.pred q, 2, 256, p;\n selp.u32 %0, 1, 0, q;\n}"
      : "=r"(r)
      : "r"((uint32_t)ok)
      : "memory");
  return r != 0;
}

template <typename T>
__global__ void __launch_bounds__(bk128::kThreads, 1)
fdc_tc_bk_n128_kernel(const __grid_constant__ CUtensorMap tm_kc,
                      const __grid_constant__ CUtensorMap tm_mix,
                      const __grid_constant__ CUtensorMap tm_go,
                      const __grid_constant__ CUtensorMap tm_go_tile,
                      const __grid_constant__ CUtensorMap tm_hw,
                      const __grid_constant__ CUtensorMap tm_gkc, const bk128::Args a) {
  using namespace bk128;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  // 1024-byte aligned base derived from the shared array itself, so that the compiler keeps
  // every pointer below in the shared window (32-bit LDS/STS addressing, not generic)
  uint8_t *smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t *kc_s = smem + kOffKc;
  uint8_t *g_s = smem + kOffG;
  uint8_t *h_s = smem + kOffH;
  uint8_t *stg_s = smem + kOffStg;
  uint64_t *bars = reinterpret_cast<uint64_t *>(smem + kOffBar);
  uint64_t *kc_full = bars;        // [2]
  uint64_t *kc_empty = bars + 2;   // [2]
  uint64_t *go_full = bars + 4;    // [2] go tile landed in the G slot
  uint64_t *g_full = bars + 6;     // [2] G built
  uint64_t *g_empty = bars + 8;    // [2] MMAs done with the G slot
  uint64_t *h_full = bars + 10;    // [2] (the h stage is released with the G slot)
  uint64_t *gk_full = bars + 14;
  uint64_t *gk_empty = bars + 15;
  uint64_t *mix_full = bars + 16;
  uint64_t *mixT_full = bars + 17;
  uint64_t *gm_done = bars + 18;
  uint32_t *tmem_hold = reinterpret_cast<uint32_t *>(bars + 19);
  volatile int *abort_flag = reinterpret_cast<volatile int *>(bars + 20);
  uint64_t *stg_full = bars + 21;   // the 4 epilogue warps wrote the staging tile
  uint64_t *stg_empty = bars + 22;  // its TMA store has read it

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int HD = a.D / 128;
  // work item = (b, tile, tap), tap fastest: the CTAs running the taps of one tile at the
  // same time share its go / h reads through L2
  const int items = a.B * a.ntile * a.K;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&kc_full[i], 1);
      mbar_init(&kc_empty[i], 1);
      mbar_init(&go_full[i], 1);
      mbar_init(&g_full[i], kNumBuildWarps);
      mbar_init(&g_empty[i], 1);
      mbar_init(&h_full[i], 1);
    }
    mbar_init(gk_full, 1);
    mbar_init(gk_empty, kNumEpiWarps);
    mbar_init(mix_full, 1);
    mbar_init(mixT_full, kNumEpiWarps);
    mbar_init(gm_done, 1);
    mbar_init(stg_full, kNumEpiWarps);
    mbar_init(stg_empty, 1);
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
  // inputs may come from the previous kernel of the stream (programmatic launch). With
  // dep_late the previous kernel is an independent one of the same backward call, which
  // triggered only after its own wait: the inputs are complete already, so this kernel
  // starts at once and waits for that kernel only before it exits (so a later kernel that
  // waits for this one also sees the earlier kernel's results).
  if (!a.dep_late) pdl_wait();
  if (threadIdx.x == 0) pdl_trigger();

  if (warp == 0) {
    // ------------------------------------------------------------ kc producer
    if (lane == 0) {
      prefetch_tensormap(&tm_kc);
      prefetch_tensormap(&tm_mix);
      prefetch_tensormap(&tm_go);
      prefetch_tensormap(&tm_hw);
      // mix [D x 128] lands in the kc ring (free until mix^T is in TMEM), so the go / h
      // producer can fill the G and h rings from the start
      mbar_arrive_expect_tx(mix_full, a.D * kN * 2);
      for (int hh = 0; hh < HD; ++hh)
        tma_load_2d(kc_s + hh * 128 * kN * 2, &tm_mix, mix_full, 0, hh * 128);
      auto prefetch_item = [&](int it2) {
        if (it2 >= items) return;
        const int b2 = it2 / (a.ntile * a.K), t2 = ((it2 / a.K) % a.ntile) * kTile;
        const int kk2 = it2 % a.K;
        const int p2 = a.off + t2 - kk2 * a.dil;
        for (int hh = 0; hh < HD; ++hh) {
          tma_prefetch_2d(&tm_go, t2, b2 * a.D + hh * 128);
          tma_prefetch_2d(&tm_hw, p2 - (p2 & 7), b2 * a.D + hh * 128);
        }
      };
      prefetch_item(blockIdx.x);
      int q = 0, last_par[kKcStages] = {-1, -1};
      bool ok = mbar_wait(mixT_full, 0, a.err, abort_flag, 164, 0);  // kc ring free again
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
        const int b = it / (a.ntile * a.K);
        const int t0 = ((it / a.K) % a.ntile) * kTile;
        const int kk = it % a.K;
        prefetch_item(it + gridDim.x);
        const int st = q % kKcStages;
        if (!mbar_wait(&kc_empty[st], ((q / kKcStages) & 1) ^ 1, a.err, abort_flag, 160, q)) { ok = false; break; }
        uint8_t *dst = kc_s + st * kKcBytes;
        mbar_arrive_expect_tx(&kc_full[st], kKcBytes);
        const int row = (b * a.K + kk) * kN;
        tma_load_2d(dst, &tm_kc, &kc_full[st], t0, row);
        tma_load_2d(dst + kN * 128, &tm_kc, &kc_full[st], t0 + 64, row);
        last_par[st] = (q / kKcStages) & 1;
      }
      for (int st = 0; st < kKcStages; ++st)
        if (last_par[st] >= 0) bk128_drain(&kc_full[st], last_par[st], a.err, 190);
      bk128_drain(mix_full, 0, a.err, 191);
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ go / h producer
    // One filler for each of the G ring and the h ring.
    if (lane == 0) {
      prefetch_tensormap(&tm_go_tile);
      prefetch_tensormap(&tm_hw);
      bool ok = true;
      int gu = 0, last_go[kGStages] = {-1, -1}, last_h[kGStages] = {-1, -1};
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x) {
        const int b = it / (a.ntile * a.K);
        const int t0 = ((it / a.K) % a.ntile) * kTile;
        const int kk = it % a.K;
        const int pos = a.off + t0 - kk * a.dil;
        const int x0 = pos - (pos & 7);  // 8-aligned window start (may be negative: zero fill)
        for (int hh = 0; hh < HD; ++hh, ++gu) {
          const int gs = gu % kGStages;
          const uint32_t par = (gu / kGStages) & 1;
          if (!mbar_wait(&g_empty[gs], par ^ 1, a.err, abort_flag, 162, gu)) { ok = false; break; }
          uint8_t *gdst = g_s + gs * kGBytes;
          mbar_arrive_expect_tx(&go_full[gs], kGBytes);
          tma_load_2d(gdst, &tm_go_tile, &go_full[gs], t0, b * a.D + hh * 128);
          tma_load_2d(gdst + 16384, &tm_go_tile, &go_full[gs], t0 + 64, b * a.D + hh * 128);
          last_go[gs] = par;
          // the h stage also held this slot's G_lo: free with the G slot (same commit)
          mbar_arrive_expect_tx(&h_full[gs], kHBytes);
          tma_load_2d(h_s + gs * kHBytes, &tm_hw, &h_full[gs], x0, b * a.D + hh * 128);
          last_h[gs] = par;
        }
      }
      for (int gs = 0; gs < kGStages; ++gs) {
        if (last_go[gs] >= 0) bk128_drain(&go_full[gs], last_go[gs], a.err, 192);
        if (last_h[gs] >= 0) bk128_drain(&h_full[gs], last_h[gs], a.err, 193);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_gm = make_idesc_f16(128, kN, IsBf16<T>::value, 0, 0);
      constexpr uint32_t idesc_kc = make_idesc_f16(kN, kTile, IsBf16<T>::value, 0, 1);
      const uint32_t kc_base = smem_u32(kc_s), g_base = smem_u32(g_s), l_base = smem_u32(h_s);
      bool ok = mbar_wait(mixT_full, 0, a.err, abort_flag, 170, 0);
      tc_fence_after();
      bool first_gm[2] = {true, true};
      int q = 0, gu = 0;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
        const int st = q % kKcStages;
        if (!mbar_wait(&kc_full[st], (q / kKcStages) & 1, a.err, abort_flag, 171, q)) break;
        const uint32_t kcb = kc_base + st * kKcBytes;
        for (int hh = 0; hh < HD; ++hh, ++gu) {
          const int gs = gu % kGStages;
          if (!mbar_wait(&g_full[gs], (gu / kGStages) & 1, a.err, abort_flag, 172, gu)) { ok = false; break; }
          tc_fence_after();
          const uint32_t gb = g_base + gs * kGBytes;   // G_hi
          const uint32_t lb = l_base + gs * kHBytes;   // G_lo (in the h stage)
          // grad_mix[half]: M = channels, K = tokens; both operands K-major
#pragma unroll
          for (int ks = 0; ks < 16; ++ks) {
            const uint32_t koff = ((ks & 7) >> 2) * 16384 + (ks & 3) * 32;
            umma_f16(tmem + kGmCol + hh * kN, make_sdesc((ks < 8 ? gb : lb) + koff, 16, 1024, kSw128),
                     make_sdesc(kcb + koff, 16, 1024, kSw128), idesc_gm,
                     (first_gm[hh] && ks == 0) ? 0u : 1u);
          }
          first_gm[hh] = false;
          if (hh == 0) {
            // the accumulator of the previous item must have been read out
            if (!mbar_wait(gk_empty, (q & 1) ^ 1, a.err, abort_flag, 173, q)) { ok = false; break; }
            tc_fence_after();
          }
          // grad_kc^T: M = basis entries (A = mix^T in TMEM), K = channels of this half,
          // N = tokens (B = G, MN-major)
#pragma unroll
          for (int ks = 0; ks < 16; ++ks)
            umma_f16_ts(tmem + kAccCol, tmem + kMixCol + hh * 64 + (ks & 7) * 8,
                        make_sdesc((ks < 8 ? gb : lb) + (ks & 7) * 2048, 16384, 1024, kSw128),
                        idesc_kc, (hh > 0 || ks > 0) ? 1u : 0u);
          umma_commit(&g_empty[gs]);
        }
        if (!ok) break;
        umma_commit(&kc_empty[st]);
        umma_commit(gk_full);
      }
      umma_commit(gm_done);
      bk128_drain(gm_done, 0, a.err, 194);
    }
  } else if (warp == 3) {
    // ------------------------------------------------------------ grad_kc stores
    // One TMA store per 64-token half of an item once the 4 epilogue warps have written
    // the staging tile; the tile is handed back after the store has read it.
    if (lane == 0) {
      prefetch_tensormap(&tm_gkc);
      int q = 0;
      bool ok = true;
      for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
        const int b = it / (a.ntile * a.K);
        const int t0 = ((it / a.K) % a.ntile) * kTile;
        const int kk = it % a.K;
        for (int hf = 0; hf < 2; ++hf) {
          const int su = 2 * q + hf;
          if (!mbar_wait(stg_full, su & 1, a.err, abort_flag, 187, su)) { ok = false; break; }
          tma_store_2d(&tm_gkc, stg_s, t0 + hf * 64, (b * a.K + kk) * kN);
          bulk_commit_group();
          bulk_wait_group_read0();
          mbar_arrive(stg_empty);
        }
      }
      bulk_wait_group0();
    }
  } else if (warp >= kEpiWarp0 && warp < kEpiWarp0 + kNumEpiWarps) {
    // ------------------------------------------------------------ epilogue
    const int qd = warp & 3;
    const int n = qd * 32 + lane;  // TMEM lane: basis entry (grad_kc), channel (grad_mix)
    const uint32_t lane_addr = tmem + ((uint32_t)(qd * 32) << 16);
    // Every handoff is an mbarrier: the warps never wait for one another. The grad_kc tile
    // leaves in two 64-token halves through the staging tile, stored by warp 3.
    bool ok = mbar_wait_warp(mix_full, 0, a.err, abort_flag, 180, 0);
    // mix^T into TMEM: thread n packs column n of mix, two channels per 32-bit column
    if (ok) {
      const uint16_t *ms = reinterpret_cast<const uint16_t *>(kc_s);
      for (int c0 = 0; c0 < a.D / 2; c0 += 16) {
        uint32_t r[16];
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const int ch = 2 * (c0 + i);
          r[i] = (uint32_t)ms[ch * kN + n] | ((uint32_t)ms[(ch + 1) * kN + n] << 16);
        }
        tmem_st16(lane_addr + kMixCol + c0, r);
      }
      tmem_wait_st();
    }
    tc_fence_before();
    __syncwarp();
    if (lane == 0) mbar_arrive(mixT_full);
    int q = 0;
    for (int it = blockIdx.x; it < items && ok; it += gridDim.x, ++q) {
      if (!mbar_wait_warp(gk_full, q & 1, a.err, abort_flag, 181, q)) break;
      tc_fence_after();
#pragma unroll
      for (int hf = 0; hf < 2; ++hf) {
        uint32_t r0[32], r1[32];
        tmem_ld32_raw(lane_addr + kAccCol + hf * 64, r0);
        tmem_ld32_raw(lane_addr + kAccCol + hf * 64 + 32, r1);
        if (hf == 1) {
          // the accumulator of this item has been read out
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(gk_empty);
        }
        // staging use 2q + hf: the store of the use before must have read the tile
        const int su = 2 * q + hf;
        if (!mbar_wait_warp(stg_empty, (su & 1) ^ 1, a.err, abort_flag, 182, su)) { ok = false; break; }
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          *reinterpret_cast<uint4 *>(stg_s + sw128_off(n, c)) = make_uint4(
              pack2<T>(__uint_as_float(r0[8 * c]), __uint_as_float(r0[8 * c + 1])),
              pack2<T>(__uint_as_float(r0[8 * c + 2]), __uint_as_float(r0[8 * c + 3])),
              pack2<T>(__uint_as_float(r0[8 * c + 4]), __uint_as_float(r0[8 * c + 5])),
              pack2<T>(__uint_as_float(r0[8 * c + 6]), __uint_as_float(r0[8 * c + 7])));
          *reinterpret_cast<uint4 *>(stg_s + sw128_off(n, 4 + c)) = make_uint4(
              pack2<T>(__uint_as_float(r1[8 * c]), __uint_as_float(r1[8 * c + 1])),
              pack2<T>(__uint_as_float(r1[8 * c + 2]), __uint_as_float(r1[8 * c + 3])),
              pack2<T>(__uint_as_float(r1[8 * c + 4]), __uint_as_float(r1[8 * c + 5])),
              pack2<T>(__uint_as_float(r1[8 * c + 6]), __uint_as_float(r1[8 * c + 7])));
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(stg_full);
      }
    }
    // grad_mix partial of this CTA: TMEM lane = channel within the half, column = n. A CTA
    // without work items (the grid is even and at least 2, so a one-item shape has one)
    // never wrote its grad_mix accumulator and contributes zeros.
    const bool gm_ok = bk128_drain(gm_done, 0, a.err, 195) && !*abort_flag;
    if (__all_sync(0xffffffffu, gm_ok)) {
      tc_fence_after();
      const bool any = (int)blockIdx.x < items;
      for (int hh = 0; hh < HD; ++hh) {
        float *dst = a.part + ((size_t)blockIdx.x * a.D + hh * 128 + n) * kN;
#pragma unroll
        for (int c = 0; c < kN / 32; ++c) {
          uint32_t r[32];
          tmem_ld32_raw(lane_addr + kGmCol + hh * kN + c * 32, r);
#pragma unroll
          for (int i = 0; i < 32; i += 4)
            *reinterpret_cast<uint4 *>(dst + c * 32 + i) =
                any ? make_uint4(r[i], r[i + 1], r[i + 2], r[i + 3]) : make_uint4(0, 0, 0, 0);
        }
      }
    }
  } else if (warp >= kBuildWarp0) {
    // ------------------------------------------------------------ G builders
    // Thread (r, j): row r of the unit's 128 channels, tokens [64j, 64j+64). It reads the 9
    // h chunks covering its shifted span from the h stage (272-byte rows: conflict free)
    // and the go chunks from the G slot, then writes G_hi over go and G_lo into the h stage
    // (same swizzled layout as the G slot). Rows of the h stage are shared by two warps, so
    // the G_lo writes wait for a barrier of all 256 builders; the barrier also ANDs their
    // wait results, so either every builder goes on or every builder stops.
    const int bid = threadIdx.x - kBuildWarp0 * 32;  // 0..255
    const int r = ((bid >> 5) & 3) * 32 + lane;
    const int j = bid >> 7;
    int gu = 0;
    for (int it = blockIdx.x; it < items; it += gridDim.x) {
      const int t0 = ((it / a.K) % a.ntile) * kTile;
      const int kk = it % a.K;
      const int sh = (a.off + t0 - kk * a.dil) & 7;
      bool ok = true;
      for (int hh = 0; hh < HD; ++hh, ++gu) {
        const int gs = gu % kGStages;
        const uint32_t par = (gu / kGStages) & 1;
        ok = mbar_wait_warp(&go_full[gs], par, a.err, abort_flag, 185, gu) &&
             mbar_wait_warp(&h_full[gs], par, a.err, abort_flag, 186, gu);
        uint4 hv[9];
        uint8_t *gbox = g_s + gs * kGBytes + j * 16384;
        uint4 gv[8];
        if (ok) {
          const uint8_t *hrow = h_s + gs * kHBytes + r * kHPitch + j * 128;
#pragma unroll
          for (int i = 0; i < 9; ++i) hv[i] = *reinterpret_cast<const uint4 *>(hrow + 16 * i);
#pragma unroll
          for (int c = 0; c < 8; ++c) gv[c] = *reinterpret_cast<const uint4 *>(gbox + sw128_off(r, c));
        }
        ok = builders_all(ok);
        if (!ok) break;
        uint8_t *lbox = h_s + gs * kHBytes + j * 16384;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          uint4 hi, lo;
          split_mul8<T>(gv[c], shift8(hv[c], hv[c + 1], sh), hi, lo);
          *reinterpret_cast<uint4 *>(gbox + sw128_off(r, c)) = hi;
          *reinterpret_cast<uint4 *>(lbox + sw128_off(r, c)) = lo;
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&g_full[gs]);
      }
      if (!ok) break;
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

bool bk128_supported(const FdcShape &s, int dtype) {
  if (dtype != DUDY_DTYPE_F16 && dtype != DUDY_DTYPE_BF16) return false;
  if (s.N != 128 || !(s.D == 128 || s.D == 256)) return false;
  return s.T % 8 == 0 && s.L % 8 == 0;
}

// Consecutive blocks take consecutive work items (taps of one tile, tap fastest); as a
// cluster they are co-scheduled, so their go / h reads of that tile reach L2 together.
constexpr unsigned kBkCluster = 2;

// Launches the kernel only; the caller runs the partial reduction.
int bk128_launch(const void *go, const void *h, const void *kc, const void *mix, void *grad_kc,
                 float *part, const FdcShape &s, int dtype, int grid, bool dep_late, int *err,
                 cudaStream_t st) {
  const bool bf16 = dtype == DUDY_DTYPE_BF16;
  bk128::Args a{};
  a.go = go;
  a.h = h;
  a.grad_kc = grad_kc;
  a.part = part;
  a.B = (int)s.B; a.D = (int)s.D; a.L = (int)s.L; a.T = (int)s.T; a.K = (int)s.K;
  a.off = (int)s.off; a.dil = (int)s.dil;
  a.ntile = (int)cdiv(s.T, bk128::kTile);
  a.dep_late = dep_late ? 1 : 0;
  a.err = err;
  CUtensorMap m_kc, m_mix, m_go, m_go_tile, m_hw, m_gkc;
  const uint64_t T = (uint64_t)s.T, rows = (uint64_t)(s.B * s.D);
  if (!make_tmap_2d(&m_kc, kc, bf16, T, (uint64_t)(s.B * s.K * 128), T * 2, 64, 128, 128) ||
      !make_tmap_2d(&m_mix, mix, bf16, 128, (uint64_t)s.D, 256, 128, 128, 0) ||
      !make_tmap_2d(&m_go, go, bf16, T, rows, T * 2, 128, 128, 0) ||
      !make_tmap_2d(&m_go_tile, go, bf16, T, rows, T * 2, 64, 128, 128) ||
      !make_tmap_2d(&m_hw, h, bf16, (uint64_t)s.L, rows, (uint64_t)s.L * 2, bk128::kHW, 128, 0) ||
      !make_tmap_2d(&m_gkc, grad_kc, bf16, T, (uint64_t)(s.B * s.K * 128), T * 2, 64, 128, 128))
    return DUDY_ERR_CUDA;
  const size_t smem = bk128::kSmemBytes + 1024;
  if (bf16) {
    auto kern = fdc_tc_bk_n128_kernel<__nv_bfloat16>;
    if (set_smem_once((const void *)kern, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(fdc_tc_bk_n128_kernel)");
    if (launch_pdl_cluster(kern, dim3(grid), dim3(bk128::kThreads), smem, st, kBkCluster, m_kc,
                           m_mix, m_go, m_go_tile, m_hw, m_gkc, a) != cudaSuccess)
      return check_launch("fdc_tc_bk_n128_kernel");
  } else {
    auto kern = fdc_tc_bk_n128_kernel<__half>;
    if (set_smem_once((const void *)kern, (int)smem) != cudaSuccess)
      return check_launch("cudaFuncSetAttribute(fdc_tc_bk_n128_kernel)");
    if (launch_pdl_cluster(kern, dim3(grid), dim3(bk128::kThreads), smem, st, kBkCluster, m_kc,
                           m_mix, m_go, m_go_tile, m_hw, m_gkc, a) != cudaSuccess)
      return check_launch("fdc_tc_bk_n128_kernel");
  }
  return DUDY_OK;
}

}  // namespace tc
}  // namespace dudy
