// Forward masked attention on sm_100a (tcgen05 + TMA), one 128-query tile of
// one (batch, head) per CTA, iterating only the live key tiles of the plan
// (attn_fwd_kernel); the rare rows outside its exponent range are recomputed
// exactly in fp32 by the epilogue warp that finds them (fix_row).
//
// Replaces confluence/confluence/layers.py:83-94: s = q k^T * scale,
// where(mask, s, -1e9), softmax, p v. Masked elements are excluded exactly
// (every row keeps its diagonal, so the reference's -1e9 entries contribute
// exp(-1e9 - max) == 0 in fp32). Also writes lse = ln sum_j exp(s_ij).
//
// The main kernel's structure (warp roles, TMEM layout, exponent reference)
// is described above attn_fwd_kernel.
#include <algorithm>

#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {
namespace fwd {

// Exponent reference offset (log2 units): p = exp2(c (s - s_ii) - kRefShift).
// The row's largest term is >= 2^-kRefShift, far above the fp32 / bf16
// normal range limit; rows whose terms grow past 2^100 go to the exact path.
constexpr float kRefShift = 64.0f;
constexpr int kMaxTiles = 65536 / RT_TILE;  // tiles per row of the plan (seq_len <= 65536)
static_assert(kMaxTiles <= 512, "tile list must fit in shared memory");

// ---------------------------------------------------------------------------
// Exact fallback for the rare rows the main kernel cannot take (their logit
// spread exceeds the range of the diagonal reference): the epilogue warp that
// finds one recomputes it on the spot, the whole warp in fp32 on the CUDA
// cores with an online max. Lanes take 32 keys at a time, o is spread over
// the lanes (DH/32 columns each), and q is read from cache for every dot
// product instead of being held in registers, so the path costs the main
// kernel no registers. In the common case it never runs.
// ---------------------------------------------------------------------------
template <int DH>
__device__ __noinline__ void fix_row(long long r, const uint16_t* __restrict__ qg, const uint16_t* __restrict__ kg,
                                     const uint16_t* __restrict__ vg, const rt_tile_plan& plan, int H, int S,
                                     float c, uint16_t* __restrict__ out, float* __restrict__ lse) {
  constexpr int kPer = DH / 32;  // output columns per lane
  const int lane = threadIdx.x & 31;
  const int T = plan.tiles;
  const int bh = (int)(r / S), i = (int)(r % S);
  const int b = bh / H, qt = i / RT_TILE, ri = i % RT_TILE;
  const uint32_t* qrow = reinterpret_cast<const uint32_t*>(qg + (size_t)r * DH);
  float m = -INFINITY, l = 0.f, o[kPer];
#pragma unroll
  for (int e = 0; e < kPer; ++e) o[e] = 0.f;
  const int lb = plan.q2k_ptr[b * T + qt], le = plan.q2k_ptr[b * T + qt + 1];
  for (int t = lb; t < le; ++t) {
    const int ent = plan.q2k_idx[t];
    const int kt = ent & 0x7FFFFFFF;
    const uint32_t* mrow = plan.tile_masks + ((((size_t)b * T + qt) * T + kt) * RT_TILE + ri) * 4;
    for (int ch = 0; ch < 4; ++ch) {
      const int j = kt * RT_TILE + ch * 32 + lane;
      const bool live = j < S && (ent < 0 || ((mrow[ch] >> lane) & 1u));
      float sc = -INFINITY;
      if (live) {
        float acc = 0.f;
        const uint32_t* krow = reinterpret_cast<const uint32_t*>(kg + ((size_t)bh * S + j) * DH);
        for (int d = 0; d < DH / 2; ++d) {
          const float2 qf = unpack_bf16x2(__ldg(qrow + d));
          const float2 kf = unpack_bf16x2(__ldg(krow + d));
          acc = fmaf(qf.x, kf.x, fmaf(qf.y, kf.y, acc));
        }
        sc = acc * c;
      }
      float cm = sc;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) cm = fmaxf(cm, __shfl_xor_sync(0xFFFFFFFFu, cm, off));
      const float mn = fmaxf(m, cm);
      if (mn == -INFINITY) continue;
      const float alpha = m == -INFINITY ? 0.f : exp2f(m - mn);
      const float p = live ? exp2f(sc - mn) : 0.f;
      float ps = p;
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) ps += __shfl_xor_sync(0xFFFFFFFFu, ps, off);
      l = l * alpha + ps;
#pragma unroll
      for (int e = 0; e < kPer; ++e) o[e] *= alpha;
      for (int src2 = 0; src2 < 32; ++src2) {
        const float pj = __shfl_sync(0xFFFFFFFFu, p, src2);
        const int jj = kt * RT_TILE + ch * 32 + src2;
        if (pj != 0.f) {
          const uint16_t* vrow = vg + ((size_t)bh * S + jj) * DH + lane * kPer;
#pragma unroll
          for (int e = 0; e < kPer; ++e) o[e] = fmaf(pj, __uint_as_float((uint32_t)vrow[e] << 16), o[e]);
        }
      }
      m = mn;
    }
  }
  const float inv_l = l > 0.f ? 1.f / l : 0.f;
  uint16_t* orow = out + (size_t)r * DH + lane * kPer;
#pragma unroll
  for (int e = 0; e < kPer; ++e) {
    const __nv_bfloat16 bv = __float2bfloat16_rn(o[e] * inv_l);
    orow[e] = *reinterpret_cast<const uint16_t*>(&bv);
  }
  if (lane == 0) lse[r] = l > 0.f ? (m + log2f(l)) * 0.6931471805599453f : -INFINITY;
}

// ---------------------------------------------------------------------------
// Main forward kernel: persistent, one CTA per SM, looping over work items
// (b, h, q-tile) c, c + G, c + 2G, ... (G = grid size) as one global sequence
// of live tiles, so the next item's loads and prologue overlap the current
// item's work and the epilogue overlaps the next item.
//   warp 0       producer: per tile, a tile-info word into a small ring, the
//                K / V tiles (TMA) and, for partial tiles, the 2 KB block of
//                mask words (bulk copy) into a 4-stage ring; per item, Q into
//                one of two slots
//   warp 1       PV issuer: O += P_g V_g into the item's O buffer (two,
//                alternating by item), in tile order
//   warp 22      S issuer: S_g = Q K_g^T into S buffer g % 3 once PV_{g-3},
//                which reads P_{g-3} from that buffer, has completed
//   warps 2..5   epilogue warpgroup: diagonal logits two items ahead, then
//                O / l -> bf16 and lse per item
//   warps 6..21  softmax: two groups of eight warps, group q taking the
//                tiles g with g % 2 == q; in a group, two warps per TMEM
//                lane quadrant, each owning a 64-column slice (two 32-column
//                chunks) of its 32 rows (thread = query row). P of a chunk
//                is packed over the first 16 of its 32 columns, so no warp
//                writes columns another warp has still to read
// Exponent reference: each row uses its own diagonal logit s_ii = q_i . k_i
// (always live), p = exp2(c (s - s_ii) - kRefShift): the largest term is at
// least 2^-kRefShift, so nothing that matters underflows, and no online max
// or O rescaling is needed (softmax is invariant to the reference). A row
// whose terms leave the safe range (row sum >= 2^100 or |O| >= 2^120, i.e. a
// logit spread above about (100 + kRefShift)/c, impossible for L2-normalised
// q, k) is recomputed exactly by the epilogue warp that finds it (fix_row).
// TMEM (512 columns): S buffers [0,128), [128,256), [256,384) fp32 with P_g
// written as bf16 pairs over columns [32 c, 32 c + 16) of its buffer for the
// 32-column chunk c, O buffers [384, 384+DH) and [384+DH, 384+2DH).
// ---------------------------------------------------------------------------
constexpr int kSBufs = 3;        // S / P buffers: tiles in flight between the MMAs and the softmax
constexpr int kSliceWarps = 4;   // softmax warps per lane quadrant
constexpr int kSoftmaxWarps = 4 * kSliceWarps;
// Softmax groups: group q takes the tiles g with g % kGroups == q, so one
// group's exponentials overlap the other's barrier hand-offs. Measured at the
// B=8, S=4096, H=16, Dh=64 workload: 1 group (all sixteen warps on every
// tile) 1.352 ms for the four kinds, 2 groups 1.267 ms.
constexpr int kGroups = 2;
constexpr int kGroupWarps = kSoftmaxWarps / kGroups;
constexpr int kChunks = kGroups;        // 32-column chunks per warp and tile
// S-ready barriers, one per (buffer, group): tile g signals barrier
// (g % kSBufs, g % kGroups), which comes round again every kStBars tiles
// because kSBufs and kGroups are coprime
constexpr int kStBars = kSBufs * kGroups;
static_assert(kGroups == 1 || kGroups == 2, "kGroups must divide the 4 slices and be coprime with kSBufs");
constexpr int kEpiWarps = 4;
constexpr int kSIssueWarp = 2 + kEpiWarps + kSoftmaxWarps;  // issues the S MMAs; warp 1 issues PV
constexpr int kMainThreads = 32 * (kSIssueWarp + 1);
constexpr int kMainTmemCols = 512;
constexpr int kOMain = kSBufs * 128;
constexpr int kStages = 4;
constexpr int kInfoRing = 8;
constexpr int kMaskBytes = RT_TILE * 16;
// tile-info word: kt (bits 0-15), fully live (16), first tile of its item (17),
// last tile of its item (18)
constexpr uint32_t kInfoFull = 1u << 16, kInfoFirst = 1u << 17, kInfoLast = 1u << 18;

// TMEM column (within an S buffer) of the bf16 pairs of P for keys
// [16 ks, 16 ks + 16): chunk ks / 2, second half of its packed run if ks is odd.
__device__ __forceinline__ uint32_t p_col(int ks) { return (uint32_t)((ks >> 1) * 32 + (ks & 1) * 8); }

template <int DH>
struct MainCfg {
  static constexpr int kRowBytes = DH * 2;
  static constexpr int kTileBytes = RT_TILE * kRowBytes;
  static constexpr uint32_t kSwizzle = DH == 64 ? SW_128B : SW_64B;
  static constexpr int kSBO = 8 * kRowBytes;
  static constexpr int kQOff = 0;                                  // two Q slots
  static constexpr int kKOff = 2 * kTileBytes;                     // K ring
  static constexpr int kVOff = kKOff + kStages * kTileBytes;       // V ring
  static constexpr int kMOff = kVOff + kStages * kTileBytes;       // mask ring
  static constexpr int kSmemBytes = kMOff + kStages * kMaskBytes;
  // all 512 TMEM columns per CTA: ask for enough shared memory that a second
  // CTA never lands on the same SM (it would only wait in tcgen05.alloc)
  static constexpr int kDynSmem = (kSmemBytes + 1024) > 118 * 1024 ? (kSmemBytes + 1024) : 118 * 1024;
};

struct __align__(8) MainBarriers {
  uint64_t q_full[2], q_empty[2];
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t st_full[kStBars], p_full[kSBufs], pv_done[kSBufs];
  uint64_t item_done[2], o_free[2];
  uint64_t sdiag_full[2], lsum_full[2];
  uint64_t drain, drain_s;
};

struct ItemCoord {
  int b, h, qt;
};
__device__ __forceinline__ ItemCoord item_coord(int item, int H, int T) {
  ItemCoord c;
  c.qt = item % T;
  const int bh = item / T;
  c.h = bh % H;
  c.b = bh / H;
  return c;
}

template <int DH>
__device__ __forceinline__ float diag_logit(const uint16_t* __restrict__ qg, const uint16_t* __restrict__ kg,
                                            size_t row) {
  const uint4* qa = reinterpret_cast<const uint4*>(qg + row * DH);
  const uint4* ka = reinterpret_cast<const uint4*>(kg + row * DH);
  float sd = 0.f;
#pragma unroll
  for (int v = 0; v < DH / 8; ++v) {
    const uint4 a = __ldg(qa + v), kk = __ldg(ka + v);
    const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, kw[4] = {kk.x, kk.y, kk.z, kk.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 af = unpack_bf16x2(aw[e]), kf = unpack_bf16x2(kw[e]);
      sd = fmaf(af.x, kf.x, fmaf(af.y, kf.y, sd));
    }
  }
  return sd;
}

template <int DH>
__global__ void __launch_bounds__(kMainThreads, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const uint16_t* __restrict__ qg,
                    const uint16_t* __restrict__ kg, const uint16_t* __restrict__ vg, const rt_tile_plan plan,
                    int H, int S, float scale_log2, uint16_t* __restrict__ out, float* __restrict__ lse) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  using C = MainCfg<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ MainBarriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ uint32_t s_info[kInfoRing];
  __shared__ float s_sdiag[2][RT_TILE];
  __shared__ float s_lpart[2][kSliceWarps][RT_TILE];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int T = plan.tiles;
  const int n_items_total = plan.batch * H * T;
  const int G = gridDim.x;
  const int n_items = (n_items_total - (int)blockIdx.x + G - 1) / G;  // items of this CTA
  auto item_id = [&](int k) { return (int)blockIdx.x + k * G; };
  auto item_ntiles = [&](int item) {
    const ItemCoord ic = item_coord(item, H, T);
    const int r = ic.b * T + ic.qt;
    return plan.q2k_ptr[r + 1] - plan.q2k_ptr[r];
  };

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars.q_full[i], 1);
      mbar_init(&bars.q_empty[i], 1);
      mbar_init(&bars.item_done[i], 1);
      mbar_init(&bars.o_free[i], kEpiWarps);
      mbar_init(&bars.sdiag_full[i], kEpiWarps);
      mbar_init(&bars.lsum_full[i], kSoftmaxWarps);
    }
    for (int i = 0; i < kStages; ++i) {
      mbar_init(&bars.kv_full[i], 1);
      mbar_init(&bars.kv_empty[i], 1);
    }
    for (int i = 0; i < kStBars; ++i) mbar_init(&bars.st_full[i], 1);
    for (int i = 0; i < kSBufs; ++i) {
      mbar_init(&bars.p_full[i], kGroupWarps);
      mbar_init(&bars.pv_done[i], 1);
    }
    mbar_init(&bars.drain, 1);
    mbar_init(&bars.drain_s, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, kMainTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    // ---------------- producer ----------------
    // item k's row pointer and first 32 list entries are loaded while item
    // k-1 streams, so item boundaries cost no L2 round trip
    auto item_list = [&](int k, int& lb, int& n, int& ent0) {
      lb = 0;
      n = 0;
      ent0 = 0;
      if (k >= n_items) return;
      const ItemCoord ic = item_coord(item_id(k), H, T);
      const int r = ic.b * T + ic.qt;
      lb = __ldg(plan.q2k_ptr + r);
      n = __ldg(plan.q2k_ptr + r + 1) - lb;
      ent0 = lane < n ? __ldg(plan.q2k_idx + lb + lane) : 0;
    };
    int g = 0;   // global tile index
    int kq = 0;  // Q loads issued
    bool ok = true;
    int lb_next, n_next, ent_next;
    item_list(0, lb_next, n_next, ent_next);
    for (int k = 0; ok && k < n_items; ++k) {
      const int lb = lb_next, n = n_next;
      int ent_l = ent_next;
      item_list(k + 1, lb_next, n_next, ent_next);
      const ItemCoord ic = item_coord(item_id(k), H, T);
      const int bh = ic.b * H + ic.h;
      const int r = ic.b * T + ic.qt;
      if (k >= 2 && !(ok = mbar_wait_warp(&bars.q_empty[k & 1], ((k - 2) >> 1) & 1, &abort_flag))) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&bars.q_full[k & 1], C::kTileBytes);
        tma_load_3d(smem + C::kQOff + (k & 1) * C::kTileBytes, &tm_q, &bars.q_full[k & 1], 0, ic.qt * RT_TILE, bh);
      }
      kq = k + 1;
      const uint32_t* mask_base = plan.tile_masks + (size_t)r * T * RT_TILE * 4;
      for (int t0 = 0; ok && t0 < n; t0 += 32) {
        if (t0 > 0) ent_l = (t0 + lane < n) ? __ldg(plan.q2k_idx + lb + t0 + lane) : 0;
        const int cnt = min(32, n - t0);
        for (int tt = 0; tt < cnt; ++tt, ++g) {
          const int ent = __shfl_sync(0xFFFFFFFFu, ent_l, tt);
          const int t = t0 + tt;
          const int st = g % kStages;
          if (g >= kStages && !(ok = mbar_wait_warp(&bars.kv_empty[st], ((g / kStages) - 1) & 1, &abort_flag))) break;
          if (lane == 0) {
            const int kt = ent & 0x7FFFFFFF;
            const bool full = ent < 0;
            s_info[g % kInfoRing] = (uint32_t)kt | (full ? kInfoFull : 0u) | (t == 0 ? kInfoFirst : 0u) |
                                    (t == n - 1 ? kInfoLast : 0u);
            mbar_arrive_expect_tx(&bars.kv_full[st], 2 * C::kTileBytes + (full ? 0 : kMaskBytes));
            tma_load_3d(smem + C::kKOff + st * C::kTileBytes, &tm_k, &bars.kv_full[st], 0, kt * RT_TILE, bh);
            tma_load_3d(smem + C::kVOff + st * C::kTileBytes, &tm_v, &bars.kv_full[st], 0, kt * RT_TILE, bh);
            if (!full)
              bulk_load(smem + C::kMOff + st * kMaskBytes, mask_base + (size_t)kt * RT_TILE * 4, kMaskBytes,
                        &bars.kv_full[st]);
          }
          __syncwarp();
        }
      }
    }
    // drain: every load issued must land before the CTA exits
    volatile int no_abort = 0;
    for (int gg = max(0, g - kStages); gg < g; ++gg)
      mbar_wait(&bars.kv_full[gg % kStages], (gg / kStages) & 1, &no_abort);
    for (int kk = max(0, kq - 2); kk < kq; ++kk) mbar_wait(&bars.q_full[kk & 1], (kk >> 1) & 1, &no_abort);
  } else if (warp == 1) {
    // ---------------- PV issue: the whole warp waits, one elected lane issues ----------------
    // Two warps issue MMAs so that each one's barrier waits overlap the other's
    // MMAs: this one O += P_g V_g in tile order, kSIssueWarp the S tiles. The
    // S tile g lands in the buffer P_{g - kSBufs} occupies, so the S warp waits
    // for pv_done (committed after that PV) before issuing it.
    {
      const bool leader = elect_one_sync();
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, DH, false, true);
      bool ok = true;
      int kP = 0, g = 0;
      int nP_next = n_items > 0 ? item_ntiles(item_id(0)) : 0;
      for (; ok && kP < n_items; ++kP) {
        const int n = nP_next;
        nP_next = kP + 1 < n_items ? item_ntiles(item_id(kP + 1)) : 0;
        const int ob = kP & 1;
        if (kP >= 2 && !(ok = mbar_wait_warp(&bars.o_free[ob], ((kP - 2) >> 1) & 1, &abort_flag))) break;
        for (int t = 0; ok && t < n; ++t, ++g) {
          const int buf = g % kSBufs;
          if (!(ok = mbar_wait_warp(&bars.p_full[buf], (g / kSBufs) & 1, &abort_flag))) break;
          tc_fence_after();
          // V is MN-major: +kRowBytes (16-byte units) per 16 keys
          const uint64_t vd = sdesc(smem_u32(smem + C::kVOff + (g % kStages) * C::kTileBytes), 0, C::kSBO, C::kSwizzle);
          if (leader) {
#pragma unroll
            for (int ks = 0; ks < RT_TILE / 16; ++ks)  // O += P_g V_g
              mma_ts(tmem + kOMain + ob * DH, tmem + buf * 128 + p_col(ks), vd + ks * C::kRowBytes, idesc_o,
                     (t > 0 || ks > 0) ? 1u : 0u);
            mma_commit(&bars.pv_done[buf]);
            mma_commit(&bars.kv_empty[g % kStages]);
            if (t == n - 1) mma_commit(&bars.item_done[ob]);
          }
          __syncwarp();
        }
        if (n == 0) {
          if (leader) mma_commit(&bars.item_done[ob]);
          __syncwarp();
        }
      }
      if (leader) mma_commit(&bars.drain);
      __syncwarp();
      volatile int no_abort = 0;
      mbar_wait_warp(&bars.drain, 0, &no_abort);
    }
  } else if (warp == kSIssueWarp) {
    // ---------------- S issue: item kS, tile tS within it, global tile gS ----------------
    const bool leader = elect_one_sync();
    constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
    bool ok = true;
    int kS = 0, tS = 0, gS = 0;
    int nS = n_items > 0 ? item_ntiles(item_id(0)) : 0;
    int nS_next = n_items > 1 ? item_ntiles(item_id(1)) : 0;
    while (ok) {
      while (kS < n_items && tS >= nS) {  // leave finished (or empty) items, releasing their Q slot
        if (nS == 0 && !(ok = mbar_wait_warp(&bars.q_full[kS & 1], (kS >> 1) & 1, &abort_flag))) break;
        if (leader) mma_commit(&bars.q_empty[kS & 1]);
        __syncwarp();
        ++kS;
        tS = 0;
        nS = nS_next;
        nS_next = kS + 1 < n_items ? item_ntiles(item_id(kS + 1)) : 0;
      }
      if (!ok || kS >= n_items) break;
      if (tS == 0 && !(ok = mbar_wait_warp(&bars.q_full[kS & 1], (kS >> 1) & 1, &abort_flag))) break;
      const int st = gS % kStages;
      if (!(ok = mbar_wait_warp(&bars.kv_full[st], (gS / kStages) & 1, &abort_flag))) break;
      // S_gS overwrites P_{gS - kSBufs}: wait until the PV that reads it has completed
      if (gS >= kSBufs && !(ok = mbar_wait_warp(&bars.pv_done[gS % kSBufs], ((gS / kSBufs) - 1) & 1, &abort_flag)))
        break;
      tc_fence_after();
      const uint64_t qd = sdesc(smem_u32(smem + C::kQOff + (kS & 1) * C::kTileBytes), 16, C::kSBO, C::kSwizzle);
      const uint64_t kd = sdesc(smem_u32(smem + C::kKOff + st * C::kTileBytes), 16, C::kSBO, C::kSwizzle);
      const uint32_t d = tmem + (gS % kSBufs) * 128;
      if (leader) {
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks) mma_ss(d, qd + ks * 2, kd + ks * 2, idesc_s, ks > 0 ? 1u : 0u);
        mma_commit(&bars.st_full[(gS % kSBufs) * kGroups + gS % kGroups]);
      }
      __syncwarp();
      ++tS;
      ++gS;
    }
    if (leader) mma_commit(&bars.drain_s);
    __syncwarp();
    volatile int no_abort = 0;
    mbar_wait_warp(&bars.drain_s, 0, &no_abort);
  } else if (warp < 2 + kEpiWarps) {
    // ---------------- epilogue warpgroup ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const float c = scale_log2;
    auto put_sdiag = [&](int k) {
      const ItemCoord ic = item_coord(item_id(k), H, T);
      const int qrow = ic.qt * RT_TILE + row;
      s_sdiag[k & 1][row] =
          qrow < S ? diag_logit<DH>(qg, kg, ((size_t)(ic.b * H + ic.h)) * S + qrow) : 0.f;
      mbar_arrive_warp(&bars.sdiag_full[k & 1]);
    };
    for (int k = 0; k < 2 && k < n_items; ++k) put_sdiag(k);
    bool ok = true;
    for (int k = 0; ok && k < n_items; ++k) {
      const int item = item_id(k);
      const ItemCoord ic = item_coord(item, H, T);
      const int bh = ic.b * H + ic.h;
      const int qrow = ic.qt * RT_TILE + row;
      const int n = item_ntiles(item);
      if (!(ok = mbar_wait_warp(&bars.lsum_full[k & 1], (k >> 1) & 1, &abort_flag))) break;
      float l = 0.f;
#pragma unroll
      for (int w = 0; w < kSliceWarps; ++w) l += s_lpart[k & 1][w][row];
      const float sd = s_sdiag[k & 1][row];
      if (k + 2 < n_items) put_sdiag(k + 2);  // the softmax warps finished item k: both buffers' readers are done
      if (!(ok = mbar_wait_warp(&bars.item_done[k & 1], (k >> 1) & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t o[DH];
#pragma unroll
      for (int cc = 0; cc < DH; cc += 32) {
        uint32_t (&oc)[32] = *reinterpret_cast<uint32_t(*)[32]>(&o[cc]);
        tmem_ld32(lane_base + kOMain + (k & 1) * DH + cc, oc);
      }
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(&bars.o_free[k & 1]);
      // accept the row only well inside the fp32 range (see above); also rejects NaN / inf
      bool bad = !(l < 0x1p100f);
      if (n > 0) {  // an item without tiles leaves its O buffer untouched
#pragma unroll
        for (int e = 0; e < DH; ++e) bad |= !(fabsf(__uint_as_float(o[e])) < 0x1p120f);
      }
      if (qrow < S) {
        const float inv_l = (n > 0 && l > 0.f) ? 1.f / l : 0.f;
        if (!bad) {
          uint4* dst = reinterpret_cast<uint4*>(out + ((size_t)bh * S + qrow) * DH);
#pragma unroll
          for (int cc = 0; cc < DH; cc += 8) {
            uint32_t w[4];
#pragma unroll
            for (int e = 0; e < 8; e += 2)
              w[e / 2] = n > 0 ? pack_bf16x2(__uint_as_float(o[cc + e]) * inv_l, __uint_as_float(o[cc + e + 1]) * inv_l)
                               : 0u;
            dst[cc / 8] = make_uint4(w[0], w[1], w[2], w[3]);
          }
        }
        lse[(size_t)bh * S + qrow] =
            bad ? __int_as_float(0x7FC00000) : (sd * c + kRefShift + __log2f(l)) * 0.6931471805599453f;
      }
      // rows outside the diagonal reference's range: the whole warp
      // recomputes each one exactly (it overwrites the NaN lse above)
      uint32_t todo = __ballot_sync(0xFFFFFFFFu, bad && qrow < S);
      __syncwarp();
      while (todo) {
        const int src = __ffs(todo) - 1;
        todo &= todo - 1;
        fix_row<DH>((long long)bh * S + ic.qt * RT_TILE + quad * 32 + src, qg, kg, vg, plan, H, S, c, out, lse);
      }
    }
    tc_fence_before();
  } else {
    // ---------------- softmax ----------------
    const int sw = warp - 2 - kEpiWarps;
    const int grp = sw / kGroupWarps;
    const int part = sw >> 2;  // (group, column slice) of this warp: its row-sum partial
    const int slice = (sw >> 2) % (4 / kGroups);  // this warp's kChunks * 32 columns of each tile
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16) + (uint32_t)(slice * kChunks * 32);
    const float c = scale_log2;
    const float2 c2 = make_float2(c, c);
    bool ok = true;
    int g = 0;  // global tile index at the start of the current item
    int n_next = n_items > 0 ? item_ntiles(item_id(0)) : 0;
    for (int k = 0; ok && k < n_items; ++k) {
      const int n = n_next;
      n_next = k + 1 < n_items ? item_ntiles(item_id(k + 1)) : 0;
      if (!(ok = mbar_wait_warp(&bars.sdiag_full[k & 1], (k >> 1) & 1, &abort_flag))) break;
      const float nref = -(s_sdiag[k & 1][row] * c + kRefShift);
      const float2 nm2 = make_float2(nref, nref);
      float2 lsum[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
      for (int t = (grp - g % kGroups + kGroups) % kGroups; t < n; t += kGroups) {
        const int gt = g + t;
        const int buf = gt % kSBufs;
        if (!(ok = mbar_wait_warp(&bars.st_full[buf * kGroups + gt % kGroups], (gt / kStBars) & 1, &abort_flag)))
          break;
        // S_gt issued implies its K / V / mask stage and tile info are in shared memory
        if (!(ok = mbar_wait_warp(&bars.kv_full[gt % kStages], (gt / kStages) & 1, &abort_flag))) break;
        tc_fence_after();
        const uint32_t info = s_info[gt % kInfoRing];
        const bool full = (info & kInfoFull) != 0;
        const uint8_t* mrow = smem + C::kMOff + (gt % kStages) * kMaskBytes + row * 16 + slice * kChunks * 4;
#pragma unroll
        for (int ch = 0; ch < kChunks; ++ch) {
          const uint32_t taddr = lane_base + (uint32_t)(buf * 128 + ch * 32);
          const uint32_t mw = full ? 0xFFFFFFFFu : reinterpret_cast<const uint32_t*>(mrow)[ch];
          uint32_t pk[16];
          if (!full && __all_sync(0xFFFFFFFFu, mw == 0u)) {
            // a 32 x 32 block with no live element: P = 0, nothing to load or exponentiate
#pragma unroll
            for (int e = 0; e < 16; ++e) pk[e] = 0u;
          } else {
            uint32_t r[32];
            tmem_ld32(taddr, r);
            tmem_wait_ld();
            if (!full) {
#pragma unroll
              for (int e = 0; e < 32; ++e) r[e] = ((mw >> e) & 1u) ? r[e] : __float_as_uint(-INFINITY);
            }
#pragma unroll
            for (int e = 0; e < 32; e += 4) {
#pragma unroll
              for (int a = 0; a < 2; ++a) {
                const float2 x =
                    ffma2(make_float2(__uint_as_float(r[e + 2 * a]), __uint_as_float(r[e + 2 * a + 1])), c2, nm2);
                // three pairs in four on the MUFU, the fourth as the polynomial on the
                // FMA and integer pipes: the polynomial costs about three times the
                // instructions of a MUFU pair, and instruction issue, not the MUFU, is
                // the softmax's limit (same-box forward A/B at B=8, S=4096, H=16,
                // Dh=64, four kinds: half polynomial 1.267 ms, a quarter 1.178 ms,
                // none 1.213 ms). At Dh = 32 all of them go to the MUFU (B=32,
                // S=1024, H=8: a quarter 0.247 ms, none 0.241 ms).
                const bool on_mufu = DH == 32 || (((e >> 1) + a) & 3) != 3;
                const float2 p = on_mufu ? make_float2(fast_exp2(x.x), fast_exp2(x.y)) : exp2_poly2(x);
                lsum[a] = fadd2(lsum[a], p);
                pk[(e >> 1) + a] = pack_bf16x2(p.x, p.y);
              }
            }
          }
          // P of these 32 columns over the first 16 of them (already read)
          tmem_st16(taddr, pk);
        }
        tmem_wait_st();
        // S_gt was issued after PV_{gt-3}, which read P_{gt-3} from this buffer,
        // had completed, so P_gt overwrites nothing an MMA still reads
        tc_fence_before();
        mbar_arrive_warp(&bars.p_full[buf]);
      }
      g += n;
      s_lpart[k & 1][part][row] = (lsum[0].x + lsum[0].y) + (lsum[1].x + lsum[1].y);
      mbar_arrive_warp(&bars.lsum_full[k & 1]);
    }
    tc_fence_before();
  }

  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kMainTmemCols);
  }
}

template <int DH>
int launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, float scale,
           const rt_tile_plan& plan, uint16_t* o, float* lse, cudaStream_t stream) {
  using M = MainCfg<DH>;
  CUtensorMap tq, tk, tv;
  if (make_qkv_tensor_map(&tq, q, B * H, S, DH) != RT_OK || make_qkv_tensor_map(&tk, k, B * H, S, DH) != RT_OK ||
      make_qkv_tensor_map(&tv, v, B * H, S, DH) != RT_OK)
    return RT_ERR_CUDA;  // detail recorded by make_qkv_tensor_map
  static bool configured[64] = {false};
  static int num_sms[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e =
        cudaFuncSetAttribute(attn_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, M::kDynSmem);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(attn_fwd_kernel)");
    e = cudaDeviceGetAttribute(&num_sms[dev], cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return cuda_failure(e, "cudaDeviceGetAttribute(multiprocessor count)");
    configured[dev] = true;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  const int sms = dev >= 0 && dev < 64 ? num_sms[dev] : 148;
  const long long items = (long long)B * H * plan.tiles;
  const int grid = (int)std::min<long long>(items, sms);
  return launch_pdl("attn_fwd_kernel launch", attn_fwd_kernel<DH>, dim3(grid), dim3(kMainThreads), M::kDynSmem,
                    stream, tq, tk, tv, q, k, v, plan, H, S, scale_log2, o, lse);
}

}  // namespace fwd

int launch_attention_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int Dh,
                         float scale, const rt_tile_plan& plan, uint16_t* o, float* lse, cudaStream_t stream) {
  if (Dh == 64) return fwd::launch<64>(q, k, v, B, H, S, scale, plan, o, lse, stream);
  if (Dh == 32) return fwd::launch<32>(q, k, v, B, H, S, scale, plan, o, lse, stream);
  return RT_ERR_UNSUPPORTED;
}

}  // namespace rt
