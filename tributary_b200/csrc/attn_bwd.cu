// Backward masked attention on sm_100a: the gradients jax autodiff takes
// through confluence/confluence/layers.py:83-94 (the reference has no
// hand-written backward; train.py:209 differentiates the forward).
//
//   delta_i = sum_d dO_id O_id                         (row_stats_kernel)
//   p_ij    = mask_ij ? exp(s_ij - lse_i) : 0,  s = scale q k^T
//   dP      = dO V^T ; dS = P o (dP - delta)
//   dQ      = scale * dS K                             (dq_kernel: thread = query)
//   dV      = P^T dO ; dK = scale * dS^T Q             (dkdv_kernel: thread = key)
//
// Both gradient kernels recompute P from lse, iterate only live tiles (q2k
// list for dQ, k2q list for dK/dV) and accumulate in TMEM, so every output
// element is written once by one CTA: results are deterministic, with no
// atomics; the only scratch is the padded row-statistics workspace.
#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {
namespace bwd {

constexpr int kThreads = 192;
constexpr int kTmemCols = 512;

template <int DH>
struct Cfg {
  static constexpr int kRowBytes = DH * 2;
  static constexpr int kTileBytes = RT_TILE * kRowBytes;
  static constexpr uint32_t kSwizzle = DH == 64 ? SW_128B : SW_64B;
  static constexpr int kSBO = 8 * kRowBytes;
  static constexpr int kStages = 3;
  // resident pair (Q,dO for dQ; K,V for dK/dV) then a ring of the other pair
  static constexpr int kA0 = 0;
  static constexpr int kA1 = kTileBytes;
  static constexpr int kR0 = 2 * kTileBytes;                 // ring tensor 0 (K or Q)
  static constexpr int kR1 = kR0 + kStages * kTileBytes;    // ring tensor 1 (V or dO)
  static constexpr int kRL = kR1 + kStages * kTileBytes;    // ring: lse2[128], delta[128] per stage
  static constexpr int kRowStatBytes = 2 * RT_TILE * 4;
  static constexpr int kSmemBytes = kRL + kStages * kRowStatBytes;
  // 512 TMEM columns per CTA: ask for enough shared memory that a second CTA
  // never lands on the same SM (it would only block in tcgen05.alloc).
  static constexpr int kDynSmem = (kSmemBytes + 1024) > 118 * 1024 ? (kSmemBytes + 1024) : 118 * 1024;
};

struct __align__(8) Barriers {
  uint64_t res_full;
  uint64_t ring_full[4];
  uint64_t ring_empty[4];
  uint64_t s_full;
  uint64_t p_full;
  uint64_t mma_done;
  uint64_t drain;
};

// Row statistics for the gradient kernels, padded to whole tiles:
//   stats[bh][0][q] = lse[bh][q] * log2(e)   (0 for q >= S)
//   stats[bh][1][q] = sum_d dO[bh][q][d] * O[bh][q][d]   (0 for q >= S)
template <int DH>
__global__ void __launch_bounds__(256) row_stats_kernel(const uint16_t* __restrict__ o,
                                                        const uint16_t* __restrict__ d_o,
                                                        const float* __restrict__ lse,
                                                        float* __restrict__ stats, int S, int Sp,
                                                        long long rows_padded) {
  constexpr int kLanesPerRow = DH / 8;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long prow = gid / kLanesPerRow;
  const int sub = (int)(gid % kLanesPerRow);
  const long long bh = prow / Sp;
  const int q = (int)(prow % Sp);
  const bool in = prow < rows_padded && q < S;
  float acc = 0.f;
  if (in) {
    const long long row = bh * S + q;
    const uint4 a = *reinterpret_cast<const uint4*>(o + row * DH + sub * 8);
    const uint4 g = *reinterpret_cast<const uint4*>(d_o + row * DH + sub * 8);
    const __nv_bfloat162* a2 = reinterpret_cast<const __nv_bfloat162*>(&a);
    const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&g);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 af = __bfloat1622float2(a2[e]);
      const float2 gf = __bfloat1622float2(g2[e]);
      acc = fmaf(af.x, gf.x, acc);
      acc = fmaf(af.y, gf.y, acc);
    }
  }
#pragma unroll
  for (int off = kLanesPerRow / 2; off > 0; off >>= 1) acc += __shfl_xor_sync(0xFFFFFFFFu, acc, off);
  if (prow < rows_padded && sub == 0) {
    float* st = stats + bh * 2 * Sp;
    st[q] = in ? lse[bh * S + q] * 1.4426950408889634f : 0.f;
    st[Sp + q] = acc;
  }
}

__device__ __forceinline__ void store_row_bf16(uint16_t* dst, const uint32_t (&pk)[8]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  d[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
}

// ---------------------------------------------------------------------------
// dQ: one CTA per (b, h, q-tile); thread = query row.
// TMEM: S [0,128) fp32, dP [128,256) fp32, dS [256,320) bf16x2, dQ [320,320+DH).
// ---------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
              const rt_tile_plan plan, int H, int S, float scale, float scale_log2,
              const float* __restrict__ stats, uint16_t* __restrict__ dq) {
  using C = Cfg<DH>;
  constexpr int kS = 0, kDP = 128, kDS = 256, kDQ = 320;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int row_list = b * T + qt;
  const int list_begin = plan.q2k_ptr[row_list];
  const int n_tiles = plan.q2k_ptr[row_list + 1] - list_begin;
  const int* list = plan.q2k_idx + list_begin;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bars.res_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars.ring_full[s], 1);
      mbar_init(&bars.ring_empty[s], 1);
    }
    mbar_init(&bars.s_full, 1);
    mbar_init(&bars.p_full, 128);
    mbar_init(&bars.mma_done, 1);
    mbar_init(&bars.drain, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(&bars.res_full, 2 * C::kTileBytes);
      tma_load_3d(smem + C::kA0, &tm_q, &bars.res_full, 0, qt * RT_TILE, bh);
      tma_load_3d(smem + C::kA1, &tm_do, &bars.res_full, 0, qt * RT_TILE, bh);
      int j = 0;
      for (; j < n_tiles; ++j) {
        const int s = j % C::kStages;
        if (j >= C::kStages && !mbar_wait(&bars.ring_empty[s], ((j / C::kStages) - 1) & 1, &abort_flag)) break;
        const int kt = list[j] & 0x7FFFFFFF;
        mbar_arrive_expect_tx(&bars.ring_full[s], 2 * C::kTileBytes);
        tma_load_3d(smem + C::kR0 + s * C::kTileBytes, &tm_k, &bars.ring_full[s], 0, kt * RT_TILE, bh);
        tma_load_3d(smem + C::kR1 + s * C::kTileBytes, &tm_v, &bars.ring_full[s], 0, kt * RT_TILE, bh);
      }
      volatile int no_abort = 0;
      for (int jj = max(0, j - C::kStages); jj < j; ++jj)
        mbar_wait(&bars.ring_full[jj % C::kStages], (jj / C::kStages) & 1, &no_abort);
      mbar_wait(&bars.res_full, 0, &no_abort);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_q = idesc_bf16_f32(128, DH, false, true);
      const uint32_t q_addr = smem_u32(smem + C::kA0);
      const uint32_t do_addr = smem_u32(smem + C::kA1);
      bool ok = mbar_wait(&bars.res_full, 0, &abort_flag);
      tc_fence_after();
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j > 0) {
          if (!(ok = mbar_wait(&bars.p_full, (j - 1) & 1, &abort_flag))) break;
          tc_fence_after();
          const int sp = (j - 1) % C::kStages;
          const uint32_t k_addr = smem_u32(smem + C::kR0 + sp * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks) {
            const uint64_t bdesc = sdesc(k_addr + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle);
            mma_ts(tmem + kDQ, tmem + kDS + ks * 8, bdesc, idesc_q, (j > 1 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&bars.mma_done);
          mma_commit(&bars.ring_empty[sp]);
        }
        if (j < n_tiles) {
          const int s = j % C::kStages;
          if (!(ok = mbar_wait(&bars.ring_full[s], (j / C::kStages) & 1, &abort_flag))) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + C::kR0 + s * C::kTileBytes);
          const uint32_t v_addr = smem_u32(smem + C::kR1 + s * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            mma_ss(tmem + kS, sdesc(q_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                   sdesc(k_addr + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            mma_ss(tmem + kDP, sdesc(do_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                   sdesc(v_addr + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bars.s_full);
        }
      }
      mma_commit(&bars.drain);
      volatile int no_abort = 0;
      mbar_wait(&bars.drain, 0, &no_abort);
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const int q = qt * RT_TILE + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t* masks = plan.tile_masks + ((size_t)row_list * T) * RT_TILE * 4;
    const int Sp = T * RT_TILE;
    const float lse2 = stats[(size_t)bh * 2 * Sp + q];
    const float dlt = stats[(size_t)bh * 2 * Sp + Sp + q];
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int ent = list[j];
      const int kt = ent & 0x7FFFFFFF;
      uint4 mk = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
      if (ent >= 0) mk = *reinterpret_cast<const uint4*>(masks + ((size_t)kt * RT_TILE + row) * 4);
      const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
      if (!(ok = mbar_wait(&bars.s_full, j & 1, &abort_flag))) break;
      if (j > 0 && !(ok = mbar_wait(&bars.mma_done, (j - 1) & 1, &abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t rs[32], rp[32];
        tmem_ld32(lane_base + kS + c * 32, rs);
        tmem_ld32(lane_base + kDP + c * 32, rp);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float p0 = ((mw[c] >> e) & 1u) ? fast_exp2(__uint_as_float(rs[e]) * scale_log2 - lse2) : 0.f;
          const float p1 =
              ((mw[c] >> (e + 1)) & 1u) ? fast_exp2(__uint_as_float(rs[e + 1]) * scale_log2 - lse2) : 0.f;
          const float d0 = p0 * (__uint_as_float(rp[e]) - dlt);
          const float d1 = p1 * (__uint_as_float(rp[e + 1]) - dlt);
          pk[e / 2] = pack_bf16x2(d0, d1);
        }
        tmem_st16(lane_base + kDS + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.p_full);
    }
    if (ok && n_tiles > 0 && mbar_wait(&bars.mma_done, (n_tiles - 1) & 1, &abort_flag)) {
      tc_fence_after();
      uint16_t* dst = dq + ((size_t)bh * S + q) * DH;
#pragma unroll
      for (int c = 0; c < DH; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_base + kDQ + c, r);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pk[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale);
        if (q < S) store_row_bf16(dst + c, pk);
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// ---------------------------------------------------------------------------
// dK, dV: one CTA per (b, h, k-tile); thread = key row.
// TMEM: S^T [0,128), dP^T [128,256), P^T [256,320) bf16x2, dS^T [320,384) bf16x2,
//       dV [384,384+DH), dK [384+DH,384+2DH).
// ---------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const rt_tile_plan plan, int H, int S, float scale, float scale_log2,
                const float* __restrict__ stats, uint16_t* __restrict__ dk, uint16_t* __restrict__ dv) {
  using C = Cfg<DH>;
  constexpr int kST = 0, kDPT = 128, kPT = 256, kDST = 320, kDV = 384, kDK = 384 + DH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int col_list = b * T + kt;
  const int list_begin = plan.k2q_ptr[col_list];
  const int n_tiles = plan.k2q_ptr[col_list + 1] - list_begin;
  const int* list = plan.k2q_idx + list_begin;
  const int Sp = T * RT_TILE;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bars.res_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars.ring_full[s], 1);
      mbar_init(&bars.ring_empty[s], 1);
    }
    mbar_init(&bars.s_full, 1);
    mbar_init(&bars.p_full, 128);
    mbar_init(&bars.mma_done, 1);
    mbar_init(&bars.drain, 1);
    fence_mbar_init();
  }
  if (warp == 0) {
    tmem_alloc(&tmem_base_s, kTmemCols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = tmem_base_s;

  if (warp == 0) {
    if (lane == 0 && n_tiles > 0) {
      mbar_arrive_expect_tx(&bars.res_full, 2 * C::kTileBytes);
      tma_load_3d(smem + C::kA0, &tm_k, &bars.res_full, 0, kt * RT_TILE, bh);
      tma_load_3d(smem + C::kA1, &tm_v, &bars.res_full, 0, kt * RT_TILE, bh);
      int i = 0;
      for (; i < n_tiles; ++i) {
        const int s = i % C::kStages;
        if (i >= C::kStages && !mbar_wait(&bars.ring_empty[s], ((i / C::kStages) - 1) & 1, &abort_flag)) break;
        const int qtile = list[i] & 0x7FFFFFFF;
        mbar_arrive_expect_tx(&bars.ring_full[s], 2 * C::kTileBytes + C::kRowStatBytes);
        tma_load_3d(smem + C::kR0 + s * C::kTileBytes, &tm_q, &bars.ring_full[s], 0, qtile * RT_TILE, bh);
        tma_load_3d(smem + C::kR1 + s * C::kTileBytes, &tm_do, &bars.ring_full[s], 0, qtile * RT_TILE, bh);
        uint8_t* st = smem + C::kRL + s * C::kRowStatBytes;
        const float* src = stats + (size_t)bh * 2 * Sp + (size_t)qtile * RT_TILE;
        bulk_load(st, src, RT_TILE * 4, &bars.ring_full[s]);
        bulk_load(st + RT_TILE * 4, src + Sp, RT_TILE * 4, &bars.ring_full[s]);
      }
      volatile int no_abort = 0;
      for (int ii = max(0, i - C::kStages); ii < i; ++ii)
        mbar_wait(&bars.ring_full[ii % C::kStages], (ii / C::kStages) & 1, &no_abort);
      mbar_wait(&bars.res_full, 0, &no_abort);
    }
  } else if (warp == 1) {
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_g = idesc_bf16_f32(128, DH, false, true);
      const uint32_t k_addr = smem_u32(smem + C::kA0);
      const uint32_t v_addr = smem_u32(smem + C::kA1);
      bool ok = mbar_wait(&bars.res_full, 0, &abort_flag);
      tc_fence_after();
      for (int i = 0; ok && i <= n_tiles; ++i) {
        if (i > 0) {
          if (!(ok = mbar_wait(&bars.p_full, (i - 1) & 1, &abort_flag))) break;
          tc_fence_after();
          const int sp = (i - 1) % C::kStages;
          const uint32_t q_addr = smem_u32(smem + C::kR0 + sp * C::kTileBytes);
          const uint32_t do_addr = smem_u32(smem + C::kR1 + sp * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks) {
            const uint32_t acc = (i > 1 || ks > 0) ? 1u : 0u;
            mma_ts(tmem + kDV, tmem + kPT + ks * 8,
                   sdesc(do_addr + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle), idesc_g, acc);
            mma_ts(tmem + kDK, tmem + kDST + ks * 8,
                   sdesc(q_addr + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle), idesc_g, acc);
          }
          mma_commit(&bars.mma_done);
          mma_commit(&bars.ring_empty[sp]);
        }
        if (i < n_tiles) {
          const int s = i % C::kStages;
          if (!(ok = mbar_wait(&bars.ring_full[s], (i / C::kStages) & 1, &abort_flag))) break;
          tc_fence_after();
          const uint32_t q_addr = smem_u32(smem + C::kR0 + s * C::kTileBytes);
          const uint32_t do_addr = smem_u32(smem + C::kR1 + s * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            mma_ss(tmem + kST, sdesc(k_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                   sdesc(q_addr + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
          }
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            mma_ss(tmem + kDPT, sdesc(v_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                   sdesc(do_addr + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bars.s_full);
        }
      }
      mma_commit(&bars.drain);
      volatile int no_abort = 0;
      mbar_wait(&bars.drain, 0, &no_abort);
    }
  } else {
    const int quad = warp & 3;
    const int row = quad * 32 + lane;           // key within the tile
    const int key = kt * RT_TILE + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t* masks_t = plan.tile_masks_t + ((size_t)col_list * T) * RT_TILE * 4;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const int ent = list[i];
      const int qtile = ent & 0x7FFFFFFF;
      uint4 mk = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
      if (ent >= 0) mk = *reinterpret_cast<const uint4*>(masks_t + ((size_t)qtile * RT_TILE + row) * 4);
      const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
      const int stage = i % C::kStages;
      if (!(ok = mbar_wait(&bars.ring_full[stage], (i / C::kStages) & 1, &abort_flag))) break;
      const float* l2 = reinterpret_cast<const float*>(smem + C::kRL + stage * C::kRowStatBytes);
      const float* dl = l2 + RT_TILE;
      if (!(ok = mbar_wait(&bars.s_full, i & 1, &abort_flag))) break;
      if (i > 0 && !(ok = mbar_wait(&bars.mma_done, (i - 1) & 1, &abort_flag))) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t rs[32], rp[32];
        tmem_ld32(lane_base + kST + c * 32, rs);
        tmem_ld32(lane_base + kDPT + c * 32, rp);
        tmem_wait_ld();
        uint32_t pk[16], dk_[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const int qa = c * 32 + e;
          const float p0 =
              ((mw[c] >> e) & 1u) ? fast_exp2(__uint_as_float(rs[e]) * scale_log2 - l2[qa]) : 0.f;
          const float p1 =
              ((mw[c] >> (e + 1)) & 1u) ? fast_exp2(__uint_as_float(rs[e + 1]) * scale_log2 - l2[qa + 1]) : 0.f;
          const float d0 = p0 * (__uint_as_float(rp[e]) - dl[qa]);
          const float d1 = p1 * (__uint_as_float(rp[e + 1]) - dl[qa + 1]);
          pk[e / 2] = pack_bf16x2(p0, p1);
          dk_[e / 2] = pack_bf16x2(d0, d1);
        }
        tmem_st16(lane_base + kPT + c * 16, pk);
        tmem_st16(lane_base + kDST + c * 16, dk_);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.p_full);
    }
    if (ok && n_tiles > 0 && mbar_wait(&bars.mma_done, (n_tiles - 1) & 1, &abort_flag)) {
      tc_fence_after();
      uint16_t* dst_v = dv + ((size_t)bh * S + key) * DH;
      uint16_t* dst_k = dk + ((size_t)bh * S + key) * DH;
#pragma unroll
      for (int c = 0; c < DH; c += 16) {
        uint32_t r[16], pk[8];
        tmem_ld16(lane_base + kDV + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2) pk[e / 2] = pack_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        if (key < S) store_row_bf16(dst_v + c, pk);
        tmem_ld16(lane_base + kDK + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pk[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale);
        if (key < S) store_row_bf16(dst_k + c, pk);
      }
    }
    tc_fence_before();
  }
  __syncthreads();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int DH>
int launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o, const uint16_t* d_o,
           const float* lse, int B, int H, int S, float scale, const rt_tile_plan& plan, uint16_t* dq,
           uint16_t* dk, uint16_t* dv, float* stats, cudaStream_t stream) {
  using C = Cfg<DH>;
  CUtensorMap tq, tk, tv, tdo;
  if (make_qkv_tensor_map(&tq, q, B * H, S, DH) != RT_OK || make_qkv_tensor_map(&tk, k, B * H, S, DH) != RT_OK ||
      make_qkv_tensor_map(&tv, v, B * H, S, DH) != RT_OK || make_qkv_tensor_map(&tdo, d_o, B * H, S, DH) != RT_OK)
    return RT_ERR_CUDA;  // detail recorded by make_qkv_tensor_map
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(dq_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmem);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(dq_kernel)");
    e = cudaFuncSetAttribute(dkdv_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmem);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(dkdv_kernel)");
    configured[dev] = true;
  }
  const int Sp = plan.tiles * RT_TILE;
  const long long rows_padded = (long long)B * H * Sp;
  const long long threads = rows_padded * (DH / 8);
  row_stats_kernel<DH><<<(unsigned)((threads + 255) / 256), 256, 0, stream>>>(o, d_o, lse, stats, S, Sp,
                                                                              rows_padded);
  if (int st = check_launch("row_stats_kernel launch")) return st;
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(plan.tiles, H, B);
  dkdv_kernel<DH><<<grid, kThreads, C::kDynSmem, stream>>>(tq, tk, tv, tdo, plan, H, S, scale, scale_log2,
                                                            stats, dk, dv);
  if (int st = check_launch("dkdv_kernel launch")) return st;
  dq_kernel<DH><<<grid, kThreads, C::kDynSmem, stream>>>(tq, tk, tv, tdo, plan, H, S, scale, scale_log2, stats,
                                                          dq);
  return check_launch("dq_kernel launch");
}

}  // namespace bwd

int launch_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                         const uint16_t* d_o, const float* lse, int B, int H, int S, int Dh, float scale,
                         const rt_tile_plan& plan, uint16_t* dq, uint16_t* dk, uint16_t* dv, float* stats,
                         cudaStream_t stream) {
  if (Dh == 64) return bwd::launch<64>(q, k, v, o, d_o, lse, B, H, S, scale, plan, dq, dk, dv, stats, stream);
  if (Dh == 32) return bwd::launch<32>(q, k, v, o, d_o, lse, B, H, S, scale, plan, dq, dk, dv, stats, stream);
  return RT_ERR_UNSUPPORTED;
}

}  // namespace rt
