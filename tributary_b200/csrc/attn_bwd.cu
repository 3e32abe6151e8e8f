// Backward masked attention on sm_100a: the gradients jax autodiff takes
// through confluence/confluence/layers.py:83-94 (the reference has no
// hand-written backward; train.py:209 differentiates the forward).
//
//   delta_i = sum_d dO_id O_id                         (row_stats_kernel)
//   p_ij    = mask_ij ? exp(s_ij - lse_i) : 0,  s = scale q k^T
//   dP      = dO V^T ; dS = P o (dP - delta)
//   dQ      = scale * dS K
//   dV      = P^T dO ; dK = scale * dS^T Q
//
// Two paths, both over live tiles only, recomputing P from lse with S
// double-buffered in tensor memory:
// - rt_attention_bwd: dkdvq_kernel, one CTA per (b, h, k-tile) over its k2q
//   list. It computes S, dP and P once per tile and yields all three
//   gradients: dK and dV accumulate in TMEM and are written once, while dQ
//   partials are reduce-added (TMA) into an fp32 workspace accumulator that
//   dq_convert_kernel scales and rounds. dQ is reproducible to fp32 rounding.
//   rt_attention_bwd_qkv runs the same kernel with token-order outputs
//   (TokenGrads): dK and dV leave its epilogue through the k normalisation's
//   Jacobian and the scatter to token order, and dq_qkv_kernel does the same
//   for dQ.
// - rt_attention_bwd_noalloc: dkdv_kernel (k2q lists, thread = key) and
//   dq_kernel (q2k lists, thread = query). Each output element is written once
//   by one CTA, so all three gradients are bit-reproducible; the only scratch
//   is the padded row statistics.
#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {
namespace bwd {

constexpr int kThreads = 576;         // producer, MMA, 16 softmax warps
constexpr int kThreadsFused = 704;    // fused kernel: the same plus four dQ reduce warps (one per TMEM lane quadrant)
constexpr int kSoftmaxThreads = 512;  // four per TMEM lane quadrant, each owning 32 of a row's 128 columns
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
  // Fused dK/dV/dQ kernel. After the Q / dO ring: a ring of row-statistic
  // operand tiles [128 queries][16 bf16] (32-byte swizzle), then two constant
  // 8-row tiles of that shape (ones in columns 0-1, resp. 2-3) that every
  // 8-row group of the MMA's A operand reads (stride 0), then the dS^T tile
  // [2 panels][128 keys][64 queries] bf16 (128-byte swizzle), then one dQ
  // staging ring per reduce warp: DH / 32 + 1 boxes [32 rows][32 fp32]
  // (128-byte swizzle), one box more than a tile's partial needs, so that
  // a box is rewritten only once the reduce issued from it three (DH = 64)
  // or two (DH = 32) boxes earlier has read it.
  static constexpr int kAuxTileBytes = RT_TILE * 32;
  static constexpr int kFAux = kR1 + kStages * kTileBytes;
  static constexpr int kFOnes = kFAux + kStages * kAuxTileBytes;
  static constexpr int kDS = (kFOnes + 512 + 1023) / 1024 * 1024;
  static constexpr int kDSPanel = RT_TILE * 128;
  static constexpr int kStg = kDS + 2 * kDSPanel;
  static constexpr int kStgBox = 32 * 32 * 4;
  static constexpr int kStgBoxesPerTile = DH / 32;
  static constexpr int kStgRing = kStgBoxesPerTile + 1;
  static constexpr int kStgSlot = kStgRing * kStgBox;
  static constexpr int kStgBytes = 4 * kStgSlot;
  static constexpr int kDynSmemFused = kStg + kStgBytes + 1024;
  static_assert(kFAux % 1024 == 0 && kDS % 1024 == 0 && kStg % 1024 == 0, "fused layout alignment");
  static_assert(kDynSmemFused + 2304 <= 227 * 1024, "fused layout and static shared memory exceed 227 KB");
};

constexpr int kMaxTiles = 65536 / RT_TILE;

struct __align__(8) Barriers {
  uint64_t res_full;       // resident pair loaded (Q,dO for dQ; K,V for dK/dV)
  uint64_t ring_full[4];   // ring stage loaded
  uint64_t ring_empty[4];  // ring stage released by the MMAs
  uint64_t st_full[2];     // S (or S^T) buffer b computed
  uint64_t dp_full;        // dP (or dP^T) computed
  uint64_t pa_full;        // softmax phase A done: S buffer read (and P^T written)
  uint64_t pa_full_odd;    // fused kernel: phase A of odd tiles (pa_full takes the even ones)
  uint64_t pb_full;        // softmax phase B done: dS (or dS^T) written
  uint64_t done;           // last gradient MMA complete
  uint64_t dq_ready;       // fused kernel: dQ partial of the tile in TMEM
  uint64_t dq_drained;     // fused kernel: the reduce warps have read the dQ partial out of TMEM
  uint64_t drain;
  uint64_t epi_red;        // fused kernel, token outputs: every softmax warp has written its share of the row sums
};

__device__ __forceinline__ void init_barriers(Barriers& bars, int stages) {
  mbar_init(&bars.res_full, 1);
  for (int s = 0; s < stages; ++s) {
    mbar_init(&bars.ring_full[s], 1);
    mbar_init(&bars.ring_empty[s], 1);
  }
  mbar_init(&bars.st_full[0], 1);
  mbar_init(&bars.st_full[1], 1);
  mbar_init(&bars.dp_full, 1);
  mbar_init(&bars.pa_full, kSoftmaxThreads / 32);  // one arrival per softmax warp
  mbar_init(&bars.pa_full_odd, kSoftmaxThreads / 32);
  mbar_init(&bars.pb_full, kSoftmaxThreads / 32);
  mbar_init(&bars.done, 1);
  mbar_init(&bars.dq_ready, 1);
  mbar_init(&bars.dq_drained, 4);
  mbar_init(&bars.drain, 1);
  mbar_init(&bars.epi_red, kSoftmaxThreads / 32);
  fence_mbar_init();
}

// Softmax phase A for a 32-column slice of one row of a 128x128 tile held in
// TMEM (one row per thread): p = exp2(c * s + nl) with nl = -lse * log2(e),
// masked entries 0, packed as 16 bf16 pairs. `nl_col` (per column, shared
// memory) is used when the rows are keys (dK/dV), `nl_row` when they are
// queries (dQ). `mw` is the mask word of these 32 columns.
template <bool kPerColumn>
__device__ __forceinline__ void softmax_phase_a(uint32_t taddr, bool full, uint32_t mw, float c,
                                                const float* nl_col, float nl_row, uint32_t (&pk)[16]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
  if (!full) {
#pragma unroll
    for (int e = 0; e < 32; ++e) r[e] = ((mw >> e) & 1u) ? r[e] : __float_as_uint(-INFINITY);
  }
  const float2 c2 = make_float2(c, c);
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    float2 nl01, nl23;
    if (kPerColumn) {
      const float4 v = *reinterpret_cast<const float4*>(nl_col + e);
      nl01 = make_float2(v.x, v.y);
      nl23 = make_float2(v.z, v.w);
    } else {
      nl01 = nl23 = make_float2(nl_row, nl_row);
    }
    const float2 x01 = ffma2(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), c2, nl01);
    const float2 x23 = ffma2(make_float2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3])), c2, nl23);
    pk[e >> 1] = pack_bf16x2(fast_exp2(x01.x), fast_exp2(x01.y));
    pk[(e >> 1) + 1] = pack_bf16x2(fast_exp2(x23.x), fast_exp2(x23.y));
  }
}

// Softmax phase B for the same slice: dS = P * (dP - delta) from the 32 dP
// columns at `taddr`, written back as 16 bf16 pairs over the first 16 of
// those columns (read before written; slices of a row never overlap).
template <bool kPerColumn>
__device__ __forceinline__ void softmax_phase_b(uint32_t taddr, const uint32_t (&pk)[16], const float* nd_col,
                                                float nd_row) {
  uint32_t d[32];
  tmem_ld32(taddr, d);
  tmem_wait_ld();
  uint32_t ds[16];
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    float2 nd01, nd23;
    if (kPerColumn) {
      const float4 v = *reinterpret_cast<const float4*>(nd_col + e);
      nd01 = make_float2(v.x, v.y);
      nd23 = make_float2(v.z, v.w);
    } else {
      nd01 = nd23 = make_float2(nd_row, nd_row);
    }
    const float2 g01 = fmul2(unpack_bf16x2(pk[e >> 1]),
                             fadd2(make_float2(__uint_as_float(d[e]), __uint_as_float(d[e + 1])), nd01));
    const float2 g23 = fmul2(unpack_bf16x2(pk[(e >> 1) + 1]),
                             fadd2(make_float2(__uint_as_float(d[e + 2]), __uint_as_float(d[e + 3])), nd23));
    ds[e >> 1] = pack_bf16x2(g01.x, g01.y);
    ds[(e >> 1) + 1] = pack_bf16x2(g23.x, g23.y);
  }
  tmem_st16(taddr, ds);
}

// Phase B math only: dS = P * (dP - delta) from the 32 dP columns at `taddr`,
// returned as 16 bf16 pairs.
template <bool kPerColumn>
__device__ __forceinline__ void softmax_phase_b_ds(uint32_t taddr, const uint32_t (&pk)[16], const float* nd_col,
                                                   float nd_row, uint32_t (&ds)[16]) {
  uint32_t d[32];
  tmem_ld32(taddr, d);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    float2 nd01, nd23;
    if (kPerColumn) {
      const float4 v = *reinterpret_cast<const float4*>(nd_col + e);
      nd01 = make_float2(v.x, v.y);
      nd23 = make_float2(v.z, v.w);
    } else {
      nd01 = nd23 = make_float2(nd_row, nd_row);
    }
    const float2 g01 = fmul2(unpack_bf16x2(pk[e >> 1]),
                             fadd2(make_float2(__uint_as_float(d[e]), __uint_as_float(d[e + 1])), nd01));
    const float2 g23 = fmul2(unpack_bf16x2(pk[(e >> 1) + 1]),
                             fadd2(make_float2(__uint_as_float(d[e + 2]), __uint_as_float(d[e + 3])), nd23));
    ds[e >> 1] = pack_bf16x2(g01.x, g01.y);
    ds[(e >> 1) + 1] = pack_bf16x2(g23.x, g23.y);
  }
}

// TMEM column of the bf16 P / dS operand for MMA k-step ks (16 rows of the
// reduction dimension): column group g = ks / 2 keeps its 32 entries packed
// in columns [32g, 32g + 16).
__device__ __forceinline__ uint32_t packed_col(int ks) { return (uint32_t)((ks >> 1) * 32 + (ks & 1) * 8); }

// Epilogue slice of the DH output columns handled by column group g.
template <int DH>
struct EpiSlice {
  static constexpr int kCols = DH / 4 < 16 ? 16 : DH / 4;
};

// Gradients in token order for the whole sublayer step [gather + QK
// normalisation + attention] (confluence/confluence/layers.py:63-97 and
// 139-142), when dqkv is set: instead of dq, dk, dv in cell order, the
// backward writes the gradient of the token-order projection qkv
// [B][S][3][H][Dh], through the normalisation's Jacobian for q and k, and
// per (b, h, cell) the row's share of d tau. With
//   y = x r, r = 1 / max(|x|, 1e-6), out = s y  (s = tau_h for q, 1 for k),
// and g the gradient of out: dx = r (s g - y yd), yd = s (y . g) while r <
// 1e6 (else 0: the clamped norm is a constant), d tau share = y . g.
struct TokenGrads {
  const uint16_t* perm;  // [B][S] cell order: cell i is token perm[b][i]
  const uint16_t* qkv;   // [B][S][3][H][Dh] the projection the forward normalised
  const float* rnorm;    // [2][B][H][S] r of q, then of k, per cell
  const float* tau;      // [H]
  uint16_t* dqkv;        // [B][S][3][H][Dh]
  float* dtau_rows;      // [B][H][S]
};

// Row statistics for the gradient kernels, padded to whole tiles and stored
// negated so they enter the exponent / difference as FMA addends:
//   stats[bh][0][q] = -lse[bh][q] * log2(e)                 (0 for q >= S)
//   stats[bh][1][q] = -sum_d dO[bh][q][d] * O[bh][q][d]     (0 for q >= S)
// when stats is given (the two-kernel path), and, when aux is given, the fused
// kernel's operand row per padded query:
//   aux[bh * Sp + q] = bf16 (a_hi, a_lo, d_hi, d_lo, 0 x 12),
//   a = -lse / scale, d = -sum_d dO O, x_hi = bf16(x), x_lo = bf16(x - x_hi),
// and, when dq_acc is given, zeroes the fused kernel's fp32 dQ accumulator
// dq_acc [bh * Sp + q][DH] (each thread clears the 8 columns it reads).
template <int DH>
__global__ void __launch_bounds__(256) row_stats_kernel(const uint16_t* __restrict__ o,
                                                        const uint16_t* __restrict__ d_o,
                                                        const float* __restrict__ lse,
                                                        float* __restrict__ stats, uint16_t* __restrict__ aux,
                                                        float* __restrict__ dq_acc, float inv_scale, int S, int Sp,
                                                        long long rows_padded) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
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
  if (dq_acc != nullptr && prow < rows_padded) {
    float4* z = reinterpret_cast<float4*>(dq_acc + prow * DH + sub * 8);
    z[0] = make_float4(0.f, 0.f, 0.f, 0.f);
    z[1] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  if (prow < rows_padded && sub == 0) {
    const float l = in ? lse[bh * S + q] : 0.f;
    if (stats != nullptr) {
      float* st = stats + bh * 2 * Sp;
      st[q] = in ? -l * 1.4426950408889634f : 0.f;
      st[Sp + q] = -acc;
    }
    if (aux != nullptr) {
      const float a = -l * inv_scale, d = -acc;
      const float a_hi = __bfloat162float(__float2bfloat16_rn(a));
      const float d_hi = __bfloat162float(__float2bfloat16_rn(d));
      uint4* dst = reinterpret_cast<uint4*>(aux + prow * 16);
      dst[0] = make_uint4(pack_bf16x2(a_hi, a - a_hi), pack_bf16x2(d_hi, d - d_hi), 0u, 0u);
      dst[1] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
}

__device__ __forceinline__ void store_row_bf16(uint16_t* dst, const uint32_t (&pk)[8]) {
  uint4* d = reinterpret_cast<uint4*>(dst);
  d[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  d[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
}

// ---------------------------------------------------------------------------
// dQ: one CTA per (b, h, q-tile); thread = query row.
// TMEM: S0 [0,128), S1 [128,256) fp32 (double buffered), dP [256,384) fp32
// with dS written as bf16 pairs over columns [32g, 32g+16) of it (one run per
// 32-column slice g), dQ [384,384+DH). Sixteen softmax warps: four per TMEM
// lane quadrant, each owning 32 of the 128 columns.
// Per k-tile j: the MMA thread issues S_{j+1} as soon as softmax phase A has
// read S_j, so QK^T overlaps phase B; dP_{j+1} follows dQ += dS_j K_j and
// overlaps the next phase A.
// ---------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(kThreads, 1)
    dq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
              const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
              const rt_tile_plan plan, int H, int S, float scale, float scale_log2,
              const float* __restrict__ stats, uint16_t* __restrict__ dq) {
  using C = Cfg<DH>;
  constexpr int kS0 = 0, kDP = 256, kDQ = 384;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ int s_list[kMaxTiles];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int row_list = b * T + qt;
  const int list_begin = plan.q2k_ptr[row_list];
  const int n_tiles = plan.q2k_ptr[row_list + 1] - list_begin;
  for (int i = threadIdx.x; i < n_tiles; i += kThreads) s_list[i] = plan.q2k_idx[list_begin + i];

  if (threadIdx.x == 0) {
    abort_flag = 0;
    init_barriers(bars, C::kStages);
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
        const int kt = s_list[j] & 0x7FFFFFFF;
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
      auto k_addr = [&](int j) { return smem_u32(smem + C::kR0 + (j % C::kStages) * C::kTileBytes); };
      auto v_addr = [&](int j) { return smem_u32(smem + C::kR1 + (j % C::kStages) * C::kTileBytes); };
      auto issue_s = [&](int j) {  // S[j%2] = Q K_j^T
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks)
          mma_ss(tmem + kS0 + (j & 1) * 128, sdesc(q_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                 sdesc(k_addr(j) + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
        mma_commit(&bars.st_full[j & 1]);
      };
      auto issue_dp = [&](int j) {  // dP = dO V_j^T
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks)
          mma_ss(tmem + kDP, sdesc(do_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                 sdesc(v_addr(j) + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
        mma_commit(&bars.dp_full);
      };
      bool ok = mbar_wait(&bars.res_full, 0, &abort_flag) && mbar_wait(&bars.ring_full[0], 0, &abort_flag);
      tc_fence_after();
      if (ok) {
        issue_s(0);
        issue_dp(0);
      }
      // S_{j+1} is issued only once phase A of tile j has been observed, so no
      // barrier can run two phases ahead of its waiter.
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (!(ok = mbar_wait(&bars.pa_full, j & 1, &abort_flag))) break;
        tc_fence_after();
        if (j + 1 < n_tiles) {
          if (!(ok = mbar_wait(&bars.ring_full[(j + 1) % C::kStages], ((j + 1) / C::kStages) & 1, &abort_flag)))
            break;
          tc_fence_after();
          issue_s(j + 1);
        }
        if (!(ok = mbar_wait(&bars.pb_full, j & 1, &abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < RT_TILE / 16; ++ks)
          mma_ts(tmem + kDQ, tmem + kDP + packed_col(ks),
                 sdesc(k_addr(j) + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle), idesc_q,
                 (j > 0 || ks > 0) ? 1u : 0u);
        mma_commit(&bars.ring_empty[j % C::kStages]);
        if (j + 1 < n_tiles) issue_dp(j + 1);
      }
      mma_commit(&bars.done);
      mma_commit(&bars.drain);
      volatile int no_abort = 0;
      mbar_wait(&bars.drain, 0, &no_abort);
    }
  } else {
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;  // column group: columns [32 grp, 32 grp + 32) of every tile
    const int row = quad * 32 + lane;
    const int q = qt * RT_TILE + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t col0 = (uint32_t)(grp * 32);
    const uint32_t* masks = plan.tile_masks + ((size_t)row_list * T) * RT_TILE * 4 + grp;
    const int Sp = T * RT_TILE;
    const float nl = stats[(size_t)bh * 2 * Sp + q];
    const float nd = stats[(size_t)bh * 2 * Sp + Sp + q];
    auto load_mask = [&](int ent) {
      return ent >= 0 ? __ldg(masks + ((size_t)(ent & 0x7FFFFFFF) * RT_TILE + row) * 4) : 0xFFFFFFFFu;
    };
    uint32_t mk_next = n_tiles > 0 ? load_mask(s_list[0]) : 0u;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const bool full = s_list[j] < 0;
      const uint32_t mk = mk_next;
      if (j + 1 < n_tiles) mk_next = load_mask(s_list[j + 1]);
      if (!(ok = mbar_wait(&bars.st_full[j & 1], (j >> 1) & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t pk[16];
      softmax_phase_a<false>(lane_base + kS0 + (j & 1) * 128 + col0, full, mk, scale_log2, nullptr, nl, pk);
      tc_fence_before();
      mbar_arrive_warp(&bars.pa_full);
      if (!(ok = mbar_wait(&bars.dp_full, j & 1, &abort_flag))) break;
      tc_fence_after();
      softmax_phase_b<false>(lane_base + kDP + col0, pk, nullptr, nd);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(&bars.pb_full);
    }
    if (ok && n_tiles > 0 && mbar_wait(&bars.done, 0, &abort_flag)) {
      tc_fence_after();
      uint16_t* dst = dq + ((size_t)bh * S + q) * DH;
#pragma unroll
      for (int c = grp * EpiSlice<DH>::kCols; c < (grp + 1) * EpiSlice<DH>::kCols && c < DH; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_base + kDQ + c, r);
        tmem_wait_ld();
        uint32_t pko[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pko[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale);
        if (q < S) store_row_bf16(dst + c, pko);
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
// TMEM: S^T0 [0,128), S^T1 [128,256) fp32 (double buffered; P^T overwrites
// columns [32g, 32g+16) as bf16 pairs, one run per 32-column slice g), dP^T
// [256,384) fp32 (dS^T likewise), dV [384,384+DH), dK [384+DH,384+2DH).
// Sixteen softmax warps: four per TMEM lane quadrant, each owning 32 columns.
// Per q-tile i: S^T_{i+1} then dV_i follow softmax phase A (overlapping phase
// B and the next phase A), dK_i and dP^T_{i+1} follow phase B.
// ---------------------------------------------------------------------------
template <int DH>
__global__ void __launch_bounds__(kThreads, 1)
    dkdv_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const rt_tile_plan plan, int H, int S, float scale, float scale_log2,
                const float* __restrict__ stats, uint16_t* __restrict__ dk, uint16_t* __restrict__ dv) {
  using C = Cfg<DH>;
  constexpr int kST0 = 0, kDPT = 256, kDV = 384, kDK = 384 + DH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ int s_list[kMaxTiles];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int col_list = b * T + kt;
  const int list_begin = plan.k2q_ptr[col_list];
  const int n_tiles = plan.k2q_ptr[col_list + 1] - list_begin;
  const int Sp = T * RT_TILE;
  for (int i = threadIdx.x; i < n_tiles; i += kThreads) s_list[i] = plan.k2q_idx[list_begin + i];

  if (threadIdx.x == 0) {
    abort_flag = 0;
    init_barriers(bars, C::kStages);
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
        const int qtile = s_list[i] & 0x7FFFFFFF;
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
      auto q_addr = [&](int i) { return smem_u32(smem + C::kR0 + (i % C::kStages) * C::kTileBytes); };
      auto do_addr = [&](int i) { return smem_u32(smem + C::kR1 + (i % C::kStages) * C::kTileBytes); };
      auto issue_st = [&](int i) {  // S^T[i%2] = K Q_i^T
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks)
          mma_ss(tmem + kST0 + (i & 1) * 128, sdesc(k_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                 sdesc(q_addr(i) + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
        mma_commit(&bars.st_full[i & 1]);
      };
      auto issue_dpt = [&](int i) {  // dP^T = V dO_i^T
#pragma unroll
        for (int ks = 0; ks < DH / 16; ++ks)
          mma_ss(tmem + kDPT, sdesc(v_addr + ks * 32, 16, C::kSBO, C::kSwizzle),
                 sdesc(do_addr(i) + ks * 32, 16, C::kSBO, C::kSwizzle), idesc_s, ks > 0 ? 1u : 0u);
        mma_commit(&bars.dp_full);
      };
      bool ok = mbar_wait(&bars.res_full, 0, &abort_flag) && mbar_wait(&bars.ring_full[0], 0, &abort_flag);
      tc_fence_after();
      if (ok) {
        issue_st(0);
        issue_dpt(0);
      }
      // S^T_{i+1} is issued only once phase A of tile i has been observed, so
      // no barrier can run two phases ahead of its waiter.
      for (int i = 0; ok && i < n_tiles; ++i) {
        if (!(ok = mbar_wait(&bars.pa_full, i & 1, &abort_flag))) break;
        tc_fence_after();
        // S^T_{i+1} first: the softmax warps start its phase A while dV_i
        // runs (MMA issue blocks for the MMA's duration, so issuing dV_i
        // first would put it on the softmax's critical path). S^T_{i+1}
        // targets the other buffer; dV_i reads P^T_i from this one.
        if (i + 1 < n_tiles) {
          if (!(ok = mbar_wait(&bars.ring_full[(i + 1) % C::kStages], ((i + 1) / C::kStages) & 1, &abort_flag)))
            break;
          tc_fence_after();
          issue_st(i + 1);
        }
#pragma unroll
        for (int ks = 0; ks < RT_TILE / 16; ++ks)  // dV += P^T_i dO_i
          mma_ts(tmem + kDV, tmem + kST0 + (i & 1) * 128 + packed_col(ks),
                 sdesc(do_addr(i) + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle), idesc_g,
                 (i > 0 || ks > 0) ? 1u : 0u);
        if (!(ok = mbar_wait(&bars.pb_full, i & 1, &abort_flag))) break;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < RT_TILE / 16; ++ks)  // dK += dS^T_i Q_i
          mma_ts(tmem + kDK, tmem + kDPT + packed_col(ks),
                 sdesc(q_addr(i) + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle), idesc_g,
                 (i > 0 || ks > 0) ? 1u : 0u);
        mma_commit(&bars.ring_empty[i % C::kStages]);
        if (i + 1 < n_tiles) issue_dpt(i + 1);
      }
      mma_commit(&bars.done);
      mma_commit(&bars.drain);
      volatile int no_abort = 0;
      mbar_wait(&bars.drain, 0, &no_abort);
    }
  } else {
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;  // column group: queries [32 grp, 32 grp + 32) of every tile
    const int row = quad * 32 + lane;  // key within the tile
    const int key = kt * RT_TILE + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t col0 = (uint32_t)(grp * 32);
    const uint32_t* masks_t = plan.tile_masks_t + ((size_t)col_list * T) * RT_TILE * 4 + grp;
    auto load_mask = [&](int ent) {
      return ent >= 0 ? __ldg(masks_t + ((size_t)(ent & 0x7FFFFFFF) * RT_TILE + row) * 4) : 0xFFFFFFFFu;
    };
    uint32_t mk_next = n_tiles > 0 ? load_mask(s_list[0]) : 0u;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const bool full = s_list[i] < 0;
      const uint32_t mk = mk_next;
      if (i + 1 < n_tiles) mk_next = load_mask(s_list[i + 1]);
      const int stage = i % C::kStages;
      if (!(ok = mbar_wait(&bars.ring_full[stage], (i / C::kStages) & 1, &abort_flag))) break;
      const float* nl = reinterpret_cast<const float*>(smem + C::kRL + stage * C::kRowStatBytes) + col0;
      const float* nd = nl + RT_TILE;
      if (!(ok = mbar_wait(&bars.st_full[i & 1], (i >> 1) & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t pk[16];
      const uint32_t st_addr = lane_base + kST0 + (i & 1) * 128 + col0;
      softmax_phase_a<true>(st_addr, full, mk, scale_log2, nl, 0.f, pk);
      tmem_st16(st_addr, pk);  // P^T over the first 16 columns of this slice
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(&bars.pa_full);
      if (!(ok = mbar_wait(&bars.dp_full, i & 1, &abort_flag))) break;
      tc_fence_after();
      softmax_phase_b<true>(lane_base + kDPT + col0, pk, nd, 0.f);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp(&bars.pb_full);
    }
    if (ok && n_tiles > 0 && mbar_wait(&bars.done, 0, &abort_flag)) {
      tc_fence_after();
      uint16_t* dst_v = dv + ((size_t)bh * S + key) * DH;
      uint16_t* dst_k = dk + ((size_t)bh * S + key) * DH;
#pragma unroll
      for (int c = grp * EpiSlice<DH>::kCols; c < (grp + 1) * EpiSlice<DH>::kCols && c < DH; c += 16) {
        uint32_t r[16], pko[8];
        tmem_ld16(lane_base + kDV + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2) pko[e / 2] = pack_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
        if (key < S) store_row_bf16(dst_v + c, pko);
        tmem_ld16(lane_base + kDK + c, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pko[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale);
        if (key < S) store_row_bf16(dst_k + c, pko);
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
// Fused dK, dV and dQ: one CTA per (b, h, k-tile), dkdv_kernel's pipeline plus
// dQ, so S, dP and P are computed once per live tile instead of twice.
//
// Row statistics ride in the MMAs. row_stats_kernel writes per query q an
// operand row aux[q] = (a_hi, a_lo, d_hi, d_lo, 0, ...) in bf16 with
// a = -lse[q] / scale and d = -delta[q], each split into two bf16 parts whose
// sum is exact to 2^-16 relative. One extra 16-deep k-step per product
// multiplies it by a constant tile of ones (columns 0-1 for S, 2-3 for dP), so
// TMEM receives S'^T = K Q^T + a and dP'^T = V dO^T - delta directly: then
//   p = exp2(scale * log2(e) * S'^T)        dS = P o dP'^T
// and the softmax warps read nothing but TMEM (warp-uniform per-column
// statistics from shared memory cost four wavefronts per 16-byte load and
// competed with the tensor core's operand reads for shared-memory bandwidth).
//
// Phase B writes dS^T (bf16) to a shared-memory tile [2 panels][128 keys][64
// queries] with the 128-byte swizzle instead of TMEM. The MMAs read it twice:
// as dS^T, K-major (dK += dS^T Q_i), and as dS, MN-major over both panels
// (dQ_i = dS K, M = the 128 queries). dQ_i lands over columns [0, DH) of the
// S^T buffer that dV_i has just consumed. Four reduce warps, one per TMEM lane
// quadrant, copy it out (32 queries x DH each), arrive on dq_drained -- the
// MMA issuer waits for that before S^T_{i+2} reuses the buffer -- and then
// stage it in shared memory (128-byte swizzle, conflict-free) and reduce-add
// it into the fp32 accumulator dq_acc [B*H][S padded][DH] with TMA
// (cp.reduce.async.bulk.tensor), each warp on its own slot and bulk group.
// The softmax warps never touch dQ.
// dq_convert_kernel scales and rounds dq_acc afterwards. Every dQ row block gets one partial per
// live key tile in an order the memory system decides, so dQ is reproducible
// to fp32 rounding; dK and dV are written once.
// TMEM as dkdv_kernel: S^T0 [0,128), S^T1 [128,256), dP^T [256,384), dV, dK.
// ---------------------------------------------------------------------------

// Phase A with the statistics already in the accumulator: p = exp2(c * s').
__device__ __forceinline__ void softmax_phase_a_aux(uint32_t taddr, bool full, uint32_t mw, float c,
                                                    uint32_t (&pk)[16]) {
  uint32_t r[32];
  tmem_ld32(taddr, r);
  tmem_wait_ld();
  if (!full) {
#pragma unroll
    for (int e = 0; e < 32; ++e) r[e] = ((mw >> e) & 1u) ? r[e] : __float_as_uint(-INFINITY);
  }
  const float2 c2 = make_float2(c, c);
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    const float2 x01 = fmul2(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), c2);
    const float2 x23 = fmul2(make_float2(__uint_as_float(r[e + 2]), __uint_as_float(r[e + 3])), c2);
    pk[e >> 1] = pack_bf16x2(fast_exp2(x01.x), fast_exp2(x01.y));
    pk[(e >> 1) + 1] = pack_bf16x2(fast_exp2(x23.x), fast_exp2(x23.y));
  }
}

// Phase B with delta already subtracted: dS = P o dP'.
__device__ __forceinline__ void softmax_phase_b_aux(uint32_t taddr, const uint32_t (&pk)[16], uint32_t (&ds)[16]) {
  uint32_t d[32];
  tmem_ld32(taddr, d);
  tmem_wait_ld();
#pragma unroll
  for (int e = 0; e < 32; e += 4) {
    const float2 g01 = fmul2(unpack_bf16x2(pk[e >> 1]), make_float2(__uint_as_float(d[e]), __uint_as_float(d[e + 1])));
    const float2 g23 =
        fmul2(unpack_bf16x2(pk[(e >> 1) + 1]), make_float2(__uint_as_float(d[e + 2]), __uint_as_float(d[e + 3])));
    ds[e >> 1] = pack_bf16x2(g01.x, g01.y);
    ds[(e >> 1) + 1] = pack_bf16x2(g23.x, g23.y);
  }
}

template <int DH, bool kTok>
__global__ void __launch_bounds__(kThreadsFused, 1)
    dkdvq_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_do,
                const __grid_constant__ CUtensorMap tm_aux, const rt_tile_plan plan, int H, int S, float scale,
                float scale_log2, uint16_t* __restrict__ dk, uint16_t* __restrict__ dv,
                const __grid_constant__ CUtensorMap tm_acc, const TokenGrads tg) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  using C = Cfg<DH>;
  constexpr int kST0 = 0, kDPT = 256, kDV = 384, kDK = 384 + DH;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;
  __shared__ int s_list[kMaxTiles];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int kt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int col_list = b * T + kt;
  const int list_begin = plan.k2q_ptr[col_list];
  const int n_tiles = plan.k2q_ptr[col_list + 1] - list_begin;
  const int Sp = T * RT_TILE;
  for (int i = threadIdx.x; i < n_tiles; i += kThreadsFused) s_list[i] = plan.k2q_idx[list_begin + i];
  // Constant ones tiles [2][8 rows][16 bf16], 32-byte swizzle (the 16-byte
  // half j of row r sits at half j ^ ((r >> 2) & 1)): tile 0 has 1.0 in
  // columns 0-1, tile 1 in columns 2-3. 32 threads write 16 bytes each.
  if (threadIdx.x < 32) {
    const int off = threadIdx.x * 16;
    const int tile = off >> 8, row = (off & 255) >> 5, half = (off & 31) >> 4;
    const bool logical0 = (half ^ ((row >> 2) & 1)) == 0;
    const uint32_t ones = 0x3F803F80u;  // two bf16 1.0
    uint4 val = make_uint4(0u, 0u, 0u, 0u);
    if (logical0) {
      if (tile == 0) val.x = ones;
      else val.y = ones;
    }
    *reinterpret_cast<uint4*>(smem + C::kFOnes + off) = val;
    fence_proxy_async_smem();
  }

  // Q, dO and the row-statistic rows of the i-th live q-tile into ring stage i % kStages
  auto load_tile = [&](int i, int qtile) {
    const int s = i % C::kStages;
    mbar_arrive_expect_tx(&bars.ring_full[s], 2 * C::kTileBytes + C::kAuxTileBytes);
    tma_load_3d(smem + C::kR0 + s * C::kTileBytes, &tm_q, &bars.ring_full[s], 0, qtile * RT_TILE, bh);
    tma_load_3d(smem + C::kR1 + s * C::kTileBytes, &tm_do, &bars.ring_full[s], 0, qtile * RT_TILE, bh);
    tma_load_2d(smem + C::kFAux + s * C::kAuxTileBytes, &tm_aux, &bars.ring_full[s], 0, bh * Sp + qtile * RT_TILE);
  };
  // The producer thread starts K, V and the first ring stages as soon as the
  // barriers exist, so their latency overlaps the TMEM allocation, the list
  // copy and the block barrier below (the list entries come from global
  // memory here; s_list is not complete yet).
  const int n_early = min(n_tiles, C::kStages);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    init_barriers(bars, C::kStages);
    if (n_tiles > 0) {
      mbar_arrive_expect_tx(&bars.res_full, 2 * C::kTileBytes);
      tma_load_3d(smem + C::kA0, &tm_k, &bars.res_full, 0, kt * RT_TILE, bh);
      tma_load_3d(smem + C::kA1, &tm_v, &bars.res_full, 0, kt * RT_TILE, bh);
      for (int i = 0; i < n_early; ++i) load_tile(i, plan.k2q_idx[list_begin + i] & 0x7FFFFFFF);
    }
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
      int i = n_early;
      for (; i < n_tiles; ++i) {
        const int s = i % C::kStages;
        if (!mbar_wait(&bars.ring_empty[s], ((i / C::kStages) - 1) & 1, &abort_flag)) break;
        load_tile(i, s_list[i] & 0x7FFFFFFF);
      }
      volatile int no_abort = 0;
      for (int ii = max(0, i - C::kStages); ii < i; ++ii)
        mbar_wait(&bars.ring_full[ii % C::kStages], (ii / C::kStages) & 1, &no_abort);
      mbar_wait(&bars.res_full, 0, &no_abort);
    }
  } else if (warp == 1) {
    // ---------------- MMA issue: the whole warp waits, one elected lane issues ----------------
    if (n_tiles > 0) {
      const bool leader = elect_one_sync();
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_g = idesc_bf16_f32(128, DH, false, true);
      constexpr uint32_t idesc_dq = idesc_bf16_f32(128, DH, true, true);
      // descriptor start addresses advance in 16-byte units: +2 per 16-deep
      // k-step along a K-major row, +kRowBytes per 16 rows of an MN-major tile
      constexpr uint32_t kRowStep = C::kRowBytes;
      const uint64_t k_kmaj = sdesc(smem_u32(smem + C::kA0), 16, C::kSBO, C::kSwizzle);
      const uint64_t v_kmaj = sdesc(smem_u32(smem + C::kA1), 16, C::kSBO, C::kSwizzle);
      const uint64_t k_mn = sdesc(smem_u32(smem + C::kA0), 0, C::kSBO, C::kSwizzle);
      const uint64_t ds_mn = sdesc(smem_u32(smem + C::kDS), C::kDSPanel, 1024, SW_128B);
      const uint64_t ds_kmaj = sdesc(smem_u32(smem + C::kDS), 16, 1024, SW_128B);
      // the 8-row ones tiles with a zero stride between 8-row groups: every group reads the same rows
      const uint64_t ones_s = sdesc(smem_u32(smem + C::kFOnes), 16, 0, SW_32B);
      const uint64_t ones_dp = sdesc(smem_u32(smem + C::kFOnes + 256), 16, 0, SW_32B);
      auto ring_desc = [&](int base, int i, uint32_t lbo) {
        return sdesc(smem_u32(smem + base + (i % C::kStages) * C::kTileBytes), lbo, C::kSBO, C::kSwizzle);
      };
      auto aux_desc = [&](int i) {
        return sdesc(smem_u32(smem + C::kFAux + (i % C::kStages) * C::kAuxTileBytes), 16, 256, SW_32B);
      };
      auto issue_st = [&](int i) {  // S'^T[i%2] = K Q_i^T + a
        const uint64_t qd = ring_desc(C::kR0, i, 16), ad = aux_desc(i);
        const uint32_t d = tmem + kST0 + (i & 1) * 128;
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) mma_ss(d, k_kmaj + ks * 2, qd + ks * 2, idesc_s, ks > 0 ? 1u : 0u);
          mma_ss(d, ones_s, ad, idesc_s, 1u);
          mma_commit(&bars.st_full[i & 1]);
        }
        __syncwarp();
      };
      auto issue_dpt = [&](int i) {  // dP'^T = V dO_i^T - delta
        const uint64_t dd = ring_desc(C::kR1, i, 16), ad = aux_desc(i);
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks)
            mma_ss(tmem + kDPT, v_kmaj + ks * 2, dd + ks * 2, idesc_s, ks > 0 ? 1u : 0u);
          mma_ss(tmem + kDPT, ones_dp, ad, idesc_s, 1u);
          mma_commit(&bars.dp_full);
        }
        __syncwarp();
      };
      // S'^T runs two tiles ahead: S'^T_{i+2} is issued as soon as its buffer
      // (i % 2) is free -- dV_i has read P^T_i from it (in-order pipe) and the
      // reduce warps have drained dQ_i -- instead of after phase A of tile
      // i + 1, so the softmax finds every S'^T waiting for it. Phase A
      // arrives on pa_full / pa_full_odd by tile parity: with S'^T_{i+1}
      // already issued, the softmax can finish phase A of tile i + 1 before
      // this warp has waited for tile i.
      bool ok = mbar_wait_warp(&bars.res_full, 0, &abort_flag) && mbar_wait_warp(&bars.ring_full[0], 0, &abort_flag);
      tc_fence_after();
      if (ok) {
        issue_st(0);
        issue_dpt(0);
        if (n_tiles > 1 && (ok = mbar_wait_warp(&bars.ring_full[1], 0, &abort_flag))) {
          tc_fence_after();
          issue_st(1);
        }
      }
      for (int i = 0; ok && i < n_tiles; ++i) {
        if (!(ok = mbar_wait_warp((i & 1) ? &bars.pa_full_odd : &bars.pa_full, (i >> 1) & 1, &abort_flag))) break;
        tc_fence_after();
        const uint64_t dom = ring_desc(C::kR1, i, 0), qm = ring_desc(C::kR0, i, 0);
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks)  // dV += P^T_i dO_i
            mma_ts(tmem + kDV, tmem + kST0 + (i & 1) * 128 + packed_col(ks), dom + ks * kRowStep, idesc_g,
                   (i > 0 || ks > 0) ? 1u : 0u);
        }
        __syncwarp();
        if (!(ok = mbar_wait_warp(&bars.pb_full, i & 1, &abort_flag))) break;
        tc_fence_after();
        if (leader) {
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks)  // dQ_i = dS K (A: the dS^T tile read MN-major over both panels)
            mma_ss(tmem + kST0 + (i & 1) * 128, ds_mn + ks * 128, k_mn + ks * kRowStep, idesc_dq, ks > 0 ? 1u : 0u);
          mma_commit(&bars.dq_ready);
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks)  // dK += dS^T_i Q_i (A: the same tile, K-major)
            mma_ss(tmem + kDK, ds_kmaj + (ks >> 2) * (C::kDSPanel / 16) + (ks & 3) * 2, qm + ks * kRowStep, idesc_g,
                   (i > 0 || ks > 0) ? 1u : 0u);
          mma_commit(&bars.ring_empty[i % C::kStages]);
        }
        __syncwarp();
        if (i + 1 < n_tiles) {
          issue_dpt(i + 1);  // its ring stage was waited for when S'^T_{i+1} was issued
          // dQ_i out of buffer i % 2 before S'^T_{i+2} lands there; this wait also
          // keeps dQ_{i+1} from completing dq_ready's next phase before every
          // reduce warp has taken this one
          if (!(ok = mbar_wait_warp(&bars.dq_drained, i & 1, &abort_flag))) break;
          if (i + 2 < n_tiles) {
            if (!(ok = mbar_wait_warp(&bars.ring_full[(i + 2) % C::kStages], ((i + 2) / C::kStages) & 1, &abort_flag)))
              break;
            tc_fence_after();
            issue_st(i + 2);
          }
        }
      }
      if (leader) {
        mma_commit(&bars.done);
        mma_commit(&bars.drain);
      }
      __syncwarp();
      volatile int no_abort = 0;
      mbar_wait_warp(&bars.drain, 0, &no_abort);
    }
  } else if (warp >= 2 + kSoftmaxThreads / 32) {
    // ---------------- dQ reduce warps ----------------
    // Warp w reads TMEM lanes [32 (w % 4), +32): queries 32 quad + lane of the
    // tile, all DH columns. Its slot is a ring of kStgRing boxes [32
    // rows][32 fp32], 16-byte chunk c of row r at chunk c ^ (r % 8) (the
    // 128-byte swizzle). Each box is reduced as its own bulk group; before
    // a box is rewritten, only the reduce issued kStgRing boxes earlier (the
    // box's previous use) must have read it, not every earlier one.
    const int quad = warp & 3;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    uint8_t* slot = smem + C::kStg + (warp - 2 - kSoftmaxThreads / 32) * C::kStgSlot;
    int rb = 0;  // ring position of the next box
    // Token-order outputs (TokenGrads): the softmax warps' epilogue reads each
    // key row's order entry and k inverse norm; they start on their way into
    // L2 now, while this warp has nothing to drain yet.
    if (kTok) {
      const int key = kt * RT_TILE + quad * 32 + lane;
      if (key < S) {
        prefetch_l2(tg.perm + (size_t)b * S + key);
        prefetch_l2(tg.rnorm + ((size_t)(gridDim.z + b) * H + h) * S + key);
      }
    }
    for (int t = 0; t < n_tiles; ++t) {
      if (!mbar_wait_warp(&bars.dq_ready, t & 1, &abort_flag)) break;
      tc_fence_after();
      uint32_t r[DH];
#pragma unroll
      for (int x = 0; x < DH / 32; ++x)
        tmem_ld32(lane_base + kST0 + (t & 1) * 128 + x * 32, *reinterpret_cast<uint32_t(*)[32]>(r + x * 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive_warp(&bars.dq_drained);
      const int row0 = bh * Sp + (s_list[t] & 0x7FFFFFFF) * RT_TILE + quad * 32;
#pragma unroll
      for (int x = 0; x < C::kStgBoxesPerTile; ++x) {
        uint8_t* box = slot + rb * C::kStgBox;
        // at most kStgRing - 1 groups still reading: the box's previous reduce is done with it
        if (lane == 0) bulk_wait_read<C::kStgRing - 1>();
        __syncwarp();
        uint8_t* srow = box + lane * 128;
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<uint4*>(srow + ((c ^ (lane & 7)) << 4)) =
              make_uint4(r[x * 32 + 4 * c], r[x * 32 + 4 * c + 1], r[x * 32 + 4 * c + 2], r[x * 32 + 4 * c + 3]);
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_2d(&tm_acc, box, x * 32, row0);
          bulk_commit_group();
        }
        rb = rb + 1 == C::kStgRing ? 0 : rb + 1;
      }
    }
    // Every reduce this warp issued has completed, its additions into dq_acc
    // included: a wait for the reads alone would let the block exit with
    // additions in flight, and nothing orders those before dq_convert_kernel.
    if (lane == 0) bulk_wait_all();
  } else {
    const int quad = warp & 3;
    const int grp = (warp - 2) >> 2;  // column group: queries [32 grp, 32 grp + 32) of every tile
    const int row = quad * 32 + lane;  // key within the tile
    const int key = kt * RT_TILE + row;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t col0 = (uint32_t)(grp * 32);
    const uint32_t* masks_t = plan.tile_masks_t + ((size_t)col_list * T) * RT_TILE * 4 + grp;
    auto load_mask = [&](int ent) {
      return ent >= 0 ? __ldg(masks_t + ((size_t)(ent & 0x7FFFFFFF) * RT_TILE + row) * 4) : 0xFFFFFFFFu;
    };
    uint32_t mk_next = n_tiles > 0 ? load_mask(s_list[0]) : 0u;
    bool ok = true;
    for (int i = 0; i < n_tiles; ++i) {
      const bool full = s_list[i] < 0;
      const uint32_t mk = mk_next;
      if (i + 1 < n_tiles) mk_next = load_mask(s_list[i + 1]);
      if (!(ok = mbar_wait_warp(&bars.st_full[i & 1], (i >> 1) & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t pk[16];
      const uint32_t st_addr = lane_base + kST0 + (i & 1) * 128 + col0;
      // a 32 x 32 block of the tile with no live element: P = dS = 0, nothing to load or exponentiate
      const bool zero = !full && __all_sync(0xFFFFFFFFu, mk == 0u);
      if (zero) {
#pragma unroll
        for (int e = 0; e < 16; ++e) pk[e] = 0u;
      } else {
        softmax_phase_a_aux(st_addr, full, mk, scale_log2, pk);
      }
      tmem_st16(st_addr, pk);  // P^T over the first 16 columns of this slice
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive_warp((i & 1) ? &bars.pa_full_odd : &bars.pa_full);
      if (!(ok = mbar_wait_warp(&bars.dp_full, i & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t ds[16];
      if (zero) {
#pragma unroll
        for (int e = 0; e < 16; ++e) ds[e] = 0u;
      } else {
        softmax_phase_b_aux(lane_base + kDPT + col0, pk, ds);
      }
      // dS^T row `row`, queries [32 grp, 32 grp + 32): panel grp / 2, 16-byte
      // chunks (grp % 2) * 4 + c of the row, stored at chunk ^ (row % 8)
      uint8_t* drow = smem + C::kDS + (grp >> 1) * C::kDSPanel + row * 128;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int chunk = (grp & 1) * 4 + c;
        *reinterpret_cast<uint4*>(drow + ((chunk ^ (row & 7)) << 4)) =
            make_uint4(ds[4 * c], ds[4 * c + 1], ds[4 * c + 2], ds[4 * c + 3]);
      }
      fence_proxy_async_smem();  // the tensor core reads the tile through the async proxy
      tc_fence_before();
      mbar_arrive_warp(&bars.pb_full);
    }
    if (ok && n_tiles > 0 && mbar_wait_warp(&bars.done, 0, &abort_flag)) {
      tc_fence_after();
      if (!kTok) {
        uint16_t* dst_v = dv + ((size_t)bh * S + key) * DH;
        uint16_t* dst_k = dk + ((size_t)bh * S + key) * DH;
#pragma unroll
        for (int c = grp * EpiSlice<DH>::kCols; c < (grp + 1) * EpiSlice<DH>::kCols && c < DH; c += 16) {
          uint32_t r[16], pko[8];
          tmem_ld16(lane_base + kDV + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 2) pko[e / 2] = pack_bf16x2(__uint_as_float(r[e]), __uint_as_float(r[e + 1]));
          if (key < S) store_row_bf16(dst_v + c, pko);
          tmem_ld16(lane_base + kDK + c, r);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 2)
            pko[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * scale, __uint_as_float(r[e + 1]) * scale);
          if (key < S) store_row_bf16(dst_k + c, pko);
        }
      } else {
        // token order (TokenGrads): dv scattered to the key's token, dk
        // through the k normalisation's Jacobian. Each warp holds 16 columns
        // of its 32 key rows (none for column groups past Dh). y = x r is
        // k_hat, the row of the resident K tile (the bf16 value the forward
        // used), so y . g needs no global load: each warp forms its share
        // from TMEM and shared memory, and the four shares of a row are added
        // in a fixed order through shared memory (the dS^T tile, which no MMA
        // reads any more) behind a bounded barrier.
        const int c = grp * 16;
        const bool has = c < DH;
        const bool kin = key < S;
        const int tok = kin ? min((int)tg.perm[(size_t)b * S + key], S - 1) : 0;  // clamps as the prepass does
        const float rk = kin ? tg.rnorm[((size_t)(gridDim.z + b) * H + h) * S + key] : 0.f;
        uint32_t g[16], kw[8];
        float part = 0.f;
        if (has) {
          uint32_t pk[8];
          tmem_ld16(lane_base + kDV + c, g);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 2) pk[e / 2] = pack_bf16x2(__uint_as_float(g[e]), __uint_as_float(g[e + 1]));
          const size_t trow = ((size_t)b * S + tok) * 3 * H * DH + (size_t)h * DH + c;
          if (kin) store_row_bf16(tg.dqkv + trow + 2 * H * DH, pk);
          tmem_ld16(lane_base + kDK + c, g);
          // 16-byte chunks c / 8 and c / 8 + 1 of the K tile's row: 128-byte
          // swizzle for DH = 64 (chunk j of row r at j ^ (r % 8)), 64-byte for
          // DH = 32 (at j ^ ((r / 2) % 4))
#pragma unroll
          for (int j = 0; j < 2; ++j) {
            const int ch = c / 8 + j;
            const int off = DH == 64 ? row * 128 + ((ch ^ (row & 7)) << 4) : row * 64 + ((ch ^ ((row >> 1) & 3)) << 4);
            const uint4 v = *reinterpret_cast<const uint4*>(smem + C::kA0 + off);
            kw[4 * j] = v.x;
            kw[4 * j + 1] = v.y;
            kw[4 * j + 2] = v.z;
            kw[4 * j + 3] = v.w;
          }
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 y = unpack_bf16x2(kw[e / 2]);
            part = fmaf(y.x, __uint_as_float(g[e]) * scale, part);
            part = fmaf(y.y, __uint_as_float(g[e + 1]) * scale, part);
          }
        }
        float* s_red = reinterpret_cast<float*>(smem + C::kDS);  // [4 column groups][128 keys]
        s_red[grp * RT_TILE + row] = part;
        mbar_arrive_warp(&bars.epi_red);
        if (mbar_wait_warp(&bars.epi_red, 0, &abort_flag) && has && kin) {
          const float yg = ((s_red[row] + s_red[RT_TILE + row]) + s_red[2 * RT_TILE + row]) + s_red[3 * RT_TILE + row];
          const float yd = rk < 1e6f ? yg : 0.f;
#pragma unroll
          for (int e = 0; e < 16; e += 2) {
            const float2 y = unpack_bf16x2(kw[e / 2]);
            kw[e / 2] = pack_bf16x2(rk * (__uint_as_float(g[e]) * scale - y.x * yd),
                                    rk * (__uint_as_float(g[e + 1]) * scale - y.y * yd));
          }
          store_row_bf16(tg.dqkv + ((size_t)b * S + tok) * 3 * H * DH + (size_t)(H + h) * DH + c, kw);
        }
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

// dQ = scale * dq_acc, rounded to bf16, for the seq_len real rows of each (b, h).
template <int DH>
__global__ void __launch_bounds__(256) dq_convert_kernel(const float* __restrict__ dq_acc, uint16_t* __restrict__ dq,
                                                         long long rows, int S, int Sp, float scale) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;  // 8 elements each
  const long long row = gid / (DH / 8);
  if (row >= rows) return;
  const int c = (int)(gid % (DH / 8)) * 8;
  const long long bh = row / S;
  const int q = (int)(row % S);
  const float4* src = reinterpret_cast<const float4*>(dq_acc + ((size_t)bh * Sp + q) * DH + c);
  const float4 a = src[0], b = src[1];
  *reinterpret_cast<uint4*>(dq + (size_t)row * DH + c) =
      make_uint4(pack_bf16x2(a.x * scale, a.y * scale), pack_bf16x2(a.z * scale, a.w * scale),
                 pack_bf16x2(b.x * scale, b.y * scale), pack_bf16x2(b.z * scale, b.w * scale));
}

// Token-order dQ (TokenGrads): g = scale * dq_acc for the seq_len real rows,
// through the q normalisation's Jacobian into dqkv's q slot of the cell's
// token, and the row's d tau share. DH / 8 consecutive threads hold one row,
// 8 elements each; the row sum is a shuffle reduction among them.
template <int DH>
__global__ void __launch_bounds__(256) dq_qkv_kernel(const float* __restrict__ dq_acc, long long rows, int H, int S,
                                                     int Sp, float scale, const TokenGrads tg) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  constexpr int kLanes = DH / 8;
  const long long gid = (long long)blockIdx.x * blockDim.x + threadIdx.x;
  const long long row = gid / kLanes;
  const bool valid = row < rows;  // every lane stays for the shuffles below
  const int c = (int)(gid % kLanes) * 8;
  const long long bh = valid ? row / S : 0;
  const int i = valid ? (int)(row % S) : 0;
  const int b = (int)(bh / H), h = (int)(bh % H);
  float g[8], y[8];
  float part = 0.f, rq = 0.f, t = 0.f;
  size_t trow = 0;
  if (valid) {
    const float4* src = reinterpret_cast<const float4*>(dq_acc + ((size_t)bh * Sp + i) * DH + c);
    const float4 a0 = src[0], a1 = src[1];
    g[0] = a0.x * scale; g[1] = a0.y * scale; g[2] = a0.z * scale; g[3] = a0.w * scale;
    g[4] = a1.x * scale; g[5] = a1.y * scale; g[6] = a1.z * scale; g[7] = a1.w * scale;
    const int tok = min((int)tg.perm[(size_t)b * S + i], S - 1);  // clamps as the prepass does
    trow = ((size_t)b * S + tok) * 3 * H * DH + (size_t)h * DH + c;
    rq = tg.rnorm[((size_t)b * H + h) * S + i];
    t = tg.tau[h];
    const uint4 x = *reinterpret_cast<const uint4*>(tg.qkv + trow);
    const uint32_t xw[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 8; e += 2) {
      const float2 xf = unpack_bf16x2(xw[e / 2]);
      y[e] = xf.x * rq;
      y[e + 1] = xf.y * rq;
      part = fmaf(y[e], g[e], part);
      part = fmaf(y[e + 1], g[e + 1], part);
    }
  }
#pragma unroll
  for (int off = 1; off < kLanes; off <<= 1) part += __shfl_xor_sync(0xFFFFFFFFu, part, off);
  if (!valid) return;
  const float yd = rq < 1e6f ? t * part : 0.f;
  uint32_t pk[4];
#pragma unroll
  for (int e = 0; e < 8; e += 2) pk[e / 2] = pack_bf16x2(rq * (t * g[e] - y[e] * yd), rq * (t * g[e + 1] - y[e + 1] * yd));
  *reinterpret_cast<uint4*>(tg.dqkv + trow) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
  if (c == 0) tg.dtau_rows[((size_t)b * H + h) * S + i] = part;
}

template <int DH>
int launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o, const uint16_t* d_o,
           const float* lse, int B, int H, int S, float scale, const rt_tile_plan& plan, uint16_t* dq,
           uint16_t* dk, uint16_t* dv, float* stats, float* dq_acc, uint16_t* aux, const TokenGrads& tg,
           cudaStream_t stream) {
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
    e = cudaFuncSetAttribute(dkdvq_kernel<DH, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmemFused);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(dkdvq_kernel)");
    e = cudaFuncSetAttribute(dkdvq_kernel<DH, true>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmemFused);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(dkdvq_kernel, token outputs)");
    configured[dev] = true;
  }
  const int Sp = plan.tiles * RT_TILE;
  const long long rows_padded = (long long)B * H * Sp;
  const long long threads = rows_padded * (DH / 8);
  // fused path: the statistics ride in the MMAs as -lse / scale, so scale > 0
  const bool fused = dq_acc != nullptr && aux != nullptr && scale > 0.f && scale < 3.0e38f;
  // fused path: operand rows and the zeroed dQ accumulator; otherwise the statistics
  if (int st = launch_pdl("row_stats_kernel launch", row_stats_kernel<DH>, dim3((unsigned)((threads + 255) / 256)),
                          dim3(256), 0, stream, o, d_o, lse, fused ? nullptr : stats, fused ? aux : nullptr,
                          fused ? dq_acc : nullptr, fused ? 1.0f / scale : 0.f, S, Sp, rows_padded))
    return st;
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(plan.tiles, H, B);
  if (fused) {  // one pass for dK, dV and dQ
    CUtensorMap tacc, taux;
    if (make_acc_tensor_map(&tacc, dq_acc, rows_padded, DH) != RT_OK) return RT_ERR_CUDA;
    if (make_aux_tensor_map(&taux, aux, rows_padded) != RT_OK) return RT_ERR_CUDA;
    if (int st = launch_pdl("dkdvq_kernel launch", tg.dqkv != nullptr ? dkdvq_kernel<DH, true> : dkdvq_kernel<DH, false>,
                            grid, dim3(kThreadsFused), C::kDynSmemFused, stream, tq, tk, tv, tdo, taux, plan, H, S,
                            scale, scale_log2, dk, dv, tacc, tg))
      return st;
    const long long rows = (long long)B * H * S;
    const long long cthreads = rows * (DH / 8);
    const dim3 cgrid((unsigned)((cthreads + 255) / 256));
    if (tg.dqkv != nullptr)
      return launch_pdl("dq_qkv_kernel launch", dq_qkv_kernel<DH>, cgrid, dim3(256), 0, stream, dq_acc, rows, H, S, Sp,
                        scale, tg);
    return launch_pdl("dq_convert_kernel launch", dq_convert_kernel<DH>, cgrid, dim3(256), 0, stream, dq_acc, dq, rows,
                      S, Sp, scale);
  }
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
                         float* dq_acc, uint16_t* aux, cudaStream_t stream) {
  const bwd::TokenGrads none{};
  if (Dh == 64)
    return bwd::launch<64>(q, k, v, o, d_o, lse, B, H, S, scale, plan, dq, dk, dv, stats, dq_acc, aux, none, stream);
  if (Dh == 32)
    return bwd::launch<32>(q, k, v, o, d_o, lse, B, H, S, scale, plan, dq, dk, dv, stats, dq_acc, aux, none, stream);
  return RT_ERR_UNSUPPORTED;
}

int launch_attention_bwd_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                             const uint16_t* d_o, const float* lse, int B, int H, int S, int Dh, float scale,
                             const rt_tile_plan& plan, const uint16_t* perm, const uint16_t* qkv, const float* tau,
                             const float* rnorm, uint16_t* dqkv, float* dtau_rows, float* dq_acc, uint16_t* aux,
                             cudaStream_t stream) {
  const bwd::TokenGrads tg{perm, qkv, rnorm, tau, dqkv, dtau_rows};
  if (Dh == 64)
    return bwd::launch<64>(q, k, v, o, d_o, lse, B, H, S, scale, plan, nullptr, nullptr, nullptr, nullptr, dq_acc,
                           aux, tg, stream);
  if (Dh == 32)
    return bwd::launch<32>(q, k, v, o, d_o, lse, B, H, S, scale, plan, nullptr, nullptr, nullptr, nullptr, dq_acc,
                           aux, tg, stream);
  return RT_ERR_UNSUPPORTED;
}

}  // namespace rt
