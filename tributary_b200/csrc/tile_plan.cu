// Prepass: token metadata -> tile occupancy bitmaps, per-tile element bits
// and compacted tile lists for one mask kind.
//
// Replaces build_attention_masks (confluence/confluence/model.py:201-264)
// followed by the mask permutation of GatedAttentionSublayer
// (confluence/confluence/layers.py:144-152). Instead of materialising
// [B,S,S] masks, each 128x128 tile of the *permuted* mask is evaluated from
// the token metadata (row id, column id, padding flag, fk adjacency bits)
// and reduced to: live / fully-live flags, and -- for live tiles that are
// not fully live -- its 128x128 element bits in both orientations (query-
// major for the forward and dQ kernels, key-major for dK/dV). Fully-live
// and dead tiles write no element bits; the attention kernels never read them.
//
// Element rule for permuted positions i, j (model.py:227-262):
//   valid = !pad[p_i] && !pad[p_j]
//   rel   = COLUMN:   col[p_i] == col[p_j]
//           FEATURE:  row_i == row_j || fk_adj[row_i][row_j]
//           NEIGHBOR: fk_adj[row_j][row_i]
//           FULL:     true
//   mask  = (rel && valid) || p_i == p_j
// with p = min(perm[b][.], S-1) and row = min(seq_row_ids[b][p], R-1): indices
// past the end clamp, as jax gathers do, so no input can read out of bounds.
#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {

constexpr int kSetupThreads = 1024;

__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, int lane);

// Set-up before the tile masks, one launch:
// - blocks [0, B): flags[b] = 1 when min(perm[b][.], S-1) is a permutation of
//   [0, S): then p_i == p_j only for i == j, and the diagonal term of the
//   element rule is the identity. The block marks each value in a shared
//   bitmap. It also clears the sample's live / fully-live bitmap words (tw =
//   T * W of them), which tile_mask_kernel then sets with atomic ORs.
// - the blocks after them (feature / neighbor kinds): fk_bits[b][r][w] bit t =
//   FEATURE: fk_adj[b][r][32w+t]; NEIGHBOR: fk_adj[b][32w+t][r]. A warp packs
//   one 32 x 32 block of fk_adj: per row, 32 lanes read 32 consecutive bytes
//   and a ballot gives the row's word; the neighbor orientation transposes
//   the 32 words across the warp.
__global__ void __launch_bounds__(kSetupThreads) plan_setup_kernel(
    const uint16_t* __restrict__ perm, int B, int S, int32_t* __restrict__ flags, uint32_t* __restrict__ live,
    uint32_t* __restrict__ full, int tw, const uint8_t* __restrict__ fk_adj, int R, int WR, int transpose,
    uint32_t* __restrict__ fk_bits) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  if ((int)blockIdx.x < B) {
    __shared__ uint32_t bm[65536 / 32];
    __shared__ int dup;
    const int b = blockIdx.x;
    const int words = (S + 31) / 32;
    for (int w = threadIdx.x; w < tw; w += blockDim.x) {
      live[(size_t)b * tw + w] = 0u;
      full[(size_t)b * tw + w] = 0u;
    }
    for (int w = threadIdx.x; w < words; w += blockDim.x) bm[w] = 0u;
    if (threadIdx.x == 0) dup = 0;
    __syncthreads();
    for (int x = threadIdx.x; x < S; x += blockDim.x) {
      const int p = min((int)perm[(size_t)b * S + x], S - 1);
      const uint32_t bit = 1u << (p & 31);
      if (atomicOr(&bm[p >> 5], bit) & bit) dup = 1;
    }
    __syncthreads();
    if (threadIdx.x == 0) flags[b] = dup ? 0 : 1;
    return;
  }
  const int lane = threadIdx.x & 31;
  const long long task = (long long)(blockIdx.x - B) * (kSetupThreads / 32) + (threadIdx.x >> 5);
  const long long per_b = (long long)WR * WR;  // 32 x 32 blocks of one sample
  if (task >= per_b * B) return;  // warp-uniform
  const int b = (int)(task / per_b);
  const int rb = (int)((task % per_b) / WR), cb = (int)(task % WR);
  const uint8_t* base = fk_adj + (size_t)b * R * R;
  const int col = cb * 32 + lane;
  uint32_t mine = 0u;  // lane t: row 32 rb + t, columns [32 cb, +32)
  for (int t = 0; t < 32; ++t) {
    const int row = rb * 32 + t;
    const bool v = row < R && col < R && base[(size_t)row * R + col] != 0;
    const uint32_t bal = __ballot_sync(0xFFFFFFFFu, v);
    if (lane == t) mine = bal;
  }
  if (!transpose) {
    if (rb * 32 + lane < R) fk_bits[((size_t)b * R + rb * 32 + lane) * WR + cb] = mine;
  } else {
    const uint32_t x = warp_transpose32(mine, lane);  // lane c: rows [32 rb, +32) of column 32 cb + c
    if (col < R) fk_bits[((size_t)b * R + col) * WR + rb] = x;
  }
}

constexpr int kTileWarps = 8;  // key tiles per CTA, one per warp
constexpr int kMaxStagedWords = 64;

// 32 x 32 bit transpose across a warp: lane l holds row l on entry and
// column l on exit (bit c of the result = bit l of lane c's row). Five
// butterfly steps; step j swaps the off-diagonal j x j blocks of each
// 2j x 2j block between lanes l and l ^ j.
__device__ __forceinline__ uint32_t warp_transpose32(uint32_t x, int lane) {
  constexpr uint32_t kMask[5] = {0x0000FFFFu, 0x00FF00FFu, 0x0F0F0F0Fu, 0x33333333u, 0x55555555u};
#pragma unroll
  for (int s = 0; s < 5; ++s) {
    const int j = 16 >> s;
    const uint32_t m = kMask[s];
    const uint32_t y = __shfl_xor_sync(0xFFFFFFFFu, x, j);
    x = (lane & j) ? ((x & ~m) | ((y & ~m) >> j)) : ((x & m) | ((y & m) << j));
  }
  return x;
}

// One CTA per (b, q-tile, run of kTileWarps key tiles); each warp evaluates
// one key tile on its own, without block barriers, so the gathers of several
// tiles are in flight at once. Lane l holds queries 32 m + l (m = 0..3) of
// the q-tile and, per 32-key word of its key tile, key 32 kw + l. The keys of
// a word are grouped by the value the relation compares -- row id (feature,
// neighbor) or column id (column) -- with __match_any_sync; in the sampler's
// cell orders a word holds runs of one row or column, so there are few groups,
// and a query evaluates its 32 key bits as the OR of the key sets whose value
// its relation admits (one test per group instead of one per key), ANDed with
// the keys' validity. The feature / neighbor relation tests bit `value` of the
// query row's packed fk row, staged in shared memory once per CTA (odd row
// stride: conflict-free) when it has at most kMaxStagedWords words. The
// diagonal term p_i == p_j is i == j for samples whose perm is a permutation
// (flags from plan_setup_kernel) and is tested key by key otherwise.
template <int KIND, bool kStaged>
__global__ void __launch_bounds__(kTileWarps * 32) tile_mask_kernel(
    const uint16_t* __restrict__ perm, const uint16_t* __restrict__ seq_row_ids,
    const int32_t* __restrict__ column_ids, const uint8_t* __restrict__ is_padding,
    const uint32_t* __restrict__ fk_bits, int S, int R, int WR, rt_tile_plan plan) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  constexpr bool kFk = KIND == RT_MASK_FEATURE || KIND == RT_MASK_NEIGHBOR;
  constexpr uint32_t kAll = 0xFFFFFFFFu;
  const int qt = blockIdx.y;
  const int b = blockIdx.z;
  const int T = plan.tiles;
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  const int kt = blockIdx.x * kTileWarps + warp;
  extern __shared__ uint32_t s_fk[];  // [128][WR | 1] when kStaged
  const size_t boff = (size_t)b * S;
  const int fk_stride = WR | 1;
  const bool have_fk = kFk && R > 0 && fk_bits != nullptr;

  // this lane's queries 32 m + lane (every warp holds the same ones)
  int pi[4], ri[4], ci[4];
  bool qin[4], act[4];
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    const int i = qt * RT_TILE + 32 * m + lane;
    qin[m] = i < S;
    pi[m] = -2;
    ri[m] = 0;
    ci[m] = 0;
    bool pad = true;
    if (qin[m]) {
      pi[m] = min((int)perm[boff + i], S - 1);
      int r = seq_row_ids[boff + pi[m]];
      if (R > 0 && r > R - 1) r = R - 1;
      ri[m] = r;
      ci[m] = column_ids[boff + pi[m]];
      pad = is_padding[boff + pi[m]] != 0;
    }
    act[m] = qin[m] && !pad;
  }
  if (kStaged && have_fk) {
#pragma unroll
    for (int m = 0; m < 4; ++m) {
      const uint32_t* row = fk_bits + ((size_t)b * R + ri[m]) * WR;
      for (int w = warp; w < WR; w += kTileWarps) s_fk[(32 * m + lane) * fk_stride + w] = __ldg(row + w);
    }
    __syncthreads();
  }
  if (kt >= T) return;  // warp-uniform, after the only block barrier
  auto fk_bit = [&](int m, int r) -> bool {
    if (!have_fk) return false;
    const uint32_t word = kStaged ? s_fk[(32 * m + lane) * fk_stride + (r >> 5)]
                                  : __ldg(fk_bits + ((size_t)b * R + ri[m]) * WR + (r >> 5));
    return (word >> (r & 31)) & 1u;
  };

  // key metadata of the tile's four words: lane holds key kt * 128 + 32 kw + lane
  int pj[4], gk[4];
  uint32_t valid[4];
#pragma unroll
  for (int kw = 0; kw < 4; ++kw) {
    const int j = kt * RT_TILE + 32 * kw + lane;
    const bool jin = j < S;
    int p = -1, r = 0, c = 0;
    bool pad = true;
    if (jin) {
      p = min((int)perm[boff + j], S - 1);  // out-of-range perm entries clamp
      r = seq_row_ids[boff + p];
      if (R > 0 && r > R - 1) r = R - 1;
      c = column_ids[boff + p];
      pad = is_padding[boff + p] != 0;
    }
    pj[kw] = p;
    gk[kw] = KIND == RT_MASK_COLUMN ? c : r;
    valid[kw] = __ballot_sync(kAll, jin && !pad);
  }

  uint32_t w[4][4];  // [query block m][key word kw]: this lane's query row, 32 keys
#pragma unroll
  for (int kw = 0; kw < 4; ++kw) {
    uint32_t rel[4] = {0u, 0u, 0u, 0u};
    if (KIND == RT_MASK_FULL) {
#pragma unroll
      for (int m = 0; m < 4; ++m) rel[m] = kAll;
    } else {
      const uint32_t same = __match_any_sync(kAll, gk[kw]);
      uint32_t leaders = __ballot_sync(kAll, (__ffs(same) - 1) == lane);
      while (leaders) {  // warp-uniform
        const int src = __ffs(leaders) - 1;
        leaders &= leaders - 1u;
        const int key = __shfl_sync(kAll, gk[kw], src);
        const uint32_t bits = __shfl_sync(kAll, same, src);
#pragma unroll
        for (int m = 0; m < 4; ++m) {
          bool r;
          if (KIND == RT_MASK_COLUMN) r = ci[m] == key;
          else if (KIND == RT_MASK_FEATURE) r = ri[m] == key || fk_bit(m, key);
          else r = fk_bit(m, key);
          if (r) rel[m] |= bits;
        }
      }
    }
#pragma unroll
    for (int m = 0; m < 4; ++m) w[m][kw] = act[m] ? (rel[m] & valid[kw]) : 0u;
  }
  if (plan.nnz[1 + b] != 0) {  // perm is a permutation: p_i == p_j exactly when i == j
    if (kt == qt) {
#pragma unroll
      for (int m = 0; m < 4; ++m)
        if (qin[m]) w[m][m] |= 1u << lane;
    }
  } else {
#pragma unroll
    for (int kw = 0; kw < 4; ++kw) {
      for (int u = 0; u < 32; ++u) {
        const int p = __shfl_sync(kAll, pj[kw], u);
#pragma unroll
        for (int m = 0; m < 4; ++m)
          if (p == pi[m]) w[m][kw] |= 1u << u;  // pi = -2 for queries past S, pj = -1 for keys past S
      }
    }
  }

  uint32_t any_v = 0u, all_v = kAll;
  bool rows_in = true;
#pragma unroll
  for (int m = 0; m < 4; ++m) {
    rows_in = rows_in && qin[m];
#pragma unroll
    for (int kw = 0; kw < 4; ++kw) {
      any_v |= w[m][kw];
      all_v &= w[m][kw];
    }
  }
  if (!__any_sync(kAll, any_v != 0u)) return;  // warp-uniform
  const bool all = __all_sync(kAll, rows_in && all_v == kAll);
  if (lane == 0) {
    const size_t wi = ((size_t)b * T + qt) * plan.words + (kt >> 5);
    atomicOr(plan.live_bits + wi, 1u << (kt & 31));
    if (all) atomicOr(plan.full_bits + wi, 1u << (kt & 31));
  }
  if (all) return;  // warp-uniform
  const size_t tile_q = ((size_t)b * T + qt) * T + kt;
  const size_t tile_k = ((size_t)b * T + kt) * T + qt;
  uint4* dst_q = reinterpret_cast<uint4*>(plan.tile_masks) + tile_q * RT_TILE;
#pragma unroll
  for (int m = 0; m < 4; ++m) dst_q[32 * m + lane] = make_uint4(w[m][0], w[m][1], w[m][2], w[m][3]);
  // key-major copy: key 32 kw + lane, its bits over query block m
  uint4* dst_k = reinterpret_cast<uint4*>(plan.tile_masks_t) + tile_k * RT_TILE;
#pragma unroll
  for (int kw = 0; kw < 4; ++kw)
    dst_k[32 * kw + lane] = make_uint4(warp_transpose32(w[0][kw], lane), warp_transpose32(w[1][kw], lane),
                                       warp_transpose32(w[2][kw], lane), warp_transpose32(w[3][kw], lane));
}

// CSR lists (q2k over (b,qt) rows, k2q over (b,kt) rows) from the bitmaps, one
// block per sample. Both lists of sample b start at the number of live tiles
// of the samples before it, which the block counts from their bitmaps; the
// sample's own bitmaps are staged in shared memory when they fit.
constexpr int kListSmemBytes = 96 * 1024;  // tile_list_kernel's staged bitmaps of one sample
constexpr int kListThreads = 512;

__global__ void __launch_bounds__(kListThreads) tile_list_kernel(rt_tile_plan plan) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const int T = plan.tiles;
  const int W = plan.words;
  const int b = blockIdx.x;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  constexpr int kWarps = kListThreads / 32;
  __shared__ int s_warp[kWarps];
  __shared__ int s_total;
  extern __shared__ uint32_t s_bits[];
  const int nwords = T * W;
  const bool staged = 2LL * nwords * (long long)sizeof(uint32_t) <= (long long)kListSmemBytes;
  const uint32_t* live = plan.live_bits + (size_t)b * nwords;
  const uint32_t* full_b = plan.full_bits + (size_t)b * nwords;

  // exclusive block scan of one value per thread; returns the prefix, leaves the sum in s_total
  auto block_scan = [&](int v) {
    int incl = v;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xFFFFFFFFu, incl, o);
      if (lane >= o) incl += u;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      const int x = lane < kWarps ? s_warp[lane] : 0;
      int xi = x;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int u = __shfl_up_sync(0xFFFFFFFFu, xi, o);
        if (lane >= o) xi += u;
      }
      if (lane < kWarps) s_warp[lane] = xi - x;
      if (lane == 31) s_total = xi;
    }
    __syncthreads();
    const int r = s_warp[warp] + incl - v;
    return r;
  };

  // live tiles of the samples before b
  int before = 0;
  for (long long i = threadIdx.x; i < (long long)b * nwords; i += kListThreads) before += __popc(plan.live_bits[i]);
  if (staged) {
    for (int i = threadIdx.x; i < nwords; i += kListThreads) {
      s_bits[i] = live[i];
      s_bits[nwords + i] = full_b[i];
    }
    live = s_bits;
    full_b = s_bits + nwords;
  }
  (void)block_scan(before);  // also orders the staging above before the reads below
  const int base = s_total;
  __syncthreads();

  // rows x of this sample in chunks of kListThreads; thread = row
  for (int pass = 0; pass < 2; ++pass) {
    const bool by_q = pass == 0;
    int* ptr = by_q ? plan.q2k_ptr : plan.k2q_ptr;
    int* idx = by_q ? plan.q2k_idx : plan.k2q_idx;
    int run = base;
    for (int x0 = 0; x0 < T; x0 += kListThreads) {
      const int x = x0 + threadIdx.x;
      int cnt = 0;
      if (x < T) {
        if (by_q) {
          for (int w = 0; w < W; ++w) cnt += __popc(live[x * W + w]);
        } else {
          for (int q = 0; q < T; ++q) cnt += (live[q * W + (x >> 5)] >> (x & 31)) & 1u;
        }
      }
      int pos = run + block_scan(cnt);
      const int chunk_total = s_total;
      if (x < T) {
        ptr[(size_t)b * T + x] = pos;
        if (by_q) {
          for (int kt = 0; kt < T; ++kt) {
            const int wi = x * W + (kt >> 5);
            if ((live[wi] >> (kt & 31)) & 1u) {
              const bool f = (full_b[wi] >> (kt & 31)) & 1u;
              idx[pos++] = kt | (f ? (int)0x80000000u : 0);
            }
          }
        } else {
          for (int qt = 0; qt < T; ++qt) {
            const int wi = qt * W + (x >> 5);
            if ((live[wi] >> (x & 31)) & 1u) {
              const bool f = (full_b[wi] >> (x & 31)) & 1u;
              idx[pos++] = qt | (f ? (int)0x80000000u : 0);
            }
          }
        }
      }
      run += chunk_total;
      __syncthreads();  // s_total / s_warp are reused by the next chunk's scan
    }
    if (b == plan.batch - 1 && threadIdx.x == 0) {
      ptr[(size_t)plan.batch * T] = run;
      if (by_q) *plan.nnz = run;
    }
  }
}

int launch_build_tile_plan(const uint16_t* perm, const uint16_t* seq_row_ids, const int32_t* column_ids,
                           const uint8_t* is_padding, const uint8_t* fk_adj, int B, int S, int R,
                           int kind, const rt_tile_plan& plan, cudaStream_t stream) {
  const int T = plan.tiles;
  const int W = plan.words;
  const int WR = (R + 31) / 32;
  const bool needs_fk = (kind == RT_MASK_FEATURE || kind == RT_MASK_NEIGHBOR) && R > 0;
  const uint32_t* fk_bits = needs_fk ? plan.fk_bits : nullptr;
  const long long fk_tasks = needs_fk ? (long long)B * WR * WR : 0;
  const int setup_blocks = B + (int)((fk_tasks + kSetupThreads / 32 - 1) / (kSetupThreads / 32));
  if (int st = launch_pdl("plan_setup_kernel launch", plan_setup_kernel, dim3(setup_blocks), dim3(kSetupThreads), 0,
                          stream, perm, B, S, plan.nnz + 1, plan.live_bits, plan.full_bits, T * W, fk_adj, R, WR,
                          kind == RT_MASK_NEIGHBOR ? 1 : 0, plan.fk_bits))
    return st;
  const dim3 grid((T + kTileWarps - 1) / kTileWarps, T, B);
  const bool staged = WR <= kMaxStagedWords;
  const size_t fk_smem = sizeof(uint32_t) * RT_TILE * (size_t)(WR | 1);
  using MaskKernel = void (*)(const uint16_t*, const uint16_t*, const int32_t*, const uint8_t*, const uint32_t*,
                              int, int, int, rt_tile_plan);
  MaskKernel mask_kernel = tile_mask_kernel<RT_MASK_FULL, false>;
  if (kind == RT_MASK_COLUMN) mask_kernel = tile_mask_kernel<RT_MASK_COLUMN, false>;
  else if (kind == RT_MASK_FEATURE) mask_kernel = staged ? tile_mask_kernel<RT_MASK_FEATURE, true>
                                                         : tile_mask_kernel<RT_MASK_FEATURE, false>;
  else if (kind == RT_MASK_NEIGHBOR) mask_kernel = staged ? tile_mask_kernel<RT_MASK_NEIGHBOR, true>
                                                          : tile_mask_kernel<RT_MASK_NEIGHBOR, false>;
  const bool uses_smem = (kind == RT_MASK_FEATURE || kind == RT_MASK_NEIGHBOR) && staged;
  if (int st = launch_pdl("tile_mask_kernel launch", mask_kernel, grid, dim3(kTileWarps * 32),
                          uses_smem ? fk_smem : 0, stream, perm, seq_row_ids, column_ids, is_padding, fk_bits, S, R,
                          WR, plan))
    return st;
  {
    const size_t bits_bytes = 2 * sizeof(uint32_t) * (size_t)plan.tiles * plan.words;  // one sample
    const size_t smem = bits_bytes <= (size_t)kListSmemBytes ? bits_bytes : 0;
    static bool list_configured[64] = {false};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev >= 0 && dev < 64 && !list_configured[dev]) {
      const cudaError_t e =
          cudaFuncSetAttribute(tile_list_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kListSmemBytes);
      if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(tile_list_kernel)");
      list_configured[dev] = true;
    }
    if (int st = launch_pdl("tile_list_kernel launch", tile_list_kernel, dim3(B), dim3(kListThreads), smem, stream, plan))
      return st;
  }
  return check_launch("tile plan kernels launch");
}

}  // namespace rt
