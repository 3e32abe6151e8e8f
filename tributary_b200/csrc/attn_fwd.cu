// Forward masked attention on sm_100a (tcgen05 + TMA), one 128-query tile of
// one (batch, head) per CTA, iterating only the live key tiles of the plan.
//
// Replaces confluence/confluence/layers.py:83-94: s = q k^T * scale,
// where(mask, s, -1e9), softmax, p v. Masked elements are excluded exactly
// (every row keeps its diagonal, so the reference's -1e9 entries contribute
// exp(-1e9 - max) == 0 in fp32). Also writes lse = ln sum_j exp(s_ij).
//
// Warp roles (192 threads):
//   warp 0      TMA producer (Q once, K/V ring) + TMEM allocation
//   warp 1      MMA issuer (one thread): S = Q K^T, O += P V
//   warps 2..5  softmax: thread = query row (TMEM lane), online softmax in
//               fp32 (log2 domain), lazy O rescale, P -> TMEM as bf16,
//               epilogue O / l -> bf16, lse.
// Tensor memory (256 columns): S [0,128) fp32, P [128,192) bf16x2, O [192,192+DH).
// Per-tile mask bits come from the prepass (query-major words); fully-live
// tiles skip the mask entirely.
#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {
namespace fwd {

constexpr int kThreads = 192;
constexpr int kSCol = 0;
constexpr int kPCol = 128;
constexpr int kOCol = 192;
constexpr int kTmemCols = 256;
constexpr float kRescaleThreshold = 8.0f;  // log2 units: rescale O only when the max grows by 2^8

template <int DH>
struct Cfg {
  static constexpr int kRowBytes = DH * 2;
  static constexpr int kTileBytes = RT_TILE * kRowBytes;
  static constexpr uint32_t kSwizzle = DH == 64 ? SW_128B : SW_64B;
  static constexpr int kSBO = 8 * kRowBytes;
  static constexpr int kStages = DH == 64 ? 2 : 4;
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kTileBytes;
  static constexpr int kVOff = kKOff + kStages * kTileBytes;
  static constexpr int kSmemBytes = kVOff + kStages * kTileBytes;
  // 256 TMEM columns per CTA: at most two CTAs may share an SM, so ask for
  // enough shared memory that a third never lands there.
  static constexpr int kDynSmem = (kSmemBytes + 1024) > 78 * 1024 ? (kSmemBytes + 1024) : 78 * 1024;
};

struct __align__(8) Barriers {
  uint64_t q_full;
  uint64_t kv_full[4];
  uint64_t kv_empty[4];
  uint64_t s_full;
  uint64_t p_full;
  uint64_t o_done;
  uint64_t drain;
};

template <int DH>
__global__ void __launch_bounds__(kThreads, 2)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const rt_tile_plan plan, int H, int S,
                    float scale_log2, uint16_t* __restrict__ out, float* __restrict__ lse) {
  using C = Cfg<DH>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ Barriers bars;
  __shared__ uint32_t tmem_base_s;
  __shared__ int abort_flag;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int qt = blockIdx.x;
  const int h = blockIdx.y;
  const int b = blockIdx.z;
  const int T = plan.tiles;
  const int bh = b * H + h;
  const int row_list = b * T + qt;
  const int list_begin = plan.q2k_ptr[row_list];
  const int n_tiles = plan.q2k_ptr[row_list + 1] - list_begin;
  const int* list = plan.q2k_idx + list_begin;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    mbar_init(&bars.q_full, 1);
    for (int s = 0; s < C::kStages; ++s) {
      mbar_init(&bars.kv_full[s], 1);
      mbar_init(&bars.kv_empty[s], 1);
    }
    mbar_init(&bars.s_full, 1);
    mbar_init(&bars.p_full, 128);
    mbar_init(&bars.o_done, 1);
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
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_tiles > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_arrive_expect_tx(&bars.q_full, C::kTileBytes);
      tma_load_3d(smem + C::kQOff, &tm_q, &bars.q_full, 0, qt * RT_TILE, bh);
      int j = 0;
      for (; j < n_tiles; ++j) {
        const int s = j % C::kStages;
        if (j >= C::kStages && !mbar_wait(&bars.kv_empty[s], ((j / C::kStages) - 1) & 1, &abort_flag)) break;
        const int kt = list[j] & 0x7FFFFFFF;
        mbar_arrive_expect_tx(&bars.kv_full[s], 2 * C::kTileBytes);
        tma_load_3d(smem + C::kKOff + s * C::kTileBytes, &tm_k, &bars.kv_full[s], 0, kt * RT_TILE, bh);
        tma_load_3d(smem + C::kVOff + s * C::kTileBytes, &tm_v, &bars.kv_full[s], 0, kt * RT_TILE, bh);
      }
      // Drain: every load issued must land before the CTA may exit.
      for (int jj = max(0, j - C::kStages); jj < j; ++jj) {
        const int s = jj % C::kStages;
        volatile int no_abort = 0;
        mbar_wait(&bars.kv_full[s], (jj / C::kStages) & 1, &no_abort);
      }
      volatile int no_abort = 0;
      mbar_wait(&bars.q_full, 0, &no_abort);
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t idesc_s = idesc_bf16_f32(128, 128, false, false);
      constexpr uint32_t idesc_o = idesc_bf16_f32(128, DH, false, true);
      const uint32_t q_addr = smem_u32(smem + C::kQOff);
      bool ok = mbar_wait(&bars.q_full, 0, &abort_flag);
      tc_fence_after();
      for (int j = 0; ok && j <= n_tiles; ++j) {
        if (j > 0) {
          // O += P_{j-1} V_{j-1}
          if (!(ok = mbar_wait(&bars.p_full, (j - 1) & 1, &abort_flag))) break;
          tc_fence_after();
          const int sp = (j - 1) % C::kStages;
          const uint32_t v_addr = smem_u32(smem + C::kVOff + sp * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < RT_TILE / 16; ++ks) {
            const uint64_t bdesc = sdesc(v_addr + ks * 16 * C::kRowBytes, 0, C::kSBO, C::kSwizzle);
            mma_ts(tmem + kOCol, tmem + kPCol + ks * 8, bdesc, idesc_o, (j > 1 || ks > 0) ? 1u : 0u);
          }
          mma_commit(&bars.o_done);
          mma_commit(&bars.kv_empty[sp]);
        }
        if (j < n_tiles) {
          // S = Q K_j^T
          const int s = j % C::kStages;
          if (!(ok = mbar_wait(&bars.kv_full[s], (j / C::kStages) & 1, &abort_flag))) break;
          tc_fence_after();
          const uint32_t k_addr = smem_u32(smem + C::kKOff + s * C::kTileBytes);
#pragma unroll
          for (int ks = 0; ks < DH / 16; ++ks) {
            const uint64_t adesc = sdesc(q_addr + ks * 32, 16, C::kSBO, C::kSwizzle);
            const uint64_t bdesc = sdesc(k_addr + ks * 32, 16, C::kSBO, C::kSwizzle);
            mma_ss(tmem + kSCol, adesc, bdesc, idesc_s, ks > 0 ? 1u : 0u);
          }
          mma_commit(&bars.s_full);
        }
      }
      // Drain: all issued MMAs complete before TMEM is released.
      mma_commit(&bars.drain);
      volatile int no_abort = 0;
      mbar_wait(&bars.drain, 0, &no_abort);
    }
  } else {
    // ---------------- softmax warpgroup ----------------
    const int quad = warp & 3;
    const int row = quad * 32 + lane;
    const uint32_t lane_base = tmem + ((uint32_t)(quad * 32) << 16);
    const uint32_t* masks = plan.tile_masks + ((size_t)row_list * T) * RT_TILE * 4;
    float m_run = -INFINITY;  // running max, log2 units
    float l_run = 0.f;
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int ent = list[j];
      const int kt = ent & 0x7FFFFFFF;
      uint4 mk = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
      if (ent >= 0) mk = *reinterpret_cast<const uint4*>(masks + ((size_t)kt * RT_TILE + row) * 4);
      const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
      if (!(ok = mbar_wait(&bars.s_full, j & 1, &abort_flag))) break;
      tc_fence_after();
      // pass 1: masked row max of this tile
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + kSCol + c * 32, r);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float v = __uint_as_float(r[e]) * scale_log2;
          mx = ((mw[c] >> e) & 1u) ? fmaxf(mx, v) : mx;
        }
      }
      const float m_new = fmaxf(m_run, mx);
      const bool need = (m_new != -INFINITY) && (m_run == -INFINITY || m_new > m_run + kRescaleThreshold);
      if (j > 0 && !(ok = mbar_wait(&bars.o_done, (j - 1) & 1, &abort_flag))) break;
      tc_fence_after();
      if (__any_sync(0xFFFFFFFFu, need)) {
        const float alpha = (m_run == -INFINITY || m_new == -INFINITY) ? (m_run == -INFINITY ? 0.f : 1.f)
                                                                        : fast_exp2(m_run - m_new);
        if (j > 0) {
#pragma unroll
          for (int c = 0; c < DH; c += 16) {
            uint32_t r[16];
            tmem_ld16(lane_base + kOCol + c, r);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 16; ++e) r[e] = __float_as_uint(__uint_as_float(r[e]) * alpha);
            tmem_st16(lane_base + kOCol + c, r);
          }
          tmem_wait_st();
        }
        l_run *= alpha;
        if (m_new != -INFINITY) m_run = m_new;
      }
      const float m_use = m_run == -INFINITY ? 0.f : m_run;
      // pass 2: p = exp2(s - m), row sum, P -> TMEM (bf16 pairs)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        uint32_t r[32];
        tmem_ld32(lane_base + kSCol + c * 32, r);
        tmem_wait_ld();
        uint32_t pk[16];
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float s0 = __uint_as_float(r[e]) * scale_log2 - m_use;
          const float s1 = __uint_as_float(r[e + 1]) * scale_log2 - m_use;
          const float p0 = ((mw[c] >> e) & 1u) ? fast_exp2(s0) : 0.f;
          const float p1 = ((mw[c] >> (e + 1)) & 1u) ? fast_exp2(s1) : 0.f;
          l_run += p0 + p1;
          pk[e / 2] = pack_bf16x2(p0, p1);
        }
        tmem_st16(lane_base + kPCol + c * 16, pk);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.p_full);
    }
    // epilogue
    if (ok && n_tiles > 0 && mbar_wait(&bars.o_done, (n_tiles - 1) & 1, &abort_flag)) {
      tc_fence_after();
      const int q = qt * RT_TILE + row;
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      uint16_t* orow = out + ((size_t)bh * S + q) * DH;
#pragma unroll
      for (int c = 0; c < DH; c += 16) {
        uint32_t r[16];
        tmem_ld16(lane_base + kOCol + c, r);
        tmem_wait_ld();
        uint32_t pk[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pk[e / 2] = pack_bf16x2(__uint_as_float(r[e]) * inv_l, __uint_as_float(r[e + 1]) * inv_l);
        if (q < S) {
          uint4* dst = reinterpret_cast<uint4*>(orow + c);
          dst[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          dst[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
        }
      }
      if (q < S)
        lse[(size_t)bh * S + q] = l_run > 0.f ? (m_run + __log2f(l_run)) * 0.6931471805599453f : -INFINITY;
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
int launch(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, float scale,
           const rt_tile_plan& plan, uint16_t* o, float* lse, cudaStream_t stream) {
  using C = Cfg<DH>;
  CUtensorMap tq, tk, tv;
  if (make_qkv_tensor_map(&tq, q, B * H, S, DH) != RT_OK || make_qkv_tensor_map(&tk, k, B * H, S, DH) != RT_OK ||
      make_qkv_tensor_map(&tv, v, B * H, S, DH) != RT_OK)
    return RT_ERR_CUDA;  // detail recorded by make_qkv_tensor_map
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_fwd_kernel<DH>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kDynSmem);
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(attn_fwd_kernel)");
    configured[dev] = true;
  }
  const float scale_log2 = scale * 1.4426950408889634f;
  dim3 grid(plan.tiles, H, B);
  attn_fwd_kernel<DH><<<grid, kThreads, C::kDynSmem, stream>>>(tq, tk, tv, plan, H, S, scale_log2, o, lse);
  return check_launch("attn_fwd_kernel launch");
}

}  // namespace fwd

int launch_attention_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S, int Dh,
                         float scale, const rt_tile_plan& plan, uint16_t* o, float* lse, cudaStream_t stream) {
  if (Dh == 64) return fwd::launch<64>(q, k, v, B, H, S, scale, plan, o, lse, stream);
  if (Dh == 32) return fwd::launch<32>(q, k, v, B, H, S, scale, plan, o, lse, stream);
  return RT_ERR_UNSUPPORTED;
}

}  // namespace rt
