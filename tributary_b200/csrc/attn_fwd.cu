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
constexpr int kMaxTiles = 65536 / RT_TILE;  // tiles per row of the plan (seq_len <= 65536)

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
  __shared__ int s_list[kMaxTiles];

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
  for (int i = threadIdx.x; i < n_tiles; i += kThreads) s_list[i] = list[i];

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
        const int kt = s_list[j] & 0x7FFFFFFF;
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
    const float c = scale_log2;
    const float kNegInf = -INFINITY;
    float m_run = kNegInf;  // running row max of raw scores (scale not applied)
    float2 l2 = make_float2(0.f, 0.f);
    auto load_mask = [&](int ent) {
      uint4 mk = make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu, 0xFFFFFFFFu);
      if (ent >= 0) mk = __ldg(reinterpret_cast<const uint4*>(masks + ((size_t)(ent & 0x7FFFFFFF) * RT_TILE + row) * 4));
      return mk;
    };
    uint4 mk_next = n_tiles > 0 ? load_mask(s_list[0]) : make_uint4(0u, 0u, 0u, 0u);
    bool ok = true;
    for (int j = 0; j < n_tiles; ++j) {
      const bool full = s_list[j] < 0;
      const uint4 mk = mk_next;
      if (j + 1 < n_tiles) mk_next = load_mask(s_list[j + 1]);
      if (!(ok = mbar_wait(&bars.s_full, j & 1, &abort_flag))) break;
      tc_fence_after();
      uint32_t r[128];
      {
        uint32_t (&r0)[64] = *reinterpret_cast<uint32_t(*)[64]>(&r[0]);
        uint32_t (&r1)[64] = *reinterpret_cast<uint32_t(*)[64]>(&r[64]);
        tmem_ld64(lane_base + kSCol, r0);
        tmem_ld64(lane_base + kSCol + 64, r1);
      }
      tmem_wait_ld();
      if (!full) {
        const uint32_t mw[4] = {mk.x, mk.y, mk.z, mk.w};
#pragma unroll
        for (int e = 0; e < 128; ++e)
          r[e] = ((mw[e >> 5] >> (e & 31)) & 1u) ? r[e] : __float_as_uint(kNegInf);
      }
      float mx = kNegInf;
#pragma unroll
      for (int e = 0; e < 128; e += 2) mx = fmax3(mx, __uint_as_float(r[e]), __uint_as_float(r[e + 1]));
      const float m_new = fmaxf(m_run, mx);
      const bool need = (m_new != kNegInf) && (m_run == kNegInf || (m_new - m_run) * c > kRescaleThreshold);
      if (j > 0 && !(ok = mbar_wait(&bars.o_done, (j - 1) & 1, &abort_flag))) break;
      tc_fence_after();
      if (__any_sync(0xFFFFFFFFu, need)) {
        const float alpha = m_run == kNegInf ? 0.f : (m_new == kNegInf ? 1.f : fast_exp2((m_run - m_new) * c));
        if (j > 0) {
#pragma unroll
          for (int cc = 0; cc < DH; cc += 32) {
            uint32_t o[32];
            tmem_ld32(lane_base + kOCol + cc, o);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st32(lane_base + kOCol + cc, o);
          }
          tmem_wait_st();
        }
        l2.x *= alpha;
        l2.y *= alpha;
        if (m_new != kNegInf) m_run = m_new;
      }
      // p = exp2(c * (s - m)); masked entries hold -inf and give exactly 0
      const float nmc = m_run == kNegInf ? 0.f : -m_run * c;
      const float2 cc2 = make_float2(c, c);
      const float2 nm2 = make_float2(nmc, nmc);
      uint32_t pk[64];
#pragma unroll
      for (int e = 0; e < 128; e += 2) {
        const float2 x = ffma2(make_float2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), cc2, nm2);
        const float2 p = make_float2(fast_exp2(x.x), fast_exp2(x.y));
        l2 = fadd2(l2, p);
        pk[e >> 1] = pack_bf16x2(p.x, p.y);
      }
      {
        uint32_t (&p0)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[0]);
        uint32_t (&p1)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32]);
        tmem_st32(lane_base + kPCol, p0);
        tmem_st32(lane_base + kPCol + 32, p1);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars.p_full);
    }
    const float l_run = l2.x + l2.y;
    // epilogue
    if (ok && n_tiles > 0 && mbar_wait(&bars.o_done, (n_tiles - 1) & 1, &abort_flag)) {
      tc_fence_after();
      const int q = qt * RT_TILE + row;
      const float inv_l = l_run > 0.f ? 1.f / l_run : 0.f;
      uint16_t* orow = out + ((size_t)bh * S + q) * DH;
#pragma unroll
      for (int cc = 0; cc < DH; cc += 16) {
        uint32_t o[16];
        tmem_ld16(lane_base + kOCol + cc, o);
        tmem_wait_ld();
        uint32_t pko[8];
#pragma unroll
        for (int e = 0; e < 16; e += 2)
          pko[e / 2] = pack_bf16x2(__uint_as_float(o[e]) * inv_l, __uint_as_float(o[e + 1]) * inv_l);
        if (q < S) {
          uint4* dst = reinterpret_cast<uint4*>(orow + cc);
          dst[0] = make_uint4(pko[0], pko[1], pko[2], pko[3]);
          dst[1] = make_uint4(pko[4], pko[5], pko[6], pko[7]);
        }
      }
      if (q < S)
        lse[(size_t)bh * S + q] =
            l_run > 0.f ? (m_run * c + __log2f(l_run)) * 0.6931471805599453f : -INFINITY;
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
