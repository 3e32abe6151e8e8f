// Token preparation around the attention kernels of one sublayer: the
// permuted-order gather / scatter of confluence/confluence/layers.py:139-167
// and the QK L2 normalisation with learned temperature of layers.py:63-80,
// fused into single memory-bound passes.
//
// A per-token linear map commutes with a permutation of the tokens, so the
// QKV projection runs on the tokens in their own order and the gather moves
// into these kernels:
//   qk_prepare   qkv[b, perm[b,i], {q,k,v}, h, :]  ->  q_hat[b,h,i,:] =
//                tau_h q / max(|q|, 1e-6), k_hat = k / max(|k|, 1e-6), v
//                (bf16, the attention kernels' [B,H,S,Dh] layout), with the
//                fp32 inverse norms kept for the backward
//   qk_prepare_bwd  the normalisation's Jacobian, scattered back through the
//                permutation (a permutation has no collisions: no atomics)
//   heads_unpermute / heads_permute  attention output [B,H,S,Dh] in permuted
//                order <-> [B,S,H*Dh] in token order (each other's backward)
// One warp per token; a warp moves each head's Dh-element row as one
// contiguous, coalesced access. Norms and products are accumulated in fp32.
// Order entries past the end clamp to S - 1, as in the prepass, so no order
// can move an access out of bounds.
#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {
namespace tok {

constexpr int kWarps = 8;  // tokens per 256-thread block

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xFFFFFFFFu, x, off);
  return x;
}

// Dh / 32 consecutive bf16 per lane: 2 for Dh = 64 (one 32-bit word), 1 for Dh = 32.
template <int DH>
struct Lane {
  static constexpr int kE = DH / 32;
  float v[kE];
  __device__ __forceinline__ void load(const uint16_t* row, int lane) {
    if (kE == 2) {
      const float2 f = unpack_bf16x2(*reinterpret_cast<const uint32_t*>(row + 2 * lane));
      v[0] = f.x;
      v[kE - 1] = f.y;
    } else {
      v[0] = __uint_as_float((uint32_t)row[lane] << 16);
    }
  }
  __device__ __forceinline__ void store(uint16_t* row, int lane, float s) const {
    if (kE == 2) {
      *reinterpret_cast<uint32_t*>(row + 2 * lane) = pack_bf16x2(v[0] * s, v[kE - 1] * s);
    } else {
      const __nv_bfloat16 b = __float2bfloat16_rn(v[0] * s);
      row[lane] = *reinterpret_cast<const uint16_t*>(&b);
    }
  }
  __device__ __forceinline__ float dot(const Lane& o) const {
    float s = 0.f;
#pragma unroll
    for (int e = 0; e < kE; ++e) s = fmaf(v[e], o.v[e], s);
    return s;
  }
};

template <int DH>
__device__ __forceinline__ void copy_row(uint16_t* dst, const uint16_t* src, int lane) {
  if (DH == 64)
    reinterpret_cast<uint32_t*>(dst)[lane] = reinterpret_cast<const uint32_t*>(src)[lane];
  else
    dst[lane] = src[lane];
}

// qk_prepare: one warp per token. The token's 3 H rows (q heads, k heads, v
// heads; Dh bf16 each) are read as 16-byte chunks, DH / 8 lanes per row and
// 32 / (DH / 8) rows per warp instruction, with up to kBatch instructions'
// loads in flight before any row is reduced: the kernel streams from HBM
// instead of waiting on one small load per head.
template <int DH>
__global__ void __launch_bounds__(32 * kWarps) qk_prepare_kernel(const uint16_t* __restrict__ qkv,
                                                                 const uint16_t* __restrict__ perm,
                                                                 const float* __restrict__ tau, int B, int H, int S,
                                                                 uint16_t* __restrict__ q, uint16_t* __restrict__ k,
                                                                 uint16_t* __restrict__ v, float* __restrict__ rnorm) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  constexpr int kL = DH / 8;      // lanes per row
  constexpr int kRows = 32 / kL;  // rows per warp instruction
  constexpr int kBatch = 6;       // instructions whose loads are issued together
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= (long long)B * S) return;  // warp-uniform
  const int b = (int)(t / S), i = (int)(t % S);
  const int sub = lane % kL, rsel = lane / kL;
  const uint16_t* row = qkv + ((size_t)b * S + min((int)perm[t], S - 1)) * 3 * H * DH;
  const int nrows = 3 * H;
  for (int r0 = 0; r0 < nrows; r0 += kRows * kBatch) {
    uint4 x[kBatch];
#pragma unroll
    for (int p = 0; p < kBatch; ++p) {
      const int r = r0 + p * kRows + rsel;
      x[p] = r < nrows ? *reinterpret_cast<const uint4*>(row + (size_t)r * DH + sub * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
#pragma unroll
    for (int p = 0; p < kBatch; ++p) {
      const int r = r0 + p * kRows + rsel;  // the kL lanes of a row share r
      const uint32_t w[4] = {x[p].x, x[p].y, x[p].z, x[p].w};
      float f[8];
      float ss = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 u = unpack_bf16x2(w[e]);
        f[2 * e] = u.x;
        f[2 * e + 1] = u.y;
        ss = fmaf(u.x, u.x, fmaf(u.y, u.y, ss));
      }
#pragma unroll
      for (int off = 1; off < kL; off <<= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
      if (r >= nrows) continue;
      const int part = r / H, h = r % H;  // 0: q, 1: k, 2: v
      const size_t o = (((size_t)b * H + h) * S + i) * DH + sub * 8;
      if (part == 2) {
        *reinterpret_cast<uint4*>(v + o) = x[p];
        continue;
      }
      const float rn = 1.f / fmaxf(sqrtf(ss), 1e-6f);
      const float sc = part == 0 ? rn * tau[h] : rn;
      *reinterpret_cast<uint4*>((part == 0 ? q : k) + o) =
          make_uint4(pack_bf16x2(f[0] * sc, f[1] * sc), pack_bf16x2(f[2] * sc, f[3] * sc),
                     pack_bf16x2(f[4] * sc, f[5] * sc), pack_bf16x2(f[6] * sc, f[7] * sc));
      if (sub == 0) rnorm[(((size_t)part * B + b) * H + h) * S + i] = rn;
    }
  }
}

// out = scale * y, y = x r, r = 1 / max(|x|, eps), upstream gradient g:
// dx = r (dy - y (y . dy)) with dy = scale * g while |x| > eps (r < 1 / eps),
// else dx = r dy (the clamped norm is a constant). Returns y . g, the row's
// share of d scale.
template <int DH>
__device__ __forceinline__ float norm_bwd(const uint16_t* x_row, const uint16_t* g_row, float r, float scale,
                                          uint16_t* dx_row, int lane) {
  Lane<DH> x, g;
  x.load(x_row, lane);
  g.load(g_row, lane);
#pragma unroll
  for (int e = 0; e < Lane<DH>::kE; ++e) x.v[e] *= r;  // y
  const float yg = warp_sum(x.dot(g));
  const float yd = r < 1e6f ? scale * yg : 0.f;
#pragma unroll
  for (int e = 0; e < Lane<DH>::kE; ++e) g.v[e] = scale * g.v[e] - x.v[e] * yd;
  g.store(dx_row, lane, r);
  return yg;
}

template <int DH>
__global__ void __launch_bounds__(32 * kWarps) qk_prepare_bwd_kernel(
    const uint16_t* __restrict__ dq, const uint16_t* __restrict__ dk, const uint16_t* __restrict__ dv,
    const uint16_t* __restrict__ qkv, const uint16_t* __restrict__ perm, const float* __restrict__ tau,
    const float* __restrict__ rnorm, int B, int H, int S, uint16_t* __restrict__ dqkv,
    float* __restrict__ dtau_rows) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= (long long)B * S) return;
  const int b = (int)(t / S), i = (int)(t % S);
  const int D = H * DH;
  const size_t r0 = ((size_t)b * S + min((int)perm[t], S - 1)) * 3 * D;
  for (int h = 0; h < H; ++h) {
    const size_t o = (((size_t)b * H + h) * S + i) * DH;
    const float rq = rnorm[((size_t)b * H + h) * S + i];
    const float rk = rnorm[(((size_t)B + b) * H + h) * S + i];
    const float yg = norm_bwd<DH>(qkv + r0 + h * DH, dq + o, rq, tau[h], dqkv + r0 + h * DH, lane);
    if (lane == 0) dtau_rows[((size_t)b * H + h) * S + i] = yg;
    norm_bwd<DH>(qkv + r0 + D + h * DH, dk + o, rk, 1.f, dqkv + r0 + D + h * DH, lane);
    copy_row<DH>(dqkv + r0 + 2 * D + h * DH, dv + o, lane);
  }
}

// kToTokens: [B,H,S,Dh] permuted -> [B,S,H*Dh] token order; else the reverse.
// One warp per token, its H rows moved as 16-byte chunks (DH / 8 lanes per
// row, 32 / (DH / 8) rows per warp instruction), up to kBatch instructions'
// loads in flight before the stores.
template <int DH, bool kToTokens>
__global__ void __launch_bounds__(32 * kWarps) heads_reorder_kernel(const uint16_t* __restrict__ src,
                                                                    const uint16_t* __restrict__ perm, int B, int H,
                                                                    int S, uint16_t* __restrict__ dst) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  constexpr int kL = DH / 8;
  constexpr int kRows = 32 / kL;
  constexpr int kBatch = 4;
  const int lane = threadIdx.x & 31;
  const long long t = (long long)blockIdx.x * kWarps + (threadIdx.x >> 5);
  if (t >= (long long)B * S) return;
  const int b = (int)(t / S), i = (int)(t % S);
  const int sub = lane % kL, rsel = lane / kL;
  const size_t tok = ((size_t)b * S + min((int)perm[t], S - 1)) * H * DH;
  for (int h0 = 0; h0 < H; h0 += kRows * kBatch) {
    uint4 x[kBatch];
#pragma unroll
    for (int p = 0; p < kBatch; ++p) {
      const int h = h0 + p * kRows + rsel;
      const size_t o = (((size_t)b * H + h) * S + i) * DH + sub * 8;
      if (h < H) x[p] = *reinterpret_cast<const uint4*>(src + (kToTokens ? o : tok + (size_t)h * DH + sub * 8));
    }
#pragma unroll
    for (int p = 0; p < kBatch; ++p) {
      const int h = h0 + p * kRows + rsel;
      const size_t o = (((size_t)b * H + h) * S + i) * DH + sub * 8;
      if (h < H) *reinterpret_cast<uint4*>(dst + (kToTokens ? tok + (size_t)h * DH + sub * 8 : o)) = x[p];
    }
  }
}

inline unsigned blocks_for(long long tokens) { return (unsigned)((tokens + kWarps - 1) / kWarps); }

}  // namespace tok
}  // namespace rt

namespace {

int check_shape(int32_t batch, int32_t heads, int32_t seq_len, int32_t head_dim) {
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len > 65536 || heads > 256) return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != 32 && head_dim != 64) return RT_ERR_UNSUPPORTED;
  return RT_OK;
}

bool all_aligned(std::initializer_list<const void*> ps) {
  for (const void* p : ps)
    if (!p || !rt::aligned16(p)) return false;
  return true;
}

}  // namespace

extern "C" int rt_qk_prepare(const uint16_t* qkv, const uint16_t* perm, const float* tau, int32_t batch,
                             int32_t heads, int32_t seq_len, int32_t head_dim, uint16_t* q, uint16_t* k,
                             uint16_t* v, float* rnorm, void* stream) {
  using namespace rt;
  if (int st = check_shape(batch, heads, seq_len, head_dim)) return st;
  if ((long long)batch * heads * seq_len == 0) return RT_OK;
  if (!all_aligned({qkv, perm, tau, q, k, v, rnorm})) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(qkv);
  if (guard.status() != RT_OK) return guard.status();
  const unsigned grid = tok::blocks_for((long long)batch * seq_len);
  auto s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    {
      if (int st_pdl = launch_pdl("qk_prepare_kernel launch", tok::qk_prepare_kernel<64>, dim3(grid), dim3(32 *
          tok::kWarps), 0, s, qkv, perm, tau, batch, heads, seq_len, q, k, v, rnorm)) return st_pdl;
    }
  else
    {
      if (int st_pdl = launch_pdl("qk_prepare_kernel launch", tok::qk_prepare_kernel<32>, dim3(grid), dim3(32 *
          tok::kWarps), 0, s, qkv, perm, tau, batch, heads, seq_len, q, k, v, rnorm)) return st_pdl;
    }
  return check_launch("qk_prepare_kernel launch");
}

extern "C" int rt_qk_prepare_bwd(const uint16_t* dq, const uint16_t* dk, const uint16_t* dv, const uint16_t* qkv,
                                 const uint16_t* perm, const float* tau, const float* rnorm, int32_t batch,
                                 int32_t heads, int32_t seq_len, int32_t head_dim, uint16_t* dqkv,
                                 float* dtau_rows, void* stream) {
  using namespace rt;
  if (int st = check_shape(batch, heads, seq_len, head_dim)) return st;
  if ((long long)batch * heads * seq_len == 0) return RT_OK;
  if (!all_aligned({dq, dk, dv, qkv, perm, tau, rnorm, dqkv, dtau_rows})) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(qkv);
  if (guard.status() != RT_OK) return guard.status();
  const unsigned grid = tok::blocks_for((long long)batch * seq_len);
  auto s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    {
      if (int st_pdl = launch_pdl("qk_prepare_bwd_kernel launch", tok::qk_prepare_bwd_kernel<64>, dim3(grid),
          dim3(32 * tok::kWarps), 0, s, dq, dk, dv, qkv, perm, tau, rnorm, batch, heads, seq_len, dqkv,
          dtau_rows)) return st_pdl;
    }
  else
    {
      if (int st_pdl = launch_pdl("qk_prepare_bwd_kernel launch", tok::qk_prepare_bwd_kernel<32>, dim3(grid),
          dim3(32 * tok::kWarps), 0, s, dq, dk, dv, qkv, perm, tau, rnorm, batch, heads, seq_len, dqkv,
          dtau_rows)) return st_pdl;
    }
  return check_launch("qk_prepare_bwd_kernel launch");
}

namespace {
template <bool kToTokens>
int heads_reorder(const uint16_t* src, const uint16_t* perm, int32_t batch, int32_t heads, int32_t seq_len,
                  int32_t head_dim, uint16_t* dst, void* stream) {
  using namespace rt;
  if (int st = check_shape(batch, heads, seq_len, head_dim)) return st;
  if ((long long)batch * heads * seq_len == 0) return RT_OK;
  if (!all_aligned({src, perm, dst})) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(src);
  if (guard.status() != RT_OK) return guard.status();
  const unsigned grid = tok::blocks_for((long long)batch * seq_len);
  auto s = static_cast<cudaStream_t>(stream);
  if (head_dim == 64)
    {
      if (int st_pdl = launch_pdl("heads_reorder_kernel launch", tok::heads_reorder_kernel<64, kToTokens>,
          dim3(grid), dim3(32 * tok::kWarps), 0, s, src, perm, batch, heads, seq_len, dst)) return st_pdl;
    }
  else
    {
      if (int st_pdl = launch_pdl("heads_reorder_kernel launch", tok::heads_reorder_kernel<32, kToTokens>,
          dim3(grid), dim3(32 * tok::kWarps), 0, s, src, perm, batch, heads, seq_len, dst)) return st_pdl;
    }
  return check_launch("heads_reorder_kernel launch");
}
}  // namespace

extern "C" int rt_heads_unpermute(const uint16_t* o, const uint16_t* perm, int32_t batch, int32_t heads,
                                  int32_t seq_len, int32_t head_dim, uint16_t* out, void* stream) {
  return heads_reorder<true>(o, perm, batch, heads, seq_len, head_dim, out, stream);
}

extern "C" int rt_heads_permute(const uint16_t* x, const uint16_t* perm, int32_t batch, int32_t heads,
                                int32_t seq_len, int32_t head_dim, uint16_t* out, void* stream) {
  return heads_reorder<false>(x, perm, batch, heads, seq_len, head_dim, out, stream);
}
