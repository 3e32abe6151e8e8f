// Fused elementwise and normalisation kernels of the encoder layer around the
// attention sublayers (the training step's non-attention work), memory-bound:
// one pass over each tensor instead of the chains of casts, multiplies and
// reductions a framework runs for them.
//
//   rms_norm      y = bf16(x / sqrt(mean(x^2) + eps) * (1 + gamma))
//                 (confluence/confluence/layers.py:16-30, ZeroCenteredRMSNorm),
//                 x fp32 [rows][d], y bf16, rstd fp32 [rows] kept for the backward
//   rms_norm_bwd  dx = rstd (g - xh mean(g xh)), g = dy (1 + gamma), xh = x rstd;
//                 dgamma = sum over rows of dy xh: per-block partial sums, then a
//                 second pass over the blocks in a fixed order (deterministic)
//   gate_residual y = x + scale * o * sigmoid(gate)   (layers.py:170-174)
//                 x fp32, o / gate bf16 [rows][d], y fp32; backward
//                 do = bf16(dy scale sigmoid(gate)), dgate = bf16(dy scale o s (1 - s))
//   residual_add  y = x + scale * h (the FFN's residual, layers.py:233-236), x fp32,
//                 h bf16 (the W_down output), y fp32; backward dh = bf16(dy scale)
//   swiglu        h = bf16(silu(a) * b) with a = u[:, :f], b = u[:, f:] of the
//                 fused [rows][2f] up-projection (layers.py:177-200); backward
//                 du = [bf16(dh b silu'(a)) | bf16(dh silu(a))]
// Each thread handles 8 consecutive elements (16-byte bf16 / 32-byte fp32
// accesses); the width d (or f) must be a multiple of 8.

namespace rt {
namespace layer {

struct F8 {
  float v[8];
};

__device__ __forceinline__ F8 load_f32x8(const float* p) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  return F8{{a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w}};
}
__device__ __forceinline__ void store_f32x8(float* p, const F8& f) {
  *reinterpret_cast<float4*>(p) = make_float4(f.v[0], f.v[1], f.v[2], f.v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(f.v[4], f.v[5], f.v[6], f.v[7]);
}
__device__ __forceinline__ F8 load_bf16x8(const uint16_t* p) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  F8 f;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = unpack_bf16x2(w[i]);
    f.v[2 * i] = t.x;
    f.v[2 * i + 1] = t.y;
  }
  return f;
}
__device__ __forceinline__ void store_bf16x8(uint16_t* p, const F8& f) {
  *reinterpret_cast<uint4*>(p) = make_uint4(pack_bf16x2(f.v[0], f.v[1]), pack_bf16x2(f.v[2], f.v[3]),
                                            pack_bf16x2(f.v[4], f.v[5]), pack_bf16x2(f.v[6], f.v[7]));
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.f / (1.f + __expf(-x)); }

constexpr int kMaxD = 1024;  // row width of the norms: at most 4 groups of 8 per lane

// One warp per row; lane handles groups lane, lane + 32, ... of 8 columns.
template <int G>
__global__ void __launch_bounds__(256) rms_norm_kernel(const float* __restrict__ x, const float* __restrict__ gamma,
                                                       long long rows, int d, float eps, uint16_t* __restrict__ y,
                                                       float* __restrict__ rstd) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const int lane = threadIdx.x & 31;
  const long long row = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int groups = d >> 3;
  const float* xr = x + row * d;
  F8 xv[G];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int gi = lane + 32 * j;
    if (gi < groups) {
      xv[j] = load_f32x8(xr + gi * 8);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(xv[j].v[e], xv[j].v[e], ss);
    }
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xFFFFFFFFu, ss, off);
  const float r = rsqrtf(ss / (float)d + eps);
  if (lane == 0) rstd[row] = r;
#pragma unroll
  for (int j = 0; j < G; ++j) {
    const int gi = lane + 32 * j;
    if (gi < groups) {
      const F8 gm = load_f32x8(gamma + gi * 8);
      F8 o;
#pragma unroll
      for (int e = 0; e < 8; ++e) o.v[e] = xv[j].v[e] * r * (1.f + gm.v[e]);
      store_bf16x8(y + row * d + gi * 8, o);
    }
  }
}

// One warp per row, warps of a block stride over rows; each block leaves its
// partial dgamma (sum over its rows) in part[blockIdx.x][d].
template <int G>
__global__ void __launch_bounds__(256) rms_norm_bwd_kernel(const uint16_t* __restrict__ dy, const float* __restrict__ x,
                                                           const float* __restrict__ gamma,
                                                           const float* __restrict__ rstd, long long rows, int d,
                                                           float* __restrict__ dx, float* __restrict__ part) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  __shared__ float sred[8][kMaxD / 8 + 1];  // per warp, one float per group slot (reduced below)
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nwarps = blockDim.x >> 5;
  const int groups = d >> 3;
  F8 dg[G];
#pragma unroll
  for (int j = 0; j < G; ++j)
#pragma unroll
    for (int e = 0; e < 8; ++e) dg[j].v[e] = 0.f;
  F8 gm[G];
#pragma unroll
  for (int j = 0; j < G; ++j)
    if (lane + 32 * j < groups) gm[j] = load_f32x8(gamma + (lane + 32 * j) * 8);
  for (long long row = (long long)blockIdx.x * nwarps + warp; row < rows; row += (long long)gridDim.x * nwarps) {
    const float r = rstd[row];
    F8 xh[G], g[G];
    float dot = 0.f;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int gi = lane + 32 * j;
      if (gi < groups) {
        const F8 xv = load_f32x8(x + row * d + gi * 8);
        const F8 dv = load_bf16x8(dy + row * d + gi * 8);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          xh[j].v[e] = xv.v[e] * r;
          g[j].v[e] = dv.v[e] * (1.f + gm[j].v[e]);
          dot = fmaf(g[j].v[e], xh[j].v[e], dot);
          dg[j].v[e] = fmaf(dv.v[e], xh[j].v[e], dg[j].v[e]);
        }
      }
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) dot += __shfl_xor_sync(0xFFFFFFFFu, dot, off);
    const float mdot = dot / (float)d;
#pragma unroll
    for (int j = 0; j < G; ++j) {
      const int gi = lane + 32 * j;
      if (gi < groups) {
        F8 o;
#pragma unroll
        for (int e = 0; e < 8; ++e) o.v[e] = r * (g[j].v[e] - xh[j].v[e] * mdot);
        store_f32x8(dx + row * d + gi * 8, o);
      }
    }
  }
  // block partial of dgamma: the warps' sums, element by element, in a fixed order
#pragma unroll
  for (int e = 0; e < 8; ++e) {
#pragma unroll
    for (int j = 0; j < G; ++j)
      if (lane + 32 * j < groups) sred[warp][lane + 32 * j] = dg[j].v[e];
    __syncthreads();
    for (int gi = threadIdx.x; gi < groups; gi += blockDim.x) {
      float s = 0.f;
      for (int w = 0; w < nwarps; ++w) s += sred[w][gi];
      part[(size_t)blockIdx.x * d + gi * 8 + e] = s;
    }
    __syncthreads();
  }
}

// dgamma[c] = sum over the blocks' partials: a block takes 32 columns, its
// eight warps each sum every eighth partial (lane = column), and the eight
// warp sums are added in warp order -- a fixed order, so the result is
// deterministic.
__global__ void __launch_bounds__(256) sum_partials_kernel(const float* __restrict__ part, int nparts, int d,
                                                           float* __restrict__ out) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  __shared__ float sw[8][32];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int c = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (c < d)
    for (int p = warp; p < nparts; p += 8) s += part[(size_t)p * d + c];
  sw[warp][lane] = s;
  __syncthreads();
  if (warp == 0 && c < d) {
    float t = 0.f;
#pragma unroll
    for (int w = 0; w < 8; ++w) t += sw[w][lane];
    out[c] = t;
  }
}

__global__ void __launch_bounds__(256) gate_residual_kernel(const float* __restrict__ x, const uint16_t* __restrict__ o,
                                                            const uint16_t* __restrict__ gate, long long n8, float scale,
                                                            float* __restrict__ y) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const F8 xv = load_f32x8(x + i * 8), ov = load_bf16x8(o + i * 8), gv = load_bf16x8(gate + i * 8);
    F8 r;
#pragma unroll
    for (int e = 0; e < 8; ++e) r.v[e] = xv.v[e] + scale * ov.v[e] * sigmoidf_(gv.v[e]);
    store_f32x8(y + i * 8, r);
  }
}

__global__ void __launch_bounds__(256) gate_residual_bwd_kernel(const float* __restrict__ dy,
                                                                const uint16_t* __restrict__ o,
                                                                const uint16_t* __restrict__ gate, long long n8,
                                                                float scale, uint16_t* __restrict__ d_o,
                                                                uint16_t* __restrict__ d_gate) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const F8 g = load_f32x8(dy + i * 8), ov = load_bf16x8(o + i * 8), gv = load_bf16x8(gate + i * 8);
    F8 a, b;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float s = sigmoidf_(gv.v[e]);
      a.v[e] = g.v[e] * scale * s;
      b.v[e] = g.v[e] * scale * ov.v[e] * s * (1.f - s);
    }
    store_bf16x8(d_o + i * 8, a);
    store_bf16x8(d_gate + i * 8, b);
  }
}

__global__ void __launch_bounds__(256) residual_add_kernel(const float* __restrict__ x, const uint16_t* __restrict__ h,
                                                           long long n8, float scale, float* __restrict__ y) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const F8 xv = load_f32x8(x + i * 8), hv = load_bf16x8(h + i * 8);
    F8 r;
#pragma unroll
    for (int e = 0; e < 8; ++e) r.v[e] = xv.v[e] + scale * hv.v[e];
    store_f32x8(y + i * 8, r);
  }
}

__global__ void __launch_bounds__(256) residual_add_bwd_kernel(const float* __restrict__ dy, long long n8, float scale,
                                                               uint16_t* __restrict__ dh) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    F8 g = load_f32x8(dy + i * 8);
#pragma unroll
    for (int e = 0; e < 8; ++e) g.v[e] *= scale;
    store_bf16x8(dh + i * 8, g);
  }
}

// u [rows][2f]: a = u[:, :f], b = u[:, f:]; h [rows][f]
__global__ void __launch_bounds__(256) swiglu_kernel(const uint16_t* __restrict__ u, long long rows, int f,
                                                     uint16_t* __restrict__ h) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const int g8 = f >> 3;
  const long long n8 = rows * g8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / g8;
    const int c = (int)(i % g8) * 8;
    const F8 a = load_bf16x8(u + row * 2 * f + c), b = load_bf16x8(u + row * 2 * f + f + c);
    F8 r;
#pragma unroll
    for (int e = 0; e < 8; ++e) r.v[e] = a.v[e] * sigmoidf_(a.v[e]) * b.v[e];
    store_bf16x8(h + row * f + c, r);
  }
}

__global__ void __launch_bounds__(256) swiglu_bwd_kernel(const uint16_t* __restrict__ dh, const uint16_t* __restrict__ u,
                                                         long long rows, int f, uint16_t* __restrict__ du) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  const int g8 = f >> 3;
  const long long n8 = rows * g8;
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (long long)gridDim.x * blockDim.x) {
    const long long row = i / g8;
    const int c = (int)(i % g8) * 8;
    const F8 g = load_bf16x8(dh + row * f + c);
    const F8 a = load_bf16x8(u + row * 2 * f + c), b = load_bf16x8(u + row * 2 * f + f + c);
    F8 da, db;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float s = sigmoidf_(a.v[e]);
      const float silu = a.v[e] * s;
      da.v[e] = g.v[e] * b.v[e] * s * (1.f + a.v[e] * (1.f - s));
      db.v[e] = g.v[e] * silu;
    }
    store_bf16x8(du + row * 2 * f + c, da);
    store_bf16x8(du + row * 2 * f + f + c, db);
  }
}

constexpr int kNormBwdBlocks = 2 * 148;  // blocks of rms_norm_bwd_kernel = dgamma partial rows

int grid_for(long long work, int per_block) {
  long long g = (work + per_block - 1) / per_block;
  return (int)std::min<long long>(std::max<long long>(g, 1), 148LL * 16);
}

}  // namespace layer
}  // namespace rt

namespace {
bool ok16(const void* p) { return p != nullptr && (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }
}  // namespace

extern "C" int rt_rms_norm(const float* x, const float* gamma, int64_t rows, int32_t d, float eps, uint16_t* y,
                           float* rstd, void* stream) {
  using namespace rt;
  if (rows < 0 || d <= 0 || d % 8 != 0 || d > layer::kMaxD || !(eps >= 0.f)) return RT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RT_OK;
  if (!ok16(x) || !ok16(gamma) || !ok16(y) || !rstd) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(x);
  if (guard.status() != RT_OK) return guard.status();
  const int blocks = (int)((rows + 7) / 8);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int gpl = (d / 8 + 31) / 32;  // groups of 8 per lane
  if (gpl <= 2) {
   if (int st_pdl = launch_pdl("rms_norm_kernel launch", layer::rms_norm_kernel<2>, dim3(blocks), dim3(256), 0,
       s, x, gamma, rows, d, eps, y, rstd)) return st_pdl;
 }
  else {
   if (int st_pdl = launch_pdl("rms_norm_kernel launch", layer::rms_norm_kernel<4>, dim3(blocks), dim3(256), 0,
       s, x, gamma, rows, d, eps, y, rstd)) return st_pdl;
 }
  return check_launch("rms_norm_kernel launch");
}

extern "C" size_t rt_rms_norm_bwd_workspace_bytes(int64_t rows, int32_t d) {
  (void)rows;
  return sizeof(float) * (size_t)rt::layer::kNormBwdBlocks * (size_t)(d > 0 ? d : 0);
}

extern "C" int rt_rms_norm_bwd(const uint16_t* dy, const float* x, const float* gamma, const float* rstd, int64_t rows,
                               int32_t d, float* dx, float* dgamma, void* workspace, size_t workspace_bytes,
                               void* stream) {
  using namespace rt;
  if (rows < 0 || d <= 0 || d % 8 != 0 || d > layer::kMaxD) return RT_ERR_INVALID_ARGUMENT;
  if (!ok16(dy) || !ok16(x) || !ok16(gamma) || !rstd || !ok16(dx) || !dgamma || !ok16(workspace))
    return RT_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < rt_rms_norm_bwd_workspace_bytes(rows, d)) return RT_ERR_WORKSPACE;
  DeviceGuard guard(x);
  if (guard.status() != RT_OK) return guard.status();
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int blocks = layer::kNormBwdBlocks;
  float* part = static_cast<float*>(workspace);
  const int gpl = (d / 8 + 31) / 32;
  if (gpl <= 2) {
   if (int st_pdl = launch_pdl("rms_norm_bwd_kernel launch", layer::rms_norm_bwd_kernel<2>, dim3(blocks),
       dim3(256), 0, s, dy, x, gamma, rstd, rows, d, dx, part)) return st_pdl;
 }
  else {
   if (int st_pdl = launch_pdl("rms_norm_bwd_kernel launch", layer::rms_norm_bwd_kernel<4>, dim3(blocks),
       dim3(256), 0, s, dy, x, gamma, rstd, rows, d, dx, part)) return st_pdl;
 }
  if (int st = check_launch("rms_norm_bwd_kernel launch")) return st;
  {
    if (int st_pdl = launch_pdl("sum_partials_kernel launch", layer::sum_partials_kernel, dim3((d + 31) / 32),
        dim3(256), 0, s, part, blocks, d, dgamma)) return st_pdl;
  }
  return check_launch("sum_partials_kernel launch");
}

extern "C" int rt_gate_residual(const float* x, const uint16_t* o, const uint16_t* gate, int64_t n, float scale,
                                float* y, void* stream) {
  using namespace rt;
  if (n < 0 || n % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  if (!ok16(x) || !ok16(o) || !ok16(gate) || !ok16(y)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(x);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("gate_residual_kernel launch", layer::gate_residual_kernel,
        dim3(layer::grid_for(n / 8, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), x, o, gate, n / 8,
        scale, y)) return st_pdl;
  }
  return check_launch("gate_residual_kernel launch");
}

extern "C" int rt_gate_residual_bwd(const float* dy, const uint16_t* o, const uint16_t* gate, int64_t n, float scale,
                                    uint16_t* d_o, uint16_t* d_gate, void* stream) {
  using namespace rt;
  if (n < 0 || n % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  if (!ok16(dy) || !ok16(o) || !ok16(gate) || !ok16(d_o) || !ok16(d_gate)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(dy);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("gate_residual_bwd_kernel launch", layer::gate_residual_bwd_kernel,
        dim3(layer::grid_for(n / 8, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), dy, o, gate, n / 8,
        scale, d_o, d_gate)) return st_pdl;
  }
  return check_launch("gate_residual_bwd_kernel launch");
}

extern "C" int rt_swiglu(const uint16_t* u, int64_t rows, int32_t f, uint16_t* h, void* stream) {
  using namespace rt;
  if (rows < 0 || f <= 0 || f % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RT_OK;
  if (!ok16(u) || !ok16(h)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(u);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("swiglu_kernel launch", layer::swiglu_kernel, dim3(layer::grid_for(rows * (f /
        8), 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), u, rows, f, h)) return st_pdl;
  }
  return check_launch("swiglu_kernel launch");
}

extern "C" int rt_swiglu_bwd(const uint16_t* dh, const uint16_t* u, int64_t rows, int32_t f, uint16_t* du,
                             void* stream) {
  using namespace rt;
  if (rows < 0 || f <= 0 || f % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (rows == 0) return RT_OK;
  if (!ok16(dh) || !ok16(u) || !ok16(du)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(u);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("swiglu_bwd_kernel launch", layer::swiglu_bwd_kernel, dim3(layer::grid_for(rows
        * (f / 8), 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), dh, u, rows, f, du)) return st_pdl;
  }
  return check_launch("swiglu_bwd_kernel launch");
}

extern "C" int rt_residual_add(const float* x, const uint16_t* h, int64_t n, float scale, float* y, void* stream) {
  using namespace rt;
  if (n < 0 || n % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  if (!ok16(x) || !ok16(h) || !ok16(y)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(x);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("residual_add_kernel launch", layer::residual_add_kernel, dim3(layer::grid_for(n
        / 8, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), x, h, n / 8, scale, y)) return st_pdl;
  }
  return check_launch("residual_add_kernel launch");
}

extern "C" int rt_residual_add_bwd(const float* dy, int64_t n, float scale, uint16_t* dh, void* stream) {
  using namespace rt;
  if (n < 0 || n % 8 != 0) return RT_ERR_INVALID_ARGUMENT;
  if (n == 0) return RT_OK;
  if (!ok16(dy) || !ok16(dh)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(dy);
  if (guard.status() != RT_OK) return guard.status();
  {
    if (int st_pdl = launch_pdl("residual_add_bwd_kernel launch", layer::residual_add_bwd_kernel,
        dim3(layer::grid_for(n / 8, 256)), dim3(256), 0, static_cast<cudaStream_t>(stream), dy, n / 8, scale,
        dh)) return st_pdl;
  }
  return check_launch("residual_add_bwd_kernel launch");
}
