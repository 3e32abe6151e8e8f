// rt_attention_bwd_noalloc: the attention backward for callers that cannot
// allocate device memory.
//
// rt_attention_bwd needs a caller-provided workspace (per-query lse and
// rowsum(dO * O), padded to whole tiles). Some callers only ever hand the
// library the buffers of the operation itself: a plugin host or FFI handler
// with no hook for scratch allocation, or a service whose device memory is
// fixed at start-up and which may not call cudaMalloc afterwards. For them
// this entry point keeps that workspace in a fixed array compiled into the
// library instead.
//
// Limits and sharing:
//   - The array holds kNoAllocRows padded query rows (batch * heads *
//     seq_len rounded up to 128) -- 8 MB of device memory that every GPU
//     loading the library keeps until the process exits. Larger problems are
//     rejected with RT_ERR_WORKSPACE before any device work.
//   - Every call on a device uses the same array and leaves its contents
//     behind. Nothing in it has to start at zero: each call rewrites every
//     entry it reads. Calls whose kernels overlap on the GPU (e.g. issued on
//     two streams without ordering) race on the array and give wrong results;
//     order them on one stream or with events.
//   - The first call on each device looks up the array's device address
//     (cudaGetSymbolAddress) with that device current; make that first call
//     before any stream capture.
#include <mutex>

namespace rt {
namespace noalloc {

constexpr long long kNoAllocRows = 1LL << 20;  // padded query rows (2 floats each)

static __device__ __align__(256) float g_bwd_scratch[2 * kNoAllocRows];

// Device addresses of g_bwd_scratch, one per device, looked up on first use.
// In host code `g_bwd_scratch` names a host-side stand-in, not device memory,
// so kernels must be given these looked-up addresses instead.
int scratch_address(float** out) {
  static std::mutex mu;
  static float* addr[64] = {nullptr};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_failure(e, "cudaGetDevice");
  if (dev < 0 || dev >= 64) return RT_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (addr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_bwd_scratch);
    if (e != cudaSuccess) return cuda_failure(e, "cudaGetSymbolAddress(g_bwd_scratch)");
    addr[dev] = static_cast<float*>(p);
  }
  *out = addr[dev];
  return RT_OK;
}

}  // namespace noalloc
}  // namespace rt

extern "C" int rt_attention_bwd_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                                        const uint16_t* o, const uint16_t* d_o, const float* lse,
                                        int32_t batch, int32_t heads, int32_t seq_len, int32_t head_dim,
                                        float scale, const rt_tile_plan* plan, uint16_t* dq,
                                        uint16_t* dk, uint16_t* dv, void* stream) {
  using namespace rt;
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len > 65536 || batch > 65535 || heads > 65535)
    return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != 32 && head_dim != 64) return RT_ERR_UNSUPPORTED;
  // masked logits enter as -inf times the scale, and the fused backward divides by it
  if (!(scale > 0.f) || !(scale < INFINITY)) return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || heads == 0 || seq_len == 0) return RT_OK;
  const long long padded_rows =
      (long long)batch * heads * ((long long)(seq_len + RT_TILE - 1) / RT_TILE) * RT_TILE;
  if (padded_rows > noalloc::kNoAllocRows) return RT_ERR_WORKSPACE;
  if (!plan_matches(plan, batch, seq_len)) return RT_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv) return RT_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {q, k, v, o, d_o, lse, dq, dk, dv};
  for (const void* p : ptrs)
    if (!aligned16(p)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(q);
  if (guard.status() != RT_OK) return guard.status();
  float* scratch = nullptr;
  const int st = noalloc::scratch_address(&scratch);
  if (st != RT_OK) return st;
  return launch_attention_bwd(q, k, v, o, d_o, lse, batch, heads, seq_len, head_dim, scale, *plan, dq, dk, dv,
                              scratch, nullptr, nullptr, static_cast<cudaStream_t>(stream));
}
