// C ABI of the library: argument validation, plan layout, TMA descriptors and
// launches. See include/rt_attention.h for the contract of each entry point.
#include <cstdio>
#include <cstring>
#include <mutex>

#include "rt_device.cuh"
#include "rt_internal.h"

namespace rt {

namespace {
thread_local char g_last_error[256] = "";
}

int cuda_failure(cudaError_t err, const char* site) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: %s (%s)", site, cudaGetErrorName(err),
           cudaGetErrorString(err));
  return RT_ERR_CUDA;
}

int driver_failure(int err, const char* site) {
  snprintf(g_last_error, sizeof(g_last_error), "%s: CUresult %d", site, err);
  return RT_ERR_CUDA;
}

namespace {

constexpr size_t kAlign = 256;
inline size_t align_up(size_t x) { return (x + kAlign - 1) & ~(kAlign - 1); }

struct PlanLayout {
  size_t live, full, q2k_ptr, q2k_idx, k2q_ptr, k2q_idx, masks, masks_t, fk, nnz, total;
};

PlanLayout plan_layout(int B, int S, int R) {
  const size_t T = (size_t)(S + RT_TILE - 1) / RT_TILE;
  const size_t W = (T + 31) / 32;
  const size_t WR = ((size_t)R + 31) / 32;
  PlanLayout L{};
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  L.live = take(sizeof(uint32_t) * B * T * W);
  L.full = take(sizeof(uint32_t) * B * T * W);
  L.q2k_ptr = take(sizeof(int32_t) * (B * T + 1));
  L.q2k_idx = take(sizeof(int32_t) * B * T * T);
  L.k2q_ptr = take(sizeof(int32_t) * (B * T + 1));
  L.k2q_idx = take(sizeof(int32_t) * B * T * T);
  L.masks = take(sizeof(uint32_t) * 4 * RT_TILE * B * T * T);
  L.masks_t = take(sizeof(uint32_t) * 4 * RT_TILE * B * T * T);
  L.fk = take(sizeof(uint32_t) * B * (size_t)R * WR);
  L.nnz = take(sizeof(int32_t) * (1 + (size_t)B));  // the count, then per-sample perm flags
  L.total = off;
  return L;
}

// sm_100 check, cached per device.
int check_device() {
  static std::mutex mu;
  static int verdict[64] = {0};  // 0 unknown, 1 ok, 2 bad
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return RT_ERR_DEVICE;
  if (dev < 0 || dev >= 64) return RT_ERR_DEVICE;
  std::lock_guard<std::mutex> lock(mu);
  if (verdict[dev] == 0) {
    int major = 0, minor = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return RT_ERR_DEVICE;
    verdict[dev] = (major == 10 && minor == 0) ? 1 : 2;
  }
  return verdict[dev] == 1 ? RT_OK : RT_ERR_DEVICE;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Makes the device that owns `ptr` current for the duration of an entry point,
// so that calls from threads with no current CUDA context (a framework's
// worker threads) and with another device current both work. A different
// previous device is restored on exit.
class DeviceGuard {
 public:
  explicit DeviceGuard(const void* ptr) {
    cudaPointerAttributes attr;
    cudaError_t e = cudaPointerGetAttributes(&attr, ptr);
    if (e != cudaSuccess) {
      status_ = cuda_failure(e, "cudaPointerGetAttributes");
      return;
    }
    if (attr.type != cudaMemoryTypeDevice && attr.type != cudaMemoryTypeManaged) {
      status_ = RT_ERR_INVALID_ARGUMENT;
      return;
    }
    int cur = -1;
    if (cudaGetDevice(&cur) != cudaSuccess) cur = -1;
    // cudaSetDevice also makes the device's primary context current on this thread.
    e = cudaSetDevice(attr.device);
    if (e != cudaSuccess) {
      status_ = cuda_failure(e, "cudaSetDevice");
      return;
    }
    if (cur >= 0 && cur != attr.device) restore_ = cur;
    status_ = check_device();
  }
  ~DeviceGuard() {
    if (restore_ >= 0) cudaSetDevice(restore_);
  }
  int status() const { return status_; }

 private:
  int status_ = RT_OK;
  int restore_ = -1;
};

bool plan_matches(const rt_tile_plan* plan, int B, int S) {
  return plan != nullptr && plan->batch == B && plan->seq_len == S &&
         plan->tiles == (S + RT_TILE - 1) / RT_TILE && plan->live_bits && plan->full_bits &&
         plan->q2k_ptr && plan->q2k_idx && plan->k2q_ptr && plan->k2q_idx && plan->tile_masks &&
         plan->tile_masks_t && plan->nnz;
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*,
                                  const cuuint64_t*, const cuuint64_t*, const cuuint32_t*,
                                  const cuuint32_t*, CUtensorMapInterleave, CUtensorMapSwizzle,
                                  CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult q;
    void* p = nullptr;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

}  // namespace

int make_qkv_tensor_map(CUtensorMap* map, const void* base, int BH, int S, int Dh) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return driver_failure(-1, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  cuuint64_t dims[3] = {(cuuint64_t)Dh, (cuuint64_t)S, (cuuint64_t)BH};
  cuuint64_t strides[2] = {(cuuint64_t)Dh * 2, (cuuint64_t)Dh * 2 * (cuuint64_t)S};
  cuuint32_t box[3] = {(cuuint32_t)Dh, (cuuint32_t)RT_TILE, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  const CUtensorMapSwizzle sw = Dh == 64 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B;
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                  estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RT_OK : driver_failure((int)r, "cuTensorMapEncodeTiled");
}

// fp32 accumulator [rows][Dh] as boxes of 32 rows x 32 floats (128 B rows,
// the 128-byte swizzle), for the TMA reduce-adds of the fused backward.
int make_acc_tensor_map(CUtensorMap* map, float* base, long long rows, int Dh) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return driver_failure(-1, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  cuuint64_t dims[2] = {(cuuint64_t)Dh, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)Dh * 4};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RT_OK : driver_failure((int)r, "cuTensorMapEncodeTiled(dq accumulator)");
}

// Row-statistic operand rows [rows][16] bf16 (32 B each) as boxes of 128 rows
// with the 32-byte swizzle: one K-major MMA operand tile per box.
int make_aux_tensor_map(CUtensorMap* map, uint16_t* base, long long rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return driver_failure(-1, "cudaGetDriverEntryPoint(cuTensorMapEncodeTiled)");
  cuuint64_t dims[2] = {16, (cuuint64_t)rows};
  cuuint64_t strides[1] = {32};
  cuuint32_t box[2] = {16, (cuuint32_t)RT_TILE};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, base, dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? RT_OK : driver_failure((int)r, "cuTensorMapEncodeTiled(row statistics)");
}

}  // namespace rt

using namespace rt;

extern "C" {

size_t rt_tile_plan_bytes(int32_t batch, int32_t seq_len, int32_t max_rows) {
  if (batch < 0 || seq_len < 0 || max_rows < 0) return 0;
  return plan_layout(batch, seq_len, max_rows).total;
}

int rt_tile_plan_bind(void* buffer, size_t bytes, int32_t batch, int32_t seq_len, int32_t max_rows,
                      rt_tile_plan* plan) {
  if (plan == nullptr || batch < 0 || seq_len < 0 || max_rows < 0) return RT_ERR_INVALID_ARGUMENT;
  if (seq_len > 65536) return RT_ERR_INVALID_ARGUMENT;  // perm is uint16
  if (batch == 0 || seq_len == 0) {  // empty problem: nothing to carve
    std::memset(plan, 0, sizeof(*plan));
    plan->batch = batch;
    plan->seq_len = seq_len;
    plan->max_rows = max_rows;
    return RT_OK;
  }
  const PlanLayout L = plan_layout(batch, seq_len, max_rows);
  if (buffer == nullptr) return RT_ERR_INVALID_ARGUMENT;
  if ((reinterpret_cast<uintptr_t>(buffer) & (kAlign - 1)) != 0) return RT_ERR_INVALID_ARGUMENT;
  if (bytes < L.total) return RT_ERR_WORKSPACE;
  uint8_t* base = static_cast<uint8_t*>(buffer);
  const int T = (seq_len + RT_TILE - 1) / RT_TILE;
  plan->batch = batch;
  plan->seq_len = seq_len;
  plan->max_rows = max_rows;
  plan->tiles = T;
  plan->words = (T + 31) / 32;
  plan->live_bits = reinterpret_cast<uint32_t*>(base + L.live);
  plan->full_bits = reinterpret_cast<uint32_t*>(base + L.full);
  plan->q2k_ptr = reinterpret_cast<int32_t*>(base + L.q2k_ptr);
  plan->q2k_idx = reinterpret_cast<int32_t*>(base + L.q2k_idx);
  plan->k2q_ptr = reinterpret_cast<int32_t*>(base + L.k2q_ptr);
  plan->k2q_idx = reinterpret_cast<int32_t*>(base + L.k2q_idx);
  plan->tile_masks = reinterpret_cast<uint32_t*>(base + L.masks);
  plan->tile_masks_t = reinterpret_cast<uint32_t*>(base + L.masks_t);
  plan->fk_bits = reinterpret_cast<uint32_t*>(base + L.fk);
  plan->nnz = reinterpret_cast<int32_t*>(base + L.nnz);
  return RT_OK;
}

int rt_build_tile_plan(const uint16_t* perm, const uint16_t* seq_row_ids, const int32_t* column_ids,
                       const uint8_t* is_padding, const uint8_t* fk_adj, int32_t batch, int32_t seq_len,
                       int32_t max_rows, int32_t kind, const rt_tile_plan* plan, void* stream) {
  if (batch < 0 || seq_len < 0 || max_rows < 0 || seq_len > 65536 || batch > 65535)
    return RT_ERR_INVALID_ARGUMENT;
  if (kind < RT_MASK_COLUMN || kind > RT_MASK_FULL) return RT_ERR_INVALID_ARGUMENT;
  if (plan == nullptr || plan->batch != batch || plan->seq_len != seq_len || plan->max_rows != max_rows)
    return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || seq_len == 0) return RT_OK;
  if (!plan_matches(plan, batch, seq_len)) return RT_ERR_INVALID_ARGUMENT;
  if (!perm || !seq_row_ids || !column_ids || !is_padding) return RT_ERR_INVALID_ARGUMENT;
  const bool needs_fk = (kind == RT_MASK_FEATURE || kind == RT_MASK_NEIGHBOR) && max_rows > 0;
  if (needs_fk && (!fk_adj || !plan->fk_bits)) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(perm);
  if (guard.status() != RT_OK) return guard.status();
  return launch_build_tile_plan(perm, seq_row_ids, column_ids, is_padding, fk_adj, batch, seq_len,
                                max_rows, kind, *plan, static_cast<cudaStream_t>(stream));
}

int rt_attention_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t batch,
                     int32_t heads, int32_t seq_len, int32_t head_dim, float scale,
                     const rt_tile_plan* plan, uint16_t* o, float* lse, void* stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len > 65536 || batch > 65535 || heads > 65535)
    return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != 32 && head_dim != 64) return RT_ERR_UNSUPPORTED;
  // masked logits enter as -inf times the scale, and the fused backward divides by it
  if (!(scale > 0.f) || !(scale < INFINITY)) return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || heads == 0 || seq_len == 0) return RT_OK;
  if (!plan_matches(plan, batch, seq_len)) return RT_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !o || !lse) return RT_ERR_INVALID_ARGUMENT;
  if (!aligned16(q) || !aligned16(k) || !aligned16(v) || !aligned16(o) || !aligned16(lse))
    return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(q);
  if (guard.status() != RT_OK) return guard.status();
  return launch_attention_fwd(q, k, v, batch, heads, seq_len, head_dim, scale, *plan, o, lse,
                              static_cast<cudaStream_t>(stream));
}

namespace {
// Workspace: the padded row statistics, then the fp32 dQ accumulator of the
// fused backward, sized for the widest head (64).
size_t bwd_stats_bytes(int32_t batch, int32_t heads, int32_t seq_len) {
  const size_t padded = (size_t)((seq_len + RT_TILE - 1) / RT_TILE) * RT_TILE;
  return align_up(2 * sizeof(float) * (size_t)batch * heads * padded);
}
}  // namespace

size_t rt_attention_bwd_workspace_bytes(int32_t batch, int32_t heads, int32_t seq_len) {
  if (batch < 0 || heads < 0 || seq_len < 0) return 0;
  const size_t padded = (size_t)((seq_len + RT_TILE - 1) / RT_TILE) * RT_TILE;
  const size_t rows = (size_t)batch * heads * padded;
  return bwd_stats_bytes(batch, heads, seq_len) + align_up(64 * sizeof(float) * rows) + align_up(32 * rows);
}

int rt_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                     const uint16_t* d_o, const float* lse, int32_t batch, int32_t heads,
                     int32_t seq_len, int32_t head_dim, float scale, const rt_tile_plan* plan,
                     uint16_t* dq, uint16_t* dk, uint16_t* dv, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len > 65536 || batch > 65535 || heads > 65535)
    return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != 32 && head_dim != 64) return RT_ERR_UNSUPPORTED;
  // masked logits enter as -inf times the scale, and the fused backward divides by it
  if (!(scale > 0.f) || !(scale < INFINITY)) return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || heads == 0 || seq_len == 0) return RT_OK;
  if (!plan_matches(plan, batch, seq_len)) return RT_ERR_INVALID_ARGUMENT;
  if (!q || !k || !v || !o || !d_o || !lse || !dq || !dk || !dv || !workspace)
    return RT_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {q, k, v, o, d_o, lse, dq, dk, dv, workspace};
  for (const void* p : ptrs)
    if (!aligned16(p)) return RT_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < rt_attention_bwd_workspace_bytes(batch, heads, seq_len)) return RT_ERR_WORKSPACE;
  DeviceGuard guard(q);
  if (guard.status() != RT_OK) return guard.status();
  float* stats = static_cast<float*>(workspace);
  const size_t padded = (size_t)((seq_len + RT_TILE - 1) / RT_TILE) * RT_TILE;
  uint8_t* acc_base = static_cast<uint8_t*>(workspace) + bwd_stats_bytes(batch, heads, seq_len);
  float* dq_acc = reinterpret_cast<float*>(acc_base);
  uint16_t* aux = reinterpret_cast<uint16_t*>(acc_base + align_up(64 * sizeof(float) * (size_t)batch * heads * padded));
  return launch_attention_bwd(q, k, v, o, d_o, lse, batch, heads, seq_len, head_dim, scale, *plan, dq,
                              dk, dv, stats, dq_acc, aux, static_cast<cudaStream_t>(stream));
}

int rt_attention_bwd_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                         const uint16_t* d_o, const float* lse, int32_t batch, int32_t heads,
                         int32_t seq_len, int32_t head_dim, float scale, const rt_tile_plan* plan,
                         const uint16_t* perm, const uint16_t* qkv, const float* tau, const float* rnorm,
                         uint16_t* dqkv, float* dtau_rows, void* workspace, size_t workspace_bytes,
                         void* stream) {
  if (batch < 0 || heads < 0 || seq_len < 0 || seq_len > 65536 || batch > 65535 || heads > 65535)
    return RT_ERR_INVALID_ARGUMENT;
  if (head_dim != 32 && head_dim != 64) return RT_ERR_UNSUPPORTED;
  if (!(scale > 0.f) || !(scale < INFINITY)) return RT_ERR_INVALID_ARGUMENT;
  if (batch == 0 || heads == 0 || seq_len == 0) return RT_OK;
  if (!plan_matches(plan, batch, seq_len)) return RT_ERR_INVALID_ARGUMENT;
  const void* ptrs[] = {q, k, v, o, d_o, lse, perm, qkv, tau, rnorm, dqkv, dtau_rows, workspace};
  for (const void* p : ptrs)
    if (!p || !aligned16(p)) return RT_ERR_INVALID_ARGUMENT;
  if (workspace_bytes < rt_attention_bwd_workspace_bytes(batch, heads, seq_len)) return RT_ERR_WORKSPACE;
  DeviceGuard guard(q);
  if (guard.status() != RT_OK) return guard.status();
  const size_t padded = (size_t)((seq_len + RT_TILE - 1) / RT_TILE) * RT_TILE;
  uint8_t* acc_base = static_cast<uint8_t*>(workspace) + bwd_stats_bytes(batch, heads, seq_len);
  float* dq_acc = reinterpret_cast<float*>(acc_base);
  uint16_t* aux = reinterpret_cast<uint16_t*>(acc_base + align_up(64 * sizeof(float) * (size_t)batch * heads * padded));
  return launch_attention_bwd_qkv(q, k, v, o, d_o, lse, batch, heads, seq_len, head_dim, scale, *plan, perm, qkv,
                                  tau, rnorm, dqkv, dtau_rows, dq_acc, aux, static_cast<cudaStream_t>(stream));
}

int rt_device_status(int32_t reset) {
  int status = 0;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_failure(e, "cudaDeviceSynchronize");
  e = cudaMemcpyFromSymbol(&status, g_device_status, sizeof(int));
  if (e != cudaSuccess) return cuda_failure(e, "cudaMemcpyFromSymbol(status)");
  if (reset) {
    const int zero = 0;
    e = cudaMemcpyToSymbol(g_device_status, &zero, sizeof(int));
    if (e != cudaSuccess) return cuda_failure(e, "cudaMemcpyToSymbol(status)");
  }
  return status;
}

const char* rt_status_string(int32_t status) {
  switch (status) {
    case RT_OK: return "ok";
    case RT_ERR_INVALID_ARGUMENT: return "invalid argument";
    case RT_ERR_UNSUPPORTED: return "unsupported configuration";
    case RT_ERR_CUDA: return "CUDA call or launch failed";
    case RT_ERR_TIMEOUT: return "device-side bounded wait ran out";
    case RT_ERR_WORKSPACE: return "workspace too small";
    case RT_ERR_DEVICE: return "no usable sm_100 device";
    default: return "unknown status";
  }
}

int32_t rt_version(void) { return 100; }

const char* rt_last_error(void) { return g_last_error; }

}  // extern "C"
