// rt_column_order_device: the column cell order of headwater/src/sampler.rs:
// 655-668 (cells sorted by padding flag, then column id, then position)
// computed on the GPU from the batch tensors already in device memory, so a
// batch goes from the sampler's raw tensors to tile plans without a host
// round trip. Bit-identical to rt_column_order (the host version).
//
// One CTA per sample sorts the sample's cells in shared memory: each cell
// becomes a 64-bit key (padding byte << 48 | column id with its sign bit
// flipped << 16 | position), unique because the position is, so any correct
// sort yields the stable order; a bitonic network over the next power of two
// of seq_len (padded with all-ones keys) sorts them, and the low 16 bits of
// the first seq_len keys are the order. Bound: shared-memory bandwidth, about
// log2(n)^2 / 2 passes over n keys; the device path takes seq_len <= 16384
// (128 KB of keys), the host path any length.

namespace rt {
namespace colsort {

constexpr int kMaxLen = 16384;
constexpr int kThreads = 1024;

__global__ void __launch_bounds__(kThreads) column_order_kernel(const int32_t* __restrict__ column_ids,
                                                                const uint8_t* __restrict__ is_padding, int S,
                                                                int n_pow2, uint16_t* __restrict__ perm) {
  pdl_wait();  // the previous kernel on the stream has completed (launch_pdl)
  pdl_trigger();
  extern __shared__ unsigned long long keys[];
  const int b = blockIdx.x;
  const int32_t* col = column_ids + (size_t)b * S;
  const uint8_t* pad = is_padding + (size_t)b * S;
  for (int i = threadIdx.x; i < n_pow2; i += kThreads) {
    unsigned long long key = ~0ull;
    if (i < S)
      key = ((unsigned long long)pad[i] << 48) | ((unsigned long long)((uint32_t)col[i] ^ 0x80000000u) << 16) |
            (unsigned long long)i;
    keys[i] = key;
  }
  __syncthreads();
  for (int k = 2; k <= n_pow2; k <<= 1) {
    for (int j = k >> 1; j > 0; j >>= 1) {
      for (int i = threadIdx.x; i < n_pow2; i += kThreads) {
        const int l = i ^ j;
        if (l > i) {
          const unsigned long long a = keys[i], c = keys[l];
          const bool up = (i & k) == 0;
          if ((a > c) == up) {
            keys[i] = c;
            keys[l] = a;
          }
        }
      }
      __syncthreads();
    }
  }
  for (int i = threadIdx.x; i < S; i += kThreads) perm[(size_t)b * S + i] = (uint16_t)(keys[i] & 0xFFFFu);
}

}  // namespace colsort
}  // namespace rt

extern "C" int rt_column_order_device(const int32_t* column_ids, const uint8_t* is_padding, int32_t batch,
                                      int32_t seq_len, uint16_t* perm, void* stream) {
  using namespace rt;
  if (batch < 0 || seq_len < 0 || batch > 65535) return RT_ERR_INVALID_ARGUMENT;
  if (seq_len > colsort::kMaxLen) return RT_ERR_UNSUPPORTED;
  if (batch == 0 || seq_len == 0) return RT_OK;
  if (!column_ids || !is_padding || !perm) return RT_ERR_INVALID_ARGUMENT;
  DeviceGuard guard(column_ids);
  if (guard.status() != RT_OK) return guard.status();
  int n_pow2 = 1;
  while (n_pow2 < seq_len) n_pow2 <<= 1;
  const size_t smem = sizeof(unsigned long long) * (size_t)n_pow2;
  static bool configured[64] = {false};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev >= 0 && dev < 64 && !configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(colsort::column_order_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               (int)(sizeof(unsigned long long) * colsort::kMaxLen));
    if (e != cudaSuccess) return cuda_failure(e, "cudaFuncSetAttribute(column_order_kernel)");
    configured[dev] = true;
  }
  {
    if (int st_pdl = launch_pdl("column_order_kernel launch", colsort::column_order_kernel, dim3(batch),
        dim3(colsort::kThreads), smem, static_cast<cudaStream_t>(stream), column_ids, is_padding, seq_len,
        n_pow2, perm)) return st_pdl;
  }
  return check_launch("column_order_kernel launch");
}
