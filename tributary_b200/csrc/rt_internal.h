// Internal declarations shared by the kernels and the C ABI (host side).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include "rt_attention.h"

namespace rt {

// Records the failing CUDA call for rt_last_error() (thread-local) and
// returns RT_ERR_CUDA.
int cuda_failure(cudaError_t err, const char* site);
int driver_failure(int err, const char* site);
inline int check_launch(const char* site) {
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? RT_OK : cuda_failure(e, site);
}

// Launches a kernel of the attention path with programmatic stream
// serialisation: the grid may be set up while the previous kernel on the
// stream drains. Every such kernel begins with pdl_wait() (griddepcontrol.wait,
// rt_device.cuh), which returns once the previous grid has completed and its
// memory is visible, before the kernel's first global access; launched any
// other way the wait is a no-op.
template <typename... KernelArgs, typename... Args>
int launch_pdl(const char* site, void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
               cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, static_cast<KernelArgs>(args)...);
  return e == cudaSuccess ? RT_OK : cuda_failure(e, site);
}

int launch_build_tile_plan(const uint16_t* perm, const uint16_t* seq_row_ids, const int32_t* column_ids,
                           const uint8_t* is_padding, const uint8_t* fk_adj, int B, int S, int R,
                           int kind, const rt_tile_plan& plan, cudaStream_t stream);

int launch_attention_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, int B, int H, int S,
                         int Dh, float scale, const rt_tile_plan& plan, uint16_t* o, float* lse,
                         cudaStream_t stream);

int launch_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                         const uint16_t* d_o, const float* lse, int B, int H, int S, int Dh,
                         float scale, const rt_tile_plan& plan, uint16_t* dq, uint16_t* dk,
                         uint16_t* dv, float* stats, float* dq_acc, uint16_t* aux, cudaStream_t stream);

// The fused backward with token-order outputs for the sublayer step [gather +
// QK normalisation + attention]: dqkv [B][S][3][H][Dh] and d tau row shares.
int launch_attention_bwd_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                             const uint16_t* d_o, const float* lse, int B, int H, int S, int Dh, float scale,
                             const rt_tile_plan& plan, const uint16_t* perm, const uint16_t* qkv, const float* tau,
                             const float* rnorm, uint16_t* dqkv, float* dtau_rows, float* dq_acc, uint16_t* aux,
                             cudaStream_t stream);

// TMA descriptor for a [rows_total][Dh] bf16 matrix viewed as (Dh, S, B*H),
// box (Dh, 128, 1), 128B swizzle for Dh = 64, 64B swizzle for Dh = 32.
int make_qkv_tensor_map(CUtensorMap* map, const void* base, int BH, int S, int Dh);
int make_acc_tensor_map(CUtensorMap* map, float* base, long long rows, int Dh);
int make_aux_tensor_map(CUtensorMap* map, uint16_t* base, long long rows);

}  // namespace rt
