// Single translation unit of libtributary_b200.so: every kernel file and the
// C ABI are compiled together so that the library-wide device status word in
// rt_device.cuh is defined once and visible to every kernel.
#include "rt_device.cuh"
#include "tile_plan.cu"
#include "attn_fwd.cu"
#include "attn_bwd.cu"
#include "api.cu"
#include "token_prep.cu"
#include "attn_bwd_noalloc.cu"
#include "row_order.cu"
#include "selftest.cu"
#include "col_sort.cu"
#include "layer_ops.cu"
