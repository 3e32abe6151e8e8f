/*
 * rt_attention.h -- C ABI of the B200 (sm_100a) Relational-Transformer masked
 * attention library (libtributary_b200.so).
 *
 * The reference computes this path in JAX:
 *   - the masks:    build_attention_masks          confluence/confluence/model.py:201-264
 *   - permutation:  GatedAttentionSublayer          confluence/confluence/layers.py:139-152
 *   - the core:     QKNormedMultiHeadAttention      confluence/confluence/layers.py:82-97
 *                   (logits, -1e9 fill, softmax, PV) and its jax autodiff backward
 *                   (jax.value_and_grad, confluence/confluence/train.py:209).
 * The reference has no native operator for it; these entry points are what an
 * XLA FFI custom call (or ctypes, cgo, ...) binds in place of those lines.
 *
 * Conventions
 *   - Every call is stream-ordered on `stream` (a cudaStream_t passed as
 *     void*, NULL = legacy default stream) and returns an rt_status.
 *   - The caller owns every buffer; all pointers are device pointers unless
 *     stated otherwise. Nothing here allocates device memory.
 *   - Attention tensors are bf16 (passed as uint16_t bit patterns), laid out
 *     [batch][heads][seq_len][head_dim] contiguous, 16-byte aligned.
 *   - Token order is the *permuted* order of the reference (x_perm = x[perm]):
 *     q/k/v row i belongs to original cell perm[b][i].
 *   - Tiles are 128 x 128 in that permuted order.
 *   - Device-side bounded waits never hang: a wait that runs out sets a
 *     sticky device status, read with rt_device_status().
 */
#ifndef RT_ATTENTION_H
#define RT_ATTENTION_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef enum rt_status {
  RT_OK = 0,
  RT_ERR_INVALID_ARGUMENT = 1, /* bad shape, null or misaligned pointer, bad kind */
  RT_ERR_UNSUPPORTED = 2,      /* valid but not implemented (e.g. head_dim) */
  RT_ERR_CUDA = 3,             /* a CUDA runtime / driver call or launch failed */
  RT_ERR_TIMEOUT = 4,          /* a device-side bounded wait ran out */
  RT_ERR_WORKSPACE = 5,        /* caller-provided buffer too small */
  RT_ERR_DEVICE = 6            /* no usable sm_100 device */
} rt_status;

/* Mask kinds. Reference names (model.py:233-245): outbound == feature,
 * inbound == neighbor. FULL (every non-padding pair, plus the diagonal) is
 * not in the reference; it is the fourth benchmark kind. */
typedef enum rt_mask_kind {
  RT_MASK_COLUMN = 0,   /* col_i == col_j                       */
  RT_MASK_FEATURE = 1,  /* row_i == row_j || fk_adj[row_i][row_j] */
  RT_MASK_NEIGHBOR = 2, /* fk_adj[row_j][row_i]                  */
  RT_MASK_FULL = 3      /* valid                                 */
} rt_mask_kind;
/* every kind is then ANDed with (!pad_i && !pad_j) and ORed with the
 * diagonal i == j, exactly as model.py:248-262 */

#define RT_TILE 128

/* Tile plan: the prepass output for one (batch, mask kind, permutation).
 * All arrays are device memory carved from one caller buffer by
 * rt_tile_plan_bind(). T = ceil(seq_len / 128), W = ceil(T / 32). */
typedef struct rt_tile_plan {
  int32_t batch;
  int32_t seq_len;
  int32_t max_rows;
  int32_t tiles;           /* T */
  int32_t words;           /* W */
  uint32_t* live_bits;     /* [batch][T][W]   bit kt of row (b,qt): tile has a true element */
  uint32_t* full_bits;     /* [batch][T][W]   tile is entirely in range and entirely true  */
  int32_t* q2k_ptr;        /* [batch*T + 1]   CSR row pointers over (b, qt)                */
  int32_t* q2k_idx;        /* [batch*T*T]     live kt ascending; bit 31 = fully live       */
  int32_t* k2q_ptr;        /* [batch*T + 1]   CSR row pointers over (b, kt)                */
  int32_t* k2q_idx;        /* [batch*T*T]     live qt ascending; bit 31 = fully live       */
  uint32_t* tile_masks;    /* [batch][T][T][128][4]  element bits, query-major (partial tiles) */
  uint32_t* tile_masks_t;  /* [batch][T][T][128][4]  element bits, key-major   (partial tiles) */
  uint32_t* fk_bits;       /* [batch][max_rows][ceil(max_rows/32)]  packed adjacency (scratch) */
  int32_t* nnz;            /* [1 + batch] number of live tiles over the batch, then scratch    */
} rt_tile_plan;

/* Bytes of device memory a tile plan needs. */
size_t rt_tile_plan_bytes(int32_t batch, int32_t seq_len, int32_t max_rows);

/* Host-only: carve `buffer` (device memory, 256-byte aligned, `bytes` long)
 * into a plan. No device work. */
int rt_tile_plan_bind(void* buffer, size_t bytes, int32_t batch, int32_t seq_len,
                      int32_t max_rows, rt_tile_plan* plan);

/* Prepass: replaces build_attention_masks (model.py:201-264) plus the mask
 * permutation of layers.py:144-152 for one kind. Inputs are the headwater
 * batch tensors (headwater/src/python.rs:17-91):
 *   perm        [batch][seq_len] uint16  (col_perm / out_perm / in_perm)
 *   seq_row_ids [batch][seq_len] uint16
 *   column_ids  [batch][seq_len] int32
 *   is_padding  [batch][seq_len] uint8
 *   fk_adj      [batch][max_rows][max_rows] uint8, fk_adj[child][parent]
 * Row ids >= max_rows are clamped to max_rows-1 (jax's gather semantics).
 * Fills every array of `plan`. */
int rt_build_tile_plan(const uint16_t* perm, const uint16_t* seq_row_ids,
                       const int32_t* column_ids, const uint8_t* is_padding,
                       const uint8_t* fk_adj, int32_t batch, int32_t seq_len,
                       int32_t max_rows, int32_t kind, const rt_tile_plan* plan,
                       void* stream);

/* Host-side cell orderings (CPU memory, synchronous; samples run on host
 * threads). The permutations the sampler attaches to every batch and under
 * which the kernels run the masks: column -> rt_column_order, feature ->
 * rt_rcm_order(outbound = 1), neighbor -> rt_rcm_order(outbound = 0).
 * rt_column_order replaces headwater/src/sampler.rs:655-668: cells sorted by
 * (padding last, column id, position).
 *   column_ids [batch][seq_len] int32, is_padding [batch][seq_len] uint8
 *   perm       [batch][seq_len] uint16 (output), seq_len <= 65536 */
int rt_column_order(const int32_t* column_ids, const uint8_t* is_padding, int32_t batch,
                    int32_t seq_len, uint16_t* perm);

/* rt_column_order on the GPU (device memory, stream-ordered): the same order,
 * bit for bit, for seq_len <= 16384 (RT_ERR_UNSUPPORTED beyond), so that a
 * batch in device memory reaches rt_build_tile_plan without a host round
 * trip. Replaces headwater/src/sampler.rs:655-668 on the device. */
int rt_column_order_device(const int32_t* column_ids, const uint8_t* is_padding, int32_t batch,
                           int32_t seq_len, uint16_t* perm, void* stream);

/* rt_rcm_order replaces headwater/src/sampler.rs:672-784: a reverse
 * Cuthill-McKee order of each sample's rows over its FK graph (fk_adj[i][j]
 * for outbound, fk_adj[j][i] for inbound), then cells sorted by (padding last,
 * row rank, position). fk_adj [batch][max_rows][max_rows] uint8 (child,
 * parent), seq_row_ids [batch][seq_len] uint16. Returns RT_ERR_WORKSPACE if
 * host memory for the sort ran out. */
int rt_rcm_order(const uint8_t* fk_adj, const uint16_t* seq_row_ids, const uint8_t* is_padding,
                 int32_t batch, int32_t seq_len, int32_t max_rows, int32_t outbound, uint16_t* perm);

/* Token preparation of one attention sublayer (device memory, stream-ordered).
 * rt_qk_prepare replaces the gather of layers.py:139-142 and the QK
 * normalisation of layers.py:63-80, applied after the QKV projection (a
 * per-token linear map commutes with the gather):
 *   qkv   [batch][seq_len][3][heads][head_dim] bf16, token order
 *   perm  [batch][seq_len] uint16, the sublayer's cell order
 *   tau   [heads] fp32
 *   q, k, v [batch][heads][seq_len][head_dim] bf16 in perm order:
 *     q = tau_h q_raw / max(|q_raw|, 1e-6), k = k_raw / max(|k_raw|, 1e-6), v = v_raw
 *   rnorm [2][batch][heads][seq_len] fp32: 1 / max(|q_raw|, 1e-6), same for k
 * head_dim in {32, 64}. */
int rt_qk_prepare(const uint16_t* qkv, const uint16_t* perm, const float* tau, int32_t batch,
                  int32_t heads, int32_t seq_len, int32_t head_dim, uint16_t* q, uint16_t* k,
                  uint16_t* v, float* rnorm, void* stream);

/* Backward of rt_qk_prepare: dqkv in token order from dq, dk, dv in perm
 * order, and dtau_rows [batch][heads][seq_len] fp32, each row's share of the
 * gradient of tau_h (d tau_h = the sum of dtau_rows over batch and rows). */
int rt_qk_prepare_bwd(const uint16_t* dq, const uint16_t* dk, const uint16_t* dv,
                      const uint16_t* qkv, const uint16_t* perm, const float* tau,
                      const float* rnorm, int32_t batch, int32_t heads, int32_t seq_len,
                      int32_t head_dim, uint16_t* dqkv, float* dtau_rows, void* stream);

/* Attention output back to token order (the scatter of layers.py:159-167 and
 * the head merge of layers.py:99): out[b][perm[b][i]][h*head_dim + d] =
 * o[b][h][i][d]. rt_heads_permute is the reverse map (its backward). */
int rt_heads_unpermute(const uint16_t* o, const uint16_t* perm, int32_t batch, int32_t heads,
                       int32_t seq_len, int32_t head_dim, uint16_t* out, void* stream);
int rt_heads_permute(const uint16_t* x, const uint16_t* perm, int32_t batch, int32_t heads,
                     int32_t seq_len, int32_t head_dim, uint16_t* out, void* stream);

/* Forward: replaces layers.py:83-94 (logits * scale, masked softmax, PV) for
 * inputs already normalised (q_hat * tau, k_hat; layers.py:65-80).
 *   q, k, v [batch][heads][seq_len][head_dim] bf16;  head_dim in {32, 64}
 *   o       same shape, bf16
 *   lse     [batch][heads][seq_len] fp32, natural-log sum of exp over live keys
 * scale multiplies q.k (the reference divides by sqrt(head_dim)); it must be
 * positive and finite (RT_ERR_INVALID_ARGUMENT otherwise), here and in the
 * backward entry points. */
int rt_attention_fwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, int32_t batch,
                     int32_t heads, int32_t seq_len, int32_t head_dim, float scale,
                     const rt_tile_plan* plan, uint16_t* o, float* lse, void* stream);

/* Workspace for the backward: [batch*heads][2][seq_len rounded up to 128]
 * fp32 -- lse (log2 units) and rowsum(dO * O) per query, zero past seq_len --
 * then the fp32 dQ accumulator [batch*heads][seq_len rounded up][64] of the
 * fused dK/dV/dQ pass, then that pass's row-statistic operand rows
 * [batch*heads][seq_len rounded up][16] bf16. */
size_t rt_attention_bwd_workspace_bytes(int32_t batch, int32_t heads, int32_t seq_len);

/* Backward: the gradients jax autodiff takes through layers.py:83-94.
 *   d_o  [batch][heads][seq_len][head_dim] bf16 (upstream gradient of o)
 *   o, lse as produced by rt_attention_fwd
 *   dq, dk, dv  bf16, same shape as q (written, not accumulated) */
int rt_attention_bwd(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                     const uint16_t* d_o, const float* lse, int32_t batch, int32_t heads,
                     int32_t seq_len, int32_t head_dim, float scale, const rt_tile_plan* plan,
                     uint16_t* dq, uint16_t* dk, uint16_t* dv, void* workspace,
                     size_t workspace_bytes, void* stream);

/* Backward of a whole attention sublayer step from the token-order
 * projection: the gather into the kind's cell order and the QK L2
 * normalisation with temperature (rt_qk_prepare, layers.py:63-80,139-142)
 * followed by the attention (layers.py:82-97). Equivalent to rt_attention_bwd
 * then rt_qk_prepare_bwd, in one pass: the normalisation's Jacobian and the
 * scatter back to token order run in the backward's own epilogues, from the
 * fp32 gradients, so dq, dk, dv never reach memory in cell order.
 *   q, k, v, rnorm  as written by rt_qk_prepare from qkv, perm, tau
 *   o, lse          as produced by rt_attention_fwd on q, k, v
 *   d_o             gradient of o, cell order [B][H][S][Dh] bf16
 *   dqkv            bf16 [B][S][3][H][Dh], gradient of qkv (written)
 *   dtau_rows       fp32 [B][H][S]: per cell, the share of d tau[h]
 *                   (sum over b and cells gives d tau)
 * The workspace is rt_attention_bwd's. Replaces dq/dk/dv + rt_qk_prepare_bwd. */
int rt_attention_bwd_qkv(const uint16_t* q, const uint16_t* k, const uint16_t* v, const uint16_t* o,
                         const uint16_t* d_o, const float* lse, int32_t batch, int32_t heads,
                         int32_t seq_len, int32_t head_dim, float scale, const rt_tile_plan* plan,
                         const uint16_t* perm, const uint16_t* qkv, const float* tau, const float* rnorm,
                         uint16_t* dqkv, float* dtau_rows, void* workspace, size_t workspace_bytes,
                         void* stream);

/* Backward for callers that cannot allocate device memory (no counterpart in
 * the reference). Same arguments and results as rt_attention_bwd minus the
 * workspace: a plugin host or FFI handler without a scratch-allocation hook,
 * or a service that may not call cudaMalloc after start-up, cannot provide
 * that workspace, so this variant keeps it in an 8 MB array compiled into the
 * library (held by every GPU that loads the library until exit). Problems
 * with batch * heads * (seq_len rounded up to 128) > 2^20 return
 * RT_ERR_WORKSPACE. All calls on a device share the array: calls that
 * overlap on the GPU race and must be ordered (one stream or events). The
 * first call on each device looks up the array's address and should come
 * before any stream capture; the address is kept for the process, so a
 * cudaDeviceReset between calls is not supported. Allocates nothing. */
int rt_attention_bwd_noalloc(const uint16_t* q, const uint16_t* k, const uint16_t* v,
                             const uint16_t* o, const uint16_t* d_o, const float* lse,
                             int32_t batch, int32_t heads, int32_t seq_len, int32_t head_dim,
                             float scale, const rt_tile_plan* plan, uint16_t* dq, uint16_t* dk,
                             uint16_t* dv, void* stream);

/* Fused kernels of the encoder layer around the attention sublayers (the
 * data-parallel training step's non-attention work; device memory,
 * stream-ordered, 16-byte aligned, widths multiples of 8).
 *
 * rt_rms_norm: ZeroCenteredRMSNorm (confluence/confluence/layers.py:16-30),
 *   y = bf16(x / sqrt(mean(x^2) + eps) * (1 + gamma)); x fp32 [rows][d]
 *   (d <= 1024), gamma fp32 [d], y bf16 [rows][d], rstd fp32 [rows] (kept
 *   for the backward).
 * rt_rms_norm_bwd: dx fp32 [rows][d] and dgamma fp32 [d] (summed in a fixed
 *   order: deterministic) from dy bf16 [rows][d]; workspace of
 *   rt_rms_norm_bwd_workspace_bytes(rows, d) bytes. */
int rt_rms_norm(const float* x, const float* gamma, int64_t rows, int32_t d, float eps, uint16_t* y,
                float* rstd, void* stream);
size_t rt_rms_norm_bwd_workspace_bytes(int64_t rows, int32_t d);
int rt_rms_norm_bwd(const uint16_t* dy, const float* x, const float* gamma, const float* rstd,
                    int64_t rows, int32_t d, float* dx, float* dgamma, void* workspace,
                    size_t workspace_bytes, void* stream);
/* rt_gate_residual: the gated residual of GatedAttentionSublayer
 *   (layers.py:170-174), y = x + scale * o * sigmoid(gate); x, y fp32 [n],
 *   o (the W_O output) and gate (the W_gate output) bf16 [n].
 * rt_gate_residual_bwd: d_o = bf16(dy scale s), d_gate = bf16(dy scale o s (1 - s)),
 *   s = sigmoid(gate); dy fp32 [n] (the gradient of x is dy itself). */
int rt_gate_residual(const float* x, const uint16_t* o, const uint16_t* gate, int64_t n, float scale,
                     float* y, void* stream);
int rt_gate_residual_bwd(const float* dy, const uint16_t* o, const uint16_t* gate, int64_t n,
                         float scale, uint16_t* d_o, uint16_t* d_gate, void* stream);
/* rt_residual_add: y = x + scale * h (the FFN's residual, layers.py:233-236);
 *   x, y fp32 [n], h bf16 [n] (the W_down output).
 * rt_residual_add_bwd: dh = bf16(dy scale) (the gradient of x is dy). */
int rt_residual_add(const float* x, const uint16_t* h, int64_t n, float scale, float* y, void* stream);
int rt_residual_add_bwd(const float* dy, int64_t n, float scale, uint16_t* dh, void* stream);
/* rt_swiglu: the SwiGLU activation (layers.py:177-200) on the fused gate/up
 *   projection u bf16 [rows][2f] (gate in columns [0, f), up in [f, 2f)):
 *   h = bf16(silu(u[:, :f]) * u[:, f:]) [rows][f].
 * rt_swiglu_bwd: du bf16 [rows][2f] = [dh up silu'(gate) | dh silu(gate)]. */
int rt_swiglu(const uint16_t* u, int64_t rows, int32_t f, uint16_t* h, void* stream);
int rt_swiglu_bwd(const uint16_t* dh, const uint16_t* u, int64_t rows, int32_t f, uint16_t* du,
                  void* stream);

/* Diagnostic for the failure path (no counterpart in the reference, which has
 * no device code). Launches one block that allocates tensor memory and waits
 * on an mbarrier nothing arrives at, through the bounded wait every kernel
 * here uses, with a limit of `limit_cycles` SM clocks (0 < limit_cycles <=
 * the kernels' own limit, about one second). The wait runs out, the block's
 * other waits leave through its abort flag, tensor memory is freed and the
 * kernel returns; rt_device_status() then reports RT_ERR_TIMEOUT and the
 * context stays usable. `report` (4 int32, device memory) receives: the
 * abort flag, the number of waits that gave up (3 expected), and the SM
 * clocks in millions that the running-out wait and the longest other wait
 * took. No fault, trap or hang is involved. */
int rt_selftest_bounded_wait(int64_t limit_cycles, int32_t* report, void* stream);

/* Sticky device status (RT_OK or RT_ERR_TIMEOUT) raised by any kernel of the
 * library on the current device. Synchronises the device. If `reset` is
 * non-zero the status is cleared after reading. */
int rt_device_status(int32_t reset);

/* Static description of a status code. */
const char* rt_status_string(int32_t status);

/* Human-readable detail of the last RT_ERR_CUDA returned on the calling
 * thread (the failing CUDA call and its error name); "" if none. */
const char* rt_last_error(void);

/* Library ABI version (major * 100 + minor). */
int32_t rt_version(void);

#ifdef __cplusplus
}
#endif

#endif /* RT_ATTENTION_H */
