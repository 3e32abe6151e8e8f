// XLA FFI handlers for the reference's JAX model: the typed custom calls that
// replace build_attention_masks (confluence/confluence/model.py:201-264, one
// tile plan per mask kind) and the masked softmax attention of
// QKNormedMultiHeadAttention (confluence/confluence/layers.py:82-97) and its
// autodiff backward, on the stream XLA hands each call.
//
// Built by build_ffi.py against the XLA FFI headers that jax ships
// (jax.ffi.include_dir()) and linked with libtributary_b200.so; where jax is
// not installed the file is not compiled. Buffers are XLA's: the plan is an
// ordinary u8 output sized by rt_tile_plan_bytes, the backward's workspace a
// u8 output sized by rt_attention_bwd_workspace_bytes (both known at trace
// time from the shapes), so nothing here allocates. Status codes become FFI
// errors carrying rt_status_string (and rt_last_error for CUDA failures).
#include <cuda_runtime_api.h>

#include <cstdint>
#include <string>

#include "rt_attention.h"
#include "xla/ffi/api/ffi.h"

namespace ffi = xla::ffi;

namespace {

ffi::Error to_error(int st, const char* what) {
  if (st == RT_OK) return ffi::Error::Success();
  std::string msg = std::string(what) + ": " + rt_status_string(st);
  if (st == RT_ERR_CUDA) msg += std::string(" (") + rt_last_error() + ")";
  const ffi::ErrorCode code = st == RT_ERR_INVALID_ARGUMENT || st == RT_ERR_WORKSPACE ? ffi::ErrorCode::kInvalidArgument
                              : st == RT_ERR_UNSUPPORTED                            ? ffi::ErrorCode::kUnimplemented
                                                                                    : ffi::ErrorCode::kInternal;
  return ffi::Error(code, msg);
}

// Binds the caller's plan buffer for [batch, seq_len] and max_rows.
int bind_plan(void* buf, size_t bytes, int64_t batch, int64_t seq_len, int32_t max_rows, rt_tile_plan* plan) {
  return rt_tile_plan_bind(buf, bytes, (int32_t)batch, (int32_t)seq_len, max_rows, plan);
}

// perm, seq_row_ids: u16 [B,S]; column_ids: s32 [B,S]; is_padding: u8 [B,S];
// fk_adj: u8 [B,R,R] -> plan: u8 [rt_tile_plan_bytes(B,S,R)]
ffi::Error TilePlan(cudaStream_t stream, ffi::Buffer<ffi::U16> perm, ffi::Buffer<ffi::U16> seq_row_ids,
                    ffi::Buffer<ffi::S32> column_ids, ffi::Buffer<ffi::U8> is_padding, ffi::Buffer<ffi::U8> fk_adj,
                    ffi::ResultBuffer<ffi::U8> plan_buf, int32_t kind) {
  const auto d = perm.dimensions();
  const auto r = fk_adj.dimensions();
  if (d.size() != 2 || r.size() != 3) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "rt_tile_plan: ranks");
  rt_tile_plan plan;
  int st = bind_plan(plan_buf->untyped_data(), plan_buf->size_bytes(), d[0], d[1], (int32_t)r[1], &plan);
  if (st == RT_OK)
    st = rt_build_tile_plan(perm.typed_data(), seq_row_ids.typed_data(), column_ids.typed_data(),
                            is_padding.typed_data(), fk_adj.typed_data(), (int32_t)d[0], (int32_t)d[1],
                            (int32_t)r[1], kind, &plan, stream);
  return to_error(st, "rt_build_tile_plan");
}

// q, k, v: bf16 [B,H,S,Dh], plan -> o: bf16 [B,H,S,Dh], lse: f32 [B,H,S]
ffi::Error AttnFwd(cudaStream_t stream, ffi::Buffer<ffi::BF16> q, ffi::Buffer<ffi::BF16> k, ffi::Buffer<ffi::BF16> v,
                   ffi::Buffer<ffi::U8> plan_buf, ffi::ResultBuffer<ffi::BF16> o, ffi::ResultBuffer<ffi::F32> lse,
                   int32_t max_rows, float scale) {
  const auto d = q.dimensions();
  if (d.size() != 4) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "rt_attention_fwd: q must be [B,H,S,Dh]");
  rt_tile_plan plan;
  int st = bind_plan(const_cast<void*>(plan_buf.untyped_data()), plan_buf.size_bytes(), d[0], d[2], max_rows, &plan);
  if (st == RT_OK)
    st = rt_attention_fwd(reinterpret_cast<const uint16_t*>(q.untyped_data()),
                          reinterpret_cast<const uint16_t*>(k.untyped_data()),
                          reinterpret_cast<const uint16_t*>(v.untyped_data()), (int32_t)d[0], (int32_t)d[1],
                          (int32_t)d[2], (int32_t)d[3], scale, &plan, reinterpret_cast<uint16_t*>(o->untyped_data()),
                          lse->typed_data(), stream);
  return to_error(st, "rt_attention_fwd");
}

// q, k, v, o, d_o: bf16 [B,H,S,Dh], lse: f32 [B,H,S], plan
//   -> dq, dk, dv: bf16 [B,H,S,Dh], workspace: u8 [rt_attention_bwd_workspace_bytes(B,H,S)]
ffi::Error AttnBwd(cudaStream_t stream, ffi::Buffer<ffi::BF16> q, ffi::Buffer<ffi::BF16> k, ffi::Buffer<ffi::BF16> v,
                   ffi::Buffer<ffi::BF16> o, ffi::Buffer<ffi::BF16> d_o, ffi::Buffer<ffi::F32> lse,
                   ffi::Buffer<ffi::U8> plan_buf, ffi::ResultBuffer<ffi::BF16> dq, ffi::ResultBuffer<ffi::BF16> dk,
                   ffi::ResultBuffer<ffi::BF16> dv, ffi::ResultBuffer<ffi::U8> workspace, int32_t max_rows,
                   float scale) {
  const auto d = q.dimensions();
  if (d.size() != 4) return ffi::Error(ffi::ErrorCode::kInvalidArgument, "rt_attention_bwd: q must be [B,H,S,Dh]");
  rt_tile_plan plan;
  int st = bind_plan(const_cast<void*>(plan_buf.untyped_data()), plan_buf.size_bytes(), d[0], d[2], max_rows, &plan);
  auto bf = [](const auto& b) { return reinterpret_cast<const uint16_t*>(b.untyped_data()); };
  if (st == RT_OK)
    st = rt_attention_bwd(bf(q), bf(k), bf(v), bf(o), bf(d_o), lse.typed_data(), (int32_t)d[0], (int32_t)d[1],
                          (int32_t)d[2], (int32_t)d[3], scale, &plan, reinterpret_cast<uint16_t*>(dq->untyped_data()),
                          reinterpret_cast<uint16_t*>(dk->untyped_data()),
                          reinterpret_cast<uint16_t*>(dv->untyped_data()), workspace->untyped_data(),
                          workspace->size_bytes(), stream);
  return to_error(st, "rt_attention_bwd");
}

}  // namespace

XLA_FFI_DEFINE_HANDLER_SYMBOL(rt_tile_plan_ffi, TilePlan,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::U16>>()
                                  .Arg<ffi::Buffer<ffi::U16>>()
                                  .Arg<ffi::Buffer<ffi::S32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int32_t>("kind"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(rt_attention_fwd_ffi, AttnFwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::F32>>()
                                  .Attr<int32_t>("max_rows")
                                  .Attr<float>("scale"));

XLA_FFI_DEFINE_HANDLER_SYMBOL(rt_attention_bwd_ffi, AttnBwd,
                              ffi::Ffi::Bind()
                                  .Ctx<ffi::PlatformStream<cudaStream_t>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::BF16>>()
                                  .Arg<ffi::Buffer<ffi::F32>>()
                                  .Arg<ffi::Buffer<ffi::U8>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::BF16>>()
                                  .Ret<ffi::Buffer<ffi::U8>>()
                                  .Attr<int32_t>("max_rows")
                                  .Attr<float>("scale"));
