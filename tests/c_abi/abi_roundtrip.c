/*
 * A caller of the C ABI with no Python and no PyTorch: the CUDA runtime for
 * device memory and copies, include/rt_attention.h for everything else, as a
 * C or C++ host (or a cgo / JNI / FFI shim) would bind it.
 *
 *   abi_roundtrip <dir> B S R H Dh kind
 *
 * Reads from <dir>: perm.u16, rows.u16, cols.i32, pad.u8, fk.u8 (the sampler's
 * batch tensors) and q.bf16, k.bf16, v.bf16, do.bf16 ([B][H][S][Dh]); builds
 * the tile plan, runs the forward and the backward, and writes o.bf16,
 * lse.f32, dq.bf16, dk.bf16, dv.bf16 and nnz.i32 back to <dir>. Exits with
 * the first non-zero rt_status (or 100 + a CUDA / file error).
 */
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <math.h>

#include <cuda_runtime_api.h>

#include "rt_attention.h"

static char g_dir[4096];

static void* read_file(const char* name, size_t bytes) {
  char path[4200];
  snprintf(path, sizeof path, "%s/%s", g_dir, name);
  FILE* f = fopen(path, "rb");
  if (!f) return NULL;
  void* buf = malloc(bytes ? bytes : 1);
  const size_t got = fread(buf, 1, bytes, f);
  fclose(f);
  if (got != bytes) {
    free(buf);
    return NULL;
  }
  return buf;
}

static int write_file(const char* name, const void* buf, size_t bytes) {
  char path[4200];
  snprintf(path, sizeof path, "%s/%s", g_dir, name);
  FILE* f = fopen(path, "wb");
  if (!f) return 0;
  const size_t put = fwrite(buf, 1, bytes, f);
  fclose(f);
  return put == bytes;
}

/* host file -> new device buffer */
static void* upload(const char* name, size_t bytes) {
  void* host = read_file(name, bytes);
  void* dev = NULL;
  if (!host) return NULL;
  if (cudaMalloc(&dev, bytes ? bytes : 16) != cudaSuccess ||
      cudaMemcpy(dev, host, bytes, cudaMemcpyHostToDevice) != cudaSuccess)
    dev = NULL;
  free(host);
  return dev;
}

static int download(const char* name, const void* dev, size_t bytes) {
  void* host = malloc(bytes);
  int ok = cudaMemcpy(host, dev, bytes, cudaMemcpyDeviceToHost) == cudaSuccess && write_file(name, host, bytes);
  free(host);
  return ok;
}

#define CHECK_RT(call)                                                       \
  do {                                                                       \
    int st_ = (call);                                                        \
    if (st_ != RT_OK) {                                                      \
      fprintf(stderr, "%s: %s %s\n", #call, rt_status_string(st_), rt_last_error()); \
      return st_;                                                            \
    }                                                                        \
  } while (0)
#define CHECK(cond, code)                              \
  do {                                                 \
    if (!(cond)) {                                     \
      fprintf(stderr, "failed: %s\n", #cond);          \
      return (code);                                   \
    }                                                  \
  } while (0)

int main(int argc, char** argv) {
  if (argc != 8) {
    fprintf(stderr, "usage: %s dir B S R H Dh kind\n", argv[0]);
    return 100;
  }
  snprintf(g_dir, sizeof g_dir, "%s", argv[1]);
  const int B = atoi(argv[2]), S = atoi(argv[3]), R = atoi(argv[4]), H = atoi(argv[5]), Dh = atoi(argv[6]);
  const int kind = atoi(argv[7]);
  const size_t bs = (size_t)B * S, elems = (size_t)B * H * S * Dh;

  void* perm = upload("perm.u16", 2 * bs);
  void* rows = upload("rows.u16", 2 * bs);
  void* cols = upload("cols.i32", 4 * bs);
  void* pad = upload("pad.u8", bs);
  void* fk = upload("fk.u8", (size_t)B * R * R);
  void* q = upload("q.bf16", 2 * elems);
  void* k = upload("k.bf16", 2 * elems);
  void* v = upload("v.bf16", 2 * elems);
  void* d_o = upload("do.bf16", 2 * elems);
  CHECK(perm && rows && cols && pad && fk && q && k && v && d_o, 101);

  /* the plan: sized and carved by the library, allocated by the caller */
  const size_t plan_bytes = rt_tile_plan_bytes(B, S, R);
  void* plan_buf = NULL;
  CHECK(cudaMalloc(&plan_buf, plan_bytes) == cudaSuccess, 102);
  rt_tile_plan plan;
  CHECK_RT(rt_tile_plan_bind(plan_buf, plan_bytes, B, S, R, &plan));
  cudaStream_t stream;
  CHECK(cudaStreamCreate(&stream) == cudaSuccess, 103);
  CHECK_RT(rt_build_tile_plan((const uint16_t*)perm, (const uint16_t*)rows, (const int32_t*)cols,
                              (const uint8_t*)pad, (const uint8_t*)fk, B, S, R, kind, &plan, stream));

  void *o = NULL, *lse = NULL, *dq = NULL, *dk = NULL, *dv = NULL, *ws = NULL;
  const size_t ws_bytes = rt_attention_bwd_workspace_bytes(B, H, S);
  CHECK(cudaMalloc(&o, 2 * elems) == cudaSuccess && cudaMalloc(&lse, 4 * (size_t)B * H * S) == cudaSuccess &&
            cudaMalloc(&dq, 2 * elems) == cudaSuccess && cudaMalloc(&dk, 2 * elems) == cudaSuccess &&
            cudaMalloc(&dv, 2 * elems) == cudaSuccess && cudaMalloc(&ws, ws_bytes) == cudaSuccess,
        104);
  const float scale = 1.0f / sqrtf((float)Dh);
  CHECK_RT(rt_attention_fwd((const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, B, H, S, Dh, scale, &plan,
                            (uint16_t*)o, (float*)lse, stream));
  CHECK_RT(rt_attention_bwd((const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, (const uint16_t*)o,
                            (const uint16_t*)d_o, (const float*)lse, B, H, S, Dh, scale, &plan, (uint16_t*)dq,
                            (uint16_t*)dk, (uint16_t*)dv, ws, ws_bytes, stream));
  CHECK(cudaStreamSynchronize(stream) == cudaSuccess, 105);
  CHECK_RT(rt_device_status(1));

  int32_t nnz = 0;
  CHECK(cudaMemcpy(&nnz, plan.nnz, sizeof nnz, cudaMemcpyDeviceToHost) == cudaSuccess, 106);
  CHECK(write_file("nnz.i32", &nnz, sizeof nnz), 107);
  CHECK(download("o.bf16", o, 2 * elems) && download("lse.f32", lse, 4 * (size_t)B * H * S) &&
            download("dq.bf16", dq, 2 * elems) && download("dk.bf16", dk, 2 * elems) &&
            download("dv.bf16", dv, 2 * elems),
        108);
  printf("ok nnz=%d\n", nnz);
  return 0;
}
