// C ABI of the Gated DeltaNet kernels.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

struct GdnConvParams {
  const __nv_bfloat16* x;  // [T, >= C] pre-conv activations (row stride x_stride)
  int64_t x_stride;
  const float* w;          // [C, 4] depthwise taps
  __nv_bfloat16* y;        // [T, C] SiLU(conv) output
  float* state;            // [slots, C, 3] last inputs (oldest first)
  float* rec_x;            // [slots, W, C] window inputs (mode 1)
  const int32_t* pending;  // [slots] accepted records to replay (mode 1)
  const int64_t* slots;    // [B] state slot per request
  const int64_t* q_start;  // [B+1] token rows per request
  int C, KW, W;
  int mode;  // 0 prefill from zero state (commits), 1 verify window (records, deferred commit)
};

struct GdnParams {
  const __nv_bfloat16* qkv;  // [T, 2*H*K + HV*V] post-conv q | k | v
  int64_t qkv_stride;
  const __nv_bfloat16* z;  // [T, HV*V] output gate
  int64_t z_stride;
  const __nv_bfloat16* ba;  // [T, 2*HV] b | a
  int64_t ba_stride;
  const float* a_log;  // [HV]
  const float* dt_bias;  // [HV]
  const __nv_bfloat16* norm_w;  // [V]
  float* state;  // [slots, HV, V, K]
  float* rec_k;  // [slots, W, HV, K]
  float* rec_v;  // [slots, W, HV, V]
  float* rec_g;  // [slots, W, HV]
  float* rec_b;  // [slots, W, HV]
  const int32_t* pending;
  const int64_t* slots;
  const int64_t* q_start;
  __nv_bfloat16* out;  // [T, HV*V]
  int64_t out_stride;
  int H, HV, K, V, W;
  int mode;
  float eps;
  int async_ok;  // set by sh_gdn_recurrent: token rows may be staged with cp.async
  int32_t* err;  // chunked prefill: set to 1 when a tensor-core wait gave up (may be null)
};

#ifdef __cplusplus
extern "C" {
#endif
int sh_gdn_conv(const GdnConvParams* p, int batch, cudaStream_t stream);
int sh_gdn_recurrent(const GdnParams* p, int batch, cudaStream_t stream);
// Prefill from zero state in chunks of 64 tokens on the tensor cores (K == V == 128); commits the final
// state like sh_gdn_recurrent mode 0.  -3: a row of qkv / z / out is not 16-byte aligned.
int sh_gdn_chunk_prefill(const GdnParams* p, int batch, cudaStream_t stream);
#ifdef __cplusplus
}
#endif
