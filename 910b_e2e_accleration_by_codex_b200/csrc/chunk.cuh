// Parameters shared by the chunked-prefill kernels and their C entry point.
#pragma once

#include "common.cuh"

namespace gdn {

struct ChunkParams {
  const void* q;
  int64_t q_st;
  const void* k;
  int64_t k_st;
  const void* v;
  int64_t v_st;
  const float* g;
  const float* beta;
  int64_t gb_st;              // token stride of g / beta, or of a_raw / b_raw
  // Raw-gate form (a_raw != nullptr): g and beta are formed in-kernel from the in_proj_a / in_proj_b
  // outputs [T, Hv] (activation dtype) and the per-head A_log / dt_bias (f32), as the prefill of
  // src/cb_tp.py:170-171 does: beta = sigmoid(b) in the activation dtype,
  // g = -exp(A_log) * softplus(float(a) + dt_bias) in fp32.
  const void* a_raw;
  const void* b_raw;
  const float* A_log;
  const float* dt_bias;
  int raw_bf16;               // a_raw / b_raw are bf16 (else f32)
  const int32_t* cu;          // cu_seqlens [B+1] (device)
  const float* init_pool;
  const int32_t* init_slot;
  const int32_t* use_init;
  float* final_pool;
  const int32_t* final_slot;
  int64_t n_slots;
  void* out;
  int64_t o_st;
  int B, Hk, Hv;
  int l2norm;
  int32_t* err;
};

// g and beta of token `tok`, value head h (0 for both past the sequence end is the caller's job).
__device__ __forceinline__ void chunk_gate(const ChunkParams& p, int64_t tok, int h, float& g, float& beta) {
  const int64_t i = tok * p.gb_st + h;
  if (p.a_raw != nullptr) {
    float a, b;
    if (p.raw_bf16) {
      a = __bfloat162float(static_cast<const __nv_bfloat16*>(p.a_raw)[i]);
      b = __bfloat162float(static_cast<const __nv_bfloat16*>(p.b_raw)[i]);
    } else {
      a = static_cast<const float*>(p.a_raw)[i];
      b = static_cast<const float*>(p.b_raw)[i];
    }
    g = -expf(p.A_log[h]) * softplus_f(a + p.dt_bias[h]);
    const float s = sigmoid_f(b);
    beta = p.raw_bf16 ? __bfloat162float(__float2bfloat16_rn(s)) : s;
  } else {
    g = p.g[i];
    beta = p.beta[i];
  }
}

int run_chunk_simt(const ChunkParams& p, int D, int dtype, cudaStream_t s);
int run_chunk_tc(const ChunkParams& p, int64_t T_total, cudaStream_t s);

}  // namespace gdn
