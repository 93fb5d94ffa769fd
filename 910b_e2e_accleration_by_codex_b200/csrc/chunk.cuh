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
  int64_t gb_st;
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

int run_chunk_simt(const ChunkParams& p, int D, int dtype, cudaStream_t s);
int run_chunk_tc(const ChunkParams& p, int64_t T_total, cudaStream_t s);

}  // namespace gdn
