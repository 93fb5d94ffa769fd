// C entry point of the chunked prefill: argument checks and kernel selection.
#include "chunk.cuh"

extern "C" int gdn_chunk_prefill(const void* q, int64_t q_st, const void* k, int64_t k_st, const void* v,
                                 int64_t v_st, const float* g, const float* beta, int64_t gb_st,
                                 const int32_t* cu_seqlens, int B, int64_t T_total, const float* init_pool,
                                 const int32_t* init_slot, const int32_t* use_initial, float* final_pool,
                                 const int32_t* final_slot, int64_t n_slots, void* out, int64_t o_st, int Hk,
                                 int Hv, int dk, int dv, int use_qk_l2norm, int dtype, int32_t* err_flag,
                                 void* stream) {
  using namespace gdn;
  if (B < 0 || T_total < 0 || Hk <= 0 || Hv <= 0)
    return fail(GDN_ERR_ARG, "gdn_chunk_prefill: B=%d T=%lld Hk=%d Hv=%d", B, (long long)T_total, Hk, Hv);
  if (B == 0) return GDN_OK;
  if (!q || !k || !v || !g || !beta || !cu_seqlens || !out)
    return fail(GDN_ERR_ARG, "gdn_chunk_prefill: null pointer");
  if (Hv % Hk != 0) return fail(GDN_ERR_SHAPE, "gdn_chunk_prefill: Hv=%d not a multiple of Hk=%d", Hv, Hk);
  if (dk != dv || (dk != 64 && dk != 128))
    return fail(GDN_ERR_SHAPE, "gdn_chunk_prefill: (dk,dv)=(%d,%d) not built", dk, dv);
  if (B > 65535) return fail(GDN_ERR_ARG, "gdn_chunk_prefill: B=%d > 65535", B);
  if ((init_pool || final_pool) && n_slots < 1)
    return fail(GDN_ERR_ARG, "gdn_chunk_prefill: n_slots=%lld", (long long)n_slots);
  if (dtype != GDN_BF16 && dtype != GDN_F32) return fail(GDN_ERR_DTYPE, "gdn_chunk_prefill: dtype %d", dtype);
  ChunkParams p{};
  p.q = q; p.q_st = q_st; p.k = k; p.k_st = k_st; p.v = v; p.v_st = v_st;
  p.g = g; p.beta = beta; p.gb_st = gb_st; p.cu = cu_seqlens;
  p.init_pool = init_pool; p.init_slot = init_slot; p.use_init = use_initial;
  p.final_pool = final_pool; p.final_slot = final_slot; p.n_slots = n_slots;
  p.out = out; p.o_st = o_st; p.B = B; p.Hk = Hk; p.Hv = Hv; p.l2norm = use_qk_l2norm; p.err = err_flag;
  // bf16 activations at dk = dv = 128 run on the tensor cores; fp32 (and d = 64) on the CUDA cores
  if (dtype == GDN_BF16 && dk == 128) return run_chunk_tc(p, T_total, as_stream(stream));
  return run_chunk_simt(p, dk, dtype, as_stream(stream));
}
