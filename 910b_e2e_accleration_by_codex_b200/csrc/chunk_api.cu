// C entry points of the chunked prefill: argument checks and kernel selection.
#include "chunk.cuh"

namespace {

using namespace gdn;

// Shared body of gdn_chunk_prefill and gdn_chunk_prefill_gates; `p` carries the gate source.
int chunk_prefill(const char* fn, ChunkParams& p, const void* q, int64_t q_st, const void* k, int64_t k_st,
                  const void* v, int64_t v_st, const int32_t* cu_seqlens, int B, int64_t T_total,
                  const float* init_pool, const int32_t* init_slot, const int32_t* use_initial, float* final_pool,
                  const int32_t* final_slot, int64_t n_slots, void* out, int64_t o_st, int Hk, int Hv, int dk,
                  int dv, int use_qk_l2norm, int dtype, int32_t* err_flag, void* stream) {
  if (B < 0 || T_total < 0 || Hk <= 0 || Hv <= 0)
    return fail(GDN_ERR_ARG, "%s: B=%d T=%lld Hk=%d Hv=%d", fn, B, (long long)T_total, Hk, Hv);
  if (B == 0) return GDN_OK;
  // with no tokens (every sequence empty) q/k/v/out are never read and may be null
  if (!cu_seqlens || (T_total > 0 && (!q || !k || !v || !out))) return fail(GDN_ERR_ARG, "%s: null pointer", fn);
  if (Hv % Hk != 0) return fail(GDN_ERR_SHAPE, "%s: Hv=%d not a multiple of Hk=%d", fn, Hv, Hk);
  if (dk != dv || (dk != 64 && dk != 128))
    return fail(GDN_ERR_SHAPE, "%s: (dk,dv)=(%d,%d) not built", fn, dk, dv);
  if (B > 65535) return fail(GDN_ERR_ARG, "%s: B=%d > 65535", fn, B);
  if ((init_pool || final_pool) && n_slots < 1) return fail(GDN_ERR_ARG, "%s: n_slots=%lld", fn, (long long)n_slots);
  if (dtype != GDN_BF16 && dtype != GDN_F32) return fail(GDN_ERR_DTYPE, "%s: dtype %d", fn, dtype);
  p.q = q; p.q_st = q_st; p.k = k; p.k_st = k_st; p.v = v; p.v_st = v_st;
  p.cu = cu_seqlens;
  p.init_pool = init_pool; p.init_slot = init_slot; p.use_init = use_initial;
  p.final_pool = final_pool; p.final_slot = final_slot; p.n_slots = n_slots;
  p.out = out; p.o_st = o_st; p.B = B; p.Hk = Hk; p.Hv = Hv; p.l2norm = use_qk_l2norm; p.err = err_flag;
  // bf16 activations at dk = dv = 128 run on the tensor cores; fp32 (and d = 64) on the CUDA cores.
  // Without tokens only the final states (initial state or zeros) are written: the CUDA-core kernel
  // does that without building tensor maps over empty arrays.
  if (dtype == GDN_BF16 && dk == 128 && T_total > 0) return run_chunk_tc(p, T_total, as_stream(stream));
  return run_chunk_simt(p, dk, dtype, as_stream(stream));
}

}  // namespace

extern "C" int gdn_chunk_prefill(const void* q, int64_t q_st, const void* k, int64_t k_st, const void* v,
                                 int64_t v_st, const float* g, const float* beta, int64_t gb_st,
                                 const int32_t* cu_seqlens, int B, int64_t T_total, const float* init_pool,
                                 const int32_t* init_slot, const int32_t* use_initial, float* final_pool,
                                 const int32_t* final_slot, int64_t n_slots, void* out, int64_t o_st, int Hk,
                                 int Hv, int dk, int dv, int use_qk_l2norm, int dtype, int32_t* err_flag,
                                 void* stream) {
  using namespace gdn;
  if (B > 0 && T_total > 0 && (!g || !beta)) return fail(GDN_ERR_ARG, "gdn_chunk_prefill: null pointer");
  ChunkParams p{};
  p.g = g; p.beta = beta; p.gb_st = gb_st;
  return chunk_prefill("gdn_chunk_prefill", p, q, q_st, k, k_st, v, v_st, cu_seqlens, B, T_total, init_pool,
                       init_slot, use_initial, final_pool, final_slot, n_slots, out, o_st, Hk, Hv, dk, dv,
                       use_qk_l2norm, dtype, err_flag, stream);
}

extern "C" int gdn_chunk_prefill_gates(const void* q, int64_t q_st, const void* k, int64_t k_st, const void* v,
                                       int64_t v_st, const void* a, const void* b, int64_t ab_st,
                                       const float* A_log, const float* dt_bias, const int32_t* cu_seqlens,
                                       int B, int64_t T_total, const float* init_pool, const int32_t* init_slot,
                                       const int32_t* use_initial, float* final_pool, const int32_t* final_slot,
                                       int64_t n_slots, void* out, int64_t o_st, int Hk, int Hv, int dk, int dv,
                                       int use_qk_l2norm, int dtype, int32_t* err_flag, void* stream) {
  using namespace gdn;
  if (B > 0 && T_total > 0 && (!a || !b || !A_log || !dt_bias))
    return fail(GDN_ERR_ARG, "gdn_chunk_prefill_gates: null pointer");
  ChunkParams p{};
  p.a_raw = a; p.b_raw = b; p.A_log = A_log; p.dt_bias = dt_bias; p.gb_st = ab_st;
  p.raw_bf16 = dtype == GDN_BF16;
  return chunk_prefill("gdn_chunk_prefill_gates", p, q, q_st, k, k_st, v, v_st, cu_seqlens, B, T_total,
                       init_pool, init_slot, use_initial, final_pool, final_slot, n_slots, out, o_st, Hk, Hv, dk,
                       dv, use_qk_l2norm, dtype, err_flag, stream);
}
