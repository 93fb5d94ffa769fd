// a2. Gated delta rule, token by token (decode), with slot-indexed state gather/scatter in-kernel,
// plus the fused decode layer (conv -> gates -> l2norm -> recurrence -> gated RMSNorm).
//
// Math per (sequence b, value head h), following recurrent_single_step
// (src/recurrent_single_step.py:14-31) and torch_recurrent_gated_delta_rule (transformers
// modeling_qwen3_5.py:314-353):
//   q,k <- l2norm in the activation dtype; q <- q / sqrt(dk)          (all later math fp32)
//   S <- S * exp(g);  m = S^T k;  delta = beta (v - m);  S <- S + k delta^T;  o = S^T q
//
// Design (HBM bound: the 64 KiB fp32 state of a (slot, head) is the traffic):
//   one CTA per (b, h); the state lives in registers for all T tokens.  Thread layout: a float4
//   column group per lane and one state row per warp per pass, so every warp load/store moves
//   whole 512-byte state rows (fully coalesced).  Reductions over dk go through shared memory.
//   The slot index is resolved in-kernel: the CTA loads pool[init_slot[b]] and stores
//   pool[final_slot[b]] -- no index_select / index_copy_ around the call.
#include "common.cuh"

namespace gdn {

struct RecParams {
  const void* q;
  int64_t q_sb, q_st;
  const void* k;
  int64_t k_sb, k_st;
  const void* v;
  int64_t v_sb, v_st;
  const float* g;     // precomputed log-decay [B,T,Hv] (null when raw gates are used)
  const float* beta;  // precomputed beta [B,T,Hv] (fp32)
  int64_t gb_sb, gb_st;
  const void* a_raw;  // raw in_proj_a output [B,Hv] (fused decode layer), with A_log, dt_bias
  const void* b_raw;  // raw in_proj_b output [B,Hv]
  const float* A_log;
  const float* dt_bias;
  const float* init_pool;
  const int32_t* init_slot;
  float* final_pool;
  const int32_t* final_slot;
  int64_t n_slots;
  void* out;
  int64_t o_sb, o_st;
  const void* z;       // gate for the fused gated RMSNorm [B,Hv,dv] (null: plain output)
  const void* norm_w;  // [dv]
  float eps;
  int B, T, Hk, Hv;
  int l2norm;
  int32_t* err;
};

template <int DK, int DV>
struct RecShape {
  static constexpr int CG = DV / 4;        // float4 column groups per state row
  static constexpr int RPW = 32 / CG;      // state rows covered by one warp per pass
  static constexpr int NW = DK == 128 ? 16 : 8;
  static constexpr int NRS = NW * RPW;     // row slots
  static constexpr int R = DK / NRS;       // state rows per thread
  static constexpr int NT = NW * 32;
  static_assert(R * NRS == DK, "row split");
};

// Load one head row of q or k (D values) with a warp, optionally l2-normalise it in the
// activation dtype (x * rsqrt(sum(x*x) + 1e-6), each op rounded to T as torch does), scale it
// and store fp32 to shared memory.
template <typename T, int D>
__device__ __forceinline__ void load_qk_row(const T* src, float* dst, bool l2, float scale, int lane) {
  constexpr int PER = D / 32;
  float x[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    x[i] = Io<T>::ld(src + lane + 32 * i);
    ss += Io<T>::rnd(x[i] * x[i]);
  }
  if (l2) {
    ss = warp_sum(ss);
    float s = Io<T>::rnd(ss);
    s = Io<T>::rnd(s + 1e-6f);
    const float inv = Io<T>::rnd(1.0f / sqrtf(s));
#pragma unroll
    for (int i = 0; i < PER; ++i) x[i] = Io<T>::rnd(x[i] * inv);
  }
#pragma unroll
  for (int i = 0; i < PER; ++i) dst[lane + 32 * i] = x[i] * scale;
}

template <typename T, int DK, int DV>
__global__ void __launch_bounds__(RecShape<DK, DV>::NT, 2) recurrent_kernel(RecParams p) {
  using Sh = RecShape<DK, DV>;
  constexpr int CG = Sh::CG, RPW = Sh::RPW, NRS = Sh::NRS, R = Sh::R;
  __shared__ float sq[DK], sk[DK], sv[DV], sdelta[DV];
  __shared__ float red[NRS][DV];
  __shared__ float sgate[2];
  __shared__ float snorm[DV / 32];

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = h / (p.Hv / p.Hk);
  const int cg = lane % CG, rs = warp * RPW + lane / CG;
  const float scale = float(1.0 / sqrt(double(DK)));

  int64_t islot = p.init_slot ? int64_t(p.init_slot[b]) : int64_t(b);
  int64_t fslot = p.final_slot ? int64_t(p.final_slot[b]) : int64_t(b);
  bool init_ok = p.init_pool != nullptr;
  bool fin_ok = p.final_pool != nullptr;
  if (init_ok && (islot < 0 || islot >= p.n_slots)) init_ok = false;
  if (fin_ok && (fslot < 0 || fslot >= p.n_slots)) fin_ok = false;
  if ((p.init_pool && !init_ok) || (p.final_pool && !fin_ok)) {
    // a bad slot index: record it and leave every pool row untouched
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    return;
  }

  float s[R][4];
  if (init_ok) {
    const float* src = p.init_pool + (islot * p.Hv + h) * int64_t(DK * DV);
#pragma unroll
    for (int r = 0; r < R; ++r) {
      const float4 t4 = *reinterpret_cast<const float4*>(src + (rs + r * NRS) * DV + cg * 4);
      s[r][0] = t4.x; s[r][1] = t4.y; s[r][2] = t4.z; s[r][3] = t4.w;
    }
  } else {
#pragma unroll
    for (int r = 0; r < R; ++r) s[r][0] = s[r][1] = s[r][2] = s[r][3] = 0.f;
  }

  const T* qb = reinterpret_cast<const T*>(p.q) + b * p.q_sb + int64_t(hk) * DK;
  const T* kb = reinterpret_cast<const T*>(p.k) + b * p.k_sb + int64_t(hk) * DK;
  const T* vb = reinterpret_cast<const T*>(p.v) + b * p.v_sb + int64_t(h) * DV;

  for (int t = 0; t < p.T; ++t) {
    // ---- phase A: q, k (normalised, fp32), v, gates into shared memory
    if (warp == 0) load_qk_row<T, DK>(qb + t * p.q_st, sq, p.l2norm, scale, lane);
    else if (warp == 1) load_qk_row<T, DK>(kb + t * p.k_st, sk, p.l2norm, 1.0f, lane);
    else if (warp == 2) {
      for (int i = lane; i < DV; i += 32) sv[i] = Io<T>::ld(vb + t * p.v_st + i);
    } else if (warp == 3 && lane == 0) {
      float beta, g;
      if (p.a_raw) {
        const float a = Io<T>::ld(reinterpret_cast<const T*>(p.a_raw) + int64_t(b) * p.Hv + h);
        const float braw = Io<T>::ld(reinterpret_cast<const T*>(p.b_raw) + int64_t(b) * p.Hv + h);
        beta = Io<T>::rnd(sigmoid_f(braw));
        g = -expf(p.A_log[h]) * softplus_f(a + p.dt_bias[h]);
      } else {
        const int64_t gi = b * p.gb_sb + t * p.gb_st + h;
        g = p.g[gi];
        beta = p.beta[gi];
      }
      sgate[0] = g;
      sgate[1] = beta;
    }
    __syncthreads();

    // ---- phase B: decay, m = S^T k
    const float decay = expf(sgate[0]);
    float kr[R], qr[R];
#pragma unroll
    for (int r = 0; r < R; ++r) {
      kr[r] = sk[rs + r * NRS];
      qr[r] = sq[rs + r * NRS];
    }
    float mp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[r][j] *= decay;
        mp[j] = fmaf(s[r][j], kr[r], mp[j]);
      }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rs][cg * 4 + j] = mp[j];
    __syncthreads();
    if (tid < DV) {
      float m = 0.f;
#pragma unroll
      for (int i = 0; i < NRS; ++i) m += red[i][tid];
      sdelta[tid] = (sv[tid] - m) * sgate[1];
    }
    __syncthreads();

    // ---- phase C: S += k delta^T; o = S^T q
    float dl[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) dl[j] = sdelta[cg * 4 + j];
    float op[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < R; ++r)
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        s[r][j] = fmaf(kr[r], dl[j], s[r][j]);
        op[j] = fmaf(s[r][j], qr[r], op[j]);
      }
#pragma unroll
    for (int j = 0; j < 4; ++j) red[rs][cg * 4 + j] = op[j];
    __syncthreads();

    // ---- phase D: output (optionally through the gated RMSNorm)
    if (tid < DV) {
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < NRS; ++i) o += red[i][tid];
      o = Io<T>::rnd(o);  // core output in the activation dtype
      if (p.z) {
        float ss = warp_sum(o * o);
        if (lane == 0) snorm[warp] = ss;
        asm volatile("bar.sync 1, %0;" ::"r"(DV));
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < DV / 32; ++i) tot += snorm[i];
        const float rinv = 1.0f / sqrtf(tot / float(DV) + p.eps);
        const T* zr = reinterpret_cast<const T*>(p.z) + (int64_t(b) * p.Hv + h) * DV;
        const float w = Io<T>::ld(reinterpret_cast<const T*>(p.norm_w) + tid);
        o = Io<T>::rnd(w * Io<T>::rnd(o * rinv)) * silu_f(Io<T>::ld(zr + tid));
      }
      Io<T>::st(reinterpret_cast<T*>(p.out) + b * p.o_sb + t * p.o_st + int64_t(h) * DV + tid, o);
    }
    __syncthreads();
  }

  if (fin_ok) {
    float* dst = p.final_pool + (fslot * p.Hv + h) * int64_t(DK * DV);
#pragma unroll
    for (int r = 0; r < R; ++r)
      *reinterpret_cast<float4*>(dst + (rs + r * NRS) * DV + cg * 4) =
          make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
  }
}

template <typename T>
static int launch_rec(const RecParams& p, int dk, int dv, cudaStream_t s) {
  dim3 grid(p.Hv, p.B);
  if (dk == 128 && dv == 128) {
    recurrent_kernel<T, 128, 128><<<grid, RecShape<128, 128>::NT, 0, s>>>(p);
  } else if (dk == 64 && dv == 64) {
    recurrent_kernel<T, 64, 64><<<grid, RecShape<64, 64>::NT, 0, s>>>(p);
  } else {
    return fail(GDN_ERR_SHAPE, "gdn_recurrent: (dk,dv)=(%d,%d) not built", dk, dv);
  }
  return check_launch("gdn_recurrent");
}

int run_recurrent(const RecParams& p, int dk, int dv, int dtype, cudaStream_t s) {
  if (dtype == GDN_BF16) return launch_rec<__nv_bfloat16>(p, dk, dv, s);
  if (dtype == GDN_F32) return launch_rec<float>(p, dk, dv, s);
  return fail(GDN_ERR_DTYPE, "gdn_recurrent: dtype %d", dtype);
}

static int check_heads(const char* who, int B, int Hk, int Hv, int dk, int dv) {
  if (B < 0 || Hk <= 0 || Hv <= 0) return fail(GDN_ERR_ARG, "%s: B=%d Hk=%d Hv=%d", who, B, Hk, Hv);
  if (Hv % Hk != 0) return fail(GDN_ERR_SHAPE, "%s: Hv=%d not a multiple of Hk=%d", who, Hv, Hk);
  if (!((dk == 128 && dv == 128) || (dk == 64 && dv == 64)))
    return fail(GDN_ERR_SHAPE, "%s: (dk,dv)=(%d,%d) not built", who, dk, dv);
  if (B > 65535) return fail(GDN_ERR_ARG, "%s: B=%d > 65535", who, B);
  return GDN_OK;
}

int launch_conv_update(const void* x, int64_t xs_b, int64_t xs_c, int64_t xs_t, void* pool,
                       const int32_t* slot_idx, int64_t n_slots, const void* w, const void* bias, void* y,
                       int64_t ys_b, int64_t ys_c, int64_t ys_t, int B, int C, int T, int K, int act,
                       int mode, int dtype, int32_t* err, cudaStream_t s);

}  // namespace gdn

extern "C" int gdn_recurrent(const void* q, int64_t q_sb, int64_t q_st, const void* k, int64_t k_sb,
                             int64_t k_st, const void* v, int64_t v_sb, int64_t v_st, const float* g,
                             const float* beta, int64_t gb_sb, int64_t gb_st, const float* init_pool,
                             const int32_t* init_slot, float* final_pool, const int32_t* final_slot,
                             int64_t n_slots, void* out, int64_t o_sb, int64_t o_st, int B, int T, int Hk,
                             int Hv, int dk, int dv, int use_qk_l2norm, int dtype, int32_t* err_flag,
                             void* stream) {
  using namespace gdn;
  int rc = check_heads("gdn_recurrent", B, Hk, Hv, dk, dv);
  if (rc) return rc;
  if (T < 0) return fail(GDN_ERR_ARG, "gdn_recurrent: T=%d", T);
  if (B == 0 || T == 0) return GDN_OK;
  if (!q || !k || !v || !g || !beta || !out) return fail(GDN_ERR_ARG, "gdn_recurrent: null pointer");
  if ((init_pool || final_pool) && n_slots < 1) return fail(GDN_ERR_ARG, "gdn_recurrent: n_slots=%lld", (long long)n_slots);
  if ((init_pool && !aligned(init_pool, 16)) || (final_pool && !aligned(final_pool, 16)))
    return fail(GDN_ERR_ARG, "gdn_recurrent: state pools must be 16-byte aligned");
  RecParams p{};
  p.q = q; p.q_sb = q_sb; p.q_st = q_st;
  p.k = k; p.k_sb = k_sb; p.k_st = k_st;
  p.v = v; p.v_sb = v_sb; p.v_st = v_st;
  p.g = g; p.beta = beta; p.gb_sb = gb_sb; p.gb_st = gb_st;
  p.init_pool = init_pool; p.init_slot = init_slot; p.final_pool = final_pool; p.final_slot = final_slot;
  p.n_slots = n_slots;
  p.out = out; p.o_sb = o_sb; p.o_st = o_st;
  p.B = B; p.T = T; p.Hk = Hk; p.Hv = Hv; p.l2norm = use_qk_l2norm; p.err = err_flag;
  return run_recurrent(p, dk, dv, dtype, as_stream(stream));
}

extern "C" size_t gdn_decode_layer_workspace_size(int n, int Hk, int Hv, int dk, int dv, int dtype) {
  const size_t es = dtype == GDN_F32 ? 4 : 2;
  const size_t C = size_t(2) * Hk * dk + size_t(Hv) * dv;
  const size_t bytes = size_t(n) * C * es;
  return (bytes + 255) & ~size_t(255);
}

extern "C" int gdn_decode_layer(const void* mixed_qkv, int64_t mixed_rs, const void* z, const void* a,
                                const void* b, const float* A_log, const float* dt_bias, const void* conv_w,
                                const void* conv_b, void* conv_pool, float* rec_pool, const int32_t* slot_idx,
                                int64_t n_slots, const void* norm_w, float eps, void* out, int n, int Hk,
                                int Hv, int dk, int dv, int K, int conv_mode, void* workspace,
                                size_t workspace_bytes, int dtype, int32_t* err_flag, void* stream) {
  using namespace gdn;
  int rc = check_heads("gdn_decode_layer", n, Hk, Hv, dk, dv);
  if (rc) return rc;
  if (n == 0) return GDN_OK;
  if (!mixed_qkv || !z || !a || !b || !A_log || !dt_bias || !conv_w || !conv_pool || !rec_pool || !norm_w || !out)
    return fail(GDN_ERR_ARG, "gdn_decode_layer: null pointer");
  if (n_slots < 1) return fail(GDN_ERR_ARG, "gdn_decode_layer: n_slots=%lld", (long long)n_slots);
  if (dtype != GDN_BF16 && dtype != GDN_F32) return fail(GDN_ERR_DTYPE, "gdn_decode_layer: dtype %d", dtype);
  const size_t need = gdn_decode_layer_workspace_size(n, Hk, Hv, dk, dv, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "gdn_decode_layer: workspace %zu bytes < %zu", workspace_bytes, need);
  if (!aligned(rec_pool, 16)) return fail(GDN_ERR_ARG, "gdn_decode_layer: rec_pool must be 16-byte aligned");
  const int C = 2 * Hk * dk + Hv * dv;
  cudaStream_t s = as_stream(stream);
  // 1) conv update + silu: mixed [n, C] -> workspace [n, C]
  rc = launch_conv_update(mixed_qkv, mixed_rs, 1, 0, conv_pool, slot_idx, n_slots, conv_w, conv_b, workspace,
                          C, 1, 0, n, C, 1, K, 1, conv_mode, dtype, err_flag, s);
  if (rc) return rc;
  // 2) gates + l2norm + recurrence (in place on rec_pool[slot_idx]) + gated RMSNorm
  const size_t es = dtype == GDN_F32 ? 4 : 2;
  const char* ws = reinterpret_cast<const char*>(workspace);
  RecParams p{};
  p.q = ws; p.q_sb = C; p.q_st = 0;
  p.k = ws + size_t(Hk) * dk * es; p.k_sb = C; p.k_st = 0;
  p.v = ws + size_t(2) * Hk * dk * es; p.v_sb = C; p.v_st = 0;
  p.a_raw = a; p.b_raw = b; p.A_log = A_log; p.dt_bias = dt_bias;
  p.init_pool = rec_pool; p.init_slot = slot_idx; p.final_pool = rec_pool; p.final_slot = slot_idx;
  p.n_slots = n_slots;
  p.out = out; p.o_sb = int64_t(Hv) * dv; p.o_st = 0;
  p.z = z; p.norm_w = norm_w; p.eps = eps;
  p.B = n; p.T = 1; p.Hk = Hk; p.Hv = Hv; p.l2norm = 1; p.err = err_flag;
  return run_recurrent(p, dk, dv, dtype, s);
}
