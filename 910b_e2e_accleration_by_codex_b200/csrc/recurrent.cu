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
#include <cstddef>
#include <type_traits>

#include "common.cuh"
#include "sm100.cuh"

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
  int64_t z_rs;        // element stride between z's rows b (Hv * dv when contiguous)
  int64_t a_rs, b_rs;  // element strides between the rows b of a_raw / b_raw (Hv when contiguous)
  const void* norm_w;  // [dv]
  float eps;
  // fused conv update (decode layer, T = 1): q/k/v are the silu(conv) of mixed_qkv [B, C] with the
  // slot's conv state; q, k, v above are then unused
  const void* mixed;
  int64_t mixed_rs;
  const void* conv_w;  // [C, K]
  const void* conv_b;  // [C] or null
  void* conv_pool;     // [n_slots, C, K], updated in place
  unsigned int* tickets;  // [B * Hk], zero between calls
  int C, K, conv_mode;
  int B, T, Hk, Hv;
  int l2norm;
  int32_t* err;
};

// One causal-conv output channel: push x into the K-window of the slot's state, return
// silu(conv) rounded to T, and hand back the new window (written to the pool by the caller).
template <typename T>
__device__ __forceinline__ float conv_channel(const T* st, const T* w, const T* bias, float x, int K, int mode,
                                              float* nwin) {
  float acc = 0.f, accr = 0.f;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    if (j < K) {
      const float wj = Io<T>::ld(w + j);
      const float xj = j + 1 < K ? Io<T>::ld(st + j + 1) : x;
      nwin[j] = xj;
      acc = fmaf(xj, wj, acc);
      accr += Io<T>::rnd(xj * wj);
    }
  }
  float o;
  if (mode == GDN_CONV_ELEM) {
    o = Io<T>::rnd(accr);
    if (bias) o = Io<T>::rnd(o + Io<T>::ld(bias));
  } else {
    if (bias) acc += Io<T>::ld(bias);
    o = Io<T>::rnd(acc);
  }
  return Io<T>::rnd(silu_f(o));
}

// atomicInc with acquire-release semantics at GPU scope: the last CTA of a k-head to take its ticket
// sees every other CTA's reads of the shared q/k windows as done before it overwrites them.
__device__ __forceinline__ unsigned ticket_inc(unsigned* p, unsigned wrap) {
  unsigned old;
  asm volatile("atom.acq_rel.gpu.global.inc.u32 %0, [%1], %2;" : "=r"(old) : "l"(p), "r"(wrap) : "memory");
  return old;
}

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

// Same as load_qk_row, for a row already in shared memory (values on the activation grid).
template <typename T, int D>
__device__ __forceinline__ void norm_qk_row(const float* src, float* dst, bool l2, float scale, int lane) {
  constexpr int PER = D / 32;
  float x[PER];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < PER; ++i) {
    x[i] = src[lane + 32 * i];
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
  static_assert(DK == DV, "fused conv assumes dk == dv");
  __shared__ float sconv[3][DK];
  __shared__ int slast;
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

  unsigned ticket = 0;  // fused conv: this CTA's place among the value heads of its k-head
  if (p.mixed) {
    // ---- fused conv update (T = 1): silu(conv) of this head's q, k and v channels.  The q/k
    //      channels are shared by the Hv/Hk value heads of the k-head; each of their CTAs reads
    //      the old window, then takes a ticket; the last one writes the new q/k window at its end
    //      (so no CTA can read a half-updated window) and the ticket counter wraps back to zero.
    const T* mixed = reinterpret_cast<const T*>(p.mixed) + int64_t(b) * p.mixed_rs;
    T* cpool = reinterpret_cast<T*>(p.conv_pool) + fslot * int64_t(p.C) * p.K;
    const T* cw = reinterpret_cast<const T*>(p.conv_w);
    const T* cb = reinterpret_cast<const T*>(p.conv_b);
    const int which = tid / DK, i = tid % DK;  // 0: q, 1: k, 2: v channel i
    float nwin[8];
    int c = 0;
    if (which < 3) {
      c = which == 0 ? hk * DK + i : which == 1 ? p.Hk * DK + hk * DK + i : 2 * p.Hk * DK + h * DV + i;
      sconv[which][i] = conv_channel<T>(cpool + int64_t(c) * p.K, cw + int64_t(c) * p.K, cb ? cb + c : nullptr,
                                        Io<T>::ld(mixed + c), p.K, p.conv_mode, nwin);
    }
    __syncthreads();  // every old window of this CTA has been read
    if (tid == 0) ticket = ticket_inc(p.tickets + int64_t(b) * p.Hk + hk, unsigned(p.Hv / p.Hk) - 1);
  }

  for (int t = 0; t < p.T; ++t) {
    // ---- phase A: q, k (normalised, fp32), v, gates into shared memory
    if (p.mixed) {
      if (warp == 0) norm_qk_row<T, DK>(sconv[0], sq, p.l2norm, scale, lane);
      else if (warp == 1) norm_qk_row<T, DK>(sconv[1], sk, p.l2norm, 1.0f, lane);
      else if (warp == 2) {
        for (int i = lane; i < DV; i += 32) sv[i] = sconv[2][i];
      }
    } else if (warp == 0) load_qk_row<T, DK>(qb + t * p.q_st, sq, p.l2norm, scale, lane);
    else if (warp == 1) load_qk_row<T, DK>(kb + t * p.k_st, sk, p.l2norm, 1.0f, lane);
    else if (warp == 2) {
      for (int i = lane; i < DV; i += 32) sv[i] = Io<T>::ld(vb + t * p.v_st + i);
    }
    if (warp == 3 && lane == 0) {
      float beta, g;
      if (p.a_raw) {
        const float a = Io<T>::ld(reinterpret_cast<const T*>(p.a_raw) + int64_t(b) * p.a_rs + h);
        const float braw = Io<T>::ld(reinterpret_cast<const T*>(p.b_raw) + int64_t(b) * p.b_rs + h);
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
        const T* zr = reinterpret_cast<const T*>(p.z) + int64_t(b) * p.z_rs + int64_t(h) * DV;
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
  if (p.mixed) {  // new conv windows: v channels always, q/k channels by the last CTA of the k-head
    if (tid == 0) slast = ticket == unsigned(p.Hv / p.Hk) - 1;
    __syncthreads();
    const int which = tid / DK, i = tid % DK;
    if (which == 2 || (which < 2 && slast)) {
      // nobody else writes this window, so the old one is still there: shift it and append x
      const int c = which == 0 ? hk * DK + i : which == 1 ? p.Hk * DK + hk * DK + i : 2 * p.Hk * DK + h * DV + i;
      T* w = reinterpret_cast<T*>(p.conv_pool) + (fslot * int64_t(p.C) + c) * p.K;
      float nw[8];
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < p.K)
          nw[j] = j + 1 < p.K ? Io<T>::ld(w + j + 1)
                              : Io<T>::ld(reinterpret_cast<const T*>(p.mixed) + int64_t(b) * p.mixed_rs + c);
#pragma unroll
      for (int j = 0; j < 8; ++j)
        if (j < p.K) Io<T>::st(w + j, nw[j]);
    }
  }
}

// ------------------------------------------------------------------ decode layer, dk = dv = 128: two kernels
//
// The decode step moves 64 KiB of fp32 state in and out per (slot, value head) and does ~4 flops
// per state element, so it is an HBM stream.  Keeping that stream full leaves every other global
// access of the step queued behind it for microseconds, so the layer is split in two:
//
//   decode_prep_kernel   (b, head row): conv update of the slot's window, silu, l2norm of the q/k
//                        rows in the activation dtype, the gates; writes compact rows
//                        prep [n, C] (dtype) and gates [n, Hv, 4] f32 = (g, beta, -, -).
//   decode_state_kernel  one CTA per SM over the items (b, h) = it, it + grid, ...: every input
//                        of an item (its 64 KiB state, the q/k/v rows, the gates, the z row) arrives by bulk
//                        copy (cp.async.bulk on the stage's mbarrier) into a 3-deep shared-memory
//                        ring, issued by one thread two items ahead; the compute warps write the
//                        new state back into its stage and the same thread stores it with a bulk
//                        copy.  The compute warps never wait on a global load, and the state
//                        traffic never passes through their load/store queues.
//
// The state kernel is launched as a programmatic dependent of the prep kernel: it starts while
// the prep kernel runs, loads its first state (which the prep kernel does not touch), and its copy
// thread waits for the prep kernel's results (griddepcontrol.wait) before loading them.
namespace dec {
constexpr int D = 128;
constexpr int kStages = 3;
constexpr int kThreads = 512;               // 16 warps; warp w owns state rows w, w+16, ..., lane 4 columns
constexpr int kRows = D / 16;
constexpr int kOutTid0 = 3 * D;             // warps 12-15 produce the output of the previous item
constexpr int kCopyTid = 11 * 32;           // issues the bulk loads and stores (not an output warp)
constexpr int kSlotCache = 512;             // slot indices of a CTA's first items kept in shared memory
constexpr uint32_t kStateBytes = D * D * 4;
constexpr int kInFloats = 4 + 4 * D;        // per stage: gates (4 floats), then q, k, v, z rows (up to f32)

struct Smem {
  float state[kStages][D * D];
  float in[kStages][kInFloats];
  float sdelta[D];
  float red[2][16][D];                      // [0]: S^T k partials, [1]: S^T q partials
  int slot[kSlotCache];
  float snorm[4];
  unsigned long long full[kStages];
};

static_assert(offsetof(Smem, red) % 16 == 0 && offsetof(Smem, sdelta) % 16 == 0 && offsetof(Smem, in) % 16 == 0,
              "float4 rows and bulk-copy targets on 16-byte offsets");
static_assert(offsetof(Smem, full) % 8 == 0, "mbarriers on 8-byte offsets");

__device__ __forceinline__ void cta_sync() { asm volatile("bar.sync 1, 512;" ::: "memory"); }
__device__ __forceinline__ void out_sync() { asm volatile("bar.sync 2, 128;" ::: "memory"); }
}  // namespace dec

// grid (C / 128, n), 128 threads: channels [128 x, 128 x + 128) of slot entry b, i.e. one q, k or v
// head row.  Conv math as conv_channel; l2norm as norm_qk_row (same summation order).
template <typename T, int KW>
__global__ void __launch_bounds__(dec::D) decode_prep_kernel(RecParams p, T* prep, float* gates) {
  using dec::D;
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ float sq2[D];
  __shared__ float sinv;
  const int row = blockIdx.x, b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t slot = p.init_slot[b];
  if (slot < 0 || slot >= p.n_slots) {  // a bad slot index: record it, leave every pool row alone
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    return;
  }
  const int c = row * D + tid;
  const T* cw = reinterpret_cast<const T*>(p.conv_w) + int64_t(c) * p.K;
  const T* cb = reinterpret_cast<const T*>(p.conv_b);
  T* win = reinterpret_cast<T*>(p.conv_pool) + (slot * int64_t(p.C) + c) * p.K;
  float nwin[8];
  float y = conv_channel<T>(win, cw, cb ? cb + c : nullptr,
                            Io<T>::ld(reinterpret_cast<const T*>(p.mixed) + int64_t(b) * p.mixed_rs + c), p.K,
                            p.conv_mode, nwin);
#pragma unroll
  for (int t = 0; t < KW; ++t)
    if (t < p.K) Io<T>::st(win + t, nwin[t]);
  if (row < 2 * p.Hk && p.l2norm) {  // q or k head row: l2norm in the activation dtype
    sq2[tid] = Io<T>::rnd(y * y);
    __syncthreads();
    if (warp == 0) {
      float ss = sq2[lane];
#pragma unroll
      for (int i = 1; i < D / 32; ++i) ss += sq2[lane + 32 * i];
      ss = warp_sum(ss);
      float s2 = Io<T>::rnd(ss);
      s2 = Io<T>::rnd(s2 + 1e-6f);
      if (lane == 0) sinv = Io<T>::rnd(1.0f / sqrtf(s2));
    }
    __syncthreads();
    y = Io<T>::rnd(y * sinv);
  }
  Io<T>::st(prep + int64_t(b) * p.C + c, y);
  if (row >= 2 * p.Hk && tid == 0) {
    const int h = row - 2 * p.Hk;
    const float a = Io<T>::ld(reinterpret_cast<const T*>(p.a_raw) + int64_t(b) * p.a_rs + h);
    const float braw = Io<T>::ld(reinterpret_cast<const T*>(p.b_raw) + int64_t(b) * p.b_rs + h);
    float* gt = gates + (int64_t(b) * p.Hv + h) * 4;
    gt[0] = -expf(p.A_log[h]) * softplus_f(a + p.dt_bias[h]);
    gt[1] = Io<T>::rnd(sigmoid_f(braw));
  }
}

template <typename T>
__global__ void __launch_bounds__(dec::kThreads, 1) decode_state_kernel(RecParams p, const T* prep,
                                                                        const float* gates) {
  using namespace dec;
  using namespace sm100;
  extern __shared__ __align__(128) unsigned char dec_smem[];
  Smem& sm = *reinterpret_cast<Smem*>(dec_smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int nitems = p.B * p.Hv;
  const int G = p.Hv / p.Hk;
  const int grid = gridDim.x;
  const int nmine = nitems > int(blockIdx.x) ? (nitems - int(blockIdx.x) + grid - 1) / grid : 0;
  constexpr uint32_t kRowBytes = D * sizeof(T);
  constexpr uint32_t kStageTx = kStateBytes + 16 + 4 * kRowBytes;

  if (tid == 0) {
    for (int k = 0; k < kStages; ++k) mbar_init(smem_u32(&sm.full[k]), 1);
    fence_mbar_init();
  }
  for (int m = tid; m < nmine && m < kSlotCache; m += kThreads)
    sm.slot[m] = p.init_slot[(int(blockIdx.x) + m * grid) / p.Hv];
  __syncthreads();
  // slot of this CTA's m-th item, or -1 when it is out of range
  auto slot_of = [&](int m) -> int64_t {
    const int it = int(blockIdx.x) + m * grid;
    const int64_t s = m < kSlotCache ? int64_t(sm.slot[m]) : int64_t(p.init_slot[it / p.Hv]);
    return s >= 0 && s < p.n_slots ? s : -1;
  };
  // copy thread: item m's state and its input rows into stage m % 3 (a bad slot completes the
  // stage's phase empty, so every item takes one phase of its stage)
  auto load_state = [&](int m) {
    const int k = m % kStages;
    const int64_t slot = slot_of(m);
    if (slot < 0) {
      mbar_arrive(smem_u32(&sm.full[k]));
      return;
    }
    const int it = int(blockIdx.x) + m * grid;
    mbar_expect_tx(smem_u32(&sm.full[k]), kStageTx);
    bulk_load(smem_u32(sm.state[k]), p.final_pool + (slot * p.Hv + it % p.Hv) * int64_t(D * D), kStateBytes,
              smem_u32(&sm.full[k]));
  };
  auto load_inputs = [&](int m) {
    const int k = m % kStages;
    if (slot_of(m) < 0) return;
    const int it = int(blockIdx.x) + m * grid;
    const int b = it / p.Hv, h = it % p.Hv, hk = h / G;
    const uint32_t bar = smem_u32(&sm.full[k]);
    const uint32_t dst = smem_u32(sm.in[k]);
    const T* row = prep + int64_t(b) * p.C;
    bulk_load(dst, gates + (int64_t(b) * p.Hv + h) * 4, 16, bar);
    bulk_load(dst + 16, row + hk * D, kRowBytes, bar);
    bulk_load(dst + 16 + kRowBytes, row + (p.Hk + hk) * D, kRowBytes, bar);
    bulk_load(dst + 16 + 2 * kRowBytes, row + (2 * p.Hk + h) * D, kRowBytes, bar);
    bulk_load(dst + 16 + 3 * kRowBytes, reinterpret_cast<const T*>(p.z) + int64_t(b) * p.z_rs + int64_t(h) * D,
              kRowBytes, bar);
  };
  if (tid == kCopyTid) {
    // item 0 first: the states do not depend on the prep kernel, its q/k/v rows and gates do; the
    // other stages are issued once item 0 has landed, so that it does not share HBM with them
    const int n0 = nmine < kStages ? nmine : kStages;
    if (n0 > 0) load_state(0);
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (n0 > 0) {
      load_inputs(0);
      if (slot_of(0) >= 0) mbar_wait(smem_u32(&sm.full[0]), 0u);
    }
    for (int m = 1; m < n0; ++m) {
      load_state(m);
      load_inputs(m);
    }
  }
  // copy thread, at the end of item m: the stage of item m - 1 takes item m + 2 once the bulk
  // store of item m - 1 has read it (the store of item m, just issued, may still be reading; an
  // item with a bad slot committed no store, so then every store must have been read)
  auto refill = [&](int m, bool stored) {
    if (m < 1 || m + kStages - 1 >= nmine) return;
    if (stored) asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    else asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    load_state(m + kStages - 1);
    load_inputs(m + kStages - 1);
  };

  const int ot = tid - kOutTid0;  // output column (warps 12-15)
  const float scale = float(1.0 / sqrt(double(D)));
  const float nwf = ot >= 0 ? Io<T>::ld(reinterpret_cast<const T*>(p.norm_w) + ot) : 0.f;

  bool ok = true;
  for (int m = 0; m < nmine; ++m) {
    const int it = int(blockIdx.x) + m * grid;
    const int b = it / p.Hv, h = it % p.Hv;
    const int k = m % kStages;
    const int64_t slot = slot_of(m);
    if (slot < 0) {  // a bad slot index: record it, leave every pool row alone
      if (tid == 0 && p.err) atomicExch(p.err, 1);
      if (tid == kCopyTid) refill(m, false);
      continue;
    }

    // B: decay, m = S^T k
    ok &= mbar_wait(smem_u32(&sm.full[k]), uint32_t(m / kStages) & 1u);
    float* st = sm.state[k];
    const float* in = sm.in[k];
    const T* qh = reinterpret_cast<const T*>(in + 4);
    const T* kh = qh + D;
    const T* vh = kh + D;
    const T* zh = vh + D;
    float s[kRows][4], kr[kRows], qr[kRows];
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
      const float4 t4 = *reinterpret_cast<const float4*>(st + (warp + 16 * r) * D + lane * 4);
      s[r][0] = t4.x; s[r][1] = t4.y; s[r][2] = t4.z; s[r][3] = t4.w;
      kr[r] = Io<T>::ld(kh + warp + 16 * r);
      qr[r] = Io<T>::ld(qh + warp + 16 * r) * scale;
    }
    const float decay = expf(in[0]);
    float mp[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kRows; ++r)
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[r][c] *= decay;
        mp[c] = fmaf(s[r][c], kr[r], mp[c]);
      }
    *reinterpret_cast<float4*>(&sm.red[0][warp][lane * 4]) = make_float4(mp[0], mp[1], mp[2], mp[3]);
    cta_sync();
    if (tid < D) {
      float mm = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) mm += sm.red[0][i][tid];
      sm.sdelta[tid] = (Io<T>::ld(vh + tid) - mm) * in[1];
    }
    cta_sync();

    // C: S += k delta^T, o = S^T q; the new state goes back into its stage
    const float4 d4 = *reinterpret_cast<const float4*>(&sm.sdelta[lane * 4]);
    const float dl[4] = {d4.x, d4.y, d4.z, d4.w};
    float op[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int r = 0; r < kRows; ++r) {
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        s[r][c] = fmaf(kr[r], dl[c], s[r][c]);
        op[c] = fmaf(s[r][c], qr[r], op[c]);
      }
      *reinterpret_cast<float4*>(st + (warp + 16 * r) * D + lane * 4) = make_float4(s[r][0], s[r][1], s[r][2], s[r][3]);
    }
    *reinterpret_cast<float4*>(&sm.red[1][warp][lane * 4]) = make_float4(op[0], op[1], op[2], op[3]);
    fence_async_smem();  // the stage's generic-proxy writes before the bulk store reads them
    cta_sync();
    if (tid == kCopyTid) {
      bulk_store(p.final_pool + (slot * p.Hv + h) * int64_t(D * D), smem_u32(st), kStateBytes);
      bulk_commit();
      refill(m, true);
    }

    // D (warps 12-15, while warps 0-11 start the next item): output through the gated RMSNorm; the
    // stage (z row) and red[1] are not overwritten before every warp has passed the next item's B
    if (ot >= 0) {
      const float z = Io<T>::ld(zh + ot);
      float o = 0.f;
#pragma unroll
      for (int i = 0; i < 16; ++i) o += sm.red[1][i][ot];
      o = Io<T>::rnd(o);
      const float ss = warp_sum(o * o);
      if (lane == 0) sm.snorm[warp - kOutTid0 / 32] = ss;
      out_sync();
      float tot = 0.f;
#pragma unroll
      for (int i = 0; i < D / 32; ++i) tot += sm.snorm[i];
      const float rinv = 1.0f / sqrtf(tot / float(D) + p.eps);
      o = Io<T>::rnd(nwf * Io<T>::rnd(o * rinv)) * silu_f(z);
      Io<T>::st(reinterpret_cast<T*>(p.out) + int64_t(b) * p.o_sb + int64_t(h) * D + ot, o);
    }
  }
  if (tid == kCopyTid) bulk_wait_all();  // every bulk store has finished before the CTA exits
  if (!ok && p.err) atomicExch(p.err, 2);
}

// workspace of the dk = dv = 128 decode layer: prep [n, C] (dtype) | gates [n, Hv, 4] f32
static size_t prep_bytes(int n, int C, int dtype) {
  const size_t e = dtype == GDN_F32 ? 4 : 2;
  return (size_t(n) * size_t(C) * e + 255) & ~size_t(255);
}

template <typename T, int KW>
static int launch_decode_layer_kw(const RecParams& p, void* workspace, cudaStream_t s) {
  static bool attr_set[64] = {};
  static int sm_count[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  if (dev >= 0 && dev < 64 && attr_set[dev]) {
    sms = sm_count[dev];
  } else {
    cudaError_t e = cudaFuncSetAttribute(decode_state_kernel<T>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(sizeof(dec::Smem)));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_decode_layer: setup: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) {
      sm_count[dev] = sms;
      attr_set[dev] = true;
    }
  }
  T* prep = reinterpret_cast<T*>(workspace);
  float* gates = reinterpret_cast<float*>(reinterpret_cast<char*>(workspace) +
                                          prep_bytes(p.B, p.C, std::is_same<T, float>::value ? GDN_F32 : GDN_BF16));
  decode_prep_kernel<T, KW><<<dim3(p.C / dec::D, p.B), dec::D, 0, s>>>(p, prep, gates);
  int rc = check_launch("gdn_decode_layer (prep)");
  if (rc) return rc;

  const int items = p.B * p.Hv;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(items < sms ? items : sms);
  cfg.blockDim = dim3(dec::kThreads);
  cfg.dynamicSmemBytes = sizeof(dec::Smem);
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, decode_state_kernel<T>, p, static_cast<const T*>(prep),
                                     static_cast<const float*>(gates));
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_decode_layer: launch: %s", cudaGetErrorString(e));
  return check_launch("gdn_decode_layer (state)");
}

template <typename T>
static int launch_decode_layer(const RecParams& p, void* workspace, cudaStream_t s) {
  return p.K <= 4 ? launch_decode_layer_kw<T, 4>(p, workspace, s) : launch_decode_layer_kw<T, 8>(p, workspace, s);
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
  n = n > 0 ? n : 0;
  Hk = Hk > 0 ? Hk : 0;
  Hv = Hv > 0 ? Hv : 0;
  if (dk == 128 && dv == 128) {
    // prepared q/k/v rows [n, C] in the activation dtype, then the gates [n, Hv, 4] f32
    const int C = 2 * Hk * dk + Hv * dv;
    return gdn::prep_bytes(n, C, dtype) + ((size_t(n) * size_t(Hv) * 16 + 255) & ~size_t(255));
  }
  // one ticket counter (uint32) per (slot entry, k-head) for the shared q/k conv windows
  (void)dtype;
  const size_t bytes = size_t(n) * size_t(Hk) * sizeof(unsigned int);
  return (bytes + 255) & ~size_t(255);
}

namespace gdn {
// Body of gdn_decode_layer and gdn_decode_layer_rows: z, a and b rows `z_rs`, `a_rs`, `b_rs` elements
// apart (Hv * dv, Hv and Hv for contiguous tensors).
static int decode_layer_impl(const char* fn, const void* mixed_qkv, int64_t mixed_rs, const void* z, int64_t z_rs,
                             const void* a, int64_t a_rs, const void* b, int64_t b_rs, const float* A_log,
                             const float* dt_bias, const void* conv_w, const void* conv_b, void* conv_pool,
                             float* rec_pool, const int32_t* slot_idx, int64_t n_slots, const void* norm_w, float eps,
                             void* out, int n, int Hk, int Hv, int dk, int dv, int K, int conv_mode, void* workspace,
                             size_t workspace_bytes, int dtype, int32_t* err_flag, void* stream) {
  int rc = check_heads(fn, n, Hk, Hv, dk, dv);
  if (rc) return rc;
  if (n == 0) return GDN_OK;
  if (!mixed_qkv || !z || !a || !b || !A_log || !dt_bias || !conv_w || !conv_pool || !rec_pool || !norm_w || !out)
    return fail(GDN_ERR_ARG, "%s: null pointer", fn);
  if (n_slots < 1) return fail(GDN_ERR_ARG, "%s: n_slots=%lld", fn, (long long)n_slots);
  if (dtype != GDN_BF16 && dtype != GDN_F32) return fail(GDN_ERR_DTYPE, "%s: dtype %d", fn, dtype);
  if (K < 1 || K > 8) return fail(GDN_ERR_SHAPE, "%s: K=%d (1..8)", fn, K);
  if (conv_mode != GDN_CONV_HF && conv_mode != GDN_CONV_ELEM) return fail(GDN_ERR_ARG, "%s: conv mode %d", fn, conv_mode);
  if (z_rs < int64_t(Hv) * dv || a_rs < Hv || b_rs < Hv || mixed_rs < 2 * Hk * dk + Hv * dv)
    return fail(GDN_ERR_ARG, "%s: row strides (mixed %lld, z %lld, a %lld, b %lld) shorter than a row", fn,
                (long long)mixed_rs, (long long)z_rs, (long long)a_rs, (long long)b_rs);
  const size_t need = gdn_decode_layer_workspace_size(n, Hk, Hv, dk, dv, dtype);
  if (!workspace || workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "%s: workspace %zu bytes < %zu", fn, workspace_bytes, need);
  const int esz = dtype == GDN_BF16 ? 2 : 4;
  // z rows move by 16-byte bulk copies
  if (!aligned(rec_pool, 16) || !aligned(workspace, 16) || !aligned(z, 16) || (z_rs * esz) % 16 != 0)
    return fail(GDN_ERR_ARG, "%s: rec_pool, z, z's row stride and the workspace must be 16-byte aligned", fn);
  // conv update of the slot's window + gates + l2norm + recurrence (in place on rec_pool[slot_idx])
  // + gated RMSNorm: two kernels for dk = dv = 128, one (ticket-ordered windows) for 64
  RecParams p{};
  p.mixed = mixed_qkv; p.mixed_rs = mixed_rs; p.conv_w = conv_w; p.conv_b = conv_b; p.conv_pool = conv_pool;
  p.tickets = reinterpret_cast<unsigned int*>(workspace);
  p.C = 2 * Hk * dk + Hv * dv; p.K = K; p.conv_mode = conv_mode;
  p.a_raw = a; p.b_raw = b; p.a_rs = a_rs; p.b_rs = b_rs; p.A_log = A_log; p.dt_bias = dt_bias;
  p.init_pool = rec_pool; p.init_slot = slot_idx; p.final_pool = rec_pool; p.final_slot = slot_idx;
  p.n_slots = n_slots;
  p.out = out; p.o_sb = int64_t(Hv) * dv; p.o_st = 0;
  p.z = z; p.z_rs = z_rs; p.norm_w = norm_w; p.eps = eps;
  p.B = n; p.T = 1; p.Hk = Hk; p.Hv = Hv; p.l2norm = 1; p.err = err_flag;
  if (dk == 128 && dv == 128)
    return dtype == GDN_BF16 ? launch_decode_layer<__nv_bfloat16>(p, workspace, as_stream(stream))
                             : launch_decode_layer<float>(p, workspace, as_stream(stream));
  return run_recurrent(p, dk, dv, dtype, as_stream(stream));
}
}  // namespace gdn

extern "C" int gdn_decode_layer(const void* mixed_qkv, int64_t mixed_rs, const void* z, const void* a,
                                const void* b, const float* A_log, const float* dt_bias, const void* conv_w,
                                const void* conv_b, void* conv_pool, float* rec_pool, const int32_t* slot_idx,
                                int64_t n_slots, const void* norm_w, float eps, void* out, int n, int Hk,
                                int Hv, int dk, int dv, int K, int conv_mode, void* workspace,
                                size_t workspace_bytes, int dtype, int32_t* err_flag, void* stream) {
  const int64_t hv = Hv > 0 ? Hv : 0;
  return gdn::decode_layer_impl("gdn_decode_layer", mixed_qkv, mixed_rs, z, hv * (dv > 0 ? dv : 0), a, hv, b, hv,
                                A_log, dt_bias, conv_w, conv_b, conv_pool, rec_pool, slot_idx, n_slots, norm_w, eps,
                                out, n, Hk, Hv, dk, dv, K, conv_mode, workspace, workspace_bytes, dtype, err_flag,
                                stream);
}

extern "C" int gdn_decode_layer_rows(const void* mixed_qkv, int64_t mixed_rs, const void* z, int64_t z_rs,
                                     const void* a, int64_t a_rs, const void* b, int64_t b_rs, const float* A_log,
                                     const float* dt_bias, const void* conv_w, const void* conv_b, void* conv_pool,
                                     float* rec_pool, const int32_t* slot_idx, int64_t n_slots, const void* norm_w,
                                     float eps, void* out, int n, int Hk, int Hv, int dk, int dv, int K,
                                     int conv_mode, void* workspace, size_t workspace_bytes, int dtype,
                                     int32_t* err_flag, void* stream) {
  return gdn::decode_layer_impl("gdn_decode_layer_rows", mixed_qkv, mixed_rs, z, z_rs, a, a_rs, b, b_rs, A_log,
                                dt_bias, conv_w, conv_b, conv_pool, rec_pool, slot_idx, n_slots, norm_w, eps, out, n,
                                Hk, Hv, dk, dv, K, conv_mode, workspace, workspace_bytes, dtype, err_flag, stream);
}
