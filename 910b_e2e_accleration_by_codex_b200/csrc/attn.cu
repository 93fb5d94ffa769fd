// Slot-indexed full-attention decode over the engine's KV pool: the decode attention of the hybrid
// model's attention layers, CBEngine._attn (src/cb_engine.py:295-316).  One call per layer does what
// the reference does with two index_copy_ writes of the new K/V rows, a masked SDPA over a
// 512-token bucket and the sigmoid output gate:
//
//   attn_decode_kernel   CTA per (entry b, kv head j, split s of 128 positions): writes entry b's new
//                        K/V row of head j at position pos[b] of pool row slot[b] (the split that
//                        holds pos[b]), then for the g = Hq / kvh query heads of head j (kv-major
//                        order, as the reference's reshape) runs an fp32 online softmax over
//                        positions [128 s, min(128 s + 128, pos[b] + 1)) and writes the split's
//                        max, exp-sum and exp-weighted V sums to the workspace.
//   attn_combine_kernel  CTA per (entry, query head), thread per dim: merges the splits, rounds the
//                        attention output to the activation dtype, multiplies by rnd(sigmoid(gate))
//                        and rounds (the reference's bf16 SDPA output times torch.sigmoid(gate)).
#include "common.cuh"

namespace gdn {
namespace attn {

constexpr int kPos = 128;    // positions per split (one per thread)
constexpr int kMaxHd = 256;  // head dim
constexpr int kMaxG = 8;     // query heads per kv head

struct Params {
  const __nv_bfloat16* q;      // [n, Hq, hd]
  const __nv_bfloat16* k_new;  // [n, kvh, hd]
  const __nv_bfloat16* v_new;
  __nv_bfloat16* kv_k;         // [n_slots, kvh, T, hd]
  __nv_bfloat16* kv_v;
  const int32_t* slot;         // [n]
  const int32_t* pos;          // [n]
  const __nv_bfloat16* gate;   // [n, Hq, hd] or null
  __nv_bfloat16* out;          // [n, Hq, hd]
  float* ws;                   // [n, Hq, S, hd + 2]
  int n, Hq, kvh, hd, T, S;
  int64_t n_slots;
  float scale;
  int32_t* err;
};

__device__ __forceinline__ void unpack8(const uint4& u, float* f) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    f[2 * i] = __uint_as_float(w[i] << 16);
    f[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Warp w streams the split's positions in groups of kU = 4: group i holds positions
// t0 + (i * kW + w) * kU + u.  Lane l holds dims [8 l, 8 l + 8) of the G query rows (scaled) and
// of its running outputs; it loads the group's kU 16-byte K and V chunks at once (a warp reads
// whole 512-byte rows), reduces the G x kU scores across the warp, and applies one online-softmax
// rescale per group.  The four warps then merge in shared memory into the split's (max, exp-sum,
// exp-weighted V sums).
template <int G>
__global__ void __launch_bounds__(kPos) attn_decode_kernel(Params p) {
  constexpr int kW = kPos / 32, kU = 4;
  __shared__ float s_m[kW][G], s_l[kW][G];
  __shared__ float s_acc[kW][G][kMaxHd];
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int s = blockIdx.x % p.S;
  const int j = (blockIdx.x / p.S) % p.kvh;
  const int b = blockIdx.x / (p.S * p.kvh);
  const int hd = p.hd;
  const int64_t slot = p.slot[b];
  const int pos = p.pos[b];
  float* ws = p.ws + ((int64_t(b) * p.Hq + int64_t(j) * G) * p.S + s) * (hd + 2);  // head j*G, split s
  const int64_t ws_head = int64_t(p.S) * (hd + 2);                                  // next query head
  if (slot < 0 || slot >= p.n_slots || pos < 0 || pos >= p.T || pos >= p.S * kPos) {  // bad entry: record it
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    if (tid < G) {
      ws[tid * ws_head + hd] = -INFINITY;
      ws[tid * ws_head + hd + 1] = 0.f;
    }
    return;
  }
  const int t0 = s * kPos;
  const int t1 = min(t0 + kPos, pos + 1);
  const int64_t head_base = (slot * p.kvh + j) * int64_t(p.T) * hd;
  __nv_bfloat16* Kp = p.kv_k + head_base;
  __nv_bfloat16* Vp = p.kv_v + head_base;
  const __nv_bfloat16* kn = p.k_new + (int64_t(b) * p.kvh + j) * hd;
  const __nv_bfloat16* vn = p.v_new + (int64_t(b) * p.kvh + j) * hd;
  // the split that holds pos writes the new row (its own reads of that position use k_new / v_new)
  if (pos >= t0 && pos < t0 + kPos)
    for (int d = tid; d < hd; d += kPos) {
      Kp[int64_t(pos) * hd + d] = kn[d];
      Vp[int64_t(pos) * hd + d] = vn[d];
    }
  const bool dl = lane < hd / 8;  // this lane holds dims 8 lane .. 8 lane + 7
  float qv[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (dl) {
      const uint4 u = reinterpret_cast<const uint4*>(p.q + (int64_t(b) * p.Hq + j * G + h) * hd)[lane];
      unpack8(u, qv[h]);
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[h][e] *= p.scale;
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) qv[h][e] = 0.f;
    }
  }
  float m[G], l[G], acc[G][8];
#pragma unroll
  for (int h = 0; h < G; ++h) {
    m[h] = -INFINITY;
    l[h] = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[h][e] = 0.f;
  }
  for (int tb = t0 + warp * kU; tb < t1; tb += kW * kU) {
    uint4 ku[kU], vu[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int t = tb + u;
      ku[u] = vu[u] = make_uint4(0, 0, 0, 0);
      if (t < t1 && dl) {
        ku[u] = reinterpret_cast<const uint4*>(t == pos ? kn : Kp + int64_t(t) * hd)[lane];
        vu[u] = reinterpret_cast<const uint4*>(t == pos ? vn : Vp + int64_t(t) * hd)[lane];
      }
    }
    float sc[G][kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      float kf[8];
      unpack8(ku[u], kf);
#pragma unroll
      for (int h = 0; h < G; ++h) {
        float a = 0.f;
#pragma unroll
        for (int e = 0; e < 8; ++e) a = fmaf(qv[h][e], kf[e], a);
        sc[h][u] = a;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1)
#pragma unroll
      for (int h = 0; h < G; ++h)
#pragma unroll
        for (int u = 0; u < kU; ++u) sc[h][u] += __shfl_xor_sync(0xffffffffu, sc[h][u], o);
#pragma unroll
    for (int h = 0; h < G; ++h) {
      float mn = m[h];
#pragma unroll
      for (int u = 0; u < kU; ++u)
        if (tb + u < t1) mn = fmaxf(mn, sc[h][u]);
      const float f = expf(m[h] - mn);
      l[h] *= f;
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[h][e] *= f;
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        if (tb + u >= t1) continue;
        const float pe = expf(sc[h][u] - mn);
        float vf[8];
        unpack8(vu[u], vf);
        l[h] += pe;
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[h][e] = fmaf(pe, vf[e], acc[h][e]);
      }
      m[h] = mn;
    }
  }
  // merge the warps
#pragma unroll
  for (int h = 0; h < G; ++h) {
    if (lane == 0) {
      s_m[warp][h] = m[h];
      s_l[warp][h] = l[h];
    }
    if (dl) {
#pragma unroll
      for (int e = 0; e < 8; ++e) s_acc[warp][h][8 * lane + e] = acc[h][e];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * hd; i += kPos) {
    const int h = i / hd, d = i - h * hd;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kW; ++w) M = fmaxf(M, s_m[w][h]);
    float a = 0.f, L = 0.f;
#pragma unroll
    for (int w = 0; w < kW; ++w) {
      if (s_m[w][h] == -INFINITY) continue;
      const float f = expf(s_m[w][h] - M);
      a = fmaf(f, s_acc[w][h][d], a);
      L = fmaf(f, s_l[w][h], L);
    }
    ws[h * ws_head + d] = a;
    if (d == 0) {
      ws[h * ws_head + hd] = M;
      ws[h * ws_head + hd + 1] = L;
    }
  }
}

__global__ void __launch_bounds__(kMaxHd) attn_combine_kernel(Params p) {
  const int bh = blockIdx.x;  // entry * Hq + query head
  const int d = threadIdx.x;
  if (d >= p.hd) return;
  const int hd = p.hd;
  const float* w = p.ws + int64_t(bh) * p.S * (hd + 2);
  float M = -INFINITY;
  for (int s = 0; s < p.S; ++s) M = fmaxf(M, w[s * (hd + 2) + hd]);
  float num = 0.f, den = 0.f;
  for (int s = 0; s < p.S; ++s) {
    const float m = w[s * (hd + 2) + hd];
    if (m == -INFINITY) continue;
    const float f = expf(m - M);
    num = fmaf(f, w[s * (hd + 2) + d], num);
    den = fmaf(f, w[s * (hd + 2) + hd + 1], den);
  }
  float o = den > 0.f ? Io<__nv_bfloat16>::rnd(num / den) : 0.f;
  if (p.gate) {
    const float gt = __bfloat162float(p.gate[int64_t(bh) * hd + d]);
    o = o * Io<__nv_bfloat16>::rnd(1.0f / (1.0f + expf(-gt)));
  }
  p.out[int64_t(bh) * hd + d] = __float2bfloat16_rn(o);
}

}  // namespace attn
}  // namespace gdn

using namespace gdn;

extern "C" size_t gdn_attn_decode_workspace_size(int n, int Hq, int hd, int max_len) {
  if (n <= 0 || Hq <= 0 || hd <= 0 || max_len <= 0) return 0;
  const size_t S = (size_t(max_len) + attn::kPos - 1) / attn::kPos;
  return size_t(n) * size_t(Hq) * S * size_t(hd + 2) * sizeof(float);
}

extern "C" int gdn_attn_decode(const void* q, const void* k_new, const void* v_new, void* kv_k, void* kv_v,
                               int64_t n_slots, int T, const int32_t* slot_idx, const int32_t* pos, int max_len,
                               const void* gate, float scale, void* out, int n, int Hq, int kvh, int hd,
                               void* workspace, size_t workspace_bytes, int dtype, int32_t* err_flag,
                               void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_attn_decode: dtype %d (bf16 only)", dtype);
  if (n < 0) return fail(GDN_ERR_ARG, "gdn_attn_decode: n=%d", n);
  if (n == 0) return GDN_OK;
  if (!q || !k_new || !v_new || !kv_k || !kv_v || !slot_idx || !pos || !out || !workspace)
    return fail(GDN_ERR_ARG, "gdn_attn_decode: null pointer");
  if (kvh <= 0 || Hq % kvh != 0 || Hq / kvh > attn::kMaxG || hd <= 0 || hd > attn::kMaxHd || hd % 8 != 0)
    return fail(GDN_ERR_SHAPE, "gdn_attn_decode: Hq=%d kvh=%d hd=%d (Hq/kvh <= %d, hd %% 8 == 0, hd <= %d)", Hq,
                kvh, hd, attn::kMaxG, attn::kMaxHd);
  if (T <= 0 || max_len <= 0 || max_len > T || n_slots < 1)
    return fail(GDN_ERR_ARG, "gdn_attn_decode: T=%d max_len=%d n_slots=%lld", T, max_len, (long long)n_slots);
  const size_t need = gdn_attn_decode_workspace_size(n, Hq, hd, max_len);
  if (workspace_bytes < need)
    return fail(GDN_ERR_WORKSPACE, "gdn_attn_decode: workspace %zu bytes < %zu", workspace_bytes, need);
  if (!aligned(q, 16) || !aligned(k_new, 16) || !aligned(kv_k, 16) || !aligned(workspace, 16))
    return fail(GDN_ERR_ARG, "gdn_attn_decode: q, k_new, kv_k and the workspace must be 16-byte aligned");
  attn::Params p{};
  p.q = static_cast<const __nv_bfloat16*>(q);
  p.k_new = static_cast<const __nv_bfloat16*>(k_new);
  p.v_new = static_cast<const __nv_bfloat16*>(v_new);
  p.kv_k = static_cast<__nv_bfloat16*>(kv_k);
  p.kv_v = static_cast<__nv_bfloat16*>(kv_v);
  p.slot = slot_idx;
  p.pos = pos;
  p.gate = static_cast<const __nv_bfloat16*>(gate);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.ws = static_cast<float*>(workspace);
  p.n = n;
  p.Hq = Hq;
  p.kvh = kvh;
  p.hd = hd;
  p.T = T;
  p.S = (max_len + attn::kPos - 1) / attn::kPos;
  p.n_slots = n_slots;
  p.scale = scale;
  p.err = err_flag;
  cudaStream_t s = as_stream(stream);
  const unsigned grid = unsigned(int64_t(n) * kvh * p.S);
  switch (Hq / kvh) {
    case 1: attn::attn_decode_kernel<1><<<grid, attn::kPos, 0, s>>>(p); break;
    case 2: attn::attn_decode_kernel<2><<<grid, attn::kPos, 0, s>>>(p); break;
    case 3: attn::attn_decode_kernel<3><<<grid, attn::kPos, 0, s>>>(p); break;
    case 4: attn::attn_decode_kernel<4><<<grid, attn::kPos, 0, s>>>(p); break;
    case 5: attn::attn_decode_kernel<5><<<grid, attn::kPos, 0, s>>>(p); break;
    case 6: attn::attn_decode_kernel<6><<<grid, attn::kPos, 0, s>>>(p); break;
    case 7: attn::attn_decode_kernel<7><<<grid, attn::kPos, 0, s>>>(p); break;
    default: attn::attn_decode_kernel<8><<<grid, attn::kPos, 0, s>>>(p); break;
  }
  int rc = check_launch("gdn_attn_decode");
  if (rc) return rc;
  attn::attn_combine_kernel<<<unsigned(int64_t(n) * Hq), attn::kMaxHd, 0, s>>>(p);
  return check_launch("gdn_attn_decode (combine)");
}

// ---------------------------------------------------------------------------------------------
// The attention layer's decode preamble in one kernel (CBEngine._attn before the attention itself,
// src/cb_engine.py:295-316, with HF's Qwen3_5Attention pieces): from one token row of the fused
// q|gate, k, v projection it writes the four contiguous inputs of gdn_attn_decode:
//   q    = rotary(q_norm(q_h))   per query head   (q_h = y[2 hd h : 2 hd h + hd])
//   gate = y[2 hd h + hd : 2 hd (h + 1)]          (the chunk of the q|gate view)
//   k    = rotary(k_norm(k_h))   per kv head      (k_h = y[nq + hd h : ...])
//   v    = y[nq + nk + hd h : ...]
// q_norm / k_norm are Qwen3_5RMSNorm over head_dim with the element order, reduction order and
// rounding of gdn_rmsnorm (one warp per head; lane t holds elements 8t .. 8t + 7), and rotary is
// apply_rotary_pos_emb on the first rd dims with every bf16 rounding of the torch ops:
//   out[i] = bf16(bf16(x[i] cos[i]) + bf16(rot[i] sin[i])),  rot = cat(-x[rd/2:rd], x[:rd/2]),
// dims rd.. passed through.  So the result equals the sequence of torch ops bit for bit.
// One warp per (token, head) over Hq + kvh heads; another warp per head copies v and gate.
namespace gdn {
namespace attn {

struct PrepParams {
  const __nv_bfloat16* y;
  int64_t y_rs;
  const __nv_bfloat16* qw;
  const __nv_bfloat16* kw;
  const __nv_bfloat16* cos;
  const __nv_bfloat16* sin;
  int64_t cs_rs;
  __nv_bfloat16 *q, *k, *v, *gate;
  int n, Hq, kvh, hd, rd;
  float eps;
};

__device__ __forceinline__ void unpack8f(const uint4& u, float* x) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ float r16(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }
__device__ __forceinline__ uint4 pack8f(const float* a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 t = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&t);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(128) attn_prep_kernel(const PrepParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t task = int64_t(blockIdx.x) * 4 + (threadIdx.x >> 5);
  const int heads = p.Hq + p.kvh;
  const int64_t norm_tasks = int64_t(p.n) * heads;
  const int groups = p.hd / 8;  // 8-element groups per head (<= 32)
  if (task < norm_tasks) {
    const int j = int(task / heads), h = int(task - int64_t(j) * heads);
    const bool isq = h < p.Hq;
    const int hh = isq ? h : h - p.Hq;
    const __nv_bfloat16* src = p.y + int64_t(j) * p.y_rs +
                               (isq ? int64_t(2) * p.hd * hh : int64_t(2) * p.hd * p.Hq + int64_t(p.hd) * hh);
    const __nv_bfloat16* w = isq ? p.qw : p.kw;
    float x[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f}, wv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    float ss = 0.f;
    if (lane < groups) {
      unpack8f(*reinterpret_cast<const uint4*>(src + lane * 8), x);
      unpack8f(*reinterpret_cast<const uint4*>(w + lane * 8), wv);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += x[i] * x[i];
    }
    ss = warp_sum(ss);
    const float r = 1.0f / sqrtf(ss / float(p.hd) + p.eps);
    float xn[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) xn[i] = r16((x[i] * r) * (1.0f + wv[i]));
    // rotary on dims [0, rd): the rotate_half partner of element i sits rd/16 lanes away
    const int half = p.rd / 16;
    float other[8];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int src_lane = lane < half ? lane + half : lane - half;
      other[i] = __shfl_sync(0xffffffffu, xn[i], src_lane < 32 ? src_lane : lane);
    }
    float out[8];
    if (lane * 8 < p.rd) {
      const __nv_bfloat16* cs = p.cos + int64_t(j) * p.cs_rs + lane * 8;
      const __nv_bfloat16* sn = p.sin + int64_t(j) * p.cs_rs + lane * 8;
      float c[8], s[8];
      unpack8f(*reinterpret_cast<const uint4*>(cs), c);
      unpack8f(*reinterpret_cast<const uint4*>(sn), s);
      const bool first = lane < half;  // rot = -x[i + rd/2] for i < rd/2, x[i - rd/2] above
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float rot = first ? -other[i] : other[i];
        out[i] = r16(r16(xn[i] * c[i]) + r16(rot * s[i]));
      }
    } else {
#pragma unroll
      for (int i = 0; i < 8; ++i) out[i] = xn[i];
    }
    if (lane < groups) {
      __nv_bfloat16* dst = (isq ? p.q + (int64_t(j) * p.Hq + hh) * p.hd : p.k + (int64_t(j) * p.kvh + hh) * p.hd);
      *reinterpret_cast<uint4*>(dst + lane * 8) = pack8f(out);
    }
    return;
  }
  // copies: v heads and gate heads
  const int64_t c = task - norm_tasks;
  if (c >= norm_tasks || lane >= groups) return;
  const int j = int(c / heads), h = int(c - int64_t(j) * heads);
  const __nv_bfloat16* row = p.y + int64_t(j) * p.y_rs;
  if (h < p.Hq) {
    const uint4 u = *reinterpret_cast<const uint4*>(row + int64_t(2) * p.hd * h + p.hd + lane * 8);
    *reinterpret_cast<uint4*>(p.gate + (int64_t(j) * p.Hq + h) * p.hd + lane * 8) = u;
  } else {
    const int hh = h - p.Hq;
    const uint4 u = *reinterpret_cast<const uint4*>(row + int64_t(2) * p.hd * p.Hq + int64_t(p.hd) * p.kvh +
                                                    int64_t(p.hd) * hh + lane * 8);
    *reinterpret_cast<uint4*>(p.v + (int64_t(j) * p.kvh + hh) * p.hd + lane * 8) = u;
  }
}

}  // namespace attn
}  // namespace gdn

extern "C" int gdn_attn_decode_prep(const void* y, int64_t y_rs, const void* q_norm_w, const void* k_norm_w, float eps,
                                    const void* cos, const void* sin, int64_t cs_rs, int rd, void* q, void* k, void* v,
                                    void* gate, int n, int Hq, int kvh, int hd, int dtype, void* stream) {
  using namespace gdn;
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_attn_decode_prep: dtype %d (bf16 only)", dtype);
  if (n < 0 || Hq < 1 || kvh < 1 || hd < 8 || hd > 256 || hd % 8 || rd < 0 || rd > hd || rd % 16 || (rd == 0))
    return fail(GDN_ERR_ARG, "gdn_attn_decode_prep: Hq %d kvh %d hd %d rd %d (hd a multiple of 8 <= 256; rd a "
                             "multiple of 16 in 16..hd)", Hq, kvh, hd, rd);
  if (n == 0) return GDN_OK;
  const void* ptrs[] = {y, q_norm_w, k_norm_w, cos, sin, q, k, v, gate};
  for (const void* ptr : ptrs)
    if (!ptr || !aligned(ptr, 16)) return fail(GDN_ERR_ARG, "gdn_attn_decode_prep: null or misaligned pointer");
  if (y_rs % 8 || cs_rs % 8 || y_rs < int64_t(2) * Hq * hd + int64_t(2) * kvh * hd || cs_rs < rd)
    return fail(GDN_ERR_ARG, "gdn_attn_decode_prep: row strides");
  attn::PrepParams p{};
  p.y = static_cast<const __nv_bfloat16*>(y);
  p.y_rs = y_rs;
  p.qw = static_cast<const __nv_bfloat16*>(q_norm_w);
  p.kw = static_cast<const __nv_bfloat16*>(k_norm_w);
  p.cos = static_cast<const __nv_bfloat16*>(cos);
  p.sin = static_cast<const __nv_bfloat16*>(sin);
  p.cs_rs = cs_rs;
  p.q = static_cast<__nv_bfloat16*>(q);
  p.k = static_cast<__nv_bfloat16*>(k);
  p.v = static_cast<__nv_bfloat16*>(v);
  p.gate = static_cast<__nv_bfloat16*>(gate);
  p.n = n;
  p.Hq = Hq;
  p.kvh = kvh;
  p.hd = hd;
  p.rd = rd;
  p.eps = eps;
  const int64_t tasks = 2 * int64_t(n) * (Hq + kvh);  // norm + rotary tasks, then copy tasks
  attn::attn_prep_kernel<<<unsigned((tasks + 3) / 4), 128, 0, as_stream(stream)>>>(p);
  return check_launch("gdn_attn_decode_prep");
}
