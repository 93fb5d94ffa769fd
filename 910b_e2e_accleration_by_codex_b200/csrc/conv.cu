// a3 / prefill conv.  Depthwise causal conv1d (kernel K) with a per-slot conv state holding the
// last K inputs (transformers' Qwen3.5 cache layout: K entries, not K-1).
//
//  * gdn_conv_update: decode form, one thread per (sequence, channel), T new tokens.  Follows
//    elem_conv_update (src/cb_engine.py:43-51) in GDN_CONV_ELEM mode and torch_causal_conv1d_update
//    (transformers modeling_qwen3_5.py:210-226) in GDN_CONV_HF mode.  The window is kept in
//    registers; the state row of the slot is read once and written once (in place).
//  * gdn_prefill_conv: packed varlen prefill, one thread per channel walking the sequence's tokens,
//    one CTA per (sequence, channel block); the first K-1 outputs see the slot's previous inputs
//    (src/cb_tp.py:236-244) or zeros (transformers modeling_qwen3_5.py:463-474), and the last K
//    inputs go back to the slot (src/cb_tp.py:158-162, :260).
#include "common.cuh"

namespace gdn {

constexpr int kMaxK = 8;

// Shift the K-window left by one and append `xv` (fixed-size loops keep `win` in registers).
__device__ __forceinline__ void push_window(float* win, float xv, int K) {
#pragma unroll
  for (int j = 0; j < kMaxK - 1; ++j)
    if (j < K - 1) win[j] = win[j + 1];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j)
    if (j == K - 1) win[j] = xv;
}

template <typename T>
__device__ __forceinline__ float conv_tap_sum(const float* win, const float* wv, float bv, bool has_bias,
                                              int K, int mode) {
  if (mode == GDN_CONV_ELEM) {
    float acc = 0.f;
#pragma unroll
    for (int j = 0; j < kMaxK; ++j)
      if (j < K) acc += Io<T>::rnd(win[j] * wv[j]);
    float o = Io<T>::rnd(acc);
    if (has_bias) o = Io<T>::rnd(o + bv);
    return o;
  }
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxK; ++j)
    if (j < K) acc = fmaf(win[j], wv[j], acc);
  if (has_bias) acc += bv;
  return Io<T>::rnd(acc);
}

template <typename T>
__global__ void __launch_bounds__(256) conv_update_kernel(
    const T* __restrict__ x, int64_t xs_b, int64_t xs_c, int64_t xs_t, T* __restrict__ pool,
    const int32_t* __restrict__ slot_idx, int64_t n_slots, const T* __restrict__ w,
    const T* __restrict__ bias, T* __restrict__ y, int64_t ys_b, int64_t ys_c, int64_t ys_t, int B, int C,
    int T_, int K, int act, int mode, int32_t* err) {
  const int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (i >= int64_t(B) * C) return;
  const int b = int(i / C), c = int(i % C);
  const int64_t slot = slot_idx ? int64_t(slot_idx[b]) : int64_t(b);
  if (slot < 0 || slot >= n_slots) {
    if (err) atomicExch(err, 1);
    return;
  }
  T* st = pool + (slot * C + c) * K;
  float win[kMaxK], wv[kMaxK];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    win[j] = j < K ? Io<T>::ld(st + j) : 0.f;
    wv[j] = j < K ? Io<T>::ld(w + int64_t(c) * K + j) : 0.f;
  }
  const bool has_bias = bias != nullptr;
  const float bv = has_bias ? Io<T>::ld(bias + c) : 0.f;
  for (int t = 0; t < T_; ++t) {
    push_window(win, Io<T>::ld(x + b * xs_b + c * xs_c + t * xs_t), K);
    float o = conv_tap_sum<T>(win, wv, bv, has_bias, K, mode);
    if (act) o = Io<T>::rnd(silu_f(o));
    Io<T>::st(y + b * ys_b + c * ys_c + t * ys_t, o);
  }
#pragma unroll
  for (int j = 0; j < kMaxK; ++j)
    if (j < K) Io<T>::st(st + j, win[j]);
}

template <typename T>
__global__ void __launch_bounds__(128) prefill_conv_kernel(
    const T* __restrict__ x, int64_t xs_t, T* __restrict__ y, int64_t ys_t,
    const int32_t* __restrict__ cu, T* __restrict__ pool, const int32_t* __restrict__ slot_idx,
    const int32_t* __restrict__ use_init, int64_t n_slots, const T* __restrict__ w,
    const T* __restrict__ bias, int C, int K, int act, int32_t* err) {
  const int b = blockIdx.y;
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const int64_t s = cu[b], e = cu[b + 1];
  const int64_t slot = slot_idx ? int64_t(slot_idx[b]) : int64_t(b);
  bool slot_ok = pool != nullptr;
  if (pool && (slot < 0 || slot >= n_slots)) {
    if (err) atomicExch(err, 1);
    slot_ok = false;
  }
  float win[kMaxK], wv[kMaxK];
  const bool from_pool = slot_ok && use_init && use_init[b];
#pragma unroll
  for (int j = 0; j < kMaxK; ++j) {
    win[j] = (j < K && from_pool) ? Io<T>::ld(pool + (slot * C + c) * K + j) : 0.f;
    wv[j] = j < K ? Io<T>::ld(w + int64_t(c) * K + j) : 0.f;
  }
  const bool has_bias = bias != nullptr;
  const float bv = has_bias ? Io<T>::ld(bias + c) : 0.f;
  constexpr int U = 8;
  int64_t t = s;
  for (; t + U <= e; t += U) {
    float xin[U];
#pragma unroll
    for (int u = 0; u < U; ++u) xin[u] = Io<T>::ld(x + (t + u) * xs_t + c);
#pragma unroll
    for (int u = 0; u < U; ++u) {
      push_window(win, xin[u], K);
      float o = conv_tap_sum<T>(win, wv, bv, has_bias, K, GDN_CONV_HF);
      if (act) o = Io<T>::rnd(silu_f(o));
      Io<T>::st(y + (t + u) * ys_t + c, o);
    }
  }
  for (; t < e; ++t) {
    push_window(win, Io<T>::ld(x + t * xs_t + c), K);
    float o = conv_tap_sum<T>(win, wv, bv, has_bias, K, GDN_CONV_HF);
    if (act) o = Io<T>::rnd(silu_f(o));
    Io<T>::st(y + t * ys_t + c, o);
  }
  if (slot_ok) {
#pragma unroll
    for (int j = 0; j < kMaxK; ++j)
      if (j < K) Io<T>::st(pool + (slot * C + c) * K + j, win[j]);
  }
}

int launch_conv_update(const void* x, int64_t xs_b, int64_t xs_c, int64_t xs_t, void* pool,
                       const int32_t* slot_idx, int64_t n_slots, const void* w, const void* bias, void* y,
                       int64_t ys_b, int64_t ys_c, int64_t ys_t, int B, int C, int T, int K, int act,
                       int mode, int dtype, int32_t* err, cudaStream_t s) {
  const int threads = 256;
  const int64_t blocks = (int64_t(B) * C + threads - 1) / threads;
  if (dtype == GDN_BF16) {
    using E = __nv_bfloat16;
    conv_update_kernel<E><<<unsigned(blocks), threads, 0, s>>>(
        (const E*)x, xs_b, xs_c, xs_t, (E*)pool, slot_idx, n_slots, (const E*)w, (const E*)bias, (E*)y,
        ys_b, ys_c, ys_t, B, C, T, K, act, mode, err);
  } else {
    conv_update_kernel<float><<<unsigned(blocks), threads, 0, s>>>(
        (const float*)x, xs_b, xs_c, xs_t, (float*)pool, slot_idx, n_slots, (const float*)w,
        (const float*)bias, (float*)y, ys_b, ys_c, ys_t, B, C, T, K, act, mode, err);
  }
  return check_launch("gdn_conv_update");
}

}  // namespace gdn

extern "C" int gdn_conv_update(const void* x, int64_t xs_b, int64_t xs_c, int64_t xs_t, void* conv_pool,
                               const int32_t* slot_idx, int64_t n_slots, const void* weight,
                               const void* bias, void* y, int64_t ys_b, int64_t ys_c, int64_t ys_t, int B,
                               int C, int T, int K, int activation, int mode, int dtype, int32_t* err_flag,
                               void* stream) {
  using namespace gdn;
  if (B < 0 || C < 0 || T < 0) return fail(GDN_ERR_ARG, "gdn_conv_update: negative size");
  if (B == 0 || C == 0 || T == 0) return GDN_OK;
  if (!x || !conv_pool || !weight || !y) return fail(GDN_ERR_ARG, "gdn_conv_update: null pointer");
  if (K < 1 || K > kMaxK) return fail(GDN_ERR_SHAPE, "gdn_conv_update: K=%d (1..%d)", K, kMaxK);
  if (mode != GDN_CONV_HF && mode != GDN_CONV_ELEM) return fail(GDN_ERR_ARG, "gdn_conv_update: mode %d", mode);
  if (dtype != GDN_BF16 && dtype != GDN_F32) return fail(GDN_ERR_DTYPE, "gdn_conv_update: dtype %d", dtype);
  if (n_slots < 1) return fail(GDN_ERR_ARG, "gdn_conv_update: n_slots=%lld", (long long)n_slots);
  return launch_conv_update(x, xs_b, xs_c, xs_t, conv_pool, slot_idx, n_slots, weight, bias, y, ys_b, ys_c,
                            ys_t, B, C, T, K, activation, mode, dtype, err_flag, as_stream(stream));
}

extern "C" int gdn_prefill_conv(const void* x, int64_t xs_t, void* y, int64_t ys_t, const int32_t* cu_seqlens,
                                int B, void* conv_pool, const int32_t* slot_idx, const int32_t* use_initial,
                                int64_t n_slots, const void* weight, const void* bias, int C, int K,
                                int activation, int dtype, int32_t* err_flag, void* stream) {
  using namespace gdn;
  if (B < 0 || C < 0) return fail(GDN_ERR_ARG, "gdn_prefill_conv: negative size");
  if (B == 0 || C == 0) return GDN_OK;
  if (!x || !y || !cu_seqlens || !weight) return fail(GDN_ERR_ARG, "gdn_prefill_conv: null pointer");
  if (K < 1 || K > kMaxK) return fail(GDN_ERR_SHAPE, "gdn_prefill_conv: K=%d (1..%d)", K, kMaxK);
  if (conv_pool && n_slots < 1) return fail(GDN_ERR_ARG, "gdn_prefill_conv: n_slots=%lld", (long long)n_slots);
  if (B > 65535) return fail(GDN_ERR_ARG, "gdn_prefill_conv: B=%d > 65535", B);
  cudaStream_t s = as_stream(stream);
  const int threads = 128;
  dim3 grid((C + threads - 1) / threads, B);
  if (dtype == GDN_BF16) {
    using E = __nv_bfloat16;
    prefill_conv_kernel<E><<<grid, threads, 0, s>>>((const E*)x, xs_t, (E*)y, ys_t, cu_seqlens, (E*)conv_pool,
                                                     slot_idx, use_initial, n_slots, (const E*)weight,
                                                     (const E*)bias, C, K, activation, err_flag);
  } else if (dtype == GDN_F32) {
    prefill_conv_kernel<float><<<grid, threads, 0, s>>>((const float*)x, xs_t, (float*)y, ys_t, cu_seqlens,
                                                         (float*)conv_pool, slot_idx, use_initial, n_slots,
                                                         (const float*)weight, (const float*)bias, C, K,
                                                         activation, err_flag);
  } else {
    return fail(GDN_ERR_DTYPE, "gdn_prefill_conv: dtype %d", dtype);
  }
  return check_launch("gdn_prefill_conv");
}
