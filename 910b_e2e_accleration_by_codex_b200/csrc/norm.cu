// a4. Gated RMSNorm: y = rnd(w * rnd(x * rsqrt(mean(x^2) + eps))) * silu(gate), one warp per row.
// Follows Qwen3_5RMSNormGated.forward (transformers modeling_qwen3_5.py:181-191): the statistics are
// fp32, the normalised row is rounded to the activation dtype before the weight multiply (which is
// itself a dtype op), and the gate product is fp32 with a final rounding.
#include "common.cuh"

namespace gdn {

template <typename T, bool VEC>
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(const T* __restrict__ x, int64_t x_rs,
                                                            const T* __restrict__ gate, int64_t g_rs,
                                                            const T* __restrict__ w, T* __restrict__ y,
                                                            int64_t y_rs, int64_t rows, int dim, float eps) {
  const int64_t row = (int64_t(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (row >= rows) return;
  const T* xr = x + row * x_rs;
  const T* gr = gate + row * g_rs;
  T* yr = y + row * y_rs;
  constexpr int G = 8;  // up to 8 groups of 4 per lane: dim <= 1024
  float4 xv[G];
  float ss = 0.f;
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < dim) {
      if (VEC) {
        xv[i] = ld4<T>(xr + c);
      } else {
        xv[i] = make_float4(Io<T>::ld(xr + c), Io<T>::ld(xr + c + 1), Io<T>::ld(xr + c + 2),
                            Io<T>::ld(xr + c + 3));
      }
      ss += xv[i].x * xv[i].x + xv[i].y * xv[i].y + xv[i].z * xv[i].z + xv[i].w * xv[i].w;
    }
  }
  ss = warp_sum(ss);
  const float r = 1.0f / sqrtf(ss / float(dim) + eps);
#pragma unroll
  for (int i = 0; i < G; ++i) {
    const int c = (i * 32 + lane) * 4;
    if (c < dim) {
      float4 gv, wv;
      if (VEC) {
        gv = ld4<T>(gr + c);
        wv = ld4<T>(w + c);
      } else {
        gv = make_float4(Io<T>::ld(gr + c), Io<T>::ld(gr + c + 1), Io<T>::ld(gr + c + 2),
                         Io<T>::ld(gr + c + 3));
        wv = make_float4(Io<T>::ld(w + c), Io<T>::ld(w + c + 1), Io<T>::ld(w + c + 2),
                         Io<T>::ld(w + c + 3));
      }
      float4 o;
      o.x = Io<T>::rnd(wv.x * Io<T>::rnd(xv[i].x * r)) * silu_f(gv.x);
      o.y = Io<T>::rnd(wv.y * Io<T>::rnd(xv[i].y * r)) * silu_f(gv.y);
      o.z = Io<T>::rnd(wv.z * Io<T>::rnd(xv[i].z * r)) * silu_f(gv.z);
      o.w = Io<T>::rnd(wv.w * Io<T>::rnd(xv[i].w * r)) * silu_f(gv.w);
      if (VEC) {
        st4<T>(yr + c, o);
      } else {
        Io<T>::st(yr + c, o.x);
        Io<T>::st(yr + c + 1, o.y);
        Io<T>::st(yr + c + 2, o.z);
        Io<T>::st(yr + c + 3, o.w);
      }
    }
  }
}

template <typename T>
static int launch_norm(const void* x, int64_t x_rs, const void* gate, int64_t g_rs, const void* w,
                       void* y, int64_t y_rs, int64_t rows, int dim, float eps, cudaStream_t s) {
  const size_t vb = 4 * sizeof(T);
  const bool vec = aligned(x, vb) && aligned(gate, vb) && aligned(w, vb) && aligned(y, vb) &&
                   (x_rs % 4 == 0) && (g_rs % 4 == 0) && (y_rs % 4 == 0);
  const int threads = 256;
  const int64_t blocks = (rows * 32 + threads - 1) / threads;
  if (vec)
    gated_rmsnorm_kernel<T, true><<<dim3(unsigned(blocks)), threads, 0, s>>>(
        (const T*)x, x_rs, (const T*)gate, g_rs, (const T*)w, (T*)y, y_rs, rows, dim, eps);
  else
    gated_rmsnorm_kernel<T, false><<<dim3(unsigned(blocks)), threads, 0, s>>>(
        (const T*)x, x_rs, (const T*)gate, g_rs, (const T*)w, (T*)y, y_rs, rows, dim, eps);
  return check_launch("gdn_gated_rmsnorm");
}

// Layer RMSNorm, Qwen3_5RMSNorm.forward (transformers modeling_qwen3_5.py): y = rnd(x * rsqrt(mean(x^2)
// + eps) * (1 + w)) with fp32 statistics and products and one final rounding -- the norm the reference
// replaces with npu_rms_norm (src/cb_engine.py:62-63, 70-71).  One CTA of 128 threads per row
// (dim <= 8192); thread t holds the 16-byte groups t, t + 128, ... of the row in registers.
template <typename T, bool VEC>
__global__ void __launch_bounds__(128) rmsnorm_kernel(const T* __restrict__ x, int64_t x_rs, const T* __restrict__ w,
                                                      T* __restrict__ y, int64_t y_rs, int dim, float eps) {
  constexpr int VW = 16 / int(sizeof(T));  // elements per group
  constexpr int NV = 8192 / (128 * VW);    // groups per thread at the largest dim
  __shared__ float red[4];
  const int tid = threadIdx.x;
  const T* xr = x + int64_t(blockIdx.x) * x_rs;
  T* yr = y + int64_t(blockIdx.x) * y_rs;
  float xv[NV][VW];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int c = (v * 128 + tid) * VW;
    if (c < dim) {
      if (VEC) {
        const uint4 u = *reinterpret_cast<const uint4*>(xr + c);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int j = 0; j < VW; ++j) xv[v][j] = Io<T>::ld(e + j);
      } else {
#pragma unroll
        for (int j = 0; j < VW; ++j) xv[v][j] = c + j < dim ? Io<T>::ld(xr + c + j) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < VW; ++j) ss += xv[v][j] * xv[v][j];
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  const float r = 1.0f / sqrtf((red[0] + red[1] + red[2] + red[3]) / float(dim) + eps);
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int c = (v * 128 + tid) * VW;
    if (c < dim) {
#pragma unroll
      for (int j = 0; j < VW; ++j)
        if (VEC || c + j < dim) Io<T>::st(yr + c + j, (xv[v][j] * r) * (1.0f + Io<T>::ld(w + c + j)));
    }
  }
}

template <typename T>
static int launch_rmsnorm(const void* x, int64_t x_rs, const void* w, void* y, int64_t y_rs, int64_t rows, int dim,
                          float eps, cudaStream_t s) {
  constexpr int VW = 16 / int(sizeof(T));
  const bool vec = aligned(x, 16) && aligned(y, 16) && dim % VW == 0 && x_rs % VW == 0 && y_rs % VW == 0;
  if (vec)
    rmsnorm_kernel<T, true><<<dim3(unsigned(rows)), 128, 0, s>>>((const T*)x, x_rs, (const T*)w, (T*)y, y_rs, dim, eps);
  else
    rmsnorm_kernel<T, false><<<dim3(unsigned(rows)), 128, 0, s>>>((const T*)x, x_rs, (const T*)w, (T*)y, y_rs, dim, eps);
  return check_launch("gdn_rmsnorm");
}

}  // namespace gdn

extern "C" int gdn_rmsnorm(const void* x, int64_t x_rs, const void* weight, void* y, int64_t y_rs, int64_t rows,
                           int dim, float eps, int dtype, void* stream) {
  using namespace gdn;
  if (rows < 0 || dim <= 0) return fail(GDN_ERR_ARG, "gdn_rmsnorm: rows=%lld dim=%d", (long long)rows, dim);
  if (rows == 0) return GDN_OK;
  if (!x || !weight || !y) return fail(GDN_ERR_ARG, "gdn_rmsnorm: null pointer");
  if (dim > 8192) return fail(GDN_ERR_SHAPE, "gdn_rmsnorm: dim=%d (<= 8192)", dim);
  if (rows > 0x7fffffffLL) return fail(GDN_ERR_ARG, "gdn_rmsnorm: rows too large");
  cudaStream_t s = as_stream(stream);
  if (dtype == GDN_BF16) return launch_rmsnorm<__nv_bfloat16>(x, x_rs, weight, y, y_rs, rows, dim, eps, s);
  if (dtype == GDN_F32) return launch_rmsnorm<float>(x, x_rs, weight, y, y_rs, rows, dim, eps, s);
  return fail(GDN_ERR_DTYPE, "gdn_rmsnorm: dtype %d", dtype);
}

extern "C" int gdn_gated_rmsnorm(const void* x, int64_t x_rs, const void* gate, int64_t g_rs,
                                 const void* weight, void* y, int64_t y_rs, int64_t rows, int dim,
                                 float eps, int dtype, void* stream) {
  using namespace gdn;
  if (rows < 0 || dim <= 0) return fail(GDN_ERR_ARG, "gdn_gated_rmsnorm: rows=%lld dim=%d", (long long)rows, dim);
  if (rows == 0) return GDN_OK;
  if (!x || !gate || !weight || !y) return fail(GDN_ERR_ARG, "gdn_gated_rmsnorm: null pointer");
  if (dim % 4 != 0 || dim > 1024) return fail(GDN_ERR_SHAPE, "gdn_gated_rmsnorm: dim=%d (need %%4==0, <=1024)", dim);
  if (rows > (int64_t(1) << 36)) return fail(GDN_ERR_ARG, "gdn_gated_rmsnorm: rows too large");
  cudaStream_t s = as_stream(stream);
  if (dtype == GDN_BF16) return launch_norm<__nv_bfloat16>(x, x_rs, gate, g_rs, weight, y, y_rs, rows, dim, eps, s);
  if (dtype == GDN_F32) return launch_norm<float>(x, x_rs, gate, g_rs, weight, y, y_rs, rows, dim, eps, s);
  return fail(GDN_ERR_DTYPE, "gdn_gated_rmsnorm: dtype %d", dtype);
}
