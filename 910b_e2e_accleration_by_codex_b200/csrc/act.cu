// The MLP activation of the decode step in one kernel: out = act_fn(gate) * up with gate and up the
// two halves of the fused gate|up projection (Qwen3_5MLP.forward, transformers modeling_qwen3_5.py:
// down_proj(act_fn(gate_proj(x)) * up_proj(x)), act_fn = SiLU).  torch runs it as two bf16 ops --
// silu (fp32 x / (1 + exp(-x)), rounded) then the product (fp32, rounded) -- and so does this
// kernel, in registers: out = bf16(bf16(silu(gate)) * up), bit for bit.
#include "common.cuh"

namespace gdn {

__global__ void __launch_bounds__(256) silu_mul_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_rs, int inter,
                                                       __nv_bfloat16* __restrict__ out, int64_t out_rs,
                                                       int64_t rows) {
  const int groups = inter / 8;
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= rows * groups) return;
  const int64_t r = gid / groups;
  const int c = int(gid - r * groups) * 8;
  const __nv_bfloat16* yr = y + r * y_rs;
  const uint4 gu = *reinterpret_cast<const uint4*>(yr + c);
  const uint4 uu = *reinterpret_cast<const uint4*>(yr + inter + c);
  const uint32_t g[4] = {gu.x, gu.y, gu.z, gu.w}, u[4] = {uu.x, uu.y, uu.z, uu.w};
  uint32_t o[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float g0 = __uint_as_float(g[i] << 16), g1 = __uint_as_float(g[i] & 0xffff0000u);
    const float u0 = __uint_as_float(u[i] << 16), u1 = __uint_as_float(u[i] & 0xffff0000u);
    const float s0 = __bfloat162float(__float2bfloat16_rn(silu_f(g0)));
    const float s1 = __bfloat162float(__float2bfloat16_rn(silu_f(g1)));
    const __nv_bfloat162 p = __floats2bfloat162_rn(s0 * u0, s1 * u1);
    o[i] = *reinterpret_cast<const uint32_t*>(&p);
  }
  *reinterpret_cast<uint4*>(out + r * out_rs + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace gdn

extern "C" int gdn_silu_mul(const void* y, int64_t y_rs, int inter, void* out, int64_t out_rs, int64_t rows, int dtype,
                            void* stream) {
  using namespace gdn;
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_silu_mul: dtype %d (bf16 only)", dtype);
  if (rows < 0 || inter < 8 || inter % 8) return fail(GDN_ERR_ARG, "gdn_silu_mul: rows %lld, inter %d (multiple of 8)",
                                                     (long long)rows, inter);
  if (rows == 0) return GDN_OK;
  if (!y || !out || !aligned(y, 16) || !aligned(out, 16) || y_rs % 8 || out_rs % 8 || y_rs < 2 * int64_t(inter) ||
      out_rs < inter)
    return fail(GDN_ERR_ARG, "gdn_silu_mul: 16-byte aligned rows with strides that are multiples of 8 needed");
  const int64_t total = rows * (inter / 8);
  if (total > (int64_t(1) << 40)) return fail(GDN_ERR_ARG, "gdn_silu_mul: too large");
  silu_mul_kernel<<<unsigned((total + 255) / 256), 256, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), y_rs, inter, static_cast<__nv_bfloat16*>(out), out_rs, rows);
  return check_launch("gdn_silu_mul");
}
