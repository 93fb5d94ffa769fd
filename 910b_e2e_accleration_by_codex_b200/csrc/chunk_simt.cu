// a1, fp32 path.  Chunked gated delta rule (chunk 64) on the CUDA cores, exact fp32 arithmetic.
//
// One CTA per (sequence, value head) walks the sequence chunk by chunk with the fp32 state S
// resident in shared memory.  Per chunk it follows fast_chunk_gated_delta_rule_v2
// (src/gdn_chunk_fast2.py:29-59) operation for operation:
//   gc = cumsum(g);  decay[i][j] = exp(gc_i - gc_j) (i >= j)
//   X = -((k*beta) k^T . decay) strictly lower;  T = (I - X)^-1 by the blocked inverse of
//       src/gdn_chunk_fast.py:21-62 (16x16 diagonal row recurrences, then pairwise merges
//       T21 = (B X21) A)
//   U = T (v*beta);  W = T (k*beta*exp(gc));  QK = (q k^T . decay) lower incl. diagonal
//   vn = U - W S;  o = (q*exp(gc)) S + QK vn;  S = S*exp(gc_last) + (k*exp(gc_last-gc))^T vn
// The last partial chunk is zero padded (k = v = g = beta = 0), exactly as F.pad does in the
// reference, so padded rows leave the state unchanged.  This kernel serves GDN_F32 (the
// reference's fp32 configuration); GDN_BF16 calls go to the tensor-core kernel.
#include "chunk.cuh"

namespace gdn {


constexpr int kC = 64;      // chunk length
constexpr int kNT = 256;    // threads per CTA

template <int D>
struct SimtSmem {
  static constexpr int LD = D + 1;   // padded row stride of [64][D] and [D][D] buffers
  static constexpr int LT = kC + 1;  // padded row stride of 64x64 buffers
  static constexpr int S_OFF = 0;
  static constexpr int Q_OFF = S_OFF + D * LD;
  static constexpr int K_OFF = Q_OFF + kC * LD;
  static constexpr int V_OFF = K_OFF + kC * LD;
  static constexpr int W_OFF = V_OFF + kC * LD;
  static constexpr int T_OFF = W_OFF + kC * LD;
  static constexpr int VEC_OFF = T_OFF + kC * LT;     // beta, gc, exp(gc), exp(gl-gc)
  static constexpr int FLOATS = VEC_OFF + 4 * kC + 4;
  static constexpr size_t BYTES = size_t(FLOATS) * 4;
};

// acc[TM][TN] = sum_k A(i,k) B(k,j) over a thread's register tile; rows i = ti + r*(M/TM),
// cols j = tj + c*(N/TN) (strided so a warp's B reads hit consecutive banks).
template <int M, int N, int KD, int TM, int TN, typename FA, typename FB>
__device__ __forceinline__ void tile_mm(float (&acc)[TM][TN], FA A, FB B, int tid) {
  constexpr int CJ = N / TN;
  const int ti = tid / CJ, tj = tid % CJ;
  constexpr int RI = M / TM;
#pragma unroll
  for (int r = 0; r < TM; ++r)
#pragma unroll
    for (int c = 0; c < TN; ++c) acc[r][c] = 0.f;
#pragma unroll 4
  for (int kk = 0; kk < KD; ++kk) {
    float a[TM], bb[TN];
#pragma unroll
    for (int r = 0; r < TM; ++r) a[r] = A(ti + r * RI, kk);
#pragma unroll
    for (int c = 0; c < TN; ++c) bb[c] = B(kk, tj + c * CJ);
#pragma unroll
    for (int r = 0; r < TM; ++r)
#pragma unroll
      for (int c = 0; c < TN; ++c) acc[r][c] = fmaf(a[r], bb[c], acc[r][c]);
  }
}

template <typename T, int D>
__global__ void __launch_bounds__(kNT, 1) chunk_simt_kernel(ChunkParams p) {
  using L = SimtSmem<D>;
  constexpr int LD = L::LD, LT = L::LT;
  extern __shared__ float sm[];
  float* S = sm + L::S_OFF;
  float* Qs = sm + L::Q_OFF;
  float* Ks = sm + L::K_OFF;
  float* Vs = sm + L::V_OFF;
  float* Ws = sm + L::W_OFF;
  float* Ts = sm + L::T_OFF;
  float* sb = sm + L::VEC_OFF;
  float* gc = sb + kC;
  float* egc = gc + kC;
  float* ekd = egc + kC;
  float* gscal = ekd + kC;  // [0] = exp(gc_last)

  const int h = blockIdx.x, b = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int hk = h / (p.Hv / p.Hk);
  const float scale = float(1.0 / sqrt(double(D)));
  const int64_t s0 = p.cu[b], s1 = p.cu[b + 1];

  const bool want_init = p.init_pool && (p.use_init == nullptr || p.use_init[b] != 0);
  const int64_t islot = p.init_slot ? int64_t(p.init_slot[b]) : int64_t(b);
  const int64_t fslot = p.final_slot ? int64_t(p.final_slot[b]) : int64_t(b);
  if ((want_init && (islot < 0 || islot >= p.n_slots)) ||
      (p.final_pool && (fslot < 0 || fslot >= p.n_slots))) {
    if (tid == 0 && p.err) atomicExch(p.err, 1);
    return;
  }
  for (int i = tid; i < D * D; i += kNT) {
    const int r = i / D, c = i % D;
    S[r * LD + c] = want_init ? p.init_pool[(islot * p.Hv + h) * int64_t(D * D) + i] : 0.f;
  }

  const T* qg = reinterpret_cast<const T*>(p.q);
  const T* kg = reinterpret_cast<const T*>(p.k);
  const T* vg = reinterpret_cast<const T*>(p.v);
  T* og = reinterpret_cast<T*>(p.out);

  for (int64_t c0 = s0; c0 < s1; c0 += kC) {
    const int nt = int((s1 - c0) < kC ? (s1 - c0) : kC);
    __syncthreads();  // previous chunk done with Qs/Ks/Vs/S
    // ---- load q, k (l2norm in the activation dtype), v, beta, g
    for (int t = warp; t < kC; t += kNT / 32) {
      const bool live = t < nt;
      const int64_t tok = c0 + t;
      constexpr int PER = D / 32;
      float xq[PER], xk[PER];
      float sq = 0.f, sk = 0.f;
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        xq[i] = live ? Io<T>::ld(qg + tok * p.q_st + int64_t(hk) * D + lane + 32 * i) : 0.f;
        xk[i] = live ? Io<T>::ld(kg + tok * p.k_st + int64_t(hk) * D + lane + 32 * i) : 0.f;
        sq += Io<T>::rnd(xq[i] * xq[i]);
        sk += Io<T>::rnd(xk[i] * xk[i]);
      }
      if (p.l2norm) {
        sq = warp_sum(sq);
        sk = warp_sum(sk);
        const float iq = Io<T>::rnd(1.0f / sqrtf(Io<T>::rnd(Io<T>::rnd(sq) + 1e-6f)));
        const float ik = Io<T>::rnd(1.0f / sqrtf(Io<T>::rnd(Io<T>::rnd(sk) + 1e-6f)));
#pragma unroll
        for (int i = 0; i < PER; ++i) {
          xq[i] = Io<T>::rnd(xq[i] * iq);
          xk[i] = Io<T>::rnd(xk[i] * ik);
        }
      }
#pragma unroll
      for (int i = 0; i < PER; ++i) {
        Qs[t * LD + lane + 32 * i] = xq[i] * scale;
        Ks[t * LD + lane + 32 * i] = xk[i];
        Vs[t * LD + lane + 32 * i] =
            live ? Io<T>::ld(vg + tok * p.v_st + int64_t(h) * D + lane + 32 * i) : 0.f;
      }
    }
    if (tid < kC) {
      const bool live = tid < nt;
      float gt = 0.f, bt = 0.f;
      if (live) chunk_gate(p, c0 + tid, h, gt, bt);
      sb[tid] = bt;
      gc[tid] = gt;
    }
    __syncthreads();
    // ---- cumulative log-decay within the chunk (warp 0, two entries per lane)
    if (warp == 0) {
      const float a0 = gc[2 * lane], a1 = gc[2 * lane + 1];
      float pre = a0 + a1;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float nb = __shfl_up_sync(0xffffffffu, pre, o);
        if (lane >= o) pre += nb;
      }
      const float excl = pre - (a0 + a1);
      __syncwarp();
      gc[2 * lane] = excl + a0;
      gc[2 * lane + 1] = excl + a0 + a1;
      __syncwarp();
      const float gl = gc[kC - 1];
      egc[2 * lane] = expf(gc[2 * lane]);
      egc[2 * lane + 1] = expf(gc[2 * lane + 1]);
      ekd[2 * lane] = expf(gl - gc[2 * lane]);
      ekd[2 * lane + 1] = expf(gl - gc[2 * lane + 1]);
      if (lane == 0) gscal[0] = expf(gl);
    }
    __syncthreads();
    // ---- X = -((k*beta) k^T . decay), strictly lower  -> Ts
    {
      float acc[4][4];
      tile_mm<kC, kC, D, 4, 4>(
          acc, [&](int i, int d) { return Ks[i * LD + d] * sb[i]; },
          [&](int d, int j) { return Ks[j * LD + d]; }, tid);
      const int ti = tid / 16, tj = tid % 16;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int i = ti + r * 16, j = tj + c * 16;
          Ts[i * LT + j] = j < i ? -(acc[r][c] * expf(gc[i] - gc[j])) : 0.f;
        }
    }
    __syncthreads();
    // ---- T = (I - X)^-1, blocked as src/gdn_chunk_fast.py:33-62
    {
      float rcol[16];
      const int blk = tid / 16, j = tid % 16, b0 = blk * 16;
      if (tid < 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) rcol[i] = 0.f;
#pragma unroll
        for (int i = 1; i < 16; ++i) {
          if (i > j) {
            float v = Ts[(b0 + i) * LT + b0 + j];
#pragma unroll
            for (int m = 0; m < 16; ++m)
              if (m > j && m < i) v = fmaf(Ts[(b0 + i) * LT + b0 + m], rcol[m], v);
            rcol[i] = v;
          }
        }
      }
      __syncthreads();
      if (tid < 64) {
#pragma unroll
        for (int i = 0; i < 16; ++i) Ts[(b0 + i) * LT + b0 + j] = i == j ? 1.f : (i > j ? rcol[i] : 0.f);
      }
      __syncthreads();
      // level 1: blocks (0,1) and (2,3): P = B X21 (16x16), T21 = P A
      float* P = Ws;  // scratch
      {
        const int m = tid / 128, idx = tid % 128;
        const int lo = m * 32, hi = lo + 16;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rr = (idx * 2 + e) / 16, cc = (idx * 2 + e) % 16;
          float v = 0.f;
          for (int t2 = 0; t2 < 16; ++t2) v = fmaf(Ts[(hi + rr) * LT + hi + t2], Ts[(hi + t2) * LT + lo + cc], v);
          P[m * 256 + rr * 16 + cc] = v;
        }
      }
      __syncthreads();
      {
        const int m = tid / 128, idx = tid % 128;
        const int lo = m * 32, hi = lo + 16;
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int rr = (idx * 2 + e) / 16, cc = (idx * 2 + e) % 16;
          float v = 0.f;
          for (int t2 = 0; t2 < 16; ++t2) v = fmaf(P[m * 256 + rr * 16 + t2], Ts[(lo + t2) * LT + lo + cc], v);
          Ts[(hi + rr) * LT + lo + cc] = v;
        }
      }
      __syncthreads();
      // level 2: P = B X21 (32x32), T21 = P A
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int o = tid * 4 + e, rr = o / 32, cc = o % 32;
        float v = 0.f;
        for (int t2 = 0; t2 < 32; ++t2) v = fmaf(Ts[(32 + rr) * LT + 32 + t2], Ts[(32 + t2) * LT + cc], v);
        P[rr * 32 + cc] = v;
      }
      __syncthreads();
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int o = tid * 4 + e, rr = o / 32, cc = o % 32;
        float v = 0.f;
        for (int t2 = 0; t2 < 32; ++t2) v = fmaf(P[rr * 32 + t2], Ts[t2 * LT + cc], v);
        Ts[(32 + rr) * LT + cc] = v;
      }
      __syncthreads();
    }
    // ---- U = T (v*beta) -> Vs;  W = T (k*beta*exp(gc)) -> Ws
    {
      constexpr int TN = D / 16;
      float u[4][TN], w[4][TN];
      tile_mm<kC, D, kC, 4, TN>(
          u, [&](int i, int j) { return Ts[i * LT + j]; }, [&](int j, int d) { return Vs[j * LD + d] * sb[j]; },
          tid);
      tile_mm<kC, D, kC, 4, TN>(
          w, [&](int i, int j) { return Ts[i * LT + j]; },
          [&](int j, int d) { return (Ks[j * LD + d] * sb[j]) * egc[j]; }, tid);
      __syncthreads();
      const int ti = tid / 16, tj = tid % 16;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < TN; ++c) {
          Vs[(ti + r * 16) * LD + tj + c * 16] = u[r][c];
          Ws[(ti + r * 16) * LD + tj + c * 16] = w[r][c];
        }
    }
    __syncthreads();
    // ---- QK (causal incl. diagonal) -> Ts;  vn = U - W S -> Vs
    {
      float acc[4][4];
      tile_mm<kC, kC, D, 4, 4>(
          acc, [&](int i, int d) { return Qs[i * LD + d]; }, [&](int d, int j) { return Ks[j * LD + d]; }, tid);
      const int ti = tid / 16, tj = tid % 16;
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int i = ti + r * 16, j = tj + c * 16;
          Ts[i * LT + j] = j <= i ? acc[r][c] * expf(gc[i] - gc[j]) : 0.f;
        }
      constexpr int TN = D / 16;
      float ws[4][TN];
      tile_mm<kC, D, D, 4, TN>(
          ws, [&](int i, int d) { return Ws[i * LD + d]; }, [&](int d, int v) { return S[d * LD + v]; }, tid);
#pragma unroll
      for (int r = 0; r < 4; ++r)
#pragma unroll
        for (int c = 0; c < TN; ++c) {
          const int i = ti + r * 16, v = tj + c * 16;
          Vs[i * LD + v] = Vs[i * LD + v] - ws[r][c];
        }
    }
    __syncthreads();
    // ---- o = (q*exp(gc)) S + QK vn
    {
      constexpr int TN = D / 16;
      float o1[4][TN], o2[4][TN];
      tile_mm<kC, D, D, 4, TN>(
          o1, [&](int i, int d) { return Qs[i * LD + d] * egc[i]; }, [&](int d, int v) { return S[d * LD + v]; },
          tid);
      tile_mm<kC, D, kC, 4, TN>(
          o2, [&](int i, int j) { return Ts[i * LT + j]; }, [&](int j, int v) { return Vs[j * LD + v]; }, tid);
      const int ti = tid / 16, tj = tid % 16;
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int i = ti + r * 16;
        if (i < nt) {
#pragma unroll
          for (int c = 0; c < TN; ++c) {
            const int v = tj + c * 16;
            Io<T>::st(og + (c0 + i) * p.o_st + int64_t(h) * D + v, o1[r][c] + o2[r][c]);
          }
        }
      }
    }
    __syncthreads();
    // ---- S = S * exp(gc_last) + (k * exp(gc_last - gc))^T vn
    {
      constexpr int TM = D / 16, TN = D / 16;
      float acc[TM][TN];
      tile_mm<D, D, kC, TM, TN>(
          acc, [&](int d, int j) { return Ks[j * LD + d] * ekd[j]; }, [&](int j, int v) { return Vs[j * LD + v]; },
          tid);
      const float gl = gscal[0];
      const int ti = tid / 16, tj = tid % 16;
#pragma unroll
      for (int r = 0; r < TM; ++r)
#pragma unroll
        for (int c = 0; c < TN; ++c) {
          float* sp = S + (ti + r * 16) * LD + tj + c * 16;
          *sp = *sp * gl + acc[r][c];
        }
    }
  }
  __syncthreads();
  if (p.final_pool) {
    float* dst = p.final_pool + (fslot * p.Hv + h) * int64_t(D * D);
    for (int i = tid; i < D * D; i += kNT) dst[i] = S[(i / D) * LD + i % D];
  }
}

template <typename T, int D>
static int launch_chunk_simt(const ChunkParams& p, cudaStream_t s) {
  auto kern = chunk_simt_kernel<T, D>;
  constexpr size_t smem = SimtSmem<D>::BYTES;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem));
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "chunk_simt: smem attribute: %s", cudaGetErrorString(e));
  kern<<<dim3(p.Hv, p.B), kNT, smem, s>>>(p);
  return check_launch("gdn_chunk_prefill (fp32)");
}

int run_chunk_simt(const ChunkParams& p, int D, int dtype, cudaStream_t s) {
  if (dtype == GDN_F32) {
    if (D == 128) return launch_chunk_simt<float, 128>(p, s);
    if (D == 64) return launch_chunk_simt<float, 64>(p, s);
  } else if (dtype == GDN_BF16) {
    if (D == 128) return launch_chunk_simt<__nv_bfloat16, 128>(p, s);
    if (D == 64) return launch_chunk_simt<__nv_bfloat16, 64>(p, s);
  }
  return fail(GDN_ERR_SHAPE, "gdn_chunk_prefill: d=%d dtype=%d not built", D, dtype);
}

}  // namespace gdn
