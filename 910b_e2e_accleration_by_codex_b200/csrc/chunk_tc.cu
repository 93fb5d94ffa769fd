// a1, tensor-core path.  Chunked gated delta rule (chunk 64, dk = dv = 128, bf16 activations,
// fp32 state) on the 5th-generation tensor cores of sm_100a.
//
// Persistent CTAs (one per SM, three warpgroups) walk a list of (sequence, value head) items; the
// fp32 state lives in TMEM, transposed (S^T: lane v, column k), for the whole item.  The chunk
// algebra of fast_chunk_gated_delta_rule_v2 (src/gdn_chunk_fast2.py:37-59) is split into the part
// that does not depend on S and the part that does, and the two run as a software pipeline:
//
//   intra-chunk group (warps 0-7), chunk j:
//       TMA loads of raw q, k (un-repeated k-head) and v tiles (128-byte swizzle; never multicast)
//       P1  [Q;K] [Q;K]^T  -> QK^T, KK^T and, on the diagonal, the squared row norms that give the
//                             l2-norm factors rq, rk (rounded in bf16 as src/gdn_chunk_fast.py:17-18)
//       CUDA cores: X = -(beta k k^T . decay) strictly lower; T = (I - X)^-1 by the blocked
//                   inverse of src/gdn_chunk_fast.py:21-62; QKm = (q k^T . decay) causal
//       P2  U^T = V^T (T diag beta)^T          P3  W^T = K^T (T diag(beta e^gc rk))^T
//   recurrence group (warps 8-11), chunk j-1 (or j once the intra group hands it over):
//       P4  vn^T = U^T - S^T W^T                (a-negated accumulate onto U^T)
//       P5  o^T  = (S^T Q^T) . (rq scale e^gc) + vn^T QKm^T    (two accumulators)
//       P6  S^T  = S^T e^gl + (vn . rk e^(gl-gc))^T K         (S pre-scaled when read)
//       S^T, vn^T and (vn . rk e^(gl-gc))^T are the A operands of P4-P6, taken from bf16 copies in
//       TMEM; the output leaves through a swizzled shared tile (TMA stores for full chunks) and the
//       final state goes to the slot's pool row.
//
// Hand-over uses mbarriers ("chunk ready" / "buffers freed"); per-chunk TMEM accumulators, the QKm
// tile and the per-chunk vectors are double buffered so the intra group can run a chunk ahead.
// All MMAs are M = 128 tcgen05.mma.kind::f16 (bf16 operands, fp32 accumulation); the state itself
// is never rounded.  Tokens past the end of the sequence are zeroed in shared memory and get
// beta = 0 and rq = rk = 0, which is what the reference's zero padding does.
#include "chunk.cuh"
#include "sm100.cuh"

namespace gdn {
namespace tcchunk {

using namespace sm100;

constexpr int kC = 64;
constexpr int kD = 128;
constexpr int kNT = 384;   // warps 0-7: intra-chunk group, warps 8-11: recurrence group
constexpr int kNI = 256;   // intra-group threads
constexpr int kRegLaunch = 168, kRegIntra = 136, kRegRec = 232;  // setmaxnreg split (see the kernel)
static_assert(2 * 128 * kRegIntra + 128 * kRegRec == kNT * kRegLaunch, "register split must match the launch");

constexpr uint32_t TMEM_COLS = 512;
constexpr int kSortMax = 256;  // sequences ranked by length in-kernel (beyond: index order)
constexpr int LT = 68;   // row stride (floats) of the fp32 64x64 scratch: 16-byte aligned rows
constexpr int LP = 36;   // row stride of the 32x32 merge scratch
constexpr float kLog2e = 1.4426950408889634f;

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ uint32_t pack2(float a, float b) {
  __nv_bfloat162 t = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&t);
}

__device__ __forceinline__ void unpack8(const uint4& u, float* x) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    x[2 * i] = __uint_as_float(w[i] << 16);
    x[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
  }
}

// Store 16 fp32 values as 2 bf16 chunks of row r, chunks cc0, cc0+1.
__device__ __forceinline__ void store_row16(uint8_t* tile, int R, int r, int cc0, const float* v) {
#pragma unroll
  for (int q = 0; q < 2; ++q) {
    uint4 u;
    u.x = pack2(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack2(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack2(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack2(v[8 * q + 6], v[8 * q + 7]);
    *reinterpret_cast<uint4*>(tile + chunk_off(r, cc0 + q, R)) = u;
  }
}

// Store 32 fp32 values as 4 bf16 chunks of row r, chunks cc0..cc0+3.
__device__ __forceinline__ void store_row32(uint8_t* tile, int R, int r, int cc0, const float* v) {
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    uint4 u;
    u.x = pack2(v[8 * q + 0], v[8 * q + 1]);
    u.y = pack2(v[8 * q + 2], v[8 * q + 3]);
    u.z = pack2(v[8 * q + 4], v[8 * q + 5]);
    u.w = pack2(v[8 * q + 6], v[8 * q + 7]);
    *reinterpret_cast<uint4*>(tile + chunk_off(r, cc0 + q, R)) = u;
  }
}

__device__ __forceinline__ float4 lds4(const float* p) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ float2 lds2(const float* p) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ float lds1(const float* p) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(smem_u32(p)));
  return v;
}
__device__ __forceinline__ float f4get(const float4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
// Named barrier over one warp group (id 1: the 256 intra threads, id 2: the 128 recurrence threads).
__device__ __forceinline__ void group_sync(int id) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(id == 1 ? kNI : 128) : "memory");
}

// T = (I - X)^-1 for the strictly lower 64x64 X held in fp32 shared memory (row stride LT), in
// place, by the blocked scheme of src/gdn_chunk_fast.py:33-62: 16x16 diagonal blocks by the row
// recurrence (evaluated column-wise, on warps 0-1, one block per half-warp), then pairwise merges
// T21 = (B X21) A.  Run by the 8 warps of the intra group (named barrier 1); P is 32 x LP floats of
// scratch.  In the products B X21 a lane owns one output column: the column operand is one
// conflict-free 32-bit load per row and the row operand a uniform-address float4; in the products P A
// a lane owns one output row (P rows are LP floats apart, so their 16-byte loads do not conflict), the
// A rows are uniform-address, and a warp owns a few output columns, so whole warps skip the k-steps
// where A's columns are zero.
__device__ __forceinline__ void tri_inverse64(float* X, float* P, int warp, int lane) {
  if (warp < 2) {  // diagonal block 2 warp + lane / 16; lane j = lane % 16 owns column j (the two half-warps'
                   // blocks are 16 banks apart, so their accesses do not conflict)
    const int b0 = 16 * (2 * warp + (lane >> 4)), j = lane & 15;
    float acc[16], r[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = lds1(X + (b0 + i) * LT + b0 + j);
#pragma unroll
    for (int mg = 0; mg < 4; ++mg) {
      // the 4 x 4 triangle of columns 4mg..4mg+3 resolves r[4mg..4mg+3] ...
      float4 xt[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) xt[u] = lds4(X + (b0 + 4 * mg + u) * LT + b0 + 4 * mg);
#pragma unroll
      for (int mm = 0; mm < 4; ++mm) {
        const int m = 4 * mg + mm;
        r[m] = m > j ? acc[m] : 0.f;
#pragma unroll
        for (int u = mm + 1; u < 4; ++u) acc[4 * mg + u] = fmaf(f4get(xt[u], mm), r[m], acc[4 * mg + u]);
      }
      // ... which then update the rows below it, one row at a time (same FMA order per row)
#pragma unroll
      for (int i = 4 * mg + 4; i < 16; ++i) {
        const float4 x = lds4(X + (b0 + i) * LT + b0 + 4 * mg);
        acc[i] = fmaf(x.x, r[4 * mg], acc[i]);
        acc[i] = fmaf(x.y, r[4 * mg + 1], acc[i]);
        acc[i] = fmaf(x.z, r[4 * mg + 2], acc[i]);
        acc[i] = fmaf(x.w, r[4 * mg + 3], acc[i]);
      }
    }
    __syncwarp();
#pragma unroll
    for (int i = 0; i < 16; ++i) X[(b0 + i) * LT + b0 + j] = i == j ? 1.f : (i > j ? r[i] : 0.f);
  }
  group_sync(1);
  // In both merge levels the first product B X21 has a lower-triangular left factor B, so the rows of
  // row group g need only the first g + 1 four-column steps; the warps that share a scheduler (w and
  // w + 4) take complementary row groups, which evens their work.  Skipped terms are exact zeros and
  // the remaining ones are summed in the same ascending order, so the result does not change.
  {  // level 1: merge m = warp / 4 (blocks (0,1) or (2,3)), column c = lane % 16, rows r0, r0 + 1 with
     // r0 = 4 rg + 2 (lane / 16), rg = warp % 4 (merge 0) or 3 - warp % 4 (merge 1): the half-warps
     // read the same column (a broadcast)
    const int m = warp >> 2, c = lane & 15, lo = m * 32, hi = lo + 16;
    const int rg = m == 0 ? (warp & 3) : 3 - (warp & 3), r0 = 4 * rg + 2 * (lane >> 4);
    float a[2] = {0.f, 0.f};
#pragma unroll 4
    for (int tq = 0; tq <= rg; ++tq) {  // B = T(hi, hi) is lower triangular: columns < 4 (rg + 1)
      float x[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) x[u] = lds1(X + (hi + 4 * tq + u) * LT + lo + c);
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        const float4 bv = lds4(X + (hi + r0 + rr) * LT + hi + 4 * tq);
        a[rr] = fmaf(bv.w, x[3], fmaf(bv.z, x[2], fmaf(bv.y, x[1], fmaf(bv.x, x[0], a[rr]))));
      }
    }
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) P[m * 16 * LP + (r0 + rr) * LP + c] = a[rr];
    group_sync(1);
    // second product T21 = P A of both merges: lane -> row (lanes 0-15 merge 0, 16-31 merge 1; P rows are
    // LP floats apart, conflict-free 16-byte loads), warp -> columns 2 g2, 2 g2 + 1 with g2 = warp or
    // 11 - warp (the warps sharing a scheduler split the triangle evenly).  A = T(lo, lo) is lower
    // triangular, so only k >= 4 (g2 / 2) contribute: the skipped terms are exact zeros after a +0 start.
    const int g2 = warp < 4 ? warp : 11 - warp, mm = lane >> 4, rm = lane & 15, lo2 = 32 * mm, c2 = 2 * g2;
    float b0 = 0.f, b1 = 0.f;
#pragma unroll 4
    for (int k4 = g2 >> 1; k4 < 4; ++k4) {
      const float4 pv = lds4(P + lane * LP + 4 * k4);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const float2 av = lds2(X + (lo2 + 4 * k4 + u) * LT + lo2 + c2);
        const float pk = f4get(pv, u);
        b0 = fmaf(pk, av.x, b0);
        b1 = fmaf(pk, av.y, b1);
      }
    }
    *reinterpret_cast<float2*>(X + (lo2 + 16 + rm) * LT + lo2 + c2) = make_float2(b0, b1);
    group_sync(1);
  }
  {  // level 2: group g = warp (warps 0-3) or 11 - warp (warps 4-7)
    const int g = warp < 4 ? warp : 11 - warp;
    {  // P = T(32:64, 32:64) X(32:64, 0:32): column c = lane, rows 4g .. 4g+3, columns of B below 4 (g + 1)
      const int c = lane, r0 = 4 * g;
      float a[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int tq = 0; tq <= g; ++tq) {
        float x[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) x[u] = lds1(X + (32 + 4 * tq + u) * LT + c);
#pragma unroll
        for (int rr = 0; rr < 4; ++rr) {
          const float4 bv = lds4(X + (32 + r0 + rr) * LT + 32 + 4 * tq);
          a[rr] = fmaf(bv.w, x[3], fmaf(bv.z, x[2], fmaf(bv.y, x[1], fmaf(bv.x, x[0], a[rr]))));
        }
      }
#pragma unroll
      for (int rr = 0; rr < 4; ++rr) P[(r0 + rr) * LP + c] = a[rr];
    }
    group_sync(1);
    {  // T(32:64, 0:32) = P T(0:32, 0:32): row r = lane, columns 4g .. 4g+3; T(0:32, 0:32) is lower
       // triangular, so only k >= 4g contribute.  P rows are 36 floats apart (conflict-free 16-byte
       // loads), the T rows are uniform across the warp (broadcast), the result leaves as one 16-byte store.
      const int r = lane, c0 = 4 * g;
      float b[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll 4
      for (int k4 = g; k4 < 8; ++k4) {
        const float4 pv = lds4(P + r * LP + 4 * k4);
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const float4 tv = lds4(X + (4 * k4 + u) * LT + c0);
          const float pk = f4get(pv, u);
          b[0] = fmaf(pk, tv.x, b[0]);
          b[1] = fmaf(pk, tv.y, b[1]);
          b[2] = fmaf(pk, tv.z, b[2]);
          b[3] = fmaf(pk, tv.w, b[3]);
        }
      }
      *reinterpret_cast<float4*>(X + (32 + r) * LT + c0) = make_float4(b[0], b[1], b[2], b[3]);
    }
    group_sync(1);
  }
}

// Per-chunk vectors handed from the intra warpgroup to the recurrence warpgroup (double buffered).
struct ChunkVec {
  float gc[64];   // log2-scaled cumulative decay
  float bt[64];   // beta (0 past the sequence end)
  float rn[128];  // l2norm factors: rq rows 0-63, rk rows 64-127 (0 past the end)
  float egc[64];  // exp(gc)
  float dkd[64];  // rk exp(gl - gc)
  float bwc[64];  // beta exp(gc) rk
  float osc[64];  // rq scale exp(gc): the output scale of S^T q_t
  float gl, Gl;   // log2-scaled total decay of the chunk and exp of it
  int nt;         // live tokens in the chunk
  int pad;
};

// One (sequence, value head) work item and a chunk cursor over a CTA's work list.
struct ItemInfo {
  int b, h, hk, nch;
  int64_t s0, s1, islot, fslot;
  bool init, ok;
};
struct Cur {
  int k, ci;
  ItemInfo it;
  bool live;
};

// shared-memory map of the warp-specialised kernel (bytes from a 1024-byte aligned base)
constexpr uint32_t W_QK0 = 0;          // QK stage 0: [Q d0-63 | K d0-63 | Q d64-127 | K d64-127]
constexpr uint32_t W_QK1 = 32768;      // QK stage 1
constexpr uint32_t W_V = 65536;        // V [s][v] (single buffer; intra group only)
constexpr uint32_t W_WT = 81920;       // W^T [k][t]; then the output staging o [t][v]
constexpr uint32_t W_INIT = 98304;     // the next item's initial state S [k][v] fp32 (64 KiB, bulk-loaded)
constexpr uint32_t W_BU = 163840;      // T diag(beta) [t][s]
constexpr uint32_t W_BW = 172032;      // T diag(beta e^gc rk) [t][s]
constexpr uint32_t W_BQK0 = 180224;    // QKm [t][s], buffer 0
constexpr uint32_t W_BQK1 = 188416;    // buffer 1
constexpr uint32_t W_X = 196608;       // fp32 64 x LT inverse scratch (17408 B) + 32 x LP merge scratch
constexpr uint32_t W_VEC = 218624;     // 2 x ChunkVec
constexpr uint32_t kVecBytes = 2304;   // one ChunkVec slot (16-byte multiple)
constexpr uint32_t W_BAR = W_VEC + 2 * kVecBytes;  // mbarriers
constexpr uint32_t W_ORD = W_BAR + 128;  // sequences ranked longest first (kSortMax ints)
constexpr uint32_t W_SMEM = W_ORD + 4 * 256 + 1024;
static_assert(sizeof(ChunkVec) <= kVecBytes && kVecBytes % 16 == 0, "ChunkVec");
static_assert(W_SMEM <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
static_assert(W_X + 64 * LT * 4 + 32 * LP * 4 <= W_VEC, "scratch");

// TMEM columns
// TMEM columns.  The state is held transposed, S^T (lane v, column k), so that S^T and the vn^T tiles
// (lane v as well) feed the recurrence group's MMAs as A operands straight from TMEM.
constexpr uint32_t T_S = 0;      // S^T fp32, 128 columns
constexpr uint32_t T_S16 = 128;  // S^T bf16 (A of P4, P5), 64 columns
constexpr uint32_t T_VN16 = 192; // vn^T bf16 (A of vn^T QKm^T), 32 columns
constexpr uint32_t T_VND = 224;  // (vn . rk e^(gl-gc))^T bf16 (A of P6), 32 columns
constexpr uint32_t T_UW = 256;   // per buffer b (128 b + 256): U^T -> vn^T -> vn^T QKm^T (64 columns),
                                 // then W^T -> S^T Q^T (64 columns); [Q;K][Q;K]^T of the intra group's
                                 // chunk occupies the same 128 columns before P2/P3 overwrite them

__global__ void __launch_bounds__(kNT, 1)
    chunk_tc_kernel(const ChunkParams p, const __grid_constant__ CUtensorMap tq,
                    const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv,
                    const __grid_constant__ CUtensorMap to, const int use_tma_store) {
  extern __shared__ __align__(1024) uint8_t smraw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smraw) + 1023) & ~uintptr_t(1023));
  const uint32_t sb = smem_u32(sm);
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + W_BAR);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(sm + W_BAR + 96);
  float* Xs = reinterpret_cast<float*>(sm + W_X);
  float* Ps = Xs + 64 * LT;
  // mbarriers: 0,1 QK stage full; 2 V full; 3 intra MMA; 4 recurrence MMA; 5,6 chunk ready; 7,8 buffers freed
  const uint32_t bar_qk0 = smem_u32(&bars[0]), bar_v = smem_u32(&bars[2]);
  const uint32_t bar_mi = smem_u32(&bars[3]), bar_mr = smem_u32(&bars[4]);
  const uint32_t bar_ready0 = smem_u32(&bars[5]), bar_free0 = smem_u32(&bars[7]);
  const uint32_t bar_init = smem_u32(&bars[9]);  // the next item's initial state landed in W_INIT

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int grp = warp >= 8 ? 1 : 0;  // 0: intra-chunk group (warps 0-7), 1: recurrence group (8-11)
  const int wg = warp & 3;            // TMEM lane quarter this warp may access
  const int hv = (warp >> 2) & 1;     // intra group: which half of the columns this warp handles
  const int row = 32 * wg + lane;     // TMEM lane of this thread
  const uint32_t lane_off = uint32_t(32 * wg) << 16;
  const float scale = float(1.0 / sqrt(double(kD)));

  // Work list.  The B * Hv (sequence, value head) items, sequences ranked longest first, are dealt
  // to the persistent CTAs in snake order (round k gives item k * P + c, or k * P + P - 1 - c on
  // odd rounds, to CTA c), which balances the rounds of unequal length.  Both warp groups walk the
  // same list; the intra group runs up to two chunks ahead, across item boundaries.
  const int P = int(gridDim.x), cta = int(blockIdx.x);
  const int nitems = p.B * p.Hv;
  int* ord = reinterpret_cast<int*>(sm + W_ORD);
  const bool sorted = p.B > 1 && p.B <= kSortMax;
  if (sorted) {
    int* lens = reinterpret_cast<int*>(sm + W_X);  // the inverse scratch is free until the first chunk
    for (int i = tid; i < p.B; i += kNT) lens[i] = p.cu[i + 1] - p.cu[i];
    __syncthreads();
    for (int i = tid; i < p.B; i += kNT) {
      const int li = lens[i];
      int rank = 0;
      for (int l = 0; l < p.B; ++l) rank += (lens[l] > li) || (lens[l] == li && l < i);
      ord[rank] = i;
    }
    __syncthreads();
  }
  // k-th item of this CTA; false past the end of its list
  auto item = [&](int k, ItemInfo& it) -> bool {
    const int u = k * P + ((k & 1) ? P - 1 - cta : cta);
    if (u >= nitems) return false;
    const int r = u / p.Hv;
    it.h = u - r * p.Hv;
    it.b = sorted ? ord[r] : r;
    it.hk = it.h / (p.Hv / p.Hk);
    it.s0 = p.cu[it.b];
    it.s1 = p.cu[it.b + 1];
    it.nch = it.s1 > it.s0 ? int((it.s1 - it.s0 + kC - 1) / kC) : 0;
    it.init = p.init_pool && (p.use_init == nullptr || p.use_init[it.b] != 0);
    it.islot = p.init_slot ? int64_t(p.init_slot[it.b]) : int64_t(it.b);
    it.fslot = p.final_slot ? int64_t(p.final_slot[it.b]) : int64_t(it.b);
    it.ok = !((it.init && (it.islot < 0 || it.islot >= p.n_slots)) ||
              (p.final_pool && (it.fslot < 0 || it.fslot >= p.n_slots)));
    return true;
  };
  // chunk cursor over the items that have chunks (valid slots, non-empty)
  auto seek = [&](Cur& x, int k) {
    for (;; ++k) {
      if (!item(k, x.it)) {
        x.live = false;
        return;
      }
      if (x.it.ok && x.it.nch > 0) {
        x.k = k;
        x.ci = 0;
        x.live = true;
        return;
      }
    }
  };
  auto step = [&](Cur& x) {
    if (!x.live) return;
    if (x.ci + 1 < x.it.nch) ++x.ci;
    else seek(x, x.k + 1);
  };

  auto issue_qk = [&](const Cur& x, int gc) {
    const int st = gc & 1;
    const uint32_t bar = bar_qk0 + 8 * st;
    const uint32_t qk = sb + (st ? W_QK1 : W_QK0);
    const int c0 = int(x.it.s0) + x.ci * kC;
    mbar_expect_tx(bar, 4 * 8192);
    tma_load_3d(qk + 0, &tq, bar, 0, x.it.hk, c0);
    tma_load_3d(qk + 8192, &tk, bar, 0, x.it.hk, c0);
    tma_load_3d(qk + 16384, &tq, bar, 64, x.it.hk, c0);
    tma_load_3d(qk + 24576, &tk, bar, 64, x.it.hk, c0);
  };
  auto issue_v = [&](const Cur& x) {
    const int c0 = int(x.it.s0) + x.ci * kC;
    mbar_expect_tx(bar_v, 2 * 8192);
    tma_load_3d(sb + W_V, &tv, bar_v, 0, x.it.h, c0);
    tma_load_3d(sb + W_V + 8192, &tv, bar_v, 64, x.it.h, c0);
  };

  if (tid == 0) {
    for (int i = 0; i < 10; ++i) mbar_init(smem_u32(&bars[i]), 1);
    fence_mbar_init();
    prefetch_tmap(&tq);
    prefetch_tmap(&tk);
    prefetch_tmap(&tv);
    Cur x;
    seek(x, 0);
    if (x.live) {
      issue_qk(x, 0);
      issue_v(x);
      step(x);
      if (x.live) issue_qk(x, 1);
    }
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(tmem_slot), TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;

  // Register split: the recurrence group's epilogues hold several 32-column TMEM rows at once, the
  // intra group needs far fewer.  Launch: 384 threads x 168 = 64512 registers; intra 2 warpgroups x
  // 128 x 136 = 34816 plus recurrence 128 x 232 = 29696 is exactly that.
  if (grp == 0) asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(kRegIntra));
  else asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(kRegRec));
  if (grp == 0) {
    // ======================================================================== intra-chunk group
    uint32_t ph_mi = 0;
    // A chunk's gate inputs are loaded one chunk ahead into registers and used at the top of their
    // chunk: g and beta as given, or in the raw-gate form in_proj_a / in_proj_b's outputs with the
    // head's A_log and dt_bias (the raw-gate maths waits for the loads, so it runs at the top too).
    float pg0 = 0.f, pg1 = 0.f, pb0 = 0.f, pb1 = 0.f, pA = 0.f, pD = 0.f;
    auto load_gates = [&](const Cur& x) {
      const int64_t c0 = x.it.s0 + int64_t(x.ci) * kC, s1 = x.it.s1;
      const int t0 = 2 * lane, t1 = 2 * lane + 1, h = x.it.h;
      const int64_t i0 = (c0 + t0) * p.gb_st + h, i1 = (c0 + t1) * p.gb_st + h;
      const bool l0 = c0 + t0 < s1, l1 = c0 + t1 < s1;
      pg0 = pg1 = pb0 = pb1 = 0.f;
      if (p.a_raw == nullptr) {
        if (l0) { pg0 = p.g[i0]; pb0 = p.beta[i0]; }
        if (l1) { pg1 = p.g[i1]; pb1 = p.beta[i1]; }
      } else {
        pA = p.A_log[h];
        pD = p.dt_bias[h];
        if (p.raw_bf16) {
          const __nv_bfloat16* ar = static_cast<const __nv_bfloat16*>(p.a_raw);
          const __nv_bfloat16* br = static_cast<const __nv_bfloat16*>(p.b_raw);
          if (l0) { pg0 = __bfloat162float(ar[i0]); pb0 = __bfloat162float(br[i0]); }
          if (l1) { pg1 = __bfloat162float(ar[i1]); pb1 = __bfloat162float(br[i1]); }
        } else {
          const float* ar = static_cast<const float*>(p.a_raw);
          const float* br = static_cast<const float*>(p.b_raw);
          if (l0) { pg0 = ar[i0]; pb0 = br[i0]; }
          if (l1) { pg1 = ar[i1]; pb1 = br[i1]; }
        }
      }
    };
    Cur cur, nx;
    seek(cur, 0);
    nx = cur;
    step(nx);
    if (warp == 0 && cur.live) load_gates(cur);
    for (int gc = 0; cur.live; ++gc) {
      const int bf = gc & 1;
      ChunkVec& cv = *reinterpret_cast<ChunkVec*>(sm + W_VEC + kVecBytes * bf);
      const int64_t c0 = cur.it.s0 + int64_t(cur.ci) * kC, s1 = cur.it.s1;
      const int nt = int((s1 - c0) < kC ? (s1 - c0) : kC);
      uint8_t* qk = sm + (bf ? W_QK1 : W_QK0);
      const uint32_t qk_a = sb + (bf ? W_QK1 : W_QK0);
      const uint32_t bqk = bf ? W_BQK1 : W_BQK0;
      // chunk gc-2 has left this buffer set (vectors, QKm tile, TMEM U/W buffers)
      if (gc >= 2 && ok && !mbar_wait(bar_free0 + 8 * bf, uint32_t((gc - 2) >> 1) & 1u)) ok = false;
      tc_fence_after();
      if (warp == 0) {  // gates: gc = cumsum(g) (log2-scaled), beta; prefetch the next chunk's
        const int t0 = 2 * lane, t1 = 2 * lane + 1;
        if (p.a_raw != nullptr) {  // g = -exp(A_log) softplus(a + dt_bias), beta = sigmoid(b); 0 past the end
          const float A = expf(pA);
          const float s0 = sigmoid_f(pb0), s1 = sigmoid_f(pb1);
          pg0 = t0 < nt ? -A * softplus_f(pg0 + pD) : 0.f;
          pg1 = t1 < nt ? -A * softplus_f(pg1 + pD) : 0.f;
          pb0 = t0 < nt ? (p.raw_bf16 ? bf16r(s0) : s0) : 0.f;
          pb1 = t1 < nt ? (p.raw_bf16 ? bf16r(s1) : s1) : 0.f;
        }
        const float g0 = pg0 * kLog2e, g1 = pg1 * kLog2e;
        cv.bt[t0] = pb0;
        cv.bt[t1] = pb1;
        float pre = g0 + g1;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
          const float nb = __shfl_up_sync(0xffffffffu, pre, o);
          if (lane >= o) pre += nb;
        }
        const float ex = pre - (g0 + g1);
        const float a0 = ex + g0, a1 = ex + g0 + g1;
        cv.gc[t0] = a0;
        cv.gc[t1] = a1;
        cv.egc[t0] = ex2(a0);
        cv.egc[t1] = ex2(a1);
        const float gl = __shfl_sync(0xffffffffu, a1, 31);
        if (lane == 0) {
          cv.gl = gl;
          cv.Gl = ex2(gl);
          cv.nt = nt;
        }
        if (nx.live) load_gates(nx);
        // the next chunk opens a new item: start its initial state towards L2 now, a chunk or two before
        // the recurrence group loads it into TMEM
        if (lane == 0 && nx.live && nx.ci == 0 && nx.it.init)
          bulk_prefetch_l2(p.init_pool + (nx.it.islot * p.Hv + nx.it.h) * int64_t(kD * kD), kD * kD * 4);
      }
      if (ok && !mbar_wait(bar_qk0 + 8 * bf, uint32_t(gc >> 1) & 1u)) ok = false;
      if (nt < kC) {  // zero the q/k rows past the sequence end (they hold the next sequence)
        for (int i = tid; i < (kC - nt) * 32; i += kNI) {
          const int r = nt + (i >> 5), tile = (i >> 3) & 3, cc = i & 7;
          *reinterpret_cast<uint4*>(qk + tile * 8192 + chunk_off(r, cc, 128)) = make_uint4(0, 0, 0, 0);
        }
        fence_async_smem();
      }
      tc_fence_before();
      group_sync(1);
      if (tid == 0) {  // P1: [Q;K] [Q;K]^T
        tc_fence_after();
        const uint32_t id = make_idesc(128, 128, false, false);
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk)
          umma(tmem + T_UW + 128 * bf, desc_kmajor(qk_a, 128, kk), desc_kmajor(qk_a, 128, kk), id, kk > 0);
        umma_commit(bar_mi);
      }
      if (ok && !mbar_wait(bar_mi, ph_mi)) ok = false;
      ph_mi ^= 1u;
      tc_fence_after();
      if (hv == 0) {  // l2-norm factors from the diagonal (bf16 arithmetic as the reference's l2norm)
        float dg[32];
        tmem_ld32(tmem + T_UW + 128 * bf + lane_off + 32 * wg, dg);
        // dg[lane] by a select tree over the lane's bits (31 selects)
#pragma unroll
        for (int w = 16; w >= 1; w >>= 1) {
          const bool hi = (lane & w) != 0;
#pragma unroll
          for (int j = 0; j < w; ++j) dg[j] = hi ? dg[j + w] : dg[j];
        }
        const float ss = dg[0];
        float inv = 1.f;
        if (p.l2norm) inv = bf16r(1.0f / sqrtf(bf16r(bf16r(ss) + 1e-6f)));
        cv.rn[row] = (row & 63) < nt ? inv : 0.f;
      }
      group_sync(1);
      {  // P1 epilogue: QKm tile (rows 0-63) and X (rows 64-127), from the K columns 64-127
        {
          const int half = hv;
          float a[32];
          // rows 0-63: QKm[t][s] = (q_t k_s) rq_t scale rk_s e^(gc_t - gc_s), s <= t; rows 64-127:
          // X[i][s] = -(k_i k_s) rk_i beta_i rk_s e^(gc_i - gc_s), s < i.  One code path for both (the
          // sign factor and the bound differ; every product is rounded as in the two separate forms).
          const bool qrow = row < 64;
          const int t = qrow ? row : row - 64;
          const int lim = qrow ? t + 1 : t;
          if (half == 1 && (wg & 1) == 0) {  // rows t < 32, columns s >= 32: all above the diagonal
#pragma unroll
            for (int j = 0; j < 32; ++j) a[j] = 0.f;
          } else {
            tmem_ld32(tmem + T_UW + 128 * bf + lane_off + 64 + 32 * half, a);
            // the X rows' minus sign rides on f (negation is exact: same values as negating each product)
            const float g0 = cv.gc[t], f = qrow ? cv.rn[t] * scale : -(cv.rn[64 + t] * cv.bt[t]);
#pragma unroll
            for (int j4 = 0; j4 < 8; ++j4) {  // the per-column vectors as 16-byte broadcast loads
              const float4 gs = lds4(cv.gc + 32 * half + 4 * j4), rs = lds4(cv.rn + 64 + 32 * half + 4 * j4);
#pragma unroll
              for (int e = 0; e < 4; ++e) {
                const int j = 4 * j4 + e, s = 32 * half + j;
                a[j] = (s < lim) ? (a[j] * f * f4get(rs, e)) * ex2(g0 - f4get(gs, e)) : 0.f;
              }
            }
          }
          if (qrow) {
            store_row32(sm + bqk, 64, t, 4 * half, a);
          } else {
            const int i = t;
            // 16-byte stores: lanes are rows LT floats apart, so scalar stores would hit 8 banks
#pragma unroll
            for (int q4 = 0; q4 < 8; ++q4)
              *reinterpret_cast<float4*>(Xs + i * LT + 32 * half + 4 * q4) =
                  make_float4(a[4 * q4], a[4 * q4 + 1], a[4 * q4 + 2], a[4 * q4 + 3]);
          }
        }
      }
      group_sync(1);
      if (warp == 2 || warp == 3) {  // per-chunk vectors of the later phases, beside the inverse's diagonal
                                     // blocks (warps 0-1); first read after the inverse
        const int i = tid - 64;
        const float rk = cv.rn[64 + i];
        cv.dkd[i] = rk * ex2(cv.gl - cv.gc[i]);
        cv.bwc[i] = cv.bt[i] * cv.egc[i] * rk;
        cv.osc[i] = cv.rn[i] * scale * cv.egc[i];
      }
      tri_inverse64(Xs, Ps, warp, lane);
      {  // B_U = T diag(beta), B_W = T diag(beta e^gc rk): warp -> 16 columns cb, lane -> row t.  Rows 0-31
         // of columns 32-63 lie above T's diagonal (warps 5 and 7, one per scheduler with the P1
         // epilogue's zero warps 4 and 6): zeros without loads.
        const int cb = 16 * (warp >> 1), t = 32 * (1 - (warp & 1)) + lane;
        float u[16], w[16];
        if (cb >= 32 && t < 32) {
#pragma unroll
          for (int e = 0; e < 16; ++e) u[e] = w[e] = 0.f;
        } else {
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const float4 tv4 = lds4(Xs + t * LT + cb + 4 * e4);
            const float4 bt4 = lds4(cv.bt + cb + 4 * e4), bw4 = lds4(cv.bwc + cb + 4 * e4);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const float tv = f4get(tv4, e);
              u[4 * e4 + e] = tv * f4get(bt4, e);
              w[4 * e4 + e] = tv * f4get(bw4, e);
            }
          }
        }
        store_row16(sm + W_BU, 64, t, cb >> 3, u);
        store_row16(sm + W_BW, 64, t, cb >> 3, w);
      }
      if (ok && !mbar_wait(bar_v, uint32_t(gc) & 1u)) ok = false;
      if (nt < kC) {
        for (int i = tid; i < (kC - nt) * 16; i += kNI) {
          const int r = nt + (i >> 4), tile = (i >> 3) & 1, cc = i & 7;
          *reinterpret_cast<uint4*>(sm + W_V + tile * 8192 + chunk_off(r, cc, 64)) = make_uint4(0, 0, 0, 0);
        }
      }
      fence_async_smem();
      tc_fence_before();
      group_sync(1);
      if (tid == 0) {  // P2: U^T = V^T B_U^T;  P3: W^T = K^T B_W^T
        tc_fence_after();
        const uint32_t id = make_idesc(128, 64, true, false);
#pragma unroll 1
        for (int kk = 0; kk < 4; ++kk)
          umma(tmem + T_UW + 128 * bf, desc_mnmajor(sb + W_V, 64, kk), desc_kmajor(sb + W_BU, 64, kk), id, kk > 0);
#pragma unroll 1
        for (int kk = 0; kk < 4; ++kk)
          umma(tmem + T_UW + 128 * bf + 64, desc_mnmajor(qk_a + 8192, 128, kk), desc_kmajor(sb + W_BW, 64, kk), id,
               kk > 0);
        umma_commit(bar_mi);
      }
      if (ok && !mbar_wait(bar_mi, ph_mi)) ok = false;
      ph_mi ^= 1u;
      tc_fence_before();
      group_sync(1);
      if (tid == 0) {
        if (nx.live) {  // the V buffer is free: fetch the next chunk's
          fence_async_smem();
          issue_v(nx);
        }
        mbar_arrive(bar_ready0 + 8 * bf);  // hand chunk gc to the recurrence group
      }
      cur = nx;
      step(nx);
    }
  } else {
    // ======================================================================== recurrence group
    const int rt = tid - kNI;
    uint32_t ph_mr = 0;
    Cur q2;  // the chunk two ahead of the current one (its Q/K tiles are fetched into the freed stage)
    seek(q2, 0);
    step(q2);
    step(q2);
    int gc = 0;
    uint32_t ph_init = 0;
    // The initial states of this CTA's items arrive by one 64 KiB bulk copy each into W_INIT, in item
    // order and one at a time: the copy for the next item that reads one is issued as soon as the
    // current one has been moved into TMEM.
    auto issue_init = [&](int k0) {  // thread rt == 0
      ItemInfo nx;
      for (int k = k0; item(k, nx); ++k) {
        if (nx.ok && nx.init) {
          fence_async_smem();  // the generic reads of the previous state are ordered before the copy
          mbar_expect_tx(bar_init, kD * kD * 4);
          bulk_load(sb + W_INIT, p.init_pool + (nx.islot * p.Hv + nx.h) * int64_t(kD * kD), kD * kD * 4, bar_init);
          return;
        }
      }
    };
    if (rt == 0) issue_init(0);
    ItemInfo itm;
    for (int k = 0; item(k, itm); ++k) {
    if (!itm.ok) {  // a bad slot index: record it and leave every pool row untouched
      if (rt == 0 && p.err) atomicExch(p.err, 1);
      continue;
    }
    const int h = itm.h;
    {  // initial state -> TMEM as S^T: thread v (TMEM lane) takes column v of S [k][v] (conflict-free)
      if (itm.init) {
        if (ok && !mbar_wait(bar_init, ph_init)) ok = false;
        ph_init ^= 1u;
      }
      const float* st = reinterpret_cast<const float*>(sm + W_INIT);
#pragma unroll 1
      for (int part = 0; part < 4; ++part) {
        float v[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) v[i] = itm.init ? st[(32 * part + i) * kD + row] : 0.f;
        tmem_st32(tmem + T_S + lane_off + 32 * part, v);
      }
      tmem_st_wait();
      if (itm.init) {
        group_sync(2);
        if (rt == 0) issue_init(k + 1);
      }
    }
    for (int ci = 0; ci < itm.nch; ++ci, ++gc) {
      const int bf = gc & 1;
      const ChunkVec& cv = *reinterpret_cast<const ChunkVec*>(sm + W_VEC + kVecBytes * bf);
      const int64_t c0 = itm.s0 + int64_t(ci) * kC;
      const uint32_t qk_a = sb + (bf ? W_QK1 : W_QK0);
      const uint32_t bqk = bf ? W_BQK1 : W_BQK0;
      const uint32_t tU = tmem + T_UW + 128 * bf, tW = tU + 64;
      if (ok && !mbar_wait(bar_ready0 + 8 * bf, uint32_t(gc >> 1) & 1u)) ok = false;
      tc_fence_after();
      if (rt == 0) bulk_wait_read();  // the previous chunk's output store has left W_WT
      group_sync(2);
      const int nt = cv.nt;
      {  // S^T -> bf16 copy in TMEM (A of P4/P5), S^T e^gl back into TMEM (P6 accumulates onto it); W^T tile
        const float Gl = cv.Gl;
#pragma unroll 1
        for (int part = 0; part < 4; ++part) {
          float sv[32];
          tmem_ld32(tmem + T_S + lane_off + 32 * part, sv);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) pk[i] = pack2(sv[2 * i], sv[2 * i + 1]);
          tmem_st16u(tmem + T_S16 + lane_off + 16 * part, pk);
#pragma unroll
          for (int j = 0; j < 32; ++j) sv[j] *= Gl;
          tmem_st32(tmem + T_S + lane_off + 32 * part, sv);
        }
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          float w[32];
          tmem_ld32(tW + lane_off + 32 * half, w);
          store_row32(sm + W_WT, 128, row, 4 * half, w);
        }
        tmem_st_wait();
      }
      fence_async_smem();
      tc_fence_before();
      group_sync(2);
      if (rt == 0) {  // P4: vn^T = U^T - S^T W^T
        tc_fence_after();
        const uint32_t id = make_idesc(128, 64, false, true, true);
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) umma_ts(tU, tmem + T_S16 + 8 * kk, desc_mnmajor(sb + W_WT, 128, kk), id, 1);
        umma_commit(bar_mr);
      }
      if (ok && !mbar_wait(bar_mr, ph_mr)) ok = false;
      ph_mr ^= 1u;
      tc_fence_after();
      {  // vn^T as bf16 copies in TMEM: plain (A of vn^T QKm^T) and scaled by rk e^(gl-gc) (A of P6)
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          float a[32], d[32];
          tmem_ld32(tU + lane_off + 32 * half, a);
#pragma unroll
          for (int j4 = 0; j4 < 8; ++j4) {
            const float4 dk4 = lds4(cv.dkd + 32 * half + 4 * j4);
#pragma unroll
            for (int e = 0; e < 4; ++e) d[4 * j4 + e] = a[4 * j4 + e] * f4get(dk4, e);
          }
          uint32_t pa[16], pd[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            pa[i] = pack2(a[2 * i], a[2 * i + 1]);
            pd[i] = pack2(d[2 * i], d[2 * i + 1]);
          }
          tmem_st16u(tmem + T_VN16 + lane_off + 16 * half, pa);
          tmem_st16u(tmem + T_VND + lane_off + 16 * half, pd);
        }
        tmem_st_wait();
      }
      fence_async_smem();
      tc_fence_before();
      group_sync(2);
      if (rt == 0) {  // P5: W = S^T Q^T, U = vn^T QKm^T;  P6: S^T += (vn . d)^T K  (A operands from TMEM)
        tc_fence_after();
        const uint32_t ia = make_idesc(128, 64, false, false);
#pragma unroll 1
        for (int kk = 0; kk < 8; ++kk) umma_ts(tW, tmem + T_S16 + 8 * kk, desc_kmajor(qk_a, 128, kk), ia, kk > 0);
#pragma unroll 1
        for (int kk = 0; kk < 4; ++kk) umma_ts(tU, tmem + T_VN16 + 8 * kk, desc_kmajor(sb + bqk, 64, kk), ia, kk > 0);
        const uint32_t ic = make_idesc(128, 128, false, true);
#pragma unroll 1
        for (int kk = 0; kk < 4; ++kk) umma_ts(tmem + T_S, tmem + T_VND + 8 * kk, desc_mnmajor(qk_a + 8192, 128, kk), ic, 1);
        umma_commit(bar_mr);
      }
      if (ok && !mbar_wait(bar_mr, ph_mr)) ok = false;
      ph_mr ^= 1u;
      tc_fence_after();
      // P5/P6 were the last readers of this chunk's Q/K stage: refill it with chunk gc+2 now, ahead of
      // the output epilogue and store
      if (rt == 0 && q2.live) {
        fence_async_smem();
        issue_qk(q2, gc + 2);
      }
      {  // output o[t][v] = rq_t scale e^gc_t (S^T q_t)[v] + (vn^T QKm^T)[v][t] -> staging (W_WT), laid out as
         // the two 128-byte-swizzled 64 x 64 boxes of the output tensor map.  The 16x256b TMEM loads give
         // this thread (v, t..t+1) pairs of 8 x 8 blocks (rows v, columns t), which stmatrix.trans writes as
         // 16-byte rows of t holding 8 consecutive v: 8 stores per thread and chunk instead of 64.
        const int qd = lane & 3, m = lane >> 3, kr = lane & 7;
#pragma unroll 1
        for (int half = 0; half < 2; ++half) {
          float2 os[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) os[j] = *reinterpret_cast<const float2*>(cv.osc + 32 * half + 8 * j + 2 * qd);
#pragma unroll 1
          for (int lg = 0; lg < 2; ++lg) {  // TMEM lanes (v) 32 wg + 16 lg .. + 15
            const uint32_t loff = uint32_t(32 * wg + 16 * lg) << 16;
            uint32_t a[16], c[16];
            tmem_ld16x256_x4(tW + loff + 32 * half, a);
            tmem_ld16x256_x4(tU + loff + 32 * half, c);
            tmem_ld_wait();
            uint32_t pk[8];  // pk[2j + vb]: v = 32 wg + 16 lg + 8 vb + g, t = 32 half + 8 j + 2 qd, +1
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
              for (int vb = 0; vb < 2; ++vb)
                pk[2 * j + vb] = pack2(__uint_as_float(a[4 * j + 2 * vb]) * os[j].x + __uint_as_float(c[4 * j + 2 * vb]),
                                       __uint_as_float(a[4 * j + 2 * vb + 1]) * os[j].y +
                                           __uint_as_float(c[4 * j + 2 * vb + 1]));
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {  // matrices (j, vb) = (2jj, 0), (2jj, 1), (2jj+1, 0), (2jj+1, 1)
              const int t = 32 * half + 8 * (2 * jj + (m >> 1)) + kr, v0 = 32 * wg + 16 * lg + 8 * (m & 1);
              stmatrix_x4_trans(sb + W_WT + chunk_off(t, v0 >> 3, 64), pk[4 * jj], pk[4 * jj + 1], pk[4 * jj + 2],
                                pk[4 * jj + 3]);
            }
          }
        }
      }
      fence_async_smem();
      tc_fence_before();
      group_sync(2);
      if (use_tma_store && nt == kC) {
        if (rt == 0) {
          tma_store_3d(&to, sb + W_WT, 0, h, int(c0));
          tma_store_3d(&to, sb + W_WT + 8192, 64, h, int(c0));
          bulk_commit();
        }
      } else {
        const uint8_t* ot = sm + W_WT;
        __nv_bfloat16* og = reinterpret_cast<__nv_bfloat16*>(p.out) + int64_t(h) * kD;
#pragma unroll 1
        for (int k8 = 0; k8 < 8; ++k8) {
          const int cidx = rt + 128 * k8, t = cidx >> 4, cc = cidx & 15;
          if (t < nt)
            *reinterpret_cast<uint4*>(og + (c0 + t) * p.o_st + cc * 8) =
                *reinterpret_cast<const uint4*>(ot + chunk_off(t, cc, 64));
        }
      }
      group_sync(2);
      if (rt == 0) mbar_arrive(bar_free0 + 8 * bf);  // chunk gc is done with its buffer set: free it
      step(q2);
    }
    // final state: thread v holds column v of S; a warp's store of row k covers 128 contiguous bytes
    if (p.final_pool) {
      float* dst = p.final_pool + (itm.fslot * p.Hv + h) * int64_t(kD * kD) + row;
#pragma unroll 1
      for (int part = 0; part < 4; ++part) {
        float v[32];
        tmem_ld32(tmem + T_S + lane_off + 32 * part, v);
#pragma unroll
        for (int i = 0; i < 32; ++i) dst[(32 * part + i) * kD] = v[i];
      }
    }
    }
    if (rt == 0) bulk_wait_all();
  }
  if (!ok && p.err) atomicExch(p.err, 2);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, TMEM_COLS);
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(f);
  }
  return fn;
}

// 3-D map over a [T, H, 128] bf16 tensor with token stride `tok_stride` elements; box = 64 dims x
// 1 head x 64 tokens, 128-byte swizzle (the UMMA canonical layout), zero fill out of bounds.
static int make_map(CUtensorMap* m, const void* base, int H, int64_t T, int64_t tok_stride) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GDN_ERR_CUDA, "gdn_chunk_prefill: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[3] = {cuuint64_t(kD), cuuint64_t(H), cuuint64_t(T)};
  cuuint64_t strides[2] = {cuuint64_t(kD) * 2, cuuint64_t(tok_stride) * 2};
  // loads and the output store: 64-element inner box (one token row half) x 64 tokens, 128-byte swizzle
  cuuint32_t box[3] = {64u, 1, 64};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "gdn_chunk_prefill: tensor map encode failed (%d)", int(r));
  return GDN_OK;
}

}  // namespace tcchunk

int run_chunk_tc(const ChunkParams& p, int64_t T_total, cudaStream_t s) {
  using namespace tcchunk;
  const void* bases[3] = {p.q, p.k, p.v};
  const int64_t strides[3] = {p.q_st, p.k_st, p.v_st};
  for (int i = 0; i < 3; ++i) {
    if (!aligned(bases[i], 16) || (strides[i] % 8) != 0)
      return fail(GDN_ERR_ARG, "gdn_chunk_prefill: q/k/v need 16-byte aligned bases and token strides "
                               "that are multiples of 8 elements");
  }
  // the state rows move as 16-byte vectors (and are prefetched into L2 by bulk prefetches)
  if (!aligned(p.init_pool, 16) || !aligned(p.final_pool, 16))
    return fail(GDN_ERR_ARG, "gdn_chunk_prefill: init_pool / final_pool need 16-byte aligned bases");
  if (T_total >= (int64_t(1) << 31)) return fail(GDN_ERR_ARG, "gdn_chunk_prefill: T_total too large");
  CUtensorMap mq, mk, mv, mo;
  int rc = make_map(&mq, p.q, p.Hk, T_total, p.q_st);
  if (!rc) rc = make_map(&mk, p.k, p.Hk, T_total, p.k_st);
  if (!rc) rc = make_map(&mv, p.v, p.Hv, T_total, p.v_st);
  if (rc) return rc;
  // full output chunks leave through a TMA store when the output rows allow one
  int use_store = aligned(p.out, 16) && (p.o_st % 8) == 0 && T_total > 0;
  if (use_store && make_map(&mo, p.out, p.Hv, T_total, p.o_st) != GDN_OK) use_store = 0;
  if (!use_store) mo = mq;  // never read
  static bool attr_set[64] = {};
  static int sm_count[64] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  int sms = 148;
  if (dev >= 0 && dev < 64 && attr_set[dev]) {
    sms = sm_count[dev];
  } else {
    cudaError_t e = cudaFuncSetAttribute(chunk_tc_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         int(W_SMEM));
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "chunk_tc: setup: %s", cudaGetErrorString(e));
    if (dev >= 0 && dev < 64) {
      sm_count[dev] = sms;
      attr_set[dev] = true;
    }
  }
  // persistent: one CTA per SM walks its share of the (sequence, head) items
  const int64_t items = int64_t(p.B) * p.Hv;
  if (items > (int64_t(1) << 30)) return fail(GDN_ERR_ARG, "gdn_chunk_prefill: B * Hv too large");
  chunk_tc_kernel<<<dim3(unsigned(items < sms ? items : sms)), kNT, W_SMEM, s>>>(p, mq, mk, mv, mo, use_store);
  return check_launch("gdn_chunk_prefill (tensor cores)");
}

}  // namespace gdn
