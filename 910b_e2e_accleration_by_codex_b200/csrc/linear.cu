// Skinny-GEMM projections of the decode step on the 5th-generation tensor cores, and the
// row-parallel projection fused with its sum over the tensor-parallel ranks.
//
//   y[n, n_out] = x[n, k] W[n_out, k]^T                       (gdn_linear)
//   y[n, n_out] = sum over ranks r of x_r W_r^T               (gdn_linear_allreduce)
//
// The second is the reference's AllReduceLinear (src/cb_tp.py:25-35: F.linear, then
// dist.all_reduce) in one kernel.  At decode sizes (n = 16-128 tokens, one per slot) the product
// is bound by streaming W from HBM, so the kernel is laid out around W:
//
//   * W supplies the tcgen05 A operand (M = 128 output features per tile, K-major, 128-byte
//     swizzle, TMA loads); the n tokens are the N dimension (n rounded up to 16, <= 256; rows past
//     n read as zeros).  Every byte of W is loaded exactly once.
//   * A tile's K range is split over the S CTAs of one thread-block cluster (S <= 8, chosen so
//     the grid covers about two CTAs per SM).  Each CTA streams its share of the k-blocks through
//     a ring of shared-memory stages (one TMA thread, one MMA thread, fp32 accumulator in TMEM).
//   * The S partial accumulators are reduced through distributed shared memory: the tile's 8
//     segments of 16 output features are dealt out to the S CTAs, each CTA sends every segment's
//     partial rows to the segment's owner, and the owner sums them in split order (fixed, so the
//     result does not depend on timing).  Nothing goes through HBM.
//   * world == 1: the owner rounds to bf16 and writes y.  world > 1: the owner rounds its segment
//     to bf16 (this rank's partial of y, as the unfused path's GEMM output), stores it with plain
//     16-byte stores into its slot on every rank's exchange buffer, raises the segment's flag on
//     every rank (system-scope release), waits (bounded) for every rank's flag on its own buffer
//     and sums the ranks' partials in rank order in fp32, so all ranks write identical y.
//     The exchange starts as soon as a tile is done; no multicast object, no TMA or bulk copy
//     reads another GPU's memory.
//
// Exchange buffer of one rank (allocated by gdn_ar_alloc, mapped by the peers through IPC):
//   [0, 16 KiB)              epoch[kMaxSegs] u32: calls that touched segment g (local use)
//   [16 KiB, 16 KiB+512 KiB) flag[2][kMaxWorld][kMaxSegs] u32: flag[p][src][g] = src's epoch of g
//   [kDataOff, ...)          data[2][world][max_out / 8][max_rows] 16-byte vectors (8 features of
//                            one token): data[p][src] holds src's bf16 partial of y
// (max_rows, max_out) are fixed for a buffer's lifetime and passed with every call.
//
// Push / pull split (gdn_linear_push + gdn_pull_add_rmsnorm): the projection kernel only sends its
// segments and raises their flags (no wait, so no limit on how many clusters are resident), and
// the kernel that follows it in the decode step -- residual add and the next RMSNorm -- waits for
// the flags, sums the ranks' partials in rank order, adds the residual and normalizes, in one pass
// per token row.  The parity argument above holds with "call" = one push and its pull.
// The data of a segment sits at an address fixed by (segment, token), whatever the call's shape,
// and the epoch of segment g counts the calls that touched it, identically on every rank.  Parity
// p = epoch & 1 double-buffers the data: a rank writes segment g of call e + 2 only after its own
// call e + 1 completed, in which it waited for every rank's flag of g, raised after that rank's
// call e (and its reads of g) completed.
#include <cstring>

#include "common.cuh"
#include "sm100.cuh"

namespace gdn {
namespace lin {

using namespace sm100;

constexpr int kBM = 128;          // output features per tile (tcgen05 M)
constexpr int kBK = 64;           // k elements per stage (one 128-byte swizzle row of bf16)
constexpr int kThreads = 128;
constexpr int kSegRows = 16;      // output features per segment (unit of DSMEM ownership and flags)
constexpr int kSegs = kBM / kSegRows;
constexpr int kMaxSplits = 8;
constexpr int kMaxStages = 16;
constexpr int kMaxTokens = 256;
constexpr int kMaxWorld = 8;
constexpr int kMaxSegs = 4096;    // n_out <= 65536 through the exchange
constexpr size_t kFlagOff = 16384;
constexpr size_t kDataOff = kFlagOff + size_t(2) * kMaxWorld * kMaxSegs * 4;
static_assert(kMaxSegs * 4 <= kFlagOff, "epoch array");

struct Params {
  int n, n_out, kb_total, splits, bn, stages, rows_cap;
  __nv_bfloat16* y;
  int64_t y_rs;
  int rank, world;
  char* bufs[kMaxWorld];
  int64_t max_rows;       // tokens per 8-feature group in the exchange buffer
  int64_t max_octs;       // 8-feature groups per rank's slot (max_out / 8)
  uint32_t spin_limit;
  int32_t* err;
  int push_only;          // world > 1: send the partials and flags, leave the sum to add_rmsnorm_kernel
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ uint32_t map_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void st_cluster_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared::cluster.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp gets lane (taddr.lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }
__device__ __forceinline__ uint32_t* flag_at(char* buf, int p, int src, int g) {
  return reinterpret_cast<uint32_t*>(buf + kFlagOff) + (size_t(p) * kMaxWorld + src) * kMaxSegs + g;
}
__device__ __forceinline__ uint4 pack8(const float* a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    __nv_bfloat162 t = __floats2bfloat162_rn(a[2 * i], a[2 * i + 1]);
    w[i] = *reinterpret_cast<uint32_t*>(&t);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}
__device__ __forceinline__ void add8(const uint4& u, float* acc) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}

// First segment of the tile owned by split ks (segments dealt out as evenly as possible).
__device__ __forceinline__ int seg_lo(int ks, int S) { return ks * kSegs / S; }

__global__ void __launch_bounds__(kThreads) linear_kernel(const __grid_constant__ CUtensorMap mw,
                                                          const __grid_constant__ CUtensorMap mx, const Params p) {
  extern __shared__ uint8_t smem_raw[];
  __shared__ __align__(8) uint64_t full_bar[kMaxStages], empty_bar[kMaxStages], acc_bar;
  __shared__ uint32_t s_tmem;
  __shared__ uint32_t s_epoch[kSegs];
  __shared__ int s_ok;
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int mt = blockIdx.x;
  const int S = p.splits;
  const int ks = int(cluster_rank());
  const int kb0 = ks * p.kb_total / S, kb1 = (ks + 1) * p.kb_total / S;
  const int nkb = kb1 - kb0;
  const int bn = p.bn, stages = p.stages;
  const uint32_t a_bytes = kBM * kBK * 2, b_bytes = uint32_t(bn) * kBK * 2;
  const uint32_t stage_bytes = a_bytes + b_bytes;
  const uint32_t ncols = bn <= 32 ? 32u : bn <= 64 ? 64u : bn <= 128 ? 128u : 256u;

  if (tid == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(smem_u32(&full_bar[s]), 1);
      mbar_init(smem_u32(&empty_bar[s]), 1);
    }
    mbar_init(smem_u32(&acc_bar), 1);
    fence_mbar_init();
    s_ok = 1;
    prefetch_tmap(&mw);
    prefetch_tmap(&mx);
  }
  if (warp == 0) {
    tmem_alloc(smem_u32(&s_tmem), ncols);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = s_tmem;

  if (warp == 0 && lane == 0) {
    // producer: W tile (128 features x 64 k) and x tile (bn tokens x 64 k) per stage
    int issued = 0;
    for (int i = 0; i < nkb; ++i) {
      const int s = i % stages;
      const uint32_t ph = uint32_t(i / stages) & 1u;
      if (i >= stages && !mbar_wait(smem_u32(&empty_bar[s]), ph ^ 1u)) {
        s_ok = 0;
        break;
      }
      const uint32_t a = sbase + uint32_t(s) * stage_bytes;
      mbar_expect_tx(smem_u32(&full_bar[s]), stage_bytes);
      tma_load_2d(a, &mw, smem_u32(&full_bar[s]), (kb0 + i) * kBK, mt * kBM);
      tma_load_2d(a + a_bytes, &mx, smem_u32(&full_bar[s]), (kb0 + i) * kBK, 0);
      ++issued;
    }
    // no load may still be landing in shared memory when the CTA moves on (the stages become the
    // reduction buffer, and the CTA may exit on an error path)
    for (int i = issued - stages > 0 ? issued - stages : 0; i < issued; ++i)
      if (!mbar_wait(smem_u32(&full_bar[i % stages]), uint32_t(i / stages) & 1u)) s_ok = 0;
  } else if (warp == 1 && lane == 0) {
    // MMA issuer: D[128 features][bn tokens] += W_tile x_tile^T, four K = 16 steps per stage
    const uint32_t idesc = make_idesc(kBM, bn, false, false);
    for (int i = 0; i < nkb; ++i) {
      const int s = i % stages;
      if (!mbar_wait(smem_u32(&full_bar[s]), uint32_t(i / stages) & 1u)) {
        s_ok = 0;
        break;
      }
      tc_fence_after();
      const uint32_t a = sbase + uint32_t(s) * stage_bytes;
#pragma unroll
      for (int kk = 0; kk < kBK / 16; ++kk)
        umma(tmem, desc_kmajor(a, kBM, kk), desc_kmajor(a + a_bytes, bn, kk), idesc, (i > 0 || kk > 0) ? 1u : 0u);
      umma_commit(smem_u32(&empty_bar[s]));
    }
    umma_commit(smem_u32(&acc_bar));
  }
  __syncwarp();
  if (!mbar_wait(smem_u32(&acc_bar), 0)) s_ok = 0;
  tc_fence_after();
  __syncthreads();
  const bool have_acc = nkb > 0;

  // ---- split-K reduction through distributed shared memory
  const int RS = bn + 4;                     // fp32 row stride of the reduction buffer
  float* red = reinterpret_cast<float*>(smem);
  cluster_sync_all();                        // every CTA of the cluster is done with its stages
  {
    const int r = warp * 32 + lane;          // TMEM lane = output feature of the tile
    const int seg = r / kSegRows;
    int owner = 0;
    while (owner + 1 < S && seg_lo(owner + 1, S) <= seg) ++owner;
    const int lrow = r - seg_lo(owner, S) * kSegRows;
    const uint32_t dst = map_rank(smem_u32(red + (size_t(ks) * p.rows_cap + lrow) * RS), uint32_t(owner));
    for (int c0 = 0; c0 < bn; c0 += 16) {
      uint32_t v[16];
      tmem_ld16(tmem + (uint32_t(warp * 32) << 16) + uint32_t(c0), v);
      tmem_ld_wait();
      if (!have_acc) {
#pragma unroll
        for (int i = 0; i < 16; ++i) v[i] = 0u;
      }
#pragma unroll
      for (int q = 0; q < 4; ++q)
        st_cluster_v4(dst + uint32_t((c0 + 4 * q) * 4), v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
    }
  }
  tc_fence_before();
  cluster_sync_all();                        // all partial rows have arrived at their owners

  // ---- this CTA's segments: sum the S partials in split order
  const int g_lo = seg_lo(ks, S), g_hi = seg_lo(ks + 1, S);
  const int octs = (g_hi - g_lo) * 2;        // 8-feature groups owned
  const int n = p.n;
  const int nvec = octs * n;                 // (oct, token) vectors of 8 features
  const int feat0 = mt * kBM + g_lo * kSegRows;
  const int64_t segs_total = (int64_t(p.n_out) + kSegRows - 1) / kSegRows;
  if (p.world == 1) {
    for (int v = tid; v < nvec; v += kThreads) {
      const int o = v / n, j = v - o * n;
      const int f = feat0 + o * 8;
      if (f >= p.n_out) continue;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int src = 0; src < S; ++src) {
        const float* row = red + (size_t(src) * p.rows_cap + o * 8) * RS + j;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += row[i * RS];
      }
      *reinterpret_cast<uint4*>(p.y + j * p.y_rs + f) = pack8(acc);
    }
  } else {
    // epochs of the owned segments that exist (segments past n_out are not touched)
    char* own = p.bufs[p.rank];
    const int gseg0 = mt * kSegs + g_lo;
    const int nseg = g_hi - g_lo;
    if (tid < nseg && gseg0 + tid < segs_total) {
      uint32_t* ep = reinterpret_cast<uint32_t*>(own) + gseg0 + tid;
      const uint32_t e = *ep + 1;
      *ep = e;
      s_epoch[tid] = e;
    }
    __syncthreads();
    for (int v = tid; v < nvec; v += kThreads) {
      const int o = v / n, j = v - o * n;
      const int f = feat0 + o * 8;
      if (f >= p.n_out) continue;
      float acc[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[i] = 0.f;
      for (int src = 0; src < S; ++src) {
        const float* row = red + (size_t(src) * p.rows_cap + o * 8) * RS + j;
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] += row[i * RS];
      }
      const uint4 val = pack8(acc);
      const int par = int(s_epoch[o >> 1] & 1u);
      const int64_t oct_g = f / 8;
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r >= p.world) break;
        uint4* slot = reinterpret_cast<uint4*>(p.bufs[r] + kDataOff) +
                      ((int64_t(par) * p.world + p.rank) * p.max_octs + oct_g) * p.max_rows;
        slot[j] = val;
      }
    }
    // the CTA barrier orders every thread's stores before each flag thread's system-scope release
    __syncthreads();
    if (tid < nseg * p.world) {
      const int sg = tid / p.world, dst = tid - sg * p.world;
      if (gseg0 + sg < segs_total)
        st_release_sys(flag_at(p.bufs[dst], int(s_epoch[sg] & 1u), p.rank, gseg0 + sg), s_epoch[sg]);
    }
    if (!p.push_only && tid < nseg * p.world) {
      const int sg = tid / p.world, src = tid - sg * p.world;
      if (gseg0 + sg < segs_total) {
        const uint32_t e = s_epoch[sg];
        const uint32_t* f = flag_at(own, int(e & 1u), src, gseg0 + sg);
        const volatile int32_t* verr = p.err;
        uint32_t it = 0;
        while (ld_acquire_sys(f) != e) {
          if (++it > p.spin_limit || (verr && *verr != 0)) {
            s_ok = 0;
            break;
          }
          __nanosleep(64);
        }
      }
    }
    __syncthreads();
    if (s_ok && !p.push_only) {
      for (int v = tid; v < nvec; v += kThreads) {
        const int o = v / n, j = v - o * n;
        const int f = feat0 + o * 8;
        if (f >= p.n_out) continue;
        const int par = int(s_epoch[o >> 1] & 1u);
        const int64_t oct_g = f / 8;
        float acc[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[i] = 0.f;
        for (int src = 0; src < p.world; ++src) {
          const uint4* slot = reinterpret_cast<const uint4*>(own + kDataOff) +
                              ((int64_t(par) * p.world + src) * p.max_octs + oct_g) * p.max_rows;
          add8(slot[j], acc);
        }
        *reinterpret_cast<uint4*>(p.y + j * p.y_rs + f) = pack8(acc);
      }
    }
  }
  if (!s_ok && tid == 0 && p.err) atomicExch(p.err, p.world > 1 ? 3 : 2);
  tc_fence_before();
  __syncthreads();
  if (warp == 0) tmem_dealloc(tmem, ncols);
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

// 2-D map over a [rows, k] bf16 matrix with row stride `rs` elements; box = 64 k x box_rows rows,
// 128-byte swizzle, zero fill out of bounds.
static int make_map(CUtensorMap* m, const void* base, int64_t rows, int64_t k, int64_t rs, int box_rows,
                    CUtensorMapL2promotion promo) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return fail(GDN_ERR_CUDA, "gdn_linear: cuTensorMapEncodeTiled unavailable");
  cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  cuuint64_t strides[1] = {cuuint64_t(rs) * 2};
  cuuint32_t box[2] = {uint32_t(kBK), uint32_t(box_rows)};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, promo,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(GDN_ERR_CUDA, "gdn_linear: tensor map encode failed (%d)", int(r));
  return GDN_OK;
}

struct Plan {
  int bn, stages, splits, rows_cap, m_tiles, kb_total;
  size_t smem;
};

constexpr int kMaxSmem = 202 * 1024;

static int device_id() {
  int dev = 0;
  cudaGetDevice(&dev);
  return dev;
}

static int sm_count() {
  static int sms[64] = {};
  const int dev = device_id();
  if (dev < 0 || dev >= 64) return 148;
  if (!sms[dev]) {
    int v = 0;
    if (cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || v <= 0) v = 148;
    sms[dev] = v;
  }
  return sms[dev];
}

static int set_smem_attr() {
  static bool done[64] = {};
  const int dev = device_id();
  if (dev >= 0 && dev < 64 && done[dev]) return GDN_OK;
  cudaError_t e = cudaFuncSetAttribute(linear_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_linear: setup: %s", cudaGetErrorString(e));
  if (dev >= 0 && dev < 64) done[dev] = true;
  return GDN_OK;
}

// Clusters of S CTAs with `smem` bytes each that the device holds at once (cached per device).
static int max_clusters(int S, size_t smem) {
  static int16_t cache[16][kMaxSplits + 1][kMaxSmem / 1024 + 2] = {};
  const int dev = device_id();
  const int kb = int(smem / 1024);
  const bool cacheable = dev >= 0 && dev < 16 && kb <= kMaxSmem / 1024 + 1;
  if (cacheable && cache[dev][S][kb]) return cache[dev][S][kb] - 1;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(1, unsigned(S), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = unsigned(S);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int v = 0;
  if (cudaOccupancyMaxActiveClusters(&v, linear_kernel, &cfg) != cudaSuccess) {
    cudaGetLastError();
    v = 0;
  }
  if (cacheable) cache[dev][S][kb] = int16_t(v + 1);
  return v;
}

// Ring depth, reduction buffer and shared memory of a launch with S splits.  Up to 128 tokens a
// CTA keeps about 110 KB of stages (two CTAs fit an SM), beyond that about 200 KB.
static void shape(Plan& pl, int S) {
  const size_t stage = size_t(kBM) * kBK * 2 + size_t(pl.bn) * kBK * 2;
  const size_t budget = pl.bn <= 128 ? 110 * 1024 : 200 * 1024;
  pl.splits = S;
  pl.stages = int(budget / stage);
  if (pl.stages > kMaxStages) pl.stages = kMaxStages;
  const int per = (pl.kb_total + S - 1) / S;  // no deeper ring than a split's k-blocks
  if (pl.stages > per) pl.stages = per < 2 ? 2 : per;
  pl.rows_cap = ((kSegs + S - 1) / S) * kSegRows;
  const size_t red = size_t(S) * pl.rows_cap * (pl.bn + 4) * 4;
  const size_t ring = size_t(pl.stages) * stage;
  pl.smem = (ring > red ? ring : red) + 1024;
}

// K splits: one CTA streams W at about 40 GB/s at most whatever its ring depth (TMA-bound), so
// the split count is what spreads a product over the SMs.  Measured on B200 for 16-128 tokens and
// 5,120 output features: about 16 k-blocks (1,024 k) per split is best, with at least 2 and at
// most 6 splits, and no more CTAs than about two per SM (wide outputs: one split).
//
// With a peer exchange (resident = true) every cluster must be resident at once, since a CTA that
// waits for the other ranks' segments holds its SM: the split count then drops until the device
// holds all m_tiles clusters together.
static Plan plan(int n, int n_out, int k, int splits, bool resident) {
  Plan pl{};
  pl.bn = (n + 15) / 16 * 16;
  pl.m_tiles = (n_out + kBM - 1) / kBM;
  pl.kb_total = (k + kBK - 1) / kBK;
  int S = splits;
  if (S <= 0) {
    S = (pl.kb_total + 8) / 16;
    if (S < 2) S = 2;
    if (S > 6) S = 6;
    const int by_sms = 2 * sm_count() / pl.m_tiles;
    if (S > by_sms) S = by_sms < 1 ? 1 : by_sms;
  }
  if (S > kMaxSplits) S = kMaxSplits;
  if (S > pl.kb_total) S = pl.kb_total;
  shape(pl, S);
  while (pl.smem > size_t(kMaxSmem) && S > 1) shape(pl, --S);  // a reduction buffer that does not fit
  if (resident)
    while (S > 1 && max_clusters(S, pl.smem) < pl.m_tiles) shape(pl, --S);
  return pl;
}

static int launch(const void* x, int64_t x_rs, const void* w, int64_t w_rs, void* y, int64_t y_rs, int n, int n_out,
                  int k, int splits, Params prm, cudaStream_t stream, const char* what) {
  if (n < 1 || n > kMaxTokens) return fail(GDN_ERR_ARG, "%s: n = %d tokens (1..%d)", what, n, kMaxTokens);
  if (n_out < 1 || n_out % 8) return fail(GDN_ERR_ARG, "%s: n_out = %d (a positive multiple of 8)", what, n_out);
  if (k < 1 || k % 8) return fail(GDN_ERR_ARG, "%s: k = %d (a positive multiple of 8)", what, k);
  const bool writes_y = !prm.push_only;  // a push leaves its result in the exchange buffers only
  if (!x || !w || (writes_y && !y)) return fail(GDN_ERR_ARG, "%s: null pointer", what);
  if (!aligned(x, 16) || !aligned(w, 16) || (writes_y && !aligned(y, 16)))
    return fail(GDN_ERR_ARG, "%s: x, W and y must be 16-byte aligned", what);
  if (x_rs < k || w_rs < k || x_rs % 8 || w_rs % 8 || (writes_y && (y_rs < n_out || y_rs % 8)))
    return fail(GDN_ERR_ARG, "%s: row strides (x %lld, W %lld, y %lld) must cover the rows and be multiples of 8",
                what, (long long)x_rs, (long long)w_rs, (long long)y_rs);
  if (splits < 0 || splits > kMaxSplits) return fail(GDN_ERR_ARG, "%s: splits = %d (0 = auto, 1..8)", what, splits);
  int rc = set_smem_attr();
  if (rc) return rc;
  const bool waits = prm.world > 1 && !prm.push_only;
  const Plan pl = plan(n, n_out, k, splits, waits);
  if (waits && max_clusters(pl.splits, pl.smem) < pl.m_tiles)
    return fail(GDN_ERR_SHAPE, "%s: %d tiles of %d CTAs do not fit the device at once", what, pl.m_tiles, pl.splits);
  CUtensorMap mw, mx;
  rc = make_map(&mw, w, n_out, k, w_rs, kBM, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  if (!rc) rc = make_map(&mx, x, n, k, x_rs, pl.bn, CU_TENSOR_MAP_L2_PROMOTION_L2_128B);
  if (rc) return rc;
  prm.n = n;
  prm.n_out = n_out;
  prm.kb_total = pl.kb_total;
  prm.splits = pl.splits;
  prm.bn = pl.bn;
  prm.stages = pl.stages;
  prm.rows_cap = pl.rows_cap;
  prm.y = static_cast<__nv_bfloat16*>(y);
  prm.y_rs = y_rs;
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(unsigned(pl.m_tiles), unsigned(pl.splits), 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = pl.smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 1;
  attr[0].val.clusterDim.y = unsigned(pl.splits);
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, linear_kernel, mw, mx, prm);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "%s: launch: %s", what, cudaGetErrorString(e));
  return check_launch(what);
}

}  // namespace lin
}  // namespace gdn

using namespace gdn;

extern "C" int gdn_linear(const void* x, int64_t x_rs, const void* w, int64_t w_rs, void* y, int64_t y_rs, int n,
                          int n_out, int k, int splits, int dtype, int32_t* err_flag, void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_linear: dtype %d (bf16 only)", dtype);
  lin::Params prm{};
  prm.rank = 0;
  prm.world = 1;
  prm.err = err_flag;
  return lin::launch(x, x_rs, w, w_rs, y, y_rs, n, n_out, k, splits, prm, as_stream(stream), "gdn_linear");
}

extern "C" int gdn_linear_plan(int n, int n_out, int k, int splits, int world, int32_t* out) {
  if (!out || n < 1 || n > lin::kMaxTokens || n_out < 1 || k < 1 || splits < 0 || splits > lin::kMaxSplits ||
      world < 1)
    return fail(GDN_ERR_ARG, "gdn_linear_plan: bad arguments");
  int rc = lin::set_smem_attr();
  if (rc) return rc;
  const lin::Plan pl = lin::plan(n, n_out, k, splits, world > 1);
  out[0] = pl.splits;
  out[1] = pl.stages;
  out[2] = int32_t(pl.smem);
  out[3] = pl.m_tiles;
  out[4] = pl.kb_total;
  return GDN_OK;
}

extern "C" size_t gdn_linear_ar_buffer_bytes(int world, int max_rows, int max_out, int dtype) {
  if (world < 1 || world > lin::kMaxWorld || dtype != GDN_BF16) return 0;
  if (max_rows < 1 || max_rows > lin::kMaxTokens || max_out < 8 || max_out > lin::kMaxSegs * lin::kSegRows)
    return 0;
  if (max_out % 8) return 0;
  const size_t slot = size_t(max_out / 8) * size_t(max_rows) * 16;
  return lin::kDataOff + 2 * size_t(world) * slot;
}

extern "C" int gdn_linear_allreduce(const void* x, int64_t x_rs, const void* w, int64_t w_rs, void* y, int64_t y_rs,
                                    int n, int n_out, int k, int splits, int rank, int world, void* const* bufs,
                                    int max_rows, int max_out, uint32_t spin_limit, int32_t* err_flag, int dtype,
                                    void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_linear_allreduce: dtype %d (bf16 only)", dtype);
  if (world < 1 || world > lin::kMaxWorld || rank < 0 || rank >= world)
    return fail(GDN_ERR_ARG, "gdn_linear_allreduce: rank %d of %d (world 1..%d)", rank, world, lin::kMaxWorld);
  if (n > max_rows) return fail(GDN_ERR_ARG, "gdn_linear_allreduce: %d tokens > buffer rows %d", n, max_rows);
  if (world > 1 && (n_out > max_out || max_out % 8 || max_out > lin::kMaxSegs * lin::kSegRows || max_rows < 1 ||
                    max_rows > lin::kMaxTokens))
    return fail(GDN_ERR_ARG, "gdn_linear_allreduce: n_out %d does not fit the buffers (max_out %d, max_rows %d)", n_out,
                max_out, max_rows);
  lin::Params prm{};
  prm.rank = rank;
  prm.world = world;
  prm.max_rows = max_rows;
  prm.max_octs = max_out / 8;
  prm.spin_limit = spin_limit ? spin_limit : (1u << 22);
  prm.err = err_flag;
  if (world > 1) {
    if (!bufs) return fail(GDN_ERR_ARG, "gdn_linear_allreduce: null buffer table");
    for (int r = 0; r < world; ++r) {
      if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_linear_allreduce: buffer %d", r);
      prm.bufs[r] = static_cast<char*>(bufs[r]);
    }
  }
  return lin::launch(x, x_rs, w, w_rs, y, y_rs, n, n_out, k, splits, prm, as_stream(stream), "gdn_linear_allreduce");
}

// ---------------------------------------------------------------------------------------------
// Residual add fused with the next RMSNorm, and (PULL) with the sum over ranks of pushed partials.
//
//   h   = PULL ? bf16(sum over src, rank order, of fp32(data[src] row j))   (the all-reduce output)
//              : h[j]                                                          (this rank's GEMM output)
//   x[j] = bf16(x[j] + h)                                     (the residual stream, updated in place)
//   out[j] = bf16((x[j] * rsqrt(mean(x[j]^2) + eps)) * (1 + w))
//
// One CTA of 128 threads per token row, with exactly the element-to-thread map, summation order
// and arithmetic of rmsnorm_kernel, so the result is bit for bit that of the unfused sequence
// all-reduce -> x + h -> Qwen3_5RMSNorm (src/cb_engine.py:295-355 runs them as separate ops).
namespace gdn {
namespace lin {

struct AddNormParams {
  __nv_bfloat16* x;
  int64_t x_rs;
  const __nv_bfloat16* h;
  int64_t h_rs;
  const __nv_bfloat16* w;
  __nv_bfloat16* out;
  int64_t out_rs;
  int dim;
  float eps;
  int rank, world;
  char* bufs[kMaxWorld];
  int64_t max_rows, max_octs;
  uint32_t spin_limit;
  int32_t* err;
};

template <bool PULL>
__global__ void __launch_bounds__(128) add_rmsnorm_kernel(const AddNormParams p) {
  constexpr int NV = 8192 / (128 * 8);  // 8-element groups per thread at the largest dim
  __shared__ float red[4];
  __shared__ int s_ok;
  const int tid = threadIdx.x, j = blockIdx.x;
  const int octs = p.dim / 8;
  char* own = PULL ? p.bufs[p.rank] : nullptr;
  if (PULL) {
    // every rank's partial of every segment of the row must be here: poll all the row's flags with
    // relaxed loads issued together (no ordering between them), round after round (bounded), then
    // one system-scope fence orders the data reads after the flags
    if (tid == 0) s_ok = 1;
    const int nseg = (p.dim + kSegRows - 1) / kSegRows;
    const volatile int32_t* verr = p.err;
    for (uint32_t it = 0;; ++it) {
      int mine = 1;
      for (int idx = tid; idx < nseg * p.world; idx += 128) {
        const int g = idx / p.world, src = idx - g * p.world;
        const uint32_t e = reinterpret_cast<const uint32_t*>(own)[g];
        mine &= ld_relaxed_sys(flag_at(own, int(e & 1u), src, g)) == e;
      }
      if (__syncthreads_and(mine)) break;
      // give up together (block-uniform) when the limit is reached or another call already failed
      if (__syncthreads_or(it > p.spin_limit || (verr && *verr != 0))) {
        if (tid == 0) s_ok = 0;
        break;
      }
      __nanosleep(64);
    }
    fence_acq_rel_sys();
    __syncthreads();
    if (!s_ok) {  // a rank did not arrive: report it and leave x and out alone
      if (tid == 0 && p.err) atomicExch(p.err, 3);
      return;
    }
  }
  __nv_bfloat16* xr = p.x + int64_t(j) * p.x_rs;
  // every load of the row first (x, h or the ranks' partials, and the norm weight), then the
  // stores: the in-place store of x must not hold back the loads behind it
  uint4 xu[NV], wu[NV];
  float xv[NV][8];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      xu[v] = *reinterpret_cast<const uint4*>(xr + o * 8);
      wu[v] = *reinterpret_cast<const uint4*>(p.w + o * 8);
#pragma unroll
      for (int i = 0; i < 8; ++i) xv[v][i] = 0.f;
      if (PULL) {
        const uint32_t e = reinterpret_cast<const uint32_t*>(own)[o >> 1];
        const int par = int(e & 1u);
        for (int src = 0; src < p.world; ++src) {
          const uint4 u = reinterpret_cast<const uint4*>(own + kDataOff)[((int64_t(par) * p.world + src) * p.max_octs + o) *
                                                                         p.max_rows + j];
          add8(u, xv[v]);
        }
      } else {
        add8(*reinterpret_cast<const uint4*>(p.h + int64_t(j) * p.h_rs + o * 8), xv[v]);
      }
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      float xin[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) xin[i] = 0.f;
      add8(xu[v], xin);
      // h rounded to bf16 (the all-reduce output, or the GEMM output as given), then x + h rounded
#pragma unroll
      for (int i = 0; i < 8; ++i)
        xv[v][i] = __bfloat162float(__float2bfloat16_rn(xin[i] + __bfloat162float(__float2bfloat16_rn(xv[v][i]))));
      *reinterpret_cast<uint4*>(xr + o * 8) = pack8(xv[v]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += xv[v][i] * xv[v][i];
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  const float r = 1.0f / sqrtf((red[0] + red[1] + red[2] + red[3]) / float(p.dim) + p.eps);
  __nv_bfloat16* yr = p.out + int64_t(j) * p.out_rs;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      float wv[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) wv[i] = 0.f;
      add8(wu[v], wv);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = (xv[v][i] * r) * (1.0f + wv[i]);
      *reinterpret_cast<uint4*>(yr + o * 8) = pack8(y);
    }
  }
}

// The push half of the exchange for a product computed elsewhere (a library GEMM): y [n, n_out]
// bf16 goes, tile of 128 features by tile, into this rank's slot of every rank's exchange buffer,
// with the same per-segment epochs, parity slots and flags as gdn_linear_push.  One CTA per tile.
__global__ void __launch_bounds__(128) push_kernel(const __nv_bfloat16* __restrict__ y, int64_t y_rs, int n,
                                                   int n_out, const Params p) {
  __shared__ uint32_t s_epoch[kSegs];
  const int tid = threadIdx.x, mt = blockIdx.x;
  const int gseg0 = mt * kSegs;
  const int segs_total = (n_out + kSegRows - 1) / kSegRows;
  const int nseg = segs_total - gseg0 < kSegs ? segs_total - gseg0 : kSegs;
  char* own = p.bufs[p.rank];
  if (tid < nseg) {
    uint32_t* ep = reinterpret_cast<uint32_t*>(own) + gseg0 + tid;
    const uint32_t e = *ep + 1;
    *ep = e;
    s_epoch[tid] = e;
  }
  __syncthreads();
  const int nvec = 2 * nseg * n;  // (8-feature group, token) vectors, token fastest
  for (int v = tid; v < nvec; v += 128) {
    const int o = v / n, j = v - o * n;
    const int f = mt * kBM + o * 8;
    if (f >= n_out) continue;
    const uint4 val = *reinterpret_cast<const uint4*>(y + int64_t(j) * y_rs + f);
    const int par = int(s_epoch[o >> 1] & 1u);
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r) {
      if (r >= p.world) break;
      reinterpret_cast<uint4*>(p.bufs[r] + kDataOff)[((int64_t(par) * p.world + p.rank) * p.max_octs + f / 8) *
                                                     p.max_rows + j] = val;
    }
  }
  __syncthreads();  // every thread's stores before the flag threads' system-scope release
  if (tid < nseg * p.world) {
    const int sg = tid / p.world, dst = tid - sg * p.world;
    st_release_sys(flag_at(p.bufs[dst], int(s_epoch[sg] & 1u), p.rank, gseg0 + sg), s_epoch[sg]);
  }
}

static int check_add_norm(const void* x, int64_t x_rs, const void* w, const void* out, int64_t out_rs, int64_t rows,
                          int dim, int dtype, const char* what) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "%s: dtype %d (bf16 only)", what, dtype);
  if (rows < 1 || rows > 0x7fffffffLL || dim < 8 || dim > 8192 || dim % 8)
    return fail(GDN_ERR_ARG, "%s: rows %lld, dim %d (a multiple of 8, <= 8192)", what, (long long)rows, dim);
  if (!x || !w || !out) return fail(GDN_ERR_ARG, "%s: null pointer", what);
  if (!aligned(x, 16) || !aligned(w, 16) || !aligned(out, 16) || x_rs % 8 || out_rs % 8 || x_rs < dim ||
      out_rs < dim)
    return fail(GDN_ERR_ARG, "%s: 16-byte aligned rows with strides that are multiples of 8 needed", what);
  return GDN_OK;
}

}  // namespace lin
}  // namespace gdn

extern "C" int gdn_add_rmsnorm(void* x, int64_t x_rs, const void* h, int64_t h_rs, const void* weight, void* out,
                               int64_t out_rs, int64_t rows, int dim, float eps, int dtype, void* stream) {
  int rc = lin::check_add_norm(x, x_rs, weight, out, out_rs, rows, dim, dtype, "gdn_add_rmsnorm");
  if (rc) return rc;
  if (!h || !aligned(h, 16) || h_rs % 8 || h_rs < dim) return fail(GDN_ERR_ARG, "gdn_add_rmsnorm: h rows");
  lin::AddNormParams p{};
  p.x = static_cast<__nv_bfloat16*>(x);
  p.x_rs = x_rs;
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.h_rs = h_rs;
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_rs = out_rs;
  p.dim = dim;
  p.eps = eps;
  p.world = 1;
  lin::add_rmsnorm_kernel<false><<<unsigned(rows), 128, 0, as_stream(stream)>>>(p);
  return check_launch("gdn_add_rmsnorm");
}

extern "C" int gdn_linear_push(const void* x, int64_t x_rs, const void* w, int64_t w_rs, int n, int n_out, int k,
                               int splits, int rank, int world, void* const* bufs, int max_rows, int max_out,
                               int32_t* err_flag, int dtype, void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_linear_push: dtype %d (bf16 only)", dtype);
  if (world < 2 || world > lin::kMaxWorld || rank < 0 || rank >= world)
    return fail(GDN_ERR_ARG, "gdn_linear_push: rank %d of %d (world 2..%d)", rank, world, lin::kMaxWorld);
  if (n > max_rows || n_out > max_out || max_out % 8 || max_out > lin::kMaxSegs * lin::kSegRows || max_rows < 1 ||
      max_rows > lin::kMaxTokens)
    return fail(GDN_ERR_ARG, "gdn_linear_push: %d x %d does not fit the buffers (max_rows %d, max_out %d)", n, n_out,
                max_rows, max_out);
  if (!bufs) return fail(GDN_ERR_ARG, "gdn_linear_push: null buffer table");
  lin::Params prm{};
  prm.rank = rank;
  prm.world = world;
  prm.max_rows = max_rows;
  prm.max_octs = max_out / 8;
  prm.err = err_flag;
  prm.push_only = 1;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_linear_push: buffer %d", r);
    prm.bufs[r] = static_cast<char*>(bufs[r]);
  }
  return lin::launch(x, x_rs, w, w_rs, nullptr, 0, n, n_out, k, splits, prm, as_stream(stream), "gdn_linear_push");
}

extern "C" int gdn_push_partial(const void* y, int64_t y_rs, int n, int n_out, int rank, int world,
                                void* const* bufs, int max_rows, int max_out, int dtype, void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_push_partial: dtype %d (bf16 only)", dtype);
  if (world < 2 || world > lin::kMaxWorld || rank < 0 || rank >= world || !bufs)
    return fail(GDN_ERR_ARG, "gdn_push_partial: rank %d of %d (world 2..%d)", rank, world, lin::kMaxWorld);
  if (n < 1 || n_out < 8 || n_out % 8 || n > max_rows || n_out > max_out || max_out % 8 ||
      max_out > lin::kMaxSegs * lin::kSegRows || max_rows > lin::kMaxTokens)
    return fail(GDN_ERR_ARG, "gdn_push_partial: %d x %d does not fit the buffers (max_rows %d, max_out %d)", n, n_out,
                max_rows, max_out);
  if (!y || !aligned(y, 16) || y_rs % 8 || y_rs < n_out) return fail(GDN_ERR_ARG, "gdn_push_partial: y rows");
  lin::Params prm{};
  prm.rank = rank;
  prm.world = world;
  prm.max_rows = max_rows;
  prm.max_octs = max_out / 8;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_push_partial: buffer %d", r);
    prm.bufs[r] = static_cast<char*>(bufs[r]);
  }
  lin::push_kernel<<<unsigned((n_out + lin::kBM - 1) / lin::kBM), 128, 0, as_stream(stream)>>>(
      static_cast<const __nv_bfloat16*>(y), y_rs, n, n_out, prm);
  return check_launch("gdn_push_partial");
}

extern "C" int gdn_pull_add_rmsnorm(void* x, int64_t x_rs, const void* weight, void* out, int64_t out_rs, int64_t rows,
                                    int dim, float eps, int rank, int world, void* const* bufs, int max_rows,
                                    int max_out, uint32_t spin_limit, int32_t* err_flag, int dtype, void* stream) {
  int rc = lin::check_add_norm(x, x_rs, weight, out, out_rs, rows, dim, dtype, "gdn_pull_add_rmsnorm");
  if (rc) return rc;
  if (world < 2 || world > lin::kMaxWorld || rank < 0 || rank >= world || !bufs)
    return fail(GDN_ERR_ARG, "gdn_pull_add_rmsnorm: rank %d of %d (world 2..%d)", rank, world, lin::kMaxWorld);
  if (rows > max_rows || dim > max_out || max_out % 8)
    return fail(GDN_ERR_ARG, "gdn_pull_add_rmsnorm: %lld x %d does not fit the buffers", (long long)rows, dim);
  lin::AddNormParams p{};
  p.x = static_cast<__nv_bfloat16*>(x);
  p.x_rs = x_rs;
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_rs = out_rs;
  p.dim = dim;
  p.eps = eps;
  p.rank = rank;
  p.world = world;
  p.max_rows = max_rows;
  p.max_octs = max_out / 8;
  p.spin_limit = spin_limit ? spin_limit : (1u << 22);
  p.err = err_flag;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_pull_add_rmsnorm: buffer %d", r);
    p.bufs[r] = static_cast<char*>(bufs[r]);
  }
  lin::add_rmsnorm_kernel<true><<<unsigned(rows), 128, 0, as_stream(stream)>>>(p);
  return check_launch("gdn_pull_add_rmsnorm");
}

// ---------------------------------------------------------------------------------------------
// All-reduce fused into its consumer: the row-parallel projection's sum over ranks, the residual
// add and the next RMSNorm (AllReduceLinear's dist.all_reduce, x + h and Qwen3_5RMSNorm,
// src/cb_tp.py:25-35, src/cb_engine.py:295-355) in one kernel, one CTA per token row:
//   1. this rank's partial row y[j] goes into its slot of every rank's buffer (plain 16-byte stores
//      over NVLink), then one flag per (row, destination) is raised with a system-scope release;
//   2. the row's flags from every other rank are polled (relaxed loads, bounded, block-uniform
//      give-up) and one system-scope fence orders the reads after them;
//   3. h = bf16(sum of the ranks' partials in rank order, fp32); x[j] = bf16(x[j] + h) in place;
//      out[j] = bf16(x[j] * rsqrt(mean(x[j]^2) + eps) * (1 + w)) with gdn_rmsnorm's arithmetic,
// bit for bit gdn_allreduce -> x + h -> gdn_rmsnorm.  Buffer of one rank:
//   [0, 1 KiB) epoch[kMaxTokens]; [1 KiB, 1 KiB + 16 KiB) flag[2][kMaxWorld][kMaxTokens];
//   [kArDataOff, ...) data[2][world][max_rows][dim] bf16 (dim fixed for the buffer's lifetime).
// The epoch of row j counts the calls that touched it, identically on every rank; parity
// double-buffers the data as in the exchange above.
namespace gdn {
namespace lin {

constexpr size_t kArFlagOff = 1024;
constexpr size_t kArDataOff = kArFlagOff + size_t(2) * kMaxWorld * kMaxTokens * 4;
static_assert(kMaxTokens * 4 <= kArFlagOff, "row epochs");

__device__ __forceinline__ uint32_t* arflag_at(char* buf, int p, int src, int j) {
  return reinterpret_cast<uint32_t*>(buf + kArFlagOff) + (size_t(p) * kMaxWorld + src) * kMaxTokens + j;
}

__global__ void __launch_bounds__(128) ar_add_rmsnorm_kernel(const AddNormParams p) {
  constexpr int NV = 8192 / (128 * 8);
  __shared__ float red[4];
  __shared__ uint32_t s_e;
  __shared__ int s_ok;
  const int tid = threadIdx.x, j = blockIdx.x;
  const int octs = p.dim / 8;
  char* own = p.bufs[p.rank];
  if (tid == 0) {
    uint32_t* ep = reinterpret_cast<uint32_t*>(own) + j;
    s_e = *ep + 1;
    *ep = s_e;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_e;
  const int par = int(e & 1u);
  auto slot = [&](char* buf, int src) {
    return reinterpret_cast<uint4*>(buf + kArDataOff) + ((int64_t(par) * p.world + src) * p.max_rows + j) * octs;
  };
  __nv_bfloat16* xr = p.x + int64_t(j) * p.x_rs;
  uint4 hu[NV], xu[NV], wu[NV];
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      hu[v] = *reinterpret_cast<const uint4*>(p.h + int64_t(j) * p.h_rs + o * 8);
      xu[v] = *reinterpret_cast<const uint4*>(xr + o * 8);
      wu[v] = *reinterpret_cast<const uint4*>(p.w + o * 8);
#pragma unroll
      for (int r = 0; r < kMaxWorld; ++r) {
        if (r >= p.world) break;
        if (r != p.rank) slot(p.bufs[r], p.rank)[o] = hu[v];
      }
    }
  }
  __syncthreads();  // every thread's stores before the flag threads' system-scope release
  if (tid < p.world && tid != p.rank) st_release_sys(arflag_at(p.bufs[tid], par, p.rank, j), e);
  // only the world - 1 polling threads wait, each with acquire loads on its source's flag; the CTA
  // barrier after them orders every thread's reads (no fence in the other threads)
  if (tid < p.world && tid != p.rank) {
    const uint32_t* f = arflag_at(own, par, tid, j);
    const volatile int32_t* verr = p.err;
    uint32_t it = 0;
    while (ld_acquire_sys(f) != e) {
      if (++it > p.spin_limit || (verr && *verr != 0)) {
        s_ok = 0;
        break;
      }
      __nanosleep(32);
    }
  }
  __syncthreads();
  if (!s_ok) {  // a rank did not arrive: report it and leave x and out alone
    if (tid == 0 && p.err) atomicExch(p.err, 3);
    return;
  }
  float xv[NV][8];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      float hv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      for (int src = 0; src < p.world; ++src) add8(src == p.rank ? hu[v] : slot(own, src)[o], hv);
      float xin[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      add8(xu[v], xin);
#pragma unroll
      for (int i = 0; i < 8; ++i)
        xv[v][i] = __bfloat162float(__float2bfloat16_rn(xin[i] + __bfloat162float(__float2bfloat16_rn(hv[i]))));
      *reinterpret_cast<uint4*>(xr + o * 8) = pack8(xv[v]);
#pragma unroll
      for (int i = 0; i < 8; ++i) ss += xv[v][i] * xv[v][i];
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  const float r = 1.0f / sqrtf((red[0] + red[1] + red[2] + red[3]) / float(p.dim) + p.eps);
  __nv_bfloat16* yr = p.out + int64_t(j) * p.out_rs;
#pragma unroll
  for (int v = 0; v < NV; ++v) {
    const int o = v * 128 + tid;
    if (o < octs) {
      float wv[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
      add8(wu[v], wv);
      float y[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) y[i] = (xv[v][i] * r) * (1.0f + wv[i]);
      *reinterpret_cast<uint4*>(yr + o * 8) = pack8(y);
    }
  }
}

}  // namespace lin
}  // namespace gdn

extern "C" size_t gdn_ar_norm_buffer_bytes(int world, int max_rows, int dim, int dtype) {
  if (world < 1 || world > lin::kMaxWorld || dtype != GDN_BF16 || max_rows < 1 || max_rows > lin::kMaxTokens ||
      dim < 8 || dim > 8192 || dim % 8)
    return 0;
  return lin::kArDataOff + 2 * size_t(world) * size_t(max_rows) * size_t(dim) * 2;
}

extern "C" int gdn_allreduce_add_rmsnorm(void* x, int64_t x_rs, const void* h, int64_t h_rs, const void* weight,
                                         void* out, int64_t out_rs, int64_t rows, int dim, float eps, int rank,
                                         int world, void* const* bufs, int max_rows, uint32_t spin_limit,
                                         int32_t* err_flag, int dtype, void* stream) {
  int rc = lin::check_add_norm(x, x_rs, weight, out, out_rs, rows, dim, dtype, "gdn_allreduce_add_rmsnorm");
  if (rc) return rc;
  if (!h || !aligned(h, 16) || h_rs % 8 || h_rs < dim) return fail(GDN_ERR_ARG, "gdn_allreduce_add_rmsnorm: h rows");
  if (world < 2 || world > lin::kMaxWorld || rank < 0 || rank >= world || !bufs)
    return fail(GDN_ERR_ARG, "gdn_allreduce_add_rmsnorm: rank %d of %d (world 2..%d)", rank, world, lin::kMaxWorld);
  if (rows > max_rows || max_rows > lin::kMaxTokens)
    return fail(GDN_ERR_ARG, "gdn_allreduce_add_rmsnorm: %lld rows > buffer rows %d", (long long)rows, max_rows);
  lin::AddNormParams p{};
  p.x = static_cast<__nv_bfloat16*>(x);
  p.x_rs = x_rs;
  p.h = static_cast<const __nv_bfloat16*>(h);
  p.h_rs = h_rs;
  p.w = static_cast<const __nv_bfloat16*>(weight);
  p.out = static_cast<__nv_bfloat16*>(out);
  p.out_rs = out_rs;
  p.dim = dim;
  p.eps = eps;
  p.rank = rank;
  p.world = world;
  p.max_rows = max_rows;
  p.spin_limit = spin_limit ? spin_limit : (1u << 22);
  p.err = err_flag;
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_allreduce_add_rmsnorm: buffer %d", r);
    p.bufs[r] = static_cast<char*>(bufs[r]);
  }
  lin::ar_add_rmsnorm_kernel<<<unsigned(rows), 128, 0, as_stream(stream)>>>(p);
  return check_launch("gdn_allreduce_add_rmsnorm");
}
