// Peer-memory all-reduce (sum) for the row-parallel projections of the tensor-parallel engine:
// the collective after out_proj / o_proj / down_proj (src/cb_tp.py:25-35) at decode sizes, where
// a library all-reduce is latency-bound.  One process per GPU; each rank owns one device buffer
// (gdn_ar_alloc) whose IPC handle the other ranks open (gdn_ar_ipc_open), so every rank holds
// plain pointers to all buffers of the node.  No multicast objects and no bulk/TMA copies of peer
// memory are used: the kernel moves data with ordinary 16-byte stores over NVLink.
//
// Buffer layout (per rank):
//   [0, 512)           per-CTA epoch counters of this rank's calls (local use only)
//   [512, 512 + 8 KiB) flags[2][kMaxWorld][kMaxCtas] u32: flags[p][src][cta] = epoch from src
//   [kDataOff, ...)    data[2][world][slot] 16-byte vectors: data[p][src] = src's partial sums
// One call (one-shot): the grid depends only on the buffer's capacity, so every CTA takes part in
// every call and CTA c's epoch e counts the calls (the same on every rank, since every rank makes
// the same calls).  CTA c takes a contiguous range of the call's vectors (possibly empty); it stores
// its range of x into data[e & 1][rank] of every rank, raises flags[e & 1][rank][c] = e on every
// rank with a system-scope release store, waits (bounded) until flags[e & 1][src][c] == e for
// every src on its own buffer, then sums data[e & 1][0..world-1] in rank order in fp32 and writes
// y.  Every rank therefore computes the identical result.  Parity e & 1 double-buffers the slots:
// a rank can write call e + 2's data only after it has seen every rank's flags of call e + 1,
// which each rank raises after its call e kernel (and all its reads) completed.
#include <cstring>

#include "common.cuh"

namespace gdn {
namespace ar {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 128;
constexpr int kThreads = 512;
constexpr int kVecsPerCta = 1024;  // 16-byte vectors per CTA before the grid grows
constexpr size_t kFlagOff = 512;
constexpr size_t kDataOff = 16384;
static_assert(kFlagOff >= kMaxCtas * 4 && kFlagOff + 2 * kMaxWorld * kMaxCtas * 4 <= kDataOff, "layout");

struct Peers {
  char* buf[kMaxWorld];
};

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t* flag_at(char* buf, int p, int src, int cta) {
  return reinterpret_cast<uint32_t*>(buf + kFlagOff) + (p * kMaxWorld + src) * kMaxCtas + cta;
}

// bf16 x 8 <-> fp32 x 8
__device__ __forceinline__ void add8(const uint4& u, float* acc) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    acc[2 * i] += __uint_as_float(w[i] << 16);
    acc[2 * i + 1] += __uint_as_float(w[i] & 0xffff0000u);
  }
}
__device__ __forceinline__ uint4 pack8(const float* a) {
  uint32_t w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t lo = __bfloat16_as_ushort(__float2bfloat16_rn(a[2 * i]));
    const uint32_t hi = __bfloat16_as_ushort(__float2bfloat16_rn(a[2 * i + 1]));
    w[i] = lo | (hi << 16);
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

__global__ void __launch_bounds__(kThreads) allreduce_bf16_kernel(const uint4* x, uint4* y, int64_t nvec,
                                                                  int64_t slot_vecs, int rank, int world, Peers peers,
                                                                  uint32_t spin_limit, int32_t* err) {
  __shared__ uint32_t s_epoch;
  __shared__ int s_ok;
  const int c = blockIdx.x, tid = threadIdx.x;
  char* own = peers.buf[rank];
  if (tid == 0) {
    uint32_t* counter = reinterpret_cast<uint32_t*>(own) + c;
    const uint32_t e = *counter + 1;
    *counter = e;
    s_epoch = e;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t e = s_epoch;
  const int p = int(e & 1u);
  const int64_t per = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = int64_t(c) * per;
  const int64_t v1 = v0 + per < nvec ? v0 + per : nvec;
  auto slot = [&](char* buf, int src) {
    return reinterpret_cast<uint4*>(buf + kDataOff) + (int64_t(p) * world + src) * slot_vecs;
  };
  // push this CTA's range of the local partial into every rank's slot [rank]
  for (int64_t v = v0 + tid; v < v1; v += kThreads) {
    const uint4 val = x[v];
#pragma unroll
    for (int r = 0; r < kMaxWorld; ++r)
      if (r < world) slot(peers.buf[r], rank)[v] = val;
  }
  // the CTA barrier orders every thread's stores before thread r's system-scope release of the
  // flag on rank r (release is cumulative), and the reader's acquire + barrier orders its reads
  // after it; a fence in every thread would add a round trip per thread (measured: 14.5 -> 8.6 us)
  __syncthreads();
  if (tid < world) st_release_sys(flag_at(peers.buf[tid], p, rank, c), e);
  // wait until every rank's range has arrived here; give up at once when an earlier call of this
  // instance already ran out (the ranks are then out of step for good)
  if (tid < world) {
    const uint32_t* f = flag_at(own, p, tid, c);
    const volatile int32_t* verr = err;
    uint32_t it = 0;
    while (ld_acquire_sys(f) != e) {
      if (++it > spin_limit || (verr && *verr != 0)) {
        s_ok = 0;
        break;
      }
      __nanosleep(64);
    }
  }
  __syncthreads();
  if (!s_ok) {  // a rank did not arrive in time: report it and leave y alone
    if (tid == 0 && err) atomicExch(err, 3);
    return;
  }
  for (int64_t v = v0 + tid; v < v1; v += kThreads) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < world; ++s) add8(slot(own, s)[v], acc);
    y[v] = pack8(acc);
  }
}

}  // namespace ar
}  // namespace gdn

using namespace gdn;

extern "C" size_t gdn_ar_buffer_bytes(int world, size_t max_elems, int dtype) {
  if (world < 1 || world > ar::kMaxWorld || dtype != GDN_BF16) return 0;
  const size_t slot = (max_elems * 2 + 15) / 16 * 16;
  return ar::kDataOff + 2 * size_t(world) * slot;
}

extern "C" int gdn_ar_alloc(size_t bytes, void** ptr) {
  if (!ptr || bytes < ar::kDataOff) return fail(GDN_ERR_ARG, "gdn_ar_alloc: %zu bytes", bytes);
  *ptr = nullptr;
  cudaError_t e = cudaMalloc(ptr, bytes);
  if (e == cudaSuccess) e = cudaMemset(*ptr, 0, bytes);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_ar_alloc: %s", cudaGetErrorString(e));
  return GDN_OK;
}

extern "C" int gdn_ar_free(void* ptr) {
  if (!ptr) return GDN_OK;
  cudaError_t e = cudaFree(ptr);
  return e == cudaSuccess ? GDN_OK : fail(GDN_ERR_CUDA, "gdn_ar_free: %s", cudaGetErrorString(e));
}

extern "C" int gdn_ar_ipc_handle(void* ptr, void* handle) {
  if (!ptr || !handle) return fail(GDN_ERR_ARG, "gdn_ar_ipc_handle: null pointer");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, ptr);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_ar_ipc_handle: %s", cudaGetErrorString(e));
  static_assert(sizeof(cudaIpcMemHandle_t) == GDN_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  return GDN_OK;
}

extern "C" int gdn_ar_ipc_open(const void* handle, void** ptr) {
  if (!ptr || !handle) return fail(GDN_ERR_ARG, "gdn_ar_ipc_open: null pointer");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  *ptr = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_ar_ipc_open: %s", cudaGetErrorString(e));
  return GDN_OK;
}

extern "C" int gdn_ar_ipc_close(void* ptr) {
  if (!ptr) return GDN_OK;
  cudaError_t e = cudaIpcCloseMemHandle(ptr);
  return e == cudaSuccess ? GDN_OK : fail(GDN_ERR_CUDA, "gdn_ar_ipc_close: %s", cudaGetErrorString(e));
}

extern "C" int gdn_allreduce(const void* x, void* y, size_t n, int dtype, int rank, int world, void* const* bufs,
                             size_t max_elems, uint32_t spin_limit, int32_t* err_flag, void* stream) {
  if (dtype != GDN_BF16) return fail(GDN_ERR_DTYPE, "gdn_allreduce: dtype %d (bf16 only)", dtype);
  if (world < 1 || world > ar::kMaxWorld || rank < 0 || rank >= world)
    return fail(GDN_ERR_ARG, "gdn_allreduce: rank %d of %d (world 1..%d)", rank, world, ar::kMaxWorld);
  if (n == 0) return GDN_OK;
  if (!x || !y || !bufs) return fail(GDN_ERR_ARG, "gdn_allreduce: null pointer");
  if (n > max_elems) return fail(GDN_ERR_ARG, "gdn_allreduce: %zu elements > buffer slot of %zu", n, max_elems);
  if ((n * 2) % 16 || !aligned(x, 16) || !aligned(y, 16))
    return fail(GDN_ERR_ARG, "gdn_allreduce: x, y must be 16-byte aligned and n a multiple of 8");
  ar::Peers peers{};
  for (int r = 0; r < world; ++r) {
    if (!bufs[r] || !aligned(bufs[r], 16)) return fail(GDN_ERR_ARG, "gdn_allreduce: buffer %d", r);
    peers.buf[r] = static_cast<char*>(bufs[r]);
  }
  const int64_t nvec = int64_t(n * 2 / 16);
  const int64_t slot_vecs = int64_t((max_elems * 2 + 15) / 16);
  // from the capacity, not from n: every call runs every CTA, so all CTAs of a call share its epoch
  int64_t ctas = (slot_vecs + ar::kVecsPerCta - 1) / ar::kVecsPerCta;
  if (ctas > ar::kMaxCtas) ctas = ar::kMaxCtas;
  ar::allreduce_bf16_kernel<<<int(ctas), ar::kThreads, 0, as_stream(stream)>>>(
      static_cast<const uint4*>(x), static_cast<uint4*>(y), nvec, slot_vecs, rank, world, peers,
      spin_limit ? spin_limit : (1u << 22), err_flag);
  return check_launch("gdn_allreduce");
}
