// gdn_decode_layer_noalloc: the fused decode layer for callers that cannot allocate device memory.
//
// Some hosts of this library never let a plugin call cudaMalloc: a serving runtime that owns the
// whole device-memory budget and hands plugins only the tensors they work on, or a latency-bound
// decode loop where cudaMalloc's implicit device synchronisation is not acceptable.  Such a
// caller still owns every input and output, but it has no way to provide the workspace that
// gdn_decode_layer needs (for dk = dv = 128 the prepared q/k/v rows and gates passed from its
// first kernel to its second; for dk = dv = 64 the counters that order the updates of the q/k
// conv windows shared by the value heads of one k-head).  This entry point takes that workspace
// from a fixed-size array in device memory that belongs to the library instead.
//
// The array (kNoAllocScratchBytes) lives in every GPU that loads the library until the process
// exits.  It has two parts that never overlap:
//   * bytes [0, kPrepBytes): the prepared rows and gates of dk = dv = 128 calls.  Every call
//     writes them before it reads them, so what an earlier call left there does not matter.
//   * bytes [kPrepBytes, kNoAllocScratchBytes): the ticket counters of dk = dv = 64 calls.  They
//     must be zero when a call starts.  The array is zero when the library loads, no dk = 128
//     call writes this part, and every dk = 64 call that runs to its end returns each counter it
//     used to zero (a call stopped by a bad slot index takes no ticket).
// Its device address is looked up once per device, on the first call made with that device
// current; make that first call before any stream capture.  The cached address belongs to the
// device's primary context: do not use this entry point across a cudaDeviceReset of that device.
// All calls on a device share the one array and it keeps whatever the last call left there.  Two
// calls whose kernels overlap on the GPU (different streams, no ordering between them) race on
// the array.  Requests larger than their part are rejected with GDN_ERR_WORKSPACE; nothing here
// calls cudaMalloc, cudaFree or any allocating library routine.
#include <mutex>

#include "common.cuh"

namespace gdn {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;  // 8 MiB per GPU
constexpr size_t kTicketBytes = size_t(256) << 10;          // dk = dv = 64 counters (the tail)
constexpr size_t kPrepBytes = kNoAllocScratchBytes - kTicketBytes;  // dk = dv = 128 rows and gates
static_assert(kPrepBytes % 256 == 0, "the ticket part keeps the array's 256-byte alignment");
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

static std::mutex g_scratch_mu;
static void* g_scratch_addr[kMaxDevices] = {};

// Device address of g_decode_scratch on the current device (looked up once per device).
static int scratch_address(void** out) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return fail(GDN_ERR_CUDA, "gdn_decode_layer_noalloc: cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return fail(GDN_ERR_ARG, "gdn_decode_layer_noalloc: device %d out of range", dev);
  std::lock_guard<std::mutex> lock(g_scratch_mu);
  if (!g_scratch_addr[dev]) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_decode_scratch);
    if (e != cudaSuccess || !p)
      return fail(GDN_ERR_CUDA, "gdn_decode_layer_noalloc: cudaGetSymbolAddress: %s", cudaGetErrorString(e));
    g_scratch_addr[dev] = p;
  }
  *out = g_scratch_addr[dev];
  return GDN_OK;
}

}  // namespace gdn

extern "C" size_t gdn_decode_layer_noalloc_max_bytes(void) { return gdn::kPrepBytes; }

extern "C" size_t gdn_decode_layer_noalloc_max_ticket_bytes(void) { return gdn::kTicketBytes; }

extern "C" int gdn_decode_layer_noalloc(const void* mixed_qkv, int64_t mixed_rs, const void* z, const void* a,
                                        const void* b, const float* A_log, const float* dt_bias,
                                        const void* conv_w, const void* conv_b, void* conv_pool, float* rec_pool,
                                        const int32_t* slot_idx, int64_t n_slots, const void* norm_w, float eps,
                                        void* out, int n, int Hk, int Hv, int dk, int dv, int K, int conv_mode,
                                        int dtype, int32_t* err_flag, void* stream) {
  using namespace gdn;
  if (n < 0 || Hk <= 0 || Hv <= 0 || dk <= 0 || dv <= 0)
    return fail(GDN_ERR_ARG, "gdn_decode_layer_noalloc: n=%d Hk=%d Hv=%d dk=%d dv=%d", n, Hk, Hv, dk, dv);
  const size_t need = gdn_decode_layer_workspace_size(n, Hk, Hv, dk, dv, dtype);
  const bool wide = dk == 128 && dv == 128;  // prepared rows (else ticket counters)
  const size_t cap = wide ? kPrepBytes : kTicketBytes;
  if (need > cap)
    return fail(GDN_ERR_WORKSPACE,
                "gdn_decode_layer_noalloc: needs %zu bytes of scratch, the built-in array's %s part holds %zu",
                need, wide ? "prepared-row" : "ticket", cap);
  void* scratch = nullptr;
  int rc = scratch_address(&scratch);
  if (rc) return rc;
  void* ws = wide ? scratch : static_cast<void*>(static_cast<unsigned char*>(scratch) + kPrepBytes);
  return gdn_decode_layer(mixed_qkv, mixed_rs, z, a, b, A_log, dt_bias, conv_w, conv_b, conv_pool, rec_pool,
                          slot_idx, n_slots, norm_w, eps, out, n, Hk, Hv, dk, dv, K, conv_mode, ws, cap, dtype,
                          err_flag, stream);
}
