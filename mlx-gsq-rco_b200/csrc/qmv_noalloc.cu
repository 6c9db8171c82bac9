// gsq_qmv_noalloc: the fused matvec for callers that cannot allocate device
// memory.
//
// gsq_qmv needs a caller-provided workspace for its split-K partial sums and
// ticket counters.  Some callers cannot provide one: code that runs where
// cudaMalloc is not allowed or not wanted (an embedding host with its own
// fixed memory budget, a plugin that is handed raw pointers only, a real-time
// loop that must never enter the allocator).  This entry point uses a fixed
// scratch array that lives in this library's device image instead, so the call
// itself allocates nothing.
//
// Limits and rules:
//  * The scratch is GSQ_QMV_NOALLOC_SCRATCH_BYTES (2 MiB) per device, held by
//    every GPU that loads the library until the process exits.  Shapes whose
//    gsq_qmv_workspace_size() exceeds it are rejected with GSQ_ERR_WORKSPACE.
//  * The first call on a device looks up the scratch's device address
//    (cudaGetSymbolAddress) with that device current; make that first call
//    before any stream capture.
//  * All calls share the one array.  Calls that overlap on the GPU (different
//    streams, or threads without ordering) race on it; order them.
//  * The array starts zero-filled (static device storage) and every completed
//    call returns the ticket counters and piece slots it used to zero, which
//    is the state the next call needs; the partial-sum region needs no
//    clearing.
//  * Bounded waits report through the same device error word as gsq_qmv
//    (gsq_device_status).  A wait that gave up can be followed by the late
//    write it waited for, which would leave a slot non-zero; when
//    gsq_device_status() reports an expired wait it also zero-fills this
//    array (a memset, no allocation), so the next call starts clean.
#include <cstdio>
#include <mutex>

#include "gsq_common.cuh"
#include "gsq_host.h"
#include "../../include/gsq_b200.h"

namespace {

constexpr size_t kScratchBytes = GSQ_QMV_NOALLOC_SCRATCH_BYTES;

__device__ __align__(256) unsigned char g_qmv_scratch[kScratchBytes];

void* g_scratch_cache[64] = {nullptr};  // device address per device, once looked up
std::mutex g_scratch_mu;

void* scratch_address(int* status) {
  void** cache = g_scratch_cache;
  std::mutex& mu = g_scratch_mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    *status = GSQ_ERR_CUDA;
    return nullptr;
  }
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_qmv_scratch);
    if (e != cudaSuccess || !p) {
      char msg[256];
      snprintf(msg, sizeof(msg), "gsq_qmv_noalloc: cudaGetSymbolAddress failed: %s", cudaGetErrorString(e));
      *status = gsq::set_last_error(GSQ_ERR_CUDA, msg);
      return nullptr;
    }
    cache[dev] = p;
  }
  return cache[dev];
}

int supported_type(int t) {
  switch (t) {
#define GSQ_NOALLOC_SUP(TT) case gsq::TT:
    GSQ_FOR_EACH_QTYPE(GSQ_NOALLOC_SUP)
    return 1;
#undef GSQ_NOALLOC_SUP
  }
  return 0;
}

}  // namespace

namespace gsq {
cudaError_t qmv_noalloc_scratch_clear() {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess || dev < 0 || dev >= 64) return e;
  void* p = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mu);
    p = g_scratch_cache[dev];
  }
  if (!p) return cudaSuccess;  // never used on this device: still zero
  // Every stream of the device: a noalloc call still running elsewhere must
  // not see the array cleared under it.
  if ((e = cudaDeviceSynchronize()) != cudaSuccess) return e;
  if ((e = cudaMemset(p, 0, kScratchBytes)) != cudaSuccess) return e;
  return cudaDeviceSynchronize();
}
}  // namespace gsq

extern "C" GSQ_API int gsq_qmv_noalloc(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N,
                                       int64_t K, int64_t rows, void* y, int y_dtype, gsq_stream_t stream) {
  // Same argument contract as gsq_qmv, minus the workspace.
  using gsq::set_last_error;
  if (!supported_type(qtype)) return set_last_error(GSQ_ERR_QTYPE, "gsq_qmv_noalloc: unsupported quant type");
  if (N < 0 || K <= 0 || K % 256 || rows < 0 || rows > (1 << 20))
    return set_last_error(GSQ_ERR_SIZE, "gsq_qmv_noalloc: invalid shape (K must be a positive multiple of 256)");
  if (rows == 0 || N == 0) return GSQ_OK;
  if (!x || !y || !packed) return set_last_error(GSQ_ERR_ARG, "gsq_qmv_noalloc: null pointer");
  if (x_dtype < 0 || x_dtype > 2 || y_dtype < 0 || y_dtype > 2)
    return set_last_error(GSQ_ERR_ARG, "gsq_qmv_noalloc: unsupported dtype");
  const size_t ysz = y_dtype == 0 ? 4 : 2;
  if ((reinterpret_cast<uintptr_t>(packed) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) ||
      (reinterpret_cast<uintptr_t>(y) % ysz))
    return set_last_error(GSQ_ERR_ALIGN, "gsq_qmv_noalloc: packed and x must be 16-byte aligned");
  const gsq::QmvPlan p = gsq::qmv_plan(qtype, N, K, (int)rows);
  if (p.ctas <= 0) return set_last_error(GSQ_ERR_SIZE, "gsq_qmv_noalloc: matrix too large for the matvec");
  if (p.workspace > kScratchBytes) {
    char msg[256];
    snprintf(msg, sizeof(msg),
             "gsq_qmv_noalloc: this shape needs %zu scratch bytes, more than the fixed %zu-byte array; "
             "use gsq_qmv with a caller workspace",
             p.workspace, kScratchBytes);
    return set_last_error(GSQ_ERR_WORKSPACE, msg);
  }
  int status = GSQ_OK;
  void* ws = p.workspace > 0 ? scratch_address(&status) : nullptr;
  if (p.workspace > 0 && !ws) return status;
  cudaError_t e = gsq::qmv_run(qtype, x, x_dtype, packed, N, K, (int)rows, y, y_dtype, ws, p,
                               gsq::device_error_word(), (cudaStream_t)stream);
  return e == cudaSuccess ? GSQ_OK : set_last_error(GSQ_ERR_CUDA, cudaGetErrorString(e));
}
