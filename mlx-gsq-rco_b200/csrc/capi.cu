// C ABI entry points (include/gsq_b200.h): argument validation, dispatch by
// quant type, and the per-device error word.  Validation mirrors the
// reference's Python contract (ValueError on size mismatch, qmv.py:540-544 /
// qmm.py:571-580; NotImplementedError on an unknown type, registry.py:29-31)
// as negative status codes.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <algorithm>
#include <mutex>

#include "gsq_common.cuh"
#include "../../include/gsq_b200.h"
#include "../../include/gsq_model.h"

#include "gsq_host.h"

using namespace gsq;

static __device__ int g_device_error;

static thread_local char g_err[512] = "";

static int fail(int code, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return code;
}

namespace gsq {
// Lets other translation units of the library report through gsq_last_error().
int set_last_error(int code, const char* msg) {
  snprintf(g_err, sizeof(g_err), "%s", msg);
  return code;
}
}  // namespace gsq

namespace gsq {
// Device address of the error word on the current device (looked up once per
// device; nullptr if CUDA cannot provide it).
int* device_error_word() {
  static int* cache[64] = {nullptr};
  static std::mutex mu;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
  std::lock_guard<std::mutex> lock(mu);
  if (!cache[dev]) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
    cache[dev] = static_cast<int*>(p);
  }
  return cache[dev];
}
}  // namespace gsq

static bool supported(int t) {
  switch (t) {
#define GSQ_SUP(TT) case TT:
    GSQ_FOR_EACH_QTYPE(GSQ_SUP)
    return true;
#undef GSQ_SUP
  }
  return false;
}

static bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
static bool dtype_ok(int d) { return d == DT_F32 || d == DT_F16 || d == DT_BF16; }
static size_t dtype_size(int d) { return d == DT_F32 ? 4 : 2; }

static int cuda_fail(cudaError_t e, const char* what) {
  return fail(GSQ_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
}

extern "C" {

const char* gsq_version(void) { return "gsq_b200 0.1.0 (sm_100a)"; }

const char* gsq_last_error(void) { return g_err; }

int gsq_block_info(int qtype, int* block_elements, int* block_bytes_out) {
  if (!supported(qtype)) return fail(GSQ_ERR_QTYPE, "unsupported quant type id %d", qtype);
  if (block_elements) *block_elements = QK;
  if (block_bytes_out) *block_bytes_out = block_bytes(qtype);
  return GSQ_OK;
}

int gsq_dequant(int qtype, const uint8_t* packed, int64_t nblocks, float* out, gsq_stream_t stream) {
  if (!supported(qtype)) return fail(GSQ_ERR_QTYPE, "validated decoder not available for type id %d", qtype);
  if (nblocks < 0) return fail(GSQ_ERR_SIZE, "negative block count");
  if (nblocks == 0) return GSQ_OK;
  if (!packed || !out) return fail(GSQ_ERR_ARG, "null pointer");
  if (!aligned(out, 16)) return fail(GSQ_ERR_ALIGN, "out must be 16-byte aligned");
  cudaError_t e = dequant_launch(qtype, packed, nblocks, out, (cudaStream_t)stream);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_dequant launch");
}

static int check_matrix(int qtype, const uint8_t* packed, int64_t N, int64_t K) {
  if (!supported(qtype)) return fail(GSQ_ERR_QTYPE, "no kernel for quant type id %d", qtype);
  if (N < 0 || K <= 0 || K % QK) return fail(GSQ_ERR_SIZE, "invalid matrix width K=%lld (must be a positive multiple of 256)", (long long)K);
  if (!packed) return fail(GSQ_ERR_ARG, "null packed pointer");
  if (!aligned(packed, 16)) return fail(GSQ_ERR_ALIGN, "packed must be 16-byte aligned");
  return GSQ_OK;
}

size_t gsq_qmv_workspace_size(int qtype, int64_t N, int64_t K, int64_t rows) {
  if (!supported(qtype) || N <= 0 || K <= 0 || K % QK || rows <= 0) return 0;
  // Also enough for gsq_qmv_gather's one-row-per-tile plan of the same shape.
  return std::max(qmv_plan(qtype, N, K, (int)rows).workspace, qmv_plan(qtype, N, K, (int)rows, true).workspace);
}

int gsq_qmv(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t rows,
            void* y, int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  int rc = check_matrix(qtype, packed, N, K);
  if (rc) return rc;
  if (rows < 0 || rows > (1 << 20)) return fail(GSQ_ERR_SIZE, "invalid row count %lld", (long long)rows);
  if (rows == 0 || N == 0) return GSQ_OK;
  if (!x || !y) return fail(GSQ_ERR_ARG, "null x or y");
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(GSQ_ERR_ARG, "unsupported dtype");
  if (!aligned(x, 16) || !aligned(y, dtype_size(y_dtype)))
    return fail(GSQ_ERR_ALIGN, "x must be 16-byte aligned and y aligned to its dtype");
  const QmvPlan p = qmv_plan(qtype, N, K, (int)rows);
  if (p.ctas <= 0)
    return fail(GSQ_ERR_SIZE, "matrix too large for the matvec (N=%lld, K=%lld)", (long long)N, (long long)K);
  if (p.workspace > 0 && (!workspace || workspace_bytes < p.workspace || !aligned(workspace, 256)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_qmv needs %zu workspace bytes (256-byte aligned), got %zu", p.workspace,
                workspace_bytes);
  cudaError_t e = qmv_run(qtype, x, x_dtype, packed, N, K, (int)rows, y, y_dtype, workspace, p, device_error_word(),
                          (cudaStream_t)stream);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_qmv launch");
}

int gsq_qmv_swiglu(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t n_out, int64_t K,
                   int64_t rows, void* y, int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  if (n_out < 0 || n_out % 8) return fail(GSQ_ERR_SIZE, "gsq_qmv_swiglu: n_out must be a multiple of 8");
  const int64_t N = 2 * n_out;  // packed rows: 8 gate rows, then the same 8 up rows, per 16
  int rc = check_matrix(qtype, packed, N, K);
  if (rc) return rc;
  if (rows < 0 || rows >= 8) return fail(GSQ_ERR_SIZE, "gsq_qmv_swiglu takes 0..7 rows (%lld)", (long long)rows);
  if (rows == 0 || N == 0) return GSQ_OK;
  if (!x || !y) return fail(GSQ_ERR_ARG, "null x or y");
  if (!dtype_ok(x_dtype) || !dtype_ok(y_dtype)) return fail(GSQ_ERR_ARG, "unsupported dtype");
  if (!aligned(x, 16) || !aligned(y, dtype_size(y_dtype)))
    return fail(GSQ_ERR_ALIGN, "x must be 16-byte aligned and y aligned to its dtype");
  const QmvPlan p = qmv_plan(qtype, N, K, (int)rows);
  if (p.ctas <= 0)
    return fail(GSQ_ERR_SIZE, "matrix too large for the matvec (N=%lld, K=%lld)", (long long)N, (long long)K);
  if (p.workspace > 0 && (!workspace || workspace_bytes < p.workspace || !aligned(workspace, 256)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_qmv_swiglu needs %zu workspace bytes (256-byte aligned), got %zu",
                p.workspace, workspace_bytes);
  cudaError_t e = qmv_run(qtype, x, x_dtype, packed, N, K, (int)rows, y, y_dtype, workspace, p, device_error_word(),
                          (cudaStream_t)stream, nullptr, 1);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_qmv_swiglu launch");
}

size_t gsq_gather_region_bytes(int64_t rows, int64_t ntot) {
  if (rows <= 0 || ntot <= 0) return 0;
  return qmv_gather_region_bytes(rows, ntot);
}

int gsq_gather_region_alloc(size_t bytes, void** region) {
  if (!region || bytes < 256) return fail(GSQ_ERR_ARG, "region pointer missing or size below the 256-byte header");
  *region = nullptr;
  cudaError_t e = cudaMalloc(region, bytes);
  if (e != cudaSuccess) return cuda_fail(e, "gsq_gather_region_alloc");
  e = cudaMemset(*region, 0, bytes);
  if (e != cudaSuccess) {
    cudaFree(*region);
    *region = nullptr;
    return cuda_fail(e, "gsq_gather_region_alloc (zero fill)");
  }
  return GSQ_OK;
}

int gsq_gather_region_free(void* region) {
  if (!region) return GSQ_OK;
  cudaError_t e = cudaFree(region);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_gather_region_free");
}

int gsq_ipc_export(void* region, uint8_t handle[64]) {
  if (!region || !handle) return fail(GSQ_ERR_ARG, "null region or handle");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, region);
  if (e != cudaSuccess) return cuda_fail(e, "gsq_ipc_export");
  static_assert(sizeof(h) == 64, "IPC handle size");
  memcpy(handle, &h, 64);
  return GSQ_OK;
}

int gsq_ipc_import(const uint8_t handle[64], void** peer) {
  if (!handle || !peer) return fail(GSQ_ERR_ARG, "null handle or output pointer");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  *peer = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(peer, h, cudaIpcMemLazyEnablePeerAccess);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_ipc_import");
}

int gsq_ipc_close(void* peer) {
  if (!peer) return GSQ_OK;
  cudaError_t e = cudaIpcCloseMemHandle(peer);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_ipc_close");
}

int gsq_qmv_gather(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                   int64_t rows, void* const* regions, int world, int rank, int64_t row0, int64_t ntot,
                   void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  int rc = check_matrix(qtype, packed, N, K);
  if (rc) return rc;
  if (world < 2 || world > 8 || rank < 0 || rank >= world) return fail(GSQ_ERR_ARG, "world must be 2..8 and rank < world");
  if (!regions) return fail(GSQ_ERR_ARG, "null region list");
  for (int i = 0; i < world; i++)
    if (!regions[i] || !aligned(regions[i], 256)) return fail(GSQ_ERR_ALIGN, "region %d missing or not 256-byte aligned", i);
  if (rows <= 0 || rows >= 8)
    return fail(GSQ_ERR_SIZE, "gsq_qmv_gather takes 1..7 activation rows, got %lld", (long long)rows);
  if (row0 < 0 || N <= 0 || row0 + N > ntot) return fail(GSQ_ERR_SIZE, "rows [%lld, %lld) outside the %lld gathered rows",
                                                         (long long)row0, (long long)(row0 + N), (long long)ntot);
  if (!x) return fail(GSQ_ERR_ARG, "null x");
  if (!dtype_ok(x_dtype)) return fail(GSQ_ERR_ARG, "unsupported dtype");
  if (!aligned(x, 16)) return fail(GSQ_ERR_ALIGN, "x must be 16-byte aligned");
  const QmvPlan p = qmv_plan(qtype, N, K, (int)rows, true);
  if (p.ctas <= 0)
    return fail(GSQ_ERR_SIZE, "matrix too large for the matvec (N=%lld, K=%lld)", (long long)N, (long long)K);
  if (p.workspace > 0 && (!workspace || workspace_bytes < p.workspace || !aligned(workspace, 256)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_qmv_gather needs %zu workspace bytes (256-byte aligned), got %zu",
                p.workspace, workspace_bytes);
  const QmvGather g = {regions, world, rank, row0, ntot};
  uint8_t* own_y = static_cast<uint8_t*>(regions[rank]) + 256;
  cudaError_t e = qmv_run(qtype, x, x_dtype, packed, N, K, (int)rows, own_y, DT_F32, workspace, p,
                          device_error_word(), (cudaStream_t)stream, &g);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_qmv_gather launch");
}

}  // extern "C"

static int qmm_gather_run(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                          int64_t M, void* const* regions, void* multicast, int world, int rank, int64_t row0,
                          int64_t ntot, int y_dtype, void* workspace, size_t workspace_bytes,
                          gsq_stream_t stream) {
  int rc = check_matrix(qtype, packed, N, K);
  if (rc) return rc;
  if (world < 2 || world > 8 || rank < 0 || rank >= world) return fail(GSQ_ERR_ARG, "world must be 2..8 and rank < world");
  if (!regions) return fail(GSQ_ERR_ARG, "null region list");
  for (int i = 0; i < world; i++)
    if (!regions[i] || !aligned(regions[i], 256)) return fail(GSQ_ERR_ALIGN, "region %d missing or not 256-byte aligned", i);
  if (y_dtype != DT_F32 && y_dtype != DT_F16) return fail(GSQ_ERR_ARG, "gathered values must be fp32 or fp16");
  if (M <= 0 || M > (1ll << 31)) return fail(GSQ_ERR_SIZE, "invalid row count %lld", (long long)M);
  if (row0 < 0 || N <= 0 || row0 + N > ntot)
    return fail(GSQ_ERR_SIZE, "rows [%lld, %lld) outside the %lld gathered rows", (long long)row0,
                (long long)(row0 + N), (long long)ntot);
  if (!x) return fail(GSQ_ERR_ARG, "null x");
  if (!dtype_ok(x_dtype)) return fail(GSQ_ERR_ARG, "unsupported x dtype");
  if (!aligned(x, 16)) return fail(GSQ_ERR_ALIGN, "x must be 16-byte aligned");
  const size_t need = qmm_workspace_bytes(qtype, N, K, M, x_dtype);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned(workspace, 256)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_qmm_gather needs %zu workspace bytes (256-byte aligned), got %zu", need,
                workspace_bytes);
  if (multicast && !aligned(multicast, 256)) return fail(GSQ_ERR_ALIGN, "multicast region not 256-byte aligned");
  const QmmGather g = {regions, world, rank, row0, ntot, multicast};
  void* own_y = static_cast<uint8_t*>(regions[rank]) + 256;
  const char* why = "";
  cudaError_t e = qmm_launch(qtype, x, x_dtype, packed, N, K, M, own_y, y_dtype, workspace, device_error_word(),
                             (cudaStream_t)stream, &why, &g);
  if (e != cudaSuccess) return fail(GSQ_ERR_CUDA, "gsq_qmm_gather launch: %s (%s)", cudaGetErrorString(e), why);
  return GSQ_OK;
}

extern "C" {

int gsq_qmm_gather(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
                   void* const* regions, int world, int rank, int64_t row0, int64_t ntot, int y_dtype,
                   void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  return qmm_gather_run(qtype, x, x_dtype, packed, N, K, M, regions, nullptr, world, rank, row0, ntot, y_dtype,
                        workspace, workspace_bytes, stream);
}

int gsq_qmm_gather_mc(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
                      void* const* regions, void* multicast_region, int world, int rank, int64_t row0, int64_t ntot,
                      int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  if (!multicast_region) return fail(GSQ_ERR_ARG, "null multicast region");
  return qmm_gather_run(qtype, x, x_dtype, packed, N, K, M, regions, multicast_region, world, rank, row0, ntot,
                        y_dtype, workspace, workspace_bytes, stream);
}

size_t gsq_qmm_workspace_size(int qtype, int64_t N, int64_t K, int64_t M, int x_dtype) {
  if (!supported(qtype) || M <= 0 || N <= 0 || K <= 0 || K % QK) return 0;
  return qmm_workspace_bytes(qtype, N, K, M, x_dtype);
}

int gsq_qmm(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
            void* y, int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream) {
  int rc = check_matrix(qtype, packed, N, K);
  if (rc) return rc;
  if (M < 0 || M > (1ll << 31)) return fail(GSQ_ERR_SIZE, "invalid row count %lld", (long long)M);
  if (M == 0 || N == 0) return GSQ_OK;
  if (!x || !y) return fail(GSQ_ERR_ARG, "null x or y");
  if (!dtype_ok(x_dtype)) return fail(GSQ_ERR_ARG, "unsupported x dtype");
  if (!dtype_ok(y_dtype)) return fail(GSQ_ERR_ARG, "unsupported y dtype");
  if (!aligned(x, 16) || !aligned(y, y_dtype == DT_F32 ? 4 : 2))
    return fail(GSQ_ERR_ALIGN, "x must be 16-byte aligned, y aligned to its type");
  const size_t need = qmm_workspace_bytes(qtype, N, K, M, x_dtype);
  if (need > 0 && (!workspace || workspace_bytes < need || !aligned(workspace, 256)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_qmm needs %zu workspace bytes (256-byte aligned), got %zu", need,
                workspace_bytes);
  const char* why = "launch";
  cudaError_t e = qmm_launch(qtype, x, x_dtype, packed, N, K, M, y, y_dtype, workspace, device_error_word(),
                             (cudaStream_t)stream, &why);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, why);
}

int gsq_embed(int qtype, const int32_t* ids, int64_t T, const uint8_t* packed, int64_t vocab, int64_t dim,
              void* out, int out_dtype, gsq_stream_t stream) {
  if (!supported(qtype)) return fail(GSQ_ERR_QTYPE, "unsupported embedding type id %d", qtype);
  if (dim <= 0 || dim % QK) return fail(GSQ_ERR_SIZE, "embedding dimensions must be divisible by 256");
  if (T < 0 || vocab <= 0) return fail(GSQ_ERR_SIZE, "invalid token count or vocab");
  if (T == 0) return GSQ_OK;
  if (!ids || !packed || !out) return fail(GSQ_ERR_ARG, "null pointer");
  if (!dtype_ok(out_dtype)) return fail(GSQ_ERR_ARG, "unsupported dtype");
  if (!aligned(out, 16)) return fail(GSQ_ERR_ALIGN, "out must be 16-byte aligned");
  cudaError_t e = embed_launch(qtype, ids, T, packed, vocab, dim, out, out_dtype, device_error_word(),
                               (cudaStream_t)stream);
  return e == cudaSuccess ? GSQ_OK : cuda_fail(e, "gsq_embed launch");
}

int gsq_device_status(gsq_stream_t stream) {
  cudaError_t e = cudaStreamSynchronize((cudaStream_t)stream);
  if (e != cudaSuccess) return cuda_fail(e, "gsq_device_status sync");
  int* w = device_error_word();
  if (!w) return fail(GSQ_ERR_CUDA, "device error word unavailable");
  int v = 0;
  e = cudaMemcpy(&v, w, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "gsq_device_status read");
  const int zero = 0;
  cudaMemcpy(w, &zero, sizeof(int), cudaMemcpyHostToDevice);
  if (v == DEV_WAIT_TIMEOUT) {
    // A wait that gave up may have been followed by the late write it was
    // waiting for, leaving a non-zero piece slot or ticket in scratch that
    // the next call expects zero.  The library's own fixed scratch
    // (gsq_qmv_noalloc) is cleared here; caller workspaces are the caller's
    // to re-zero (include/gsq_b200.h).
    e = qmv_noalloc_scratch_clear();
    if (e != cudaSuccess) return cuda_fail(e, "gsq_device_status scratch reset");
  }
  return v;
}

}  // extern "C"
