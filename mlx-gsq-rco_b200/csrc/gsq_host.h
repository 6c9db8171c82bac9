// Host-side declarations shared by the kernel translation units and the C ABI.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stddef.h>
#include <stdint.h>

#include <utility>

namespace gsq {

// Launch with programmatic stream serialization (PDL): the kernel may begin
// while the previous kernel of the stream finishes; it synchronises with
// griddepcontrol.wait before touching that kernel's results.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                                     cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// launch_pdl with thread-block clusters of `cluster_x` CTAs along x (grid.x
// a multiple of cluster_x), no dynamic shared memory.
template <typename... KArgs, typename... Args>
static inline cudaError_t launch_pdl_cluster(void (*kernel)(KArgs...), dim3 grid, dim3 block, unsigned cluster_x,
                                             cudaStream_t st, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = cluster_x;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Launch plan of one QMV call: grid shape, work split and scratch layout.
struct QmvPlan {
  int nb;            // activation rows per tile (1 or 2)
  int btiles;        // activation-row tiles (grid.z)
  int64_t tiles;     // 16-row weight tiles
  int slices;        // K-slices (grid.y)
  int bps;           // 256-blocks per K-slice
  int ctas;          // persistent CTAs per K-slice (grid.x)
  int aligned;       // 1: CTAs own whole tiles (no partial sums, no tickets)
  int ns;            // ring stages (2..4)
  int cb, rowb, stage;  // ring geometry: blocks per stage, staged row stride, stage bytes
  int pre;           // stages issued before the activations are quantised
  size_t smem;       // dynamic shared memory bytes
  size_t off_full, off_piece;  // scratch layout (bytes)
  size_t workspace;  // scratch bytes (tickets + partial sums), 0 when no tile is split
};

// one_row_tiles: one activation row per tile (the gathering kernel exists
// only in that form).
QmvPlan qmv_plan(int t, int64_t N, int64_t K, int rows, bool one_row_tiles = false);

// Runs QMV with `ws` as scratch (must hold plan.workspace bytes, zero-filled
// tickets; left zero-filled on completion).
// Fused row gather of a rank's output rows into every rank's region (see
// gsq_qmv_gather); regions[i] is rank i's region, mapped in this process.
struct QmvGather {
  void* const* regions;
  int world, rank;
  int64_t row0, ntot;
};

cudaError_t qmv_run(int t, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int rows,
                    void* y, int y_dtype, void* ws, const QmvPlan& p, int* err, cudaStream_t st,
                    const QmvGather* gather = nullptr, int glu = 0);
size_t qmv_gather_inbox_offset(int64_t rows, int64_t ntot);
size_t qmv_gather_region_bytes(int64_t rows, int64_t ntot);

cudaError_t dequant_launch(int t, const uint8_t* packed, int64_t nblocks, float* out, cudaStream_t st);
cudaError_t embed_launch(int t, const int32_t* ids, int64_t n, const uint8_t* packed, int64_t vocab, int64_t dim,
                         void* out, int dtype, int* err, cudaStream_t st);
// Launch plan of one QMM call: token tile T = bn x nacc, grid = row tiles x
// token groups x K splits, and the scratch layout.
struct QmmPlan {
  int bn, nacc;              // MMA N per accumulator (<= 256), accumulators per CTA (1 or 2)
  int ksplit, kbs;           // K splits, 256-blocks per split (of the split launch)
  int64_t row_tiles, token_groups;
  int64_t whole_tiles;       // > 0: a first launch of whole-K tiles [0, whole_tiles) in full waves,
                             // then the remaining tiles with K split ksplit ways
  size_t off_part, off_x16;  // scratch layout: tickets at 0, partial tiles, fp16 activations
  size_t workspace;          // scratch bytes
};

QmmPlan qmm_plan(int t, int64_t N, int64_t K, int64_t M, int x_dtype);
size_t qmm_workspace_bytes(int t, int64_t N, int64_t K, int64_t M, int x_dtype);
// ws: the plan's scratch, zero-filled once by the caller.
// Fused row gather of a rank's output rows into every rank's region (see
// gsq_qmm_gather); regions[i] is rank i's region, mapped in this process.
struct QmmGather {
  void* const* regions;
  int world, rank;
  int64_t row0, ntot;
  void* multicast;  // NVSwitch multicast mapping of the regions, or nullptr
};

// y: M x N values of y_dtype (DT_F32 / DT_F16 / DT_BF16), or with `gather`
// this rank's region values (DT_F32 / DT_F16).
cudaError_t qmm_launch(int t, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
                       void* y, int y_dtype, void* ws, int* err, cudaStream_t st, const char** why,
                       const struct QmmGather* gather = nullptr);

// Device address of the library's error word on the current device (the
// word gsq_device_status reads); nullptr if it cannot be looked up.
int* device_error_word();

// Zero-fills gsq_qmv_noalloc's fixed scratch array on the current device
// (synchronising the device first, so no kernel is still using it).  No-op on
// a device where the array was never used.  Allocates nothing.
cudaError_t qmv_noalloc_scratch_clear();

// Records `msg` as this thread's gsq_last_error() text and returns `code`.
int set_last_error(int code, const char* msg);

}  // namespace gsq
