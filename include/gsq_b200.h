/*
 * gsq_b200 -- C ABI of the B200 (sm_100a) packed-GGUF hot path.
 *
 * Drop-in replacement for the kernel layer of mlx-GSQ-RCO
 * (mlx_gsq/runtime/kernels/): dequantize, fused dequantize-matvec (decode),
 * tiled dequantize-matmul (prefill) and the packed embedding gather, for the
 * eleven GGUF block types IQ1_M, IQ1_S, IQ2_XXS, IQ2_XS, IQ2_S, IQ3_XXS,
 * IQ3_S, IQ4_XS, Q2_K, Q4_K, Q6_K, read directly from the unmodified packed
 * payloads.
 *
 * Conventions
 *  - qtype is the GGML type id (mlx_gsq/gguf/parser.py:26-32): IQ1_M=29,
 *    IQ1_S=19, IQ2_XXS=16, IQ2_XS=17, IQ2_S=22, IQ3_XXS=18, IQ3_S=21,
 *    IQ4_XS=23, Q2_K=10, Q4_K=12, Q6_K=14.
 *  - A packed matrix of N output rows and K inputs is N rows of K/256 blocks,
 *    row n occupying bytes [n*(K/256)*bb, (n+1)*(K/256)*bb) (bb = block bytes).
 *  - All pointers are device pointers; every call is asynchronous on
 *    `stream` (a cudaStream_t; NULL = legacy default stream) and allocates
 *    nothing: buffers, including workspaces, belong to the caller.
 *  - Return value: GSQ_OK (0) or a negative gsq_status; gsq_last_error()
 *    then describes the failure (per calling thread).
 *  - Calls are thread-safe; concurrent calls that share a workspace must be
 *    ordered by the caller (same stream, or events).
 */
#ifndef GSQ_B200_H
#define GSQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GSQ_API __attribute__((visibility("default")))
#else
#define GSQ_API
#endif

typedef struct CUstream_st* gsq_stream_t; /* == cudaStream_t */

typedef enum {
  GSQ_OK = 0,
  GSQ_ERR_QTYPE = -1,     /* unsupported quant type (reference: NotImplementedError, registry.py:29-31) */
  GSQ_ERR_SIZE = -2,      /* shape / payload size mismatch (reference: ValueError, qmv.py:541-544) */
  GSQ_ERR_ALIGN = -3,     /* pointer alignment requirement not met */
  GSQ_ERR_ARG = -4,       /* other invalid argument (dtype, null pointer) */
  GSQ_ERR_CUDA = -5,      /* CUDA runtime error at launch */
  GSQ_ERR_WORKSPACE = -6, /* workspace missing or too small */
  GSQ_ERR_DEVICE = -7     /* a kernel reported an error (gsq_device_status) */
} gsq_status;

typedef enum { GSQ_F32 = 0, GSQ_F16 = 1, GSQ_BF16 = 2 } gsq_dtype;

/* Library version string. */
GSQ_API const char* gsq_version(void);

/* Description of the last error returned on this thread. */
GSQ_API const char* gsq_last_error(void);

/* Block geometry of a type: elements and stored bytes per block.
 * Replaces QUANT_BLOCK_SIZES lookups (mlx_gsq/gguf/parser.py:35-42). */
GSQ_API int gsq_block_info(int qtype, int* block_elements, int* block_bytes);

/* Flat fp32 dequantization of nblocks packed blocks, bit-identical to
 * gguf-py 0.19.0 (finite inputs).  out: nblocks*256 floats, 16-byte aligned.
 * Replaces registry.decode / decode_weight (mlx_gsq/runtime/kernels/registry.py:28-46). */
GSQ_API int gsq_dequant(int qtype, const uint8_t* packed, int64_t nblocks, float* out, gsq_stream_t stream);

/* Workspace bytes gsq_qmv needs for this shape (0 when none is needed). */
GSQ_API size_t gsq_qmv_workspace_size(int qtype, int64_t N, int64_t K, int64_t rows);

/* Fused dequantize + matvec for few activation rows (decode):
 *   y[r, n] = sum_k x[r, k] * deq(W)[n, k],  r < rows, fp32 accumulation.
 * x: rows x K (x_dtype), 16-byte aligned.  y: rows x N (y_dtype).
 * packed: 16-byte aligned, N*(K/256)*bb bytes.  K % 256 == 0.
 * workspace: gsq_qmv_workspace_size() bytes, zero-filled before its first use;
 * every completed call leaves it zero-filled again -- except after a bounded
 * wait expired (gsq_device_status() == 1), which can leave stale slots: zero
 * the workspace again before its next use.
 * Replaces quantized_matvec (mlx_gsq/runtime/kernels/qmv.py:537-576). */
GSQ_API int gsq_qmv(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t rows,
            void* y, int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream);

/* Workspace bytes gsq_qmm needs (an fp16 copy of x unless x is fp16). */
GSQ_API size_t gsq_qmm_workspace_size(int qtype, int64_t N, int64_t K, int64_t M, int x_dtype);

/* Tiled dequantize + matmul on tcgen05 tensor cores (prefill):
 *   y[m, n] = sum_k x[m, k] * deq(W)[n, k],  M x N row-major in y_dtype
 *   (fp32, or fp16 / bf16 rounded once to nearest even from the fp32 sum).
 * x: M x K (x_dtype), 16-byte aligned; weights decoded to fp16, fp32 accumulation.
 * Replaces quantized_matmul (mlx_gsq/runtime/kernels/qmm.py:559-594), whose
 * output has x's dtype. */
GSQ_API int gsq_qmm(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
                    void* y, int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream);

/* Packed embedding gather: out[t, :] = deq(W)[ids[t], :] rounded once to
 * out_dtype; W is vocab x dim packed rows.  Out-of-range ids leave their row
 * untouched and set GSQ_ERR_DEVICE in gsq_device_status.
 * Replaces iq2_s_embedding (mlx_gsq/runtime/kernels/embedding.py:28-36),
 * generalised from IQ2_S to all eleven types. */
GSQ_API int gsq_embed(int qtype, const int32_t* ids, int64_t T, const uint8_t* packed, int64_t vocab, int64_t dim,
              void* out, int out_dtype, gsq_stream_t stream);

/* Fixed size of the device scratch array behind gsq_qmv_noalloc. */
#define GSQ_QMV_NOALLOC_SCRATCH_BYTES (2u * 1024u * 1024u)

/* gsq_qmv for callers that cannot allocate device memory (no reference
 * counterpart: the reference's Metal kernels need no scratch).  Same
 * arguments and results as gsq_qmv, without the workspace: the split-K
 * scratch is a fixed GSQ_QMV_NOALLOC_SCRATCH_BYTES array inside the library
 * (held by every GPU that loads it until exit), so the call allocates nothing.
 * Shapes that need more scratch return GSQ_ERR_WORKSPACE.  The first call on
 * a device looks up the array's address and should come before any stream
 * capture.  Every call shares the array: calls that overlap on the GPU race,
 * so order them (one stream, or events).  Bounded waits report through
 * gsq_device_status() like gsq_qmv; when it reports an expired wait it also
 * zero-fills this array, so calls after it start from a clean array. */
GSQ_API int gsq_qmv_noalloc(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                            int64_t rows, void* y, int y_dtype, gsq_stream_t stream);

/* ---- Row-parallel decode with the gather fused into the matvec ----------
 * No reference counterpart: the reference runs on one device (its only
 * trace of parallelism is mlx-lm's unexercised all_sum hook,
 * mlx_gsq/models/qwen35.py:104-105).  Each rank of a row split holds one
 * gather region per projection call site: 256 bytes of control words, the
 * gathered output (fp32 rows x ntot, at byte 256), then an inbox the peers
 * write.  Regions are exchanged between the ranks' processes with CUDA IPC
 * handles. */
GSQ_API size_t gsq_gather_region_bytes(int64_t rows, int64_t ntot);
/* Device allocation of `bytes` (>= 256), zero-filled; 256-byte aligned. */
GSQ_API int gsq_gather_region_alloc(size_t bytes, void** region);
GSQ_API int gsq_gather_region_free(void* region);
/* 64-byte CUDA IPC handle of a region, and its mapping in another process. */
GSQ_API int gsq_ipc_export(void* region, uint8_t handle[64]);
GSQ_API int gsq_ipc_import(const uint8_t handle[64], void** peer);
GSQ_API int gsq_ipc_close(void* peer);

/* gsq_qmv for 1..7 activation rows on rank `rank` of `world` (2..8) holding output rows
 * [row0, row0 + N) of ntot: the kernel sends its rows into every rank's
 * region (regions[i] = rank i's region, mapped in this process) over NVLink
 * and ends with the exchange of the rows through the regions' inboxes, so
 * that once the call has completed on `stream` every rank's region holds all
 * ntot rows of this call.  Every rank must make the same sequence of calls on a region; a
 * region must serve one call site.  Its rows stay valid until any rank calls
 * the region again: that call stores into every rank's copy, so a rank must
 * not issue it before every rank has consumed the previous rows (another
 * gathered call in between orders them, as does a barrier).  The flag wait is bounded: a rank that never arrives makes the
 * others return with gsq_device_status() == 1.  Output is fp32. */
GSQ_API int gsq_qmv_gather(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                           int64_t rows, void* const* regions, int world, int rank, int64_t row0, int64_t ntot,
                           void* workspace, size_t workspace_bytes, gsq_stream_t stream);

/* gsq_qmm for rank `rank` of `world` (2..8) holding output rows
 * [row0, row0 + N) of ntot (prefill): every output tile is stored into every
 * rank's region (M x ntot values at byte 256: fp32 for y_dtype 0, fp16
 * rounded to nearest even for y_dtype 1, which halves the bytes that cross
 * NVLink) over NVLink as the epilogue writes it, and each rank counts the
 * tiles its peers delivered, so that once the call has completed on `stream`
 * every rank's region holds all ntot rows.  Every call on a region uses the
 * same y_dtype.  Same region rules and bounded wait as gsq_qmv_gather (a
 * region for M >= 8 rows has no inbox: gsq_gather_region_bytes(M, ntot)
 * bytes, enough for either value type). */
GSQ_API int gsq_qmm_gather(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                           int64_t M, void* const* regions, int world, int rank, int64_t row0, int64_t ntot,
                           int y_dtype, void* workspace, size_t workspace_bytes, gsq_stream_t stream);

/* gsq_qmm_gather writing every output value once, through an NVSwitch
 * multicast mapping of the ranks' regions (multimem stores: the switch
 * delivers each value to every rank, this one included), instead of once per
 * rank.  multicast_region maps all ranks' regions at the same byte offsets
 * (e.g. torch symmetric memory's multicast_ptr for buffers holding the
 * regions); regions[] are still each rank's unicast mapping (the tile counts
 * go through them).  Same rules and bounded wait as gsq_qmm_gather.  No
 * reference counterpart (the reference runs on one device). */
GSQ_API int gsq_qmm_gather_mc(int qtype, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K,
                              int64_t M, void* const* regions, void* multicast_region, int world, int rank,
                              int64_t row0, int64_t ntot, int y_dtype, void* workspace, size_t workspace_bytes,
                              gsq_stream_t stream);

/* Synchronises `stream`, then returns and clears the device error word the
 * kernels of the current device write (0 = none; 1 = a bounded wait expired;
 * 2 = an embedding id was out of range).  On 1 it also synchronises the
 * device and zero-fills gsq_qmv_noalloc's fixed scratch array; workspaces
 * that the caller passed to gsq_qmv / gsq_qmm / the gathers must be
 * zero-filled again by the caller.  No reference counterpart: the
 * reference's Metal kernels have no device-side error path. */
GSQ_API int gsq_device_status(gsq_stream_t stream);

#ifdef __cplusplus
}
#endif

#endif /* GSQ_B200_H */
