// Tiled dequantize + matmul (QMM, prefill) on the 5th-gen tensor cores, sm_100a.
//
// Replaces the reference's tiled Metal QMM (mlx_gsq/runtime/kernels/qmm.py:
// template _source :252-325, decode bodies :38-143, entry quantized_matmul
// :559-594): Y[m, n] = sum_k X[m, k] * deq(W)[n, k], fp32 accumulation.
//
// Output tile = 128 weight rows (MMA M) x T tokens, K stepped 64 at a time;
// T = nacc x BN with one or two fp32 accumulators of BN <= 256 columns in
// TMEM (two when M > 256: every decoded weight tile then feeds 512 tokens).
// When there are too few row tiles to fill the GPU, K is split over several
// CTAs; each writes its partial tile to scratch and the last one to finish
// (acquire-release ticket) sums them in split order and writes Y, so the
// result stays deterministic.  Warp roles in a 352-thread CTA:
//   warp 0      TMA tensor-map loads of the fp16 activation tile (128B swizzle);
//   warp 1      allocates TMEM and issues tcgen05.mma (kind::f16, fp32 accum
//               in TMEM) from one elected lane, committing to mbarriers;
//   warp 2      1-D bulk copies of each row's packed 256-weight block into a
//               PST-deep staging ring, running ahead of the decoders;
//   warps 3..10 decode the packed blocks into fp16 in the canonical K-major
//               SW128 layout the MMA reads (each weight once per BN tokens),
//               two warps per TMEM sub-partition, then run the epilogue
//               (tcgen05.ld TMEM -> registers -> fp32 Y).
// Weights are decoded to fp16, not bf16: bf16-rounded weights miss the
// rel-L2 <= 1e-3 bar, fp16 ones pass; activations are converted to fp16 by
// a pre-pass (exact for |x| >= 2^-14).  All waits are time-bounded.
#include <cuda.h>
#include <algorithm>

#include "gsq_exact.cuh"
#include "gsq_fast.cuh"
#include "gsq_host.h"

namespace gsq {

constexpr int QMM_BM = 128;
constexpr int QMM_BK = 64;
constexpr int QMM_DEC_WARPS = 8;                 // two per TMEM sub-partition
constexpr int QMM_DEC0 = 3;                       // first decoder warp
constexpr int QMM_THREADS = 32 * (QMM_DEC0 + QMM_DEC_WARPS);
// Scratch: a fixed region of ticket counters (left zero-filled by every
// call), then the partial tiles of split-K plans, then the fp16 activations.
constexpr int QMM_TICKETS = 16384;
constexpr int QMM_KSPLIT_MAX = 8;
constexpr size_t QMM_TICKET_BYTES = QMM_TICKETS * sizeof(unsigned);

template <int T>
struct QmmGeom {
  static constexpr int BB = block_bytes(T);
  static constexpr int PROWB = ((BB + 30) + 15) / 16 * 16;   // staged packed row stride
  static constexpr int PSTAGE = QMM_BM * PROWB;               // one 256-block column of 128 rows
  static constexpr int TAB = (Fast<T>::TAB_BYTES + 127) / 128 * 128;
};

constexpr size_t QMM_SMEM_LIMIT = 227 * 1024;

// Pipeline shape for an activation stage of `bstage` bytes (T tokens x 64 k
// fp16): PST packed stages (3, or 2 when space is short) and as many A/B
// stages (<= 4) as fit.
template <int T>
struct QmmPipe {
  static constexpr size_t fixed(int pst) { return 1024 + (size_t)pst * QmmGeom<T>::PSTAGE + QmmGeom<T>::TAB + 256; }
  static constexpr int stages_for(size_t bstage, int pst) {
    const size_t per = (size_t)QMM_BM * 128 + bstage;
    const size_t n = fixed(pst) < QMM_SMEM_LIMIT ? (QMM_SMEM_LIMIT - fixed(pst)) / per : 0;
    return n >= 4 ? 4 : (int)n;
  }
  static constexpr int pst(size_t bstage) { return stages_for(bstage, 3) >= 3 ? 3 : 2; }
  static constexpr int ns(size_t bstage) { return stages_for(bstage, pst(bstage)); }
  static constexpr size_t smem(size_t bstage) {
    return fixed(pst(bstage)) + (size_t)ns(bstage) * ((size_t)QMM_BM * 128 + bstage);
  }
  // 512 tokens (the widest tile) must still leave two stages.
  static_assert(stages_for((size_t)512 * 128, 2) >= 2, "QMM ring must hold two stages at 512 tokens");
};

constexpr int QMM_GATHER_MAX = 8;
constexpr int QMM_GFLAG_TICKET = 62, QMM_GFLAG_COUNT = 63;  // owner's words of a gather region header

struct QmmArgs {
  const uint8_t* packed;
  int64_t N, K, M, row_bytes, packed_bytes;
  void* y;            // M x N, ydt (without the gather)
  int ydt;            // DT_F32 / DT_F16 / DT_BF16 (rounded to nearest even)
  float* part;        // [row tiles x token groups][ksplit][T][128] partial tiles (ksplit > 1)
  unsigned* tickets;  // [row tiles x token groups] (ksplit > 1)
  int bn, nacc;       // MMA N per accumulator, accumulators per CTA
  int ksplit, kbs;    // K splits, 256-blocks per split
  int64_t tile0;      // tile of CTA (0, 0): tiles are numbered row tile fastest
  int64_t row_tiles;
  int* err;
  // Fused row gather (world > 1, gsq_qmm_gather): output rows
  // [row0, row0 + N) of ntot go to every rank's region ([M][ntot] fp32, or
  // fp16 with yh, after a 256-byte header whose word p counts the tiles rank
  // p has delivered).
  float* gy[QMM_GATHER_MAX];
  unsigned* gflags[QMM_GATHER_MAX];
  float* mcy;         // or: the output through the regions' NVSwitch multicast address
  int yh;             // the regions hold fp16 values (round to nearest even)
  int gvec;           // 16-byte pieces of 4 (fp32) or 8 (fp16) consecutive rows are aligned in the regions
  int world, rank;
  int64_t row0, ntot;
};

// One output value: y, or every rank's gather region (coalesced per warp:
// 32 consecutive rows of one token).
template <bool GATHER>
__device__ __forceinline__ void qmm_store(const QmmArgs& a, int64_t m, int64_t erow, float v) {
  if constexpr (!GATHER) {
    store_out(a.y, a.ydt, m * a.N + erow, v);
    return;
  }
  const int64_t off = m * a.ntot + a.row0 + erow;
  if (a.yh) {
    // (multimem stores have no single-fp16 form: one store per rank through
    // the unicast mappings, which a multicast call also holds)
    const __half h = __float2half_rn(v);
#pragma unroll
    for (int p = 0; p < QMM_GATHER_MAX; p++)
      if (p < a.world) reinterpret_cast<__half*>(a.gy[p])[off] = h;
    return;
  }
  if (a.mcy) {
    // One store through the multicast address: the switch writes it into
    // every rank's region (this rank's included).
    asm volatile("multimem.st.relaxed.sys.global.f32 [%0], %1;" ::"l"(a.mcy + off), "f"(v) : "memory");
    return;
  }
#pragma unroll
  for (int p = 0; p < QMM_GATHER_MAX; p++)
    if (p < a.world) a.gy[p][off] = v;
}

// Four consecutive output rows [erow, erow + 4) of token m (16-byte
// aligned: a.gvec): one 16-byte store per rank, or one multicast store.
__device__ __forceinline__ void qmm_store_v4(const QmmArgs& a, int64_t m, int64_t erow, float4 v) {
  const int64_t off = m * a.ntot + a.row0 + erow;
  if (a.mcy) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(a.mcy + off), "f"(v.x),
                 "f"(v.y), "f"(v.z), "f"(v.w)
                 : "memory");
    return;
  }
#pragma unroll
  for (int p = 0; p < QMM_GATHER_MAX; p++)
    if (p < a.world) *reinterpret_cast<float4*>(a.gy[p] + off) = v;
}

// Eight consecutive output rows [erow, erow + 8) of token m as fp16 (16-byte
// aligned: a.gvec with a.yh).
__device__ __forceinline__ void qmm_store_h8(const QmmArgs& a, int64_t m, int64_t erow, uint4 v) {
  const int64_t off = m * a.ntot + a.row0 + erow;
  __half* mc = reinterpret_cast<__half*>(a.mcy);
  if (mc) {
    asm volatile("multimem.st.relaxed.sys.global.v4.f16x2 [%0], {%1, %2, %3, %4};" ::"l"(mc + off), "r"(v.x),
                 "r"(v.y), "r"(v.z), "r"(v.w)
                 : "memory");
    return;
  }
#pragma unroll
  for (int p = 0; p < QMM_GATHER_MAX; p++)
    if (p < a.world) *reinterpret_cast<uint4*>(reinterpret_cast<__half*>(a.gy[p]) + off) = v;
}

// A warp's 32 rows (lanes) x NJ tokens of a gathering epilogue: staged in
// shared memory (token-major), then written as 16-byte stores of 4 (fp32)
// or 8 (fp16) consecutive rows -- remote and multicast stores move whole
// 16-byte pieces instead of 4- or 2-byte ones.  `stage`: 32 * NJ floats of
// this warp.
template <int NJ>
__device__ __forceinline__ void gather_store_rows(const QmmArgs& a, float* stage, const float (&v)[NJ], int lane,
                                                  int64_t m_first, int64_t row_first) {
  static_assert(NJ % 8 == 0, "whole 8-row pieces per lane");
#pragma unroll
  for (int j = 0; j < NJ; j++) stage[j * 32 + lane] = v[j];
  __syncwarp();
  if (a.yh) {
#pragma unroll
    for (int i = 0; i < NJ / 8; i++) {
      const int idx = lane + 32 * i;         // (token, 8-row group) pairs
      const int t = idx >> 2, r8 = (idx & 3) * 8;
      const int64_t m = m_first + t, row = row_first + r8;
      if (m >= a.M || row >= a.N) continue;
      const float4 q0 = *reinterpret_cast<const float4*>(stage + t * 32 + r8);
      const float4 q1 = *reinterpret_cast<const float4*>(stage + t * 32 + r8 + 4);
      if (row + 7 < a.N) {
        const __half2 h0 = __floats2half2_rn(q0.x, q0.y), h1 = __floats2half2_rn(q0.z, q0.w);
        const __half2 h2 = __floats2half2_rn(q1.x, q1.y), h3 = __floats2half2_rn(q1.z, q1.w);
        qmm_store_h8(a, m, row,
                     make_uint4(*reinterpret_cast<const uint32_t*>(&h0), *reinterpret_cast<const uint32_t*>(&h1),
                                *reinterpret_cast<const uint32_t*>(&h2), *reinterpret_cast<const uint32_t*>(&h3)));
      } else {
        const float e[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
        for (int k = 0; k < 8 && row + k < a.N; k++) qmm_store<true>(a, m, row + k, e[k]);
      }
    }
    __syncwarp();
    return;
  }
#pragma unroll
  for (int i = 0; i < NJ / 4; i++) {
    const int idx = lane + 32 * i;         // (token, 4-row group) pairs
    const int t = idx >> 3, r4 = (idx & 7) * 4;
    const int64_t m = m_first + t, row = row_first + r4;
    if (m >= a.M || row >= a.N) continue;
    const float4 q = *reinterpret_cast<const float4*>(stage + t * 32 + r4);
    if (row + 3 < a.N) {
      qmm_store_v4(a, m, row, q);
    } else {
      const float e[4] = {q.x, q.y, q.z, q.w};
      for (int k = 0; k < 4 && row + k < a.N; k++) qmm_store<true>(a, m, row + k, e[k]);
    }
  }
  __syncwarp();
}

// End of a gathering call, one thread per CTA, after the decoder warps'
// barrier.  A CTA that completed an output tile (every CTA without split-K,
// the split that finishes the tile's reduction otherwise) adds 1 to this
// rank's word in every peer's region (release, system scope; the storing
// threads fenced their peer stores at system scope before the barrier).  The
// last CTA of the grid (gpu-scope ticket) then waits, bounded, until every
// peer's word in the own region reaches the running total of tiles of all
// calls on the region so far, this one included (acquire): when the kernel
// completes, every rank's tiles of this call are in every region.
// Every rank must make the same sequence of calls on a region.
__device__ void qmm_gather_signal(const QmmArgs& a, bool stored) {
  unsigned* own = a.gflags[a.rank];
  if (stored) {
    for (int p = 0; p < a.world; p++)
      if (p != a.rank)
        asm volatile("red.release.sys.global.add.u32 [%0], 1;" ::"l"(a.gflags[p] + a.rank) : "memory");
  }
  __threadfence();
  const unsigned ctas = gridDim.x * gridDim.y * gridDim.z;
  if (atomicAdd(own + QMM_GFLAG_TICKET, 1u) != ctas - 1u) return;
  own[QMM_GFLAG_TICKET] = 0u;
  // Running total of the tiles every peer has delivered into this region
  // once this call is done: calls on a region may differ in token count (a
  // shared prefill region sees prompts of any length), so the total grows
  // by this call's tile count, which every rank computes the same way.
  const unsigned expected = own[QMM_GFLAG_COUNT] + gridDim.x * gridDim.y;
  own[QMM_GFLAG_COUNT] = expected;
  const long long t0 = clock64();
  for (int p = 0; p < a.world; p++) {
    if (p == a.rank) continue;
    for (;;) {
      unsigned v;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(own + p) : "memory");
      if ((int)(v - expected) >= 0) break;
      if (clock64() - t0 > (1ll << 31)) {
        if (a.err) atomicExch(a.err, DEV_WAIT_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
  }
}

__device__ __forceinline__ uint32_t elect_lane0() { return (threadIdx.x & 31) == 0; }

// Barrier 2: the decoder warps only.
__device__ __forceinline__ void named_sync_decoders() {
  asm volatile("bar.sync 2, %0;" ::"n"(32 * QMM_DEC_WARPS) : "memory");
}

// tcgen05 wrappers ------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate) : "memory");
}
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int c0, int c1, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(map), "r"(c0), "r"(c1), "r"(smem_u32(bar)) : "memory");
}

// Shared-memory matrix descriptor: K-major, 128B swizzle, 8-row atoms of 1024 B.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)1 << 16;                 // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;       // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                 // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                 // SWIZZLE_128B
  return d;
}

// Instruction descriptor: D=f32, A=B=f16, both K-major, M=128, N=bn.
__host__ __device__ constexpr uint32_t f16_idesc(int bn) {
  return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(bn >> 3) << 17) | ((uint32_t)(QMM_BM >> 4) << 24);
}

// Store 8 fp16 values as one 16-byte chunk of a swizzled K-major row.
__device__ __forceinline__ void st_sw128(uint8_t* tile, int row, int chunk, const float (&v)[8]) {
  __half2 h[4];
#pragma unroll
  for (int j = 0; j < 4; j++) h[j] = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
  *reinterpret_cast<uint4*>(tile + row * 128 + ((chunk ^ (row & 7)) << 4)) = *reinterpret_cast<const uint4*>(h);
}

// GATHER: the instance used by gsq_qmm_gather (a separate instance, so the
// single-GPU kernel carries none of its code).
template <int T, bool GATHER>
__global__ void __launch_bounds__(QMM_THREADS, 1) qmm_kernel(const QmmArgs a, const __grid_constant__ CUtensorMap xmap) {
  using G = QmmGeom<T>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((0u - smem_u32(smem_raw)) & 1023u);  // 1024-aligned, shared provenance kept
  const int bn = a.bn, nacc = a.nacc, ttok = a.bn * a.nacc;
  const size_t bbytes = (size_t)ttok * 128;                   // one activation stage: T tokens x 64 k fp16
  const int NS = QmmPipe<T>::ns(bbytes);
  const int PST = QmmPipe<T>::pst(bbytes);
  uint8_t* astage = smem;                                     // NS x 16 KB
  uint8_t* bstage = astage + (size_t)NS * QMM_BM * 128;       // NS x T*128
  uint8_t* pstage = bstage + (size_t)NS * bbytes;             // PST x PSTAGE
  uint8_t* tab = pstage + (size_t)PST * G::PSTAGE;            // decode tables
  uint64_t* bars = reinterpret_cast<uint64_t*>(tab + G::TAB);
  uint64_t* full_a = bars;          // [NS]  count 8 (decoder warps)
  uint64_t* full_b = bars + 4;      // [NS]  count 1 (TMA)
  uint64_t* empty = bars + 8;       // [NS]  count 1 (tcgen05.commit)
  uint64_t* accf = bars + 20;       // [1]   count 1
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 21);
  unsigned* last_flag = reinterpret_cast<unsigned*>(bars + 22);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // This CTA's output tile: row tile fastest over the whole call; a launch
  // covers tiles [tile0, tile0 + gridDim.x * gridDim.y).
  const int64_t tile_id = a.tile0 + (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
  const int64_t n0 = (tile_id % a.row_tiles) * QMM_BM;
  const int m0 = (int)(tile_id / a.row_tiles) * ttok;
  const int split = blockIdx.z;
  const int kb0 = split * a.kbs;                                  // this CTA's 256-blocks
  const int nkb = min(a.kbs, (int)(a.K / QK) - kb0);
  const int nks = nkb * (QK / QMM_BK);
  const uint32_t tcols = ttok <= 32 ? 32 : ttok <= 64 ? 64 : ttok <= 128 ? 128 : ttok <= 256 ? 256 : 512;

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full_a[s], QMM_DEC_WARPS);
      mbar_init(&full_b[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, tcols);
  Fast<T>::load_tables(tab, threadIdx.x, blockDim.x);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_d = *tmem_slot;
  bool ok = true;

  if (warp == 0) {
    // ---------------- activation tiles (TMA) ----------------
    pdl_wait();  // the activations are written by the preceding kernel
    int s = 0, n = 0;  // stage and its use count, advanced without divisions
    for (int ks = 0; ks < nks && ok; ks++) {
      if (n > 0) ok = mbar_wait_bounded(&empty[s], (uint32_t)((n - 1) & 1), a.err);
      if (!ok) break;
      if (lane == 0) {
        mbar_arrive_expect_tx(&full_b[s], (uint32_t)bbytes);
        for (int j = 0; j < nacc; j++)
          tma_load_2d(bstage + (size_t)s * bbytes + (size_t)j * bn * 128, &xmap, kb0 * QK + ks * QMM_BK, m0 + j * bn,
                      &full_b[s]);
      }
      __syncwarp();
      if (++s == NS) { s = 0; n++; }
    }
  } else if (warp == 2) {
    // (idle: the decoder warps fetch their own packed rows)
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    const uint32_t idesc = f16_idesc(bn);
    int s = 0, n = 0;
    for (int ks = 0; ks < nks && ok; ks++, (++s == NS ? (s = 0, n++) : 0)) {
      ok = mbar_wait_bounded(&full_a[s], (uint32_t)(n & 1), a.err) &&
           mbar_wait_bounded(&full_b[s], (uint32_t)(n & 1), a.err);
      if (!ok) break;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t aaddr = smem_u32(astage + (size_t)s * QMM_BM * 128);
        const uint32_t baddr = smem_u32(bstage + (size_t)s * bbytes);
        for (int j = 0; j < nacc; j++) {
#pragma unroll
          for (int kk = 0; kk < QMM_BK / 16; kk++)
            tc_mma_f16(tmem_d + (uint32_t)(j * bn), sw128_desc(aaddr + kk * 32),
                       sw128_desc(baddr + (uint32_t)(j * bn * 128) + kk * 32), idesc, (ks | kk) != 0 ? 1u : 0u);
        }
        tc_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (lane == 0) tc_commit(accf);
    __syncwarp();
  } else {
    // ---------------- decoders + epilogue ----------------
    // Decoding: warp dw owns tile rows 16dw .. 16dw+15; lanes 2i and 2i+1
    // share row 16dw+i, `half` 0 decoding k 0..31 and `half` 1 k 32..63 of
    // every 64-wide step.  Each warp fetches its own rows' packed blocks with
    // per-thread 16-byte async copies into a PST-deep ring (every slot but
    // the one being decoded is in flight), so no producer or barrier sits
    // between HBM and the decoders.  In the epilogue the TMEM sub-partition
    // decides the rows.
    using F = Fast<T>;
    const int dw = warp - QMM_DEC0;
    const int half = lane & 1;
    const int r = 16 * dw + (lane >> 1);  // tile row decoded by this lane
    const int64_t row = n0 + r;
    const bool live = row < a.N;
    const int64_t roff = row * a.row_bytes;
    const __half2 off2 = __float2half2_rn(1152.f);
    const uintptr_t pbase = reinterpret_cast<uintptr_t>(a.packed);
    const uint64_t policy = l2_policy_evict_first();
    uint8_t* pslot = pstage + r * G::PROWB;
    // Copies block kb of this row into ring slot ps (this lane's alternate
    // 16-byte chunks); always commits a group so group counts stay uniform.
    auto fetch = [&](int kb, int ps) {
      if (live && kb < nkb) {
        const int64_t off = roff + (int64_t)(kb0 + kb) * G::BB;
        const int64_t end = off + G::BB;
        const int64_t off_al = off & ~int64_t(15);
        int64_t end_al = (end + 15) & ~int64_t(15);
        if (end_al > a.packed_bytes) end_al = end & ~int64_t(15);
        uint8_t* dst = pslot + (size_t)ps * G::PSTAGE;
        const int nch = (int)((end_al - off_al) >> 4);
        for (int c = half; c < nch; c += 2)
          cp_async16_stream(dst + 16 * c, reinterpret_cast<const void*>(pbase + off_al + 16 * c), policy);
        // Tail beyond the last 16-byte boundary of the buffer: plain loads.
        if (half == 0)
          for (int64_t t = max(end_al, off_al); t < end; t++) dst[t - off_al] = a.packed[t];
      }
      cp_async_commit();
    };
    for (int j = 0; j < PST; j++) fetch(j, j);
    int ps = 0;        // packed ring slot
    int s = 0, n = 0;  // A/B stage / use count
    for (int kb = 0; kb < nkb && ok; kb++) {
      if (PST == 3) cp_async_wait<2>(); else cp_async_wait<1>();  // block kb landed
      __syncwarp();  // both lanes' chunks of the row are visible
      const uint8_t* blk = pslot + (size_t)ps * G::PSTAGE + (int)((roff + (int64_t)(kb0 + kb) * G::BB) & 15);
      for (int q = 0; q < 4 && ok; q++, (++s == NS ? (s = 0, n++) : 0)) {
        if (n > 0) ok = mbar_wait_bounded(&empty[s], (uint32_t)((n - 1) & 1), a.err);
        if (!ok) break;
        uint8_t* trow = astage + (size_t)s * QMM_BM * 128 + r * 128;
        const int c32 = 2 * q + half;
        // 32 weights of this row: int8 entries -> exact fp16 integers via a
        // 0x64xx byte-permute (1024 + a + 128) - 1152, then one fp16 FMA with
        // the unit's scale/offset: w = a * S + B.
        uint32_t out[16];
        if (live) {
          __half2 S2[2], B2[2];
          if constexpr (F::UNIT == 32) {
            float S, B;
            F::affine(blk, c32, S, B);
            S2[0] = S2[1] = __float2half2_rn(S);
            B2[0] = B2[1] = __float2half2_rn(B);
          } else {
            float S0, B0, S1, B1;
            F::affine(blk, 2 * c32, S0, B0);
            F::affine(blk, 2 * c32 + 1, S1, B1);
            S2[0] = __float2half2_rn(S0); B2[0] = __float2half2_rn(B0);
            S2[1] = __float2half2_rn(S1); B2[1] = __float2half2_rn(B1);
          }
#pragma unroll
          for (int tq = 0; tq < 4; tq++) {
            uint32_t lo, hi;
            F::entry(blk, c32, tq, tab, lo, hi);
            const int u = F::BLOCKED ? (8 * tq) / F::UNIT : 0;
            const uint32_t w2[2] = {lo ^ 0x80808080u, hi ^ 0x80808080u};
#pragma unroll
            for (int h = 0; h < 2; h++) {
#pragma unroll
              for (int p = 0; p < 2; p++) {
                const uint32_t m = __byte_perm(w2[h], 0x64646464u, p ? 0x4342u : 0x4140u);
                __half2 v = __hsub2(*reinterpret_cast<const __half2*>(&m), off2);
                v = __hfma2(v, S2[u], B2[u]);
                // BLOCKED: 8 consecutive weights per entry; identity: lo/hi are
                // the 4-weight runs at 4tq and 16+4tq.
                const int idx = F::BLOCKED ? 4 * tq + 2 * h + p : (h ? 8 : 0) + 2 * tq + p;
                out[idx] = *reinterpret_cast<const uint32_t*>(&v);
              }
            }
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; j++) out[j] = 0u;
        }
#pragma unroll
        for (int c = 0; c < 4; c++) {
          const int chunk = 4 * half + c;
          *reinterpret_cast<uint4*>(trow + ((chunk ^ (r & 7)) << 4)) =
              make_uint4(out[4 * c], out[4 * c + 1], out[4 * c + 2], out[4 * c + 3]);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(&full_a[s]);
      }
      __syncwarp();  // the ring slot is no longer read: refill it
      fetch(kb + PST, ps);
      if (++ps == PST) ps = 0;
    }
    cp_async_wait<0>();
    // Epilogue rows: TMEM sub-partition (warp & 3) x lane; the two warps of a
    // sub-partition take half of the T columns each.
    const int sub = warp & 3, ehalf = dw >> 2;
    const int er = 32 * sub + lane;
    const int64_t erow = n0 + er;
    const bool elive = erow < a.N;
    // epilogue: this warp's TMEM lanes, half of the T columns
    pdl_launch_dependents();
    pdl_wait();  // global writes only after the preceding kernel completed
    if (ok) ok = mbar_wait_bounded(accf, 0u, a.err);
    tc_fence_after();
    const uint32_t lane_base = (uint32_t)(32 * sub) << 16;
    // Gathering epilogue staging: 2 KB per decoder warp in the A stages,
    // which no MMA reads any more (accf completed).
    float* gstage = reinterpret_cast<float*>(astage) + dw * 32 * 16;
    const int cols = ttok / 2;
    const int64_t tile = (int64_t)blockIdx.y * gridDim.x + blockIdx.x;
    if (a.ksplit == 1) {
      if (ok) {
        for (int j0 = ehalf * cols; j0 < (ehalf + 1) * cols; j0 += 16) {
          uint32_t vv[16];
          tmem_ld16(tmem_d + lane_base + (uint32_t)j0, vv);
          if constexpr (GATHER) {
            if (a.gvec) {  // whole warp: the staging needs every lane
              float f[16];
#pragma unroll
              for (int jj = 0; jj < 16; jj++) f[jj] = __uint_as_float(vv[jj]);
              gather_store_rows<16>(a, gstage, f, lane, (int64_t)m0 + j0, n0 + 32 * sub);
              continue;
            }
          }
          if (elive) {
#pragma unroll
            for (int jj = 0; jj < 16; jj++) {
              const int64_t m = (int64_t)m0 + j0 + jj;
              if (m < a.M) qmm_store<GATHER>(a, m, erow, __uint_as_float(vv[jj]));
            }
          }
        }
      }
    } else {
      // Partial tile of this split -> scratch [tile][split][T][128] (rows
      // contiguous: coalesced).  The tile's ticket then counts the splits
      // twice: the first ksplit arrivals say that every partial is written
      // (each split waits, bounded, until all are: the plan keeps every
      // split of a call resident at once), then every split sums its share
      // of the tile's 8-column chunks over all splits, in split order
      // (deterministic), and arrives again; the last of those arrivals
      // resets the ticket to zero for the next call.
      float* mine = a.part + ((tile * a.ksplit + split) * ttok) * QMM_BM;
      if (ok) {
        for (int j0 = ehalf * cols; j0 < (ehalf + 1) * cols; j0 += 16) {
          uint32_t vv[16];
          tmem_ld16(tmem_d + lane_base + (uint32_t)j0, vv);
#pragma unroll
          for (int jj = 0; jj < 16; jj++) mine[(int64_t)(j0 + jj) * QMM_BM + er] = __uint_as_float(vv[jj]);
        }
      }
      unsigned* tk = a.tickets + tile;
      named_sync_decoders();
      if (warp == QMM_DEC0 && lane == 0) {
        atom_add_acq_rel_gpu(tk, 1u);
        bool all_in = true;
        const long long t0 = clock64();
        for (;;) {
          unsigned v;
          asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(tk) : "memory");
          if (v >= (unsigned)a.ksplit) break;
          if (clock64() - t0 > (1ll << 31)) {
            if (a.err) atomicExch(a.err, DEV_WAIT_TIMEOUT);
            all_in = false;
            break;
          }
          __nanosleep(64);
        }
        *last_flag = all_in ? 1u : 0u;
      }
      named_sync_decoders();
      const bool reduce = ok && *last_flag != 0u;
      if (reduce) {
        // This split's chunks of 8 columns in this warp's column half: 8
        // columns x all splits (<= QMM_KSPLIT_MAX) of loads in flight.
        const float* base = a.part + (tile * a.ksplit * ttok) * QMM_BM;
        for (int c = split; c < cols / 8; c += a.ksplit) {
          const int j0 = ehalf * cols + 8 * c;
          if (m0 + j0 >= a.M) break;
          float v[QMM_KSPLIT_MAX][8];
#pragma unroll
          for (int z = 0; z < QMM_KSPLIT_MAX; z++) {
#pragma unroll
            for (int jj = 0; jj < 8; jj++)
              v[z][jj] = z < a.ksplit ? __ldcg(base + ((int64_t)z * ttok + j0 + jj) * QMM_BM + er) : 0.f;
          }
          float accs[8];
#pragma unroll
          for (int jj = 0; jj < 8; jj++) {
            float acc = v[0][jj];
#pragma unroll
            for (int z = 1; z < QMM_KSPLIT_MAX; z++) acc += v[z][jj];  // zeros beyond ksplit
            accs[jj] = acc;
          }
          if constexpr (GATHER) {
            if (a.gvec) {  // whole warp (the loop bounds are uniform over the warp)
              gather_store_rows<8>(a, gstage, accs, lane, (int64_t)m0 + j0, n0 + 32 * sub);
              continue;
            }
          }
          if (elive) {
#pragma unroll
            for (int jj = 0; jj < 8; jj++) {
              const int64_t m = (int64_t)m0 + j0 + jj;
              if (m < a.M) qmm_store<GATHER>(a, m, erow, accs[jj]);
            }
          }
        }
      }
      if constexpr (GATHER) {
        if (reduce) __threadfence_system();  // this thread's stores into the peers' regions
      }
      named_sync_decoders();
      if (warp == QMM_DEC0 && lane == 0) {
        const unsigned prev = atom_add_acq_rel_gpu(tk, 1u);
        const bool done = prev + 1u == 2u * (unsigned)a.ksplit;
        if (done) *tk = 0u;
        *last_flag = done && reduce ? 1u : 0u;  // the tile is complete: this split signals it
      }
    }
  }
  if constexpr (GATHER) {
    if (warp >= QMM_DEC0) {
      if (a.ksplit == 1) __threadfence_system();  // this thread's stores into the peers' regions
      named_sync_decoders();
      const bool signal = a.ksplit == 1 || *last_flag;
      if (warp == QMM_DEC0 && lane == 0) qmm_gather_signal(a, signal);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) tmem_dealloc(tmem_d, tcols);
}

// Activations -> fp16 (row-major [M, K]); the tensor map reads this copy.
// Eight values per thread and step (one 16-byte fp16 store; one 16-byte
// bf16 or two fp32 loads), four steps' loads issued before their stores;
// each value rounds to nearest even.  n8 = M*K/8 (K is a multiple of 256,
// x is 16-byte aligned).
__device__ __forceinline__ uint4 to_f16_8(const void* x, int dtype, int64_t i) {
  float f[8];
  if (dtype == DT_BF16) {
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(x) + i);
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int j = 0; j < 4; j++) {
      f[2 * j] = __uint_as_float(w[j] << 16);
      f[2 * j + 1] = __uint_as_float(w[j] & 0xFFFF0000u);
    }
  } else {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  }
  uint32_t h[4];
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const __half2 p = __floats2half2_rn(f[2 * j], f[2 * j + 1]);
    h[j] = *reinterpret_cast<const uint32_t*>(&p);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

__global__ void __launch_bounds__(256) to_f16_kernel(const void* x, int dtype, int64_t n8, uint4* out) {
  pdl_launch_dependents();
  pdl_wait();  // x is written by the preceding kernel; out may still be read by the previous matmul
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  for (; i + 3 * stride < n8; i += 4 * stride) {
    uint4 v[4];
#pragma unroll
    for (int u = 0; u < 4; u++) v[u] = to_f16_8(x, dtype, i + u * stride);
#pragma unroll
    for (int u = 0; u < 4; u++) out[i + u * stride] = v[u];
  }
  for (; i < n8; i += stride) out[i] = to_f16_8(x, dtype, i);
}

// --------------------------------------------------------------------------
// Host side.

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn get_encode_fn() {
  static EncodeTiledFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  }
  return fn;
}

// Launch plan: token tile T (one accumulator of round32(M) tokens up to 256,
// else two accumulators of up to 256 tokens each), row tiles x token groups,
// and a K split when that grid would leave most SMs idle.
static int qmm_sm_count() {
  static int sms = 0;
  if (!sms) {
    int dev = 0, n = 0;
    if (cudaGetDevice(&dev) == cudaSuccess &&
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0)
      sms = n;
    else {
      cudaGetLastError();
      sms = 148;
    }
  }
  return sms;
}

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

QmmPlan qmm_plan(int t, int64_t N, int64_t K, int64_t M, int x_dtype) {
  (void)t;
  QmmPlan p = {};
  if (M <= 256) {
    p.nacc = 1;
    p.bn = (int)std::max<int64_t>(32, (M + 31) / 32 * 32);
  } else {
    p.nacc = 2;
    const int64_t groups = (M + 511) / 512;
    const int64_t per = (M + groups - 1) / groups;            // tokens per group, <= 512
    p.bn = (int)std::min<int64_t>(256, ((per + 1) / 2 + 31) / 32 * 32);
  }
  const int64_t ttok = (int64_t)p.bn * p.nacc;
  p.row_tiles = (N + QMM_BM - 1) / QMM_BM;
  p.token_groups = (M + ttok - 1) / ttok;
  const int64_t ctas = p.row_tiles * p.token_groups;
  const int nkb = (int)(K / QK);
  const int sms = qmm_sm_count();
  p.ksplit = 1;
  p.whole_tiles = 0;
  int64_t split_tiles = ctas;  // tiles whose K is split (their partials live in the scratch)
  if (ctas * 4 < (int64_t)sms * 3 && ctas <= QMM_TICKETS) {
    p.ksplit = (int)std::max<int64_t>(1, std::min<int64_t>(std::min<int64_t>(nkb, QMM_KSPLIT_MAX), sms / ctas));
  } else if (ctas > sms && ctas % sms != 0 && (ctas % sms) * 2 <= sms) {
    // A last wave at most half full: its tiles split K over the idle SMs.
    const int64_t tail = ctas % sms;
    const int s = (int)std::min<int64_t>(std::min<int64_t>(nkb, QMM_KSPLIT_MAX), sms / tail);
    if (s >= 2) {
      p.whole_tiles = ctas - tail;
      p.ksplit = s;
      split_tiles = tail;
    }
  }
  p.kbs = (nkb + p.ksplit - 1) / p.ksplit;
  p.ksplit = (nkb + p.kbs - 1) / p.kbs;
  if (p.ksplit == 1) p.whole_tiles = 0;
  // Nothing but tickets is ever written to [0, QMM_TICKET_BYTES), whatever
  // the shape, so a workspace zero-filled once keeps zero tickets.
  size_t off = QMM_TICKET_BYTES;
  if (p.ksplit > 1) {
    p.off_part = off;
    off += align256((size_t)split_tiles * p.ksplit * ttok * QMM_BM * sizeof(float));
  }
  p.off_x16 = off;
  if (x_dtype != DT_F16) off += align256((size_t)M * K * 2);
  p.workspace = off > QMM_TICKET_BYTES ? off : 0;
  return p;
}

size_t qmm_workspace_bytes(int t, int64_t N, int64_t K, int64_t M, int x_dtype) {
  return qmm_plan(t, N, K, M, x_dtype).workspace;
}

template <int T, bool GATHER>
static cudaError_t qmm_launch_g(const QmmArgs& a, const QmmPlan& p, const CUtensorMap& map, cudaStream_t st) {
  const size_t smem = QmmPipe<T>::smem((size_t)a.bn * a.nacc * 128);
  static int configured[64] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 64 && configured[dev] < (int)smem) {
    cudaError_t e =
        cudaFuncSetAttribute(qmm_kernel<T, GATHER>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    configured[dev] = (int)smem;
  }
  if (p.whole_tiles == 0) {
    const dim3 grid((unsigned)p.row_tiles, (unsigned)p.token_groups, (unsigned)p.ksplit);
    return launch_pdl(qmm_kernel<T, GATHER>, grid, dim3(QMM_THREADS), smem, st, a, map);
  }
  // Full waves of whole-K tiles, then the last wave's tiles split along K
  // (every split CTA of that launch fits on the GPU at once).
  QmmArgs w = a;
  w.ksplit = 1;
  w.kbs = (int)(a.K / QK);
  w.tile0 = 0;
  cudaError_t e = launch_pdl(qmm_kernel<T, GATHER>, dim3((unsigned)p.whole_tiles, 1, 1), dim3(QMM_THREADS), smem,
                             st, w, map);
  if (e != cudaSuccess) return e;
  QmmArgs s = a;
  s.tile0 = p.whole_tiles;
  const int64_t rest = p.row_tiles * p.token_groups - p.whole_tiles;
  return launch_pdl(qmm_kernel<T, GATHER>, dim3((unsigned)rest, 1, (unsigned)p.ksplit), dim3(QMM_THREADS), smem, st,
                    s, map);
}

template <int T>
static cudaError_t qmm_launch_t(const QmmArgs& a, const QmmPlan& p, const CUtensorMap& map, cudaStream_t st) {
  return a.world > 1 ? qmm_launch_g<T, true>(a, p, map, st) : qmm_launch_g<T, false>(a, p, map, st);
}

#define GSQ_QMM_LAUNCH_CASE(TT) case TT: return qmm_launch_t<TT>(a, p, map, st);

// ws holds the plan's scratch (zero-filled once by the caller; the ticket
// region is left zero-filled by every call).
cudaError_t qmm_launch(int t, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int64_t M,
                       void* y, int y_dtype, void* ws, int* err, cudaStream_t st, const char** why,
                       const QmmGather* gather) {
  const QmmPlan p = qmm_plan(t, N, K, M, x_dtype);
  uint8_t* wsb = static_cast<uint8_t*>(ws);
  __half* x16 = reinterpret_cast<__half*>(wsb + p.off_x16);
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) { *why = "cuTensorMapEncodeTiled unavailable"; return cudaErrorNotSupported; }
  if (x_dtype != DT_F16) {
    // about four 8-value steps per thread, at most 8 CTAs of 256 per SM
    const int64_t n8 = M * K / 8;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>((n8 + 1023) / 1024, (int64_t)qmm_sm_count() * 8));
    cudaError_t e = launch_pdl(to_f16_kernel, dim3((unsigned)grid), dim3(256), 0, st, x, x_dtype, n8,
                               reinterpret_cast<uint4*>(x16));
    if (e != cudaSuccess) return e;
  } else {
    x16 = reinterpret_cast<__half*>(const_cast<void*>(x));
  }
  QmmArgs a;
  a.packed = packed; a.N = N; a.K = K; a.M = M;
  a.row_bytes = (K / QK) * block_bytes(t);
  a.packed_bytes = N * a.row_bytes;
  a.y = y; a.ydt = y_dtype; a.err = err;
  a.bn = p.bn; a.nacc = p.nacc; a.ksplit = p.ksplit; a.kbs = p.kbs;
  a.tickets = p.ksplit > 1 ? reinterpret_cast<unsigned*>(wsb) : nullptr;
  a.tile0 = 0;
  a.row_tiles = p.row_tiles;
  a.part = p.ksplit > 1 ? reinterpret_cast<float*>(wsb + p.off_part) : nullptr;
  a.world = 0;
  a.rank = 0;
  a.row0 = 0;
  a.ntot = N;
  for (int i = 0; i < QMM_GATHER_MAX; i++) {
    a.gy[i] = nullptr;
    a.gflags[i] = nullptr;
  }
  a.mcy = nullptr;
  a.yh = 0;
  a.gvec = 0;
  if (gather && gather->world > 1) {
    if (gather->world > QMM_GATHER_MAX || gather->rank < 0 || gather->rank >= gather->world) {
      *why = "invalid gather world/rank";
      return cudaErrorInvalidValue;
    }
    a.world = gather->world;
    a.rank = gather->rank;
    a.row0 = gather->row0;
    a.ntot = gather->ntot;
    for (int i = 0; i < gather->world; i++) {
      uint8_t* r = static_cast<uint8_t*>(gather->regions[i]);
      a.gflags[i] = reinterpret_cast<unsigned*>(r);
      a.gy[i] = reinterpret_cast<float*>(r + 256);
    }
    if (gather->multicast) a.mcy = reinterpret_cast<float*>(static_cast<uint8_t*>(gather->multicast) + 256);
    a.yh = y_dtype == DT_F16 ? 1 : 0;
    const int piece = a.yh ? 8 : 4;  // rows per 16-byte piece
    a.gvec = (gather->row0 % piece == 0 && gather->ntot % piece == 0) ? 1 : 0;
  }
  CUtensorMap map;
  const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)M};
  const cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  const cuuint32_t box[2] = {QMM_BK, (cuuint32_t)a.bn};
  const cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, x16, dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) { *why = "cuTensorMapEncodeTiled failed"; return cudaErrorInvalidValue; }
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMM_LAUNCH_CASE) }
  return cudaErrorInvalidValue;
}

}  // namespace gsq
