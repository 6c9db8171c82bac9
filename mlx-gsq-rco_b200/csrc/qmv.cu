// Fused dequantize + matvec (QMV) over packed GGUF super-blocks, sm_100a.
//
// Replaces the reference's per-type Metal matvec kernels
// (mlx_gsq/runtime/kernels/qmv.py:76-528, dispatched by quantized_matvec,
// qmv.py:537-576).  y[b, n] = sum_k x[b, k] * deq(W)[n, k] for a few
// activation rows b (decode), W stored as N rows of K/256 packed blocks.
//
// Design (B200):
//  * Work unit = 16 weight rows x one K-slice per warp; a CTA of 4 warps owns
//    64 rows and one K-slice, so the grid is (N/64, slices, row-pairs).  The
//    host picks the slice count so that the grid fills the 148 SMs in one
//    wave; partial sums of the slices are combined deterministically by the
//    last CTA to finish a row group (an atomic ticket, no spinning).
//  * Packed bytes stream HBM -> shared memory with 1-D bulk async copies
//    (one per weight row and chunk, issued by 16 lanes in parallel) into a
//    3-stage per-warp ring completed on mbarriers; waits are time-bounded.
//  * Activations are quantised once per CTA into two int8 levels per 32-wide
//    group (x ~= s * (hi + lo/256)), so each weight is decoded to an int8
//    value a_k (gsq_fast.cuh) and multiplied on the tensor cores with
//    mma.sync.m16n8k32.s8 -- decode cost is a few integer ops per 8 weights.
//  * The 8 MMA columns carry (unit, batch row, level) triples; each quad lane
//    ends up holding the integer dot products of a different sub-block, which
//    it scales once: acc += S_u * s_x * (256*C_hi + C_lo) + B_u * sum(x_u).
#include <algorithm>

#include "gsq_fast.cuh"
#include "gsq_host.h"

namespace gsq {

constexpr int QMV_WARPS = 4;
constexpr int QMV_ROWS = 16 * QMV_WARPS;
constexpr int QMV_STAGES = 2;
constexpr int QMV_THREADS = 32 * QMV_WARPS;
constexpr int QMV_MAX_SLICE_BLOCKS = 32;
// Split-K scratch layout: a fixed region of ticket counters first, then the
// partial sums.  Every completed call returns the tickets it used to zero, and
// no call ever writes partial sums over the ticket region, so one zero-filled
// workspace can serve calls of any shape in sequence.
constexpr int QMV_TICKET_SLOTS = 65536;
constexpr size_t QMV_TICKET_BYTES = QMV_TICKET_SLOTS * sizeof(unsigned);

struct QmvArgs {
  const uint8_t* packed;
  int64_t N, K, row_bytes;
  int64_t packed_bytes;
  const void* x;
  int x_dtype;
  int rows;        // activation rows
  void* y;
  int y_dtype;
  int kblocks;     // K / 256
  int bps;         // blocks per K-slice
  int slices;
  float* partial;  // [slices][rows_pad][N] when slices > 1
  unsigned* tickets;
  int* err;
};

template <int T>
struct QmvGeom {
  static constexpr int BB = block_bytes(T);
  static constexpr int CB = BB <= 66 ? 8 : BB <= 98 ? 4 : 2;       // blocks per chunk (~400-600 B a row)
  static constexpr int ROWB = ((CB * BB + 30) + 15) / 16 * 16;     // staged row stride
  static constexpr int STAGE = 16 * ROWB;
  static constexpr int TAB = (Fast<T>::TAB_BYTES + 127) / 128 * 128;
};

template <int T, int NB>
__host__ __device__ constexpr size_t qmv_smem_bytes(int bps) {
  // tables | mbarriers | xq [NB][2][KS] | xs [NB][KS/32] | xsum [NB][KS/16] | stages
  return (size_t)QmvGeom<T>::TAB + 128 + (size_t)NB * 2 * bps * 256 + (size_t)NB * bps * 8 * 4 +
         (size_t)NB * bps * 16 * 4 + (size_t)QMV_WARPS * QMV_STAGES * QmvGeom<T>::STAGE + 128;
}

// Load 32 consecutive activations starting at element `i` (a multiple of 32;
// the row base is 16-byte aligned) with 16-byte loads.
template <typename XT> __device__ __forceinline__ void load32(const void* x, int64_t i, float (&v)[32]);
template <> __device__ __forceinline__ void load32<float>(const void* x, int64_t i, float (&v)[32]) {
  const float4* p = reinterpret_cast<const float4*>(reinterpret_cast<const float*>(x) + i);
#pragma unroll
  for (int j = 0; j < 8; j++) {
    const float4 f = p[j];
    v[4 * j] = f.x; v[4 * j + 1] = f.y; v[4 * j + 2] = f.z; v[4 * j + 3] = f.w;
  }
}
template <> __device__ __forceinline__ void load32<__half>(const void* x, int64_t i, float (&v)[32]) {
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __half*>(x) + i);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint4 u = p[j];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; t++) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[t]));
      v[8 * j + 2 * t] = f.x; v[8 * j + 2 * t + 1] = f.y;
    }
  }
}
template <> __device__ __forceinline__ void load32<__nv_bfloat16>(const void* x, int64_t i, float (&v)[32]) {
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const __nv_bfloat16*>(x) + i);
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const uint4 u = p[j];
    const uint32_t w[4] = {u.x, u.y, u.z, u.w};
#pragma unroll
    for (int t = 0; t < 4; t++) {
      v[8 * j + 2 * t] = __uint_as_float(w[t] << 16);
      v[8 * j + 2 * t + 1] = __uint_as_float(w[t] & 0xFFFF0000u);
    }
  }
}

// Quantise the activation slice for this CTA into shared memory: per 32-wide
// group, x ~= s * (hi + lo/256) with int8 hi, lo and s = max|x|/127; also the
// fp32 sums of each 16-wide half (for the per-unit offsets B_u).
template <int NB, typename XT>
__device__ void qmv_quantize_x(const QmvArgs& a, int k0, int ks, int ksmax, int batch0, int8_t* xq,
                               float* xs, float* xsum) {
  const int ng = ks / 32;
  for (int task = threadIdx.x; task < NB * ng; task += blockDim.x) {
    const int b = task / ng, gi = task - b * ng;
    const int row = batch0 + b;
    int8_t* qh = xq + (size_t)(2 * b) * ksmax + gi * 32;
    int8_t* ql = qh + ksmax;
    if (row >= a.rows) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(qh)[0] = z; reinterpret_cast<uint4*>(qh)[1] = z;
      reinterpret_cast<uint4*>(ql)[0] = z; reinterpret_cast<uint4*>(ql)[1] = z;
      xs[b * (ksmax / 32) + gi] = 0.f;
      xsum[b * (ksmax / 16) + 2 * gi] = 0.f;
      xsum[b * (ksmax / 16) + 2 * gi + 1] = 0.f;
      continue;
    }
    float v[32];
    load32<XT>(a.x, (int64_t)row * a.K + k0 + gi * 32, v);
    float amax = 0.f, s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int j = 0; j < 32; j++) {
      amax = fmaxf(amax, fabsf(v[j]));
      if (j < 16) s0 += v[j]; else s1 += v[j];
    }
    const float inv = amax > 0.f ? 127.f / amax : 0.f;
    uint32_t wh[8], wl[8];
#pragma unroll
    for (int j = 0; j < 8; j++) {
      wh[j] = 0u; wl[j] = 0u;
#pragma unroll
      for (int t = 0; t < 4; t++) {
        const float u = v[4 * j + t] * inv;
        const float h = fminf(fmaxf(rintf(u), -127.f), 127.f);
        const float l = fminf(fmaxf(rintf((u - h) * 256.f), -127.f), 127.f);
        wh[j] |= ((uint32_t)(uint8_t)(int8_t)(int)h) << (8 * t);
        wl[j] |= ((uint32_t)(uint8_t)(int8_t)(int)l) << (8 * t);
      }
    }
    reinterpret_cast<uint4*>(qh)[0] = make_uint4(wh[0], wh[1], wh[2], wh[3]);
    reinterpret_cast<uint4*>(qh)[1] = make_uint4(wh[4], wh[5], wh[6], wh[7]);
    reinterpret_cast<uint4*>(ql)[0] = make_uint4(wl[0], wl[1], wl[2], wl[3]);
    reinterpret_cast<uint4*>(ql)[1] = make_uint4(wl[4], wl[5], wl[6], wl[7]);
    xs[b * (ksmax / 32) + gi] = amax / (127.f * 256.f);
    xsum[b * (ksmax / 16) + 2 * gi] = s0;
    xsum[b * (ksmax / 16) + 2 * gi + 1] = s1;
  }
}

template <int T, int NB>
__global__ void __launch_bounds__(QMV_THREADS, 4) qmv_kernel(const QmvArgs a) {
  using F = Fast<T>;
  using G = QmvGeom<T>;
  constexpr int UNIT = F::UNIT;
  constexpr int UPS = 4 / NB;            // units per set
  constexpr int KSET = UNIT * UPS;       // k per set
  constexpr int MMAS = KSET / 32;        // MMAs per set
  constexpr int SETS = QK / KSET;        // sets per block
  static_assert(MMAS >= 1, "set must cover at least one MMA");
  static_assert(F::BLOCKED || UNIT == 32, "identity mapping needs 32-wide units");

  extern __shared__ __align__(128) uint8_t smem[];
  const int ksmax = a.bps * QK;
  uint8_t* tab = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::TAB);
  int8_t* xq = reinterpret_cast<int8_t*>(smem + G::TAB + 128);
  float* xs = reinterpret_cast<float*>(xq + (size_t)NB * 2 * ksmax);
  float* xsum = xs + NB * (ksmax / 32);
  uint8_t* stages = reinterpret_cast<uint8_t*>(xsum + NB * (ksmax / 16));
  stages += (0u - smem_u32(stages)) & 127u;  // align in the shared window, keeping shared provenance

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int row_group = blockIdx.x, slice = blockIdx.y, btile = blockIdx.z;
  const int64_t row0 = (int64_t)row_group * QMV_ROWS + warp * 16;
  const int blk0 = slice * a.bps;
  const int nblk = min(a.bps, a.kblocks - blk0);
  const int nchunks = (nblk + G::CB - 1) / G::CB;
  uint64_t* wbars = bars + warp * QMV_STAGES;
  uint8_t* wstage = stages + (size_t)warp * QMV_STAGES * G::STAGE;
  const uintptr_t pbase = reinterpret_cast<uintptr_t>(a.packed);
  const uint64_t policy = l2_policy_evict_first();

  if (lane == 0)
    for (int s = 0; s < QMV_STAGES; s++) mbar_init(&wbars[s], 1);
  fence_mbar_init();
  __syncwarp();

  // Stage chunk c of this warp's 16 rows: lanes 0..15 each copy one row span.
  auto issue = [&](int c) {
    const int s = c % QMV_STAGES;
    uint32_t bytes = 0;
    if (lane < 16) {
      const int64_t r = row0 + lane;
      if (r < a.N) {
        const int nb_c = min(G::CB, nblk - c * G::CB);
        const int64_t off = r * a.row_bytes + (int64_t)(blk0 + c * G::CB) * G::BB;
        const int64_t end = off + (int64_t)nb_c * G::BB;
        const int64_t off_al = off & ~int64_t(15);
        int64_t end_al = (end + 15) & ~int64_t(15);
        if (end_al > a.packed_bytes) end_al = end & ~int64_t(15);
        uint8_t* dst = wstage + (size_t)s * G::STAGE + lane * G::ROWB;
        if (end_al > off_al) {
          bytes = (uint32_t)(end_al - off_al);
          fence_proxy_async_smem();
          bulk_g2s_stream(dst, reinterpret_cast<const void*>(pbase + off_al), bytes, &wbars[s], policy);
        }
        // Tail beyond the last 16-byte boundary of the buffer: plain loads.
        for (int64_t t = max(end_al, off_al); t < end; t++) dst[t - off_al] = a.packed[t];
      }
    }
    const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
    __syncwarp();
    if (lane == 0) mbar_arrive_expect_tx(&wbars[s], total);
  };

  const int npro = min(QMV_STAGES, nchunks);
  for (int c = 0; c < npro; c++) issue(c);

  F::load_tables(tab, threadIdx.x, blockDim.x);
  // Everything above reads only weights and tables; from here on the kernel
  // reads activations / scratch that an earlier kernel in the stream may write.
  pdl_wait();
  if (a.x_dtype == DT_F16)
    qmv_quantize_x<NB, __half>(a, blk0 * QK, nblk * QK, ksmax, btile * NB, xq, xs, xsum);
  else if (a.x_dtype == DT_BF16)
    qmv_quantize_x<NB, __nv_bfloat16>(a, blk0 * QK, nblk * QK, ksmax, btile * NB, xq, xs, xsum);
  else
    qmv_quantize_x<NB, float>(a, blk0 * QK, nblk * QK, ksmax, btile * NB, xq, xs, xsum);
  __syncthreads();

  // Per-thread constants of the activation operand (column g of the MMA).
  const int pcol = g >> 1, level = g & 1;
  const int s_col = pcol / NB, b_col = pcol % NB;
  const int8_t* xrow = xq + (size_t)(2 * b_col + level) * ksmax;
  // Epilogue identity of this lane: unit s_ep of each set, activation row b_ep.
  const int s_ep = tq / NB, b_ep = tq % NB;
  const float* xs_row = xs + b_ep * (ksmax / 32);
  const float* xsum_row = xsum + b_ep * (ksmax / 16);

  const int64_t roff0 = (row0 + g) * a.row_bytes + (int64_t)blk0 * G::BB;
  const int64_t roff1 = (row0 + g + 8) * a.row_bytes + (int64_t)blk0 * G::BB;

  float acc0 = 0.f, acc1 = 0.f;
  bool ok = true;
  int waited = 0;
  for (int c = 0; c < nchunks && ok; c++) {
    const int s = c % QMV_STAGES;
    ok = mbar_wait_bounded(&wbars[s], (uint32_t)((c / QMV_STAGES) & 1), a.err);
    if (!ok) break;
    waited = c + 1;
    const int nb_c = min(G::CB, nblk - c * G::CB);
    const int64_t coff = (int64_t)c * G::CB * G::BB;
    const uint8_t* st = wstage + (size_t)s * G::STAGE;
    const uint8_t* r0p = st + g * G::ROWB + (int)((roff0 + coff) & 15);
    const uint8_t* r1p = st + (g + 8) * G::ROWB + (int)((roff1 + coff) & 15);
    for (int bi = 0; bi < nb_c; bi++) {
      const uint8_t* b0 = r0p + bi * G::BB;
      const uint8_t* b1 = r1p + bi * G::BB;
      const int kblk = (c * G::CB + bi) * QK;
#pragma unroll
      for (int set = 0; set < SETS; set++) {
        const int kset = kblk + set * KSET;
        // Activation words for the one MMA of this set where column g is live.
        uint32_t xw0, xw1;
        int jsel;
        bool live;
        if constexpr (UNIT == 32) {
          jsel = s_col;
          live = true;
          if constexpr (F::BLOCKED) {
            const uint2 w = lds64(reinterpret_cast<const uint8_t*>(xrow + kset + 32 * s_col + 8 * tq));
            xw0 = w.x; xw1 = w.y;
          } else {
            xw0 = lds32(reinterpret_cast<const uint8_t*>(xrow + kset + 32 * s_col + 4 * tq));
            xw1 = lds32(reinterpret_cast<const uint8_t*>(xrow + kset + 32 * s_col + 16 + 4 * tq));
          }
        } else {
          jsel = s_col >> 1;
          live = (s_col & 1) == (tq >> 1);
          const uint2 w = lds64(reinterpret_cast<const uint8_t*>(xrow + kset + 32 * jsel + 8 * tq));
          xw0 = live ? w.x : 0u;
          xw1 = live ? w.y : 0u;
        }
        // Two independent accumulator chains (even / odd MMAs) halve the
        // dependent tensor-core latency per set.
        int C[4] = {0, 0, 0, 0}, Cb[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < MMAS; j++) {
          const int c32 = set * MMAS + j;
          uint32_t a0, a1, a2, a3;
          F::entry(b0, c32, tq, tab, a0, a2);
          F::entry(b1, c32, tq, tab, a1, a3);
          const bool on = (j == jsel);
          if (j & 1) mma_s8(Cb, a0, a1, a2, a3, on ? xw0 : 0u, on ? xw1 : 0u);
          else mma_s8(C, a0, a1, a2, a3, on ? xw0 : 0u, on ? xw1 : 0u);
        }
        if constexpr (MMAS > 1) {
#pragma unroll
          for (int i = 0; i < 4; i++) C[i] += Cb[i];
        }
        (void)live;
        const int unit = set * UPS + s_ep;
        const int ku = kblk + unit * UNIT;
        const float xsv = xs_row[ku >> 5];
        float S0, B0, S1, B1;
        F::affine(b0, unit, S0, B0);
        F::affine(b1, unit, S1, B1);
        const float d0 = (float)(C[0] * 256 + C[1]) * xsv;
        const float d1 = (float)(C[2] * 256 + C[3]) * xsv;
        acc0 = fmaf(S0, d0, acc0);
        acc1 = fmaf(S1, d1, acc1);
        if constexpr (F::HAS_BIAS) {
          float xu = xsum_row[ku >> 4];
          if constexpr (UNIT == 32) xu += xsum_row[(ku >> 4) + 1];
          acc0 = fmaf(B0, xu, acc0);
          acc1 = fmaf(B1, xu, acc1);
        }
      }
    }
    __syncwarp();
    if (c + QMV_STAGES < nchunks) issue(c + QMV_STAGES);
  }
  pdl_launch_dependents();
  if (!ok) {
    // Drain the copies this warp still has in flight before the CTA exits.
    for (int c = waited; c < min(nchunks, waited + QMV_STAGES); c++)
      mbar_wait_bounded(&wbars[c % QMV_STAGES], (uint32_t)((c / QMV_STAGES) & 1), nullptr);
  }

  // Sum the quad lanes that hold the same activation row.
  if constexpr (NB == 1) {
    acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
    acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
  }
  acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
  acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);

  const int batch = btile * NB + b_ep;
  const int64_t rg0 = row0 + g, rg1 = row0 + g + 8;
  const bool writer = ok && tq < NB && batch < a.rows;
  if (a.slices == 1) {
    if (writer) {
      if (rg0 < a.N) store_out(a.y, a.y_dtype, (int64_t)batch * a.N + rg0, acc0);
      if (rg1 < a.N) store_out(a.y, a.y_dtype, (int64_t)batch * a.N + rg1, acc1);
    }
    return;
  }
  const int rows_pad = gridDim.z * NB;
  if (writer) {
    float* p = a.partial + ((int64_t)slice * rows_pad + batch) * a.N;
    if (rg0 < a.N) p[rg0] = acc0;
    if (rg1 < a.N) p[rg1] = acc1;
  }
  __shared__ int s_last;
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const unsigned t = atomicAdd(&a.tickets[row_group * gridDim.z + btile], 1u);
    s_last = (t == (unsigned)(a.slices - 1));
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int i = threadIdx.x; i < QMV_ROWS * NB; i += blockDim.x) {
    const int b = i / QMV_ROWS;
    const int64_t r = (int64_t)row_group * QMV_ROWS + (i - b * QMV_ROWS);
    const int bt = btile * NB + b;
    if (r >= a.N || bt >= a.rows) continue;
    float sum = 0.f;
    for (int sl = 0; sl < a.slices; sl++) sum += __ldcg(a.partial + ((int64_t)sl * rows_pad + bt) * a.N + r);
    store_out(a.y, a.y_dtype, (int64_t)bt * a.N + r, sum);
  }
  if (threadIdx.x == 0) a.tickets[row_group * gridDim.z + btile] = 0u;
}

// --------------------------------------------------------------------------
// Host side.

template <int T, int NB>
static size_t qmv_smem(int bps) { return qmv_smem_bytes<T, NB>(bps); }

// Resident CTAs per SM for an instantiation and its shared-memory size (the
// occupancy API when a device is present, else a shared-memory estimate).
template <int T, int NB>
static int qmv_occupancy(size_t smem) {
  static size_t cached_smem = 0;
  static int cached_occ = 0;
  if (cached_occ > 0 && cached_smem == smem) return cached_occ;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qmv_kernel<T, NB>, QMV_THREADS, smem) != cudaSuccess ||
      occ <= 0) {
    cudaGetLastError();
    occ = (int)std::max<size_t>(1, std::min<size_t>(16, (227u * 1024u) / (smem + 1024)));
  }
  cached_smem = smem;
  cached_occ = occ;
  return occ;
}

static int qmv_sm_count() {
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

// Blocks per K-slice so that row_groups x slices fills the resident CTA slots
// of the GPU in a single wave (every CTA streams about the same bytes).
static int qmv_pick_bps(int64_t row_groups, int kblocks, int slots) {
  int slices = (int)std::max<int64_t>(1, slots / std::max<int64_t>(1, row_groups));
  slices = std::min(slices, kblocks);
  int bps = (kblocks + slices - 1) / slices;
  bps = std::min(bps, QMV_MAX_SLICE_BLOCKS);
  return std::max(bps, 1);
}

#define GSQ_QMV_SMEM_CASE(TT)                                                   \
  case TT:                                                                      \
    return nb == 1 ? qmv_smem<TT, 1>(bps) : qmv_smem<TT, 2>(bps);

static size_t qmv_smem_dispatch(int t, int nb, int bps) {
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_SMEM_CASE) }
  return 0;
}

#define GSQ_QMV_OCC_CASE(TT)                                                                       \
  case TT:                                                                                         \
    return nb == 1 ? qmv_occupancy<TT, 1>(qmv_smem<TT, 1>(bps)) : qmv_occupancy<TT, 2>(qmv_smem<TT, 2>(bps));

static int qmv_occ_dispatch(int t, int nb, int bps) {
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_OCC_CASE) }
  return 1;
}

QmvPlan qmv_plan(int t, int64_t N, int64_t K, int rows) {
  QmvPlan p;
  const int kblocks = (int)(K / QK);
  p.nb = rows == 1 ? 1 : 2;
  p.btiles = (rows + p.nb - 1) / p.nb;
  p.row_groups = (int)((N + QMV_ROWS - 1) / QMV_ROWS);
  // The occupancy is evaluated at the largest slice (the smem of the x slice
  // grows with it), so the chosen grid never exceeds one wave.
  const int occ = qmv_occ_dispatch(t, p.nb, std::min(kblocks, QMV_MAX_SLICE_BLOCKS));
  const int slots = occ * qmv_sm_count();
  p.bps = qmv_pick_bps((int64_t)p.row_groups * p.btiles, kblocks, slots);
  p.slices = (kblocks + p.bps - 1) / p.bps;
  if ((int64_t)p.row_groups * p.btiles > QMV_TICKET_SLOTS) {  // too many row groups to ticket: no split
    p.bps = kblocks;
    p.slices = 1;
  }
  p.smem = qmv_smem_dispatch(t, p.nb, p.bps);
  p.workspace = 0;
  if (p.slices > 1) {
    const size_t partial = (size_t)p.slices * p.btiles * p.nb * N * sizeof(float);
    p.workspace = QMV_TICKET_BYTES + partial;
  }
  return p;
}

template <int T, int NB>
static cudaError_t qmv_launch_t(const QmvArgs& a, const QmvPlan& p, cudaStream_t st) {
  auto kern = qmv_kernel<T, NB>;
  static int configured[64] = {0};  // max dynamic smem already set, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || (int)p.smem > configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = (int)p.smem;
  }
  return launch_pdl(kern, dim3(p.row_groups, p.slices, p.btiles), dim3(QMV_THREADS), p.smem, st, a);
}

#define GSQ_QMV_LAUNCH_CASE(TT) \
  case TT:                      \
    return p.nb == 1 ? qmv_launch_t<TT, 1>(a, p, st) : qmv_launch_t<TT, 2>(a, p, st);

static cudaError_t qmv_launch(int t, const QmvArgs& a, const QmvPlan& p, cudaStream_t st) {
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_LAUNCH_CASE) }
  return cudaErrorInvalidValue;
}

cudaError_t qmv_run(int t, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int rows,
                    void* y, int y_dtype, void* ws, const QmvPlan& p, int* err, cudaStream_t st) {
  QmvArgs a;
  a.packed = packed;
  a.N = N;
  a.K = K;
  a.row_bytes = (K / QK) * block_bytes(t);
  a.packed_bytes = N * a.row_bytes;
  a.x = x;
  a.x_dtype = x_dtype;
  a.rows = rows;
  a.y = y;
  a.y_dtype = y_dtype;
  a.kblocks = (int)(K / QK);
  a.bps = p.bps;
  a.slices = p.slices;
  a.partial = nullptr;
  a.tickets = nullptr;
  if (p.slices > 1) {
    a.tickets = static_cast<unsigned*>(ws);
    a.partial = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + QMV_TICKET_BYTES);
  }
  a.err = err;
  return qmv_launch(t, a, p, st);
}

}  // namespace gsq
