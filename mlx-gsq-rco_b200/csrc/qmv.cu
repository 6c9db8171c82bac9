// Fused dequantize + matvec (QMV) over packed GGUF super-blocks, sm_100a.
//
// Replaces the reference's per-type Metal matvec kernels
// (mlx_gsq/runtime/kernels/qmv.py:76-528, dispatched by quantized_matvec,
// qmv.py:537-576).  y[b, n] = sum_k x[b, k] * deq(W)[n, k] for a few
// activation rows b (decode), W stored as N rows of K/256 packed blocks.
//
// Design (B200):
//  * A pre-kernel quantises the activations once per call into two int8
//    levels per 32-wide group (x ~= s * (hi + lo/256), s = max|x|/127) and
//    the fp32 sums of each 16-wide half; the matvec kernel reads them from
//    L1/L2.
//  * Work = 16-row weight tiles x 256-weight blocks.  The units are split
//    evenly over every resident warp (warp-level stream-K): no wave
//    quantisation and no tail imbalance whatever N and K are.  A warp whose
//    range covers a whole tile writes y directly; tiles shared by several
//    warps are combined by the last warp to finish (atomic ticket, no
//    spinning), summing the partials in warp order so results are
//    deterministic.
//  * Packed bytes stream HBM -> shared memory with 1-D bulk async copies (one
//    per weight row and chunk, issued by 16 lanes in parallel) into a 2-stage
//    per-warp ring completed on mbarriers; waits are time-bounded.
//  * Each weight is decoded to an int8 value a_k (gsq_fast.cuh) and
//    multiplied with the int8 activations on the tensor cores
//    (mma.sync.m16n8k32.s8).  The 8 MMA columns carry (sub-block, activation
//    row, level) triples so each quad lane ends up holding the integer dot
//    products of a different sub-block, which it scales once:
//    acc += S_u * s_x * (256*C_hi + C_lo) + B_u * sum(x_u).
//  * Programmatic dependent launch: the weight prefetch and table load run
//    before griddepcontrol.wait, overlapping the previous kernel.
#include <algorithm>

#include "gsq_fast.cuh"
#include "gsq_host.h"

namespace gsq {

constexpr int QMV_WARPS = 4;
constexpr int QMV_STAGES = 2;
constexpr int QMV_THREADS = 32 * QMV_WARPS;
// Scratch layout: a fixed region of ticket counters first, then the
// quantised activations and the partial sums.  Every completed call returns
// the tickets it used to zero and nothing else is ever written over the
// ticket region, so one zero-filled workspace serves calls of any shape.
constexpr int QMV_TICKET_SLOTS = 65536;
constexpr size_t QMV_TICKET_BYTES = QMV_TICKET_SLOTS * sizeof(unsigned);

struct QmvArgs {
  const uint8_t* packed;
  int64_t N, K, row_bytes, packed_bytes;
  const int8_t* xq;    // [rows_pad][2][K]
  const float* xs;     // [rows_pad][K/32]   (s/256)
  const float* xsum;   // [rows_pad][K/16]
  int rows, rows_pad;
  void* y;
  int y_dtype;
  int kblocks;
  int64_t tiles, units;
  int aligned;
  float* partial;      // [btiles][warps][2][NB][16]
  unsigned* tickets;   // [btiles][tiles]
  int* err;
};

template <int T>
struct QmvGeom {
  static constexpr int BB = block_bytes(T);
  static constexpr int CB = BB <= 66 ? 8 : BB <= 98 ? 4 : 2;       // blocks per chunk (~400-600 B a row)
  static constexpr int ROWB = ((CB * BB + 30) + 15) / 16 * 16;     // staged row stride
  static constexpr int STAGE = 16 * ROWB;
  static constexpr int TAB = (Fast<T>::TAB_BYTES + 127) / 128 * 128;
  static constexpr size_t SMEM = TAB + 128 /*mbarriers*/ + 128 /*align*/ + (size_t)QMV_WARPS * QMV_STAGES * STAGE;
};

// ---------------------------------------------------------------------------
// Activation quantisation pre-kernel.

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

// One thread per (row, 32-wide group): hi/lo int8 levels, s/256, half sums.
// Rows in [rows, rows_pad) are written as zeros.
template <typename XT>
__global__ void __launch_bounds__(256) qmv_xquant_kernel(const void* x, int rows, int rows_pad, int64_t K,
                                                         int8_t* xq, float* xs, float* xsum) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t ng = K / 32;
  for (int64_t task = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; task < rows_pad * ng;
       task += (int64_t)gridDim.x * blockDim.x) {
    const int64_t row = task / ng, gi = task - row * ng;
    int8_t* qh = xq + (row * 2) * K + gi * 32;
    int8_t* ql = qh + K;
    if (row >= rows) {
      const uint4 z = make_uint4(0, 0, 0, 0);
      reinterpret_cast<uint4*>(qh)[0] = z; reinterpret_cast<uint4*>(qh)[1] = z;
      reinterpret_cast<uint4*>(ql)[0] = z; reinterpret_cast<uint4*>(ql)[1] = z;
      xs[row * ng + gi] = 0.f;
      xsum[row * 2 * ng + 2 * gi] = 0.f;
      xsum[row * 2 * ng + 2 * gi + 1] = 0.f;
      continue;
    }
    float v[32];
    load32<XT>(x, row * K + gi * 32, v);
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
    xs[row * ng + gi] = amax / (127.f * 256.f);
    xsum[row * 2 * ng + 2 * gi] = s0;
    xsum[row * 2 * ng + 2 * gi + 1] = s1;
  }
}

// ---------------------------------------------------------------------------
// The matvec kernel.

// Warp range [u0, u1) of the unit space for global warp gw of GW.
__device__ __forceinline__ void warp_range(const QmvArgs& a, int64_t gw, int64_t GW, int64_t& u0, int64_t& u1) {
  if (a.aligned) {
    u0 = (gw * a.tiles / GW) * a.kblocks;
    u1 = ((gw + 1) * a.tiles / GW) * a.kblocks;
  } else {
    u0 = gw * a.units / GW;
    u1 = (gw + 1) * a.units / GW;
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
  uint8_t* tab = smem;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + G::TAB);
  uint8_t* stages = smem + G::TAB + 128;
  stages += (0u - smem_u32(stages)) & 127u;  // align in the shared window, keeping shared provenance

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, tq = lane & 3;
  const int btile = blockIdx.y;
  const int64_t GW = (int64_t)gridDim.x * QMV_WARPS;
  const int64_t gw = (int64_t)blockIdx.x * QMV_WARPS + warp;
  const int kb = a.kblocks;
  int64_t u0, u1;
  warp_range(a, gw, GW, u0, u1);

  uint64_t* wbars = bars + warp * QMV_STAGES;
  uint8_t* wstage = stages + (size_t)warp * QMV_STAGES * G::STAGE;
  const uintptr_t pbase = reinterpret_cast<uintptr_t>(a.packed);
  const uint64_t policy = l2_policy_evict_first();

  if (lane == 0)
    for (int s = 0; s < QMV_STAGES; s++) mbar_init(&wbars[s], 1);
  fence_mbar_init();
  __syncwarp();

  // Producer: stage the next chunk (16 rows of one tile, up to CB blocks,
  // never crossing the tile's end or the warp's range end).
  // Iterators walk (tile, block) incrementally: no divisions in the loop.
  int64_t pu = u0, ptile = u0 / kb;
  int pkb = (int)(u0 - ptile * kb);
  int issued = 0;
  auto issue_next = [&]() {
    const int s = issued % QMV_STAGES;
    const int64_t tile = ptile;
    const int kb0 = pkb;
    const int nb = (int)(u1 - pu < (int64_t)min(G::CB, kb - kb0) ? u1 - pu : (int64_t)min(G::CB, kb - kb0));
    uint32_t bytes = 0;
    if (lane < 16) {
      const int64_t r = tile * 16 + lane;
      if (r < a.N) {
        const int64_t off = r * a.row_bytes + (int64_t)kb0 * G::BB;
        const int64_t end = off + (int64_t)nb * G::BB;
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
    pu += nb;
    pkb += nb;
    if (pkb == kb) { pkb = 0; ptile++; }
    issued++;
  };
  while (issued < QMV_STAGES && pu < u1) issue_next();

  F::load_tables(tab, threadIdx.x, blockDim.x);
  __syncthreads();
  // Everything above reads only weights and tables; from here on the kernel
  // reads activations / scratch that an earlier kernel in the stream writes.
  pdl_wait();

  // Activation-operand identity of this lane (column g of the MMA) and its
  // epilogue identity (sub-block s_ep of each set, activation row b_ep).
  const int pcol = g >> 1, level = g & 1;
  const int s_col = pcol / NB, b_col = pcol % NB;
  const int s_ep = tq / NB, b_ep = tq % NB;
  const int64_t K = a.K;
  const int8_t* xrow = a.xq + ((int64_t)(btile * NB + b_col) * 2 + level) * K;
  const float* xs_row = a.xs + (int64_t)(btile * NB + b_ep) * (K / 32);
  const float* xsum_row = a.xsum + (int64_t)(btile * NB + b_ep) * (K / 16);
  const int batch = btile * NB + b_ep;
  const bool writer = tq < NB && batch < a.rows;

  float acc0 = 0.f, acc1 = 0.f;
  bool ok = true;
  int consumed = 0;
  int64_t cu = u0, seg = u0, ctile = u0 / kb;
  int ckb = (int)(u0 - ctile * kb);
  const int64_t first_tile = ctile;
  while (cu < u1) {
    const int s = consumed % QMV_STAGES;
    ok = mbar_wait_bounded(&wbars[s], (uint32_t)((consumed / QMV_STAGES) & 1), a.err);
    if (!ok) break;
    const int64_t tile = ctile;
    const int kb0 = ckb;
    const int nb = (int)(u1 - cu < (int64_t)min(G::CB, kb - kb0) ? u1 - cu : (int64_t)min(G::CB, kb - kb0));
    const int64_t row0 = tile * 16 + g;
    const uint8_t* st = wstage + (size_t)s * G::STAGE;
    const uint8_t* r0p = st + g * G::ROWB + (int)((row0 * a.row_bytes + (int64_t)kb0 * G::BB) & 15);
    const uint8_t* r1p = st + (g + 8) * G::ROWB + (int)(((row0 + 8) * a.row_bytes + (int64_t)kb0 * G::BB) & 15);
    for (int bi = 0; bi < nb; bi++) {
      const uint8_t* b0 = r0p + bi * G::BB;
      const uint8_t* b1 = r1p + bi * G::BB;
      const int kblk = (kb0 + bi) * QK;
      // Per-block activation bases: the set loop below then uses immediate offsets.
      const int8_t* xb = xrow + kblk;
      const float* xsb = xs_row + (kblk >> 5);
      const float* xub = xsum_row + (kblk >> 4);
#pragma unroll
      for (int set = 0; set < SETS; set++) {
        const int kset = set * KSET;
        // Activation words for the one MMA of this set where column g is live.
        uint32_t xw0, xw1;
        int jsel;
        if constexpr (UNIT == 32) {
          jsel = s_col;
          if constexpr (F::BLOCKED) {
            const uint2 w = __ldg(reinterpret_cast<const uint2*>(xb + kset + 32 * s_col + 8 * tq));
            xw0 = w.x; xw1 = w.y;
          } else {
            xw0 = __ldg(reinterpret_cast<const uint32_t*>(xb + kset + 32 * s_col + 4 * tq));
            xw1 = __ldg(reinterpret_cast<const uint32_t*>(xb + kset + 32 * s_col + 16 + 4 * tq));
          }
        } else {
          jsel = s_col >> 1;
          const bool live = (s_col & 1) == (tq >> 1);
          const uint2 w = __ldg(reinterpret_cast<const uint2*>(xb + kset + 32 * jsel + 8 * tq));
          xw0 = live ? w.x : 0u;
          xw1 = live ? w.y : 0u;
        }
        // Two independent accumulator chains (even / odd MMAs) halve the
        // dependent tensor-core latency per set.  Sign-carrying formats run a
        // second pair of chains on the negative-position magnitudes.
        int C[4] = {0, 0, 0, 0}, Cb[4] = {0, 0, 0, 0};
        int Nn[4] = {0, 0, 0, 0}, Nb[4] = {0, 0, 0, 0};
#pragma unroll
        for (int j = 0; j < MMAS; j++) {
          const int c32 = set * MMAS + j;
          const bool on = (j == jsel);
          const uint32_t bx0 = on ? xw0 : 0u, bx1 = on ? xw1 : 0u;
          if constexpr (F::SPLIT) {
            uint32_t a0, a1, a2, a3, m0, m1, m2, m3;
            F::entry_split(b0, c32, tq, tab, a0, a2, m0, m2);
            F::entry_split(b1, c32, tq, tab, a1, a3, m1, m3);
            if (j & 1) {
              mma_s8(Cb, a0, a1, a2, a3, bx0, bx1);
              mma_s8(Nb, a0 & m0, a1 & m1, a2 & m2, a3 & m3, bx0, bx1);
            } else {
              mma_s8(C, a0, a1, a2, a3, bx0, bx1);
              mma_s8(Nn, a0 & m0, a1 & m1, a2 & m2, a3 & m3, bx0, bx1);
            }
          } else {
            uint32_t a0, a1, a2, a3;
            F::entry(b0, c32, tq, tab, a0, a2);
            F::entry(b1, c32, tq, tab, a1, a3);
            if (j & 1) mma_s8(Cb, a0, a1, a2, a3, bx0, bx1);
            else mma_s8(C, a0, a1, a2, a3, bx0, bx1);
          }
        }
        if constexpr (MMAS > 1) {
#pragma unroll
          for (int i = 0; i < 4; i++) C[i] += Cb[i];
        }
        if constexpr (F::SPLIT) {
#pragma unroll
          for (int i = 0; i < 4; i++) C[i] -= 2 * (Nn[i] + Nb[i]);
        }
        const int unit = set * UPS + s_ep;
        const int ku = unit * UNIT;  // within the block
        const float xsv = __ldg(xsb + (ku >> 5));
        float S0, B0, S1, B1;
        F::affine(b0, unit, S0, B0);
        F::affine(b1, unit, S1, B1);
        acc0 = fmaf(S0, (float)(C[0] * 256 + C[1]) * xsv, acc0);
        acc1 = fmaf(S1, (float)(C[2] * 256 + C[3]) * xsv, acc1);
        if constexpr (F::HAS_BIAS) {
          float xu = __ldg(xub + (ku >> 4));
          if constexpr (UNIT == 32) xu += __ldg(xub + (ku >> 4) + 1);
          acc0 = fmaf(B0, xu, acc0);
          acc1 = fmaf(B1, xu, acc1);
        }
      }
    }
    __syncwarp();
    consumed++;
    if (pu < u1) issue_next();  // refill the stage just released
    cu += nb;
    ckb += nb;
    if (ckb == kb) { ckb = 0; ctile++; }

    if (kb0 + nb == kb || cu == u1) {
      // ---- end of this warp's segment of `tile`: reduce the quad lanes that
      // hold the same activation row, then write or combine.
      if constexpr (NB == 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      }
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
      const int64_t rg0 = tile * 16 + g, rg1 = rg0 + 8;
      const int seg_len = (int)(cu - seg);
      if (seg_len == kb) {
        if (writer) {
          if (rg0 < a.N) store_out(a.y, a.y_dtype, (int64_t)batch * a.N + rg0, acc0);
          if (rg1 < a.N) store_out(a.y, a.y_dtype, (int64_t)batch * a.N + rg1, acc1);
        }
      } else {
        const int slot = (tile == first_tile) ? 0 : 1;
        float* pp = a.partial + (((int64_t)btile * GW + gw) * 2 + slot) * NB * 16 + b_ep * 16;
        if (writer) {
          pp[g] = acc0;
          pp[g + 8] = acc1;
        }
        __threadfence();
        __syncwarp();
        unsigned last = 0;
        if (lane == 0) {
          const unsigned prev = atomicAdd(&a.tickets[(int64_t)btile * a.tiles + tile], (unsigned)seg_len);
          last = (prev + (unsigned)seg_len == (unsigned)kb);
        }
        last = __shfl_sync(0xffffffffu, last, 0);
        if (last) {
          __threadfence();
          // Sum the segments of every warp that covered this tile, in warp order.
          const int64_t ut0 = tile * kb, ut1 = ut0 + kb;
          const int64_t g0 = ((ut0 + 1) * GW - 1) / a.units;
          const int64_t g1 = (ut1 * GW - 1) / a.units;
          if (lane < NB * 16) {
            const int b = lane >> 4, r = lane & 15;
            float sum = 0.f;
            for (int64_t gg = g0; gg <= g1; gg++) {
              const int64_t s0 = gg * a.units / GW, s1 = (gg + 1) * a.units / GW;
              if (s0 == s1 || s1 <= ut0 || s0 >= ut1) continue;  // empty or not covering this tile
              const int sl = (s0 / kb == tile) ? 0 : 1;
              sum += __ldcg(a.partial + (((int64_t)btile * GW + gg) * 2 + sl) * NB * 16 + b * 16 + r);
            }
            const int bt = btile * NB + b;
            const int64_t rr = tile * 16 + r;
            if (bt < a.rows && rr < a.N) store_out(a.y, a.y_dtype, (int64_t)bt * a.N + rr, sum);
          }
          if (lane == 0) a.tickets[(int64_t)btile * a.tiles + tile] = 0u;
        }
      }
      acc0 = acc1 = 0.f;
      seg = cu;
    }
  }
  pdl_launch_dependents();
  if (!ok) {
    // Drain the copies this warp still has in flight before the CTA exits.
    for (int c = consumed; c < issued; c++)
      mbar_wait_bounded(&wbars[c % QMV_STAGES], (uint32_t)((c / QMV_STAGES) & 1), nullptr);
  }
}

// --------------------------------------------------------------------------
// Host side.

// Resident CTAs per SM for an instantiation (the occupancy API when a device
// is present, else a shared-memory estimate).
template <int T, int NB>
static int qmv_occupancy() {
  static int cached = 0;
  if (cached > 0) return cached;
  int occ = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qmv_kernel<T, NB>, QMV_THREADS, QmvGeom<T>::SMEM) !=
          cudaSuccess ||
      occ <= 0) {
    cudaGetLastError();
    occ = (int)std::max<size_t>(1, std::min<size_t>(4, (227u * 1024u) / (QmvGeom<T>::SMEM + 1024)));
  }
  cached = occ;
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

#define GSQ_QMV_GEOM_CASE(TT)                                                           \
  case TT:                                                                              \
    smem = QmvGeom<TT>::SMEM;                                                           \
    occ = nb == 1 ? qmv_occupancy<TT, 1>() : qmv_occupancy<TT, 2>();                    \
    break;

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

QmvPlan qmv_plan(int t, int64_t N, int64_t K, int rows) {
  QmvPlan p = {};
  const int kblocks = (int)(K / QK);
  p.nb = rows == 1 ? 1 : 2;
  p.btiles = (rows + p.nb - 1) / p.nb;
  p.tiles = (N + 15) / 16;
  p.units = p.tiles * kblocks;
  size_t smem = 0;
  int occ = 1;
  const int nb = p.nb;
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_GEOM_CASE) default: break; }
  p.smem = smem;
  const int64_t slots = (int64_t)occ * qmv_sm_count() / std::max(1, p.btiles);
  const int64_t want_warps = std::min<int64_t>(std::max<int64_t>(1, slots) * QMV_WARPS, p.units);
  p.ctas = (int)std::max<int64_t>(1, (want_warps + QMV_WARPS - 1) / QMV_WARPS);
  p.aligned = (p.tiles * p.btiles > QMV_TICKET_SLOTS) ? 1 : 0;
  const int64_t GW = (int64_t)p.ctas * QMV_WARPS;
  const size_t rows_pad = (size_t)p.btiles * p.nb;
  p.off_xq = QMV_TICKET_BYTES;
  p.off_xs = p.off_xq + align256(rows_pad * 2 * (size_t)K);
  p.off_xsum = p.off_xs + align256(rows_pad * (size_t)(K / 32) * 4);
  p.off_partial = p.off_xsum + align256(rows_pad * (size_t)(K / 16) * 4);
  p.workspace = p.off_partial + align256((size_t)p.btiles * GW * 2 * p.nb * 16 * 4);
  return p;
}

template <int T, int NB>
static cudaError_t qmv_launch_t(const QmvArgs& a, const QmvPlan& p, cudaStream_t st) {
  auto kern = qmv_kernel<T, NB>;
  static int configured[64] = {0};  // dynamic smem attribute already set, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  return launch_pdl(kern, dim3(p.ctas, p.btiles), dim3(QMV_THREADS), p.smem, st, a);
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
  uint8_t* w = static_cast<uint8_t*>(ws);
  QmvArgs a;
  a.packed = packed;
  a.N = N;
  a.K = K;
  a.row_bytes = (K / QK) * block_bytes(t);
  a.packed_bytes = N * a.row_bytes;
  a.rows = rows;
  a.rows_pad = p.btiles * p.nb;
  a.y = y;
  a.y_dtype = y_dtype;
  a.kblocks = (int)(K / QK);
  a.tiles = p.tiles;
  a.units = p.units;
  a.aligned = p.aligned;
  a.tickets = reinterpret_cast<unsigned*>(w);
  a.xq = reinterpret_cast<const int8_t*>(w + p.off_xq);
  a.xs = reinterpret_cast<const float*>(w + p.off_xs);
  a.xsum = reinterpret_cast<const float*>(w + p.off_xsum);
  a.partial = reinterpret_cast<float*>(w + p.off_partial);
  a.err = err;

  // 1) quantise the activations into the scratch
  const int64_t tasks = (int64_t)a.rows_pad * (K / 32);
  const int grid = (int)std::min<int64_t>((tasks + 255) / 256, 148 * 8);
  int8_t* xq = reinterpret_cast<int8_t*>(w + p.off_xq);
  float* xs = reinterpret_cast<float*>(w + p.off_xs);
  float* xsum = reinterpret_cast<float*>(w + p.off_xsum);
  cudaError_t e;
  if (x_dtype == DT_F16)
    e = launch_pdl(qmv_xquant_kernel<__half>, dim3(grid), dim3(256), 0, st, x, rows, a.rows_pad, K, xq, xs, xsum);
  else if (x_dtype == DT_BF16)
    e = launch_pdl(qmv_xquant_kernel<__nv_bfloat16>, dim3(grid), dim3(256), 0, st, x, rows, a.rows_pad, K, xq, xs,
                   xsum);
  else
    e = launch_pdl(qmv_xquant_kernel<float>, dim3(grid), dim3(256), 0, st, x, rows, a.rows_pad, K, xq, xs, xsum);
  if (e != cudaSuccess) return e;
  // 2) the matvec
  return qmv_launch(t, a, p, st);
}

}  // namespace gsq
