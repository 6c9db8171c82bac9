// Fused dequantize + matvec (QMV) over packed GGUF super-blocks, sm_100a.
//
// Replaces the reference's per-type Metal matvec kernels
// (mlx_gsq/runtime/kernels/qmv.py:76-528, dispatched by quantized_matvec,
// qmv.py:537-576).  y[b, n] = sum_k x[b, k] * deq(W)[n, k] for a few
// activation rows b (decode), W stored as N rows of K/256 packed blocks.
//
// Design (B200):
//  * One kernel per call.  Work = 16-row weight tiles x 256-weight blocks.
//    K is cut into `slices` (grid.y) only when the activations of a whole
//    row would not fit the per-CTA budget; inside a slice the (tile, block)
//    units are split evenly over the persistent CTAs (grid.x), so there is
//    no wave quantisation whatever N and K are.
//  * Each CTA = 8 consumer warps + 1 producer warp.  The producer streams
//    the packed bytes HBM -> shared memory with 1-D bulk async copies (one
//    per weight row per stage, ~1 KB each) into an NS-deep ring completed on
//    mbarriers; consumers release stages on a second set of mbarriers.  All
//    waits are time-bounded.
//  * The consumer warps split every stage's blocks among themselves and
//    combine their per-tile row sums through shared memory in warp order.
//    Tiles split between CTAs (at most the first and last tile of a CTA's
//    range) are combined by the last CTA to finish (atomic ticket, no
//    spinning), summing the pieces in slice and CTA order: results are
//    deterministic.
//  * Before the main loop each CTA quantises its slice of the activations
//    into shared memory: two int8 levels per 32-wide group
//    (x ~= s * (hi + lo/256), s = max|x|/127) and fp32 sums of each 16-wide
//    half.  Each weight is decoded to an int8 value a_k (gsq_fast.cuh) and
//    multiplied with them on the tensor cores (mma.sync.m16n8k32.s8).  The 8
//    MMA columns carry (sub-block, activation row, level) triples so each
//    quad lane ends up holding the integer dot products of a different
//    sub-block, which it scales once:
//    acc += S_u * s_x * (256*C_hi + C_lo) + B_u * sum(x_u).
//  * Programmatic dependent launch: the weight stream and the table load
//    start before griddepcontrol.wait, overlapping the previous kernel; the
//    activations are read after it.
#include <algorithm>
#include <type_traits>

#include "gsq_mv.cuh"
#include "gsq_host.h"

namespace gsq {

constexpr int QMV_CWARPS = 8;                          // consumer (tensor-core) warps per CTA
constexpr int QMV_CTHREADS = 32 * QMV_CWARPS;
constexpr int QMV_PRODUCER = QMV_CWARPS;               // warp streaming packed bytes into the ring
constexpr int QMV_COMBINER = QMV_CWARPS + 1;           // warp combining tiles split between CTAs
constexpr int QMV_THREADS = QMV_CTHREADS + 64;
constexpr int QMV_NS_MAX = 4;                          // ring stages at most
constexpr int QMV_MIN_UNITS = 8;                       // (tile, block) units per CTA at least
constexpr int QMV_CTA_SMEM = 112 * 1024;               // two CTAs per SM
constexpr int QMV_XBYTES_PER_BLOCK = 2 * QK + 8 * 4 + 16 * 4;  // per activation row: levels, scales, half sums
constexpr int QMV_RED_BUFS = QMV_NS_MAX + 1;          // per-warp row-sum buffers (ring depth + 1)
constexpr int QMV_RED_BYTES = QMV_RED_BUFS * QMV_CWARPS * 32 * 4;
// Scratch layout: a fixed region that every completed call leaves zero-filled
// (ticket counters, or the published-piece slots of single-slice plans), then
// the partial sums of multi-slice plans.  Nothing else is ever written over
// the fixed region, so one zero-filled workspace serves calls of any shape.
constexpr int QMV_TICKET_SLOTS = 65536;
// Gather regions (fused row gather): 64 words of which the last two are the
// owner's CTA ticket and call count, then fp32 y [rows][ntot], then an
// inbox of two [rows][ntot] arrays of {value, call count} 8-byte pairs that
// the peers write (slot = call count & 1).
constexpr int QMV_GATHER_MAX = 8;
constexpr int QMV_GFLAG_TICKET = 62, QMV_GFLAG_COUNT = 63;
constexpr size_t QMV_GATHER_HEADER = 64 * sizeof(unsigned);
constexpr size_t QMV_TICKET_BYTES = QMV_TICKET_SLOTS * sizeof(unsigned);

// Non-negative division and remainder with a 32-bit path: the work-split
// arithmetic fits 32 bits for every plannable shape, and a 64-bit division
// is a long software sequence.
__device__ __forceinline__ int64_t udiv(int64_t a, int64_t b) {
  return ((uint64_t)a | (uint64_t)b) >> 32 ? a / b : (int64_t)((uint32_t)a / (uint32_t)b);
}
__device__ __forceinline__ int64_t umod(int64_t a, int64_t b) { return a - udiv(a, b) * b; }

struct QmvArgs {
  const uint8_t* packed;
  const void* x;
  void* y;
  float* part_full;    // [btiles][slices][tiles][NB*16]   whole-slice pieces of a tile
  float* part_piece;   // [btiles][slices][ctas][2][NB*16] first / last piece of a CTA's range
  unsigned* tickets;   // [btiles][tiles]
  uint32_t* slots;     // [btiles][ctas][NB*16] published pieces, one slice (encoded, 0 = empty)
  int* err;
  int64_t N, K, row_bytes, packed_bytes, tiles;
  int rows, x_dtype, y_dtype, kb, bps, slices, aligned, ns;
  int cb, rowb, stage;  // ring geometry: blocks per stage, staged row stride, stage bytes
  int pre;              // stages issued before the activations are quantised (<= ns)
  int xbulk;            // one 16-bit activation row, copied into shared memory in bulk
  int glu;              // SwiGLU epilogue (gsq_qmv_swiglu): y = silu(gate) * up, N/2 columns
  // Fused row gather (world > 1): output rows [row0, row0 + N) of ntot are
  // stored into every rank's gather region (fp32, [rows][ntot]) over
  // NVLink, and the regions' flag words synchronise the ranks at the end.
  float* gy[QMV_GATHER_MAX];
  unsigned* gflags[QMV_GATHER_MAX];
  uint2* ginbox[QMV_GATHER_MAX];
  int world, rank;
  int64_t row0, ntot;
};

// 8-byte {value, call count} pairs: one single-copy-atomic access each.
__device__ __forceinline__ void st_pair_sys(uint2* p, float v, unsigned ep) {
  const unsigned long long w = ((unsigned long long)ep << 32) | __float_as_uint(v);
  asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(w) : "memory");
}
__device__ __forceinline__ unsigned long long ld_pair_sys(const uint2* p) {
  unsigned long long w;
  asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(w) : "l"(p) : "memory");
  return w;
}

// Store one output value: y, or (gathering) this rank's own region and, as
// a {value, call count} pair, every peer's inbox slot for call count ep.
template <bool GATHER>
__device__ __forceinline__ void store_y(const QmvArgs& a, int batch, int64_t rr, float v, unsigned ep) {
  if constexpr (!GATHER) {
    store_out(a.y, a.y_dtype, (int64_t)batch * a.N + rr, v);
    return;
  }
  const int64_t off = (int64_t)batch * a.ntot + a.row0 + rr;
  a.gy[a.rank][off] = v;
  const int64_t slot = (int64_t)(ep & 1u) * a.rows * a.ntot;
#pragma unroll
  for (int p = 0; p < QMV_GATHER_MAX; p++)
    if (p < a.world && p != a.rank) st_pair_sys(a.ginbox[p] + slot + off, v, ep);
}

// Final value v of packed row 16*tile + r for activation row `batch`, by the
// lanes in `mask` (the tile's 16 rows per activation row, lane = b*16 + r);
// `ok`: this lane's row exists.  With the SwiGLU epilogue the packed rows of a
// tile are 8 gate rows then the same 8 up rows (gsq_qmv_swiglu): lane r < 8
// takes its up value from lane r + 8 and stores silu(gate) * up as output
// column 8*tile + r.
template <bool GATHER>
__device__ __forceinline__ void final_store(const QmvArgs& a, unsigned mask, int batch, int64_t tile, int r, float v,
                                            bool ok, unsigned ep) {
  if constexpr (!GATHER) {
    if (a.glu) {
      const float up = __shfl_xor_sync(mask, v, 8);
      if (ok && r < 8)
        store_out(a.y, a.y_dtype, (int64_t)batch * (a.N >> 1) + tile * 8 + r, v / (1.f + __expf(-v)) * up);
      return;
    }
  }
  if (ok) store_y<GATHER>(a, batch, tile * 16 + r, v, ep);
}

// Call count of this call on the gather region (read after griddepcontrol.wait:
// the previous call on the region may be the kernel just before).
template <bool GATHER>
__device__ __forceinline__ unsigned gather_count(const QmvArgs& a) {
  if constexpr (GATHER) return a.gflags[a.rank][QMV_GFLAG_COUNT] + 1u;
  return 0u;
}

// End of a gathering call, run by the consumer and combiner threads of every
// CTA after their last store.  Every output value already went to the
// peers' inboxes as a {value, call count} pair when it was stored (8-byte
// stores over NVLink, no fences: each pair carries its own readiness).
// Here the CTA takes its share of the other ranks' values of this call from
// its own inbox into y -- about one value per thread, spread over all CTAs --
// waiting (bounded) until each pair's call count is this call's.  The kernel
// completes only when every share is in, i.e. every rank's rows of this call
// are in every rank's y.  The last CTA to finish (gpu-scope ticket) records
// the call count.  The inbox slot alternates with the call count; a rank
// cannot finish a call before every peer has computed its rows of that call,
// and it sends the next call's rows only after this call's kernel completed,
// so a peer is never two calls ahead in one slot.  Every rank must make the
// same sequence of calls on a region.
__device__ void gather_finish(const QmvArgs& a, unsigned ep) {
  constexpr int NT = QMV_CTHREADS + 32;  // consumer and combiner threads
  const int t = threadIdx.x < QMV_CTHREADS ? threadIdx.x : threadIdx.x - 32;  // skip the producer warp
  const int64_t cta = (int64_t)blockIdx.x + (int64_t)gridDim.x * ((int64_t)blockIdx.y + (int64_t)gridDim.y * blockIdx.z);
  const int64_t nthreads = (int64_t)gridDim.x * gridDim.y * gridDim.z * NT;
  const int64_t total = (int64_t)a.rows * a.ntot;
  const uint2* in = a.ginbox[a.rank] + (int64_t)(ep & 1u) * total;
  float* y = a.gy[a.rank];
  const long long t0 = clock64();
  bool late = false;  // a timed-out thread still reaches the barrier below
  for (int64_t i = cta * NT + t; i < total && !late; i += nthreads) {
    const int64_t col = umod(i, a.ntot);
    if (col >= a.row0 && col < a.row0 + a.N) continue;  // this rank's own rows
    unsigned long long w = ld_pair_sys(in + i);
    while ((unsigned)(w >> 32) != ep) {
      if (clock64() - t0 > (1ll << 31)) {
        if (a.err) atomicExch(a.err, DEV_WAIT_TIMEOUT);
        late = true;
        break;
      }
      __nanosleep(32);
      w = ld_pair_sys(in + i);
    }
    if (!late) y[i] = __uint_as_float((unsigned)w);
  }
  asm volatile("bar.sync 2, %0;" ::"n"(NT) : "memory");
  if (threadIdx.x == 0) {
    unsigned* own = a.gflags[a.rank];
    __threadfence();
    const unsigned ctas = gridDim.x * gridDim.y * gridDim.z;
    if (atomicAdd(own + QMV_GFLAG_TICKET, 1u) == ctas - 1u) {
      own[QMV_GFLAG_TICKET] = 0u;
      own[QMV_GFLAG_COUNT] = ep;
    }
  }
}

// Staged row stride for cb blocks: the copied bytes plus head/tail 16-byte
// rounding, padded to an odd number of 16-byte units so that the 8 rows a
// warp reads at once (rows g = 0..7) start in 8 different 16-byte bank groups.
__host__ __device__ constexpr int qmv_rowb(int cb, int bb) {
  return (((cb * bb + 30) + 15) / 16) % 2 ? ((cb * bb + 30) + 15) / 16 * 16 : ((cb * bb + 30) + 15) / 16 * 16 + 16;
}

template <int T>
struct QmvGeom {
  static constexpr int BB = block_bytes(T);
  static constexpr int TAB = (Mv<T>::TAB_BYTES + 127) / 128 * 128;
  static constexpr int FIXED = 128 /*align*/ + TAB + 256 /*mbarriers*/ + QK /*zeros*/ + QMV_RED_BYTES;
  // Stages of 8 blocks: two of them plus the activations of one block always
  // fit; the plan may choose wider stages (16 or 32 blocks) per call.
  static_assert(FIXED + 2 * 16 * qmv_rowb(8, BB) + 2 * QMV_XBYTES_PER_BLOCK <= QMV_CTA_SMEM,
                "ring must hold two stages");
};

// Calls f(std::integral_constant<int, i>) for i = I..N-1 (compile-time loop).
template <int I, int N, typename Fn>
__device__ __forceinline__ void static_for(Fn&& f) {
  if constexpr (I < N) {
    f(std::integral_constant<int, I>{});
    static_for<I + 1, N>(f);
  }
}

__device__ __forceinline__ void named_sync_consumers() {
  asm volatile("bar.sync 1, %0;" ::"n"(QMV_CTHREADS) : "memory");
}

// ---------------------------------------------------------------------------
// Activation quantisation (CTA prologue).

// 8 consecutive activations, as raw 16-byte words (two for fp32).
template <typename XT>
__device__ __forceinline__ void load8(const void* x, int64_t i, uint4 (&r)[2]) {
  const uint4* p = reinterpret_cast<const uint4*>(reinterpret_cast<const XT*>(x) + i);
  r[0] = __ldcg(p);
  r[1] = sizeof(XT) == 4 ? __ldcg(p + 1) : make_uint4(0, 0, 0, 0);
}

template <typename XT> __device__ __forceinline__ void unpack8(const uint4 (&r)[2], float (&v)[8]);
template <> __device__ __forceinline__ void unpack8<float>(const uint4 (&r)[2], float (&v)[8]) {
  v[0] = __uint_as_float(r[0].x); v[1] = __uint_as_float(r[0].y);
  v[2] = __uint_as_float(r[0].z); v[3] = __uint_as_float(r[0].w);
  v[4] = __uint_as_float(r[1].x); v[5] = __uint_as_float(r[1].y);
  v[6] = __uint_as_float(r[1].z); v[7] = __uint_as_float(r[1].w);
}
template <> __device__ __forceinline__ void unpack8<__half>(const uint4 (&r)[2], float (&v)[8]) {
  const uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[t]));
    v[2 * t] = f.x; v[2 * t + 1] = f.y;
  }
}
template <> __device__ __forceinline__ void unpack8<__nv_bfloat16>(const uint4 (&r)[2], float (&v)[8]) {
  const uint32_t w[4] = {r[0].x, r[0].y, r[0].z, r[0].w};
#pragma unroll
  for (int t = 0; t < 4; t++) {
    v[2 * t] = __uint_as_float(w[t] << 16);
    v[2 * t + 1] = __uint_as_float(w[t] & 0xFFFF0000u);
  }
}

// Slice layout in shared memory (KS = bps*256 activations per row):
//   xq   [NB][2][KS] int8   levels hi, lo:  x ~= s * (hi + lo/256)
//   xs   [NB][KS/32] fp32   s/256 per 32-group (s = max|x|/127)
//   xsum [NB][KS/16] fp32   sum of each 16-wide half
// Every consumer thread issues the loads of up to CH chunks of 8 values
// first (one round trip per CH * 256 chunks, a K = 20480 row at fp16), then
// quantises them; the four lanes holding a 32-group combine max and sums with
// shuffles.
// Levels of one 32-group (words 0..7 = elements 4q..4q+3) into the nibble
// order of MvDecode<T>::NIBBLE_ORDER formats: word tq = elements
// 4tq, 16+4tq, 4tq+1, 17+4tq; word 4+tq = 4tq+2, 18+4tq, 4tq+3, 19+4tq.
__device__ __forceinline__ void nibble_order(uint32_t (&hw)[8], uint32_t (&lw)[8]) {
#pragma unroll
  for (int tq = 0; tq < 4; tq++) {
    const uint32_t h0 = hw[tq], h1 = hw[4 + tq], l0 = lw[tq], l1 = lw[4 + tq];
    hw[tq] = __byte_perm(h0, h1, 0x5140u);
    hw[4 + tq] = __byte_perm(h0, h1, 0x7362u);
    lw[tq] = __byte_perm(l0, l1, 0x5140u);
    lw[4 + tq] = __byte_perm(l0, l1, 0x7362u);
  }
}

template <int T, int NB, bool SUMS, typename XT, int CH>
__device__ __forceinline__ void quantise_round(const QmvArgs& a, int btile, int kb0, int KS, int per_row, int total,
                                               int base, int8_t* xq, float* xs, float* xsum) {
  uint4 raw[CH][2];
#pragma unroll
  for (int i = 0; i < CH; i++) {
    const int c = base + threadIdx.x + i * QMV_CTHREADS;
    const int b = c >= per_row ? 1 : 0;  // NB <= 2
    const int row = btile * NB + b;
    if (c < total && row < a.rows) {
      load8<XT>(a.x, (int64_t)row * a.K + (int64_t)kb0 * QK + (c - b * per_row) * 8, raw[i]);
    } else {
      raw[i][0] = raw[i][1] = make_uint4(0, 0, 0, 0);
    }
  }
#pragma unroll
  for (int i = 0; i < CH; i++) {
    if (base + i * QMV_CTHREADS >= total) break;  // uniform over the CTA
    const int c = base + threadIdx.x + i * QMV_CTHREADS;
    float v[8];
    unpack8<XT>(raw[i], v);
    float am = 0.f, sum = 0.f;
#pragma unroll
    for (int j = 0; j < 8; j++) {
      am = fmaxf(am, fabsf(v[j]));
      if constexpr (SUMS) sum += v[j];
    }
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 1));
    am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, 2));
    float half = 0.f;
    if constexpr (SUMS) half = sum + __shfl_xor_sync(0xffffffffu, sum, 1);
    // With u = x * 127 / max|x| in [-127, 127], t = rint(256 u) + 128 is
    // 256 hi + (lo + 128) with lo in [-128, 127]: byte 1 of t is the level
    // hi, byte 0 is lo + 128, and hi + lo/256 = rint(256 u)/256.  The scale
    // and its reciprocal need only agree to a few ulps: the levels are
    // reconstructed with xs, never with inv.
    // Rounding: adding 1.5 * 2^23 leaves the float grid at spacing 1, so the
    // fma rounds 256 u + 128 once, to nearest even, and its bit pattern is
    // 0x4B400000 + t: bytes 0 and 1 are those of t (|t| < 2^15).  This
    // replaces a float-to-int conversion per value.
    const float inv = am > 0.f ? __fdividef(127.f * 256.f, am) : 0.f;
    uint32_t t[8];
#pragma unroll
    for (int j = 0; j < 8; j++) t[j] = __float_as_uint(fmaf(v[j], inv, 12582912.f + 128.f));
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int q = 0; q < 2; q++) {
      const uint32_t z01 = __byte_perm(t[4 * q], t[4 * q + 1], 0x5140);      // b0(t0) b0(t1) b1(t0) b1(t1)
      const uint32_t z23 = __byte_perm(t[4 * q + 2], t[4 * q + 3], 0x5140);
      lw[q] = __byte_perm(z01, z23, 0x5410) ^ 0x80808080u;
      hw[q] = __byte_perm(z01, z23, 0x7632);
    }
    if constexpr (MvDecode<T>::NIBBLE_ORDER) {
      // This thread holds words 2lc, 2lc+1 of its 32-group (lc = chunk & 3);
      // words q and q + 4 pair up, so chunk lc pairs with chunk lc ^ 2 (the
      // thread two lanes away: consecutive chunks are consecutive threads).
      const int lc = (base + threadIdx.x) & 3;
#pragma unroll
      for (int q = 0; q < 2; q++) {
        const uint32_t ph = __shfl_xor_sync(0xffffffffu, hw[q], 2);
        const uint32_t pl = __shfl_xor_sync(0xffffffffu, lw[q], 2);
        if (lc < 2) {
          hw[q] = __byte_perm(hw[q], ph, 0x5140u);
          lw[q] = __byte_perm(lw[q], pl, 0x5140u);
        } else {
          hw[q] = __byte_perm(ph, hw[q], 0x7362u);
          lw[q] = __byte_perm(pl, lw[q], 0x7362u);
        }
      }
    }
    if (c < total) {
      const int b = c >= per_row ? 1 : 0;
      const int cc = c - b * per_row;
      int8_t* qh = xq + (b * 2) * KS + cc * 8;
      *reinterpret_cast<uint2*>(qh) = make_uint2(hw[0], hw[1]);
      *reinterpret_cast<uint2*>(qh + KS) = make_uint2(lw[0], lw[1]);
      if ((cc & 3) == 0) xs[b * (KS / 32) + (cc >> 2)] = am * (1.f / (127.f * 256.f)) * MvDecode<T>::xgroup_scale(cc >> 2);
      if constexpr (SUMS) {
        if ((cc & 1) == 0) xsum[b * (KS / 16) + (cc >> 1)] = half;
      }
    }
  }
}

// Staged row (bulk path): each consumer thread quantises whole 32-groups of
// the 16-bit row that the bulk copy left at xq -- every value of a group in
// one thread, so no shuffles, about half the instructions per value of the
// per-chunk form.  All threads read their raw words (up to QMV_XSTAGE_G groups)
// before the first level is written over the staged row.
constexpr int QMV_XSTAGE_G = 3;

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}
template <typename XT> __device__ __forceinline__ float amax32(const uint4 (&r)[4]);
template <> __device__ __forceinline__ float amax32<__half>(const uint4 (&r)[4]) {
  __half2 m = __habs2(*reinterpret_cast<const __half2*>(&r[0].x));
#pragma unroll
  for (int i = 1; i < 16; i++) {
    const uint32_t u = word_of(r[i >> 2], i & 3);
    m = __hmax2(m, __habs2(*reinterpret_cast<const __half2*>(&u)));
  }
  const float2 f = __half22float2(m);
  return fmaxf(f.x, f.y);
}
template <> __device__ __forceinline__ float amax32<__nv_bfloat16>(const uint4 (&r)[4]) {
  uint32_t m = 0;  // |bf16| orders as its 15 low bits
#pragma unroll
  for (int i = 0; i < 16; i++) {
    const uint32_t u = word_of(r[i >> 2], i & 3);
    m = max(m, max(u & 0x7FFFu, (u >> 16) & 0x7FFFu));
  }
  return __uint_as_float(m << 16);
}
template <typename XT> __device__ __forceinline__ float2 pair32(const uint4 (&r)[4], int j);  // values 2j, 2j+1
template <> __device__ __forceinline__ float2 pair32<__half>(const uint4 (&r)[4], int j) {
  const uint32_t u = word_of(r[j >> 2], j & 3);
  return __half22float2(*reinterpret_cast<const __half2*>(&u));
}
template <> __device__ __forceinline__ float2 pair32<__nv_bfloat16>(const uint4 (&r)[4], int j) {
  const uint32_t u = word_of(r[j >> 2], j & 3);
  return make_float2(__uint_as_float(u << 16), __uint_as_float(u & 0xFFFF0000u));
}

template <int T, bool SUMS, typename XT>
__device__ void quantise_staged(int groups, int KS, int8_t* xq, float* xs, float* xsum) {
  uint4 raw[QMV_XSTAGE_G][4];
#pragma unroll
  for (int i = 0; i < QMV_XSTAGE_G; i++) {
    const int gg = threadIdx.x + i * QMV_CTHREADS;
    const uint4* p = reinterpret_cast<const uint4*>(xq + 64 * gg);
#pragma unroll
    for (int w2 = 0; w2 < 4; w2++) raw[i][w2] = gg < groups ? p[w2] : make_uint4(0, 0, 0, 0);
  }
  named_sync_consumers();
#pragma unroll
  for (int i = 0; i < QMV_XSTAGE_G; i++) {
    const int gg = threadIdx.x + i * QMV_CTHREADS;
    if (gg >= groups) break;
    const float am = amax32<XT>(raw[i]);
    // Levels and rounding as in quantise_round.
    const float inv = am > 0.f ? __fdividef(127.f * 256.f, am) : 0.f;
    uint32_t hw[8], lw[8];
    float s0 = 0.f, s1 = 0.f;
#pragma unroll
    for (int q = 0; q < 8; q++) {
      const float2 p0 = pair32<XT>(raw[i], 2 * q), p1 = pair32<XT>(raw[i], 2 * q + 1);
      if constexpr (SUMS) {
        if (q < 4) s0 += (p0.x + p0.y) + (p1.x + p1.y);
        else s1 += (p0.x + p0.y) + (p1.x + p1.y);
      }
      const uint32_t t0 = __float_as_uint(fmaf(p0.x, inv, 12582912.f + 128.f));
      const uint32_t t1 = __float_as_uint(fmaf(p0.y, inv, 12582912.f + 128.f));
      const uint32_t t2 = __float_as_uint(fmaf(p1.x, inv, 12582912.f + 128.f));
      const uint32_t t3 = __float_as_uint(fmaf(p1.y, inv, 12582912.f + 128.f));
      const uint32_t z01 = __byte_perm(t0, t1, 0x5140);
      const uint32_t z23 = __byte_perm(t2, t3, 0x5140);
      lw[q] = __byte_perm(z01, z23, 0x5410) ^ 0x80808080u;
      hw[q] = __byte_perm(z01, z23, 0x7632);
    }
    if constexpr (MvDecode<T>::NIBBLE_ORDER) nibble_order(hw, lw);
    uint4* qh = reinterpret_cast<uint4*>(xq + gg * 32);
    uint4* ql = reinterpret_cast<uint4*>(xq + KS + gg * 32);
    qh[0] = make_uint4(hw[0], hw[1], hw[2], hw[3]);
    qh[1] = make_uint4(hw[4], hw[5], hw[6], hw[7]);
    ql[0] = make_uint4(lw[0], lw[1], lw[2], lw[3]);
    ql[1] = make_uint4(lw[4], lw[5], lw[6], lw[7]);
    xs[gg] = am * (1.f / (127.f * 256.f)) * MvDecode<T>::xgroup_scale(gg);
    if constexpr (SUMS) *reinterpret_cast<float2*>(xsum + 2 * gg) = make_float2(s0, s1);
  }
}

template <int T, int NB, bool SUMS, typename XT>
__device__ void quantise_slice_t(const QmvArgs& a, int btile, int kb0, int w, int KS, int8_t* xq, float* xs,
                                 float* xsum) {
  constexpr int CH = sizeof(XT) == 4 ? 5 : 10;
  const int per_row = w * 32;  // 8-value chunks per activation row
  const int total = NB * per_row;
  if constexpr (NB == 1 && sizeof(XT) == 2) {
    if (a.xbulk) {  // the plan guarantees w * 8 <= QMV_XSTAGE_G * QMV_CTHREADS
      quantise_staged<T, SUMS, XT>(w * (QK / 32), KS, xq, xs, xsum);
      return;
    }
  }
  for (int base = 0; base < total; base += CH * QMV_CTHREADS)
    quantise_round<T, NB, SUMS, XT, CH>(a, btile, kb0, KS, per_row, total, base, xq, xs, xsum);
}

template <int T, int NB, bool SUMS>
__device__ __forceinline__ void quantise_slice(const QmvArgs& a, int btile, int kb0, int w, int KS, int8_t* xq,
                                               float* xs, float* xsum) {
  if (a.x_dtype == DT_F16) quantise_slice_t<T, NB, SUMS, __half>(a, btile, kb0, w, KS, xq, xs, xsum);
  else if (a.x_dtype == DT_BF16) quantise_slice_t<T, NB, SUMS, __nv_bfloat16>(a, btile, kb0, w, KS, xq, xs, xsum);
  else quantise_slice_t<T, NB, SUMS, float>(a, btile, kb0, w, KS, xq, xs, xsum);
}

// ---------------------------------------------------------------------------
// Work cursor over the (tile, block) units of one CTA's range [u0, u1) in its
// slice (tile-major, `w` blocks per tile).  The range is whole tiles framed by
// at most two tiles shared with neighbouring CTAs.  The cursor visits the
// shared tiles first -- the last one (whose piece other CTAs wait for), then
// the first one -- and the whole tiles after them, so that pieces are
// published early and the end of the kernel only finishes whole tiles.
struct QmvCursor {
  int64_t tile, t_hi;   // current tile, end of the current phase's tiles
  int64_t t0, t1;       // first / last tile of the range
  int blk, bend;        // current block, end block of the current tile
  int w, b0, e1;        // slice width, first block in t0, end block in t1
  int phase;            // 0 last shared tile, 1 first shared tile, 2 whole tiles, 3 done
  __device__ QmvCursor(int64_t u0, int64_t u1, int width) : w(width) {
    t0 = udiv(u0, width);
    b0 = (int)(u0 - t0 * width);
    t1 = udiv(u1 - 1, width);
    e1 = (int)(u1 - t1 * width);
    phase = u1 > u0 ? 0 : 3;
    enter();
  }
  __device__ void set(int64_t t, int64_t hi, int b, int e) {
    tile = t; t_hi = hi; blk = b; bend = e;
  }
  // Set up the current phase, skipping empty ones.
  __device__ void enter() {
    if (phase == 0) {
      if (t0 == t1) { set(t0, t0 + 1, b0, e1); return; }  // the range lies in one tile
      if (e1 < w) { set(t1, t1 + 1, 0, e1); return; }
      phase = 1;
    }
    if (phase == 1) {
      if (b0 > 0) { set(t0, t0 + 1, b0, w); return; }
      phase = 2;
    }
    if (phase == 2) {
      const int64_t lo = b0 > 0 ? t0 + 1 : t0, hi = e1 < w ? t1 : t1 + 1;
      if (lo < hi) { set(lo, hi, 0, w); return; }
      phase = 3;
    }
  }
  __device__ bool done() const { return phase == 3; }
  __device__ int chunk(int cb) const { return min(cb, bend - blk); }
  // Advances by n blocks; returns true when this ends the CTA's part of the
  // current tile.
  __device__ bool advance(int n) {
    blk += n;
    if (blk < bend) return false;
    tile++;
    if (tile < t_hi) {
      blk = 0;
      bend = w;
    } else {
      phase = (phase == 0 && t0 == t1) ? 3 : phase + 1;
      enter();
    }
    return true;
  }
};

// Unit range [u0, u1) of CTA c among C over U units (whole tiles of width w
// when `aligned`).
__device__ __forceinline__ void cta_range(const QmvArgs& a, int64_t U, int w, int c, int C, int64_t& u0,
                                          int64_t& u1) {
  if (a.aligned) {
    u0 = udiv((int64_t)c * a.tiles, C) * w;
    u1 = udiv((int64_t)(c + 1) * a.tiles, C) * w;
  } else {
    u0 = udiv((int64_t)c * U, C);
    u1 = udiv((int64_t)(c + 1) * U, C);
  }
}

// ---------------------------------------------------------------------------
// The matvec kernel.

// Single-slice plans: a tile shared by consecutive CTAs c0 < ... < ck is
// finished by ck, the CTA holding its last block.  Every other CTA publishes
// its piece (one per CTA: the end of its range) with plain stores, encoded so
// that no float maps to 0 (the one 32-bit pattern that would, 0xFFBFFFFF, is
// a NaN payload arithmetic never produces); ck reads them in CTA order,
// resets the slots to 0 and writes y.  The pieces are visited first by their
// CTAs, so ck rarely waits; the wait is bounded.
__device__ __forceinline__ uint32_t piece_enc(float v) { return __float_as_uint(v) + 0x00400001u; }
__device__ __forceinline__ float piece_dec(uint32_t e) { return __uint_as_float(e - 0x00400001u); }
__device__ __forceinline__ uint32_t ld_relaxed_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ void st_relaxed_gpu(uint32_t* p, uint32_t v) {
  asm volatile("st.relaxed.gpu.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

template <int NB>
__device__ void publish_piece(const QmvArgs& a, int btile, int C, int c, float v) {
  const int lane = threadIdx.x & 31;
  if (lane < NB * 16) st_relaxed_gpu(a.slots + ((int64_t)btile * C + c) * (NB * 16) + lane, piece_enc(v));
}

template <int NB, bool GATHER>
__device__ void gather_pieces(const QmvArgs& a, int btile, int C, int c, int64_t U, int w, int64_t tile, float v,
                              unsigned ep) {
  const int lane = threadIdx.x & 31;
  if (lane >= NB * 16) return;
  const int64_t c0 = udiv((tile * w + 1) * C - 1, U);  // first CTA touching the tile
  float sum = 0.f;
  for (int64_t c2 = c0; c2 < c; c2++) {
    uint32_t* p = a.slots + ((int64_t)btile * C + c2) * (NB * 16) + lane;
    uint32_t e = ld_relaxed_gpu(p);
    if (e == 0u) {
      const long long t0 = clock64();
      while (e == 0u) {
        __nanosleep(64);
        e = ld_relaxed_gpu(p);
        if (e == 0u && clock64() - t0 > (1ll << 31)) {
          if (a.err) atomicExch(a.err, DEV_WAIT_TIMEOUT);
          break;
        }
      }
    }
    sum += piece_dec(e);
    st_relaxed_gpu(p, 0u);
  }
  sum += v;
  const int b = lane >> 4, r = lane & 15;
  const int batch = btile * NB + b;
  const int64_t rr = tile * 16 + r;
  final_store<GATHER>(a, NB == 1 ? 0xffffu : 0xffffffffu, batch, tile, r, sum, batch < a.rows && rr < a.N, ep);
}

// Global combination of one piece of a tile shared with other CTAs (other
// slices and/or neighbouring CTAs of the same slice): publish the piece, take
// a ticket, and if this was the last piece, sum all pieces of the tile in
// slice order then CTA order and write y.  Executed by the combiner warp; v
// is this piece's row sum (lane = b*16 + r).
template <int NB, bool GATHER>
__device__ void combine_piece(const QmvArgs& a, int btile, int slice, int C, int c, int w, int64_t tile,
                              int64_t first_tile, int seg_len, float v, unsigned ep) {
  const int lane = threadIdx.x & 31;
  float* pp;
  if (seg_len == w)
    pp = a.part_full + (((int64_t)btile * a.slices + slice) * a.tiles + tile) * (NB * 16);
  else
    pp = a.part_piece + ((((int64_t)btile * a.slices + slice) * C + c) * 2 + (tile == first_tile ? 0 : 1)) * (NB * 16);
  if (lane < NB * 16) pp[lane] = v;
  // The warp barrier orders every lane's store before lane 0's ticket, whose
  // release makes them visible with it; its acquire (for the last piece)
  // orders the reads of the other pieces after all of their tickets.
  __syncwarp();
  unsigned last = 0;
  unsigned* tk = a.tickets + (int64_t)btile * a.tiles + tile;
  if (lane == 0) {
    const unsigned prev = atom_add_acq_rel_gpu(tk, (unsigned)seg_len);
    last = (prev + (unsigned)seg_len == (unsigned)a.kb);
  }
  last = __shfl_sync(0xffffffffu, last, 0);
  if (!last) return;
  if (lane < NB * 16) {
    float sum = 0.f;
    for (int s2 = 0; s2 < a.slices; s2++) {
      const int w2 = min(a.bps, a.kb - s2 * a.bps);
      const int64_t U2 = a.tiles * w2;
      const int64_t ut0 = tile * w2, ut1 = ut0 + w2;
      const int64_t c0 = udiv((ut0 + 1) * C - 1, U2);
      const int64_t c1 = udiv(ut1 * C - 1, U2);
      const int64_t base = (int64_t)btile * a.slices + s2;
      if (c0 == c1) {  // one CTA covered the whole slice of this tile
        sum += __ldcg(a.part_full + (base * a.tiles + tile) * (NB * 16) + lane);
        continue;
      }
      for (int64_t c2 = c0; c2 <= c1; c2++) {
        const int64_t s0 = udiv(c2 * U2, C), s1 = udiv((c2 + 1) * U2, C);
        if (s0 == s1 || s1 <= ut0 || s0 >= ut1) continue;  // empty or not covering this tile
        const int sl = (udiv(s0, w2) == tile) ? 0 : 1;
        sum += __ldcg(a.part_piece + ((base * C + c2) * 2 + sl) * (NB * 16) + lane);
      }
    }
    const int b = lane >> 4, r = lane & 15;
    const int batch = btile * NB + b;
    const int64_t rr = tile * 16 + r;
    final_store<GATHER>(a, NB == 1 ? 0xffffu : 0xffffffffu, batch, tile, r, sum, batch < a.rows && rr < a.N, ep);
  }
  if (lane == 0) *tk = 0u;
}

// GATHER: the row-parallel variant (gsq_qmv_gather), instantiated for
// one-activation-row tiles only; the ordinary kernel carries none of its code
// (its presence alone cost ~2 % in the single-GPU sweep).
template <int T, int NB, bool GATHER>
__global__ void __launch_bounds__(QMV_THREADS, 2) qmv_kernel(const QmvArgs a) {
  using MV = Mv<T>;
  using G = QmvGeom<T>;
  constexpr int UNIT = MV::UNIT;
  constexpr int UPS = 4 / NB;            // unit slots (lanes of a quad per activation row)
  constexpr int SETS = QK / (UNIT * UPS);  // units per slot and block
  constexpr int MMAS = UNIT / (8 * NB);  // MMAs per set
  static_assert(MMAS >= 1, "set must cover at least one MMA");
  static_assert(!MV::IDENT || UNIT == 32, "identity mapping needs 32-wide units");
  const int NS = a.ns, RB = a.ns + 1;

  // Shared memory: tables | mbarriers | row-sum buffers | ring | activations.
  extern __shared__ __align__(128) uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((0u - smem_u32(smem_raw)) & 127u);  // keeps shared provenance
  uint8_t* tab = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + G::TAB);  // [NS] stage landed (tx bytes)
  uint64_t* empty = full + QMV_NS_MAX;                          // [NS] stage released by all consumers
  uint64_t* segb = empty + QMV_NS_MAX;                          // [RB] segment row sums posted by all consumers
  uint64_t* rfree = segb + QMV_RED_BUFS;                        // [RB] segment row sums read
  uint64_t* xready = rfree + QMV_RED_BUFS;                      // activations quantised
  uint64_t* xcopy = xready + 1;                                  // bulk copy of the activations landed
  // B operand of the columns a lane does not feed: one block of zero
  // activations (offsets within a block stay below QK).
  int8_t* zeros = reinterpret_cast<int8_t*>(smem + G::TAB + 256);
  float* red = reinterpret_cast<float*>(smem + G::TAB + 256 + QK);
  uint8_t* ring = smem + G::TAB + 256 + QK + QMV_RED_BYTES;
  const int CB = a.cb, ROWB = a.rowb, STAGE = a.stage;
  const int KS = a.bps * QK;
  int8_t* xq_s = reinterpret_cast<int8_t*>(ring + NS * STAGE);
  float* xs_s = reinterpret_cast<float*>(ring + NS * STAGE + NB * 2 * KS);
  float* xsum_s = xs_s + NB * (KS / 32);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = gridDim.x, c = blockIdx.x;
  const int slice = blockIdx.y, btile = blockIdx.z;
  const int kb0 = slice * a.bps;                       // first block of the slice
  const int w = min(a.bps, a.kb - kb0);                // slice width in blocks
  const int64_t U = a.tiles * w;
  int64_t ub, ue;
  cta_range(a, U, w, c, C, ub, ue);

  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; s++) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], QMV_CWARPS);
    }
    for (int s = 0; s < RB; s++) {
      mbar_init(&segb[s], QMV_CWARPS);
      mbar_init(&rfree[s], 1);
    }
    mbar_init(xready, 1);
    mbar_init(xcopy, 1);
    fence_mbar_init();
  }
  __syncthreads();
  pdl_launch_dependents();

  if (warp == QMV_PRODUCER) {
    // ------------------------------------------------------------ producer
    const uintptr_t pbase = reinterpret_cast<uintptr_t>(a.packed);
    const uint64_t policy = l2_policy_evict_first();
    QmvCursor cur(ub, ue, w);
    int i = 0, s = 0;
    uint32_t ph = 0;
    bool dead = false;
    while (!cur.done()) {
      // The first `pre` stages go out at once (before the previous kernel
      // has finished: weights only); further stages wait until the
      // activations are in, so their loads do not queue behind weights.
      if (i == a.pre && i < NS && !dead && !mbar_wait_bounded(xready, 0u, a.err)) dead = true;
      if (i >= NS && !dead && !mbar_wait_bounded(&empty[s], ph ^ 1u, a.err)) dead = true;
      const int nblk = cur.chunk(CB);
      uint32_t bytes = 0;
      if (lane < 16 && !dead) {
        const int64_t r = cur.tile * 16 + lane;
        if (r < a.N) {
          const int64_t off = r * a.row_bytes + (int64_t)(kb0 + cur.blk) * G::BB;
          const int64_t end = off + (int64_t)nblk * G::BB;
          const int64_t off_al = off & ~int64_t(15);
          int64_t end_al = (end + 15) & ~int64_t(15);
          if (end_al > a.packed_bytes) end_al = end & ~int64_t(15);
          uint8_t* dst = ring + s * STAGE + lane * ROWB;
          if (end_al > off_al) {
            bytes = (uint32_t)(end_al - off_al);
            fence_proxy_async_smem();
            bulk_g2s_stream(dst, reinterpret_cast<const void*>(pbase + off_al), bytes, &full[s], policy);
          }
          // Tail beyond the last 16-byte boundary of the buffer: plain loads.
          for (int64_t t = max(end_al, off_al); t < end; t++) dst[t - off_al] = a.packed[t];
        }
      }
      const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
      __syncwarp();
      if (lane == 0) mbar_arrive_expect_tx(&full[s], total);
      cur.advance(nblk);
      i++;
      if (++s == NS) { s = 0; ph ^= 1u; }
    }
    // Every issued copy has landed before the CTA may exit (the consumers
    // wait for them too; this covers the timed-out path).
    for (int j = max(0, i - NS); j < i; j++)
      mbar_wait_bounded(&full[j % NS], (uint32_t)((j / NS) & 1), nullptr);
    return;
  }

  if (warp == QMV_COMBINER) {
    // ------------------------------------------------------------ combiner
    // Walks the same segments as the consumers (one per tile touched) and
    // takes over every piece that needs other CTAs' pieces, so that the
    // tensor-core warps never wait on global-memory round trips.
    pdl_wait();  // before any global write
    const unsigned gep = gather_count<GATHER>(a);
    QmvCursor cur(ub, ue, w);
    const int64_t first_tile = cur.t0;
    int rbuf = 0;
    uint32_t rph = 0;
    bool dead = false;
    while (!cur.done()) {
      const int64_t tile = cur.tile;
      const int sb = cur.blk;
      const int seg_len = cur.chunk(1 << 30);
      cur.advance(seg_len);
      if (seg_len != a.kb) {
        if (!dead && !mbar_wait_bounded(&segb[rbuf], rph, a.err)) dead = true;
        float v = 0.f;
        if (lane < NB * 16) {
#pragma unroll
          for (int w2 = 0; w2 < QMV_CWARPS; w2++) v += red[(rbuf * QMV_CWARPS + w2) * 32 + lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfree[rbuf]);
        if (a.slices > 1)
          combine_piece<NB, GATHER>(a, btile, slice, C, c, w, tile, first_tile, seg_len, v, gep);
        else if (sb + seg_len < w)
          publish_piece<NB>(a, btile, C, c, v);  // later CTAs hold the rest of this tile
        else
          gather_pieces<NB, GATHER>(a, btile, C, c, U, w, tile, v, gep);
      }
      if (++rbuf == RB) { rbuf = 0; rph ^= 1u; }
    }
    if constexpr (GATHER) gather_finish(a, gep);
    return;
  }

  // -------------------------------------------------------------- consumers
  MV::load_tables(tab, threadIdx.x, QMV_CTHREADS);
  if (threadIdx.x < QK / 4) reinterpret_cast<uint32_t*>(zeros)[threadIdx.x] = 0u;
  // Everything above reads only weights and tables; from here on the kernel
  // reads activations / scratch that an earlier kernel in the stream writes.
  pdl_wait();
  if (a.xbulk) {
    // One bulk copy brings the slice of the activation row (16-bit values)
    // into the level area; per-thread loads of the same bytes from every CTA
    // at once queue on each SM's outstanding-miss limit.
    if (threadIdx.x == 0) {
      const uint32_t bytes = (uint32_t)w * QK * 2u;
      mbar_arrive_expect_tx(xcopy, bytes);
      bulk_g2s(xq_s, reinterpret_cast<const uint8_t*>(a.x) + ((int64_t)btile * a.K + (int64_t)kb0 * QK) * 2, bytes,
               xcopy);
    }
    mbar_wait_bounded(xcopy, 0u, a.err);
  }
  quantise_slice<T, NB, MV::BIAS>(a, btile, kb0, w, KS, xq_s, xs_s, xsum_s);
  const unsigned gep = gather_count<GATHER>(a);
  named_sync_consumers();
  if (threadIdx.x == 0) mbar_arrive(xready);

  const int g = lane >> 2, tq = lane & 3;
  // A operand: unit slot q and first entry e0 of this lane.  B operand:
  // column g = (unit slot s_col, activation row b_col, level), live in the
  // k rows of the lanes that feed slot s_col -- this lane's own k rows when
  // s_col == q; otherwise it reads zeros.  Epilogue: slot q, activation row e0.
  const int q = tq / NB, e0 = tq % NB;
  const int pcol = g >> 1, level = g & 1;
  const int s_col = pcol / NB, b_col = pcol % NB;
  const bool xlive = s_col == q;
  const int8_t* xbase = xq_s + (b_col * 2 + level) * KS + (MV::IDENT ? 32 * q + 4 * e0 : UNIT * q + 8 * e0);
  const float* xs_row = xs_s + e0 * (KS / 32);
  const float* xsum_row = xsum_s + e0 * (KS / 16);
  // Per-entry path (formats without a lane-unit view): the four lanes of a
  // quad feed consecutive entries of one 32-weight chunk; column g is live in
  // the one MMA of a set whose unit slot is s_col, and lane (g, tq) scales
  // unit slot q of every set.
  using FO = Fast<T>;
  using MD = MvDecode<T>;
  constexpr int KSET = UNIT * UPS;  // k per set
  const int8_t* xrow_o = xq_s + (b_col * 2 + level) * KS;
  const int s_ep = q;

  // Row starts keep their offset modulo 16 from tile to tile (a tile is 16
  // rows), so the staged position of a block needs only 32-bit arithmetic.
  const uint32_t rb16 = (uint32_t)a.row_bytes & 15u;
  const uint32_t h0 = (rb16 * (uint32_t)g) & 15u, h1 = (rb16 * (uint32_t)(g + 8)) & 15u;
  const uint8_t* lane_st0 = ring + g * ROWB;
  const uint8_t* lane_st1 = ring + (g + 8) * ROWB;

  float acc0 = 0.f, acc1 = 0.f;
  QmvCursor cur(ub, ue, w);
  int seg_len = 0;
  int s = 0, rbuf = 0, seg_no = 0;
  uint32_t ph = 0, rph = 0;
  bool dead = false;
  while (!cur.done()) {
    if (!dead && !mbar_wait_bounded(&full[s], ph, a.err)) dead = true;
    const int nblk = cur.chunk(CB);
    const int64_t tile = cur.tile;
    const uint32_t kb16 = ((uint32_t)(kb0 + cur.blk) * (uint32_t)G::BB) & 15u;
    const uint8_t* r0p = lane_st0 + s * STAGE + ((h0 + kb16) & 15u);
    const uint8_t* r1p = lane_st1 + s * STAGE + ((h1 + kb16) & 15u);
    for (int bi = warp; bi < nblk; bi += QMV_CWARPS) {
      const uint8_t* b0 = r0p + bi * G::BB;
      const uint8_t* b1 = r1p + bi * G::BB;
      const int kk = (cur.blk + bi) * QK;  // within the slice
      if constexpr (MV::LANE_UNITS) {
        const int8_t* xl = xlive ? xbase + kk : zeros;
        const auto row0 = MV::template row<NB>(b0, q);
        const auto row1 = MV::template row<NB>(b1, q);
        float A0 = 0.f, A1 = 0.f, M0 = 0.f, M1 = 0.f;
        static_for<0, SETS>([&](auto s_) {
          constexpr int S = decltype(s_)::value;
          const int u = UPS * S + q;  // this lane's unit
          int C[4] = {0, 0, 0, 0}, N[4] = {0, 0, 0, 0};
#pragma unroll
          for (int j = 0; j < MMAS; j++) {
            const int e = e0 + NB * j;
            uint32_t bx0, bx1;
            if constexpr (MV::IDENT) {
              bx0 = *reinterpret_cast<const uint32_t*>(xl + 32 * UPS * S + 4 * NB * j);
              bx1 = *reinterpret_cast<const uint32_t*>(xl + 32 * UPS * S + 16 + 4 * NB * j);
            } else {
              const uint2 v = *reinterpret_cast<const uint2*>(xl + UNIT * UPS * S + 8 * NB * j);
              bx0 = v.x;
              bx1 = v.y;
            }
            uint32_t a0, a1, a2, a3, m0, m1, m2, m3;
            MV::template entry<S, NB>(b0, row0, u, e, tab, a0, a2, m0, m2);
            MV::template entry<S, NB>(b1, row1, u, e, tab, a1, a3, m1, m3);
            if constexpr (MV::UNSIGNED) mma_u8s8(C, a0, a1, a2, a3, bx0, bx1);
            else mma_s8(C, a0, a1, a2, a3, bx0, bx1);
            if constexpr (MV::SPLIT) mma_s8(N, a0 & m0, a1 & m1, a2 & m2, a3 & m3, bx0, bx1);
          }
          const int ku = kk + UNIT * u;  // within the slice
          const float xs = xs_row[ku >> 5];
          float xsum = 0.f;
          if constexpr (MV::BIAS) {
            xsum = xsum_row[ku >> 4];
            if constexpr (UNIT == 32) xsum += xsum_row[(ku >> 4) + 1];
          }
          MV::template unit<S, NB>(b0, row0, u, C[0] * 256 + C[1], N[0] * 256 + N[1], xs, xsum, A0, M0);
          MV::template unit<S, NB>(b1, row1, u, C[2] * 256 + C[3], N[2] * 256 + N[3], xs, xsum, A1, M1);
        });
        acc0 += MV::finish(b0, row0, A0, M0);
        acc1 += MV::finish(b1, row1, A1, M1);
      } else {
        const int8_t* xb = xrow_o + kk;
        const float* xsb = xs_row + (kk >> 5);
        const float* xub = xsum_row + (kk >> 4);
        // Block accumulators in units of the block scales (dscale).
        float A0 = 0.f, A1 = 0.f, M0 = 0.f, M1 = 0.f;
#pragma unroll
        for (int set = 0; set < SETS; set++) {
          const int kset = set * KSET;
          // Activation words for the one MMA of this set where column g is live.
          uint32_t xw0, xw1;
          int jsel;
          if constexpr (UNIT == 32) {
            jsel = s_col;
            if constexpr (FO::BLOCKED) {
              const uint2 v = *reinterpret_cast<const uint2*>(xb + kset + 32 * s_col + 8 * tq);
              xw0 = v.x; xw1 = v.y;
            } else {
              xw0 = *reinterpret_cast<const uint32_t*>(xb + kset + 32 * s_col + 4 * tq);
              xw1 = *reinterpret_cast<const uint32_t*>(xb + kset + 32 * s_col + 16 + 4 * tq);
            }
          } else {
            jsel = s_col >> 1;
            const bool live = (s_col & 1) == (tq >> 1);
            const uint2 v = *reinterpret_cast<const uint2*>(xb + kset + 32 * jsel + 8 * tq);
            xw0 = live ? v.x : 0u;
            xw1 = live ? v.y : 0u;
          }
          // Two independent accumulator chains (even / odd MMAs) halve the
          // dependent tensor-core latency per set.  Sign-carrying formats run a
          // second pair of chains on the negative-position magnitudes.
          int Cc[4] = {0, 0, 0, 0}, Cb[4] = {0, 0, 0, 0};
          int Nn[4] = {0, 0, 0, 0}, Nb[4] = {0, 0, 0, 0};
#pragma unroll
          for (int j = 0; j < MMAS; j++) {
            const int c32 = set * MMAS + j;
            const bool on = (j == jsel);
            const uint32_t bx0 = on ? xw0 : 0u, bx1 = on ? xw1 : 0u;
            if constexpr (MD::SPLIT) {
              uint32_t a0, a1, a2, a3, m0, m1, m2, m3;
              FO::entry_split(b0, c32, tq, tab, a0, a2, m0, m2);
              FO::entry_split(b1, c32, tq, tab, a1, a3, m1, m3);
              if (j & 1) {
                mma_s8(Cb, a0, a1, a2, a3, bx0, bx1);
                mma_s8(Nb, a0 & m0, a1 & m1, a2 & m2, a3 & m3, bx0, bx1);
              } else {
                mma_s8(Cc, a0, a1, a2, a3, bx0, bx1);
                mma_s8(Nn, a0 & m0, a1 & m1, a2 & m2, a3 & m3, bx0, bx1);
              }
            } else {
              uint32_t a0, a1, a2, a3;
              MD::entry(b0, c32, tq, tab, a0, a2);
              MD::entry(b1, c32, tq, tab, a1, a3);
              if constexpr (MD::UNSIGNED) {
                if (j & 1) mma_u8s8(Cb, a0, a1, a2, a3, bx0, bx1);
                else mma_u8s8(Cc, a0, a1, a2, a3, bx0, bx1);
              } else {
                if (j & 1) mma_s8(Cb, a0, a1, a2, a3, bx0, bx1);
                else mma_s8(Cc, a0, a1, a2, a3, bx0, bx1);
              }
            }
          }
          if constexpr (MMAS > 1) {
#pragma unroll
            for (int i = 0; i < 4; i++) Cc[i] += Cb[i];
          }
          if constexpr (MD::SPLIT) {
#pragma unroll
            for (int i = 0; i < 4; i++) Cc[i] -= 2 * (Nn[i] + Nb[i]);
          }
          const int unit = set * UPS + s_ep;
          const int ku = unit * UNIT;  // within the block
          const float xsv = xsb[ku >> 5];
          int k0, m0, k1, m1;
          FO::kscale(b0, unit, k0, m0);
          FO::kscale(b1, unit, k1, m1);
          const int c0 = Cc[0] * 256 + Cc[1], c1 = Cc[2] * 256 + Cc[3];
          if constexpr (FO::KINT) {
            A0 = fmaf(xsv, (float)(k0 * c0), A0);
            A1 = fmaf(xsv, (float)(k1 * c1), A1);
          } else {
            A0 = fmaf(xsv * (float)k0, (float)c0, A0);
            A1 = fmaf(xsv * (float)k1, (float)c1, A1);
          }
          if constexpr (FO::HAS_BIAS) {
            float xu = xub[ku >> 4];
            if constexpr (UNIT == 32) xu += xub[(ku >> 4) + 1];
            M0 = fmaf((float)m0, xu, M0);
            M1 = fmaf((float)m1, xu, M1);
          }
        }
        float D0, DM0, D1, DM1;
        FO::dscale(b0, D0, DM0);
        FO::dscale(b1, D1, DM1);
        acc0 = fmaf(D0, A0, acc0);
        acc1 = fmaf(D1, A1, acc1);
        if constexpr (FO::HAS_BIAS) {
          acc0 = fmaf(DM0, M0, acc0);
          acc1 = fmaf(DM1, M1, acc1);
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&empty[s]);
    if (++s == NS) { s = 0; ph ^= 1u; }
    seg_len += nblk;
    if (cur.advance(nblk)) {
      // ---- end of this CTA's segment of `tile`: reduce the quad lanes that
      // hold the same activation row, post the warp's row sums, move on.
      if constexpr (NB == 1) {
        acc0 += __shfl_xor_sync(0xffffffffu, acc0, 1);
        acc1 += __shfl_xor_sync(0xffffffffu, acc1, 1);
      }
      acc0 += __shfl_xor_sync(0xffffffffu, acc0, 2);
      acc1 += __shfl_xor_sync(0xffffffffu, acc1, 2);
      // Buffer rbuf was last used RB segments ago; wait until it was read.
      if (seg_no >= RB && !dead && !mbar_wait_bounded(&rfree[rbuf], rph ^ 1u, a.err)) dead = true;
      float* rb = red + (rbuf * QMV_CWARPS + warp) * 32;
      if (tq < NB) {
        rb[e0 * 16 + g] = acc0;
        rb[e0 * 16 + g + 8] = acc1;
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&segb[rbuf]);
      // A whole tile is finished here by one consumer warp (rotating); tiles
      // shared with other CTAs go to the combiner warp.
      if (seg_len == a.kb && warp == (seg_no & (QMV_CWARPS - 1))) {
        if (!dead && !mbar_wait_bounded(&segb[rbuf], rph, a.err)) dead = true;
        float v = 0.f;
        if (lane < NB * 16) {
#pragma unroll
          for (int w2 = 0; w2 < QMV_CWARPS; w2++) v += red[(rbuf * QMV_CWARPS + w2) * 32 + lane];
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&rfree[rbuf]);
        const int b = lane >> 4, r = lane & 15;
        const int batch = btile * NB + b;
        const int64_t rr = tile * 16 + r;
        final_store<GATHER>(a, 0xffffffffu, batch, tile, r, v, lane < NB * 16 && batch < a.rows && rr < a.N, gep);
      }
      if (++rbuf == RB) { rbuf = 0; rph ^= 1u; }
      seg_no++;
      acc0 = acc1 = 0.f;
      seg_len = 0;
    }
  }
  if constexpr (GATHER) gather_finish(a, gep);
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
  const size_t smem = QMV_CTA_SMEM;
  if (cudaFuncSetAttribute(qmv_kernel<T, NB, false>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) !=
          cudaSuccess ||
      cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, qmv_kernel<T, NB, false>, QMV_THREADS, smem) != cudaSuccess ||
      occ <= 0) {
    cudaGetLastError();
    occ = (int)std::max<size_t>(1, std::min<size_t>(2, (228u * 1024u) / (smem + 1024)));
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
    fixed = QmvGeom<TT>::FIXED;                                                         \
    bb = QmvGeom<TT>::BB;                                                               \
    occ = nb == 1 ? qmv_occupancy<TT, 1>() : qmv_occupancy<TT, 2>();                    \
    break;

static size_t align256(size_t v) { return (v + 255) / 256 * 256; }

static QmvPlan qmv_plan_compute(int t, int64_t N, int64_t K, int rows, bool one_row_tiles) {
  QmvPlan p = {};
  const int kb = (int)(K / QK);
  p.nb = rows == 1 || one_row_tiles ? 1 : 2;
  p.btiles = (rows + p.nb - 1) / p.nb;
  p.tiles = (N + 15) / 16;
  size_t fixed = 0;
  int occ = 1, bb = 0;
  const int nb = p.nb;
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_GEOM_CASE) default: break; }
  // Shared memory per CTA = fixed part + ring (2..4 stages) + the activations
  // of one K-slice.  Wider stages (more blocks per consumer warp between
  // ring synchronisations) are taken when the activations of a whole row
  // still fit next to two of them; otherwise stages of 8 blocks, and as few
  // K-slices as fit.
  const size_t avail = QMV_CTA_SMEM - fixed;
  auto xbytes = [&](int bps) { return align256((size_t)nb * bps * QMV_XBYTES_PER_BLOCK); };
  const int cb_max = bb <= 84 ? 32 : 16;
  p.cb = 8;
  for (int cb = cb_max; cb > 8; cb /= 2) {
    if (cb > 2 * kb) continue;  // wider than two tile rows: no gain
    if (xbytes(kb) + 2 * (size_t)(16 * qmv_rowb(cb, bb)) <= avail) { p.cb = cb; break; }
  }
  const size_t stage = 16 * (size_t)qmv_rowb(p.cb, bb);
  p.slices = 1;
  while (p.slices < kb && xbytes((kb + p.slices - 1) / p.slices) + 2 * stage > avail) p.slices++;
  p.bps = (kb + p.slices - 1) / p.slices;
  p.slices = (kb + p.bps - 1) / p.bps;
  p.ns = (int)std::min<size_t>(QMV_NS_MAX, (avail - xbytes(p.bps)) / stage);
  if (p.ns < 2) {  // cannot happen for 8-block stages (static_assert); refuse rather than run a 1-stage ring
    p.ctas = 0;
    return p;
  }
  const int w_min = kb - (p.slices - 1) * p.bps;  // the last slice is the narrowest
  // CTAs per slice: fill every resident slot once.
  const int64_t slots = std::max<int64_t>(1, (int64_t)occ * qmv_sm_count() / p.btiles);
  int64_t ctas = std::max<int64_t>(1, slots / p.slices);
  ctas = std::min<int64_t>(ctas, p.tiles * w_min);
  // At least QMV_MIN_UNITS (tile, block) units per CTA: a CTA quantises the
  // whole activation slice whatever its share, so small matrices (the row
  // shards of 4-8 ranks) ran faster on fewer CTAs (the 33-configuration
  // sweep at 1/8 of the rows: 268 -> 246 us; at 1/4: 287 -> 278 us; full
  // and half matrices keep one CTA per resident slot).
  ctas = std::min<int64_t>(ctas, std::max<int64_t>(1, p.tiles * w_min / QMV_MIN_UNITS));
  // Single-slice piece slots must fit the always-zero fixed region.
  ctas = std::min<int64_t>(ctas, (int64_t)(QMV_TICKET_BYTES / ((size_t)p.btiles * nb * 16 * sizeof(float))));
  p.aligned = 0;
  if (p.tiles * p.btiles > QMV_TICKET_SLOTS) {
    // Too many tiles for the ticket region: CTAs own whole tiles.  With that
    // many tiles per CTA the split is balanced anyway.
    p.aligned = 1;
    ctas = std::min<int64_t>(ctas, p.tiles);
  }
  p.ctas = (int)ctas;
  p.smem = fixed + (size_t)p.ns * stage + xbytes(p.bps);
  p.rowb = qmv_rowb(p.cb, bb);
  p.stage = (int)stage;
  p.pre = p.ns;
  const bool split = !(p.slices == 1 && (p.aligned || p.tiles % p.ctas == 0));
  if (split && p.aligned) {
    p.ctas = 0;  // not plannable: slices need tickets (K beyond the activation budget with > 1M rows)
    return p;
  }
  if (split && p.slices == 1) {
    // Published-piece slots only, inside the always-zero fixed region.
    p.off_full = p.off_piece = 0;
    p.workspace = align256((size_t)p.btiles * p.ctas * nb * 16 * sizeof(float));
  } else if (split) {
    const size_t seg = (size_t)nb * 16 * sizeof(float);
    p.off_full = QMV_TICKET_BYTES;
    p.off_piece = p.off_full + align256((size_t)p.btiles * p.slices * p.tiles * seg);
    p.workspace = p.off_piece + align256((size_t)p.btiles * p.slices * p.ctas * 2 * seg);
  } else {
    p.off_full = p.off_piece = 0;
    p.workspace = 0;
  }
  return p;
}

// The plan depends only on the shape (and the device model): the last few are
// kept per host thread, so a call does not redo it (the workspace query and
// the launch of one call both need it).
QmvPlan qmv_plan(int t, int64_t N, int64_t K, int rows, bool one_row_tiles) {
  struct Entry {
    int t, rows, one;
    int64_t N, K;
    QmvPlan p;
  };
  static thread_local Entry cache[8];
  static thread_local int filled = 0, next = 0;
  for (int i = 0; i < filled; i++) {
    const Entry& e = cache[i];
    if (e.t == t && e.N == N && e.K == K && e.rows == rows && e.one == (int)one_row_tiles) return e.p;
  }
  const QmvPlan p = qmv_plan_compute(t, N, K, rows, one_row_tiles);
  cache[next] = Entry{t, rows, (int)one_row_tiles, N, K, p};
  next = (next + 1) % 8;
  filled = std::min(filled + 1, 8);
  return p;
}

template <int T, int NB, bool GATHER>
static cudaError_t qmv_launch_t(const QmvArgs& a, const QmvPlan& p, cudaStream_t st) {
  auto kern = qmv_kernel<T, NB, GATHER>;
  static int configured[64] = {0};  // dynamic smem attribute already set, per device
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= 64 || !configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)QMV_CTA_SMEM);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) configured[dev] = 1;
  }
  return launch_pdl(kern, dim3(p.ctas, p.slices, p.btiles), dim3(QMV_THREADS), p.smem, st, a);
}

#define GSQ_QMV_LAUNCH_CASE(TT)                                                     \
  case TT:                                                                          \
    if (a.world > 1) return p.nb == 1 ? qmv_launch_t<TT, 1, true>(a, p, st) : cudaErrorInvalidValue; \
    return p.nb == 1 ? qmv_launch_t<TT, 1, false>(a, p, st) : qmv_launch_t<TT, 2, false>(a, p, st);

static cudaError_t qmv_launch(int t, const QmvArgs& a, const QmvPlan& p, cudaStream_t st) {
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_QMV_LAUNCH_CASE) }
  return cudaErrorInvalidValue;
}

size_t qmv_gather_inbox_offset(int64_t rows, int64_t ntot) {
  return (QMV_GATHER_HEADER + (size_t)rows * ntot * sizeof(float) + 15) / 16 * 16;
}

// The inbox exists only for decode-sized regions (fewer than 8 rows: the
// matvec's gather); a prefill region (the tiled matmul's gather) is header
// and output only.
size_t qmv_gather_region_bytes(int64_t rows, int64_t ntot) {
  return qmv_gather_inbox_offset(rows, ntot) + (rows < 8 ? 2 * (size_t)rows * ntot * sizeof(uint2) : 0);
}

cudaError_t qmv_run(int t, const void* x, int x_dtype, const uint8_t* packed, int64_t N, int64_t K, int rows,
                    void* y, int y_dtype, void* ws, const QmvPlan& p, int* err, cudaStream_t st,
                    const QmvGather* gather, int glu) {
  if (p.ctas <= 0) return cudaErrorInvalidValue;
  if (glu && ((N & 15) || (gather && gather->world > 1))) return cudaErrorInvalidValue;
  uint8_t* w = static_cast<uint8_t*>(ws);
  QmvArgs a;
  a.packed = packed;
  a.x = x;
  a.y = y;
  a.tickets = p.workspace ? reinterpret_cast<unsigned*>(w) : nullptr;
  a.slots = p.workspace ? reinterpret_cast<uint32_t*>(w) : nullptr;
  a.part_full = p.workspace ? reinterpret_cast<float*>(w + p.off_full) : nullptr;
  a.part_piece = p.workspace ? reinterpret_cast<float*>(w + p.off_piece) : nullptr;
  a.err = err;
  a.N = N;
  a.K = K;
  a.row_bytes = (K / QK) * block_bytes(t);
  a.packed_bytes = N * a.row_bytes;
  a.tiles = p.tiles;
  a.rows = rows;
  a.x_dtype = x_dtype;
  a.y_dtype = y_dtype;
  a.kb = (int)(K / QK);
  a.bps = p.bps;
  a.slices = p.slices;
  a.aligned = p.aligned;
  a.ns = p.ns;
  a.cb = p.cb;
  a.rowb = p.rowb;
  a.stage = p.stage;
  a.pre = p.pre;
  a.glu = glu ? 1 : 0;
  a.world = 0;
  a.rank = 0;
  a.row0 = 0;
  a.ntot = N;
  for (int i = 0; i < QMV_GATHER_MAX; i++) {
    a.gy[i] = nullptr;
    a.gflags[i] = nullptr;
    a.ginbox[i] = nullptr;
  }
  if (gather && gather->world > 1) {
    if (gather->world > QMV_GATHER_MAX || gather->rank < 0 || gather->rank >= gather->world)
      return cudaErrorInvalidValue;
    a.world = gather->world;
    a.rank = gather->rank;
    a.row0 = gather->row0;
    a.ntot = gather->ntot;
    for (int i = 0; i < gather->world; i++) {
      uint8_t* r = static_cast<uint8_t*>(gather->regions[i]);
      a.gflags[i] = reinterpret_cast<unsigned*>(r);
      a.gy[i] = reinterpret_cast<float*>(r + QMV_GATHER_HEADER);
      a.ginbox[i] = reinterpret_cast<uint2*>(r + qmv_gather_inbox_offset(rows, gather->ntot));
    }
  }
  // Bulk activation copy: one 16-bit row, 16-byte aligned, at most
  // QMV_XSTAGE_G 32-groups per consumer thread.
  a.xbulk = (rows == 1 && p.nb == 1 && (x_dtype == DT_F16 || x_dtype == DT_BF16) &&
             (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && p.bps * (QK / 32) <= QMV_XSTAGE_G * QMV_CTHREADS)
                ? 1
                : 0;
  return qmv_launch(t, a, p, st);
}

}  // namespace gsq
