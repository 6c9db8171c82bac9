// Matvec views of the block formats: what the tensor-core matvec (qmv.cu)
// needs from a packed block, organised by the lanes that need it.
//
// Lane layout.  A warp multiplies 16 weight rows (g and g+8 per lane) of one
// 256-weight block with the activations, mma.m16n8k32 at a time.  Lane
// (g, tq) owns unit slot q = tq / NB and the units u = UPS*S + q,
// S = 0..SETS-1 (UPS = 4 / NB slots): the lanes of a quad hold neighbouring
// units, so that their packed bytes are neighbours in shared memory (no bank
// conflicts between the rows of a warp).  In the MMAs of set S
// the lane supplies entry e = tq % NB + NB*j (j = 0..MMAS-1) of its unit for
// both rows: 8 weights as int8 in two registers (lo, hi), which the MMA
// places at k = 4tq..4tq+3 and 16+4tq..16+4tq+3.  The B operand carries the
// activations of the same positions in the 8 columns (unit slot, activation
// row, level), zero outside the column's unit, so that the accumulator of
// lane (g, tq) ends up holding the integer dot products of its own unit for
// rows g and g+8 (levels hi, lo) -- the epilogue needs no shuffles.
//
// Entry positions in the block: BLOCKED formats use elements UNIT*u + 8e ..
// UNIT*u + 8e + 7 (lo = first four); the identity layout (IQ4_XS) uses
// 32u + 4e .. +3 (lo) and 32u + 16 + 4e .. +3 (hi), one packed word.
//
// Each view provides
//   UNIT, SPLIT (sign-carrying: entries come as magnitudes plus byte masks of
//   the negative positions, the matvec runs a second MMA on the masked
//   magnitudes), UNSIGNED (entries are u8), IDENT, BIAS (per-unit offsets
//   multiplied with activation sums), TAB_BYTES / load_tables (shared memory
//   tables),
//   Row<NB>: per (block, row) values the lane decodes once,
//   row<NB>(b, q), entry<S>(b, r, u, e, tab, lo, hi, mlo, mhi),
//   unit<S>(b, r, u, C, N, xs, xsum, A, M): accumulate the unit's dot
//   products (C = 256*C_hi + C_lo; N the same for the masked MMA) into the
//   block accumulators A (scaled) and M (bias),
//   finish(b, r, A, M): the block's contribution to the row sum.
// The generic view adapts the per-entry decoders of gsq_fast.cuh; formats
// with a specialised view decode and scale with fewer instructions.
//
// LANE_UNITS selects this lane layout in the matvec.  Formats without it use
// the per-entry layout (the lanes of a quad feed consecutive entries of one
// 32-weight chunk, and a select keeps each column's activations to one MMA
// per set), which measured faster for them: their per-entry decoders read
// neighbouring bytes across a quad, and one activation load per set costs
// fewer shared-memory wavefronts than one per MMA.
#pragma once

#include "gsq_fast.cuh"

namespace gsq {

template <int T> struct MvLaneUnits { static constexpr bool value = false; };
template <> struct MvLaneUnits<T_IQ4_XS> { static constexpr bool value = true; };

template <int T>
struct Mv {
  using F = Fast<T>;
  using MD = MvDecode<T>;
  static constexpr bool LANE_UNITS = MvLaneUnits<T>::value;
  static constexpr int UNIT = F::UNIT;
  static constexpr bool SPLIT = MD::SPLIT, UNSIGNED = MD::UNSIGNED, IDENT = !F::BLOCKED, BIAS = F::HAS_BIAS;
  static constexpr int TAB_BYTES = MD::TAB_BYTES;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { MD::load_tables(tab, tid, nthr); }
  template <int NB> struct Row {};
  template <int NB> __device__ static Row<NB> row(const uint8_t*, int) { return {}; }
  template <int S, int NB>
  __device__ static void entry(const uint8_t* b, const Row<NB>&, int u, int e, const uint8_t* tab, uint32_t& lo,
                               uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    int c32, t;
    if constexpr (IDENT) {
      c32 = u;
      t = e;
    } else {
      const int el = UNIT * u + 8 * e;
      c32 = el >> 5;
      t = (el & 31) >> 3;
    }
    if constexpr (SPLIT) F::entry_split(b, c32, t, tab, lo, hi, mlo, mhi);
    else {
      MD::entry(b, c32, t, tab, lo, hi);
      mlo = mhi = 0u;
    }
  }
  template <int S, int NB>
  __device__ static void unit(const uint8_t* b, const Row<NB>&, int u, int C, int N, float xs, float xsum, float& A,
                              float& M) {
    int k, m;
    F::kscale(b, u, k, m);
    const int c = SPLIT ? C - 2 * N : C;
    if constexpr (F::KINT) A = fmaf(xs, (float)(k * c), A);
    else A = fmaf(xs * (float)k, (float)c, A);
    if constexpr (BIAS) M = fmaf((float)m, xsum, M);
  }
  template <int NB>
  __device__ static float finish(const uint8_t* b, const Row<NB>&, float A, float M) {
    float D, DM;
    F::dscale(b, D, DM);
    return BIAS ? fmaf(D, A, DM * M) : D * A;
  }
};

// IQ2_XXS: units of 32 weights, 8 bytes each at 2 + 8u: four grid indices
// (one per entry of 8 weights) and a word of four 7-bit sign indices plus
// the 4-bit scale s: w = d * (0.5 + s) / 4 * grid * sign = d/8 * (2s + 1) * ...
template <>
struct Mv<T_IQ2_XXS> {
  static constexpr int UNIT = 32, GRID = 256 * 8;
  static constexpr bool LANE_UNITS = true, SPLIT = true, UNSIGNED = false, IDENT = false, BIAS = false;
  static constexpr int TAB_BYTES = GRID;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ2XXS, GRID, tid, nthr); }
  template <int NB> struct Row {
    uint32_t grid[2 * NB], aux[2 * NB];
  };
  template <int NB> __device__ static Row<NB> row(const uint8_t* b, int q) {
    Row<NB> r;
#pragma unroll
    for (int S = 0; S < 2 * NB; S++) {
      const uint8_t* p = b + 2 + 8 * ((4 / NB) * S + q);
      r.grid[S] = ld32a2(p);
      r.aux[S] = ld32a2(p + 4);
    }
    return r;
  }
  template <int S, int NB>
  __device__ static void entry(const uint8_t*, const Row<NB>& r, int, int e, const uint8_t* tab, uint32_t& lo,
                               uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    const uint2 g = lds64(tab + 8 * ((r.grid[S] >> (8 * e)) & 255u));
    lo = g.x; hi = g.y;
    ksign_masks((r.aux[S] >> (7 * e)) & 127u, mlo, mhi);
  }
  template <int S, int NB>
  __device__ static void unit(const uint8_t*, const Row<NB>& r, int, int C, int N, float xs, float, float& A, float&) {
    const int k = 2 * (int)(r.aux[S] >> 28) + 1;  // |C - 2N| * k < 32 * 43 * 2^15 * 31 < 2^31
    A = fmaf(xs, (float)(k * (C - 2 * N)), A);
  }
  template <int NB>
  __device__ static float finish(const uint8_t* b, const Row<NB>&, float A, float) {
    return h2f_bits(ld16a2(b)) * 0.125f * A;
  }
};

}  // namespace gsq
