// Integer-entry decoders for the tensor-core matvec.
//
// Every supported format can be written, per sub-block ("unit") of 16 or 32
// weights, as   w_k = S_u * a_k + B_u   with a_k a small integer that fits in
// int8 and S_u, B_u fp32 per-unit constants:
//
//   Q2_K   (unit 16)  a = q in [0,3]          S = d*(sc&15)      B = -dmin*(sc>>4)
//   Q4_K   (unit 32)  a = q in [0,15]         S = d*sc           B = -dmin*m
//   Q6_K   (unit 16)  a = q in [0,63]         S = d*scale        B = -32*S
//   IQ4_XS (unit 32)  a = kvalues[q]          S = d*(scale-32)   B = 0
//   IQ2_*  (unit 32/16) a = +-grid            S = d*(0.5+s)/4    B = 0
//   IQ3_XXS (unit 32) a = +-grid              S = d*(0.5+s)/2    B = 0
//   IQ3_S  (unit 32)  a = +-grid              S = d*(1+2s)       B = 0
//   IQ1_S/M           a = 8*grid +- 1         S = d*(2s+1)/8     B = 0
//
// (derived from the block layouts that gguf-py 0.19.0 quants.py dequantizes;
// the reference's fused kernels apply the same decode per weight in fp32,
// mlx_gsq/runtime/kernels/qmv.py:76-528).  The matvec multiplies the a_k with
// int8 activations on the tensor cores and applies S_u, B_u once per unit.
//
// Entry layout.  For a 32-weight MMA chunk c32 (0..7) of a block and a thread
// quad index tq (0..3), entry() returns the 8 int8 values that thread feeds to
// mma.m16n8k32: `lo` holds MMA k = 4tq..4tq+3 and `hi` holds 16+4tq..16+4tq+3.
// BLOCKED formats map them to block elements 32*c32 + 8tq .. +7 (one grid
// entry); the identity mapping (IQ4_XS) uses 32*c32 + 4tq.. and +16+4tq...
// The activation operand is laid out with the same mapping.
//
// Sign-carrying IQ types (SPLIT = true) also expose entry_split(): the
// unsigned grid magnitudes and the byte mask of the negative positions, so
// the matvec computes sum x*(+-g) = sum x*g - 2*sum x*(g & mask) with two
// integer MMAs instead of negating bytes.  Sign masks are expanded from the
// 8 sign bits in registers (multiply to spread, prmt to sign-replicate).
//
// Blocks live in shared memory at the byte alignment the packed stream gives
// them: every block start is 2-byte aligned; blocks of 56/84/136/144 bytes are
// 4/8/16-byte aligned.  The readers below use the widest access that the
// format's guaranteed alignment allows.
#pragma once

#include "gsq_common.cuh"

namespace gsq {

// Negate the bytes of (lo, hi) selected by the mask.  Magnitudes are >= 1, so
// (v ^ 0xFF) + 1 == -v never carries into the neighbouring byte.
__device__ __forceinline__ void apply_sign(uint32_t& lo, uint32_t& hi, uint2 m) {
  lo = (lo ^ m.x) + (m.x & 0x01010101u);
  hi = (hi ^ m.y) + (m.y & 0x01010101u);
}

__device__ __forceinline__ uint2 lds64(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }

// Byte masks for 4 sign bits (s4 in [0,15]): byte j = 0xFF if bit j is set.
// The multiply moves bit j to bit 8j+7 (no carries between the four terms);
// prmt's sign-replicate mode (selector nibbles 8..B) spreads each byte's msb.
__device__ __forceinline__ uint32_t byte_mask4(uint32_t s4) {
  const uint32_t t = s4 * 0x10204080u;
  uint32_t m;
  asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(m) : "r"(t));
  return m;
}

// The IQ2/IQ3 sign byte of a 7-bit sign index: bit 7 is the parity of the
// seven stored bits, so that every 8-sign group has an even count of minus
// signs (equal to gguf-py's ksigns table, entry for entry).
__device__ __forceinline__ uint32_t ksign(uint32_t i7) { return i7 | ((__popc(i7) & 1u) << 7); }

__device__ __forceinline__ void sign_masks(uint32_t s8, uint32_t& mlo, uint32_t& mhi) {
  mlo = byte_mask4(s8 & 15u);
  mhi = byte_mask4((s8 >> 4) & 15u);
}

// sign_masks(ksign(i7)) straight from the 7-bit index: i7 times
// sum_{m<7} 2^(7m+7) puts bit j of i7 on bit 8j+7, the sign bit of byte j
// (the partial products sit on distinct bits, since j + 7m differs for every
// j, m < 7, so nothing carries); bit 63 is free and takes the parity.  One
// wide multiply on the FMA pipe replaces the two 4-bit multiplies and the
// shifts and masks of the separate sign byte.
__device__ __forceinline__ void ksign_masks(uint32_t i7, uint32_t& mlo, uint32_t& mhi) {
  const uint64_t t = (uint64_t)i7 * 0x0002040810204080ull;
  const uint32_t hi = (uint32_t)(t >> 32) | ((uint32_t)__popc(i7) << 31);
  asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(mlo) : "r"((uint32_t)t));
  asm("prmt.b32 %0, %1, 0, 0xBA98;" : "=r"(mhi) : "r"(hi));
}
__device__ __forceinline__ uint32_t lds32(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

template <int T> struct Fast;

// Derived lookup tables, generated at build time from the gguf-py codebooks.
// kIq1Dual: IQ1 grid x 8 with the +1/8 delta folded in (first 2048 entries)
//           and with -1/8 (next 2048 entries).
static __device__ __align__(16) const int8_t kIq1Dual[2 * 2048 * 8] = GSQ_INIT_IQ1_DUAL;

// Copy a 16-byte aligned table into shared memory with 16-byte accesses.
__device__ __forceinline__ void copy16(uint8_t* dst, const void* src, int bytes, int tid, int nthr) {
  const uint4* s = reinterpret_cast<const uint4*>(src);
  uint4* d = reinterpret_cast<uint4*>(dst);
  for (int i = tid; i < bytes / 16; i += nthr) d[i] = s[i];
}

// --- K-quants ----------------------------------------------------------------

template <> struct Fast<T_Q2_K> {
  static constexpr int UNIT = 16, TAB_BYTES = 0;
  static constexpr bool BLOCKED = true, HAS_BIAS = true, SPLIT = false;
  __device__ static void load_tables(uint8_t*, int, int) {}
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t*, uint32_t& lo, uint32_t& hi) {
    const int i = 4 * c32 + tq;
    const int chunk = i >> 4, plane = (i & 15) >> 2;
    const uint2 w = ld64a4(b + 16 + chunk * 32 + 8 * (i & 3));
    lo = (w.x >> (2 * plane)) & 0x03030303u;
    hi = (w.y >> (2 * plane)) & 0x03030303u;
  }
  __device__ static void affine(const uint8_t* b, int u, float& S, float& B) {
    const uint32_t sc = b[u];
    S = h2f_bits(ld16a2(b + 80)) * (float)(sc & 15u);
    B = -h2f_bits(ld16a2(b + 82)) * (float)(sc >> 4);
  }
  // Integer unit scale k and min m: S_u = D * k, B_u = DM * m (kscale, dscale);
  // KINT: k times any dot product the matvec forms fits int32 (entries <= 192
  // as fed: 16 * 192 * 2^15 * 15 < 2^31).
  static constexpr bool KINT = true;
  __device__ static void kscale(const uint8_t* b, int u, int& k, int& m) {
    const uint32_t sc = b[u];
    k = (int)(sc & 15u);
    m = (int)(sc >> 4);
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b + 80));
    DM = -h2f_bits(ld16a2(b + 82));
  }
};

template <> struct Fast<T_Q4_K> {
  static constexpr int UNIT = 32, TAB_BYTES = 0;
  static constexpr bool BLOCKED = true, HAS_BIAS = true, SPLIT = false;
  __device__ static void load_tables(uint8_t*, int, int) {}
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t*, uint32_t& lo, uint32_t& hi) {
    const uint2 w = ld64a8(b + 16 + (c32 >> 1) * 32 + 8 * tq);
    const int sh = 4 * (c32 & 1);
    lo = (w.x >> sh) & 0x0F0F0F0Fu;
    hi = (w.y >> sh) & 0x0F0F0F0Fu;
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    // 6-bit scale/min of group g from the 12 packed bytes (branch-free):
    // g < 4: low 6 bits of bytes g, 4+g; g >= 4: nibbles of byte 8+j plus the
    // top 2 bits of bytes j, 4+j (j = g-4).  Q4_K blocks are 16-byte aligned,
    // so the header is read as four words that every call on the same block
    // shares.
    const uint32_t dm = ld32a4(b), q0 = ld32a4(b + 4), q1 = ld32a4(b + 8), q2 = ld32a4(b + 12);
    const int sh = 8 * (g & 3);
    const bool hi = g >= 4;
    const uint32_t sc = hi ? ((q2 >> sh) & 15u) | ((q0 >> (sh + 2)) & 48u) : (q0 >> sh) & 63u;
    const uint32_t mn = hi ? ((q2 >> (sh + 4)) & 15u) | ((q1 >> (sh + 2)) & 48u) : (q1 >> sh) & 63u;
    S = h2f_bits(dm & 0xFFFFu) * (float)sc;
    B = -h2f_bits(dm >> 16) * (float)mn;
  }
  static constexpr bool KINT = false;  // 32 * 240 * 2^15 * 63 > 2^31
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    const uint32_t q0 = ld32a4(b + 4), q1 = ld32a4(b + 8), q2 = ld32a4(b + 12);
    const int sh = 8 * (g & 3);
    const bool hi = g >= 4;
    k = (int)(hi ? ((q2 >> sh) & 15u) | ((q0 >> (sh + 2)) & 48u) : (q0 >> sh) & 63u);
    m = (int)(hi ? ((q2 >> (sh + 4)) & 15u) | ((q1 >> (sh + 2)) & 48u) : (q1 >> sh) & 63u);
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    const uint32_t dm = ld32a4(b);
    D = h2f_bits(dm & 0xFFFFu);
    DM = -h2f_bits(dm >> 16);
  }
};

template <> struct Fast<T_Q6_K> {
  static constexpr int UNIT = 16, TAB_BYTES = 0;
  static constexpr bool BLOCKED = true, HAS_BIAS = true, SPLIT = false;
  __device__ static void load_tables(uint8_t*, int, int) {}
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t*, uint32_t& lo, uint32_t& hi) {
    const int i = 4 * c32 + tq;
    const int c = i >> 4, r0 = 8 * (i & 15);
    const uint2 ql = ld64a2(b + c * 64 + (r0 & 63));
    const uint2 qh = ld64a2(b + 128 + c * 32 + (r0 & 31));
    const int s1 = 4 * (r0 >> 6), s2 = 2 * (r0 >> 5 & 3);
    lo = ((ql.x >> s1) & 0x0F0F0F0Fu) | (((qh.x >> s2) & 0x03030303u) << 4);
    hi = ((ql.y >> s1) & 0x0F0F0F0Fu) | (((qh.y >> s2) & 0x03030303u) << 4);
  }
  __device__ static void affine(const uint8_t* b, int u, float& S, float& B) {
    S = h2f_bits(ld16a2(b + 208)) * (float)(int8_t)b[192 + u];
    B = -32.0f * S;
  }
  static constexpr bool KINT = false;  // 16 * 63 * 2^15 * 128 > 2^31
  __device__ static void kscale(const uint8_t* b, int u, int& k, int& m) {
    k = (int)(int8_t)b[192 + u];
    m = k;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b + 208));
    DM = -32.0f * D;
  }
};

// 16-entry int8 table lookup of the four nibbles in the low 16 bits of `sel`,
// using byte permutes over the table held in four registers.
__device__ __forceinline__ uint32_t lut16(uint32_t sel, uint32_t t0, uint32_t t1, uint32_t t2, uint32_t t3) {
  const uint32_t lowp = __byte_perm(t0, t1, sel & 0x7777u);
  const uint32_t highp = __byte_perm(t2, t3, sel & 0x7777u);
  const uint32_t pick = 0x3210u | ((sel >> 1) & 0x4444u);
  return __byte_perm(lowp, highp, pick);
}

template <> struct Fast<T_IQ4_XS> {
  static constexpr int UNIT = 32, TAB_BYTES = 16;
  static constexpr bool BLOCKED = false, HAS_BIAS = false, SPLIT = false;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) {
    copy16(tab, kKvalues, 16, tid, nthr);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const uint4 kv = *reinterpret_cast<const uint4*>(tab);
    const uint32_t w = ld32a4(b + 8 + 16 * c32 + 4 * tq);
    // nibble order in w: lo0 hi0 lo1 hi1 lo2 hi2 lo3 hi3
    const uint32_t r01 = lut16(w, kv.x, kv.y, kv.z, kv.w);
    const uint32_t r23 = lut16(w >> 16, kv.x, kv.y, kv.z, kv.w);
    lo = __byte_perm(r01, r23, 0x6420u);
    hi = __byte_perm(r01, r23, 0x7531u);
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    const uint32_t l = (b[4 + (g >> 1)] >> (4 * (g & 1))) & 15u;
    const uint32_t h = (ld16a2(b + 2) >> (2 * g)) & 3u;
    S = h2f_bits(ld16a2(b)) * (float)((int)(l | (h << 4)) - 32);
    B = 0.f;
  }
  static constexpr bool KINT = false;  // 32 * 127 * 2^15 * 32 > 2^31
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    const uint32_t l = (b[4 + (g >> 1)] >> (4 * (g & 1))) & 15u;
    const uint32_t h = (ld16a2(b + 2) >> (2 * g)) & 3u;
    k = (int)(l | (h << 4)) - 32;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b));
    DM = 0.f;
  }
};

// --- IQ lookup types ------------------------------------------------------------

template <> struct Fast<T_IQ2_XXS> {
  static constexpr int UNIT = 32, GRID = 256 * 8, TAB_BYTES = GRID;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = true;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ2XXS, GRID, tid, nthr); }
  __device__ static void entry_split(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo,
                                     uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    const uint8_t* q = b + 2 + 8 * c32;
    const uint32_t aux = ld32a2(q + 4);
    const uint2 g = lds64(tab + 8 * q[tq]);
    lo = g.x; hi = g.y;
    ksign_masks((aux >> (7 * tq)) & 127u, mlo, mhi);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    uint32_t mlo, mhi;
    entry_split(b, c32, tq, tab, lo, hi, mlo, mhi);
    apply_sign(lo, hi, make_uint2(mlo, mhi));
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    const uint32_t aux = ld32a2(b + 2 + 8 * g + 4);
    S = h2f_bits(ld16a2(b)) * (0.5f + (float)(aux >> 28)) * 0.25f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 32 * 43 * 2^15 * 31 < 2^31
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    k = 2 * (int)(ld32a2(b + 2 + 8 * g + 4) >> 28) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b)) * 0.125f;
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ2_XS> {
  static constexpr int UNIT = 16, GRID = 512 * 8, TAB_BYTES = GRID;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = true;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ2XS, GRID, tid, nthr); }
  __device__ static void entry_split(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo,
                                     uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    // The matvec's split form keeps the separate sign byte: with the wide
    // multiply of ksign_masks it measured 1 % slower (its FMA pipe is already
    // busy with the grid addressing), while the signed form below gains.
    const uint32_t q = ld16a2(b + 2 + 2 * (4 * c32 + tq));
    const uint2 g = lds64(tab + 8 * (q & 511u));
    lo = g.x; hi = g.y;
    sign_masks(ksign(q >> 9), mlo, mhi);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const uint32_t q = ld16a2(b + 2 + 2 * (4 * c32 + tq));
    const uint2 g = lds64(tab + 8 * (q & 511u));
    uint32_t mlo, mhi;
    ksign_masks(q >> 9, mlo, mhi);
    lo = g.x; hi = g.y;
    apply_sign(lo, hi, make_uint2(mlo, mhi));
  }
  __device__ static void affine(const uint8_t* b, int s, float& S, float& B) {
    const uint32_t sc = (b[66 + (s >> 1)] >> (4 * (s & 1))) & 15u;
    S = h2f_bits(ld16a2(b)) * (0.5f + (float)sc) * 0.25f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 16 * 43 * 2^15 * 31 < 2^31
  __device__ static void kscale(const uint8_t* b, int s, int& k, int& m) {
    k = 2 * (int)((b[66 + (s >> 1)] >> (4 * (s & 1))) & 15u) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b)) * 0.125f;
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ2_S> {
  static constexpr int UNIT = 16, GRID = 1024 * 8, TAB_BYTES = GRID;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = true;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ2S, GRID, tid, nthr); }
  __device__ static void entry_split(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo,
                                     uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    const int i = 4 * c32 + tq;
    const uint32_t h = (b[66 + (i >> 2)] >> (2 * (i & 3))) & 3u;
    const uint2 g = lds64(tab + 8 * (b[2 + i] | (h << 8)));
    lo = g.x; hi = g.y;
    sign_masks(b[34 + i], mlo, mhi);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    uint32_t mlo, mhi;
    entry_split(b, c32, tq, tab, lo, hi, mlo, mhi);
    apply_sign(lo, hi, make_uint2(mlo, mhi));
  }
  __device__ static void affine(const uint8_t* b, int s, float& S, float& B) {
    const uint32_t sc = (b[74 + (s >> 1)] >> (4 * (s & 1))) & 15u;
    S = h2f_bits(ld16a2(b)) * (0.5f + (float)sc) * 0.25f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 16 * 43 * 2^15 * 31 < 2^31
  __device__ static void kscale(const uint8_t* b, int s, int& k, int& m) {
    k = 2 * (int)((b[74 + (s >> 1)] >> (4 * (s & 1))) & 15u) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b)) * 0.125f;
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ3_XXS> {
  static constexpr int UNIT = 32, GRID = 256 * 4, TAB_BYTES = GRID;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = true;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ3XXS, GRID, tid, nthr); }
  __device__ static void entry_split(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo,
                                     uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    const uint32_t idx = ld16a2(b + 2 + 8 * c32 + 2 * tq);
    const uint32_t aux = ld32a2(b + 66 + 4 * c32);
    lo = lds32(tab + 4 * (idx & 255u));
    hi = lds32(tab + 4 * (idx >> 8));
    ksign_masks((aux >> (7 * tq)) & 127u, mlo, mhi);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    uint32_t mlo, mhi;
    entry_split(b, c32, tq, tab, lo, hi, mlo, mhi);
    apply_sign(lo, hi, make_uint2(mlo, mhi));
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    const uint32_t aux = ld32a2(b + 66 + 4 * g);
    S = h2f_bits(ld16a2(b)) * (0.5f + (float)(aux >> 28)) * 0.5f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 32 * 62 * 2^15 * 31 < 2^31 (grid values <= 62)
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    k = 2 * (int)(ld32a2(b + 66 + 4 * g) >> 28) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b)) * 0.25f;
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ3_S> {
  static constexpr int UNIT = 32, GRID = 512 * 4, TAB_BYTES = GRID;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = true;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kGridIQ3S, GRID, tid, nthr); }
  __device__ static void entry_split(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo,
                                     uint32_t& hi, uint32_t& mlo, uint32_t& mhi) {
    const uint32_t idx = ld16a2(b + 2 + 8 * c32 + 2 * tq);
    const uint32_t qh = b[66 + c32] >> (2 * tq);
    lo = lds32(tab + 4 * ((idx & 255u) | ((qh & 1u) << 8)));
    hi = lds32(tab + 4 * ((idx >> 8) | ((qh & 2u) << 7)));
    sign_masks(b[74 + 4 * c32 + tq], mlo, mhi);
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    uint32_t mlo, mhi;
    entry_split(b, c32, tq, tab, lo, hi, mlo, mhi);
    apply_sign(lo, hi, make_uint2(mlo, mhi));
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    const uint32_t sc = (b[106 + (g >> 1)] >> (4 * (g & 1))) & 15u;
    S = h2f_bits(ld16a2(b)) * (float)(1u + 2u * sc);
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 32 * 15 * 2^15 * 31 < 2^31
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    k = 1 + 2 * (int)((b[106 + (g >> 1)] >> (4 * (g & 1))) & 15u);
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b));
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ1_S> {
  static constexpr int UNIT = 32, TAB_BYTES = 2 * 2048 * 8;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = false;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kIq1Dual, TAB_BYTES, tid, nthr); }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const uint32_t qh = ld16a2(b + 34 + 2 * c32);
    const uint32_t idx = b[2 + 4 * c32 + tq] | (((qh >> (3 * tq)) & 7u) << 8) | ((qh >> 15) << 11);
    const uint2 g = lds64(tab + 8 * idx);
    lo = g.x; hi = g.y;
  }
  __device__ static void affine(const uint8_t* b, int g, float& S, float& B) {
    const uint32_t qh = ld16a2(b + 34 + 2 * g);
    S = h2f_bits(ld16a2(b)) * (float)(2u * ((qh >> 12) & 7u) + 1u) * 0.125f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 32 * 9 * 2^15 * 15 < 2^31
  __device__ static void kscale(const uint8_t* b, int g, int& k, int& m) {
    k = 2 * (int)((ld16a2(b + 34 + 2 * g) >> 12) & 7u) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    D = h2f_bits(ld16a2(b)) * 0.125f;
    DM = 0.f;
  }
};

template <> struct Fast<T_IQ1_M> {
  static constexpr int UNIT = 16, TAB_BYTES = 2 * 2048 * 8;
  static constexpr bool BLOCKED = true, HAS_BIAS = false, SPLIT = false;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kIq1Dual, TAB_BYTES, tid, nthr); }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const int i = 4 * c32 + tq;
    const uint32_t hn = (b[32 + (i >> 1)] >> (4 * (i & 1))) & 15u;
    const uint2 g = lds64(tab + 8 * (b[i] | (hn << 8)));  // bit 3 of hn selects the -1/8 half
    lo = g.x; hi = g.y;
  }
  __device__ static void affine(const uint8_t* b, int s, float& S, float& B) {
    const uint2 w = ld64a8(b + 48);
    const uint32_t w0 = w.x & 0xFFFFu, w1 = w.x >> 16, w2 = w.y & 0xFFFFu, w3 = w.y >> 16;
    const uint32_t dbits = ((w0 & 0xF000u) >> 12) | ((w1 & 0xF000u) >> 8) | ((w2 & 0xF000u) >> 4) | (w3 & 0xF000u);
    const uint32_t ws = (s >> 2) == 0 ? w0 : (s >> 2) == 1 ? w1 : (s >> 2) == 2 ? w2 : w3;
    const uint32_t sc = (ws >> (3 * (s & 3))) & 7u;
    S = h2f_bits(dbits) * (float)(2u * sc + 1u) * 0.125f;
    B = 0.f;
  }
  static constexpr bool KINT = true;  // 16 * 9 * 2^15 * 15 < 2^31
  __device__ static void kscale(const uint8_t* b, int s, int& k, int& m) {
    const uint32_t ws = ld16a2(b + 48 + 2 * (s >> 2));
    k = 2 * (int)((ws >> (3 * (s & 3))) & 7u) + 1;
    m = 0;
  }
  __device__ static void dscale(const uint8_t* b, float& D, float& DM) {
    const uint2 w = ld64a8(b + 48);
    const uint32_t w0 = w.x & 0xFFFFu, w1 = w.x >> 16, w2 = w.y & 0xFFFFu, w3 = w.y >> 16;
    const uint32_t dbits = ((w0 & 0xF000u) >> 12) | ((w1 & 0xF000u) >> 8) | ((w2 & 0xF000u) >> 4) | (w3 & 0xF000u);
    D = h2f_bits(dbits) * 0.125f;
    DM = 0.f;
  }
};

// Matvec-only variants of the integer entries.  Where an entry read in place
// (a nibble or 2-bit plane masked but not shifted) is the true entry times a
// power of two, the matvec feeds it unshifted to the u8 x s8 tensor-core MMA
// and folds the power of two into the scale of that 32-wide activation group
// (xgroup_scale(g), g = group index along K).  Entries stay below 256.
//
// IQ3_XXS reads its entries from a pre-signed table (grid word x 4-bit sign
// group, 16 KB, gen_tables.py) instead of expanding sign masks: the same
// number of shared loads, no mask arithmetic and no second (masked) MMA.
// (The same scheme for IQ3_S and IQ2_XXS needs 32 KB tables; the shared
// memory they take from the stage ring costs more than the masks save.)
template <int T>
struct MvDecode {
  static constexpr bool UNSIGNED = false;
  static constexpr bool NIBBLE_ORDER = false;  // activations of a 32-group in natural order
  static constexpr bool SPLIT = Fast<T>::SPLIT;
  static constexpr int TAB_BYTES = Fast<T>::TAB_BYTES;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { Fast<T>::load_tables(tab, tid, nthr); }
  __device__ static float xgroup_scale(int) { return 1.f; }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    Fast<T>::entry(b, c32, tq, tab, lo, hi);
  }
};

static __device__ __align__(16) const int8_t kIq3xxsSigned[256 * 16 * 4] = GSQ_INIT_IQ3XXS_SIGNED;

// IQ4_XS: the matvec stores the activations of every 32-group in the
// order of the packed word's nibbles (byte 4tq + i of the group holds
// element 4tq + i/2 (i even) or 16 + 4tq + i/2 (i odd), and byte 16 + 4tq + i
// element 4tq + 2 + i/2 or 18 + 4tq + i/2), so the two lookups of a word
// feed the MMA as they come and the two byte permutes that restore element
// order (Fast<T_IQ4_XS>::entry) go away.  The MMA's sum is the same in any
// k order that weights and activations share.
template <>
struct MvDecode<T_IQ4_XS> {
  static constexpr bool UNSIGNED = false, SPLIT = false, NIBBLE_ORDER = true;
  static constexpr int TAB_BYTES = Fast<T_IQ4_XS>::TAB_BYTES;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { Fast<T_IQ4_XS>::load_tables(tab, tid, nthr); }
  __device__ static float xgroup_scale(int) { return 1.f; }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const uint4 kv = *reinterpret_cast<const uint4*>(tab);
    const uint32_t w = ld32a4(b + 8 + 16 * c32 + 4 * tq);
    lo = lut16(w, kv.x, kv.y, kv.z, kv.w);          // elements 4tq, 16+4tq, 4tq+1, 17+4tq
    hi = lut16(w >> 16, kv.x, kv.y, kv.z, kv.w);    // elements 4tq+2, 18+4tq, 4tq+3, 19+4tq
  }
};

template <>
struct MvDecode<T_IQ3_XXS> {
  static constexpr bool UNSIGNED = false, SPLIT = false, NIBBLE_ORDER = false;
  static constexpr int TAB_BYTES = 256 * 16 * 4;
  __device__ static void load_tables(uint8_t* tab, int tid, int nthr) { copy16(tab, kIq3xxsSigned, TAB_BYTES, tid, nthr); }
  __device__ static float xgroup_scale(int) { return 1.f; }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t* tab, uint32_t& lo, uint32_t& hi) {
    const uint32_t idx = ld16a2(b + 2 + 8 * c32 + 2 * tq);
    const uint32_t s8 = ksign((ld32a2(b + 66 + 4 * c32) >> (7 * tq)) & 127u);
    lo = lds32(tab + 4 * (((idx & 255u) << 4) | (s8 & 15u)));
    hi = lds32(tab + 4 * (((idx >> 8) << 4) | (s8 >> 4)));
  }
};

template <>
struct MvDecode<T_Q4_K> {  // odd 32-groups are the high nibbles: 16 q <= 240
  static constexpr bool UNSIGNED = true, SPLIT = false, NIBBLE_ORDER = false;
  static constexpr int TAB_BYTES = 0;
  __device__ static void load_tables(uint8_t*, int, int) {}
  __device__ static float xgroup_scale(int g) { return (g & 1) ? 0.0625f : 1.f; }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t*, uint32_t& lo, uint32_t& hi) {
    const uint2 w = ld64a8(b + 16 + (c32 >> 1) * 32 + 8 * tq);
    const uint32_t m = (c32 & 1) ? 0xF0F0F0F0u : 0x0F0F0F0Fu;
    lo = w.x & m;
    hi = w.y & m;
  }
};

template <>
struct MvDecode<T_Q2_K> {  // 32-group g reads bit plane g & 3: 4^p q <= 192
  static constexpr bool UNSIGNED = true, SPLIT = false, NIBBLE_ORDER = false;
  static constexpr int TAB_BYTES = 0;
  __device__ static void load_tables(uint8_t*, int, int) {}
  __device__ static float xgroup_scale(int g) {
    return (g & 3) == 0 ? 1.f : (g & 3) == 1 ? 0.25f : (g & 3) == 2 ? 0.0625f : 0.015625f;
  }
  __device__ static void entry(const uint8_t* b, int c32, int tq, const uint8_t*, uint32_t& lo, uint32_t& hi) {
    const uint2 w = ld64a4(b + 16 + (c32 >> 2) * 32 + 8 * tq);
    const uint32_t m = 0x03030303u << (2 * (c32 & 3));
    lo = w.x & m;
    hi = w.y & m;
  }
};

}  // namespace gsq
