// Bit-exact fp32 decode of one 8-weight entry of a 256-weight block.
//
// Entry i (0..31) covers block elements 8i .. 8i+7.  Every product and sum is
// an explicit round-to-nearest fp32 operation (__fmul_rn / __fadd_rn /
// __fsub_rn), so nvcc cannot contract them into FMAs; the operation order is
// the one gguf-py 0.19.0 gguf/quants.py uses, which is what the reference's
// tests compare against with assert_array_equal
// (tests/test_metal_decoders.py:21-23).  Byte reads are alignment-agnostic.
#pragma once

#include "gsq_common.cuh"

namespace gsq {

__device__ __forceinline__ float sgn_mul(float v, uint32_t neg) { return neg ? -v : v; }

template <int T> struct Exact;

// gguf-py quants.py:404-428.  Reference Metal: k_decode.py:18-30.
template <> struct Exact<T_Q2_K> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b + 80)), dmin = h2f_bits(rd16u(b + 82));
    const int chunk = i >> 4, plane = (i & 15) >> 2, pos0 = 8 * (i & 3);
    const uint32_t sc = rd8(b + (i >> 1));
    const float dl = __fmul_rn(d, (float)(sc & 15u));
    const float ml = __fmul_rn(dmin, (float)(sc >> 4));
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t q = (rd8(b + 16 + chunk * 32 + pos0 + j) >> (2 * plane)) & 3u;
      o[j] = __fsub_rn(__fmul_rn(dl, (float)q), ml);
    }
  }
};

__device__ __forceinline__ void q4k_scale_min(const uint8_t* s, int g, uint32_t& sc, uint32_t& mn) {
  if (g < 4) {
    sc = rd8(s + g) & 63u;
    mn = rd8(s + 4 + g) & 63u;
  } else {
    const int j = g - 4;
    sc = (rd8(s + 8 + j) & 15u) | ((rd8(s + j) >> 2) & 48u);
    mn = (rd8(s + 8 + j) >> 4) | ((rd8(s + 4 + j) >> 2) & 48u);
  }
}

// gguf-py quants.py:475-522.  Reference Metal: k_decode.py:31-50.
template <> struct Exact<T_Q4_K> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b)), dmin = h2f_bits(rd16u(b + 2));
    const int g = i >> 2, p0 = 8 * (i & 3);
    uint32_t sc, mn;
    q4k_scale_min(b + 4, g, sc, mn);
    const float dl = __fmul_rn(d, (float)sc), dm = __fmul_rn(dmin, (float)mn);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const uint32_t q = (rd8(b + 16 + (g >> 1) * 32 + p0 + j) >> (4 * (g & 1))) & 15u;
      o[j] = __fsub_rn(__fmul_rn(dl, (float)q), dm);
    }
  }
};

// gguf-py quants.py:552-572.  Reference Metal: k_decode.py:51-65.
template <> struct Exact<T_Q6_K> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b + 208));
    const int c = i >> 4, r0 = 8 * (i & 15);
    const int sc = (int)(int8_t)rd8(b + 192 + (i >> 1));
    const float dl = __fmul_rn(d, (float)sc);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int r = r0 + j;
      const uint32_t ql = (rd8(b + c * 64 + (r & 63)) >> (4 * (r >> 6))) & 15u;
      const uint32_t qh = (rd8(b + 128 + c * 32 + (r & 31)) >> (2 * (r >> 5))) & 3u;
      o[j] = __fmul_rn(dl, (float)((int)(ql | (qh << 4)) - 32));
    }
  }
};

// gguf-py quants.py:1351-1377.  Reference Metal: k_decode.py:66-81.
template <> struct Exact<T_IQ4_XS> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const int g = i >> 2, p0 = 8 * (i & 3);
    const uint32_t lo = (rd8(b + 4 + (g >> 1)) >> (4 * (g & 1))) & 15u;
    const uint32_t hi = (rd16u(b + 2) >> (2 * g)) & 3u;
    const int scale = (int)(lo | (hi << 4)) - 32;
    const float dl = __fmul_rn(d, (float)scale);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const int p = p0 + j;
      const uint32_t q = (rd8(b + 8 + 16 * g + (p & 15)) >> (4 * (p >> 4))) & 15u;
      o[j] = __fmul_rn(dl, (float)kKvalues[q]);
    }
  }
};

// gguf-py quants.py:800-828.  Reference Metal: iq_lookup_decode.py:23-26.
template <> struct Exact<T_IQ2_XXS> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const int g = i >> 2, l = i & 3;
    const uint32_t aux = rd32u(b + 2 + 8 * g + 4);
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.25f);
    const uint32_t signs = kKsigns[(aux >> (7 * l)) & 127u];
    const int8_t* row = kGridIQ2XXS + 8 * rd8(b + 2 + 8 * g + l);
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = sgn_mul(__fmul_rn(db, (float)row[j]), (signs >> j) & 1u);
  }
};

// gguf-py quants.py:870-898.  Reference Metal: iq_lookup_decode.py:13-17.
template <> struct Exact<T_IQ2_XS> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const uint32_t q = rd16u(b + 2 + 2 * i);
    const int s = i >> 1;
    const uint32_t sc = (rd8(b + 66 + (s >> 1)) >> (4 * (s & 1))) & 15u;
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)sc)), 0.25f);
    const uint32_t signs = kKsigns[q >> 9];
    const int8_t* row = kGridIQ2XS + 8 * (q & 511u);
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = sgn_mul(__fmul_rn(db, (float)row[j]), (signs >> j) & 1u);
  }
};

// gguf-py quants.py:972-1002.  Reference Metal: iq_lookup_decode.py:18-22.
template <> struct Exact<T_IQ2_S> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const uint32_t hi = (rd8(b + 66 + (i >> 2)) >> (2 * (i & 3))) & 3u;
    const uint32_t idx = rd8(b + 2 + i) | (hi << 8);
    const int s = i >> 1;
    const uint32_t sc = (rd8(b + 74 + (s >> 1)) >> (4 * (s & 1))) & 15u;
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)sc)), 0.25f);
    const uint32_t signs = rd8(b + 34 + i);
    const int8_t* row = kGridIQ2S + 8 * idx;
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = sgn_mul(__fmul_rn(db, (float)row[j]), (signs >> j) & 1u);
  }
};

// gguf-py quants.py:1026-1054.  Reference Metal: iq_lookup_decode.py:7-12.
template <> struct Exact<T_IQ3_XXS> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const int g = i >> 2, l = i & 3;
    const uint32_t aux = rd32u(b + 66 + 4 * g);
    const float db = __fmul_rn(__fmul_rn(d, __fadd_rn(0.5f, (float)(aux >> 28))), 0.5f);
    const uint32_t signs = kKsigns[(aux >> (7 * l)) & 127u];
    const int8_t* r0 = kGridIQ3XXS + 4 * rd8(b + 2 + 2 * i);
    const int8_t* r1 = kGridIQ3XXS + 4 * rd8(b + 2 + 2 * i + 1);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float v = (float)(j < 4 ? r0[j] : r1[j - 4]);
      o[j] = sgn_mul(__fmul_rn(db, v), (signs >> j) & 1u);
    }
  }
};

// gguf-py quants.py:1094-1125.  Reference Metal: iq3_s_decode.py:16-40.
template <> struct Exact<T_IQ3_S> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const int g = i >> 2;
    const uint32_t sc = (rd8(b + 106 + (g >> 1)) >> (4 * (g & 1))) & 15u;
    const float db = __fmul_rn(d, (float)(1u + 2u * sc));
    const int k0 = 2 * i, k1 = 2 * i + 1;
    const uint32_t qh = rd8(b + 66 + (k0 >> 3));
    const uint32_t i0 = rd8(b + 2 + k0) | (((qh >> (k0 & 7)) & 1u) << 8);
    const uint32_t i1 = rd8(b + 2 + k1) | (((qh >> (k1 & 7)) & 1u) << 8);
    const uint32_t signs = rd8(b + 74 + i);
#pragma unroll
    for (int j = 0; j < 8; j++) {
      const float v = (float)(j < 4 ? kGridIQ3S[4 * i0 + j] : kGridIQ3S[4 * i1 + j - 4]);
      o[j] = sgn_mul(__fmul_rn(db, v), (signs >> j) & 1u);
    }
  }
};

// gguf-py quants.py:1265-1288.  Reference Metal: iq_lookup_decode.py:27-30.
template <> struct Exact<T_IQ1_S> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const float d = h2f_bits(rd16u(b));
    const int g = i >> 2, l = i & 3;
    const uint32_t qh = rd16u(b + 34 + 2 * g);
    const float dl = __fmul_rn(d, (float)(2u * ((qh >> 12) & 7u) + 1u));
    const float delta = (qh & 0x8000u) ? -0.125f : 0.125f;
    const uint32_t idx = rd8(b + 2 + 4 * g + l) | (((qh >> (3 * l)) & 7u) << 8);
    const int8_t* row = kGridIQ1S + 8 * idx;
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = __fmul_rn(dl, __fadd_rn((float)row[j], delta));
  }
};

// gguf-py quants.py:1298-1327.  Reference Metal: iq_lookup_decode.py:31-37.
template <> struct Exact<T_IQ1_M> {
  __device__ static void entry(const uint8_t* b, int i, float o[8]) {
    const uint32_t w0 = rd16u(b + 48), w1 = rd16u(b + 50), w2 = rd16u(b + 52), w3 = rd16u(b + 54);
    const uint32_t dbits = ((w0 & 0xF000u) >> 12) | ((w1 & 0xF000u) >> 8) | ((w2 & 0xF000u) >> 4) | (w3 & 0xF000u);
    const float d = h2f_bits(dbits);
    const int s = i >> 1;
    const uint32_t wsel = (s >> 2) == 0 ? w0 : (s >> 2) == 1 ? w1 : (s >> 2) == 2 ? w2 : w3;
    const uint32_t sc = (wsel >> (3 * (s & 3))) & 7u;
    const float dl = __fmul_rn(d, (float)(2u * sc + 1u));
    const uint32_t hn = (rd8(b + 32 + (i >> 1)) >> (4 * (i & 1))) & 15u;
    const uint32_t idx = rd8(b + i) | ((hn & 7u) << 8);
    const float delta = (hn & 8u) ? -0.125f : 0.125f;
    const int8_t* row = kGridIQ1S + 8 * idx;
#pragma unroll
    for (int j = 0; j < 8; j++) o[j] = __fmul_rn(dl, __fadd_rn((float)row[j], delta));
  }
};

}  // namespace gsq
