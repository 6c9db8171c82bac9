/*
 * CPU oracle for the packed-GGUF hot path.  TEST INFRASTRUCTURE ONLY: the
 * product never links, loads or calls this file; tests, smoke() and the
 * bench's CPU-baseline leg use it as the checker.
 *
 * What it restates.  The reference's trusted decoder is
 * mlx_gsq/quant/reference.py:10-18 (dequantize_reference), which calls the
 * third-party gguf-py package (pinned here: gguf 0.19.0, not vendored in the
 * reference, pyproject.toml:13 says gguf>=0.17).  Each function below follows
 * the float32 operation order of gguf-py 0.19.0 gguf/quants.py so that the
 * result is bit-identical: every product and sum is rounded to float32 on its
 * own (build with -ffp-contract=off, no fast-math).  The matvec/matmul follow
 * the reference tests' expected value x @ deq.T (tests/test_all_qmv.py:22,
 * tests/test_all_qmm.py:34-35), accumulated here in double.
 *
 * Tables (grids, ksigns, kvalues) are passed in by the caller, which takes
 * them from gguf-py exactly as mlx_gsq/runtime/kernels/iq_lookup_decode.py:46-53
 * does.
 */
#include <stdint.h>
#include <string.h>
#include <math.h>

#define QK 256

static float h2f(uint16_t h) {
    /* IEEE binary16 -> binary32, exact for every input (incl. subnormal/inf/nan). */
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1fu;
    uint32_t man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {
            int e = -1;
            do { e++; man <<= 1; } while (!(man & 0x400u));
            man &= 0x3ffu;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 0x1f) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

static uint16_t rd16(const uint8_t* p) { return (uint16_t)(p[0] | (p[1] << 8)); }
static uint32_t rd32(const uint8_t* p) {
    return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

/* gguf-py quants.py:404-428 (Q2_K): dl*q - ml with dl = d*(sc&15), ml = dmin*(sc>>4). */
static void deq_q2_k(const uint8_t* b, float* o) {
    float d = h2f(rd16(b + 80)), dmin = h2f(rd16(b + 82));
    for (int e = 0; e < QK; e++) {
        int chunk = e / 128, plane = (e % 128) / 32, pos = e % 32;
        uint32_t q = (b[16 + chunk * 32 + pos] >> (2 * plane)) & 3u;
        uint8_t sc = b[e / 16];
        float dl = d * (float)(sc & 15);
        float ml = dmin * (float)(sc >> 4);
        float t = dl * (float)q;
        o[e] = t - ml;
    }
}

/* gguf-py quants.py:475-522 (Q4_K, get_scale_min). */
static void q4k_scale_min(const uint8_t* s, int g, uint32_t* sc, uint32_t* mn) {
    if (g < 4) {
        *sc = s[g] & 63u;
        *mn = s[4 + g] & 63u;
    } else {
        int j = g - 4;
        *sc = (s[8 + j] & 15u) | ((s[j] >> 2) & 48u);
        *mn = (s[8 + j] >> 4) | ((s[4 + j] >> 2) & 48u);
    }
}

static void deq_q4_k(const uint8_t* b, float* o) {
    float d = h2f(rd16(b)), dmin = h2f(rd16(b + 2));
    for (int g = 0; g < 8; g++) {
        uint32_t sc, mn;
        q4k_scale_min(b + 4, g, &sc, &mn);
        float dl = d * (float)sc;
        float dm = dmin * (float)mn;
        for (int p = 0; p < 32; p++) {
            uint32_t q = (b[16 + (g / 2) * 32 + p] >> (4 * (g & 1))) & 15u;
            float t = dl * (float)q;
            o[g * 32 + p] = t - dm;
        }
    }
}

/* gguf-py quants.py:552-572 (Q6_K): (d*scale) * (q - 32). */
static void deq_q6_k(const uint8_t* b, float* o) {
    float d = h2f(rd16(b + 208));
    for (int e = 0; e < QK; e++) {
        int c = e / 128, r = e % 128;
        uint32_t ql = (b[c * 64 + (r % 64)] >> (4 * (r / 64))) & 15u;
        uint32_t qh = (b[128 + c * 32 + (r % 32)] >> (2 * (r / 32))) & 3u;
        int q = (int)(ql | (qh << 4)) - 32;
        int8_t sc = (int8_t)b[192 + e / 16];
        float dl = d * (float)sc;
        o[e] = dl * (float)q;
    }
}

/* gguf-py quants.py:1351-1377 (IQ4_XS): (d*(scale-32)) * kvalues[q]. */
static void deq_iq4_xs(const uint8_t* b, float* o, const int8_t* kv) {
    float d = h2f(rd16(b));
    uint32_t sh = rd16(b + 2);
    for (int g = 0; g < 8; g++) {
        uint32_t lo = (b[4 + g / 2] >> (4 * (g & 1))) & 15u;
        uint32_t hi = (sh >> (2 * g)) & 3u;
        int scale = (int)(int8_t)(uint8_t)(lo | (hi << 4)) - 32;
        float dl = d * (float)scale;
        for (int p = 0; p < 32; p++) {
            uint32_t q = (b[8 + g * 16 + (p & 15)] >> (4 * (p / 16))) & 15u;
            o[g * 32 + p] = dl * (float)kv[q];
        }
    }
}

/* gguf-py quants.py:800-828 (IQ2_XXS). */
static void deq_iq2_xxs(const uint8_t* b, float* o, const int8_t* grid, const uint8_t* ks) {
    float d = h2f(rd16(b));
    for (int g = 0; g < 8; g++) {
        const uint8_t* q = b + 2 + 8 * g;
        uint32_t aux = rd32(q + 4);
        float db = (d * (0.5f + (float)(aux >> 28))) * 0.25f;
        for (int l = 0; l < 4; l++) {
            uint8_t signs = ks[(aux >> (7 * l)) & 127u];
            const int8_t* row = grid + 8 * q[l];
            for (int j = 0; j < 8; j++) {
                float v = db * (float)row[j];
                o[g * 32 + l * 8 + j] = ((signs >> j) & 1) ? v * -1.0f : v * 1.0f;
            }
        }
    }
}

/* gguf-py quants.py:870-898 (IQ2_XS). */
static void deq_iq2_xs(const uint8_t* b, float* o, const int8_t* grid, const uint8_t* ks) {
    float d = h2f(rd16(b));
    for (int i = 0; i < 32; i++) {
        uint32_t q = rd16(b + 2 + 2 * i);
        int s = i / 2;
        uint32_t sc = (b[66 + s / 2] >> (4 * (s & 1))) & 15u;
        float db = (d * (0.5f + (float)sc)) * 0.25f;
        uint8_t signs = ks[q >> 9];
        const int8_t* row = grid + 8 * (q & 511u);
        for (int j = 0; j < 8; j++) {
            float v = db * (float)row[j];
            o[i * 8 + j] = ((signs >> j) & 1) ? v * -1.0f : v * 1.0f;
        }
    }
}

/* gguf-py quants.py:972-1002 (IQ2_S). */
static void deq_iq2_s(const uint8_t* b, float* o, const int8_t* grid) {
    float d = h2f(rd16(b));
    for (int i = 0; i < 32; i++) {
        uint32_t hi = (b[66 + i / 4] >> (2 * (i % 4))) & 3u;
        uint32_t idx = b[2 + i] | (hi << 8);
        int s = i / 2;
        uint32_t sc = (b[74 + s / 2] >> (4 * (s & 1))) & 15u;
        float db = (d * (0.5f + (float)sc)) * 0.25f;
        uint8_t signs = b[34 + i];
        const int8_t* row = grid + 8 * idx;
        for (int j = 0; j < 8; j++) {
            float v = db * (float)row[j];
            o[i * 8 + j] = ((signs >> j) & 1) ? v * -1.0f : v * 1.0f;
        }
    }
}

/* gguf-py quants.py:1026-1054 (IQ3_XXS). */
static void deq_iq3_xxs(const uint8_t* b, float* o, const int8_t* grid, const uint8_t* ks) {
    float d = h2f(rd16(b));
    for (int g = 0; g < 8; g++) {
        uint32_t aux = rd32(b + 66 + 4 * g);
        float db = (d * (0.5f + (float)(aux >> 28))) * 0.5f;
        for (int l = 0; l < 4; l++) {
            uint8_t signs = ks[(aux >> (7 * l)) & 127u];
            for (int j = 0; j < 8; j++) {
                int e = g * 32 + l * 8 + j;
                const int8_t* row = grid + 4 * b[2 + e / 4];
                float v = db * (float)row[e % 4];
                o[e] = ((signs >> j) & 1) ? v * -1.0f : v * 1.0f;
            }
        }
    }
}

/* gguf-py quants.py:1094-1125 (IQ3_S): db = d*(1+2*scale) (integer factor). */
static void deq_iq3_s(const uint8_t* b, float* o, const int8_t* grid) {
    float d = h2f(rd16(b));
    for (int g = 0; g < 8; g++) {
        uint32_t sc = (b[106 + g / 2] >> (4 * (g & 1))) & 15u;
        float db = d * (float)(1u + 2u * sc);
        for (int p = 0; p < 32; p++) {
            int e = g * 32 + p;
            int i = e / 4;
            uint32_t idx = b[2 + i] | (((b[66 + i / 8] >> (i % 8)) & 1u) << 8);
            float v = db * (float)grid[4 * idx + (e % 4)];
            o[e] = ((b[74 + e / 8] >> (e % 8)) & 1) ? v * -1.0f : v * 1.0f;
        }
    }
}

/* gguf-py quants.py:1265-1288 (IQ1_S): dl*(grid + delta), delta = +-0.125. */
static void deq_iq1_s(const uint8_t* b, float* o, const int8_t* grid) {
    float d = h2f(rd16(b));
    for (int g = 0; g < 8; g++) {
        uint32_t qh = rd16(b + 34 + 2 * g);
        float dl = d * (float)(2u * ((qh >> 12) & 7u) + 1u);
        float delta = (qh & 0x8000u) ? -0.125f : 0.125f;
        for (int l = 0; l < 4; l++) {
            uint32_t idx = b[2 + 4 * g + l] | (((qh >> (3 * l)) & 7u) << 8);
            for (int j = 0; j < 8; j++) {
                float gv = (float)grid[8 * idx + j] + delta;
                o[g * 32 + l * 8 + j] = dl * gv;
            }
        }
    }
}

/* gguf-py quants.py:1298-1327 (IQ1_M): fp16 d assembled from the top nibbles. */
static void deq_iq1_m(const uint8_t* b, float* o, const int8_t* grid) {
    uint32_t w[4];
    for (int i = 0; i < 4; i++) w[i] = rd16(b + 48 + 2 * i);
    uint16_t dbits = (uint16_t)(((w[0] & 0xF000u) >> 12) | ((w[1] & 0xF000u) >> 8) |
                                ((w[2] & 0xF000u) >> 4) | (w[3] & 0xF000u));
    float d = h2f(dbits);
    for (int i = 0; i < 32; i++) {          /* 8-weight entries */
        int s = i / 2;                       /* 16-weight sub-block scale index */
        uint32_t sc = (w[s / 4] >> (3 * (s % 4))) & 7u;
        float dl = d * (float)(2u * sc + 1u);
        uint32_t hn = (b[32 + i / 2] >> (4 * (i % 2))) & 15u;
        uint32_t idx = b[i] | ((hn & 7u) << 8);
        float delta = (hn & 8u) ? -0.125f : 0.125f;
        for (int j = 0; j < 8; j++) {
            float gv = (float)grid[8 * idx + j] + delta;
            o[i * 8 + j] = dl * gv;
        }
    }
}

enum {
    T_Q2_K = 10, T_Q4_K = 12, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18,
    T_IQ1_S = 19, T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_IQ1_M = 29
};

int oracle_block_bytes(int t) {
    switch (t) {
        case T_Q2_K: return 84; case T_Q4_K: return 144; case T_Q6_K: return 210;
        case T_IQ2_XXS: return 66; case T_IQ2_XS: return 74; case T_IQ3_XXS: return 98;
        case T_IQ1_S: return 50; case T_IQ3_S: return 110; case T_IQ2_S: return 82;
        case T_IQ4_XS: return 136; case T_IQ1_M: return 56;
    }
    return -1;
}

static int deq_block(int t, const uint8_t* b, float* o, const int8_t* grid, const uint8_t* ks,
                     const int8_t* kv) {
    switch (t) {
        case T_Q2_K: deq_q2_k(b, o); return 0;
        case T_Q4_K: deq_q4_k(b, o); return 0;
        case T_Q6_K: deq_q6_k(b, o); return 0;
        case T_IQ4_XS: deq_iq4_xs(b, o, kv); return 0;
        case T_IQ2_XXS: deq_iq2_xxs(b, o, grid, ks); return 0;
        case T_IQ2_XS: deq_iq2_xs(b, o, grid, ks); return 0;
        case T_IQ2_S: deq_iq2_s(b, o, grid); return 0;
        case T_IQ3_XXS: deq_iq3_xxs(b, o, grid, ks); return 0;
        case T_IQ3_S: deq_iq3_s(b, o, grid); return 0;
        case T_IQ1_S: deq_iq1_s(b, o, grid); return 0;
        case T_IQ1_M: deq_iq1_m(b, o, grid); return 0;
    }
    return -1;
}

/* Flat fp32 dequant of nblocks blocks (reference registry.decode contract,
 * mlx_gsq/runtime/kernels/registry.py:28-32). */
int oracle_dequant(int t, const uint8_t* packed, int64_t nblocks, float* out,
                   const int8_t* grid, const uint8_t* ks, const int8_t* kv) {
    int bb = oracle_block_bytes(t);
    if (bb < 0) return -1;
    int err = 0;
#pragma omp parallel for schedule(static) reduction(| : err)
    for (int64_t i = 0; i < nblocks; i++)
        err |= deq_block(t, packed + i * bb, out + i * QK, grid, ks, kv) != 0;
    return err ? -1 : 0;
}

/* y[m, n] = sum_k x[m, k] * deq(W)[n, k], double accumulation of fp32 terms.
 * W is N rows of K/256 blocks (reference quantized_matvec/quantized_matmul
 * contract, qmv.py:537-576, qmm.py:559-594). */
int oracle_matmul(int t, const float* x, int64_t M, const uint8_t* packed, int64_t N, int64_t K,
                  double* y, const int8_t* grid, const uint8_t* ks, const int8_t* kv) {
    int bb = oracle_block_bytes(t);
    if (bb < 0 || K % QK) return -1;
    int64_t nb = K / QK;
    int err = 0;
#pragma omp parallel for schedule(static) reduction(| : err)
    for (int64_t n = 0; n < N; n++) {
        float w[QK];
        double acc[64];
        int64_t m0;
        for (m0 = 0; m0 < M; m0 += 64) {
            int64_t mc = M - m0 < 64 ? M - m0 : 64;
            for (int64_t m = 0; m < mc; m++) acc[m] = 0.0;
            for (int64_t j = 0; j < nb; j++) {
                err |= deq_block(t, packed + (n * nb + j) * bb, w, grid, ks, kv) != 0;
                for (int64_t m = 0; m < mc; m++) {
                    const float* xr = x + (m0 + m) * K + j * QK;
                    double s = 0.0;
                    for (int e = 0; e < QK; e++) s += (double)xr[e] * (double)w[e];
                    acc[m] += s;
                }
            }
            for (int64_t m = 0; m < mc; m++) y[(m0 + m) * N + n] = acc[m];
        }
    }
    return err ? -1 : 0;
}

/* out[i, :] = deq(W)[ids[i], :] as fp32 (reference iq2_s_embedding,
 * mlx_gsq/runtime/kernels/embedding.py:9-36, generalised to every type). */
int oracle_embed(int t, const int32_t* ids, int64_t T, const uint8_t* packed, int64_t vocab,
                 int64_t dim, float* out, const int8_t* grid, const uint8_t* ks, const int8_t* kv) {
    int bb = oracle_block_bytes(t);
    if (bb < 0 || dim % QK) return -1;
    int64_t nb = dim / QK;
    for (int64_t i = 0; i < T; i++) {
        if (ids[i] < 0 || ids[i] >= vocab) return -2;
        for (int64_t j = 0; j < nb; j++)
            deq_block(t, packed + ((int64_t)ids[i] * nb + j) * bb, out + i * dim + j * QK, grid, ks, kv);
    }
    return 0;
}
