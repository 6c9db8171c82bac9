// Decoder-glue kernels of the Qwen3.5-hybrid model harness (include/gsq_model.h):
// the work between the packed projections of one decoder layer.
//
//  * rmsnorm_kernel: one CTA per row; the residual add is fused in (the
//    projection that produced `delta` writes fp32, the next projection reads
//    the normalised row as 16-bit).
//  * gated-DeltaNet, three launches per layer call:
//      gdn_prep_kernel  (T x (nk + nv) CTAs of 128 threads): causal conv of
//                       one head's q|k (or v) channels over the last four
//                       inputs, SiLU, the q/k RMS scaling, the gates;
//      gdn_scan_kernel  (nv x 8 CTAs of 128 threads): the delta-rule
//                       recurrence over the T tokens, 16 value columns per
//                       CTA.  The columns of S evolve independently (every
//                       update reads only its own column and the shared k, q),
//                       so a head splits over CTAs with no exchange.  Each
//                       thread keeps 16 entries of one column in registers
//                       (key index i = seg + 8r, r = 0..15, so the eight
//                       threads of a column read consecutive shared words),
//                       and the next token's q, k, v and gates are loaded
//                       while the current one is applied: one barrier per
//                       token.  The same launch advances the conv window;
//      gdn_norm_kernel  (T x nv CTAs): gated RMSNorm of each head's output.
//  * attn_decode_kernel: one CTA per query head for a single token; the CTA
//    normalises and rotates its own key (the first query head of each group
//    also stores it), so no CTA reads a cache row another CTA is writing.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>

#include "gsq_common.cuh"
#include "../../include/gsq_model.h"

namespace gsq {
int set_last_error(int code, const char* msg);
}

using namespace gsq;

namespace {

constexpr int GDN_D = 128;      // gated-DeltaNet key / value head width
constexpr int GDN_COLS = 16;    // value columns per scan CTA
constexpr int ATT_D = 256;      // attention head width

__device__ __forceinline__ float silu(float v) { return v / (1.f + __expf(-v)); }

// Sum over the CTA (blockDim.x a multiple of 32); every thread gets the sum.
__device__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();  // earlier readers of red are done
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = 0.f;
  for (int i = 0; i < nw; i++) s += red[i];
  return s;
}

__device__ float block_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int w = threadIdx.x >> 5, nw = blockDim.x >> 5;
  __syncthreads();
  if ((threadIdx.x & 31) == 0) red[w] = v;
  __syncthreads();
  float s = red[0];
  for (int i = 1; i < nw; i++) s = fmaxf(s, red[i]);
  return s;
}

__global__ void __launch_bounds__(256) rmsnorm_kernel(float* resid, const float* delta, int64_t dim, const float* w,
                                                      float eps, void* out, int dt) {
  __shared__ float red[32];
  const int64_t r = blockIdx.x;
  float* x = resid + r * dim;
  const float* d = delta ? delta + r * dim : nullptr;
  float ss = 0.f;
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) {
    float v = x[i];
    if (d) {
      v += d[i];
      x[i] = v;
    }
    ss = fmaf(v, v, ss);
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)dim + eps);
  for (int64_t i = threadIdx.x; i < dim; i += blockDim.x) store_out(out, dt, r * dim + i, x[i] * inv * w[i]);
}

__global__ void silu_mul_kernel(const float* gu, int64_t rows, int64_t n, void* out, int dt) {
  const int64_t total = rows * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    store_out(out, dt, i, silu(gu[r * 2 * n + c]) * gu[r * 2 * n + n + c]);
  }
}

struct GdnArgs {
  const float* proj;
  int64_t ps;
  const __half* ab;
  int64_t abs;
  int T, nk, nv, C;
  float* conv_state;
  const float* conv_w;
  const float* A;
  const float* dt_bias;
  const float* norm_w;
  float eps;
  float* state;
  float* qn;    // [T, nk, 128]
  float* kn;    // [T, nk, 128]
  float* vv;    // [T, nv, 128]
  float* gdec;  // [T, nv]
  float* beta;  // [T, nv]
  float* o;     // [T, nv, 128]
  void* out;
  int dt;
};

// SiLU of the causal depthwise conv of channel c at token t: taps 0..3 meet
// inputs t-3..t; inputs before the first token come from the conv window.
__device__ __forceinline__ float gdn_conv(const GdnArgs& a, int t, int c) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int s = t - 3 + j;
    const float in = s >= 0 ? a.proj[(int64_t)s * a.ps + c] : a.conv_state[(int64_t)(3 + s) * a.C + c];
    acc = fmaf(a.conv_w[(int64_t)c * 4 + j], in, acc);
  }
  return silu(acc);
}

__global__ void __launch_bounds__(GDN_D) gdn_prep_kernel(GdnArgs a) {
  __shared__ float red[32];
  const int t = blockIdx.x, grp = blockIdx.y, i = threadIdx.x;
  if (grp < a.nk) {
    const float q = gdn_conv(a, t, grp * GDN_D + i);
    const float k = gdn_conv(a, t, a.nk * GDN_D + grp * GDN_D + i);
    const float sq = block_sum(q * q, red);
    const float sk = block_sum(k * k, red);
    const int64_t o = ((int64_t)t * a.nk + grp) * GDN_D + i;
    a.qn[o] = q * rsqrtf(sq / GDN_D + 1e-6f) * (1.f / GDN_D);
    a.kn[o] = k * rsqrtf(sk / GDN_D + 1e-6f) * rsqrtf((float)GDN_D);
  } else {
    const int h = grp - a.nk;
    a.vv[((int64_t)t * a.nv + h) * GDN_D + i] = gdn_conv(a, t, 2 * a.nk * GDN_D + h * GDN_D + i);
    if (i == 0) {
      const float av = __half2float(a.ab[(int64_t)t * a.abs + h]) + a.dt_bias[h];
      const float bv = __half2float(a.ab[(int64_t)t * a.abs + a.nv + h]);
      const float sp = av > 20.f ? av : log1pf(__expf(av));
      a.gdec[(int64_t)t * a.nv + h] = __expf(a.A[h] * sp);
      a.beta[(int64_t)t * a.nv + h] = 1.f / (1.f + __expf(-bv));
    }
  }
}

__global__ void __launch_bounds__(GDN_D) gdn_scan_kernel(GdnArgs a) {
  __shared__ float qs[2][GDN_D], ks[2][GDN_D];
  const int h = blockIdx.x, kh = h % a.nk;
  const int tid = threadIdx.x, col = tid >> 3, seg = tid & 7;
  const int j = blockIdx.y * GDN_COLS + col;
  float* sp = a.state + ((int64_t)h * GDN_D + j) * GDN_D + seg;
  float S[16];
#pragma unroll
  for (int r = 0; r < 16; r++) S[r] = sp[8 * r];

  float nq = 0.f, nkv = 0.f, nv = 0.f, ng = 0.f, nb = 0.f;
  if (a.T > 0) {
    qs[0][tid] = a.qn[(int64_t)kh * GDN_D + tid];
    ks[0][tid] = a.kn[(int64_t)kh * GDN_D + tid];
    nv = a.vv[(int64_t)h * GDN_D + j];
    ng = a.gdec[h];
    nb = a.beta[h];
  }
  __syncthreads();
  for (int t = 0; t < a.T; t++) {
    const int b = t & 1;
    const float vj = nv, d = ng, be = nb;
    if (t + 1 < a.T) {
      const int64_t base = ((int64_t)(t + 1) * a.nk + kh) * GDN_D + tid;
      nq = a.qn[base];
      nkv = a.kn[base];
      nv = a.vv[((int64_t)(t + 1) * a.nv + h) * GDN_D + j];
      ng = a.gdec[(int64_t)(t + 1) * a.nv + h];
      nb = a.beta[(int64_t)(t + 1) * a.nv + h];
    }
    float kv = 0.f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      S[r] *= d;
      kv = fmaf(S[r], ks[b][seg + 8 * r], kv);
    }
    kv += __shfl_xor_sync(0xffffffffu, kv, 1);
    kv += __shfl_xor_sync(0xffffffffu, kv, 2);
    kv += __shfl_xor_sync(0xffffffffu, kv, 4);
    const float u = (vj - kv) * be;
    float y = 0.f;
#pragma unroll
    for (int r = 0; r < 16; r++) {
      S[r] = fmaf(ks[b][seg + 8 * r], u, S[r]);
      y = fmaf(S[r], qs[b][seg + 8 * r], y);
    }
    y += __shfl_xor_sync(0xffffffffu, y, 1);
    y += __shfl_xor_sync(0xffffffffu, y, 2);
    y += __shfl_xor_sync(0xffffffffu, y, 4);
    if (seg == 0) a.o[((int64_t)t * a.nv + h) * GDN_D + j] = y;
    if (t + 1 < a.T) {
      qs[b ^ 1][tid] = nq;
      ks[b ^ 1][tid] = nkv;
    }
    __syncthreads();
  }
#pragma unroll
  for (int r = 0; r < 16; r++) sp[8 * r] = S[r];

  // Advance the conv window by T inputs (the prep launch, which read it, has
  // completed).  Rows ascend, and new row r reads old row r + T > r.
  const int64_t nthr = (int64_t)gridDim.x * gridDim.y * blockDim.x;
  const int64_t gid = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid;
  for (int64_t c = gid; c < a.C; c += nthr) {
#pragma unroll
    for (int r = 0; r < 3; r++) {
      const int s = a.T - 3 + r;
      a.conv_state[(int64_t)r * a.C + c] =
          s >= 0 ? a.proj[(int64_t)s * a.ps + c] : a.conv_state[(int64_t)(r + a.T) * a.C + c];
    }
  }
}

__global__ void __launch_bounds__(GDN_D) gdn_norm_kernel(GdnArgs a) {
  __shared__ float red[32];
  const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  const float v = a.o[((int64_t)t * a.nv + h) * GDN_D + i];
  const float ss = block_sum(v * v, red);
  const float z = a.proj[(int64_t)t * a.ps + a.C + h * GDN_D + i];
  store_out(a.out, a.dt, ((int64_t)t * a.nv + h) * GDN_D + i,
            v * rsqrtf(ss / GDN_D + a.eps) * a.norm_w[i] * silu(z));
}

// One decode token of gated GQA attention; CTA = query head, 256 threads =
// head dimensions.  Dynamic shared memory: scores of positions 0..pos.
__global__ void __launch_bounds__(ATT_D) attn_decode_kernel(const float* qkv, int nq, int nkv, const float* qw,
                                                            const float* kw, float eps, int rot, float theta,
                                                            float* kc, float* vc, int max_len, const int* pos_p,
                                                            void* out, int dt) {
  extern __shared__ float sc[];
  __shared__ float red[32];
  __shared__ float qs[ATT_D], ks[ATT_D], vs[ATT_D];
  const int h = blockIdx.x, d = threadIdx.x;
  const int group = nq / nkv, kvh = h / group;
  const int pos = min(max(*pos_p, 0), max_len - 1);
  float q = qkv[(int64_t)h * 2 * ATT_D + d];
  const float gate = qkv[(int64_t)h * 2 * ATT_D + ATT_D + d];
  float k = qkv[(int64_t)nq * 2 * ATT_D + kvh * ATT_D + d];
  const float v = qkv[(int64_t)nq * 2 * ATT_D + nkv * ATT_D + kvh * ATT_D + d];
  q *= rsqrtf(block_sum(q * q, red) / ATT_D + eps) * qw[d];
  k *= rsqrtf(block_sum(k * k, red) / ATT_D + eps) * kw[d];
  qs[d] = q;
  ks[d] = k;
  vs[d] = v;
  __syncthreads();
  if (d < rot) {
    const int half = rot / 2, i = d % half;
    const float ang = (float)pos * powf(theta, -2.f * (float)i / (float)rot);
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float qo = d < half ? -qs[d + half] : qs[d - half];
    const float ko = d < half ? -ks[d + half] : ks[d - half];
    q = q * cs + qo * sn;
    k = k * cs + ko * sn;
  }
  __syncthreads();
  qs[d] = q;
  ks[d] = k;
  if (h % group == 0) {
    kc[((int64_t)pos * nkv + kvh) * ATT_D + d] = k;
    vc[((int64_t)pos * nkv + kvh) * ATT_D + d] = v;
  }
  __syncthreads();

  // Scores: warp w takes positions w, w + 8, ...; lane l holds dimensions
  // 8l..8l+7.  The current position's key comes from shared memory.
  const int warp = d >> 5, lane = d & 31;
  float qr[8];
#pragma unroll
  for (int e = 0; e < 8; e++) qr[e] = qs[8 * lane + e];
  const float scale = rsqrtf((float)ATT_D);
  for (int s = warp; s <= pos; s += ATT_D / 32) {
    const float* kr = s == pos ? ks : kc + ((int64_t)s * nkv + kvh) * ATT_D;
    const float4 k0 = *reinterpret_cast<const float4*>(kr + 8 * lane);
    const float4 k1 = *reinterpret_cast<const float4*>(kr + 8 * lane + 4);
    float p = qr[0] * k0.x + qr[1] * k0.y + qr[2] * k0.z + qr[3] * k0.w + qr[4] * k1.x + qr[5] * k1.y +
              qr[6] * k1.z + qr[7] * k1.w;
#pragma unroll
    for (int o = 16; o; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
    if (lane == 0) sc[s] = p * scale;
  }
  __syncthreads();
  float m = -INFINITY;
  for (int s = d; s <= pos; s += ATT_D) m = fmaxf(m, sc[s]);
  m = block_max(m, red);
  float l = 0.f;
  for (int s = d; s <= pos; s += ATT_D) {
    const float e = __expf(sc[s] - m);
    sc[s] = e;
    l += e;
  }
  l = block_sum(l, red);  // its barriers also publish sc
  float acc = 0.f;
  for (int s = 0; s < pos; s++) acc = fmaf(sc[s], vc[((int64_t)s * nkv + kvh) * ATT_D + d], acc);
  acc = fmaf(sc[pos], vs[d], acc);
  store_out(out, dt, (int64_t)h * ATT_D + d, acc / l / (1.f + __expf(-gate)));
}

bool dt_ok(int d) { return d == DT_F32 || d == DT_F16 || d == DT_BF16; }

int fail(int code, const char* msg) { return set_last_error(code, msg); }

int launched(const char* what) {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    char buf[256];
    snprintf(buf, sizeof(buf), "%s: %s", what, cudaGetErrorString(e));
    return fail(GSQ_ERR_CUDA, buf);
  }
  return GSQ_OK;
}

size_t align16(size_t v) { return (v + 15) & ~size_t(15); }

}  // namespace

extern "C" {

int gsq_rmsnorm(float* resid, const float* delta, int64_t rows, int64_t dim, const float* weight, float eps,
                void* out, int out_dtype, gsq_stream_t stream) {
  if (!resid || !weight || !out) return fail(GSQ_ERR_ARG, "gsq_rmsnorm: null pointer");
  if (rows < 0 || dim <= 0 || rows > INT32_MAX) return fail(GSQ_ERR_SIZE, "gsq_rmsnorm: bad shape");
  if (!dt_ok(out_dtype)) return fail(GSQ_ERR_ARG, "gsq_rmsnorm: bad output dtype");
  if (rows == 0) return GSQ_OK;
  rmsnorm_kernel<<<(unsigned)rows, 256, 0, (cudaStream_t)stream>>>(resid, delta, dim, weight, eps, out, out_dtype);
  return launched("gsq_rmsnorm");
}

int gsq_silu_mul(const float* gu, int64_t rows, int64_t n, void* out, int out_dtype, gsq_stream_t stream) {
  if (!gu || !out) return fail(GSQ_ERR_ARG, "gsq_silu_mul: null pointer");
  if (rows < 0 || n <= 0) return fail(GSQ_ERR_SIZE, "gsq_silu_mul: bad shape");
  if (!dt_ok(out_dtype)) return fail(GSQ_ERR_ARG, "gsq_silu_mul: bad output dtype");
  if (rows == 0) return GSQ_OK;
  const int64_t total = rows * n;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  silu_mul_kernel<<<blocks, 256, 0, (cudaStream_t)stream>>>(gu, rows, n, out, out_dtype);
  return launched("gsq_silu_mul");
}

size_t gsq_gdn_scratch_bytes(int64_t T, int64_t nk, int64_t nv) {
  if (T <= 0 || nk <= 0 || nv <= 0) return 0;
  const size_t f = sizeof(float);
  return 2 * align16(T * nk * GDN_D * f) + 2 * align16(T * nv * GDN_D * f) + 2 * align16(T * nv * f);
}

int gsq_gdn(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride, int64_t T, int64_t nk,
            int64_t nv, float* conv_state, const float* conv_w, const float* A, const float* dt_bias,
            const float* norm_w, float eps, float* state, void* scratch, size_t scratch_bytes, void* out,
            int out_dtype, gsq_stream_t stream) {
  if (!proj || !ab || !conv_state || !conv_w || !A || !dt_bias || !norm_w || !state || !out)
    return fail(GSQ_ERR_ARG, "gsq_gdn: null pointer");
  if (T < 0 || T > INT32_MAX / 2 || nk <= 0 || nv <= 0 || nv % nk || nv > 65535 || nk > 65535)
    return fail(GSQ_ERR_SIZE, "gsq_gdn: bad shape (nv must be a multiple of nk)");
  const int64_t C = 2 * nk * GDN_D + nv * GDN_D;
  if (proj_stride < C + nv * GDN_D || ab_stride < 2 * nv) return fail(GSQ_ERR_SIZE, "gsq_gdn: stride too small");
  if (!dt_ok(out_dtype)) return fail(GSQ_ERR_ARG, "gsq_gdn: bad output dtype");
  if (T == 0) return GSQ_OK;
  if (!scratch || scratch_bytes < gsq_gdn_scratch_bytes(T, nk, nv))
    return fail(GSQ_ERR_WORKSPACE, "gsq_gdn: scratch missing or too small");
  if (reinterpret_cast<uintptr_t>(scratch) % 16) return fail(GSQ_ERR_ALIGN, "gsq_gdn: scratch not 16-byte aligned");
  GdnArgs a;
  a.proj = proj;
  a.ps = proj_stride;
  a.ab = reinterpret_cast<const __half*>(ab);
  a.abs = ab_stride;
  a.T = (int)T;
  a.nk = (int)nk;
  a.nv = (int)nv;
  a.C = (int)C;
  a.conv_state = conv_state;
  a.conv_w = conv_w;
  a.A = A;
  a.dt_bias = dt_bias;
  a.norm_w = norm_w;
  a.eps = eps;
  a.state = state;
  uint8_t* p = static_cast<uint8_t*>(scratch);
  const size_t f = sizeof(float);
  a.qn = reinterpret_cast<float*>(p);
  p += align16(T * nk * GDN_D * f);
  a.kn = reinterpret_cast<float*>(p);
  p += align16(T * nk * GDN_D * f);
  a.vv = reinterpret_cast<float*>(p);
  p += align16(T * nv * GDN_D * f);
  a.o = reinterpret_cast<float*>(p);
  p += align16(T * nv * GDN_D * f);
  a.gdec = reinterpret_cast<float*>(p);
  p += align16(T * nv * f);
  a.beta = reinterpret_cast<float*>(p);
  a.out = out;
  a.dt = out_dtype;
  cudaStream_t st = (cudaStream_t)stream;
  gdn_prep_kernel<<<dim3((unsigned)T, (unsigned)(nk + nv)), GDN_D, 0, st>>>(a);
  int rc = launched("gsq_gdn (prep)");
  if (rc) return rc;
  gdn_scan_kernel<<<dim3((unsigned)nv, GDN_D / GDN_COLS), GDN_D, 0, st>>>(a);
  if ((rc = launched("gsq_gdn (scan)"))) return rc;
  gdn_norm_kernel<<<dim3((unsigned)T, (unsigned)nv), GDN_D, 0, st>>>(a);
  return launched("gsq_gdn (norm)");
}

int gsq_attn_decode(const float* qkv, int64_t nq, int64_t nkv, const float* q_norm_w, const float* k_norm_w,
                    float eps, int64_t rot, float theta, float* k_cache, float* v_cache, int64_t max_len,
                    const int32_t* pos, void* out, int out_dtype, gsq_stream_t stream) {
  if (!qkv || !q_norm_w || !k_norm_w || !k_cache || !v_cache || !pos || !out)
    return fail(GSQ_ERR_ARG, "gsq_attn_decode: null pointer");
  if (nq <= 0 || nkv <= 0 || nq % nkv || nq > 65535) return fail(GSQ_ERR_SIZE, "gsq_attn_decode: bad head counts");
  if (rot < 0 || rot > ATT_D || rot % 2) return fail(GSQ_ERR_SIZE, "gsq_attn_decode: bad rotary width");
  if (max_len <= 0 || max_len > 48 * 1024) return fail(GSQ_ERR_SIZE, "gsq_attn_decode: max_len out of range");
  if (!dt_ok(out_dtype)) return fail(GSQ_ERR_ARG, "gsq_attn_decode: bad output dtype");
  if (reinterpret_cast<uintptr_t>(k_cache) % 16 || reinterpret_cast<uintptr_t>(v_cache) % 16)
    return fail(GSQ_ERR_ALIGN, "gsq_attn_decode: caches not 16-byte aligned");
  const size_t smem = (size_t)max_len * sizeof(float);
  cudaStream_t st = (cudaStream_t)stream;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(GSQ_ERR_CUDA, "gsq_attn_decode: shared memory attribute");
  }
  attn_decode_kernel<<<(unsigned)nq, ATT_D, smem, st>>>(qkv, (int)nq, (int)nkv, q_norm_w, k_norm_w, eps, (int)rot,
                                                        theta, k_cache, v_cache, (int)max_len, pos, out,
                                                        out_dtype);
  return launched("gsq_attn_decode");
}

}  // extern "C"
