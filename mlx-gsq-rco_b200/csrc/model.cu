// Decoder-glue kernels of the Qwen3.5-hybrid model harness (include/gsq_model.h):
// the work between the packed projections of one decoder layer.
//
//  * rmsnorm_vec_kernel: one CTA per row, the row held in registers; the
//    residual add is fused in (the projection that produced `delta` writes
//    fp32, the next projection reads the normalised row as 16-bit).
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
//  * Every kernel is launched with programmatic dependent launch: it lets the
//    next kernel of the stream start (a matvec's weight stream overlaps it),
//    loads only static weights before griddepcontrol.wait, and everything
//    the previous kernels wrote after it.
//  * attn_decode_kernel: one CTA per query head for a single token; the CTA
//    normalises and rotates its own key (the first query head of each group
//    also stores it), so no CTA reads a cache row another CTA is writing.
#include <cuda_fp16.h>

#include <algorithm>
#include <cstdio>

#include "gsq_common.cuh"
#include "gsq_host.h"
#include "../../include/gsq_model.h"

namespace gsq {
int set_last_error(int code, const char* msg);
}

using namespace gsq;

namespace {

constexpr int GDN_D = 128;      // gated-DeltaNet key / value head width
constexpr int GDN_COLS = 16;    // value columns per scan CTA
constexpr int ATT_D = 256;      // attention head width
constexpr int ATT_U = 8;        // key positions per warp step of the decode attention

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

// Thread-block cluster barrier (all threads of every CTA of the cluster;
// release / acquire order the shared-memory writes before it).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// A float in the shared memory of CTA `rank` of this cluster, at the address
// `p` has in this CTA.
__device__ __forceinline__ float ld_shared_cluster_f32(const float* p, uint32_t rank) {
  uint32_t remote;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(smem_u32(p)), "r"(rank));
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
  return v;
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

// Rows of up to RMS_MAXV float4 per thread x 256 threads (dim <= 8192): the
// whole row is loaded into registers before anything is stored, so every
// load of the row is in flight at once (a loop that stores the residual
// between loads waits for each load in turn).
constexpr int RMS_THREADS = 256, RMS_MAXV = 8;

__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_vec_kernel(float* __restrict__ resid,
                                                                 const float* __restrict__ delta, int dim,
                                                                 const float* __restrict__ w, float eps,
                                                                 void* __restrict__ out, int dt) {
  __shared__ float red[32];
  pdl_launch_dependents();
  const int64_t r = blockIdx.x;
  const int n4 = dim >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[RMS_MAXV];  // static weights: loaded while the previous kernel finishes
#pragma unroll
  for (int u = 0; u < RMS_MAXV; u++) {
    const int i = threadIdx.x + u * RMS_THREADS;
    if (i < n4) wv[u] = w4[i];
  }
  pdl_wait();
  float4* x = reinterpret_cast<float4*>(resid + r * dim);
  const float4* d = delta ? reinterpret_cast<const float4*>(delta + r * dim) : nullptr;
  float4 v[RMS_MAXV];
  float ss = 0.f;
#pragma unroll
  for (int u = 0; u < RMS_MAXV; u++) {
    const int i = threadIdx.x + u * RMS_THREADS;
    if (i < n4) {
      v[u] = x[i];
      if (d) {
        const float4 b = d[i];
        v[u].x += b.x;
        v[u].y += b.y;
        v[u].z += b.z;
        v[u].w += b.w;
      }
    }
  }
#pragma unroll
  for (int u = 0; u < RMS_MAXV; u++) {
    const int i = threadIdx.x + u * RMS_THREADS;
    if (i < n4) {
      if (d) x[i] = v[u];
      ss = fmaf(v[u].x, v[u].x, fmaf(v[u].y, v[u].y, fmaf(v[u].z, v[u].z, fmaf(v[u].w, v[u].w, ss))));
    }
  }
  const float inv = rsqrtf(block_sum(ss, red) / (float)dim + eps);
#pragma unroll
  for (int u = 0; u < RMS_MAXV; u++) {
    const int i = threadIdx.x + u * RMS_THREADS;
    if (i < n4) {
      const float4 g = wv[u];
      const float o0 = v[u].x * inv * g.x, o1 = v[u].y * inv * g.y, o2 = v[u].z * inv * g.z, o3 = v[u].w * inv * g.w;
      const int64_t e = r * dim + 4 * (int64_t)i;
      if (dt == DT_F32) {
        reinterpret_cast<float4*>(out)[e >> 2] = make_float4(o0, o1, o2, o3);
      } else if (dt == DT_F16) {
        __half2 h[2] = {__floats2half2_rn(o0, o1), __floats2half2_rn(o2, o3)};
        reinterpret_cast<uint2*>(out)[e >> 2] = *reinterpret_cast<uint2*>(h);
      } else {
        __nv_bfloat162 h[2] = {__floats2bfloat162_rn(o0, o1), __floats2bfloat162_rn(o2, o3)};
        reinterpret_cast<uint2*>(out)[e >> 2] = *reinterpret_cast<uint2*>(h);
      }
    }
  }
}

// Any width and alignment.
__global__ void __launch_bounds__(RMS_THREADS) rmsnorm_kernel(float* resid, const float* delta, int64_t dim,
                                                             const float* w, float eps, void* out, int dt) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
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

// group 0: gu = [gate | up] halves; group g > 0: gate and up interleaved in
// groups of g columns (g gate columns, then the same g up columns).  gu is
// fp32, fp16 or bf16 (gu_dt).
__global__ void silu_mul_kernel(const void* gu, int gu_dt, int64_t rows, int64_t n, int64_t group, void* out,
                                int dt) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t total = rows * n;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t r = i / n, c = i - r * n;
    int64_t gcol = c, ucol = n + c;
    if (group > 0) {
      const int64_t q = c / group;
      gcol = c + q * group;
      ucol = gcol + group;
    }
    store_out(out, dt, i, silu(load_act(gu, gu_dt, r * 2 * n + gcol)) * load_act(gu, gu_dt, r * 2 * n + ucol));
  }
}

// Eight outputs per thread: the gate values at gu[row][g0 .. g0+7] and the
// up values at gu[row][u0 .. u0+7] (16-byte loads of fp16 / bf16, two of
// fp32), out[row][8c .. 8c+7] as one 16-byte store (fp16 / bf16) or two
// (fp32).  grid.y = rows; group 8: g0 = 16c, u0 = 16c + 8; group 0: g0 = 8c,
// u0 = n + 8c.
template <typename IT>
__device__ __forceinline__ void load8(const IT* p, float (&f)[8]) {
  if constexpr (sizeof(IT) == 4) {
    const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w; f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
    const uint4 v = *reinterpret_cast<const uint4*>(p);
    const IT* e = reinterpret_cast<const IT*>(&v);
#pragma unroll
    for (int i = 0; i < 8; i++) f[i] = to_f32(e[i]);
  }
}

template <typename IT>
__global__ void silu_mul8_kernel(const IT* gu, int64_t n, int64_t group, void* out, int dt) {
  pdl_launch_dependents();
  pdl_wait();
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= n / 8) return;
  const int64_t row = blockIdx.y;
  const IT* base = gu + row * 2 * n;
  float g[8], u[8], y[8];
  load8(base + (group ? 16 * c : 8 * c), g);
  load8(base + (group ? 16 * c + 8 : n + 8 * c), u);
#pragma unroll
  for (int i = 0; i < 8; i++) y[i] = silu(g[i]) * u[i];
  const int64_t o = row * n + 8 * c;
  if (dt == DT_F32) {
    float4* p = reinterpret_cast<float4*>(reinterpret_cast<float*>(out) + o);
    p[0] = make_float4(y[0], y[1], y[2], y[3]);
    p[1] = make_float4(y[4], y[5], y[6], y[7]);
  } else {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; i++) {
      if (dt == DT_F16) {
        const __half2 h = __floats2half2_rn(y[2 * i], y[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      } else {
        const __nv_bfloat162 h = __floats2bfloat162_rn(y[2 * i], y[2 * i + 1]);
        w[i] = *reinterpret_cast<const uint32_t*>(&h);
      }
    }
    *reinterpret_cast<uint4*>(reinterpret_cast<uint16_t*>(out) + o) = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

struct GdnArgs {
  const float* proj;
  int64_t ps;
  const __half* ab;   // precomputed gate inputs, or null:
  int64_t abs;
  const __half* x;    // ... then from the layer input x [T, hidden]
  int64_t xs;
  const __half* abw;  // and the gate weights [2nv, hidden]
  int hidden;
  int T, nk, nv, C;
  float* conv_state;  // [4, C] ring: slot p & 3 holds the input of position p
  const int* pos;     // position of token 0 (device)
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

// SiLU of the causal depthwise conv of channel c at token t (position
// p0 + t): taps 0..3 meet inputs t-3..t; inputs before the first token come
// from the conv window's ring slots.
__device__ __forceinline__ float gdn_conv(const GdnArgs& a, int p0, int t, int c) {
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; j++) {
    const int s = t - 3 + j;
    const float in = s >= 0 ? a.proj[(int64_t)s * a.ps + c] : a.conv_state[(int64_t)((p0 + s) & 3) * a.C + c];
    acc = fmaf(a.conv_w[(int64_t)c * 4 + j], in, acc);
  }
  return silu(acc);
}

// Dot products of one fp16 input row with two fp16 weight rows, summed over
// the CTA (8 halves per 16-byte load; hidden % 8 == 0, rows 16-byte aligned).
__device__ __forceinline__ void dot2_rows(const __half* x, const __half* wa, const __half* wb, int hidden,
                                          float* red, float& da, float& db) {
  const uint4* xr = reinterpret_cast<const uint4*>(x);
  const uint4* ar = reinterpret_cast<const uint4*>(wa);
  const uint4* br = reinterpret_cast<const uint4*>(wb);
  float sa = 0.f, sb = 0.f;
#pragma unroll 4
  for (int e = threadIdx.x; e < hidden / 8; e += blockDim.x) {
    const uint4 xv = xr[e], av = ar[e], bv = br[e];
    const __half2* xh = reinterpret_cast<const __half2*>(&xv);
    const __half2* ah = reinterpret_cast<const __half2*>(&av);
    const __half2* bh = reinterpret_cast<const __half2*>(&bv);
#pragma unroll
    for (int q = 0; q < 4; q++) {
      const float2 xf = __half22float2(xh[q]), af = __half22float2(ah[q]), bf = __half22float2(bh[q]);
      sa = fmaf(xf.x, af.x, fmaf(xf.y, af.y, sa));
      sb = fmaf(xf.x, bf.x, fmaf(xf.y, bf.y, sb));
    }
  }
  da = block_sum(sa, red);
  db = block_sum(sb, red);
}

__device__ __forceinline__ void gdn_gates(const GdnArgs& a, int h, float av, float bv, float& g, float& beta) {
  av += a.dt_bias[h];
  const float sp = av > 20.f ? av : log1pf(__expf(av));
  g = __expf(a.A[h] * sp);
  beta = 1.f / (1.f + __expf(-bv));
}

__global__ void __launch_bounds__(GDN_D) gdn_prep_kernel(GdnArgs a) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, grp = blockIdx.y, i = threadIdx.x;
  const int p0 = *a.pos;
  if (grp < a.nk) {
    const float q = gdn_conv(a, p0, t, grp * GDN_D + i);
    const float k = gdn_conv(a, p0, t, a.nk * GDN_D + grp * GDN_D + i);
    const float sq = block_sum(q * q, red);
    const float sk = block_sum(k * k, red);
    const int64_t o = ((int64_t)t * a.nk + grp) * GDN_D + i;
    a.qn[o] = q * rsqrtf(sq / GDN_D + 1e-6f) * (1.f / GDN_D);
    a.kn[o] = k * rsqrtf(sk / GDN_D + 1e-6f) * rsqrtf((float)GDN_D);
  } else {
    const int h = grp - a.nk;
    a.vv[((int64_t)t * a.nv + h) * GDN_D + i] = gdn_conv(a, p0, t, 2 * a.nk * GDN_D + h * GDN_D + i);
    float av = 0.f, bv = 0.f;
    if (!a.ab)  // the two gate rows of this head against the token's input
      dot2_rows(a.x + (int64_t)t * a.xs, a.abw + (int64_t)h * a.hidden, a.abw + (int64_t)(a.nv + h) * a.hidden,
                a.hidden, red, av, bv);
    if (i == 0) {
      if (a.ab) {
        av = __half2float(a.ab[(int64_t)t * a.abs + h]);
        bv = __half2float(a.ab[(int64_t)t * a.abs + a.nv + h]);
      }
      gdn_gates(a, h, av, bv, a.gdec[(int64_t)t * a.nv + h], a.beta[(int64_t)t * a.nv + h]);
    }
  }
}

__global__ void __launch_bounds__(GDN_D) gdn_scan_kernel(GdnArgs a) {
  __shared__ float qs[2][GDN_D], ks[2][GDN_D];
  pdl_launch_dependents();
  pdl_wait();
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
  // completed): the last (up to) four inputs go to their positions' slots.
  const int64_t nthr = (int64_t)gridDim.x * gridDim.y * blockDim.x;
  const int64_t gid = ((int64_t)blockIdx.y * gridDim.x + blockIdx.x) * blockDim.x + tid;
  const int p0 = *a.pos;
  for (int64_t c = gid; c < a.C; c += nthr) {
    for (int t = max(0, a.T - 4); t < a.T; t++)
      a.conv_state[(int64_t)((p0 + t) & 3) * a.C + c] = a.proj[(int64_t)t * a.ps + c];
  }
}

// One token (T == 1) of the whole block in one launch, SPLIT CTAs per value
// head h (SPLIT = 4: a thread-block cluster, for few heads x sequences;
// SPLIT = 1: one CTA of 1024 threads per head, for batches that fill the
// GPU anyway -- every CTA of a cluster repeats the head's q/k conv and norms
// and gate dot products, which a large batch pays 4 times).  Every CTA forms
// the q and k channels of key head h % nk (threads 0..127 q, 128..255 k:
// conv, then the rms norms) and the two gate dot products; CTA rank c owns
// value columns COLS c .. COLS c + COLS - 1 (COLS = 128 / SPLIT): thread
// (col = tid / 8, seg = tid % 8) holds column COLS c + col at key indices
// seg, seg + 8, ..., seg + 120 in registers and applies the recurrence
// (8-lane shuffle reductions).  The gated norm needs the sum of y^2 over the
// head's 128 columns: with SPLIT > 1 each CTA posts its columns' sum in
// shared memory and reads the others' through the cluster's distributed
// shared memory.  The conv window slot of this position is written by rank 0
// of the CTAs that own the channels (q/k: h < nk) and is not read by any CTA
// at this position.
// Batched decode: blockIdx.y is the sequence b of the batch, whose token is
// row b of proj / x / ab, whose conv ring and state follow the previous
// sequence's (4*C and nv*128*128 floats), and whose output is row b of out;
// every sequence is at position *pos.
template <int SPLIT>
__global__ void __launch_bounds__(8 * GDN_D / SPLIT) gdn_decode_kernel(const GdnArgs a0) {
  constexpr int GDN_DEC_SPLIT = SPLIT, GDN_DEC_COLS = GDN_D / SPLIT;
  __shared__ float red[32];
  __shared__ float qs[GDN_D], ks[GDN_D], vs[GDN_DEC_COLS];
  __shared__ float part_ss;
  pdl_launch_dependents();
  pdl_wait();
  const int64_t seq = blockIdx.y;
  GdnArgs a = a0;
  a.proj = a0.proj + seq * a0.ps;
  if (a0.ab) a.ab = a0.ab + seq * a0.abs;
  if (a0.x) a.x = a0.x + seq * a0.xs;
  a.conv_state = a0.conv_state + seq * 4 * a0.C;
  a.state = a0.state + seq * a0.nv * GDN_D * GDN_D;
  const int64_t obase = seq * a0.nv * GDN_D;
  const int crank = blockIdx.x % GDN_DEC_SPLIT;  // == %cluster_ctarank (cluster dims SPLIT x 1 x 1)
  const int h = blockIdx.x / GDN_DEC_SPLIT, kh = h % a.nk, tid = threadIdx.x, warp = tid >> 5;
  const int pos = *a.pos;
  const int i = tid & (GDN_D - 1);
  const int cqk = (tid < GDN_D ? 0 : a.nk * GDN_D) + kh * GDN_D + i;
  const int col0 = crank * GDN_DEC_COLS;
  const int cv = 2 * a.nk * GDN_D + h * GDN_D + col0 + tid;  // threads 0..31: this CTA's v channels
  // this thread's state entries first: their loads overlap the conv, norms and gates below
  const int col = tid >> 3, seg = tid & 7;
  const int j = col0 + col;
  float* sp = a.state + ((int64_t)h * GDN_D + j) * GDN_D + seg;
  float S[16];
#pragma unroll
  for (int r = 0; r < 16; r++) S[r] = sp[8 * r];
  const float c = tid < 2 * GDN_D ? gdn_conv(a, pos, 0, cqk) : 0.f;  // threads past 255: state columns only
  const float v = tid < GDN_DEC_COLS ? gdn_conv(a, pos, 0, cv) : 0.f;
  float av = 0.f, bv = 0.f;
  if (a.ab) {
    av = __half2float(a.ab[h]);
    bv = __half2float(a.ab[a.nv + h]);
  } else {
    dot2_rows(a.x, a.abw + (int64_t)h * a.hidden, a.abw + (int64_t)(a.nv + h) * a.hidden, a.hidden, red, av, bv);
  }
  float g, beta;
  gdn_gates(a, h, av, bv, g, beta);
  // q and k norms: warps 0-3 hold q, warps 4-7 k
  float sq = c * c;
#pragma unroll
  for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
  __syncthreads();  // red is free again
  if ((tid & 31) == 0) red[warp] = sq;
  __syncthreads();
  const float part = tid < GDN_D ? red[0] + red[1] + red[2] + red[3] : red[4] + red[5] + red[6] + red[7];
  if (tid < GDN_D) qs[i] = c * rsqrtf(part / GDN_D + 1e-6f) * (1.f / GDN_D);
  else if (tid < 2 * GDN_D) ks[i] = c * rsqrtf(part / GDN_D + 1e-6f) * rsqrtf((float)GDN_D);
  if (tid < GDN_DEC_COLS) vs[tid] = v;
  const int slot = pos & 3;
  if (crank == 0 && h < a.nk && tid < 2 * GDN_D) a.conv_state[(int64_t)slot * a.C + cqk] = a.proj[cqk];
  if (tid < GDN_DEC_COLS) a.conv_state[(int64_t)slot * a.C + cv] = a.proj[cv];
  __syncthreads();

  float kv0 = 0.f, kv1 = 0.f;
#pragma unroll
  for (int r = 0; r < 16; r += 2) {
    S[r] *= g;
    S[r + 1] *= g;
    kv0 = fmaf(S[r], ks[seg + 8 * r], kv0);
    kv1 = fmaf(S[r + 1], ks[seg + 8 * r + 8], kv1);
  }
  float kv = kv0 + kv1;
  kv += __shfl_xor_sync(0xffffffffu, kv, 1);
  kv += __shfl_xor_sync(0xffffffffu, kv, 2);
  kv += __shfl_xor_sync(0xffffffffu, kv, 4);
  const float u = (vs[col] - kv) * beta;
  float y0 = 0.f, y1 = 0.f;
#pragma unroll
  for (int r = 0; r < 16; r += 2) {
    S[r] = fmaf(ks[seg + 8 * r], u, S[r]);
    S[r + 1] = fmaf(ks[seg + 8 * r + 8], u, S[r + 1]);
    y0 = fmaf(S[r], qs[seg + 8 * r], y0);
    y1 = fmaf(S[r + 1], qs[seg + 8 * r + 8], y1);
  }
  float y = y0 + y1;
  y += __shfl_xor_sync(0xffffffffu, y, 1);
  y += __shfl_xor_sync(0xffffffffu, y, 2);
  y += __shfl_xor_sync(0xffffffffu, y, 4);
#pragma unroll
  for (int r = 0; r < 16; r++) sp[8 * r] = S[r];
  // sum of y^2 over this CTA's columns, then over the cluster's CTAs
  const float ss_cta = block_sum(seg == 0 ? y * y : 0.f, red);
  float ss = ss_cta;
  if constexpr (SPLIT > 1) {
    if (tid == 0) part_ss = ss_cta;
    cluster_sync_all();
    ss = 0.f;
#pragma unroll
    for (int q = 0; q < GDN_DEC_SPLIT; q++) ss += ld_shared_cluster_f32(&part_ss, (uint32_t)q);
    cluster_sync_all();  // no CTA leaves while a peer may still read its part_ss
  }
  if (seg == 0) {
    const float z = a.proj[a.C + h * GDN_D + j];
    store_out(a.out, a.dt, obase + (int64_t)h * GDN_D + j, y * rsqrtf(ss / GDN_D + a.eps) * a.norm_w[j] * silu(z));
  }
}

__global__ void __launch_bounds__(GDN_D) gdn_norm_kernel(GdnArgs a) {
  __shared__ float red[32];
  pdl_launch_dependents();
  pdl_wait();
  const int t = blockIdx.x, h = blockIdx.y, i = threadIdx.x;
  const float v = a.o[((int64_t)t * a.nv + h) * GDN_D + i];
  const float ss = block_sum(v * v, red);
  const float z = a.proj[(int64_t)t * a.ps + a.C + h * GDN_D + i];
  store_out(a.out, a.dt, ((int64_t)t * a.nv + h) * GDN_D + i,
            v * rsqrtf(ss / GDN_D + a.eps) * a.norm_w[i] * silu(z));
}

// One decode token of gated GQA attention; CTA = query head, 256 threads =
// head dimensions.  Dynamic shared memory: scores of positions 0..pos.
// Batched decode: blockIdx.y is the sequence b, whose qkv row follows the
// previous sequence's (nq*512 + 2*nkv*256 floats), whose caches follow the
// previous sequence's (max_len*nkv*256 floats each), and whose output is row
// b of out; every sequence is at position *pos.
__global__ void __launch_bounds__(ATT_D) attn_decode_kernel(const float* qkv0, int nq, int nkv, const float* qw,
                                                            const float* kw, float eps, int rot, float theta,
                                                            float* kc0, float* vc0, int max_len, const int* pos_p,
                                                            void* out, int dt) {
  extern __shared__ float sc[];
  __shared__ float red[32];
  __shared__ __align__(16) float qs[ATT_D], ks[ATT_D], vs[ATT_D];
  pdl_launch_dependents();
  pdl_wait();
  const int64_t seq = blockIdx.y;
  const float* qkv = qkv0 + seq * ((int64_t)nq * 2 * ATT_D + (int64_t)nkv * 2 * ATT_D);
  float* kc = kc0 + seq * (int64_t)max_len * nkv * ATT_D;
  float* vc = vc0 + seq * (int64_t)max_len * nkv * ATT_D;
  const int64_t obase = seq * (int64_t)nq * ATT_D;
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

  // Scores: warp w takes positions ATT_U*w.., then 8*ATT_U further on; lane
  // l holds dimensions 8l..8l+7.  ATT_U positions' loads are in flight at once.
  // The current position's key comes from shared memory.
  const int warp = d >> 5, lane = d & 31;
  float qr[8];
#pragma unroll
  for (int e = 0; e < 8; e++) qr[e] = qs[8 * lane + e];
  const float scale = rsqrtf((float)ATT_D);
  for (int s0 = ATT_U * warp; s0 <= pos; s0 += ATT_U * (ATT_D / 32)) {
    float4 k0[ATT_U], k1[ATT_U];
#pragma unroll
    for (int u = 0; u < ATT_U; u++) {
      const int s = min(s0 + u, pos);
      const float* kr = s == pos ? ks : kc + ((int64_t)s * nkv + kvh) * ATT_D;
      k0[u] = *reinterpret_cast<const float4*>(kr + 8 * lane);
      k1[u] = *reinterpret_cast<const float4*>(kr + 8 * lane + 4);
    }
#pragma unroll
    for (int u = 0; u < ATT_U; u++) {
      float p = qr[0] * k0[u].x + qr[1] * k0[u].y + qr[2] * k0[u].z + qr[3] * k0[u].w + qr[4] * k1[u].x +
                qr[5] * k1[u].y + qr[6] * k1[u].z + qr[7] * k1[u].w;
#pragma unroll
      for (int o = 16; o; o >>= 1) p += __shfl_xor_sync(0xffffffffu, p, o);
      if (lane == 0 && s0 + u <= pos) sc[s0 + u] = p * scale;
    }
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

  // Weighted values: warp w takes positions w, w + 8, ... (lane: dimensions
  // 8l..8l+7), then the eight warps' partial sums are added per dimension.
  float acc[8];
#pragma unroll
  for (int e = 0; e < 8; e++) acc[e] = 0.f;
#pragma unroll 8
  for (int s = warp; s <= pos; s += ATT_D / 32) {
    const float* vr = s == pos ? vs : vc + ((int64_t)s * nkv + kvh) * ATT_D;
    const float4 a0 = *reinterpret_cast<const float4*>(vr + 8 * lane);
    const float4 a1 = *reinterpret_cast<const float4*>(vr + 8 * lane + 4);
    const float pr = sc[s];
    acc[0] = fmaf(pr, a0.x, acc[0]);
    acc[1] = fmaf(pr, a0.y, acc[1]);
    acc[2] = fmaf(pr, a0.z, acc[2]);
    acc[3] = fmaf(pr, a0.w, acc[3]);
    acc[4] = fmaf(pr, a1.x, acc[4]);
    acc[5] = fmaf(pr, a1.y, acc[5]);
    acc[6] = fmaf(pr, a1.z, acc[6]);
    acc[7] = fmaf(pr, a1.w, acc[7]);
  }
  __shared__ float part[ATT_D / 32][ATT_D];
#pragma unroll
  for (int e = 0; e < 8; e++) part[warp][8 * lane + e] = acc[e];
  __syncthreads();
  float o = 0.f;
#pragma unroll
  for (int w = 0; w < ATT_D / 32; w++) o += part[w][d];
  store_out(out, dt, obase + (int64_t)h * ATT_D + d, o / l / (1.f + __expf(-gate)));
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
  auto al = [](const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; };
  const bool vec = dim % 4 == 0 && dim <= (int64_t)RMS_THREADS * RMS_MAXV * 4 && al(resid) && al(weight) &&
                   (!delta || al(delta)) && reinterpret_cast<uintptr_t>(out) % (out_dtype == DT_F32 ? 16 : 8) == 0;
  if (vec)
    launch_pdl(rmsnorm_vec_kernel, dim3((unsigned)rows), dim3(RMS_THREADS), 0, (cudaStream_t)stream, resid, delta,
               (int)dim, weight, eps, out, out_dtype);
  else
    launch_pdl(rmsnorm_kernel, dim3((unsigned)rows), dim3(RMS_THREADS), 0, (cudaStream_t)stream, resid, delta, dim,
               weight, eps, out, out_dtype);
  return launched("gsq_rmsnorm");
}

int gsq_silu_mul(const void* gu, int gu_dtype, int64_t rows, int64_t n, int64_t group, void* out, int out_dtype,
                 gsq_stream_t stream) {
  if (!gu || !out) return fail(GSQ_ERR_ARG, "gsq_silu_mul: null pointer");
  if (rows < 0 || n <= 0 || group < 0 || (group > 0 && n % group)) return fail(GSQ_ERR_SIZE, "gsq_silu_mul: bad shape");
  if (!dt_ok(out_dtype) || !dt_ok(gu_dtype)) return fail(GSQ_ERR_ARG, "gsq_silu_mul: bad dtype");
  if (rows == 0) return GSQ_OK;
  // Eight outputs per thread where every 8-value piece is 16-byte aligned.
  const size_t isz = gu_dtype == DT_F32 ? 4 : 2;
  if ((group == 0 || group == 8) && n % 8 == 0 && rows <= 65535 && (2 * n * isz) % 16 == 0 &&
      reinterpret_cast<uintptr_t>(gu) % 16 == 0 && reinterpret_cast<uintptr_t>(out) % 16 == 0) {
    const dim3 grid((unsigned)((n / 8 + 255) / 256), (unsigned)rows);
    cudaStream_t st = (cudaStream_t)stream;
    if (gu_dtype == DT_F16)
      launch_pdl(silu_mul8_kernel<__half>, grid, dim3(256), 0, st, static_cast<const __half*>(gu), n, group, out,
                 out_dtype);
    else if (gu_dtype == DT_BF16)
      launch_pdl(silu_mul8_kernel<__nv_bfloat16>, grid, dim3(256), 0, st, static_cast<const __nv_bfloat16*>(gu), n,
                 group, out, out_dtype);
    else
      launch_pdl(silu_mul8_kernel<float>, grid, dim3(256), 0, st, static_cast<const float*>(gu), n, group, out,
                 out_dtype);
    return launched("gsq_silu_mul");
  }
  const int64_t total = rows * n;
  const unsigned blocks = (unsigned)std::min<int64_t>((total + 255) / 256, 148 * 16);
  launch_pdl(silu_mul_kernel, dim3(blocks), dim3(256), 0, (cudaStream_t)stream, gu, gu_dtype, rows, n, group, out,
             out_dtype);
  return launched("gsq_silu_mul");
}

size_t gsq_gdn_scratch_bytes(int64_t T, int64_t nk, int64_t nv) {
  if (T <= 1 || nk <= 0 || nv <= 0) return 0;  // one token needs none
  const size_t f = sizeof(float);
  return 2 * align16(T * nk * GDN_D * f) + 2 * align16(T * nv * GDN_D * f) + 2 * align16(T * nv * f);
}

}  // extern "C"

namespace {

// gsq_gdn (batch == 1: T tokens of one sequence) and gsq_gdn_batch (T == 1:
// one token of each of `batch` sequences).
int gdn_run(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride, const uint16_t* x,
            int64_t x_stride, const uint16_t* ab_w, int64_t hidden, int64_t T, int64_t nk, int64_t nv,
            float* conv_state, const int32_t* pos, const float* conv_w, const float* A, const float* dt_bias,
            const float* norm_w, float eps, float* state, void* scratch, size_t scratch_bytes, void* out,
            int out_dtype, int64_t batch, gsq_stream_t stream) {
  auto al16 = [](const void* q) { return reinterpret_cast<uintptr_t>(q) % 16 == 0; };
  if (batch < 0 || batch > 65535 || (batch > 1 && T != 1)) return fail(GSQ_ERR_SIZE, "gsq_gdn: bad batch");
  if (batch == 0) return GSQ_OK;
  if (!proj || !conv_state || !pos || !conv_w || !A || !dt_bias || !norm_w || !state || !out)
    return fail(GSQ_ERR_ARG, "gsq_gdn: null pointer");
  if (!ab && (!x || !ab_w || hidden <= 0 || hidden > INT32_MAX || x_stride < hidden))
    return fail(GSQ_ERR_ARG, "gsq_gdn: without ab, x and ab_w are required");
  if (!ab && (hidden % 8 || x_stride % 8 || !al16(x) || !al16(ab_w)))
    return fail(GSQ_ERR_ALIGN, "gsq_gdn: x and ab_w rows must be 16-byte aligned (hidden % 8 == 0)");
  if (T < 0 || T > INT32_MAX / 2 || nk <= 0 || nv <= 0 || nv % nk || nv > 65535 || nk > 65535)
    return fail(GSQ_ERR_SIZE, "gsq_gdn: bad shape (nv must be a multiple of nk)");
  const int64_t C = 2 * nk * GDN_D + nv * GDN_D;
  if (proj_stride < C + nv * GDN_D || (ab && ab_stride < 2 * nv))
    return fail(GSQ_ERR_SIZE, "gsq_gdn: stride too small");
  if (!dt_ok(out_dtype)) return fail(GSQ_ERR_ARG, "gsq_gdn: bad output dtype");
  if (!al16(state)) return fail(GSQ_ERR_ALIGN, "gsq_gdn: state not 16-byte aligned");
  if (T == 0) return GSQ_OK;
  if (T > 1 && (!scratch || scratch_bytes < gsq_gdn_scratch_bytes(T, nk, nv)))
    return fail(GSQ_ERR_WORKSPACE, "gsq_gdn: scratch missing or too small");
  if (T > 1 && !al16(scratch)) return fail(GSQ_ERR_ALIGN, "gsq_gdn: scratch not 16-byte aligned");
  GdnArgs a = {};
  a.proj = proj;
  a.ps = proj_stride;
  a.ab = reinterpret_cast<const __half*>(ab);
  a.abs = ab_stride;
  a.x = reinterpret_cast<const __half*>(x);
  a.xs = x_stride;
  a.abw = reinterpret_cast<const __half*>(ab_w);
  a.hidden = (int)hidden;
  a.T = (int)T;
  a.nk = (int)nk;
  a.nv = (int)nv;
  a.C = (int)C;
  a.conv_state = conv_state;
  a.pos = pos;
  a.conv_w = conv_w;
  a.A = A;
  a.dt_bias = dt_bias;
  a.norm_w = norm_w;
  a.eps = eps;
  a.state = state;
  a.out = out;
  a.dt = out_dtype;
  cudaStream_t st = (cudaStream_t)stream;
  if (T == 1) {
    if (nv * batch < 2 * 148)  // few heads x sequences: 4 CTAs (a cluster) per head
      launch_pdl_cluster(gdn_decode_kernel<4>, dim3((unsigned)(nv * 4), (unsigned)batch), dim3(2 * GDN_D), 4, st, a);
    else
      launch_pdl(gdn_decode_kernel<1>, dim3((unsigned)nv, (unsigned)batch), dim3(8 * GDN_D), 0, st, a);
    return launched("gsq_gdn (one token)");
  }
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
  launch_pdl(gdn_prep_kernel, dim3((unsigned)T, (unsigned)(nk + nv)), dim3(GDN_D), 0, st, a);
  int rc = launched("gsq_gdn (prep)");
  if (rc) return rc;
  launch_pdl(gdn_scan_kernel, dim3((unsigned)nv, GDN_D / GDN_COLS), dim3(GDN_D), 0, st, a);
  if ((rc = launched("gsq_gdn (scan)"))) return rc;
  launch_pdl(gdn_norm_kernel, dim3((unsigned)T, (unsigned)nv), dim3(GDN_D), 0, st, a);
  return launched("gsq_gdn (norm)");
}

}  // namespace

extern "C" {

int gsq_gdn(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride, const uint16_t* x,
            int64_t x_stride, const uint16_t* ab_w, int64_t hidden, int64_t T, int64_t nk, int64_t nv,
            float* conv_state, const int32_t* pos, const float* conv_w, const float* A, const float* dt_bias,
            const float* norm_w, float eps, float* state, void* scratch, size_t scratch_bytes, void* out,
            int out_dtype, gsq_stream_t stream) {
  return gdn_run(proj, proj_stride, ab, ab_stride, x, x_stride, ab_w, hidden, T, nk, nv, conv_state, pos, conv_w, A,
                 dt_bias, norm_w, eps, state, scratch, scratch_bytes, out, out_dtype, 1, stream);
}

int gsq_gdn_batch(const float* proj, int64_t proj_stride, const uint16_t* ab, int64_t ab_stride, const uint16_t* x,
                  int64_t x_stride, const uint16_t* ab_w, int64_t hidden, int64_t batch, int64_t nk, int64_t nv,
                  float* conv_state, const int32_t* pos, const float* conv_w, const float* A, const float* dt_bias,
                  const float* norm_w, float eps, float* state, void* out, int out_dtype, gsq_stream_t stream) {
  return gdn_run(proj, proj_stride, ab, ab_stride, x, x_stride, ab_w, hidden, 1, nk, nv, conv_state, pos, conv_w, A,
                 dt_bias, norm_w, eps, state, nullptr, 0, out, out_dtype, batch, stream);
}

int gsq_attn_decode(const float* qkv, int64_t nq, int64_t nkv, const float* q_norm_w, const float* k_norm_w,
                    float eps, int64_t rot, float theta, float* k_cache, float* v_cache, int64_t max_len,
                    const int32_t* pos, void* out, int out_dtype, gsq_stream_t stream) {
  return gsq_attn_decode_batch(qkv, nq, nkv, q_norm_w, k_norm_w, eps, rot, theta, k_cache, v_cache, max_len, pos,
                               out, out_dtype, 1, stream);
}

int gsq_attn_decode_batch(const float* qkv, int64_t nq, int64_t nkv, const float* q_norm_w, const float* k_norm_w,
                          float eps, int64_t rot, float theta, float* k_cache, float* v_cache, int64_t max_len,
                          const int32_t* pos, void* out, int out_dtype, int64_t batch, gsq_stream_t stream) {
  if (batch < 0 || batch > 65535) return fail(GSQ_ERR_SIZE, "gsq_attn_decode: bad batch");
  if (batch == 0) return GSQ_OK;
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
  if (smem + 12 * 1024 > 48 * 1024) {  // with the static arrays (about 11 KB)
    const cudaError_t e =
        cudaFuncSetAttribute(attn_decode_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return fail(GSQ_ERR_CUDA, "gsq_attn_decode: shared memory attribute");
  }
  launch_pdl(attn_decode_kernel, dim3((unsigned)nq, (unsigned)batch), dim3(ATT_D), smem, st, qkv, (int)nq, (int)nkv,
             q_norm_w,
             k_norm_w, eps, (int)rot, theta, k_cache, v_cache, (int)max_len, pos, out, out_dtype);
  return launched("gsq_attn_decode");
}

}  // extern "C"
