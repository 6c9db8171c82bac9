// Bit-exact dequantization and packed embedding gather, sm_100a.
//
// gsq_dequant replaces the reference's decode-only Metal kernels
// (mlx_gsq/runtime/kernels/k_decode.py, iq_lookup_decode.py, iq3_s_decode.py;
// dispatched by registry.decode, registry.py:28-32): packed blocks -> flat
// fp32, identical bits to gguf-py.  gsq_embed replaces iq2_s_embedding
// (mlx_gsq/runtime/kernels/embedding.py:9-36) for all eleven types: out[t, :]
// = deq(W)[ids[t], :], rounded once to the output dtype.
//
// One thread decodes one 8-weight entry and writes it with two 16-byte
// stores; both kernels are bound by the output bytes they write.
#include <algorithm>
#include <type_traits>

#include "gsq_exact.cuh"
#include "gsq_host.h"

namespace gsq {

template <int T>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ packed, int64_t n_entries,
                                                      float* __restrict__ out) {
  constexpr int BB = block_bytes(T);
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n_entries;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t blk = e >> 5;
    const int i = (int)(e & 31);
    float o[8];
    Exact<T>::entry(packed + blk * BB, i, o);
    float4* dst = reinterpret_cast<float4*>(out + e * 8);
    dst[0] = make_float4(o[0], o[1], o[2], o[3]);
    dst[1] = make_float4(o[4], o[5], o[6], o[7]);
  }
}

template <int T, typename OutT>
__global__ void __launch_bounds__(256) embed_kernel(const int32_t* __restrict__ ids, int64_t T_, const uint8_t* __restrict__ packed,
                                                    int64_t vocab, int64_t dim, OutT* __restrict__ out, int* err) {
  constexpr int BB = block_bytes(T);
  const int64_t epr = dim / 8;  // entries per row
  const int64_t total = T_ * epr;
  for (int64_t e = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < total;
       e += (int64_t)gridDim.x * blockDim.x) {
    const int64_t t = e / epr, f8 = e - t * epr;
    const int32_t id = ids[t];
    OutT* dst = out + t * dim + f8 * 8;
    if (id < 0 || id >= vocab) {
      if (err) atomicExch(err, 2);
      continue;
    }
    const int64_t blk = (int64_t)id * (dim / QK) + (f8 >> 5);
    float o[8];
    Exact<T>::entry(packed + blk * BB, (int)(f8 & 31), o);
    if constexpr (sizeof(OutT) == 4) {
      reinterpret_cast<float4*>(dst)[0] = make_float4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<float4*>(dst)[1] = make_float4(o[4], o[5], o[6], o[7]);
    } else {
      OutT h[8];
#pragma unroll
      for (int j = 0; j < 8; j++) {
        if constexpr (sizeof(OutT) == 2 && std::is_same<OutT, __half>::value) h[j] = __float2half_rn(o[j]);
        else h[j] = __float2bfloat16_rn(o[j]);
      }
      *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(h);
    }
  }
}

static int grid_for(int64_t work, int threads) {
  int64_t b = (work + threads - 1) / threads;
  const int64_t cap = 148LL * 16;
  return (int)std::max<int64_t>(1, std::min(b, cap));
}

#define GSQ_DEQ_CASE(TT)                                                          \
  case TT:                                                                        \
    dequant_kernel<TT><<<grid_for(n_entries, 256), 256, 0, st>>>(packed, n_entries, out); \
    return cudaGetLastError();

cudaError_t dequant_launch(int t, const uint8_t* packed, int64_t nblocks, float* out, cudaStream_t st) {
  const int64_t n_entries = nblocks * 32;
  if (n_entries == 0) return cudaSuccess;
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_DEQ_CASE) }
  return cudaErrorInvalidValue;
}

template <int T>
static cudaError_t embed_t(const int32_t* ids, int64_t n, const uint8_t* packed, int64_t vocab, int64_t dim,
                           void* out, int dtype, int* err, cudaStream_t st) {
  const int grid = grid_for(n * (dim / 8), 256);
  if (dtype == DT_F16)
    embed_kernel<T, __half><<<grid, 256, 0, st>>>(ids, n, packed, vocab, dim, (__half*)out, err);
  else if (dtype == DT_BF16)
    embed_kernel<T, __nv_bfloat16><<<grid, 256, 0, st>>>(ids, n, packed, vocab, dim, (__nv_bfloat16*)out, err);
  else
    embed_kernel<T, float><<<grid, 256, 0, st>>>(ids, n, packed, vocab, dim, (float*)out, err);
  return cudaGetLastError();
}

#define GSQ_EMB_CASE(TT) \
  case TT:               \
    return embed_t<TT>(ids, n, packed, vocab, dim, out, dtype, err, st);

cudaError_t embed_launch(int t, const int32_t* ids, int64_t n, const uint8_t* packed, int64_t vocab, int64_t dim,
                         void* out, int dtype, int* err, cudaStream_t st) {
  if (n == 0) return cudaSuccess;
  switch (t) { GSQ_FOR_EACH_QTYPE(GSQ_EMB_CASE) }
  return cudaErrorInvalidValue;
}

}  // namespace gsq
