// Common definitions for the packed-GGUF kernels (sm_100a).
//
// Type ids, per-type block geometry, the codebook tables, and thin inline-PTX
// wrappers (mbarrier, bulk async copy, int8 mma.sync, tcgen05).  Everything
// here is device-side plumbing; the per-type decoders live in gsq_exact.cuh
// (bit-exact fp32) and gsq_fast.cuh (int8 entries for the matvec).
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "_gen/gsq_grids.h"

namespace gsq {

// GGML type ids (reference mlx_gsq/gguf/parser.py:26-32).
enum QType : int {
  T_Q2_K = 10, T_Q4_K = 12, T_Q6_K = 14, T_IQ2_XXS = 16, T_IQ2_XS = 17, T_IQ3_XXS = 18,
  T_IQ1_S = 19, T_IQ3_S = 21, T_IQ2_S = 22, T_IQ4_XS = 23, T_IQ1_M = 29,
};

enum DType : int { DT_F32 = 0, DT_F16 = 1, DT_BF16 = 2 };

constexpr int QK = 256;

// Stored bytes per 256-weight block (parser.py:35-42).
__host__ __device__ constexpr int block_bytes(int t) {
  return t == T_Q2_K ? 84 : t == T_Q4_K ? 144 : t == T_Q6_K ? 210 : t == T_IQ2_XXS ? 66
       : t == T_IQ2_XS ? 74 : t == T_IQ3_XXS ? 98 : t == T_IQ1_S ? 50 : t == T_IQ3_S ? 110
       : t == T_IQ2_S ? 82 : t == T_IQ4_XS ? 136 : t == T_IQ1_M ? 56 : -1;
}

// X-macro over the eleven supported types, used for dispatch tables.
#define GSQ_FOR_EACH_QTYPE(X) \
  X(T_IQ1_M) X(T_IQ1_S) X(T_IQ2_XXS) X(T_IQ2_XS) X(T_IQ2_S) X(T_IQ3_XXS) \
  X(T_IQ3_S) X(T_IQ4_XS) X(T_Q2_K) X(T_Q4_K) X(T_Q6_K)

// ---------------------------------------------------------------------------
// Codebooks (int8, exact), generated from gguf-py at build time.
static __device__ __align__(16) const int8_t kGridIQ2XXS[256 * 8] = GSQ_INIT_GRID_IQ2_XXS;
static __device__ __align__(16) const int8_t kGridIQ2XS[512 * 8] = GSQ_INIT_GRID_IQ2_XS;
static __device__ __align__(16) const int8_t kGridIQ2S[1024 * 8] = GSQ_INIT_GRID_IQ2_S;
static __device__ __align__(16) const int8_t kGridIQ3XXS[256 * 4] = GSQ_INIT_GRID_IQ3_XXS;
static __device__ __align__(16) const int8_t kGridIQ3S[512 * 4] = GSQ_INIT_GRID_IQ3_S;
static __device__ __align__(16) const int8_t kGridIQ1S[2048 * 8] = GSQ_INIT_GRID_IQ1_S;
static __device__ __align__(16) const uint8_t kKsigns[128] = GSQ_INIT_KSIGNS;
static __device__ __align__(16) const int8_t kKvalues[16] = GSQ_INIT_KVALUES;

template <int T> struct GridOf { static __device__ const int8_t* ptr() { return nullptr; } static constexpr int entries = 0, width = 0; };
template <> struct GridOf<T_IQ2_XXS> { static __device__ const int8_t* ptr() { return kGridIQ2XXS; } static constexpr int entries = 256, width = 8; };
template <> struct GridOf<T_IQ2_XS> { static __device__ const int8_t* ptr() { return kGridIQ2XS; } static constexpr int entries = 512, width = 8; };
template <> struct GridOf<T_IQ2_S> { static __device__ const int8_t* ptr() { return kGridIQ2S; } static constexpr int entries = 1024, width = 8; };
template <> struct GridOf<T_IQ3_XXS> { static __device__ const int8_t* ptr() { return kGridIQ3XXS; } static constexpr int entries = 256, width = 4; };
template <> struct GridOf<T_IQ3_S> { static __device__ const int8_t* ptr() { return kGridIQ3S; } static constexpr int entries = 512, width = 4; };
template <> struct GridOf<T_IQ1_S> { static __device__ const int8_t* ptr() { return kGridIQ1S; } static constexpr int entries = 2048, width = 8; };
template <> struct GridOf<T_IQ1_M> { static __device__ const int8_t* ptr() { return kGridIQ1S; } static constexpr int entries = 2048, width = 8; };

// ---------------------------------------------------------------------------
// Scalar helpers.
__device__ __forceinline__ float h2f_bits(uint32_t bits) {
  return __half2float(__ushort_as_half((unsigned short)bits));
}

// Byte-granular reads, safe at any alignment (global or shared, generic address).
__device__ __forceinline__ uint32_t rd8(const uint8_t* p) { return *p; }
__device__ __forceinline__ uint32_t rd16u(const uint8_t* p) { return (uint32_t)p[0] | ((uint32_t)p[1] << 8); }
__device__ __forceinline__ uint32_t rd32u(const uint8_t* p) {
  return (uint32_t)p[0] | ((uint32_t)p[1] << 8) | ((uint32_t)p[2] << 16) | ((uint32_t)p[3] << 24);
}

// Reads that rely on a guaranteed minimum alignment of p.
__device__ __forceinline__ uint32_t ld16a2(const uint8_t* p) { return *reinterpret_cast<const uint16_t*>(p); }
__device__ __forceinline__ uint32_t ld32a4(const uint8_t* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ uint32_t ld32a2(const uint8_t* p) {
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return __byte_perm((uint32_t)q[0], (uint32_t)q[1], 0x5410);
}
__device__ __forceinline__ uint2 ld64a8(const uint8_t* p) { return *reinterpret_cast<const uint2*>(p); }
__device__ __forceinline__ uint2 ld64a4(const uint8_t* p) {
  const uint32_t* q = reinterpret_cast<const uint32_t*>(p);
  return make_uint2(q[0], q[1]);
}
__device__ __forceinline__ uint2 ld64a2(const uint8_t* p) {
  const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
  return make_uint2(__byte_perm((uint32_t)q[0], (uint32_t)q[1], 0x5410),
                    __byte_perm((uint32_t)q[2], (uint32_t)q[3], 0x5410));
}

template <typename T> __device__ __forceinline__ float to_f32(T v);
template <> __device__ __forceinline__ float to_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ float to_f32<__half>(__half v) { return __half2float(v); }
template <> __device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 v) { return __bfloat162float(v); }

__device__ __forceinline__ float load_act(const void* base, int dtype, int64_t i) {
  if (dtype == DT_F16) return __half2float(reinterpret_cast<const __half*>(base)[i]);
  if (dtype == DT_BF16) return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(base)[i]);
  return reinterpret_cast<const float*>(base)[i];
}

__device__ __forceinline__ void store_out(void* base, int dtype, int64_t i, float v) {
  if (dtype == DT_F16) reinterpret_cast<__half*>(base)[i] = __float2half_rn(v);
  else if (dtype == DT_BF16) reinterpret_cast<__nv_bfloat16*>(base)[i] = __float2bfloat16_rn(v);
  else reinterpret_cast<float*>(base)[i] = v;
}

// ---------------------------------------------------------------------------
// Shared-memory / async-proxy PTX wrappers.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
               ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity) : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps until the phase
// completes or about `ns` nanoseconds pass, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok) : "r"(smem_u32(bar)), "r"(parity), "r"(ns) : "memory");
  return ok != 0;
}

// Programmatic dependent launch.  A kernel launched with the programmatic
// stream-serialization attribute may start while the previous kernel in the
// stream is still running; pdl_wait() blocks the calling thread until that
// kernel has completed and its memory is visible, so it must precede every
// read of the previous kernel's outputs and every global write.
// pdl_launch_dependents() lets the next kernel start its own prologue.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Error codes a kernel can record in the device status word.
enum DeviceError : int { DEV_OK = 0, DEV_WAIT_TIMEOUT = 1 };

// Spin on an mbarrier phase with a time limit (~2^31 SM cycles, about a
// second).  On expiry it records DEV_WAIT_TIMEOUT in *err and returns false so
// the caller can unwind instead of hanging the GPU.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 20000u)) return true;
    if (clock64() - t0 > (1ll << 31)) {
      if (err) atomicExch(err, DEV_WAIT_TIMEOUT);
      return false;
    }
  }
}

// Atomic add with acquire-release semantics at GPU scope: one round trip
// that publishes the caller's earlier writes and sees the earlier writers'.
__device__ __forceinline__ unsigned atom_add_acq_rel_gpu(unsigned* p, unsigned v) {
  unsigned r;
  asm volatile("atom.add.acq_rel.gpu.global.u32 %0, [%1], %2;" : "=r"(r) : "l"(p), "r"(v) : "memory");
  return r;
}

// Per-thread 16-byte async copy global -> shared (L2 evict-first), tracked by
// commit groups; dst and src must be 16-byte aligned.
__device__ __forceinline__ void cp_async16_stream(void* dst, const void* src, uint64_t policy) {
  asm volatile("cp.async.cg.shared.global.L2::cache_hint [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "l"(policy) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// One-dimensional bulk async copy global -> shared, completing on an mbarrier.
// dst, src and bytes must all be multiples of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)) : "memory");
}

// Same, with an L2 evict-first policy for data that is streamed exactly once.
__device__ __forceinline__ void bulk_g2s_stream(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                                uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
      ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// uint8 (A) x int8 (B) -> int32 tensor-core MMA, m16n8k32, for formats whose
// integer entries are unsigned (0..255).
__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// int8 x int8 -> int32 tensor-core MMA, m16n8k32 (A row-major, B column-major).
// Pure register computation: not volatile, so the compiler may schedule it.
__device__ __forceinline__ void mma_s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm(
      "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

}  // namespace gsq
