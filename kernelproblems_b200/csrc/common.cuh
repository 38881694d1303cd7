// common.cuh — helpers shared by the libfrag.so kernels (sm_100a).
//
// bf16 values travel as raw 16-bit patterns packed in uint32/uint4 words so
// every global access is a 128-bit vector op.  Widening bf16 -> fp32 is a
// shift; narrowing uses the hardware round-to-nearest-even conversion.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "frag.h"

namespace frag {

// ---------------------------------------------------------------- host side

// Per-thread record of the last CUDA error seen by an entry point.
void set_last_cuda_error(cudaError_t e);

// Returns FRAG_OK, or FRAG_ERR_CUDA after recording the error.
inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return FRAG_ERR_CUDA;
  }
  return FRAG_OK;
}

inline int cuda_status(cudaError_t e) {
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return FRAG_ERR_CUDA;
  }
  return FRAG_OK;
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

// Number of SMs on the current device (cached per device).
int sm_count();
// Device address of the library's error word on the current device (kernels
// atomicOr FRAG_DEVFLAG_* bits into it), or nullptr if it cannot be found.
int* device_error_word();
// Opt a kernel into `bytes` of dynamic shared memory (once per kernel/device).
bool allow_dynamic_smem(const void* kernel, int bytes);
// Current device ordinal or -1.
int current_device();

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }
inline size_t align_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// ---------------------------------------------------------------- device side

__device__ __forceinline__ float bf16lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float bf16hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
__device__ __forceinline__ float bf16_to_f(uint16_t u) {
  return __uint_as_float(static_cast<uint32_t>(u) << 16);
}

// Two fp32 -> packed bf16x2 (lo in the low half), round to nearest even.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
__device__ __forceinline__ uint16_t f_to_bf16(float f) {
  __nv_bfloat16 v = __float2bfloat16_rn(f);
  return *reinterpret_cast<uint16_t*>(&v);
}
// Round an fp32 value to the nearest bf16 and widen it back.
__device__ __forceinline__ float round_bf16(float f) {
  return bf16_to_f(f_to_bf16(f));
}

// 8 bf16 <-> 8 fp32
__device__ __forceinline__ void unpack8(const uint4& v, float (&f)[8]) {
  f[0] = bf16lo(v.x); f[1] = bf16hi(v.x);
  f[2] = bf16lo(v.y); f[3] = bf16hi(v.y);
  f[4] = bf16lo(v.z); f[5] = bf16hi(v.z);
  f[6] = bf16lo(v.w); f[7] = bf16hi(v.w);
}
__device__ __forceinline__ uint4 pack8(const float (&f)[8]) {
  uint4 v;
  v.x = pack_bf16x2(f[0], f[1]);
  v.y = pack_bf16x2(f[2], f[3]);
  v.z = pack_bf16x2(f[4], f[5]);
  v.w = pack_bf16x2(f[6], f[7]);
  return v;
}

// bf16 pair (lo in the low half) <-> fp32 pair, for the f32x2 arithmetic
// (__fmul2_rn / __ffma2_rn: one instruction for both lanes).
__device__ __forceinline__ float2 bf16x2_to_f2(uint32_t v) {
  return make_float2(__uint_as_float(v << 16), __uint_as_float(v & 0xffff0000u));
}
__device__ __forceinline__ uint32_t f2_to_bf16x2(float2 v) { return pack_bf16x2(v.x, v.y); }
__device__ __forceinline__ uint32_t u4_word(const uint4& v, int q) {
  return q == 0 ? v.x : q == 1 ? v.y : q == 2 ? v.z : v.w;
}

// Streaming 128-bit load: read-only, not kept in L1 (each byte is read once).
__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Plain 128-bit load (the coherent path, default L1 policy).  For the
// streaming reads of the embedding gather, RoPE and residual add + RMSNorm
// kernels it measured faster than ld_stream on B200 (same-box suite A/B:
// gather 9%, RoPE 1.4%, add + RMSNorm 1%); the plain RMSNorm forward and the
// backward kernels measured equal or slower with it and keep ld_stream.
__device__ __forceinline__ uint4 ld_plain(const void* p) {
  uint4 v;
  asm volatile("ld.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
// Cached 128-bit read-only load (data shared by many CTAs: weights, tables).
__device__ __forceinline__ uint4 ld_cached(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}
__device__ __forceinline__ float4 ld_stream_f4(const void* p) {
  float4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.f32 {%0,%1,%2,%3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p));
  return v;
}
// Plain 128-bit store (result is consumed by the next op, keep default policy).
__device__ __forceinline__ void st_global(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}
// Streaming 128-bit store (evict-first: large outputs nobody re-reads soon).
__device__ __forceinline__ void st_stream(void* p, const uint4& v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x),
               "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}
__device__ __forceinline__ void st_stream_f4(void* p, const float4& v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x),
               "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float2 warp_sum2(float2 v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    v.x += __shfl_xor_sync(0xffffffffu, v.x, o);
    v.y += __shfl_xor_sync(0xffffffffu, v.y, o);
  }
  return v;
}

// Block-wide sum in a fixed order (warp butterflies, then warps 0..nw-1 in
// order), result broadcast to every thread.  `slots` is a [2][32] shared
// array; `parity` alternates between consecutive calls so only one barrier
// per call is needed (a warp cannot overwrite a slot another warp still reads:
// it must first pass the barrier of the call in between).
__device__ __forceinline__ float2 block_sum2(float2 v, float2 (*slots)[32], int parity) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum2(v);
  if (lane == 0) slots[parity][warp] = v;
  __syncthreads();
  float2 t = make_float2(0.f, 0.f);
  for (int i = 0; i < nw; ++i) {
    float2 s = slots[parity][i];
    t.x += s.x;
    t.y += s.y;
  }
  return t;
}
__device__ __forceinline__ float block_sum(float v, float (*slots)[32], int parity) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int nw = (blockDim.x + 31) >> 5;
  v = warp_sum(v);
  if (lane == 0) slots[parity][warp] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += slots[parity][i];
  return t;
}

// Elementwise sum of two bf16x2 words rounded to bf16 (ties to even).  The
// fp32 sum of two bf16 values rounded to bf16 (what an aten bf16 add
// computes) is the correctly rounded bf16 sum, which is what the packed bf16
// add gives: the two agree for every input.
__device__ __forceinline__ uint32_t add_bf16x2(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hadd2(*reinterpret_cast<const __nv_bfloat162*>(&a),
                             *reinterpret_cast<const __nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
__device__ __forceinline__ uint4 add_bf16x8(const uint4& a, const uint4& b) {
  return make_uint4(add_bf16x2(a.x, b.x), add_bf16x2(a.y, b.y), add_bf16x2(a.z, b.z),
                    add_bf16x2(a.w, b.w));
}

// Round two fp32 values to the nearest bf16 (ties to even) with one packed
// conversion and widen them back.
__device__ __forceinline__ void round_bf16x2(float& a, float& b) {
  const uint32_t u = pack_bf16x2(a, b);
  a = bf16lo(u);
  b = bf16hi(u);
}

// --------------------------------------------- TMA bulk copies + mbarriers
//
// One-dimensional bulk copies (cp.async.bulk) move whole rows from global to
// shared memory asynchronously; an mbarrier per stage counts the bytes in.
// Every wait is bounded: after kWaitCycles it sets FRAG_DEVFLAG_WAIT_TIMEOUT
// in the error word and returns false instead of spinning forever.

constexpr long long kWaitCycles = 4000000000LL;  // ~2 s at 2 GHz

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
// Arrive without expecting bytes (a stage that receives no copy).
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
      " selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// Wait for phase `parity` of `bar` to complete; false (and the error bit set)
// if it has not after `limit` clock cycles.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err,
                                              long long limit) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - t0 > limit) {
      if (err) atomicOr(err, FRAG_DEVFLAG_WAIT_TIMEOUT);
      return false;
    }
  }
  return true;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, int* err) {
  return mbar_wait_for(bar, parity, err, kWaitCycles);
}
// L2 policy "evict first" for data read once: when the L2 must make room,
// these lines go before others (a clean input line costs no write-back).
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
// bulk_g2s (below) with an L2 cache policy for the source lines.
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                              uint64_t pol) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
      "%4;" ::"r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
      : "memory");
}
// Global -> shared bulk copy of `bytes` (multiple of 16, both addresses
// 16-byte aligned), completing on `bar`.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

}  // namespace frag
