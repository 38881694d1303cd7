// peer_dweight.cu — the data-parallel dweight exchange of the RMSNorm
// backward over NVLink peer memory.
//
// With rows sharded over W ranks every rank ends its backward with an fp32
// dweight over its own rows, and every rank needs the sum.  The vector is
// 16-32 KB, so an NCCL all-gather costs its launch and protocol latency
// (~25 us measured at 2 ranks), far more than moving the bytes.  Here one CTA
// per rank does the whole exchange:
//   entry  every rank writes `epoch` into slot [0][rank] of every rank's flag
//          block and waits for all W (no rank overwrites a slot row that a
//          peer's previous call may still be summing);
//   store  its dweight into row `rank` of every rank's [W, N] slot buffer
//          (plain 16-byte peer stores), then fence at system scope;
//   exit   writes `epoch` into slot [1][rank] of every flag block and waits
//          for all W;
//   sum    dw_out[n] = sum over r = 0..W-1 of slots[r][n], in rank order.
// The sum adds the same W vectors in the same order on every rank, so every
// rank gets the same bits, and they equal a fixed-order dw_reduce of the
// gathered [W, N] block.  Every wait is bounded (~2 s): on expiry the kernel
// sets FRAG_DEVFLAG_WAIT_TIMEOUT in the library's error word and returns
// without writing dw_out.  The call count (the epoch the flags are compared
// against) lives in this rank's device state word and advances in the kernel,
// so the launch has no per-call arguments and can be captured in a graph.
#include <cuda_runtime.h>

#include "common.cuh"

namespace frag {
namespace {

struct PeerSlots {
  float* slots[FRAG_PEER_MAX_RANKS];    // each rank's [W, N] fp32 rows
  int32_t* flags[FRAG_PEER_MAX_RANKS];  // each rank's [2][W] int32 flags
};

__device__ __forceinline__ void st_release_sys_i32(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys_i32(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Warp-wide: lane q < W signals itself on every rank (lane q writes rank q's
// block) and waits for rank q's signal on this rank.  Returns false (and sets
// the error bit) if any wait ran out.
__device__ bool flag_barrier(const PeerSlots& ps, int slot, int rank, int W, int32_t epoch, int* err) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane < W) {
    st_release_sys_i32(ps.flags[lane] + slot * W + rank, epoch);
    const int32_t* f = ps.flags[rank] + slot * W + lane;
    const long long t0 = clock64();
    while (ld_acquire_sys_i32(f) < epoch) {
      if (clock64() - t0 > kWaitCycles) {
        if (err) atomicOr(err, FRAG_DEVFLAG_WAIT_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

__global__ void __launch_bounds__(1024)
dw_exchange_peer(const float* __restrict__ dw_local, int N, const __grid_constant__ PeerSlots ps,
                 int rank, int W, int32_t* state, float* __restrict__ dw_out, int* err) {
  __shared__ int s_ok, s_epoch;
  if (threadIdx.x == 0) s_epoch = *state + 1;
  __syncthreads();
  const int32_t epoch = s_epoch;
  // every rank advances its count identically, also when a wait gives up
  if (threadIdx.x == 0) *state = epoch;
  if (threadIdx.x < 32) {
    const bool ok = flag_barrier(ps, 0, rank, W, epoch, err);
    if (threadIdx.x == 0) s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const int n4 = N >> 2;
  const float4* src = reinterpret_cast<const float4*>(dw_local);
  for (int i = threadIdx.x; i < n4; i += blockDim.x) {
    const float4 v = src[i];
    for (int j = 1; j <= W; ++j) {  // peers first, this rank's own row last
      float4* dst = reinterpret_cast<float4*>(ps.slots[(rank + j) % W] + static_cast<size_t>(rank) * N);
      dst[i] = v;
    }
  }
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x < 32) {
    const bool ok = flag_barrier(ps, 1, rank, W, epoch, err);
    if (threadIdx.x == 0) s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  const float* own = ps.slots[rank];
  for (int i = threadIdx.x; i < N; i += blockDim.x) {
    float s = 0.f;
    for (int r = 0; r < W; ++r) s += __ldcv(own + static_cast<size_t>(r) * N + i);
    // dw_reduce adds the (zero) sums of its unused warps after the W rows;
    // adding +0 here too keeps the result identical for a -0 column sum
    dw_out[i] = s + 0.0f;
  }
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" int frag_dw_exchange_peer(const float* dw_local, int64_t N, float* const* slot_ptrs,
                                     int32_t* const* flag_ptrs, int32_t* state, int rank, int world,
                                     float* dw_out, frag_stream_t stream) {
  if (world < 1 || world > FRAG_PEER_MAX_RANKS || rank < 0 || rank >= world || !state)
    return FRAG_ERR_INVALID_ARG;
  if (N < 0 || !slot_ptrs || !flag_ptrs || (N > 0 && (!dw_local || !dw_out))) return FRAG_ERR_INVALID_ARG;
  if (N % 4 != 0 || N > (1 << 24)) return FRAG_ERR_SHAPE;
  PeerSlots ps = {};
  for (int r = 0; r < world; ++r) {
    if (!slot_ptrs[r] || !flag_ptrs[r]) return FRAG_ERR_INVALID_ARG;
    if (!aligned16(slot_ptrs[r])) return FRAG_ERR_ALIGN;
    ps.slots[r] = slot_ptrs[r];
    ps.flags[r] = flag_ptrs[r];
  }
  if (N > 0 && !aligned16(dw_local)) return FRAG_ERR_ALIGN;
  dw_exchange_peer<<<1, 1024, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      dw_local, static_cast<int>(N), ps, rank, world, state, dw_out, device_error_word());
  return check_launch();
}
