// peer_embedding.cu — vocab-parallel embedding forward fused with its
// exchange over NVLink peer memory.
//
// The vocab-parallel forward (8 contiguous vocab shards, the layout of
// v7/1e49beb8a123/problem.py:16-23 across an 8-rank FSDP group) is usually a
// masked gather followed by an all-reduce of the whole [T, D] output: every
// element is the sum of one table value and W-1 zeros.  Here every token's
// row has exactly one owner, so the owner gathers table_shard[id - lo] once
// and stores it straight into the output buffer of every rank (its own and
// the peers', mapped with CUDA IPC): (W-1)/W of the output crosses NVLink per
// rank instead of a ring all-reduce's 2(W-1)/W, there is no reduction
// arithmetic, and the result is the table row bit for bit (no -0.0 -> +0.0).
//
// Two bounded flag barriers order the ranks (plain peer loads and stores
// only):
//   entry  (one warp) every rank writes `epoch` into slot [0][rank] of every
//          rank's flag block, then waits until all W slots [0][*] of its own
//          block reach `epoch`.  A rank enters call k only after its stream
//          finished everything before it, including reading call k-1's
//          output, so after this barrier no peer still reads the buffer this
//          call writes.
//   exit   every CTA fences its stores (system scope) and counts itself in;
//          the last CTA writes `epoch` into slot [1][rank] of every block
//          and waits for all W slots [1][*] of its own block: when the kernel
//          ends, every peer's rows for this call are in this rank's buffer.
// Every wait gives up after ~2 s of clock cycles, sets
// FRAG_DEVFLAG_WAIT_TIMEOUT in the library's error word and returns.  The
// call count (the epoch the flags are compared against) and the CTA counter
// live in this rank's device state words; the exit barrier's last CTA
// advances the count, so the launches take no per-call arguments and can be
// captured in a graph.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "common.cuh"

namespace frag {
namespace {

struct PeerPtrs {
  uint16_t* out[FRAG_PEER_MAX_RANKS];
  int32_t* flags[FRAG_PEER_MAX_RANKS];
};

__device__ __forceinline__ void st_release_sys(int32_t* p, int32_t v) {
  asm volatile("st.release.sys.global.b32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ int32_t ld_acquire_sys(const int32_t* p) {
  int32_t v;
  asm volatile("ld.acquire.sys.global.b32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Lane q < W waits until own_flags[slot * W + q] >= epoch; false (error bit
// set) after kWaitCycles.
__device__ bool wait_all_ranks(const int32_t* own_flags, int slot, int W, int32_t epoch, int* err) {
  const int lane = threadIdx.x & 31;
  bool ok = true;
  if (lane < W) {
    const int32_t* f = own_flags + slot * W + lane;
    const long long t0 = clock64();
    while (ld_acquire_sys(f) < epoch) {
      if (clock64() - t0 > kWaitCycles) {
        if (err) atomicOr(err, FRAG_DEVFLAG_WAIT_TIMEOUT);
        ok = false;
        break;
      }
    }
  }
  return __all_sync(0xffffffffu, ok);
}

// state[0]: CTA counter of the exit barrier; state[1]: calls completed.
__global__ void vp_entry_barrier(const __grid_constant__ PeerPtrs pp, int rank, int W, const int32_t* state,
                                 int* err) {
  const int32_t epoch = state[1] + 1;
  const int lane = threadIdx.x & 31;
  if (lane < W) st_release_sys(pp.flags[lane] + 0 * W + rank, epoch);
  wait_all_ranks(pp.flags[rank], 0, W, epoch, err);
}

// One warp per token (grid-stride over tokens).  Owned rows are loaded once
// (16-byte loads, all of a lane's loads before its stores) and stored to
// every rank's buffer; ids outside the vocabulary give a zero row, written
// by rank 0, and set FRAG_DEVFLAG_INDEX_OOB.
template <int UNROLL>
__global__ void __launch_bounds__(256)
vp_gather_store(const __grid_constant__ PeerPtrs pp, const int64_t* __restrict__ ids,
                const uint16_t* __restrict__ table, int64_t T, int64_t shard_rows, int D,
                int64_t vocab_lo, int64_t vocab_total, int rank, int W, int32_t* state,
                int32_t* status, int* err) {
  __shared__ int s_last;
  int32_t* counter = state;
  const int32_t epoch = *reinterpret_cast<volatile int32_t*>(state + 1) + 1;
  const int lane = threadIdx.x & 31;
  const int chunks = D >> 3;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x >> 5);
  for (int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5); t < T;
       t += warps) {
    const int64_t id = __ldg(ids + t);
    const bool oob = id < 0 || id >= vocab_total;
    const int64_t v = id - vocab_lo;
    const bool mine = !oob && v >= 0 && v < shard_rows;
    if (oob && lane == 0 && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
    if (!mine && !(oob && rank == 0)) continue;
    const uint16_t* src = table + (mine ? v : 0) * static_cast<int64_t>(D);
    const size_t dst = static_cast<size_t>(t) * D;
    for (int c0 = 0; c0 < chunks; c0 += 32 * UNROLL) {
      uint4 buf[UNROLL];
#pragma unroll
      for (int u = 0; u < UNROLL; ++u) {
        const int c = c0 + u * 32 + lane;
        buf[u] = (mine && c < chunks) ? ld_plain(src + c * 8) : make_uint4(0, 0, 0, 0);
      }
      // the peers' copies first, this rank's own last: rank r starts with
      // peer r+1, so the W writers spread over the W destinations
      for (int j = 1; j <= W; ++j) {
        uint16_t* out = pp.out[(rank + j) % W];
#pragma unroll
        for (int u = 0; u < UNROLL; ++u) {
          const int c = c0 + u * 32 + lane;
          if (c < chunks) st_global(out + dst + c * 8, buf[u]);
        }
      }
    }
  }
  // exit barrier: this CTA's stores are visible system-wide before it counts in
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const int prev = atomicAdd(counter, 1);
    s_last = (prev == static_cast<int>(gridDim.x) - 1);
  }
  __syncthreads();
  if (!s_last || threadIdx.x >= 32) return;
  if (lane == 0) *counter = 0;  // every CTA has counted in: reset for the next call
  __threadfence_system();
  if (lane < W) st_release_sys(pp.flags[lane] + 1 * W + rank, epoch);
  wait_all_ranks(pp.flags[rank], 1, W, epoch, err);
  if (lane == 0) state[1] = epoch;  // this call is complete on this rank
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" {

int frag_peer_alloc(size_t bytes, void** dev_ptr, void* ipc_handle) {
  if (!dev_ptr || !ipc_handle || bytes == 0) return FRAG_ERR_INVALID_ARG;
  *dev_ptr = nullptr;
  void* p = nullptr;
  if (cuda_status(cudaMalloc(&p, bytes)) != FRAG_OK) return FRAG_ERR_CUDA;
  if (cuda_status(cudaMemset(p, 0, bytes)) != FRAG_OK ||
      cuda_status(cudaIpcGetMemHandle(static_cast<cudaIpcMemHandle_t*>(ipc_handle), p)) != FRAG_OK) {
    cudaFree(p);
    return FRAG_ERR_CUDA;
  }
  *dev_ptr = p;
  return FRAG_OK;
}

int frag_peer_open(const void* ipc_handle, void** dev_ptr) {
  if (!dev_ptr || !ipc_handle) return FRAG_ERR_INVALID_ARG;
  *dev_ptr = nullptr;
  cudaIpcMemHandle_t h;
  memcpy(&h, ipc_handle, sizeof(h));
  return cuda_status(cudaIpcOpenMemHandle(dev_ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int frag_peer_close(void* dev_ptr) {
  if (!dev_ptr) return FRAG_ERR_INVALID_ARG;
  return cuda_status(cudaIpcCloseMemHandle(dev_ptr));
}

int frag_peer_free(void* dev_ptr) {
  if (!dev_ptr) return FRAG_ERR_INVALID_ARG;
  return cuda_status(cudaFree(dev_ptr));
}

int frag_embedding_fwd_vp_peer(const int64_t* ids, const void* table_shard, int64_t T,
                               int64_t shard_rows, int64_t D, int64_t vocab_lo, int64_t vocab_total,
                               void* const* out_ptrs, int32_t* const* flag_ptrs, int32_t* state,
                               int rank, int world, int32_t* status, frag_stream_t stream) {
  if (world < 1 || world > FRAG_PEER_MAX_RANKS || rank < 0 || rank >= world) return FRAG_ERR_INVALID_ARG;
  if (T < 0 || shard_rows < 0 || D < 0 || vocab_lo < 0 || vocab_total < 0) return FRAG_ERR_INVALID_ARG;
  if (!out_ptrs || !flag_ptrs || !state || (T > 0 && !ids) || (shard_rows > 0 && !table_shard))
    return FRAG_ERR_INVALID_ARG;
  if (D % 8 != 0 || D > (1 << 20) || T > 0x7fffffffLL) return FRAG_ERR_SHAPE;
  PeerPtrs pp = {};
  for (int r = 0; r < world; ++r) {
    if (!out_ptrs[r] || !flag_ptrs[r]) return FRAG_ERR_INVALID_ARG;
    if (!aligned16(out_ptrs[r])) return FRAG_ERR_ALIGN;
    pp.out[r] = static_cast<uint16_t*>(out_ptrs[r]);
    pp.flags[r] = flag_ptrs[r];
  }
  if (shard_rows > 0 && !aligned16(table_shard)) return FRAG_ERR_ALIGN;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int* err = device_error_word();
  vp_entry_barrier<<<1, 32, 0, s>>>(pp, rank, world, state, err);
  int st = check_launch();
  if (st != FRAG_OK) return st;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const int64_t need = ceil_div(T, 8);  // 8 warps (tokens) per CTA
  // at least one CTA even for T == 0: the exit barrier advances the count
  const unsigned grid = static_cast<unsigned>(
      std::max<int64_t>(1, std::min<int64_t>(need, static_cast<int64_t>(sms) * 8)));
  vp_gather_store<16><<<grid, 256, 0, s>>>(pp, ids, static_cast<const uint16_t*>(table_shard), T,
                                           shard_rows, static_cast<int>(D), vocab_lo, vocab_total,
                                           rank, world, state, status, err);
  return check_launch();
}

}  // extern "C"
