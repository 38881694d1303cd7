// embedding.cu — token-embedding gather and its deterministic backward.
//
// Forward (aten.embedding, v7/1e49beb8a123/problem.py:20-23): one warp per
// token copies table[ids[t]] to out[t] with 128-bit loads/stores, all of a
// row's loads issued before its stores.  A vocab shard [vocab_lo,
// vocab_lo + shard_rows) writes zero rows for ids outside the shard, which is
// the masked half of a vocab-parallel embedding (the other half is the
// all-reduce done by the caller).  The copy is bit exact.
//
// Backward (aten.embedding_dense_backward -> fp32, v7/a12a160cb11b/problem.py:16,19):
//   1. prep:  key[t] = shard-local row of ids[t] (or a sentinel that sorts
//             last for padding / out-of-shard ids), val[t] = t
//   2. sort:  stable LSD radix sort of (key, val) — tokens of one row end up
//             contiguous and in increasing t order
//   3. rows:  every table row of the shard is owned by exactly one CTA, which
//             sums that row's token gradients in t order in fp32 registers and
//             writes the row once (zero rows included: no separate memset of
//             the 2 GB gradient).  Summation order is fixed by (ids, t), so the
//             result is bitwise reproducible, unlike the fp32-atomic reference
//             kernel (v7/a12a160cb11b/optimized_kernel.py:34).
#include <cub/device/device_radix_sort.cuh>

#include <algorithm>

#include "common.cuh"

namespace frag {
namespace {

// ------------------------------------------------------------------ forward

template <int UNROLL>
__global__ void __launch_bounds__(256)
emb_fwd_vec(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
            uint16_t* __restrict__ out, int64_t T, int64_t shard_rows, int D,
            int64_t vocab_lo, int64_t vocab_total, int32_t* status) {
  const int lane = threadIdx.x & 31;
  const int64_t t = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (t >= T) return;
  const int64_t id = __ldg(ids + t);
  const bool oob = id < 0 || id >= vocab_total;
  const int64_t v = id - vocab_lo;
  const bool hit = !oob && v >= 0 && v < shard_rows;
  if (oob && lane == 0 && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  const int chunks = D >> 3;
  const uint16_t* src = table + (hit ? v : 0) * static_cast<int64_t>(D);
  uint16_t* dst = out + t * static_cast<int64_t>(D);
  for (int c0 = 0; c0 < chunks; c0 += 32 * UNROLL) {
    uint4 buf[UNROLL];
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int c = c0 + u * 32 + lane;
      buf[u] = (hit && c < chunks) ? ld_stream(src + c * 8) : make_uint4(0, 0, 0, 0);
    }
#pragma unroll
    for (int u = 0; u < UNROLL; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < chunks) st_global(dst + c * 8, buf[u]);
    }
  }
}

__global__ void __launch_bounds__(256)
emb_fwd_generic(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
                uint16_t* __restrict__ out, int64_t T, int64_t shard_rows, int64_t D,
                int64_t vocab_lo, int64_t vocab_total, int32_t* status) {
  const int64_t t = blockIdx.x;
  const int64_t id = ids[t];
  const bool oob = id < 0 || id >= vocab_total;
  const int64_t v = id - vocab_lo;
  const bool hit = !oob && v >= 0 && v < shard_rows;
  if (oob && threadIdx.x == 0 && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  for (int64_t n = threadIdx.x; n < D; n += blockDim.x)
    out[t * D + n] = hit ? table[v * D + n] : static_cast<uint16_t>(0);
}

// ----------------------------------------------------------------- backward

__global__ void __launch_bounds__(256)
emb_bwd_prep(const int64_t* __restrict__ ids, int T, int64_t vocab_lo, int64_t shard_rows,
             int64_t vocab_total, int64_t padding_idx, uint32_t* __restrict__ keys,
             uint32_t* __restrict__ vals, int32_t* status) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int64_t id = ids[t];
  const bool oob = id < 0 || id >= vocab_total;
  if (oob && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  const int64_t v = id - vocab_lo;
  const bool ok = !oob && id != padding_idx && v >= 0 && v < shard_rows;
  keys[t] = ok ? static_cast<uint32_t>(v) : static_cast<uint32_t>(shard_rows);
  vals[t] = static_cast<uint32_t>(t);
}

// First index i in [0, n) with keys[i] >= target (n if none), keys sorted
// ascending.  32-way search: each round probes 31 evenly spaced keys and keeps
// the one interval that must hold the answer, so 32768 keys take 3 rounds.
__device__ int warp_lower_bound(const uint32_t* __restrict__ keys, int n, uint32_t target) {
  const int lane = threadIdx.x & 31;
  int lo = 0, hi = n;
  while (hi - lo > 32) {
    const int64_t span = hi - lo;
    const int pos = lo + static_cast<int>(span * lane / 32);
    const bool less = lane > 0 && keys[pos] < target;
    const int c = __popc(__ballot_sync(0xffffffffu, less));
    const int nlo = (c == 0) ? lo : lo + static_cast<int>(span * c / 32) + 1;
    const int nhi = (c == 31) ? hi : lo + static_cast<int>(span * (c + 1) / 32);
    lo = nlo;
    hi = nhi;
  }
  const bool less = lo + lane < hi && keys[lo + lane] < target;
  return lo + __popc(__ballot_sync(0xffffffffu, less));
}

// Rows [b*R, min(shard_rows, (b+1)*R)) belong to CTA b.  Thread i owns
// 16-byte column chunks i, i+256, ... (KPT of them), so each row is summed in
// registers and written with 128-bit streaming stores.
template <int KPT>
__global__ void __launch_bounds__(256)
emb_bwd_rows_vec(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, int T,
                 const uint16_t* __restrict__ grad, float* __restrict__ G, int64_t shard_rows,
                 int D, int64_t rows_per_block) {
  __shared__ int bounds[2];
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t hi = min(shard_rows, lo + rows_per_block);
  if (lo >= hi) return;
  const int warp = threadIdx.x >> 5;
  if (warp < 2) {
    const int b = warp_lower_bound(keys, T, static_cast<uint32_t>(warp == 0 ? lo : hi));
    if ((threadIdx.x & 31) == 0) bounds[warp] = b;
  }
  __syncthreads();
  int p = bounds[0];
  const int pend = bounds[1];
  const int chunks = D >> 3;

  for (int64_t v = lo; v < hi; ++v) {
    float acc[KPT][8];
#pragma unroll
    for (int k = 0; k < KPT; ++k)
#pragma unroll
      for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;
    // Tokens of row v: keys[p..] == v (uniform across the CTA).
    while (p < pend && keys[p] == static_cast<uint32_t>(v)) {
      // Up to 4 tokens of the run per round: their loads are all issued
      // before the adds, which still happen in token order.
      int tok[4];
      bool has[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        has[j] = p < pend && keys[p] == static_cast<uint32_t>(v);
        tok[j] = has[j] ? static_cast<int>(vals[p]) : 0;
        if (has[j]) ++p;
      }
      uint4 gv[4][KPT];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (has[j]) {
#pragma unroll
          for (int k = 0; k < KPT; ++k) {
            const int c = threadIdx.x + k * 256;
            gv[j][k] = (c < chunks)
                           ? ld_stream(grad + static_cast<int64_t>(tok[j]) * D + c * 8)
                           : make_uint4(0, 0, 0, 0);
          }
        }
      }
      // Add in token order.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (has[j]) {
#pragma unroll
          for (int k = 0; k < KPT; ++k) {
            float f[8];
            unpack8(gv[j][k], f);
#pragma unroll
            for (int i = 0; i < 8; ++i) acc[k][i] += f[i];
          }
        }
      }
    }
    float* row = G + v * static_cast<int64_t>(D);
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int c = threadIdx.x + k * 256;
      if (c < chunks) {
        st_stream_f4(row + c * 8, make_float4(acc[k][0], acc[k][1], acc[k][2], acc[k][3]));
        st_stream_f4(row + c * 8 + 4, make_float4(acc[k][4], acc[k][5], acc[k][6], acc[k][7]));
      }
    }
  }
}

__global__ void __launch_bounds__(256)
emb_bwd_rows_generic(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, int T,
                     const uint16_t* __restrict__ grad, float* __restrict__ G,
                     int64_t shard_rows, int64_t D, int64_t rows_per_block) {
  __shared__ int bounds[2];
  const int64_t lo = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t hi = min(shard_rows, lo + rows_per_block);
  if (lo >= hi) return;
  const int warp = threadIdx.x >> 5;
  if (warp < 2) {
    const int b = warp_lower_bound(keys, T, static_cast<uint32_t>(warp == 0 ? lo : hi));
    if ((threadIdx.x & 31) == 0) bounds[warp] = b;
  }
  __syncthreads();
  int p = bounds[0];
  const int pend = bounds[1];
  for (int64_t v = lo; v < hi; ++v) {
    const int ps = p;
    while (p < pend && keys[p] == static_cast<uint32_t>(v)) ++p;
    for (int64_t n = threadIdx.x; n < D; n += blockDim.x) {
      float acc = 0.f;
      for (int q = ps; q < p; ++q) acc += bf16_to_f(grad[static_cast<int64_t>(vals[q]) * D + n]);
      G[v * D + n] = acc;
    }
  }
}

struct BwdLayout {
  size_t keys_in, vals_in, keys_out, vals_out, temp, temp_bytes, total;
};

int sort_end_bit(int64_t shard_rows) {
  int b = 0;
  while (b < 32 && (static_cast<uint64_t>(shard_rows) >> b) != 0) ++b;
  return std::max(b, 1);
}

bool bwd_layout(int64_t T, int64_t shard_rows, BwdLayout* L) {
  size_t temp_bytes = 0;
  const int n = static_cast<int>(std::max<int64_t>(T, 1));
  if (cub::DeviceRadixSort::SortPairs(nullptr, temp_bytes, static_cast<const uint32_t*>(nullptr),
                                      static_cast<uint32_t*>(nullptr),
                                      static_cast<const uint32_t*>(nullptr),
                                      static_cast<uint32_t*>(nullptr), n, 0,
                                      sort_end_bit(shard_rows)) != cudaSuccess) {
    cudaGetLastError();
    return false;
  }
  const size_t a = align_up(static_cast<size_t>(std::max<int64_t>(T, 1)) * 4, 256);
  L->keys_in = 0;
  L->vals_in = a;
  L->keys_out = 2 * a;
  L->vals_out = 3 * a;
  L->temp = 4 * a;
  L->temp_bytes = align_up(temp_bytes, 256);
  L->total = L->temp + L->temp_bytes;
  return true;
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" {

int frag_embedding_fwd(const int64_t* ids, const void* table, void* out, int64_t T,
                       int64_t shard_rows, int64_t D, int64_t vocab_lo, int64_t vocab_total,
                       int32_t* status, frag_stream_t stream) {
  if (T < 0 || D < 0 || shard_rows < 0 || vocab_total < 0) return FRAG_ERR_INVALID_ARG;
  if (T == 0 || D == 0) return FRAG_OK;
  if (!ids || !out || (shard_rows > 0 && !table)) return FRAG_ERR_INVALID_ARG;
  if (T > 0x7fffffffLL * 8) return FRAG_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  auto tab = static_cast<const uint16_t*>(table);
  auto o = static_cast<uint16_t*>(out);
  const bool vec = D % 8 == 0 && D <= (1 << 30) && aligned16(out) && (!table || aligned16(table));
  if (vec) {
    const dim3 grid(static_cast<unsigned>(ceil_div(T, 8)));
    if (D / 8 >= 32 * 16)
      emb_fwd_vec<16><<<grid, 256, 0, s>>>(ids, tab, o, T, shard_rows, static_cast<int>(D), vocab_lo, vocab_total, status);
    else if (D / 8 >= 32 * 4)
      emb_fwd_vec<4><<<grid, 256, 0, s>>>(ids, tab, o, T, shard_rows, static_cast<int>(D), vocab_lo, vocab_total, status);
    else
      emb_fwd_vec<1><<<grid, 256, 0, s>>>(ids, tab, o, T, shard_rows, static_cast<int>(D), vocab_lo, vocab_total, status);
  } else {
    if (T > 0x7fffffffLL) return FRAG_ERR_SHAPE;
    emb_fwd_generic<<<dim3(static_cast<unsigned>(T)), 256, 0, s>>>(ids, tab, o, T, shard_rows, D, vocab_lo, vocab_total, status);
  }
  return check_launch();
}

size_t frag_embedding_bwd_workspace_bytes(int64_t T, int64_t shard_rows) {
  if (T < 0 || shard_rows < 0 || T > 0x7fffffffLL || shard_rows >= 0xffffffffLL) return 0;
  BwdLayout L;
  if (!bwd_layout(T, shard_rows, &L)) return 0;
  return L.total;
}

int frag_embedding_bwd(const int64_t* ids, const void* grad, float* G, int64_t T,
                       int64_t shard_rows, int64_t D, int64_t vocab_lo, int64_t vocab_total,
                       int64_t padding_idx, void* workspace, size_t workspace_bytes,
                       int32_t* status, frag_stream_t stream) {
  if (T < 0 || D < 0 || shard_rows < 0 || vocab_total < 0) return FRAG_ERR_INVALID_ARG;
  if (shard_rows == 0 || D == 0) return FRAG_OK;
  if (!G || (T > 0 && (!ids || !grad))) return FRAG_ERR_INVALID_ARG;
  if (T > 0x7fffffffLL || shard_rows >= 0xffffffffLL) return FRAG_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  BwdLayout L;
  if (!bwd_layout(T, shard_rows, &L)) return FRAG_ERR_CUDA;
  if (!workspace || workspace_bytes < L.total) return FRAG_ERR_WORKSPACE;
  if (!aligned16(workspace)) return FRAG_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  auto keys_in = reinterpret_cast<uint32_t*>(ws + L.keys_in);
  auto vals_in = reinterpret_cast<uint32_t*>(ws + L.vals_in);
  auto keys_out = reinterpret_cast<uint32_t*>(ws + L.keys_out);
  auto vals_out = reinterpret_cast<uint32_t*>(ws + L.vals_out);
  const int Ti = static_cast<int>(T);

  if (Ti > 0) {
    emb_bwd_prep<<<dim3(static_cast<unsigned>(ceil_div(T, 256))), 256, 0, s>>>(
        ids, Ti, vocab_lo, shard_rows, vocab_total, padding_idx, keys_in, vals_in, status);
    int st = check_launch();
    if (st != FRAG_OK) return st;
    size_t tb = L.temp_bytes;
    if (cuda_status(cub::DeviceRadixSort::SortPairs(ws + L.temp, tb, keys_in, keys_out, vals_in,
                                                    vals_out, Ti, 0, sort_end_bit(shard_rows),
                                                    s)) != FRAG_OK)
      return FRAG_ERR_CUDA;
  }

  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const int64_t target = std::max<int64_t>(1, std::min<int64_t>(shard_rows, static_cast<int64_t>(sms) * 8));
  const int64_t rpb = ceil_div(shard_rows, target);
  const dim3 grid(static_cast<unsigned>(ceil_div(shard_rows, rpb)));
  auto g = static_cast<const uint16_t*>(grad);
  const int64_t chunks = D / 8;
  const bool vec = D % 8 == 0 && chunks <= 8 * 256 && (Ti == 0 || aligned16(grad)) && aligned16(G);
  if (vec) {
    const int Di = static_cast<int>(D);
    if (chunks <= 256)
      emb_bwd_rows_vec<1><<<grid, 256, 0, s>>>(keys_out, vals_out, Ti, g, G, shard_rows, Di, rpb);
    else if (chunks <= 512)
      emb_bwd_rows_vec<2><<<grid, 256, 0, s>>>(keys_out, vals_out, Ti, g, G, shard_rows, Di, rpb);
    else if (chunks <= 1024)
      emb_bwd_rows_vec<4><<<grid, 256, 0, s>>>(keys_out, vals_out, Ti, g, G, shard_rows, Di, rpb);
    else
      emb_bwd_rows_vec<8><<<grid, 256, 0, s>>>(keys_out, vals_out, Ti, g, G, shard_rows, Di, rpb);
  } else {
    emb_bwd_rows_generic<<<grid, 256, 0, s>>>(keys_out, vals_out, Ti, g, G, shard_rows, D, rpb);
  }
  return check_launch();
}

}  // extern "C"
