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
//   3. rows:  every table row of the shard is written exactly once (no
//             separate memset of the 2 GB gradient): rows without tokens as
//             zeros, rows with tokens as the fp32 sum of their gradient rows in
//             increasing t (emb_bwd_zero + emb_bwd_tokens).  Summation order is
//             fixed by (ids, t), so the result is bitwise reproducible, unlike
//             the fp32-atomic reference kernel
//             (v7/a12a160cb11b/optimized_kernel.py:34).
#include <cub/device/device_radix_sort.cuh>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "emb_bwd.cuh"

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
      buf[u] = (hit && c < chunks) ? ld_plain(src + c * 8) : make_uint4(0, 0, 0, 0);
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

// keys/values for the sort, plus a bitmap of the shard rows that have tokens
// (zeroed by the caller).
__global__ void __launch_bounds__(256)
emb_bwd_prep(const int64_t* __restrict__ ids, int T, int64_t vocab_lo, int64_t shard_rows,
             int64_t vocab_total, int64_t padding_idx, uint32_t* __restrict__ keys,
             uint32_t* __restrict__ vals, uint32_t* __restrict__ touched, int32_t* status) {
  const int t = blockIdx.x * blockDim.x + threadIdx.x;
  if (t >= T) return;
  const int64_t id = ids[t];
  const bool oob = id < 0 || id >= vocab_total;
  if (oob && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  const int64_t v = id - vocab_lo;
  const bool ok = !oob && id != padding_idx && v >= 0 && v < shard_rows;
  keys[t] = ok ? static_cast<uint32_t>(v) : static_cast<uint32_t>(shard_rows);
  vals[t] = static_cast<uint32_t>(t);
  if (ok && touched) atomicOr(&touched[v >> 5], 1u << (v & 31));
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

// Rows [b*R, min(shard_rows, (b+1)*R)) belong to CTA b.  Thread i owns the
// 4-column groups i, i+256, ... (KPT of them): it reads 8-byte bf16 quads and
// writes 16-byte fp32 quads, so every load and store instruction of a warp is
// one contiguous span (a thread owning 8 columns would write two float4s 32 B
// apart per instruction and half-fill every sector: ~45% slower on B200).
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
  const int quads = D >> 2;

  for (int64_t v = lo; v < hi; ++v) {
    float4 acc[KPT];
#pragma unroll
    for (int k = 0; k < KPT; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
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
      uint2 gv[4][KPT];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (has[j]) {
          const uint16_t* src = grad + static_cast<int64_t>(tok[j]) * D;
#pragma unroll
          for (int k = 0; k < KPT; ++k) {
            const int q = threadIdx.x + k * 256;
            if (q < quads) {
              asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];"
                           : "=r"(gv[j][k].x), "=r"(gv[j][k].y) : "l"(src + q * 4));
            } else {
              gv[j][k] = make_uint2(0, 0);
            }
          }
        }
      }
      // Add in token order.
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        if (has[j]) {
#pragma unroll
          for (int k = 0; k < KPT; ++k) {
            acc[k].x += bf16lo(gv[j][k].x);
            acc[k].y += bf16hi(gv[j][k].x);
            acc[k].z += bf16lo(gv[j][k].y);
            acc[k].w += bf16hi(gv[j][k].y);
          }
        }
      }
    }
    float4* row = reinterpret_cast<float4*>(G + v * static_cast<int64_t>(D));
#pragma unroll
    for (int k = 0; k < KPT; ++k) {
      const int q = threadIdx.x + k * 256;
      if (q < quads) st_stream_f4(row + q, acc[k]);
    }
  }
}

// Default row kernels (widths that are multiples of 8, up to 4096), two
// launches that together write every table row of the shard exactly once:
//
// emb_bwd_zero: every row the bitmap does not mark is zeroed by a grid-stride
//   sweep in 32-byte units with 256-bit stores.  All CTAs write neighbouring
//   addresses at the same time, which on B200 streams at ~6.9 TB/s (a CTA per
//   block of rows reaches ~6.2 TB/s).
// emb_bwd_tokens: many small CTAs, each owning the runs (rows) that start in
//   its slice of kTokPerCta sorted tokens; a run's gradient rows are added in
//   token order in fp32 and the row is written once.  Thousands of CTAs keep
//   enough runs in flight to hide each run's dependent load chain.
constexpr int kTokPerCta = 8;

__global__ void __launch_bounds__(256)
emb_bwd_zero(const uint32_t* __restrict__ touched, float* __restrict__ G, int64_t shard_rows, int D) {
  const int units_row = D >> 3;
  const int64_t total = shard_rows * units_row;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = u / units_row;
    if (__ldg(touched + (row >> 5)) & (1u << (row & 31))) continue;
    asm volatile("st.global.cs.v8.f32 [%0], {%1,%1,%1,%1,%1,%1,%1,%1};" ::"l"(G + u * 8), "f"(0.f)
                 : "memory");
  }
}

// Zero sweep for any width and alignment (scalar stores).
__global__ void __launch_bounds__(256)
emb_bwd_zero_generic(const uint32_t* __restrict__ touched, float* __restrict__ G, int64_t shard_rows,
                     int64_t D) {
  const int64_t total = shard_rows * D;
  for (int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; u < total;
       u += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t row = u / D;
    if (__ldg(touched + (row >> 5)) & (1u << (row & 31))) continue;
    G[u] = 0.f;
  }
}

template <int U>  // 8-float units per thread and row (128 threads)
__global__ void __launch_bounds__(128)
emb_bwd_tokens(const uint32_t* __restrict__ keys, const uint32_t* __restrict__ vals, int T,
               const uint16_t* __restrict__ grad, float* __restrict__ G, int64_t shard_rows, int D) {
  __shared__ int bounds[2];
  const int warp = threadIdx.x >> 5;
  if (warp < 2) {
    // slice start/end moved forward to the first run that starts at or after it
    int sx = static_cast<int>(min(static_cast<int64_t>(T),
                                  (static_cast<int64_t>(blockIdx.x) + warp) * kTokPerCta));
    if (sx > 0 && sx < T && __ldg(keys + sx) == __ldg(keys + sx - 1))
      sx = warp_lower_bound(keys, T, __ldg(keys + sx - 1) + 1);
    if ((threadIdx.x & 31) == 0) bounds[warp] = sx;
  }
  __syncthreads();
  int q = bounds[0];
  const int s1 = bounds[1];
  const int units_row = D >> 3;
  while (q < s1) {
    const uint32_t key = __ldg(keys + q);
    if (key >= static_cast<uint64_t>(shard_rows)) break;  // padding / other shards sort last
    float acc[U][8];
#pragma unroll
    for (int k = 0; k < U; ++k)
#pragma unroll
      for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
    while (q < s1 && __ldg(keys + q) == key) {
      // two tokens per round: both loads in flight, then the in-order adds
      const bool two = q + 1 < s1 && __ldg(keys + q + 1) == key;
      const uint16_t* s0p = grad + static_cast<int64_t>(__ldg(vals + q)) * D;
      const uint16_t* s1p = two ? grad + static_cast<int64_t>(__ldg(vals + q + 1)) * D : s0p;
      uint4 g0[U], g1[U];
#pragma unroll
      for (int k = 0; k < U; ++k) {
        const int c = threadIdx.x + k * 128;
        const bool in = c < units_row;
        g0[k] = in ? ld_stream(s0p + c * 8) : make_uint4(0, 0, 0, 0);
        g1[k] = (in && two) ? ld_stream(s1p + c * 8) : make_uint4(0, 0, 0, 0);
      }
#pragma unroll
      for (int k = 0; k < U; ++k) {
        float f[8];
        unpack8(g0[k], f);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc[k][e] += f[e];
        if (two) {
          unpack8(g1[k], f);
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[k][e] += f[e];
        }
      }
      q += two ? 2 : 1;
    }
    float* row = G + static_cast<int64_t>(key) * D;
#pragma unroll
    for (int k = 0; k < U; ++k) {
      const int c = threadIdx.x + k * 128;
      if (c < units_row)
        asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(row + c * 8),
                     "f"(acc[k][0]), "f"(acc[k][1]), "f"(acc[k][2]), "f"(acc[k][3]), "f"(acc[k][4]),
                     "f"(acc[k][5]), "f"(acc[k][6]), "f"(acc[k][7])
                     : "memory");
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

// A second stream per device for the zero sweep, so it runs while the sort
// and the token kernel run on the caller's stream (joined before returning).
cudaStream_t side_stream() {
  static std::mutex mu;
  static cudaStream_t streams[64] = {};
  const int d = current_device();
  if (d < 0 || d >= 64) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  if (streams[d] == nullptr) {
    cudaStream_t st = nullptr;
    if (cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    streams[d] = st;
  }
  return streams[d];
}

int sort_end_bit(int64_t shard_rows) {
  int b = 0;
  while (b < 32 && (static_cast<uint64_t>(shard_rows) >> b) != 0) ++b;
  return std::max(b, 1);
}

}  // namespace

bool emb_bwd_layout(int64_t T, int64_t shard_rows, EmbBwdLayout* L) {
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
  L->touched = 4 * a;
  L->touched_bytes = align_up(static_cast<size_t>((shard_rows + 31) / 32) * 4, 256);
  L->temp = L->touched + L->touched_bytes;
  L->temp_bytes = align_up(temp_bytes, 256);
  L->total = L->temp + L->temp_bytes;
  return true;
}

int emb_bwd_front(const int64_t* ids, int T, int64_t shard_rows, int64_t D, int64_t vocab_lo,
                  int64_t vocab_total, int64_t padding_idx, float* G, bool zero_sweep,
                  int zero_ctas_per_sm, bool sort_first, char* ws, const EmbBwdLayout& L,
                  int32_t* status, cudaStream_t s, EmbBwdFront* f) {
  auto keys_in = reinterpret_cast<uint32_t*>(ws + L.keys_in);
  auto vals_in = reinterpret_cast<uint32_t*>(ws + L.vals_in);
  auto keys_out = reinterpret_cast<uint32_t*>(ws + L.keys_out);
  auto vals_out = reinterpret_cast<uint32_t*>(ws + L.vals_out);
  auto touched = reinterpret_cast<uint32_t*>(ws + L.touched);
  f->keys = keys_out;
  f->vals = vals_out;
  f->touched = touched;
  f->fork = f->join = nullptr;

  if (cuda_status(cudaMemsetAsync(touched, 0, L.touched_bytes, s)) != FRAG_OK) return FRAG_ERR_CUDA;
  if (T > 0) {
    emb_bwd_prep<<<dim3(static_cast<unsigned>(ceil_div(T, 256))), 256, 0, s>>>(
        ids, T, vocab_lo, shard_rows, vocab_total, padding_idx, keys_in, vals_in, touched, status);
    const int st = check_launch();
    if (st != FRAG_OK) return st;
  }
  auto sort = [&]() -> int {
    if (T <= 0) return FRAG_OK;
    size_t tb = L.temp_bytes;
    return cuda_status(cub::DeviceRadixSort::SortPairs(ws + L.temp, tb, keys_in, keys_out, vals_in,
                                                       vals_out, T, 0, sort_end_bit(shard_rows), s));
  };
  if (sort_first) {
    const int st = sort();
    if (st != FRAG_OK) return st;
  }
  if (zero_sweep) {
    int sms = sm_count();
    if (sms <= 0) sms = 148;
    // The sweep depends only on the bitmap: with tokens to sort (and the
    // sort still to come) it runs on a side stream, forked here and joined
    // by emb_bwd_join; after the sort it runs on `s` itself.
    cudaStream_t zs = (T > 0 && !sort_first) ? side_stream() : nullptr;
    if (zs && (cudaEventCreateWithFlags(&f->fork, cudaEventDisableTiming) != cudaSuccess ||
               cudaEventCreateWithFlags(&f->join, cudaEventDisableTiming) != cudaSuccess)) {
      cudaGetLastError();
      if (f->fork) cudaEventDestroy(f->fork);
      f->fork = f->join = nullptr;
      zs = nullptr;
    }
    if (zs) {
      const int a = cuda_status(cudaEventRecord(f->fork, s));
      const int b = (a == FRAG_OK) ? cuda_status(cudaStreamWaitEvent(zs, f->fork, 0)) : a;
      if (b != FRAG_OK) {
        cudaEventDestroy(f->fork);
        cudaEventDestroy(f->join);
        f->fork = f->join = nullptr;
        return b;
      }
    }
    cudaStream_t on = zs ? zs : s;
    const bool vec = D % 8 == 0 && (reinterpret_cast<uintptr_t>(G) & 31) == 0;
    const int64_t per_thread = vec ? D / 8 : D;
    const int64_t zgrid = std::min<int64_t>(static_cast<int64_t>(sms) * std::max(zero_ctas_per_sm, 1),
                                            std::max<int64_t>(1, ceil_div(shard_rows * per_thread, 256)));
    if (vec) {
      emb_bwd_zero<<<dim3(static_cast<unsigned>(zgrid)), 256, 0, on>>>(touched, G, shard_rows,
                                                                       static_cast<int>(D));
    } else {
      emb_bwd_zero_generic<<<dim3(static_cast<unsigned>(zgrid)), 256, 0, on>>>(touched, G, shard_rows, D);
    }
    int st = check_launch();
    if (zs) {
      // recorded whatever happened above, so the join always has an event
      const int sj = cuda_status(cudaEventRecord(f->join, zs));
      if (st == FRAG_OK) st = sj;
    }
    if (st != FRAG_OK) return st;
  }
  return sort_first ? FRAG_OK : sort();
}

int emb_bwd_join(EmbBwdFront* f, cudaStream_t s, int st) {
  if (f->join) {
    const int sj = cuda_status(cudaStreamWaitEvent(s, f->join, 0));
    if (st == FRAG_OK) st = sj;
  }
  if (f->fork) cudaEventDestroy(f->fork);
  if (f->join) cudaEventDestroy(f->join);
  f->fork = f->join = nullptr;
  return st;
}

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
  EmbBwdLayout L;
  if (!emb_bwd_layout(T, shard_rows, &L)) return 0;
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
  EmbBwdLayout L;
  if (!emb_bwd_layout(T, shard_rows, &L)) return FRAG_ERR_CUDA;
  if (!workspace || workspace_bytes < L.total) return FRAG_ERR_WORKSPACE;
  if (!aligned16(workspace)) return FRAG_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  const int Ti = static_cast<int>(T);
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  auto g = static_cast<const uint16_t*>(grad);

  // Zero sweep + token CTAs: widths that are multiples of 8 up to 4096, rows
  // 32-byte aligned (256-bit stores) and gradient rows 16-byte aligned.  The
  // sweep runs on the side stream while the sort and the token kernel run on
  // `s`.
  const int64_t units = D / 8;
  if (D % 8 == 0 && units <= 4 * 128 && (reinterpret_cast<uintptr_t>(G) & 31) == 0 &&
      (Ti == 0 || aligned16(grad))) {
    EmbBwdFront f;
    // one persistent wave of the sweep (8 x 256 threads per SM; measured
    // faster than several waves of a larger grid, or fewer CTAs per SM)
    int st = emb_bwd_front(ids, Ti, shard_rows, D, vocab_lo, vocab_total, padding_idx, G,
                           /*zero_sweep=*/true, /*zero_ctas_per_sm=*/8, /*sort_first=*/false, ws,
                           L, status, s, &f);
    if (st == FRAG_OK && Ti > 0) {
      const int Di = static_cast<int>(D);
      const dim3 tgrid(static_cast<unsigned>(ceil_div(T, kTokPerCta)));
      if (units <= 128)
        emb_bwd_tokens<1><<<tgrid, 128, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di);
      else if (units <= 256)
        emb_bwd_tokens<2><<<tgrid, 128, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di);
      else
        emb_bwd_tokens<4><<<tgrid, 128, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di);
      st = check_launch();
    }
    return emb_bwd_join(&f, s, st);
  }

  // Fallback row kernels (other widths / alignments): a CTA per block of
  // rows writes every row of its block, so no zero sweep.
  EmbBwdFront f;
  int st = emb_bwd_front(ids, Ti, shard_rows, D, vocab_lo, vocab_total, padding_idx, G,
                         /*zero_sweep=*/false, 0, /*sort_first=*/true, ws, L, status, s, &f);
  st = emb_bwd_join(&f, s, st);
  if (st != FRAG_OK) return st;
  const int64_t quads = D / 4;
  const bool vec = D % 4 == 0 && quads <= 8 * 256 && (Ti == 0 || (reinterpret_cast<uintptr_t>(grad) & 7) == 0) &&
                   aligned16(G);
  int per_sm = 0;
  cudaError_t oe;
  if (!vec) oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, emb_bwd_rows_generic, 256, 0);
  else if (quads <= 256) oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, emb_bwd_rows_vec<1>, 256, 0);
  else if (quads <= 512) oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, emb_bwd_rows_vec<2>, 256, 0);
  else if (quads <= 1024) oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, emb_bwd_rows_vec<4>, 256, 0);
  else oe = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, emb_bwd_rows_vec<8>, 256, 0);
  if (oe != cudaSuccess) {
    cudaGetLastError();
    per_sm = 4;
  }
  const int64_t target =
      std::max<int64_t>(1, std::min<int64_t>(shard_rows, static_cast<int64_t>(sms) * std::max(per_sm, 1)));
  const int64_t rpb = ceil_div(shard_rows, target);
  const dim3 grid(static_cast<unsigned>(ceil_div(shard_rows, rpb)));
  if (vec) {
    const int Di = static_cast<int>(D);
    if (quads <= 256)
      emb_bwd_rows_vec<1><<<grid, 256, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di, rpb);
    else if (quads <= 512)
      emb_bwd_rows_vec<2><<<grid, 256, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di, rpb);
    else if (quads <= 1024)
      emb_bwd_rows_vec<4><<<grid, 256, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di, rpb);
    else
      emb_bwd_rows_vec<8><<<grid, 256, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, Di, rpb);
  } else {
    emb_bwd_rows_generic<<<grid, 256, 0, s>>>(f.keys, f.vals, Ti, g, G, shard_rows, D, rpb);
  }
  return check_launch();
}

}  // extern "C"
