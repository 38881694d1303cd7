// rmsnorm.cu — RMSNorm forward / residual-add + RMSNorm forward / RMSNorm
// backward with a deterministic two-pass dweight, for bf16 rows on sm_100a.
//
// Math follows the fragments' torch reference path:
//   forward  aten._fused_rms_norm   (v8/f4e9e58fef73/problem.py:28)
//            rstd = 1/sqrt(mean(x^2) + eps), y = bf16((x * rstd) * w), fp32 math
//   add      aten.add.Tensor in bf16 (v8/7884328a5557/problem.py:20): h = bf16(res + x)
//   backward torch._decomp _fused_rms_norm_backward (torch 2.11,
//            torch/_decomp/decompositions.py:1862-1933), called by
//            v7/45990c83cfd6/problem.py:23 and v7/7f544ceb2120/problem.py:23-38:
//            xhat = x*rstd, gw = dy*w,
//            dx = (gw - xhat/N * sum(xhat*gw)) * rstd, dw = sum_rows(dy*xhat)
//   The fused backward fragments round the grad sum and dx to bf16 before the
//   residual add (v7/7f544ceb2120/problem.py:23-32), and so do we.
//
// Vector path (N % 8 == 0, 16-byte aligned pointers, N <= 16384): the row is
// held in registers — thread t owns 16-byte chunks t, t+T, ..., so every load
// instruction of a block is one fully coalesced span — and each element is
// read from HBM exactly once.  Generic path: any N, two passes over the row.
#include <algorithm>
#include <mutex>

#include "common.cuh"

namespace frag {
namespace {

struct RowCfg {
  int vpt;      // 16-byte chunks per thread (0 = generic kernel)
  int threads;  // block size, multiple of 32
};

RowCfg pick_row_cfg(int64_t N, bool aligned) {
  // Register-resident rows: at most 512 threads x 4 chunks (N <= 16384), so
  // every thread keeps <= 128 registers without spilling.
  if (!aligned || N % 8 != 0 || N > 16384) return {0, 256};
  const int64_t chunks = N / 8;
  const int vpts[2] = {2, 4};
  for (int vpt : vpts) {
    int64_t t = (chunks + vpt - 1) / vpt;
    t = (t + 31) / 32 * 32;
    if (t <= 512) return {vpt, static_cast<int>(t)};
  }
  return {0, 256};
}

// ------------------------------------------------------------------ forward

template <int VPT, bool HAS_RES, bool WRITE_H, bool WRITE_RSTD>
__global__ void __launch_bounds__(512)
rmsnorm_fwd_vec(const uint16_t* __restrict__ x, const uint16_t* __restrict__ res,
                const uint16_t* __restrict__ w, uint16_t* __restrict__ h,
                uint16_t* __restrict__ y, float* __restrict__ rstd, int N, float eps) {
  __shared__ float slots[2][32];
  const int chunks = N >> 3;
  const int64_t row = blockIdx.x;
  const size_t base = static_cast<size_t>(row) * N;

  uint4 xv[VPT], rv[VPT], wv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      xv[k] = HAS_RES ? ld_plain(x + base + c * 8) : ld_stream(x + base + c * 8);
      if (HAS_RES) rv[k] = ld_plain(res + base + c * 8);
      wv[k] = ld_cached(w + c * 8);
    } else {
      xv[k] = rv[k] = wv[k] = make_uint4(0, 0, 0, 0);
    }
  }

  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    unpack8(xv[k], v[k]);
    if (HAS_RES) {
      float r8[8];
      unpack8(rv[k], r8);
#pragma unroll
      for (int i = 0; i < 8; ++i) v[k][i] = round_bf16(r8[i] + v[k][i]);
      const int c = threadIdx.x + k * blockDim.x;
      if (WRITE_H && c < chunks) st_global(h + base + c * 8, pack8(v[k]));
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[k][i], v[k][i], ss);
  }
  const float tot = block_sum(ss, slots, 0);
  const float r = rsqrtf(tot / static_cast<float>(N) + eps);
  if (WRITE_RSTD && threadIdx.x == 0) rstd[row] = r;

#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      float wf[8], o[8];
      unpack8(wv[k], wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[k][i] * r) * wf[i];
      st_global(y + base + c * 8, pack8(o));
    }
  }
}

// Embedding gather fused with RMSNorm (v8/12545c1e9b06/problem.py:16-51:
// aten.embedding -> aten._fused_rms_norm): the row is read from
// table[ids[row]] and normalised in registers, so the gathered embedding is
// written only when the caller asks for it.  Ids outside [0, V) give a zero
// row and set FRAG_DEVFLAG_INDEX_OOB.
template <int VPT, bool WRITE_EMB, bool WRITE_RSTD>
__global__ void __launch_bounds__(512)
emb_rmsnorm_fwd_vec(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
                    const uint16_t* __restrict__ w, uint16_t* __restrict__ emb,
                    uint16_t* __restrict__ y, float* __restrict__ rstd, int64_t V, int N,
                    float eps, int32_t* status) {
  __shared__ float slots[2][32];
  const int chunks = N >> 3;
  const int64_t row = blockIdx.x;
  const int64_t id = __ldg(ids + row);
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  const uint16_t* src = table + (ok ? id : 0) * static_cast<int64_t>(N);
  const size_t base = static_cast<size_t>(row) * N;
  uint4 xv[VPT], wv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    xv[k] = (ok && c < chunks) ? ld_plain(src + c * 8) : make_uint4(0, 0, 0, 0);
    wv[k] = (c < chunks) ? ld_cached(w + c * 8) : make_uint4(0, 0, 0, 0);
  }
  float v[VPT][8];
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (WRITE_EMB && c < chunks) st_global(emb + base + c * 8, xv[k]);
    unpack8(xv[k], v[k]);
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(v[k][i], v[k][i], ss);
  }
  const float tot = block_sum(ss, slots, 0);
  const float r = rsqrtf(tot / static_cast<float>(N) + eps);
  if (WRITE_RSTD && threadIdx.x == 0) rstd[row] = r;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      float wf[8], o[8];
      unpack8(wv[k], wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) o[i] = (v[k][i] * r) * wf[i];
      st_stream(y + base + c * 8, pack8(o));  // evict-first: 8% faster at C2N
    }
  }
}

template <bool WRITE_EMB, bool WRITE_RSTD>
__global__ void __launch_bounds__(256)
emb_rmsnorm_fwd_generic(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
                        const uint16_t* __restrict__ w, uint16_t* __restrict__ emb,
                        uint16_t* __restrict__ y, float* __restrict__ rstd, int64_t V, int64_t N,
                        float eps, int32_t* status) {
  __shared__ float slots[2][32];
  const int64_t row = blockIdx.x;
  const int64_t id = ids[row];
  const bool ok = id >= 0 && id < V;
  if (!ok && threadIdx.x == 0 && status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
  const uint16_t* src = table + (ok ? id : 0) * N;
  const size_t base = static_cast<size_t>(row) * N;
  float ss = 0.f;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    const uint16_t u = ok ? src[n] : static_cast<uint16_t>(0);
    if (WRITE_EMB) emb[base + n] = u;
    const float v = bf16_to_f(u);
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, slots, 0);
  const float r = rsqrtf(tot / static_cast<float>(N) + eps);
  if (WRITE_RSTD && threadIdx.x == 0) rstd[row] = r;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    const float v = ok ? bf16_to_f(src[n]) : 0.f;
    y[base + n] = f_to_bf16((v * r) * bf16_to_f(w[n]));
  }
}

// The gather + RMSNorm as a bulk-copy ring, for rows of two 8-column chunks
// per thread at up to 256 threads (D <= 4096, the C2 shapes).  CTA b owns the
// rows [b*R, min(T, (b+1)*R)); their ids are staged in shared memory, and
// thread 0 keeps S gathered rows in flight (one cp.async.bulk of the 2D-byte
// table row per ring stage), so the id -> row dependency and the row loads
// overlap the reduction and stores of earlier rows; a row per CTA (above)
// waits for its own id, then its own row, every time.  An out-of-range id
// marks its stage as a zero row, and the stage's barrier completes without
// bytes.  Same per-thread and block summation order as emb_rmsnorm_fwd_vec,
// so the same bits.  Same-box timing at C2 (T = 32768, D = 4096), 3 CTAs per
// SM: 98.3 -> 91.0 us with a clean L2, 103.3 -> 93.6 us with a dirty one
// (2 or 4 CTAs per SM, 128-thread CTAs, two rows per barrier, and a
// register-pipelined version without the ring all measured slower).
constexpr int kEmbRingCps = 3;
constexpr int64_t kEmbRingMaxRows = 1024;  // ids staged per CTA (8 KB)

template <bool WRITE_EMB, bool WRITE_RSTD>
__global__ void __launch_bounds__(256, kEmbRingCps)
emb_rmsnorm_fwd_ring(const int64_t* __restrict__ ids, const uint16_t* __restrict__ table,
                     const uint16_t* __restrict__ w, uint16_t* __restrict__ emb, uint16_t* __restrict__ y,
                     float* __restrict__ rstd, int64_t T, int64_t V, int N, float eps, int64_t rows_per_block,
                     int S, int32_t* status, int* err) {
  constexpr int VPT = 2;
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float slots[2][32];
  __shared__ int s_abort;
  const int row_bytes = N * 2;
  // layout: S row stages | S barriers | the block's ids | S zero-row flags
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * row_bytes);
  int64_t* sid = reinterpret_cast<int64_t*>(bars + S);
  int* okf = reinterpret_cast<int*>(sid + rows_per_block);
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t r1 = min(T, r0 + rows_per_block);
  const int nrows = static_cast<int>(r1 - r0);
  const int chunks = N >> 3;
  for (int i = threadIdx.x; i < nrows; i += blockDim.x) sid[i] = __ldg(ids + r0 + i);
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int i) {  // thread 0: row i into stage i % S
    if (i >= nrows) return;
    const int st = i % S;
    const int64_t id = sid[i];
    const bool ok = id >= 0 && id < V;
    okf[st] = ok ? 1 : 0;
    if (ok) {
      mbar_arrive_expect_tx(&bars[st], row_bytes);
      bulk_g2s(smem + static_cast<size_t>(st) * row_bytes, table + id * static_cast<int64_t>(N), row_bytes,
               &bars[st]);
    } else {
      if (status) atomicOr(status, FRAG_DEVFLAG_INDEX_OOB);
      mbar_arrive(&bars[st]);
    }
    issued = i + 1;
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < S; ++i) issue(i);
  float wf[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    unpack8((c < chunks) ? ld_cached(w + c * 8) : make_uint4(0, 0, 0, 0), wf[k]);
  }
  int parity = 0;
  int i = 0;
  for (; i < nrows; ++i) {
    const int st = i % S;
    if (!mbar_wait(&bars[st], (i / S) & 1, err)) s_abort = 1;
    const bool ok = okf[st] != 0;
    const unsigned char* src = smem + static_cast<size_t>(st) * row_bytes;
    const size_t base = static_cast<size_t>(r0 + i) * N;
    uint4 xv[VPT];
    float v[VPT][8];
    float ss = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      xv[k] = (ok && c < chunks) ? *reinterpret_cast<const uint4*>(src + c * 16) : make_uint4(0, 0, 0, 0);
      unpack8(xv[k], v[k]);
#pragma unroll
      for (int e = 0; e < 8; ++e) ss = fmaf(v[k][e], v[k][e], ss);
    }
    const float tot = block_sum(ss, slots, parity);
    parity ^= 1;
    if (s_abort) break;
    if (threadIdx.x == 0) issue(i + S);  // every thread has read stage st
    const float r = rsqrtf(tot / static_cast<float>(N) + eps);
    if (WRITE_RSTD && threadIdx.x == 0) rstd[r0 + i] = r;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < chunks) {
        if (WRITE_EMB) st_global(emb + base + c * 8, xv[k]);
        float o[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) o[e] = (v[k][e] * r) * wf[k][e];
        st_stream(y + base + c * 8, pack8(o));
      }
    }
  }
  if (threadIdx.x == 0 && s_abort)
    for (int j = i; j < issued; ++j) mbar_wait(&bars[j % S], (j / S) & 1, nullptr);
}

// Launches the ring when the shape fits it; returns -1 (nothing launched)
// when it does not.
template <bool WRITE_EMB, bool WRITE_RSTD>
int launch_emb_rms_ring(const RowCfg& cfg, const int64_t* ids, const uint16_t* table, const uint16_t* w,
                        uint16_t* emb, uint16_t* y, float* rstd, int64_t T, int64_t V, int64_t N, float eps,
                        int32_t* status, cudaStream_t s) {
  if (cfg.vpt != 2 || cfg.threads > 256) return -1;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const int64_t target = std::max<int64_t>(1, std::min<int64_t>(T, static_cast<int64_t>(sms) * kEmbRingCps));
  const int64_t R = ceil_div(T, target);
  if (R > kEmbRingMaxRows) return -1;
  const int64_t G = ceil_div(T, R);
  const int row_bytes = static_cast<int>(N) * 2;
  const int fixed = static_cast<int>(R) * 8 + 1024;  // ids + static shared memory and slack
  const int S = std::min(16, (220 * 1024 / kEmbRingCps - fixed) / (row_bytes + 12));
  if (S < 2) return -1;
  const int smem = S * row_bytes + S * 8 + static_cast<int>(R) * 8 + S * 4;
  auto kern = emb_rmsnorm_fwd_ring<WRITE_EMB, WRITE_RSTD>;
  if (!allow_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) return -1;
  kern<<<dim3(static_cast<unsigned>(G)), cfg.threads, smem, s>>>(ids, table, w, emb, y, rstd, T, V,
                                                                  static_cast<int>(N), eps, R, S, status,
                                                                  device_error_word());
  return check_launch();
}

template <bool WRITE_EMB, bool WRITE_RSTD>
int launch_emb_rms_t(const RowCfg& cfg, const int64_t* ids, const uint16_t* table, const uint16_t* w,
                     uint16_t* emb, uint16_t* y, float* rstd, int64_t T, int64_t V, int64_t N,
                     float eps, int32_t* status, cudaStream_t s) {
  const int rs = launch_emb_rms_ring<WRITE_EMB, WRITE_RSTD>(cfg, ids, table, w, emb, y, rstd, T, V, N, eps,
                                                            status, s);
  if (rs != -1) return rs;
  const dim3 grid(static_cast<unsigned>(T));
  switch (cfg.vpt) {
    case 2:
      emb_rmsnorm_fwd_vec<2, WRITE_EMB, WRITE_RSTD><<<grid, cfg.threads, 0, s>>>(
          ids, table, w, emb, y, rstd, V, static_cast<int>(N), eps, status);
      break;
    case 4:
      emb_rmsnorm_fwd_vec<4, WRITE_EMB, WRITE_RSTD><<<grid, cfg.threads, 0, s>>>(
          ids, table, w, emb, y, rstd, V, static_cast<int>(N), eps, status);
      break;
    default:
      emb_rmsnorm_fwd_generic<WRITE_EMB, WRITE_RSTD><<<grid, 256, 0, s>>>(ids, table, w, emb, y, rstd, V, N,
                                                                           eps, status);
  }
  return check_launch();
}

template <bool HAS_RES, bool WRITE_H, bool WRITE_RSTD>
__global__ void __launch_bounds__(256)
rmsnorm_fwd_generic(const uint16_t* __restrict__ x, const uint16_t* __restrict__ res,
                    const uint16_t* __restrict__ w, uint16_t* __restrict__ h,
                    uint16_t* __restrict__ y, float* __restrict__ rstd, int64_t N, float eps) {
  __shared__ float slots[2][32];
  const int64_t row = blockIdx.x;
  const size_t base = static_cast<size_t>(row) * N;
  float ss = 0.f;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    float v = bf16_to_f(x[base + n]);
    if (HAS_RES) {
      v = round_bf16(bf16_to_f(res[base + n]) + v);
      if (WRITE_H) h[base + n] = f_to_bf16(v);
    }
    ss = fmaf(v, v, ss);
  }
  const float tot = block_sum(ss, slots, 0);
  const float r = rsqrtf(tot / static_cast<float>(N) + eps);
  if (WRITE_RSTD && threadIdx.x == 0) rstd[row] = r;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    float v = bf16_to_f(x[base + n]);
    if (HAS_RES) v = round_bf16(bf16_to_f(res[base + n]) + v);
    y[base + n] = f_to_bf16((v * r) * bf16_to_f(w[n]));
  }
}

template <bool HAS_RES, bool WRITE_H, bool WRITE_RSTD>
int launch_fwd_t(const RowCfg& cfg, const uint16_t* x, const uint16_t* res,
                 const uint16_t* w, uint16_t* h, uint16_t* y, float* rstd,
                 int64_t M, int64_t N, float eps, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(M));
  switch (cfg.vpt) {
    case 2:
      rmsnorm_fwd_vec<2, HAS_RES, WRITE_H, WRITE_RSTD>
          <<<grid, cfg.threads, 0, s>>>(x, res, w, h, y, rstd, static_cast<int>(N), eps);
      break;
    case 4:
      rmsnorm_fwd_vec<4, HAS_RES, WRITE_H, WRITE_RSTD>
          <<<grid, cfg.threads, 0, s>>>(x, res, w, h, y, rstd, static_cast<int>(N), eps);
      break;
    default:
      rmsnorm_fwd_generic<HAS_RES, WRITE_H, WRITE_RSTD>
          <<<grid, 256, 0, s>>>(x, res, w, h, y, rstd, N, eps);
  }
  return check_launch();
}

int launch_fwd(const void* res, const void* x, const void* w, void* h, void* y,
               float* rstd, int64_t M, int64_t N, float eps, cudaStream_t s) {
  if (M < 0 || N < 0) return FRAG_ERR_INVALID_ARG;
  if (M == 0) return FRAG_OK;
  if (!x || !w || !y) return FRAG_ERR_INVALID_ARG;
  if (N == 0 || M > 0x7fffffffLL) return FRAG_ERR_SHAPE;
  bool aligned = aligned16(x) && aligned16(w) && aligned16(y);
  if (res) aligned = aligned && aligned16(res);
  if (h) aligned = aligned && aligned16(h);
  RowCfg cfg = pick_row_cfg(N, aligned);
  // Rows of 2048-4096 elements: four chunks per thread at 64-128 threads
  // (more CTAs resident per SM) measured 9% faster than two at 128-256 at
  // width 4096, and slower at width 8192.
  if (cfg.vpt == 2 && N % 32 == 0 && N >= 2048 && N <= 4096) cfg = RowCfg{4, static_cast<int>(N / 32)};
  auto X = static_cast<const uint16_t*>(x);
  auto R = static_cast<const uint16_t*>(res);
  auto W = static_cast<const uint16_t*>(w);
  auto H = static_cast<uint16_t*>(h);
  auto Y = static_cast<uint16_t*>(y);
  if (!res) {
    return rstd ? launch_fwd_t<false, false, true>(cfg, X, R, W, H, Y, rstd, M, N, eps, s)
                : launch_fwd_t<false, false, false>(cfg, X, R, W, H, Y, rstd, M, N, eps, s);
  }
  if (h) {
    return rstd ? launch_fwd_t<true, true, true>(cfg, X, R, W, H, Y, rstd, M, N, eps, s)
                : launch_fwd_t<true, true, false>(cfg, X, R, W, H, Y, rstd, M, N, eps, s);
  }
  return rstd ? launch_fwd_t<true, false, true>(cfg, X, R, W, H, Y, rstd, M, N, eps, s)
              : launch_fwd_t<true, false, false>(cfg, X, R, W, H, Y, rstd, M, N, eps, s);
}

// ----------------------------------------------------------------- backward

struct BwdIn {
  const uint16_t* dy;
  const uint16_t* dy2;
  const uint16_t* dy3;  // third gradient term (only with dy2), or nullptr
  const uint16_t* x;
  const float* rstd;
  const uint16_t* w;
  const uint16_t* dres;
  uint16_t* dx;
  float* partials;  // [G, N]
  float* rws;       // [M] rstd scratch (generic path)
  // forward recomputed in the backward (FWD kernels only): the normalised
  // input is h = bf16(bf16(x + x2) + x3), y = bf16((h * rstd) * w)
  const uint16_t* x2;  // or nullptr
  const uint16_t* x3;  // or nullptr (only with x2)
  uint16_t* y;         // or nullptr
  float* rstd_out;     // or nullptr
};

// One row block per CTA: rows [b*R, min(M, (b+1)*R)).  The next row's inputs
// are loaded before the current row is reduced, so each thread keeps up to two
// rows of loads in flight; rows stay packed (bf16) in registers and are
// widened on the fly.  dweight partial sums stay in registers (each thread
// owns fixed columns) and are written once per block.
template <int VPT, bool HAS_DY2, bool HAS_DRES, bool RECOMPUTE>
__device__ __forceinline__ void bwd_load_row(const BwdIn& p, int64_t row, int N, int chunks,
                                             uint4 (&dy)[VPT], uint4 (&xx)[VPT],
                                             uint4 (&dy2)[VPT], uint4 (&dy3)[VPT],
                                             uint4 (&dr)[VPT], float& rr) {
  const size_t base = static_cast<size_t>(row) * N;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < chunks) {
      dy[k] = ld_stream(p.dy + base + c * 8);
      xx[k] = ld_stream(p.x + base + c * 8);
      if (HAS_DY2) dy2[k] = ld_stream(p.dy2 + base + c * 8);
      if (HAS_DY2) dy3[k] = p.dy3 ? ld_stream(p.dy3 + base + c * 8) : make_uint4(0, 0, 0, 0);
      if (HAS_DRES) dr[k] = ld_stream(p.dres + base + c * 8);
    } else {
      dy[k] = xx[k] = make_uint4(0, 0, 0, 0);
      if (HAS_DY2) dy2[k] = dy3[k] = make_uint4(0, 0, 0, 0);
      if (HAS_DRES) dr[k] = make_uint4(0, 0, 0, 0);
    }
  }
  if (!RECOMPUTE) rr = __ldg(p.rstd + row);
}

template <int VPT, bool HAS_DY2, bool HAS_DRES, bool RECOMPUTE>
__global__ void __launch_bounds__(512)
rmsnorm_bwd_vec(BwdIn p, int64_t M, int N, float eps, int64_t rows_per_block) {
  __shared__ float2 slots[2][32];
  const int chunks = N >> 3;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t r1 = min(M, r0 + rows_per_block);
  const float invN = 1.0f / static_cast<float>(N);

  float acc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k)
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[k][i] = 0.f;

  uint4 cdy[VPT], cx[VPT], cdy2[VPT], cdy3[VPT], cdr[VPT];
  float cr = 0.f;
  if (r0 < r1) bwd_load_row<VPT, HAS_DY2, HAS_DRES, RECOMPUTE>(p, r0, N, chunks, cdy, cx, cdy2, cdy3, cdr, cr);
  int parity = 0;
  for (int64_t row = r0; row < r1; ++row) {
    uint4 ndy[VPT], nx[VPT], ndy2[VPT], ndy3[VPT], ndr[VPT];
    float nr = 0.f;
    if (row + 1 < r1)
      bwd_load_row<VPT, HAS_DY2, HAS_DRES, RECOMPUTE>(p, row + 1, N, chunks, ndy, nx, ndy2, ndy3, ndr, nr);

    float s1 = 0.f, s2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      const uint4 wv = (c < chunks) ? ld_cached(p.w + c * 8) : make_uint4(0, 0, 0, 0);
      float g[8], xf[8], wf[8];
      unpack8(cdy[k], g);
      if (HAS_DY2) {
        // Each partial sum of the gradients is a bf16 tensor in the graph.
        float g2[8];
        unpack8(cdy2[k], g2);
#pragma unroll
        for (int i = 0; i < 8; ++i) g[i] = g[i] + g2[i];
        cdy[k] = pack8(g);
        unpack8(cdy[k], g);
        if (p.dy3) {
          unpack8(cdy3[k], g2);
#pragma unroll
          for (int i = 0; i < 8; ++i) g[i] = g[i] + g2[i];
          cdy[k] = pack8(g);
          unpack8(cdy[k], g);
        }
      }
      unpack8(cx[k], xf);
      unpack8(wv, wf);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        if (RECOMPUTE) s1 = fmaf(xf[i], xf[i], s1);
        s2 = fmaf(xf[i], g[i] * wf[i], s2);
      }
    }
    const float2 tot = block_sum2(make_float2(s1, s2), slots, parity);
    parity ^= 1;
    const float r = RECOMPUTE ? rsqrtf(tot.x * invN + eps) : cr;
    // mean(xhat * gw) = r * sum(x * gw) / N
    const float cmean = r * tot.y * invN;
    const size_t base = static_cast<size_t>(row) * N;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      const uint4 wv = (c < chunks) ? ld_cached(p.w + c * 8) : make_uint4(0, 0, 0, 0);
      float g[8], xf[8], wf[8], o[8];
      unpack8(cdy[k], g);
      unpack8(cx[k], xf);
      unpack8(wv, wf);
      if (HAS_DRES) unpack8(cdr[k], o);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float xhat = xf[i] * r;
        const float dx = (g[i] * wf[i] - xhat * cmean) * r;
        acc[k][i] = fmaf(g[i], xhat, acc[k][i]);
        o[i] = HAS_DRES ? o[i] + round_bf16(dx) : dx;
      }
      if (c < chunks) st_global(p.dx + base + c * 8, pack8(o));
    }
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      cdy[k] = ndy[k];
      cx[k] = nx[k];
      if (HAS_DY2) cdy2[k] = ndy2[k];
      if (HAS_DY2) cdy3[k] = ndy3[k];
      if (HAS_DRES) cdr[k] = ndr[k];
    }
    cr = nr;
  }

  // Write this block's partials [N] with contiguous 16-byte stores: a warp's
  // 32 chunks (8 floats each) become 64 float4s; lane l stores float4
  // 2*base + l (and + 32), taken from lane l/2 (16 + l/2) by shuffles.
  float4* part = reinterpret_cast<float4*>(p.partials + static_cast<size_t>(blockIdx.x) * N);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int base = (threadIdx.x & ~31) + k * blockDim.x;  // chunk of lane 0
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int src = half * 16 + (lane >> 1);
      float v[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = __shfl_sync(0xffffffffu, acc[k][i], src);
      const bool hi = lane & 1;
      const float4 o = hi ? make_float4(v[4], v[5], v[6], v[7]) : make_float4(v[0], v[1], v[2], v[3]);
      if (base + src < chunks) part[2 * base + half * 32 + lane] = o;
    }
  }
}

// TMA-ring backward: CTA b owns the contiguous rows [b*R, min(M, (b+1)*R))
// (fixed blocks keep the dweight sum order fixed); one thread streams each
// row's inputs (dy, x, then dy2 and dres when present) into a ring of S
// shared-memory stages, S rows ahead.  dweight partials stay in registers and
// are written once per block, coalesced, like the register kernel above.
//
// FWD: the forward recomputed in the same pass (activation checkpointing,
// v6/822931829090/problem.py:19-66): x2 / x3 are streamed with the other
// inputs and summed into h in bf16 before anything else reads the row; rstd
// is recomputed from h and y (and rstd) are stored next to dx.
//
// PLAIN (saved rstd, one gradient, no residual gradient, no fused forward --
// the C1 backward): the per-row arithmetic runs on fp32 pairs (f32x2 multiply
// and fused multiply-add, one instruction for two columns) and the row
// copies carry an L2 evict-first policy, so a fill evicts consumed input
// lines (clean) before others.  Same-box timing of the C1 shape, 8192 x 4096:
// row pass 38.9 -> 34.8 us with a clean L2, unchanged (43 us) with an L2 full
// of another kernel's dirty lines.  The other variants keep the scalar
// arithmetic (packed arithmetic there measured slower: the residual-gradient
// variant 1.235 -> 1.331 ms at the C4 shape).
template <int VPT, bool HAS_DY2, bool HAS_DRES, bool RECOMPUTE, bool FWD = false>
__global__ void __launch_bounds__(512)
rmsnorm_bwd_tma(BwdIn p, int64_t M, int N, float eps, int64_t rows_per_block, int S, int* err) {
  static_assert(!FWD || RECOMPUTE, "the fused forward recomputes rstd");
  constexpr bool PLAIN = !HAS_DY2 && !HAS_DRES && !RECOMPUTE && !FWD;
  // The dweight reduce that follows may be launched now; it waits for this
  // grid to finish before reading the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float2 slots[2][32];
  __shared__ int s_abort;
  const bool has3 = HAS_DY2 && p.dy3 != nullptr;
  const bool hasx2 = FWD && p.x2 != nullptr;
  const bool hasx3 = hasx2 && p.x3 != nullptr;
  // stage layout: dy, x, [dy2], [dy3], [dres], [x2], [x3]
  const int sdres = 2 + (HAS_DY2 ? 1 : 0) + (has3 ? 1 : 0);
  const int sx2 = sdres + (HAS_DRES ? 1 : 0);
  const int nin = sx2 + (hasx2 ? 1 : 0) + (hasx3 ? 1 : 0);
  const int row_bytes = N * 2;
  const int stage_bytes = nin * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * stage_bytes);
  const int chunks = N >> 3;
  const int64_t r0 = static_cast<int64_t>(blockIdx.x) * rows_per_block;
  const int64_t r1 = min(M, r0 + rows_per_block);
  const float invN = 1.0f / static_cast<float>(N);
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  int issued = 0;
  auto issue = [&](int i) {
    const int64_t row = r0 + i;
    if (row >= r1) return;
    unsigned char* st = smem + static_cast<size_t>(i % S) * stage_bytes;
    uint64_t* bar = &bars[i % S];
    const size_t off = static_cast<size_t>(row) * N;
    mbar_arrive_expect_tx(bar, stage_bytes);
    if (PLAIN) {
      const uint64_t pol = l2_policy_evict_first();
      bulk_g2s_hint(st, p.dy + off, row_bytes, bar, pol);
      bulk_g2s_hint(st + row_bytes, p.x + off, row_bytes, bar, pol);
    } else {
      bulk_g2s(st, p.dy + off, row_bytes, bar);
      bulk_g2s(st + row_bytes, p.x + off, row_bytes, bar);
    }
    int slot = 2;
    if (HAS_DY2) bulk_g2s(st + (slot++) * row_bytes, p.dy2 + off, row_bytes, bar);
    if (has3) bulk_g2s(st + (slot++) * row_bytes, p.dy3 + off, row_bytes, bar);
    if (HAS_DRES) bulk_g2s(st + slot * row_bytes, p.dres + off, row_bytes, bar);
    if (hasx2) bulk_g2s(st + sx2 * row_bytes, p.x2 + off, row_bytes, bar);
    if (hasx3) bulk_g2s(st + (sx2 + 1) * row_bytes, p.x3 + off, row_bytes, bar);
    issued = i + 1;
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < S; ++i) issue(i);

  float wf[VPT][8];
  float acc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    unpack8((c < chunks) ? ld_cached(p.w + c * 8) : make_uint4(0, 0, 0, 0), wf[k]);
#pragma unroll
    for (int e = 0; e < 8; ++e) acc[k][e] = 0.f;
  }
  int parity = 0;
  int i = 0;
  for (; r0 + i < r1; ++i) {
    const int64_t row = r0 + i;
    const float rr = RECOMPUTE ? 0.f : __ldg(p.rstd + row);
    const unsigned char* st = smem + static_cast<size_t>(i % S) * stage_bytes;
    if (!mbar_wait(&bars[i % S], (i / S) & 1, err)) s_abort = 1;
    uint4 gdy[VPT], gx[VPT], gdr[VPT];
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < chunks) {
        gdy[k] = *reinterpret_cast<const uint4*>(st + c * 16);
        gx[k] = *reinterpret_cast<const uint4*>(st + row_bytes + c * 16);
        if (FWD && hasx2) {  // h = bf16(bf16(x + x2) + x3): bf16 tensors in the graph
          gx[k] = add_bf16x8(gx[k], *reinterpret_cast<const uint4*>(st + sx2 * row_bytes + c * 16));
          if (hasx3)
            gx[k] = add_bf16x8(gx[k], *reinterpret_cast<const uint4*>(st + (sx2 + 1) * row_bytes + c * 16));
        }
        if (HAS_DY2) {
          // Each partial sum of the gradients is a bf16 tensor in the graph.
          float g[8], g2[8];
          unpack8(gdy[k], g);
          unpack8(*reinterpret_cast<const uint4*>(st + 2 * row_bytes + c * 16), g2);
#pragma unroll
          for (int e = 0; e < 8; ++e) g[e] += g2[e];
          gdy[k] = pack8(g);
          if (has3) {
            unpack8(gdy[k], g);
            unpack8(*reinterpret_cast<const uint4*>(st + 3 * row_bytes + c * 16), g2);
#pragma unroll
            for (int e = 0; e < 8; ++e) g[e] += g2[e];
            gdy[k] = pack8(g);
          }
        }
        if (HAS_DRES)
          gdr[k] = *reinterpret_cast<const uint4*>(st + sdres * row_bytes + c * 16);
      } else {
        gdy[k] = gx[k] = gdr[k] = make_uint4(0, 0, 0, 0);
      }
    }
    float s1 = 0.f, s2 = 0.f;
    if (PLAIN) {
      // sum of x * (g * w): one f32x2 chain per chunk, added in chunk order
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float2 v = make_float2(0.f, 0.f);
#pragma unroll
        for (int q = 0; q < 4; ++q)
          v = __ffma2_rn(bf16x2_to_f2(u4_word(gx[k], q)),
                         __fmul2_rn(bf16x2_to_f2(u4_word(gdy[k], q)), make_float2(wf[k][2 * q], wf[k][2 * q + 1])),
                         v);
        s2 += v.x + v.y;
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        float g[8], xf[8];
        unpack8(gdy[k], g);
        unpack8(gx[k], xf);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          if (RECOMPUTE) s1 = fmaf(xf[e], xf[e], s1);
          s2 = fmaf(xf[e], g[e] * wf[k][e], s2);
        }
      }
    }
    const float2 tot = block_sum2(make_float2(s1, s2), slots, parity);
    parity ^= 1;
    if (s_abort) break;
    if (threadIdx.x == 0) issue(i + S);  // stage i % S is free again
    // the fused forward rounds rstd like the forward kernel (sum / N)
    const float r = FWD ? rsqrtf(tot.x / static_cast<float>(N) + eps)
                        : (RECOMPUTE ? rsqrtf(tot.x * invN + eps) : rr);
    if (FWD && p.rstd_out && threadIdx.x == 0) p.rstd_out[row] = r;
    const float cmean = r * tot.y * invN;  // mean(xhat * gw)
    const size_t base = static_cast<size_t>(row) * N;
    if (PLAIN) {
      // dx = r * (g * w - x * (r * cmean)); dweight += g * (x * r)
      const float2 r2 = make_float2(r, r);
      const float nrc = -(r * cmean);
      const float2 n2 = make_float2(nrc, nrc);
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        uint32_t o[4];
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 g2 = bf16x2_to_f2(u4_word(gdy[k], q));
          const float2 x2 = bf16x2_to_f2(u4_word(gx[k], q));
          const float2 t = __ffma2_rn(x2, n2, __fmul2_rn(g2, make_float2(wf[k][2 * q], wf[k][2 * q + 1])));
          o[q] = f2_to_bf16x2(__fmul2_rn(t, r2));
          const float2 a = __ffma2_rn(g2, __fmul2_rn(x2, r2), make_float2(acc[k][2 * q], acc[k][2 * q + 1]));
          acc[k][2 * q] = a.x;
          acc[k][2 * q + 1] = a.y;
        }
        if (c < chunks) st_global(p.dx + base + c * 8, make_uint4(o[0], o[1], o[2], o[3]));
      }
    } else {
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        float g[8], xf[8], o[8], yv[8];
        unpack8(gdy[k], g);
        unpack8(gx[k], xf);
        if (HAS_DRES) unpack8(gdr[k], o);
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float xhat = xf[e] * r;
          const float dx = (g[e] * wf[k][e] - xhat * cmean) * r;
          acc[k][e] = fmaf(g[e], xhat, acc[k][e]);
          o[e] = HAS_DRES ? o[e] + round_bf16(dx) : dx;
          if (FWD) yv[e] = xhat * wf[k][e];
        }
        if (c < chunks) st_global(p.dx + base + c * 8, pack8(o));
        if (FWD && p.y && c < chunks) st_global(p.y + base + c * 8, pack8(yv));
      }
    }
  }
  if (threadIdx.x == 0 && s_abort)
    for (int j = i; j < issued; ++j) mbar_wait(&bars[j % S], (j / S) & 1, nullptr);

  float4* part = reinterpret_cast<float4*>(p.partials + static_cast<size_t>(blockIdx.x) * N);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int base = (threadIdx.x & ~31) + k * blockDim.x;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int src = half * 16 + (lane >> 1);
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __shfl_sync(0xffffffffu, acc[k][e], src);
      const float4 o = (lane & 1) ? make_float4(v[4], v[5], v[6], v[7]) : make_float4(v[0], v[1], v[2], v[3]);
      if (base + src < chunks) part[2 * base + half * 32 + lane] = o;
    }
  }
}

// The normalised input of element i: x, or with the fused forward
// h = bf16(bf16(x + x2) + x3).
template <bool FWD>
__device__ __forceinline__ float norm_input(const BwdIn& p, size_t i) {
  float h = bf16_to_f(p.x[i]);
  if (FWD && p.x2) {
    h = round_bf16(h + bf16_to_f(p.x2[i]));
    if (p.x3) h = round_bf16(h + bf16_to_f(p.x3[i]));
  }
  return h;
}

// Generic backward, pass 1: dx per row (one CTA per row), rstd copied or
// recomputed into p.rws for pass 2 (with FWD also y and rstd_out).
template <bool HAS_DY2, bool HAS_DRES, bool RECOMPUTE, bool FWD = false>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_generic_dx(BwdIn p, int64_t N, float eps) {
  __shared__ float2 slots[2][32];
  const int64_t row = blockIdx.x;
  const size_t base = static_cast<size_t>(row) * N;
  float s1 = 0.f, s2 = 0.f;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    float g = bf16_to_f(p.dy[base + n]);
    if (HAS_DY2) g = round_bf16(g + bf16_to_f(p.dy2[base + n]));
    if (HAS_DY2 && p.dy3) g = round_bf16(g + bf16_to_f(p.dy3[base + n]));
    const float xf = norm_input<FWD>(p, base + n);
    if (RECOMPUTE) s1 = fmaf(xf, xf, s1);
    s2 = fmaf(xf, g * bf16_to_f(p.w[n]), s2);
  }
  const float2 tot = block_sum2(make_float2(s1, s2), slots, 0);
  const float invN = 1.0f / static_cast<float>(N);
  const float r = FWD ? rsqrtf(tot.x / static_cast<float>(N) + eps)
                      : (RECOMPUTE ? rsqrtf(tot.x * invN + eps) : p.rstd[row]);
  if (threadIdx.x == 0) p.rws[row] = r;
  if (FWD && p.rstd_out && threadIdx.x == 0) p.rstd_out[row] = r;
  const float cmean = r * tot.y * invN;
  for (int64_t n = threadIdx.x; n < N; n += blockDim.x) {
    float g = bf16_to_f(p.dy[base + n]);
    if (HAS_DY2) g = round_bf16(g + bf16_to_f(p.dy2[base + n]));
    if (HAS_DY2 && p.dy3) g = round_bf16(g + bf16_to_f(p.dy3[base + n]));
    const float xhat = norm_input<FWD>(p, base + n) * r;
    const float dx = (g * bf16_to_f(p.w[n]) - xhat * cmean) * r;
    const float o = HAS_DRES ? bf16_to_f(p.dres[base + n]) + round_bf16(dx) : dx;
    p.dx[base + n] = f_to_bf16(o);
    if (FWD && p.y) p.y[base + n] = f_to_bf16(xhat * bf16_to_f(p.w[n]));
  }
}

// Generic backward, pass 2: dweight partials, one thread per column per block.
template <bool HAS_DY2, bool FWD = false>
__global__ void __launch_bounds__(256)
rmsnorm_bwd_generic_dw(BwdIn p, int64_t M, int64_t N, int64_t rows_per_block) {
  const int64_t col = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (col >= N) return;
  const int64_t r0 = static_cast<int64_t>(blockIdx.y) * rows_per_block;
  const int64_t r1 = min(M, r0 + rows_per_block);
  float acc = 0.f;
  for (int64_t row = r0; row < r1; ++row) {
    const size_t i = static_cast<size_t>(row) * N + col;
    float g = bf16_to_f(p.dy[i]);
    if (HAS_DY2) g = round_bf16(g + bf16_to_f(p.dy2[i]));
    if (HAS_DY2 && p.dy3) g = round_bf16(g + bf16_to_f(p.dy3[i]));
    acc = fmaf(g, norm_input<FWD>(p, i) * p.rws[row], acc);
  }
  p.partials[static_cast<size_t>(blockIdx.y) * N + col] = acc;
}

// dw[n] = sum_{b=0}^{G-1} partials[b, n].  A CTA owns 32 columns (one per
// lane); warp w adds the blocks w, w+32, ... in order, then the 32 warp sums
// of a column are added in warp order.  The order is fixed, so the result is
// bitwise reproducible.  Each lane issues all of its (up to 16) loads before
// the first add, so the kernel costs one memory round trip for G <= 512.
__global__ void __launch_bounds__(1024)
dw_reduce_kernel(const float* __restrict__ partials, int64_t G, int64_t N,
                 float* __restrict__ dw, uint16_t* __restrict__ dw_bf16) {
  __shared__ float red[32][33];
  // Launched as a programmatic dependent of the row kernel: wait until that
  // grid has completed and its partials are visible (no-op otherwise).
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t col = static_cast<int64_t>(blockIdx.x) * 32 + lane;
  float a = 0.f;
  if (col < N) {
    for (int64_t b0 = warp; b0 < G; b0 += 32 * 16) {
      float v[16];
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        const int64_t b = b0 + 32 * j;
        v[j] = (b < G) ? __ldg(partials + b * N + col) : 0.f;
      }
#pragma unroll
      for (int j = 0; j < 16; ++j) a += v[j];
    }
  }
  red[warp][lane] = a;
  __syncthreads();
  if (warp == 0 && col < N) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < 32; ++w) s += red[w][lane];
    if (dw) dw[col] = s;
    if (dw_bf16) dw_bf16[col] = f_to_bf16(s);
  }
}

int launch_dw_reduce(const float* partials, int64_t G, int64_t N, float* dw,
                     uint16_t* dw_bf16, cudaStream_t s, bool after_row_kernel = false) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(ceil_div(N, 32)));
  cfg.blockDim = dim3(1024);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  // Directly behind the row kernel: a programmatic dependent launch, so its
  // launch overlaps that kernel's tail.
  cfg.attrs = attr;
  cfg.numAttrs = after_row_kernel ? 1 : 0;
  return cuda_status(cudaLaunchKernelEx(&cfg, dw_reduce_kernel, partials, G, N, dw, dw_bf16));
}

// Row-block plan shared by the workspace query and the launch: the number of
// blocks G is the number of CTAs of the heaviest vector variant that fit on
// the device at once, so the whole grid runs as one wave.
struct BwdPlan {
  RowCfg cfg;
  int64_t G;
  int64_t rows_per_block;
  bool tma = false;  // TMA-ring kernel
  int cps = 0;       // its CTAs per SM (same for every input set)
};

int vec_blocks_per_sm(int vpt, int threads) {
  int n = 0;
  cudaError_t e = cudaSuccess;
  switch (vpt) {
    case 2: e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, rmsnorm_bwd_vec<2, true, true, true>, threads, 0); break;
    default: n = 8;
  }
  if (e != cudaSuccess) {
    cudaGetLastError();
    n = 1;
  }
  return std::max(1, n);
}

BwdPlan make_bwd_plan(int64_t M, int64_t N, bool aligned) {
  BwdPlan pl;
  pl.cfg = pick_row_cfg(N, aligned);
  // The backward keeps two rows of up to four inputs in registers: only the
  // 2-chunks-per-thread variant fits (N <= 8192 at 512 threads).
  if (pl.cfg.vpt != 2) pl.cfg = RowCfg{0, 256};
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  if (pl.cfg.vpt == 2) {
    // TMA ring: CTAs per SM from the register footprint of the heaviest input
    // set (at most 2), the same for every input set (the stage count adapts),
    // so the block count, and with it the partials layout, depends on M, N only.
    int occ = 0;
    const cudaError_t oe =
        pl.cfg.vpt == 1
            ? cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, rmsnorm_bwd_tma<1, true, true, true>,
                                                            pl.cfg.threads, 0)
            : cudaOccupancyMaxActiveBlocksPerMultiprocessor(&occ, rmsnorm_bwd_tma<2, true, true, true>,
                                                            pl.cfg.threads, 0);
    if (oe != cudaSuccess) {
      cudaGetLastError();
      occ = 1;
    }
    pl.tma = true;
    pl.cps = std::max(1, std::min(2, occ));
    const int64_t target = std::max<int64_t>(1, std::min<int64_t>(M, static_cast<int64_t>(pl.cps) * sms));
    pl.rows_per_block = ceil_div(M, target);
    pl.G = ceil_div(M, pl.rows_per_block);
    return pl;
  }
  int64_t target = static_cast<int64_t>(sms) * vec_blocks_per_sm(pl.cfg.vpt, pl.cfg.threads);
  if (pl.cfg.vpt == 0) target = static_cast<int64_t>(sms) * 4;
  target = std::max<int64_t>(1, std::min<int64_t>(target, M));
  pl.rows_per_block = ceil_div(M, target);
  pl.G = ceil_div(M, pl.rows_per_block);
  return pl;
}

size_t bwd_partials_bytes(const BwdPlan& pl, int64_t N) {
  return align_up(static_cast<size_t>(pl.G) * N * sizeof(float), 256);
}
size_t bwd_rstd_copy_bytes(int64_t M) { return align_up(static_cast<size_t>(M) * sizeof(float), 256); }

// What a launch with this plan needs: the [G, N] partials, plus the rstd
// copy (p.rws) that only the generic kernels keep.
size_t bwd_workspace_bytes(const BwdPlan& pl, int64_t M, int64_t N) {
  return bwd_partials_bytes(pl, N) + (pl.tma ? 0 : bwd_rstd_copy_bytes(M));
}

template <bool HAS_DY2, bool HAS_DRES, bool RECOMPUTE, bool FWD = false>
int launch_bwd_t(const BwdPlan& pl, BwdIn p, int64_t M, int64_t N, float eps, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(pl.G));
  const int T = pl.cfg.threads;
  if (pl.tma) {
    const int nx = FWD && p.x2 ? (p.x3 ? 2 : 1) : 0;
    const int nin = 2 + (HAS_DY2 ? 1 : 0) + (HAS_DY2 && p.dy3 ? 1 : 0) + (HAS_DRES ? 1 : 0) + nx;
    const int stage_bytes = nin * static_cast<int>(N) * 2;
    const int S = std::min(8, (220 * 1024 / pl.cps - 1024) / stage_bytes);
    auto kern = pl.cfg.vpt == 1 ? rmsnorm_bwd_tma<1, HAS_DY2, HAS_DRES, RECOMPUTE, FWD>
                                : rmsnorm_bwd_tma<2, HAS_DY2, HAS_DRES, RECOMPUTE, FWD>;
    const int smem = std::max(S, 1) * stage_bytes + 8 * std::max(S, 1);
    if (S >= 1 && allow_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) {
      kern<<<grid, T, smem, s>>>(p, M, static_cast<int>(N), eps, pl.rows_per_block, S,
                                 device_error_word());
      return check_launch();
    }
    // no room for the ring: the register-prefetch kernel on the same blocks
    // (the fused forward takes the generic kernels)
  }
  if (!FWD && pl.cfg.vpt == 2) {
    rmsnorm_bwd_vec<2, HAS_DY2, HAS_DRES, RECOMPUTE><<<grid, T, 0, s>>>(p, M, static_cast<int>(N), eps, pl.rows_per_block);
    return check_launch();
  }
  // the generic kernels keep a copy of rstd after the partials; a caller
  // whose workspace was sized for the ring plan has no room for it
  if (p.rws == nullptr) return FRAG_ERR_WORKSPACE;
  rmsnorm_bwd_generic_dx<HAS_DY2, HAS_DRES, RECOMPUTE, FWD>
      <<<dim3(static_cast<unsigned>(M)), 256, 0, s>>>(p, N, eps);
  int st = check_launch();
  if (st != FRAG_OK) return st;
  const dim3 g2(static_cast<unsigned>(ceil_div(N, 256)), static_cast<unsigned>(pl.G));
  rmsnorm_bwd_generic_dw<HAS_DY2, FWD><<<g2, 256, 0, s>>>(p, M, N, pl.rows_per_block);
  return check_launch();
}

}  // namespace
}  // namespace frag

using namespace frag;

namespace {

// frag_rmsnorm_bwd3 (fwd == false) and frag_rmsnorm_fwd_bwd (fwd == true:
// rstd recomputed from h = x [+ x2 [+ x3]], y / rstd stored when given).
int rmsnorm_bwd_impl(bool fwd, const void* dy, const void* dy2, const void* dy3, const void* x,
                     const void* x2, const void* x3, const float* rstd, const void* w,
                     const void* dres, void* y_out, float* rstd_out, void* dx_out, float* dw,
                     void* dw_bf16, int64_t M, int64_t N, float eps, void* workspace,
                     size_t workspace_bytes, frag_stream_t stream) {
  if (M < 0 || N < 0) return FRAG_ERR_INVALID_ARG;
  if (dy3 && !dy2) return FRAG_ERR_INVALID_ARG;
  if (N == 0 && M > 0) return FRAG_ERR_SHAPE;
  if (M > 0 && (!dy || !x || !w || !dx_out)) return FRAG_ERR_INVALID_ARG;
  if (M > 0x7fffffffLL || N > 0x7fffffffLL) return FRAG_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (M == 0) {
    // Empty batch: dweight is an empty sum.
    if (dw && cuda_status(cudaMemsetAsync(dw, 0, N * sizeof(float), s)) != FRAG_OK)
      return FRAG_ERR_CUDA;
    if (dw_bf16 && cuda_status(cudaMemsetAsync(dw_bf16, 0, N * 2, s)) != FRAG_OK)
      return FRAG_ERR_CUDA;
    return FRAG_OK;
  }
  bool aligned = aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx_out);
  if (dy2) aligned = aligned && aligned16(dy2);
  if (dy3) aligned = aligned && aligned16(dy3);
  if (dres) aligned = aligned && aligned16(dres);
  if (x2) aligned = aligned && aligned16(x2);
  if (x3) aligned = aligned && aligned16(x3);
  if (y_out) aligned = aligned && aligned16(y_out);
  const BwdPlan pl = make_bwd_plan(M, N, aligned);
  if (!workspace || workspace_bytes < bwd_workspace_bytes(pl, M, N)) return FRAG_ERR_WORKSPACE;
  if (!aligned16(workspace)) return FRAG_ERR_ALIGN;

  BwdIn p;
  p.dy = static_cast<const uint16_t*>(dy);
  p.dy2 = static_cast<const uint16_t*>(dy2);
  p.dy3 = static_cast<const uint16_t*>(dy3);
  p.x = static_cast<const uint16_t*>(x);
  p.rstd = rstd;
  p.w = static_cast<const uint16_t*>(w);
  p.dres = static_cast<const uint16_t*>(dres);
  p.dx = static_cast<uint16_t*>(dx_out);
  p.partials = static_cast<float*>(workspace);
  const size_t part_bytes = bwd_partials_bytes(pl, N);
  p.rws = workspace_bytes >= part_bytes + bwd_rstd_copy_bytes(M)
              ? reinterpret_cast<float*>(static_cast<char*>(workspace) + part_bytes)
              : nullptr;
  p.x2 = static_cast<const uint16_t*>(x2);
  p.x3 = static_cast<const uint16_t*>(x3);
  p.y = static_cast<uint16_t*>(y_out);
  p.rstd_out = rstd_out;

  const bool rc = (rstd == nullptr);
  int st;
  if (fwd) {
    if (dy2) st = dres ? launch_bwd_t<true, true, true, true>(pl, p, M, N, eps, s)
                       : launch_bwd_t<true, false, true, true>(pl, p, M, N, eps, s);
    else st = dres ? launch_bwd_t<false, true, true, true>(pl, p, M, N, eps, s)
                   : launch_bwd_t<false, false, true, true>(pl, p, M, N, eps, s);
  } else if (dy2) {
    if (dres) st = rc ? launch_bwd_t<true, true, true>(pl, p, M, N, eps, s) : launch_bwd_t<true, true, false>(pl, p, M, N, eps, s);
    else st = rc ? launch_bwd_t<true, false, true>(pl, p, M, N, eps, s) : launch_bwd_t<true, false, false>(pl, p, M, N, eps, s);
  } else {
    if (dres) st = rc ? launch_bwd_t<false, true, true>(pl, p, M, N, eps, s) : launch_bwd_t<false, true, false>(pl, p, M, N, eps, s);
    else st = rc ? launch_bwd_t<false, false, true>(pl, p, M, N, eps, s) : launch_bwd_t<false, false, false>(pl, p, M, N, eps, s);
  }
  if (st != FRAG_OK) return st;
  if (dw || dw_bf16)
    return launch_dw_reduce(p.partials, pl.G, N, dw, static_cast<uint16_t*>(dw_bf16), s, pl.tma);
  return FRAG_OK;
}

}  // namespace

extern "C" {

int frag_rmsnorm_fwd(const void* x, const void* w, void* y, float* rstd, int64_t M,
                     int64_t N, float eps, frag_stream_t stream) {
  return launch_fwd(nullptr, x, w, nullptr, y, rstd, M, N, eps,
                    reinterpret_cast<cudaStream_t>(stream));
}

int frag_add_rmsnorm_fwd(const void* res, const void* x, const void* w, void* h, void* y,
                         float* rstd, int64_t M, int64_t N, float eps,
                         frag_stream_t stream) {
  if (!res && M > 0) return FRAG_ERR_INVALID_ARG;
  return launch_fwd(res, x, w, h, y, rstd, M, N, eps, reinterpret_cast<cudaStream_t>(stream));
}

size_t frag_rmsnorm_bwd_workspace_bytes(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  // Enough for either plan (aligned or not) and for every kernel a plan may
  // fall back to: the larger partials block plus the generic kernels' rstd copy.
  const BwdPlan a = make_bwd_plan(M, N, true);
  const BwdPlan b = make_bwd_plan(M, N, false);
  return std::max(bwd_partials_bytes(a, N), bwd_partials_bytes(b, N)) + bwd_rstd_copy_bytes(M);
}

int64_t frag_rmsnorm_bwd_num_blocks(int64_t M, int64_t N) {
  if (M <= 0 || N <= 0) return 0;
  return make_bwd_plan(M, N, true).G;
}

int64_t frag_rmsnorm_bwd_plan_blocks(int64_t M, int64_t N, int aligned) {
  if (M <= 0 || N <= 0) return 0;
  return make_bwd_plan(M, N, aligned != 0).G;
}

int frag_dw_reduce(const float* partials, int64_t G, int64_t N, float* dw, void* dw_bf16,
                   frag_stream_t stream) {
  if (!partials || (!dw && !dw_bf16) || G < 0 || N < 0) return FRAG_ERR_INVALID_ARG;
  if (N == 0) return FRAG_OK;
  return launch_dw_reduce(partials, G, N, dw, static_cast<uint16_t*>(dw_bf16),
                          reinterpret_cast<cudaStream_t>(stream));
}

int frag_rmsnorm_bwd(const void* dy, const void* dy2, const void* x, const float* rstd,
                     const void* w, const void* dres, void* dx_out, float* dw, void* dw_bf16,
                     int64_t M, int64_t N, float eps, void* workspace,
                     size_t workspace_bytes, frag_stream_t stream) {
  return frag_rmsnorm_bwd3(dy, dy2, nullptr, x, rstd, w, dres, dx_out, dw, dw_bf16, M, N, eps,
                           workspace, workspace_bytes, stream);
}

int frag_rmsnorm_bwd3(const void* dy, const void* dy2, const void* dy3, const void* x,
                      const float* rstd, const void* w, const void* dres, void* dx_out, float* dw,
                      void* dw_bf16, int64_t M, int64_t N, float eps, void* workspace,
                      size_t workspace_bytes, frag_stream_t stream) {
  return rmsnorm_bwd_impl(false, dy, dy2, dy3, x, nullptr, nullptr, rstd, w, dres, nullptr, nullptr,
                          dx_out, dw, dw_bf16, M, N, eps, workspace, workspace_bytes, stream);
}

int frag_rmsnorm_fwd_bwd(const void* x, const void* x2, const void* x3, const void* w,
                         const void* dy, const void* dy2, const void* dy3, const void* dres,
                         void* y_out, float* rstd_out, void* dx_out, float* dw, void* dw_bf16,
                         int64_t M, int64_t N, float eps, void* workspace, size_t workspace_bytes,
                         frag_stream_t stream) {
  if (x3 && !x2) return FRAG_ERR_INVALID_ARG;
  return rmsnorm_bwd_impl(true, dy, dy2, dy3, x, x2, x3, nullptr, w, dres, y_out, rstd_out, dx_out,
                          dw, dw_bf16, M, N, eps, workspace, workspace_bytes, stream);
}

}  // extern "C"

// ----------------------------------------------- backward without a workspace
//
// frag_rmsnorm_bwd_noalloc runs frag_rmsnorm_bwd with a file-scope device
// array as its workspace, for callers that cannot allocate (see frag.h).

namespace frag {
namespace {

__device__ __align__(256) unsigned char g_noalloc_scratch[FRAG_NOALLOC_SCRATCH_BYTES];

std::mutex g_noalloc_mu;
void* g_noalloc_addr[64] = {};

// In host code `g_noalloc_scratch` names a host-side shadow, not device
// memory; the device address is looked up once per device, with that device
// current, and cached.
int noalloc_scratch_address(void** out) {
  const int d = current_device();
  if (d < 0 || d >= 64) return FRAG_ERR_NO_DEVICE;
  std::lock_guard<std::mutex> lk(g_noalloc_mu);
  if (g_noalloc_addr[d] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess) {
      cudaGetLastError();
      set_last_cuda_error(e);
      return FRAG_ERR_CUDA;
    }
    g_noalloc_addr[d] = p;
  }
  *out = g_noalloc_addr[d];
  return FRAG_OK;
}

}  // namespace
}  // namespace frag

extern "C" int frag_rmsnorm_bwd_noalloc(const void* dy, const void* dy2, const void* x,
                                        const float* rstd, const void* w, const void* dres,
                                        void* dx_out, float* dw, void* dw_bf16, int64_t M,
                                        int64_t N, float eps, frag_stream_t stream) {
  if (M < 0 || N < 0) return FRAG_ERR_INVALID_ARG;
  if (M == 0 || N == 0)  // nothing to reduce: no scratch needed
    return frag_rmsnorm_bwd(dy, dy2, x, rstd, w, dres, dx_out, dw, dw_bf16, M, N, eps, nullptr,
                            0, stream);
  bool aligned = aligned16(dy) && aligned16(x) && aligned16(w) && aligned16(dx_out) &&
                 aligned16(dy2) && aligned16(dres);
  const BwdPlan pl = make_bwd_plan(M, N, aligned);
  if (bwd_workspace_bytes(pl, M, N) > FRAG_NOALLOC_SCRATCH_BYTES) return FRAG_ERR_SCRATCH_LIMIT;
  void* ws = nullptr;
  const int st = noalloc_scratch_address(&ws);
  if (st != FRAG_OK) return st;
  return frag_rmsnorm_bwd(dy, dy2, x, rstd, w, dres, dx_out, dw, dw_bf16, M, N, eps, ws,
                          FRAG_NOALLOC_SCRATCH_BYTES, stream);
}

extern "C" int frag_embedding_rmsnorm_fwd(const int64_t* ids, const void* table, const void* w,
                                          void* y, float* rstd, void* emb_out, int64_t T,
                                          int64_t V, int64_t D, float eps, int32_t* status,
                                          frag_stream_t stream) {
  if (T < 0 || V < 0 || D < 0) return FRAG_ERR_INVALID_ARG;
  if (T == 0) return FRAG_OK;
  if (D == 0 || T > 0x7fffffffLL) return FRAG_ERR_SHAPE;
  if (!ids || !w || !y || (V > 0 && !table)) return FRAG_ERR_INVALID_ARG;
  bool aligned = aligned16(w) && aligned16(y) && (V == 0 || aligned16(table));
  if (emb_out) aligned = aligned && aligned16(emb_out);
  const RowCfg cfg = pick_row_cfg(D, aligned);
  auto tab = static_cast<const uint16_t*>(table);
  auto W = static_cast<const uint16_t*>(w);
  auto E = static_cast<uint16_t*>(emb_out);
  auto Y = static_cast<uint16_t*>(y);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  if (emb_out)
    return rstd ? launch_emb_rms_t<true, true>(cfg, ids, tab, W, E, Y, rstd, T, V, D, eps, status, s)
                : launch_emb_rms_t<true, false>(cfg, ids, tab, W, E, Y, rstd, T, V, D, eps, status, s);
  return rstd ? launch_emb_rms_t<false, true>(cfg, ids, tab, W, E, Y, rstd, T, V, D, eps, status, s)
              : launch_emb_rms_t<false, false>(cfg, ids, tab, W, E, Y, rstd, T, V, D, eps, status, s);
}
