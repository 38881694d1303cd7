// norm_embedding.cu — RMSNorm backward fused into the token-embedding
// backward: the first layer's attention_norm and the table-gradient scatter
// of its input gradient (v6/0b493aad68f0/problem.py:21-70,
// v5/118d525f44e0/problem.py and v1-v4/680e4c57cdc8/problem.py, and the
// v8/f6251e84e3fa/problem.py:22-57 variant that takes the saved rstd):
//
//   dy    = bf16(bf16(dy_a + dy_b) + dy_c)             (aten.add chain)
//   rstd  = rsqrt(mean(x^2) + eps)  or the saved one
//   y     = bf16((x * rstd) * w)                       (optional forward output)
//   dx    = bf16(rstd * (dy*w - xhat * mean(dy*w*xhat)))   xhat = x * rstd
//   d_emb = bf16(dres + dx)                            (dres optional)
//   dw    = sum_t dy * xhat                            (fp32, fixed order)
//   G[v]  = sum_{t : ids[t] = v} d_emb[t]              (fp32, fixed order)
//
// The unfused chain writes d_emb (T x D bf16) to HBM and reads it back for
// the scatter; here it never leaves the SM.  Tokens are processed in sorted
// id order: CTA b owns the sorted positions [b*R, (b+1)*R), streams each
// token's rows (x, the dy terms, dres) through a TMA ring in shared memory,
// and keeps the running sum of the current table row in registers.  A row
// whose tokens all lie in the CTA's range is written to G directly; a run
// that crosses a range boundary leaves fp32 partial rows in a workspace slot
// and a small fixup kernel adds them in range order.  Every sum therefore has
// a fixed order, even when one id covers all tokens, and the result is
// bitwise reproducible.  Rows of G without tokens are zeroed by the sweep of
// the shared front end (emb_bwd.cuh), on a side stream, while the sort and
// the fused kernel run.
#include <algorithm>

#include "common.cuh"
#include "emb_bwd.cuh"

namespace frag {
namespace {

struct ChainIn {
  const uint16_t* x;
  const uint16_t* w;
  const float* rstd;      // saved rstd [T] (RECOMPUTE = false)
  const uint16_t* dy0;
  const uint16_t* dy1;    // optional
  const uint16_t* dy2;    // optional (only with dy1)
  const uint16_t* dres;   // optional
  uint16_t* y;            // optional forward output
  uint16_t* demb;         // optional d_emb output
  const uint32_t* keys;   // sorted rows (sentinel shard_rows for skipped tokens)
  const uint32_t* vals;   // token of each sorted position
  float* G;
  int64_t shard_rows;
  float* partials;  // [P, D] dweight partial sums
  float* slots;     // [P, 3, D]: 0 = head run, 1 = tail run, 2 = generic accumulator
  int T;
  int D;
  int R;  // sorted positions per CTA
  float eps;
};

// 8 consecutive fp32 values, one 256-bit store (32-byte aligned address).
__device__ __forceinline__ void st_v8(float* p, const float (&v)[8]) {
  asm volatile("st.global.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}
__device__ __forceinline__ void st_v8_cs(float* p, const float (&v)[8]) {
  asm volatile("st.global.cs.v8.f32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "f"(v[0]), "f"(v[1]),
               "f"(v[2]), "f"(v[3]), "f"(v[4]), "f"(v[5]), "f"(v[6]), "f"(v[7])
               : "memory");
}

// Where a finished run's sum goes: the head slot when the run began before
// this CTA's range, the tail slot when it continues past it, else its row.
__device__ __forceinline__ float* run_dest(const ChainIn& p, bool head, bool cont, uint32_t key) {
  if (head) return p.slots + (static_cast<size_t>(blockIdx.x) * 3 + 0) * p.D;
  if (cont) return p.slots + (static_cast<size_t>(blockIdx.x) * 3 + 1) * p.D;
  return p.G + static_cast<size_t>(key) * p.D;
}

// One token's data between the two halves of its work: x and dres packed,
// the folded gradient (bf16-exact values) in fp32 at one chunk per thread,
// packed as bf16 at two (so two tokens' data fit in the registers).
template <int VPT>
struct TokRegs {
  static constexpr bool kF32 = VPT == 1;
  uint4 x[VPT], r[VPT];
  float g[kF32 ? VPT : 1][8];
  uint4 gp[kF32 ? 1 : VPT];
  __device__ __forceinline__ void set_g(int k, const float (&v)[8]) {
    if (kF32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) g[kF32 ? k : 0][e] = v[e];
    } else {
      gp[kF32 ? 0 : k] = pack8(v);
    }
  }
  __device__ __forceinline__ void get_g(int k, float (&v)[8]) const {
    if (kF32) {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = g[kF32 ? k : 0][e];
    } else {
      unpack8(gp[kF32 ? 0 : k], v);
    }
  }
};

// TMA-ring kernel: D % 8 == 0, blockDim.x * VPT * 8 >= D.  Thread 0 keeps S
// tokens' rows in flight; every wait is bounded.  Each token's work has two
// halves split by the block reduction of its row sums: stage -> registers,
// folded gradient and the sums (first half), then dx, d_emb, y and the run
// sums (second half).  The second half of token i and the first half of
// token i + 1 share one barrier interval, so warps that reach the barrier
// late still leave the others independent work, and a token costs one
// barrier.
template <int VPT, bool RECOMPUTE>
__global__ void __launch_bounds__(512)
norm_emb_bwd_tma(ChainIn p, int S, int* err) {
  extern __shared__ __align__(128) unsigned char smem[];
  __shared__ float2 red[2][32];
  __shared__ int s_abort;
  const int ndy = 1 + (p.dy1 ? 1 : 0) + (p.dy2 ? 1 : 0);
  const int nin = 1 + ndy + (p.dres ? 1 : 0);
  const int row_bytes = p.D * 2;
  const int stage_bytes = nin * row_bytes;
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(S) * stage_bytes);
  const int chunks = p.D >> 3;
  const int lo = blockIdx.x * p.R;
  const int hi = min(p.T, lo + p.R);
  const int n = hi - lo;
  const float invN = 1.0f / static_cast<float>(p.D);
  if (threadIdx.x == 0) {
    s_abort = 0;
    for (int i = 0; i < S; ++i) mbar_init(&bars[i], 1);
    mbar_init_fence();
  }
  __syncthreads();
  int issued = 0;
  // thread 0's next token index, loaded one copy ahead so issuing a stage
  // never waits on a global load (the CTA would wait for it at the barrier)
  int64_t next_tok = (threadIdx.x == 0 && n > 0) ? __ldg(p.vals + lo) : 0;
  auto issue = [&](int i) {
    if (i >= n) return;
    const size_t off = static_cast<size_t>(next_tok) * p.D;
    if (i + 1 < n) next_tok = __ldg(p.vals + lo + i + 1);
    unsigned char* st = smem + static_cast<size_t>(i % S) * stage_bytes;
    uint64_t* bar = &bars[i % S];
    mbar_arrive_expect_tx(bar, stage_bytes);
    bulk_g2s(st, p.x + off, row_bytes, bar);
    bulk_g2s(st + row_bytes, p.dy0 + off, row_bytes, bar);
    int slot = 2;
    if (p.dy1) bulk_g2s(st + (slot++) * row_bytes, p.dy1 + off, row_bytes, bar);
    if (p.dy2) bulk_g2s(st + (slot++) * row_bytes, p.dy2 + off, row_bytes, bar);
    if (p.dres) bulk_g2s(st + slot * row_bytes, p.dres + off, row_bytes, bar);
    issued = i + 1;
  };
  if (threadIdx.x == 0)
    for (int i = 0; i < S; ++i) issue(i);

  // The weight stays in registers at one chunk per thread; with two, two
  // tokens' data plus the accumulators would not fit in 128 registers, so it
  // is re-read from L1 (16 KB at width 8192) where it is used.
  constexpr bool kWRegs = VPT == 1;
  float wf[kWRegs ? VPT : 1][8], gacc[VPT][8], dwacc[VPT][8];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (kWRegs) unpack8((c < chunks) ? ld_cached(p.w + c * 8) : make_uint4(0, 0, 0, 0), wf[kWRegs ? k : 0]);
#pragma unroll
    for (int e = 0; e < 8; ++e) gacc[k][e] = dwacc[k][e] = 0.f;
  }
  auto weight = [&](int k, float (&out)[8]) {
    if (kWRegs) {
#pragma unroll
      for (int e = 0; e < 8; ++e) out[e] = wf[kWRegs ? k : 0][e];
    } else {
      const int c = threadIdx.x + k * blockDim.x;
      unpack8((c < chunks) ? ld_cached(p.w + c * 8) : make_uint4(0, 0, 0, 0), out);
    }
  };

  // First half of token i: wait for its stage, copy what it needs to
  // registers (the barrier that follows frees the stage), fold the
  // gradients, partial row sums.
  auto first_half = [&](int i, TokRegs<VPT>& R, float& s1, float& s2) {
    const unsigned char* st = smem + static_cast<size_t>(i % S) * stage_bytes;
    if (!mbar_wait(&bars[i % S], (i / S) & 1, err)) s_abort = 1;
    s1 = s2 = 0.f;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      const bool in = c < chunks;
      const uint4 z = make_uint4(0, 0, 0, 0);
      R.x[k] = in ? *reinterpret_cast<const uint4*>(st + c * 16) : z;
      // each partial sum of the gradients is a bf16 tensor in the graph:
      // packed bf16 adds give exactly those sums
      uint4 gp = in ? *reinterpret_cast<const uint4*>(st + row_bytes + c * 16) : z;
      int slot = 2;
      if (p.dy1)
        gp = add_bf16x8(gp, in ? *reinterpret_cast<const uint4*>(st + (slot++) * row_bytes + c * 16) : z);
      if (p.dy2)
        gp = add_bf16x8(gp, in ? *reinterpret_cast<const uint4*>(st + (slot++) * row_bytes + c * 16) : z);
      float g[8];
      unpack8(gp, g);
      R.set_g(k, g);
      R.r[k] = (p.dres && in) ? *reinterpret_cast<const uint4*>(st + slot * row_bytes + c * 16) : z;
      float xf[8], wv[8];
      unpack8(R.x[k], xf);
      weight(k, wv);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        if (RECOMPUTE) s1 = fmaf(xf[e], xf[e], s1);
        s2 = fmaf(xf[e], g[e] * wv[e], s2);
      }
    }
  };

  // Per-token scalars, software-pipelined: token i's key, next key, token
  // index and saved rstd are loaded while token i - 1 is in flight.
  auto key_at = [&](int q) { return q < p.T ? __ldg(p.keys + q) : 0xffffffffu; };
  // the first run continues one that began in an earlier range
  bool head = n > 0 && lo > 0 && __ldg(p.keys + lo - 1) == __ldg(p.keys + lo);
  uint32_t key = n > 0 ? key_at(lo) : 0u;
  uint32_t nkey = n > 0 ? key_at(lo + 1) : 0u;
  int64_t t = n > 0 ? __ldg(p.vals + lo) : 0;
  int64_t t1 = n > 1 ? __ldg(p.vals + lo + 1) : 0;
  float rr = (!RECOMPUTE && n > 0) ? __ldg(p.rstd + t) : 0.f;

  TokRegs<VPT> A, B;
  float2 totA = make_float2(0.f, 0.f);
  int parity = 0;
  int failed = -1;  // token whose stage wait gave up
  if (n > 0) {
    float s1, s2;
    first_half(0, A, s1, s2);
    totA = block_sum2(make_float2(s1, s2), red, parity);
    parity ^= 1;
    if (s_abort) failed = 0;
    else if (threadIdx.x == 0) issue(S);  // stage 0 is free again
  }
  for (int i = 0; i < n && failed < 0; ++i) {
    const bool more = i + 1 < n;
    // next tokens' scalars
    const uint32_t nnkey = key_at(lo + i + 2);
    const int64_t t2 = (i + 2 < n) ? __ldg(p.vals + lo + i + 2) : 0;
    const float rr1 = (!RECOMPUTE && more) ? __ldg(p.rstd + t1) : 0.f;
    float bs1 = 0.f, bs2 = 0.f;
    if (more) first_half(i + 1, B, bs1, bs2);

    // second half of token i
    const float r = RECOMPUTE ? rsqrtf(totA.x * invN + p.eps) : rr;
    const float cmean = r * totA.y * invN;  // mean(xhat * dy * w)
    const bool in_shard = key < static_cast<uint64_t>(p.shard_rows);
    const size_t base = static_cast<size_t>(t) * p.D;
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      float xf[8], d[8], yv[8], wv[8], g[8];
      unpack8(A.x[k], xf);
      A.get_g(k, g);
      weight(k, wv);
      float dx[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float xhat = xf[e] * r;
        yv[e] = xhat * wv[e];
        dx[e] = (g[e] * wv[e] - xhat * cmean) * r;
        dwacc[k][e] = fmaf(g[e], xhat, dwacc[k][e]);
      }
      // d_emb = bf16(dres + bf16(dx)): round dx, then one packed bf16 add
      uint4 dp = pack8(dx);
      if (p.dres) dp = add_bf16x8(A.r[k], dp);
      unpack8(dp, d);
      if (in_shard) {
#pragma unroll
        for (int e = 0; e < 8; ++e) gacc[k][e] += d[e];
      }
      if (c < chunks) {
        if (p.y) st_global(p.y + base + c * 8, pack8(yv));
        if (p.demb) st_global(p.demb + base + c * 8, dp);
      }
    }
    // end of a run: its table row (or a boundary slot) is written once
    const bool last = (i == n - 1);
    if (in_shard && (last || nkey != key)) {
      const bool cont = last && nkey == key;
      float* dst = run_dest(p, head, cont, key);
      const bool to_g = !head && !cont;
#pragma unroll
      for (int k = 0; k < VPT; ++k) {
        const int c = threadIdx.x + k * blockDim.x;
        if (c < chunks) {
          if (to_g) st_v8_cs(dst + c * 8, gacc[k]);
          else st_v8(dst + c * 8, gacc[k]);
        }
#pragma unroll
        for (int e = 0; e < 8; ++e) gacc[k][e] = 0.f;
      }
    }
    if (last || nkey != key) head = false;

    if (more) {
      totA = block_sum2(make_float2(bs1, bs2), red, parity);
      parity ^= 1;
      if (s_abort) {
        failed = i + 1;
        break;
      }
      if (threadIdx.x == 0) issue(i + 1 + S);  // stage (i + 1) % S is free again
      A = B;
    }
    key = nkey;
    nkey = nnkey;
    t = t1;
    t1 = t2;
    rr = rr1;
  }
  // a wait gave up: wait (bounded) for this CTA's copies still in flight
  if (threadIdx.x == 0 && failed >= 0)
    for (int j = failed; j < issued; ++j) mbar_wait(&bars[j % S], (j / S) & 1, nullptr);

  // dweight partials of this range, coalesced: a warp's 32 chunks (8 floats
  // each) become 64 float4s; lane l stores float4 2*base + l (and + 32).
  float4* part = reinterpret_cast<float4*>(p.partials + static_cast<size_t>(blockIdx.x) * p.D);
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int cb = (threadIdx.x & ~31) + k * blockDim.x;
#pragma unroll
    for (int half = 0; half < 2; ++half) {
      const int src = half * 16 + (lane >> 1);
      float v[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = __shfl_sync(0xffffffffu, dwacc[k][e], src);
      const float4 o = (lane & 1) ? make_float4(v[4], v[5], v[6], v[7]) : make_float4(v[0], v[1], v[2], v[3]);
      if (cb + src < chunks) part[2 * cb + half * 32 + lane] = o;
    }
  }
}

// Any width and alignment: the same ranges and runs, rows re-read from
// global memory for the second pass, the run sum and the dweight partials
// accumulated in this CTA's own workspace rows (thread-private columns).
template <bool RECOMPUTE>
__global__ void __launch_bounds__(256)
norm_emb_bwd_generic(ChainIn p) {
  __shared__ float2 red[2][32];
  const int64_t D = p.D;
  const int lo = blockIdx.x * p.R;
  const int hi = min(p.T, lo + p.R);
  const float invN = 1.0f / static_cast<float>(D);
  float* part = p.partials + static_cast<size_t>(blockIdx.x) * D;
  float* acc = p.slots + (static_cast<size_t>(blockIdx.x) * 3 + 2) * D;
  for (int64_t c = threadIdx.x; c < D; c += blockDim.x) part[c] = acc[c] = 0.f;
  auto grad = [&](size_t off) {
    float g = bf16_to_f(p.dy0[off]);
    if (p.dy1) g = round_bf16(g + bf16_to_f(p.dy1[off]));
    if (p.dy2) g = round_bf16(g + bf16_to_f(p.dy2[off]));
    return g;
  };
  bool head = hi > lo && lo > 0 && p.keys[lo - 1] == p.keys[lo];
  int parity = 0;
  for (int pos = lo; pos < hi; ++pos) {
    const uint32_t key = p.keys[pos];
    const uint32_t nkey = (pos + 1 < p.T) ? p.keys[pos + 1] : 0xffffffffu;
    const size_t base = static_cast<size_t>(p.vals[pos]) * D;
    float s1 = 0.f, s2 = 0.f;
    for (int64_t c = threadIdx.x; c < D; c += blockDim.x) {
      const float xf = bf16_to_f(p.x[base + c]);
      if (RECOMPUTE) s1 = fmaf(xf, xf, s1);
      s2 = fmaf(xf, grad(base + c) * bf16_to_f(p.w[c]), s2);
    }
    const float2 tot = block_sum2(make_float2(s1, s2), red, parity);
    parity ^= 1;
    const float r = RECOMPUTE ? rsqrtf(tot.x * invN + p.eps) : p.rstd[p.vals[pos]];
    const float cmean = r * tot.y * invN;
    const bool in_shard = key < static_cast<uint64_t>(p.shard_rows);
    const bool last = (pos == hi - 1);
    const bool end = in_shard && (last || nkey != key);
    float* dst = end ? run_dest(p, head, last && nkey == key, key) : nullptr;
    for (int64_t c = threadIdx.x; c < D; c += blockDim.x) {
      const float xf = bf16_to_f(p.x[base + c]);
      const float wv = bf16_to_f(p.w[c]);
      const float g = grad(base + c);
      const float xhat = xf * r;
      const float dx = round_bf16((g * wv - xhat * cmean) * r);
      const float d = p.dres ? round_bf16(bf16_to_f(p.dres[base + c]) + dx) : dx;
      if (p.y) p.y[base + c] = f_to_bf16(xhat * wv);
      if (p.demb) p.demb[base + c] = f_to_bf16(d);
      part[c] = fmaf(g, xhat, part[c]);
      if (in_shard) acc[c] += d;
      if (end) {
        dst[c] = acc[c];
        acc[c] = 0.f;
      }
    }
    if (last || nkey != key) head = false;
  }
}

// Runs that cross range boundaries.  CTA b looks at the boundary after range
// b: when a run crosses it and began inside range b, the run's sum is range
// b's tail slot plus the head slots of the following ranges it covers, added
// in range order.  VEC: D % 4 == 0 (16-byte slot and table rows).
template <bool VEC>
__global__ void __launch_bounds__(1024)
norm_emb_fixup(const uint32_t* __restrict__ keys, int T, int R, int P, int64_t shard_rows,
               const float* __restrict__ slots, float* __restrict__ G, int D) {
  const int b = blockIdx.x;
  const int64_t lo = static_cast<int64_t>(b) * R, hi = lo + R;
  if (hi >= T) return;
  const uint32_t k = __ldg(keys + hi - 1);
  if (k >= static_cast<uint64_t>(shard_rows) || __ldg(keys + hi) != k) return;
  if (lo > 0 && __ldg(keys + lo - 1) == k) return;  // began in an earlier range
  int c_end = b + 1;                                  // ranges b+1 .. c_end-1 hold head slots
  while (c_end < P && static_cast<int64_t>(c_end) * R < T && __ldg(keys + static_cast<int64_t>(c_end) * R) == k)
    ++c_end;
  const size_t D3 = static_cast<size_t>(D) * 3;
  const float* tail = slots + static_cast<size_t>(b) * D3 + D;
  float* row = G + static_cast<size_t>(k) * D;
  if (VEC) {
    for (int c = threadIdx.x; c < D / 4; c += blockDim.x) {
      float4 s = __ldcg(reinterpret_cast<const float4*>(tail) + c);
      int q = b + 1;
      // four head slots in flight per round, added in range order
      for (; q + 4 <= c_end; q += 4) {
        float4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j)
          v[j] = __ldcg(reinterpret_cast<const float4*>(slots + static_cast<size_t>(q + j) * D3) + c);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          s.x += v[j].x; s.y += v[j].y; s.z += v[j].z; s.w += v[j].w;
        }
      }
      for (; q < c_end; ++q) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(slots + static_cast<size_t>(q) * D3) + c);
        s.x += v.x; s.y += v.y; s.z += v.z; s.w += v.w;
      }
      reinterpret_cast<float4*>(row)[c] = s;
    }
  } else {
    for (int c = threadIdx.x; c < D; c += blockDim.x) {
      float s = tail[c];
      for (int q = b + 1; q < c_end; ++q) s += slots[static_cast<size_t>(q) * D3 + c];
      row[c] = s;
    }
  }
}

// Launch plan, shared by the workspace query and the launch.
struct ChainPlan {
  bool tma = false;
  int vpt = 0, threads = 256;
  int P = 0;  // CTAs (ranges)
  int cps = 1;  // CTAs per SM the ring is sized for
  int R = 1;  // sorted positions per range
};

ChainPlan make_chain_plan(int64_t T, int64_t D, bool aligned) {
  ChainPlan pl;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const int64_t chunks = D / 8;
  if (aligned && D % 8 == 0 && chunks >= 1 && chunks <= 1024) {
    pl.tma = true;
    // Up to width 4096: at most 256 threads (one chunk per thread up to 256
    // chunks, two above) and two CTAs per SM, each with half the shared
    // memory for its ring: two token streams per SM and half the warps at
    // each token's barrier (measured 3% faster at width 4096 than one
    // 512-thread CTA per SM).  Wider rows: two chunks per thread, up to 512
    // threads, one CTA per SM (a ring stage of five 16 KB rows needs it).
    pl.vpt = chunks <= 256 ? 1 : 2;
    pl.threads = static_cast<int>((ceil_div(chunks, pl.vpt) + 31) / 32 * 32);
    pl.cps = pl.threads <= 256 ? 2 : 1;
    const int64_t target = std::max<int64_t>(1, std::min<int64_t>(T, static_cast<int64_t>(pl.cps) * sms));
    pl.R = static_cast<int>(ceil_div(std::max<int64_t>(T, 1), target));
  } else {
    const int64_t target = std::max<int64_t>(1, std::min<int64_t>(T, static_cast<int64_t>(sms) * 4));
    pl.R = static_cast<int>(ceil_div(std::max<int64_t>(T, 1), target));
  }
  pl.P = static_cast<int>(ceil_div(T, pl.R));
  return pl;
}

struct ChainLayout {
  EmbBwdLayout emb;
  size_t partials, slots, total;
};

bool chain_layout(int64_t T, int64_t D, int64_t shard_rows, const ChainPlan& pl, ChainLayout* L) {
  if (!emb_bwd_layout(T, shard_rows, &L->emb)) return false;
  L->partials = L->emb.total;
  const size_t pb = align_up(static_cast<size_t>(std::max(pl.P, 1)) * D * 4, 256);
  L->slots = L->partials + pb;
  L->total = L->slots + align_up(static_cast<size_t>(std::max(pl.P, 1)) * 3 * D * 4, 256);
  return true;
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" {

size_t frag_rmsnorm_embedding_bwd_workspace_bytes(int64_t T, int64_t D, int64_t shard_rows) {
  if (T < 0 || D <= 0 || shard_rows < 0 || T > 0x7fffffffLL || shard_rows >= 0xffffffffLL ||
      D > 0x7fffffffLL / 2)
    return 0;
  // The plan of the aligned path has the most ranges; either plan fits.
  const ChainPlan a = make_chain_plan(T, D, true), b = make_chain_plan(T, D, false);
  ChainLayout La, Lb;
  if (!chain_layout(T, D, shard_rows, a, &La) || !chain_layout(T, D, shard_rows, b, &Lb)) return 0;
  return std::max(La.total, Lb.total);
}

int frag_rmsnorm_embedding_bwd(const void* x, const void* w, const float* rstd, void* y,
                               const void* dy_a, const void* dy_b, const void* dy_c,
                               const void* dres, void* d_emb, const int64_t* ids, float* G,
                               float* dw, void* dw_bf16, int64_t T, int64_t D, int64_t shard_rows,
                               int64_t vocab_lo, int64_t vocab_total, int64_t padding_idx, float eps,
                               void* workspace, size_t workspace_bytes, int32_t* status,
                               frag_stream_t stream) {
  if (T < 0 || D < 0 || shard_rows < 0 || vocab_total < 0) return FRAG_ERR_INVALID_ARG;
  if (D == 0) return FRAG_OK;
  if (dy_c && !dy_b) return FRAG_ERR_INVALID_ARG;
  if (T > 0 && (!x || !w || !dy_a || !ids)) return FRAG_ERR_INVALID_ARG;
  if (shard_rows > 0 && !G) return FRAG_ERR_INVALID_ARG;
  if (!dw && !dw_bf16) return FRAG_ERR_INVALID_ARG;
  if (T > 0x7fffffffLL || shard_rows >= 0xffffffffLL || D > 0x7fffffffLL / 2) return FRAG_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const int Ti = static_cast<int>(T);
  const bool aligned = aligned16(x) && aligned16(dy_a) && (!dy_b || aligned16(dy_b)) &&
                       (!dy_c || aligned16(dy_c)) && (!dres || aligned16(dres)) &&
                       (!y || aligned16(y)) && (!d_emb || aligned16(d_emb)) && aligned16(w) &&
                       (reinterpret_cast<uintptr_t>(G) & 31) == 0;
  const ChainPlan pl = make_chain_plan(T, D, aligned);
  ChainLayout L;
  if (!chain_layout(T, D, shard_rows, pl, &L)) return FRAG_ERR_CUDA;
  if (!workspace || workspace_bytes < L.total) return FRAG_ERR_WORKSPACE;
  if (!aligned16(workspace)) return FRAG_ERR_ALIGN;
  char* ws = static_cast<char*>(workspace);
  float* partials = reinterpret_cast<float*>(ws + L.partials);

  // 1-2: the zero sweep of untouched rows on the side stream, the sort and
  // then the fused kernel on `s`.  The sweep's grid fills the GPU, so the
  // sort's kernels start in its last wave and the fused kernel starts about
  // when the sweep ends: the sort hides under the sweep, and the fused
  // kernel (a gathering reader) barely overlaps the streaming sweep, which
  // would lower the throughput of both (measured on B200: 0.45 ms per call at
  // the reference shapes, 0.49 ms with the phases strictly serial).
  EmbBwdFront f;
  int st = FRAG_OK;
  if (shard_rows > 0 || Ti > 0) {
    st = emb_bwd_front(ids, Ti, std::max<int64_t>(shard_rows, 0), D, vocab_lo, vocab_total, padding_idx,
                       G, /*zero_sweep=*/shard_rows > 0, /*zero_ctas_per_sm=*/32, /*sort_first=*/false, ws,
                       L.emb, status, s, &f);
  }
  if (st == FRAG_OK && Ti > 0) {
    ChainIn p;
    p.x = static_cast<const uint16_t*>(x);
    p.w = static_cast<const uint16_t*>(w);
    p.rstd = rstd;
    p.dy0 = static_cast<const uint16_t*>(dy_a);
    p.dy1 = static_cast<const uint16_t*>(dy_b);
    p.dy2 = static_cast<const uint16_t*>(dy_c);
    p.dres = static_cast<const uint16_t*>(dres);
    p.y = static_cast<uint16_t*>(y);
    p.demb = static_cast<uint16_t*>(d_emb);
    p.keys = f.keys;
    p.vals = f.vals;
    p.G = G;
    p.shard_rows = shard_rows;
    p.partials = partials;
    p.slots = reinterpret_cast<float*>(ws + L.slots);
    p.T = Ti;
    p.D = static_cast<int>(D);
    p.R = pl.R;
    p.eps = eps;
    const dim3 grid(static_cast<unsigned>(pl.P));
    if (pl.tma) {
      const int nin = 2 + (dy_b ? 1 : 0) + (dy_c ? 1 : 0) + (dres ? 1 : 0);
      const int stage_bytes = nin * static_cast<int>(D) * 2;
      const int S = std::min(8, (200 * 1024 / pl.cps) / stage_bytes);
      const int smem = S * stage_bytes + 8 * S;
      auto kern = pl.vpt == 1 ? (rstd ? norm_emb_bwd_tma<1, false> : norm_emb_bwd_tma<1, true>)
                              : (rstd ? norm_emb_bwd_tma<2, false> : norm_emb_bwd_tma<2, true>);
      if (S >= 2 && allow_dynamic_smem(reinterpret_cast<const void*>(kern), smem)) {
        kern<<<grid, pl.threads, smem, s>>>(p, S, device_error_word());
        st = check_launch();
      } else {
        st = FRAG_ERR_SHAPE;
      }
    } else {
      if (rstd) norm_emb_bwd_generic<false><<<grid, 256, 0, s>>>(p);
      else norm_emb_bwd_generic<true><<<grid, 256, 0, s>>>(p);
      st = check_launch();
    }
    if (st == FRAG_OK && pl.P > 1 && shard_rows > 0) {
      const dim3 fg(static_cast<unsigned>(pl.P - 1));
      const int ft = static_cast<int>(std::min<int64_t>(1024, (D % 4 == 0 ? D / 4 : D) + 31) / 32 * 32);
      if (D % 4 == 0 && (reinterpret_cast<uintptr_t>(G) & 15) == 0)
        norm_emb_fixup<true><<<fg, ft, 0, s>>>(f.keys, Ti, pl.R, pl.P, shard_rows, p.slots, G,
                                               static_cast<int>(D));
      else
        norm_emb_fixup<false><<<fg, ft, 0, s>>>(f.keys, Ti, pl.R, pl.P, shard_rows, p.slots, G,
                                                static_cast<int>(D));
      st = check_launch();
    }
  }
  // 3: dweight in a fixed order over the ranges (zeros without tokens)
  if (st == FRAG_OK) st = frag_dw_reduce(partials, Ti > 0 ? pl.P : 0, D, dw, dw_bf16, stream);
  return emb_bwd_join(&f, s, st);
}

}  // extern "C"
