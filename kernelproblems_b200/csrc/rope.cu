// rope.cu — rotary position embedding (forward and its inverse) on q and k.
//
// Reference math (v8/c8c60d8f7015/problem.py:18-70): x is widened to fp32,
// viewed as complex pairs, multiplied by freqs_cis[pos] and rounded back to
// bf16.  Here the pair layout is a template parameter:
//   INTERLEAVED  pairs (x[2j], x[2j+1])        (the reference's view_as_complex)
//   NEOX         pairs (x[j], x[j + D/2])      (rotate-half)
// and (cos, sin) either come from the caller's complex64 table (the
// reference's freqs_cis input) or are evaluated in registers from
//   angle_j = float(pos) * inv_freq[j],  inv_freq[j] = theta^(-2j/D)
// with the accurate sincosf, so no cache tensor is read from HBM.
// The backward is the same rotation by the conjugate (v6/03d64c25b654/problem.py:12-43
// multiplies the incoming gradient by conj(freqs_cis)).  The v1/v2 snapshots
// multiply complex64 tensors directly (v2/075cb40f3d5d/problem.py:15-27:
// view_as_complex inputs times freqs_cis[pos], complex64 out): fp32 input
// with the interleaved layout, fp32 output, no rounding anywhere.
//
// Vector path: one warp per token; D/16 lanes per head.  Lane j owns the two
// 16-byte chunks at element offsets 8j and D/2 + 8j of every head, so each
// load/store instruction of a warp covers contiguous 128-byte spans.  Those
// chunks hold 8 rotation pairs: (x[8j+i], x[D/2+8j+i]) for neox, or the pairs
// 4j..4j+3 and D/4+4j..D/4+4j+3 for the interleaved layout; the lane computes
// their 8 (cos, sin) values once per token and reuses them for every head.
#include <math.h>

#include <algorithm>

#include "common.cuh"

namespace frag {
namespace {

constexpr int kMaxHalf = 256;  // D <= 512

struct RopeT {
  const void* x;  // bf16, or fp32 with if32
  void* out;      // bf16, or fp32 with of32
  int H;
  int64_t xsb, xss, xsh, osb, oss, osh;  // elements of x's / out's type
  int of32;
  int if32;
};

struct RopeP {
  RopeT t[2];
  int nt;
  int64_t B, S;
  int D;
  const void* pos;
  int pos_dtype;
  int64_t psb, pss;
  const float* freqs;  // complex64 as (re, im) float pairs
  int64_t fstride;     // complex elements per table row
  int64_t frows;       // table rows: positions outside [0, frows) are flagged
  int* err;            // library error word (FRAG_DEVFLAG_INDEX_OOB)
  float sign;          // +1 forward, -1 inverse
  float inv_freq[kMaxHalf];
};

__device__ __forceinline__ int64_t load_pos(const RopeP& p, int64_t b, int64_t s) {
  if (p.pos_dtype == FRAG_POS_I32)
    return __ldg(static_cast<const int32_t*>(p.pos) + b * p.psb + s * p.pss);
  if (p.pos_dtype == FRAG_POS_I64)
    return __ldg(static_cast<const int64_t*>(p.pos) + b * p.psb + s * p.pss);
  return s;
}

template <bool NEOX>
__device__ __forceinline__ void rotate_vals(const float (&fa)[8], const float (&fc)[8],
                                            const float (&cs)[8], const float (&sn)[8],
                                            float (&ra)[8], float (&rc)[8]) {
  if (NEOX) {
    // a = x[8j..8j+8), c = x[D/2+8j..): pair i is (fa[i], fc[i]).
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      ra[i] = fa[i] * cs[i] - fc[i] * sn[i];
      rc[i] = fc[i] * cs[i] + fa[i] * sn[i];
    }
  } else {
    // a, c hold 4 (re, im) pairs each: a's use cs[0..3], c's use cs[4..7].
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float re = fa[2 * i], im = fa[2 * i + 1];
      ra[2 * i] = re * cs[i] - im * sn[i];
      ra[2 * i + 1] = re * sn[i] + im * cs[i];
      const float re2 = fc[2 * i], im2 = fc[2 * i + 1];
      rc[2 * i] = re2 * cs[4 + i] - im2 * sn[4 + i];
      rc[2 * i + 1] = re2 * sn[4 + i] + im2 * cs[4 + i];
    }
  }
}

template <bool NEOX>
__device__ __forceinline__ void rotate_f(const uint4& a, const uint4& c, const float (&cs)[8],
                                         const float (&sn)[8], float (&ra)[8], float (&rc)[8]) {
  float fa[8], fc[8];
  unpack8(a, fa);
  unpack8(c, fc);
  rotate_vals<NEOX>(fa, fc, cs, sn, ra, rc);
}

// 8 fp32 values (32 bytes) from x at element offset `off`.
__device__ __forceinline__ void load_f32x8(const float* x, float (&v)[8]) {
  const float4 a = ld_stream_f4(x), b = ld_stream_f4(x + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

template <bool NEOX>
__device__ __forceinline__ void rotate(const uint4& a, const uint4& c, const float (&cs)[8],
                                       const float (&sn)[8], uint4& oa, uint4& oc) {
  float ra[8], rc[8];
  rotate_f<NEOX>(a, c, cs, sn, ra, rc);
  oa = pack8(ra);
  oc = pack8(rc);
}

// 8 fp32 values (32 bytes) to out at element offset `off`.
__device__ __forceinline__ void store_f32x8(const RopeT& T, int64_t off, const float (&v)[8]) {
  float4* o = reinterpret_cast<float4*>(static_cast<float*>(T.out) + off);
  o[0] = make_float4(v[0], v[1], v[2], v[3]);
  o[1] = make_float4(v[4], v[5], v[6], v[7]);
}

// The 8 (cos, sin) of lane j's rotation pairs at position `pos` (the
// conjugate for the inverse); a position outside the table is flagged and
// rotates by nothing instead of reading outside it.
template <bool NEOX, bool TABLE>
__device__ __forceinline__ void lane_freqs(const RopeP& p, int64_t pos, int j, int half,
                                           const float* sfreq, bool report, float (&cs)[8],
                                           float (&sn)[8]) {
  const bool bad = TABLE && (pos < 0 || pos >= p.frows);
  if (bad && report && p.err) atomicOr(p.err, FRAG_DEVFLAG_INDEX_OOB);
  // Frequency index of pair i (0..7) of this lane.
  auto fidx = [&](int i) { return NEOX ? 8 * j + i : (i < 4 ? 4 * j + i : (half >> 1) + 4 * j + i - 4); };
  if (bad) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      cs[i] = 1.f;
      sn[i] = 0.f;
    }
  } else if (TABLE) {
    // pairs i = 0..3 and 4..7 are 4 consecutive complex values each
    const float* row = p.freqs + 2 * pos * p.fstride;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float4* f = reinterpret_cast<const float4*>(row + 2 * fidx(4 * h));
      const float4 v0 = __ldg(f), v1 = __ldg(f + 1);
      cs[4 * h + 0] = v0.x; sn[4 * h + 0] = v0.y * p.sign;
      cs[4 * h + 1] = v0.z; sn[4 * h + 1] = v0.w * p.sign;
      cs[4 * h + 2] = v1.x; sn[4 * h + 2] = v1.y * p.sign;
      cs[4 * h + 3] = v1.z; sn[4 * h + 3] = v1.w * p.sign;
    }
  } else {
    const float fp = static_cast<float>(pos);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      float sv, cv;
      sincosf(fp * sfreq[fidx(i)], &sv, &cv);
      cs[i] = cv;
      sn[i] = sv * p.sign;
    }
  }
}

template <int LPH, bool NEOX, bool TABLE, bool ANYF32>
__global__ void __launch_bounds__(256) rope_vec(const RopeP p) {
  __shared__ float sfreq[kMaxHalf];
  const int half = p.D >> 1;
  if (!TABLE)
    for (int i = threadIdx.x; i < half; i += blockDim.x) sfreq[i] = p.inv_freq[i];
  __syncthreads();
  constexpr int HPI = 32 / LPH;  // heads per warp iteration
  constexpr int UNR = 4;
  const int lane = threadIdx.x & 31;
  const int64_t tok = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (tok >= p.B * p.S) return;
  const int64_t b = tok / p.S, s = tok - b * p.S;
  const int64_t pos = load_pos(p, b, s);
  const int j = lane % LPH, hs = lane / LPH;
  float cs[8], sn[8];
  lane_freqs<NEOX, TABLE>(p, pos, j, half, sfreq, lane == 0, cs, sn);

  // Element offsets of this lane's two 16-byte chunks within a head.
  const int oa = 8 * j;
  const int oc = half + 8 * j;
#pragma unroll
  for (int ti = 0; ti < 2; ++ti) {
    if (ti >= p.nt) break;
    const RopeT& T = p.t[ti];
    const int64_t ob = b * T.osb + s * T.oss;
    const uint16_t* xb = static_cast<const uint16_t*>(T.x) + b * T.xsb + s * T.xss;
    for (int h0 = hs; h0 < T.H; h0 += HPI * UNR) {
      uint4 va[UNR], vc[UNR];
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int h = h0 + u * HPI;
        if (h < T.H) {
          va[u] = ld_plain(xb + h * T.xsh + oa);
          vc[u] = ld_plain(xb + h * T.xsh + oc);
        }
      }
#pragma unroll
      for (int u = 0; u < UNR; ++u) {
        const int h = h0 + u * HPI;
        if (h < T.H) {
          if (ANYF32 && T.of32) {  // fp32 output: the rotated values unrounded
            float ra[8], rc[8];
            rotate_f<NEOX>(va[u], vc[u], cs, sn, ra, rc);
            store_f32x8(T, ob + h * T.osh + oa, ra);
            store_f32x8(T, ob + h * T.osh + oc, rc);
          } else {
            uint4 ra, rc;
            rotate<NEOX>(va[u], vc[u], cs, sn, ra, rc);
            st_global(static_cast<uint16_t*>(T.out) + ob + h * T.osh + oa, ra);
            st_global(static_cast<uint16_t*>(T.out) + ob + h * T.osh + oc, rc);
          }
        }
      }
    }
  }
}

// fp32 (complex64) inputs and outputs, interleaved pairs: one warp per unit
// = (token, group of HG heads of one tensor), so a short sequence still
// fills every resident warp several times over (a persistent grid walking
// the units measured slower).  A lane's two groups of 8 elements sit at the
// bf16 chunks' element offsets, 32 bytes each.
template <int LPH, bool TABLE>
__global__ void __launch_bounds__(256) rope_vec_f32(const RopeP p, int units_q, int units_k) {
  __shared__ float sfreq[kMaxHalf];
  const int half = p.D >> 1;
  if (!TABLE)
    for (int i = threadIdx.x; i < half; i += blockDim.x) sfreq[i] = p.inv_freq[i];
  __syncthreads();
  constexpr int HPI = 32 / LPH;  // heads per warp iteration
  constexpr int UF = 2;          // iterations per unit, loads issued together
  constexpr int HG = HPI * UF;   // heads per unit
  const int U = units_q + units_k;
  const int lane = threadIdx.x & 31;
  const int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x >> 5) + (threadIdx.x >> 5);
  if (w >= p.B * p.S * U) return;
  const int64_t tok = w / U;
  const int u = static_cast<int>(w - tok * U);
  const int ti = u < units_q ? 0 : 1;
  const int hbase = (ti == 0 ? u : u - units_q) * HG;
  const int64_t b = tok / p.S, s = tok - b * p.S;
  const int64_t pos = load_pos(p, b, s);
  const int j = lane % LPH, hs = lane / LPH;
  float cs[8], sn[8];
  // one report per token: the unit holding its first q heads
  lane_freqs<false, TABLE>(p, pos, j, half, sfreq, lane == 0 && u == 0, cs, sn);
  const RopeT& T = p.t[ti];
  const float* xf = static_cast<const float*>(T.x) + b * T.xsb + s * T.xss;
  const int64_t ob = b * T.osb + s * T.oss;
  const int oa = 8 * j, oc = half + 8 * j;
  float fa[UF][8], fc[UF][8];
#pragma unroll
  for (int k = 0; k < UF; ++k) {
    const int h = hbase + hs + k * HPI;
    if (h < T.H) {
      load_f32x8(xf + h * T.xsh + oa, fa[k]);
      load_f32x8(xf + h * T.xsh + oc, fc[k]);
    }
  }
#pragma unroll
  for (int k = 0; k < UF; ++k) {
    const int h = hbase + hs + k * HPI;
    if (h < T.H) {
      float ra[8], rc[8];
      rotate_vals<false>(fa[k], fc[k], cs, sn, ra, rc);
      store_f32x8(T, ob + h * T.osh + oa, ra);
      store_f32x8(T, ob + h * T.osh + oc, rc);
    }
  }
}

// Any even D, any strides: one CTA per token, one thread per (head, pair).
template <bool NEOX, bool TABLE>
__global__ void __launch_bounds__(256) rope_generic(const RopeP p) {
  __shared__ float sfreq[kMaxHalf];
  const int half = p.D >> 1;
  if (!TABLE)
    for (int i = threadIdx.x; i < half; i += blockDim.x) sfreq[i] = p.inv_freq[i];
  __syncthreads();
  const int64_t tok = blockIdx.x;
  const int64_t b = tok / p.S, s = tok - b * p.S;
  const int64_t pos = load_pos(p, b, s);
  const bool bad = TABLE && (pos < 0 || pos >= p.frows);  // flagged, no table read
  if (bad && threadIdx.x == 0 && p.err) atomicOr(p.err, FRAG_DEVFLAG_INDEX_OOB);
#pragma unroll
  for (int ti = 0; ti < 2; ++ti) {
    if (ti >= p.nt) break;
    const RopeT& T = p.t[ti];
    const uint16_t* xb = static_cast<const uint16_t*>(T.x) + b * T.xsb + s * T.xss;
    const float* xf = static_cast<const float*>(T.x) + b * T.xsb + s * T.xss;
    const int64_t ob = b * T.osb + s * T.oss;
    for (int64_t q = threadIdx.x; q < static_cast<int64_t>(T.H) * half; q += blockDim.x) {
      const int h = static_cast<int>(q / half), jj = static_cast<int>(q - static_cast<int64_t>(h) * half);
      float cv, sv;
      if (bad) {
        cv = 1.f;
        sv = 0.f;
      } else if (TABLE) {
        cv = p.freqs[2 * (pos * p.fstride + jj)];
        sv = p.freqs[2 * (pos * p.fstride + jj) + 1];
      } else {
        sincosf(static_cast<float>(pos) * sfreq[jj], &sv, &cv);
      }
      sv *= p.sign;
      const int ia = NEOX ? jj : 2 * jj;
      const int ic = NEOX ? jj + half : 2 * jj + 1;
      const float a = T.if32 ? xf[h * T.xsh + ia] : bf16_to_f(xb[h * T.xsh + ia]);
      const float c = T.if32 ? xf[h * T.xsh + ic] : bf16_to_f(xb[h * T.xsh + ic]);
      const float ra = a * cv - c * sv;
      const float rc = NEOX ? c * cv + a * sv : a * sv + c * cv;
      if (T.of32) {
        static_cast<float*>(T.out)[ob + h * T.osh + ia] = ra;
        static_cast<float*>(T.out)[ob + h * T.osh + ic] = rc;
      } else {
        static_cast<uint16_t*>(T.out)[ob + h * T.osh + ia] = f_to_bf16(ra);
        static_cast<uint16_t*>(T.out)[ob + h * T.osh + ic] = f_to_bf16(rc);
      }
    }
  }
}

template <bool NEOX, bool TABLE, bool ANYF32>
int launch_rope_vec(const RopeP& p, cudaStream_t s) {
  const dim3 grid(static_cast<unsigned>(ceil_div(p.B * p.S, 8)));
  switch (p.D / 16) {
    case 1: rope_vec<1, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    case 2: rope_vec<2, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    case 4: rope_vec<4, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    case 8: rope_vec<8, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    case 16: rope_vec<16, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    case 32: rope_vec<32, NEOX, TABLE, ANYF32><<<grid, 256, 0, s>>>(p); break;
    default: return FRAG_ERR_SHAPE;
  }
  return check_launch();
}

template <int LPH, bool TABLE>
int launch_rope_f32_lph(const RopeP& p, cudaStream_t s) {
  constexpr int HG = 2 * (32 / LPH);
  const int uq = static_cast<int>(ceil_div(p.t[0].H, HG));
  const int uk = p.nt > 1 ? static_cast<int>(ceil_div(p.t[1].H, HG)) : 0;
  const int64_t warps = p.B * p.S * (uq + uk);
  if (warps == 0) return FRAG_OK;
  if (ceil_div(warps, 8) > 0x7fffffffLL) return FRAG_ERR_SHAPE;
  rope_vec_f32<LPH, TABLE><<<static_cast<unsigned>(ceil_div(warps, 8)), 256, 0, s>>>(p, uq, uk);
  return check_launch();
}

template <bool TABLE>
int launch_rope_f32(const RopeP& p, cudaStream_t s) {
  switch (p.D / 16) {
    case 1: return launch_rope_f32_lph<1, TABLE>(p, s);
    case 2: return launch_rope_f32_lph<2, TABLE>(p, s);
    case 4: return launch_rope_f32_lph<4, TABLE>(p, s);
    case 8: return launch_rope_f32_lph<8, TABLE>(p, s);
    case 16: return launch_rope_f32_lph<16, TABLE>(p, s);
    case 32: return launch_rope_f32_lph<32, TABLE>(p, s);
    default: return FRAG_ERR_SHAPE;
  }
}

template <bool NEOX, bool TABLE>
int launch_rope_t(const RopeP& p, bool vec, cudaStream_t s) {
  if (vec) {
    // fp32 outputs get their own instantiation: the bf16-only kernel keeps
    // its register count (and CTAs per SM); fp32 inputs (all tensors of the
    // call) another, interleaved pairs only (complex64 tensors)
    if (p.t[0].if32) {
      if constexpr (NEOX) return FRAG_ERR_SHAPE;
      else return launch_rope_f32<TABLE>(p, s);
    }
    const bool anyf32 = p.t[0].of32 || (p.nt > 1 && p.t[1].of32);
    return anyf32 ? launch_rope_vec<NEOX, TABLE, true>(p, s) : launch_rope_vec<NEOX, TABLE, false>(p, s);
  }
  rope_generic<NEOX, TABLE><<<dim3(static_cast<unsigned>(p.B * p.S)), 256, 0, s>>>(p);
  return check_launch();
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" int frag_rope(const frag_rope_tensor* tensors, int num_tensors, int64_t B, int64_t S,
                         int64_t D, const void* pos, int pos_dtype, int64_t pos_stride_b,
                         int64_t pos_stride_s, const float* freqs, int64_t freqs_stride,
                         int64_t freqs_rows, float theta, int layout, int inverse,
                         frag_stream_t stream) {
  if (!tensors || num_tensors < 1 || num_tensors > 2) return FRAG_ERR_INVALID_ARG;
  if (B < 0 || S < 0 || D < 0) return FRAG_ERR_INVALID_ARG;
  if (layout != FRAG_ROPE_NEOX && layout != FRAG_ROPE_INTERLEAVED) return FRAG_ERR_INVALID_ARG;
  if (pos_dtype != FRAG_POS_NONE && pos_dtype != FRAG_POS_I32 && pos_dtype != FRAG_POS_I64)
    return FRAG_ERR_INVALID_ARG;
  if (pos_dtype != FRAG_POS_NONE && !pos) return FRAG_ERR_INVALID_ARG;
  if (B * S == 0) return FRAG_OK;
  if (D == 0 || D % 2 != 0 || D / 2 > kMaxHalf) return FRAG_ERR_SHAPE;
  if (B * S > 0x7fffffffLL) return FRAG_ERR_SHAPE;

  RopeP p;
  p.nt = num_tensors;
  p.B = B;
  p.S = S;
  p.D = static_cast<int>(D);
  p.pos = pos;
  p.pos_dtype = pos_dtype;
  p.psb = pos_stride_b;
  p.pss = pos_stride_s;
  if (freqs && freqs_rows < 0) return FRAG_ERR_INVALID_ARG;
  p.freqs = freqs;
  p.fstride = freqs_stride;
  p.frows = freqs_rows;
  p.err = freqs ? device_error_word() : nullptr;
  p.sign = inverse ? -1.0f : 1.0f;
  const int half = static_cast<int>(D / 2);
  for (int i = 0; i < kMaxHalf; ++i) p.inv_freq[i] = 0.f;
  if (!freqs) {
    if (!(theta > 0.f)) return FRAG_ERR_INVALID_ARG;
    for (int i = 0; i < half; ++i)
      p.inv_freq[i] = static_cast<float>(1.0 / pow(static_cast<double>(theta),
                                                   static_cast<double>(2 * i) / static_cast<double>(D)));
  }

  bool vec = D % 16 == 0 && (D / 16) <= 32 && (32 % (D / 16)) == 0;
  if (freqs) vec = vec && aligned16(freqs) && freqs_stride % 2 == 0;
  p.t[1] = RopeT{nullptr, nullptr, 0, 0, 0, 0, 0, 0, 0, 0, 0};
  for (int i = 0; i < num_tensors; ++i) {
    const frag_rope_tensor& t = tensors[i];
    if (t.H < 0 || t.H > 0x7fffffffLL) return FRAG_ERR_SHAPE;
    if (t.H > 0 && (!t.x || !t.out)) return FRAG_ERR_INVALID_ARG;
    if (t.out_dtype != FRAG_ROPE_OUT_BF16 && t.out_dtype != FRAG_ROPE_OUT_F32) return FRAG_ERR_INVALID_ARG;
    if (t.in_dtype != FRAG_ROPE_IN_BF16 && t.in_dtype != FRAG_ROPE_IN_F32) return FRAG_ERR_INVALID_ARG;
    // fp32 (complex64) inputs: fp32 outputs, the interleaved layout, and the
    // same input type for every tensor of the call
    if (t.in_dtype == FRAG_ROPE_IN_F32 &&
        (t.out_dtype != FRAG_ROPE_OUT_F32 || layout != FRAG_ROPE_INTERLEAVED))
      return FRAG_ERR_INVALID_ARG;
    if (i > 0 && t.in_dtype != tensors[0].in_dtype) return FRAG_ERR_INVALID_ARG;
    p.t[i] = RopeT{t.x, t.out, static_cast<int>(t.H), t.x_stride_b,
                   t.x_stride_s, t.x_stride_h, t.out_stride_b, t.out_stride_s, t.out_stride_h,
                   t.out_dtype == FRAG_ROPE_OUT_F32 ? 1 : 0, t.in_dtype == FRAG_ROPE_IN_F32 ? 1 : 0};
    const int64_t st[6] = {t.x_stride_b, t.x_stride_s, t.x_stride_h,
                           t.out_stride_b, t.out_stride_s, t.out_stride_h};
    for (int k = 0; k < 6; ++k) vec = vec && (st[k] % 8 == 0);
    vec = vec && aligned16(t.x) && aligned16(t.out);
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool neox = layout == FRAG_ROPE_NEOX;
  if (neox) return freqs ? launch_rope_t<true, true>(p, vec, s) : launch_rope_t<true, false>(p, vec, s);
  return freqs ? launch_rope_t<false, true>(p, vec, s) : launch_rope_t<false, false>(p, vec, s);
}
