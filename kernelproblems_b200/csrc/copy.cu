// copy.cu — row-strided copies: the FSDP unshard of a parameter out of the
// all-gather buffer (v8/8e33a91b7364/problem.py:23-51: wait_tensor viewed
// [8, -1], split_with_sizes, clone of the [8, 65667072] split into a
// contiguous [128256, 4096] table) and the small weight gathers of the other
// FSDP fragments; the grouped form copies every split of one parameter group
// (v8/7815074de963/problem.py:23-103) in a single launch.
//
// dst row r <- src row r, `row_bytes` each, rows `src_stride` / `dst_stride`
// bytes apart.  With 16-byte aligned rows the copy moves 16-byte units, each
// thread keeping four loads in flight before its stores; the grid is (CTAs
// per row, rows), so no unit index is ever divided by the row length.
#include <algorithm>

#include "common.cuh"

namespace frag {
namespace {

constexpr int kCopyUnroll = 4;

// Rows by, by + yb, ... of one copy; in each, unit bx*256 + tid and every
// (xb*256)-th after it.  Shared by the single and the grouped launch.
__device__ __forceinline__ void copy_rows_part(const unsigned char* __restrict__ src, int64_t src_stride,
                                               unsigned char* __restrict__ dst, int64_t dst_stride,
                                               int64_t rows, int64_t units, int64_t bx, int64_t xb,
                                               int64_t by, int64_t yb) {
  const int64_t step = xb * blockDim.x;
  for (int64_t r = by; r < rows; r += yb) {
    const unsigned char* s = src + r * src_stride;
    unsigned char* d = dst + r * dst_stride;
    int64_t u = bx * blockDim.x + threadIdx.x;
    for (; u + (kCopyUnroll - 1) * step < units; u += kCopyUnroll * step) {
      uint4 v[kCopyUnroll];
#pragma unroll
      for (int j = 0; j < kCopyUnroll; ++j) v[j] = ld_stream(s + (u + j * step) * 16);
#pragma unroll
      for (int j = 0; j < kCopyUnroll; ++j) st_stream(d + (u + j * step) * 16, v[j]);
    }
    for (; u < units; u += step) st_stream(d + u * 16, ld_stream(s + u * 16));
  }
}

__global__ void __launch_bounds__(256)
copy_rows_vec(const unsigned char* __restrict__ src, int64_t src_stride, unsigned char* __restrict__ dst,
              int64_t dst_stride, int64_t rows, int64_t units) {
  copy_rows_part(src, src_stride, dst, dst_stride, rows, units, blockIdx.x, gridDim.x, blockIdx.y,
                 gridDim.y);
}

// One segment of a grouped copy: its CTAs are [first, first + xb*yb) of the
// 1-D grid, xb of them per row and yb row groups.
struct CopySeg {
  const unsigned char* src;
  unsigned char* dst;
  int64_t src_stride, dst_stride, rows, units;
  int64_t first, xb, yb;
};

struct CopyGroup {
  CopySeg seg[FRAG_COPY_MAX_SEGMENTS];
  int n;
};

__global__ void __launch_bounds__(256) copy_rows_grouped_vec(const __grid_constant__ CopyGroup g) {
  int i = 0;
  while (i + 1 < g.n && static_cast<int64_t>(blockIdx.x) >= g.seg[i + 1].first) ++i;
  const CopySeg& c = g.seg[i];
  const int64_t b = static_cast<int64_t>(blockIdx.x) - c.first;
  copy_rows_part(c.src, c.src_stride, c.dst, c.dst_stride, c.rows, c.units, b % c.xb, c.xb, b / c.xb,
                 c.yb);
}

__global__ void __launch_bounds__(256)
copy_rows_bytes(const unsigned char* __restrict__ src, int64_t src_stride, unsigned char* __restrict__ dst,
                int64_t dst_stride, int64_t rows, int64_t row_bytes) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y)
    for (int64_t b = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; b < row_bytes; b += step)
      dst[r * dst_stride + b] = src[r * src_stride + b];
}

}  // namespace
}  // namespace frag

using namespace frag;

extern "C" int frag_copy_rows(const void* src, int64_t src_stride, void* dst, int64_t dst_stride,
                              int64_t rows, int64_t row_bytes, frag_stream_t stream) {
  if (rows < 0 || row_bytes < 0 || src_stride < 0 || dst_stride < 0) return FRAG_ERR_INVALID_ARG;
  if (rows == 0 || row_bytes == 0) return FRAG_OK;
  if (!src || !dst) return FRAG_ERR_INVALID_ARG;
  if (rows > 1 && (src_stride < row_bytes || dst_stride < row_bytes)) return FRAG_ERR_SHAPE;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  const bool vec = aligned16(src) && aligned16(dst) && src_stride % 16 == 0 && dst_stride % 16 == 0 &&
                   row_bytes % 16 == 0;
  const int64_t per_row = vec ? row_bytes / 16 : row_bytes;
  // about 8 CTAs of 256 threads per SM in total, split over the rows
  const int64_t ytot = std::min<int64_t>(rows, 65535);
  const int64_t want = std::max<int64_t>(1, static_cast<int64_t>(sms) * 8 / ytot);
  const int64_t xblocks = std::max<int64_t>(1, std::min<int64_t>(want, ceil_div(per_row, 256)));
  const dim3 grid(static_cast<unsigned>(std::min<int64_t>(xblocks, 0x7fffffffLL)),
                  static_cast<unsigned>(ytot));
  auto sp = static_cast<const unsigned char*>(src);
  auto dp = static_cast<unsigned char*>(dst);
  if (vec)
    copy_rows_vec<<<grid, 256, 0, s>>>(sp, src_stride, dp, dst_stride, rows, per_row);
  else
    copy_rows_bytes<<<grid, 256, 0, s>>>(sp, src_stride, dp, dst_stride, rows, row_bytes);
  return check_launch();
}

extern "C" int frag_copy_rows_grouped(const frag_copy_segment* segs, int32_t n, frag_stream_t stream) {
  if (n < 0 || n > FRAG_COPY_MAX_SEGMENTS) return FRAG_ERR_INVALID_ARG;
  if (n == 0) return FRAG_OK;
  if (!segs) return FRAG_ERR_INVALID_ARG;
  bool vec = true;
  int64_t total = 0;
  for (int i = 0; i < n; ++i) {
    const frag_copy_segment& c = segs[i];
    if (c.rows < 0 || c.row_bytes < 0 || c.src_stride < 0 || c.dst_stride < 0) return FRAG_ERR_INVALID_ARG;
    if (c.rows == 0 || c.row_bytes == 0) continue;
    if (!c.src || !c.dst) return FRAG_ERR_INVALID_ARG;
    if (c.rows > 1 && (c.src_stride < c.row_bytes || c.dst_stride < c.row_bytes)) return FRAG_ERR_SHAPE;
    vec = vec && aligned16(c.src) && aligned16(c.dst) && c.src_stride % 16 == 0 && c.dst_stride % 16 == 0 &&
          c.row_bytes % 16 == 0;
    total += c.rows * (c.row_bytes / 16);
  }
  if (!vec) {  // byte-granular segments: one launch each
    for (int i = 0; i < n; ++i) {
      const frag_copy_segment& c = segs[i];
      const int st = frag_copy_rows(c.src, c.src_stride, c.dst, c.dst_stride, c.rows, c.row_bytes, stream);
      if (st != FRAG_OK) return st;
    }
    return FRAG_OK;
  }
  if (total == 0) return FRAG_OK;
  int sms = sm_count();
  if (sms <= 0) sms = 148;
  // about 8 CTAs of 256 threads per SM in total, shared out by bytes; every
  // non-empty segment gets at least one CTA and no CTA less than one unit per
  // thread of a row
  const int64_t target = static_cast<int64_t>(sms) * 8;
  CopyGroup g{};
  int64_t first = 0;
  int m = 0;
  for (int i = 0; i < n; ++i) {
    const frag_copy_segment& c = segs[i];
    if (c.rows == 0 || c.row_bytes == 0) continue;
    const int64_t units = c.row_bytes / 16;
    const int64_t per_row = ceil_div(units, 256);
    const int64_t share = ceil_div(target * c.rows * units, total);
    const int64_t nb = std::max<int64_t>(1, std::min<int64_t>(share, c.rows * per_row));
    CopySeg& d = g.seg[m++];
    d.src = static_cast<const unsigned char*>(c.src);
    d.dst = static_cast<unsigned char*>(c.dst);
    d.src_stride = c.src_stride;
    d.dst_stride = c.dst_stride;
    d.rows = c.rows;
    d.units = units;
    d.first = first;
    if (c.rows >= nb) {
      d.yb = nb;
      d.xb = 1;
    } else {
      d.yb = c.rows;
      d.xb = std::max<int64_t>(1, std::min<int64_t>(nb / c.rows, per_row));
    }
    first += d.xb * d.yb;
  }
  g.n = m;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  copy_rows_grouped_vec<<<static_cast<unsigned>(first), 256, 0, s>>>(g);
  return check_launch();
}
