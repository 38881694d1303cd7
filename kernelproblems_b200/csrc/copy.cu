// copy.cu — row-strided copies: the FSDP unshard of a parameter out of the
// all-gather buffer (v8/8e33a91b7364/problem.py:23-51: wait_tensor viewed
// [8, -1], split_with_sizes, clone of the [8, 65667072] split into a
// contiguous [128256, 4096] table) and the small weight gathers of the other
// FSDP fragments.
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

__global__ void __launch_bounds__(256)
copy_rows_vec(const unsigned char* __restrict__ src, int64_t src_stride, unsigned char* __restrict__ dst,
              int64_t dst_stride, int64_t rows, int64_t units) {
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = blockIdx.y; r < rows; r += gridDim.y) {
    const unsigned char* s = src + r * src_stride;
    unsigned char* d = dst + r * dst_stride;
    int64_t u = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
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
