// emb_bwd.cuh — the sort front end of the table-gradient backward, shared by
// frag_embedding_bwd (embedding.cu) and frag_rmsnorm_embedding_bwd
// (norm_embedding.cu).  Host-side declarations; the kernels live in
// embedding.cu.
#pragma once

#include "common.cuh"

namespace frag {

// Workspace layout: sort keys/values in and out, the touched-row bitmap and
// CUB's temporary storage, each 256-byte aligned.
struct EmbBwdLayout {
  size_t keys_in, vals_in, keys_out, vals_out, touched, touched_bytes, temp, temp_bytes, total;
};
bool emb_bwd_layout(int64_t T, int64_t shard_rows, EmbBwdLayout* L);

// State handed from the front end to the row kernels.
struct EmbBwdFront {
  const uint32_t* keys = nullptr;     // sorted shard-local rows; padding and other
                                      // shards' ids carry the sentinel shard_rows
  const uint32_t* vals = nullptr;     // token index of each sorted position
  const uint32_t* touched = nullptr;  // bit v set: row v has at least one token
  cudaEvent_t fork = nullptr, join = nullptr;  // zero sweep on the side stream
};

// On `s`: clear the bitmap, build keys/values/bitmap from ids, radix-sort
// them (stable, so each row's tokens stay in increasing t).  With
// `zero_sweep`, every row of G that no token touches is written with zeros
// by a grid-stride sweep (`zero_ctas_per_sm` sizes its grid):
//   sort_first = false: on a per-device side stream forked before the sort,
//     so it overlaps the sort and the caller's row kernel on `s`;
//   sort_first = true: on `s` after the sort, alone.
// Measured on B200: the sort's small latency-bound kernels slow down several
// times while a sweep saturates HBM beside them, and a gathering row kernel
// next to the streaming sweep lowers their combined throughput.  With a grid
// that fills the GPU (32 CTAs per SM) forked before the sort, the sort's
// kernels get SMs only in the sweep's last wave and the row kernel starts
// about when the sweep ends, which is the fastest order measured for both
// callers.  The caller must end with emb_bwd_join on the same front,
// whatever happened.
int emb_bwd_front(const int64_t* ids, int T, int64_t shard_rows, int64_t D, int64_t vocab_lo,
                  int64_t vocab_total, int64_t padding_idx, float* G, bool zero_sweep,
                  int zero_ctas_per_sm, bool sort_first, char* ws, const EmbBwdLayout& L,
                  int32_t* status, cudaStream_t s, EmbBwdFront* f);

// Joins the side stream back into `s` (a stream capture must not end
// forked) and releases the events.  Returns `st`, or the join's error when
// `st` is FRAG_OK.
int emb_bwd_join(EmbBwdFront* f, cudaStream_t s, int st);

}  // namespace frag
