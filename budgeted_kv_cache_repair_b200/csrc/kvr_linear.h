// Internal entry of the sm_100a projection kernel (kvr_linear.cu), shared with
// the native layer loop (kvr_refresh.cu).
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/kvr_b200.h"

namespace kvr {

// Rows of x per launch (MMA N); more rows run as several launches.
constexpr int64_t kMaxRows = 256;

size_t linear_workspace_size(int64_t rows, int64_t k, const kvr_linear_segment* segments, int count);

// The same size from the segments' geometry alone (n, gated or not); the
// first linear_zero_bytes(tiles) bytes must be zero before the first launch.
size_t linear_workspace_bytes(int64_t rows, int64_t k, const int64_t* n, const bool* paired, int count);

// Bytes at the start of a workspace that hold the status word and tile
// counters of a launch with `tiles` tiles.
constexpr size_t linear_zero_bytes(int64_t tiles) { return 256 + (static_cast<size_t>(tiles) * 4 + 255) / 256 * 256; }

// Deferred reduction: instead of the rounded output, each of the `split` CTAs
// that share a tile writes its fp32 partial over its k range to
// part[i] + slice * part_slice + row * part_stride + column (segment i). The
// consumer sums the `split` slices in order and rounds (the projection's own
// rounding). No cluster, no reduction in the projection kernel. Gated
// segments cannot be deferred. `split` is chosen by the call and returned.
struct Deferred {
  float* part[KVR_LINEAR_MAX_SEGMENTS];
  int64_t part_stride;  // floats between rows of one slice
  int64_t part_slice;   // floats between slices
  int max_split;        // slices the buffer holds
  int split;            // out: slices written
};

// kvr_linear; with counters_zeroed the caller guarantees that the status word
// and tile counters at the start of `workspace` are zero (every launch leaves
// the counters zero), and no memset is issued.
int linear_forward(const void* x, int64_t x_stride, int64_t rows, int64_t k, const kvr_linear_segment* segments,
                   int count, void* workspace, size_t workspace_bytes, int dtype, bool counters_zeroed,
                   cudaStream_t stream, Deferred* deferred = nullptr);

// Slices a deferred launch of `tiles` 128-row tiles over k would use.
int deferred_split(int64_t tiles, int64_t k);

}  // namespace kvr
