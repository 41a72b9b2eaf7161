// Internal entry of the fused projection kernel (kvr_proj.cu), used by the
// native layer loop (kvr_refresh.cu) for requests of up to kProjMaxRows rows.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

#include "../../include/kvr_b200.h"

namespace kvr {

// Rows of x one fused projection launch takes (MMA N <= 128).
constexpr int64_t kProjMaxRows = 128;

// What a fused projection does around out = x . W^T.
enum ProjEpilogue : int {
  // o_proj / down_proj: h[r, n] = round(h[r, n] + round(out[r, n])) in place,
  // and for every 128-column tile t and row r the fp32 sum of squares of the
  // new h[r, t*128 .. t*128+127] into ssq_out[t * kProjMaxRows + r].
  PROJ_RESIDUAL = 0,
  // gate/up pair: act = round(round(silu(round(gate))) * round(up)).
  PROJ_GATED = 1,
  // q/k/v (head_dim 128, one tile per head): round, per-head q/k RMSNorm when
  // weights are given, RoPE at the row's absolute position, then q heads to
  // q_out[r][head][:], k and v heads into the cache at row positions[r].
  PROJ_QKV_ROPE = 2,
};

struct ProjParams {
  int epilogue;
  int dtype;
  int64_t rows, k;
  // x: either the rows of a 16-bit matrix read as they are (x, x_stride), or,
  // with norm_w set, RMSNorm(x) computed while the stages are filled:
  // round(norm_w * round(x * rsqrt(sum_t ssq_in[t][r] / k + eps))), the
  // sums of squares coming from the PROJ_RESIDUAL launch that wrote x.
  const void* x;
  int64_t x_stride;
  const void* norm_w;
  const float* ssq_in;
  int ssq_tiles;
  float eps;
  // weights [n, k] row-major: w[0] (q, gate or the single matrix), w[1]
  // (k or up), w[2] (v); n_w[i] rows each.
  const void* w[3];
  int64_t n_w[3];
  // PROJ_RESIDUAL / PROJ_GATED output [rows, n] with row stride out_stride.
  void* out;
  int64_t out_stride;
  float* ssq_out;  // PROJ_RESIDUAL: [n / 128][kProjMaxRows]
  // PROJ_QKV_ROPE
  int q_heads, kv_heads;  // q_heads = 0: k and v only (no q_out)
  void* q_out;            // [rows][q_heads][128]
  void* k_cache;
  void* v_cache;          // [kv_heads][cache_rows][128] with (c_hs, c_rs) strides
  int64_t cache_rows, c_hs, c_rs;
  const int64_t* positions;
  const void* cos_tab;
  const void* sin_tab;  // [rows][128]
  const void* q_norm;
  const void* k_norm;  // [128] or NULL
};

// Workspace bytes of launches with `rows` rows and up to `tiles` 128-row
// weight tiles (64 gate + 64 up rows per tile for PROJ_GATED); the first
// proj_zero_bytes(tiles) bytes must be zero before the first launch (every
// launch leaves them zero). Launches of different tile counts may share one
// workspace: the partial results sit at its end.
size_t proj_workspace_bytes(int64_t rows, int64_t tiles);
constexpr size_t proj_zero_bytes(int64_t tiles) { return 256 + (static_cast<size_t>(tiles) * 4 + 255) / 256 * 256; }

// Tiles of a launch with these parameters (0 if they are not supported).
int64_t proj_tiles(const ProjParams& p);

int proj_forward(const ProjParams& p, void* workspace, size_t workspace_bytes, cudaStream_t stream);

}  // namespace kvr
