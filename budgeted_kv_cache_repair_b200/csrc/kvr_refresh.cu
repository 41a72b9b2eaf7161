// Native layer loop of the packed refresh: one C-ABI call runs the selected
// rows through every decoder layer on the caller's stream. When the request
// also asks for the ownership copy of a source cache, the loop runs on an
// internal high-priority stream beside a low-priority copy stream (layer l is
// copied before its first write), and the caller's stream waits for both.
//
// Per layer: residual add + input RMSNorm, q/k/v projection, fused q/k-norm +
// RoPE + K/V scatter into the cache, selected-query attention, o projection,
// residual add + post-attention RMSNorm, gate/up projections with
// SiLU(gate)*up, down projection. The last layer stops after its K/V scatter
// (and projects no queries): nothing after it reaches the cache.
//
// Projections run on cuBLAS, or (request.projections) up to kMaxRows rows on
// the sm_100a weight-streaming kernel (kvr_linear.cu: q/k/v in one launch,
// gate/up fused with the SiLU product); more rows always run on cuBLAS, where
// the GEMMs are no longer weight-bound.
//
// Host work per layer is a handful of launches from C++, so the GPU, not the
// Python interpreter, sets the pace at a few dozen rows.
//
// Tensor parallelism (optional): each rank holds its share of the query/KV
// heads (column-parallel q/k/v and gate/up, row-parallel o and down, its heads'
// cache) and the two row-parallel projections' partial sums are all-reduced in
// place with NCCL on the same stream, before the residual add.
#include <cublas_v2.h>
#include <nccl.h>

#include <string.h>

#include <algorithm>
#include <mutex>
#include <unordered_map>
#include <vector>

#include "kvr_common.cuh"
#include "kvr_linear.h"
#include "kvr_proj.h"

namespace kvr {
namespace {

constexpr size_t kAlign = 256;

inline size_t align_up(size_t v) { return (v + kAlign - 1) / kAlign * kAlign; }

struct Buffers {
  bool lin;   // room for the sm_100a projection kernel (rows <= kMaxRows)
  bool fused; // room for the fused projections (rows <= kProjMaxRows, head_dim 128)
  size_t hidden, normed, delta, qkv, q_rot, attn, gate, up, act, lin_ws, lin_bytes, lin_zero, parts, attn_ws, total;
  size_t proj_ws, proj_bytes, proj_zero, ssq;
  int max_split;  // slices the deferred-projection buffer holds
};

// The fused projections' geometry rule: head_dim 128 (one tile per head),
// hidden a multiple of 128 (whole residual tiles), at most kProjMaxRows rows.
bool fused_geometry(const kvr_model* m, int64_t rows) {
  return rows <= kProjMaxRows && m->head_dim == 128 && m->hidden % 128 == 0 && m->intermediate % 8 == 0;
}

// Workspace of the projection launches of one layer: the largest of the four
// (q/k/v, o, gate/up, down); every launch leaves its counters zero, so one
// memset of the largest counter region serves the whole call.
void linear_plan(const kvr_model* m, int64_t rows, size_t* bytes, size_t* zero) {
  const int64_t qd = static_cast<int64_t>(m->q_heads) * m->head_dim;
  const int64_t kd = static_cast<int64_t>(m->kv_heads) * m->head_dim;
  const int64_t H = m->hidden, I = m->intermediate;
  const int64_t n_qkv[3] = {qd, kd, kd};
  const bool plain[3] = {false, false, false};
  const bool gated[1] = {true};
  size_t b = linear_workspace_bytes(rows, H, n_qkv, plain, 3);
  const size_t b_o = linear_workspace_bytes(rows, qd, &H, plain, 1);
  const size_t b_mlp = linear_workspace_bytes(rows, H, &I, gated, 1);
  const size_t b_down = linear_workspace_bytes(rows, I, &H, plain, 1);
  b = b > b_o ? b : b_o;
  b = b > b_mlp ? b : b_mlp;
  *bytes = b > b_down ? b : b_down;
  int64_t tiles = (qd + 127) / 128 + 2 * ((kd + 127) / 128);
  if ((H + 127) / 128 > tiles) tiles = (H + 127) / 128;
  if ((I + 63) / 64 > tiles) tiles = (I + 63) / 64;
  *zero = linear_zero_bytes(tiles);
}

Buffers layout(const kvr_model* m, int64_t rows, int64_t cache_rows) {
  const size_t e = 2;  // bf16 / fp16
  const size_t qd = static_cast<size_t>(m->q_heads) * m->head_dim;
  const size_t kd = static_cast<size_t>(m->kv_heads) * m->head_dim;
  Buffers b;
  b.lin = rows <= kMaxRows;
  size_t off = 0;
  auto take = [&](size_t bytes) {
    const size_t at = off;
    off = align_up(off + bytes);
    return at;
  };
  b.hidden = take(rows * m->hidden * e);
  b.normed = take(rows * m->hidden * e);
  b.delta = take(rows * m->hidden * e);
  b.qkv = take(rows * (qd + 2 * kd) * e);
  b.q_rot = take(rows * qd * e);
  b.attn = take(rows * qd * e);
  b.gate = take(rows * static_cast<size_t>(m->intermediate) * e);
  b.up = take(rows * static_cast<size_t>(m->intermediate) * e);
  b.act = take(rows * static_cast<size_t>(m->intermediate) * e);
  b.lin_bytes = b.lin_zero = 0;
  if (b.lin) linear_plan(m, rows, &b.lin_bytes, &b.lin_zero);
  b.lin_ws = take(b.lin_bytes);
  // fp32 partial slices of the deferred projections (q/k/v, o, down), summed
  // by the kernel that consumes each projection.
  b.max_split = 0;
  size_t parts_floats = 0;
  if (b.lin) {
    const int64_t H = m->hidden, I = m->intermediate;
    const int64_t qkv_tiles = (static_cast<int64_t>(qd) + 127) / 128 + 2 * ((static_cast<int64_t>(kd) + 127) / 128);
    const int64_t kv_tiles = 2 * ((static_cast<int64_t>(kd) + 127) / 128);
    const int s_qkv = deferred_split(qkv_tiles, H), s_kv = deferred_split(kv_tiles, H);
    const int s_o = deferred_split((H + 127) / 128, static_cast<int64_t>(qd));
    const int s_down = deferred_split((H + 127) / 128, I);
    const size_t w_qkv = qd + 2 * kd;
    auto need = [&](int sp, size_t width) {
      const size_t f = static_cast<size_t>(sp) * rows * width;
      if (f > parts_floats) parts_floats = f;
      if (sp > b.max_split) b.max_split = sp;
    };
    need(s_qkv, w_qkv);
    need(s_kv, w_qkv);
    need(s_o, H);
    need(s_down, H);
  }
  b.parts = take(parts_floats * sizeof(float));
  // Fused projections: one workspace for the four launches of a layer (the
  // largest tile count: q/k/v heads, hidden / 128 or intermediate / 64) and
  // the per-tile row sums of squares of the residual stream.
  b.fused = fused_geometry(m, rows);
  b.proj_bytes = b.proj_zero = 0;
  int64_t proj_tiles_max = 0;
  if (b.fused) {
    proj_tiles_max = static_cast<int64_t>(m->q_heads) + 2 * m->kv_heads;
    if (m->hidden / 128 > proj_tiles_max) proj_tiles_max = m->hidden / 128;
    if ((m->intermediate + 63) / 64 > proj_tiles_max) proj_tiles_max = (m->intermediate + 63) / 64;
    b.proj_bytes = proj_workspace_bytes(rows, proj_tiles_max);
    b.proj_zero = proj_zero_bytes(proj_tiles_max);
  }
  b.proj_ws = take(b.proj_bytes);
  b.ssq = take(b.fused ? static_cast<size_t>(m->hidden / 128) * kProjMaxRows * sizeof(float) : 0);
  b.attn_ws = take(kvr_attention_workspace_size(rows, m->q_heads, m->kv_heads, m->head_dim, cache_rows));
  b.total = off;
  return b;
}

// One cuBLAS handle per (thread, device); cuBLAS handles are not shared
// across threads.
cublasHandle_t handle_for_current_device(int* status) {
  thread_local std::unordered_map<int, cublasHandle_t> handles;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    *status = KVR_ERR_CUDA;
    return nullptr;
  }
  auto it = handles.find(dev);
  if (it != handles.end()) return it->second;
  cublasHandle_t h = nullptr;
  if (cublasCreate(&h) != CUBLAS_STATUS_SUCCESS) {
    *status = KVR_ERR_CUDA;
    return nullptr;
  }
  handles.emplace(dev, h);
  return h;
}

// Y[M, N] = X[M, K] * W[N, K]^T, row-major, fp32 accumulation (nn.Linear).
int gemm(cublasHandle_t h, const void* x, int64_t ldx, const void* w, void* y, int64_t ldy, int64_t m, int64_t n,
         int64_t k, cudaDataType_t t) {
  const float one = 1.0f, zero = 0.0f;
  const cublasStatus_t st = cublasGemmEx(h, CUBLAS_OP_T, CUBLAS_OP_N, static_cast<int>(n), static_cast<int>(m),
                                         static_cast<int>(k), &one, w, t, static_cast<int>(k), x, t,
                                         static_cast<int>(ldx), &zero, y, t, static_cast<int>(ldy),
                                         CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  return st == CUBLAS_STATUS_SUCCESS ? KVR_OK : KVR_ERR_CUDA;
}

// Two projections of the same input with same-shape weights (gate and up) as
// one strided-batched GEMM, one launch instead of two (config 2: 128.7 ->
// 125.2 us per layer replayed): Y_i[M, N] = X[M, K] * W_i^T. The batch strides
// are the address differences of the two weights and of the two outputs; the
// lower-addressed weight is batch 0 and writes the lower output, so both
// strides are positive. `first_is_w0` reports which weight went to `y_lo`.
int gemm_pair(cublasHandle_t h, const void* x, int64_t ldx, const void* w0, const void* w1, void* y_lo, void* y_hi,
              int64_t ldy, int64_t m, int64_t n, int64_t k, cudaDataType_t t, bool* first_is_w0) {
  const bool order = reinterpret_cast<uintptr_t>(w0) < reinterpret_cast<uintptr_t>(w1);
  const uint8_t* wa = static_cast<const uint8_t*>(order ? w0 : w1);
  const uint8_t* wb = static_cast<const uint8_t*>(order ? w1 : w0);
  const long long stride_w = static_cast<long long>(wb - wa) / 2;
  const long long stride_y = static_cast<long long>(static_cast<uint8_t*>(y_hi) - static_cast<uint8_t*>(y_lo)) / 2;
  *first_is_w0 = order;
  const float one = 1.0f, zero = 0.0f;
  const cublasStatus_t st = cublasGemmStridedBatchedEx(
      h, CUBLAS_OP_T, CUBLAS_OP_N, static_cast<int>(n), static_cast<int>(m), static_cast<int>(k), &one, wa, t,
      static_cast<int>(k), stride_w, x, t, static_cast<int>(ldx), 0, &zero, y_lo, t, static_cast<int>(ldy), stride_y, 2,
      CUBLAS_COMPUTE_32F, CUBLAS_GEMM_DEFAULT);
  return st == CUBLAS_STATUS_SUCCESS ? KVR_OK : KVR_ERR_CUDA;
}

// Per (thread, device) streams for a refresh that also makes the ownership
// copy: `work` (the highest stream priority) runs the layer loop, `copy` (the
// lowest) copies one layer per launch. The block scheduler dispatches pending
// CTAs of `work` first, so the copy's short CTAs fill the SM slots and HBM time
// that the layer loop leaves idle instead of delaying it. Events: `start`
// (both streams wait for the caller's earlier work), one per copied layer, and
// `done` (the caller's stream waits for `work`).
struct RefreshStreams {
  cudaStream_t work = nullptr;
  cudaStream_t copy = nullptr;
  cudaStream_t capture = nullptr;  // only ever captured into a graph, never run
  cudaEvent_t start = nullptr;
  cudaEvent_t done = nullptr;
  cudaEvent_t layer[KVR_MAX_LAYER_TENSORS / 2] = {};
};

int refresh_streams_for_current_device(RefreshStreams** out) {
  thread_local std::unordered_map<int, RefreshStreams> pools;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  RefreshStreams& c = pools[dev];
  if (!c.layer[KVR_MAX_LAYER_TENSORS / 2 - 1]) {
    int least = 0, greatest = 0;
    e = cudaDeviceGetStreamPriorityRange(&least, &greatest);
    if (e == cudaSuccess && !c.work) e = cudaStreamCreateWithPriority(&c.work, cudaStreamNonBlocking, greatest);
    if (e == cudaSuccess && !c.copy) e = cudaStreamCreateWithPriority(&c.copy, cudaStreamNonBlocking, least);
    if (e == cudaSuccess && !c.capture) e = cudaStreamCreateWithFlags(&c.capture, cudaStreamNonBlocking);
    if (e == cudaSuccess && !c.start) e = cudaEventCreateWithFlags(&c.start, cudaEventDisableTiming);
    if (e == cudaSuccess && !c.done) e = cudaEventCreateWithFlags(&c.done, cudaEventDisableTiming);
    for (int l = 0; e == cudaSuccess && l < KVR_MAX_LAYER_TENSORS / 2; ++l)
      if (!c.layer[l]) e = cudaEventCreateWithFlags(&c.layer[l], cudaEventDisableTiming);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
  }
  *out = &c;
  return KVR_OK;
}

// Makes the caller's stream wait for the internal work stream when the
// refresh returns, on success and on every error path alike.
struct JoinCaller {
  cudaStream_t caller = nullptr;
  const RefreshStreams* streams = nullptr;
  ~JoinCaller() {
    if (!streams) return;
    cudaError_t e = cudaEventRecord(streams->done, streams->work);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, streams->done, 0);
    if (e != cudaSuccess) set_last_cuda_error(e);
  }
};

int allreduce(void* buf, int64_t count, int dtype, void* comm, cudaStream_t s) {
  const ncclResult_t st = ncclAllReduce(buf, buf, static_cast<size_t>(count),
                                        dtype == KVR_DTYPE_BF16 ? ncclBfloat16 : ncclFloat16, ncclSum,
                                        static_cast<ncclComm_t>(comm), s);
  return st == ncclSuccess ? KVR_OK : KVR_ERR_CUDA;
}

// Test hook (kvr_debug_fail_refresh_after_layer): the layer after whose K/V
// scatter this thread's next refresh reports KVR_ERR_INJECTED; -1 when unarmed.
thread_local int g_fail_after_layer = -1;

bool valid_model(const kvr_model* m) {
  if (!m || !m->layers || !m->embed || m->num_layers <= 0 || m->num_layers > KVR_MAX_LAYER_TENSORS / 2) return false;
  if (m->hidden <= 0 || m->hidden % 8 || m->q_heads <= 0 || m->kv_heads <= 0 || m->q_heads % m->kv_heads) return false;
  if ((m->head_dim != 64 && m->head_dim != 128) || m->intermediate <= 0 || m->intermediate % 8 || m->vocab <= 0)
    return false;
  if (m->dtype != KVR_DTYPE_BF16 && m->dtype != KVR_DTYPE_F16) return false;
  for (int l = 0; l < m->num_layers; ++l) {
    const kvr_layer_weights& w = m->layers[l];
    if (!w.input_norm || !w.o || !w.post_norm || !w.gate || !w.up || !w.down) return false;
    if (!w.qkv && (!w.q || !w.k || !w.v)) return false;
    if ((w.q_norm == nullptr) != (w.k_norm == nullptr)) return false;
  }
  return true;
}

}  // namespace
}  // namespace kvr

using namespace kvr;

extern "C" {

size_t kvr_packed_refresh_workspace_size(const kvr_model* model, int64_t rows, int64_t cache_rows) {
  if (!valid_model(model) || rows <= 0 || cache_rows <= 0) return 0;
  return layout(model, rows, cache_rows).total;
}

static int refresh_direct(const kvr_model* model, const kvr_refresh_request* req, void* workspace,
                          size_t workspace_bytes, void* stream) {
  if (!valid_model(model) || !req) return KVR_ERR_INVALID_ARG;
  const kvr_model& m = *model;
  const kvr_refresh_request& r = *req;
  if (r.rows < 0 || r.cache_rows <= 0 || !r.k_cache || !r.v_cache) return KVR_ERR_INVALID_ARG;
  for (int l = 0; l < m.num_layers; ++l)
    if (!r.k_cache[l] || !r.v_cache[l]) return KVR_ERR_INVALID_ARG;
  if ((r.k_src == nullptr) != (r.v_src == nullptr)) return KVR_ERR_INVALID_ARG;
  if (r.k_src)
    for (int l = 0; l < m.num_layers; ++l)
      if (!r.k_src[l] || !r.v_src[l]) return KVR_ERR_INVALID_ARG;
  if (r.rows == 0) {
    // Nothing to recompute: the ownership copy is the whole call.
    if (!r.k_src) return KVR_OK;
    const void* src[KVR_MAX_LAYER_TENSORS];
    void* dst[KVR_MAX_LAYER_TENSORS];
    for (int l = 0; l < m.num_layers; ++l) {
      src[2 * l] = r.k_src[l];
      src[2 * l + 1] = r.v_src[l];
      dst[2 * l] = r.k_cache[l];
      dst[2 * l + 1] = r.v_cache[l];
    }
    return kvr_copy_layers(src, dst, 2 * m.num_layers, m.kv_heads, r.cache_rows, m.head_dim, r.src_head_stride,
                           r.src_row_stride, r.cache_head_stride, r.cache_row_stride, m.dtype, stream);
  }
  if (!r.ids || !r.positions || !r.cos_tab || !r.sin_tab || r.id_count <= 0 || r.max_position < 0 ||
      r.max_position >= r.cache_rows)
    return KVR_ERR_INVALID_ARG;
  if (r.rows > 0x7fffffffLL) return KVR_ERR_UNSUPPORTED;
  if (r.projections != KVR_PROJ_CUBLAS && r.projections != KVR_PROJ_SM100 && r.projections != KVR_PROJ_FUSED)
    return KVR_ERR_INVALID_ARG;
  const Buffers b = layout(&m, r.rows, r.cache_rows);
  if (!workspace || workspace_bytes < b.total || !aligned16(workspace)) return KVR_ERR_INVALID_ARG;

  int st = KVR_OK;
  cublasHandle_t h = handle_for_current_device(&st);
  if (!h) return st;
  auto s = static_cast<cudaStream_t>(stream);
  if (cublasSetStream(h, s) != CUBLAS_STATUS_SUCCESS) return KVR_ERR_CUDA;
  const cudaDataType_t t = m.dtype == KVR_DTYPE_BF16 ? CUDA_R_16BF : CUDA_R_16F;

  uint8_t* ws = static_cast<uint8_t*>(workspace);
  void* hidden = ws + b.hidden;
  void* normed = ws + b.normed;
  void* delta = ws + b.delta;
  uint8_t* qkv = ws + b.qkv;
  void* q_rot = ws + b.q_rot;
  void* attn = ws + b.attn;
  void* gate = ws + b.gate;
  void* up = ws + b.up;
  void* act = ws + b.act;
  void* attn_ws = ws + b.attn_ws;
  const size_t attn_ws_bytes = b.total - b.attn_ws;

  const int64_t rows = r.rows;
  const int H = m.hidden, D = m.head_dim, I = m.intermediate;
  const int64_t qd = static_cast<int64_t>(m.q_heads) * D, kd = static_cast<int64_t>(m.kv_heads) * D;
  const int64_t qkv_w = qd + 2 * kd;
  const float scale = 1.0f / sqrtf(static_cast<float>(D));

#define KVR_TRY(expr)            \
  do {                           \
    const int _st = (expr);      \
    if (_st != KVR_OK) return _st; \
  } while (0)

  void* lin_ws = ws + b.lin_ws;
  float* parts = reinterpret_cast<float*>(ws + b.parts);
  // Fused projections (requests outside their geometry or tensor-parallel run
  // on cuBLAS instead).
  const bool fused = b.fused && r.projections == KVR_PROJ_FUSED && !r.tp_comm;
  const bool lin = b.lin && r.projections == KVR_PROJ_SM100;
  // Deferred reduction of q/k/v, o and down (their consumers sum the fp32
  // slices); the tensor-parallel all-reduce needs the rounded sums, so there
  // the projection kernel reduces in-cluster instead.
  const bool defer = lin && !r.tp_comm;
  int down_split = 0;  // slices of the previous layer's down projection
  // Projection on the sm_100a kernel: `count` segments sharing input x.
  auto project = [&](const void* x, int64_t x_stride, int64_t k, const kvr_linear_segment* segs, int count,
                     Deferred* d = nullptr) {
    return linear_forward(x, x_stride, rows, k, segs, count, lin_ws, b.lin_bytes, m.dtype, true, s, d);
  };
  auto deferred = [&](int64_t width, float* p0, float* p1 = nullptr, float* p2 = nullptr) {
    Deferred d{};
    d.part[0] = p0;
    d.part[1] = p1;
    d.part[2] = p2;
    d.part_stride = width;
    d.part_slice = rows * width;
    d.max_split = b.max_split;
    return d;
  };
  // Status words (attention, projections) and tile counters start at zero;
  // each launch leaves its counters zero, so the layer loop needs no memset
  // between kernels (a memset would break the programmatic launch chain).
  {
    cudaError_t e = cudaMemsetAsync(attn_ws, 0, sizeof(int), s);
    if (e == cudaSuccess && lin) e = cudaMemsetAsync(lin_ws, 0, b.lin_zero, s);
    if (e == cudaSuccess && fused) e = cudaMemsetAsync(ws + b.proj_ws, 0, b.proj_zero, s);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
  }

  // Ownership copy of the source layers: from here on the layer loop runs on
  // the internal high-priority stream and the copy on the low-priority one,
  // one launch and one event per layer, both after the caller's earlier work.
  JoinCaller join;
  RefreshStreams* cp = nullptr;
  if (r.k_src) {
    KVR_TRY(refresh_streams_for_current_device(&cp));
    cudaError_t e = cudaEventRecord(cp->start, s);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cp->work, cp->start, 0);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(cp->copy, cp->start, 0);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    join.caller = s;
    join.streams = cp;
    s = cp->work;
    stream = cp->work;
    if (cublasSetStream(h, s) != CUBLAS_STATUS_SUCCESS) return KVR_ERR_CUDA;
    for (int l = 0; l < m.num_layers; ++l) {
      const void* src[2] = {r.k_src[l], r.v_src[l]};
      void* dst[2] = {r.k_cache[l], r.v_cache[l]};
      KVR_TRY(kvr_copy_layers(src, dst, 2, m.kv_heads, r.cache_rows, D, r.src_head_stride, r.src_row_stride,
                              r.cache_head_stride, r.cache_row_stride, m.dtype, cp->copy));
      e = cudaEventRecord(cp->layer[l], cp->copy);
      if (e != cudaSuccess) {
        set_last_cuda_error(e);
        return KVR_ERR_CUDA;
      }
    }
  }
  // Layer l of the owned cache is first written by its K/V scatter.
  auto copied = [&](int l) -> int {
    if (!cp) return KVR_OK;
    const cudaError_t e = cudaStreamWaitEvent(s, cp->layer[l], 0);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    return KVR_OK;
  };

  KVR_TRY(kvr_embed_rows(m.embed, m.vocab, H, r.ids, r.id_count, r.positions, rows, hidden, nullptr, m.dtype,
                         stream));
  if (fused) {
    // Four fused projection launches and the attention per layer; layer 0's
    // input norm is the one separate RMSNorm (no residual sums exist yet).
    void* proj_ws = ws + b.proj_ws;
    float* ssq = reinterpret_cast<float*>(ws + b.ssq);
    const int ssq_tiles = H / 128;
    KVR_TRY(add_rmsnorm_ex(hidden, nullptr, nullptr, 0, 0, 0, m.layers[0].input_norm, normed, rows, H, H, H, H,
                           m.eps, m.dtype, stream, true));
    // The four projections of layer l, in launch order.
    auto qkv_params = [&](int l) {
      const kvr_layer_weights& w = m.layers[l];
      const bool final = l == m.num_layers - 1;
      const uint8_t* wq = static_cast<const uint8_t*>(w.qkv ? w.qkv : w.q);
      ProjParams qp{};
      qp.epilogue = PROJ_QKV_ROPE;
      qp.dtype = m.dtype;
      qp.rows = rows;
      qp.k = H;
      qp.x = l == 0 ? normed : hidden;
      qp.x_stride = H;
      if (l > 0) {
        qp.norm_w = w.input_norm;
        qp.ssq_in = ssq;
        qp.ssq_tiles = ssq_tiles;
      }
      qp.eps = m.eps;
      qp.w[0] = final ? nullptr : wq;
      qp.w[1] = w.qkv ? static_cast<const void*>(wq + qd * H * 2) : w.k;
      qp.w[2] = w.qkv ? static_cast<const void*>(wq + (qd + kd) * H * 2) : w.v;
      qp.n_w[0] = final ? 0 : qd;
      qp.n_w[1] = kd;
      qp.n_w[2] = kd;
      qp.q_heads = final ? 0 : m.q_heads;
      qp.kv_heads = m.kv_heads;
      qp.q_out = final ? nullptr : q_rot;
      qp.k_cache = r.k_cache[l];
      qp.v_cache = r.v_cache[l];
      qp.cache_rows = r.cache_rows;
      qp.c_hs = r.cache_head_stride;
      qp.c_rs = r.cache_row_stride;
      qp.positions = r.positions;
      qp.cos_tab = r.cos_tab;
      qp.sin_tab = r.sin_tab;
      qp.q_norm = w.q_norm;
      qp.k_norm = w.k_norm;
      return qp;
    };
    auto residual_params = [&](const void* x, int64_t k, const void* wt) {
      ProjParams op{};
      op.epilogue = PROJ_RESIDUAL;
      op.dtype = m.dtype;
      op.rows = rows;
      op.k = k;
      op.x = x;
      op.x_stride = k;
      op.w[0] = wt;
      op.n_w[0] = H;
      op.out = hidden;
      op.out_stride = H;
      op.ssq_out = ssq;
      return op;
    };
    auto gated_params = [&](const kvr_layer_weights& w) {
      ProjParams gp{};
      gp.epilogue = PROJ_GATED;
      gp.dtype = m.dtype;
      gp.rows = rows;
      gp.k = H;
      gp.x = hidden;
      gp.x_stride = H;
      gp.norm_w = w.post_norm;
      gp.ssq_in = ssq;
      gp.ssq_tiles = ssq_tiles;
      gp.eps = m.eps;
      gp.w[0] = w.gate;
      gp.w[1] = w.up;
      gp.n_w[0] = I;
      gp.n_w[1] = I;
      gp.out = act;
      gp.out_stride = I;
      return gp;
    };
    for (int l = 0; l < m.num_layers; ++l) {
      const kvr_layer_weights& w = m.layers[l];
      const bool final = l == m.num_layers - 1;
      const ProjParams qp = qkv_params(l);
      if (final) {
        KVR_TRY(copied(l));  // the q/k/v launch writes layer l of the owned cache: its copy first
        KVR_TRY(proj_forward(qp, proj_ws, b.proj_bytes, s));
        if (l == g_fail_after_layer) {
          g_fail_after_layer = -1;
          return KVR_ERR_INJECTED;
        }
        break;
      }
      KVR_TRY(copied(l));
      KVR_TRY(proj_forward(qp, proj_ws, b.proj_bytes, s));
      if (l == g_fail_after_layer) {
        g_fail_after_layer = -1;
        return KVR_ERR_INJECTED;
      }
      KVR_TRY(selected_attention(q_rot, r.k_cache[l], r.v_cache[l], attn, r.positions, rows, m.q_heads, m.kv_heads,
                                 D, r.cache_rows, r.cache_head_stride, r.cache_row_stride, r.max_position, scale,
                                 r.attention_precision, attn_ws, attn_ws_bytes, m.dtype, stream, true));
      KVR_TRY(proj_forward(residual_params(attn, qd, w.o), proj_ws, b.proj_bytes, s));
      KVR_TRY(proj_forward(gated_params(w), proj_ws, b.proj_bytes, s));
      KVR_TRY(proj_forward(residual_params(act, I, w.down), proj_ws, b.proj_bytes, s));
    }
    return KVR_OK;
  }
  for (int l = 0; l < m.num_layers; ++l) {
    const kvr_layer_weights& w = m.layers[l];
    const bool final = l == m.num_layers - 1;
    if (defer && l)
      KVR_TRY(add_rmsnorm_ex(hidden, nullptr, parts, down_split, H, rows * H, w.input_norm, normed, rows, H, H, H,
                             H, m.eps, m.dtype, stream, true));
    else
      KVR_TRY(add_rmsnorm_ex(hidden, l ? delta : nullptr, nullptr, 0, 0, 0, w.input_norm, normed, rows, H, H, H, H,
                             m.eps, m.dtype, stream, true));
    QkvParts qkv_parts{};
    // Layer l of the owned cache must be copied before its K/V scatter. The
    // wait is a full dependency: on the cuBLAS path it goes on the q/k/v GEMM,
    // which waits for its predecessor anyway, so that the scatter keeps its
    // programmatic launch; on the kvr_linear path every kernel is in the
    // programmatic chain and it stays on the scatter, so that the projection
    // can start streaming its weights early.
    if (!lin) KVR_TRY(copied(l));
    if (lin) {
      // q/k/v from separate weights or from row ranges of the stacked matrix.
      const uint8_t* wq = static_cast<const uint8_t*>(w.qkv ? w.qkv : w.q);
      const void* wk = w.qkv ? wq + qd * H * 2 : w.k;
      const void* wv = w.qkv ? wq + (qd + kd) * H * 2 : w.v;
      kvr_linear_segment segs[3] = {
          {wq, nullptr, qd, qkv, qkv_w},
          {wk, nullptr, kd, qkv + qd * 2, qkv_w},
          {wv, nullptr, kd, qkv + (qd + kd) * 2, qkv_w},
      };
      // The last layer needs no queries.
      if (defer) {
        Deferred d = final ? deferred(qkv_w, parts + qd, parts + qd + kd) : deferred(qkv_w, parts, parts + qd, parts + qd + kd);
        KVR_TRY(final ? project(normed, H, H, segs + 1, 2, &d) : project(normed, H, H, segs, 3, &d));
        qkv_parts = QkvParts{parts, d.split, qkv_w, rows * qkv_w, 0, qd, qd + kd};
      } else {
        KVR_TRY(final ? project(normed, H, H, segs + 1, 2) : project(normed, H, H, segs, 3));
      }
    } else if (w.qkv) {
      KVR_TRY(gemm(h, normed, H, w.qkv, qkv, qkv_w, rows, qkv_w, H, t));
    } else {
      if (!final) KVR_TRY(gemm(h, normed, H, w.q, qkv, qkv_w, rows, qd, H, t));
      KVR_TRY(gemm(h, normed, H, w.k, qkv + qd * 2, qkv_w, rows, kd, H, t));
      KVR_TRY(gemm(h, normed, H, w.v, qkv + (qd + kd) * 2, qkv_w, rows, kd, H, t));
    }
    if (lin) KVR_TRY(copied(l));
    KVR_TRY(qkv_rope_scatter_ex(qkv, qkv + qd * 2, qkv + (qd + kd) * 2, qkv_w, qkv_w, qkv_w, w.q_norm, w.k_norm,
                                m.eps, r.cos_tab, r.sin_tab, r.positions, rows, m.q_heads, m.kv_heads, D,
                                final ? nullptr : q_rot, r.k_cache[l], r.v_cache[l], r.cache_rows,
                                r.cache_head_stride, r.cache_row_stride, nullptr, m.dtype, stream,
                                defer ? &qkv_parts : nullptr, true));
    if (l == g_fail_after_layer) {
      // Injected failure: layer l of the owned cache is written, the rest of
      // the call is not issued, as after a CUDA call failing part-way.
      g_fail_after_layer = -1;
      return KVR_ERR_INJECTED;
    }
    if (final) break;
    KVR_TRY(selected_attention(q_rot, r.k_cache[l], r.v_cache[l], attn, r.positions, rows, m.q_heads, m.kv_heads,
                               D, r.cache_rows, r.cache_head_stride, r.cache_row_stride, r.max_position, scale,
                               r.attention_precision, attn_ws, attn_ws_bytes, m.dtype, stream, true));
    int o_split = 0;
    if (lin) {
      const kvr_linear_segment o_seg = {w.o, nullptr, H, delta, H};
      if (defer) {
        Deferred d = deferred(H, parts);
        KVR_TRY(project(attn, qd, qd, &o_seg, 1, &d));
        o_split = d.split;
      } else {
        KVR_TRY(project(attn, qd, qd, &o_seg, 1));
      }
    } else {
      KVR_TRY(gemm(h, attn, qd, w.o, delta, H, rows, H, qd, t));
    }
    if (r.tp_comm) KVR_TRY(allreduce(delta, rows * H, m.dtype, r.tp_comm, s));
    if (defer)
      KVR_TRY(add_rmsnorm_ex(hidden, nullptr, parts, o_split, H, rows * H, w.post_norm, normed, rows, H, H, H, H,
                             m.eps, m.dtype, stream, true));
    else
      KVR_TRY(add_rmsnorm_ex(hidden, delta, nullptr, 0, 0, 0, w.post_norm, normed, rows, H, H, H, H, m.eps, m.dtype,
                             stream, true));
    if (lin) {
      const kvr_linear_segment mlp = {w.gate, w.up, I, act, I};
      const kvr_linear_segment down = {w.down, nullptr, H, delta, H};
      KVR_TRY(project(normed, H, H, &mlp, 1));
      if (defer) {
        Deferred d = deferred(H, parts);
        KVR_TRY(project(act, I, I, &down, 1, &d));
        down_split = d.split;
      } else {
        KVR_TRY(project(act, I, I, &down, 1));
      }
    } else {
      bool gate_first = true;
      KVR_TRY(gemm_pair(h, normed, H, w.gate, w.up, gate, up, I, rows, I, H, t, &gate_first));
      KVR_TRY(kvr_silu_mul(gate_first ? gate : up, gate_first ? up : gate, act, rows, I, I, I, I, m.dtype, stream));
      KVR_TRY(gemm(h, act, I, w.down, delta, H, rows, H, I, t));
    }
    if (r.tp_comm) KVR_TRY(allreduce(delta, rows * H, m.dtype, r.tp_comm, s));
  }
#undef KVR_TRY
  return KVR_OK;
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Replay of repeated requests as CUDA graphs (request.graph_replay).
//
// The layer loop issues ~14 launches per layer; the cuBLAS kernels among them
// cannot start before their predecessor has drained (no programmatic launch),
// which costs ~2.5 us of idle GPU per boundary when launched into a stream and
// less inside a graph. A request that repeats an earlier call's launch key (the
// same model weights, geometry, options and every device pointer: cache,
// sources, ids, positions, rotary tables, workspace) issues exactly the same
// launches, so its second occurrence is captured once and later ones replay
// the graph. Positions and ids are read by the kernels at run time: a caller
// that stages each request's values into the same buffers (and drops or reuses
// its output cache) hits the cache with new data.
// ---------------------------------------------------------------------------
namespace kvr {
namespace {

constexpr size_t kGraphs = 4;  // executable graphs kept per (thread, device)
constexpr size_t kSeen = 8;    // keys run once, remembered for a capture on the next
unsigned long long g_replays = 0;

std::vector<uint64_t> graph_key(int dev, const kvr_model& m, const kvr_refresh_request& r, const void* ws,
                                size_t bytes) {
  std::vector<uint64_t> k;
  k.reserve(40 + 16 * static_cast<size_t>(m.num_layers));
  auto p = [&](const void* x) { k.push_back(static_cast<uint64_t>(reinterpret_cast<uintptr_t>(x))); };
  auto v = [&](int64_t x) { k.push_back(static_cast<uint64_t>(x)); };
  uint32_t eps_bits = 0;
  memcpy(&eps_bits, &m.eps, sizeof(eps_bits));
  v(dev), v(m.num_layers), v(m.hidden), v(m.q_heads), v(m.kv_heads), v(m.head_dim), v(m.intermediate);
  v(m.vocab), v(eps_bits), v(m.dtype), p(m.embed);
  for (int l = 0; l < m.num_layers; ++l) {
    const kvr_layer_weights& w = m.layers[l];
    for (const void* x : {w.input_norm, w.qkv, w.q, w.k, w.v, w.q_norm, w.k_norm, w.o, w.post_norm, w.gate, w.up,
                          w.down})
      p(x);
    p(r.k_cache[l]), p(r.v_cache[l]);
    if (r.k_src) p(r.k_src[l]), p(r.v_src[l]);
  }
  v(r.cache_rows), v(r.cache_head_stride), v(r.cache_row_stride), p(r.ids), v(r.id_count), p(r.positions);
  v(r.rows), v(r.max_position), p(r.cos_tab), p(r.sin_tab), v(r.attention_precision), p(r.tp_comm);
  v(r.projections), v(r.k_src != nullptr), v(r.src_head_stride), v(r.src_row_stride), p(ws), v(bytes);
  return k;
}

struct GraphEntry {
  std::vector<uint64_t> key;
  cudaGraphExec_t exec = nullptr;
  cudaEvent_t last = nullptr;  // recorded after each launch; eviction waits for it
  uint64_t launches = 0;       // library kernels in the graph
  uint64_t used = 0;
};

struct GraphCache {
  std::vector<GraphEntry> entries;
  std::vector<std::vector<uint64_t>> seen;  // oldest first
  uint64_t clock = 0;
  // Destroys every graph once its latest launch has finished and forgets the
  // keys; a thread that exits does this for its caches (at process exit the
  // runtime may already be gone, and its errors are ignored).
  int release() {
    cudaError_t first = cudaSuccess;
    for (GraphEntry& e : entries) {
      cudaError_t err = cudaEventSynchronize(e.last);
      if (err == cudaSuccess) err = cudaGraphExecDestroy(e.exec);
      cudaEventDestroy(e.last);
      if (first == cudaSuccess) first = err;
    }
    entries.clear();
    seen.clear();
    (void)cudaGetLastError();
    if (first != cudaSuccess) {
      set_last_cuda_error(first);
      return KVR_ERR_CUDA;
    }
    return KVR_OK;
  }
  ~GraphCache() { release(); }
};

std::unordered_map<int, GraphCache>& graph_caches() {
  thread_local std::unordered_map<int, GraphCache> caches;
  return caches;
}

GraphCache& graph_cache_for(int dev) { return graph_caches()[dev]; }

int launch_entry(GraphEntry& e, cudaStream_t s) {
  cudaError_t err = cudaGraphLaunch(e.exec, s);
  if (err == cudaSuccess) err = cudaEventRecord(e.last, s);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return KVR_ERR_CUDA;
  }
  count_launches(e.launches);
  __atomic_add_fetch(&g_replays, 1ull, __ATOMIC_RELAXED);
  return KVR_OK;
}

// Drops the least recently used graph once its latest launch has finished.
int evict_oldest(GraphCache& c) {
  size_t at = 0;
  for (size_t i = 1; i < c.entries.size(); ++i)
    if (c.entries[i].used < c.entries[at].used) at = i;
  GraphEntry& e = c.entries[at];
  cudaError_t err = cudaEventSynchronize(e.last);
  if (err == cudaSuccess) err = cudaGraphExecDestroy(e.exec);
  cudaEventDestroy(e.last);
  c.entries.erase(c.entries.begin() + static_cast<std::ptrdiff_t>(at));
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return KVR_ERR_CUDA;
  }
  return KVR_OK;
}

int refresh_graphed(const kvr_model* model, const kvr_refresh_request* req, void* ws, size_t bytes, void* stream) {
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return KVR_ERR_CUDA;
  }
  GraphCache& c = graph_cache_for(dev);
  std::vector<uint64_t> key = graph_key(dev, *model, *req, ws, bytes);
  const auto s = static_cast<cudaStream_t>(stream);
  for (GraphEntry& e : c.entries)
    if (e.key == key) {
      e.used = ++c.clock;
      return launch_entry(e, s);
    }
  auto seen = std::find(c.seen.begin(), c.seen.end(), key);
  if (seen == c.seen.end()) {
    // First occurrence: run directly and remember the key.
    const int st = refresh_direct(model, req, ws, bytes, stream);
    if (st == KVR_OK) {
      if (c.seen.size() >= kSeen) c.seen.erase(c.seen.begin());
      c.seen.push_back(std::move(key));
    }
    return st;
  }
  c.seen.erase(seen);
  // Second occurrence: capture the same launches on the idle capture stream,
  // then run the graph on the caller's stream. Anything that fails during the
  // capture leaves nothing behind and the call runs directly instead.
  RefreshStreams* cp = nullptr;
  int st = refresh_streams_for_current_device(&cp);
  if (st != KVR_OK) return st;
  err = cudaStreamBeginCapture(cp->capture, cudaStreamCaptureModeThreadLocal);
  if (err != cudaSuccess) {
    (void)cudaGetLastError();
    return refresh_direct(model, req, ws, bytes, stream);
  }
  uint64_t captured = 0;
  count_captured_launches(&captured);
  st = refresh_direct(model, req, ws, bytes, cp->capture);
  count_captured_launches(nullptr);
  cudaGraph_t graph = nullptr;
  err = cudaStreamEndCapture(cp->capture, &graph);
  cudaGraphExec_t exec = nullptr;
  // Kernel nodes keep the priority of the stream they were captured from (the
  // layer loop's high one, the copy's low one); without this flag the whole
  // graph would run at the priority of the stream it is launched into.
  if (st == KVR_OK && err == cudaSuccess && graph)
    err = cudaGraphInstantiate(&exec, graph, cudaGraphInstantiateFlagUseNodePriority);
  if (graph) cudaGraphDestroy(graph);
  if (st != KVR_OK || err != cudaSuccess || !exec) {
    if (exec) cudaGraphExecDestroy(exec);
    (void)cudaGetLastError();
    return refresh_direct(model, req, ws, bytes, stream);
  }
  GraphEntry e;
  e.key = std::move(key);
  e.exec = exec;
  e.launches = captured;
  e.used = ++c.clock;
  err = cudaEventCreateWithFlags(&e.last, cudaEventDisableTiming);
  if (err != cudaSuccess) {
    cudaGraphExecDestroy(exec);
    set_last_cuda_error(err);
    return KVR_ERR_CUDA;
  }
  if (c.entries.size() >= kGraphs) {
    st = evict_oldest(c);
    if (st != KVR_OK) {
      cudaGraphExecDestroy(exec);
      cudaEventDestroy(e.last);
      return st;
    }
  }
  c.entries.push_back(std::move(e));
  return launch_entry(c.entries.back(), s);
}

}  // namespace
}  // namespace kvr

extern "C" {

int kvr_debug_fail_refresh_after_layer(int layer) {
  g_fail_after_layer = layer < 0 ? -1 : layer;
  return KVR_OK;
}

int kvr_packed_refresh(const kvr_model* model, const kvr_refresh_request* req, void* workspace,
                       size_t workspace_bytes, void* stream) {
  if (g_fail_after_layer >= 0) return refresh_direct(model, req, workspace, workspace_bytes, stream);
  if (req && req->graph_replay && req->rows > 0 && !req->tp_comm && valid_model(model) && req->k_cache &&
      req->v_cache) {
    // The key and cache bookkeeping allocate host memory: no exception may
    // cross the C ABI.
    try {
      return refresh_graphed(model, req, workspace, workspace_bytes, stream);
    } catch (...) {
      count_captured_launches(nullptr);
      return KVR_ERR_CUDA;
    }
  }
  return refresh_direct(model, req, workspace, workspace_bytes, stream);
}

uint64_t kvr_graph_replays(void) { return __atomic_load_n(&g_replays, __ATOMIC_RELAXED); }

int kvr_release_graphs(void) {
  int st = KVR_OK;
  for (auto& entry : graph_caches()) {
    const int s = entry.second.release();
    if (st == KVR_OK) st = s;
  }
  return st;
}

int kvr_tp_unique_id(void* out) {
  if (!out) return KVR_ERR_INVALID_ARG;
  static_assert(sizeof(ncclUniqueId) == KVR_TP_ID_BYTES, "NCCL unique id size");
  ncclUniqueId id;
  if (ncclGetUniqueId(&id) != ncclSuccess) return KVR_ERR_CUDA;
  memcpy(out, &id, sizeof(id));
  return KVR_OK;
}

int kvr_tp_comm_init(const void* unique_id, int nranks, int rank, void** comm_out) {
  if (!unique_id || !comm_out || nranks < 1 || rank < 0 || rank >= nranks) return KVR_ERR_INVALID_ARG;
  ncclUniqueId id;
  memcpy(&id, unique_id, sizeof(id));
  ncclComm_t comm = nullptr;
  if (ncclCommInitRank(&comm, nranks, id, rank) != ncclSuccess) return KVR_ERR_CUDA;
  *comm_out = comm;
  return KVR_OK;
}

int kvr_tp_comm_destroy(void* comm) {
  if (!comm) return KVR_OK;
  return ncclCommDestroy(static_cast<ncclComm_t>(comm)) == ncclSuccess ? KVR_OK : KVR_ERR_CUDA;
}

}  // extern "C"
