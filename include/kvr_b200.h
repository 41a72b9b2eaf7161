/*
 * kvr_b200.h - C ABI of the B200 packed refresh engine (libkvr_b200.so).
 *
 * Plain pointers, sizes and strides only. Every entry point:
 *   - returns an int status (KVR_OK or one of the KVR_ERR_* codes below),
 *   - validates its arguments on the host before launching anything,
 *   - launches on the caller's stream (`stream` is a cudaStream_t; NULL is the
 *     legacy default stream), never synchronises and never reads device memory
 *     back to the host,
 *   - lets no C++ exception cross the ABI.
 * Device pointers must belong to the current device. Element type codes are
 * KVR_DTYPE_BF16 and KVR_DTYPE_F16. Strides are in elements.
 *
 * Cache tensors use the reference layout [1, Hkv, N, D] per layer (transformers
 * DynamicCache), addressed here as (head_stride, row_stride) with unit stride
 * along D. Reference paths below are relative to yh0903/budgeted-kv-cache-repair.
 */
#ifndef KVR_B200_H
#define KVR_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define KVR_API __attribute__((visibility("default")))
#else
#define KVR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define KVR_OK 0
#define KVR_ERR_INVALID_ARG 1   /* bad pointer, size, stride or alignment */
#define KVR_ERR_UNSUPPORTED 2   /* shape/dtype outside the built kernels */
#define KVR_ERR_CUDA 3          /* a CUDA runtime call failed; see kvr_last_cuda_error */
#define KVR_ERR_TIMEOUT 4       /* a bounded device wait gave up */
#define KVR_ERR_SCRATCH_LIMIT 5 /* problem needs more than the static scratch array holds */
#define KVR_ERR_INJECTED 6      /* failure injected by kvr_debug_fail_refresh_after_layer */

#define KVR_DTYPE_BF16 0
#define KVR_DTYPE_F16 1
#define KVR_DTYPE_F32 2  /* kvr_query_relevance's embedding table only */

/* Largest number of per-layer tensors one multi-layer launch takes (K and V of
 * 128 layers). */
#define KVR_MAX_LAYER_TENSORS 256

/* Library identification and diagnostics. */
KVR_API const char* kvr_version(void);
KVR_API const char* kvr_status_string(int status);
/* cudaError_t of the last failing CUDA call in this thread (0 if none). */
KVR_API int kvr_last_cuda_error(void);
/* Kernels this library has launched in this process (all threads, all
 * devices), those run by replayed graphs included; a diagnostic counter for
 * benchmarks and tests. */
KVR_API uint64_t kvr_kernel_launches(void);
/* Packed refreshes this process ran as a CUDA graph (request.graph_replay):
 * the graph launches of captured keys, the capturing call's own included. */
KVR_API uint64_t kvr_graph_replays(void);
/* Diagnostics for failure handling; neither has a counterpart in the
 * reference, whose tests inject failures by patching Python (tests/
 * test_packed_cache.py:227-252).
 * kvr_set_wait_limit: SM clocks after which the pipeline waits of the kernels
 * launched from now on (attention, projections) give up and record an error
 * code in their workspace status word; 0 restores the default (~2 s). The
 * waits in which a CTA drains its own copies and MMAs before exiting keep the
 * default, so an early give-up still leaves nothing in flight. Process-wide.
 * kvr_debug_fail_refresh_after_layer: the calling thread's next
 * kvr_packed_refresh returns KVR_ERR_INJECTED right after launching layer
 * `layer`'s K/V scatter (the owned output cache is then partly written), the
 * way a CUDA call failing part-way through would end it; that call runs
 * directly, never from a cached graph. A negative layer disarms it. */
KVR_API int kvr_set_wait_limit(int64_t cycles);
KVR_API int kvr_debug_fail_refresh_after_layer(int layer);
/* Destroys the calling thread's cached refresh graphs (on every device, each
 * after its latest launch has finished) and forgets the keys seen once, e.g.
 * when a model is unloaded; later calls start over (direct, then capture). */
KVR_API int kvr_release_graphs(void);

/*
 * Output ownership copy of every layer: dst[t][h, n, :] = src[t][h, n, :] for
 * t < num_tensors (K and V of each layer, any order), h < heads, n < rows.
 * Replaces clone_cache (cache.py:31-44) as used by packed_interval_repair
 * (kernels/packed_cache.py:287). One launch for all given tensors.
 */
KVR_API int kvr_copy_layers(const void* const* src, void* const* dst, int num_tensors,
                    int heads, int64_t rows, int head_dim,
                    int64_t src_head_stride, int64_t src_row_stride,
                    int64_t dst_head_stride, int64_t dst_row_stride,
                    int dtype, void* stream);

/*
 * Delta-RoPE of retained suffix keys for every layer at once:
 *   dst[l][h, r, :] = src[l][h, r, :] * cos + rotate_half(src[l][h, r, :]) * sin
 * with cos/sin = cos_sin[0:D], cos_sin[D:2D] (one angle set: every row moves
 * by the same shift), each product and the sum rounded to the element type the
 * way torch's bf16/fp16 elementwise ops round them. src == dst is allowed;
 * otherwise a layer's src and dst must not overlap.
 * Replaces shifted_suffix_keys (cache.py:47-77) called per layer by
 * build_halo_cache (cache.py:129-139).
 */
KVR_API int kvr_rope_shift_layers(const void* const* src, void* const* dst, int num_layers,
                          int heads, int64_t rows, int head_dim,
                          int64_t src_head_stride, int64_t src_row_stride,
                          int64_t dst_head_stride, int64_t dst_row_stride,
                          const void* cos_sin, int dtype, void* stream);

/*
 * Whole shift cache for every layer in one launch (build_halo_cache with
 * halo 0, cache.py:103-144): for each layer, head and new row n < new_rows
 *   n <  prefix          : K, V copied from old row n
 *   n >= new_tail_start  : K rotated (as above; copied when apply_rope == 0)
 *                          and V copied from old row n - new_tail_start + old_tail_start
 * Rows in [prefix, new_tail_start) are left untouched (changed boundary tokens,
 * recomputed afterwards). k_old/v_old/k_new/v_new each hold num_layers pointers;
 * the new tensors must not overlap the old ones (the old rows are read through
 * the read-only data path while the new ones are written).
 */
KVR_API int kvr_shift_cache_layers(const void* const* k_old, const void* const* v_old,
                           void* const* k_new, void* const* v_new, int num_layers,
                           int heads, int head_dim, int64_t new_rows, int64_t prefix,
                           int64_t old_tail_start, int64_t new_tail_start,
                           int64_t old_head_stride, int64_t old_row_stride,
                           int64_t new_head_stride, int64_t new_row_stride,
                           const void* cos_sin, int apply_rope, int dtype, void* stream);

/*
 * Bitwise row scatter of fresh K/V into one layer's cache:
 *   k_cache[h, positions[r], :] = k_fresh[h, r, :] (same for V).
 * Positions outside [0, cache_rows) are skipped and counted in *error_count
 * (device int, may be NULL). Replaces indexed_kv_scatter_
 * (kernels/indexed_attention.py:179-204) and _PackedLayer.update's index_copy_
 * (kernels/packed_cache.py:189-191).
 */
KVR_API int kvr_scatter_rows(const void* k_fresh, const void* v_fresh, void* k_cache, void* v_cache,
                     const int64_t* positions, int64_t rows, int heads, int head_dim,
                     int64_t cache_rows,
                     int64_t fresh_head_stride, int64_t fresh_row_stride,
                     int64_t cache_head_stride, int64_t cache_row_stride,
                     int* error_count, int dtype, void* stream);

/*
 * Rotary cos/sin tables at the selected positions ([rows, 2*half_dim] each, the
 * element type), by the op sequence of the transformers rotary forward that
 * the reference's packed forward calls (LlamaRotaryEmbedding.forward, default
 * rope type): freq = inv_freq[i] * float(positions[r]) in fp32, cos/sin of
 * cat(freq, freq), times `scaling` (attention_scaling), cast to the element
 * type. inv_freq: device fp32 [half_dim].
 */
KVR_API int kvr_rope_tables(const float* inv_freq, int half_dim, const int64_t* positions, int64_t rows,
                            float scaling, void* cos_out, void* sin_out, int dtype, void* stream);

/*
 * Embedding gather of the selected rows (the native forward's embed_tokens on
 * edited_ids.index_select(1, positions), kernels/packed_cache.py:291):
 *   out[r, :] = embed[ids[positions[r]], :]
 * Out-of-range positions or ids write a zero row and increment *error_count.
 */
KVR_API int kvr_embed_rows(const void* embed, int64_t vocab, int hidden,
                   const int64_t* ids, int64_t id_count, const int64_t* positions, int64_t rows,
                   void* out, int* error_count, int dtype, void* stream);

/*
 * Residual add fused with RMSNorm (transformers LlamaRMSNorm / Qwen3RMSNorm and
 * the decoder layer's `residual + hidden_states`):
 *   if delta != NULL: hidden = round(hidden + delta)   (written back in place)
 *   out = round(weight * round(hidden * rsqrt(mean(hidden^2) + eps)))
 * mean in fp32. Row-major [rows, hidden_size] with row strides.
 */
KVR_API int kvr_add_rmsnorm(void* hidden, const void* delta, const void* weight, void* out,
                    int64_t rows, int hidden_size, int64_t hidden_stride, int64_t delta_stride,
                    int64_t out_stride, float eps, int dtype, void* stream);

/*
 * Per-layer K/V epilogue of the packed forward, fused (kernels/packed_cache.py:
 * 290-295 through the native attention module and _PackedLayer.update):
 *   q  = RoPE(q_norm(q))       -> q_out[r, head, :]       (q_norm only if q_norm_w)
 *   k  = RoPE(k_norm(k))       -> k_cache[h, positions[r], :]
 *   v                          -> v_cache[h, positions[r], :]   (bitwise)
 * q_in/k_in/v_in: GEMM outputs [rows, heads*D] with row strides. cos/sin:
 * [rows, D] tables of the element type (rotary_emb at the selected positions).
 * q_out: [rows, q_heads, D] contiguous; may be NULL (K/V only, e.g. the last
 * layer). Out-of-range positions are skipped and counted in *error_count.
 */
KVR_API int kvr_qkv_rope_scatter(const void* q_in, const void* k_in, const void* v_in,
                         int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                         const void* q_norm_w, const void* k_norm_w, float eps,
                         const void* cos_tab, const void* sin_tab, const int64_t* positions,
                         int64_t rows, int q_heads, int kv_heads, int head_dim,
                         void* q_out, void* k_cache, void* v_cache, int64_t cache_rows,
                         int64_t cache_head_stride, int64_t cache_row_stride,
                         int* error_count, int dtype, void* stream);

/*
 * MLP activation: out = round(round(silu(gate)) * up), elementwise over
 * [rows, width] (transformers LlamaMLP.forward: act_fn(gate_proj(x)) * up_proj(x)).
 */
KVR_API int kvr_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int64_t width,
                 int64_t gate_stride, int64_t up_stride, int64_t out_stride,
                 int dtype, void* stream);

/*
 * Projections of the selected rows on sm_100a tensor cores, for the few
 * dozen rows of a refresh: out = x . weight^T (nn.Linear, fp32 accumulation,
 * one rounding), for up to KVR_LINEAR_MAX_SEGMENTS weight matrices that share
 * the input x in ONE launch (q/k/v as three segments). A segment with
 * weight_up set is the gated MLP: out = round(round(silu(round(x . weight^T)))
 * * round(x . weight_up^T)) (LlamaMLP's act_fn(gate_proj(x)) * up_proj(x)).
 * Replaces the nn.Linear calls of the decoder modules that the reference's
 * packed forward runs (q/k/v/o_proj, gate/up/down_proj under
 * kernels/packed_cache.py:284-297); cuBLAS stays the path for many rows.
 *
 * x: [rows, k] with row stride x_stride (16-byte aligned base, stride and k
 * multiples of 8). weight(_up): [n, k] contiguous, 16-byte aligned. out:
 * [rows, n] with row stride out_stride. Summation order is fixed: results do
 * not depend on the run. `workspace` (kvr_linear_workspace_size bytes, any
 * contents) starts with a status word: 0, or the code of a bounded
 * device-side wait that gave up. Calls that overlap on the GPU must not share
 * a workspace.
 */
#define KVR_LINEAR_MAX_SEGMENTS 4
typedef struct kvr_linear_segment {
  const void* weight;      /* [n, k] */
  const void* weight_up;   /* NULL, or [n, k]: gated-MLP segment */
  int64_t n;
  void* out;               /* [rows, out_stride] */
  int64_t out_stride;
} kvr_linear_segment;
KVR_API size_t kvr_linear_workspace_size(int64_t rows, int64_t k, const kvr_linear_segment* segments, int count);
KVR_API int kvr_linear(const void* x, int64_t x_stride, int64_t rows, int64_t k,
                       const kvr_linear_segment* segments, int count, void* workspace,
                       size_t workspace_bytes, int dtype, void* stream);

/*
 * Selected-query absolute-causal attention with GQA on sm_100a tensor cores
 * (tcgen05 MMA with TMEM accumulators, TMA-fed K/V).
 * q [rows, q_heads, D] contiguous; K/V [kv_heads, cache_rows, D] with strides;
 * out [rows, q_heads, D] contiguous. Row r attends keys 0..positions[r]
 * (inclusive); positions must be strictly increasing (as IndexedPlan
 * guarantees) and max_position must equal positions[rows-1]. Query head j
 * reads KV head j / (q_heads / kv_heads). softmax(scale * q.k) in fp32, one
 * rounding on output. `precision` selects how probabilities enter the P.V
 * product: KVR_ATTN_P_SPLIT (P = P_hi + P_lo in the element type, ~16
 * mantissa bits) or KVR_ATTN_P_ROUNDED (one rounding, as fused SDPA kernels do).
 * Replaces _packed_attention's SDPA call with its dense [1,1,B,N] mask and
 * repeat_kv (kernels/packed_cache.py:47-67, 203-207) and the experimental
 * indexed_causal_attention (kernels/indexed_attention.py:207-241).
 *
 * `workspace` is device memory of at least kvr_attention_workspace_size()
 * bytes (any contents). Its first 4 bytes receive a status word: 0, or the
 * code of a bounded device-side wait that gave up (then the output is not
 * valid). When rows are few the key range is split across CTAs and partial
 * results go to the rest of the workspace, merged by a second launch on the
 * same stream. Calls that overlap on the GPU must not share a workspace.
 */
#define KVR_ATTN_P_SPLIT 0
#define KVR_ATTN_P_ROUNDED 1
KVR_API size_t kvr_attention_workspace_size(int64_t rows, int q_heads, int kv_heads, int head_dim,
                                            int64_t cache_rows);
KVR_API int kvr_selected_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                                   const int64_t* positions, int64_t rows, int q_heads, int kv_heads,
                                   int head_dim, int64_t cache_rows,
                                   int64_t cache_head_stride, int64_t cache_row_stride,
                                   int64_t max_position, float scale, int precision,
                                   void* workspace, size_t workspace_bytes, int dtype, void* stream);

/*
 * Whole packed refresh in one call: the selected rows run through every
 * decoder layer of a dense Llama/Qwen3 model on `stream`, and each layer's
 * fresh K/V rows are written into the cache at their absolute positions.
 * Replaces the native transformers forward of packed_interval_repair
 * (kernels/packed_cache.py:284-297: _make_native_view, the _PackedLayer cache
 * and the per-layer decoder modules). Weights are the model's own tensors
 * (row-major [out, in], nn.Linear layout); `qkv` may point to the rows of
 * Wq, Wk, Wv stacked into one matrix (one GEMM per layer) or be NULL with
 * q/k/v set. q_norm/k_norm are the Qwen3 per-head RMSNorm weights or NULL.
 * The caller owns the output cache and has already copied the base into it;
 * cos_tab/sin_tab are the model's rotary cos/sin at the selected positions
 * ([rows, head_dim], model dtype). `workspace` holds
 * kvr_packed_refresh_workspace_size() bytes of activations and attention
 * scratch (any contents). Projections run on cuBLAS or on the kvr_linear
 * kernel (request.projections), with fp32 accumulation either way.
 */
typedef struct kvr_layer_weights {
  const void* input_norm;  /* [hidden] */
  const void* qkv;         /* [(q_heads + 2*kv_heads) * head_dim, hidden] or NULL */
  const void* q;           /* [q_heads * head_dim, hidden] (when qkv == NULL) */
  const void* k;           /* [kv_heads * head_dim, hidden] */
  const void* v;           /* [kv_heads * head_dim, hidden] */
  const void* q_norm;      /* [head_dim] or NULL */
  const void* k_norm;      /* [head_dim] or NULL */
  const void* o;           /* [hidden, q_heads * head_dim] */
  const void* post_norm;   /* [hidden] */
  const void* gate;        /* [intermediate, hidden] */
  const void* up;          /* [intermediate, hidden] */
  const void* down;        /* [hidden, intermediate] */
} kvr_layer_weights;

typedef struct kvr_model {
  int num_layers, hidden, q_heads, kv_heads, head_dim, intermediate;
  int64_t vocab;
  float eps;               /* rms_norm_eps */
  int dtype;               /* KVR_DTYPE_* of weights, cache and activations */
  const void* embed;       /* [vocab, hidden] */
  const kvr_layer_weights* layers;  /* num_layers entries (host memory) */
} kvr_model;

typedef struct kvr_refresh_request {
  void* const* k_cache;    /* num_layers device pointers, [kv_heads, cache_rows, head_dim] */
  void* const* v_cache;
  int64_t cache_rows, cache_head_stride, cache_row_stride;
  const int64_t* ids;      /* device [id_count] token ids of the edited prompt */
  int64_t id_count;
  const int64_t* positions;  /* device [rows], strictly increasing */
  int64_t rows;
  int64_t max_position;    /* positions[rows-1], from the host plan */
  const void* cos_tab;     /* device [rows, head_dim] */
  const void* sin_tab;
  int attention_precision; /* KVR_ATTN_P_* */
  void* tp_comm;           /* NULL, or a communicator from kvr_tp_comm_init: the model is this
                              rank's head/column shard and the o/down partial sums are
                              all-reduced (sum) across the group after each projection */
  int projections;         /* KVR_PROJ_*: which GEMMs run the q/k/v, o, gate/up and down
                              projections (requests above 256 rows always use cuBLAS) */
  const void* const* k_src;  /* NULL, or num_layers source layers (same geometry as the cache):
                              the call first makes k_cache/v_cache an ownership copy of
                              k_src/v_src (clone_cache, kernels/packed_cache.py:287). The layer
                              loop then runs on an internal high-priority stream and layer l
                              is copied on a low-priority one while earlier layers compute
                              (layer l is first written only after its copy); `stream` waits
                              for both before any later work on it */
  const void* const* v_src;
  int64_t src_head_stride, src_row_stride;
  int graph_replay;        /* 0: launch every kernel into `stream`. 1: key the call on the model's
                              weights, the geometry and options and every pointer of the request
                              and the workspace; a key's second call is captured into a CUDA graph
                              (on an internal stream, nothing runs during the capture) and that and
                              later calls with the key launch the graph into `stream` (same kernels
                              and results; the cuBLAS boundaries drain faster inside a graph).
                              Kernels read ids, positions, tables, weights and sources at run time,
                              so staging new values into the same buffers replays with them. Up to 4
                              graphs per (thread, device); tensor-parallel calls run directly. */
} kvr_refresh_request;
#define KVR_PROJ_CUBLAS 0  /* cuBLAS GEMMs, fp32 accumulation */
#define KVR_PROJ_SM100 1   /* kvr_linear's weight-streaming kernel, gate/up fused with SiLU */
#define KVR_PROJ_FUSED 2   /* fused projections (up to 128 rows, head_dim 128, no tensor parallelism;
                              other requests run on cuBLAS): four launches per layer, the q/k/v one
                              with q/k-norm + RoPE + K/V scatter, o and down with the residual add,
                              gate/up with the post-attention RMSNorm applied to its input and SiLU*up */

/*
 * Tensor-parallel group for kvr_packed_refresh (NCCL over NVLink). No
 * counterpart in the reference, which runs on one device (api.py:156-160).
 * kvr_tp_unique_id writes KVR_TP_ID_BYTES bytes on one rank; every rank passes
 * the same bytes to kvr_tp_comm_init (collective over the group, with each
 * rank's device current). kvr_tp_comm_destroy releases it.
 */
#define KVR_TP_ID_BYTES 128
KVR_API int kvr_tp_unique_id(void* out);
KVR_API int kvr_tp_comm_init(const void* unique_id, int nranks, int rank, void** comm_out);
KVR_API int kvr_tp_comm_destroy(void* comm);

KVR_API size_t kvr_packed_refresh_workspace_size(const kvr_model* model, int64_t rows, int64_t cache_rows);
KVR_API int kvr_packed_refresh(const kvr_model* model, const kvr_refresh_request* request, void* workspace,
                               size_t workspace_bytes, void* stream);

/*
 * kvr_selected_attention without a caller-provided workspace, for callers
 * that cannot allocate device memory per call (for example a host runtime
 * reaching this library over a plain C FFI with a fixed, pre-planned GPU
 * memory budget and no caching allocator, where a cudaMalloc would
 * synchronise the device). It has no counterpart in the reference.
 *
 * Scratch comes from one file-scope device array of KVR_STATIC_SCRATCH_BYTES
 * (16 MiB) that every GPU loading the library holds until the process exits.
 * Problems whose partial results need more return KVR_ERR_SCRATCH_LIMIT
 * before any launch (kvr_attention_workspace_size() tells the need). The
 * first call on a device looks up the array's device address with that
 * device current, so make it before any stream capture. All calls share the
 * array and it keeps the last call's contents (the status word at offset 0 is
 * cleared on the stream before each launch): calls that overlap on the GPU,
 * on any streams, race. Nothing here calls cudaMalloc, cudaFree or an
 * allocating library routine. Arguments and results otherwise match
 * kvr_selected_attention; the status word (0, or the code of a bounded device
 * wait that gave up, when the output is not valid) lives in the array's first
 * 4 bytes and kvr_attention_static_status reads it.
 */
#define KVR_STATIC_SCRATCH_BYTES (16u << 20)
KVR_API int kvr_selected_attention_static(const void* q, const void* k_cache, const void* v_cache, void* out,
                                          const int64_t* positions, int64_t rows, int q_heads, int kv_heads,
                                          int head_dim, int64_t cache_rows,
                                          int64_t cache_head_stride, int64_t cache_row_stride,
                                          int64_t max_position, float scale, int precision,
                                          int dtype, void* stream);
/* Copies the status word of the last kvr_selected_attention_static call on the
 * current device into *status_out (host or device memory) with one 4-byte
 * cudaMemcpyAsync on `stream`; read it after the stream has reached the copy.
 * Like the variant it serves, it has no counterpart in the reference. */
KVR_API int kvr_attention_static_status(int* status_out, void* stream);

/*
 * Query relevance of prompt tokens from the frozen input embeddings
 * (dense_query_relevance_scores, scoring.py:11-72), the scoring step of
 * select_support's SUR allocation (api.py:83-96):
 *   scores[t] = max_q cos(E[prompt_ids[t]], E[query_ids[q]])
 *               + exact_boost * [prompt_ids[t] in query_ids]
 * with E the [vocab, hidden] table (dtype KVR_DTYPE_BF16/F16/F32, rows
 * contiguous), cosine through x / max(||x||, 1e-12) in fp32. scores: fp32
 * [prompt_count] on the device. The workspace (kvr_query_relevance_workspace_size
 * bytes) holds the normalised query rows; its first 4 bytes count ids outside
 * [0, vocab) (those scores are NaN): read it with the scores.
 */
KVR_API size_t kvr_query_relevance_workspace_size(int hidden, int query_count);
KVR_API int kvr_query_relevance(const void* embed, int64_t vocab, int hidden, int dtype, const int64_t* prompt_ids,
                                int64_t prompt_count, const int64_t* query_ids, int query_count, float exact_boost,
                                float* scores, void* workspace, size_t workspace_bytes, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* KVR_B200_H */
