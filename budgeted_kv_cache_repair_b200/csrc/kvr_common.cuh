// Shared helpers for the kvr_b200 kernels: element types, torch-compatible
// rounding, launch bookkeeping and the C-ABI status plumbing.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/kvr_b200.h"

namespace kvr {

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

// Records the CUDA error of the calling thread for kvr_last_cuda_error().
void set_last_cuda_error(cudaError_t e);
// Adds to the process-wide launch counter behind kvr_kernel_launches().
void count_launch();
// Adds n launches at once (the kernels of a replayed CUDA graph).
void count_launches(uint64_t n);
// Default limit, in SM clocks (~2 s), of every bounded device wait.
constexpr long long kDefaultWaitLimit = 4000000000LL;
// Limit of the pipeline waits (producer/consumer hand-offs) of the kernels
// launched from now on: kDefaultWaitLimit unless kvr_set_wait_limit changed
// it. The waits that drain a CTA's own copies and MMAs before it exits always
// use kDefaultWaitLimit.
long long pipeline_wait_limit();
// While `sink` is set, this thread's launches are being captured into a graph
// (recorded, not run): count_launch() adds to *sink instead. NULL ends it.
void count_captured_launches(uint64_t* sink);

// kvr_selected_attention; with status_zeroed the caller has zeroed the status
// word at the start of `workspace` and no memset is issued.
int selected_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                       const int64_t* positions, int64_t rows, int q_heads, int kv_heads, int head_dim,
                       int64_t cache_rows, int64_t cache_head_stride, int64_t cache_row_stride,
                       int64_t max_position, float scale, int precision, void* workspace, size_t workspace_bytes,
                       int dtype, void* stream, bool status_zeroed);

// kvr_add_rmsnorm whose delta may instead be a deferred projection: nparts
// fp32 slices (row stride part_stride, slice stride part_slice floats),
// summed in order and rounded before the residual add. weight_early: the norm
// weight is not written by any kernel of the programmatic launch chain, so it
// is loaded before the wait on the previous kernel.
int add_rmsnorm_ex(void* hidden, const void* delta, const float* parts, int nparts, int64_t part_stride,
                   int64_t part_slice, const void* weight, void* out, int64_t rows, int hidden_size,
                   int64_t hidden_stride, int64_t delta_stride, int64_t out_stride, float eps, int dtype,
                   void* stream, bool weight_early);

// Deferred q/k/v projection for qkv_rope_scatter_ex: `count` fp32 slices of
// [rows][row_stride] (slice stride `slice` floats), q/k/v at columns
// q_col/k_col/v_col.
struct QkvParts {
  const float* data;
  int count;
  int64_t row_stride, slice, q_col, k_col, v_col;
};

// kvr_qkv_rope_scatter reading q/k/v from `parts` when given (q_in/k_in/v_in
// are then unused). consts_early: positions, cos/sin and norm weights are
// written by no kernel of the programmatic launch chain, so they are loaded
// before the wait on the previous kernel.
int qkv_rope_scatter_ex(const void* q_in, const void* k_in, const void* v_in, int64_t q_row_stride,
                        int64_t k_row_stride, int64_t v_row_stride, const void* q_norm_w, const void* k_norm_w,
                        float eps, const void* cos_tab, const void* sin_tab, const int64_t* positions,
                        int64_t rows, int q_heads, int kv_heads, int head_dim, void* q_out, void* k_cache,
                        void* v_cache, int64_t cache_rows, int64_t cache_head_stride, int64_t cache_row_stride,
                        int* error_count, int dtype, void* stream, const QkvParts* parts, bool consts_early);

// Two fp32 values in one 64-bit register, for the packed fp32 ALU ops of
// sm_100 (one instruction for two lanes of a row).
__device__ __forceinline__ uint64_t f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// Call right after each kernel launch.
inline int check_launch() {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  count_launch();
  return KVR_OK;
}

inline bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// ---------------------------------------------------------------------------
// Programmatic dependent launch. Every kernel of the library is launched with
// programmatic stream serialization allowed, so it may start while the
// kernel before it in the stream is still running. Its threads call
// pdl_wait() before touching any memory that an earlier kernel writes or
// reads (then all earlier kernels have completed and their writes are
// visible), and pdl_launch_dependents() first thing, so that the kernel after
// it may start its own independent prologue early (the projection kernel uses
// that time to load its first weight tiles; everything it does before its own
// pdl_wait() reads only weights). Without the launch attribute both are no-ops.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;\n" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;\n" ::: "memory");
}

// Per-device once: prefer the largest shared-memory split of L1 for `kernel`,
// so that the SM keeps one configuration across the layer loop's kernels (the
// projection and attention kernels need it) instead of switching between
// consecutive launches. The HBM-streaming cache kernels opt out
// (launch_pdl_default_carveout).
template <auto kernel>
inline void prefer_shared_once() {
  static int done[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
    cudaGetLastError();
    return;
  }
  if (__atomic_load_n(&done[dev], __ATOMIC_ACQUIRE)) return;
  if (cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared) != cudaSuccess)
    cudaGetLastError();  // a preference only
  __atomic_store_n(&done[dev], 1, __ATOMIC_RELEASE);
}

// Launch `kernel` on `stream` with programmatic dependent launch allowed
// (optionally in clusters of `cluster` CTAs along x); counts the launch. The
// kernel keeps the driver's choice of L1 / shared-memory split: for kernels
// that stream HBM through L1-allocating loads, whose loads in flight need L1
// space (a cache copy ran at 1.05 of the measured copy peak with the default
// split and at 0.89 with the largest shared-memory one).
template <auto kernel, class... Args>
inline int launch_pdl_default_carveout(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster,
                                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  int n = 1;
  if (cluster > 1) {
    attr[1].id = cudaLaunchAttributeClusterDimension;
    attr[1].val.clusterDim.x = static_cast<unsigned>(cluster);
    attr[1].val.clusterDim.y = 1;
    attr[1].val.clusterDim.z = 1;
    n = 2;
  }
  cfg.attrs = attr;
  cfg.numAttrs = n;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kernel, args...);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    cudaGetLastError();
    return KVR_ERR_CUDA;
  }
  return check_launch();
}

// launch_pdl_default_carveout after preferring the largest shared-memory split
// for `kernel` (the library's default, see prefer_shared_once).
template <auto kernel, class... Args>
inline int launch_pdl(dim3 grid, dim3 block, size_t smem, cudaStream_t stream, int cluster, Args... args) {
  prefer_shared_once<kernel>();
  return launch_pdl_default_carveout<kernel>(grid, block, smem, stream, cluster, args...);
}

// ---------------------------------------------------------------------------
// Element types. Storage is 16-bit; arithmetic is fp32 with one rounding per
// torch elementwise op, which is what torch's CUDA/CPU kernels do for
// bf16/fp16 tensors (load -> float -> op -> round to nearest even).
// ---------------------------------------------------------------------------

// fp32 -> bf16, round to nearest even; NaN becomes the canonical quiet NaN
// 0x7FC0 (c10::BFloat16's conversion, used by every torch op on bf16).
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0u;
  u += 0x7fffu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

__device__ __forceinline__ float bf16_bits_to_f32(uint16_t h) {
  return __uint_as_float(static_cast<uint32_t>(h) << 16);
}

struct BF16 {
  static __device__ __forceinline__ float to_f(uint16_t b) { return bf16_bits_to_f32(b); }
  static __device__ __forceinline__ uint16_t from_f(float f) { return f32_to_bf16_bits(f); }
};

struct F16 {
  static __device__ __forceinline__ float to_f(uint16_t b) {
    return __half2float(__ushort_as_half(b));
  }
  static __device__ __forceinline__ uint16_t from_f(float f) {
    return __half_as_ushort(__float2half_rn(f));
  }
};

// Round-trip through the element type.
template <class T>
__device__ __forceinline__ float rnd(float f) {
  return T::to_f(T::from_f(f));
}

// SiLU(gate) * up with the transformers MLP's roundings (act_fn(gate_proj(x)) *
// up_proj(x) on 16-bit tensors): SiLU of the rounded gate in fp32, rounded,
// then the product rounded. `gate` and `up` are already element-type values.
template <class T>
__device__ __forceinline__ uint16_t silu_mul_elem(float gate, float up) {
  const float act = rnd<T>(gate / (1.0f + expf(-gate)));
  return T::from_f(__fmul_rn(act, up));
}

// The same with the quotient of SiLU from the fast division (within 2 fp32
// ulps of gate / (1 + exp(-gate)); the rounded 16-bit result differs from the
// exact one only when the fp32 quotient lies within 2 ulps of a rounding
// boundary, about 2^-14 of inputs). IEEE division carries a slow-path call
// that made the projection epilogue several times slower.
template <class T>
__device__ __forceinline__ uint16_t silu_mul_elem_fast(float gate, float up) {
  const float act = rnd<T>(__fdividef(gate, 1.0f + expf(-gate)));
  return T::from_f(__fmul_rn(act, up));
}

// 8 x 16-bit elements = one 128-bit access.
struct alignas(16) Vec8 {
  uint16_t h[8];
};

__device__ __forceinline__ Vec8 ld_vec8(const void* p) {
  uint4 u = *reinterpret_cast<const uint4*>(p);
  Vec8 v;
  *reinterpret_cast<uint4*>(&v) = u;
  return v;
}

__device__ __forceinline__ Vec8 ld_vec8_stream(const void* p) {
  uint4 u = __ldcs(reinterpret_cast<const uint4*>(p));
  Vec8 v;
  *reinterpret_cast<uint4*>(&v) = u;
  return v;
}

__device__ __forceinline__ void st_vec8(void* p, const Vec8& v) {
  *reinterpret_cast<uint4*>(p) = *reinterpret_cast<const uint4*>(&v);
}

__device__ __forceinline__ void st_vec8_stream(void* p, const Vec8& v) {
  __stcs(reinterpret_cast<uint4*>(p), *reinterpret_cast<const uint4*>(&v));
}

// ---------------------------------------------------------------------------
// RoPE in torch's op order: out = round(round(x*c) + round(rotate_half(x)*s)).
// rotate_half(x)[d] = -x[d + D/2] for d < D/2, x[d - D/2] otherwise.
// ---------------------------------------------------------------------------
template <class T>
__device__ __forceinline__ uint16_t rope_elem(float x, float partner_rot, float c, float s) {
  // partner_rot is rotate_half(x)[d] already negated where needed (exact).
  float t1 = rnd<T>(__fmul_rn(x, c));
  float t2 = rnd<T>(__fmul_rn(partner_rot, s));
  return T::from_f(__fadd_rn(t1, t2));
}

// The same value with the hardware round-to-nearest-even conversions
// (cvt.rn.bf16.f32 / cvt.rn.f16.f32 instead of the integer rounding of
// f32_to_bf16_bits): a few instructions per rounding instead of about ten.
// Finite values round identically; a NaN result becomes the quiet NaN that
// torch's conversion writes (0x7FC0 for bf16), so the result is bit-identical
// to rope_elem.
template <class T>
__device__ __forceinline__ uint16_t rope_elem_hw(float x, float partner_rot, float c, float s);

template <>
__device__ __forceinline__ uint16_t rope_elem_hw<BF16>(float x, float partner_rot, float c, float s) {
  const float t1 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(x, c)));
  const float t2 = __bfloat162float(__float2bfloat16_rn(__fmul_rn(partner_rot, s)));
  const float r = __fadd_rn(t1, t2);
  const uint16_t b = __bfloat16_as_ushort(__float2bfloat16_rn(r));
  return r != r ? static_cast<uint16_t>(0x7fc0u) : b;
}

template <>
__device__ __forceinline__ uint16_t rope_elem_hw<F16>(float x, float partner_rot, float c, float s) {
  return rope_elem<F16>(x, partner_rot, c, s);  // F16 rounding is already the hardware conversion
}

// Pointer arrays passed by value (kernel parameters hold up to 32 KB).
struct LayerPtrs {
  const void* src[KVR_MAX_LAYER_TENSORS];
  void* dst[KVR_MAX_LAYER_TENSORS];
};

inline int grid_for(int64_t work_items, int threads, int per_sm = 8) {
  int64_t blocks = (work_items + threads - 1) / threads;
  int64_t cap = static_cast<int64_t>(kNumSMs) * per_sm;
  if (blocks > cap) blocks = cap;
  if (blocks < 1) blocks = 1;
  return static_cast<int>(blocks);
}

}  // namespace kvr
