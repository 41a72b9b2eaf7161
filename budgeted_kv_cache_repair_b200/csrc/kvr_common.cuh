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

// Call right after each <<<>>> launch.
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
