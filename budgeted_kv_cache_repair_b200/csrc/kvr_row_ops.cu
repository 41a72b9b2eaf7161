// Per-layer row kernels of the packed forward: residual add + RMSNorm, the
// fused K/V epilogue (q/k-norm, RoPE, q packing, K/V scatter into the cache),
// and the MLP activation. Each reproduces the rounding points of the
// transformers modules the reference drives (one rounding per torch op).
#include "kvr_common.cuh"

namespace kvr {

constexpr int kNormThreads = 256;
constexpr int kNormMaxVecs = 4;  // hidden_size <= 256 * 4 * 8 = 8192

// A kernel as a type, for generic launch helpers.
template <auto K>
struct KernelRef {
  static constexpr auto value = K;
};

// Sum of `n` fp32 partial slices of 8 consecutive values, in slice order,
// rounded to the element type (a deferred projection output).
// Loads of up to kPartBatch slices are all issued before any add (one memory
// round trip per batch); the adds keep slice order.
constexpr int kPartBatch = 8;

template <class T>
__device__ __forceinline__ Vec8 sum_parts8(const float* p, int n, int64_t slice) {
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
  for (int s0 = 0; s0 < n; s0 += kPartBatch) {
    float4 a[kPartBatch], b[kPartBatch];
#pragma unroll
    for (int i = 0; i < kPartBatch; ++i) {
      if (s0 + i < n) {
        a[i] = __ldcg(reinterpret_cast<const float4*>(p + (s0 + i) * slice));
        b[i] = __ldcg(reinterpret_cast<const float4*>(p + (s0 + i) * slice + 4));
      }
    }
#pragma unroll
    for (int i = 0; i < kPartBatch; ++i) {
      if (s0 + i < n) {
        acc[0] += a[i].x; acc[1] += a[i].y; acc[2] += a[i].z; acc[3] += a[i].w;
        acc[4] += b[i].x; acc[5] += b[i].y; acc[6] += b[i].z; acc[7] += b[i].w;
      }
    }
  }
  Vec8 v;
#pragma unroll
  for (int e = 0; e < 8; ++e) v.h[e] = T::from_f(acc[e]);
  return v;
}

// With nparts > 0 the delta is a deferred projection: nparts fp32 slices
// (row stride p_stride, slice stride p_slice floats), summed and rounded here.
// VPT: 16-byte vectors per thread (ceil(hidden / 8 / kNormThreads)) and
// PARTS (the delta is deferred fp32 slices) are template parameters so that
// registers, and with them the CTAs resident per SM, follow the work
// (hundreds of rows run in many waves).
template <class T, int VPT, bool PARTS>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(
    uint16_t* hidden, const uint16_t* __restrict__ delta, const uint16_t* __restrict__ weight,
    uint16_t* out, int vpr, int64_t h_stride, int64_t d_stride, int64_t o_stride, float inv_h,
    float eps, const float* __restrict__ parts, int nparts, int64_t p_stride, int64_t p_slice, int weight_early) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  // With weight_early (the layer loop: the norm weight is a model constant)
  // the weight is fetched before the wait, so its load overlaps the previous
  // kernel instead of following the reduction.
  Vec8 w[VPT];
  if (weight_early) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * kNormThreads;
      if (v < vpr) w[k] = ld_vec8(weight + v * 8);
    }
  }
  pdl_wait();  // every other input may come from the previous kernel
  if (!weight_early) {
#pragma unroll
    for (int k = 0; k < VPT; ++k) {
      const int v = threadIdx.x + k * kNormThreads;
      if (v < vpr) w[k] = ld_vec8(weight + v * 8);
    }
  }
  const int64_t r = blockIdx.x;
  uint16_t* hrow = hidden + r * h_stride;
  // Every load of the row (hidden, then the delta or its partial slices) is
  // issued before the first store back to `hidden`: one memory round trip.
  Vec8 x[VPT], dv[VPT];
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * kNormThreads;
    if (v < vpr) {
      x[k] = ld_vec8(hrow + v * 8);
      if constexpr (PARTS)
        dv[k] = sum_parts8<T>(parts + r * p_stride + v * 8, nparts, p_slice);
      else if (delta)
        dv[k] = ld_vec8(delta + r * d_stride + v * 8);
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * kNormThreads;
    if (v < vpr) {
      if (PARTS || delta) {
        // residual + hidden_states, rounded to the element type.
#pragma unroll
        for (int e = 0; e < 8; ++e) x[k].h[e] = T::from_f(__fadd_rn(T::to_f(x[k].h[e]), T::to_f(dv[k].h[e])));
        st_vec8(hrow + v * 8, x[k]);
      }
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float f = T::to_f(x[k].h[e]);
        ss = __fmaf_rn(f, f, ss);
      }
    }
  }
  // Block reduction of the sum of squares.
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
    if (threadIdx.x == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = rsqrtf(__fadd_rn(red[0] * inv_h, eps));
#pragma unroll
  for (int k = 0; k < VPT; ++k) {
    const int v = threadIdx.x + k * kNormThreads;
    if (v < vpr) {
      Vec8 y;
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        const float normed = rnd<T>(__fmul_rn(T::to_f(x[k].h[e]), inv));
        y.h[e] = T::from_f(__fmul_rn(T::to_f(w[k].h[e]), normed));
      }
      st_vec8(out + r * o_stride + v * 8, y);
    }
  }
}

// One warp per (row, head slot). Slots [0, q_heads) are query heads (when q_out
// is given), then kv_heads key heads, then kv_heads value heads. Lane l holds
// elements [l*E, l*E+E) of the head (E = D/32); its RoPE partner d +- D/2
// lives in lane l ^ 16.
struct QkvArgs {
  const uint16_t* q_in;
  const uint16_t* k_in;
  const uint16_t* v_in;
  int64_t q_rs, k_rs, v_rs;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  float eps;
  const uint16_t* cos_tab;
  const uint16_t* sin_tab;
  const int64_t* positions;
  int64_t rows;
  int q_heads, kv_heads;
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int64_t cache_rows, c_hs, c_rs;
  int* error_count;
  // Deferred projection (nparts > 0): q/k/v are nparts fp32 slices of
  // [rows][p_rs] at columns q_col/k_col/v_col, summed and rounded here.
  const float* parts;
  int nparts;
  int64_t p_rs, p_slice, q_col, k_col, v_col;
  // Positions, cos/sin tables and norm weights are written by no kernel of the
  // programmatic launch chain (the layer loop): load them before the wait.
  int consts_early;
};

// PARTS: q/k/v come as deferred fp32 slices (a.nparts > 0); a template
// parameter so the direct path keeps the registers of the slice sums free.
template <class T, int D, bool PARTS>
__global__ void __launch_bounds__(256) qkv_rope_scatter_kernel(QkvArgs a) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  constexpr int E = D / 32;  // 4 for D=128, 2 for D=64
  const int lane = threadIdx.x & 31;
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
  const int qh = a.q_out ? a.q_heads : 0;
  const int slots = qh + 2 * a.kv_heads;
  const int64_t r = warp / slots;
  if (r >= a.rows) {
    pdl_wait();
    return;
  }
  const int slot = static_cast<int>(warp - r * slots);
  const bool is_q = slot < qh;
  const bool is_v = slot >= qh + a.kv_heads;
  const int head = is_q ? slot : (is_v ? slot - qh - a.kv_heads : slot - qh);
  const uint16_t* nw = is_q ? a.q_norm : a.k_norm;
  // Row constants: position, cos/sin of this lane's elements, norm weights.
  int64_t p = 0;
  uint16_t cb[E], sb[E], wb[E];
  auto load_consts = [&]() {
    p = a.positions[r];
    if (is_v) return;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      cb[e] = a.cos_tab[r * D + lane * E + e];
      sb[e] = a.sin_tab[r * D + lane * E + e];
      wb[e] = nw ? nw[lane * E + e] : 0;
    }
  };
  if (a.consts_early) load_consts();
  pdl_wait();  // q/k/v (or their partial slices) come from the previous kernel
  if (!a.consts_early) load_consts();
  if (!is_q && (p < 0 || p >= a.cache_rows)) {
    if (lane == 0 && head == 0 && !is_v && a.error_count) atomicAdd(a.error_count, 1);
    return;
  }
  const uint16_t* src = is_q ? a.q_in + r * a.q_rs : (is_v ? a.v_in + r * a.v_rs : a.k_in + r * a.k_rs);
  src += head * D + lane * E;
  uint16_t* dst = is_q ? a.q_out + (r * a.q_heads + head) * D
                       : (is_v ? a.v_cache : a.k_cache) + head * a.c_hs + p * a.c_rs;
  dst += lane * E;
  uint16_t xb[E];
  if constexpr (PARTS) {
    const float* ps =
        a.parts + r * a.p_rs + (is_q ? a.q_col : (is_v ? a.v_col : a.k_col)) + head * D + lane * E;
    float acc[E];
#pragma unroll
    for (int e = 0; e < E; ++e) acc[e] = 0.f;
    for (int s0 = 0; s0 < a.nparts; s0 += kPartBatch) {
      float pv[kPartBatch][E];
#pragma unroll
      for (int i = 0; i < kPartBatch; ++i)
        if (s0 + i < a.nparts) {
          if constexpr (E == 4) {
            const float4 t = __ldcg(reinterpret_cast<const float4*>(ps + (s0 + i) * a.p_slice));
            pv[i][0] = t.x; pv[i][1] = t.y; pv[i][2] = t.z; pv[i][3] = t.w;
          } else {
            const float2 t = __ldcg(reinterpret_cast<const float2*>(ps + (s0 + i) * a.p_slice));
            pv[i][0] = t.x; pv[i][1] = t.y;
          }
        }
#pragma unroll
      for (int i = 0; i < kPartBatch; ++i)
        if (s0 + i < a.nparts)
#pragma unroll
          for (int e = 0; e < E; ++e) acc[e] += pv[i][e];
    }
#pragma unroll
    for (int e = 0; e < E; ++e) xb[e] = T::from_f(acc[e]);
  } else if constexpr (E == 4) {
    uint2 u = *reinterpret_cast<const uint2*>(src);
    *reinterpret_cast<uint2*>(xb) = u;
  } else {
    uint32_t u = *reinterpret_cast<const uint32_t*>(src);
    *reinterpret_cast<uint32_t*>(xb) = u;
  }
  if (is_v) {  // bitwise copy into the cache row
    if constexpr (E == 4) *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(xb);
    else *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(xb);
    return;
  }
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = T::to_f(xb[e]);
  if (nw) {  // Qwen3 per-head RMSNorm over head_dim
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < E; ++e) ss = __fmaf_rn(x[e], x[e], ss);
#pragma unroll
    for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float inv = rsqrtf(__fadd_rn(ss * (1.0f / D), a.eps));
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float normed = rnd<T>(__fmul_rn(x[e], inv));
      x[e] = rnd<T>(__fmul_rn(T::to_f(wb[e]), normed));
    }
  }
  // RoPE at the row's absolute position: out = x*cos + rotate_half(x)*sin.
  const bool low = lane < 16;
  uint16_t ob[E];
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
    const float rot = low ? -partner : partner;
    ob[e] = rope_elem<T>(x[e], rot, T::to_f(cb[e]), T::to_f(sb[e]));
  }
  if constexpr (E == 4) *reinterpret_cast<uint2*>(dst) = *reinterpret_cast<const uint2*>(ob);
  else *reinterpret_cast<uint32_t*>(dst) = *reinterpret_cast<const uint32_t*>(ob);
}

template <class T>
__global__ void __launch_bounds__(256) silu_mul_kernel(const uint16_t* __restrict__ gate,
                                                       const uint16_t* __restrict__ up,
                                                       uint16_t* out, int64_t rows, int vpr,
                                                       int64_t g_rs, int64_t u_rs, int64_t o_rs) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  const int64_t n = rows * vpr;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += step) {
    const int64_t r = i / vpr;
    const int v = static_cast<int>(i - r * vpr);
    Vec8 g = ld_vec8(gate + r * g_rs + v * 8);
    Vec8 u = ld_vec8(up + r * u_rs + v * 8);
    Vec8 o;
#pragma unroll
    for (int e = 0; e < 8; ++e) o.h[e] = silu_mul_elem<T>(T::to_f(g.h[e]), T::to_f(u.h[e]));
    st_vec8(out + r * o_rs + v * 8, o);
  }
}

}  // namespace kvr

using namespace kvr;

extern "C" {

int kvr_add_rmsnorm(void* hidden, const void* delta, const void* weight, void* out, int64_t rows,
                    int hidden_size, int64_t hidden_stride, int64_t delta_stride,
                    int64_t out_stride, float eps, int dtype, void* stream) {
  return kvr::add_rmsnorm_ex(hidden, delta, nullptr, 0, 0, 0, weight, out, rows, hidden_size, hidden_stride,
                             delta_stride, out_stride, eps, dtype, stream, false);
}

}  // extern "C"

namespace kvr {

int add_rmsnorm_ex(void* hidden, const void* delta, const float* parts, int nparts, int64_t part_stride,
                   int64_t part_slice, const void* weight, void* out, int64_t rows, int hidden_size,
                   int64_t hidden_stride, int64_t delta_stride, int64_t out_stride, float eps, int dtype,
                   void* stream, bool weight_early) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || hidden_size <= 0 || hidden_size % 8) return KVR_ERR_INVALID_ARG;
  if (hidden_size > kNormThreads * kNormMaxVecs * 8) return KVR_ERR_UNSUPPORTED;
  if (rows == 0) return KVR_OK;
  if (rows > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  if (!hidden || !weight || !out || !aligned16(hidden) || !aligned16(weight) || !aligned16(out) ||
      (delta && !aligned16(delta)) || hidden_stride % 8 || out_stride % 8 ||
      (delta && delta_stride % 8))
    return KVR_ERR_INVALID_ARG;
  if (nparts < 0 || (nparts && (!parts || !aligned16(parts) || part_stride % 4 || part_slice % 4)))
    return KVR_ERR_INVALID_ARG;
  auto s = static_cast<cudaStream_t>(stream);
  const int vpr = hidden_size / 8;
  const float inv_h = 1.0f / static_cast<float>(hidden_size);
  int st = KVR_OK;
  auto go = [&](auto kernel) {
    return launch_pdl<decltype(kernel)::value>(static_cast<unsigned>(rows), dim3(kNormThreads), 0, s, 1,
        static_cast<uint16_t*>(hidden), static_cast<const uint16_t*>(delta),
        static_cast<const uint16_t*>(weight), static_cast<uint16_t*>(out), vpr, hidden_stride,
        delta_stride, out_stride, inv_h, eps, parts, nparts, part_stride, part_slice, weight_early ? 1 : 0);
  };
  const int vpt = (vpr + kNormThreads - 1) / kNormThreads;
  auto pick = [&](auto elem) {
    using T = decltype(elem);
    if (nparts) {
      if (vpt <= 1) return go(KernelRef<add_rmsnorm_kernel<T, 1, true>>{});
      if (vpt == 2) return go(KernelRef<add_rmsnorm_kernel<T, 2, true>>{});
      return go(KernelRef<add_rmsnorm_kernel<T, 4, true>>{});
    }
    if (vpt <= 1) return go(KernelRef<add_rmsnorm_kernel<T, 1, false>>{});
    if (vpt == 2) return go(KernelRef<add_rmsnorm_kernel<T, 2, false>>{});
    return go(KernelRef<add_rmsnorm_kernel<T, 4, false>>{});
  };
  st = dtype == KVR_DTYPE_BF16 ? pick(BF16{}) : pick(F16{});
  return st;
}

}  // namespace kvr

extern "C" {

int kvr_qkv_rope_scatter(const void* q_in, const void* k_in, const void* v_in,
                         int64_t q_row_stride, int64_t k_row_stride, int64_t v_row_stride,
                         const void* q_norm_w, const void* k_norm_w, float eps, const void* cos_tab,
                         const void* sin_tab, const int64_t* positions, int64_t rows, int q_heads,
                         int kv_heads, int head_dim, void* q_out, void* k_cache, void* v_cache,
                         int64_t cache_rows, int64_t cache_head_stride, int64_t cache_row_stride,
                         int* error_count, int dtype, void* stream) {
  return kvr::qkv_rope_scatter_ex(q_in, k_in, v_in, q_row_stride, k_row_stride, v_row_stride, q_norm_w, k_norm_w,
                                  eps, cos_tab, sin_tab, positions, rows, q_heads, kv_heads, head_dim, q_out,
                                  k_cache, v_cache, cache_rows, cache_head_stride, cache_row_stride, error_count,
                                  dtype, stream, nullptr, false);
}

}  // extern "C"

namespace kvr {

int qkv_rope_scatter_ex(const void* q_in, const void* k_in, const void* v_in, int64_t q_row_stride,
                        int64_t k_row_stride, int64_t v_row_stride, const void* q_norm_w, const void* k_norm_w,
                        float eps, const void* cos_tab, const void* sin_tab, const int64_t* positions,
                        int64_t rows, int q_heads, int kv_heads, int head_dim, void* q_out, void* k_cache,
                        void* v_cache, int64_t cache_rows, int64_t cache_head_stride, int64_t cache_row_stride,
                        int* error_count, int dtype, void* stream, const QkvParts* parts, bool consts_early) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || q_heads <= 0 || kv_heads <= 0 || cache_rows < 0) return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!cos_tab || !sin_tab || !positions || !k_cache || !v_cache) return KVR_ERR_INVALID_ARG;
  if (!parts && (!k_in || !v_in || (q_out && !q_in))) return KVR_ERR_INVALID_ARG;
  if (parts && (!parts->data || parts->count < 1 || (reinterpret_cast<uintptr_t>(parts->data) & 15u) ||
                parts->row_stride % 4 || parts->slice % 4 || parts->q_col % 4 || parts->k_col % 4 ||
                parts->v_col % 4))
    return KVR_ERR_INVALID_ARG;
  // Lanes move 4/8-byte slices of a head: require 8-byte alignment of every base/stride.
  const void* ptrs[] = {q_in, k_in, v_in, q_out, k_cache, v_cache, cos_tab, sin_tab};
  for (const void* p : ptrs)
    if (p && (reinterpret_cast<uintptr_t>(p) & 7u)) return KVR_ERR_INVALID_ARG;
  if (q_row_stride % 4 || k_row_stride % 4 || v_row_stride % 4 || cache_head_stride % 4 ||
      cache_row_stride % 4)
    return KVR_ERR_INVALID_ARG;
  QkvArgs a;
  a.q_in = static_cast<const uint16_t*>(q_in);
  a.k_in = static_cast<const uint16_t*>(k_in);
  a.v_in = static_cast<const uint16_t*>(v_in);
  a.q_rs = q_row_stride;
  a.k_rs = k_row_stride;
  a.v_rs = v_row_stride;
  a.q_norm = static_cast<const uint16_t*>(q_norm_w);
  a.k_norm = static_cast<const uint16_t*>(k_norm_w);
  a.eps = eps;
  a.cos_tab = static_cast<const uint16_t*>(cos_tab);
  a.sin_tab = static_cast<const uint16_t*>(sin_tab);
  a.positions = positions;
  a.rows = rows;
  a.q_heads = q_heads;
  a.kv_heads = kv_heads;
  a.q_out = static_cast<uint16_t*>(q_out);
  a.k_cache = static_cast<uint16_t*>(k_cache);
  a.v_cache = static_cast<uint16_t*>(v_cache);
  a.cache_rows = cache_rows;
  a.c_hs = cache_head_stride;
  a.c_rs = cache_row_stride;
  a.error_count = error_count;
  a.parts = parts ? parts->data : nullptr;
  a.nparts = parts ? parts->count : 0;
  a.p_rs = parts ? parts->row_stride : 0;
  a.p_slice = parts ? parts->slice : 0;
  a.q_col = parts ? parts->q_col : 0;
  a.k_col = parts ? parts->k_col : 0;
  a.v_col = parts ? parts->v_col : 0;
  a.consts_early = consts_early ? 1 : 0;
  const int slots = (q_out ? q_heads : 0) + 2 * kv_heads;
  const int64_t warps = rows * slots;
  const int64_t blocks = (warps + 7) / 8;
  if (blocks > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  auto s = static_cast<cudaStream_t>(stream);
  int st = KVR_OK;
  const unsigned grid = static_cast<unsigned>(blocks);
  auto go = [&](auto kernel) { return launch_pdl<decltype(kernel)::value>(grid, dim3(256), 0, s, 1, a); };
  const bool with_parts = a.nparts > 0;
  if (dtype == KVR_DTYPE_BF16) {
    if (head_dim == 128)
      st = with_parts ? go(KernelRef<qkv_rope_scatter_kernel<BF16, 128, true>>{})
                      : go(KernelRef<qkv_rope_scatter_kernel<BF16, 128, false>>{});
    else
      st = with_parts ? go(KernelRef<qkv_rope_scatter_kernel<BF16, 64, true>>{})
                      : go(KernelRef<qkv_rope_scatter_kernel<BF16, 64, false>>{});
  } else {
    if (head_dim == 128)
      st = with_parts ? go(KernelRef<qkv_rope_scatter_kernel<F16, 128, true>>{})
                      : go(KernelRef<qkv_rope_scatter_kernel<F16, 128, false>>{});
    else
      st = with_parts ? go(KernelRef<qkv_rope_scatter_kernel<F16, 64, true>>{})
                      : go(KernelRef<qkv_rope_scatter_kernel<F16, 64, false>>{});
  }
  return st;
}

}  // namespace kvr

extern "C" {

int kvr_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int64_t width,
                 int64_t gate_stride, int64_t up_stride, int64_t out_stride, int dtype,
                 void* stream) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || width <= 0 || width % 8) return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!gate || !up || !out || !aligned16(gate) || !aligned16(up) || !aligned16(out) ||
      gate_stride % 8 || up_stride % 8 || out_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (width / 8 > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  const int vpr = static_cast<int>(width / 8);
  auto s = static_cast<cudaStream_t>(stream);
  const int grid = grid_for(rows * vpr, 256);
  int st = KVR_OK;
  if (dtype == KVR_DTYPE_BF16)
    st = launch_pdl<silu_mul_kernel<BF16>>(grid, dim3(256), 0, s, 1, static_cast<const uint16_t*>(gate),
                                                static_cast<const uint16_t*>(up),
                                                static_cast<uint16_t*>(out), rows, vpr, gate_stride,
                                                up_stride, out_stride);
  else
    st = launch_pdl<silu_mul_kernel<F16>>(grid, dim3(256), 0, s, 1, static_cast<const uint16_t*>(gate),
                                               static_cast<const uint16_t*>(up),
                                               static_cast<uint16_t*>(out), rows, vpr, gate_stride,
                                               up_stride, out_stride);
  return st;
}

}  // extern "C"
