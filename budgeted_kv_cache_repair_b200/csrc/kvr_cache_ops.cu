// HBM-bound cache kernels: ownership copy, delta-RoPE positional correction,
// fused shift cache, indexed row scatter and embedding gather.
//
// All of them move 16- or 32-byte vectors with consecutive threads on
// consecutive addresses. A "segment" is one (tensor, head) plane of rows*D
// elements. The copy runs one short CTA per 16 KB chunk, the shift and the
// delta-RoPE one short CTA per 256 vector pairs, all over work units that
// span every segment; the scatter walks its (head, row, vector) items in a
// grid-stride loop and the embedding gather takes one CTA per row. The
// streaming kernels keep the driver's L1 / shared-memory split
// (launch_pdl_default_carveout).
#include <stdio.h>

#include <algorithm>

#include "kvr_common.cuh"

namespace kvr {

namespace {
thread_local int g_last_cuda_error = 0;
unsigned long long g_launches = 0;
thread_local uint64_t* g_captured = nullptr;  // set while this thread captures a graph
}

void set_last_cuda_error(cudaError_t e) { g_last_cuda_error = static_cast<int>(e); }
void count_launch() {
  if (g_captured)
    ++*g_captured;
  else
    __atomic_add_fetch(&g_launches, 1ull, __ATOMIC_RELAXED);
}
long long g_wait_limit = kDefaultWaitLimit;
long long pipeline_wait_limit() { return __atomic_load_n(&g_wait_limit, __ATOMIC_RELAXED); }

void count_launches(uint64_t n) { __atomic_add_fetch(&g_launches, static_cast<unsigned long long>(n), __ATOMIC_RELAXED); }
void count_captured_launches(uint64_t* sink) { g_captured = sink; }

// ---------------------------------------------------------------------------
// Ownership copy (clone_cache, cache.py:31-44).
// ---------------------------------------------------------------------------
struct CopyArgs {
  int heads;
  int vecs_per_row;  // head_dim / 8
  int64_t src_hs, src_rs, dst_hs, dst_rs;  // element strides
  bool dense;        // rows of both sides are contiguous inside a head
  int64_t nvec;      // 16-byte vectors per segment (rows * vecs_per_row)
  int64_t chunks_per_seg, chunks;
};

constexpr int kCopyThreads = 256;
constexpr int kCopyUnroll = 4;
constexpr int kCopyChunk = kCopyThreads * kCopyUnroll;  // vectors per chunk (16 KB)

// One short CTA per 16 KB chunk of a segment: one division per chunk maps it
// to (segment, offset), and each thread has kCopyUnroll coalesced 16-byte loads in flight
// before its stores. Short CTAs measured faster than a persistent grid here,
// and a copy running beside higher-priority work gives SM slots back to it
// within microseconds.
__global__ void __launch_bounds__(kCopyThreads) copy_layers_kernel(LayerPtrs ptrs, CopyArgs a) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  for (int64_t c = blockIdx.x; c < a.chunks; c += gridDim.x) {
    const int64_t seg = c / a.chunks_per_seg;
    const int64_t base = (c - seg * a.chunks_per_seg) * kCopyChunk + threadIdx.x;
    const int t = static_cast<int>(seg / a.heads);
    const int h = static_cast<int>(seg - static_cast<int64_t>(t) * a.heads);
    const uint16_t* src = static_cast<const uint16_t*>(ptrs.src[t]) + h * a.src_hs;
    uint16_t* dst = static_cast<uint16_t*>(ptrs.dst[t]) + h * a.dst_hs;
    Vec8 v[kCopyUnroll];
    if (a.dense) {
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * kCopyThreads;
        if (i < a.nvec) v[u] = ld_vec8_stream(src + i * 8);
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * kCopyThreads;
        if (i < a.nvec) st_vec8_stream(dst + i * 8, v[u]);
      }
    } else {
      const int vpr = a.vecs_per_row;
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * kCopyThreads;
        if (i < a.nvec) {
          const int64_t r = i / vpr;
          v[u] = ld_vec8_stream(src + r * a.src_rs + (i - r * vpr) * 8);
        }
      }
#pragma unroll
      for (int u = 0; u < kCopyUnroll; ++u) {
        const int64_t i = base + u * kCopyThreads;
        if (i < a.nvec) {
          const int64_t r = i / vpr;
          st_vec8_stream(dst + r * a.dst_rs + (i - r * vpr) * 8, v[u]);
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Delta-RoPE (shifted_suffix_keys, cache.py:47-77): every layer's rows
// rotated in one launch, in the shift kernel's layout (below).
// ---------------------------------------------------------------------------
struct RopeArgs {
  int heads;
  int segments;  // num_layers * heads
  int64_t rows;
  int64_t src_hs, src_rs, dst_hs, dst_rs;
};

// ---------------------------------------------------------------------------
// Fused shift cache (build_halo_cache, cache.py:103-144, halo 0): prefix rows
// copied, tail rows moved up by the deleted span with K re-rotated.
// Segment = (layer, head, component) with component 0 = K, 1 = V.
// ---------------------------------------------------------------------------
struct ShiftArgs {
  int heads;
  int segments;  // num_layers * heads * 2
  int64_t new_rows, prefix, old_tail, new_tail;
  int64_t old_hs, old_rs, new_hs, new_rs;
  int apply_rope;
};

struct ShiftPtrs {
  const void* k_old[KVR_MAX_LAYER_TENSORS / 2];
  const void* v_old[KVR_MAX_LAYER_TENSORS / 2];
  void* k_new[KVR_MAX_LAYER_TENSORS / 2];
  void* v_new[KVR_MAX_LAYER_TENSORS / 2];
};

// The grid covers all (layer, head, component) segments as one flat sequence
// of "pairs" (a vector of a row's low half and its partner in the high half,
// so rotate_half needs no data exchange): one short CTA per 256 pairs, one
// pair per thread, VB-byte vectors (32 when every pointer and stride allows
// 256-bit accesses, else 16). CTAs of 256 threads are a multiple of the pairs
// per row, so a thread's pair index is its thread index modulo that count.
// cos/sin sit in shared memory as one 16-byte (cos_lo, sin_lo, cos_hi,
// sin_hi) entry per element, padded by one entry per pair index so that the
// pair indices of a warp read disjoint banks.
//
// Measured at config 2 (32 layers, 2.08 GB): 309 us = 1.04 of the measured
// copy peak, launched with the driver's L1 / shared-memory split; the same
// kernel under the largest shared-memory split, and persistent grids (all of
// a thread's loads in flight, then its stores; or a per-thread cp.async ring
// in shared memory), took 350-380 us. The old rows are read through the
// non-coherent path, so the new tensors must not overlap them.
constexpr int kShiftThreads = 256;

template <int VB>
struct ShiftVec {
  uint32_t w[VB / 4];
};

template <int VB>
__device__ __forceinline__ ShiftVec<VB> ld_shift(const void* p) {
  ShiftVec<VB> v;
  if constexpr (VB == 32) {
    asm volatile("ld.global.nc.L1::no_allocate.L2::evict_first.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p));
  } else {
    asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p));
  }
  return v;
}

template <int VB>
__device__ __forceinline__ void st_shift(void* p, const ShiftVec<VB>& v) {
  if constexpr (VB == 32) {
    asm volatile("st.global.v8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]),
                 "r"(v.w[2]), "r"(v.w[3]), "r"(v.w[4]), "r"(v.w[5]), "r"(v.w[6]), "r"(v.w[7])
                 : "memory");
  } else {
    asm volatile("st.global.v4.b32 [%0], {%1,%2,%3,%4};\n" ::"l"(p), "r"(v.w[0]), "r"(v.w[1]), "r"(v.w[2]),
                 "r"(v.w[3])
                 : "memory");
  }
}

template <class T, int D, int VB>
__global__ void __launch_bounds__(kShiftThreads) shift_cache_kernel(ShiftPtrs ptrs, ShiftArgs a,
                                                                 const uint16_t* __restrict__ cos_sin) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  constexpr int EV = VB / 2;           // 16-bit elements per vector
  constexpr int PAIRS = D / (2 * EV);  // vector pairs per row
  constexpr int HALF = D / 2;
  constexpr int PAD = EV + 1;
  static_assert(kShiftThreads % PAIRS == 0, "a CTA covers whole rows");
  __shared__ float4 cs4[PAIRS * PAD];  // [pair index][element (+1 pad)] = (cos_lo, sin_lo, cos_hi, sin_hi)
  if (a.apply_rope) {  // the table is only non-null when the tail rotates
    for (int i = threadIdx.x; i < HALF; i += blockDim.x) {
      cs4[(i / EV) * PAD + (i % EV)] = make_float4(T::to_f(cos_sin[i]), T::to_f(cos_sin[D + i]),
                                                  T::to_f(cos_sin[HALF + i]), T::to_f(cos_sin[D + HALF + i]));
    }
  }
  __syncthreads();
  const int j = threadIdx.x % PAIRS;
  const uint32_t per_seg = static_cast<uint32_t>(a.new_rows) * PAIRS;
  const uint32_t i = blockIdx.x * kShiftThreads + threadIdx.x;  // < 2^32 (host-checked)
  if (i >= per_seg * static_cast<uint32_t>(a.segments)) return;
  const uint32_t seg = i / per_seg;
  const int64_t r = (i - seg * per_seg) / PAIRS;
  const int comp = seg & 1;
  const int lh = seg >> 1;
  const int l = lh / a.heads;
  const int h = lh - l * a.heads;
  int64_t sr;
  if (r < a.prefix) sr = r;
  else if (r >= a.new_tail) sr = r - a.new_tail + a.old_tail;
  else return;  // rows in [prefix, new_tail) are recomputed by the caller
  const uint16_t* src = static_cast<const uint16_t*>(comp ? ptrs.v_old[l] : ptrs.k_old[l]) + h * a.old_hs +
                        sr * a.old_rs + j * EV;
  uint16_t* dst = static_cast<uint16_t*>(comp ? ptrs.v_new[l] : ptrs.k_new[l]) + h * a.new_hs + r * a.new_rs +
                  j * EV;
  const ShiftVec<VB> lo = ld_shift<VB>(src);
  const ShiftVec<VB> hi = ld_shift<VB>(src + HALF);
  if (comp == 0 && a.apply_rope && r >= a.new_tail) {
    const float4* csj = cs4 + j * PAD;
    const uint16_t* xl = reinterpret_cast<const uint16_t*>(lo.w);
    const uint16_t* xh = reinterpret_cast<const uint16_t*>(hi.w);
    ShiftVec<VB> olo, ohi;
    uint16_t* ol = reinterpret_cast<uint16_t*>(olo.w);
    uint16_t* oh = reinterpret_cast<uint16_t*>(ohi.w);
#pragma unroll
    for (int e = 0; e < EV; ++e) {
      const float fl = T::to_f(xl[e]);
      const float fh = T::to_f(xh[e]);
      // d < D/2: rotate_half = -x[d + D/2];  d >= D/2: rotate_half = x[d - D/2].
      const float4 c = csj[e];
      ol[e] = rope_elem_hw<T>(fl, -fh, c.x, c.y);
      oh[e] = rope_elem_hw<T>(fh, fl, c.z, c.w);
    }
    st_shift<VB>(dst, olo);
    st_shift<VB>(dst + HALF, ohi);
  } else {
    st_shift<VB>(dst, lo);
    st_shift<VB>(dst + HALF, hi);
  }
}

// Delta-RoPE with the shift kernel's layout: one short CTA per 256 vector
// pairs over all (layer, head, row), one pair per thread, 32-byte vectors
// where pointers and strides allow, launched with the driver's L1 split. The
// rotation may run in place (src == dst): every element is read and written
// by the same thread, so the loads take the coherent path (not the read-only
// one) and skip L1 allocation; read-only loads for out-of-place calls
// measured the same (164.9 against 167.3 us for 0.9 GB).
template <int VB>
__device__ __forceinline__ ShiftVec<VB> ld_rope(const void* p) {
  ShiftVec<VB> v;
  if constexpr (VB == 32) {
    asm volatile("ld.global.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3]), "=r"(v.w[4]), "=r"(v.w[5]),
                   "=r"(v.w[6]), "=r"(v.w[7])
                 : "l"(p)
                 : "memory");
  } else {
    asm volatile("ld.global.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(v.w[0]), "=r"(v.w[1]), "=r"(v.w[2]), "=r"(v.w[3])
                 : "l"(p)
                 : "memory");
  }
  return v;
}

template <class T, int D, int VB>
__global__ void __launch_bounds__(kShiftThreads) rope_shift_kernel(LayerPtrs ptrs, RopeArgs a,
                                                                const uint16_t* __restrict__ cos_sin) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  constexpr int EV = VB / 2;           // 16-bit elements per vector
  constexpr int PAIRS = D / (2 * EV);  // vector pairs per row
  constexpr int HALF = D / 2;
  constexpr int PAD = EV + 1;
  static_assert(kShiftThreads % PAIRS == 0, "a CTA covers whole rows");
  __shared__ float4 cs4[PAIRS * PAD];  // [pair index][element (+1 pad)] = (cos_lo, sin_lo, cos_hi, sin_hi)
  for (int i = threadIdx.x; i < HALF; i += blockDim.x) {
    cs4[(i / EV) * PAD + (i % EV)] = make_float4(T::to_f(cos_sin[i]), T::to_f(cos_sin[D + i]),
                                                T::to_f(cos_sin[HALF + i]), T::to_f(cos_sin[D + HALF + i]));
  }
  __syncthreads();
  const int j = threadIdx.x % PAIRS;
  const uint32_t per_seg = static_cast<uint32_t>(a.rows) * PAIRS;
  const uint32_t i = blockIdx.x * kShiftThreads + threadIdx.x;  // < 2^32 (host-checked)
  if (i >= per_seg * static_cast<uint32_t>(a.segments)) return;
  const uint32_t seg = i / per_seg;
  const int64_t r = (i - seg * per_seg) / PAIRS;
  const int l = static_cast<int>(seg) / a.heads;
  const int h = static_cast<int>(seg) - l * a.heads;
  const uint16_t* src = static_cast<const uint16_t*>(ptrs.src[l]) + h * a.src_hs + r * a.src_rs + j * EV;
  uint16_t* dst = static_cast<uint16_t*>(ptrs.dst[l]) + h * a.dst_hs + r * a.dst_rs + j * EV;
  const ShiftVec<VB> lo = ld_rope<VB>(src);
  const ShiftVec<VB> hi = ld_rope<VB>(src + HALF);
  const float4* csj = cs4 + j * PAD;
  const uint16_t* xl = reinterpret_cast<const uint16_t*>(lo.w);
  const uint16_t* xh = reinterpret_cast<const uint16_t*>(hi.w);
  ShiftVec<VB> olo, ohi;
  uint16_t* ol = reinterpret_cast<uint16_t*>(olo.w);
  uint16_t* oh = reinterpret_cast<uint16_t*>(ohi.w);
#pragma unroll
  for (int e = 0; e < EV; ++e) {
    const float fl = T::to_f(xl[e]);
    const float fh = T::to_f(xh[e]);
    // d < D/2: rotate_half = -x[d + D/2];  d >= D/2: rotate_half = x[d - D/2].
    const float4 c = csj[e];
    ol[e] = rope_elem_hw<T>(fl, -fh, c.x, c.y);
    oh[e] = rope_elem_hw<T>(fh, fl, c.z, c.w);
  }
  st_shift<VB>(dst, olo);
  st_shift<VB>(dst + HALF, ohi);
}

template <class T, int D>
int launch_rope(bool wide, dim3 grid, cudaStream_t s, const LayerPtrs& p, const RopeArgs& a, const uint16_t* cs) {
  const dim3 block(kShiftThreads);
  return wide ? launch_pdl_default_carveout<rope_shift_kernel<T, D, 32>>(grid, block, 0, s, 1, p, a, cs)
              : launch_pdl_default_carveout<rope_shift_kernel<T, D, 16>>(grid, block, 0, s, 1, p, a, cs);
}

// ---------------------------------------------------------------------------
// Bitwise scatter (indexed_kv_scatter_ / index_copy_). One warp-slice of
// D/8 threads per (head, row); positions read once per row.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) scatter_rows_kernel(
    const uint16_t* __restrict__ kf, const uint16_t* __restrict__ vf, uint16_t* kc, uint16_t* vc,
    const int64_t* __restrict__ positions, int64_t rows, int heads, int vpr, int64_t cache_rows,
    int64_t f_hs, int64_t f_rs, int64_t c_hs, int64_t c_rs, int* error_count) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  const int64_t n = static_cast<int64_t>(heads) * rows * vpr;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n; i += step) {
    const int64_t hr = i / vpr;
    const int v = static_cast<int>(i - hr * vpr);
    const int64_t h = hr / rows;
    const int64_t r = hr - h * rows;
    const int64_t p = positions[r];
    if (p < 0 || p >= cache_rows) {
      if (v == 0 && h == 0 && error_count) atomicAdd(error_count, 1);
      continue;
    }
    const int64_t so = h * f_hs + r * f_rs + v * 8;
    const int64_t dofs = h * c_hs + p * c_rs + v * 8;
    st_vec8(kc + dofs, ld_vec8(kf + so));
    st_vec8(vc + dofs, ld_vec8(vf + so));
  }
}

// ---------------------------------------------------------------------------
// Embedding gather of the selected rows.
// ---------------------------------------------------------------------------
__global__ void __launch_bounds__(256) embed_rows_kernel(
    const uint16_t* __restrict__ embed, int64_t vocab, int vpr, const int64_t* __restrict__ ids,
    int64_t id_count, const int64_t* __restrict__ positions, int64_t rows, uint16_t* out,
    int* error_count) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  const int64_t r = blockIdx.x;
  if (r >= rows) return;
  const int64_t p = positions[r];
  int64_t id = -1;
  if (p >= 0 && p < id_count) id = ids[p];
  const bool ok = id >= 0 && id < vocab;
  if (!ok && threadIdx.x == 0 && error_count) atomicAdd(error_count, 1);
  uint16_t* o = out + r * static_cast<int64_t>(vpr) * 8;
  for (int v = threadIdx.x; v < vpr; v += blockDim.x) {
    Vec8 x;
    if (ok) {
      x = ld_vec8(embed + id * static_cast<int64_t>(vpr) * 8 + v * 8);
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x.h[e] = 0;
    }
    st_vec8(o + v * 8, x);
  }
}

// ---------------------------------------------------------------------------
// Rotary tables at the selected positions, by the op sequence of the
// transformers rotary forward (LlamaRotaryEmbedding / Qwen3RotaryEmbedding):
// freq = inv_freq[i] * float(position) (its K=1 matmul: one fp32 product),
// cos/sin of the duplicated halves, times attention_scaling, rounded to the
// element type. cosf/sinf are CUDA's full-precision functions, as torch's
// elementwise cos/sin kernels call them.
// ---------------------------------------------------------------------------
template <class T>
__global__ void __launch_bounds__(128) rope_tables_kernel(const float* __restrict__ inv_freq, int half,
                                                          const int64_t* __restrict__ positions, int64_t rows,
                                                          float scaling, uint16_t* __restrict__ cos_out,
                                                          uint16_t* __restrict__ sin_out) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // positions may come from the previous kernel
  const int64_t idx = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= rows * half) return;
  const int64_t r = idx / half;
  const int i = static_cast<int>(idx - r * half);
  const float f = __fmul_rn(inv_freq[i], static_cast<float>(positions[r]));
  const uint16_t c = T::from_f(__fmul_rn(cosf(f), scaling));
  const uint16_t sn = T::from_f(__fmul_rn(sinf(f), scaling));
  const int64_t o = r * 2 * half + i;
  cos_out[o] = c;
  cos_out[o + half] = c;
  sin_out[o] = sn;
  sin_out[o + half] = sn;
}

}  // namespace kvr

using namespace kvr;

namespace {

bool valid_dtype(int dtype) { return dtype == KVR_DTYPE_BF16 || dtype == KVR_DTYPE_F16; }

bool aligned32(const void* ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 31u) == 0; }

// A kernel as a type, so that one generic lambda can launch any of them.
template <auto kernel>
struct Kernel {
  static constexpr auto value = kernel;
};

}  // namespace

extern "C" {

const char* kvr_version(void) { return "kvr_b200 0.1 (sm_100a)"; }

const char* kvr_status_string(int status) {
  switch (status) {
    case KVR_OK: return "ok";
    case KVR_ERR_INVALID_ARG: return "invalid argument";
    case KVR_ERR_UNSUPPORTED: return "unsupported shape or dtype";
    case KVR_ERR_CUDA: return "CUDA error";
    case KVR_ERR_TIMEOUT: return "bounded device wait timed out";
    case KVR_ERR_SCRATCH_LIMIT: return "needs more scratch than the static device array holds";
    case KVR_ERR_INJECTED: return "failure injected by a test hook";
    default: return "unknown status";
  }
}

int kvr_last_cuda_error(void) { return g_last_cuda_error; }

int kvr_set_wait_limit(int64_t cycles) {
  if (cycles < 0) return KVR_ERR_INVALID_ARG;
  __atomic_store_n(&g_wait_limit, cycles ? static_cast<long long>(cycles) : kDefaultWaitLimit, __ATOMIC_RELAXED);
  return KVR_OK;
}

uint64_t kvr_kernel_launches(void) { return __atomic_load_n(&g_launches, __ATOMIC_RELAXED); }

int kvr_copy_layers(const void* const* src, void* const* dst, int num_tensors, int heads,
                    int64_t rows, int head_dim, int64_t src_head_stride, int64_t src_row_stride,
                    int64_t dst_head_stride, int64_t dst_row_stride, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return KVR_ERR_UNSUPPORTED;
  if (!src || !dst || num_tensors < 0 || num_tensors > KVR_MAX_LAYER_TENSORS || heads <= 0 ||
      rows < 0 || head_dim <= 0 || head_dim % 8)
    return KVR_ERR_INVALID_ARG;
  if (src_row_stride % 8 || dst_row_stride % 8 || src_head_stride % 8 || dst_head_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (num_tensors == 0 || rows == 0) return KVR_OK;
  LayerPtrs p;
  for (int t = 0; t < num_tensors; ++t) {
    if (!src[t] || !dst[t] || !aligned16(src[t]) || !aligned16(dst[t])) return KVR_ERR_INVALID_ARG;
    p.src[t] = src[t];
    p.dst[t] = dst[t];
  }
  CopyArgs a;
  a.heads = heads;
  a.vecs_per_row = head_dim / 8;
  a.src_hs = src_head_stride;
  a.src_rs = src_row_stride;
  a.dst_hs = dst_head_stride;
  a.dst_rs = dst_row_stride;
  a.dense = src_row_stride == head_dim && dst_row_stride == head_dim;
  a.nvec = rows * a.vecs_per_row;
  a.chunks_per_seg = (a.nvec + kCopyChunk - 1) / kCopyChunk;
  a.chunks = a.chunks_per_seg * num_tensors * heads;
  if (a.chunks > 0x7fffffffLL) return KVR_ERR_UNSUPPORTED;
  dim3 grid(static_cast<unsigned>(a.chunks));
  return launch_pdl_default_carveout<copy_layers_kernel>(grid, dim3(kCopyThreads), 0,
                                                         static_cast<cudaStream_t>(stream), 1, p, a);
}

int kvr_rope_shift_layers(const void* const* src, void* const* dst, int num_layers, int heads,
                          int64_t rows, int head_dim, int64_t src_head_stride,
                          int64_t src_row_stride, int64_t dst_head_stride, int64_t dst_row_stride,
                          const void* cos_sin, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return KVR_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (!src || !dst || !cos_sin || num_layers < 0 || num_layers > KVR_MAX_LAYER_TENSORS ||
      heads <= 0 || rows < 0)
    return KVR_ERR_INVALID_ARG;
  if (src_row_stride % 8 || dst_row_stride % 8 || src_head_stride % 8 || dst_head_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (num_layers == 0 || rows == 0) return KVR_OK;
  if (static_cast<int64_t>(num_layers) * heads > 65535) return KVR_ERR_UNSUPPORTED;
  LayerPtrs p;
  for (int l = 0; l < num_layers; ++l) {
    if (!src[l] || !dst[l] || !aligned16(src[l]) || !aligned16(dst[l])) return KVR_ERR_INVALID_ARG;
    p.src[l] = src[l];
    p.dst[l] = dst[l];
  }
  const int segs = num_layers * heads;
  RopeArgs a{heads, segs, rows, src_head_stride, src_row_stride, dst_head_stride, dst_row_stride};
  const bool wide = (src_row_stride | dst_row_stride | src_head_stride | dst_head_stride) % 16 == 0 &&
                    std::all_of(p.src, p.src + num_layers, aligned32) &&
                    std::all_of(p.dst, p.dst + num_layers, aligned32);
  const int64_t pairs = rows * (head_dim / (wide ? 32 : 16)) * segs;
  if (pairs > 0xffffffffLL) return KVR_ERR_UNSUPPORTED;  // 32-bit pair index
  const dim3 grid(static_cast<unsigned>((pairs + kShiftThreads - 1) / kShiftThreads));
  auto s = static_cast<cudaStream_t>(stream);
  const uint16_t* cs = static_cast<const uint16_t*>(cos_sin);
  if (dtype == KVR_DTYPE_BF16)
    return head_dim == 128 ? launch_rope<BF16, 128>(wide, grid, s, p, a, cs)
                           : launch_rope<BF16, 64>(wide, grid, s, p, a, cs);
  return head_dim == 128 ? launch_rope<F16, 128>(wide, grid, s, p, a, cs)
                         : launch_rope<F16, 64>(wide, grid, s, p, a, cs);
}

int kvr_shift_cache_layers(const void* const* k_old, const void* const* v_old, void* const* k_new,
                           void* const* v_new, int num_layers, int heads, int head_dim,
                           int64_t new_rows, int64_t prefix, int64_t old_tail_start,
                           int64_t new_tail_start, int64_t old_head_stride, int64_t old_row_stride,
                           int64_t new_head_stride, int64_t new_row_stride, const void* cos_sin,
                           int apply_rope, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return KVR_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (!k_old || !v_old || !k_new || !v_new || (apply_rope && !cos_sin) || num_layers < 0 ||
      num_layers > KVR_MAX_LAYER_TENSORS / 2 || heads <= 0 || new_rows < 0 || prefix < 0 ||
      prefix > new_tail_start || new_tail_start > new_rows || old_tail_start < prefix)
    return KVR_ERR_INVALID_ARG;
  if (old_row_stride % 8 || new_row_stride % 8 || old_head_stride % 8 || new_head_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (num_layers == 0 || new_rows == 0) return KVR_OK;
  if (static_cast<int64_t>(num_layers) * heads * 2 > 65535) return KVR_ERR_UNSUPPORTED;
  ShiftPtrs p;
  for (int l = 0; l < num_layers; ++l) {
    const void* ptrs[4] = {k_old[l], v_old[l], k_new[l], v_new[l]};
    for (const void* q : ptrs)
      if (!q || !aligned16(q)) return KVR_ERR_INVALID_ARG;
    p.k_old[l] = k_old[l];
    p.v_old[l] = v_old[l];
    p.k_new[l] = k_new[l];
    p.v_new[l] = v_new[l];
  }
  const int segs = num_layers * heads * 2;
  ShiftArgs a{heads, segs, new_rows, prefix, old_tail_start, new_tail_start,
              old_head_stride, old_row_stride, new_head_stride, new_row_stride, apply_rope};
  const bool wide = (old_row_stride | new_row_stride | old_head_stride | new_head_stride) % 16 == 0 &&
                    std::all_of(p.k_old, p.k_old + num_layers, aligned32) &&
                    std::all_of(p.v_old, p.v_old + num_layers, aligned32) &&
                    std::all_of(p.k_new, p.k_new + num_layers, aligned32) &&
                    std::all_of(p.v_new, p.v_new + num_layers, aligned32);
  const int64_t pairs = new_rows * (head_dim / (wide ? 32 : 16)) * segs;
  if (pairs > 0xffffffffLL) return KVR_ERR_UNSUPPORTED;  // 32-bit pair index
  const dim3 grid(static_cast<unsigned>((pairs + kShiftThreads - 1) / kShiftThreads));
  auto s = static_cast<cudaStream_t>(stream);
  const uint16_t* cs = static_cast<const uint16_t*>(cos_sin);
  auto go = [&](auto kernel) {
    return launch_pdl_default_carveout<decltype(kernel)::value>(grid, dim3(kShiftThreads), 0, s, 1, p, a, cs);
  };
  if (dtype == KVR_DTYPE_BF16) {
    if (head_dim == 128)
      return wide ? go(Kernel<shift_cache_kernel<BF16, 128, 32>>{})
                  : go(Kernel<shift_cache_kernel<BF16, 128, 16>>{});
    return wide ? go(Kernel<shift_cache_kernel<BF16, 64, 32>>{}) : go(Kernel<shift_cache_kernel<BF16, 64, 16>>{});
  }
  if (head_dim == 128)
    return wide ? go(Kernel<shift_cache_kernel<F16, 128, 32>>{}) : go(Kernel<shift_cache_kernel<F16, 128, 16>>{});
  return wide ? go(Kernel<shift_cache_kernel<F16, 64, 32>>{}) : go(Kernel<shift_cache_kernel<F16, 64, 16>>{});
}

int kvr_scatter_rows(const void* k_fresh, const void* v_fresh, void* k_cache, void* v_cache,
                     const int64_t* positions, int64_t rows, int heads, int head_dim,
                     int64_t cache_rows, int64_t fresh_head_stride, int64_t fresh_row_stride,
                     int64_t cache_head_stride, int64_t cache_row_stride, int* error_count,
                     int dtype, void* stream) {
  if (!valid_dtype(dtype)) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || heads <= 0 || head_dim <= 0 || head_dim % 8 || cache_rows < 0)
    return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!k_fresh || !v_fresh || !k_cache || !v_cache || !positions) return KVR_ERR_INVALID_ARG;
  if (!aligned16(k_fresh) || !aligned16(v_fresh) || !aligned16(k_cache) || !aligned16(v_cache) ||
      fresh_head_stride % 8 || fresh_row_stride % 8 || cache_head_stride % 8 || cache_row_stride % 8)
    return KVR_ERR_INVALID_ARG;
  const int vpr = head_dim / 8;
  const int64_t n = static_cast<int64_t>(heads) * rows * vpr;
  return launch_pdl<scatter_rows_kernel>(grid_for(n, 256), dim3(256), 0, static_cast<cudaStream_t>(stream), 1, 
      static_cast<const uint16_t*>(k_fresh), static_cast<const uint16_t*>(v_fresh),
      static_cast<uint16_t*>(k_cache), static_cast<uint16_t*>(v_cache), positions, rows, heads,
      vpr, cache_rows, fresh_head_stride, fresh_row_stride, cache_head_stride, cache_row_stride,
      error_count);
}

int kvr_rope_tables(const float* inv_freq, int half_dim, const int64_t* positions, int64_t rows, float scaling,
                    void* cos_out, void* sin_out, int dtype, void* stream) {
  if (!inv_freq || !positions || !cos_out || !sin_out || half_dim <= 0 || rows < 0 || !valid_dtype(dtype))
    return KVR_ERR_INVALID_ARG;
  if (!rows) return KVR_OK;
  const int64_t n = rows * half_dim;
  if ((n + 127) / 128 > 0x7fffffffLL) return KVR_ERR_UNSUPPORTED;
  const dim3 grid(static_cast<unsigned>((n + 127) / 128));
  auto s = static_cast<cudaStream_t>(stream);
  auto* c = static_cast<uint16_t*>(cos_out);
  auto* sn = static_cast<uint16_t*>(sin_out);
  if (dtype == KVR_DTYPE_BF16)
    return launch_pdl<rope_tables_kernel<BF16>>(grid, dim3(128), 0, s, 1, inv_freq, half_dim, positions, rows, scaling,
                                                c, sn);
  return launch_pdl<rope_tables_kernel<F16>>(grid, dim3(128), 0, s, 1, inv_freq, half_dim, positions, rows, scaling, c,
                                             sn);
}

int kvr_embed_rows(const void* embed, int64_t vocab, int hidden, const int64_t* ids,
                   int64_t id_count, const int64_t* positions, int64_t rows, void* out,
                   int* error_count, int dtype, void* stream) {
  if (!valid_dtype(dtype)) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || hidden <= 0 || hidden % 8 || vocab <= 0 || id_count < 0)
    return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!embed || !ids || !positions || !out || !aligned16(embed) || !aligned16(out))
    return KVR_ERR_INVALID_ARG;
  if (rows > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  return launch_pdl<embed_rows_kernel>(static_cast<unsigned>(rows), dim3(128), 0, static_cast<cudaStream_t>(stream), 1, 
      static_cast<const uint16_t*>(embed), vocab, hidden / 8, ids, id_count, positions, rows,
      static_cast<uint16_t*>(out), error_count);
}

}  // extern "C"
