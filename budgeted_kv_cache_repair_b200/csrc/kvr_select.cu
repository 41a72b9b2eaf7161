// Query relevance of every prompt token from the model's frozen input
// embeddings (dense_query_relevance_scores, scoring.py:11-72): the score of
// token t is max over query tokens q of cos(E[t], E[q]) plus a fixed boost
// when t's id is one of the query ids.
//
// Two launches. The first normalises the query tokens' embedding rows into an
// fp32 workspace (one warp per query token). The second gives each prompt
// token one warp: it streams the token's embedding row once (16-byte loads,
// HBM-bound: N * hidden * element bytes), accumulates the squared norm and
// the dot products with up to kQueryBlock normalised query rows per pass
// (the query rows come from L1/L2: every warp reads the same ones), reduces
// them across the warp and writes max_q dot / max(norm, 1e-12) + boost.
// F.normalize divides by max(||x||, 1e-12) before the product; dividing the
// dot product afterwards differs only in the last bits.
//
// Token ids outside [0, vocab) are counted in the workspace's status word and
// their score is left as NaN; the host reads the count with the scores.
#include <type_traits>

#include "kvr_common.cuh"

namespace kvr {
namespace sel {

constexpr int kThreads = 256;
constexpr int kQueryBlock = 8;   // query rows per pass over a token's row
constexpr int kMaxQuery = 512;   // query ids held in shared memory for the exact-match test
constexpr int STATUS_BYTES = 256;

struct F32 {};

// Eight consecutive elements i..i+7 of an embedding table as fp32.
template <class T>
__device__ __forceinline__ void load8(const void* base, int64_t i, float (&v)[8]) {
  if constexpr (std::is_same<T, F32>::value) {
    const float* p = static_cast<const float*>(base) + i;
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
    v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
  } else {
    const Vec8 x = ld_vec8(static_cast<const uint16_t*>(base) + i);
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = T::to_f(x.h[e]);
  }
}
// Eight raw table elements held in registers until use (16 bytes for bf16/fp16,
// 32 for fp32), so that a warp can keep several chunks of loads in flight.
template <class T>
struct Raw8 {
  Vec8 x;
  // The table is read-only here and a row is read once per pass: no L1
  // allocation (3 % faster than plain loads on the Qwen3-8B table).
  __device__ __forceinline__ void load(const void* base, int64_t i) {
    uint4 u;
    asm volatile("ld.global.nc.L1::no_allocate.v4.b32 {%0,%1,%2,%3}, [%4];\n"
                 : "=r"(u.x), "=r"(u.y), "=r"(u.z), "=r"(u.w)
                 : "l"(static_cast<const uint16_t*>(base) + i));
    *reinterpret_cast<uint4*>(&x) = u;
  }
  __device__ __forceinline__ float get(int e) const { return T::to_f(x.h[e]); }
};
template <>
struct Raw8<F32> {
  float4 a, b;
  __device__ __forceinline__ void load(const void* base, int64_t i) {
    const float* p = static_cast<const float*>(base) + i;
    a = *reinterpret_cast<const float4*>(p);
    b = *reinterpret_cast<const float4*>(p + 4);
  }
  __device__ __forceinline__ float get(int e) const {
    const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
    return v[e];
  }
};

__device__ __forceinline__ void load8f(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w;
  v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// qn[i] = E[query_ids[i]] / max(||E[query_ids[i]]||, 1e-12), fp32.
template <class E>
__global__ void __launch_bounds__(kThreads) normalize_query_kernel(const void* embed, int64_t vocab, int hidden,
                                                                   const int64_t* query_ids, int nq, float* qn,
                                                                   int* status) {
  pdl_launch_dependents();
  pdl_wait();
  const int lane = threadIdx.x & 31;
  const int i = static_cast<int>((blockIdx.x * blockDim.x + threadIdx.x) >> 5);
  if (i >= nq) return;
  const int64_t id = query_ids[i];
  float* dst = qn + static_cast<int64_t>(i) * hidden;
  if (id < 0 || id >= vocab) {
    if (lane == 0) atomicAdd(status, 1);
    for (int d = lane; d < hidden; d += 32) dst[d] = __int_as_float(0x7fc00000);
    return;
  }
  const int64_t row = id * hidden;
  float ss = 0.f;
  for (int d = lane * 8; d < hidden; d += 256) {
    float v[8];
    load8<E>(embed, row + d, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) ss = fmaf(v[e], v[e], ss);
  }
  const float inv = 1.0f / fmaxf(sqrtf(warp_sum(ss)), 1e-12f);
  for (int d = lane * 8; d < hidden; d += 256) {
    float v[8];
    load8<E>(embed, row + d, v);
#pragma unroll
    for (int e = 0; e < 8; ++e) dst[d + e] = v[e] * inv;
  }
}

// One CTA stages up to `qb` normalised query rows in shared memory per pass;
// each warp then takes kTokens prompt tokens at a time, so every query value
// read from shared memory serves kTokens rows (shared-memory traffic per
// token = qb * hidden * 4 / kTokens bytes). Products accumulate as packed fp32
// pairs; three tokens keep the accumulators, the converted rows and two
// chunks of loads in flight within 128 registers.
// Persistent grid over token groups; scores are max over passes.
constexpr int kTokens = 3;

// hidden rounded up to whole 256-element chunks (the staged row length).
__host__ __device__ __forceinline__ int64_t padded_hidden(int hidden) { return (static_cast<int64_t>(hidden) + 255) / 256 * 256; }
constexpr int kUnroll = 2;  // row chunks in flight per token
constexpr int kScoreThreads = 512;  // 16 warps share one staged query block

template <class E>
__global__ void __launch_bounds__(kScoreThreads, 1) relevance_kernel(const void* embed, int64_t vocab, int hidden,
                                                             const int64_t* prompt_ids, int64_t n,
                                                             const int64_t* query_ids, int nq, const float* qn,
                                                             int qb, float boost, float* scores, int* status) {
  extern __shared__ float4 smem4[];
  // Staged query rows: row stride rs4 float4s = hidden rounded up to whole
  // 256-element chunks, so the permuted chunk layout below stays in its row.
  const int64_t rs4 = padded_hidden(hidden) / 4;
  int64_t* qids = reinterpret_cast<int64_t*>(smem4 + static_cast<int64_t>(qb) * rs4);  // [min(nq, kMaxQuery)]
  const int nqs = nq < kMaxQuery ? nq : kMaxQuery;
  pdl_launch_dependents();
  pdl_wait();
  for (int i = threadIdx.x; i < nqs; i += blockDim.x) qids[i] = query_ids[i];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int64_t groups = (n + kTokens - 1) / kTokens;
  const int64_t gstep = static_cast<int64_t>(gridDim.x) * (kScoreThreads / 32);
  for (int q0 = 0; q0 < nq; q0 += qb) {
    const int qn_here = nq - q0 < qb ? nq - q0 : qb;
    __syncthreads();  // the previous pass is done with qs
    // Staged in the order the lanes read: for each 256-element chunk, the first
    // four of every lane's eight elements (lane-contiguous), then the last four,
    // so a warp's 16-byte shared loads are conflict-free.
    for (int64_t i = threadIdx.x; i < static_cast<int64_t>(qn_here) * hidden / 4; i += blockDim.x) {
      const int64_t j = i / (hidden / 4), r = i - j * (hidden / 4);  // float4 r of query row j
      const int64_t c = r / 64, l = (r % 64) / 2, h = r % 2;          // chunk, lane, half
      smem4[j * rs4 + (c * 2 + h) * 32 + l] =
          reinterpret_cast<const float4*>(qn + static_cast<int64_t>(q0 + j) * hidden)[r];
    }
    __syncthreads();
    for (int64_t g = static_cast<int64_t>(blockIdx.x) * (kScoreThreads / 32) + warp; g < groups; g += gstep) {
      int64_t rows[kTokens];
      bool ok[kTokens];
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        const int64_t tok = g * kTokens + t;
        const int64_t id = tok < n ? prompt_ids[tok] : -1;
        ok[t] = id >= 0 && id < vocab;
        rows[t] = ok[t] ? id * hidden : 0;
      }
      // Packed fp32 pairs (even, odd element): one fma.rn.f32x2 per two products.
      uint64_t dot[kTokens][kQueryBlock], ss[kTokens];
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        ss[t] = 0;
#pragma unroll
        for (int j = 0; j < kQueryBlock; ++j) dot[t][j] = 0;
      }
      // kUnroll chunks of every token row are loaded before any is used.
      for (int d0 = lane * 8; d0 < hidden; d0 += 256 * kUnroll) {
        Raw8<E> raw[kUnroll][kTokens];
#pragma unroll
        for (int u = 0; u < kUnroll; ++u)
          if (d0 + u * 256 < hidden)
#pragma unroll
            for (int t = 0; t < kTokens; ++t) raw[u][t].load(embed, rows[t] + d0 + u * 256);
#pragma unroll
        for (int u = 0; u < kUnroll; ++u) {
          const int d = d0 + u * 256;
          if (d >= hidden) break;
          uint64_t v2[kTokens][4];
#pragma unroll
          for (int t = 0; t < kTokens; ++t)
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              v2[t][k] = f2(raw[u][t].get(2 * k), raw[u][t].get(2 * k + 1));
              ss[t] = f2_fma(v2[t][k], v2[t][k], ss[t]);
            }
          const int c = (d - lane * 8) / 256;  // 256-element chunk of the row
#pragma unroll
          for (int j = 0; j < kQueryBlock; ++j) {
            if (j < qn_here) {
              const float4* qrow = smem4 + static_cast<int64_t>(j) * rs4;
              const float4 lo = qrow[(2 * c) * 32 + lane];
              const float4 hi = qrow[(2 * c + 1) * 32 + lane];
              const uint64_t w2[4] = {f2(lo.x, lo.y), f2(lo.z, lo.w), f2(hi.x, hi.y), f2(hi.z, hi.w)};
#pragma unroll
              for (int t = 0; t < kTokens; ++t)
#pragma unroll
                for (int k = 0; k < 4; ++k) dot[t][j] = f2_fma(v2[t][k], w2[k], dot[t][j]);
            }
          }
        }
      }
#pragma unroll
      for (int t = 0; t < kTokens; ++t) {
        const int64_t tok = g * kTokens + t;
        float best = -INFINITY;
#pragma unroll
        for (int j = 0; j < kQueryBlock; ++j) {
          if (j < qn_here) {
            float a, b;
            f2_split(dot[t][j], a, b);
            best = fmaxf(best, warp_sum(a + b));
          }
        }
        // Every pass streams the row again, so the norm comes with it.
        float sa, sb;
        f2_split(ss[t], sa, sb);
        const float norm = fmaxf(sqrtf(warp_sum(sa + sb)), 1e-12f);
        if (lane == 0 && tok < n) {
          if (!ok[t]) {
            if (q0 == 0) {
              atomicAdd(status, 1);
              scores[tok] = __int_as_float(0x7fc00000);
            }
          } else {
            scores[tok] = q0 == 0 ? best / norm : fmaxf(scores[tok], best / norm);
          }
        }
      }
    }
  }
  // Exact-match boost, after every pass.
  __syncthreads();
  for (int64_t g = static_cast<int64_t>(blockIdx.x) * (kScoreThreads / 32) + warp; g < groups; g += gstep) {
    const int64_t tok = g * kTokens + lane;
    if (lane < kTokens && tok < n) {
      const int64_t id = prompt_ids[tok];
      if (id >= 0 && id < vocab) {
        bool exact = false;
        for (int i = 0; i < nqs && !exact; ++i) exact = qids[i] == id;
        for (int i = nqs; i < nq && !exact; ++i) exact = query_ids[i] == id;
        if (exact) scores[tok] += boost;
      }
    }
  }
}

// Query rows staged per pass: up to kQueryBlock, within ~200 KB of shared memory.
inline int query_block(int hidden) {
  const int fit = static_cast<int>((200 * 1024 - kMaxQuery * 8) / (padded_hidden(hidden) * 4));
  return fit < kQueryBlock ? (fit < 1 ? 0 : fit) : kQueryBlock;
}

template <class E>
int launch(const void* embed, int64_t vocab, int hidden, const int64_t* prompt_ids, int64_t n,
           const int64_t* query_ids, int nq, float boost, float* scores, float* qn, int* status, cudaStream_t s) {
  const void* e = embed;
  const unsigned qblocks = static_cast<unsigned>((static_cast<int64_t>(nq) * 32 + kThreads - 1) / kThreads);
  int st = launch_pdl<normalize_query_kernel<E>>(dim3(qblocks), dim3(kThreads), 0, s, 1, e, vocab, hidden, query_ids,
                                                 nq, qn, status);
  if (st != KVR_OK) return st;
  const int qb = query_block(hidden);
  const int nqs = nq < kMaxQuery ? nq : kMaxQuery;
  const size_t smem = static_cast<size_t>(qb) * padded_hidden(hidden) * 4 + static_cast<size_t>(nqs) * 8;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t err = cudaGetDevice(&dev);
  if (err == cudaSuccess && (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE))) {
    err = cudaFuncSetAttribute(relevance_kernel<E>, cudaFuncAttributeMaxDynamicSharedMemorySize, 210 * 1024);
    if (err == cudaSuccess && dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  if (err != cudaSuccess) {
    set_last_cuda_error(err);
    return KVR_ERR_CUDA;
  }
  const int64_t groups = (n + kTokens - 1) / kTokens;
  const int64_t want = (groups + kScoreThreads / 32 - 1) / (kScoreThreads / 32);
  const unsigned blocks = static_cast<unsigned>(want < kNumSMs ? want : kNumSMs);
  return launch_pdl_default_carveout<relevance_kernel<E>>(dim3(blocks), dim3(kScoreThreads), smem, s, 1, e, vocab,
                                                         hidden, prompt_ids, n, query_ids, nq,
                                                         static_cast<const float*>(qn), qb, boost, scores, status);
}

}  // namespace sel
}  // namespace kvr

using namespace kvr;

extern "C" {

size_t kvr_query_relevance_workspace_size(int hidden, int query_count) {
  if (hidden <= 0 || query_count <= 0) return sel::STATUS_BYTES;
  return sel::STATUS_BYTES + static_cast<size_t>(hidden) * query_count * sizeof(float);
}

int kvr_query_relevance(const void* embed, int64_t vocab, int hidden, int dtype, const int64_t* prompt_ids,
                        int64_t prompt_count, const int64_t* query_ids, int query_count, float exact_boost,
                        float* scores, void* workspace, size_t workspace_bytes, void* stream) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16 && dtype != KVR_DTYPE_F32) return KVR_ERR_UNSUPPORTED;
  if (vocab <= 0 || hidden <= 0 || hidden % 8 || prompt_count < 0 || query_count <= 0) return KVR_ERR_INVALID_ARG;
  if (sel::query_block(hidden) < 1) return KVR_ERR_UNSUPPORTED;  // one fp32 query row must fit in shared memory
  if (!embed || !aligned16(embed) || !query_ids || (prompt_count && (!prompt_ids || !scores)) || !workspace ||
      !aligned16(workspace) || workspace_bytes < kvr_query_relevance_workspace_size(hidden, query_count))
    return KVR_ERR_INVALID_ARG;
  auto s = static_cast<cudaStream_t>(stream);
  int* status = static_cast<int*>(workspace);
  float* qn = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + sel::STATUS_BYTES);
  const cudaError_t e = cudaMemsetAsync(status, 0, sizeof(int), s);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (prompt_count == 0) return KVR_OK;
  switch (dtype) {
    case KVR_DTYPE_BF16:
      return sel::launch<BF16>(embed, vocab, hidden, prompt_ids, prompt_count, query_ids, query_count, exact_boost,
                               scores, qn, status, s);
    case KVR_DTYPE_F16:
      return sel::launch<F16>(embed, vocab, hidden, prompt_ids, prompt_count, query_ids, query_count, exact_boost,
                              scores, qn, status, s);
    default:
      return sel::launch<sel::F32>(embed, vocab, hidden, prompt_ids, prompt_count, query_ids, query_count, exact_boost,
                                scores, qn, status, s);
  }
}

}  // extern "C"
