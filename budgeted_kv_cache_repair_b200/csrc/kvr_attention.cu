// Selected-query absolute-causal attention with GQA packing and split-KV.
//
// Work unit (CTA): one KV head h, one tile of BM=64 "m-entries", one key chunk.
// An m-entry is a (selected row r, query head of group g) pair, m = r*G + g, so
// the G query heads that share KV head h ride in the same MMA rows and every
// K/V tile read from HBM serves all of them (no repeat_kv). Rows are sorted by
// absolute position, so a tile's causal span is [0, pos(last row)] and keys
// below pos(first row) need no mask.
//
// Inside a CTA, 4 warps each own 16 m-entries. K/V blocks of 64 keys stream
// through a cp.async double buffer in XOR-swizzled shared memory; S = Q K^T and
// O += P V run on the tensor cores (m16n8k16, fp32 accumulate). The online
// softmax is fp32. P is split as P = P_hi + P_lo (both in the element type)
// and both halves multiply V, so probabilities keep ~16 mantissa bits, close
// to the reference's fp32-probability P@V (kernels/_indexed_triton.py:58).
//
// When the (head, tile) grid is too small for 148 SMs the key range is cut
// into chunks; each chunk CTA writes unnormalised partials (O, running max,
// running sum) to the workspace and attn_combine_kernel merges them.
#include <math.h>

#include "kvr_common.cuh"

namespace kvr {

namespace attn {

constexpr int BM = 64;        // m-entries per CTA
constexpr int BN = 64;        // keys per block
constexpr int THREADS = 128;  // 4 warps x 16 m-entries

struct Args {
  const uint16_t* q;
  const uint16_t* k;
  const uint16_t* v;
  uint16_t* out;
  const int64_t* positions;
  int64_t rows;
  int hq, hkv, group;
  int64_t cache_rows, c_hs, c_rs;
  float scale_log2;
  int tiles, nchunks;
  int64_t chunk;  // keys per chunk (multiple of BN)
  float* ws_o;    // [hkv][tiles][nchunks][BM][D]
  float* ws_ml;   // [hkv][tiles][nchunks][BM][2]
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;  // src-size 0 zero-fills the 16 bytes
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n));
}
__device__ __forceinline__ void cp_commit() { asm volatile("cp.async.commit_group;\n" ::); }
template <int N>
__device__ __forceinline__ void cp_wait() {
  asm volatile("cp.async.wait_group %0;\n" ::"n"(N));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                          uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];\n"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <class T>
__device__ __forceinline__ void mma16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1);

template <>
__device__ __forceinline__ void mma16816<BF16>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
template <>
__device__ __forceinline__ void mma16816<F16>(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Two floats -> packed pair of 16-bit elements (low half = first).
template <class T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return static_cast<uint32_t>(T::from_f(lo)) | (static_cast<uint32_t>(T::from_f(hi)) << 16);
}

// Byte offset of 16-byte chunk c of row r in a swizzled [rows][D] tile.
template <int D>
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * (D * 2) + ((c ^ (r & 7)) << 4));
}

template <class T, int D>
__global__ void __launch_bounds__(THREADS) attn_kernel(Args a) {
  constexpr int CPR = D / 8;              // 16-byte chunks per row
  constexpr int TILE_BYTES = BN * D * 2;  // one K or V block
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t* sq = smem;                        // [BM][D]
  uint8_t* skv = smem + BM * D * 2;          // 2 stages x (K, V)

  const int tid = threadIdx.x;
  const int warp = tid >> 5, lane = tid & 31;
  const int gq = lane >> 2, tq = lane & 3;
  const int h = blockIdx.y;
  const int tile = blockIdx.x / a.nchunks;
  const int chunk = blockIdx.x - tile * a.nchunks;
  const int G = a.group;
  const int64_t total_m = a.rows * G;
  const int64_t m0 = static_cast<int64_t>(tile) * BM;
  const int64_t r_first = m0 / G;
  int64_t r_last = (m0 + BM - 1) / G;
  if (r_last > a.rows - 1) r_last = a.rows - 1;
  const int64_t pmin = a.positions[r_first];
  const int64_t pmax = a.positions[r_last];
  const int64_t k_begin = chunk * a.chunk;
  if (k_begin > pmax) return;  // this chunk lies past every row of the tile
  int64_t k_end = k_begin + a.chunk;
  if (k_end > pmax + 1) k_end = pmax + 1;

  // Absolute positions of this thread's two MMA rows (padding entries see key 0).
  int64_t pos_ab[2];
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int64_t m = m0 + warp * 16 + gq + i * 8;
    pos_ab[i] = m < total_m ? a.positions[m / G] : 0;
  }

  // Q tile -> shared (cp.async group 0 together with the first K/V block).
  for (int idx = tid; idx < BM * CPR; idx += THREADS) {
    const int row = idx / CPR, c = idx - row * CPR;
    const int64_t m = m0 + row;
    const bool ok = m < total_m;
    const int64_t r = ok ? m / G : 0;
    const int g = ok ? static_cast<int>(m - r * G) : 0;
    const uint16_t* src = a.q + ((r * a.hq + static_cast<int64_t>(h) * G + g) * D + c * 8);
    cp_async16(smem_u32(sq + swz<D>(row, c)), ok ? src : a.q, ok);
  }
  const uint16_t* kbase = a.k + static_cast<int64_t>(h) * a.c_hs;
  const uint16_t* vbase = a.v + static_cast<int64_t>(h) * a.c_hs;
  auto load_kv = [&](int stage, int64_t key0) {
    uint8_t* sk = skv + stage * 2 * TILE_BYTES;
    uint8_t* sv = sk + TILE_BYTES;
    for (int idx = tid; idx < BN * CPR; idx += THREADS) {
      const int row = idx / CPR, c = idx - row * CPR;
      const int64_t key = key0 + row;
      const bool ok = key < k_end;
      const int64_t off = ok ? key * a.c_rs + c * 8 : 0;
      cp_async16(smem_u32(sk + swz<D>(row, c)), kbase + off, ok);
      cp_async16(smem_u32(sv + swz<D>(row, c)), vbase + off, ok);
    }
  };
  load_kv(0, k_begin);
  cp_commit();

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
  float mrow[2] = {-INFINITY, -INFINITY};
  float lrow[2] = {0.f, 0.f};
  uint32_t qf[D / 16][4];
  bool have_q = false;

  int stage = 0;
  for (int64_t blk = k_begin; blk < k_end; blk += BN, stage ^= 1) {
    const bool has_next = blk + BN < k_end;
    if (has_next) {
      load_kv(stage ^ 1, blk + BN);
      cp_commit();
      cp_wait<1>();
    } else {
      cp_wait<0>();
    }
    __syncthreads();
    if (!have_q) {
#pragma unroll
      for (int kk = 0; kk < D / 16; ++kk) {
        const int i = lane >> 3;
        const int row = warp * 16 + (i & 1) * 8 + (lane & 7);
        ldsm_x4(smem_u32(sq + swz<D>(row, kk * 2 + (i >> 1))), qf[kk][0], qf[kk][1], qf[kk][2],
                qf[kk][3]);
      }
      have_q = true;
    }
    const uint8_t* sk = skv + stage * 2 * TILE_BYTES;
    const uint8_t* sv = sk + TILE_BYTES;

    // S = Q K^T for 64 keys: 8 n-tiles of 8 keys.
    float s[BN / 8][4];
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
#pragma unroll
      for (int jp = 0; jp < BN / 16; ++jp) {
        const int i = lane >> 3;
        const int key = (jp * 2 + (i >> 1)) * 8 + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4(smem_u32(sk + swz<D>(key, kk * 2 + (i & 1))), b0, b1, b2, b3);
        mma16816<T>(s[jp * 2], qf[kk], b0, b1);
        mma16816<T>(s[jp * 2 + 1], qf[kk], b2, b3);
      }
    }

    // Scale, causal/chunk mask, online softmax (fp32, base-2).
    const bool need_mask = blk + BN - 1 > pmin || blk + BN > k_end;
    float mx[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float x = s[j][e] * a.scale_log2;
        if (need_mask) {
          const int64_t key = blk + j * 8 + tq * 2 + (e & 1);
          if (key > pos_ab[e >> 1] || key >= k_end) x = -INFINITY;
        }
        s[j][e] = x;
        mx[e >> 1] = fmaxf(mx[e >> 1], x);
      }
    }
    float alpha[2], base[2];
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 1));
      mx[i] = fmaxf(mx[i], __shfl_xor_sync(0xffffffffu, mx[i], 2));
      const float mnew = fmaxf(mrow[i], mx[i]);
      base[i] = mnew == -INFINITY ? 0.f : mnew;
      alpha[i] = exp2f(mrow[i] - base[i]);
      mrow[i] = mnew;
      lrow[i] *= alpha[i];
    }
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= alpha[0];
      o[n][1] *= alpha[0];
      o[n][2] *= alpha[1];
      o[n][3] *= alpha[1];
    }
#pragma unroll
    for (int j = 0; j < BN / 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float p = exp2f(s[j][e] - base[e >> 1]);
        s[j][e] = p;
        lrow[e >> 1] += p;
      }
    }

    // O += P V with P = P_hi + P_lo.
#pragma unroll
    for (int kk = 0; kk < BN / 16; ++kk) {
      uint32_t ph[4], pl[4];
      const float* s0 = s[kk * 2];
      const float* s1 = s[kk * 2 + 1];
      const float src[8] = {s0[0], s0[1], s0[2], s0[3], s1[0], s1[1], s1[2], s1[3]};
      float hi[8], lo[8];
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        hi[e] = rnd<T>(src[e]);
        lo[e] = src[e] - hi[e];
      }
      ph[0] = pack2<T>(hi[0], hi[1]);
      ph[1] = pack2<T>(hi[2], hi[3]);
      ph[2] = pack2<T>(hi[4], hi[5]);
      ph[3] = pack2<T>(hi[6], hi[7]);
      pl[0] = pack2<T>(lo[0], lo[1]);
      pl[1] = pack2<T>(lo[2], lo[3]);
      pl[2] = pack2<T>(lo[4], lo[5]);
      pl[3] = pack2<T>(lo[6], lo[7]);
#pragma unroll
      for (int np = 0; np < D / 16; ++np) {
        const int i = lane >> 3;
        const int key = kk * 16 + (i & 1) * 8 + (lane & 7);
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(smem_u32(sv + swz<D>(key, np * 2 + (i >> 1))), b0, b1, b2, b3);
        mma16816<T>(o[np * 2], ph, b0, b1);
        mma16816<T>(o[np * 2], pl, b0, b1);
        mma16816<T>(o[np * 2 + 1], ph, b2, b3);
        mma16816<T>(o[np * 2 + 1], pl, b2, b3);
      }
    }
    __syncthreads();  // stage is refilled by the next iteration's prefetch
  }

#pragma unroll
  for (int i = 0; i < 2; ++i) {
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 1);
    lrow[i] += __shfl_xor_sync(0xffffffffu, lrow[i], 2);
  }
  if (a.nchunks == 1) {
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const int64_t m = m0 + warp * 16 + gq + i * 8;
      if (m >= total_m) continue;
      const int64_t r = m / G;
      const int g = static_cast<int>(m - r * G);
      uint16_t* dst = a.out + (r * a.hq + static_cast<int64_t>(h) * G + g) * D;
      const float inv = 1.0f / lrow[i];
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        const uint32_t pr = pack2<T>(o[n][i * 2] * inv, o[n][i * 2 + 1] * inv);
        *reinterpret_cast<uint32_t*>(dst + n * 8 + tq * 2) = pr;
      }
    }
    return;
  }
  const int64_t w = (static_cast<int64_t>(h) * a.tiles + tile) * a.nchunks + chunk;
  float* wo = a.ws_o + w * BM * D;
  float* wml = a.ws_ml + w * BM * 2;
#pragma unroll
  for (int i = 0; i < 2; ++i) {
    const int ml = warp * 16 + gq + i * 8;
#pragma unroll
    for (int n = 0; n < D / 8; ++n)
      *reinterpret_cast<float2*>(wo + ml * D + n * 8 + tq * 2) = make_float2(o[n][i * 2], o[n][i * 2 + 1]);
    if (tq == 0) *reinterpret_cast<float2*>(wml + ml * 2) = make_float2(mrow[i], lrow[i]);
  }
}

// Merge the chunk partials of one (head, tile): O = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.
template <class T, int D>
__global__ void __launch_bounds__(256) attn_combine_kernel(Args a) {
  const int h = blockIdx.y;
  const int tile = blockIdx.x;
  const int G = a.group;
  const int64_t total_m = a.rows * G;
  const int64_t m0 = static_cast<int64_t>(tile) * BM;
  int64_t r_last = (m0 + BM - 1) / G;
  if (r_last > a.rows - 1) r_last = a.rows - 1;
  const int64_t pmax = a.positions[r_last];
  int nv = static_cast<int>(pmax / a.chunk) + 1;
  if (nv > a.nchunks) nv = a.nchunks;
  const int64_t w0 = (static_cast<int64_t>(h) * a.tiles + tile) * a.nchunks;
  constexpr int VPR = D / 8;
  for (int idx = threadIdx.x; idx < BM * VPR; idx += blockDim.x) {
    const int ml = idx / VPR, v = idx - ml * VPR;
    const int64_t m = m0 + ml;
    if (m >= total_m) continue;
    float M = -INFINITY;
    for (int c = 0; c < nv; ++c) M = fmaxf(M, a.ws_ml[(w0 + c) * BM * 2 + ml * 2]);
    float L = 0.f;
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int c = 0; c < nv; ++c) {
      const float2 ml2 = *reinterpret_cast<const float2*>(a.ws_ml + (w0 + c) * BM * 2 + ml * 2);
      const float wgt = exp2f(ml2.x - M);  // 0 for rows fully masked in chunk c
      if (wgt == 0.f) continue;
      L += wgt * ml2.y;
      const float4* src = reinterpret_cast<const float4*>(a.ws_o + ((w0 + c) * BM + ml) * D + v * 8);
      const float4 x0 = src[0], x1 = src[1];
      acc[0] += wgt * x0.x; acc[1] += wgt * x0.y; acc[2] += wgt * x0.z; acc[3] += wgt * x0.w;
      acc[4] += wgt * x1.x; acc[5] += wgt * x1.y; acc[6] += wgt * x1.z; acc[7] += wgt * x1.w;
    }
    const float inv = 1.0f / L;
    const int64_t r = m / G;
    const int g = static_cast<int>(m - r * G);
    Vec8 out;
#pragma unroll
    for (int e = 0; e < 8; ++e) out.h[e] = T::from_f(acc[e] * inv);
    st_vec8(a.out + (r * a.hq + static_cast<int64_t>(h) * G + g) * D + v * 8, out);
  }
}

struct Plan {
  int tiles, nchunks;
  int64_t chunk;
};

inline Plan make_plan(int64_t rows, int hq, int hkv, int64_t max_position) {
  Plan p;
  const int group = hq / hkv;
  const int64_t total_m = rows * group;
  p.tiles = static_cast<int>((total_m + BM - 1) / BM);
  const int64_t keys = max_position + 1;
  const int64_t blocks = (keys + BN - 1) / BN;
  const int64_t base = static_cast<int64_t>(p.tiles) * hkv;
  // Aim for >= 3 CTAs per SM (2 resident + tail) but keep >= 4 key blocks per chunk.
  const int64_t target = static_cast<int64_t>(kNumSMs) * 3;
  int64_t n = (target + base - 1) / base;
  int64_t max_n = (blocks + 3) / 4;
  if (n > max_n) n = max_n;
  if (n < 1) n = 1;
  const int64_t chunk_blocks = (blocks + n - 1) / n;
  p.chunk = chunk_blocks * BN;
  p.nchunks = static_cast<int>((keys + p.chunk - 1) / p.chunk);
  return p;
}

inline size_t workspace_bytes(const Plan& p, int hkv, int head_dim) {
  if (p.nchunks <= 1) return 0;
  const size_t units = static_cast<size_t>(hkv) * p.tiles * p.nchunks;
  return units * BM * (head_dim + 2) * sizeof(float) + 256;
}

template <class T, int D>
int launch(const Args& a, cudaStream_t s) {
  const int smem = BM * D * 2 + 2 * 2 * BN * D * 2;
  // The shared-memory opt-in is a per-device function attribute: set it once
  // per device (one process drives one GPU, but a process may see several).
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    e = cudaFuncSetAttribute(attn_kernel<T, D>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  dim3 grid(a.tiles * a.nchunks, a.hkv);
  attn_kernel<T, D><<<grid, THREADS, smem, s>>>(a);
  int st = check_launch();
  if (st != KVR_OK || a.nchunks == 1) return st;
  attn_combine_kernel<T, D><<<dim3(a.tiles, a.hkv), 256, 0, s>>>(a);
  return check_launch();
}

}  // namespace attn
}  // namespace kvr

using namespace kvr;

extern "C" {

size_t kvr_attention_workspace_size(int64_t rows, int q_heads, int kv_heads, int head_dim,
                                    int64_t cache_rows) {
  if (rows <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || cache_rows <= 0)
    return 0;
  attn::Plan p = attn::make_plan(rows, q_heads, kv_heads, cache_rows - 1);
  return attn::workspace_bytes(p, kv_heads, head_dim);
}

int kvr_selected_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                           const int64_t* positions, int64_t rows, int q_heads, int kv_heads,
                           int head_dim, int64_t cache_rows, int64_t cache_head_stride,
                           int64_t cache_row_stride, int64_t max_position, float scale,
                           void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || cache_rows < 0)
    return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!q || !k_cache || !v_cache || !out || !positions || !aligned16(q) || !aligned16(k_cache) ||
      !aligned16(v_cache) || !aligned16(out) || cache_head_stride % 8 || cache_row_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (max_position < 0 || max_position >= cache_rows || !(scale == scale)) return KVR_ERR_INVALID_ARG;
  attn::Plan p = attn::make_plan(rows, q_heads, kv_heads, max_position);
  if (static_cast<int64_t>(p.tiles) * p.nchunks > 0x7fffffff || kv_heads > 65535)
    return KVR_ERR_UNSUPPORTED;
  const size_t need = attn::workspace_bytes(p, kv_heads, head_dim);
  if (need && (!workspace || workspace_bytes < need || !aligned16(workspace)))
    return KVR_ERR_INVALID_ARG;
  attn::Args a;
  a.q = static_cast<const uint16_t*>(q);
  a.k = static_cast<const uint16_t*>(k_cache);
  a.v = static_cast<const uint16_t*>(v_cache);
  a.out = static_cast<uint16_t*>(out);
  a.positions = positions;
  a.rows = rows;
  a.hq = q_heads;
  a.hkv = kv_heads;
  a.group = q_heads / kv_heads;
  a.cache_rows = cache_rows;
  a.c_hs = cache_head_stride;
  a.c_rs = cache_row_stride;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.tiles = p.tiles;
  a.nchunks = p.nchunks;
  a.chunk = p.chunk;
  const size_t units = static_cast<size_t>(kv_heads) * p.tiles * p.nchunks;
  a.ws_o = static_cast<float*>(workspace);
  a.ws_ml = need ? a.ws_o + units * attn::BM * head_dim : nullptr;
  auto s = static_cast<cudaStream_t>(stream);
  if (dtype == KVR_DTYPE_BF16)
    return head_dim == 128 ? attn::launch<BF16, 128>(a, s) : attn::launch<BF16, 64>(a, s);
  return head_dim == 128 ? attn::launch<F16, 128>(a, s) : attn::launch<F16, 64>(a, s);
}

}  // extern "C"
