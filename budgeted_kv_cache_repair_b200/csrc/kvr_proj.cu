// Fused projections of the packed layer loop on sm_100a (tcgen05 + TMEM +
// TMA): out = x . W^T, with the elementwise work that surrounds each
// projection in the transformers decoder layer done by the same launch, so a
// layer is four projection launches and the attention:
//
//   q/k/v   x = RMSNorm(h) (input norm) formed while the stages are filled;
//           epilogue per 128-column tile (= one head of head_dim 128): round,
//           q/k RMSNorm (Qwen3), RoPE at the row's absolute position, q into
//           the packed query buffer, k and v into the cache at that position
//   o       x = attention output; epilogue h = round(h + round(o)) in place,
//           plus each tile's per-row sum of squares of the new h
//   gate/up x = RMSNorm(h) (post-attention norm) from those sums; epilogue
//           act = round(silu(round(gate))) * round(up), rounded
//   down    x = act; epilogue as o
//
// which replaces, per layer, the residual-add + RMSNorm kernels, the K/V
// epilogue kernel and the SiLU product of the separate-kernel loop, and with
// them four kernel boundaries (each a drain of one grid and the start of the
// next) on a path whose floor is the weight stream.
//
// Measured (Llama-3-8B shape, 64 rows, 12 layers replayed from a CUDA graph):
// 166 us per layer against 131 us for the cuBLAS loop, so it is a request
// option (KVR_PROJ_FUSED), not the default. Without its epilogues the same
// launches take 134 us per layer: the stream-K fix-up and the row passes at
// the end of each launch cost ~8 us that the next launch cannot overlap, and
// the weight stream alone reaches 4.2-4.5 TB/s (ncu, one launch, no x and no
// epilogue), below cuBLAS's ~5 TB/s at these shapes. Neither deeper stages
// along k (2 and 4 TMA boxes per stage: same DRAM throughput) nor prefetching
// the next launch's first weight tiles into L2 changed that.
//
// The work of a launch is (tile, 64-wide k-chunk) units split into one
// contiguous range per CTA over a persistent grid of one CTA per SM (stream-K):
// every SM streams the same number of weight bytes. A tile inside one range is
// finished straight from TMEM; a tile cut by a range boundary leaves fp32
// partials in the workspace and its last contributor (tile counter) sums them
// in CTA order and finishes it, so results do not depend on timing. Counters
// are zero on entry and left zero.
//
// Warp roles (384 threads): warps 0-7 epilogue (warp w reads TMEM lanes
// 32*(w%4).., the tile's weight rows; warpgroup w/4 takes every other 32-row
// chunk of x), warp 8 TMA producer (weight and x tiles into a ring of
// 128B-swizzled stages, no multicast), warp 9 MMA issuer, warps 10-11 x
// normaliser when x is RMSNorm(h): they turn each stage's raw h tile into the
// normalised one in place (the rows' inverse RMS from the sums of squares the
// previous launch left) before the MMA may read it. Every
// mbarrier wait is bounded; on a give-up the kernel records an error code in
// the status word, stops issuing, drains its own copies and MMAs, frees TMEM
// and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <type_traits>

#include "kvr_common.cuh"
#include "kvr_proj.h"
#include "kvr_sm100.cuh"

namespace kvr {
namespace proj {

constexpr int BM = 128;  // weight rows per tile (MMA M, TMEM lanes)
constexpr int SUBK = 64;  // k elements of one TMA box: one 128-byte swizzle row
#ifndef KVR_PROJ_KSUB
#define KVR_PROJ_KSUB 1
#endif
constexpr int KSUB = KVR_PROJ_KSUB;  // boxes per stage along k
constexpr int BK = SUBK * KSUB;      // k elements per stage (one unit of work)
constexpr int W_BYTES = BM * 128 * KSUB;  // weight tile of one stage
constexpr int kEpiThreads = 256;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kXWarp0 = 10;
constexpr int kXThreads = 64;
constexpr int THREADS = 384;
constexpr int STATUS_BYTES = 256;
constexpr long long WAIT_LIMIT = kDefaultWaitLimit;  // drains of the CTA's own copies and MMAs
// Named barriers: kAllEpi (the 256 epilogue threads), kTmemBar (every warp
// but the TMA producer, after the TMEM allocation), kXBar (the x warps).
constexpr int kAllEpi = 3;
constexpr int kTmemBar = 4;
constexpr int kXBar = 5;

enum Err : int { ERR_EMPTY = 1, ERR_FULL, ERR_ACC_EMPTY, ERR_ACC_FULL, ERR_DRAIN, ERR_SMEM_ALIGN };

template <int BN>
struct Layout {
  static constexpr int X_BYTES = BN * 128 * KSUB;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  // Ring of at most ~192 KB (BN 64) / 128 KB (BN 128, whose fp32 tile is larger).
  static constexpr int NS = (BN <= 64 ? 196608 : 131072) / STAGE;
  static constexpr int RING = NS * STAGE;
  // A finished tile in fp32, [x row][weight row] (row stride BM floats), for
  // the row-wise epilogue passes and the stream-K fix-up.
  static constexpr int TILE_OFF = RING;
  static constexpr int TILE_BYTES = BN * BM * 4;
  static constexpr int INV_OFF = TILE_OFF + TILE_BYTES;  // float [BN]: inverse RMS of each x row
  static constexpr int BAR_OFF = INV_OFF + BN * 4;
  // wfull[NS] (weight bytes, and x bytes when x is used as loaded), xfull[NS]
  // (x-warp arrivals once normalised), empty[NS], xraw[NS] (x bytes to be
  // normalised), acc_full[2], acc_empty[2], drain
  static constexpr int NBAR = 4 * NS + 5;
  static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // abort flag, TMEM address, fix-up flag
  static constexpr int USED = MISC_OFF + 16;
  static constexpr int BYTES = USED + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators
  static_assert(BYTES <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
  static_assert(STAGE % 1024 == 0 && W_BYTES % 1024 == 0, "swizzled tiles need 1 KB alignment");
};

struct Args {
  int rows, kchunks, tiles, grid;
  int64_t units, k;
  int q_tiles, k_tiles;  // PROJ_QKV_ROPE: tiles [0, q_tiles) q heads, then k_tiles k heads, then v heads
  int64_t n_out;         // output columns (PROJ_RESIDUAL, PROJ_GATED)
  uint16_t* out;
  int64_t out_stride;
  float* ssq_out;
  // x producer: RMSNorm of h
  const uint16_t* x;
  int64_t x_stride;
  const uint16_t* norm_w;
  const float* ssq_in;
  int ssq_tiles;
  float inv_k, eps;
  // PROJ_QKV_ROPE
  int q_heads;
  uint16_t* q_out;
  uint16_t* k_cache;
  uint16_t* v_cache;
  int64_t cache_rows, c_hs, c_rs;
  const int64_t* positions;
  const uint16_t* cos_tab;
  const uint16_t* sin_tab;
  const uint16_t* q_norm;
  const uint16_t* k_norm;
  int* status;
  int* counters;    // [tiles]
  float* partials;  // [grid][2 slots][BN x rows][128] fp32
  long long wait_limit;
};

// Weight-tile coordinates of unit (t, c): which map and its row offset.
__device__ __forceinline__ void tile_rows(int epi, int q_tiles, int k_tiles, int t, int& map, int& row0) {
  map = 0;
  if (epi == PROJ_QKV_ROPE) {
    if (t < q_tiles) {
      row0 = t * BM;
    } else if (t < q_tiles + k_tiles) {
      map = 1;
      row0 = (t - q_tiles) * BM;
    } else {
      map = 2;
      row0 = (t - q_tiles - k_tiles) * BM;
    }
  } else if (epi == PROJ_GATED) {
    row0 = t * 64;
  } else {
    row0 = t * BM;
  }
}

struct Maps {
  CUtensorMap x;
  CUtensorMap w[3];
};



// First unit of CTA b's range and the CTA that owns unit u (its inverse).
__device__ __forceinline__ int64_t range_begin(int64_t units, int grid, int b) { return units * b / grid; }
__device__ __forceinline__ int owner(int64_t units, int grid, int64_t u) {
  return static_cast<int>(((u + 1) * grid + units - 1) / units - 1);
}

// The (tile, k range) jobs of one CTA, in the order every role walks them.
struct Cursor {
  int64_t u, u_end, kc;
  __device__ __forceinline__ bool next(int& t, int& c0, int& c1) {
    if (u >= u_end) return false;
    const int64_t tt = u / kc;
    c0 = static_cast<int>(u - tt * kc);
    c1 = static_cast<int>(kc < c0 + (u_end - u) ? kc : c0 + (u_end - u));
    u += c1 - c0;
    t = static_cast<int>(tt);
    return true;
  }
};

__device__ __forceinline__ Cursor make_cursor(const Args& a, int b) {
  Cursor c;
  c.kc = a.kchunks;
  c.u = range_begin(a.units, a.grid, b);
  c.u_end = range_begin(a.units, a.grid, b + 1);
  return c;
}

// Byte offset of 16-byte chunk c (0..7) of row r in a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

// ------------------------------------------------- 16-bit conversions
// Round to nearest even with the hardware conversion; a NaN becomes the quiet
// NaN torch writes (0x7FC0 for bf16), so the bits equal T::from_f's.
template <class T>
__device__ __forceinline__ uint16_t to16(float f);
template <>
__device__ __forceinline__ uint16_t to16<BF16>(float f) {
  const uint16_t b = __bfloat16_as_ushort(__float2bfloat16_rn(f));
  return f != f ? static_cast<uint16_t>(0x7fc0u) : b;
}
template <>
__device__ __forceinline__ uint16_t to16<F16>(float f) {
  return __half_as_ushort(__float2half_rn(f));
}
template <class T>
__device__ __forceinline__ float rnd16(float f) {
  return T::to_f(to16<T>(f));
}
// Two values at once (finite inputs: the x normaliser's).
template <class T>
__device__ __forceinline__ uint32_t cvt2(float lo, float hi) {
  if constexpr (std::is_same<T, BF16>::value) {
    const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  } else {
    const __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<const uint32_t*>(&v);
  }
}
template <class T>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  return make_float2(T::to_f(static_cast<uint16_t>(v & 0xffffu)), T::to_f(static_cast<uint16_t>(v >> 16)));
}

// ------------------------------------------------------------- epilogues
// Row-wise passes over a finished tile staged in shared memory as fp32
// [x row][weight row] (stride BM), run by the 256 epilogue threads together
// after a barrier.

// o / down: h[r, t*128 + c] = round(h + round(tile[r][c])) in place, 16 bytes
// per access (16 threads per x row), and the row's sum of squares of its 128
// new values: each thread's 8 in order, then across the 16 threads by
// shuffles in a fixed tree, into ssq_out[t][r].
template <class T, int BN>
__device__ __forceinline__ void epi_residual(const Args& a, int t, const float* tile, int tid) {
  constexpr int TASKS = BN * 16 / kEpiThreads;  // (x row, 8-column chunk) pairs per thread
  uint4 hv[TASKS];
#pragma unroll
  for (int i = 0; i < TASKS; ++i) {
    const int task = tid + i * kEpiThreads, r = task >> 4, cc = task & 15;
    hv[i] = make_uint4(0, 0, 0, 0);
    if (r < a.rows) hv[i] = *reinterpret_cast<const uint4*>(a.out + static_cast<int64_t>(r) * a.out_stride +
                                                          static_cast<int64_t>(t) * BM + cc * 8);
  }
#pragma unroll
  for (int i = 0; i < TASKS; ++i) {
    const int task = tid + i * kEpiThreads, r = task >> 4, cc = task & 15;
    const float4 v0 = *reinterpret_cast<const float4*>(tile + r * BM + cc * 8);
    const float4 v1 = *reinterpret_cast<const float4*>(tile + r * BM + cc * 8 + 4);
    const float dv[8] = {v0.x, v0.y, v0.z, v0.w, v1.x, v1.y, v1.z, v1.w};
    uint16_t hb[8], ob[8];
    *reinterpret_cast<uint4*>(hb) = hv[i];
    float ss = 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const float nv = rnd16<T>(__fadd_rn(T::to_f(hb[e]), rnd16<T>(dv[e])));
      ob[e] = to16<T>(nv);
      ss = __fmaf_rn(nv, nv, ss);
    }
#pragma unroll
    for (int o = 8; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    if (r < a.rows) {
      *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(r) * a.out_stride + static_cast<int64_t>(t) * BM +
                                cc * 8) = *reinterpret_cast<const uint4*>(ob);
      if (cc == 0) a.ssq_out[static_cast<int64_t>(t) * kProjMaxRows + r] = ss;
    }
  }
}

// gate/up pair: tile columns [0, 64) are gate rows, [64, 128) the same up
// rows; act[r, t*64 + j] = round(round(silu(round(gate))) * round(up)).
template <class T, int BN>
__device__ __forceinline__ void epi_gated(const Args& a, int t, const float* tile, int tid) {
  constexpr int TASKS = BN * 8 / kEpiThreads;  // (x row, 8-column chunk of the 64) pairs per thread
#pragma unroll
  for (int i = 0; i < TASKS; ++i) {
    const int task = tid + i * kEpiThreads, r = task >> 3, jc = task & 7;
    const int64_t n = static_cast<int64_t>(t) * 64 + jc * 8;
    if (r >= a.rows || n >= a.n_out) continue;
    const float* g = tile + r * BM + jc * 8;
    const float* u = g + 64;
    uint16_t ob[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) ob[e] = silu_mul_elem_fast<T>(rnd16<T>(g[e]), rnd16<T>(u[e]));
    *reinterpret_cast<uint4*>(a.out + static_cast<int64_t>(r) * a.out_stride + n) =
        *reinterpret_cast<const uint4*>(ob);
  }
}

// q/k/v tile (head_dim 128): warp w takes x rows w, w+8, ...; lane l holds
// head dims [4l, 4l+4), whose RoPE partners d +- 64 sit in lane l ^ 16. The
// op order and roundings are those of the separate K/V epilogue kernel
// (kvr_row_ops.cu): round the projection, q/k RMSNorm (fp32 sum of squares,
// round, times weight, round), RoPE with each product and the sum rounded.
template <class T>
__device__ __forceinline__ void epi_qkv_rows(const Args& a, int t, int warp, int lane, const float* tile) {
  constexpr int D = BM, E = 4;
  const bool is_q = t < a.q_tiles;
  const bool is_v = t >= a.q_tiles + a.k_tiles;
  const int head = is_q ? t : (is_v ? t - a.q_tiles - a.k_tiles : t - a.q_tiles);
  const uint16_t* nw = is_q ? a.q_norm : a.k_norm;
  float wv[E] = {0.f, 0.f, 0.f, 0.f};
  if (nw && !is_v) {
#pragma unroll
    for (int e = 0; e < E; ++e) wv[e] = T::to_f(nw[lane * E + e]);
  }
  for (int r = warp; r < a.rows; r += kEpiThreads / 32) {
    const float4 raw = *reinterpret_cast<const float4*>(tile + r * BM + lane * E);
    const int64_t p = a.positions[r];
    if (!is_q && (p < 0 || p >= a.cache_rows)) continue;  // the position check of the plan failed
    uint16_t xb[E] = {to16<T>(raw.x), to16<T>(raw.y), to16<T>(raw.z), to16<T>(raw.w)};
    if (is_v) {  // the rounded projection, bitwise into the cache row
      *reinterpret_cast<uint2*>(a.v_cache + head * a.c_hs + p * a.c_rs + lane * E) =
          *reinterpret_cast<const uint2*>(xb);
      continue;
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
      for (int e = 0; e < E; ++e) x[e] = rnd16<T>(__fmul_rn(wv[e], rnd16<T>(__fmul_rn(x[e], inv))));
    }
    const uint2 cr = *reinterpret_cast<const uint2*>(a.cos_tab + r * D + lane * E);
    const uint2 sr = *reinterpret_cast<const uint2*>(a.sin_tab + r * D + lane * E);
    uint16_t cb[E], sb[E], ob[E];
    *reinterpret_cast<uint2*>(cb) = cr;
    *reinterpret_cast<uint2*>(sb) = sr;
    const bool low = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float partner = __shfl_xor_sync(0xffffffffu, x[e], 16);
      ob[e] = rope_elem_hw<T>(x[e], low ? -partner : partner, T::to_f(cb[e]), T::to_f(sb[e]));
    }
    uint16_t* dst = is_q ? a.q_out + (static_cast<int64_t>(r) * a.q_heads + head) * D
                         : a.k_cache + head * a.c_hs + p * a.c_rs;
    *reinterpret_cast<uint2*>(dst + lane * E) = *reinterpret_cast<const uint2*>(ob);
  }
}

template <class T, int BN, int EPI, bool XNORM>
__global__ void __launch_bounds__(THREADS, 1) proj_kernel(const __grid_constant__ Maps maps, const Args a) {
  using L = Layout<BN>;
  constexpr int NS = L::NS;
  constexpr bool kBF16 = std::is_same<T, BF16>::value;
  extern __shared__ uint8_t smem_raw[];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int b = blockIdx.x;
  const int64_t KC = a.kchunks;

  const uint32_t raw = sm100::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  if (base - raw + L::USED > static_cast<uint32_t>(L::BYTES)) {  // uniform across the grid
    if (tid == 0) atomicCAS(a.status, 0, ERR_SMEM_ALIGN);
    return;
  }
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + L::BAR_OFF;
  auto wfull = [&](int s) { return bar0 + 8u * s; };
  auto xfull = [&](int s) { return bar0 + 8u * (NS + s); };
  auto empty = [&](int s) { return bar0 + 8u * (2 * NS + s); };
  auto xraw = [&](int s) { return bar0 + 8u * (3 * NS + s); };
  auto acc_full = [&](int buf) { return bar0 + 8u * (4 * NS + buf); };
  auto acc_empty = [&](int buf) { return bar0 + 8u * (4 * NS + 2 + buf); };
  const uint32_t drain = bar0 + 8u * (4 * NS + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(gbase + L::MISC_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L::MISC_OFF + 4);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(gbase + L::MISC_OFF + 8);
  int* err = a.status;

  if (tid == 0) {
    *abort = 0;
    for (int s = 0; s < NS; ++s) {
      sm100::mbar_init(wfull(s), 1);
      sm100::mbar_init(xfull(s), kXThreads);
      sm100::mbar_init(xraw(s), 1);
      sm100::mbar_init(empty(s), 1);
    }
    for (int buf = 0; buf < 2; ++buf) {
      sm100::mbar_init(acc_full(buf), 1);
      sm100::mbar_init(acc_empty(buf), kEpiThreads);
    }
    sm100::mbar_init(drain, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  uint32_t tmem = 0;
  if (warp != kTmaWarp) {
    // All but the producer wait here for the previous kernel in the stream (it
    // writes x and what the epilogue reads); TMEM is taken only after that, so
    // no CTA holds it while it waits.
    pdl_wait();
    if (warp == kMmaWarp) {
      sm100::tmem_alloc(sm100::smem_u32(tmem_slot), L::TMEM_COLS);
      sm100::tmem_relinquish();
    }
    sm100::tc_fence_before();
    sm100::bar_sync_named(kTmemBar, THREADS - 32);
    sm100::tc_fence_after();
    tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  }

  int it = 0;  // stages the producer has filled (an aborted CTA drains them)
  if (warp == kTmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      sm100::prefetch_tmap(&maps.x);
      sm100::prefetch_tmap(&maps.w[0]);
      if (EPI != PROJ_RESIDUAL) sm100::prefetch_tmap(&maps.w[1]);
      if (EPI == PROJ_QKV_ROPE) sm100::prefetch_tmap(&maps.w[2]);
      Cursor cur = make_cursor(a, b);
      int t, c0, c1;
      bool ok = true;
      // The first NS stages get their weight tiles before the previous kernel
      // has finished (weights are never written); their x tiles, which that
      // kernel produces, follow once pdl_wait() returns. An x tile to be
      // normalised lands on xraw (the x warps take it from there), one used
      // as loaded on wfull with the weights.
      int pre_c[NS];
      bool waited = false;
      auto load_x = [&](int s, int c) {
        const uint32_t xs = base + s * L::STAGE + W_BYTES;
        if constexpr (XNORM) sm100::mbar_arrive_expect_tx(xraw(s), L::X_BYTES);
#pragma unroll
        for (int j = 0; j < KSUB; ++j)
          sm100::tma_load_2d(xs + j * BN * 128, &maps.x, XNORM ? xraw(s) : wfull(s), c * BK + j * SUBK, 0);
      };
      auto release_x = [&]() {
        pdl_wait();
        const int n = it < NS ? it : NS;
        for (int j = 0; j < n; ++j) load_x(j, pre_c[j]);
        waited = true;
      };
      while (ok && cur.next(t, c0, c1)) {
        int map, row0;
        tile_rows(EPI, a.q_tiles, a.k_tiles, t, map, row0);
        for (int c = c0; c < c1; ++c, ++it) {
          if (!waited && it == NS) release_x();
          const int s = it % NS;
          if (it >= NS && !sm100::mbar_wait(empty(s), ((it / NS) - 1) & 1, abort, err, ERR_EMPTY, a.wait_limit)) {
            ok = false;
            break;
          }
          sm100::mbar_arrive_expect_tx(wfull(s), XNORM ? W_BYTES : L::STAGE);
          const uint32_t ws = base + s * L::STAGE;
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
            const uint32_t wj = ws + j * BM * 128;
            if constexpr (EPI == PROJ_GATED) {
              sm100::tma_load_2d(wj, &maps.w[0], wfull(s), c * BK + j * SUBK, row0);
              sm100::tma_load_2d(wj + 64 * 128, &maps.w[1], wfull(s), c * BK + j * SUBK, row0);
            } else {
              sm100::tma_load_2d(wj, &maps.w[map], wfull(s), c * BK + j * SUBK, row0);
            }
          }
          if (waited) load_x(s, c);
          else pre_c[it] = c;
        }
      }
      if (!waited) release_x();
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- MMA issuer ----------------
      constexpr uint32_t IDESC = sm100::idesc_f16(kBF16, BM, BN, false);
      Cursor cur = make_cursor(a, b);
      int mit = 0, job = 0, t, c0, c1;
      bool ok = true;
      for (; ok && cur.next(t, c0, c1); ++job) {
        const int buf = job & 1;
        if (job >= 2 &&
            !sm100::mbar_wait(acc_empty(buf), ((job >> 1) - 1) & 1, abort, err, ERR_ACC_EMPTY, a.wait_limit))
          break;
        sm100::tc_fence_after();
        for (int c = c0; c < c1; ++c, ++mit) {
          const int s = mit % NS;
          if (!sm100::mbar_wait(wfull(s), (mit / NS) & 1, abort, err, ERR_FULL, a.wait_limit) ||
              (XNORM && !sm100::mbar_wait(xfull(s), (mit / NS) & 1, abort, err, ERR_FULL, a.wait_limit))) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t ws = base + s * L::STAGE;
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
#pragma unroll
            for (int kk = 0; kk < SUBK / 16; ++kk) {
              const uint64_t da = sm100::desc_sw128(ws + j * BM * 128 + kk * 32, 16, 1024);
              const uint64_t db = sm100::desc_sw128(ws + W_BYTES + j * BN * 128 + kk * 32, 16, 1024);
              sm100::mma_f16_ss(tmem + buf * BN, da, db, IDESC, (c > c0 || j > 0 || kk > 0) ? 1u : 0u);
            }
          }
          sm100::mma_commit(empty(s));
        }
        if (!ok) break;
        sm100::mma_commit(acc_full(buf));
      }
      // Nothing of ours may still be writing TMEM when it is freed.
      sm100::mma_commit(drain);
      volatile int keep_waiting = 0;
      sm100::mbar_wait(drain, 0, &keep_waiting, err, ERR_DRAIN, WAIT_LIMIT);
    }
  } else if (warp >= kXWarp0) {
    if constexpr (XNORM) {
      // ---------------- x producer: RMSNorm(h) stages ----------------
      // The TMA producer brings the raw h tile of every stage (xraw); these
      // warps normalise it in place, 16 bytes at a time, and release it to
      // the MMA (xfull).
      const int xt = tid - kXWarp0 * 32;
      float* inv = reinterpret_cast<float*>(gbase + L::INV_OFF);
      for (int r = xt; r < BN; r += kXThreads) {
        float v = 0.f;
        if (r < a.rows) {
          // Tile sums in tile order, eight loads in flight at a time.
          float s = 0.f;
          for (int t0 = 0; t0 < a.ssq_tiles; t0 += 8) {
            float part[8];
#pragma unroll
            for (int i = 0; i < 8; ++i)
              part[i] = t0 + i < a.ssq_tiles ? __ldcg(a.ssq_in + static_cast<int64_t>(t0 + i) * kProjMaxRows + r) : 0.f;
#pragma unroll
            for (int i = 0; i < 8; ++i)
              if (t0 + i < a.ssq_tiles) s += part[i];
          }
          v = rsqrtf(__fadd_rn(s * a.inv_k, a.eps));
        }
        inv[r] = v;
      }
      sm100::bar_sync_named(kXBar, kXThreads);
      const int cc = xt & 7;   // 16-byte chunk of the 64-column stage
      const int rb = xt >> 3;  // rows rb, rb + 8, ...
      constexpr int RPT = BN / 8;
      float rinv[RPT];
#pragma unroll
      for (int i = 0; i < RPT; ++i) rinv[i] = inv[rb + 8 * i];
      Cursor cur = make_cursor(a, b);
      int xit = 0, t, c0, c1;
      bool ok = true;
      while (ok && cur.next(t, c0, c1)) {
        for (int c = c0; c < c1; ++c, ++xit) {
          const int s = xit % NS;
          if (!sm100::mbar_wait(xraw(s), (xit / NS) & 1, abort, err, ERR_FULL, a.wait_limit)) {
            ok = false;
            break;
          }
#pragma unroll
          for (int j = 0; j < KSUB; ++j) {
          const int64_t col = static_cast<int64_t>(c) * BK + j * SUBK + cc * 8;
          const bool in = col < a.k;  // k is a multiple of 8: whole chunks are in or out
          uint4 w4 = make_uint4(0, 0, 0, 0);
          if (in) w4 = *reinterpret_cast<const uint4*>(a.norm_w + col);
          const uint32_t wpk[4] = {w4.x, w4.y, w4.z, w4.w};
          uint8_t* xs = gbase + s * L::STAGE + W_BYTES + j * BN * 128;
#pragma unroll
          for (int i = 0; i < RPT; ++i) {
            uint4* slot = reinterpret_cast<uint4*>(xs + swz(rb + 8 * i, cc));
            const uint4 xv = *slot;
            const uint32_t xpk[4] = {xv.x, xv.y, xv.z, xv.w};
            uint32_t ypk[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              // round(w * round(x * inv)), two elements per conversion
              const float2 xf = unpack2<T>(xpk[e]);
              const float2 nf = unpack2<T>(cvt2<T>(__fmul_rn(xf.x, rinv[i]), __fmul_rn(xf.y, rinv[i])));
              const float2 wf = unpack2<T>(wpk[e]);
              ypk[e] = cvt2<T>(__fmul_rn(wf.x, nf.x), __fmul_rn(wf.y, nf.y));
            }
            *slot = make_uint4(ypk[0], ypk[1], ypk[2], ypk[3]);
          }
          }
          sm100::fence_proxy_async_smem();  // generic-proxy stores -> read by the MMA
          sm100::mbar_arrive(xfull(s));
        }
      }
    }
  } else {
    // ---------------- epilogue ----------------
    // Each finished tile goes TMEM -> shared memory (fp32 [x row][weight row])
    // and is then processed row-wise with 16-byte global accesses. A tile cut
    // by a range boundary is first written to this CTA's partial slot (the same
    // layout) and, by its last contributor, summed over its contributors in
    // CTA order back into shared memory.
    const int wg = warp >> 2;                // warpgroup: x-row chunks q with q % 2 == wg
    const int row = (warp & 3) * 32 + lane;  // TMEM lane = weight row of the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    float* tile = reinterpret_cast<float*>(gbase + L::TILE_OFF);
    constexpr int F4 = BN * BM / 4;            // float4s in a tile
    constexpr int F4T = F4 / kEpiThreads;      // per thread
    const int qn = (a.rows + 31) / 32;
    Cursor cur = make_cursor(a, b);
    int job = 0, t, c0, c1;
    auto finish = [&]() {
      sm100::bar_sync_named(kAllEpi, kEpiThreads);  // the tile is complete in shared memory
      if constexpr (EPI == PROJ_RESIDUAL) epi_residual<T, BN>(a, t, tile, tid);
      else if constexpr (EPI == PROJ_GATED) epi_gated<T, BN>(a, t, tile, tid);
      else epi_qkv_rows<T>(a, t, warp, lane, tile);
      sm100::bar_sync_named(kAllEpi, kEpiThreads);  // before the next tile reuses it
    };
    for (; cur.next(t, c0, c1); ++job) {
      const int buf = job & 1;
      // One decision for all eight warps (they meet at named barriers below).
      const bool ready = sm100::mbar_wait(acc_full(buf), (job >> 1) & 1, abort, err, ERR_ACC_FULL, a.wait_limit);
      if (!sm100::bar_and_named(kAllEpi, kEpiThreads, ready)) break;
      sm100::tc_fence_after();
      const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(buf * BN);
      for (int q = wg; q < qn; q += 2) {
        uint32_t r[32];
        sm100::tmem_ld32(acc + q * 32, r);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) tile[(q * 32 + e) * BM + row] = __uint_as_float(r[e]);
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(acc_empty(buf));  // the accumulator is free for the job after next
      if (c0 == 0 && c1 == KC) {  // whole tile in this CTA
        finish();
        continue;
      }
      // Part of a tile: slot 0 for the range's first job, 1 for its last (a
      // range inside one tile has one job).
      sm100::bar_sync_named(kAllEpi, kEpiThreads);
      const int slot = job == 0 ? 0 : 1;
      float4* part = reinterpret_cast<float4*>(a.partials + (static_cast<int64_t>(b) * 2 + slot) * BN * BM);
      const float4* tile4 = reinterpret_cast<const float4*>(tile);
#pragma unroll
      for (int i = 0; i < F4T; ++i) __stcg(part + tid + i * kEpiThreads, tile4[tid + i * kEpiThreads]);
      __threadfence();  // this thread's partial stores before the count below
      sm100::bar_sync_named(kAllEpi, kEpiThreads);
      const int64_t t_first_unit = static_cast<int64_t>(t) * KC;
      const int b_first = owner(a.units, a.grid, t_first_unit);
      const int b_last = owner(a.units, a.grid, t_first_unit + KC - 1);
      if (tid == 0) {
        const int old = atomicAdd(a.counters + t, 1);
        const int last = old == b_last - b_first;
        if (last) a.counters[t] = 0;  // every contributor has arrived: reset for the next launch
        __threadfence();
        *fix_flag = last;
      }
      sm100::bar_sync_named(kAllEpi, kEpiThreads);
      // fix_flag is next written after the barriers of the next partial tile,
      // which every thread reaches only after this read.
      if (*fix_flag == 0) continue;
      // Fix-up: the contributors' partials summed in CTA order (independent
      // of the arrival order); eight float4s per thread at a time, two
      // contributors' loads in flight.
#pragma unroll
      for (int i0 = 0; i0 < F4T; i0 += 8) {
        float4 sum[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sum[i] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int b0 = b_first; b0 <= b_last; b0 += 2) {
          float4 pv[2][8];
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            const int bb = b0 + k;
            if (bb <= b_last) {
              const int sl = range_begin(a.units, a.grid, bb) >= t_first_unit ? 0 : 1;
              const float4* src =
                  reinterpret_cast<const float4*>(a.partials + (static_cast<int64_t>(bb) * 2 + sl) * BN * BM);
#pragma unroll
              for (int i = 0; i < 8; ++i) pv[k][i] = __ldcg(src + tid + (i0 + i) * kEpiThreads);
            }
          }
#pragma unroll
          for (int k = 0; k < 2; ++k) {
            if (b0 + k <= b_last) {
#pragma unroll
              for (int i = 0; i < 8; ++i) {
                sum[i].x += pv[k][i].x;
                sum[i].y += pv[k][i].y;
                sum[i].z += pv[k][i].z;
                sum[i].w += pv[k][i].w;
              }
            }
          }
        }
#pragma unroll
        for (int i = 0; i < 8; ++i) reinterpret_cast<float4*>(tile)[tid + (i0 + i) * kEpiThreads] = sum[i];
      }
      finish();
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  // Every role has stopped; `abort` is final. After an abort, consumers may
  // have left stages unread: never leave the CTA while one of our copies may
  // still land in shared memory. (Without an abort every stage was waited for.)
  if (*abort && warp == kTmaWarp && lane == 0) {
    volatile int keep_waiting = 0;
    for (int j = it > NS ? it - NS : 0; j < it; ++j) {
      sm100::mbar_wait(wfull(j % NS), (j / NS) & 1, &keep_waiting, nullptr, 0, WAIT_LIMIT);
      if (XNORM) sm100::mbar_wait(xraw(j % NS), (j / NS) & 1, &keep_waiting, nullptr, 0, WAIT_LIMIT);
    }
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ------------------------------------------------------------------ host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

EncodeFn encode_fn() {
  static EncodeFn fn = nullptr;
  if (!fn) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeFn>(p);
  }
  return fn;
}

// Row-major [rows][k] (row stride `stride` elements), box 64 x box_rows, 128B swizzle.
bool make_map(CUtensorMap* map, const void* ptr, bool bf16, int64_t k, int64_t rows, int64_t stride, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
  cuuint32_t box[2] = {SUBK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int pick_bn(int64_t rows) { return rows <= 64 ? 64 : 128; }

size_t partial_bytes(int bn) { return static_cast<size_t>(kNumSMs) * 2 * bn * BM * sizeof(float); }

template <class T, int BN, int EPI, bool XNORM>
int launch(const Maps& maps, const Args& a, cudaStream_t s) {
  using L = Layout<BN>;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    e = cudaFuncSetAttribute(proj_kernel<T, BN, EPI, XNORM>, cudaFuncAttributeMaxDynamicSharedMemorySize, L::BYTES);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  return launch_pdl<proj_kernel<T, BN, EPI, XNORM>>(dim3(static_cast<unsigned>(a.grid)), dim3(THREADS), L::BYTES, s,
                                                     1, maps, a);
}

template <class T, int BN>
int launch_epi(const Maps& maps, const Args& a, int epi, bool xnorm, cudaStream_t s) {
  switch (epi) {
    case PROJ_RESIDUAL: return launch<T, BN, PROJ_RESIDUAL, false>(maps, a, s);
    case PROJ_GATED: return xnorm ? launch<T, BN, PROJ_GATED, true>(maps, a, s) : launch<T, BN, PROJ_GATED, false>(maps, a, s);
    default:
      return xnorm ? launch<T, BN, PROJ_QKV_ROPE, true>(maps, a, s) : launch<T, BN, PROJ_QKV_ROPE, false>(maps, a, s);
  }
}

}  // namespace proj

int64_t proj_tiles(const ProjParams& p) {
  switch (p.epilogue) {
    case PROJ_RESIDUAL: return (p.n_w[0] + proj::BM - 1) / proj::BM;
    case PROJ_GATED: return (p.n_w[0] + 63) / 64;
    case PROJ_QKV_ROPE: return static_cast<int64_t>(p.q_heads) + 2 * p.kv_heads;
    default: return 0;
  }
}

size_t proj_workspace_bytes(int64_t rows, int64_t tiles) {
  return proj_zero_bytes(tiles) + proj::partial_bytes(proj::pick_bn(rows));
}

int proj_forward(const ProjParams& p, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  using namespace proj;
  if (p.dtype != KVR_DTYPE_BF16 && p.dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (p.rows <= 0 || p.rows > kProjMaxRows || p.k <= 0 || p.k % 8 || p.k > 0x7fffffffLL) return KVR_ERR_INVALID_ARG;
  const bool xnorm = p.norm_w != nullptr;
  if (xnorm) {
    if (p.epilogue == PROJ_RESIDUAL || !p.x || !p.ssq_in || p.ssq_tiles <= 0 || !aligned16(p.x) || !aligned16(p.norm_w) ||
        p.x_stride < p.k || p.x_stride % 8)
      return KVR_ERR_INVALID_ARG;
  } else if (!p.x || !aligned16(p.x) || p.x_stride < p.k || p.x_stride % 8) {
    return KVR_ERR_INVALID_ARG;
  }
  const int64_t tiles = proj_tiles(p);
  if (tiles <= 0) return KVR_ERR_INVALID_ARG;
  const int nmaps = p.epilogue == PROJ_QKV_ROPE ? 3 : (p.epilogue == PROJ_GATED ? 2 : 1);
  for (int i = 0; i < nmaps; ++i) {
    const bool needed = !(p.epilogue == PROJ_QKV_ROPE && i == 0 && p.q_heads == 0);
    if (needed && (!p.w[i] || !aligned16(p.w[i]) || p.n_w[i] <= 0)) return KVR_ERR_INVALID_ARG;
  }
  if (p.epilogue == PROJ_QKV_ROPE) {
    if (p.kv_heads <= 0 || p.q_heads < 0 || (p.q_heads > 0 && (!p.q_out || p.n_w[0] != p.q_heads * 128LL)) ||
        p.n_w[1] != p.kv_heads * 128LL || p.n_w[2] != p.kv_heads * 128LL || !p.k_cache || !p.v_cache ||
        !p.positions || !p.cos_tab || !p.sin_tab || p.cache_rows <= 0 || (p.q_norm == nullptr) != (p.k_norm == nullptr))
      return KVR_ERR_INVALID_ARG;
  } else {
    if (!p.out || !aligned16(p.out) || p.out_stride < p.n_w[0] || p.out_stride % 8 || p.n_w[0] % 8)
      return KVR_ERR_INVALID_ARG;
    if (p.epilogue == PROJ_RESIDUAL && (!p.ssq_out || p.n_w[0] % BM)) return KVR_ERR_INVALID_ARG;
    if (p.epilogue == PROJ_GATED && (!p.w[1] || p.n_w[1] != p.n_w[0])) return KVR_ERR_INVALID_ARG;
  }
  const int bn = pick_bn(p.rows);
  const size_t need = proj_workspace_bytes(p.rows, tiles);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return KVR_ERR_INVALID_ARG;
  const bool bf16 = p.dtype == KVR_DTYPE_BF16;

  Maps maps;
  memset(&maps, 0, sizeof(maps));
  const int box = p.epilogue == PROJ_GATED ? 64 : BM;
  for (int i = 0; i < nmaps; ++i) {
    const void* w = p.w[i] ? p.w[i] : p.w[1];  // a k/v-only launch never reads map 0
    const int64_t n = p.w[i] ? p.n_w[i] : p.n_w[1];
    if (!make_map(&maps.w[i], w, bf16, p.k, n, p.k, box)) return KVR_ERR_UNSUPPORTED;
  }
  for (int i = nmaps; i < 3; ++i) maps.w[i] = maps.w[0];
  if (!make_map(&maps.x, p.x, bf16, p.k, p.rows, p.x_stride, bn)) return KVR_ERR_UNSUPPORTED;

  Args a{};
  a.rows = static_cast<int>(p.rows);
  a.k = p.k;
  a.kchunks = static_cast<int>((p.k + BK - 1) / BK);
  a.tiles = static_cast<int>(tiles);
  a.units = tiles * a.kchunks;
  a.grid = static_cast<int>(a.units < kNumSMs ? a.units : kNumSMs);
  a.q_tiles = p.epilogue == PROJ_QKV_ROPE ? p.q_heads : 0;
  a.k_tiles = p.epilogue == PROJ_QKV_ROPE ? p.kv_heads : 0;
  a.n_out = p.n_w[0];
  a.out = static_cast<uint16_t*>(p.out);
  a.out_stride = p.out_stride;
  a.ssq_out = p.ssq_out;
  a.x = static_cast<const uint16_t*>(p.x);
  a.x_stride = p.x_stride;
  a.norm_w = static_cast<const uint16_t*>(p.norm_w);
  a.ssq_in = p.ssq_in;
  a.ssq_tiles = p.ssq_tiles;
  a.inv_k = 1.0f / static_cast<float>(p.k);
  a.eps = p.eps;
  a.q_heads = p.q_heads;
  a.q_out = static_cast<uint16_t*>(p.q_out);
  a.k_cache = static_cast<uint16_t*>(p.k_cache);
  a.v_cache = static_cast<uint16_t*>(p.v_cache);
  a.cache_rows = p.cache_rows;
  a.c_hs = p.c_hs;
  a.c_rs = p.c_rs;
  a.positions = p.positions;
  a.cos_tab = static_cast<const uint16_t*>(p.cos_tab);
  a.sin_tab = static_cast<const uint16_t*>(p.sin_tab);
  a.q_norm = static_cast<const uint16_t*>(p.q_norm);
  a.k_norm = static_cast<const uint16_t*>(p.k_norm);
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.status = reinterpret_cast<int*>(ws);
  a.counters = reinterpret_cast<int*>(ws + STATUS_BYTES);
  // Partials at the end of the workspace: the same place for every launch
  // that shares it, whatever its own tile count (the counters of a launch
  // with more tiles lie below them and stay zero).
  a.partials = reinterpret_cast<float*>(ws + ((workspace_bytes - partial_bytes(bn)) & ~static_cast<size_t>(255)));
  a.wait_limit = pipeline_wait_limit();
  if (bn == 64)
    return bf16 ? launch_epi<BF16, 64>(maps, a, p.epilogue, xnorm, stream)
                : launch_epi<F16, 64>(maps, a, p.epilogue, xnorm, stream);
  return bf16 ? launch_epi<BF16, 128>(maps, a, p.epilogue, xnorm, stream)
              : launch_epi<F16, 128>(maps, a, p.epilogue, xnorm, stream);
}

}  // namespace kvr
