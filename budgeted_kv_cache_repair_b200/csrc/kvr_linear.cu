// Projections of the selected rows on sm_100a tensor cores (tcgen05 + TMEM +
// TMA): out = x . W^T for nn.Linear weights W [n, k].
//
// A refresh pushes a few dozen rows through each projection, so every weight
// byte is read once and used by at most 256 rows: the work is a weight stream
// and its roofline is HBM bandwidth over n*k*2 bytes. The kernel
//   * puts the weight rows on the MMA M side: a tile is 128 weight rows, the
//     MMA is D[128 x BN] += W[128 x 64] . X[BN x 64]^T with the (<= 256) rows
//     of x as N, accumulated in TMEM (two accumulators, so the epilogue of one
//     tile overlaps the next tile's MMAs);
//   * feeds both operands by TMA into a ring of 128B-swizzled stages (no
//     multicast); x is tiny and stays in L2 across CTAs;
//   * takes up to four weight matrices that share x in one launch (q/k/v), and
//     fuses the gated MLP: a "paired" tile holds 64 rows of W_gate and the same
//     64 rows of W_up, and its epilogue writes silu(gate) * up directly.
//
// Work is spread over the 148 SMs in one of two ways, so that every SM streams
// about the same number of weight bytes and the end of the kernel carries no
// slow reduction:
//   * fewer tiles than SMs (q/k/v, o, down of an 8B model): split-K inside a
//     thread-block cluster. The S CTAs of a cluster (S <= 8, chosen so the
//     whole grid is resident) share one tile, each a contiguous k range; each
//     leaves its fp32 partial in its own shared memory, and after a cluster
//     barrier pushes every peer's slice of x rows into that peer's shared
//     memory with one bulk copy; CTA r then sums its slice over the S partials
//     (in rank order) and writes the output;
//   * at least as many tiles as SMs (the gated MLP): a persistent grid of one
//     CTA per SM. The tiles beyond the last whole wave are cut into (tile,
//     64-wide k-chunk) units and dealt out stream-K first, as one contiguous
//     range per CTA; then each CTA streams whole tiles. A tile cut by a range
//     boundary is finished by fix-up: its contributors store fp32 partials to
//     the workspace and the last one to arrive (tile counter) sums them in CTA
//     order, while its own producer and MMA warps already stream the next
//     whole tile. Counters are zero on entry and left zero on exit.
// Both ways fix the summation order: results do not depend on timing.
//
// Warp roles (320 threads): warps 0-7 epilogue in two warpgroups (warp w reads
// TMEM lanes 32*(w%4).., i.e. weight rows; warpgroup w/4 takes every other
// 32-row chunk of x), warp 8 TMA producer, warp 9 MMA issuer. Every mbarrier
// wait is bounded: on timeout the kernel records an error code in the status
// word, stops issuing, drains its own TMA and MMA work, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <type_traits>

#include "kvr_common.cuh"
#include "kvr_linear.h"
#include "kvr_sm100.cuh"

namespace kvr {
namespace lin {

constexpr int BM = 128;             // weight rows per tile (MMA M, TMEM lanes)
constexpr int BK = 64;              // k elements per stage: one 128-byte swizzle row
constexpr int W_BYTES = BM * 128;   // weight tile of one stage
constexpr int kEpiWarps = 8;
constexpr int kEpiThreads = 256;
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int THREADS = 320;
constexpr int kMaxSplit = 8;        // portable cluster size
constexpr int MAX_SEGS = KVR_LINEAR_MAX_SEGMENTS;
constexpr int STATUS_BYTES = 256;
constexpr long long WAIT_LIMIT = kDefaultWaitLimit;  // drains of the CTA's own copies and MMAs
// Named barriers: 1 + warpgroup (128 threads each), kAllEpi (all 256 epilogue
// threads), kTmemBar (every warp but the producer, after TMEM allocation).
constexpr int kAllEpi = 3;
constexpr int kTmemBar = 4;

enum Err : int { ERR_EMPTY = 1, ERR_FULL, ERR_ACC_EMPTY, ERR_ACC_FULL, ERR_DRAIN, ERR_SMEM_ALIGN, ERR_REDUCE };

template <int BN>
struct Layout {
  static constexpr int X_BYTES = BN * 128;
  static constexpr int STAGE = W_BYTES + X_BYTES;
  static constexpr int NS = BN <= 64 ? 8 : (BN == 128 ? 6 : 4);  // 160-192 KB of ring
  // gate/up exchange of a paired tile, per warpgroup: [64 rows][34] 16-bit
  // values of the gate half, then of the up half (stride 34: no bank conflicts)
  static constexpr int XCH_STRIDE = 34;
  static constexpr int XCH_WG = 2 * 64 * XCH_STRIDE * 2;
  static constexpr int XCH_OFF = NS * STAGE;
  static constexpr int BAR_OFF = XCH_OFF + 2 * XCH_WG;
  // full[NS], empty[NS], acc_full[2], acc_empty[2], drain, red_full
  static constexpr int NBAR = 2 * NS + 6;
  static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;  // abort flag, TMEM address, fix-up flag
  static constexpr int USED = MISC_OFF + 16;
  static constexpr int BYTES = USED + 1024 <= 232448 ? USED + 1024 : 232448;
  static constexpr uint32_t STAGE_TX = STAGE;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // two accumulators; BN >= 32 keeps it a power of two >= 64
  static_assert(USED <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
  static_assert(STAGE % 1024 == 0 && W_BYTES % 1024 == 0, "swizzled tiles need 1 KB alignment");
  // Split-K: the fp32 partial [BN x rows][128] at the ring's start, then the
  // receive area for the peers' slices of this CTA's rows.
  static constexpr int PART_BYTES = BN * BM * 4;
  static constexpr int RING_BYTES = NS * STAGE;
  static_assert(PART_BYTES <= RING_BYTES, "split-K partial must fit in the ring");
};

struct Segment {
  uint16_t* out;
  int64_t out_stride;
  float* part;  // deferred mode: this segment's fp32 partial buffer (slice 0, row 0, column 0)
  int64_t n;
  int tile_begin;  // first global tile of this segment
  int paired;      // 64 rows of gate + 64 rows of up per tile; out = silu(gate) * up
};

struct Args {
  Segment seg[MAX_SEGS];
  int nseg;
  int rows;      // rows of x in this launch (<= BN)
  int kchunks;   // ceil(k / 64)
  int tiles;
  int split;     // > 0: split-K mode, CTAs (cluster size) per tile; 0: persistent stream-K mode
  int grid;      // stream-K mode: persistent CTAs
  int dp_tiles;  // stream-K mode: tiles [0, dp_tiles) are streamed whole, after the stream-K part
  int sk_grid;   // stream-K mode: CTAs that share the stream-K part (<= grid, <= sk_units)
  int64_t sk_units;  // stream-K mode: (tiles - dp_tiles) * kchunks
  int64_t part_stride, part_slice;  // deferred mode (part_slice > 0): partial layout, floats
  int* status;
  int* counters;    // [tiles - dp_tiles]
  float* partials;  // [sk_grid][2 slots][BN / 4][128][4]
  long long wait_limit;  // SM clocks before a pipeline wait gives up
};

struct Maps {
  CUtensorMap x;
  CUtensorMap w[2 * MAX_SEGS];  // weight, weight_up per segment
};

__device__ __forceinline__ Segment seg_at(const Args& a, int i) {
  switch (i) {
    case 0: return a.seg[0];
    case 1: return a.seg[1];
    case 2: return a.seg[2];
    default: return a.seg[3];
  }
}

__device__ __forceinline__ int seg_index(const Args& a, int tile) {
  int si = 0;
#pragma unroll
  for (int i = 1; i < MAX_SEGS; ++i)
    if (i < a.nseg && tile >= a.seg[i].tile_begin) si = i;
  return si;
}

// First stream-K unit of CTA b and the CTA that owns unit u (inverse of the
// split; every CTA below sk_grid owns at least one unit).
__device__ __forceinline__ int64_t range_begin(int64_t units, int grid, int b) {
  return units * b / grid;
}
__device__ __forceinline__ int owner(int64_t units, int grid, int64_t u) {
  return static_cast<int>(((u + 1) * grid + units - 1) / units - 1);
}

// The jobs of one CTA, in the order all three roles walk them: a (tile, k
// range) run of stream-K units first, then whole tiles.
struct Cursor {
  int64_t u, u_end, kc;
  int tile_off;
  int dp, dp_step, dp_end;

  __device__ __forceinline__ bool next(int& t, int& c0, int& c1) {
    if (u < u_end) {
      const int64_t tt = u / kc;
      c0 = static_cast<int>(u - tt * kc);
      c1 = static_cast<int>(kc < c0 + (u_end - u) ? kc : c0 + (u_end - u));
      u += c1 - c0;
      t = tile_off + static_cast<int>(tt);
      return true;
    }
    if (dp < dp_end) {
      t = dp;
      c0 = 0;
      c1 = static_cast<int>(kc);
      dp += dp_step;
      return true;
    }
    return false;
  }
};

__device__ __forceinline__ Cursor make_cursor(const Args& a, int b) {
  Cursor c;
  c.kc = a.kchunks;
  if (a.split > 0) {  // one tile, k range r of `split`
    const int t = b / a.split, r = b % a.split;
    c.u = static_cast<int64_t>(t) * c.kc + c.kc * r / a.split;
    c.u_end = static_cast<int64_t>(t) * c.kc + c.kc * (r + 1) / a.split;
    c.tile_off = 0;
    c.dp = c.dp_end = 0;
    c.dp_step = 1;
  } else {
    const bool sk = b < a.sk_grid;
    c.u = sk ? range_begin(a.sk_units, a.sk_grid, b) : 0;
    c.u_end = sk ? range_begin(a.sk_units, a.sk_grid, b + 1) : 0;
    c.tile_off = a.dp_tiles;
    c.dp = b;
    c.dp_step = a.grid;
    c.dp_end = a.dp_tiles;
  }
  return c;
}

// One 32-column chunk (x rows q*32 .. q*32+31) of this thread's weight row
// `row`: round and store, or, for a paired tile, exchange with the other half
// through shared memory and store silu(gate) * up (the gate threads take
// columns 0-15 of the pair, the up threads 16-31). The 128 threads of the
// warpgroup call it together.
template <class T>
__device__ __forceinline__ void finalize(const Args& a, const Segment& sg, int local_tile, int q, const float (&v)[32],
                                         uint16_t* xch, int row, int wg) {
  const int r0 = q * 32;
  if (!sg.paired) {
    const int64_t n = static_cast<int64_t>(local_tile) * BM + row;
    if (n < sg.n) {
      uint16_t* dst = sg.out + n;
#pragma unroll
      for (int e = 0; e < 32; ++e)
        if (r0 + e < a.rows) dst[static_cast<int64_t>(r0 + e) * sg.out_stride] = T::from_f(v[e]);
    }
    return;
  }
  constexpr int XS = 34;
  const int j = row & 63, half = row >> 6;  // half 0: gate row j, half 1: up row j
  uint16_t* mine = xch + (half * 64 + j) * XS;
#pragma unroll
  for (int e = 0; e < 32; ++e) mine[e] = T::from_f(v[e]);
  sm100::bar_sync_named(1 + wg, 128);
  const int64_t n = static_cast<int64_t>(local_tile) * 64 + j;
  if (n < sg.n) {
    const uint16_t* g = xch + j * XS;
    const uint16_t* u = xch + (64 + j) * XS;
    uint16_t* dst = sg.out + n;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e = half * 16 + i;
      if (r0 + e < a.rows)
        dst[static_cast<int64_t>(r0 + e) * sg.out_stride] = silu_mul_elem_fast<T>(T::to_f(g[e]), T::to_f(u[e]));
    }
  }
  sm100::bar_sync_named(1 + wg, 128);
}

template <class T, int BN>
__global__ void __launch_bounds__(THREADS, 1) linear_kernel(const __grid_constant__ Maps maps, const Args a) {
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
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (NS + s); };
  auto acc_full = [&](int buf) { return bar0 + 8u * (2 * NS + buf); };
  auto acc_empty = [&](int buf) { return bar0 + 8u * (2 * NS + 2 + buf); };
  const uint32_t drain = bar0 + 8u * (2 * NS + 4);
  const uint32_t red_full = bar0 + 8u * (2 * NS + 5);
  volatile int* abort = reinterpret_cast<volatile int*>(gbase + L::MISC_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L::MISC_OFF + 4);
  volatile int* fix_flag = reinterpret_cast<volatile int*>(gbase + L::MISC_OFF + 8);
  int* err = a.status;

  if (tid == 0) {
    *abort = 0;
    for (int s = 0; s < NS; ++s) {
      sm100::mbar_init(full(s), 1);
      sm100::mbar_init(empty(s), 1);
    }
    for (int buf = 0; buf < 2; ++buf) {
      sm100::mbar_init(acc_full(buf), 1);
      sm100::mbar_init(acc_empty(buf), kEpiThreads);
    }
    sm100::mbar_init(drain, 1);
    sm100::mbar_init(red_full, 1);
    sm100::fence_barrier_init();
  }
  __syncthreads();
  pdl_launch_dependents();
  uint32_t tmem = 0;
  if (warp != kTmaWarp) {
    // All but the producer wait here for the previous kernel in the stream
    // (its outputs are x, and it may still read what this kernel writes).
    // TMEM is taken only after that, so no CTA holds it while it waits.
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

  // Stages this CTA's producer has filled (each with its weight and x tiles
  // issued): an aborted CTA waits for them to land before it exits.
  int it = 0;
  if (warp == kTmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      sm100::prefetch_tmap(&maps.x);
      for (int i = 0; i < a.nseg; ++i) {
        sm100::prefetch_tmap(&maps.w[2 * i]);
        if (seg_at(a, i).paired) sm100::prefetch_tmap(&maps.w[2 * i + 1]);
      }
      Cursor cur = make_cursor(a, b);
      int t, c0, c1;
      bool ok = true;
      // The first NS stages get their weight tiles before the previous kernel
      // has finished (weights are never written); their x tiles, which that
      // kernel produces, follow once pdl_wait() returns.
      int pre_c[NS];
      bool waited = false;
      auto release_x = [&]() {
        pdl_wait();
        const int n = it < NS ? it : NS;
        for (int j = 0; j < n; ++j)
          sm100::tma_load_2d(base + j * L::STAGE + W_BYTES, &maps.x, full(j), pre_c[j] * BK, 0);
        waited = true;
      };
      while (ok && cur.next(t, c0, c1)) {
        const int si = seg_index(a, t);
        const Segment sg = seg_at(a, si);
        const int lt = t - sg.tile_begin;
        for (int c = c0; c < c1; ++c, ++it) {
          if (!waited && it == NS) release_x();
          const int s = it % NS;
          if (it >= NS && !sm100::mbar_wait(empty(s), ((it / NS) - 1) & 1, abort, err, ERR_EMPTY, a.wait_limit)) {
            ok = false;
            break;
          }
          sm100::mbar_arrive_expect_tx(full(s), L::STAGE_TX);
          const uint32_t ws = base + s * L::STAGE;
          if (sg.paired) {
            sm100::tma_load_2d(ws, &maps.w[2 * si], full(s), c * BK, lt * 64);
            sm100::tma_load_2d(ws + W_BYTES / 2, &maps.w[2 * si + 1], full(s), c * BK, lt * 64);
          } else {
            sm100::tma_load_2d(ws, &maps.w[2 * si], full(s), c * BK, lt * BM);
          }
          if (waited) sm100::tma_load_2d(ws + W_BYTES, &maps.x, full(s), c * BK, 0);
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
      int it = 0, job = 0, t, c0, c1;
      bool ok = true;
      for (; ok && cur.next(t, c0, c1); ++job) {
        const int buf = job & 1;
        if (job >= 2 &&
            !sm100::mbar_wait(acc_empty(buf), ((job >> 1) - 1) & 1, abort, err, ERR_ACC_EMPTY, a.wait_limit))
          break;
        sm100::tc_fence_after();
        for (int c = c0; c < c1; ++c, ++it) {
          const int s = it % NS;
          if (!sm100::mbar_wait(full(s), (it / NS) & 1, abort, err, ERR_FULL, a.wait_limit)) {
            ok = false;
            break;
          }
          sm100::tc_fence_after();
          const uint32_t ws = base + s * L::STAGE;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t da = sm100::desc_sw128(ws + kk * 32, 16, 1024);
            const uint64_t db = sm100::desc_sw128(ws + W_BYTES + kk * 32, 16, 1024);
            sm100::mma_f16_ss(tmem + buf * BN, da, db, IDESC, (c > c0 || kk > 0) ? 1u : 0u);
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
  } else {
    // ---------------- epilogue ----------------
    const int wg = warp >> 2;                    // warpgroup: x-row chunks q with q % 2 == wg
    const int row = (warp & 3) * 32 + lane;      // TMEM lane = weight row of the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    uint16_t* xch = reinterpret_cast<uint16_t*>(gbase + L::XCH_OFF + wg * L::XCH_WG);
    const int qn = (a.rows + 31) / 32;
    const int first_sk_tile = a.split == 0 && b < a.sk_grid
                                  ? a.dp_tiles + static_cast<int>(range_begin(a.sk_units, a.sk_grid, b) / KC)
                                  : -1;
    Cursor cur = make_cursor(a, b);
    int job = 0, t, c0, c1;
    for (; cur.next(t, c0, c1); ++job) {
      const int buf = job & 1;
      // One decision for all eight warps (they meet at named barriers below).
      const bool ready = sm100::mbar_wait(acc_full(buf), (job >> 1) & 1, abort, err, ERR_ACC_FULL, a.wait_limit);
      if (!sm100::bar_and_named(kAllEpi, kEpiThreads, ready)) break;
      sm100::tc_fence_after();
      const Segment sg = seg_at(a, seg_index(a, t));
      const int lt = t - sg.tile_begin;
      const uint32_t acc = tmem + lane_base + static_cast<uint32_t>(buf * BN);
      if (a.part_slice) {
        // Deferred reduction: this CTA's fp32 partial (k range b % split) of
        // weight row n for every x row; the consumer sums the slices.
        const int64_t n = static_cast<int64_t>(lt) * BM + row;
        float* dst = sg.part + (b % a.split) * a.part_slice + n;
        for (int q = wg; q < qn; q += 2) {
          uint32_t r[32];
          sm100::tmem_ld32(acc + q * 32, r);
          sm100::tmem_wait_ld();
          if (n < sg.n) {
#pragma unroll
            for (int e = 0; e < 32; ++e)
              if (q * 32 + e < a.rows) dst[static_cast<int64_t>(q * 32 + e) * a.part_stride] = __uint_as_float(r[e]);
          }
        }
        sm100::tc_fence_before();
        sm100::mbar_arrive(acc_empty(buf));
        continue;
      }
      if (a.split > 1) {
        // Split-K: the fp32 partial goes to this CTA's ring ([x row][weight
        // row]), free now that every MMA has read its stage; the cluster sums
        // the partials after the loop.
        float* part = reinterpret_cast<float*>(gbase);
        for (int q = wg; q < qn; q += 2) {
          uint32_t r[32];
          sm100::tmem_ld32(acc + q * 32, r);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) part[(q * 32 + e) * BM + row] = __uint_as_float(r[e]);
        }
        sm100::fence_proxy_async_smem();  // read next by bulk copies
        sm100::tc_fence_before();
        sm100::mbar_arrive(acc_empty(buf));
        continue;
      }
      if (c0 == 0 && c1 == KC) {
        // Whole tile in this CTA: round and store straight from TMEM.
        for (int q = wg; q < qn; q += 2) {
          uint32_t r[32];
          sm100::tmem_ld32(acc + q * 32, r);
          sm100::tmem_wait_ld();
          float v[32];
#pragma unroll
          for (int e = 0; e < 32; ++e) v[e] = __uint_as_float(r[e]);
          finalize<T>(a, sg, lt, q, v, xch, row, wg);
        }
        sm100::tc_fence_before();
        sm100::mbar_arrive(acc_empty(buf));
        continue;
      }
      // Stream-K part of a tile: partial to the workspace, slot 0 for the
      // range's first tile, 1 for its last (a range cut on both sides holds
      // one tile). Slot layout [x row / 4][weight row][4]: one 16-byte store
      // per thread and 4 x rows, 512 contiguous bytes per warp.
      const int slot = t == first_sk_tile ? 0 : 1;
      float4* part = reinterpret_cast<float4*>(a.partials + (static_cast<int64_t>(b) * 2 + slot) * BN * BM) + row;
      for (int q = wg; q < qn; q += 2) {
        uint32_t r[32];
        sm100::tmem_ld32(acc + q * 32, r);
        sm100::tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 8; ++j)
          __stcg(part + (q * 8 + j) * BM, make_float4(__uint_as_float(r[4 * j]), __uint_as_float(r[4 * j + 1]),
                                                      __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3])));
      }
      sm100::tc_fence_before();
      sm100::mbar_arrive(acc_empty(buf));
      sm100::bar_sync_named(kAllEpi, kEpiThreads);
      const int sk_t = t - a.dp_tiles;
      const int64_t t_first_unit = static_cast<int64_t>(sk_t) * KC;
      const int b_first = owner(a.sk_units, a.sk_grid, t_first_unit);
      const int b_last = owner(a.sk_units, a.sk_grid, t_first_unit + KC - 1);
      if (tid == 0) {
        // The barrier ordered every thread's partial stores before this
        // thread's fence (cumulative), which orders them before the count.
        __threadfence();
        const int old = atomicAdd(a.counters + sk_t, 1);
        const int last = old == b_last - b_first;
        if (last) a.counters[sk_t] = 0;  // every contributor has arrived: reset for the next launch
        __threadfence();
        *fix_flag = last;
      }
      sm100::bar_sync_named(kAllEpi, kEpiThreads);
      // fix_flag is next written after the first barrier of the next partial
      // tile, which every thread reaches only after this read.
      if (*fix_flag == 0) continue;
      // Fix-up: sum the tile's partials in CTA order (independent of arrival
      // order), two contributors' loads in flight before their adds.
      for (int q = wg; q < qn; q += 2) {
        float v[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) v[e] = 0.f;
        for (int b0 = b_first; b0 <= b_last; b0 += 2) {
          float4 pv[2][8];
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            const int bb = b0 + i;
            if (bb <= b_last) {
              const int sl = range_begin(a.sk_units, a.sk_grid, bb) >= t_first_unit ? 0 : 1;
              const float4* src =
                  reinterpret_cast<const float4*>(a.partials + (static_cast<int64_t>(bb) * 2 + sl) * BN * BM) + row;
#pragma unroll
              for (int j = 0; j < 8; ++j) pv[i][j] = __ldcg(src + (q * 8 + j) * BM);
            }
          }
#pragma unroll
          for (int i = 0; i < 2; ++i) {
            if (b0 + i <= b_last) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                v[4 * j] += pv[i][j].x;
                v[4 * j + 1] += pv[i][j].y;
                v[4 * j + 2] += pv[i][j].z;
                v[4 * j + 3] += pv[i][j].w;
              }
            }
          }
        }
        finalize<T>(a, sg, lt, q, v, xch, row, wg);
      }
    }
  }

  if (a.split > 1 && !a.part_slice) {
    // Split-K reduction. Once the whole cluster is here, every CTA's partial
    // is in its shared memory and every ring is idle. x rows [rows*r/S,
    // rows*(r+1)/S) belong to rank r: each rank pushes each peer's rows of its
    // partial into that peer's receive area (one bulk copy per peer, counted
    // on the peer's red_full barrier), then sums its own rows over all ranks
    // in rank order and writes them.
    sm100::cluster_sync();
    const int S = a.split;
    const int me = static_cast<int>(sm100::cluster_rank());
    const int t = b / S;
    const Segment sg = seg_at(a, seg_index(a, t));
    const int lt = t - sg.tile_begin;
    const int m0 = a.rows * me / S, m1 = a.rows * (me + 1) / S;
    const uint32_t row_bytes = BM * 4;
    const uint32_t slice_bytes = static_cast<uint32_t>((a.rows + S - 1) / S) * row_bytes;  // receive slot
    const uint32_t recv = base + L::PART_BYTES;
    if (tid == 0) {
      const uint32_t mine = static_cast<uint32_t>(m1 - m0) * row_bytes;
      if (mine) sm100::mbar_arrive_expect_tx(red_full, static_cast<uint32_t>(S - 1) * mine);
      else sm100::mbar_arrive(red_full);
      for (int q = 0; q < S; ++q) {
        const int q0 = a.rows * q / S, q1 = a.rows * (q + 1) / S;
        if (q == me || q1 == q0) continue;
        const uint32_t slot = static_cast<uint32_t>(me < q ? me : me - 1);  // my slot at rank q
        sm100::bulk_copy_to_peer(sm100::map_peer(recv + slot * slice_bytes, q), base + q0 * row_bytes,
                                 static_cast<uint32_t>(q1 - q0) * row_bytes, sm100::map_peer(red_full, q));
      }
      sm100::bulk_commit();
    }
    if (warp < kEpiWarps) {
      // Every peer sends its slices once past the barrier above, aborted or
      // not, so this waits for them in any case: they must land before the
      // CTA may exit.
      volatile int keep_waiting = 0;
      const bool got = sm100::mbar_wait(red_full, 0, &keep_waiting, err, ERR_REDUCE, WAIT_LIMIT);
      if (sm100::bar_and_named(kAllEpi, kEpiThreads, got && !*abort)) {
        const float* part = reinterpret_cast<const float*>(gbase);
        const float* rcv = reinterpret_cast<const float*>(gbase + L::PART_BYTES);
        const int slot_f = static_cast<int>(slice_bytes / 4);
        // Rank p's partial of (x row m, weight row n), m in [m0, m1).
        auto value = [&](int p, int m, int n) -> float {
          return p == me ? part[m * BM + n] : rcv[(p < me ? p : p - 1) * slot_f + (m - m0) * BM + n];
        };
        if (!sg.paired) {
          const int n = tid & (BM - 1);
          const int64_t col = static_cast<int64_t>(lt) * BM + n;
          if (col < sg.n) {
            for (int m = m0 + (tid >> 7); m < m1; m += 2) {
              float v = 0.f;
#pragma unroll
              for (int p = 0; p < kMaxSplit; ++p)
                if (p < S) v += value(p, m, n);
              sg.out[static_cast<int64_t>(m) * sg.out_stride + col] = T::from_f(v);
            }
          }
        } else {
          const int j = tid & 63;
          const int64_t col = static_cast<int64_t>(lt) * 64 + j;
          if (col < sg.n) {
            for (int m = m0 + (tid >> 6); m < m1; m += 4) {
              float g = 0.f, u = 0.f;
#pragma unroll
              for (int p = 0; p < kMaxSplit; ++p)
                if (p < S) {
                  g += value(p, m, j);
                  u += value(p, m, 64 + j);
                }
              sg.out[static_cast<int64_t>(m) * sg.out_stride + col] = silu_mul_elem_fast<T>(rnd<T>(g), rnd<T>(u));
            }
          }
        }
      }
    }
    if (tid == 0) sm100::bulk_wait_read();
    // No CTA leaves while a copy into its shared memory may be in flight.
    sm100::cluster_sync();
  }

  sm100::tc_fence_before();
  __syncthreads();
  // Every role has stopped; `abort` is final. After an abort, consumers may
  // have left stages unread: never leave the CTA while one of our copies may
  // still land in shared memory. (Without an abort every stage was waited for.)
  if (*abort && warp == kTmaWarp && lane == 0) {
    volatile int keep_waiting = 0;
    for (int j = it > NS ? it - NS : 0; j < it; ++j)
      sm100::mbar_wait(full(j % NS), (j / NS) & 1, &keep_waiting, nullptr, 0, WAIT_LIMIT);
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

// Row-major [rows][k] (row stride `stride` elements), box 64 x box_rows.
bool make_map(CUtensorMap* map, const void* ptr, bool bf16, int64_t k, int64_t rows, int64_t stride, int box_rows) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(stride) * 2};
  cuuint32_t box[2] = {BK, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

int pick_bn(int64_t rows) {
  if (rows <= 32) return 32;
  if (rows <= 64) return 64;
  if (rows <= 128) return 128;
  return 256;
}

// Geometry-only part of the plan (the split-K cluster size needs the device
// and is chosen at launch).
struct Plan {
  int bn, tiles, kchunks;
  bool stream_k;
  int grid, dp_tiles, sk_grid;
  int64_t sk_units;
  int tile_begin[MAX_SEGS];
};

Plan make_plan(int64_t rows, int64_t k, const kvr_linear_segment* segs, int count) {
  Plan p{};
  p.bn = pick_bn(rows < kMaxRows ? rows : kMaxRows);
  p.kchunks = static_cast<int>((k + BK - 1) / BK);
  int tiles = 0;
  for (int i = 0; i < count; ++i) {
    p.tile_begin[i] = tiles;
    const int per = segs[i].weight_up ? 64 : BM;
    tiles += static_cast<int>((segs[i].n + per - 1) / per);
  }
  p.tiles = tiles;
  p.stream_k = tiles >= kNumSMs;
  if (p.stream_k) {
    p.grid = kNumSMs;
    p.dp_tiles = tiles - tiles % kNumSMs;
    p.sk_units = static_cast<int64_t>(tiles - p.dp_tiles) * p.kchunks;
    p.sk_grid = static_cast<int>(p.sk_units < kNumSMs ? p.sk_units : kNumSMs);
  }
  return p;
}

size_t partial_bytes(const Plan& p) { return static_cast<size_t>(p.sk_grid) * 2 * p.bn * BM * sizeof(float); }

size_t workspace_bytes(const Plan& p) {
  if (!p.stream_k || p.sk_units == 0) return STATUS_BYTES;
  const size_t counters = (static_cast<size_t>(p.tiles - p.dp_tiles) * sizeof(int) + 255) / 256 * 256;
  return STATUS_BYTES + counters + partial_bytes(p);
}

template <class T, int BN>
int configure(int dev) {
  static int configured[64] = {0};
  if (dev >= 0 && dev < 64 && __atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) return KVR_OK;
  const cudaError_t e =
      cudaFuncSetAttribute(linear_kernel<T, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize, Layout<BN>::BYTES);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  return KVR_OK;
}

// Largest cluster size S <= min(8, kchunks, SMs / tiles) for which `tiles`
// clusters are resident at once (one wave), else 1. Occupancy answers are
// cached per device and S.
template <class T, int BN>
int choose_split(int dev, int tiles, int kchunks, int rows) {
  static int cache[64][kMaxSplit + 1] = {};  // 0 = not queried, else clusters + 1
  int s_max = kNumSMs / tiles;
  if (s_max > kMaxSplit) s_max = kMaxSplit;
  if (s_max > kchunks) s_max = kchunks;
  for (int s = s_max; s >= 2; --s) {
    // partial + receive slots for the S-1 peers' slices of this CTA's rows
    const int64_t need = Layout<BN>::PART_BYTES + static_cast<int64_t>(s - 1) * ((rows + s - 1) / s) * BM * 4;
    if (need > Layout<BN>::RING_BYTES) continue;
    int clusters = 0;
    if (dev >= 0 && dev < 64 && __atomic_load_n(&cache[dev][s], __ATOMIC_ACQUIRE)) {
      clusters = cache[dev][s] - 1;
    } else {
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(s));
      cfg.blockDim = dim3(THREADS);
      cfg.dynamicSmemBytes = Layout<BN>::BYTES;
      cudaLaunchAttribute attr;
      attr.id = cudaLaunchAttributeClusterDimension;
      attr.val.clusterDim.x = static_cast<unsigned>(s);
      attr.val.clusterDim.y = 1;
      attr.val.clusterDim.z = 1;
      cfg.attrs = &attr;
      cfg.numAttrs = 1;
      if (cudaOccupancyMaxActiveClusters(&clusters, linear_kernel<T, BN>, &cfg) != cudaSuccess) {
        cudaGetLastError();  // not sticky: fall back to a smaller cluster
        clusters = 0;
      }
      if (dev >= 0 && dev < 64) __atomic_store_n(&cache[dev][s], clusters + 1, __ATOMIC_RELEASE);
    }
    if (clusters >= tiles) return s;
  }
  return 1;
}

template <class T, int BN>
int launch(const Maps& maps, Args a, const Plan& p, cudaStream_t s, int deferred) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  const int st = configure<T, BN>(dev);
  if (st != KVR_OK) return st;
  unsigned grid = static_cast<unsigned>(p.grid);
  int cluster = 1;
  if (deferred > 0) {  // one wave of independent CTAs, no cluster
    a.split = deferred;
    grid = static_cast<unsigned>(p.tiles * a.split);
  } else if (p.stream_k) {
    a.split = 0;
  } else {
    a.split = choose_split<T, BN>(dev, p.tiles, p.kchunks, a.rows);
    cluster = a.split;
    grid = static_cast<unsigned>(p.tiles * a.split);
  }
  return launch_pdl<linear_kernel<T, BN>>(dim3(grid), dim3(THREADS), Layout<BN>::BYTES, s, cluster, maps, a);
}

template <class T>
int launch_bn(const Maps& maps, const Args& a, const Plan& p, cudaStream_t s, int deferred) {
  switch (p.bn) {
    case 32: return launch<T, 32>(maps, a, p, s, deferred);
    case 64: return launch<T, 64>(maps, a, p, s, deferred);
    case 128: return launch<T, 128>(maps, a, p, s, deferred);
    default: return launch<T, 256>(maps, a, p, s, deferred);
  }
}

bool valid_segments(int64_t k, const kvr_linear_segment* segs, int count) {
  if (!segs || count < 1 || count > MAX_SEGS) return false;
  for (int i = 0; i < count; ++i) {
    const kvr_linear_segment& sg = segs[i];
    if (!sg.weight || !aligned16(sg.weight) || sg.n <= 0 || !sg.out || sg.out_stride < sg.n) return false;
    if (sg.weight_up && !aligned16(sg.weight_up)) return false;
  }
  return k > 0 && k % 8 == 0;
}

}  // namespace lin

size_t linear_workspace_bytes(int64_t rows, int64_t k, const int64_t* n, const bool* paired, int count) {
  if (rows <= 0 || k <= 0 || count < 1 || count > lin::MAX_SEGS) return lin::STATUS_BYTES;
  kvr_linear_segment segs[lin::MAX_SEGS] = {};
  for (int i = 0; i < count; ++i) {
    segs[i].n = n[i];
    segs[i].weight_up = paired[i] ? segs : nullptr;  // only its presence matters to the plan
  }
  return lin::workspace_bytes(lin::make_plan(rows, k, segs, count));
}

size_t linear_workspace_size(int64_t rows, int64_t k, const kvr_linear_segment* segments, int count) {
  if (rows <= 0 || !lin::valid_segments(k, segments, count)) return lin::STATUS_BYTES;
  return lin::workspace_bytes(lin::make_plan(rows, k, segments, count));
}

int deferred_split(int64_t tiles, int64_t k) {
  const int64_t kc = (k + lin::BK - 1) / lin::BK;
  int64_t s = tiles > 0 ? kNumSMs / tiles : 1;
  if (s > kc) s = kc;
  if (s > 16) s = 16;
  return s < 1 ? 1 : static_cast<int>(s);
}

int linear_forward(const void* x, int64_t x_stride, int64_t rows, int64_t k, const kvr_linear_segment* segments,
                   int count, void* workspace, size_t workspace_bytes, int dtype, bool counters_zeroed,
                   cudaStream_t stream, Deferred* deferred) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (rows < 0 || !lin::valid_segments(k, segments, count)) return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!x || !aligned16(x) || x_stride < k || x_stride % 8) return KVR_ERR_INVALID_ARG;
  if (k > 0x7fffffffLL) return KVR_ERR_UNSUPPORTED;
  for (int i = 0; i < count; ++i)
    if (segments[i].n > 0x3fffffffLL) return KVR_ERR_UNSUPPORTED;
  lin::Plan p = lin::make_plan(rows, k, segments, count);
  if (static_cast<int64_t>(p.tiles) * p.kchunks > 0x7fffffffLL) return KVR_ERR_UNSUPPORTED;
  int defer = 0;
  if (deferred) {
    for (int i = 0; i < count; ++i)
      if (segments[i].weight_up || !deferred->part[i]) return KVR_ERR_INVALID_ARG;
    if (rows > kMaxRows) return KVR_ERR_UNSUPPORTED;  // one launch: one set of slices
    defer = deferred_split(p.tiles, k);
    if (defer > deferred->max_split) defer = deferred->max_split;
    deferred->split = defer;
    p.stream_k = false;  // independent CTAs, no stream-K workspace
    p.dp_tiles = p.sk_grid = 0;
    p.sk_units = 0;
  }
  const size_t need = lin::workspace_bytes(p);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return KVR_ERR_INVALID_ARG;
  const bool bf16 = dtype == KVR_DTYPE_BF16;

  lin::Maps maps;
  memset(&maps, 0, sizeof(maps));
  lin::Args a{};
  for (int i = 0; i < count; ++i) {
    const kvr_linear_segment& sg = segments[i];
    const bool paired = sg.weight_up != nullptr;
    const int box = paired ? 64 : lin::BM;
    if (!lin::make_map(&maps.w[2 * i], sg.weight, bf16, k, sg.n, k, box)) return KVR_ERR_UNSUPPORTED;
    if (paired && !lin::make_map(&maps.w[2 * i + 1], sg.weight_up, bf16, k, sg.n, k, box))
      return KVR_ERR_UNSUPPORTED;
    a.seg[i].out = static_cast<uint16_t*>(sg.out);
    a.seg[i].out_stride = sg.out_stride;
    a.seg[i].n = sg.n;
    a.seg[i].tile_begin = p.tile_begin[i];
    a.seg[i].paired = paired ? 1 : 0;
    a.seg[i].part = deferred ? deferred->part[i] : nullptr;
  }
  if (deferred) {
    a.part_stride = deferred->part_stride;
    a.part_slice = deferred->part_slice;
  }
  a.nseg = count;
  a.kchunks = p.kchunks;
  a.tiles = p.tiles;
  a.grid = p.grid;
  a.dp_tiles = p.dp_tiles;
  a.sk_grid = p.sk_grid;
  a.sk_units = p.sk_units;
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  a.status = reinterpret_cast<int*>(ws);
  a.counters = reinterpret_cast<int*>(ws + lin::STATUS_BYTES);
  a.partials = reinterpret_cast<float*>(ws + need - lin::partial_bytes(p));
  a.wait_limit = pipeline_wait_limit();
  if (!counters_zeroed) {
    const cudaError_t e = cudaMemsetAsync(ws, 0, need - lin::partial_bytes(p), stream);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
  }
  // Blocks of at most kMaxRows rows; each block streams the weights again.
  const uint8_t* xb = static_cast<const uint8_t*>(x);
  for (int64_t r0 = 0; r0 < rows; r0 += kMaxRows) {
    const int64_t nr = rows - r0 < kMaxRows ? rows - r0 : kMaxRows;
    if (!lin::make_map(&maps.x, xb + r0 * x_stride * 2, bf16, k, nr, x_stride, p.bn)) return KVR_ERR_UNSUPPORTED;
    a.rows = static_cast<int>(nr);
    for (int i = 0; i < count; ++i)
      a.seg[i].out = static_cast<uint16_t*>(segments[i].out) + r0 * segments[i].out_stride;
    const int st =
        bf16 ? lin::launch_bn<BF16>(maps, a, p, stream, defer) : lin::launch_bn<F16>(maps, a, p, stream, defer);
    if (st != KVR_OK) return st;
  }
  return KVR_OK;
}

}  // namespace kvr

extern "C" {

size_t kvr_linear_workspace_size(int64_t rows, int64_t k, const kvr_linear_segment* segments, int count) {
  return kvr::linear_workspace_size(rows, k, segments, count);
}

int kvr_linear(const void* x, int64_t x_stride, int64_t rows, int64_t k, const kvr_linear_segment* segments,
               int count, void* workspace, size_t workspace_bytes, int dtype, void* stream) {
  return kvr::linear_forward(x, x_stride, rows, k, segments, count, workspace, workspace_bytes, dtype, false,
                             static_cast<cudaStream_t>(stream));
}

}  // extern "C"
