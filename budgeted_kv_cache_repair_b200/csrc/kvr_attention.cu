// Selected-query absolute-causal attention on sm_100a tensor cores (tcgen05 +
// TMEM + TMA), GQA-packed and split over the key range.
//
// Work unit (CTA): one KV head h, one tile of 128 "m-entries" and one key
// chunk. An m-entry is a (selected row r, query head g of the group) pair,
// m = r*G + g: the G query heads that share KV head h occupy MMA rows of the
// same tile, so each K/V tile brought on chip serves all of them (no
// repeat_kv). Rows are sorted by absolute position; a tile's causal span is
// [0, pos(last row)].
//
// One CTA per SM, 11 warps:
//   warp 8  TMA producer: K and V blocks of 128 keys, 128B-swizzled, into
//           rings of NS stages with separate K and V barriers, so a K stage is
//           refilled as soon as its Q.K^T is done (bounded waits, no multicast)
//   warp 10 Q.K^T issuer (one thread): S_j = Q K_j^T into TMEM S buffer j & 1
//   warp 9  P.V issuer (one thread): O += P_j V_j into the TMEM O accumulators,
//           with P_j read from tensor memory; it also owns the TMEM allocation.
//           Two issuing threads, because tcgen05.mma issue blocks while the
//           tensor pipe is busy: S_{j+2} must not queue behind P.V of block j+1.
//   warps 0-7  softmax: two threads per m-entry row (TMEM lane = row), each
//           owning 64 keys of every block with its own running max, sum and
//           TMEM O accumulator. A thread loads its S half-row, applies the
//           causal/chunk mask, keeps a running max, writes P = 2^(s - m) over
//           its own S columns in tensor memory (the A operand of P.V), and
//           rescales its O half in TMEM only when the max grew by more than 2^8
//           (exact: the final normalisation uses the same stale max). The two
//           halves merge once, in the epilogue.
// QK^T of block j+1 overlaps the softmax of block j.
//
// Precision: QK^T and PV run on bf16/fp16 operands with fp32 accumulation.
// With SPLIT, P is issued as P_hi + P_lo (two element-type halves, two PV
// MMAs), keeping ~16 mantissa bits of the probabilities as the reference's
// fp32-probability P@V does (kernels/_indexed_triton.py:58); without SPLIT, P
// is rounded once, as in fused SDPA kernels.
//
// Partial results of a split key range go to the workspace as (O, max, sum)
// and attn_combine_kernel merges them. Every wait is bounded: on timeout the
// kernel records an error code in the workspace status word, stops issuing,
// drains its own in-flight TMA and MMA work, frees TMEM and returns.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <math.h>

#include <type_traits>

#include "kvr_common.cuh"
#include "kvr_sm100.cuh"

namespace kvr {
namespace attn {

constexpr int BM = 128;  // m-entries per CTA (MMA M, TMEM lanes)
constexpr int BN = 128;  // keys per block (MMA N of QK^T, K of PV)
constexpr int kSoftmaxThreads = 256;  // warps 0-7: two threads per m-entry row
constexpr int kTmaWarp = 8;
constexpr int kMmaWarp = 9;   // P.V issuer; also allocates and frees tensor memory
constexpr int kQkWarp = 10;   // Q.K^T issuer
constexpr int THREADS = 352;
constexpr int SUB = BM * 128;  // one [128 rows x 128 B] swizzled sub-tile
constexpr int STATUS_BYTES = 256;
constexpr int kEpilogueBar = 1;        // named barrier of the softmax warps (0 is __syncthreads)
constexpr long long WAIT_LIMIT = kDefaultWaitLimit;  // drains of the CTA's own copies and MMAs

enum Err : int { ERR_KV_EMPTY = 1, ERR_Q_FULL, ERR_KV_FULL, ERR_S_FREE, ERR_P_FULL, ERR_S_FULL,
                 ERR_PV_DONE, ERR_DRAIN, ERR_RED, ERR_SMEM_ALIGN };

struct Args {
  const uint16_t* q;
  uint16_t* out;
  const int64_t* positions;
  int64_t rows;
  int hq, hkv, group;
  float scale_log2;
  int tiles, nchunks;
  int64_t chunk;  // keys per chunk (multiple of BN)
  int* status;    // workspace status word (error code, 0 = ok)
  int q_by_tma;   // Q tile fetched by TMA (128 % group == 0) or by cp.async
  float* ws_o;    // [hkv][tiles][nchunks][BM][D] unnormalised O
  float* ws_ml;   // [hkv][tiles][nchunks][BM][2] (running max, sum)
  long long wait_limit;  // SM clocks before a pipeline wait gives up
};

template <int D, bool SPLIT>
struct Layout {
  static constexpr int DS = D / 64;  // 64-element (128 B) sub-tiles across head_dim
  // K/V ring stages. P lives in tensor memory (over its own S columns), so
  // shared memory holds only Q and the rings.
  static constexpr int NS = D == 128 ? 3 : 4;
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + DS * SUB;
  static constexpr int V_OFF = K_OFF + NS * DS * SUB;
  static constexpr int NP = 2;  // P buffers = the two S buffers
  static constexpr int BAR_OFF = V_OFF + NS * DS * SUB;
  // q_full, k_full[NS], k_empty[NS], v_full[NS], v_empty[NS], s_full[2], s_free[2], p_full[NP],
  // pv_done[NP], drain, red_bar, drain_qk
  static constexpr int NBAR = 1 + 4 * NS + 4 + 2 * NP + 1 + 1 + 1;
  static constexpr int MISC_OFF = BAR_OFF + NBAR * 8;
  static constexpr int RED_OFF = MISC_OFF + 16;  // float [2 halves][128 rows][max, sum]
  static constexpr int USED = RED_OFF + 2 * BM * 2 * 4;
  // Swizzled tiles need a 1 KB-aligned base; the allocation carries what slack
  // fits under the per-CTA limit and the kernel checks it at run time.
  static constexpr int BYTES = USED + 1024 <= 232448 ? USED + 1024 : 232448;
  // Staged output rows (epilogue, in the K ring): D floats plus a 16-byte
  // shift per row, so a warp's row-per-lane float4 stores hit distinct banks.
  static constexpr int STAGE_STRIDE = D + 4;
  static_assert(NS * DS * SUB >= BM * STAGE_STRIDE * 4, "the K ring holds the staged output tile");
  static constexpr uint32_t HALF_TX = DS * SUB;  // one K or one V block
  static_assert(USED <= 232448, "dynamic shared memory above the 227 KB per-CTA limit");
};

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  const int n = valid ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;\n" ::"r"(dst), "l"(src), "r"(n) : "memory");
}

template <class T>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  return static_cast<uint32_t>(T::from_f(lo)) | (static_cast<uint32_t>(T::from_f(hi)) << 16);
}

// Two floats -> packed pair with the hardware round-to-nearest conversion
// (cvt.rn.bf16x2.f32 / cvt.rn.f16x2.f32); used for probabilities, which are
// finite and non-negative, so NaN payload conventions do not arise.
template <class T>
__device__ __forceinline__ uint32_t pack2_hw(float lo, float hi) {
  if constexpr (std::is_same<T, BF16>::value) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  } else {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
}
template <class T>
__device__ __forceinline__ float lo_half(uint32_t v) {
  return T::to_f(static_cast<uint16_t>(v & 0xffffu));
}
template <class T>
__device__ __forceinline__ float hi_half(uint32_t v) {
  return T::to_f(static_cast<uint16_t>(v >> 16));
}

// 2^x with the MUFU approximation (relative error ~2^-22; inputs here are <= 8).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// max(a, b, c) in one instruction (sm_100).
__device__ __forceinline__ float max3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

// Byte offset of 16-byte chunk c (0..7) of row r in a 128B-swizzled sub-tile.
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

template <class T, int D, bool SPLIT>
__global__ void __launch_bounds__(THREADS, 1)
    attn_tc_kernel(const __grid_constant__ CUtensorMap tmap_k, const __grid_constant__ CUtensorMap tmap_v,
                   const __grid_constant__ CUtensorMap tmap_q, Args a) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  using L = Layout<D, SPLIT>;
  constexpr int DS = L::DS, NS = L::NS, NP = L::NP;
  constexpr int HD = D / 2;  // output columns per softmax thread in the epilogue
  constexpr bool kBF16 = std::is_same<T, BF16>::value;
  extern __shared__ uint8_t smem_raw[];

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  // Launch order (1-D grid): key chunk, then KV head, then tiles from the last
  // (latest positions, longest causal span) down, so that the block scheduler
  // starts the longest work first and the tiles sharing a K/V chunk run
  // together (the chunk stays in L2).
  const int tile = a.tiles - 1 - static_cast<int>(blockIdx.x % a.tiles);
  const int h = static_cast<int>((blockIdx.x / a.tiles) % a.hkv);
  const int chunk = static_cast<int>(blockIdx.x / a.tiles / a.hkv);
  const int G = a.group;
  const int64_t total_m = a.rows * G;
  const int64_t m0 = static_cast<int64_t>(tile) * BM;
  int64_t r_last = (m0 + BM - 1) / G;
  if (r_last > a.rows - 1) r_last = a.rows - 1;
  const int64_t k_begin = static_cast<int64_t>(chunk) * a.chunk;

  const uint32_t raw = sm100::smem_u32(smem_raw);
  const uint32_t base = (raw + 1023u) & ~1023u;
  if (base - raw + L::USED > static_cast<uint32_t>(L::BYTES)) {  // uniform: every thread sees the same
    if (tid == 0) atomicCAS(a.status, 0, ERR_SMEM_ALIGN);
    return;
  }
  uint8_t* gbase = smem_raw + (base - raw);
  const uint32_t bar0 = base + L::BAR_OFF;
  const uint32_t q_full = bar0;
  // K and V blocks have their own barriers: a K stage is refilled as soon as
  // its Q.K^T MMA is done, a V stage once its P.V MMA is done.
  auto k_full = [&](int s) { return bar0 + 8u * (1 + s); };
  auto k_empty = [&](int s) { return bar0 + 8u * (1 + NS + s); };
  auto v_full = [&](int s) { return bar0 + 8u * (1 + 2 * NS + s); };
  auto v_empty = [&](int s) { return bar0 + 8u * (1 + 3 * NS + s); };
  auto s_full = [&](int b) { return bar0 + 8u * (1 + 4 * NS + b); };
  auto s_free = [&](int b) { return bar0 + 8u * (3 + 4 * NS + b); };
  auto p_full = [&](int pb) { return bar0 + 8u * (5 + 4 * NS + pb); };
  auto pv_done = [&](int pb) { return bar0 + 8u * (5 + 4 * NS + NP + pb); };
  const uint32_t drain = bar0 + 8u * (5 + 4 * NS + 2 * NP);
  const uint32_t red_bar = bar0 + 8u * (6 + 4 * NS + 2 * NP);
  const uint32_t drain_qk = bar0 + 8u * (7 + 4 * NS + 2 * NP);
  volatile int* abort = reinterpret_cast<volatile int*>(gbase + L::MISC_OFF);
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(gbase + L::MISC_OFF + 4);
  float* red = reinterpret_cast<float*>(gbase + L::RED_OFF);  // [2 halves][128 rows][max, sum]
  int* err = a.status;

  if (tid == 0) {
    *abort = 0;
    sm100::mbar_init(q_full, a.q_by_tma ? 1 : kSoftmaxThreads);
    for (int s = 0; s < NS; ++s) {
      sm100::mbar_init(k_full(s), 1);
      sm100::mbar_init(k_empty(s), 1);
      sm100::mbar_init(v_full(s), 1);
      sm100::mbar_init(v_empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      sm100::mbar_init(s_full(b), 1);
      sm100::mbar_init(s_free(b), 1);  // committed after the P.V that reads P (in S's columns)
    }
    for (int pb = 0; pb < NP; ++pb) {
      sm100::mbar_init(p_full(pb), kSoftmaxThreads);
      sm100::mbar_init(pv_done(pb), 1);
    }
    sm100::mbar_init(drain, 1);
    sm100::mbar_init(drain_qk, 1);
    sm100::mbar_init(red_bar, kSoftmaxThreads);
    sm100::fence_barrier_init();
  }
  if (warp == kMmaWarp) {
    sm100::tmem_alloc(sm100::smem_u32(tmem_slot), 512);
    sm100::tmem_relinquish();
  }
  if (warp == kTmaWarp && lane == 0) {
    sm100::prefetch_tmap(&tmap_k);
    sm100::prefetch_tmap(&tmap_v);
  }
  sm100::tc_fence_before();
  __syncthreads();
  sm100::tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(tmem_slot);
  // Everything above (barriers, tensor memory, descriptor prefetch) overlaps
  // the previous kernel; the positions, queries and cache may come from it.
  pdl_wait();
  const int64_t pmax = a.positions[r_last];
  int64_t k_end = k_begin + a.chunk;
  if (k_end > pmax + 1) k_end = pmax + 1;
  // A chunk past every row of the tile has no blocks (uniform): straight to teardown.
  const int nblk = k_begin > pmax ? 0 : static_cast<int>((k_end - k_begin + BN - 1) / BN);
  // TMEM columns: S buffers [0,128) and [128,256); one O accumulator per key
  // half, [256, 256+D) and [256+D, 256+2D).
  constexpr uint32_t TM_O = 256;

  // Copies this CTA's producer has issued (Q by TMA, K and V blocks): an
  // aborted CTA waits for them to land before it exits (see the teardown).
  int issued_k = 0, issued_v = 0;
  if (nblk == 0) {
    // No keys for this tile in this chunk: no role has work, but the combine
    // reads every chunk's (max, sum), so the rows record an empty chunk.
    if (a.nchunks > 1 && tid < BM) {
      const int64_t wu = (static_cast<int64_t>(h) * a.tiles + tile) * a.nchunks + chunk;
      *reinterpret_cast<float2*>(a.ws_ml + (wu * BM + tid) * 2) = make_float2(-INFINITY, 0.f);
    }
  } else if (warp == kTmaWarp) {
    if (lane == 0) {
      // ---------------- TMA producer ----------------
      if (a.q_by_tma) {
        // The tile's 128 m-entries are 128/G consecutive rows x the G heads of
        // KV head h: one box per 64-column half of head_dim.
        sm100::mbar_arrive_expect_tx(q_full, DS * SUB);
#pragma unroll
        for (int ds = 0; ds < DS; ++ds)
          sm100::tma_load_3d(base + L::Q_OFF + ds * SUB, &tmap_q, q_full, ds * 64, h * G,
                             static_cast<int>(m0 / G));
      }
      for (int j = 0; j < nblk; ++j) {
        const int s = j % NS;
        const int key0 = static_cast<int>(k_begin + static_cast<int64_t>(j) * BN);
        if (j >= NS && !sm100::mbar_wait(k_empty(s), ((j / NS) - 1) & 1, abort, err, ERR_KV_EMPTY, a.wait_limit))
          break;
        sm100::mbar_arrive_expect_tx(k_full(s), L::HALF_TX);
#pragma unroll
        for (int ds = 0; ds < DS; ++ds)
          sm100::tma_load_3d(base + L::K_OFF + (s * DS + ds) * SUB, &tmap_k, k_full(s), ds * 64, key0, h);
        issued_k = j + 1;
        if (j >= NS && !sm100::mbar_wait(v_empty(s), ((j / NS) - 1) & 1, abort, err, ERR_KV_EMPTY, a.wait_limit))
          break;
        sm100::mbar_arrive_expect_tx(v_full(s), L::HALF_TX);
#pragma unroll
        for (int ds = 0; ds < DS; ++ds)
          sm100::tma_load_3d(base + L::V_OFF + (s * DS + ds) * SUB, &tmap_v, v_full(s), ds * 64, key0, h);
        issued_v = j + 1;
      }
    }
  } else if (warp == kQkWarp) {
    if (lane == 0) {
      // ---------------- Q.K^T issuer ----------------
      // Its own thread, so that S of block j+2 is issued the moment P.V of
      // block j has freed the buffer, never behind a P.V issue (tcgen05.mma
      // issue blocks while the tensor pipe is busy).
      constexpr uint32_t IQK = sm100::idesc_f16(kBF16, BM, BN, false);
      bool ok = sm100::mbar_wait(q_full, 0, abort, err, ERR_Q_FULL, a.wait_limit);
      for (int j = 0; ok && j < nblk; ++j) {
        const int s = j % NS, b = j & 1;
        if (!sm100::mbar_wait(k_full(s), (j / NS) & 1, abort, err, ERR_KV_FULL, a.wait_limit)) break;
        if (j >= 2 && !sm100::mbar_wait(s_free(b), ((j >> 1) - 1) & 1, abort, err, ERR_S_FREE, a.wait_limit)) break;
        sm100::tc_fence_after();
#pragma unroll
        for (int k = 0; k < D / 16; ++k) {
          const int ds = k >> 2, kk = k & 3;
          const uint64_t da = sm100::desc_sw128(base + L::Q_OFF + ds * SUB + kk * 32, 16, 1024);
          const uint64_t db = sm100::desc_sw128(base + L::K_OFF + (s * DS + ds) * SUB + kk * 32, 16, 1024);
          sm100::mma_f16_ss(tmem + b * BN, da, db, IQK, k > 0);
        }
        sm100::mma_commit(s_full(b));
        sm100::mma_commit(k_empty(s));  // K block free once Q.K^T is done
      }
      // Nothing of ours may still be writing TMEM when it is freed.
      sm100::mma_commit(drain_qk);
      volatile int keep_waiting = 0;
      sm100::mbar_wait(drain_qk, 0, &keep_waiting, err, ERR_DRAIN, WAIT_LIMIT);
    }
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      // ---------------- P.V issuer ----------------
      constexpr uint32_t IPV = sm100::idesc_f16(kBF16, BM, D, true);
      for (int j = 0; j < nblk; ++j) {
        const int pb = j & 1;  // P of block j sits in S buffer j & 1
        if (!sm100::mbar_wait(p_full(pb), (j >> 1) & 1, abort, err, ERR_P_FULL, a.wait_limit)) break;
        if (!sm100::mbar_wait(v_full(j % NS), (j / NS) & 1, abort, err, ERR_KV_FULL, a.wait_limit)) break;
        sm100::tc_fence_after();
        const int s = j % NS;
        // P of key half `half`: 32 TMEM columns at pb*BN + half*64 (two 16-bit
        // values per column), the low halves of split P in the next 32.
        const uint32_t pcol = tmem + static_cast<uint32_t>(pb * BN);
#pragma unroll
        for (int half = 0; half < 2; ++half) {
#pragma unroll
          for (int k = 0; k < 4; ++k) {  // 16 keys per MMA, 64 keys per half
            // V block: MN-major (head_dim contiguous); 16 keys = two 8-row groups.
            const uint64_t db =
                sm100::desc_sw128(base + L::V_OFF + s * DS * SUB + (half * 4 + k) * 2048, SUB, 1024);
            const uint32_t acc = (j > 0 || k > 0) ? 1u : 0u;
            sm100::mma_f16_ts(tmem + TM_O + half * D, pcol + half * 64 + k * 8, db, IPV, acc);
            if constexpr (SPLIT) sm100::mma_f16_ts(tmem + TM_O + half * D, pcol + half * 64 + 32 + k * 8, db, IPV, 1u);
          }
        }
        sm100::mma_commit(pv_done(pb));
        sm100::mma_commit(v_empty(s));
        sm100::mma_commit(s_free(pb));  // S/P buffer free for block j + 2
      }
      // Nothing of ours may still be writing TMEM when it is freed.
      sm100::mma_commit(drain);
      volatile int keep_waiting = 0;
      sm100::mbar_wait(drain, 0, &keep_waiting, err, ERR_DRAIN, WAIT_LIMIT);
    }
  } else {
    // ------- softmax warps: thread (half, row) owns TMEM lane `row` and the keys
    // [64*half, 64*half+64) of every block, with its own running max, sum and O
    // accumulator (merged with the other half once, in the epilogue) -------
    const int row = tid & (BM - 1);
    const int half = tid >> 7;
    const int64_t m_abs = m0 + row;
    const bool valid = m_abs < total_m;
    const int64_t r = valid ? m_abs / G : 0;
    const int g = valid ? static_cast<int>(m_abs - r * G) : 0;
    const int64_t pos = valid ? a.positions[r] : 0;  // padding rows see key 0 only
    if (!a.q_by_tma) {
      const uint16_t* qsrc = a.q + ((r * a.hq + static_cast<int64_t>(h) * G + g) * D);
#pragma unroll
      for (int c = half * (D / 16); c < (half + 1) * (D / 16); ++c)
        cp_async16(base + L::Q_OFF + (c >> 3) * SUB + swz(row, c & 7), valid ? qsrc + c * 8 : a.q, valid);
      asm volatile("cp.async.commit_group;\ncp.async.wait_all;\n" ::: "memory");
      sm100::fence_proxy_async_smem();
      sm100::mbar_arrive(q_full);
    }

    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t scol = static_cast<uint32_t>(half * 64);
    const uint32_t ocol = TM_O + static_cast<uint32_t>(half * D);
    const float sl2 = a.scale_log2;
    float m_used = -INFINITY, lsum = 0.f;
    bool ok = true;
    for (int j = 0; j < nblk; ++j) {
      const int b = j & 1;
      // Warp-uniform decisions: tcgen05.ld/st are .sync.aligned.
      if (!__all_sync(0xffffffffu, sm100::mbar_wait(s_full(b), (j >> 1) & 1, abort, err, ERR_S_FULL, a.wait_limit))) {
        ok = false;
        break;
      }
      sm100::tc_fence_after();
      uint32_t sv[2][32];
      sm100::tmem_ld32(tmem + lane_base + b * BN + scol, sv[0]);
      sm100::tmem_ld32(tmem + lane_base + b * BN + scol + 32, sv[1]);
      sm100::tmem_wait_ld();

      const int64_t key0 = k_begin + static_cast<int64_t>(j) * BN + half * 64;
      // Visible columns of this half-block for this row: [0, lim).
      const int64_t lim64 = (pos + 1 < k_end ? pos + 1 : k_end) - key0;
      const int lim = lim64 < 0 ? 0 : (lim64 > 64 ? 64 : static_cast<int>(lim64));
      // Masked columns become -inf (then P = 2^-inf = 0); four independent
      // three-input max chains.
      if (lim < 64) {
#pragma unroll
        for (int e = 0; e < 64; ++e)
          if (e >= lim) sv[e >> 5][e & 31] = __float_as_uint(-INFINITY);
      }
      float mx4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int e = 0; e < 64; e += 8) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
          mx4[q] = max3(mx4[q], __uint_as_float(sv[e >> 5][(e + 2 * q) & 31]),
                        __uint_as_float(sv[e >> 5][(e + 2 * q + 1) & 31]));
      }
      const float mx = fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3]));
      const float m_new = fmaxf(m_used, mx * sl2);  // scale > 0: max commutes with scaling
      const bool rescale = m_used != -INFINITY && m_new > m_used + 8.0f;
      if (__any_sync(0xffffffffu, rescale)) {
        // This half's O must be final up to block j-1 before it is rescaled in TMEM.
        if (j > 0 && !__all_sync(0xffffffffu, sm100::mbar_wait(pv_done((j - 1) & 1), ((j - 1) >> 1) & 1, abort,
                                                                err, ERR_PV_DONE, a.wait_limit))) {
          ok = false;
          break;
        }
        sm100::tc_fence_after();
        const float f = rescale ? ex2_approx(m_used - m_new) : 1.0f;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t ov[32];
          sm100::tmem_ld32(tmem + lane_base + ocol + c * 32, ov);
          sm100::tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) ov[e] = __float_as_uint(__uint_as_float(ov[e]) * f);
          sm100::tmem_st32(tmem + lane_base + ocol + c * 32, ov);
        }
        sm100::tmem_wait_st();
        if (rescale) {
          lsum *= f;
          m_used = m_new;
        }
      }
      if (m_used == -INFINITY) m_used = m_new;  // first visible keys: this O row is still zero
      const float neg_mb = m_used == -INFINITY ? 0.f : -m_used;
      // P overwrites this thread's own S columns (already loaded): hi in the
      // first 32, split lo in the next 32; two 16-bit values per column.
      uint32_t phi[32], plo[32];
      // P = 2^(s*scale*log2e - m) two columns at a time (packed fp32 FMA and
      // adds, MUFU ex2 per value); four independent pair sums.
      const uint64_t scale2 = f2(sl2, sl2), shift2 = f2(neg_mb, neg_mb);
      uint64_t sum2[4] = {0, 0, 0, 0};
#pragma unroll
      for (int e = 0; e < 64; e += 2) {
        float t0, t1;
        f2_split(f2_fma(f2(__uint_as_float(sv[e >> 5][e & 31]), __uint_as_float(sv[e >> 5][(e + 1) & 31])), scale2,
                        shift2),
                 t0, t1);
        const float p0 = ex2_approx(t0), p1 = ex2_approx(t1);
        const uint64_t pp = f2(p0, p1);
        sum2[(e >> 1) & 3] = f2_add(sum2[(e >> 1) & 3], pp);
        const uint32_t h2 = pack2_hw<T>(p0, p1);
        phi[e >> 1] = h2;
        if constexpr (SPLIT) {
          // Low halves: P - round(P), exact in fp32, rounded once more.
          float d0, d1;
          f2_split(f2_sub(pp, f2(lo_half<T>(h2), hi_half<T>(h2))), d0, d1);
          plo[e >> 1] = pack2_hw<T>(d0, d1);
        }
      }
      {
        float a0, a1;
        f2_split(f2_add(f2_add(sum2[0], sum2[1]), f2_add(sum2[2], sum2[3])), a0, a1);
        lsum += a0 + a1;
      }
      sm100::tmem_st32(tmem + lane_base + b * BN + scol, phi);
      if constexpr (SPLIT) sm100::tmem_st32(tmem + lane_base + b * BN + scol + 32, plo);
      sm100::tmem_wait_st();
      sm100::tc_fence_before();
      sm100::mbar_arrive(p_full(b));
    }
    // Merge the two halves of each row: both threads of a row read (max, sum)
    // of both halves, then each produces HD output columns from both O halves.
    float w_self = 0.f, w_other = 0.f, lrow = 0.f, mrow = -INFINITY;
    if (ok) {
      red[(half * BM + row) * 2 + 0] = m_used;
      red[(half * BM + row) * 2 + 1] = lsum;
      sm100::mbar_arrive(red_bar);
      ok = __all_sync(0xffffffffu, sm100::mbar_wait(red_bar, 0, abort, err, ERR_RED, a.wait_limit));
      if (ok) {
        const float m_o = red[((half ^ 1) * BM + row) * 2 + 0];
        const float l_o = red[((half ^ 1) * BM + row) * 2 + 1];
        mrow = fmaxf(m_used, m_o);
        w_self = m_used == -INFINITY ? 0.f : ex2_approx(m_used - mrow);
        w_other = m_o == -INFINITY ? 0.f : ex2_approx(m_o - mrow);
        lrow = w_self * lsum + w_other * l_o;
      }
    }
    bool ready = ok && __all_sync(0xffffffffu, sm100::mbar_wait(pv_done((nblk - 1) & 1), ((nblk - 1) >> 1) & 1,
                                                                abort, err, ERR_PV_DONE, a.wait_limit));
    // One decision for all softmax warps (the staging below has a barrier).
    ready = sm100::bar_and_named(kEpilogueBar, kSoftmaxThreads, ready);
    if (ready) {
      sm100::tc_fence_after();
      // O columns [half*HD, half*HD+HD) of this row = w_self*O_self + w_other*O_other,
      // staged row-major in the K ring (idle: every K/V load landed before the
      // MMAs that read it, and the last P.V is done) so that the global writes
      // below are whole coalesced rows.
      const float w0 = half == 0 ? w_self : w_other;
      const float w1 = half == 0 ? w_other : w_self;
      const bool final_out = a.nchunks == 1;
      const float inv = final_out ? 1.0f / lrow : 1.0f;
      float* stage = reinterpret_cast<float*>(gbase + L::K_OFF);
#pragma unroll
      for (int c = 0; c < HD / 32; ++c) {
        uint32_t o0[32], o1[32];
        sm100::tmem_ld32(tmem + lane_base + TM_O + half * HD + c * 32, o0);
        sm100::tmem_ld32(tmem + lane_base + TM_O + D + half * HD + c * 32, o1);
        sm100::tmem_wait_ld();
        float* srow = stage + row * L::STAGE_STRIDE + half * HD + c * 32;
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          float4 v;
          v.x = (w0 * __uint_as_float(o0[q * 4 + 0]) + w1 * __uint_as_float(o1[q * 4 + 0])) * inv;
          v.y = (w0 * __uint_as_float(o0[q * 4 + 1]) + w1 * __uint_as_float(o1[q * 4 + 1])) * inv;
          v.z = (w0 * __uint_as_float(o0[q * 4 + 2]) + w1 * __uint_as_float(o1[q * 4 + 2])) * inv;
          v.w = (w0 * __uint_as_float(o0[q * 4 + 3]) + w1 * __uint_as_float(o1[q * 4 + 3])) * inv;
          *reinterpret_cast<float4*>(srow + q * 4) = v;
        }
      }
      const int64_t wu = (static_cast<int64_t>(h) * a.tiles + tile) * a.nchunks + chunk;
      if (!final_out && half == 0)
        *reinterpret_cast<float2*>(a.ws_ml + (wu * BM + row) * 2) = make_float2(mrow, lrow);
      sm100::bar_sync_named(kEpilogueBar, kSoftmaxThreads);
      // Copy-out: each warp writes whole rows, lane l the columns [l*D/32, (l+1)*D/32).
      constexpr int PER = D / 32;
      for (int rr = warp; rr < BM; rr += kSoftmaxThreads / 32) {
        const float* srow = stage + rr * L::STAGE_STRIDE + lane * PER;
        if (final_out) {
          const int64_t mr = m0 + rr;
          if (mr >= total_m) continue;
          const int64_t rw = mr / G;
          const int gw = static_cast<int>(mr - rw * G);
          uint16_t* dst = a.out + (rw * a.hq + static_cast<int64_t>(h) * G + gw) * D + lane * PER;
          if constexpr (PER == 4) {
            const float4 v = *reinterpret_cast<const float4*>(srow);
            *reinterpret_cast<uint2*>(dst) = make_uint2(pack2<T>(v.x, v.y), pack2<T>(v.z, v.w));
          } else {
            const float2 v = *reinterpret_cast<const float2*>(srow);
            *reinterpret_cast<uint32_t*>(dst) = pack2<T>(v.x, v.y);
          }
        } else {
          float* wo = a.ws_o + (wu * BM + rr) * D + lane * PER;
          if constexpr (PER == 4)
            *reinterpret_cast<float4*>(wo) = *reinterpret_cast<const float4*>(srow);
          else
            *reinterpret_cast<float2*>(wo) = *reinterpret_cast<const float2*>(srow);
        }
      }
    }
  }

  sm100::tc_fence_before();
  __syncthreads();
  // Every role has stopped; `abort` is final. After an abort, consumers may
  // have left copies unread: never leave the CTA while one of ours may still
  // land in shared memory. (Without an abort every copy was waited for.)
  if (*abort && nblk > 0 && warp == kTmaWarp && lane == 0) {
    volatile int keep_waiting = 0;
    if (a.q_by_tma) sm100::mbar_wait(q_full, 0, &keep_waiting, nullptr, 0, WAIT_LIMIT);
    for (int j = issued_k > NS ? issued_k - NS : 0; j < issued_k; ++j)
      sm100::mbar_wait(k_full(j % NS), (j / NS) & 1, &keep_waiting, nullptr, 0, WAIT_LIMIT);
    for (int j = issued_v > NS ? issued_v - NS : 0; j < issued_v; ++j)
      sm100::mbar_wait(v_full(j % NS), (j / NS) & 1, &keep_waiting, nullptr, 0, WAIT_LIMIT);
  }
  __syncthreads();
  if (warp == kMmaWarp) {
    sm100::tc_fence_after();
    sm100::tmem_dealloc(tmem, 512);
  }
}

// One warp per m-entry: O = sum_c 2^(m_c - M) O_c / sum_c 2^(m_c - M) l_c.
// Every chunk of the tile has a (max, sum) record (an empty chunk: max -inf,
// and no O, whose weight 0 skips it), so nothing here waits on the positions:
// lane c loads (m_c, l_c) of chunk c while the O rows of the first chunks are
// already in flight (lane l owns columns [l*D/32, (l+1)*D/32)); the warp
// reduces M and L with shuffles and takes each chunk's weight by shuffle. The
// chunk order of the sum is fixed, so the result is too.
// BATCH (chunks whose O rows are loaded together) is a template parameter:
// the launch picks the smallest of 4 and 16 that holds every chunk, so that
// few-chunk plans keep the registers, and the warps resident per SM, of a
// small batch.
template <class T, int D, int BATCH>
__global__ void __launch_bounds__(256) attn_combine_kernel(Args a) {
  pdl_launch_dependents();  // the next kernel may start its independent prologue
  pdl_wait();  // every input may come from the previous kernel
  constexpr int PER = D / 32;  // values per lane: 4 (D=128) or 2 (D=64)
  using Vec = typename std::conditional<PER == 4, float4, float2>::type;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int h = blockIdx.y;
  const int64_t m_abs = static_cast<int64_t>(blockIdx.x) * 8 + warp;
  const int G = a.group;
  const int64_t total_m = a.rows * G;
  if (m_abs >= total_m) return;
  const int tile = static_cast<int>(m_abs / BM);
  const int row = static_cast<int>(m_abs - static_cast<int64_t>(tile) * BM);
  const int nc = a.nchunks;
  const int64_t w0 = (static_cast<int64_t>(h) * a.tiles + tile) * nc;
  float M = -INFINITY, Lsum = 0.f, acc[PER];
#pragma unroll
  for (int e = 0; e < PER; ++e) acc[e] = 0.f;
  for (int c0 = 0; c0 < nc; c0 += 32) {
    const int cn = nc - c0 < 32 ? nc - c0 : 32;
    const float* o_base = a.ws_o + ((w0 + c0) * BM + row) * D + lane * PER;
    Vec ov[BATCH];
#pragma unroll
    for (int i = 0; i < BATCH; ++i)
      if (i < cn) ov[i] = *reinterpret_cast<const Vec*>(o_base + static_cast<int64_t>(i) * BM * D);
    const float2 ml = lane < cn ? *reinterpret_cast<const float2*>(a.ws_ml + ((w0 + c0 + lane) * BM + row) * 2)
                                : make_float2(-INFINITY, 0.f);
    float mb = ml.x;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mb = fmaxf(mb, __shfl_xor_sync(0xffffffffu, mb, o));
    mb = fmaxf(mb, M);
    const float keep = M == -INFINITY ? 0.f : exp2f(M - mb);  // rescale what earlier groups summed
    const float wgt = ml.x == -INFINITY ? 0.f : exp2f(ml.x - mb);
    float lw = wgt * ml.y;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) lw += __shfl_xor_sync(0xffffffffu, lw, o);
    Lsum = Lsum * keep + lw;
#pragma unroll
    for (int e = 0; e < PER; ++e) acc[e] *= keep;
    for (int b = 0; b < cn; b += BATCH) {
      if (b > 0) {
#pragma unroll
        for (int i = 0; i < BATCH; ++i)
          if (b + i < cn) ov[i] = *reinterpret_cast<const Vec*>(o_base + static_cast<int64_t>(b + i) * BM * D);
      }
#pragma unroll
      for (int i = 0; i < BATCH; ++i) {
        const float wi = __shfl_sync(0xffffffffu, wgt, (b + i) & 31);
        if (b + i < cn && wi != 0.f) {  // an empty chunk's O was never written
          const float* v = reinterpret_cast<const float*>(&ov[i]);
#pragma unroll
          for (int e = 0; e < PER; ++e) acc[e] += wi * v[e];
        }
      }
    }
    M = mb;
  }
  const float inv = 1.0f / Lsum;
  const int64_t r = m_abs / G;
  const int g = static_cast<int>(m_abs - r * G);
  uint16_t* dst = a.out + (r * a.hq + static_cast<int64_t>(h) * G + g) * D + lane * PER;
#pragma unroll
  for (int e = 0; e < PER; e += 2) *reinterpret_cast<uint32_t*>(dst + e) = pack2<T>(acc[e] * inv, acc[e + 1] * inv);
}

struct Plan {
  int tiles, nchunks;
  int64_t chunk;
  int64_t max_chunks;  // upper bound on nchunks for any max_position up to this one
};

inline Plan make_plan(int64_t rows, int hq, int hkv, int64_t max_position) {
  Plan p;
  const int64_t total_m = rows * (hq / hkv);
  p.tiles = static_cast<int>((total_m + BM - 1) / BM);
  const int64_t keys = max_position + 1;
  const int64_t blocks = (keys + BN - 1) / BN;
  const int64_t base = static_cast<int64_t>(p.tiles) * hkv;
  // One CTA per SM and a per-CTA prologue/epilogue of a few microseconds: with
  // few (head, tile) units, cut the key range into about one wave of chunks;
  // with many, use ~6 waves so that short and long causal spans balance out
  // (config-3 geometry, 352 units: 4/5/6/7/8/12/16 waves measured
  // 504-516/516/471-476/497/491/518/524 us per call). Chunks hold >= 4 key
  // blocks.
  const int64_t waves = base >= kNumSMs ? 6 : 1;
  int64_t cb = (base * blocks + waves * kNumSMs - 1) / (waves * kNumSMs);
  if (cb < 4) cb = 4;
  if (cb > blocks) cb = blocks;
  if (cb < 1) cb = 1;
  p.chunk = cb * BN;
  p.nchunks = static_cast<int>((blocks + cb - 1) / cb);
  // nchunks = ceil(blocks / cb) <= min(ceil(blocks / 4), ceil(waves * SMs / base)),
  // a bound that only grows with max_position: it sizes workspaces from cache_rows.
  int64_t bound = (waves * kNumSMs + base - 1) / base;
  const int64_t by_blocks = (blocks + 3) / 4;
  if (bound > by_blocks) bound = by_blocks;
  if (bound < p.nchunks) bound = p.nchunks;
  p.max_chunks = bound;
  return p;
}

// Partials are laid out with `stride_chunks` chunk slots per (head, tile).
inline size_t workspace_bytes(int tiles, int64_t chunks, int hkv, int head_dim) {
  size_t bytes = STATUS_BYTES;
  if (chunks > 1) {
    const size_t units = static_cast<size_t>(hkv) * tiles * chunks;
    bytes += units * BM * (head_dim + 2) * sizeof(float);
  }
  return bytes;
}

// ------------------------------------------------------------------ host side
using EncodeFn = PFN_cuTensorMapEncodeTiled_v12000;

inline EncodeFn encode_fn() {
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

// [kv_heads][cache_rows][D] with element strides (head, row); box 64 x 128 x 1.
inline bool make_kv_map(CUtensorMap* map, const void* ptr, bool bf16, int head_dim, int64_t rows,
                        int kv_heads, int64_t hs, int64_t rs) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(kv_heads)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(rs) * 2, static_cast<cuuint64_t>(hs) * 2};
  cuuint32_t box[3] = {64, BN, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

// Packed queries [rows][q_heads][D] seen as {D, q_heads, rows}; box 64 x G x 128/G
// covers the 128 m-entries (row, head of the group) of one tile.
inline bool make_q_map(CUtensorMap* map, const void* ptr, bool bf16, int head_dim, int q_heads, int64_t rows,
                       int group) {
  EncodeFn fn = encode_fn();
  if (!fn) return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(head_dim), static_cast<cuuint64_t>(q_heads),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(head_dim) * 2,
                           static_cast<cuuint64_t>(q_heads) * head_dim * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(group), static_cast<cuuint32_t>(BM / group)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = fn(map, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3,
                  const_cast<void*>(ptr), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS;
}

template <class T, int D, bool SPLIT>
int launch(const CUtensorMap& mk, const CUtensorMap& mv, const CUtensorMap& mq, const Args& a, cudaStream_t s,
           bool status_zeroed) {
  constexpr int smem = Layout<D, SPLIT>::BYTES;
  static int configured[64] = {0};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64 || !__atomic_load_n(&configured[dev], __ATOMIC_ACQUIRE)) {
    e = cudaFuncSetAttribute(attn_tc_kernel<T, D, SPLIT>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    if (dev >= 0 && dev < 64) __atomic_store_n(&configured[dev], 1, __ATOMIC_RELEASE);
  }
  if (!status_zeroed) {
    e = cudaMemsetAsync(a.status, 0, sizeof(int), s);
    if (e != cudaSuccess) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
  }
  dim3 grid(static_cast<unsigned>(a.tiles) * a.nchunks * a.hkv);
  int st = launch_pdl<attn_tc_kernel<T, D, SPLIT>>(grid, dim3(THREADS), smem, s, 1, mk, mv, mq, a);
  if (st != KVR_OK || a.nchunks == 1) return st;
  const int64_t total_m = a.rows * a.group;
  const dim3 cgrid(static_cast<unsigned>((total_m + 7) / 8), a.hkv);
  if (a.nchunks <= 4) return launch_pdl<attn_combine_kernel<T, D, 4>>(cgrid, dim3(256), 0, s, 1, a);
  return launch_pdl<attn_combine_kernel<T, D, 16>>(cgrid, dim3(256), 0, s, 1, a);
}

}  // namespace attn
}  // namespace kvr

using namespace kvr;

extern "C" {

size_t kvr_attention_workspace_size(int64_t rows, int q_heads, int kv_heads, int head_dim,
                                    int64_t cache_rows) {
  if (rows <= 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || cache_rows <= 0)
    return attn::STATUS_BYTES;
  attn::Plan p = attn::make_plan(rows, q_heads, kv_heads, cache_rows - 1);
  return attn::workspace_bytes(p.tiles, p.max_chunks, kv_heads, head_dim);
}

int kvr_selected_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                           const int64_t* positions, int64_t rows, int q_heads, int kv_heads,
                           int head_dim, int64_t cache_rows, int64_t cache_head_stride,
                           int64_t cache_row_stride, int64_t max_position, float scale,
                           int precision, void* workspace, size_t workspace_bytes, int dtype,
                           void* stream) {
  return kvr::selected_attention(q, k_cache, v_cache, out, positions, rows, q_heads, kv_heads, head_dim, cache_rows,
                                 cache_head_stride, cache_row_stride, max_position, scale, precision, workspace,
                                 workspace_bytes, dtype, stream, false);
}

}  // extern "C"

namespace kvr {

int selected_attention(const void* q, const void* k_cache, const void* v_cache, void* out,
                       const int64_t* positions, int64_t rows, int q_heads, int kv_heads, int head_dim,
                       int64_t cache_rows, int64_t cache_head_stride, int64_t cache_row_stride,
                       int64_t max_position, float scale, int precision, void* workspace, size_t workspace_bytes,
                       int dtype, void* stream, bool status_zeroed) {
  if (dtype != KVR_DTYPE_BF16 && dtype != KVR_DTYPE_F16) return KVR_ERR_UNSUPPORTED;
  if (head_dim != 64 && head_dim != 128) return KVR_ERR_UNSUPPORTED;
  if (precision != KVR_ATTN_P_SPLIT && precision != KVR_ATTN_P_ROUNDED) return KVR_ERR_INVALID_ARG;
  if (rows < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || cache_rows < 0)
    return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  if (!q || !k_cache || !v_cache || !out || !positions || !aligned16(q) || !aligned16(k_cache) ||
      !aligned16(v_cache) || !aligned16(out) || cache_head_stride % 8 || cache_row_stride % 8)
    return KVR_ERR_INVALID_ARG;
  if (max_position < 0 || max_position >= cache_rows || !(scale == scale)) return KVR_ERR_INVALID_ARG;
  if (cache_rows > 0x7fffffffLL || kv_heads > 65535) return KVR_ERR_UNSUPPORTED;
  attn::Plan p = attn::make_plan(rows, q_heads, kv_heads, max_position);
  if (static_cast<int64_t>(p.tiles) * p.nchunks * kv_heads > 0x7fffffff) return KVR_ERR_UNSUPPORTED;
  const size_t need = attn::workspace_bytes(p.tiles, p.nchunks, kv_heads, head_dim);
  if (!workspace || workspace_bytes < need || !aligned16(workspace)) return KVR_ERR_INVALID_ARG;
  const bool bf16 = dtype == KVR_DTYPE_BF16;
  CUtensorMap mk, mv, mq;
  if (!attn::make_kv_map(&mk, k_cache, bf16, head_dim, cache_rows, kv_heads, cache_head_stride,
                         cache_row_stride) ||
      !attn::make_kv_map(&mv, v_cache, bf16, head_dim, cache_rows, kv_heads, cache_head_stride,
                         cache_row_stride))
    return KVR_ERR_UNSUPPORTED;
  const int group = q_heads / kv_heads;
  // Q by TMA when the tile's 128 m-entries are whole rows x group heads.
  const bool q_by_tma = group <= attn::BM && attn::BM % group == 0 &&
                        attn::make_q_map(&mq, q, bf16, head_dim, q_heads, rows, group);
  if (!q_by_tma) mq = mk;  // unused placeholder
  attn::Args a;
  a.q_by_tma = q_by_tma ? 1 : 0;
  a.q = static_cast<const uint16_t*>(q);
  a.out = static_cast<uint16_t*>(out);
  a.positions = positions;
  a.rows = rows;
  a.hq = q_heads;
  a.hkv = kv_heads;
  a.group = q_heads / kv_heads;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.tiles = p.tiles;
  a.nchunks = p.nchunks;
  a.chunk = p.chunk;
  a.status = static_cast<int*>(workspace);
  a.wait_limit = pipeline_wait_limit();
  a.ws_o = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + attn::STATUS_BYTES);
  const size_t units = static_cast<size_t>(kv_heads) * p.tiles * p.nchunks;
  a.ws_ml = a.ws_o + units * attn::BM * head_dim;
  auto s = static_cast<cudaStream_t>(stream);
  const bool split = precision == KVR_ATTN_P_SPLIT;
  if (bf16) {
    if (head_dim == 128)
      return split ? attn::launch<BF16, 128, true>(mk, mv, mq, a, s, status_zeroed) : attn::launch<BF16, 128, false>(mk, mv, mq, a, s, status_zeroed);
    return split ? attn::launch<BF16, 64, true>(mk, mv, mq, a, s, status_zeroed) : attn::launch<BF16, 64, false>(mk, mv, mq, a, s, status_zeroed);
  }
  if (head_dim == 128)
    return split ? attn::launch<F16, 128, true>(mk, mv, mq, a, s, status_zeroed) : attn::launch<F16, 128, false>(mk, mv, mq, a, s, status_zeroed);
  return split ? attn::launch<F16, 64, true>(mk, mv, mq, a, s, status_zeroed) : attn::launch<F16, 64, false>(mk, mv, mq, a, s, status_zeroed);
}

}  // namespace kvr

extern "C" {

// ---------------------------------------------------------------------------
// No-allocation variant. Some callers cannot allocate device memory per call:
// a host runtime that reaches this library over a plain C FFI with a fixed,
// pre-planned GPU memory budget and no caching allocator, for which a
// cudaMalloc would synchronise the device and fragment its pool. For them the
// split-KV partials live in one file-scope device array of fixed size,
// reserved on every GPU that loads the library for the life of the process.
// ---------------------------------------------------------------------------
static __device__ __align__(256) uint8_t g_attention_scratch[KVR_STATIC_SCRATCH_BYTES];

namespace {

// Device address of g_attention_scratch, looked up once per device with that
// device current (host code cannot use the symbol itself as a pointer).
void* g_scratch_ptr[64] = {nullptr};
int g_scratch_ready[64] = {0};

int scratch_address(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  if (dev < 0 || dev >= 64) return KVR_ERR_UNSUPPORTED;
  if (!__atomic_load_n(&g_scratch_ready[dev], __ATOMIC_ACQUIRE)) {
    void* ptr = nullptr;
    e = cudaGetSymbolAddress(&ptr, g_attention_scratch);
    if (e != cudaSuccess || !ptr) {
      set_last_cuda_error(e);
      return KVR_ERR_CUDA;
    }
    g_scratch_ptr[dev] = ptr;  // identical value from any racing thread
    __atomic_store_n(&g_scratch_ready[dev], 1, __ATOMIC_RELEASE);
  }
  *out = g_scratch_ptr[dev];
  return KVR_OK;
}

}  // namespace

int kvr_selected_attention_static(const void* q, const void* k_cache, const void* v_cache, void* out,
                                  const int64_t* positions, int64_t rows, int q_heads, int kv_heads,
                                  int head_dim, int64_t cache_rows, int64_t cache_head_stride,
                                  int64_t cache_row_stride, int64_t max_position, float scale, int precision,
                                  int dtype, void* stream) {
  if (rows < 0 || q_heads <= 0 || kv_heads <= 0 || q_heads % kv_heads || cache_rows < 0 || max_position < 0)
    return KVR_ERR_INVALID_ARG;
  if (rows == 0) return KVR_OK;
  const attn::Plan p = attn::make_plan(rows, q_heads, kv_heads, max_position);
  if (attn::workspace_bytes(p.tiles, p.nchunks, kv_heads, head_dim) > KVR_STATIC_SCRATCH_BYTES)
    return KVR_ERR_SCRATCH_LIMIT;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != KVR_OK) return st;
  return kvr_selected_attention(q, k_cache, v_cache, out, positions, rows, q_heads, kv_heads, head_dim,
                                cache_rows, cache_head_stride, cache_row_stride, max_position, scale, precision,
                                scratch, KVR_STATIC_SCRATCH_BYTES, dtype, stream);
}

// The status word of the last kvr_selected_attention_static call on the
// current device, copied on `stream` (one 4-byte cudaMemcpyAsync, no
// allocation) into `status_out`, which may be host or device memory; the
// value is there once the stream has reached the copy.
int kvr_attention_static_status(int* status_out, void* stream) {
  if (!status_out) return KVR_ERR_INVALID_ARG;
  void* scratch = nullptr;
  const int st = scratch_address(&scratch);
  if (st != KVR_OK) return st;
  const cudaError_t e =
      cudaMemcpyAsync(status_out, scratch, sizeof(int), cudaMemcpyDefault, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    set_last_cuda_error(e);
    return KVR_ERR_CUDA;
  }
  return KVR_OK;
}

}  // extern "C"
