// fp32 backward, second stage of the GEMM route: dQ, dK and dV as plain
// 3xTF32 GEMMs over the score-shaped gradients the score pass materialised
// (tf32_scores.cuh):
//
//   dQ[b] = scale * dS[b] K[b]        M = S_q rows,  K-dim = S_kv
//   dK[b] = scale * dS[b]^T Q[b]      M = S_kv rows, K-dim = S_q (dS read MN-major)
//   dV[b] =         P~[b]^T dO[b]     M = S_kv rows, K-dim = S_q (P~ read MN-major)
//
// with dS = P (kf dP - D) and P~ = kf P, exactly the matrices the reference's
// dQ and dK/dV kernels form element by element (sdpa/sdpa_bwd.cu.cc:125-170).
// Recomputing them per pass (S, dP for dQ and dK; S for dV) costs the fp32
// path more tensor time than reading them back: every recomputed product is
// three tf32 MMAs, and with hi / lo operands resident the recomputing passes
// only fit N = 32 tiles in TMEM, where a tf32 MMA runs at half its rate.
//
// A work item = 128 rows of the result, all N columns; persistent CTAs take
// items in turn (below).  Streams K-dim tiles of kK = 64 (32 at N = 128):
// the A tile (128 x 32) and the B tile (32 x N, MN-major, 32-byte swizzle
// atoms) by TMA.  Four converter warps split A row by row into tf32 hi / lo
// in TMEM and B in place in shared memory; one thread issues kK / 8 x 3 TS MMAs
// per tile (A from TMEM: only B is read from shared memory, whose bandwidth
// bounded the all-shared-memory form) into one of two TMEM accumulators,
// which 8 epilogue warps fold into an fp32 running total every tile (the
// tensor cores' accumulation is not round-to-nearest).
// Causal ranges: dQ row tile m0 needs keys < m0 + 128, dK / dV row tile m0
// queries >= m0; every entry inside those ranges was written (masked ones as
// zero).
#pragma once
#include "common.cuh"
#include "fwd_tc.cuh"
#include "ptx.cuh"
#include "tf32_fwd.cuh"

namespace sdpa_b200 {
namespace tf32 {

constexpr int kGemmThreads = 448;

// Timing probe for tuning builds (-DSDPA_B200_TF32_PROBE=3
// -DSDPA_B200_GEMM_PROBE_N=<N>): SM cycles of CTA 0's roles, as in the passes.
#if defined(SDPA_B200_TF32_PROBE) && defined(SDPA_B200_GEMM_PROBE_N)
#define GEMM_PROBE_T0(v) const long long v = clock64()
#define GEMM_PROBE_ADD(slot, t0)                                      \
  if (blockIdx.x == 0 && N == SDPA_B200_GEMM_PROBE_N) \
  atomicAdd(&g_tf32_probe[slot], static_cast<unsigned long long>(clock64() - (t0)))
#else
#define GEMM_PROBE_T0(v)
#define GEMM_PROBE_ADD(slot, t0)
#endif

struct GemmArgs {
  float* c;          // result [B/H, M, H, D] (H = 1: [B, M, D])
  int64_t B, H, M, K;
  int D;             // result columns (<= N)
  float alpha;
  int range;         // 0: whole K-dim, 1: K-dim < m0 + 128 (dQ, causal), 2: K-dim >= m0 (dK, dV, causal)
  uint64_t timeout_ns;
};

#ifndef SDPA_B200_GEMM_K
#define SDPA_B200_GEMM_K 64
#endif
template <int N>
struct GemmCfg {
  // K-dim per tile (kK / 32 boxes of 128-byte rows): 64 halves the per-tile
  // hand-offs (cfg5 dQ 0.43 -> 0.37 ms, dK 0.39 -> 0.34); at N = 128 it
  // leaves TMEM and shared memory two stages only, and 32 with four measured
  // as fast (dV 0.51 / 0.52 ms)
  static constexpr int kK = N >= 128 ? 32 : SDPA_B200_GEMM_K;
  static_assert(kK == 32 || kK == 64, "K tile");
  static constexpr uint32_t kABytes = 128 * kK * 4;      // 16 or 32 KB
  static constexpr uint32_t kBBytes = kK * N * 4;        // N / 32 boxes of 32 columns x kK
  static constexpr uint32_t kStageBytes = kABytes + 2 * kBBytes;  // raw A, B hi, B lo
  // TMEM: two accumulators (N columns each), then per stage A hi, A lo (kK each)
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kAslot0 = 2 * N;
  static constexpr int kSmemStages = 200 * 1024 / kStageBytes;
  static constexpr int kTmemStages = (512 - 2 * N) / (2 * kK);
  static constexpr int kStages = kSmemStages < kTmemStages ? (kSmemStages < 4 ? kSmemStages : 4)
                                                           : (kTmemStages < 4 ? kTmemStages : 4);
  static_assert(kStages >= 2, "pipeline depth");
  static constexpr uint32_t kBarOff = kStages * kStageBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kAslot0 + kStages * 2 * kK <= kTmemCols, "TMEM budget");
  static constexpr int kHC = N / 2;                      // columns per epilogue thread
  static_assert(N == 32 || N == 64 || N == 128, "N");
  static_assert(kSmemBytes <= 232448, "shared memory");
  static __device__ __forceinline__ uint32_t a_raw(int s) { return s * kStageBytes; }
  static __device__ __forceinline__ uint32_t b_hi(int s) { return s * kStageBytes + kABytes; }
  static __device__ __forceinline__ uint32_t b_lo(int s) { return s * kStageBytes + kABytes + kBBytes; }
};

struct GemmBarriers {
  uint64_t st_full[4], st_ready[4], st_empty[4];
  uint64_t acc_full[2], acc_empty[2];
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

template <int N>
__device__ __forceinline__ void gemm_tmem_ld(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 16) {
    SDPA_TMEM_LD16(taddr, r);
  } else {
    SDPA_TMEM_LD32(taddr, r);
  }
}

// One work item = 128 result rows of one batch row: its K-dim tiles [tile0,
// tile0 + n) (causal ranges) and its TMA coordinates.
struct GemmItem {
  int64_t b, m0;
  int hb, ob, tile0, n;
};
template <bool HEADS>
__device__ __forceinline__ GemmItem gemm_item(const GemmArgs& g, int64_t item, int kK) {
  GemmItem it;
  const int64_t n_mt = (g.M + 127) / 128;
  int64_t tord;
  raster(item, g.B, n_mt, it.b, tord);
  it.hb = HEADS ? static_cast<int>(it.b % g.H) : 0;
  it.ob = HEADS ? static_cast<int>(it.b / g.H) : static_cast<int>(it.b);
  // heaviest causal row tiles first: high ones for dQ, low ones for dK / dV
  it.m0 = (g.range == 1 ? n_mt - 1 - tord : tord) * 128;
  const int64_t n_all = (g.K + kK - 1) / kK;
  it.tile0 = 0;
  it.n = static_cast<int>(n_all);
  if (g.range == 1) {
    it.n = static_cast<int>(min(n_all, (it.m0 + 127) / kK + 1));
  } else if (g.range == 2) {
    it.tile0 = static_cast<int>(it.m0 / kK);
    it.n = static_cast<int>(n_all - it.tile0 > 0 ? n_all - it.tile0 : 0);
  }
  return it;
}

// Persistent: CTA c takes work items c, c + gridDim.x, ... (heaviest first),
// and every role runs one continuous pipeline over the concatenated K-dim
// tiles of its items (index q), so a short item (dK / dV: 16 tiles at cfg5)
// does not pay the pipeline's fill and drain, and the epilogue of one item
// overlaps the next item's loads and MMAs.
// tm_a: 3-D map of the materialised matrix: K-major (A_MN false: K-dim
// innermost, kK / 32 boxes of 32 x 128 rows, 128-byte swizzle) or MN-major (A_MN
// true: the stored matrix is A^T, rows innermost, boxes of 32 rows x kK K-dim with 32-byte
// atoms; dK and dV read dS and P~ this way).  tm_b: MN-major map of K, Q or
// dO, box 32 columns x kK K-dim.
template <int N, bool HEADS, bool A_MN>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tm_a, const __grid_constant__ CUtensorMap tm_b, const GemmArgs g) {
  using Cfg = GemmCfg<N>;
  constexpr int kK = Cfg::kK, kStages = Cfg::kStages, kHC = Cfg::kHC;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc::align1024(smem_raw);
  GemmBarriers* bars = reinterpret_cast<GemmBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int64_t n_items = ((g.M + 127) / 128) * g.B;
  int n_tiles = 0;  // K-dim tiles of all this CTA's items
  for (int64_t item = blockIdx.x; item < n_items; item += gridDim.x) n_tiles += gemm_item<HEADS>(g, item, kK).n;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_ready[s], 128);
      mbar_init(&bars->st_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->acc_full[s], 1);
      mbar_init(&bars->acc_empty[s], 256);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 13) tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // before any global access and before the wait deadline starts
  const uint32_t tmem = bars->tmem_base;
  WaitCtl ctl;
  ctl.deadline_ns = globaltimer_ns() + g.timeout_ns;
  ctl.abort_flag = &bars->abort_flag;

  if (warp == 12) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&tm_a);
      tma_prefetch_desc(&tm_b);
      int q = 0;  // tiles issued
      bool ok = true;
      for (int64_t item = blockIdx.x; ok && item < n_items; item += gridDim.x) {
        const GemmItem it = gemm_item<HEADS>(g, item, kK);
        for (int t = 0; t < it.n; ++t, ++q) {
          ctl.deadline_ns = globaltimer_ns() + g.timeout_ns;  // per tile: a persistent CTA may run long
          const int s = q % kStages;
          GEMM_PROBE_T0(p0);
          if (!mbar_wait(&bars->st_empty[s], ((q / kStages) & 1) ^ 1, ctl)) {
            ok = false;
            break;
          }
          GEMM_PROBE_ADD(8, p0);
          const int k0 = (it.tile0 + t) * kK;
          mbar_expect_tx(&bars->st_full[s], Cfg::kABytes + Cfg::kBBytes);
          if (A_MN) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              tma_load_3d(smem + Cfg::a_raw(s) + c * kK * 128, &tm_a, static_cast<int>(it.m0) + c * 32, k0,
                          static_cast<int>(it.b), &bars->st_full[s]);
          } else {
#pragma unroll
            for (int c = 0; c < kK / 32; ++c)
              tma_load_3d(smem + Cfg::a_raw(s) + c * (128 * 128), &tm_a, k0 + c * 32, static_cast<int>(it.m0),
                          static_cast<int>(it.b), &bars->st_full[s]);
          }
#pragma unroll
          for (int c = 0; c < N / 32; ++c)
            tma_load_rows(smem + Cfg::b_hi(s) + c * kK * 128, &tm_b, c * 32, k0, it.hb, it.ob, &bars->st_full[s],
                          HEADS);
        }
      }
      if (*ctl.abort_flag) {  // let the copies in flight land before the CTA exits
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + g.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        for (int t = (q > kStages ? q - kStages : 0); t < q; ++t)
          mbar_wait(&bars->st_full[t % kStages], (t / kStages) & 1, drain);
      }
    }
  } else if (warp == 13) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0) {
      const uint32_t sb = smem_u32(smem);
      constexpr uint32_t idesc = make_idesc(128, N, false, true, true);  // A from TMEM
      for (int q = 0; q < n_tiles; ++q) {
        ctl.deadline_ns = globaltimer_ns() + g.timeout_ns;
        const int s = q % kStages, ab = q & 1;
        // accumulator ab was folded by the epilogue (its use q - 2)
        GEMM_PROBE_T0(w0);
        if (q >= 2 && !mbar_wait(&bars->acc_empty[ab], ((q >> 1) - 1) & 1, ctl)) break;
        GEMM_PROBE_ADD(0, w0);
        GEMM_PROBE_T0(w1);
        if (!mbar_wait(&bars->st_ready[s], (q / kStages) & 1, ctl)) break;
        GEMM_PROBE_ADD(1, w1);
        GEMM_PROBE_T0(w2);
        tc_fence_after();
        const uint32_t acc = tmem + ab * N;
        const uint32_t ah = tmem + Cfg::kAslot0 + s * 2 * kK, al = ah + kK;
#pragma unroll
        for (int kk = 0; kk < kK / 8; ++kk) {
          const uint64_t bh = make_sw128_32b_desc(sb + Cfg::b_hi(s) + kk * 1024, kK * 128, 512);
          const uint64_t bl = make_sw128_32b_desc(sb + Cfg::b_lo(s) + kk * 1024, kK * 128, 512);
          mma_tf32_ts(acc, ah + kk * 8, bh, idesc, kk > 0 ? 1u : 0u);  // a fresh accumulator every tile
          mma_tf32_ts(acc, ah + kk * 8, bl, idesc, 1u);
          mma_tf32_ts(acc, al + kk * 8, bh, idesc, 1u);
        }
        mma_commit(&bars->st_empty[s]);
        mma_commit(&bars->acc_full[ab]);
        GEMM_PROBE_ADD(2, w2);
      }
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + g.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------- converters
    // Thread tid owns A row tid (= its warp's TMEM lane quarter): it splits the
    // row's 32 K-dim values into TMEM, where the MMAs read A (sparing shared-
    // memory bandwidth); all 128 split the B tile in place.  (Splitting B in
    // the epilogue warps instead measured no faster.)
    const int tid = threadIdx.x - 256;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    for (int q = 0; q < n_tiles; ++q) {
      ctl.deadline_ns = globaltimer_ns() + g.timeout_ns;
      const int s = q % kStages;
      GEMM_PROBE_T0(c0);
      if (!tc::warp_wait(&bars->st_full[s], (q / kStages) & 1, ctl)) break;
      if (tid == 0) GEMM_PROBE_ADD(6, c0);
      GEMM_PROBE_T0(c1);
      const uint8_t* a = smem + Cfg::a_raw(s);
      const uint32_t ta = tmem + lane_base + Cfg::kAslot0 + s * 2 * kK;
#pragma unroll
      for (int kh = 0; kh < kK / 32; ++kh) {  // 32 K-dim values of the row at a time
        uint32_t h[32], l[32];
        if (A_MN) {  // box tid / 32, element tid % 32 of each 128-byte K row (32-byte atoms, XOR row & 3)
          const uint8_t* box = a + (tid >> 5) * (kK * 128) + ((lane & 7) << 2);
#pragma unroll
          for (int k0 = 0; k0 < 32; ++k0) {
            const int k = kh * 32 + k0;
            float hi, lo;
            split_tf32(*reinterpret_cast<const float*>(box + k * 128 + (((lane >> 3) ^ (k & 3)) << 5)), hi, lo);
            h[k0] = __float_as_uint(hi);
            l[k0] = __float_as_uint(lo);
          }
        } else {  // box kh, row tid: 16-byte chunk j at chunk j ^ (row & 7) (128-byte swizzle)
          const uint8_t* row = a + kh * (128 * 128) + tid * 128;
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const float4 x = *reinterpret_cast<const float4*>(row + ((j ^ (tid & 7)) << 4));
            const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              float hi, lo;
              split_tf32(xv[e], hi, lo);
              h[4 * j + e] = __float_as_uint(hi);
              l[4 * j + e] = __float_as_uint(lo);
            }
          }
        }
        SDPA_TMEM_ST32(ta + kh * 32, h);
        SDPA_TMEM_ST32(ta + kK + kh * 32, l);
      }
      split_tile(smem + Cfg::b_hi(s), smem + Cfg::b_lo(s), Cfg::kBBytes, tid, 128);
      tmem_wait_st();
      fence_proxy_async_smem();
      tc_fence_before();
      if (tid == 0) GEMM_PROBE_ADD(7, c1);
      mbar_arrive(&bars->st_ready[s]);
    }
  } else {
    // ---------------------------------------------------- epilogue warps
    // Tile q's accumulator is folded into the running total of its item; the
    // item's rows are written after its last tile.
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    int64_t f_item = blockIdx.x;  // the item being folded, and its next tile
    GemmItem f_it = gemm_item<HEADS>(g, f_item < n_items ? f_item : 0, kK);
    int f_t = 0;
    float tot[kHC];
#pragma unroll
    for (int e = 0; e < kHC; ++e) tot[e] = 0.0f;
    for (int qf = 0; qf < n_tiles; ++qf) {
      ctl.deadline_ns = globaltimer_ns() + g.timeout_ns;
      const int ab = qf & 1;
      GEMM_PROBE_T0(e0);
      if (!tc::warp_wait(&bars->acc_full[ab], (qf >> 1) & 1, ctl)) break;
      if (threadIdx.x == 0) GEMM_PROBE_ADD(4, e0);
      GEMM_PROBE_T0(e1);
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < (kHC + 31) / 32; ++c) {
        constexpr int W = kHC < 32 ? kHC : 32;
        uint32_t a[W];
        gemm_tmem_ld<W>(tmem + lane_base + ab * N + half * kHC + c * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < W; ++e) tot[c * 32 + e] += __uint_as_float(a[e]);
      }
      tc_fence_before();
      if (threadIdx.x == 0) GEMM_PROBE_ADD(5, e1);
      mbar_arrive(&bars->acc_empty[ab]);
      if (++f_t < f_it.n) continue;
      // last tile of the item: its rows (every item has n >= 1: K >= 1, and the
      // causal ranges start at or before the row tile's diagonal)
      const int64_t m = f_it.m0 + r;
      if (m < g.M) {
        float* crow = g.c + row_offset_t<HEADS>(g.H, f_it.b, m, g.M, g.D);
#pragma unroll
        for (int c4 = 0; c4 < kHC / 4; ++c4) {
          const int col = half * kHC + 4 * c4;
          if (col < g.D)
            *reinterpret_cast<float4*>(crow + col) =
                make_float4(tot[4 * c4] * g.alpha, tot[4 * c4 + 1] * g.alpha, tot[4 * c4 + 2] * g.alpha,
                            tot[4 * c4 + 3] * g.alpha);
        }
      }
#pragma unroll
      for (int e = 0; e < kHC; ++e) tot[e] = 0.0f;
      f_item += gridDim.x;
      if (f_item < n_items) f_it = gemm_item<HEADS>(g, f_item, kK);
      f_t = 0;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// D_i = rowsum(dO_i * O_i) - dstats_i for every query row (the DQ pass of the
// recomputing route computes it in its prologue): one warp per row.
template <bool HEADS>
__global__ void __launch_bounds__(256) delta_kernel(const Params p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= p.B * p.S_q) return;
  const int64_t b = row / p.S_q, i = row - b * p.S_q;
  const float* orow = static_cast<const float*>(p.o) + row_offset_t<HEADS>(p.H, b, i, p.S_q, p.D_v);
  const float* grow = static_cast<const float*>(p.d_o) + row_offset_t<HEADS>(p.H, b, i, p.S_q, p.D_v);
  float acc = 0.0f;
  for (int c = 4 * lane; c < p.D_v; c += 128) {
    const float4 o4 = *reinterpret_cast<const float4*>(orow + c);
    const float4 g4 = *reinterpret_cast<const float4*>(grow + c);
    acc = fmaf(g4.x, o4.x, acc);
    acc = fmaf(g4.y, o4.y, acc);
    acc = fmaf(g4.z, o4.z, acc);
    acc = fmaf(g4.w, o4.w, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if (lane == 0) p.delta[row] = p.d_stats ? acc - p.d_stats[row] : acc;
}

}  // namespace tf32
}  // namespace sdpa_b200
