// fp32 backward, first stage of the GEMM route: the score pass.  One CTA =
// 128 key rows j of one batch row, K and V (tf32 hi / lo) resident in TMEM;
// streams query tiles i (Q, dO, lse, D) and per tile
//
//   S^T = K Q^T, dP^T = V dO^T          (TS MMAs, 3xTF32, into one TMEM buffer)
//   P~ = kf p, dS = p (kf dP - D)       (8 elementwise warps; p = exp(S - lse))
//
// and writes dS and P~, both [B, S_q, ld_k], to the workspace,
// where the three GEMMs of tf32_gemm.cuh turn them into dQ, dK and dV.  The
// elementwise formulas, skip rule (p <= 1e-6) and dropout counters are the
// reference's dK/dV kernel's (sdpa/sdpa_bwd.cu.cc:125-170), as in the passes
// of tf32_bwd.cuh.  Without an accumulator or dS operand in TMEM, the tile is
// 64 query rows wide (against 32 in the recomputing DK pass; 32 again with
// both D at 128): half as many MMA instructions per score, each at a better
// rate.  The elementwise warps
// read S^T / dP^T into registers and release the buffer at once, so the next
// tile's MMAs run under this tile's elementwise work.
//
// Roles: warps 0-7 elementwise (warp w: TMEM lanes 32*(w%4).., column half
// w/4), 8-11 split each streamed tile into hi / lo and stage lse / D, warp 12
// TMA, warp 13 MMA issuer + TMEM owner.
#pragma once
#include "common.cuh"
#include "fwd_tc.cuh"
#include "ptx.cuh"
#include "tf32_bwd.cuh"
#include "tf32_fwd.cuh"

namespace sdpa_b200 {
namespace tf32 {

constexpr int kScoreThreads = 448;

// Timing probe for tuning builds (-DSDPA_B200_TF32_PROBE=4): SM cycles of
// CTA 0's roles, as in the passes.
#if defined(SDPA_B200_TF32_PROBE) && SDPA_B200_TF32_PROBE == 4
#define SCORE_PROBE_T0(v) const long long v = clock64()
#define SCORE_PROBE_ADD(slot, t0) \
  if (blockIdx.x == 0) atomicAdd(&g_tf32_probe[slot], static_cast<unsigned long long>(clock64() - (t0)))
#else
#define SCORE_PROBE_T0(v)
#define SCORE_PROBE_ADD(slot, t0)
#endif

template <int DQK, int DV>
struct ScoreCfg {
  // TMEM columns: K hi / lo, V hi / lo, then S^T (kN) and dP^T (kN).  With
  // both D at 128 that leaves no room for a tile: V lo moves to shared memory
  // (kVlSmem; its product with dO hi becomes an SS MMA) and tiles are 32 rows.
  static constexpr bool kVlSmem = 2 * DQK + 2 * DV + 2 * 32 > 512;
  static constexpr uint32_t kKh = 0, kKl = DQK, kVh = 2 * DQK, kVl = 2 * DQK + DV;  // kVl: TMEM (unless kVlSmem)
  static constexpr uint32_t kT = 2 * DQK + (kVlSmem ? 1 : 2) * DV;
  static constexpr int kN = !kVlSmem && (512 - static_cast<int>(kT)) / 2 >= 64 ? 64 : 32;  // query rows per tile
  static constexpr int kHalf = kN / 2;
  static_assert(kT + 2 * kN <= 512, "TMEM budget");
  // shared memory per stage: Q hi, Q lo (kN x DQK), dO hi, dO lo (kN x DV),
  // K-major with 128-byte swizzle.  lse (log2 units) and D of a tile's kN
  // rows sit in a separate ring of kVecSlots, so that a stage is free for the
  // next load as soon as its MMAs complete, while the elementwise warps still
  // read the tile's lse / D.
  static constexpr uint32_t kQBytes = kN * DQK * 4, kOBytes = kN * DV * 4;
  static constexpr uint32_t kStageBytes = 2 * kQBytes + 2 * kOBytes;
  static constexpr uint32_t kStageAligned = (kStageBytes + 1023) / 1024 * 1024;
  static constexpr uint32_t kVlBytes = kVlSmem ? 128 * DV * 4 : 0;  // K-major, 128-byte swizzle
  static constexpr int kStages = 3 * kStageAligned + kVlBytes <= 200 * 1024 ? 3 : 2;
  static constexpr int kVecSlots = 4;
  static constexpr uint32_t kVlOff = kStages * kStageAligned;
  static constexpr uint32_t kVecOff = kVlOff + kVlBytes;
  static constexpr uint32_t kBarOff = kVecOff + kVecSlots * 2 * kN * 4;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory");
  static __device__ __forceinline__ uint32_t q_hi(int s) { return s * kStageAligned; }
  static __device__ __forceinline__ uint32_t q_lo(int s) { return s * kStageAligned + kQBytes; }
  static __device__ __forceinline__ uint32_t o_hi(int s) { return s * kStageAligned + 2 * kQBytes; }
  static __device__ __forceinline__ uint32_t o_lo(int s) { return s * kStageAligned + 2 * kQBytes + kOBytes; }
  static __device__ __forceinline__ uint32_t vec(int v) { return kVecOff + v * 2 * kN * 4; }
};

struct ScoreBarriers {
  uint64_t res_ready;
  uint64_t st_full[3], st_ready[3], st_empty[3];
  uint64_t vec_full[4], vec_empty[4];
  uint64_t s_full, t_free;
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

// issue_scores (tf32_bwd.cuh) with the A lo operand in shared memory (128
// rows, K-major, 128-byte swizzle, boxes of 32 columns): out = A B^T.
template <int D, int kN>
__device__ __forceinline__ void issue_scores_lo_smem(uint32_t out, uint32_t ah, uint32_t al_smem, uint32_t bh,
                                                     uint32_t bl) {
  constexpr uint32_t idesc = make_idesc(128, kN, false, false, true);
#pragma unroll
  for (int kk = 0; kk < D / 8; ++kk) {
    const uint32_t off = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
    const uint64_t dh = make_sw128_desc(bh + off, 16, 1024);
    const uint64_t dl = make_sw128_desc(bl + off, 16, 1024);
    const uint64_t da = make_sw128_desc(al_smem + (kk >> 2) * (128 * 128) + (kk & 3) * 32, 16, 1024);
    mma_tf32_ts(out, ah + kk * 8, dh, idesc, kk > 0 ? 1u : 0u);
    mma_tf32_ts(out, ah + kk * 8, dl, idesc, 1u);
    mma_tf32_ss(out, da, dh, idesc, 1u);
  }
}

// tm_q: Q [B/H, S_q, H, D_qk], tm_o: dO [B/H, S_q, H, D_v], both box 32 x kN.
template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kScoreThreads, 1)
    score_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_o, const Params p) {
  using Cfg = ScoreCfg<DQK, DV>;
  constexpr int kN = Cfg::kN, kHalf = Cfg::kHalf, kStages = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc::align1024(smem_raw);
  ScoreBarriers* bars = reinterpret_cast<ScoreBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;

  int64_t b, kt;  // low key tiles see the most causal query rows: issued first
  raster(blockIdx.x, p.B, (p.S_kv + 127) / 128, b, kt);
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  const int64_t r0 = kt * 128;
  const int64_t n_all = (p.S_q + kN - 1) / kN;
  int tile0 = 0, n = static_cast<int>(n_all);
  if (p.causal) {  // query rows i >= j only
    tile0 = static_cast<int>(r0 / kN);
    n = static_cast<int>(n_all - tile0 > 0 ? n_all - tile0 : 0);
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->res_ready, 256);
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_ready[s], 128);
      mbar_init(&bars->st_empty[s], 1);
    }
    for (int v = 0; v < Cfg::kVecSlots; ++v) {
      mbar_init(&bars->vec_full[v], 128);
      mbar_init(&bars->vec_empty[v], 256);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->t_free, 256);
    mbar_init(&bars->mma_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 13) tmem_alloc(&bars->tmem_base, 512);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // before any global access and before the wait deadline starts
  const uint32_t tmem = bars->tmem_base;
  WaitCtl ctl;
  ctl.deadline_ns = globaltimer_ns() + p.timeout_ns;
  ctl.abort_flag = &bars->abort_flag;

  if (warp == 12) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && n > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_o);
      int issued = 0;
      for (int t = 0; t < n; ++t) {
        const int s = t % kStages;
        SCORE_PROBE_T0(p0);
        if (!mbar_wait(&bars->st_empty[s], ((t / kStages) & 1) ^ 1, ctl)) break;
        SCORE_PROBE_ADD(8, p0);
        const int row0 = (tile0 + t) * kN;
        mbar_expect_tx(&bars->st_full[s], Cfg::kQBytes + Cfg::kOBytes);
#pragma unroll
        for (int c = 0; c < DQK / 32; ++c)
          tma_load_rows(smem + Cfg::q_hi(s) + c * kN * 128, &tm_q, c * 32, row0, hb, ob, &bars->st_full[s], HEADS);
#pragma unroll
        for (int c = 0; c < DV / 32; ++c)
          tma_load_rows(smem + Cfg::o_hi(s) + c * kN * 128, &tm_o, c * 32, row0, hb, ob, &bars->st_full[s], HEADS);
        issued = t + 1;
      }
      if (*ctl.abort_flag) {  // let the copies in flight land before the CTA exits
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        for (int t = (issued > kStages ? issued - kStages : 0); t < issued; ++t)
          mbar_wait(&bars->st_full[t % kStages], (t / kStages) & 1, drain);
      }
    }
  } else if (warp == 13) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && n > 0) {
      const uint32_t sb = smem_u32(smem);
      const uint32_t tT = tmem + Cfg::kT;
      bool ok = mbar_wait(&bars->res_ready, 0, ctl);
      for (int t = 0; ok && t < n; ++t) {
        const int s = t % kStages;
        // the buffer is free once every elementwise thread loaded tile t - 1
        SCORE_PROBE_T0(w0);
        if (t > 0 && !mbar_wait(&bars->t_free, (t - 1) & 1, ctl)) break;
        SCORE_PROBE_ADD(0, w0);
        SCORE_PROBE_T0(w1);
        if (!mbar_wait(&bars->st_ready[s], (t / kStages) & 1, ctl)) break;
        SCORE_PROBE_ADD(1, w1);
        SCORE_PROBE_T0(w2);
        tc_fence_after();
        issue_scores<DQK, kN>(tT, tmem + Cfg::kKh, tmem + Cfg::kKl, sb + Cfg::q_hi(s), sb + Cfg::q_lo(s));
        if constexpr (Cfg::kVlSmem)
          issue_scores_lo_smem<DV, kN>(tT + kN, tmem + Cfg::kVh, sb + Cfg::kVlOff, sb + Cfg::o_hi(s), sb + Cfg::o_lo(s));
        else
          issue_scores<DV, kN>(tT + kN, tmem + Cfg::kVh, tmem + Cfg::kVl, sb + Cfg::o_hi(s), sb + Cfg::o_lo(s));
        mma_commit(&bars->s_full);
        mma_commit(&bars->st_empty[s]);
        SCORE_PROBE_ADD(2, w2);
      }
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else if (warp >= 8) {
    // ------------------------------------------------------- converters
    const int tid = threadIdx.x - 256;
    for (int t = 0; t < n; ++t) {
      const int s = t % kStages;
      SCORE_PROBE_T0(c0);
      if (!tc::warp_wait(&bars->st_full[s], (t / kStages) & 1, ctl)) break;
      if (tid == 0) SCORE_PROBE_ADD(6, c0);
      SCORE_PROBE_T0(c1);
      const int vs = t % Cfg::kVecSlots;
      if (!tc::warp_wait(&bars->vec_empty[vs], ((t / Cfg::kVecSlots) & 1) ^ 1, ctl)) break;
      float* vec = reinterpret_cast<float*>(smem + Cfg::vec(vs));
      const int64_t i = static_cast<int64_t>(tile0 + t) * kN + (tid % kN);
      const bool in = i < p.S_q;
      if (tid < kN) vec[tid] = in ? p.lse[b * p.S_q + i] * kLog2e : INFINITY;  // p = 0 beyond S_q
      else if (tid < 2 * kN) vec[tid] = in ? p.delta[b * p.S_q + i] : 0.0f;
      mbar_arrive(&bars->vec_full[vs]);
      split_tile(smem + Cfg::q_hi(s), smem + Cfg::q_lo(s), Cfg::kQBytes, tid, 128);
      split_tile(smem + Cfg::o_hi(s), smem + Cfg::o_lo(s), Cfg::kOBytes, tid, 128);
      fence_proxy_async_smem();
      if (tid == 0) SCORE_PROBE_ADD(7, c1);
      mbar_arrive(&bars->st_ready[s]);
    }
  } else {
    // ------------------------------------------------ elementwise warps
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // TMEM lane = key row in the tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int col0 = half * kHalf;
    const int64_t rr = r0 + r;  // key row j
    const bool row_ok = rr < p.S_kv;
    const float sl2 = p.scale_log2, dp_inv = p.dp_inv;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    SCORE_PROBE_T0(e9);
    {  // K and V rows to TMEM (hi / lo): this thread's half of the columns
      const float* krow = static_cast<const float*>(p.k) + (row_ok ? row_offset_t<HEADS>(p.H, b, rr, p.S_kv, p.D_qk) : 0);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c) {
        const int cc = half * (DQK / 2) + c * 32;
        row_to_tmem(krow, cc, p.D_qk, row_ok, tmem + lane_base + Cfg::kKh + cc, tmem + lane_base + Cfg::kKl + cc);
      }
      const float* vrow = static_cast<const float*>(p.v) + (row_ok ? row_offset_t<HEADS>(p.H, b, rr, p.S_kv, p.D_v) : 0);
      constexpr int HC = DV / 2 < 32 ? 32 : DV / 2;  // columns per half (D_v = 32: half 0 takes all)
      if (half * HC < DV) {
#pragma unroll
        for (int c = 0; c < HC / 32; ++c) {
          const int cc = half * HC + c * 32;
          if constexpr (Cfg::kVlSmem)  // lo: row r of box cc / 32, 16-byte chunk g at g ^ (r & 7)
            row_to_tmem_smem(vrow, cc, p.D_v, row_ok, tmem + lane_base + Cfg::kVh + cc,
                             smem + Cfg::kVlOff + (cc / 32) * (128 * 128) + r * 128, r & 7);
          else
            row_to_tmem(vrow, cc, p.D_v, row_ok, tmem + lane_base + Cfg::kVh + cc, tmem + lane_base + Cfg::kVl + cc);
        }
      }
      if (Cfg::kVlSmem) fence_proxy_async_smem();
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->res_ready);
    }
    if (threadIdx.x == 0) SCORE_PROBE_ADD(9, e9);
    const uint64_t step_i = static_cast<uint64_t>(p.S_kv) * kLcgA;  // counter step between query rows
    const uint32_t step_lo = static_cast<uint32_t>(step_i), step_hi = static_cast<uint32_t>(step_i >> 32);
    for (int t = 0; t < n; ++t) {
      SCORE_PROBE_T0(e0);
      const int vs = t % Cfg::kVecSlots;
      if (!tc::warp_wait(&bars->s_full, t & 1, ctl) ||
          !tc::warp_wait(&bars->vec_full[vs], (t / Cfg::kVecSlots) & 1, ctl))
        break;
      if (threadIdx.x == 0) SCORE_PROBE_ADD(4, e0);
      SCORE_PROBE_T0(e1);
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + Cfg::kT + col0;
      uint32_t sv[kHalf], dpv[kHalf];
      tmem_ld_cols<kHalf>(tS, sv);
      tmem_ld_cols<kHalf>(tS + kN, dpv);
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars->t_free);
      // columns are query rows i = c0g + c of key row j = rr
      const int64_t c0g = static_cast<int64_t>(tile0 + t) * kN + col0;
      const float* vec = reinterpret_cast<const float*>(smem + Cfg::vec(vs)) + col0;
      int lo = -1;  // causal: column c valid iff c0g + c >= j
      if (p.causal) {
        const int64_t d = rr - c0g;
        lo = static_cast<int>(d < -1 ? -1 : (d > kHalf ? kHalf : d));
      }
      LcgWalk st(DROP ? lcg_state(p.rng_base + static_cast<uint64_t>(b * p.S_q + c0g) * static_cast<uint64_t>(p.S_kv),
                                  static_cast<uint64_t>(rr))
                      : 0);
      // column j of dS and P~, query rows c0g.. < S_q: consecutive lanes write
      // consecutive keys, so each store of a warp fills one 128-byte line
      // (rows of a thread's own, written with vector stores, would touch 32
      // lines per store and measured 1.5x slower)
      const int64_t col_off = (b * p.S_q + c0g) * p.ld_k + rr;
      float* const ds_col = p.ws_ds + col_off;
      float* const p_col = p.ws_p + col_off;
      const int lim = static_cast<int>(p.S_q - c0g < kHalf ? p.S_q - c0g : kHalf);
#pragma unroll
      for (int c = 0; c < kHalf; ++c) {
        float pr = ex2(fmaf(__uint_as_float(sv[c]), sl2, -vec[c]));
        pr = (pr > kEps && c >= lo) ? pr : 0.0f;
        float kf = 1.0f;
        if (DROP) {
          kf = st.dropped(thr_m1) ? 0.0f : dp_inv;
          st.step(step_lo, step_hi);
        }
        if (row_ok && c < lim) {
          p_col[static_cast<int64_t>(c) * p.ld_k] = pr * kf;
          ds_col[static_cast<int64_t>(c) * p.ld_k] = pr * fmaf(kf, __uint_as_float(dpv[c]), -vec[kN + c]);
        }
      }
      if (threadIdx.x == 0) SCORE_PROBE_ADD(5, e1);
      mbar_arrive(&bars->vec_empty[vs]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 13) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tf32
}  // namespace sdpa_b200
