// Backward attention on the 5th-generation tensor cores (sm_100a), fp16 in,
// fp32 accumulate.  Two kernels, as the reference splits it (sdpa/sdpa_bwd.cu.cc:
// a dK/dV pass over key tiles and a dQ pass over query tiles, no atomics):
//
// dkdv_kernel: one CTA = 128 key rows (TMEM lanes) of one batch row; streams
//   64-row tiles of Q and dO (3-stage TMA ring) and per tile computes
//     S^T  = K Q^T,  dP^T = V dO^T              (SS MMA, M=128, N=64)
//     P^T  = exp2(S^T*scale*log2e - lse*log2e), dropout, skip p <= 1e-6
//     dS^T = P~ (dP^T - D/dp_inv)  or  -p D when dropped   (unscaled)
//     dV  += P~^T dO,  dK += dS^T Q             (TS MMA: A = P~ / dS read
//                                                from TMEM, written over S^T / dP^T)
//   dK is multiplied by `scale` in the epilogue.
// dq2_kernel: one CTA = 128 query rows; streams 128-row K/V tiles; S = Q K^T,
//   dP = dO V^T, dS as above, dQ += dS K (TS MMA); dQ *= scale at the end
//   (layout and pipeline at its definition below).
//
// Roles: warps 0-7 elementwise (warp w serves TMEM lanes 32*(w%4).. and
// column half w/4 of each 64-column tile), warp 8 TMA producer, warp 9 MMA
// issuer + TMEM owner; dkdv_kernel adds warp 10, which issues the gradient
// MMAs while warp 9 issues the score MMAs.  S / dP are double-buffered in
// TMEM so the MMAs of tile j+1 overlap the elementwise work of tile j.
//
// Semantics: sdpa/sdpa_bwd.cu.cc:125-170 (dS formulas, skip rule, dropout).
#pragma once
#include "common.cuh"
#include "fwd_tc.cuh"
#include "ptx.cuh"

namespace sdpa_b200 {
namespace tc {

constexpr int kBwdTcThreads = 352;  // 8 elementwise warps, TMA producer, two MMA-issuing warps
constexpr int kBwdRows = 128;   // rows owned by a CTA (TMEM lanes)
constexpr int kBwdTile = 64;    // rows of each streamed tile
constexpr int kBwdStages = 3;

template <int DQK, int DV>
struct BwdCfg {
  // resident operand (128 rows) and streamed operands (64 rows per stage)
  static constexpr uint32_t kResA = kBwdRows * DQK * 2;  // K (dkdv) or Q (dq)
  static constexpr uint32_t kResB = kBwdRows * DV * 2;   // V (dkdv) or dO (dq)
  static constexpr uint32_t kStA = kBwdTile * DQK * 2;   // Q (dkdv) or K (dq)
  static constexpr uint32_t kStB = kBwdTile * DV * 2;    // dO (dkdv) or V (dq)
  static constexpr uint32_t kResAOff = 0;
  static constexpr uint32_t kResBOff = kResAOff + kResA;
  static constexpr uint32_t kStAOff = kResBOff + kResB;
  static constexpr uint32_t kStBOff = kStAOff + kBwdStages * kStA;
  static constexpr uint32_t kVecOff = kStBOff + kBwdStages * kStB;  // per-tile row vectors
  static constexpr uint32_t kVecBytes = 2 * 2 * kBwdTile * 4;       // 2 buffers x {lse2, delta}
  static constexpr uint32_t kBarOff = kVecOff + kVecBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  // TMEM columns
  static constexpr uint32_t kAcc0 = 0;     // dV (dkdv) or dQ (dq)
  static constexpr uint32_t kAcc1 = DV;    // dK (dkdv)
  static constexpr uint32_t kS = 256;      // S / S^T buffers: 256 + sb*64
  static constexpr uint32_t kDP = 384;     // dP / dP^T buffers: 384 + sb*64
  static_assert(DQK + DV <= 256, "TMEM budget");
};

struct BwdBarriers {
  uint64_t res_full;
  uint64_t st_full[kBwdStages];
  uint64_t st_empty[kBwdStages];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t vec_ready[2];
  uint64_t acc_done;
  uint64_t mma_done;
  uint64_t gv_done[2];   // dK/dV kernel: dV MMAs of the tile in buffer sb completed (P~^T read)
  uint64_t gk_done[2];   // dK/dV kernel: dK MMAs of the tile in buffer sb completed (dS^T read)
  uint64_t mma_done2;    // dK/dV kernel: drain of the second issuing thread
  uint32_t tmem_base;
  int abort_flag;
};

// Shared prologue of both backward kernels: barriers, TMEM, wait control.
__device__ __forceinline__ void bwd_setup(BwdBarriers* bars, uint32_t tmem_cols, int warp) {
  if (threadIdx.x == 0) {
    mbar_init(&bars->res_full, 1);
    for (int s = 0; s < kBwdStages; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 256);
      mbar_init(&bars->vec_ready[s], 256);
    }
    mbar_init(&bars->acc_done, 1);
    mbar_init(&bars->mma_done, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->gv_done[s], 1);
      mbar_init(&bars->gk_done[s], 1);
    }
    mbar_init(&bars->mma_done2, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(&bars->tmem_base, tmem_cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // before any global access and before the wait deadline starts
}

// Producer of both kernels: the resident 128-row pair once, then n 64-row
// tiles (rows tile0*64 ..) of the streamed pair through the stage ring.
template <int DA, int DB, typename Cfg>
__device__ __forceinline__ void bwd_producer(uint8_t* smem, BwdBarriers* bars, const CUtensorMap* ra,
                                             const CUtensorMap* rb, const CUtensorMap* sa, const CUtensorMap* sb,
                                             int res_row0, int tile0, int n, int hb, int ob, bool heads, const WaitCtl& ctl,
                                             uint64_t timeout_ns) {
  mbar_expect_tx(&bars->res_full, Cfg::kResA + Cfg::kResB);
#pragma unroll
  for (int c = 0; c < DA / 64; ++c)
    tma_load_rows(smem + Cfg::kResAOff + c * kBwdRows * 128, ra, c * 64, res_row0, hb, ob, &bars->res_full, heads);
#pragma unroll
  for (int c = 0; c < DB / 64; ++c)
    tma_load_rows(smem + Cfg::kResBOff + c * kBwdRows * 128, rb, c * 64, res_row0, hb, ob, &bars->res_full, heads);
  int issued = 0;
  for (int t = 0; t < n; ++t) {
    const int s = t % kBwdStages;
    if (!mbar_wait(&bars->st_empty[s], ((t / kBwdStages) & 1) ^ 1, ctl)) break;
    const int row0 = (tile0 + t) * kBwdTile;
    mbar_expect_tx(&bars->st_full[s], Cfg::kStA + Cfg::kStB);
#pragma unroll
    for (int c = 0; c < DA / 64; ++c)
      tma_load_rows(smem + Cfg::kStAOff + s * Cfg::kStA + c * kBwdTile * 128, sa, c * 64, row0, hb, ob, &bars->st_full[s], heads);
#pragma unroll
    for (int c = 0; c < DB / 64; ++c)
      tma_load_rows(smem + Cfg::kStBOff + s * Cfg::kStB + c * kBwdTile * 128, sb, c * 64, row0, hb, ob, &bars->st_full[s], heads);
    issued = t + 1;
  }
  if (*ctl.abort_flag) {  // let copies in flight land before the CTA exits
    WaitCtl drain = ctl;
    drain.deadline_ns = globaltimer_ns() + timeout_ns;
    int dummy = 0;
    drain.abort_flag = &dummy;
    mbar_wait(&bars->res_full, 0, drain);
    for (int t = (issued > kBwdStages ? issued - kBwdStages : 0); t < issued; ++t)
      mbar_wait(&bars->st_full[t % kBwdStages], (t / kBwdStages) & 1, drain);
  }
}

// One of the two score products of the dK/dV kernel: TMEM columns OUT + sb*64
// (+)= resident (at smem RES) * stage tile (at smem ST + s*STB)^T, K = D.
template <int D, typename Cfg, uint32_t OUT, uint32_t RES, uint32_t ST, uint32_t STB>
__device__ __forceinline__ void bwd_issue_scores_half(uint32_t tmem, uint32_t smem_base, int s, int sb) {
  constexpr uint32_t idesc = make_idesc(kBwdRows, kBwdTile, false, false, false);
  const uint32_t ra = smem_base + RES, sa = smem_base + ST + s * STB;
#pragma unroll
  for (int kk = 0; kk < D / 16; ++kk) {
    const uint64_t a = make_sw128_desc(ra + (kk >> 2) * (kBwdRows * 128) + (kk & 3) * 32, 16, 1024);
    const uint64_t bb = make_sw128_desc(sa + (kk >> 2) * (kBwdTile * 128) + (kk & 3) * 32, 16, 1024);
    mma_f16_ss(tmem + OUT + sb * kBwdTile, a, bb, idesc, kk > 0 ? 1u : 0u);
  }
}

// acc (+)= A[tmem: fp16 pairs over buffer `a_col`, 64 K-elements in two
// 16-column runs at +0 and +32] * B[64-row stage tile, MN-major, N = DN].
template <int DN>
__device__ __forceinline__ void bwd_issue_acc(uint32_t acc_tmem, uint32_t a_col, uint32_t b_tile, bool first) {
  constexpr uint32_t idesc = make_idesc(kBwdRows, DN, false, true, false);
#pragma unroll
  for (int kk = 0; kk < kBwdTile / 16; ++kk) {
    const uint64_t bd = make_sw128_desc(b_tile + kk * 16 * 128, kBwdTile * 128, 1024);
    mma_f16_ts(acc_tmem, a_col + (kk >> 1) * 32 + (kk & 1) * 8, bd, idesc, (!first || kk > 0) ? 1u : 0u);
  }
}

// Epilogue: TMEM accumulator columns [col0, col0 + 32*nchunks) of this
// thread's lane, times `mul`, to fp16 row `dst` (columns < D valid).
__device__ __forceinline__ void store_acc_row(uint32_t taddr, int nchunks, int col0, float mul, bool have_acc,
                                              bool active, __half* dst, int D) {
  for (int c = 0; c < nchunks; ++c) {
    uint32_t o[32];
    if (have_acc) {
      SDPA_TMEM_LD32(taddr + c * 32, o);
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = 0u;
    }
    uint32_t h[16];
#pragma unroll
    for (int e = 0; e < 16; ++e) h[e] = pack_half2(__uint_as_float(o[2 * e]) * mul, __uint_as_float(o[2 * e + 1]) * mul);
    if (active) {
#pragma unroll
      for (int w = 0; w < 4; ++w) {
        const int col = col0 + c * 32 + w * 8;
        if (col < D) *reinterpret_cast<uint4*>(dst + col) = make_uint4(h[4 * w], h[4 * w + 1], h[4 * w + 2], h[4 * w + 3]);
      }
    }
  }
}

// Elementwise pass of the dK/dV kernel over 32 columns (query rows) of one key
// row: P~^T and the unscaled dS^T as packed fp16 pairs.  MASK: some columns
// fail the causal test c >= lo (only warps on the diagonal).
template <bool DROP, bool MASK>
__device__ __forceinline__ void dkdv_elems(const uint32_t* sv, const uint32_t* dpv, const float* vbc, int lo,
                                           float sl2, float dp_inv, LcgWalk& st, uint32_t thr_m1, uint32_t step_lo,
                                           uint32_t step_hi, uint32_t* pk, uint32_t* dk) {
#pragma unroll
  for (int c4 = 0; c4 < 8; ++c4) {
    const float4 L4 = *reinterpret_cast<const float4*>(vbc + 4 * c4);
    const float4 D4 = *reinterpret_cast<const float4*>(vbc + kBwdTile + 4 * c4);
    const float Lv[4] = {L4.x, L4.y, L4.z, L4.w}, Dv[4] = {D4.x, D4.y, D4.z, D4.w};
    float ptv[4], dsv[4];
    // element pairs in packed f32x2 arithmetic (same rounding as scalar)
#pragma unroll
    for (int e = 0; e < 4; e += 2) {
      const int c = 4 * c4 + e;
      float x0, x1;
      ffma2(x0, x1, __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]), sl2, sl2, -Lv[e], -Lv[e + 1]);
      float pr0 = ex2(x0), pr1 = ex2(x1);
      // skip rule of sdpa/sdpa_bwd.cu.cc:131, causal mask
      pr0 = (pr0 > kEps && (!MASK || c >= lo)) ? pr0 : 0.0f;
      pr1 = (pr1 > kEps && (!MASK || c + 1 >= lo)) ? pr1 : 0.0f;
      // dropped: P~ = 0, dS = -p D; kept: P~ = p/(1-r), dS = P~ (dP - D (1-r)) = p (dP/(1-r) - D)
      float kf0 = 1.0f, kf1 = 1.0f;
      if (DROP) {
        const bool dr0 = st.dropped(thr_m1);
        st.step(step_lo, step_hi);
        const bool dr1 = st.dropped(thr_m1);
        st.step(step_lo, step_hi);
        kf0 = dr0 ? 0.0f : dp_inv;
        kf1 = dr1 ? 0.0f : dp_inv;
        fmul2(ptv[e], ptv[e + 1], pr0, pr1, kf0, kf1);
      } else {
        ptv[e] = pr0;
        ptv[e + 1] = pr1;
      }
      float t0, t1;
      ffma2(t0, t1, kf0, kf1, __uint_as_float(dpv[c]), __uint_as_float(dpv[c + 1]), -Dv[e], -Dv[e + 1]);
      fmul2(dsv[e], dsv[e + 1], pr0, pr1, t0, t1);
    }
    pk[2 * c4] = pack_half2(ptv[0], ptv[1]);
    pk[2 * c4 + 1] = pack_half2(ptv[2], ptv[3]);
    dk[2 * c4] = pack_half2(dsv[0], dsv[1]);
    dk[2 * c4 + 1] = pack_half2(dsv[2], dsv[3]);
  }
}

// Elementwise pass of the dQ kernel over 32 columns (keys) of one query row:
// the unscaled dS as packed fp16 pairs.  MASK: some columns fail c < lim.
template <bool DROP, bool MASK>
__device__ __forceinline__ void dq_elems(const uint32_t* sv, const uint32_t* dpv, int lim, float sl2, float lse2,
                                         float delta, float dp_inv, LcgWalk& st, uint32_t thr_m1, uint32_t* dk) {
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
    float dsv[2];
    // exponent arguments: a packed f32x2 pair without dropout (same rounding as
    // scalar); with dropout the scalar form measured faster in this kernel
    float x0, x1;
    if (DROP) {
      x0 = fmaf(__uint_as_float(sv[c]), sl2, -lse2);
      x1 = fmaf(__uint_as_float(sv[c + 1]), sl2, -lse2);
    } else {
      ffma2(x0, x1, __uint_as_float(sv[c]), __uint_as_float(sv[c + 1]), sl2, sl2, -lse2, -lse2);
    }
    float pr0 = ex2(x0), pr1 = ex2(x1);
    pr0 = (pr0 > kEps && (!MASK || c < lim)) ? pr0 : 0.0f;  // skip rule, key range, causal mask
    pr1 = (pr1 > kEps && (!MASK || c + 1 < lim)) ? pr1 : 0.0f;
    float kf0 = 1.0f, kf1 = 1.0f;  // see dkdv_elems: dS = p (kf dP - D)
    if (DROP) {
      const bool dr0 = st.dropped(thr_m1);
      st.step();
      const bool dr1 = st.dropped(thr_m1);
      st.step();
      kf0 = dr0 ? 0.0f : dp_inv;
      kf1 = dr1 ? 0.0f : dp_inv;
    }
    dsv[0] = pr0 * fmaf(kf0, __uint_as_float(dpv[c]), -delta);
    dsv[1] = pr1 * fmaf(kf1, __uint_as_float(dpv[c + 1]), -delta);
    dk[c / 2] = pack_half2(dsv[0], dsv[1]);
  }
}

// dq_elems with dropout over a thread's two 32-column halves at once (no
// masking): element c of each half in the same iteration, each half with its
// own RNG walker, so the two 64-bit carry chains interleave.
template <bool DROP>
__device__ __forceinline__ void dq_elems_x2(const uint32_t* sv, const uint32_t* dpv, float sl2, float lse2,
                                            float delta, float dp_inv, LcgWalk& st0, LcgWalk& st1, uint32_t thr_m1,
                                            uint32_t* dk) {
#pragma unroll
  for (int c = 0; c < 32; c += 2) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      LcgWalk& st = h ? st1 : st0;
      const int cc = 32 * h + c;
      float pr0 = ex2(fmaf(__uint_as_float(sv[cc]), sl2, -lse2));
      float pr1 = ex2(fmaf(__uint_as_float(sv[cc + 1]), sl2, -lse2));
      pr0 = pr0 > kEps ? pr0 : 0.0f;  // skip rule
      pr1 = pr1 > kEps ? pr1 : 0.0f;
      float kf0 = 1.0f, kf1 = 1.0f;  // see dkdv_elems: dS = p (kf dP - D)
      if (DROP) {
        const bool dr0 = st.dropped(thr_m1);
        st.step();
        const bool dr1 = st.dropped(thr_m1);
        st.step();
        kf0 = dr0 ? 0.0f : dp_inv;
        kf1 = dr1 ? 0.0f : dp_inv;
      }
      const float d0 = pr0 * fmaf(kf0, __uint_as_float(dpv[cc]), -delta);
      const float d1 = pr1 * fmaf(kf1, __uint_as_float(dpv[cc + 1]), -delta);
      dk[cc / 2] = pack_half2(d0, d1);
    }
  }
}

template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kBwdTcThreads, 1)
    dkdv_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v,
                const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do, const Params p) {
  using Cfg = BwdCfg<DQK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  BwdBarriers* bars = reinterpret_cast<BwdBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  int64_t b, kt;  // low key tiles see the most causal rows: issued first
  raster(blockIdx.x, p.B, (p.S_kv + kBwdRows - 1) / kBwdRows, b, kt);
  // head and outer batch of folded row b (layout [B/H, S, H, D] when HEADS)
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  constexpr bool heads = HEADS;
  const int64_t n0 = kt * kBwdRows;
  const int n_qtiles = static_cast<int>((p.S_q + kBwdTile - 1) / kBwdTile);
  const int tile0 = p.causal ? static_cast<int>(n0 / kBwdTile) : 0;
  const int nq = n_qtiles - tile0 > 0 ? n_qtiles - tile0 : 0;

  bwd_setup(bars, Cfg::kTmemCols, warp);
  const uint32_t tmem = bars->tmem_base;
  WaitCtl ctl;
  ctl.deadline_ns = globaltimer_ns() + p.timeout_ns;
  ctl.abort_flag = &bars->abort_flag;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 8) {
    if (lane == 0 && nq > 0)
      bwd_producer<DQK, DV, Cfg>(smem, bars, &tm_k, &tm_v, &tm_q, &tm_do, static_cast<int>(n0), tile0, nq, hb, ob,
                                 heads, ctl, p.timeout_ns);
  } else if (warp == 9) {
    // Score MMAs.  S^T / dP^T of tile t go to buffer t&1, whose halves the
    // dV / dK MMAs of tile t-2 read (as P~^T / dS^T): S^T waits only for the
    // dV MMAs, dP^T for the dK MMAs, so S^T enters the pipe while dK runs.
    if (lane == 0 && nq > 0) {
      bool ok = mbar_wait(&bars->res_full, 0, ctl);
      for (int t = 0; ok && t < nq; ++t) {
        const int s = t % kBwdStages, sb = t & 1;
        const uint32_t ph = ((t >> 1) - 1) & 1;
        if (!mbar_wait(&bars->st_full[s], (t / kBwdStages) & 1, ctl) ||
            (t >= 2 && !mbar_wait(&bars->gv_done[sb], ph, ctl))) {
          ok = false;
          break;
        }
        tc_fence_after();
        bwd_issue_scores_half<DQK, Cfg, Cfg::kS, Cfg::kResAOff, Cfg::kStAOff, Cfg::kStA>(tmem, sbase, s, sb);
        if (t >= 2 && !mbar_wait(&bars->gk_done[sb], ph, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        bwd_issue_scores_half<DV, Cfg, Cfg::kDP, Cfg::kResBOff, Cfg::kStBOff, Cfg::kStB>(tmem, sbase, s, sb);
        mma_commit(&bars->s_full[sb]);
      }
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else if (warp == 10) {
    // Gradient MMAs, issued from their own thread so that its waits overlap
    // the score MMAs in the tensor pipe (and the other way round).
    if (lane == 0 && nq > 0) {
      bool ok = true;
      for (int t = 0; ok && t < nq; ++t) {
        const int s = t % kBwdStages, sb = t & 1;
        if (!mbar_wait(&bars->p_full[sb], (t >> 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        // dV += P~^T dO_t ; dK += dS^T Q_t
        bwd_issue_acc<DV>(tmem + Cfg::kAcc0, tmem + Cfg::kS + sb * kBwdTile, sbase + Cfg::kStBOff + s * Cfg::kStB,
                          t == 0);
        mma_commit(&bars->gv_done[sb]);
        bwd_issue_acc<DQK>(tmem + Cfg::kAcc1, tmem + Cfg::kDP + sb * kBwdTile, sbase + Cfg::kStAOff + s * Cfg::kStA,
                           t == 0);
        mma_commit(&bars->st_empty[s]);
        mma_commit(&bars->gk_done[sb]);
      }
      mma_commit(&bars->acc_done);
      mma_commit(&bars->mma_done2);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done2, 0, drain);
    }
  } else {
    // ------------------------------------------------ elementwise warps
    const int e = threadIdx.x;                // 0..255
    const int half = warp >> 2;               // column half of each 64-wide tile
    const int r = (warp & 3) * 32 + lane;     // TMEM lane = key row in tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int col0 = half * 32;
    const int64_t j = n0 + r;                 // key row
    float* vec = reinterpret_cast<float*>(smem + Cfg::kVecOff);  // [2][2][64]
    const float sl2 = p.scale_log2, dp_inv = p.dp_inv;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    const int64_t jw0 = n0 + (warp & 3) * 32;  // first key row of this warp
    const uint64_t step_i = static_cast<uint64_t>(p.S_kv) * kLcgA;  // counter step between query rows
    const uint32_t step_lo = static_cast<uint32_t>(step_i), step_hi = static_cast<uint32_t>(step_i >> 32);
    // Row vectors of tile t (thread e < 128 owns one value): the global load
    // is issued a tile ahead and only consumed when stored to shared memory,
    // so its latency overlaps the current tile's work.
    const int which = e >> 6;  // 0: lse (log2 units), 1: delta
    auto row_load = [&](int t, bool& in_range) -> float {
      const int64_t i = static_cast<int64_t>(tile0 + t) * kBwdTile + (e & 63);
      in_range = which < 2 && i < p.S_q;
      if (!in_range) return 0.0f;
      return which == 0 ? p.lse[b * p.S_q + i] : p.delta[b * p.S_q + i];
    };
    bool pre_ok = false;
    float pre = nq > 0 ? row_load(0, pre_ok) : 0.0f;
    bool ok = true;
    for (int t = 0; t < nq; ++t) {
      const int sb = t & 1;
      float* vb = vec + sb * 2 * kBwdTile;
      if (e < 2 * kBwdTile) vb[e] = which == 0 ? (pre_ok ? pre * kLog2e : INFINITY) : (pre_ok ? pre : 0.0f);
      mbar_arrive(&bars->vec_ready[sb]);
      if (t + 1 < nq) pre = row_load(t + 1, pre_ok);
      if (!warp_wait(&bars->vec_ready[sb], (t >> 1) & 1, ctl) || !warp_wait(&bars->s_full[sb], (t >> 1) & 1, ctl)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[32], dpv[32];
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kS + sb * kBwdTile + col0, sv);
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kDP + sb * kBwdTile + col0, dpv);
      tmem_wait_ld();
      const int64_t i0 = static_cast<int64_t>(tile0 + t) * kBwdTile + col0;
      // causal: column c is valid iff i0 + c >= j; only warps on the diagonal test it
      const bool masked = p.causal && i0 < jw0 + 31;  // warp-uniform
      int lo = -1;
      if (masked) {
        const int64_t d = j - i0;
        lo = static_cast<int>(d < -1 ? -1 : (d > 32 ? 32 : d));
      }
      LcgWalk st(DROP ? lcg_state(p.rng_base + static_cast<uint64_t>(b * p.S_q + i0) *
                                                static_cast<uint64_t>(p.S_kv),
                                  static_cast<uint64_t>(j))
                      : 0);
      uint32_t pk[16], dk[16];
      if (masked)
        dkdv_elems<DROP, true>(sv, dpv, vb + col0, lo, sl2, dp_inv, st, thr_m1, step_lo, step_hi, pk, dk);
      else
        dkdv_elems<DROP, false>(sv, dpv, vb + col0, lo, sl2, dp_inv, st, thr_m1, step_lo, step_hi, pk, dk);
      SDPA_TMEM_ST16(tmem + lane_base + Cfg::kS + sb * kBwdTile + col0, pk);
      SDPA_TMEM_ST16(tmem + lane_base + Cfg::kDP + sb * kBwdTile + col0, dk);
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[sb]);
    }
    if (ok && nq > 0) ok = warp_wait(&bars->acc_done, 0, ctl);
    if (ok) {
      tc_fence_after();
      const bool active = j < p.S_kv;
      __half* dv_row = static_cast<__half*>(p.dv) + row_offset_t<HEADS>(p.H, b, j, p.S_kv, p.D_v);
      __half* dk_row = static_cast<__half*>(p.dk) + row_offset_t<HEADS>(p.H, b, j, p.S_kv, p.D_qk);
      store_acc_row(tmem + lane_base + Cfg::kAcc0 + half * (DV / 2), DV / 64, half * (DV / 2), 1.0f, nq > 0, active,
                    dv_row, p.D_v);
      store_acc_row(tmem + lane_base + Cfg::kAcc1 + half * (DQK / 2), DQK / 64, half * (DQK / 2), p.scale, nq > 0,
                    active, dk_row, p.D_qk);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ============================================================================
// dQ kernel with 128-key tiles.  One CTA = 128 query rows; per key tile t
// (warp 9 issues S/dP, warp 10 issues dQ):
//     S = Q K_t^T, dP = dO V_t^T      (SS MMA, N = 128: full rate)
//     dS = p (kf dP - D)               (8 elementwise warps, 64 columns each)
//     dQ += dS K_t                     (TS MMA, A = dS from its own TMEM buffer)
// The elementwise warps release S/dP as soon as they have loaded them, so the
// MMAs of tile t+1 run while dS of tile t is computed.  TMEM: dQ [0,128),
// dS [128,256) (two buffers of fp16 pairs), S [256,384), dP [384,512).  K is held until dQ
// consumed it (3-stage ring), V only until dP (2 stages); Q and dO resident.
template <int DQK, int DV>
struct Dq2Cfg {
  static constexpr int kKStages = 3, kVStages = 2;
  static constexpr uint32_t kQBytes = kBwdRows * DQK * 2, kOBytes = kBwdRows * DV * 2;
  static constexpr uint32_t kKBytes = kBwdRows * DQK * 2, kVBytes = kBwdRows * DV * 2;
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kOOff = kQOff + kQBytes;
  static constexpr uint32_t kKOff = kOOff + kOBytes;
  static constexpr uint32_t kVOff = kKOff + kKStages * kKBytes;
  static constexpr uint32_t kBarOff = kVOff + kVStages * kVBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static constexpr uint32_t kDQ = 0, kDS = 128, kS = 256, kDP = 384;
  static_assert(kSmemBytes <= 232448, "shared memory");
};

struct Dq2Barriers {
  uint64_t res_full;
  uint64_t k_full[3], k_empty[3];
  uint64_t v_full[2], v_empty[2];
  uint64_t s_full, sdp_free, ds_full[2], ds_empty[2];
  uint64_t acc_done, mma_done, mma_done2;
  uint32_t tmem_base;
  int abort_flag;
};

template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kBwdTcThreads, 1)
    dq2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_do,
               const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using Cfg = Dq2Cfg<DQK, DV>;
  constexpr int TN = kBwdRows;  // keys per tile
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  Dq2Barriers* bars = reinterpret_cast<Dq2Barriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const int64_t n_qt = (p.S_q + kBwdRows - 1) / kBwdRows;
  int64_t b, tord;
  raster(blockIdx.x, p.B, n_qt, b, tord);
  // head and outer batch of folded row b (layout [B/H, S, H, D] when HEADS)
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  constexpr bool heads = HEADS;
  const int64_t qt = n_qt - 1 - tord;  // longest causal rows first
  const int64_t m0 = qt * kBwdRows;
  const int64_t n_kv_all = (p.S_kv + TN - 1) / TN;
  const int nkv = static_cast<int>(p.causal ? min(n_kv_all, qt + 1) : n_kv_all);

  if (threadIdx.x == 0) {
    mbar_init(&bars->res_full, 1);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->k_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->v_empty[s], 1);
    }
    mbar_init(&bars->s_full, 1);
    mbar_init(&bars->sdp_free, 256);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->ds_full[s], 256);
      mbar_init(&bars->ds_empty[s], 1);
    }
    mbar_init(&bars->acc_done, 1);
    mbar_init(&bars->mma_done, 1);
    mbar_init(&bars->mma_done2, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // before any global access and before the wait deadline starts
  const uint32_t tmem = bars->tmem_base;
  WaitCtl ctl;
  ctl.deadline_ns = globaltimer_ns() + p.timeout_ns;
  ctl.abort_flag = &bars->abort_flag;
  const uint32_t sbase = smem_u32(smem);

  if (warp == 8) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && nkv > 0) {
      mbar_expect_tx(&bars->res_full, Cfg::kQBytes + Cfg::kOBytes);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c)
        tma_load_rows(smem + Cfg::kQOff + c * kBwdRows * 128, &tm_q, c * 64, static_cast<int>(m0), hb, ob,
                    &bars->res_full, heads);
#pragma unroll
      for (int c = 0; c < DV / 64; ++c)
        tma_load_rows(smem + Cfg::kOOff + c * kBwdRows * 128, &tm_do, c * 64, static_cast<int>(m0),
                    hb, ob, &bars->res_full, heads);
      int issued = 0;
      for (int t = 0; t < nkv; ++t) {
        const int ks = t % 3, vs = t & 1;
        if (!mbar_wait(&bars->k_empty[ks], ((t / 3) & 1) ^ 1, ctl)) break;
        mbar_expect_tx(&bars->k_full[ks], Cfg::kKBytes);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_rows(smem + Cfg::kKOff + ks * Cfg::kKBytes + c * TN * 128, &tm_k, c * 64, t * TN,
                      hb, ob, &bars->k_full[ks], heads);
        if (!mbar_wait(&bars->v_empty[vs], ((t >> 1) & 1) ^ 1, ctl)) break;
        mbar_expect_tx(&bars->v_full[vs], Cfg::kVBytes);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_rows(smem + Cfg::kVOff + vs * Cfg::kVBytes + c * TN * 128, &tm_v, c * 64, t * TN,
                      hb, ob, &bars->v_full[vs], heads);
        issued = t + 1;
      }
      if (*ctl.abort_flag) {  // let copies in flight land before the CTA exits
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        mbar_wait(&bars->res_full, 0, drain);
        for (int t = (issued > 2 ? issued - 2 : 0); t < issued; ++t) {
          mbar_wait(&bars->k_full[t % 3], (t / 3) & 1, drain);
          mbar_wait(&bars->v_full[t & 1], (t >> 1) & 1, drain);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------- score MMA issuer (S, dP)
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t idesc_s = make_idesc(kBwdRows, TN, false, false, false);
      bool ok = mbar_wait(&bars->res_full, 0, ctl);
      for (int t = 0; ok && t < nkv; ++t) {
        const int ks = t % 3, vs = t & 1;
        // S/dP of tile t-1 must be in registers of the elementwise warps
        if ((t > 0 && !mbar_wait(&bars->sdp_free, (t - 1) & 1, ctl)) || !mbar_wait(&bars->k_full[ks], (t / 3) & 1, ctl) ||
            !mbar_wait(&bars->v_full[vs], (t >> 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sbase + Cfg::kKOff + ks * Cfg::kKBytes, vb = sbase + Cfg::kVOff + vs * Cfg::kVBytes;
        const uint32_t qb = sbase + Cfg::kQOff, ob = sbase + Cfg::kOOff;
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kBwdRows * 128) + (kk & 3) * 32;
          mma_f16_ss(tmem + Cfg::kS, make_sw128_desc(qb + off, 16, 1024), make_sw128_desc(kb + off, 16, 1024),
                     idesc_s, kk > 0 ? 1u : 0u);
        }
#pragma unroll
        for (int kk = 0; kk < DV / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kBwdRows * 128) + (kk & 3) * 32;
          mma_f16_ss(tmem + Cfg::kDP, make_sw128_desc(ob + off, 16, 1024), make_sw128_desc(vb + off, 16, 1024),
                     idesc_s, kk > 0 ? 1u : 0u);
        }
        mma_commit(&bars->v_empty[vs]);  // V_t is no longer read
        mma_commit(&bars->s_full);
      }
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else if (warp == 10) {
    // -------------------------------------------- dQ MMA issuer (dQ += dS K)
    if (lane == 0 && nkv > 0) {
      constexpr uint32_t idesc_dq = make_idesc(kBwdRows, DQK, false, true, false);
      bool ok = true;
      for (int t = 0; ok && t < nkv; ++t) {
        const int db = t & 1;
        if (!mbar_wait(&bars->ds_full[db], (t >> 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kb = sbase + Cfg::kKOff + (t % 3) * Cfg::kKBytes;
#pragma unroll
        for (int kk = 0; kk < TN / 16; ++kk)
          mma_f16_ts(tmem + Cfg::kDQ, tmem + Cfg::kDS + db * 64 + kk * 8,
                     make_sw128_desc(kb + kk * 16 * 128, TN * 128, 1024), idesc_dq, (t > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars->k_empty[t % 3]);
        mma_commit(&bars->ds_empty[db]);
      }
      mma_commit(&bars->acc_done);
      mma_commit(&bars->mma_done2);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done2, 0, drain);
    }
  } else {
    // ------------------------------------------------ elementwise warps
    const int half = warp >> 2;            // 64-column half of each 128-key tile
    const int r = (warp & 3) * 32 + lane;  // TMEM lane = query row in tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int col0 = half * 64;
    const int64_t i = m0 + r;
    const int64_t iw0 = m0 + (warp & 3) * 32;
    const bool row_ok = i < p.S_q;
    const float lse2 = row_ok ? p.lse[b * p.S_q + i] * kLog2e : INFINITY;
    const float sl2 = p.scale_log2, dp_inv = p.dp_inv;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + i) * static_cast<uint64_t>(p.S_kv);
    // D_i = sum_d dO[i,d] O[i,d] (minus the stats gradient, when given) of this
    // CTA's rows, from the resident dO tile (128B-swizzled: 16-byte chunk k of
    // row r at r*128 + ((k ^ (r & 7)) << 4) in box k/8) and O in global
    // memory; both threads of a row compute the whole sum (no exchange), the
    // first writes it for the dK/dV kernel, which runs after this one.  The O
    // row is loaded before the resident tiles arrive, so its latency overlaps
    // theirs.
    uint4 orow_v[DV / 8];
    if (row_ok) {
      const __half* orow = static_cast<const __half*>(p.o) + row_offset_t<HEADS>(p.H, b, i, p.S_q, p.D_v);
#pragma unroll
      for (int g = 0; g < DV / 8; ++g)
        orow_v[g] = g * 8 < p.D_v ? *reinterpret_cast<const uint4*>(orow + g * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    bool ok = warp_wait(&bars->res_full, 0, ctl);
    float delta = 0.0f;
    if (ok && row_ok) {
      const uint8_t* dO_s = smem + Cfg::kOOff;
      float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int g = 0; g < DV / 8; ++g) {
        const uint4 ov = orow_v[g];
        const uint4 dv = *reinterpret_cast<const uint4*>(dO_s + (g >> 3) * (kBwdRows * 128) + r * 128 +
                                                           (((g & 7) ^ (r & 7)) << 4));
        const uint32_t ow[4] = {ov.x, ov.y, ov.z, ov.w}, dw[4] = {dv.x, dv.y, dv.z, dv.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float2 of = __half22float2(*reinterpret_cast<const __half2*>(&ow[e]));
          const float2 df = __half22float2(*reinterpret_cast<const __half2*>(&dw[e]));
          acc[e] = fmaf(df.x, of.x, acc[e]);
          acc[e] = fmaf(df.y, of.y, acc[e]);
        }
      }
      delta = (acc[0] + acc[1]) + (acc[2] + acc[3]);
      // A gradient g_i reaching stats_i = logsumexp adds g_i * p_ij to dS_ij,
      // i.e. it enters dS = p (dP - D) as D - g.
      if (p.d_stats) delta -= p.d_stats[b * p.S_q + i];
      if (half == 0) p.delta[b * p.S_q + i] = delta;
    }
    for (int t = 0; t < nkv; ++t) {
      if (!warp_wait(&bars->s_full, t & 1, ctl)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t sv[64], dpv[64];
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kS + col0, sv);
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kS + col0 + 32, (sv + 32));
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kDP + col0, dpv);
      SDPA_TMEM_LD32(tmem + lane_base + Cfg::kDP + col0 + 32, (dpv + 32));
      tmem_wait_ld();
      tc_fence_before();
      mbar_arrive(&bars->sdp_free);  // S/dP may be overwritten by the next tile's MMAs
      uint32_t dk[32];
      const int64_t jt = static_cast<int64_t>(t) * TN + col0;  // first key of this thread's 64 columns
      const bool interior = (p.S_kv - jt >= 64) && (!p.causal || iw0 - jt + 1 >= 64);  // warp-uniform
      if (DROP && interior) {
        // both 32-column halves in one interleaved loop: two independent RNG
        // carry chains per thread (measured faster with dropout only)
        LcgWalk st0(DROP ? lcg_state(rbase, static_cast<uint64_t>(jt)) : 0);
        LcgWalk st1(DROP ? lcg_state(rbase, static_cast<uint64_t>(jt + 32)) : 0);
        dq_elems_x2<DROP>(sv, dpv, sl2, lse2, delta, dp_inv, st0, st1, thr_m1, dk);
      } else
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        const int64_t j0 = static_cast<int64_t>(t) * TN + col0 + 32 * h2;
        int64_t lim64 = p.S_kv - j0;
        if (p.causal) lim64 = min(lim64, i - j0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > 32 ? 32 : lim64));
        const bool masked = (p.S_kv - j0 < 32) || (p.causal && iw0 - j0 + 1 < 32);  // warp-uniform
        LcgWalk st(DROP ? lcg_state(rbase, static_cast<uint64_t>(j0)) : 0);
        if (masked)
          dq_elems<DROP, true>(sv + 32 * h2, dpv + 32 * h2, lim, sl2, lse2, delta, dp_inv, st, thr_m1, dk + 16 * h2);
        else
          dq_elems<DROP, false>(sv + 32 * h2, dpv + 32 * h2, lim, sl2, lse2, delta, dp_inv, st, thr_m1, dk + 16 * h2);
      }
      const int db = t & 1;
      if (t > 1) {  // dQ of tile t-2 must have read dS buffer db
        if (!warp_wait(&bars->ds_empty[db], ((t >> 1) - 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
      }
      SDPA_TMEM_ST16(tmem + lane_base + Cfg::kDS + db * 64 + half * 32, dk);
      SDPA_TMEM_ST16(tmem + lane_base + Cfg::kDS + db * 64 + half * 32 + 16, (dk + 16));
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->ds_full[db]);
    }
    if (ok && nkv > 0) ok = warp_wait(&bars->acc_done, 0, ctl);
    if (ok) {
      tc_fence_after();
      __half* dq_row = static_cast<__half*>(p.dq) + row_offset_t<HEADS>(p.H, b, i, p.S_q, p.D_qk);
      store_acc_row(tmem + lane_base + Cfg::kDQ + half * (DQK / 2), DQK / 64, half * (DQK / 2), p.scale, nkv > 0,
                    row_ok, dq_row, p.D_qk);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

}  // namespace tc
}  // namespace sdpa_b200
