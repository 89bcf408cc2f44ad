// fp32 backward attention on the 5th-generation tensor cores with the 3xTF32
// split (see tf32_fwd.cuh).  Three passes, one template:
//
//   DQ  one CTA = 128 query rows.  Resident in TMEM: Q and dO (hi / lo), dQ.
//       Streams key tiles (K, V).  Per tile
//         S = Q K^T, dP = dO V^T            (TS MMAs, A = Q / dO from TMEM)
//         dS = p (kf dP - D)                (8 elementwise warps)
//         dQ += dS K                        (TS MMA, A = dS hi/lo from TMEM)
//       Its prologue writes D_i = rowsum(dO O) (- the stats gradient) to the
//       workspace for the DK pass.
//   DK  one CTA = 128 key rows.  Resident: K and V (hi / lo), dK.  Streams
//       query tiles (Q, dO) and computes S^T = K Q^T, dP^T = V dO^T,
//       dS^T, dK += dS^T Q.
//   DV  one CTA = 128 key rows.  Resident: K (hi / lo), dV.  Streams query
//       tiles (Q, dO): S^T = K Q^T, P~^T, dV += P~^T dO.  Two tile buffers,
//       so the next S^T overlaps the elementwise pass.
//
// The reference splits its backward the same way (no atomics,
// sdpa/sdpa_bwd.cu.cc); dK and dV are computed in two passes here because
// K, V (hi / lo) and both accumulators do not fit in TMEM at once in fp32.
// Every product is issued as three kind::tf32 MMAs (ah bh + ah bl + al bh).
//
// Roles: warps 0-7 elementwise (warp w serves TMEM lanes 32*(w%4).. and
// column half w/4 of each tile), warps 8-11 convert each streamed tile in
// shared memory into hi / lo (and stage lse / D of its query rows for DK and
// DV), warp 12 TMA producer, warp 13 MMA issuer + TMEM owner.
// Semantics: sdpa/sdpa_bwd.cu.cc:125-170 (dS formulas, skip rule p <= 1e-6,
// dropout), as in the fp16 kernels.
#pragma once
#include "common.cuh"
#include "fwd_tc.cuh"
#include "ptx.cuh"
#include "tf32_fwd.cuh"

namespace sdpa_b200 {
namespace tf32 {

enum BwdMode { kDQ = 0, kDK = 1, kDV = 2 };

// Timing probe for tuning builds (-DSDPA_B200_TF32_PROBE): SM cycles spent by
// the roles of CTA 0 in each phase, summed into slots of g_tf32_probe.
#ifdef SDPA_B200_TF32_PROBE
__device__ unsigned long long g_tf32_probe[16];
#define TF32_PROBE_T0(v) const long long v = clock64()
#define TF32_PROBE_ADD(slot, t0) \
  if (blockIdx.x == 0 && MODE == SDPA_B200_TF32_PROBE) atomicAdd(&g_tf32_probe[slot], static_cast<unsigned long long>(clock64() - (t0)))
#else
#define TF32_PROBE_T0(v)
#define TF32_PROBE_ADD(slot, t0)
#endif
constexpr int kBwdThreads = 448;

template <int MODE, int DQK, int DV>
struct BwdCfg {
  static constexpr bool kHasY = MODE != kDV;
  static constexpr int kAccCols = MODE == kDV ? DV : DQK;
  // TMEM columns
  static constexpr uint32_t kXh = 0, kXl = DQK;                 // Q (DQ) or K (DK, DV)
  static constexpr uint32_t kYh = 2 * DQK, kYl = 2 * DQK + DV;  // dO (DQ) or V (DK)
  static constexpr uint32_t kAcc = kHasY ? 2 * DQK + 2 * DV : 2 * DQK;
  static constexpr uint32_t kT = kAcc + kAccCols;               // tile buffers
  static constexpr int kNbuf = kHasY ? 1 : 2;
  static constexpr int kN = (512 - static_cast<int>(kT)) / (2 * kNbuf) >= 64 ? 64 : 32;  // streamed rows per tile
  static constexpr int kHalf = kN / 2;                           // columns per elementwise thread
  static_assert(kT + kNbuf * 2 * kN <= 512, "TMEM budget");
  // shared memory per stage: SA hi, SA lo (kN x DQK, 128B-swizzled K-major, for
  // the score MMAs), SB hi, SB lo (kN x DV), for DQ / DK the SA tile again as
  // hi / lo with 32-byte swizzle atoms (the accumulating MMA reads SA
  // MN-major, which tf32 takes only in that layout), row vectors (2 x kN
  // floats).  In DV, SB is read MN-major only and lands in that layout.
  static constexpr uint32_t kSABytes = kN * DQK * 4, kSBBytes = kN * DV * 4;
  static constexpr uint32_t kStageBytes = (kHasY ? 4 : 2) * kSABytes + 2 * kSBBytes + 2 * kN * 4;
  static constexpr uint32_t kStageAligned = (kStageBytes + 1023) / 1024 * 1024;
  static constexpr int kStages = 3 * kStageAligned <= 200 * 1024 ? 3 : 2;
  static constexpr uint32_t kBarOff = kStages * kStageAligned;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static_assert(kSmemBytes <= 232448, "shared memory");
  static __device__ __forceinline__ uint32_t sa_hi(int s) { return s * kStageAligned; }
  static __device__ __forceinline__ uint32_t sa_lo(int s) { return s * kStageAligned + kSABytes; }
  static __device__ __forceinline__ uint32_t sb_hi(int s) { return s * kStageAligned + 2 * kSABytes; }
  static __device__ __forceinline__ uint32_t sb_lo(int s) { return s * kStageAligned + 2 * kSABytes + kSBBytes; }
  static __device__ __forceinline__ uint32_t sa_mh(int s) { return s * kStageAligned + 2 * kSABytes + 2 * kSBBytes; }
  static __device__ __forceinline__ uint32_t sa_ml(int s) { return sa_mh(s) + kSABytes; }
  static __device__ __forceinline__ uint32_t vec(int s) {
    return s * kStageAligned + (kHasY ? 4 : 2) * kSABytes + 2 * kSBBytes;
  }
};

struct BwdBarriers {
  uint64_t res_ready;
  uint64_t st_full[3], st_ready[3], st_empty[3];
  uint64_t s_full[2], p_full[2];
  uint64_t acc_done, mma_done;
  uint64_t acc_step;  // DV: the accumulating MMAs of a tile completed
  uint32_t tmem_base;
  int abort_flag;
};

// split_tile for a tile read both K-major and MN-major: the raw tile at `hi`
// (128B swizzle: 16-byte chunk k of row r at r*128 + ((k ^ (r & 7)) << 4) in
// each box of ROWS rows) becomes hi / lo in place / at `lo`, and hi / lo again
// at `mh` / `ml` with 32-byte atoms (32-byte chunk c of row r at
// r*128 + ((c ^ (r & 3)) << 5)).
template <int ROWS>
__device__ __forceinline__ void split_tile_dual(uint8_t* hi, uint8_t* lo, uint8_t* mh, uint8_t* ml, uint32_t bytes,
                                                int tid, int nthr) {
  const int n4 = static_cast<int>(bytes / 16);
#pragma unroll 4
  for (int i = tid; i < n4; i += nthr) {
    const uint32_t o = static_cast<uint32_t>(i) * 16u;
    const uint32_t r = (o >> 7) % ROWS;
    const uint32_t kb = ((o >> 4) & 7u) ^ (r & 7u);  // logical 16-byte chunk in the row
    const uint32_t d = (o & ~127u) | ((((kb >> 1) ^ (r & 3u)) << 5) | ((kb & 1u) << 4));
    const float4 x = *reinterpret_cast<const float4*>(hi + o);
    float4 a, b;
    split_tf32(x.x, a.x, b.x);
    split_tf32(x.y, a.y, b.y);
    split_tf32(x.z, a.z, b.z);
    split_tf32(x.w, a.w, b.w);
    *reinterpret_cast<float4*>(hi + o) = a;
    *reinterpret_cast<float4*>(lo + o) = b;
    *reinterpret_cast<float4*>(mh + d) = a;
    *reinterpret_cast<float4*>(ml + d) = b;
  }
}

template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 16) {
    SDPA_TMEM_LD16(taddr, r);
  } else {
    SDPA_TMEM_LD32(taddr, r);
  }
}
template <int N>
__device__ __forceinline__ void tmem_st_cols(uint32_t taddr, uint32_t* r) {
  if constexpr (N == 16) {
    SDPA_TMEM_ST16(taddr, r);
  } else {
    SDPA_TMEM_ST32(taddr, r);
  }
}

// acc (+)= A[tmem hi / lo, K = kN] * B[stage tile hi / lo, MN-major with
// 32-byte swizzle atoms, N = DN]
template <int DN, int kN>
__device__ __forceinline__ void issue_acc(uint32_t acc, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl,
                                          bool first) {
  constexpr uint32_t idesc = make_idesc(128, DN, false, true, true);
#pragma unroll
  for (int kk = 0; kk < kN / 8; ++kk) {
    const uint64_t dh = make_sw128_32b_desc(bh + kk * 1024, kN * 128, 512);
    const uint64_t dl = make_sw128_32b_desc(bl + kk * 1024, kN * 128, 512);
    mma_tf32_ts(acc, ah + kk * 8, dh, idesc, (!first || kk > 0) ? 1u : 0u);
    mma_tf32_ts(acc, ah + kk * 8, dl, idesc, 1u);
    mma_tf32_ts(acc, al + kk * 8, dh, idesc, 1u);
  }
}

// out = A[tmem hi / lo, K = D] * B[stage tile hi / lo, K-major, N = kN]^T
template <int D, int kN>
__device__ __forceinline__ void issue_scores(uint32_t out, uint32_t ah, uint32_t al, uint32_t bh, uint32_t bl) {
  constexpr uint32_t idesc = make_idesc(128, kN, false, false, true);
#pragma unroll
  for (int kk = 0; kk < D / 8; ++kk) {
    const uint32_t off = (kk >> 2) * (kN * 128) + (kk & 3) * 32;
    const uint64_t dh = make_sw128_desc(bh + off, 16, 1024);
    const uint64_t dl = make_sw128_desc(bl + off, 16, 1024);
    mma_tf32_ts(out, ah + kk * 8, dh, idesc, kk > 0 ? 1u : 0u);
    mma_tf32_ts(out, ah + kk * 8, dl, idesc, 1u);
    mma_tf32_ts(out, al + kk * 8, dh, idesc, 1u);
  }
}

template <int MODE, int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kBwdThreads, 1)
    bwd_kernel(const __grid_constant__ CUtensorMap tm_sa, const __grid_constant__ CUtensorMap tm_sb, const Params p) {
  using Cfg = BwdCfg<MODE, DQK, DV>;
  constexpr int kN = Cfg::kN, kHalf = Cfg::kHalf, kStages = Cfg::kStages;
  constexpr bool kRowsAreQueries = MODE == kDQ;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc::align1024(smem_raw);
  BwdBarriers* bars = reinterpret_cast<BwdBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;

  const int64_t S_res = kRowsAreQueries ? p.S_q : p.S_kv;  // resident rows
  const int64_t S_str = kRowsAreQueries ? p.S_kv : p.S_q;  // streamed rows
  int64_t b, tord;
  raster(blockIdx.x, p.B, (S_res + 127) / 128, b, tord);
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  // DQ: longest causal query tiles first; DK / DV: low key tiles (most query rows) first
  const int64_t rt = kRowsAreQueries ? (S_res + 127) / 128 - 1 - tord : tord;
  const int64_t r0 = rt * 128;
  const int64_t n_all = (S_str + kN - 1) / kN;
  int tile0 = 0, n = static_cast<int>(n_all);
  if (p.causal) {
    if (kRowsAreQueries) {
      n = static_cast<int>(min(n_all, (r0 + 127) / kN + 1));
    } else {
      tile0 = static_cast<int>(r0 / kN);
      n = static_cast<int>(n_all - tile0 > 0 ? n_all - tile0 : 0);
    }
  }

  if (threadIdx.x == 0) {
    mbar_init(&bars->res_ready, 256);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars->st_full[s], 1);
      mbar_init(&bars->st_ready[s], 128);
      mbar_init(&bars->st_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], 256);
    }
    mbar_init(&bars->acc_done, 1);
    mbar_init(&bars->mma_done, 1);
    mbar_init(&bars->acc_step, 1);
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
      tma_prefetch_desc(&tm_sa);
      tma_prefetch_desc(&tm_sb);
      int issued = 0;
      for (int t = 0; t < n; ++t) {
        const int s = t % kStages;
        TF32_PROBE_T0(p0);
        if (!mbar_wait(&bars->st_empty[s], ((t / kStages) & 1) ^ 1, ctl)) break;
        TF32_PROBE_ADD(8, p0);
        const int row0 = (tile0 + t) * kN;
        mbar_expect_tx(&bars->st_full[s], Cfg::kSABytes + Cfg::kSBBytes);
#pragma unroll
        for (int c = 0; c < DQK / 32; ++c)
          tma_load_rows(smem + Cfg::sa_hi(s) + c * kN * 128, &tm_sa, c * 32, row0, hb, ob, &bars->st_full[s], HEADS);
#pragma unroll
        for (int c = 0; c < DV / 32; ++c)
          tma_load_rows(smem + Cfg::sb_hi(s) + c * kN * 128, &tm_sb, c * 32, row0, hb, ob, &bars->st_full[s], HEADS);
        issued = t + 1;
      }
      if (*ctl.abort_flag) {
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
      if constexpr (Cfg::kHasY) {
        // one tile buffer: S at tT, dP at tT + kN; dS hi / lo written over them
        for (int t = 0; ok && t <= n; ++t) {
          if (t > 0) {  // dQ / dK (+)= dS(t-1) SA(t-1)
            const int sp = (t - 1) % kStages;
            TF32_PROBE_T0(w0);
            if (!mbar_wait(&bars->p_full[0], (t - 1) & 1, ctl)) {
              ok = false;
              break;
            }
            TF32_PROBE_ADD(0, w0);
            tc_fence_after();
            // a fresh accumulator every tile: the elementwise threads fold the
            // previous tile's into their fp32 running total (see below)
            issue_acc<DQK, kN>(tmem + Cfg::kAcc, tT, tT + kN, sb + Cfg::sa_mh(sp), sb + Cfg::sa_ml(sp), true);
            mma_commit(&bars->st_empty[sp]);
          }
          if (t == n) break;
          const int s = t % kStages;
          TF32_PROBE_T0(w1);
          if (!mbar_wait(&bars->st_ready[s], (t / kStages) & 1, ctl)) {
            ok = false;
            break;
          }
          TF32_PROBE_ADD(1, w1);
          tc_fence_after();
          TF32_PROBE_T0(w3);
          issue_scores<DQK, kN>(tT, tmem + Cfg::kXh, tmem + Cfg::kXl, sb + Cfg::sa_hi(s), sb + Cfg::sa_lo(s));
          issue_scores<DV, kN>(tT + kN, tmem + Cfg::kYh, tmem + Cfg::kYl, sb + Cfg::sb_hi(s), sb + Cfg::sb_lo(s));
          mma_commit(&bars->s_full[0]);
          TF32_PROBE_ADD(3, w3);
        }
      } else {
        // two tile buffers (S^T / P~^T hi, P~^T lo) of 2 kN columns
        auto issue_dv = [&](int t) -> bool {
          const int s = t % kStages, bb = t & 1;
          if (!mbar_wait(&bars->p_full[bb], (t >> 1) & 1, ctl)) return false;
          tc_fence_after();
          const uint32_t buf = tT + bb * 2 * kN;
          // fresh accumulator every tile, folded into the elementwise threads' total
          issue_acc<DV, kN>(tmem + Cfg::kAcc, buf, buf + kN, sb + Cfg::sb_hi(s), sb + Cfg::sb_lo(s), true);
          mma_commit(&bars->st_empty[s]);
          mma_commit(&bars->acc_step);
          return true;
        };
        for (int t = 0; ok && t < n; ++t) {
          const int s = t % kStages, bb = t & 1;
          if (!mbar_wait(&bars->st_ready[s], (t / kStages) & 1, ctl)) {
            ok = false;
            break;
          }
          tc_fence_after();
          issue_scores<DQK, kN>(tT + bb * 2 * kN, tmem + Cfg::kXh, tmem + Cfg::kXl, sb + Cfg::sa_hi(s),
                                sb + Cfg::sa_lo(s));
          mma_commit(&bars->s_full[bb]);
          if (t > 0 && !issue_dv(t - 1)) {
            ok = false;
            break;
          }
        }
        if (ok) issue_dv(n - 1);
      }
      mma_commit(&bars->acc_done);
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
      TF32_PROBE_T0(c0);
      if (!tc::warp_wait(&bars->st_full[s], (t / kStages) & 1, ctl)) break;
      if (tid == 0) TF32_PROBE_ADD(6, c0);
      TF32_PROBE_T0(c1);
      if (!kRowsAreQueries) {  // lse (log2 units) and D of the tile's query rows
        float* vec = reinterpret_cast<float*>(smem + Cfg::vec(s));
        const int64_t i = static_cast<int64_t>(tile0 + t) * kN + (tid % kN);
        const bool in = i < p.S_q;
        if (tid < kN) vec[tid] = in ? p.lse[b * p.S_q + i] * kLog2e : INFINITY;
        else if (MODE == kDK && tid < 2 * kN) vec[tid] = in ? p.delta[b * p.S_q + i] : 0.0f;
      }
      if constexpr (Cfg::kHasY)
        split_tile_dual<kN>(smem + Cfg::sa_hi(s), smem + Cfg::sa_lo(s), smem + Cfg::sa_mh(s), smem + Cfg::sa_ml(s),
                            Cfg::kSABytes, tid, 128);
      else
        split_tile(smem + Cfg::sa_hi(s), smem + Cfg::sa_lo(s), Cfg::kSABytes, tid, 128);
      split_tile(smem + Cfg::sb_hi(s), smem + Cfg::sb_lo(s), Cfg::kSBBytes, tid, 128);
      fence_proxy_async_smem();
      if (tid == 0) TF32_PROBE_ADD(7, c1);
      mbar_arrive(&bars->st_ready[s]);
    }
  } else {
    // ------------------------------------------------ elementwise warps
    const int half = warp >> 2;
    const int r = (warp & 3) * 32 + lane;  // TMEM lane = resident row in tile
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const int col0 = half * kHalf;
    const int64_t rr = r0 + r;             // resident row (query for DQ, key for DK / DV)
    const bool row_ok = rr < S_res;
    const float sl2 = p.scale_log2, dp_inv = p.dp_inv;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    // resident operands to TMEM: this thread's half of the columns of its row
    {
      const void* xsrc = kRowsAreQueries ? p.q : p.k;
      const float* xrow = static_cast<const float*>(xsrc) + (row_ok ? row_offset_t<HEADS>(p.H, b, rr, S_res, p.D_qk) : 0);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c) {
        const int cc = half * (DQK / 2) + c * 32;
        row_to_tmem(xrow, cc, p.D_qk, row_ok, tmem + lane_base + Cfg::kXh + cc, tmem + lane_base + Cfg::kXl + cc);
      }
      if constexpr (Cfg::kHasY) {
        const void* ysrc = kRowsAreQueries ? p.d_o : p.v;
        const float* yrow = static_cast<const float*>(ysrc) + (row_ok ? row_offset_t<HEADS>(p.H, b, rr, S_res, p.D_v) : 0);
        constexpr int HC = DV / 2 < 32 ? 32 : DV / 2;  // columns per half (D_v = 32: half 0 takes all)
        if (half * HC < DV) {
#pragma unroll
          for (int c = 0; c < HC / 32; ++c) {
            const int cc = half * HC + c * 32;
            row_to_tmem(yrow, cc, p.D_v, row_ok, tmem + lane_base + Cfg::kYh + cc, tmem + lane_base + Cfg::kYl + cc);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->res_ready);
    }
    // DQ: D_i = sum_d dO O (minus the stats gradient) over the whole row, and lse
    float delta = 0.0f, lse2 = INFINITY;
    if (MODE == kDQ && row_ok) {
      const float* orow = static_cast<const float*>(p.o) + row_offset_t<HEADS>(p.H, b, rr, p.S_q, p.D_v);
      const float* grow = static_cast<const float*>(p.d_o) + row_offset_t<HEADS>(p.H, b, rr, p.S_q, p.D_v);
      float acc[4] = {0.f, 0.f, 0.f, 0.f};
      for (int c = 0; c < p.D_v; c += 4) {
        const float4 o4 = *reinterpret_cast<const float4*>(orow + c);
        const float4 g4 = *reinterpret_cast<const float4*>(grow + c);
        acc[0] = fmaf(g4.x, o4.x, acc[0]);
        acc[1] = fmaf(g4.y, o4.y, acc[1]);
        acc[2] = fmaf(g4.z, o4.z, acc[2]);
        acc[3] = fmaf(g4.w, o4.w, acc[3]);
      }
      delta = (acc[0] + acc[1]) + (acc[2] + acc[3]);
      if (p.d_stats) delta -= p.d_stats[b * p.S_q + rr];
      if (half == 0) p.delta[b * p.S_q + rr] = delta;
      lse2 = p.lse[b * p.S_q + rr] * kLog2e;
    }
    const uint64_t step_i = static_cast<uint64_t>(p.S_kv) * kLcgA;  // counter step between query rows
    const uint32_t step_lo = static_cast<uint32_t>(step_i), step_hi = static_cast<uint32_t>(step_i >> 32);
    // DQ / DK: running total of this thread's half of the accumulator row.  The
    // tensor cores' fp32 accumulation is not round-to-nearest; over thousands
    // of MMAs (dQ over S_kv = 4096 keys) its error reaches a few 1e-5.  So
    // each tile's products go to a fresh accumulator, folded in here in fp32:
    // s_full(t) is committed after acc(t-1) was issued, so it is complete.
    // DV: the same, with the total of this thread's kTotCols columns of dV,
    // folded at the end of every tile after acc_step shows the previous tile's
    // accumulating MMAs complete (the next tile's restart the accumulator).
    static_assert(!Cfg::kHasY || Cfg::kAccCols == 64, "running total sized for D_qk = 64");
    constexpr int kTotCols = Cfg::kHasY ? 32 : (DV / 2 < 32 ? 32 : DV / 2);
    const bool has_cols = Cfg::kHasY || half * kTotCols < DV;  // D_v = 32: half 1 holds none
    float tot[kTotCols];
#pragma unroll
    for (int e = 0; e < kTotCols; ++e) tot[e] = 0.0f;
    bool ok = true;
    for (int t = 0; t < n; ++t) {
      const int s = t % kStages;
      const int bb = Cfg::kHasY ? 0 : (t & 1);
      const uint32_t ph = Cfg::kHasY ? (t & 1) : ((t >> 1) & 1);
      TF32_PROBE_T0(e0);
      if (!tc::warp_wait(&bars->s_full[bb], ph, ctl) ||
          (!kRowsAreQueries && !tc::warp_wait(&bars->st_ready[s], (t / kStages) & 1, ctl))) {
        ok = false;
        break;
      }
      if (threadIdx.x == 0) TF32_PROBE_ADD(4, e0);
      TF32_PROBE_T0(e1);
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + Cfg::kT + bb * 2 * kN + col0;  // S / S^T (hi written back here)
      const uint32_t tD = tS + kN;                                          // dP / dP^T, or P~^T lo
      uint32_t sv[kHalf], dpv[kHalf];
      tmem_ld_cols<kHalf>(tS, sv);
      if (Cfg::kHasY) tmem_ld_cols<kHalf>(tD, dpv);
      if (Cfg::kHasY && t > 0) {
        uint32_t a[32];
        SDPA_TMEM_LD32(tmem + lane_base + Cfg::kAcc + half * 32, a);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) tot[e] += __uint_as_float(a[e]);
      }
      tmem_wait_ld();
      const int64_t c0g = static_cast<int64_t>(tile0 + t) * kN + col0;  // first streamed row of these columns
      uint32_t hv[kHalf], lv[kHalf];
      if (kRowsAreQueries) {
        // columns are keys j = c0g + c of query row i = rr
        int64_t lim64 = p.S_kv - c0g;
        if (p.causal) lim64 = min(lim64, rr - c0g + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kHalf ? kHalf : lim64));
        LcgWalk st(DROP ? lcg_state(p.rng_base + static_cast<uint64_t>(b * p.S_q + rr) * static_cast<uint64_t>(p.S_kv),
                                    static_cast<uint64_t>(c0g))
                        : 0);
#pragma unroll
        for (int c = 0; c < kHalf; ++c) {
          float pr = ex2(fmaf(__uint_as_float(sv[c]), sl2, -lse2));
          pr = (pr > kEps && c < lim) ? pr : 0.0f;
          float kf = 1.0f;
          if (DROP) {
            kf = st.dropped(thr_m1) ? 0.0f : dp_inv;
            st.step();
          }
          const float ds = pr * fmaf(kf, __uint_as_float(dpv[c]), -delta);
          float h, w;
          split_tf32(ds, h, w);
          hv[c] = __float_as_uint(h);
          lv[c] = __float_as_uint(w);
        }
      } else {
        // columns are query rows i = c0g + c of key row j = rr
        const float* vec = reinterpret_cast<const float*>(smem + Cfg::vec(s)) + col0;
        int lo = -1;  // causal: column c valid iff c0g + c >= j
        if (p.causal) {
          const int64_t d = rr - c0g;
          lo = static_cast<int>(d < -1 ? -1 : (d > kHalf ? kHalf : d));
        }
        LcgWalk st(DROP ? lcg_state(p.rng_base + static_cast<uint64_t>(b * p.S_q + c0g) * static_cast<uint64_t>(p.S_kv),
                                    static_cast<uint64_t>(rr))
                        : 0);
#pragma unroll
        for (int c = 0; c < kHalf; ++c) {
          float pr = ex2(fmaf(__uint_as_float(sv[c]), sl2, -vec[c]));
          pr = (pr > kEps && c >= lo) ? pr : 0.0f;
          float kf = 1.0f;
          if (DROP) {
            kf = st.dropped(thr_m1) ? 0.0f : dp_inv;
            st.step(step_lo, step_hi);
          }
          const float x = MODE == kDK ? pr * fmaf(kf, __uint_as_float(dpv[c]), -vec[kN + c]) : pr * kf;
          float h, w;
          split_tf32(x, h, w);
          hv[c] = __float_as_uint(h);
          lv[c] = __float_as_uint(w);
        }
      }
      tmem_st_cols<kHalf>(tS, hv);
      tmem_st_cols<kHalf>(tD, lv);
      if (!Cfg::kHasY && t > 0 && has_cols) {
        // acc_step is waited every tile by these warps, so never two phases behind
        if (!tc::warp_wait(&bars->acc_step, (t - 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < kTotCols / 32; ++c) {
          uint32_t a[32];
          SDPA_TMEM_LD32(tmem + lane_base + Cfg::kAcc + half * kTotCols + c * 32, a);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) tot[c * 32 + e] += __uint_as_float(a[e]);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      if (threadIdx.x == 0) TF32_PROBE_ADD(5, e1);
      mbar_arrive(&bars->p_full[bb]);
    }
    if (ok && n > 0) ok = tc::warp_wait(&bars->acc_done, 0, ctl);
    if (ok) {
      tc_fence_after();
      void* dst = MODE == kDQ ? p.dq : (MODE == kDK ? p.dk : p.dv);
      const int D = MODE == kDV ? p.D_v : p.D_qk;
      constexpr int DA = Cfg::kAccCols;
      float* drow = static_cast<float*>(dst) + (row_ok ? row_offset_t<HEADS>(p.H, b, rr, S_res, D) : 0);
      if constexpr (Cfg::kHasY) {
        uint32_t a[32];
        if (n > 0) {
          SDPA_TMEM_LD32(tmem + lane_base + Cfg::kAcc + half * 32, a);
          tmem_wait_ld();
        }
        if (row_ok) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            const int col = half * 32 + 4 * g;
            float v4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) v4[e] = (tot[4 * g + e] + (n > 0 ? __uint_as_float(a[4 * g + e]) : 0.0f)) * p.scale;
            if (col < D) *reinterpret_cast<float4*>(drow + col) = make_float4(v4[0], v4[1], v4[2], v4[3]);
          }
        }
      } else {
        if (has_cols) {
#pragma unroll
          for (int c = 0; c < kTotCols / 32; ++c) {
            uint32_t a[32];
            if (n > 0) {
              SDPA_TMEM_LD32(tmem + lane_base + Cfg::kAcc + half * kTotCols + c * 32, a);
              tmem_wait_ld();
            }
            if (row_ok) {
#pragma unroll
              for (int g = 0; g < 8; ++g) {
                const int col = half * kTotCols + c * 32 + 4 * g;
                float v4[4];
#pragma unroll
                for (int e = 0; e < 4; ++e)
                  v4[e] = tot[c * 32 + 4 * g + e] + (n > 0 ? __uint_as_float(a[4 * g + e]) : 0.0f);
                if (col < D) *reinterpret_cast<float4*>(drow + col) = make_float4(v4[0], v4[1], v4[2], v4[3]);
              }
            }
          }
        }
      }
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
