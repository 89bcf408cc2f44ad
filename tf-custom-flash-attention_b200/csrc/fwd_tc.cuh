// Forward attention on the 5th-generation tensor cores (sm_100a), fp16 in,
// fp32 accumulate.  One CTA = one 128-row query tile of one batch row.
//
//   warp 4      TMA producer: Q once, then K/V tiles (128 keys) into a
//               2-stage ring of 128B-swizzled shared-memory buffers
//   warp 5      MMA issuer (one thread) + TMEM owner:
//                 S[j%2] = Q K_j^T           (SS MMA, 128x128, K = D_qk)
//                 O     += P_{j-1} V_{j-1}   (TS MMA, A = P read from TMEM)
//   warps 0-3   softmax: thread t owns query row t = TMEM lane t.  Reads its
//               S row (128 fp32) from TMEM, masks, online max in log2 units
//               with scale folded into the exponent, exp2, row sum, dropout,
//               writes P (fp16 pairs) back over S, rescales O only when the
//               running max grew by more than 2^8 (exact: the final division
//               uses the same reference max), then the epilogue.
//
// TMEM columns: [0,128) S0/P0, [128,256) S1/P1, [256,256+DV) O.
// Semantics follow sdpa/sdpa_fwd.cu.cc:60-173: l sums pre-dropout p,
// stats = max + ln(l + 1e-6), O = acc / l guarded by l > 1e-6.
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace sdpa_b200 {
namespace tc {

constexpr int kBM = 128;  // query rows per CTA (= TMEM lanes)
constexpr int kBN = 128;  // keys per tile
constexpr int kFwdThreads = 192;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int DQK, int DV>
struct FwdCfg {
  static constexpr int kStages = 2;
  static constexpr uint32_t kQBytes = kBM * DQK * 2;
  static constexpr uint32_t kKBytes = kBN * DQK * 2;
  static constexpr uint32_t kVBytes = kBN * DV * 2;
  static constexpr uint32_t kQOff = 0;
  static constexpr uint32_t kKOff = kQOff + kQBytes;
  static constexpr uint32_t kVOff = kKOff + kStages * kKBytes;
  static constexpr uint32_t kBarOff = kVOff + kStages * kVBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;  // + barriers + alignment slack
  static constexpr uint32_t kTmemCols = 512;
  static_assert(256 + DV <= 512, "TMEM budget");
};

struct FwdBarriers {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t o_final;  // every PV MMA done (one phase)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

// Warp-uniform bounded wait: every lane spins until all lanes observed the
// phase; the give-up decision is taken by lane 0 and broadcast, so the warp
// never diverges in front of a .sync.aligned instruction.
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, const WaitCtl& ctl) {
  bool done = mbar_try_wait(bar, parity);
  uint32_t spins = 0;
  while (!__all_sync(0xffffffffu, done)) {
    if (!done) done = mbar_try_wait(bar, parity);
    if ((++spins & 255u) == 0) {
      int give_up = 0;
      if ((threadIdx.x & 31) == 0) give_up = (*ctl.abort_flag) || (globaltimer_ns() > ctl.deadline_ns);
      give_up = __shfl_sync(0xffffffffu, give_up, 0);
      if (give_up) {
        if ((threadIdx.x & 31) == 0) {
          *ctl.abort_flag = 1;
          atomicOr(&g_status_word, kStatusTimeout);
        }
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ uint8_t* align1024(uint8_t* raw) {
  const uint32_t a = smem_u32(raw);
  return raw + ((1024u - (a & 1023u)) & 1023u);
}

template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
               const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using Cfg = FwdCfg<DQK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  FwdBarriers* bars = reinterpret_cast<FwdBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  const int64_t n_qt = (p.S_q + kBM - 1) / kBM;
  int64_t b, tord;
  raster(blockIdx.x, p.B, n_qt, b, tord);
  // head and outer batch of folded row b (layout [B/H, S, H, D] when HEADS)
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  constexpr bool heads = HEADS;
  const int64_t qt = n_qt - 1 - tord;  // longest causal rows first
  const int64_t m0 = qt * kBM;
  const int64_t n_kv_all = (p.S_kv + kBN - 1) / kBN;
  const int n_kv = static_cast<int>(p.causal ? min(n_kv_all, qt + 1) : n_kv_all);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], kBM);
    }
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->o_final, 1);
    mbar_init(&bars->mma_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(&bars->tmem_base, Cfg::kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  pdl_launch_dependents();
  pdl_wait();  // before any global access and before the wait deadline starts
  const uint32_t tmem = bars->tmem_base;
  WaitCtl ctl;
  ctl.deadline_ns = globaltimer_ns() + p.timeout_ns;
  ctl.abort_flag = &bars->abort_flag;

  const uint32_t sQ = smem_u32(smem + Cfg::kQOff);
  const uint32_t sK0 = smem_u32(smem + Cfg::kKOff);
  const uint32_t sV0 = smem_u32(smem + Cfg::kVOff);

  if (warp == 4) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && n_kv > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_expect_tx(&bars->q_full, Cfg::kQBytes);
#pragma unroll
      for (int c = 0; c < DQK / 64; ++c)
        tma_load_rows(smem + Cfg::kQOff + c * kBM * 128, &tm_q, c * 64, static_cast<int>(m0), hb, ob,
                    &bars->q_full, heads);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bars->kv_empty[s], ((j >> 1) & 1) ^ 1, ctl)) break;
        uint8_t* kdst = smem + Cfg::kKOff + s * Cfg::kKBytes;
        uint8_t* vdst = smem + Cfg::kVOff + s * Cfg::kVBytes;
        mbar_expect_tx(&bars->k_full[s], Cfg::kKBytes);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_rows(kdst + c * kBN * 128, &tm_k, c * 64, j * kBN, hb, ob, &bars->k_full[s], heads);
        mbar_expect_tx(&bars->v_full[s], Cfg::kVBytes);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_rows(vdst + c * kBN * 128, &tm_v, c * 64, j * kBN, hb, ob, &bars->v_full[s], heads);
        issued = j + 1;
      }
      if (*ctl.abort_flag) {
        // Let the copies already in flight land before the CTA exits.
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          mbar_wait(&bars->k_full[j & 1], (j >> 1) & 1, drain);
          mbar_wait(&bars->v_full[j & 1], (j >> 1) & 1, drain);
        }
        if (issued == 0) mbar_wait(&bars->q_full, 0, drain);
      }
    }
  } else if (warp == 5) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_qk = make_idesc(kBM, kBN, false, false, false);
      constexpr uint32_t idesc_pv = make_idesc(kBM, DV, false, true, false);
      const uint32_t tO = tmem + 256;
      bool ok = mbar_wait(&bars->q_full, 0, ctl);
      auto issue_pv = [&](int t) -> bool {
        const int s = t & 1;
        if (!mbar_wait(&bars->p_full[s], (t >> 1) & 1, ctl)) return false;
        if (!mbar_wait(&bars->v_full[s], (t >> 1) & 1, ctl)) return false;
        tc_fence_after();
        const uint32_t vbase = sV0 + s * Cfg::kVBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t bdesc = make_sw128_desc(vbase + kk * 16 * 128, kBN * 128, 1024);
          mma_f16_ts(tO, tmem + s * 128 + kk * 8, bdesc, idesc_pv, (t > 0 || kk > 0) ? 1u : 0u);
        }
        mma_commit(&bars->kv_empty[s]);
        mma_commit(&bars->o_done);
        return true;
      };
      for (int j = 0; ok && j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bars->k_full[s], (j >> 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t kbase = sK0 + s * Cfg::kKBytes;
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          const uint64_t adesc = make_sw128_desc(sQ + koff, 16, 1024);
          const uint64_t bdesc = make_sw128_desc(kbase + koff, 16, 1024);
          mma_f16_ss(tmem + s * 128, adesc, bdesc, idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(&bars->s_full[s]);
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(n_kv - 1);
      mma_commit(&bars->o_final);
      // Every MMA issued so far must finish before TMEM is released.
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else {
    // ------------------------------------------------ softmax warpgroup
    const int t = threadIdx.x;  // 0..127 = TMEM lane = query row in tile
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t row = m0 + t;
    const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + row) * static_cast<uint64_t>(p.S_kv);
    float m_run = -INFINITY;  // true running max (log2 units, scaled)
    float m_use = -INFINITY;  // reference max the exponentials are taken against
    float l = 0.0f;           // sum of exp2(x - m_use), pre-dropout
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;
      if (!warp_wait(&bars->s_full[s], (j >> 1) & 1, ctl)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[128];
      SDPA_TMEM_LD32(tmem + lane_base + s * 128 + 0, (r + 0));
      SDPA_TMEM_LD32(tmem + lane_base + s * 128 + 32, (r + 32));
      SDPA_TMEM_LD32(tmem + lane_base + s * 128 + 64, (r + 64));
      SDPA_TMEM_LD32(tmem + lane_base + s * 128 + 96, (r + 96));
      tmem_wait_ld();
      const int64_t kv0 = static_cast<int64_t>(j) * kBN;
      // Scale is folded into one FFMA per element when positive (max over the
      // raw scores); otherwise the scores are scaled first.
      const bool fold = p.scale_log2 > 0.0f;
      const float sl = fold ? p.scale_log2 : 1.0f;
      if (!fold) {
#pragma unroll
        for (int c = 0; c < 128; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * p.scale_log2);
      }
      // Masking only where this warp's rows meet the key range or the diagonal.
      const int64_t row_w0 = m0 + warp * 32;
      const bool edge = (kv0 + kBN > p.S_kv) || (p.causal && kv0 + kBN - 1 > row_w0);
      if (edge) {
        int64_t lim64 = p.S_kv - kv0;
        if (p.causal) lim64 = min(lim64, row - kv0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kBN ? kBN : lim64));
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= lim) r[c] = __float_as_uint(-INFINITY);
      }
      float tmax_raw = -INFINITY;
#pragma unroll
      for (int c = 0; c < 128; ++c) tmax_raw = fmaxf(tmax_raw, __uint_as_float(r[c]));
      const float tmax = tmax_raw * sl;
      m_run = fmaxf(m_run, tmax);
      float alpha = 1.0f;
      bool rescale_o = false;
      if (tmax > m_use + kRescaleThreshold) {
        alpha = ex2(m_use - m_run);  // 0 when m_use = -inf
        rescale_o = (j > 0) && (m_use != -INFINITY);
        m_use = m_run;
        l *= alpha;
      }
      const float mu = (m_use == -INFINITY) ? 0.0f : m_use;
      float rs = 0.0f;
      uint32_t pk[64];
      if (DROP) {
        LcgWalk st(lcg_state(rbase, static_cast<uint64_t>(kv0)));
        const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          float p0 = ex2(fmaf(__uint_as_float(r[c]), sl, -mu));
          float p1 = ex2(fmaf(__uint_as_float(r[c + 1]), sl, -mu));
          rs += p0 + p1;
          const bool d0 = st.dropped(thr_m1);
          st.step();
          const bool d1 = st.dropped(thr_m1);
          st.step();
          pk[c / 2] = pack_half2(d0 ? 0.0f : p0, d1 ? 0.0f : p1);
        }
      } else {
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(r[c]), sl, -mu));
          const float p1 = ex2(fmaf(__uint_as_float(r[c + 1]), sl, -mu));
          rs += p0 + p1;
          pk[c / 2] = pack_half2(p0, p1);
        }
      }
      l += rs;
      SDPA_TMEM_ST32(tmem + lane_base + s * 128 + 0, (pk + 0));
      SDPA_TMEM_ST32(tmem + lane_base + s * 128 + 32, (pk + 32));
      if (__any_sync(0xffffffffu, rescale_o)) {
        // O must hold PV_{j-1} before it is rescaled (and before PV_j).
        if (!warp_wait(&bars->o_done, (j - 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float a = rescale_o ? alpha : 1.0f;
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t o[32];
          SDPA_TMEM_LD32(tmem + lane_base + 256 + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
          SDPA_TMEM_ST32(tmem + lane_base + 256 + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[s]);
    }
    // ----------------------------------------------------------- epilogue
    // Not o_done with parity (n_kv - 1) & 1: PV(j-1) is issued after S(j), so
    // o_done may still be two phases behind here and that parity would match
    // an older phase.
    if (ok && n_kv > 0) ok = warp_wait(&bars->o_final, 0, ctl);
    if (ok) {
      tc_fence_after();
      float lse, inv;
      if (m_run == -INFINITY) {
        lse = kNegInit + logf(kEps);
        inv = 0.0f;
      } else {
        const float l_true = l * ex2(m_use - m_run);  // sum relative to the true max
        lse = m_run * kLn2 + logf(l_true + kEps);
        inv = (l_true > kEps) ? p.dp_inv / l : 0.0f;
      }
      const bool active = row < p.S_q;
      if (active) p.stats[b * p.S_q + row] = lse;
      __half* orow = static_cast<__half*>(p.out) + row_offset_t<HEADS>(p.H, b, row, p.S_q, p.D_v);
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
        uint32_t o[32];
        if (n_kv > 0) {
          SDPA_TMEM_LD32(tmem + lane_base + 256 + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        uint32_t h[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          h[e] = pack_half2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        if (active) {
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int col = c * 32 + w * 8;
            if (col < p.D_v)
              *reinterpret_cast<uint4*>(orow + col) = make_uint4(h[4 * w], h[4 * w + 1], h[4 * w + 2], h[4 * w + 3]);
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 5) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, Cfg::kTmemCols);
  }
}

// ============================================================================
// Paired forward: one CTA = two 128-row query tiles (A = rows m0.., B = rows
// m0+128..) of one batch row, sharing every K/V tile.  Two softmax
// warpgroups (warps 0-3 tile A, warps 4-7 tile B) alternate on the tensor
// pipe; the MMA warp issues, per key tile j,
//     S_A(j)  S_B(j)  PV_A(j)  S_A(j+1)  PV_B(j)  S_B(j+1)  PV_A(j+1) ...
// so each softmax pass overlaps two MMAs of the other tile.  TMEM: S_A/P_A
// [0,128), S_B/P_B [128,256), O_A [256, 256+DV), O_B [256+DV, 256+2*DV).
// Warp 8 = TMA producer, warp 9 = MMA issuer + TMEM owner.
constexpr int kPairThreads = 320;

template <int DQK, int DV>
struct PairCfg {
  static constexpr int kStages = 2;
  static constexpr uint32_t kQBytes = kBM * DQK * 2;  // one tile
  static constexpr uint32_t kKBytes = kBN * DQK * 2;
  static constexpr uint32_t kVBytes = kBN * DV * 2;
  static constexpr uint32_t kQOff = 0;  // A then B
  static constexpr uint32_t kKOff = kQOff + 2 * kQBytes;
  static constexpr uint32_t kVOff = kKOff + kStages * kKBytes;
  static constexpr uint32_t kBarOff = kVOff + kStages * kVBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static constexpr uint32_t kTmemCols = 512;
  static_assert(256 + 2 * DV <= 512, "TMEM budget");
};

struct PairBarriers {
  uint64_t q_full;
  uint64_t k_full[2];
  uint64_t v_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];   // per tile
  uint64_t p_full[2];   // per tile
  uint64_t o_done[2];   // per tile
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kPairThreads, 1)
    fwd_pair_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                    const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using Cfg = PairCfg<DQK, DV>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = align1024(smem_raw);
  PairBarriers* bars = reinterpret_cast<PairBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  const int64_t n_pairs = (p.S_q + 2 * kBM - 1) / (2 * kBM);
  int64_t b, tord;
  raster(blockIdx.x, p.B, n_pairs, b, tord);
  // head and outer batch of folded row b (layout [B/H, S, H, D] when HEADS)
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  constexpr bool heads = HEADS;
  const int64_t pq = n_pairs - 1 - tord;  // longest causal rows first
  const int64_t m0 = pq * 2 * kBM;
  const int64_t n_kv_all = (p.S_kv + kBN - 1) / kBN;
  // key tiles per query tile; tile A never needs more than tile B
  int n_t[2];
  n_t[0] = static_cast<int>(p.causal ? min(n_kv_all, 2 * pq + 1) : n_kv_all);
  n_t[1] = static_cast<int>(p.causal ? min(n_kv_all, 2 * pq + 2) : n_kv_all);
  const int n_kv = n_t[1];

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->kv_empty[s], 1);
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], kBM);
      mbar_init(&bars->o_done[s], 1);
    }
    mbar_init(&bars->mma_done, 1);
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

  if (warp == 8) {
    // ------------------------------------------------------ TMA producer
    if (lane == 0 && n_kv > 0) {
      tma_prefetch_desc(&tm_q);
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      mbar_expect_tx(&bars->q_full, 2 * Cfg::kQBytes);
#pragma unroll
      for (int t = 0; t < 2; ++t)
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_rows(smem + Cfg::kQOff + t * Cfg::kQBytes + c * kBM * 128, &tm_q, c * 64,
                      static_cast<int>(m0 + t * kBM), hb, ob, &bars->q_full, heads);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j & 1;
        if (!mbar_wait(&bars->kv_empty[s], ((j >> 1) & 1) ^ 1, ctl)) break;
        uint8_t* kdst = smem + Cfg::kKOff + s * Cfg::kKBytes;
        uint8_t* vdst = smem + Cfg::kVOff + s * Cfg::kVBytes;
        mbar_expect_tx(&bars->k_full[s], Cfg::kKBytes);
#pragma unroll
        for (int c = 0; c < DQK / 64; ++c)
          tma_load_rows(kdst + c * kBN * 128, &tm_k, c * 64, j * kBN, hb, ob, &bars->k_full[s], heads);
        mbar_expect_tx(&bars->v_full[s], Cfg::kVBytes);
#pragma unroll
        for (int c = 0; c < DV / 64; ++c)
          tma_load_rows(vdst + c * kBN * 128, &tm_v, c * 64, j * kBN, hb, ob, &bars->v_full[s], heads);
        issued = j + 1;
      }
      if (*ctl.abort_flag) {  // let copies in flight land before the CTA exits
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        mbar_wait(&bars->q_full, 0, drain);
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          mbar_wait(&bars->k_full[j & 1], (j >> 1) & 1, drain);
          mbar_wait(&bars->v_full[j & 1], (j >> 1) & 1, drain);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_qk = make_idesc(kBM, kBN, false, false, false);
      constexpr uint32_t idesc_pv = make_idesc(kBM, DV, false, true, false);
      const uint32_t sQ = smem_u32(smem + Cfg::kQOff);
      const uint32_t sK0 = smem_u32(smem + Cfg::kKOff);
      const uint32_t sV0 = smem_u32(smem + Cfg::kVOff);
      auto issue_s = [&](int t, int j) -> bool {  // S_t = Q_t K_j^T
        const int s = j & 1;
        if (t == 0 && !mbar_wait(&bars->k_full[s], (j >> 1) & 1, ctl)) return false;
        tc_fence_after();
        const uint32_t kbase = sK0 + s * Cfg::kKBytes, qbase = sQ + t * Cfg::kQBytes;
#pragma unroll
        for (int kk = 0; kk < DQK / 16; ++kk) {
          const uint32_t koff = (kk >> 2) * (kBM * 128) + (kk & 3) * 32;
          mma_f16_ss(tmem + t * 128, make_sw128_desc(qbase + koff, 16, 1024), make_sw128_desc(kbase + koff, 16, 1024),
                     idesc_qk, kk > 0 ? 1u : 0u);
        }
        mma_commit(&bars->s_full[t]);
        return true;
      };
      auto issue_pv = [&](int t, int j) -> bool {  // O_t += P_t V_j
        const int s = j & 1;
        if (!mbar_wait(&bars->p_full[t], j & 1, ctl)) return false;
        if (t == 0 || n_t[0] <= j)  // first user of V_j waits for it
          if (!mbar_wait(&bars->v_full[s], (j >> 1) & 1, ctl)) return false;
        tc_fence_after();
        const uint32_t vbase = sV0 + s * Cfg::kVBytes;
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk)
          mma_f16_ts(tmem + 256 + t * DV, tmem + t * 128 + kk * 8,
                     make_sw128_desc(vbase + kk * 16 * 128, kBN * 128, 1024), idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        mma_commit(&bars->o_done[t]);
        return true;
      };
      bool ok = mbar_wait(&bars->q_full, 0, ctl);
      // prologue: S_A(0) (when tile A has keys), S_B(0)
      if (ok && n_t[0] > 0) ok = issue_s(0, 0);
      if (ok) {
        if (n_t[0] == 0 && !mbar_wait(&bars->k_full[0], 0, ctl)) ok = false;
        if (ok) ok = issue_s(1, 0);
      }
      for (int j = 0; ok && j < n_kv; ++j) {
        if (j < n_t[0]) {
          if (!issue_pv(0, j)) { ok = false; break; }
          if (j + 1 < n_t[0] && !issue_s(0, j + 1)) { ok = false; break; }
        }
        if (!issue_pv(1, j)) { ok = false; break; }
        mma_commit(&bars->kv_empty[j & 1]);  // K_j, V_j no longer read
        if (j + 1 < n_kv) {
          if (j + 1 >= n_t[0] && !mbar_wait(&bars->k_full[(j + 1) & 1], ((j + 1) >> 1) & 1, ctl)) { ok = false; break; }
          if (!issue_s(1, j + 1)) { ok = false; break; }
        }
      }
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else {
    // ------------------------------------------------ softmax warpgroups
    const int t = warp >> 2;                     // query tile of this warpgroup
    const int wq = warp & 3;                     // TMEM lane quadrant
    const int r_in = wq * 32 + lane;             // TMEM lane = row in tile
    const uint32_t lane_base = static_cast<uint32_t>(wq * 32) << 16;
    const uint32_t tS = tmem + lane_base + t * 128;
    const uint32_t tO = tmem + lane_base + 256 + t * DV;
    const int64_t row = m0 + t * kBM + r_in;
    const int64_t row_w0 = m0 + t * kBM + wq * 32;
    const int n_my = n_t[t];
    const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + row) * static_cast<uint64_t>(p.S_kv);
    const bool fold = p.scale_log2 > 0.0f;  // scale folded into one FFMA (max over raw scores)
    const float sl = fold ? p.scale_log2 : 1.0f;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    float m_run = -INFINITY;  // true running max (log2 units, scaled)
    float m_use = -INFINITY;  // reference max the exponentials are taken against
    float l = 0.0f;           // sum of exp2(x - m_use), pre-dropout
    bool ok = true;
    for (int j = 0; j < n_my; ++j) {
      if (!warp_wait(&bars->s_full[t], j & 1, ctl)) {
        ok = false;
        break;
      }
      tc_fence_after();
      uint32_t r[128];
      SDPA_TMEM_LD32(tS + 0, (r + 0));
      SDPA_TMEM_LD32(tS + 32, (r + 32));
      SDPA_TMEM_LD32(tS + 64, (r + 64));
      SDPA_TMEM_LD32(tS + 96, (r + 96));
      tmem_wait_ld();
      const int64_t kv0 = static_cast<int64_t>(j) * kBN;
      if (!fold) {
#pragma unroll
        for (int c = 0; c < 128; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * p.scale_log2);
      }
      if ((kv0 + kBN > p.S_kv) || (p.causal && kv0 + kBN - 1 > row_w0)) {  // this warp meets an edge
        int64_t lim64 = p.S_kv - kv0;
        if (p.causal) lim64 = min(lim64, row - kv0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kBN ? kBN : lim64));
#pragma unroll
        for (int c = 0; c < 128; ++c)
          if (c >= lim) r[c] = __float_as_uint(-INFINITY);
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};  // four independent chains
#pragma unroll
      for (int c = 0; c < 128; c += 8)
#pragma unroll
        for (int q = 0; q < 4; ++q) mx[q] = fmax3(mx[q], __uint_as_float(r[c + 2 * q]), __uint_as_float(r[c + 2 * q + 1]));
      const float tmax_raw = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3]));
      const float tmax = tmax_raw * sl;
      m_run = fmaxf(m_run, tmax);
      float alpha = 1.0f;
      bool rescale_o = false;
      if (tmax > m_use + kRescaleThreshold) {
        alpha = ex2(m_use - m_run);  // 0 when m_use = -inf
        rescale_o = (j > 0) && (m_use != -INFINITY);
        m_use = m_run;
        l *= alpha;
      }
      const float mu = (m_use == -INFINITY) ? 0.0f : m_use;
      // P packed in place: r[c/2] <- (p_c, p_c+1) once both are read.  With
      // dropout (issue-bound) argument and row sum go in packed pairs; four
      // partial sums keep the add chains short.
      float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      const float nmu = -mu;
      if (DROP) {
        const uint64_t s0 = lcg_state(rbase, static_cast<uint64_t>(kv0));
        const uint32_t s0_lo = static_cast<uint32_t>(s0), s0_hi = static_cast<uint32_t>(s0 >> 32);
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          float x0, x1;
          ffma2(x0, x1, __uint_as_float(r[c]), __uint_as_float(r[c + 1]), sl, sl, nmu, nmu);
          const float p0 = ex2(x0), p1 = ex2(x1);
          const int q = (c >> 1) & 1;
          fadd2(rs[2 * q], rs[2 * q + 1], p0, p1);
          // state of column kv0 + c is s0 + c * A (dropped iff its hi32 < thr)
          const bool d0 = lcg_hi_at(s0_lo, s0_hi, p.one, static_cast<uint64_t>(c) * kLcgA) <= thr_m1;
          const bool d1 = lcg_hi_at(s0_lo, s0_hi, p.one, static_cast<uint64_t>(c + 1) * kLcgA) <= thr_m1;
          r[c / 2] = pack_half2(d0 ? 0.0f : p0, d1 ? 0.0f : p1);
        }
      } else {  // bound by MUFU and the tensor pipe, not by issue: scalar forms
#pragma unroll
        for (int c = 0; c < 128; c += 2) {
          const float p0 = ex2(fmaf(__uint_as_float(r[c]), sl, nmu));
          const float p1 = ex2(fmaf(__uint_as_float(r[c + 1]), sl, nmu));
          rs[(c >> 1) & 3] += p0 + p1;
          r[c / 2] = pack_half2(p0, p1);
        }
      }
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
      SDPA_TMEM_ST32(tS + 0, (r + 0));
      SDPA_TMEM_ST32(tS + 32, (r + 32));
      if (__any_sync(0xffffffffu, rescale_o)) {
        // O_t holds PV_t(j-1) (committed before S_t(j)); rescale it before PV_t(j)
        if (!warp_wait(&bars->o_done[t], (j - 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float a = rescale_o ? alpha : 1.0f;
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t o[32];
          SDPA_TMEM_LD32(tO + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
          SDPA_TMEM_ST32(tO + c * 32, o);
        }
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->p_full[t]);
    }
    // ----------------------------------------------------------- epilogue
    if (ok && n_my > 0) ok = warp_wait(&bars->o_done[t], (n_my - 1) & 1, ctl);
    if (ok) {
      tc_fence_after();
      float lse, inv;
      if (m_run == -INFINITY) {
        lse = kNegInit + logf(kEps);
        inv = 0.0f;
      } else {
        const float l_true = l * ex2(m_use - m_run);  // sum relative to the true max
        lse = m_run * kLn2 + logf(l_true + kEps);
        inv = (l_true > kEps) ? p.dp_inv / l : 0.0f;
      }
      const bool active = row < p.S_q;
      if (active) p.stats[b * p.S_q + row] = lse;
      __half* orow = static_cast<__half*>(p.out) + row_offset_t<HEADS>(p.H, b, row, p.S_q, p.D_v);
#pragma unroll
      for (int c = 0; c < DV / 32; ++c) {
        uint32_t o[32];
        if (n_my > 0) {
          SDPA_TMEM_LD32(tO + c * 32, o);
          tmem_wait_ld();
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = 0u;
        }
        uint32_t h[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          h[e] = pack_half2(__uint_as_float(o[2 * e]) * inv, __uint_as_float(o[2 * e + 1]) * inv);
        if (active) {
#pragma unroll
          for (int w = 0; w < 4; ++w) {
            const int col = c * 32 + w * 8;
            if (col < p.D_v)
              *reinterpret_cast<uint4*>(orow + col) = make_uint4(h[4 * w], h[4 * w + 1], h[4 * w + 2], h[4 * w + 3]);
          }
        }
      }
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
