// fp32 forward attention on the 5th-generation tensor cores (sm_100a) with
// the 3xTF32 split: every fp32 operand x is held as two tf32 values
// x = hi + lo (split_tf32) and each product a*b is issued as three
// kind::tf32 MMAs ah*bh + ah*bl + al*bh, which keeps the error near 2^-21 of
// the product (fp32-level) where one tf32 product would be off by 2^-11.
//
// One CTA = 128 query rows of one batch row (TMEM lanes); key tiles of kBN
// rows (64 or 32, see FwdCfg).
//   warps 0-3  softmax: thread t owns query row t.  First loads its Q row from
//              HBM, splits it and writes Qh / Ql into TMEM (the A operand of
//              S = Q K^T stays on chip: no shared-memory traffic for it).  Per
//              tile: S row from TMEM, masks, online max, exp2, row sum,
//              dropout, P split into Ph (written over S) and Pl, lazy O
//              rescale, folding of O into the running total, then the
//              epilogue (O / l, stats).
//   warps 4-7  converters: each K / V tile lands raw (fp32) in shared memory
//              by TMA; they rewrite it in place as hi and add the lo copy.
//   warp 8     TMA producer (K, V tiles; 2- or 3-stage ring).  K lands in the
//              128B-swizzled K-major layout, V (read MN-major by the PV
//              MMAs) with 32-byte swizzle atoms, the layout MN-major tf32
//              operands need.
//   warp 9     MMA issuer + TMEM owner:
//                S_b  = Qh Kh^T + Qh Kl^T + Ql Kh^T      (TS MMA, N = kBN)
//                O   += Ph Vh + Ph Vl + Pl Vh            (TS MMA, N = DV)
//
// TMEM columns: Qh [0,DQK), Ql [DQK,2DQK), O [2DQK,2DQK+DV), the running
// total OT [2DQK+DV, 2DQK+2DV) (see FwdCfg), then two tile buffers of 2*kBN
// columns (S/Ph, Pl).
// Semantics follow sdpa/sdpa_fwd.cu.cc:60-173 exactly as the fp16 kernels do:
// l sums pre-dropout p, stats = max + ln(l + 1e-6), O = acc / l guarded by
// l > 1e-6, dropout by the counter-based LCG.
#pragma once
#include "common.cuh"
#include "fwd_tc.cuh"
#include "ptx.cuh"

namespace sdpa_b200 {
namespace tf32 {

constexpr int kBM = 128;

// Timing probe of tuning builds (-DSDPA_B200_TF32_FWD_PROBE): SM cycles of the
// roles of CTA 0, summed into slots of g_tf32_fwd_probe.
#ifdef SDPA_B200_TF32_FWD_PROBE
__device__ unsigned long long g_tf32_fwd_probe[16];
#define TF32F_T0(v) const long long v = clock64()
#define TF32F_ADD(slot, t0) \
  if (blockIdx.x == 0) atomicAdd(&g_tf32_fwd_probe[slot], static_cast<unsigned long long>(clock64() - (t0)))
#else
#define TF32F_T0(v)
#define TF32F_ADD(slot, t0)
#endif
constexpr int kFwdThreads = 320;

template <int DQK, int DV>
struct FwdCfg {
  // Key rows per tile, and how the output is accumulated.  The tensor cores'
  // fp32 accumulation is not round-to-nearest: summed over thousands of MMAs
  // (S_kv = 4096) its error reaches a few 1e-5 of |O|.  So where TMEM has
  // room, PV accumulates only kFlush tiles at a time (fresh accumulator at
  // every kFlush-th tile) and the softmax threads add each segment into a
  // running total OT (separate TMEM columns) in fp32 round-to-nearest.  With
  // D_qk and D_v both over 64 that leaves no room for Q lo: it moves to shared
  // memory (kQlSmem; the Q lo x K hi product becomes an SS MMA) and tiles are
  // 32 keys.
  static constexpr bool kFits64 = 2 * DQK + 2 * DV + 4 * 64 <= 512;
  static constexpr bool kFits32 = 2 * DQK + 2 * DV + 4 * 32 <= 512;
  static constexpr bool kQlSmem = !kFits32;
  static_assert(!kQlSmem || DQK + 2 * DV + 4 * 32 <= 512, "TMEM budget with Q lo in shared memory");
  static constexpr int kBN = kFits64 ? 64 : 32;
  static constexpr int kFlush = kFits64 ? 1 : 2;
  static constexpr uint32_t kKBytes = kBN * DQK * 4;  // one of hi / lo
  static constexpr uint32_t kVBytes = kBN * DV * 4;
  static constexpr uint32_t kStageBytes = 2 * (kKBytes + kVBytes);
  static constexpr uint32_t kQlBytes = kQlSmem ? kBM * DQK * 4 : 0;  // K-major, 128-byte swizzle
  static constexpr int kStages = 3 * kStageBytes + kQlBytes <= 200 * 1024 ? 3 : 2;
  static constexpr uint32_t kQlOff = kStages * kStageBytes;
  static constexpr uint32_t kBarOff = kQlOff + kQlBytes;
  static constexpr uint32_t kSmemBytes = kBarOff + 256 + 1024;
  static constexpr uint32_t kQh = 0, kQl = DQK;                       // kQl: TMEM (unless kQlSmem)
  static constexpr uint32_t kO = kQlSmem ? DQK : 2 * DQK;
  static constexpr uint32_t kOT = kO + DV;                            // running total
  static constexpr uint32_t kS = kOT + DV;                            // two buffers of 2 kBN columns
  static_assert(kS + 4 * kBN <= 512, "TMEM budget");
  static_assert(kSmemBytes <= 232448, "shared memory");
  // stage s: K hi, K lo, V hi, V lo
  static __device__ __forceinline__ uint32_t khi(int s) { return s * kStageBytes; }
  static __device__ __forceinline__ uint32_t klo(int s) { return s * kStageBytes + kKBytes; }
  static __device__ __forceinline__ uint32_t vhi(int s) { return s * kStageBytes + 2 * kKBytes; }
  static __device__ __forceinline__ uint32_t vlo(int s) { return s * kStageBytes + 2 * kKBytes + kVBytes; }
};

struct FwdBarriers {
  uint64_t q_ready;
  uint64_t k_full[3], v_full[3];
  uint64_t k_ready[3], v_ready[3];
  uint64_t kv_empty[3];
  uint64_t s_full[2];
  uint64_t p_full[2];
  uint64_t o_done;
  uint64_t o_final;  // every PV MMA done (one phase)
  uint64_t mma_done;
  uint32_t tmem_base;
  int abort_flag;
};

// Rewrites `bytes` of fp32 in shared memory at `hi` as tf32 hi parts and
// writes the lo parts to `lo` (same layout); `tid` of `nthr` threads.
__device__ __forceinline__ void split_tile(uint8_t* hi, uint8_t* lo, uint32_t bytes, int tid, int nthr) {
  float4* h4 = reinterpret_cast<float4*>(hi);
  float4* l4 = reinterpret_cast<float4*>(lo);
  const int n4 = static_cast<int>(bytes / 16);
#pragma unroll 4
  for (int i = tid; i < n4; i += nthr) {
    const float4 x = h4[i];
    float4 a, b;
    split_tf32(x.x, a.x, b.x);
    split_tf32(x.y, a.y, b.y);
    split_tf32(x.z, a.z, b.z);
    split_tf32(x.w, a.w, b.w);
    h4[i] = a;
    l4[i] = b;
  }
}

// Loads 32 consecutive fp32 columns [c0, c0+32) of a row (zeros at and beyond
// `ncols`, or everywhere when !valid), splits them and writes hi / lo to this
// thread's TMEM lane at columns th / tl.
__device__ __forceinline__ void row_to_tmem(const float* row, int c0, int ncols, bool valid, uint32_t th,
                                            uint32_t tl) {
  uint32_t h[32], l[32];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid && c0 + 4 * g < ncols) x = *reinterpret_cast<const float4*>(row + c0 + 4 * g);
    const float xv[4] = {x.x, x.y, x.z, x.w};
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a, b;
      split_tf32(xv[e], a, b);
      h[4 * g + e] = __float_as_uint(a);
      l[4 * g + e] = __float_as_uint(b);
    }
  }
  SDPA_TMEM_ST32(th, h);
  SDPA_TMEM_ST32(tl, l);
}

// row_to_tmem with the lo parts to a 128-byte shared-memory row (16-byte chunk
// g at chunk g ^ sw) instead of TMEM.
__device__ __forceinline__ void row_to_tmem_smem(const float* row, int c0, int ncols, bool valid, uint32_t th,
                                                 uint8_t* lo_row, int sw) {
  uint32_t h[32];
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    float4 x = make_float4(0.f, 0.f, 0.f, 0.f);
    if (valid && c0 + 4 * g < ncols) x = *reinterpret_cast<const float4*>(row + c0 + 4 * g);
    const float xv[4] = {x.x, x.y, x.z, x.w};
    float lv[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float a;
      split_tf32(xv[e], a, lv[e]);
      h[4 * g + e] = __float_as_uint(a);
    }
    *reinterpret_cast<float4*>(lo_row + ((g ^ sw) << 4)) = make_float4(lv[0], lv[1], lv[2], lv[3]);
  }
  SDPA_TMEM_ST32(th, h);
}

// Stores TMEM columns [0, 32*nchunks) of this lane (from taddr), times mul, to
// fp32 row `dst` at columns col0.. (columns < D).  With `total` nonzero, the
// TMEM columns at `total` are added first.
__device__ __forceinline__ void store_acc_row_f32(uint32_t taddr, int nchunks, int col0, float mul, bool have_acc,
                                                  bool active, float* dst, int D, uint32_t total = 0u) {
  for (int c = 0; c < nchunks; ++c) {
    uint32_t o[32];
    if (have_acc) {
      SDPA_TMEM_LD32(taddr + c * 32, o);
      if (total) {
        uint32_t ot[32];
        SDPA_TMEM_LD32(total + c * 32, ot);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) + __uint_as_float(ot[e]));
      }
      tmem_wait_ld();
    } else {
#pragma unroll
      for (int e = 0; e < 32; ++e) o[e] = 0u;
    }
    if (active) {
#pragma unroll
      for (int g = 0; g < 8; ++g) {
        const int col = col0 + c * 32 + 4 * g;
        if (col < D)
          *reinterpret_cast<float4*>(dst + col) =
              make_float4(__uint_as_float(o[4 * g]) * mul, __uint_as_float(o[4 * g + 1]) * mul,
                          __uint_as_float(o[4 * g + 2]) * mul, __uint_as_float(o[4 * g + 3]) * mul);
      }
    }
  }
}

template <int DQK, int DV, bool DROP, bool HEADS>
__global__ void __launch_bounds__(kFwdThreads, 1)
    fwd_kernel(const __grid_constant__ CUtensorMap tm_k, const __grid_constant__ CUtensorMap tm_v, const Params p) {
  using Cfg = FwdCfg<DQK, DV>;
  constexpr int kBN = Cfg::kBN;
  constexpr int NS = Cfg::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = tc::align1024(smem_raw);
  FwdBarriers* bars = reinterpret_cast<FwdBarriers*>(smem + Cfg::kBarOff);
  const int warp = threadIdx.x / 32;
  const int lane = threadIdx.x & 31;

  const int64_t n_qt = (p.S_q + kBM - 1) / kBM;
  int64_t b, tord;
  raster(blockIdx.x, p.B, n_qt, b, tord);
  const int hb = HEADS ? static_cast<int>(b % p.H) : 0, ob = HEADS ? static_cast<int>(b / p.H) : static_cast<int>(b);
  const int64_t qt = n_qt - 1 - tord;  // longest causal rows first
  const int64_t m0 = qt * kBM;
  const int64_t n_kv_all = (p.S_kv + kBN - 1) / kBN;
  const int n_kv = static_cast<int>(p.causal ? min(n_kv_all, (m0 + kBM - 1) / kBN + 1) : n_kv_all);

  if (threadIdx.x == 0) {
    mbar_init(&bars->q_ready, kBM);
    for (int s = 0; s < 3; ++s) {
      mbar_init(&bars->k_full[s], 1);
      mbar_init(&bars->v_full[s], 1);
      mbar_init(&bars->k_ready[s], 128);
      mbar_init(&bars->v_ready[s], 128);
      mbar_init(&bars->kv_empty[s], 1);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&bars->s_full[s], 1);
      mbar_init(&bars->p_full[s], kBM);
    }
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->o_final, 1);
    mbar_init(&bars->mma_done, 1);
    bars->abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 9) tmem_alloc(&bars->tmem_base, 512);
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
      tma_prefetch_desc(&tm_k);
      tma_prefetch_desc(&tm_v);
      int issued = 0;
      for (int j = 0; j < n_kv; ++j) {
        const int s = j % NS;
        if (!mbar_wait(&bars->kv_empty[s], ((j / NS) & 1) ^ 1, ctl)) break;
        mbar_expect_tx(&bars->k_full[s], Cfg::kKBytes);
#pragma unroll
        for (int c = 0; c < DQK / 32; ++c)
          tma_load_rows(smem + Cfg::khi(s) + c * kBN * 128, &tm_k, c * 32, j * kBN, hb, ob, &bars->k_full[s], HEADS);
        mbar_expect_tx(&bars->v_full[s], Cfg::kVBytes);
#pragma unroll
        for (int c = 0; c < DV / 32; ++c)
          tma_load_rows(smem + Cfg::vhi(s) + c * kBN * 128, &tm_v, c * 32, j * kBN, hb, ob, &bars->v_full[s], HEADS);
        issued = j + 1;
      }
      if (*ctl.abort_flag) {  // let copies in flight land before the CTA exits
        WaitCtl drain = ctl;
        drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
        int dummy = 0;
        drain.abort_flag = &dummy;
        for (int j = (issued > NS ? issued - NS : 0); j < issued; ++j) {
          mbar_wait(&bars->k_full[j % NS], (j / NS) & 1, drain);
          mbar_wait(&bars->v_full[j % NS], (j / NS) & 1, drain);
        }
      }
    }
  } else if (warp == 9) {
    // ------------------------------------------------------- MMA issuer
    if (lane == 0 && n_kv > 0) {
      constexpr uint32_t idesc_s = make_idesc(kBM, kBN, false, false, true);
      constexpr uint32_t idesc_pv = make_idesc(kBM, DV, false, true, true);
      const uint32_t sb = smem_u32(smem);
      auto issue_s = [&](int j) -> bool {
        const int s = j % NS;
        TF32F_T0(a0);
        if (!mbar_wait(&bars->k_ready[s], (j / NS) & 1, ctl)) return false;
        TF32F_ADD(0, a0);
        TF32F_T0(a1);
        tc_fence_after();
        const uint32_t tS = tmem + Cfg::kS + (j & 1) * 2 * kBN;
#pragma unroll
        for (int kk = 0; kk < DQK / 8; ++kk) {
          const uint32_t off = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          const uint64_t bh = make_sw128_desc(sb + Cfg::khi(s) + off, 16, 1024);
          const uint64_t bl = make_sw128_desc(sb + Cfg::klo(s) + off, 16, 1024);
          mma_tf32_ts(tS, tmem + Cfg::kQh + kk * 8, bh, idesc_s, kk > 0 ? 1u : 0u);
          mma_tf32_ts(tS, tmem + Cfg::kQh + kk * 8, bl, idesc_s, 1u);
          if constexpr (Cfg::kQlSmem)  // Q lo from shared memory: box kk / 4, 32-byte step kk % 4
            mma_tf32_ss(tS, make_sw128_desc(sb + Cfg::kQlOff + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024),
                        bh, idesc_s, 1u);
          else
            mma_tf32_ts(tS, tmem + Cfg::kQl + kk * 8, bh, idesc_s, 1u);
        }
        mma_commit(&bars->s_full[j & 1]);
        TF32F_ADD(1, a1);
        return true;
      };
      auto issue_pv = [&](int t) -> bool {
        const int s = t % NS;
        TF32F_T0(a2);
        if (!mbar_wait(&bars->p_full[t & 1], (t >> 1) & 1, ctl)) return false;
        TF32F_ADD(2, a2);
        TF32F_T0(a3);
        if (!mbar_wait(&bars->v_ready[s], (t / NS) & 1, ctl)) return false;
        tc_fence_after();
        const uint32_t tPh = tmem + Cfg::kS + (t & 1) * 2 * kBN, tPl = tPh + kBN;
        // a fresh accumulator at the first tile of each flush segment
        const bool fresh = Cfg::kFlush ? (t % (Cfg::kFlush * p.tf32_fold)) == 0 : t == 0;
#pragma unroll
        for (int kk = 0; kk < kBN / 8; ++kk) {
          const uint64_t vh = make_sw128_32b_desc(sb + Cfg::vhi(s) + kk * 1024, kBN * 128, 512);
          const uint64_t vl = make_sw128_32b_desc(sb + Cfg::vlo(s) + kk * 1024, kBN * 128, 512);
          mma_tf32_ts(tmem + Cfg::kO, tPh + kk * 8, vh, idesc_pv, (!fresh || kk > 0) ? 1u : 0u);
          mma_tf32_ts(tmem + Cfg::kO, tPh + kk * 8, vl, idesc_pv, 1u);
          mma_tf32_ts(tmem + Cfg::kO, tPl + kk * 8, vh, idesc_pv, 1u);
        }
        mma_commit(&bars->kv_empty[s]);
        TF32F_ADD(3, a3);
        mma_commit(&bars->o_done);
        return true;
      };
      bool ok = mbar_wait(&bars->q_ready, 0, ctl);
      for (int j = 0; ok && j < n_kv; ++j) {
        if (!issue_s(j)) {
          ok = false;
          break;
        }
        if (j > 0 && !issue_pv(j - 1)) {
          ok = false;
          break;
        }
      }
      if (ok) issue_pv(n_kv - 1);
      mma_commit(&bars->o_final);
      mma_commit(&bars->mma_done);
      WaitCtl drain = ctl;
      drain.deadline_ns = globaltimer_ns() + p.timeout_ns;
      int dummy = 0;
      drain.abort_flag = &dummy;
      mbar_wait(&bars->mma_done, 0, drain);
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------- converters
    const int tid = threadIdx.x - 128;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j % NS;
      TF32F_T0(c0);
      if (!tc::warp_wait(&bars->k_full[s], (j / NS) & 1, ctl)) break;
      if (tid == 0) TF32F_ADD(4, c0);
      TF32F_T0(c1);
      split_tile(smem + Cfg::khi(s), smem + Cfg::klo(s), Cfg::kKBytes, tid, 128);
      fence_proxy_async_smem();
      mbar_arrive(&bars->k_ready[s]);
      if (!tc::warp_wait(&bars->v_full[s], (j / NS) & 1, ctl)) break;
      split_tile(smem + Cfg::vhi(s), smem + Cfg::vlo(s), Cfg::kVBytes, tid, 128);
      fence_proxy_async_smem();
      if (tid == 0) TF32F_ADD(5, c1);
      mbar_arrive(&bars->v_ready[s]);
    }
  } else {
    // ------------------------------------------------ softmax warpgroup
    const int t = threadIdx.x;  // TMEM lane = query row in tile
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const int64_t row = m0 + t;
    const bool row_ok = row < p.S_q;
    {
      const float* qrow = static_cast<const float*>(p.q) + (row_ok ? row_offset_t<HEADS>(p.H, b, row, p.S_q, p.D_qk) : 0);
#pragma unroll
      for (int c = 0; c < DQK / 32; ++c) {
        if constexpr (Cfg::kQlSmem)  // lo: row t of box c, 16-byte chunk g at g ^ (t & 7)
          row_to_tmem_smem(qrow, c * 32, p.D_qk, row_ok, tmem + lane_base + Cfg::kQh + c * 32,
                           smem + Cfg::kQlOff + c * (kBM * 128) + t * 128, t & 7);
        else
          row_to_tmem(qrow, c * 32, p.D_qk, row_ok, tmem + lane_base + Cfg::kQh + c * 32,
                      tmem + lane_base + Cfg::kQl + c * 32);
      }
      if (Cfg::kQlSmem) fence_proxy_async_smem();
      if (Cfg::kFlush) {  // running output total starts at zero
        uint32_t z[32];
#pragma unroll
        for (int e = 0; e < 32; ++e) z[e] = 0u;
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) SDPA_TMEM_ST32(tmem + lane_base + Cfg::kOT + c * 32, z);
      }
      tmem_wait_st();
      tc_fence_before();
      mbar_arrive(&bars->q_ready);
    }
    const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + row) * static_cast<uint64_t>(p.S_kv);
    const bool fold = p.scale_log2 > 0.0f;
    const float sl = fold ? p.scale_log2 : 1.0f;
    const uint32_t thr_m1 = drop_thr_m1(p.drop_thr);
    const int64_t row_w0 = m0 + warp * 32;
    float m_run = -INFINITY, m_use = -INFINITY, l = 0.0f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int s = j & 1;  // TMEM tile buffer
      TF32F_T0(e0);
      if (!tc::warp_wait(&bars->s_full[s], (j >> 1) & 1, ctl)) {
        ok = false;
        break;
      }
      if (t == 0) TF32F_ADD(6, e0);
      TF32F_T0(e1);
      tc_fence_after();
      const uint32_t tS = tmem + lane_base + Cfg::kS + s * 2 * kBN;
      uint32_t r[kBN];
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) SDPA_TMEM_LD32(tS + c * 32, (r + c * 32));
      tmem_wait_ld();
      const int64_t kv0 = static_cast<int64_t>(j) * kBN;
      if (!fold) {
#pragma unroll
        for (int c = 0; c < kBN; ++c) r[c] = __float_as_uint(__uint_as_float(r[c]) * p.scale_log2);
      }
      if ((kv0 + kBN > p.S_kv) || (p.causal && kv0 + kBN - 1 > row_w0)) {
        int64_t lim64 = p.S_kv - kv0;
        if (p.causal) lim64 = min(lim64, row - kv0 + 1);
        const int lim = static_cast<int>(lim64 < 0 ? 0 : (lim64 > kBN ? kBN : lim64));
#pragma unroll
        for (int c = 0; c < kBN; ++c)
          if (c >= lim) r[c] = __float_as_uint(-INFINITY);
      }
      float mx[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
      for (int c = 0; c < kBN; c += 8)
#pragma unroll
        for (int q = 0; q < 4; ++q) mx[q] = fmax3(mx[q], __uint_as_float(r[c + 2 * q]), __uint_as_float(r[c + 2 * q + 1]));
      const float tmax = fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])) * sl;
      m_run = fmaxf(m_run, tmax);
      float alpha = 1.0f;
      bool rescale_o = false;
      if (tmax > m_use + tc::kRescaleThreshold) {
        alpha = ex2(m_use - m_run);
        rescale_o = (j > 0) && (m_use != -INFINITY);
        m_use = m_run;
        l *= alpha;
      }
      const float nmu = (m_use == -INFINITY) ? 0.0f : -m_use;
      float rs[4] = {0.0f, 0.0f, 0.0f, 0.0f};
      uint32_t lo[kBN];
      uint32_t s0_lo = 0, s0_hi = 0;
      if (DROP) {
        const uint64_t s0 = lcg_state(rbase, static_cast<uint64_t>(kv0));
        s0_lo = static_cast<uint32_t>(s0);
        s0_hi = static_cast<uint32_t>(s0 >> 32);
      }
#pragma unroll
      for (int c = 0; c < kBN; ++c) {
        float pv = ex2(fmaf(__uint_as_float(r[c]), sl, nmu));
        rs[c & 3] += pv;
        if (DROP && lcg_hi_at(s0_lo, s0_hi, p.one, static_cast<uint64_t>(c) * kLcgA) <= thr_m1) pv = 0.0f;
        float h, w;
        split_tf32(pv, h, w);
        r[c] = __float_as_uint(h);
        lo[c] = __float_as_uint(w);
      }
      l += (rs[0] + rs[1]) + (rs[2] + rs[3]);
#pragma unroll
      for (int c = 0; c < kBN / 32; ++c) {
        SDPA_TMEM_ST32(tS + c * 32, (r + c * 32));
        SDPA_TMEM_ST32(tS + kBN + c * 32, (lo + c * 32));
      }
      // PV(j-1) is in O: fold it into the running total at the end of a flush
      // segment, and whenever the reference max moved (then O and the total
      // are rescaled by alpha and O restarts from zero).  s_full(j) implies
      // PV(j-2) completed, so o_done is at most one phase behind here.
      const bool flush_now = Cfg::kFlush && j > 0 && (j % (Cfg::kFlush * p.tf32_fold)) == 0;
      if (flush_now || __any_sync(0xffffffffu, rescale_o)) {
        if (!tc::warp_wait(&bars->o_done, (j - 1) & 1, ctl)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float a = rescale_o ? alpha : 1.0f;
#pragma unroll
        for (int c = 0; c < DV / 32; ++c) {
          uint32_t o[32];
          SDPA_TMEM_LD32(tmem + lane_base + Cfg::kO + c * 32, o);
          if (Cfg::kFlush) {
            uint32_t ot[32];
            SDPA_TMEM_LD32(tmem + lane_base + Cfg::kOT + c * 32, ot);
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) ot[e] = __float_as_uint((__uint_as_float(ot[e]) + __uint_as_float(o[e])) * a);
            SDPA_TMEM_ST32(tmem + lane_base + Cfg::kOT + c * 32, ot);
            if (!flush_now) {  // PV(j) accumulates onto O: restart it
#pragma unroll
              for (int e = 0; e < 32; ++e) o[e] = 0u;
              SDPA_TMEM_ST32(tmem + lane_base + Cfg::kO + c * 32, o);
            }
          } else {
            tmem_wait_ld();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * a);
            SDPA_TMEM_ST32(tmem + lane_base + Cfg::kO + c * 32, o);
          }
        }
      }
      tmem_wait_st();
      tc_fence_before();
      if (t == 0) TF32F_ADD(7, e1);
      mbar_arrive(&bars->p_full[s]);
    }
    // ----------------------------------------------------------- epilogue
    // Not o_done with parity (n_kv - 1) & 1: PV(j-1) is issued after S(j), so
    // o_done may still be two phases behind here and that parity would match
    // an older phase.
    if (ok && n_kv > 0) ok = tc::warp_wait(&bars->o_final, 0, ctl);
    if (ok) {
      tc_fence_after();
      float lse, inv;
      if (m_run == -INFINITY) {
        lse = kNegInit + logf(kEps);
        inv = 0.0f;
      } else {
        const float l_true = l * ex2(m_use - m_run);
        lse = m_run * kLn2 + logf(l_true + kEps);
        inv = (l_true > kEps) ? p.dp_inv / l : 0.0f;
      }
      if (row_ok) p.stats[b * p.S_q + row] = lse;
      float* orow = static_cast<float*>(p.out) + (row_ok ? row_offset_t<HEADS>(p.H, b, row, p.S_q, p.D_v) : 0);
      store_acc_row_f32(tmem + lane_base + Cfg::kO, DV / 32, 0, inv, n_kv > 0, row_ok, orow, p.D_v,
                        Cfg::kFlush ? tmem + lane_base + Cfg::kOT : 0u);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 9) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

}  // namespace tf32
}  // namespace sdpa_b200
