// SIMT kernels: the general path for shapes the tensor-core kernels do not
// take (head-dim rows that are not a multiple of 16 bytes, hence not
// TMA-addressable) and for fp32 until its tensor-core path serves it.
// Same semantics as the tensor-core kernels (see api.cu); FP32 arithmetic.
//   fwd      one thread per query row, K/V tiles staged in shared memory
//   delta    one warp per query row: D_i = sum_d dO*O
//   dkdv     one thread per key row, Q/dO tiles staged, K/V transposed in smem
//   dq       one thread per query row, K/V tiles staged, Q/dO transposed in smem
#pragma once
#include "common.cuh"
#include "ptx.cuh"

namespace sdpa_b200 {
namespace simt {

constexpr int kFwdRows = 128;  // query rows per CTA
constexpr int kFwdKeys = 32;   // keys per staged tile
constexpr int kBwdRows = 64;   // rows owned per CTA in dkdv / dq
constexpr int kBwdTile = 32;   // rows per staged tile of the other side

// dst[r][d] (row-major, width DM) <- src rows row0.. (row stride ld; zero
// outside).  Rows whose start and length are 16-byte multiples (and a 16-byte
// aligned base) move in 16-byte vectors, one per thread per step, coalesced
// along the row; others element by element.
template <typename T>
__device__ __forceinline__ void stage_rows(float* dst, const T* src, int64_t ld, int64_t row0, int64_t nrows_total,
                                           int rows, int D, int DM, int tid, int nthreads) {
  constexpr int V = 16 / static_cast<int>(sizeof(T));  // elements per 16-byte vector
  const bool vec = (D % V == 0) && (ld % V == 0) && (DM % V == 0) &&
                   ((reinterpret_cast<uintptr_t>(src) & 15u) == 0);
  if (vec) {
    const int per_row = DM / V;
    for (int idx = tid; idx < rows * per_row; idx += nthreads) {
      const int r = idx / per_row, d = (idx - r * per_row) * V;
      const int64_t gr = row0 + r;
      float f[V];
      if (gr < nrows_total && d < D) {
        const uint4 u = *reinterpret_cast<const uint4*>(src + gr * ld + d);
        const T* e = reinterpret_cast<const T*>(&u);
#pragma unroll
        for (int i = 0; i < V; ++i) f[i] = to_f<T>(e[i]);
      } else {
#pragma unroll
        for (int i = 0; i < V; ++i) f[i] = 0.0f;
      }
#pragma unroll
      for (int i = 0; i < V; i += 4)
        *reinterpret_cast<float4*>(dst + r * DM + d + i) = make_float4(f[i], f[i + 1], f[i + 2], f[i + 3]);
    }
    return;
  }
  for (int idx = tid; idx < rows * DM; idx += nthreads) {
    int r = idx / DM, d = idx - r * DM;
    int64_t gr = row0 + r;
    dst[idx] = (gr < nrows_total && d < D) ? to_f<T>(src[gr * ld + d]) : 0.0f;
  }
}

// acc + a*b as the reference's `score += T(a*b)`: for half the product is
// rounded to half before the fp32 sum (Eigen::half arithmetic,
// sdpa/sdpa_fwd.cu.cc:108, sdpa/sdpa_bwd.cu.cc:98, 128, 154); for float a fused
// multiply-add.  On these kernels' small head dims (rows that are not 16-byte
// multiples) the rounding is a visible part of the reference's result.
template <typename T>
__device__ __forceinline__ float dot_step(float acc, float a, float b);
template <>
__device__ __forceinline__ float dot_step<float>(float acc, float a, float b) {
  return fmaf(a, b, acc);
}
template <>
__device__ __forceinline__ float dot_step<__half>(float acc, float a, float b) {
  return acc + __half2float(__float2half_rn(a * b));
}

template <typename T, int DM>
__global__ void __launch_bounds__(kFwdRows) fwd_kernel(Params p) {
  __shared__ __align__(16) float Ks[kFwdKeys * DM];
  __shared__ __align__(16) float Vs[kFwdKeys * DM];
  const int64_t n_qt = (p.S_q + kFwdRows - 1) / kFwdRows;
  const int64_t b = blockIdx.x % p.B;
  const int64_t qt = n_qt - 1 - blockIdx.x / p.B;  // heavy causal tiles first
  const int tid = threadIdx.x;
  const int64_t row = qt * kFwdRows + tid;
  const bool active = row < p.S_q;
  // rows of folded batch row b; row strides H*D ([B/H, S, H, D] layout)
  const T* Q = static_cast<const T*>(p.q) + row_offset(p.H, b, 0, p.S_q, p.D_qk);
  const T* K = static_cast<const T*>(p.k) + row_offset(p.H, b, 0, p.S_kv, p.D_qk);
  const T* V = static_cast<const T*>(p.v) + row_offset(p.H, b, 0, p.S_kv, p.D_v);
  const int64_t ldqk = p.H * p.D_qk, ldv = p.H * p.D_v;

  float qr[DM], acc[DM];
#pragma unroll
  for (int d = 0; d < DM; ++d) {
    // float: scale folded into q; half: products of the raw values, scaled after the sum
    qr[d] = (active && d < p.D_qk) ? to_f<T>(Q[row * ldqk + d]) * (sizeof(T) == 2 ? 1.0f : p.scale_log2) : 0.0f;
    acc[d] = 0.0f;
  }
  float m = -INFINITY, l = 0.0f;
  const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + row) * static_cast<uint64_t>(p.S_kv);
  int64_t kv_end = p.S_kv;
  if (p.causal) kv_end = min(p.S_kv, (qt + 1) * kFwdRows);
  for (int64_t kv0 = 0; kv0 < kv_end; kv0 += kFwdKeys) {
    __syncthreads();
    stage_rows<T>(Ks, K, ldqk, kv0, p.S_kv, kFwdKeys, p.D_qk, DM, tid, kFwdRows);
    stage_rows<T>(Vs, V, ldv, kv0, p.S_kv, kFwdKeys, p.D_v, DM, tid, kFwdRows);
    __syncthreads();
    if (!active) continue;
    float sc[kFwdKeys];
    float tmax = -INFINITY;
#pragma unroll
    for (int jj = 0; jj < kFwdKeys; ++jj) {
      const int64_t j = kv0 + jj;
      const bool valid = j < p.S_kv && (!p.causal || j <= row);
      float s = 0.0f;
#pragma unroll
      for (int d = 0; d < DM; ++d) s = dot_step<T>(s, qr[d], Ks[jj * DM + d]);
      if (sizeof(T) == 2) s *= p.scale_log2;
      sc[jj] = valid ? s : -INFINITY;
      tmax = fmaxf(tmax, sc[jj]);
    }
    if (tmax == -INFINITY) continue;
    const float m_new = fmaxf(m, tmax);
    const float alpha = ex2(m - m_new);
    m = m_new;
    l *= alpha;
#pragma unroll
    for (int d = 0; d < DM; ++d) acc[d] *= alpha;
#pragma unroll
    for (int jj = 0; jj < kFwdKeys; ++jj) {
      float pr = ex2(sc[jj] - m);
      l += pr;
      if (p.dropout_on && dropped(lcg_state(rbase, static_cast<uint64_t>(kv0 + jj)), p.drop_thr)) pr = 0.0f;
#pragma unroll
      for (int d = 0; d < DM; ++d) acc[d] = fmaf(pr, Vs[jj * DM + d], acc[d]);
    }
  }
  if (!active) return;
  const int64_t orow = b * p.S_q + row;
  const float lse = (m == -INFINITY) ? kNegInit + logf(kEps) : m * kLn2 + logf(l + kEps);
  p.stats[orow] = lse;
  const float inv = (l > kEps) ? p.dp_inv / l : 0.0f;
  T* O = static_cast<T*>(p.out) + row_offset(p.H, b, row, p.S_q, p.D_v);
#pragma unroll
  for (int d = 0; d < DM; ++d)
    if (d < p.D_v) O[d] = from_f<T>(acc[d] * inv);
}

// D_i = sum_d dO[i,d] * O[i,d] (fp32), one warp per row (minus the stats gradient, if any).
template <typename T>
__global__ void __launch_bounds__(256) delta_kernel(Params p) {
  const int64_t row = static_cast<int64_t>(blockIdx.x) * 8 + threadIdx.x / 32;
  const int lane = threadIdx.x & 31;
  if (row >= p.B * p.S_q) return;
  const int64_t off = p.H == 1 ? row * p.D_v : row_offset(p.H, row / p.S_q, row % p.S_q, p.S_q, p.D_v);
  const T* dO = static_cast<const T*>(p.d_o) + off;
  const T* O = static_cast<const T*>(p.o) + off;
  float s = 0.0f;
  for (int d = lane; d < p.D_v; d += 32) s = dot_step<T>(s, to_f<T>(dO[d]), to_f<T>(O[d]));
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
  // A gradient g_i reaching stats_i = logsumexp adds g_i * p_ij to dS_ij,
  // i.e. it enters dS = p (dP - D) as D - g.
  if (lane == 0) p.delta[row] = p.d_stats ? s - p.d_stats[row] : s;
}

// Gradient of one score element.  Returns false when skipped (p <= 1e-6,
// sdpa/sdpa_bwd.cu.cc:131); otherwise the dropped-out probability and dS
// (sdpa/sdpa_bwd.cu.cc:133-157).
__device__ __forceinline__ bool elem_grad(const Params& p, float s_log2, float lse2, float delta, uint64_t state,
                                          float dPdot, float& prob, float& dS) {
  float pr = ex2(s_log2 - lse2);
  if (!(pr > kEps)) return false;
  if (p.dropout_on) {
    if (dropped(state, p.drop_thr)) {
      dS = p.scale * (-pr * delta);
      prob = 0.0f;
      return true;
    }
    pr *= p.dp_inv;
  }
  dS = p.scale * (pr * (dPdot - delta / p.dp_inv));
  prob = pr;
  return true;
}

// Threads per key row in dkdv_kernel: wide head dims split the dK / dV
// accumulators over two threads (partial dot products joined by a shuffle)
// so they stay in registers.
template <int DM>
__host__ __device__ constexpr int dkdv_split() {
  return DM >= 64 ? 2 : 1;
}

template <typename T, int DM>
__global__ void __launch_bounds__(kBwdRows * dkdv_split<DM>()) dkdv_kernel(Params p) {
  constexpr int SPLIT = dkdv_split<DM>();
  constexpr int DH = DM / SPLIT;              // head-dim slice owned by this thread
  constexpr int NT = kBwdRows * SPLIT;
  extern __shared__ float sm[];
  float* Kt = sm;                         // [DM][kBwdRows]
  float* Vt = Kt + DM * kBwdRows;         // [DM][kBwdRows]
  float* Qs = Vt + DM * kBwdRows;         // [kBwdTile][DM]
  float* dOs = Qs + kBwdTile * DM;        // [kBwdTile][DM]
  float* lse_s = dOs + kBwdTile * DM;     // [kBwdTile] (log2 units)
  float* del_s = lse_s + kBwdTile;        // [kBwdTile]
  const int64_t b = blockIdx.x % p.B;
  const int64_t kt = blockIdx.x / p.B;
  const int tid = threadIdx.x;
  const int r = tid / SPLIT, h = tid % SPLIT, d0 = h * DH;
  const int64_t kv = kt * kBwdRows + r;
  const bool active = kv < p.S_kv;
  // rows of folded batch row b; row strides H*D ([B/H, S, H, D] layout)
  const T* Q = static_cast<const T*>(p.q) + row_offset(p.H, b, 0, p.S_q, p.D_qk);
  const T* K = static_cast<const T*>(p.k) + row_offset(p.H, b, 0, p.S_kv, p.D_qk);
  const T* V = static_cast<const T*>(p.v) + row_offset(p.H, b, 0, p.S_kv, p.D_v);
  const int64_t ldqk = p.H * p.D_qk, ldv = p.H * p.D_v;
  const T* dO = static_cast<const T*>(p.d_o) + row_offset(p.H, b, 0, p.S_q, p.D_v);
  for (int idx = tid; idx < DM * kBwdRows; idx += NT) {
    const int d = idx / kBwdRows, rr = idx - d * kBwdRows;
    const int64_t kvr = kt * kBwdRows + rr;
    Kt[idx] = (kvr < p.S_kv && d < p.D_qk) ? to_f<T>(K[kvr * ldqk + d]) : 0.0f;
    Vt[idx] = (kvr < p.S_kv && d < p.D_v) ? to_f<T>(V[kvr * ldv + d]) : 0.0f;
  }
  float dk[DH], dv[DH];
#pragma unroll
  for (int d = 0; d < DH; ++d) dk[d] = dv[d] = 0.0f;
  const int64_t q_start = p.causal ? (kt * kBwdRows / kBwdTile) * kBwdTile : 0;
  for (int64_t q0 = q_start; q0 < p.S_q; q0 += kBwdTile) {
    __syncthreads();
    stage_rows<T>(Qs, Q, ldqk, q0, p.S_q, kBwdTile, p.D_qk, DM, tid, NT);
    stage_rows<T>(dOs, dO, ldv, q0, p.S_q, kBwdTile, p.D_v, DM, tid, NT);
    for (int rr = tid; rr < kBwdTile; rr += NT) {
      const int64_t i = q0 + rr;
      lse_s[rr] = i < p.S_q ? p.lse[b * p.S_q + i] * kLog2e : 0.0f;
      del_s[rr] = i < p.S_q ? p.delta[b * p.S_q + i] : 0.0f;
    }
    __syncthreads();
    if (!active) continue;  // both threads of a row take the same path
    for (int rr = 0; rr < kBwdTile; ++rr) {
      const int64_t i = q0 + rr;
      if (i >= p.S_q) break;
      if (p.causal && i < kv) continue;
      float s = 0.0f, dP = 0.0f;
#pragma unroll
      for (int d = 0; d < DH; ++d) s = dot_step<T>(s, Qs[rr * DM + d0 + d], Kt[(d0 + d) * kBwdRows + r]);
#pragma unroll
      for (int d = 0; d < DH; ++d) dP = dot_step<T>(dP, dOs[rr * DM + d0 + d], Vt[(d0 + d) * kBwdRows + r]);
      if (SPLIT == 2) {
        // Only the two threads of this key row are guaranteed to be here (rows
        // of a warp skip different query rows), so the shuffle names just them.
        const unsigned pair = 0x3u << (threadIdx.x & 30);
        s += __shfl_xor_sync(pair, s, 1);
        dP += __shfl_xor_sync(pair, dP, 1);
      }
      const uint64_t st =
          lcg_state(p.rng_base + static_cast<uint64_t>(b * p.S_q + i) * static_cast<uint64_t>(p.S_kv),
                    static_cast<uint64_t>(kv));
      float pr, dS;
      if (!elem_grad(p, s * p.scale_log2, lse_s[rr], del_s[rr], st, dP, pr, dS)) continue;
#pragma unroll
      for (int d = 0; d < DH; ++d) {
        dv[d] = fmaf(pr, dOs[rr * DM + d0 + d], dv[d]);
        dk[d] = fmaf(dS, Qs[rr * DM + d0 + d], dk[d]);
      }
    }
  }
  if (!active) return;
  T* dK = static_cast<T*>(p.dk) + row_offset(p.H, b, kv, p.S_kv, p.D_qk);
  T* dV = static_cast<T*>(p.dv) + row_offset(p.H, b, kv, p.S_kv, p.D_v);
#pragma unroll
  for (int d = 0; d < DH; ++d) {
    if (d0 + d < p.D_qk) dK[d0 + d] = from_f<T>(dk[d]);
    if (d0 + d < p.D_v) dV[d0 + d] = from_f<T>(dv[d]);
  }
}

template <typename T, int DM>
__global__ void __launch_bounds__(kBwdRows) dq_kernel(Params p) {
  extern __shared__ float sm[];
  float* Qt = sm;                     // [DM][kBwdRows]
  float* dOt = Qt + DM * kBwdRows;    // [DM][kBwdRows]
  float* Ks = dOt + DM * kBwdRows;    // [kBwdTile][DM]
  float* Vs = Ks + kBwdTile * DM;     // [kBwdTile][DM]
  const int64_t n_qt = (p.S_q + kBwdRows - 1) / kBwdRows;
  const int64_t b = blockIdx.x % p.B;
  const int64_t qt = n_qt - 1 - blockIdx.x / p.B;
  const int tid = threadIdx.x;
  const int64_t row = qt * kBwdRows + tid;
  const bool active = row < p.S_q;
  // rows of folded batch row b; row strides H*D ([B/H, S, H, D] layout)
  const T* Q = static_cast<const T*>(p.q) + row_offset(p.H, b, 0, p.S_q, p.D_qk);
  const T* K = static_cast<const T*>(p.k) + row_offset(p.H, b, 0, p.S_kv, p.D_qk);
  const T* V = static_cast<const T*>(p.v) + row_offset(p.H, b, 0, p.S_kv, p.D_v);
  const int64_t ldqk = p.H * p.D_qk, ldv = p.H * p.D_v;
  const T* dO = static_cast<const T*>(p.d_o) + row_offset(p.H, b, 0, p.S_q, p.D_v);
  for (int d = 0; d < DM; ++d) {
    Qt[d * kBwdRows + tid] = (active && d < p.D_qk) ? to_f<T>(Q[row * ldqk + d]) : 0.0f;
    dOt[d * kBwdRows + tid] = (active && d < p.D_v) ? to_f<T>(dO[row * ldv + d]) : 0.0f;
  }
  const float lse2 = active ? p.lse[b * p.S_q + row] * kLog2e : 0.0f;
  const float delta = active ? p.delta[b * p.S_q + row] : 0.0f;
  const uint64_t rbase = p.rng_base + static_cast<uint64_t>(b * p.S_q + row) * static_cast<uint64_t>(p.S_kv);
  float dq[DM];
#pragma unroll
  for (int d = 0; d < DM; ++d) dq[d] = 0.0f;
  int64_t kv_end = p.S_kv;
  if (p.causal) kv_end = min(p.S_kv, (qt + 1) * kBwdRows);
  for (int64_t kv0 = 0; kv0 < kv_end; kv0 += kBwdTile) {
    __syncthreads();
    stage_rows<T>(Ks, K, ldqk, kv0, p.S_kv, kBwdTile, p.D_qk, DM, tid, kBwdRows);
    stage_rows<T>(Vs, V, ldv, kv0, p.S_kv, kBwdTile, p.D_v, DM, tid, kBwdRows);
    __syncthreads();
    if (!active) continue;
    for (int jj = 0; jj < kBwdTile; ++jj) {
      const int64_t j = kv0 + jj;
      if (j >= p.S_kv) break;
      if (p.causal && j > row) break;
      float s = 0.0f, dP = 0.0f;
#pragma unroll
      for (int d = 0; d < DM; ++d) s = dot_step<T>(s, Qt[d * kBwdRows + tid], Ks[jj * DM + d]);
#pragma unroll
      for (int d = 0; d < DM; ++d) dP = dot_step<T>(dP, dOt[d * kBwdRows + tid], Vs[jj * DM + d]);
      float pr, dS;
      if (!elem_grad(p, s * p.scale_log2, lse2, delta, lcg_state(rbase, static_cast<uint64_t>(j)), dP, pr, dS))
        continue;
#pragma unroll
      for (int d = 0; d < DM; ++d) dq[d] = fmaf(dS, Ks[jj * DM + d], dq[d]);
    }
  }
  if (!active) return;
  T* dQ = static_cast<T*>(p.dq) + row_offset(p.H, b, row, p.S_q, p.D_qk);
#pragma unroll
  for (int d = 0; d < DM; ++d)
    if (d < p.D_qk) dQ[d] = from_f<T>(dq[d]);
}

template <int DM>
constexpr size_t dkdv_smem() {
  return sizeof(float) * (2 * DM * kBwdRows + 2 * kBwdTile * DM + 2 * kBwdTile);
}
template <int DM>
constexpr size_t dq_smem() {
  return sizeof(float) * (2 * DM * kBwdRows + 2 * kBwdTile * DM);
}

}  // namespace simt
}  // namespace sdpa_b200
