/*
 * CPU restatement of the reference GPU algorithm for the Sdpa / SdpaGrad hot
 * path -- TEST INFRASTRUCTURE ONLY (parity checker, never the product path).
 * Loaded by tests/, __graft_entry__.smoke() and bench.py's cpu_baseline leg.
 *
 * Parity pin: checked against the reference itself (its unmodified sources
 * built by oracle/build_ref.sh, see tests/test_oracle.py) and against the
 * committed golden vectors in tests/golden/.
 *
 * It follows the reference's GPU kernels step by step (file:line are paths in
 * the reference project):
 *   RNG            sdpa/sdpa_utils.cuh:13-19   (== sdpa/sdpa_cpu.cc:198-211)
 *   forward        sdpa/sdpa_fwd.cu.cc:60-173  (online softmax with a max per
 *                  key tile of Bc columns, Bc from sdpa/sdpa_utils.cuh:58-93)
 *   backward dK/dV sdpa/sdpa_bwd.cu.cc:46-193
 *   backward dQ    sdpa/sdpa_bwd.cu.cc:227-344
 * including: half products rounded to half before the fp32 sum (Eigen::half
 * operator*), l summing pre-dropout p, stats = m + ln(l + 1e-6), O guarded by
 * l > 1e-6, dropout enabled iff rate > 1e-6, the backward skip rule p <= 1e-6,
 * and the dropped / kept dS formulas.
 *
 * Threads: rows are shared out over pthreads (set by oracle_set_threads).
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define ORACLE_F16 0
#define ORACLE_F32 1

static const float EPSF = 1e-6f;    /* sdpa/sdpa_utils.cuh:9 */
static const float NEGINF = -1e9f;  /* sdpa/sdpa_utils.cuh:11 */

static int g_threads = 1;
void oracle_set_threads(int n) { g_threads = n > 0 ? n : 1; }

/* ---------------------------------------------------------------- RNG */
/* state = seed + offset + (b*S_q + i)*S_kv + j (mod 2^64), one LCG step,
 * u = hi32(state) / 2^32 as float.  sdpa/sdpa_utils.cuh:13-19. */
float oracle_rng_uniform(uint64_t seed, uint64_t offset, uint64_t b, uint64_t i, uint64_t j, uint64_t S_q,
                         uint64_t S_kv) {
  uint64_t state = seed + offset + (b * S_q + i) * S_kv + j;
  state = state * 6364136223846793005ULL + 1442695040888963407ULL;
  uint32_t val = (uint32_t)(state >> 32);
  return (float)val / 4294967296.0f;
}

/* mask[b][i][j] = 1 where the element is dropped (u < rate); all zero when
 * rate <= 1e-6 (the GPU kernels' enable rule, sdpa/sdpa_fwd.cu.cc:136). */
void oracle_dropout_mask(uint64_t seed, uint64_t offset, int64_t B, int64_t S_q, int64_t S_kv, float rate,
                         uint8_t* mask) {
  for (int64_t b = 0; b < B; ++b)
    for (int64_t i = 0; i < S_q; ++i)
      for (int64_t j = 0; j < S_kv; ++j)
        mask[(b * S_q + i) * S_kv + j] =
            (rate > EPSF) && oracle_rng_uniform(seed, offset, b, i, j, S_q, S_kv) < rate;
}

/* ------------------------------------------------------- element access */
static inline float ld(const void* p, int64_t idx, int dtype) {
  if (dtype == ORACLE_F16) return (float)((const _Float16*)p)[idx];
  return ((const float*)p)[idx];
}
static inline void st(void* p, int64_t idx, float v, int dtype) {
  if (dtype == ORACLE_F16)
    ((_Float16*)p)[idx] = (_Float16)v;
  else
    ((float*)p)[idx] = v;
}
/* score += T(a*b): half products round to half first; fp32 uses a fused
 * multiply-add as the GPU compiler does for `score += q*k`. */
static inline float dot_acc(float acc, float a, float b, int dtype) {
  if (dtype == ORACLE_F16) return acc + (float)(_Float16)(a * b);
  return fmaf(a, b, acc);
}

/* Reference tile widths per head-dim bucket D_MAX in {8,16,32,64,128}
 * (sdpa/sdpa_utils.cuh:58-162).  Only the forward key tile Bc changes results
 * (the running max is taken per tile); the others only drive tile skipping. */
static int dmax_bucket(int64_t D) {
  if (D <= 8) return 8;
  if (D <= 16) return 16;
  if (D <= 32) return 32;
  if (D <= 64) return 64;
  return 128;
}
int oracle_fwd_tile_kv(int64_t D_qk, int64_t D_v) {
  int dm = dmax_bucket(D_qk > D_v ? D_qk : D_v);
  switch (dm) {
    case 8: return 256;
    case 16: return 256;
    case 32: return 128;
    case 64: return 32;
    default: return 16;
  }
}

/* ---------------------------------------------------------- thread pool */
typedef struct {
  void (*fn)(void* ctx, int64_t item);
  void* ctx;
  int64_t n;
  int64_t next;
  pthread_mutex_t mu;
} pool_t;

static void* pool_worker(void* arg) {
  pool_t* p = (pool_t*)arg;
  for (;;) {
    pthread_mutex_lock(&p->mu);
    int64_t it = p->next;
    p->next += 1;
    pthread_mutex_unlock(&p->mu);
    if (it >= p->n) break;
    p->fn(p->ctx, it);
  }
  return NULL;
}

static void run_items(void (*fn)(void*, int64_t), void* ctx, int64_t n) {
  pool_t p;
  p.fn = fn;
  p.ctx = ctx;
  p.n = n;
  p.next = 0;
  pthread_mutex_init(&p.mu, NULL);
  int nt = g_threads;
  if (nt > n) nt = (int)n;
  if (nt <= 1) {
    pool_worker(&p);
  } else {
    pthread_t* th = (pthread_t*)malloc(sizeof(pthread_t) * nt);
    for (int t = 0; t < nt; ++t) pthread_create(&th[t], NULL, pool_worker, &p);
    for (int t = 0; t < nt; ++t) pthread_join(th[t], NULL);
    free(th);
  }
  pthread_mutex_destroy(&p.mu);
}

/* --------------------------------------------------------------- common */
typedef struct {
  int dtype;
  const void *q, *k, *v, *o, *d_o;
  const float* stats_in;
  void *out, *dq, *dk, *dv;
  float* stats;
  int64_t B, S_q, S_kv, D_qk, D_v;
  float scale, dropout;
  int causal;
  uint64_t seed, offset;
  int tile_kv;
} job_t;

static inline float dp_inverse_of(float rate) { return rate > EPSF ? 1.0f / (1.0f - rate) : 1.0f; }

/* u64 counter of element (row q_idx = b*S_q + i, column j): base + j */
static inline float rng_at(uint64_t base, uint64_t j) {
  uint64_t state = base + j;
  state = state * 6364136223846793005ULL + 1442695040888963407ULL;
  return (float)(uint32_t)(state >> 32) / 4294967296.0f;
}

/* --------------------------------------------------------------- forward */
/* One query row (b, i): sdpa/sdpa_fwd.cu.cc:60-173. */
static void fwd_row(void* vctx, int64_t item) {
  const job_t* J = (const job_t*)vctx;
  const int64_t b = item / J->S_q, i = item % J->S_q;
  const int64_t S_kv = J->S_kv, D_qk = J->D_qk, D_v = J->D_v;
  const int Bc = J->tile_kv;
  const float dp_inv = dp_inverse_of(J->dropout);
  float* acc = (float*)calloc((size_t)(D_v > 0 ? D_v : 1), sizeof(float));
  float* sc = (float*)malloc(sizeof(float) * (size_t)Bc);
  float* qrow = (float*)malloc(sizeof(float) * (size_t)(D_qk > 0 ? D_qk : 1));
  for (int64_t d = 0; d < D_qk; ++d) qrow[d] = ld(J->q, (b * J->S_q + i) * D_qk + d, J->dtype);
  float m = NEGINF, l = 0.0f;
  const uint64_t base = J->seed + J->offset + (uint64_t)(b * J->S_q + i) * (uint64_t)S_kv;
  for (int64_t kv0 = 0; kv0 < S_kv; kv0 += Bc) {
    int64_t valid_end = (kv0 + Bc > S_kv) ? (S_kv - kv0) : Bc;
    if (J->causal && kv0 + valid_end > i) valid_end = i - kv0 + 1;
    if (valid_end <= 0) continue;
    float smax = NEGINF;
    for (int64_t jj = 0; jj < valid_end; ++jj) {
      const int64_t j = kv0 + jj;
      float s = 0.0f;
      for (int64_t d = 0; d < D_qk; ++d) s = dot_acc(s, qrow[d], ld(J->k, (b * S_kv + j) * D_qk + d, J->dtype), J->dtype);
      s *= J->scale;
      sc[jj] = s;
      if (s > smax) smax = s;
    }
    const float m_prev = m;
    m = smax > m ? smax : m;
    const float ratio = expf(m_prev - m);
    l *= ratio;
    for (int64_t d = 0; d < D_v; ++d) acc[d] *= ratio;
    for (int64_t jj = 0; jj < valid_end; ++jj) {
      const int64_t j = kv0 + jj;
      float p = expf(sc[jj] - m);
      l += p;
      if (J->dropout > EPSF) {
        if (rng_at(base, (uint64_t)j) < J->dropout)
          p = 0.0f;
        else
          p *= dp_inv;
      }
      for (int64_t d = 0; d < D_v; ++d) acc[d] = fmaf(p, ld(J->v, (b * S_kv + j) * D_v + d, J->dtype), acc[d]);
    }
  }
  J->stats[b * J->S_q + i] = m + logf(l + EPSF);
  const float inv_l = (l > EPSF) ? (1.0f / l) : 0.0f;
  for (int64_t d = 0; d < D_v; ++d) st(J->out, (b * J->S_q + i) * D_v + d, acc[d] * inv_l, J->dtype);
  free(acc);
  free(sc);
  free(qrow);
}

/* Forward: O [B,S_q,D_v] (dtype), stats [B,S_q] f32.  tile_kv <= 0 selects
 * the reference's Bc for this head dim. */
int oracle_sdpa_fwd(int dtype, const void* q, const void* k, const void* v, void* out, float* stats, int64_t B,
                    int64_t S_q, int64_t S_kv, int64_t D_qk, int64_t D_v, float scale, float dropout, int causal,
                    uint64_t seed, uint64_t offset, int tile_kv) {
  job_t J;
  memset(&J, 0, sizeof(J));
  J.dtype = dtype;
  J.q = q;
  J.k = k;
  J.v = v;
  J.out = out;
  J.stats = stats;
  J.B = B;
  J.S_q = S_q;
  J.S_kv = S_kv;
  J.D_qk = D_qk;
  J.D_v = D_v;
  J.scale = scale;
  J.dropout = dropout;
  J.causal = causal;
  J.seed = seed;
  J.offset = offset;
  J.tile_kv = tile_kv > 0 ? tile_kv : oracle_fwd_tile_kv(D_qk, D_v);
  run_items(fwd_row, &J, B * S_q);
  return 0;
}

/* -------------------------------------------------------------- backward */
/* D_i = sum_d T(dO*O) (sdpa/sdpa_bwd.cu.cc:87-104 and :248-257) */
static float row_delta(const job_t* J, int64_t q_idx) {
  float s = 0.0f;
  for (int64_t d = 0; d < J->D_v; ++d)
    s = dot_acc(s, ld(J->d_o, q_idx * J->D_v + d, J->dtype), ld(J->o, q_idx * J->D_v + d, J->dtype), J->dtype);
  return s;
}

/* dS and the dropped-out probability for element (q_idx, j); returns 0 when
 * the element is skipped (p <= 1e-6).  sdpa/sdpa_bwd.cu.cc:125-157. */
static int elem_grad(const job_t* J, int64_t b, int64_t i, int64_t j, float delta, float* p_out, float* ds_out) {
  const int64_t q_idx = b * J->S_q + i;
  float s = 0.0f;
  for (int64_t d = 0; d < J->D_qk; ++d)
    s = dot_acc(s, ld(J->q, q_idx * J->D_qk + d, J->dtype), ld(J->k, (b * J->S_kv + j) * J->D_qk + d, J->dtype),
                J->dtype);
  float p = expf(s * J->scale - J->stats_in[q_idx]);
  if (!(p > EPSF)) return 0;
  const float dp_inv = dp_inverse_of(J->dropout);
  float dS = J->scale;
  int dropped = 0;
  if (J->dropout > EPSF) {
    const uint64_t base = J->seed + J->offset + (uint64_t)q_idx * (uint64_t)J->S_kv;
    if (rng_at(base, (uint64_t)j) < J->dropout) {
      dropped = 1;
      dS *= -p * delta;
      p = 0.0f;
    } else {
      p *= dp_inv;
    }
  }
  if (!dropped) {
    float dP = 0.0f;
    for (int64_t d = 0; d < J->D_v; ++d)
      dP = dot_acc(dP, ld(J->d_o, q_idx * J->D_v + d, J->dtype), ld(J->v, (b * J->S_kv + j) * J->D_v + d, J->dtype),
                   J->dtype);
    dS *= p * (dP - delta / dp_inv);
  }
  *p_out = p;
  *ds_out = dS;
  return 1;
}

/* One key row (b, j): dK, dV (sdpa/sdpa_bwd.cu.cc:46-193). */
static void bwd_kv_row(void* vctx, int64_t item) {
  const job_t* J = (const job_t*)vctx;
  const int64_t b = item / J->S_kv, j = item % J->S_kv;
  float* dk = (float*)calloc((size_t)(J->D_qk > 0 ? J->D_qk : 1), sizeof(float));
  float* dv = (float*)calloc((size_t)(J->D_v > 0 ? J->D_v : 1), sizeof(float));
  for (int64_t i = 0; i < J->S_q; ++i) {
    if (J->causal && i < j) continue;
    const int64_t q_idx = b * J->S_q + i;
    const float delta = row_delta(J, q_idx);
    float p, dS;
    if (!elem_grad(J, b, i, j, delta, &p, &dS)) continue;
    for (int64_t d = 0; d < J->D_v; ++d) dv[d] = fmaf(p, ld(J->d_o, q_idx * J->D_v + d, J->dtype), dv[d]);
    for (int64_t d = 0; d < J->D_qk; ++d) dk[d] = fmaf(dS, ld(J->q, q_idx * J->D_qk + d, J->dtype), dk[d]);
  }
  for (int64_t d = 0; d < J->D_qk; ++d) st(J->dk, (b * J->S_kv + j) * J->D_qk + d, dk[d], J->dtype);
  for (int64_t d = 0; d < J->D_v; ++d) st(J->dv, (b * J->S_kv + j) * J->D_v + d, dv[d], J->dtype);
  free(dk);
  free(dv);
}

/* One query row (b, i): dQ (sdpa/sdpa_bwd.cu.cc:227-344). */
static void bwd_q_row(void* vctx, int64_t item) {
  const job_t* J = (const job_t*)vctx;
  const int64_t b = item / J->S_q, i = item % J->S_q;
  const int64_t q_idx = b * J->S_q + i;
  float* dq = (float*)calloc((size_t)(J->D_qk > 0 ? J->D_qk : 1), sizeof(float));
  const float delta = row_delta(J, q_idx);
  for (int64_t j = 0; j < J->S_kv; ++j) {
    if (J->causal && i < j) continue;
    float p, dS;
    if (!elem_grad(J, b, i, j, delta, &p, &dS)) continue;
    for (int64_t d = 0; d < J->D_qk; ++d) dq[d] = fmaf(dS, ld(J->k, (b * J->S_kv + j) * J->D_qk + d, J->dtype), dq[d]);
  }
  for (int64_t d = 0; d < J->D_qk; ++d) st(J->dq, q_idx * J->D_qk + d, dq[d], J->dtype);
  free(dq);
}

/* Backward: dq, dk, dv shaped like q, k, v. */
int oracle_sdpa_bwd(int dtype, const void* q, const void* k, const void* v, const void* o, const float* stats,
                    const void* d_o, void* dq, void* dk, void* dv, int64_t B, int64_t S_q, int64_t S_kv, int64_t D_qk,
                    int64_t D_v, float scale, float dropout, int causal, uint64_t seed, uint64_t offset) {
  job_t J;
  memset(&J, 0, sizeof(J));
  J.dtype = dtype;
  J.q = q;
  J.k = k;
  J.v = v;
  J.o = o;
  J.stats_in = stats;
  J.d_o = d_o;
  J.dq = dq;
  J.dk = dk;
  J.dv = dv;
  J.B = B;
  J.S_q = S_q;
  J.S_kv = S_kv;
  J.D_qk = D_qk;
  J.D_v = D_v;
  J.scale = scale;
  J.dropout = dropout;
  J.causal = causal;
  J.seed = seed;
  J.offset = offset;
  run_items(bwd_kv_row, &J, B * S_kv);
  run_items(bwd_q_row, &J, B * S_q);
  return 0;
}
