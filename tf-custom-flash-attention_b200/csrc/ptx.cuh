// Thin inline-PTX wrappers for the sm_100a features the kernels use:
// mbarriers with bounded waits, TMA tile loads (no multicast), tcgen05 MMA /
// TMEM alloc / ld / st / commit / fences, and UMMA shared-memory and
// instruction descriptors.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>

namespace sdpa_b200 {

// ------------------------------------------------------------ status word
// Bit 0: a bounded wait gave up.  One word per device and translation unit
// (static: each .cu file's kernels raise their own; the C ABI reads them all).
static __device__ unsigned int g_status_word;
constexpr unsigned int kStatusTimeout = 1u;

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Shared state every role of a CTA sees: an abort flag raised by the first
// wait that gives up, so the other roles leave their loops promptly.
struct WaitCtl {
  uint64_t deadline_ns;
  volatile int* abort_flag;  // in shared memory
};

// Waits for phase `parity` of `bar`.  Gives up when the deadline passes or
// another role aborted; on giving up raises the device status word and the
// CTA abort flag and returns false.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtl& ctl) {
  if (mbar_try_wait(bar, parity)) return true;
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*ctl.abort_flag) return false;
      if (globaltimer_ns() > ctl.deadline_ns) {
        *ctl.abort_flag = 1;
        atomicOr(&g_status_word, kStatusTimeout);
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
// 3-D tiled load of one box into shared memory, completing on `bar`.
// x (innermost coordinate) must be a multiple of 16 bytes / element size.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* m, int x, int y, int z, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], [%5];" ::
          "r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

// 4-D tiled load (coordinates x, y, z, w innermost first); same rule for x.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* m, int x, int y, int z, int w,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(x), "r"(y), "r"(z), "r"(w), "r"(smem_u32(bar))
      : "memory");
}
// Rows [row, row + box) of folded batch row (head h, outer batch bo) of a map
// made by make_map_f16: with heads, 4-D coordinates (column x, head, row,
// outer batch); without (H = 1), the 3-D map (column x, row, batch).
__device__ __forceinline__ void tma_load_rows(void* dst, const CUtensorMap* m, int x, int row, int h, int bo,
                                              uint64_t* bar, bool heads) {
  if (heads)
    tma_load_4d(dst, m, x, h, row, bo, bar);
  else
    tma_load_3d(dst, m, x, row, bo, bar);
}

// ------------------------------------------- programmatic dependent launch
// With the launch attribute ProgrammaticStreamSerialization a kernel may start
// while the previous kernel on the stream is still finishing; it must wait
// here before touching global memory the previous kernel may read or write
// (a no-op without the attribute).  Each tensor-core kernel calls both right
// after its set-up (barrier init, TMEM alloc), so the set-up of the next
// kernel's CTAs overlaps this kernel's tail.
__device__ __forceinline__ void pdl_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// --------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]
__device__ __forceinline__ void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same products for fp32 data read as tf32 (K = 8 per instruction; the
// operands hold tf32 values, i.e. fp32 with the 13 low mantissa bits zero).
__device__ __forceinline__ void mma_tf32_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_tf32_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on `bar` when every tcgen05 op issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Warp-collective TMEM loads / stores, 32 lanes x 32-bit, N consecutive columns.
// Thread t of the warp gets lane (taddr.lane + t), columns taddr.col .. +N-1.
#define SDPA_TMEM_LD32(taddr, r)                                                                                     \
  asm volatile(                                                                                                    \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                   \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),  \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),     \
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),    \
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])                  \
      : "r"(taddr))

#define SDPA_TMEM_ST32(taddr, r)                                                                                      \
  asm volatile(                                                                                                     \
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18," \
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),                                      \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),   \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),     \
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),     \
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])                                                                 \
      : "memory")


#define SDPA_TMEM_ST16(taddr, r)                                                                                      \
  asm volatile(                                                                                                     \
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::      \
          "r"(taddr),                                                                                               \
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),   \
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])                                         \
      : "memory")

#define SDPA_TMEM_LD16(taddr, r)                                                                                    \
  asm volatile(                                                                                                    \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"      \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),  \
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])                   \
      : "r"(taddr))

__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------ descriptors
// Shared-memory matrix descriptor, 128-byte swizzle (sm_100 "version 1").
//   K-major operand: rows of 128 B (64 halves / 32 floats) in 8-row, 1024-B
//   swizzle atoms; sbo = 1024 (next 8 rows); lbo unused (1).
//   MN-major operand: 64 halves contiguous along M/N per row of K; sbo = 1024
//   (next 8 K-rows), lbo = byte distance to the next 64-wide M/N block.
// The buffer must be 1024-byte aligned (base offset 0); advancing the start
// address by 32 B inside a 128-B row steps K by 16 halves / 8 floats.
__device__ __forceinline__ uint64_t make_sw128_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm_100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// MN-major operand of 32-bit (tf32) elements: the only layout the tensor
// cores take for it is the 128-byte swizzle with 32-byte atoms (descriptor
// layout type 1): rows of 128 B (32 elements along M/N), the 32-byte chunk
// index XORed with (row & 3); sbo = byte distance between 4-row K groups,
// lbo = byte distance to the next 32-wide M/N block.  TMA writes it with
// CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B.
__device__ __forceinline__ uint64_t make_sw128_32b_desc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(1) << 61;  // SWIZZLE_128B_BASE32B
  return d;
}

// Instruction descriptor for kind::f16 (fp16 x fp16 -> fp32) or kind::tf32.
//   a_mn / b_mn: 1 when the operand is M/N-major in shared memory.
__host__ __device__ constexpr uint32_t make_idesc(int M, int N, bool a_mn, bool b_mn, bool tf32) {
  return (1u << 4)                                  // D format: f32
         | ((tf32 ? 2u : 0u) << 7)                  // A format: f16 (0) / tf32 (2)
         | ((tf32 ? 2u : 0u) << 10)                 // B format
         | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         (static_cast<uint32_t>(N >> 3) << 17)      // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24);   // M / 16
}

// ------------------------------------------------------------- 3xTF32
// x = hi + lo with hi, lo both tf32 values: hi = x rounded to tf32 (nearest,
// ties away), lo = the rounded remainder.  A product a*b is then taken as
// ah*bh + ah*bl + al*bh, whose error is about 2^-21 of |a*b| (al*bl and the
// rounding of the remainders are what is dropped), against 2^-11 for one
// tf32 product.
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
__device__ __forceinline__ void split_tf32(float x, float& hi, float& lo) {
  hi = tf32_rna(x);
  lo = tf32_rna(x - hi);
}
// Generic-proxy writes to shared memory become visible to the async proxy
// (TMA, tcgen05.mma operand reads) after this fence.
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// -------------------------------------------------------------- math bits
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);  // .x (low 16 bits) = lo
  return *reinterpret_cast<uint32_t*>(&h);
}

// Counter-based dropout (sdpa/sdpa_utils.cuh:13-19): the LCG state of element
// (row, column j) is (base + j) * A + C with base = seed + offset + row*S_kv.
// An element is dropped iff hi32(state) < thr, where the host derived thr from
// the rate so that hi32 < thr <=> float(hi32) / 2^32 < rate exactly.
constexpr uint64_t kLcgA = 6364136223846793005ULL;
constexpr uint64_t kLcgC = 1442695040888963407ULL;
__device__ __forceinline__ uint64_t lcg_state(uint64_t base, uint64_t j) { return (base + j) * kLcgA + kLcgC; }
__device__ __forceinline__ bool dropped(uint64_t state, uint64_t thr) { return (state >> 32) < thr; }

// The same walk on the two 32-bit halves of the state: one step adds A with a
// carry from the low word (2 instructions); the drop test reads the high word.
// Packed fp32 pairs (sm_100 f32x2 ALU forms): one instruction for two lanes
// of work.  Same rounding as the scalar forms (round-to-nearest).
__device__ __forceinline__ void ffma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0,
                                      float c1) {
  asm("{\n\t.reg .b64 a, b, c, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\tmov.b64 c, {%6, %7};\n\t"
      "fma.rn.f32x2 d, a, b, c;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void fadd2(float& d0, float& d1, float a0, float a1) {  // (d0, d1) += (a0, a1)
  asm("{\n\t.reg .b64 a, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 d, {%0, %1};\n\t"
      "add.rn.f32x2 d, d, a;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "+f"(d0), "+f"(d1)
      : "f"(a0), "f"(a1));
}
__device__ __forceinline__ void fmul2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n\t.reg .b64 a, b, d;\n\t"
      "mov.b64 a, {%2, %3};\n\tmov.b64 b, {%4, %5};\n\t"
      "mul.rn.f32x2 d, a, b;\n\tmov.b64 {%0, %1}, d;\n\t}"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
// Three-input maximum (exact).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

struct LcgWalk {
  uint32_t lo, hi;
  __device__ __forceinline__ explicit LcgWalk(uint64_t s)
      : lo(static_cast<uint32_t>(s)), hi(static_cast<uint32_t>(s >> 32)) {}
  __device__ __forceinline__ void step() {
    asm("add.cc.u32 %0, %0, %2;\n\taddc.u32 %1, %1, %3;"
        : "+r"(lo), "+r"(hi)
        : "n"(static_cast<uint32_t>(kLcgA & 0xffffffffu)), "n"(static_cast<uint32_t>(kLcgA >> 32)));
  }
  __device__ __forceinline__ void step(uint32_t inc_lo, uint32_t inc_hi) {
    asm("add.cc.u32 %0, %0, %2;\n\taddc.u32 %1, %1, %3;" : "+r"(lo), "+r"(hi) : "r"(inc_lo), "r"(inc_hi));
  }
  // dropped iff hi32(state) < thr, tested as hi <= thr - 1 (thr in [1, 2^32]),
  // so rate >= 1 (thr = 2^32) needs no separate case
  __device__ __forceinline__ bool dropped(uint32_t thr_m1) const { return hi <= thr_m1; }
};
__host__ __device__ inline uint32_t drop_thr_m1(uint64_t thr) { return static_cast<uint32_t>(thr - 1); }

// hi32 of the LCG state s + kc (mod 2^64), s = (s_hi, s_lo), kc a
// compile-time per-element constant (j * A), for the forward softmax, whose
// busiest pipe is the ALU pipe: one 32x32+64 multiply-add by `one` (a kernel
// parameter equal to 1, so the compiler keeps it) does the low add and its
// carry on the integer multiply-add unit, then one ALU add of s_hi, instead
// of a two-instruction 64-bit add chain on the ALU pipe.  (Measured: +3 % on
// the forward with dropout; the same in the backward passes, or the final add
// as a multiply-add too, measured slower.)
__device__ __forceinline__ uint32_t lcg_hi_at(uint32_t s_lo, uint32_t s_hi, uint32_t one, uint64_t kc) {
  uint64_t d;
  asm("mad.wide.u32 %0, %1, %2, %3;" : "=l"(d) : "r"(s_lo), "r"(one), "l"(kc));
  return static_cast<uint32_t>(d >> 32) + s_hi;
}

}  // namespace sdpa_b200
