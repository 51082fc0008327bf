// Shared device helpers for every sm_100a kernel in this extension.
//
// Thin inline-PTX wrappers around the Blackwell primitives the kernels use:
// mbarriers, TMA tiled loads, tcgen05 (TMEM alloc / MMA / commit / ld), and
// the system-scope acquire/release accesses + %globaltimer used by the
// cross-GPU signalling in the collective kernels.  Every wait helper here is
// bounded: after its budget it records an error code and returns false, so a
// missing peer or a broken pipeline never hangs the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#define MNB_DEVICE __device__ __forceinline__

namespace mnb {

// Error codes written to a kernel's status word.
enum : int {
  kOk = 0,
  kErrPeerTimeout = 1,     // a peer's signal did not arrive before the deadline
  kErrPipelineTimeout = 2, // an intra-CTA mbarrier wait exceeded its budget
  kErrBadArgument = 3,
};

// ---------------------------------------------------------------------------
// scalar conversions
// ---------------------------------------------------------------------------
MNB_DEVICE float bf16_to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
MNB_DEVICE __nv_bfloat16 f32_to_bf16(float x) { return __float2bfloat16_rn(x); }

MNB_DEVICE uint32_t pack_bf16x2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}
MNB_DEVICE float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// ---------------------------------------------------------------------------
// time and system-scope memory ordering (cross-GPU flags)
// ---------------------------------------------------------------------------
MNB_DEVICE uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

MNB_DEVICE uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
MNB_DEVICE void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
MNB_DEVICE uint32_t ld_relaxed_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.relaxed.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// 16-byte vector access through the generic address space (peer pointers).
MNB_DEVICE uint4 ld_v4(const void* p) { return *reinterpret_cast<const uint4*>(p); }
MNB_DEVICE void st_v4(void* p, uint4 v) { *reinterpret_cast<uint4*>(p) = v; }
// Non-coherent-with-L1 (volatile) 16-byte load for data another GPU wrote.
MNB_DEVICE uint4 ld_v4_volatile(const void* p) {
  uint4 v;
  asm volatile("ld.volatile.global.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// ---------------------------------------------------------------------------
// shared memory addressing
// ---------------------------------------------------------------------------
MNB_DEVICE uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
MNB_DEVICE void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
MNB_DEVICE void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
MNB_DEVICE void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
MNB_DEVICE void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}
MNB_DEVICE bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait on an mbarrier phase.  `abort` is a per-launch status word in
// global memory: once any thread of the launch has given up, everyone else
// stops waiting too.  Returns false on timeout/abort.
constexpr uint32_t kMbarSpinBudget = 1u << 27;
MNB_DEVICE bool mbar_wait(uint32_t bar, uint32_t parity, int* abort) {
  for (uint32_t i = 0;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 1023u) == 1023u) {
      if (abort != nullptr && *reinterpret_cast<volatile int*>(abort) != 0) return false;
      if (i >= kMbarSpinBudget) {
        if (abort != nullptr) atomicCAS(abort, 0, kErrPipelineTimeout);
        return false;
      }
    }
  }
}

// ---------------------------------------------------------------------------
// TMA (cp.async.bulk.tensor) -- plain per-CTA loads only, never multicast.
// ---------------------------------------------------------------------------
MNB_DEVICE void tma_load_2d(uint32_t dst, const CUtensorMap* map, int32_t x, int32_t y,
                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
MNB_DEVICE void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// Shared -> global tile store, and the same tile added element-wise into global
// memory by the TMA unit (the adds happen at L2; the issuing thread does not wait).
// Both are tracked by the issuing thread's bulk async-group.
MNB_DEVICE void tma_store_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
MNB_DEVICE void tma_reduce_add_2d(const CUtensorMap* map, uint32_t src, int32_t x, int32_t y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%1, %2}], [%3];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(src)
               : "memory");
}
MNB_DEVICE void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N groups still read their shared-memory source.
template <int N>
MNB_DEVICE void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until every group has fully completed (global writes done).
MNB_DEVICE void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// ---------------------------------------------------------------------------
// tcgen05 (5th-generation tensor cores, accumulators in TMEM)
// ---------------------------------------------------------------------------
MNB_DEVICE void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
MNB_DEVICE void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
MNB_DEVICE void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
MNB_DEVICE void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
MNB_DEVICE void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 in, fp32 acc).
MNB_DEVICE void tc_mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                       uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Same, with the A operand read from TMEM instead of shared memory.
MNB_DEVICE void tc_mma_tmem_a(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                              uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every previously issued tcgen05.mma of this thread is done.
MNB_DEVICE void tc_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// Load 32 consecutive fp32 columns of this thread's TMEM lane.
MNB_DEVICE void tmem_ld_32(uint32_t taddr, float* out) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) out[i] = __uint_as_float(r[i]);
}

// Load 16 consecutive fp32 columns of this thread's TMEM lane.
MNB_DEVICE void tmem_ld_16(uint32_t taddr, float* out) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) out[i] = __uint_as_float(r[i]);
}

// 64 consecutive fp32 columns of this thread's TMEM lane with a single wait
// (one load instruction instead of two dependent x32 round trips).
MNB_DEVICE void tmem_ld_64(uint32_t taddr, float* out) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,"
      "%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) out[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive 32-bit columns into this thread's TMEM lane.
MNB_DEVICE void tmem_st_16(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]),
      "r"(v[15])
      : "memory");
}
MNB_DEVICE void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Shared-memory matrix descriptor (tcgen05 format, version 1) for a tile laid
// out in the 128-byte swizzle canonical form.  `lbo`/`sbo` in bytes.
MNB_DEVICE uint64_t smem_desc_sw128(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);
  d |= static_cast<uint64_t>((lbo & 0x3FFFFu) >> 4) << 16;
  d |= static_cast<uint64_t>((sbo & 0x3FFFFu) >> 4) << 32;
  d |= 1ull << 46;  // descriptor version for tcgen05
  d |= 2ull << 61;  // 128-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16 with bf16 A/B and fp32 D.
// a_mn / b_mn select the MN-major ("transposed") operand layout.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn, bool b_mn) {
  return (1u << 4)                        // D format: f32
         | (1u << 7)                      // A format: bf16
         | (1u << 10)                     // B format: bf16
         | ((a_mn ? 1u : 0u) << 15)       // A major-ness
         | ((b_mn ? 1u : 0u) << 16)       // B major-ness
         | ((static_cast<uint32_t>(n) >> 3) << 17)
         | ((static_cast<uint32_t>(m) >> 4) << 24);
}

// ---------------------------------------------------------------------------
// math
// ---------------------------------------------------------------------------
// GELU with the exact (erf) definition, x * Phi(x).  erf is evaluated with
// Abramowitz & Stegun, Handbook of Mathematical Functions, formula 7.1.26:
//   erf(z) = 1 - (a1 t + a2 t^2 + a3 t^3 + a4 t^4 + a5 t^5) exp(-z^2),
//   t = 1 / (1 + p z),  z >= 0,  |error| <= 1.5e-7,
// with the hardware reciprocal and base-2 exponential (checked against the
// exact erf to 1.4e-7 absolute over [-10, 10]; GELU outputs are rounded to
// bf16, whose resolution is ~4e-3).  The same exp(-z^2) = exp(-x^2 / 2) is
// the normal density's factor, so GELU' costs one more FMA.
MNB_DEVICE float rcp_approx(float x) {
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
MNB_DEVICE float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// returns Phi(x) = 0.5 (1 + erf(x / sqrt 2)) and e = exp(-x^2 / 2)
MNB_DEVICE float normal_cdf_as(float x, float* e_out) {
  const float z = fabsf(x) * 0.70710678118654752f;
  const float t = rcp_approx(fmaf(0.3275911f, z, 1.0f));
  const float poly =
      t * fmaf(t, fmaf(t, fmaf(t, fmaf(t, 1.061405429f, -1.453152027f), 1.421413741f), -0.284496736f), 0.254829592f);
  const float e = ex2_approx(-z * z * 1.4426950408889634f);
  const float erf_abs = fmaf(-poly, e, 1.0f);
  *e_out = e;
  return 0.5f + copysignf(0.5f * erf_abs, x);
}
MNB_DEVICE float gelu_exact(float x) {
  float e;
  return x * normal_cdf_as(x, &e);
}

// Packed fp32 pairs: sm_100's f32x2 add / mul / fma do two lanes' worth of
// fp32 math in one instruction (same IEEE rounding as two scalar ops).
MNB_DEVICE uint64_t f2_bits(float2 a) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a.x), "f"(a.y));
  return r;
}
MNB_DEVICE float2 f2_of(uint64_t r) {
  float2 a;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a.x), "=f"(a.y) : "l"(r));
  return a;
}
MNB_DEVICE float2 add2(float2 a, float2 b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_of(d);
}
MNB_DEVICE float2 mul2(float2 a, float2 b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_of(d);
}
MNB_DEVICE float2 fma2(float2 a, float2 b, float2 c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)), "l"(f2_bits(c)));
  return f2_of(d);
}
MNB_DEVICE float2 sub2(float2 a, float2 b) {
  uint64_t d;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(f2_bits(a)), "l"(f2_bits(b)));
  return f2_of(d);
}
MNB_DEVICE float2 splat2(float a) { return make_float2(a, a); }
// max of three floats in one instruction (sm_100)
MNB_DEVICE float max3f(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// normal_cdf_as on a pair, the polynomial and products in f32x2; the same
// formula and rounding as the scalar version except that the polynomial's
// sign is folded into its coefficients (exact).
MNB_DEVICE float2 normal_cdf_as2(float2 x, float2* e_out) {
  const float2 z = mul2(make_float2(fabsf(x.x), fabsf(x.y)), splat2(0.70710678118654752f));
  const float2 d = fma2(splat2(0.3275911f), z, splat2(1.0f));
  const float2 t = make_float2(rcp_approx(d.x), rcp_approx(d.y));
  float2 q = fma2(t, splat2(-1.061405429f), splat2(1.453152027f));
  q = fma2(t, q, splat2(-1.421413741f));
  q = fma2(t, q, splat2(0.284496736f));
  q = fma2(t, q, splat2(-0.254829592f));
  const float2 negpoly = mul2(t, q);  // -(a1 t + ... + a5 t^5)
  const float2 w = mul2(z, mul2(z, splat2(-1.4426950408889634f)));
  const float2 e = make_float2(ex2_approx(w.x), ex2_approx(w.y));
  const float2 erf_abs = fma2(negpoly, e, splat2(1.0f));
  *e_out = e;
  return fma2(erf_abs, make_float2(copysignf(0.5f, x.x), copysignf(0.5f, x.y)), splat2(0.5f));
}
MNB_DEVICE float2 gelu_exact2(float2 x) {
  float2 e;
  return mul2(x, normal_cdf_as2(x, &e));
}
MNB_DEVICE float2 gelu_grad2(float2 x) {
  float2 e;
  const float2 cdf = normal_cdf_as2(x, &e);
  return fma2(mul2(x, splat2(0.3989422804014327f)), e, cdf);
}
// d/dx [x * Phi(x)] = Phi(x) + x * phi(x), phi(x) = exp(-x^2 / 2) / sqrt(2 pi).
MNB_DEVICE float gelu_grad(float x) {
  float e;
  const float cdf = normal_cdf_as(x, &e);
  return fmaf(x * 0.3989422804014327f, e, cdf);
}

MNB_DEVICE float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
MNB_DEVICE float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace mnb
