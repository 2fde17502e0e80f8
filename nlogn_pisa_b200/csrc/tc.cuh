// Blackwell (sm_100a) tensor-core building blocks written as inline PTX:
// tensor memory (TMEM) allocation, tcgen05.mma with shared-memory operand
// descriptors, commit to an mbarrier, tcgen05.ld of the accumulator, and the
// bounded mbarrier wait used everywhere a thread waits on asynchronous work.
//
// Operand layout used throughout: K-major bf16/fp16 tiles whose rows are
// 128 bytes (64 elements) wide, stored with the 128-byte swizzle -- within
// each 1024-byte atom of 8 rows, the 16-byte chunk c of row r lives at chunk
// position (c ^ r).  A tile of R rows x 64 elements occupies R*128 bytes and
// must be 1024-byte aligned; wider K is a sequence of such tiles.
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace pisa {
namespace tc {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// Byte offset of 16-byte chunk `c` (0..7) of row `r` inside a 128B-swizzled tile.
__device__ __forceinline__ uint32_t swizzle128(int r, int c) {
  return uint32_t(r) * 128u + (uint32_t((c ^ (r & 7)) & 7) << 4);
}

// Shared-memory matrix descriptor: K-major, 128-byte swizzle, 8-row core
// groups 1024 bytes apart (stride byte offset), descriptor version 1.
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFFu) >> 4);      // start address
  d |= uint64_t(1) << 16;                       // leading byte offset (unused when swizzled)
  d |= uint64_t(1024 >> 4) << 32;               // stride byte offset
  d |= uint64_t(1) << 46;                       // version
  d |= uint64_t(2) << 61;                       // 128-byte swizzle
  return d;
}

// Instruction descriptor for kind::f16 with fp32 accumulation.
// ab_bf16: 1 for bf16 operands, 0 for fp16.  Both operands K-major unless
// b_mn_major (B stored with N contiguous, e.g. V in [keys][dims] order).
__host__ __device__ __forceinline__ uint32_t idesc_f16(int M, int N, int ab_bf16, int b_mn_major = 0) {
  uint32_t d = 0;
  d |= 1u << 4;                          // D format: f32
  d |= uint32_t(ab_bf16) << 7;           // A format
  d |= uint32_t(ab_bf16) << 10;          // B format
  d |= uint32_t(b_mn_major) << 16;       // B major-ness
  d |= uint32_t(N >> 3) << 17;
  d |= uint32_t(M >> 4) << 24;
  return d;
}

__device__ __forceinline__ void fence_before_sync() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void fence_after_sync() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// Make generic-proxy shared-memory writes visible to the tensor core.
__device__ __forceinline__ void fence_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// Warp-collective: allocate `ncols` TMEM columns (power of two >= 32); the
// base address is written to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(slot)), "r"(ncols) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(base), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                        uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      :: "r"(d_tmem), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Arrive on `mbar` once every MMA issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t* mbar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(smem_u32(mbar)) : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* mbar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(smem_u32(mbar)), "r"(count) : "memory");
}

// Make mbarrier initialisation visible to the async proxy (tcgen05.commit).
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* mbar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(smem_u32(mbar)) : "memory");
}

// Arrive on `mbar` once every cp.async issued so far by this thread has
// landed (the arrival counts toward the barrier's initial count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* mbar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" :: "r"(smem_u32(mbar)) : "memory");
}

// One arrival that also expects `bytes` more transaction bytes (TMA) this phase.
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* mbar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;"
               :: "r"(smem_u32(mbar)), "r"(bytes) : "memory");
}

// TMA: copy the box at coordinates (c0..c3) of a 4-D tensor map into shared
// memory at `dst` (the map's swizzle applies); completion counts the box's
// bytes on `mbar`.  c0 (innermost) is always a multiple of 64 elements here.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint64_t* mbar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];"
      :: "r"(dst), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
         "r"(smem_u32(mbar))
      : "memory");
}

// Barrier among `count` threads of the CTA on hardware barrier `id` (1..15).
__device__ __forceinline__ void named_sync(int id, int count) {
  asm volatile("bar.sync %0, %1;" :: "r"(id), "r"(count) : "memory");
}

// Non-blocking test of the phase with parity `phase` (no suspension).
__device__ __forceinline__ bool mbar_test(uint64_t* mbar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(mbar)), "r"(phase) : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* mbar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok) : "r"(smem_u32(mbar)), "r"(phase) : "memory");
  return ok != 0;
}

// Bounded wait for the phase with parity `phase` to complete.  Returns false
// (and the caller records a timeout status) instead of spinning forever.
__device__ __forceinline__ bool mbar_wait(uint64_t* mbar, uint32_t phase, uint32_t max_tries = 1u << 22) {
  for (uint32_t i = 0; i < max_tries; ++i)
    if (mbar_try_wait(mbar, phase)) return true;
  return false;
}

// 32 lanes x 32 consecutive 32-bit TMEM columns -> 32 registers per thread
// (thread i of warp w reads lane 32*(w%4) + i), waiting for completion inside
// the same asm statement so no consumer can be scheduled before the data lands.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]),
        "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]),
        "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 lanes x 64 consecutive 32-bit TMEM columns -> 64 registers per thread, waited.
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// The same load without waiting: registers are valid after tmem_wait_ld2().
__device__ __forceinline__ void tmem_ld64_nowait(uint32_t taddr, uint32_t (&r)[64]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr)
      : "memory");
}

// Wait for the loads into a and b; the registers pass through the asm
// statements so no use of them can be scheduled before the wait.
__device__ __forceinline__ void tmem_wait_ld2(uint32_t (&a)[64], uint32_t (&b)[64]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;" : "+r"(a[0]), "+r"(a[1]), "+r"(a[2]), "+r"(a[3]), "+r"(a[4]), "+r"(a[5]), "+r"(a[6]), "+r"(a[7]), "+r"(a[8]), "+r"(a[9]), "+r"(a[10]), "+r"(a[11]), "+r"(a[12]), "+r"(a[13]), "+r"(a[14]), "+r"(a[15]), "+r"(a[16]), "+r"(a[17]), "+r"(a[18]), "+r"(a[19]), "+r"(a[20]), "+r"(a[21]), "+r"(a[22]), "+r"(a[23]), "+r"(a[24]), "+r"(a[25]), "+r"(a[26]), "+r"(a[27]), "+r"(a[28]), "+r"(a[29]), "+r"(a[30]), "+r"(a[31]), "+r"(a[32]), "+r"(a[33]), "+r"(a[34]), "+r"(a[35]), "+r"(a[36]), "+r"(a[37]), "+r"(a[38]), "+r"(a[39]), "+r"(a[40]), "+r"(a[41]), "+r"(a[42]), "+r"(a[43]), "+r"(a[44]), "+r"(a[45]), "+r"(a[46]), "+r"(a[47]), "+r"(a[48]), "+r"(a[49]), "+r"(a[50]), "+r"(a[51]), "+r"(a[52]), "+r"(a[53]), "+r"(a[54]), "+r"(a[55]), "+r"(a[56]), "+r"(a[57]), "+r"(a[58]), "+r"(a[59]), "+r"(a[60]), "+r"(a[61]), "+r"(a[62]), "+r"(a[63]) :: "memory");
  asm volatile("" : "+r"(b[0]), "+r"(b[1]), "+r"(b[2]), "+r"(b[3]), "+r"(b[4]), "+r"(b[5]), "+r"(b[6]), "+r"(b[7]), "+r"(b[8]), "+r"(b[9]), "+r"(b[10]), "+r"(b[11]), "+r"(b[12]), "+r"(b[13]), "+r"(b[14]), "+r"(b[15]), "+r"(b[16]), "+r"(b[17]), "+r"(b[18]), "+r"(b[19]), "+r"(b[20]), "+r"(b[21]), "+r"(b[22]), "+r"(b[23]), "+r"(b[24]), "+r"(b[25]), "+r"(b[26]), "+r"(b[27]), "+r"(b[28]), "+r"(b[29]), "+r"(b[30]), "+r"(b[31]), "+r"(b[32]), "+r"(b[33]), "+r"(b[34]), "+r"(b[35]), "+r"(b[36]), "+r"(b[37]), "+r"(b[38]), "+r"(b[39]), "+r"(b[40]), "+r"(b[41]), "+r"(b[42]), "+r"(b[43]), "+r"(b[44]), "+r"(b[45]), "+r"(b[46]), "+r"(b[47]), "+r"(b[48]), "+r"(b[49]), "+r"(b[50]), "+r"(b[51]), "+r"(b[52]), "+r"(b[53]), "+r"(b[54]), "+r"(b[55]), "+r"(b[56]), "+r"(b[57]), "+r"(b[58]), "+r"(b[59]), "+r"(b[60]), "+r"(b[61]), "+r"(b[62]), "+r"(b[63]) :: "memory");
}

// ---- fp32 helpers on the packed / special-function paths ----
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// 2^x on the special-function unit (approximate, flush-to-zero).
__device__ __forceinline__ float ex2f(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
// (a*b + c) on two lanes at once.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 add2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "add.rn.f32x2 rd, ra, rb;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Max of 64 values with four independent 3-input max chains.
// 2^x for a pair of fp32 values on the FMA and integer pipes, leaving the
// MUFU unit (ex2.approx) free for the other exponentials of an epilogue.
// Range reduction: adding 1.5 * 2^23 rounds x to the nearest integer j, which
// lands in the low mantissa bits of the sum; f = x - j lies in [-0.5, 0.5].
// 2^f is a degree-5 polynomial whose coefficients were fitted for minimum
// maximum relative error on [-0.5, 0.5] (Lawson-weighted least squares;
// 2.3e-7 maximum relative error with fp32 Horner evaluation, the size of
// ex2.approx.f32's error); 2^j is applied by adding j to the exponent field
// (j << 23 equals the sum's bits << 23, since the constant's low 9 bits are 0).
// Inputs are clamped at -125: results below 2^-125 are not exact.
__device__ __forceinline__ float2 ex2_poly2(float2 x) {
  x.x = fmaxf(x.x, -125.f);
  x.y = fmaxf(x.y, -125.f);
  const float2 magic = make_float2(12582912.f, 12582912.f);
  const float2 t = add2(x, magic);
  const float2 j = add2(t, make_float2(-12582912.f, -12582912.f));
  const float2 f = fma2(j, make_float2(-1.f, -1.f), x);
  float2 p = fma2(make_float2(1.3276325771585107e-3f, 1.3276325771585107e-3f), f,
                  make_float2(9.675491601228714e-3f, 9.675491601228714e-3f));
  p = fma2(p, f, make_float2(5.550713092088699e-2f, 5.550713092088699e-2f));
  p = fma2(p, f, make_float2(2.4022120237350464e-1f, 2.4022120237350464e-1f));
  p = fma2(p, f, make_float2(6.931469440460205e-1f, 6.931469440460205e-1f));
  p = fma2(p, f, make_float2(1.0000001192092896f, 1.0000001192092896f));
  return make_float2(__int_as_float(__float_as_int(p.x) + (__float_as_int(t.x) << 23)),
                     __int_as_float(__float_as_int(p.y) + (__float_as_int(t.y) << 23)));
}

__device__ __forceinline__ float max32(const float (&v)[32]) {
  float m0 = v[0], m1 = v[1], m2 = v[2], m3 = v[3];
#pragma unroll
  for (int i = 4; i < 32; i += 8) {
    m0 = max3f(m0, v[i], v[i + 1]);
    m1 = max3f(m1, v[i + 2], v[i + 3]);
    m2 = max3f(m2, v[i + 4], v[i + 5]);
    m3 = max3f(m3, v[i + 6], v[i + 7]);
  }
  return fmaxf(max3f(m0, m1, m2), m3);
}

// sum_i 2^(v_i * k - c) over 32 values, packed pairs, two accumulators
__device__ __forceinline__ float sum_ex2_32(const float (&v)[32], float k, float c) {
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  const float2 kk = make_float2(k, k), cc = make_float2(-c, -c);
#pragma unroll
  for (int i = 0; i < 32; i += 4) {
    float2 x0 = fma2(make_float2(v[i], v[i + 1]), kk, cc);
    float2 x1 = fma2(make_float2(v[i + 2], v[i + 3]), kk, cc);
    acc0 = add2(acc0, make_float2(ex2f(x0.x), ex2f(x0.y)));
    acc1 = add2(acc1, make_float2(ex2f(x1.x), ex2f(x1.y)));
  }
  const float2 t = add2(acc0, acc1);
  return t.x + t.y;
}

__device__ __forceinline__ float max64(const float (&v)[64]) {
  float m0 = v[0], m1 = v[1], m2 = v[2], m3 = v[3];
#pragma unroll
  for (int i = 4; i < 64; i += 8) {
    m0 = max3f(m0, v[i], v[i + 1]);
    m1 = max3f(m1, v[i + 2], v[i + 3]);
    m2 = max3f(m2, v[i + 4], v[i + 5]);
    m3 = max3f(m3, v[i + 6], v[i + 7]);
  }
  return fmaxf(max3f(m0, m1, m2), m3);
}

// sum_i 2^(v_i * k - c) over 64 values (packed FMA for the arguments).
__device__ __forceinline__ float sum_ex2_64(const float (&v)[64], float k, float c) {
  float2 acc0 = make_float2(0.f, 0.f), acc1 = make_float2(0.f, 0.f);
  const float2 kk = make_float2(k, k), cc = make_float2(-c, -c);
#pragma unroll
  for (int i = 0; i < 64; i += 4) {
    float2 x0 = fma2(make_float2(v[i], v[i + 1]), kk, cc);
    float2 x1 = fma2(make_float2(v[i + 2], v[i + 3]), kk, cc);
    acc0 = add2(acc0, make_float2(ex2f(x0.x), ex2f(x0.y)));
    acc1 = add2(acc1, make_float2(ex2f(x1.x), ex2f(x1.y)));
  }
  const float2 t = add2(acc0, acc1);
  return t.x + t.y;
}

// 32 lanes x 16 consecutive 32-bit TMEM columns -> 16 registers per thread, waited.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// Store 16 consecutive 32-bit columns of this thread's TMEM lane and wait.
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
         "r"(r[7]), "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]),
         "r"(r[14]), "r"(r[15])
      : "memory");
}

// Store 8 consecutive 32-bit columns of this thread's TMEM lane and wait.
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      :: "r"(taddr), "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
         "r"(r[7])
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]; A is K-major in TMEM (lane = row).
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      :: "r"(d_tmem), "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate) : "memory");
}

// Generic descriptor with explicit byte offsets (for layout experiments and
// MN-major operands): leading/stride byte offsets and swizzle code.
__device__ __forceinline__ uint64_t desc_make(uint32_t saddr, uint32_t lbo, uint32_t sbo, uint32_t swizzle) {
  uint64_t d = 0;
  d |= uint64_t((saddr & 0x3FFFFu) >> 4);
  d |= uint64_t((lbo >> 4) & 0x3FFFu) << 16;
  d |= uint64_t((sbo >> 4) & 0x3FFFu) << 32;
  d |= uint64_t(1) << 46;
  d |= uint64_t(swizzle & 7u) << 61;
  return d;
}

}  // namespace tc
}  // namespace pisa
