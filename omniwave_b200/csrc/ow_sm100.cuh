// sm_100a building blocks for the tensor-core BiGEMM kernels: mbarriers with
// bounded waits, bulk copies, tcgen05 (TMEM alloc, UMMA issue/commit, TMEM
// loads), warp-level mma.sync for the 16x16 token mixes, ldmatrix, and the
// 128-byte-swizzled K-major shared-memory layout the UMMA descriptors use.
//
// Layout convention ("SW128 K-major"): an operand with R rows and K columns
// (K a multiple of 64 16-bit elements) is stored as K/64 "atoms"; atom a holds
// columns [64a, 64a+64) of every row as one 128-byte line per row, 8-row
// groups 1024 bytes apart, and the 16-byte chunk j of row r stored at chunk
// position j ^ (r % 8).  Every atom starts on a 1024-byte boundary.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace ow {
namespace sm100 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Wait for the phase with the given parity to complete.  Gives up after
// ``limit_ns`` of wall time (kWaitLimitNs unless told otherwise) and sets
// *abort (a flag in the CTA's shared memory) so that the caller's loops wind
// down instead of hanging; once *abort is set every wait returns false
// immediately.  The kernel reports an aborted CTA through report_abort().
constexpr uint64_t kWaitLimitNs = 2000000000ull;

// Code a kernel writes into the library's device fault word when one of its
// bounded waits gave up.
constexpr int kFaultWait = 1;

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (*abort) return false;
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  for (;;) {
    for (int i = 0; i < 256; ++i)
      if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer_ns() - t0 > limit_ns) {
      *abort = 1;
      return false;
    }
  }
}

// Wait-timeout self-check: with ``probe_ns`` > 0 the calling thread waits
// that long on ``bar``, a barrier nothing arrives on, before any copy or MMA
// of the kernel is issued.  The wait runs out, the CTA's abort flag is set,
// and every role skips its work.  Lets a test exercise the bounded-wait and
// fault-reporting path without a copy or MMA in flight.
__device__ __forceinline__ void wait_probe(uint64_t* bar, volatile int* abort, uint32_t probe_ns) {
  if (probe_ns) mbar_wait(bar, 0, abort, probe_ns);
}

// Called by every thread after the kernel's final __syncthreads: the first
// thread of an aborted CTA records kFaultWait in the device fault word.
__device__ __forceinline__ void report_abort(volatile int* abort, int* fault) {
  if (threadIdx.x == 0 && *abort && fault) atomicOr(fault, kFaultWait);
}

// ---------------------------------------------------------------- bulk copy
// 1-D global -> shared copy completing on an mbarrier (both addresses 16-byte
// aligned, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// 1-D shared -> global copy (bulk-group completion); both addresses 16-byte
// aligned, size a multiple of 16.  bulk_commit() closes a group;
// bulk_wait_read() waits until every committed group has read its source,
// bulk_wait_all() until every group has completed.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)),
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
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16/f16 in, f32 acc).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on ``bar`` once every tcgen05 op this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Instruction descriptor: kind::f16, f32 accumulate, A and B K-major.
// ``bf16`` selects bf16 operands (else f16).
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16) {
  return (1u << 4)                                   // D format: f32
         | ((bf16 ? 1u : 0u) << 7)                   // A format
         | ((bf16 ? 1u : 0u) << 10)                  // B format
         | ((uint32_t)(N >> 3) << 17)                // N / 8
         | ((uint32_t)(M >> 4) << 24);               // M / 16
}

// Shared-memory matrix descriptor for an SW128 K-major operand whose current
// 16-element K step starts at byte address ``addr`` (inside a 1024-aligned atom).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t addr) {
  return (uint64_t)((addr >> 4) & 0x3FFF)          // start address
         | ((uint64_t)1 << 16)                     // leading byte offset (unused for SW128 K-major)
         | ((uint64_t)(1024 >> 4) << 32)           // stride byte offset: 8 rows x 128 B
         | ((uint64_t)1 << 46)                     // descriptor version (sm100)
         | ((uint64_t)2 << 61);                    // layout: 128-byte swizzle
}

// Byte offset of element (r, k) in an SW128 K-major operand of ``rows`` rows.
__host__ __device__ __forceinline__ uint32_t sw128_off(int r, int k, int rows) {
  return (uint32_t)((k >> 6) * rows * 128 + (r >> 3) * 1024 + (r & 7) * 128 +
                    ((((k & 63) >> 3) ^ (r & 7)) << 4) + (k & 7) * 2);
}

// Address of the K step ``kk`` (16 elements) of an SW128 operand at ``base``.
__device__ __forceinline__ uint32_t sw128_kstep(uint32_t base, int kk, int rows) {
  return base + (uint32_t)((kk >> 2) * rows * 128 + (kk & 3) * 32);
}

// TMEM load: 32 lanes x 32 consecutive 32-bit columns (thread i <- lane i).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]),
        "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]),
        "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]),
        "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

// 32 lanes x N consecutive 32-bit columns (N = 16 or 32), one lane per thread.
template <int N>
__device__ __forceinline__ void tmem_ld_cols(uint32_t taddr, uint32_t (&r)[N]) {
  static_assert(N == 16 || N == 32, "tmem_ld_cols: N is 16 or 32");
  if constexpr (N == 32) tmem_ld32(taddr, r);
  else tmem_ld16(taddr, r);
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// TMEM load in the m16n8 C-fragment layout: 16 lanes x 16 columns from
// ``taddr``; r[0..3] hold columns 0-7 (row g: r0, r1; row g + 8: r2, r3 at
// columns 2 t4, 2 t4 + 1), r[4..7] the same for columns 8-15.
__device__ __forceinline__ void tmem_ld16x256_x2(uint32_t taddr, uint32_t (&r)[8]) {
  asm volatile("tcgen05.ld.sync.aligned.16x256b.x2.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7])
               : "r"(taddr));
}

// 8x8 16-bit transpose across the warp: turns a C-fragment pair into the
// matching B-fragment pair.
__device__ __forceinline__ uint32_t movm_trans(uint32_t v) {
  uint32_t o;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(o) : "r"(v));
  return o;
}

// m16n8k16 A fragment of a 16x16 matrix in shared/global row-major 16-bit
// storage (optionally transposed).
__device__ __forceinline__ void load_afrag(const uint16_t* A, bool trans, int g, int t4, uint32_t (&f)[4]) {
  auto el = [&](int m, int k) -> uint32_t { return trans ? A[k * 16 + m] : A[m * 16 + k]; };
  f[0] = el(g, 2 * t4) | (el(g, 2 * t4 + 1) << 16);
  f[1] = el(g + 8, 2 * t4) | (el(g + 8, 2 * t4 + 1) << 16);
  f[2] = el(g, 2 * t4 + 8) | (el(g, 2 * t4 + 9) << 16);
  f[3] = el(g + 8, 2 * t4 + 8) | (el(g + 8, 2 * t4 + 9) << 16);
}

// ---------------------------------------------------------------- warp MMA
template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  if constexpr (BF16) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  } else {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
}

__device__ __forceinline__ void ldsm_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                              uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                        uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

// Two floats -> packed 16-bit pair (low = a, high = b).
template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
  if constexpr (BF16) {
    __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  } else {
    __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<uint32_t*>(&h);
  }
}

template <bool BF16>
__device__ __forceinline__ float2 unpack2(uint32_t v) {
  if constexpr (BF16) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162*>(&v);
    return __bfloat1622float2(h);
  } else {
    __half2 h = *reinterpret_cast<__half2*>(&v);
    return __half22float2(h);
  }
}

// Packed f32x2 arithmetic (sm_100: one instruction for two f32 lanes, each
// rounded as the scalar operation would be).  Halves the instruction count
// of f32 element-wise code.
__device__ __forceinline__ uint64_t f2pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ float2 f2unpack(uint64_t v) {
  float2 r;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r.x), "=f"(r.y) : "l"(v));
  return r;
}
__device__ __forceinline__ uint64_t fma2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t d;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
  return d;
}
__device__ __forceinline__ uint64_t mul2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}
__device__ __forceinline__ uint64_t add2(uint64_t a, uint64_t b) {
  uint64_t d;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
  return d;
}

// silu(u) * v on a packed 16-bit pair, sigmoid via the hardware tanh:
// sigmoid(u) = 0.5 + 0.5 tanh(u / 2).
template <bool BF16>
__device__ __forceinline__ uint32_t silu_mul2(uint32_t u, uint32_t v) {
  uint32_t out;
  const uint32_t half2 = BF16 ? 0x3F003F00u : 0x38003800u;  // (0.5, 0.5)
  if constexpr (BF16) {
    asm("{\n\t.reg .b32 h, t, s, z;\n\t"
        "mul.rn.bf16x2 h, %1, %3;\n\t"        // u / 2
        "tanh.approx.bf16x2 t, h;\n\t"
        "fma.rn.bf16x2 s, t, %3, %3;\n\t"     // 0.5 t + 0.5 = sigmoid(u)
        "mul.rn.bf16x2 z, %1, s;\n\t"
        "mul.rn.bf16x2 %0, z, %2;\n\t}"
        : "=r"(out)
        : "r"(u), "r"(v), "r"(half2));
  } else {
    asm("{\n\t.reg .b32 h, t, s, z;\n\t"
        "mul.rn.f16x2 h, %1, %3;\n\t"
        "tanh.approx.f16x2 t, h;\n\t"
        "fma.rn.f16x2 s, t, %3, %3;\n\t"
        "mul.rn.f16x2 z, %1, s;\n\t"
        "mul.rn.f16x2 %0, z, %2;\n\t}"
        : "=r"(out)
        : "r"(u), "r"(v), "r"(half2));
  }
  return out;
}

}  // namespace sm100
}  // namespace ow
