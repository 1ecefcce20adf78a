// Shared device helpers for the sm_100a kernels: status reporting, mbarriers with bounded
// waits, TMA tiled loads, tcgen05 (TMEM alloc, MMA, commit, loads), UMMA descriptors and the
// exact MXFP4 (E2M1 codes + E8M0 block-32 scales) decode into fp16.
#pragma once
#include <cstdint>
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include "lazylora_b200.h"

#define LL_DEV __device__ __forceinline__

// Programmatic dependent launch. A kernel launched with the programmatic-serialization
// attribute (launch_pdl) may be scheduled while the kernel before it on the stream still runs;
// pdl_wait() returns once that kernel has completed and its writes are visible. Since that
// kernel waited in the same way, everything earlier on the stream has completed too. A kernel
// launched so calls pdl_wait() in every block before its first read or write of global memory
// another kernel produces or consumes, and before it can exit (so that completion stays
// ordered). pdl_launch_next() lets the next kernel's blocks be scheduled now; kernels that
// allocate tensor memory call it only after their allocation, so that a waiting successor never
// holds columns a running predecessor still has to allocate.
LL_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
LL_DEV void pdl_launch_next() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// K per tensor-memory / activation ring stage of the grouped GEMM (64 or 128); each 128-K
// packed weight stage feeds 128 / LL_KS ring stages. 64-K stages double the ring depth for the
// same tensor memory but also every per-stage barrier and commit; they measured 16 % slower
// on configs[1] and 3 % on 128-row tiles, so 128 is the default.
#ifndef LL_KS
#define LL_KS 128
#endif

namespace ll {

// ------------------------------------------------------------------------------ status
// Kernels never trap. A wait that runs out records LL_ERR_TIMEOUT (and where) in a
// caller-visible status word and the kernel winds down; the host reads the word back.
struct DevStatus {
  int code;
  int where;
  int info;
  int pad;
};

LL_DEV void report(DevStatus* st, int code, int where, int info) {
  if (st && atomicCAS(&st->code, 0, code) == 0) {
    st->where = where;
    st->info = info;
  }
}

// ---------------------------------------------------------------------------- mbarrier
LL_DEV uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

LL_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

LL_DEV void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

LL_DEV void fence_async_smem() {  // generic-proxy smem writes -> visible to the async proxy
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

LL_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

LL_DEV void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

LL_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
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

// ~1 s at the B200's clocks: a healthy pipeline waits microseconds.
constexpr long long kWaitLimitCycles = 2000000000LL;

// Bounded wait. Returns false (after recording the timeout and raising the CTA abort flag)
// when the phase does not complete in time, or when another role already aborted.
LL_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, DevStatus* st,
                      int where) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      report(st, LL_ERR_TIMEOUT, where, 0);
      return false;
    }
  }
}

// Bounded wait for a warp off the critical path (a producer that is ahead, an issuer, an
// epilogue waiting for the next tile): polls with a __nanosleep back-off that doubles from
// 32 ns up to ns_max, so the waiting warp stops taking issue slots from the warps that work.
LL_DEV bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort_flag, DevStatus* st, int where,
                            uint32_t ns_max) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  uint32_t ns = 32;
  while (true) {
    __nanosleep(ns);
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      report(st, LL_ERR_TIMEOUT, where, 0);
      return false;
    }
    ns = ns < ns_max ? ns * 2 : ns_max;
  }
}

// A monotonic event counter in shared memory, published by one thread and polled by another:
// release / acquire at CTA scope carry the publisher's observations (e.g. an mbarrier phase it
// waited for) to the poller.
LL_DEV void seq_publish(uint32_t* seq, uint32_t v) {
  asm volatile("st.release.cta.shared::cta.u32 [%0], %1;" ::"r"(smem_u32(seq)), "r"(v) : "memory");
}
LL_DEV uint32_t seq_read(uint32_t* seq) {
  uint32_t v;
  asm volatile("ld.acquire.cta.shared::cta.u32 %0, [%1];" : "=r"(v) : "r"(smem_u32(seq)) : "memory");
  return v;
}
// Bounded poll until *seq >= target; false after a timeout (recorded) or another role's abort.
LL_DEV bool seq_wait(uint32_t* seq, uint32_t target, volatile int* abort_flag, DevStatus* st, int where) {
  if (seq_read(seq) >= target) return true;
  const long long t0 = clock64();
  while (true) {
    if (seq_read(seq) >= target) return true;
    if (*abort_flag) return false;
    if (clock64() - t0 > kWaitLimitCycles) {
      *abort_flag = 1;
      report(st, LL_ERR_TIMEOUT, where, 0);
      return false;
    }
  }
}

// Named barriers (bar.sync / bar.arrive): warp-granular, all 32 lanes of a warp execute them.
LL_DEV void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}
LL_DEV void named_bar_arrive(int id, int nthreads) {
  asm volatile("bar.arrive %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// --------------------------------------------------------------------------------- TMA
LL_DEV void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

LL_DEV void tma_load_2d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1)
      : "memory");
}

LL_DEV void tma_load_3d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}

LL_DEV void tma_load_4d(void* dst, const CUtensorMap* m, uint64_t* bar, int c0, int c1, int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

// ----------------------------------------------------------------------------- tcgen05
LL_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

LL_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {  // whole warp
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

LL_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
LL_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (fp16 or bf16 in, fp32 accumulate)
LL_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A occupies 128 lanes (lane = row m); a
// 32-bit column c holds k = 2c (low half) and k = 2c + 1 (high half), 8 columns per K = 16.
LL_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 16 consecutive 32-bit columns from registers; thread i writes lane (base + i).
LL_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

LL_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
LL_DEV void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

LL_DEV void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 16 consecutive 32-bit columns; thread i of the warp gets lane (base lane + i).
LL_DEV void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
#pragma unroll
  for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}

// The same load without the conversion: the registers are valid only after tcgen05.wait::ld
// and tmem_regs_ready (which ties them to a point after the wait, so no use is scheduled
// earlier).
LL_DEV void tmem_ld16_u(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
}

LL_DEV void tmem_regs_ready(uint32_t (&r)[16]) {
  asm volatile(""
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15])
               :
               : "memory");
}

// UMMA shared-memory descriptor (tcgen05 format): start address, leading / stride byte
// offsets (all >> 4), version 1 at bits 46-47, layout type at bits 61-63.
enum : uint32_t { kSwizzleNone = 0, kSwizzle128B = 2, kSwizzle64B = 4, kSwizzle32B = 6 };

LL_DEV uint64_t umma_desc(uint32_t smem_addr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)(layout & 0x7) << 61;
  return d;
}

// Instruction descriptor, kind::f16: fp16 A and B, fp32 D, M = 128, N = n (multiple of 16).
LL_DEV uint32_t idesc_f16_m128(uint32_t n, bool a_mn_major, bool b_mn_major) {
  uint32_t d = 0;
  d |= 1u << 4;                  // D format F32
  d |= 0u << 7;                  // A format F16
  d |= 0u << 10;                 // B format F16
  d |= (a_mn_major ? 1u : 0u) << 15;
  d |= (b_mn_major ? 1u : 0u) << 16;
  d |= (n >> 3) << 17;
  d |= (128u >> 4) << 24;
  return d;
}

// ------------------------------------------------------------- block-scaled tcgen05 MMA
// D[tmem] (+)= (A * SFA)[smem desc] * (B * SFB)[smem desc], kind::mxf8f6f4 with one E8M0 scale
// per 32 K elements of every A row and B row, read from tensor memory at sfa / sfb (the byte
// of each 32-bit word selected by bits 30-31 of the address and the ids in the descriptor).
LL_DEV void mma_mxf8f6f4_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa,
                            uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::mxf8f6f4 block-scaled: A E2M1 (K-major), B E4M3 (K-major), fp32
// D, E8M0 scales, M = 128, N = n (multiple of 16, <= 256), K = 32; sf_a / sf_b select the scale
// byte (the 32-K block within a 32-bit scale word) of A and B.
LL_DEV uint32_t idesc_mxf4xe4m3_m128(uint32_t n, uint32_t sf_a, uint32_t sf_b) {
  uint32_t d = 0;
  d |= (sf_b & 3u) << 4;        // B scale-factor id
  d |= 5u << 7;                 // A format E2M1
  d |= 0u << 10;                // B format E4M3
  d |= (n >> 3) << 17;          // N
  d |= 1u << 23;                // scale format E8M0
  d |= (128u >> 4) << 24;       // M
  d |= (sf_a & 3u) << 29;       // A scale-factor id
  return d;
}

// D[tmem] (+)= (A * SFA) * (B * SFB), kind::mxf4: A and B packed E2M1 (two per byte) in shared
// memory, one E8M0 scale per 32 K elements of every row, K = 64 per instruction (two scale
// bytes of each row: those at sf_id and sf_id + 1).
LL_DEV void mma_mxf4_bs(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t sfa,
                        uint32_t sfb, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %6, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf4.block_scale.block32 [%0], %1, %2, %3, [%4], [%5], p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(sfa), "r"(sfb), "r"(accumulate)
      : "memory");
}

// Instruction descriptor, kind::mxf4: A and B E2M1 (K-major), fp32 D, E8M0 scales, M = 128,
// N = n (multiple of 16, <= 256), K = 64; sf_a / sf_b the first scale byte of each row used.
LL_DEV uint32_t idesc_mxf4_m128(uint32_t n, uint32_t sf_a, uint32_t sf_b) {
  uint32_t d = 0;
  d |= (sf_b & 3u) << 4;        // B scale-factor id
  d |= 1u << 7;                 // A format E2M1
  d |= 1u << 10;                // B format E2M1
  d |= (n >> 3) << 17;          // N
  d |= 1u << 23;                // scale format E8M0
  d |= (128u >> 4) << 24;       // M
  d |= (sf_a & 3u) << 29;       // A scale-factor id
  return d;
}

// Two floats -> two E2M1 codes in one byte (lo in the low nibble), round to nearest even,
// saturating to +-6.
LL_DEV uint32_t f32x2_to_e2m1x2(float lo, float hi) {
  uint32_t r;
  asm("{\n\t.reg .b8 b;\n\t"
      "cvt.rn.satfinite.e2m1x2.f32 b, %1, %2;\n\t"
      "cvt.u32.u8 %0, b;\n\t}"
      : "=r"(r)
      : "f"(hi), "f"(lo));
  return r;
}

// 32 rows x 128 bits from shared memory (descriptor, no swizzle, 16-byte rows) into tensor
// memory lanes 0..31 at columns taddr .. taddr + 3, replicated into all four lane quarters.
LL_DEV void tmem_cp_32x128b_x4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// L2 prefetch of a 2-D TMA box (no shared memory, no barrier).
LL_DEV void tma_prefetch_l2_2d(const CUtensorMap* m, int c0, int c1) {
  asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(reinterpret_cast<uint64_t>(m)),
               "r"(c0), "r"(c1)
               : "memory");
}

// L2 prefetch of a contiguous range (16-byte aligned, size % 16 == 0).
LL_DEV void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(reinterpret_cast<uint64_t>(src)), "r"(bytes)
               : "memory");
}

// Contiguous global -> shared copy on the async proxy (16-byte aligned, size % 16 == 0),
// completing `bytes` transactions on bar.
LL_DEV void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Two floats -> two E4M3 bytes, round to nearest, saturating to +-448 (lo in the low byte).
LL_DEV uint32_t f32x2_to_e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}

// Two E4M3 bytes (low byte = first) -> their exact values.
LL_DEV float2 e4m3x2_to_f32x2(uint32_t b2) {
  uint32_t h2;
  const uint16_t b = (uint16_t)b2;
  asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(h2) : "h"(b));
  return __half22float2(*reinterpret_cast<const __half2*>(&h2));
}

// Power-of-two exponent e that brings max|row| into [2^7, 2^8): the first E4M3 term of a row
// scaled by 2^e keeps its largest entries at full E4M3 precision, well inside the +-448 range.
LL_DEV int e4m3_scale_exp(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 0;
  int e;
  frexpf(maxabs, &e);   // maxabs in [2^(e-1), 2^e)
  return 8 - e;
}

// ------------------------------------------------------------------------ MXFP4 decode
// fp16 bit pattern of 2^(b - 127 + bias) for an E8M0 scale byte b; 0 for b >= 253 (an
// unrepresentable / damaged group contributes nothing) and for exponents below fp16's
// smallest subnormal 2^-24. The caller picks `bias` so that 6 * 2^(b-127+bias) <= 2^15.
LL_DEV uint32_t e8m0_to_half_bits(uint32_t b, int bias) {
  // 2^(b - 127 + bias) built as an fp32 power of two and rounded to fp16: exact for normal
  // and subnormal fp16 powers of two, 0 below 2^-24 (2^-25 rounds to even, 0)
  const int t = (int)b + bias;                      // biased fp32 exponent of the scale
  const uint32_t h = __half_as_ushort(__float2half_rn(__int_as_float(t << 23)));
  return (b >= 253u || t <= 0) ? 0u : h;
}

// The same scale in both halves of an fp16x2 (one f32x2 -> f16x2 conversion packs the pair).
LL_DEV uint32_t e8m0_to_half2_bits(uint32_t b, int bias) {
  const int t = (int)b + bias;
  const float f = __int_as_float(t << 23);
  uint32_t h2;
  asm("cvt.rn.f16x2.f32 %0, %1, %1;" : "=r"(h2) : "f"(f));
  return (b >= 253u || t <= 0) ? 0u : h2;
}

// Two E2M1 codes (low nibble = even element) -> fp16x2 (even element in the low half),
// exact. One hardware conversion per byte.
LL_DEV uint32_t e2m1x2_to_half2(uint32_t byte) {
  uint32_t out;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t}"
      : "=r"(out)
      : "r"(byte));
  return out;
}

// Four bytes (8 codes) -> 4 x fp16x2, scaled by an fp16x2 splat of the group scale.
LL_DEV void decode8(uint32_t w, uint32_t scale2, uint32_t (&o)[4]) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(h0), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[1]) : "r"(h1), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[2]) : "r"(h2), "r"(scale2));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[3]) : "r"(h3), "r"(scale2));
}

// Four bytes (8 codes) -> 4 x fp16x2, output pair j scaled by its own fp16x2 scale sc[j].
LL_DEV void decode8v(uint32_t w, const uint32_t* sc, uint32_t* o) {
  uint32_t h0, h1, h2, h3;
  asm("{\n\t.reg .b8 b0, b1, b2, b3;\n\t"
      "mov.b32 {b0, b1, b2, b3}, %4;\n\t"
      "cvt.rn.f16x2.e2m1x2 %0, b0;\n\t"
      "cvt.rn.f16x2.e2m1x2 %1, b1;\n\t"
      "cvt.rn.f16x2.e2m1x2 %2, b2;\n\t"
      "cvt.rn.f16x2.e2m1x2 %3, b3;\n\t}"
      : "=r"(h0), "=r"(h1), "=r"(h2), "=r"(h3)
      : "r"(w));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[0]) : "r"(h0), "r"(sc[0]));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[1]) : "r"(h1), "r"(sc[1]));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[2]) : "r"(h2), "r"(sc[2]));
  asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(o[3]) : "r"(h3), "r"(sc[3]));
}

LL_DEV void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}

LL_DEV uint4 ld_shared_v4(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// -------------------------------------------------------------------------- SiTU-GLU
// situ(g) = 4 tanh(g/4) sigmoid(g);  u' = 25 tanh(u/25)   (beta 4, linear beta 25)
constexpr float kSituBeta = 4.0f;
constexpr float kSituLinBeta = 25.0f;

LL_DEV float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

LL_DEV float situ_glu_fwd(float g, float u) {
  const float a = kSituBeta * tanhf(g / kSituBeta) * sigmoidf_(g);
  return a * (kSituLinBeta * tanhf(u / kSituLinBeta));
}

LL_DEV void situ_glu_bwd(float go, float g, float u, float& dg, float& du) {
  const float t = tanhf(g / kSituBeta);
  const float s = sigmoidf_(g);
  const float a = kSituBeta * t * s;
  const float da = (1.0f - t * t) * s + kSituBeta * t * s * (1.0f - s);
  const float tu = tanhf(u / kSituLinBeta);
  dg = go * (kSituLinBeta * tu) * da;
  du = go * a * (1.0f - tu * tu);
}

// power-of-two exponent that brings max|row| into [2^14, 2^15): fp16 keeps full precision
// for the large entries and has headroom below 65504.
LL_DEV int row_scale_exp(float maxabs) {
  if (!(maxabs > 0.f) || !isfinite(maxabs)) return 0;
  int e;
  frexpf(maxabs, &e);   // maxabs = m * 2^e, m in [0.5, 1)
  return 15 - e;        // maxabs * 2^(15-e) in [2^14, 2^15)
}

}  // namespace ll
