// Thin inline-PTX wrappers for the sm_100a features the FA2 forward kernel uses:
// mbarriers (with bounded waits), TMA tile loads/stores, tcgen05 MMA / TMEM
// load-store / commit / fences, and the UMMA shared-memory + instruction
// descriptors. Everything here is written against the public PTX ISA (8.7+).
#pragma once

#include <cstdint>
#include <cuda.h>

namespace fa2 {

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;" ::"r"(bar),
               "r"(bytes)
               : "memory");
}

#ifndef FA2_WAIT_SUSPEND_NS
#define FA2_WAIT_SUSPEND_NS 0  // >0: suspend-time hint (ns) for waits; measured: no gain, off
#endif

// One potentially-blocking probe: the thread may be suspended (without issuing) until the
// phase completes or the suspend-time hint expires.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
#if FA2_WAIT_SUSPEND_NS > 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(static_cast<uint32_t>(FA2_WAIT_SUSPEND_NS))
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

#ifndef FA2_WAIT_UNROLL
// 8: the slow path of mbar_wait probes 8 times per call in one PTX block (two instructions a
// probe instead of ~6). Measured against 1 on one box: headline -2.6%, mha_causal -2.5%,
// pack_tail -3.9%, full_long (D = 64) +2%. 1 (shipped): one probe per loop iteration.
#define FA2_WAIT_UNROLL 1
#endif

// Up to 8 potentially-blocking probes back to back (two instructions each): true as soon as one
// sees the phase complete.
__device__ __forceinline__ bool mbar_try_wait8(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t@p bra DONE;\n\t"
      "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n"
      "DONE:\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait that polls without suspending the thread (lowest wake-up latency; for the
// single MMA-issuing thread, whose waits sit on the critical path).
__device__ __forceinline__ bool mbar_wait_spin(uint32_t bar, uint32_t parity, long long timeout_cycles,
                                               const int* err) {
  if (mbar_test_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (mbar_test_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (clock64() - t0 > timeout_cycles) return false;
      if (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0) return false;
    }
  }
}

// Waits for the phase of `bar` with the given parity to complete. Gives up after
// `timeout_cycles` SM clocks, or as soon as another CTA has raised the kernel's error
// word, and returns false; the caller then abandons its role and joins the teardown.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, long long timeout_cycles,
                                          const int* err) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (FA2_WAIT_UNROLL > 1 ? mbar_try_wait8(bar, parity) : mbar_try_wait(bar, parity)) return true;
    if ((it & (FA2_WAIT_UNROLL > 1 ? 7u : 63u)) == 0u) {
      if (clock64() - t0 > timeout_cycles) return false;
      if (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0) return false;
    }
  }
}

// As mbar_wait for a whole warp (all 32 lanes call it): every probe and every exit test is a
// warp vote, so the loop's branches are warp-uniform. Returns the same value in every lane.
__device__ __forceinline__ bool mbar_wait_warp(uint32_t bar, uint32_t parity, long long timeout_cycles,
                                               const int* err) {
  if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity))) return true;
    if ((it & 63u) == 0u) {
      const bool stop = (clock64() - t0 > timeout_cycles) ||
                        (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0);
      if (__any_sync(0xffffffffu, stop)) return false;
    }
  }
}

// Waits until the device word *flag becomes non-zero (written by another kernel or the
// host), bounded like mbar_wait.
__device__ __forceinline__ bool flag_wait(const int* flag, long long timeout_cycles, const int* err) {
  const volatile int* f = reinterpret_cast<const volatile int*>(flag);
  if (*f != 0) return true;
  const long long t0 = clock64();
  for (uint32_t it = 1;; ++it) {
    __nanosleep(256);
    if (*f != 0) return true;
    if ((it & 15u) == 0u) {
      if (clock64() - t0 > timeout_cycles) return false;
      if (err != nullptr && *reinterpret_cast<const volatile int*>(err) != 0) return false;
    }
  }
}

// ----------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* m, uint32_t bar,
                                            int c0, int c1, int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_store_4d(const CUtensorMap* m, uint32_t src, int c0, int c1,
                                             int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
          reinterpret_cast<uint64_t>(m)),
      "r"(src), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// The shared-memory source of every committed bulk store has been read (the slot is reusable).
__device__ __forceinline__ void bulk_wait_read() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// Warpgroup register re-balancing (all four warps of a warpgroup execute the same one).
template <int N>
__device__ __forceinline__ void reg_alloc() {
  asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}
template <int N>
__device__ __forceinline__ void reg_dealloc() {
  asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// ------------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// D[tmem] (+)= A[smem] * B[smem]
__device__ __forceinline__ void mma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]
__device__ __forceinline__ void mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                       uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive once on `bar` when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   bar)
               : "memory");
}

#define FA2_R8(i) "=r"(r[i]), "=r"(r[i + 1]), "=r"(r[i + 2]), "=r"(r[i + 3]), "=r"(r[i + 4]), \
                  "=r"(r[i + 5]), "=r"(r[i + 6]), "=r"(r[i + 7])
#define FA2_S8(i) "r"(r[i]), "r"(r[i + 1]), "r"(r[i + 2]), "r"(r[i + 3]), "r"(r[i + 4]), \
                  "r"(r[i + 5]), "r"(r[i + 6]), "r"(r[i + 7])

// 32 lanes x 32 consecutive 32-bit columns: this thread gets its lane's 32 columns.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : FA2_R8(0), FA2_R8(8), FA2_R8(16), FA2_R8(24)
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : FA2_R8(0), FA2_R8(8)
      : "r"(taddr));
}

// 64 or 128 consecutive 32-bit columns in one instruction, into 32-column register chunks.
#define FA2_RA8(a, i) "=r"(a[i]), "=r"(a[i + 1]), "=r"(a[i + 2]), "=r"(a[i + 3]), "=r"(a[i + 4]), \
                      "=r"(a[i + 5]), "=r"(a[i + 6]), "=r"(a[i + 7])
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, uint32_t (&a0)[32], uint32_t (&a1)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%64];"
      : FA2_RA8(a0, 0), FA2_RA8(a0, 8), FA2_RA8(a0, 16), FA2_RA8(a0, 24), FA2_RA8(a1, 0), FA2_RA8(a1, 8), FA2_RA8(a1, 16), FA2_RA8(a1, 24)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, uint32_t (&a0)[32], uint32_t (&a1)[32], uint32_t (&a2)[32], uint32_t (&a3)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x128.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63,%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95,%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%128];"
      : FA2_RA8(a0, 0), FA2_RA8(a0, 8), FA2_RA8(a0, 16), FA2_RA8(a0, 24), FA2_RA8(a1, 0), FA2_RA8(a1, 8), FA2_RA8(a1, 16), FA2_RA8(a1, 24), FA2_RA8(a2, 0), FA2_RA8(a2, 8), FA2_RA8(a2, 16), FA2_RA8(a2, 24), FA2_RA8(a3, 0), FA2_RA8(a3, 8), FA2_RA8(a3, 16), FA2_RA8(a3, 24)
      : "r"(taddr));
}
#undef FA2_RA8

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      FA2_S8(0), FA2_S8(8)
      : "memory");
}

// One 32-bit column of this warp's 32 lanes: store, and load followed by its wait (one asm
// statement, so no use of the value can be scheduled above the wait).
__device__ __forceinline__ void tmem_st1(uint32_t taddr, uint32_t v) {
  asm volatile("tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};" ::"r"(taddr), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t tmem_ld1_wait(uint32_t taddr) {
  uint32_t v;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v)
      : "r"(taddr)
      : "memory");
  return v;
}

// tcgen05.ld writes its destination registers asynchronously; they are valid only after
// tcgen05.wait::ld. This empty asm "redefines" the registers after the wait so the
// compiler cannot schedule any use of them above it.
#define FA2_W8(i) "+r"(r[i]), "+r"(r[i + 1]), "+r"(r[i + 2]), "+r"(r[i + 3]), "+r"(r[i + 4]), \
                  "+r"(r[i + 5]), "+r"(r[i + 6]), "+r"(r[i + 7])
__device__ __forceinline__ void reg_fence32(uint32_t (&r)[32]) {
  asm volatile("" : FA2_W8(0), FA2_W8(8), FA2_W8(16), FA2_W8(24) : : "memory");
}
__device__ __forceinline__ void reg_fence16(uint32_t (&r)[16]) {
  asm volatile("" : FA2_W8(0), FA2_W8(8) : : "memory");
}
#undef FA2_W8

#undef FA2_R8
#undef FA2_S8

// ------------------------------------------------------------- descriptors
// UMMA shared-memory matrix descriptor, 128-byte swizzle (layout type 2), sm100 version 1.
// Byte offsets are encoded >> 4. For K-major operands `sbo` is the stride between 8-row
// groups and `lbo` is unused (1); for MN-major operands `lbo` is the stride between
// 64-element MN chunks and `sbo` the stride between 8-row K groups.
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;  // descriptor version for sm100
  d |= static_cast<uint64_t>(2) << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::f16 with FP32 accumulation.
__host__ __device__ constexpr uint32_t idesc_f16(bool bf16, int M, int N, bool b_mn_major) {
  return (1u << 4)                                // D format: F32
         | ((bf16 ? 1u : 0u) << 7)                // A format: F16 = 0, BF16 = 1
         | ((bf16 ? 1u : 0u) << 10)               // B format
         | (0u << 15)                             // A is K-major
         | ((b_mn_major ? 1u : 0u) << 16)         // B major
         | (static_cast<uint32_t>(N >> 3) << 17)  // N / 8
         | (static_cast<uint32_t>(M >> 4) << 24); // M / 16
}

// ------------------------------------------------------------- f32 helpers
__device__ __forceinline__ uint64_t f2_pack(float a, float b) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
  return r;
}
__device__ __forceinline__ void f2_unpack(uint64_t v, float& a, float& b) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
// Hardware MUFU base-2 exponential (PTX ex2.approx), the instruction the reference's
// tl.math.exp2 lowers to.
__device__ __forceinline__ float ex2_mufu(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}

template <bool BF16>
__device__ __forceinline__ uint32_t cvt_pack2(float lo, float hi) {
  uint32_t r;
  if constexpr (BF16) {
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  } else {
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  }
  return r;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.b32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d)
               : "memory");
}


}  // namespace fa2
