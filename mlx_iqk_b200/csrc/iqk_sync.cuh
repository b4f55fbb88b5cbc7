// Device primitives shared by the tensor-memory kernels: shared-memory
// addressing, bounded mbarrier waits, TMA / bulk copies, and the tcgen05
// (5th-generation tensor core + tensor memory) instructions, as inline PTX
// (PTX ISA 8.6+: mbarrier, cp.async.bulk.tensor, tcgen05.*).
#pragma once

#include <cuda.h>
#include <stdint.h>

namespace iqk {
namespace dev {

constexpr unsigned long long kWaitNs = 2000000000ull;  // every wait gives up after 2 s

__device__ __forceinline__ uint32_t saddr(const void *p) {
    return (uint32_t)__cvta_generic_to_shared(p);
}
__device__ __forceinline__ unsigned long long now_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;\n" : "=l"(t));
    return t;
}

// ---- mbarrier
__device__ __forceinline__ void bar_init(uint64_t *b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;\n" ::"r"(saddr(b)), "r"(count) : "memory");
}
__device__ __forceinline__ void bar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory");
}
__device__ __forceinline__ void bar_expect_tx(uint64_t *b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;\n" ::"r"(saddr(b)),
                 "r"(bytes) : "memory");
}
__device__ __forceinline__ void bar_arrive(uint64_t *b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];\n" ::"r"(saddr(b)) : "memory");
}
__device__ __forceinline__ bool bar_test(uint64_t *b, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(saddr(b)), "r"(parity) : "memory");
    return ok != 0;
}
// Like bar_test, but the thread may sleep in hardware (up to `hint_ns`) until
// the phase completes, instead of spinning and taking issue slots from the
// warps that do the work.
__device__ __forceinline__ bool bar_test_sleep(uint64_t *b, uint32_t parity, uint32_t hint_ns) {
    uint32_t ok;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
        " selp.u32 %0, 1, 0, p;\n}\n"
        : "=r"(ok) : "r"(saddr(b)), "r"(parity), "r"(hint_ns) : "memory");
    return ok != 0;
}
// Wait for the phase with the given parity. Gives up (returns false) after
// kWaitNs, or -- when `abort` is not null -- as soon as *abort is set by
// another warp that gave up. Drains of copies in flight pass null.
__device__ __forceinline__ bool bar_wait(uint64_t *b, uint32_t parity, volatile int *abort) {
    if (bar_test(b, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!bar_test_sleep(b, parity, 20000u)) {
        if (abort && *abort) return false;
        if (now_ns() - t0 > kWaitNs) return false;
    }
    return true;
}

// One lane of a converged warp (elect.sync); the others get false.
__device__ __forceinline__ bool elect_one() {
    uint32_t pred = 0;
    asm volatile("{\n .reg .pred P;\n elect.sync _|P, 0xffffffff;\n selp.b32 %0, 1, 0, P;\n}\n"
                 : "=r"(pred));
    return pred != 0;
}

// bar_wait without the hardware sleep: for warps whose lanes must stay
// converged (the MMA issuers).
__device__ __forceinline__ bool bar_wait_spin(uint64_t *b, uint32_t parity, volatile int *abort) {
    if (bar_test(b, parity)) return true;
    const unsigned long long t0 = now_ns();
    while (!bar_test(b, parity)) {
        if (abort && *abort) return false;
        if (now_ns() - t0 > kWaitNs) return false;
    }
    return true;
}

// ---- TMA (no multicast anywhere)
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap *map, int x, int y,
                                       uint64_t *b) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(dst),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(saddr(b))
        : "memory");
}

// ---- tensor memory
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t cols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;\n"
                 ::"r"(saddr(dst_smem)), "r"(cols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(cols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;\n" ::: "memory");
}
__device__ __forceinline__ void tc_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tc_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory");
}
// Arrive once on `b` when every tcgen05.mma this thread issued so far is done.
__device__ __forceinline__ void tc_commit(uint64_t *b) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(
            saddr(b))
        : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T, kind::f16 (A and B both f16), f32 accumulate.
__device__ __forceinline__ void tc_mma_ts(uint32_t d, uint32_t a, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d),
        "r"(a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// 32 lanes x 32-bit, 32 consecutive columns per thread (its own lane).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,"
        "%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// 32 lanes x 32-bit, 8 consecutive columns per thread (its own lane).
__device__ __forceinline__ void tmem_st8(uint32_t taddr, const uint32_t (&r)[8]) {
    asm volatile("tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};\n" ::"r"(
                     taddr),
                 "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]),
                 "r"(r[7])
                 : "memory");
}
// 32 lanes x 32-bit, 8 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld8(uint32_t taddr, uint32_t (&r)[8]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];\n"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7])
                 : "r"(taddr)
                 : "memory");
}

// Shared-memory matrix descriptor of a K-major operand tile stored in the
// 128-byte swizzle layout (rows of 128 B, 8-row groups of 1024 B):
// start address and strides in 16-byte units, version 1, layout 2 (SW128).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t smem_addr) {
    return (uint64_t)((smem_addr >> 4) & 0x3FFFu) | ((uint64_t)1u << 16) /* LBO: 16 B */ |
           ((uint64_t)(1024u >> 4) << 32) /* SBO: 8 rows */ | ((uint64_t)1u << 46) |
           ((uint64_t)2u << 61);
}

// Instruction descriptor, kind::f16: f32 accumulator, f16 A and B, both
// K-major, shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int m, int n) {
    return (1u << 4) | (0u << 7) | (0u << 10) | ((uint32_t)(n >> 3) << 17) |
           ((uint32_t)(m >> 4) << 24);
}

}  // namespace dev
}  // namespace iqk
