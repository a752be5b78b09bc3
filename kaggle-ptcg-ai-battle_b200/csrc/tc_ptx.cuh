// Inline-PTX building blocks of the hand-written tcgen05 kernels: mbarriers
// with bounded waits, 2-D TMA loads (no multicast), tcgen05.mma with shared
// memory descriptors, commits, TMEM loads / stores and the UMMA descriptor
// formats.  Each kernel file includes it inside its own anonymous namespace
// use; nothing here allocates or launches.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "common.cuh"

namespace tcx {

constexpr long long WAIT_BUDGET = 4000000000LL;   // clock cycles (~2 s)

PTCG_DEV uint32_t saddr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
PTCG_DEV void bar_init(uint32_t b, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(b), "r"(count));
}
PTCG_DEV void bar_expect_tx(uint32_t b, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(b), "r"(bytes)
                 : "memory");
}
PTCG_DEV void bar_arrive(uint32_t b) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(b) : "memory");
}
PTCG_DEV bool bar_try(uint32_t b, uint32_t parity) {
    uint32_t ok;
    asm volatile("{\n\t.reg .pred P;\n\t"
                 "mbarrier.try_wait.parity.shared::cta.b64 P, [%1], %2;\n\t"
                 "selp.u32 %0, 1, 0, P;\n\t}"
                 : "=r"(ok) : "r"(b), "r"(parity) : "memory");
    return ok != 0;
}
// bounded wait; false once the CTA's abort flag is set (by this wait on
// expiry, which records `code` in *err, or by another role)
PTCG_DEV bool bar_wait(uint32_t b, uint32_t parity, volatile int* abort_flag, int* err, int code) {
    if (*abort_flag) return false;
    const long long t0 = clock64();
    while (!bar_try(b, parity)) {
        if (*abort_flag) return false;
        if (clock64() - t0 > WAIT_BUDGET) {
            *abort_flag = 1;
            atomicCAS(err, 0, code);
            return false;
        }
    }
    return true;
}
// wait for a barrier phase regardless of the abort flag, still bounded (the
// exit path: copies and MMAs already issued must land before the CTA leaves)
PTCG_DEV void bar_drain(uint32_t b, uint32_t parity) {
    const long long t0 = clock64();
    while (!bar_try(b, parity) && clock64() - t0 < WAIT_BUDGET) {}
}
PTCG_DEV void tma_2d(uint32_t dst, const CUtensorMap* map, uint32_t b, int x, int y) {
    asm volatile("cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
                 " [%0], [%1, {%3, %4}], [%2];"
                 :: "r"(dst), "l"((uint64_t)map), "r"(b), "r"(x), "r"(y) : "memory");
}
PTCG_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
PTCG_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
PTCG_DEV void mma_bf16(uint32_t d, uint64_t a, uint64_t b, uint32_t idesc, uint32_t acc) {
    asm volatile("{\n\t.reg .pred p;\n\t"
                 "setp.ne.b32 p, %4, 0;\n\t"
                 "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
                 :: "r"(d), "l"(a), "l"(b), "r"(idesc), "r"(acc) : "memory");
}
PTCG_DEV void mma_commit_to(uint32_t b) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 :: "r"(b) : "memory");
}
PTCG_DEV void tmem_ld32x32_x16(uint32_t taddr, float (&v)[16]) {
    uint32_t r[16];
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 "
                 "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]),
                   "=r"(r[6]), "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]),
                   "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
                 : "r"(taddr));
    #pragma unroll
    for (int i = 0; i < 16; i++) v[i] = __uint_as_float(r[i]);
}
PTCG_DEV void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// UMMA shared-memory descriptor (sm_100): start, leading / stride byte
// offsets, layout (2 = 128-byte swizzle, 4 = 64-byte swizzle)
PTCG_DEV uint64_t sdesc(uint32_t a, uint32_t lbo, uint32_t sbo, uint32_t layout) {
    uint64_t d = 0;
    d |= (uint64_t)((a >> 4) & 0x3FFF);
    d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
    d |= (uint64_t)((sbo >> 4) & 0x3FFF) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)layout << 61;
    return d;
}
// instruction descriptor, kind::f16: fp32 accumulate, bf16 A and B, A / B
// major-ness (1 = MN-major), N, M = 128
__host__ __device__ inline uint32_t idesc_bf16(int n, int a_mn, int b_mn) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)a_mn << 15) | ((uint32_t)b_mn << 16) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(128 >> 4) << 24);
}

}  // namespace tcx
