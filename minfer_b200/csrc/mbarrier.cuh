// mbarrier and 1-D bulk-copy helpers shared by the TMA-fed kernels
// (decode GEMV, batched-prefill GEMM and attention).
#pragma once

#include "mf_common.cuh"

namespace mf {

MF_DEVICE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

MF_DEVICE void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
MF_DEVICE void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
MF_DEVICE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Wait for the phase of `parity` to complete, until `deadline` (and at most
// 2^26 polls). Returns false, and sets `failed`, when it gives up; a caller
// that already failed does not wait again.
MF_DEVICE bool mbar_wait(uint64_t* bar, uint32_t parity, unsigned long long deadline, bool& failed) {
    if (failed) return false;
    for (long long i = 0; i < (1ll << 26); ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 15) == 15 && globaltimer_ns() > deadline) break;
    }
    failed = true;
    return false;
}

MF_DEVICE void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// 1-D bulk copy global -> shared (no multicast): `bytes` (a multiple of 16)
// from a 16-byte aligned source, completing on `bar` (complete_tx).
MF_DEVICE void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                     smem_u32(dst)),
                 "l"(src), "r"(bytes), "r"(smem_u32(bar))
                 : "memory");
}

}  // namespace mf
