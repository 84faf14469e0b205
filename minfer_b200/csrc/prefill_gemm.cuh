// Batched-prefill GEMM on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).
//
//   C[M, N] = A[M, K] · W[N, K]^T     (A: activations of M prompt tokens,
//                                      W: a projection weight, row-major)
//
// The reference has no batched prefill: it runs the prompt as M sequential
// decode steps (src/base/model.cpp:120-129), each an fp32-activation GEMV
// over bf16 weights widened to fp32 (src/ops/kernels.cpp:297-343). To keep
// that numeric contract on bf16 tensor cores the fp32 activation is split
// into two bf16 terms, a = hi + lo with hi = bf16(a), lo = bf16(a - hi)
// (|a - hi - lo| <= 2^-16 |a|), and C = hi·W^T + lo·W^T is accumulated in
// fp32 in TMEM: the weights are exact in bf16, so the result matches the fp32
// GEMV to ~1e-5 relative instead of bf16's ~4e-3.
//
// One CTA computes one 128 x 256 output tile:
//  * warp 0 (one lane): TMA producer. Per 64-wide K block it loads the
//    A_hi, A_lo (128 x 64) and W (256 x 64) tiles with 128-byte swizzle into
//    a PG_STAGES-deep shared-memory ring, completion on a "full" mbarrier.
//  * warp 1: allocates 256 TMEM columns; one lane issues the MMAs
//    (tcgen05.mma kind::f16, M=128 N=256 K=16, bf16 x bf16 -> fp32, both
//    operands K-major from shared memory): 4 K-steps x (hi, lo) per block,
//    then tcgen05.commit to the stage's "empty" mbarrier; after the last
//    block a commit to the accumulator mbarrier.
//  * warps 2-5: epilogue. Each reads its 32 TMEM lanes (rows) 32 columns at
//    a time (tcgen05.ld 32x32b.x32) and applies the mode: store fp32, add to
//    a residual, or SwiGLU on interleaved gate/up columns written back as
//    the next GEMM's bf16 hi/lo operands.
// Every mbarrier wait is bounded by a wall-clock deadline; on expiry the
// kernel records an error, stops issuing, waits (bounded) for its own copies
// in flight, frees its TMEM and returns.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>

#include "mbarrier.cuh"
#include "mf_common.cuh"

namespace mf {

constexpr int PG_BM = 128, PG_BN = 256, PG_BK = 64;
constexpr int PG_STAGES = 3;
constexpr int PG_A_BYTES = PG_BM * PG_BK * 2;                 // 16 KB
constexpr int PG_B_BYTES = PG_BN * PG_BK * 2;                 // 32 KB
constexpr int PG_STAGE_BYTES = 2 * PG_A_BYTES + PG_B_BYTES;   // 64 KB
constexpr int PG_THREADS = 192;
constexpr int PG_TMEM_COLS = 256;
constexpr int PG_SMEM_BYTES = PG_STAGES * PG_STAGE_BYTES + 1024;  // + alignment slack

enum PgMode { PG_STORE = 0, PG_RESID = 1, PG_SWIGLU_SPLIT = 2 };

struct PgParams {
    int M, N, K;
    // grouped mode (MoE experts; grp_rows == nullptr: one plain GEMM): A holds
    // the rows of every group back to back, group g at rows [grp_rows[g],
    // grp_rows[g + 1]); W holds n_groups matrices of N rows each. CTA row
    // blockIdx.y is tile blockIdx.y - grp_tiles[g] of the group g with
    // grp_tiles[g] <= blockIdx.y < grp_tiles[g + 1] (the tables come from the
    // previous kernel); rows past the group's end are computed but not stored.
    const int* grp_rows;   // [n_groups + 1]
    const int* grp_tiles;  // [n_groups + 1]
    int n_groups;
    float* y;              // PG_STORE: y[m*ldy + n] = C; PG_RESID: y[m*ldy + n] += C
    int ldy;
    __nv_bfloat16* h_hi;   // PG_SWIGLU_SPLIT: h = silu(C[:, 2i]) * C[:, 2i+1] as hi/lo [M][N/2]
    __nv_bfloat16* h_lo;
    int* status;           // bit 1: a wait gave up
    unsigned long long timeout_ns;
};

// 2-D TMA tile load (no multicast) into shared memory, completing on `bar`.
// x (the inner, K coordinate) is always a multiple of 64 elements.
MF_DEVICE void tma_load_2d(void* dst, const CUtensorMap* tm, uint64_t* bar, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
            smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}

// Shared-memory matrix descriptor: K-major tile, 128-byte swizzle, rows of
// 128 bytes (64 bf16 of K) stacked contiguously, 8-row groups 1024 bytes apart.
MF_DEVICE uint64_t sw128_kmajor_desc(uint32_t saddr) {
    uint64_t d = 0;
    d |= (uint64_t)((saddr >> 4) & 0x3FFFu);        // start address (16-byte units)
    d |= (uint64_t)((1024u >> 4) & 0x3FFFu) << 32;  // stride byte offset: next 8-row group
    d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
    d |= (uint64_t)2 << 61;                         // layout: 128-byte swizzle
    return d;
}

// Instruction descriptor of tcgen05.mma kind::f16: bf16 A and B, fp32
// accumulator, both K-major, M = PG_BM, N = PG_BN.
constexpr uint32_t pg_idesc() {
    return (1u << 4)                        // accumulator format: f32
           | (1u << 7)                      // A: bf16
           | (1u << 10)                     // B: bf16
           | ((uint32_t)(PG_BN >> 3) << 17)  // N / 8
           | ((uint32_t)(PG_BM >> 4) << 24);  // M / 16
}

MF_DEVICE void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}
MF_DEVICE void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
MF_DEVICE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
MF_DEVICE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (lane = row).
MF_DEVICE void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// fp32 -> (hi, lo) bf16 with hi = bf16(v), lo = bf16(v - hi), both round-to-nearest-even.
MF_DEVICE void split_bf16(float v, __nv_bfloat16& hi, __nv_bfloat16& lo) {
    hi = __float2bfloat16_rn(v);
    lo = __float2bfloat16_rn(v - __bfloat162float(hi));
}

template <int MODE>
__global__ void __launch_bounds__(PG_THREADS, 1)
    prefill_gemm_kernel(const __grid_constant__ CUtensorMap tm_ahi, const __grid_constant__ CUtensorMap tm_alo,
                        const __grid_constant__ CUtensorMap tm_w, const PgParams p) {
    extern __shared__ uint8_t pg_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(pg_smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t full_bar[PG_STAGES], empty_bar[PG_STAGES], acc_bar;
    __shared__ uint32_t tmem_base_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n0 = blockIdx.x * PG_BN;
    int m0 = blockIdx.y * PG_BM, m_end = p.M, w_row0 = n0;
    if (p.grp_rows) {
        // the group tables are the previous kernel's output
        pdl_wait();
        const int y = blockIdx.y;
        if (y >= __ldcg(p.grp_tiles + p.n_groups)) return;  // past the last tile: the whole CTA leaves
        int lo = 0, hi = p.n_groups - 1;  // the group g with grp_tiles[g] <= y < grp_tiles[g + 1]
        while (lo < hi) {
            const int mid = (lo + hi + 1) >> 1;
            if (__ldcg(p.grp_tiles + mid) <= y) lo = mid;
            else hi = mid - 1;
        }
        m0 = __ldcg(p.grp_rows + lo) + (y - __ldcg(p.grp_tiles + lo)) * PG_BM;
        m_end = __ldcg(p.grp_rows + lo + 1);
        w_row0 = lo * p.N + n0;
    }
    const int KB = (p.K + PG_BK - 1) / PG_BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < PG_STAGES; ++s) {
            mbar_init(&full_bar[s], 1);
            mbar_init(&empty_bar[s], 1);
        }
        mbar_init(&acc_bar, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(PG_TMEM_COLS)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_base_s;

    pdl_launch_dependents();
    pdl_wait();
    const unsigned long long deadline = globaltimer_ns() + p.timeout_ns;
    bool failed = false;

    if (warp == 0) {
        if (lane == 0) {
            int issued = 0;
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % PG_STAGES;
                const uint32_t ph = (uint32_t)(kb / PG_STAGES) & 1u;
                // slot s is free once the MMAs of block kb - PG_STAGES completed
                if (kb >= PG_STAGES && !mbar_wait(&empty_bar[s], ph ^ 1u, deadline, failed)) break;
                uint8_t* st = smem + (size_t)s * PG_STAGE_BYTES;
                mbar_expect_tx(&full_bar[s], PG_STAGE_BYTES);
                tma_load_2d(st, &tm_ahi, &full_bar[s], kb * PG_BK, m0);
                tma_load_2d(st + PG_A_BYTES, &tm_alo, &full_bar[s], kb * PG_BK, m0);
                tma_load_2d(st + 2 * PG_A_BYTES, &tm_w, &full_bar[s], kb * PG_BK, w_row0);
                issued = kb + 1;
            }
            if (failed) {
                // let the copies this thread started land before shared memory goes away
                bool f2 = false;
                for (int kb = issued > PG_STAGES ? issued - PG_STAGES : 0; kb < issued; ++kb)
                    mbar_wait(&full_bar[kb % PG_STAGES], (uint32_t)(kb / PG_STAGES) & 1u,
                              globaltimer_ns() + p.timeout_ns, f2);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc = pg_idesc();
            for (int kb = 0; kb < KB; ++kb) {
                const int s = kb % PG_STAGES;
                const uint32_t ph = (uint32_t)(kb / PG_STAGES) & 1u;
                if (!mbar_wait(&full_bar[s], ph, deadline, failed)) break;
                tc_fence_after();
                const uint32_t a_hi = smem_u32(smem + (size_t)s * PG_STAGE_BYTES);
                const uint32_t a_lo = a_hi + PG_A_BYTES, b = a_hi + 2 * PG_A_BYTES;
#pragma unroll
                for (int k = 0; k < PG_BK / 16; ++k) {
                    const uint64_t db = sw128_kmajor_desc(b + k * 32);
                    umma_bf16(tmem, sw128_kmajor_desc(a_hi + k * 32), db, idesc, (kb > 0 || k > 0) ? 1u : 0u);
                    umma_bf16(tmem, sw128_kmajor_desc(a_lo + k * 32), db, idesc, 1u);
                }
                umma_commit(&empty_bar[s]);  // frees the slot when these MMAs have read it
            }
            umma_commit(&acc_bar);  // the accumulator is final once every MMA above completes
        }
    } else {
        // epilogue: warp w may access TMEM lanes [32*(w%4), 32*(w%4) + 32)
        const int q = warp & 3;
        mbar_wait(&acc_bar, 0, deadline, failed);
        tc_fence_after();
        const int row = m0 + q * 32 + lane;
#pragma unroll 1
        for (int c0 = 0; c0 < PG_BN; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)c0, r);
            const int col = n0 + c0;
            if (failed || row >= m_end || col >= p.N) continue;
            const bool full = col + 32 <= p.N;
            if (MODE == PG_SWIGLU_SPLIT) {
                // columns 2i / 2i+1 are gate_i / up_i (src/models/qwen3/module.cpp:466-468)
                const int F = p.N >> 1;
                __nv_bfloat16* hh = p.h_hi + (size_t)row * F + (col >> 1);
                __nv_bfloat16* hl = p.h_lo + (size_t)row * F + (col >> 1);
                if (full && (F & 7) == 0) {
                    // 16 outputs of this row: packed into two 16-byte stores per operand
                    // (col / 2 is a multiple of 16, so both are 16-byte aligned)
                    uint32_t ph[8], pl[8];
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        __nv_bfloat16 h0, l0, h1, l1;
                        split_bf16(silu(__uint_as_float(r[j])) * __uint_as_float(r[j + 1]), h0, l0);
                        split_bf16(silu(__uint_as_float(r[j + 2])) * __uint_as_float(r[j + 3]), h1, l1);
                        ph[j >> 2] = (uint32_t)__bfloat16_as_ushort(h0) | ((uint32_t)__bfloat16_as_ushort(h1) << 16);
                        pl[j >> 2] = (uint32_t)__bfloat16_as_ushort(l0) | ((uint32_t)__bfloat16_as_ushort(l1) << 16);
                    }
                    uint4* dh = reinterpret_cast<uint4*>(hh);
                    uint4* dl = reinterpret_cast<uint4*>(hl);
                    dh[0] = make_uint4(ph[0], ph[1], ph[2], ph[3]);
                    dh[1] = make_uint4(ph[4], ph[5], ph[6], ph[7]);
                    dl[0] = make_uint4(pl[0], pl[1], pl[2], pl[3]);
                    dl[1] = make_uint4(pl[4], pl[5], pl[6], pl[7]);
                } else {
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        if (!full && col + j + 1 >= p.N) break;
                        const float h = silu(__uint_as_float(r[j])) * __uint_as_float(r[j + 1]);
                        split_bf16(h, hh[j >> 1], hl[j >> 1]);
                    }
                }
            } else {
                float* yr = p.y + (size_t)row * p.ldy + col;
                if (full) {
#pragma unroll
                    for (int j = 0; j < 32; j += 4) {
                        float4 v = make_float4(__uint_as_float(r[j]), __uint_as_float(r[j + 1]),
                                               __uint_as_float(r[j + 2]), __uint_as_float(r[j + 3]));
                        if (MODE == PG_RESID) {
                            const float4 o = *reinterpret_cast<const float4*>(yr + j);
                            v.x += o.x;
                            v.y += o.y;
                            v.z += o.z;
                            v.w += o.w;
                        }
                        *reinterpret_cast<float4*>(yr + j) = v;
                    }
                } else {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (col + j < p.N) yr[j] = (MODE == PG_RESID ? yr[j] : 0.f) + __uint_as_float(r[j]);
                }
            }
        }
    }
    if (failed) atomicOr(p.status, 1);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(PG_TMEM_COLS) : "memory");
    }
}

}  // namespace mf
