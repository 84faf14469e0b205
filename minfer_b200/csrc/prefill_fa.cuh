// Causal prefill attention on the 5th-generation tensor cores (tcgen05).
//
// Same result as prefill_attn_kernel (and the reference's per-token softmax
// attention, src/ops/kernels.cpp:31-110): for query row (token t, head h) the
// softmax over cache positions [0, pos0 + t] of (q.k)/sqrt(128), weighted sum
// of V rows. Q, K and V are fp32; each product sums hi*hi + hi*lo + lo*hi of
// operands split into hi + lo halves:
//  * Q and K as fp16 hi + lo (22 mantissa bits, ~2^-22 relative): scores keep
//    near-fp32 accuracy, which matters because their error is absolute in the
//    exponent. Normalised, rotated q/k rows are bounded by 16 * max|norm
//    weight|; the split kernel flags values outside the fp16 range (status
//    bit 4) and the host keeps such models on the SIMT kernel.
//  * P and V as bf16 hi + lo (~2^-17 relative; V has no range bound).
//
// CTA = 128 query rows (QT tokens x G query heads of one KV head) x one KV
// head; 192 threads:
//  * warp 0, one lane: TMA producer. Q hi/lo once (2 x 32 KB), then per 64-key
//    tile the K hi/lo tile and the V^T hi/lo tile (both double-buffered), all
//    with 128-byte swizzle; OOB rows (past the keys this call may see) read zero.
//  * warp 1: TMEM owner; one lane issues S = Q K^T (M128 N64 K16, 24 MMAs per
//    tile) into TMEM columns [0, 64) and O += P V (M128 N128 K16, 12 MMAs per
//    tile) into columns [128, 256), committing to mbarriers.
//  * warps 2-5: one thread per query row (its TMEM lane). Per tile: read the
//    row's 64 scores from TMEM, causal mask, online softmax in registers,
//    write P hi/lo into the swizzled shared-memory tile of the next MMA,
//    rescale the row of O in TMEM when the running max grew by more than 2^8
//    (base-2 softmax; a stale max changes rounding only). At the end,
//    O / l is written as the O projection's bf16 hi/lo operands.
// Every wait is bounded by a wall-clock deadline; on expiry the kernel records
// it (status bit 2), stops issuing, waits (bounded) for its copies in flight,
// frees its TMEM and returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attention.cuh"
#include "prefill_gemm.cuh"

namespace mf {

constexpr int FA_BM = 128;  // query rows per CTA
constexpr int FA_BN = 64;   // keys per tile
constexpr int FA_THREADS = 192;
constexpr int FA_TMEM_COLS = 256;
constexpr int FA_TMEM_O = 128;  // first TMEM column of O
// shared-memory layout (each matrix K-major, 128-byte swizzle, 128-byte rows)
constexpr int FA_Q_ATOM = FA_BM * 128;         // 128 rows x 64 dims (16 KB)
constexpr int FA_K_ATOM = FA_BN * 128;         // 64 rows x 64 dims (8 KB)
constexpr int FA_V_TILE = ATT_D * 128;         // 128 rows (dims) x 64 keys (16 KB)
constexpr int FA_P_TILE = FA_BM * 128;         // 128 rows x 64 keys (16 KB)
constexpr int FA_OFF_QHI = 0, FA_OFF_QLO = 2 * FA_Q_ATOM;                // 32 KB each
constexpr int FA_OFF_K = 4 * FA_Q_ATOM;                                  // 2 stages x (hi, lo) x 2 atoms
constexpr int FA_K_STAGE = 4 * FA_K_ATOM;                                // 32 KB
constexpr int FA_OFF_V = FA_OFF_K + 2 * FA_K_STAGE;                      // 2 stages x V^T (hi, lo)
constexpr int FA_V_STAGE = 2 * FA_V_TILE;                                // 32 KB
constexpr int FA_OFF_P = FA_OFF_V + 2 * FA_V_STAGE;                      // P hi, lo
constexpr int FA_SMEM_BYTES = FA_OFF_P + 2 * FA_P_TILE + 1024;           // + alignment slack
static_assert(FA_SMEM_BYTES + 256 <= 227 * 1024, "shared memory of one CTA (dynamic + barriers)");

// kind::f16 instruction descriptor: bf16 x bf16 -> f32, both K-major, M x N.
// kind::f16 instruction descriptor: A and B both bf16 (bf16 = true) or both
// fp16, f32 accumulator, both K-major, M x N.
constexpr uint32_t fa_idesc(int M, int N, bool bf16) {
    const uint32_t ab = bf16 ? 1u : 0u;
    return (1u << 4) | (ab << 7) | (ab << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

MF_DEVICE void tma_load_3d(void* dst, const CUtensorMap* tm, uint64_t* bar, int x, int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}
MF_DEVICE void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
MF_DEVICE void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

struct FaParams {
    int P;              // prompt tokens of this call
    int pos0;           // position of token 0
    int n_heads;        // query heads (Hq)
    int n_keys_max;     // keys the tensor maps cover (pos0 + P)
    __nv_bfloat16* out_hi;  // [P][Hq * 128]
    __nv_bfloat16* out_lo;
    int* status;        // bit 2: a wait gave up
    unsigned long long timeout_ns;
};

// Q maps: 2-D over [Hkv * P * G rows][128] (row = kvh*P*G + t*G + g), box {64, 128}.
// K maps: 3-D [Hkv][keys][128], box {64, 64, 1}. V^T maps: 3-D [Hkv][128][keys], box {64, 128, 1}.
template <int G>
__global__ void __launch_bounds__(FA_THREADS, 1)
    prefill_fa_kernel(const __grid_constant__ CUtensorMap tq_hi, const __grid_constant__ CUtensorMap tq_lo,
                      const __grid_constant__ CUtensorMap tk_hi, const __grid_constant__ CUtensorMap tk_lo,
                      const __grid_constant__ CUtensorMap tv_hi, const __grid_constant__ CUtensorMap tv_lo,
                      const FaParams p) {
    constexpr int QT = FA_BM / G;  // tokens per CTA
    extern __shared__ uint8_t fa_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t q_full, k_full[2], k_free[2], v_full[2], v_free[2], s_full, s_free, p_full,
        o_done, drain;
    __shared__ uint32_t tmem_base_s;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int n_qt = (p.P + QT - 1) / QT;
    const int qt = n_qt - 1 - (int)blockIdx.x;  // the latest tokens (most keys) first
    const int kvh = blockIdx.y;
    const int t0 = qt * QT;
    const int t_last = min(t0 + QT, p.P) - 1;
    const int n_keys = p.pos0 + t_last + 1;
    const int nt = (n_keys + FA_BN - 1) / FA_BN;

    if (threadIdx.x == 0) {
        mbar_init(&q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_free[s], 1);
            mbar_init(&v_full[s], 1);
            mbar_init(&v_free[s], 1);
        }
        mbar_init(&s_full, 1);
        mbar_init(&s_free, 128);
        mbar_init(&p_full, 128);
        mbar_init(&o_done, 1);
        mbar_init(&drain, 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&tmem_base_s)),
                     "r"(FA_TMEM_COLS)
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
    const int qrow0 = kvh * p.P * G + t0 * G;  // first Q row of this CTA

    if (warp == 0) {
        if (lane == 0) {
            mbar_expect_tx(&q_full, 4 * FA_Q_ATOM);
            tma_load_2d(smem + FA_OFF_QHI, &tq_hi, &q_full, 0, qrow0);
            tma_load_2d(smem + FA_OFF_QHI + FA_Q_ATOM, &tq_hi, &q_full, 64, qrow0);
            tma_load_2d(smem + FA_OFF_QLO, &tq_lo, &q_full, 0, qrow0);
            tma_load_2d(smem + FA_OFF_QLO + FA_Q_ATOM, &tq_lo, &q_full, 64, qrow0);
            int k_issued = 0, v_issued = 0;
            for (int j = 0; j < nt; ++j) {
                const int s = j & 1;
                if (j >= 2 && !mbar_wait(&k_free[s], ((uint32_t)(j >> 1) & 1u) ^ 1u, deadline, failed)) break;
                uint8_t* kb = smem + FA_OFF_K + s * FA_K_STAGE;
                mbar_expect_tx(&k_full[s], FA_K_STAGE);
                tma_load_3d(kb, &tk_hi, &k_full[s], 0, j * FA_BN, kvh);
                tma_load_3d(kb + FA_K_ATOM, &tk_hi, &k_full[s], 64, j * FA_BN, kvh);
                tma_load_3d(kb + 2 * FA_K_ATOM, &tk_lo, &k_full[s], 0, j * FA_BN, kvh);
                tma_load_3d(kb + 3 * FA_K_ATOM, &tk_lo, &k_full[s], 64, j * FA_BN, kvh);
                k_issued = j + 1;
                if (j >= 2 && !mbar_wait(&v_free[s], ((uint32_t)(j >> 1) & 1u) ^ 1u, deadline, failed)) break;
                uint8_t* vb = smem + FA_OFF_V + s * FA_V_STAGE;
                mbar_expect_tx(&v_full[s], FA_V_STAGE);
                tma_load_3d(vb, &tv_hi, &v_full[s], j * FA_BN, 0, kvh);
                tma_load_3d(vb + FA_V_TILE, &tv_lo, &v_full[s], j * FA_BN, 0, kvh);
                v_issued = j + 1;
            }
            if (failed) {
                // let this thread's copies land before shared memory goes away
                bool f2 = false;
                const unsigned long long d2 = globaltimer_ns() + p.timeout_ns;
                mbar_wait(&q_full, 0, d2, f2);
                for (int j = max(0, k_issued - 2); j < k_issued; ++j)
                    mbar_wait(&k_full[j & 1], (uint32_t)(j >> 1) & 1u, d2, f2);
                for (int j = max(0, v_issued - 2); j < v_issued; ++j)
                    mbar_wait(&v_full[j & 1], (uint32_t)(j >> 1) & 1u, d2, f2);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = fa_idesc(FA_BM, FA_BN, false);  // Q, K: fp16 hi/lo
            constexpr uint32_t idesc_o = fa_idesc(FA_BM, ATT_D, true);   // P, V: bf16 hi/lo
            const uint32_t qhi = smem_u32(smem + FA_OFF_QHI), qlo = smem_u32(smem + FA_OFF_QLO);
            const uint32_t phi = smem_u32(smem + FA_OFF_P), plo = phi + FA_P_TILE;
            auto issue_s = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(&k_full[s], (uint32_t)(j >> 1) & 1u, deadline, failed)) return false;
                if (j >= 1 && !mbar_wait(&s_free, (uint32_t)(j - 1) & 1u, deadline, failed)) return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(smem + FA_OFF_K + s * FA_K_STAGE);
#pragma unroll
                for (int ks = 0; ks < ATT_D / 16; ++ks) {
                    const uint32_t off = (uint32_t)(ks & 3) * 32;  // 16 dims = 32 bytes inside a 64-dim atom
                    const uint32_t qa = (uint32_t)(ks >> 2) * FA_Q_ATOM + off;
                    const uint32_t ka = (uint32_t)(ks >> 2) * FA_K_ATOM + off;
                    const uint64_t dkh = sw128_kmajor_desc(kb + ka), dkl = sw128_kmajor_desc(kb + 2 * FA_K_ATOM + ka);
                    umma_bf16(tmem, sw128_kmajor_desc(qhi + qa), dkh, idesc_s, ks > 0 ? 1u : 0u);
                    umma_bf16(tmem, sw128_kmajor_desc(qhi + qa), dkl, idesc_s, 1u);
                    umma_bf16(tmem, sw128_kmajor_desc(qlo + qa), dkh, idesc_s, 1u);
                }
                umma_commit(&k_free[s]);  // the K stage may be refilled once these MMAs read it
                umma_commit(&s_full);     // the scores are in TMEM
                return true;
            };
            if (mbar_wait(&q_full, 0, deadline, failed) && nt > 0) issue_s(0);
            for (int j = 0; j < nt && !failed; ++j) {
                if (j + 1 < nt && !issue_s(j + 1)) break;
                if (!mbar_wait(&p_full, (uint32_t)j & 1u, deadline, failed)) break;
                if (!mbar_wait(&v_full[j & 1], (uint32_t)(j >> 1) & 1u, deadline, failed)) break;
                tc_fence_after();
                const uint32_t vhi = smem_u32(smem + FA_OFF_V + (j & 1) * FA_V_STAGE), vlo = vhi + FA_V_TILE;
#pragma unroll
                for (int ks = 0; ks < FA_BN / 16; ++ks) {
                    const uint32_t off = (uint32_t)ks * 32;
                    const uint64_t dvh = sw128_kmajor_desc(vhi + off), dvl = sw128_kmajor_desc(vlo + off);
                    umma_bf16(tmem + FA_TMEM_O, sw128_kmajor_desc(phi + off), dvh, idesc_o, (j > 0 || ks > 0) ? 1u : 0u);
                    umma_bf16(tmem + FA_TMEM_O, sw128_kmajor_desc(phi + off), dvl, idesc_o, 1u);
                    umma_bf16(tmem + FA_TMEM_O, sw128_kmajor_desc(plo + off), dvh, idesc_o, 1u);
                }
                umma_commit(&v_free[j & 1]);  // the V^T stage and P may be rewritten once these MMAs read them
                umma_commit(&o_done);
            }
            if (failed) {
                // the MMAs already issued finish before TMEM is freed
                umma_commit(&drain);
                bool f2 = false;
                mbar_wait(&drain, 0, globaltimer_ns() + p.timeout_ns, f2);
            }
        }
    } else {
        // softmax warps: warp w owns TMEM lanes [32*(w%4), 32*(w%4) + 32): row r
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;
        const uint32_t lane_base = (uint32_t)(q4 * 32) << 16;
        const int my_pos = p.pos0 + t0 + r / G;
        const int cta_pos = p.pos0 + t0;  // smallest position among the CTA's rows
        // softmax in base 2: exp(x * scale) = 2^(x * scale * log2(e)); scale = 1/sqrt(128) (src/ops/kernels.cpp:88)
        const float c2 = (1.0f / sqrtf((float)ATT_D)) * 1.4426950408889634f;
        float m = -INFINITY, l = 0.f;
        uint8_t* phi = smem + FA_OFF_P;
        uint8_t* plo = phi + FA_P_TILE;
        for (int j = 0; j < nt; ++j) {
            mbar_wait(&s_full, (uint32_t)j & 1u, deadline, failed);
            tc_fence_after();
            uint32_t sr[64];
            tmem_ld32(tmem + lane_base + 0, *reinterpret_cast<uint32_t(*)[32]>(sr));
            tmem_ld32(tmem + lane_base + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
            tc_fence_before();
            mbar_arrive(&s_free);
            // scaled, causally masked scores (tiles below the CTA's first position need no mask)
            float sv[64];
            float mx = -INFINITY;
            if ((j + 1) * FA_BN - 1 <= cta_pos) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sv[c] = __uint_as_float(sr[c]) * c2;
                    mx = fmaxf(mx, sv[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sv[c] = (j * FA_BN + c <= my_pos) ? __uint_as_float(sr[c]) * c2 : -INFINITY;
                    mx = fmaxf(mx, sv[c]);
                }
            }
            // The running max m moves only when the tile's max exceeds it by more than 8 (a factor
            // 2^8): softmax is shift-invariant and O and l share m, so a stale m changes rounding
            // only (p <= 2^8), and O is rescaled rarely. Key 0 (tile 0) is visible to every row,
            // so the first tile sets a finite m and alpha = 2^-inf = 0.
            const bool bump = mx > m + 8.f;
            const float mu = bump ? mx : m;
            const float alpha = exp2f(m - mu);
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                sv[c] = exp2f(sv[c] - mu);
                s4[c & 3] += sv[c];
            }
            l = fmaf(l, alpha, (s4[0] + s4[1]) + (s4[2] + s4[3]));
            m = mu;
            // PV of the previous tile is done: the P tile is free and O is stable
            if (j >= 1) mbar_wait(&o_done, (uint32_t)(j - 1) & 1u, deadline, failed);
            tc_fence_after();
            // P hi/lo row r into the 128-byte-swizzled K-major tile (chunk c of 8 keys at c ^ (r % 8))
#pragma unroll
            for (int c = 0; c < 8; ++c) {
                uint4 hw, lw;
                uint32_t* hp = &hw.x;
                uint32_t* lp = &lw.x;
#pragma unroll
                for (int e = 0; e < 4; ++e) {
                    const float a0 = sv[8 * c + 2 * e], a1 = sv[8 * c + 2 * e + 1];
                    const __nv_bfloat162 h2 = __floats2bfloat162_rn(a0, a1);
                    const float2 hf = __bfloat1622float2(h2);
                    const __nv_bfloat162 l2 = __floats2bfloat162_rn(a0 - hf.x, a1 - hf.y);
                    hp[e] = *reinterpret_cast<const uint32_t*>(&h2);
                    lp[e] = *reinterpret_cast<const uint32_t*>(&l2);
                }
                const int off = r * 128 + ((c ^ (r & 7)) << 4);
                *reinterpret_cast<uint4*>(phi + off) = hw;
                *reinterpret_cast<uint4*>(plo + off) = lw;
            }
            // rescale this row of O when its running max moved (warp-collective TMEM access)
            if (j >= 1 && __any_sync(0xffffffffu, bump)) {
#pragma unroll 1
                for (int cc = 0; cc < ATT_D; cc += 32) {
                    uint32_t o[32];
                    tmem_ld32(tmem + lane_base + FA_TMEM_O + cc, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tmem_st32(tmem + lane_base + FA_TMEM_O + cc, o);
                }
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor core
            tc_fence_before();
            mbar_arrive(&p_full);
        }
        // final: O / l as the O projection's bf16 hi/lo operands
        if (nt > 0) mbar_wait(&o_done, (uint32_t)(nt - 1) & 1u, deadline, failed);
        tc_fence_after();
        const int t = t0 + r / G, g = r % G;
        const float inv = 1.0f / l;
#pragma unroll 1
        for (int cc = 0; cc < ATT_D; cc += 32) {
            uint32_t o[32];
            tmem_ld32(tmem + lane_base + FA_TMEM_O + cc, o);
            if (t < p.P && !failed) {
                const size_t base = ((size_t)t * p.n_heads + kvh * G + g) * ATT_D + cc;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    __align__(16) __nv_bfloat16 h[8], lo8[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) split_bf16(__uint_as_float(o[e + u]) * inv, h[u], lo8[u]);
                    *reinterpret_cast<uint4*>(p.out_hi + base + e) = *reinterpret_cast<const uint4*>(h);
                    *reinterpret_cast<uint4*>(p.out_lo + base + e) = *reinterpret_cast<const uint4*>(lo8);
                }
            }
        }
    }
    if (failed) atomicOr(p.status, 2);
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(FA_TMEM_COLS) : "memory");
    }
}

// Operand preparation for prefill_fa_kernel, one warp per 128-float row:
//  * Q [P][Hq][128] fp32 -> fp16 hi/lo [Hkv][P * G][128] (row t*G + g of KV head h/G)
//  * K cache rows [0, n_keys) of [Hkv][max_seq][128] -> fp16 hi/lo [Hkv][ld][128]
// A value outside the fp16 range (or not finite) sets status bit 4.
MF_DEVICE void split_f16(float v, __half& hi, __half& lo, bool& bad) {
    bad |= !(fabsf(v) < 65504.f);
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}

__global__ void __launch_bounds__(256) fa_qk_split_kernel(const float* __restrict__ q, const float* __restrict__ k_cache,
                                                          int P, int Hq, int Hkv, int max_seq, int n_keys, int ld,
                                                          __half* qh, __half* ql, __half* kh, __half* kl,
                                                          int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const int G = Hq / Hkv;
    const long long nq = (long long)P * Hq, rows = nq + (long long)Hkv * n_keys;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    bool bad = false;
    for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < rows; w += warps) {
        const float* src;
        size_t dst;
        if (w < nq) {
            const int t = (int)(w / Hq), h = (int)(w % Hq);
            src = q + (size_t)w * ATT_D;
            dst = (((size_t)(h / G) * P + t) * G + (h % G)) * ATT_D;
        } else {
            const long long j = w - nq;
            const int h = (int)(j / n_keys), key = (int)(j % n_keys);
            src = k_cache + ((size_t)h * max_seq + key) * ATT_D;
            dst = ((size_t)h * ld + key) * ATT_D;
        }
        const float4 v = reinterpret_cast<const float4*>(src)[lane];
        __align__(8) __half h4[4], l4[4];
        split_f16(v.x, h4[0], l4[0], bad);
        split_f16(v.y, h4[1], l4[1], bad);
        split_f16(v.z, h4[2], l4[2], bad);
        split_f16(v.w, h4[3], l4[3], bad);
        __half* oh = w < nq ? qh : kh;
        __half* ol = w < nq ? ql : kl;
        *reinterpret_cast<uint2*>(oh + dst + 4 * lane) = *reinterpret_cast<const uint2*>(h4);
        *reinterpret_cast<uint2*>(ol + dst + 4 * lane) = *reinterpret_cast<const uint2*>(l4);
    }
    if (bad) atomicOr(status, 4);
}

// V cache rows [0, n_keys) of [Hkv][max_seq][128] -> V^T hi/lo [Hkv][128][ld]
// (tiles of 64 keys x 128 dims through shared memory; grid (ceil(n_keys/64), Hkv)).
__global__ void __launch_bounds__(256) fa_v_split_kernel(const float* __restrict__ v_cache, int max_seq, int n_keys,
                                                         int ld, __nv_bfloat16* vh, __nv_bfloat16* vl) {
    __shared__ float tile[64][ATT_D + 1];
    pdl_launch_dependents();
    pdl_wait();
    const int k0 = blockIdx.x * 64, h = blockIdx.y;
    for (int i = threadIdx.x; i < 64 * ATT_D; i += blockDim.x) {
        const int kk = i / ATT_D, d = i % ATT_D;
        tile[kk][d] = (k0 + kk < n_keys) ? v_cache[((size_t)h * max_seq + k0 + kk) * ATT_D + d] : 0.f;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < 64 * ATT_D; i += blockDim.x) {
        const int d = i / 64, kk = i % 64;
        if (k0 + kk < n_keys) {
            const size_t o = ((size_t)h * ATT_D + d) * ld + k0 + kk;
            split_bf16(tile[kk][d], vh[o], vl[o]);
        }
    }
}

}  // namespace mf
