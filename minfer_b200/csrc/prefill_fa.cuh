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
//    weight|; values outside the fp16 range set status bit 4 and the host
//    keeps such models on the SIMT kernel.
//  * P and V as bf16 hi + lo (~2^-17 relative; V has no range bound).
//
// CTA = 128 query rows (QT tokens x G query heads of one KV head) x one KV
// head, 352 threads. The 64-key tiles alternate between two softmax groups:
// group g takes tiles j = g, g + 2, ... with its own running max, row sum and
// O accumulator, so the groups never wait on each other until the final
// merge (O = (O_0 2^(m_0 - m) + O_1 2^(m_1 - m)) / (l_0 2^(m_0 - m) + l_1 2^(m_1 - m))).
// TMEM (512 columns): S of group g at [64 g, 64 g + 64), O_g at
// [128 + 128 g, 256 + 128 g), Q hi/lo at [384, 512) (the A operand of
// Q K^T straight from TMEM: 16-bit elements packed two per 32-bit column,
// row = lane). Shared memory: K hi/lo and V^T hi/lo rings, and each group's
// P hi/lo tile (the A operand of P V).
//  * warps 0 and 10, one lane each: TMA producers of the K and of the V^T
//    tiles (128-byte swizzle; rows past the keys this call may see read zero).
//  * warp 1: TMEM owner; one lane issues S = Q K^T (M128 N64 K16, 24 MMAs per
//    tile) and O_g += P V (M128 N128 K16, 12 MMAs per tile).
//  * warps 2-5 (group 0) and 6-9 (group 1): one thread per query row (its
//    TMEM lane) in each group. Group 0 first puts the rows of Q (fp32 split to
//    fp16 hi/lo) into TMEM. Per tile: read the row's 64 scores, causal mask,
//    online softmax in registers (base 2; the running max moves only when it
//    grows by more than 2^8 - a stale max changes rounding only - and O_g is
//    rescaled then), P hi/lo into the group's swizzled tile. At the end the
//    groups merge and write O / l as the O projection's bf16 hi/lo operands.
// Every wait is bounded by a wall-clock deadline; on expiry the kernel records
// it (status bit 2), stops issuing, waits (bounded) for its copies and MMAs in
// flight, frees its TMEM and returns.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "attention.cuh"
#include "prefill_gemm.cuh"

namespace mf {

constexpr int FA_BM = 128;  // query rows per CTA
constexpr int FA_BN = 64;   // keys per tile
constexpr int FA_THREADS = 352;  // K producer, MMA, two softmax groups of 4 warps, V producer
constexpr int FA_STAGES = 2;     // depth of the K ring
constexpr int FA_VSTAGES = 3;    // depth of the V^T ring
constexpr int FA_TMEM_COLS = 512;
constexpr uint32_t FA_T_S = 0, FA_T_O = 128, FA_T_QH = 384, FA_T_QL = 448;
// shared-memory layout (each matrix K-major, 128-byte swizzle, 128-byte rows)
constexpr int FA_K_ATOM = FA_BN * 128;    // 64 keys x 64 dims (8 KB)
constexpr int FA_K_STAGE = 4 * FA_K_ATOM;  // hi d0-63, hi d64-127, lo d0-63, lo d64-127 (32 KB)
constexpr int FA_V_TILE = ATT_D * 128;     // 128 dims x 64 keys (16 KB)
constexpr int FA_V_STAGE = 2 * FA_V_TILE;  // hi, lo (32 KB)
constexpr int FA_P_TILE = FA_BM * 128;     // 128 rows x 64 keys (16 KB)
constexpr int FA_OFF_V = FA_STAGES * FA_K_STAGE;
constexpr int FA_OFF_P = FA_OFF_V + FA_VSTAGES * FA_V_STAGE;  // group g: hi at + 2 g P_TILE, lo after it
constexpr int FA_SMEM_BYTES = FA_OFF_P + 4 * FA_P_TILE + 1024;   // + alignment slack
static_assert(FA_SMEM_BYTES + 256 <= 227 * 1024, "shared memory of one CTA (dynamic + barriers)");

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
// D (TMEM) (+)= A (TMEM) * B (shared-memory descriptor); no output lane disabled.
MF_DEVICE void umma_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    const uint32_t z = 0;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, {%5, %5, %5, %5}, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(db), "r"(idesc), "r"(accumulate), "r"(z)
        : "memory");
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
}
MF_DEVICE void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// 32 columns of this warp's lanes without waiting (pair with tmem_wait_ld).
MF_DEVICE void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
}
MF_DEVICE void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
MF_DEVICE void named_bar_sync(int id, int n_threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n_threads) : "memory");
}
// 2^x by the hardware approximation (PTX ex2.approx.ftz.f32: relative error
// about 2^-22; 2^-inf = +0, results below 2^-126 flush to zero).
MF_DEVICE float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// fp32 -> fp16 hi + lo; `bad` records a value outside the fp16 range (or not finite).
MF_DEVICE void split_f16(float v, __half& hi, __half& lo, bool& bad) {
    bad |= !(fabsf(v) < 65504.f);
    hi = __float2half_rn(v);
    lo = __float2half_rn(v - __half2float(hi));
}
MF_DEVICE uint32_t pack_half2(__half a, __half b) {
    return (uint32_t)__half_as_ushort(a) | ((uint32_t)__half_as_ushort(b) << 16);
}

struct FaParams {
    const float* q;     // [P][Hq][128] (normed, rotated)
    int P;              // prompt tokens of this call
    int pos0;           // position of token 0
    int n_heads;        // query heads (Hq)
    __nv_bfloat16* out_hi;  // [P][Hq * 128]
    __nv_bfloat16* out_lo;
    int* status;        // bit 2: a wait gave up; bit 4: q outside the fp16 range
    unsigned long long timeout_ns;
};

// K maps: 3-D fp16 [Hkv][keys][128], box {64, 64, 1}. V^T maps: 3-D bf16 [Hkv][128][keys], box {64, 128, 1}.
template <int G>
__global__ void __launch_bounds__(FA_THREADS, 1)
    prefill_fa_kernel(const __grid_constant__ CUtensorMap tk_hi, const __grid_constant__ CUtensorMap tk_lo,
                      const __grid_constant__ CUtensorMap tv_hi, const __grid_constant__ CUtensorMap tv_lo,
                      const FaParams p) {
    constexpr int QT = FA_BM / G;  // tokens per CTA
    extern __shared__ uint8_t fa_smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(fa_smem_raw) + 1023) & ~(uintptr_t)1023);
    __shared__ __align__(8) uint64_t k_full[FA_STAGES], k_free[FA_STAGES], v_full[FA_VSTAGES], v_free[FA_VSTAGES];
    __shared__ __align__(8) uint64_t q_full, s_full[2], s_free[2], p_full[2], pv_done[2], drain;
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
        for (int s = 0; s < FA_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_free[s], 1);
        }
        for (int s = 0; s < FA_VSTAGES; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_free[s], 1);
        }
        mbar_init(&q_full, 128);
        for (int b = 0; b < 2; ++b) {
            mbar_init(&s_full[b], 1);
            mbar_init(&s_free[b], 128);
            mbar_init(&p_full[b], 128);
            mbar_init(&pv_done[b], 1);
        }
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

    if (warp == 0 || warp == 10) {
        // TMA producers: warp 0 streams the K tiles (refilled once Q K^T of the tile two back is
        // done), warp 10 the V^T tiles (refilled once P V of the tile three back is done)
        if (lane == 0) {
            const bool is_k = warp == 0;
            const int n_st = is_k ? FA_STAGES : FA_VSTAGES;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* free_ = is_k ? k_free : v_free;
            int issued = 0;
            for (int j = 0; j < nt; ++j) {
                const int s = j % n_st;
                if (j >= n_st && !mbar_wait(&free_[s], ((uint32_t)(j / n_st) & 1u) ^ 1u, deadline, failed)) break;
                if (is_k) {
                    uint8_t* kb = smem + s * FA_K_STAGE;
                    mbar_expect_tx(&full[s], FA_K_STAGE);
                    tma_load_3d(kb, &tk_hi, &full[s], 0, j * FA_BN, kvh);
                    tma_load_3d(kb + FA_K_ATOM, &tk_hi, &full[s], 64, j * FA_BN, kvh);
                    tma_load_3d(kb + 2 * FA_K_ATOM, &tk_lo, &full[s], 0, j * FA_BN, kvh);
                    tma_load_3d(kb + 3 * FA_K_ATOM, &tk_lo, &full[s], 64, j * FA_BN, kvh);
                } else {
                    uint8_t* vb = smem + FA_OFF_V + s * FA_V_STAGE;
                    mbar_expect_tx(&full[s], FA_V_STAGE);
                    tma_load_3d(vb, &tv_hi, &full[s], j * FA_BN, 0, kvh);
                    tma_load_3d(vb + FA_V_TILE, &tv_lo, &full[s], j * FA_BN, 0, kvh);
                }
                issued = j + 1;
            }
            if (failed) {
                // let this thread's copies land before shared memory goes away
                bool f2 = false;
                const unsigned long long d2 = globaltimer_ns() + p.timeout_ns;
                for (int j = max(0, issued - n_st); j < issued; ++j)
                    mbar_wait(&full[j % n_st], (uint32_t)(j / n_st) & 1u, d2, f2);
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {
            constexpr uint32_t idesc_s = fa_idesc(FA_BM, FA_BN, false);  // Q, K: fp16 hi/lo
            constexpr uint32_t idesc_o = fa_idesc(FA_BM, ATT_D, true);   // P, V: bf16 hi/lo
            bool issued = false;
            // S(j) -> group j & 1's columns; needs K tile j and that group's read of S(j - 2)
            auto issue_s = [&](int j) -> bool {
                const int s = j % FA_STAGES, b = j & 1;
                if (!mbar_wait(&k_full[s], (uint32_t)(j / FA_STAGES) & 1u, deadline, failed)) return false;
                if (j >= 2 && !mbar_wait(&s_free[b], (uint32_t)((j - 2) >> 1) & 1u, deadline, failed)) return false;
                tc_fence_after();
                const uint32_t kb = smem_u32(smem + s * FA_K_STAGE);
                const uint32_t d = tmem + FA_T_S + 64u * (uint32_t)b;
#pragma unroll
                for (int ks = 0; ks < ATT_D / 16; ++ks) {
                    // 16 dims: 8 TMEM columns of Q; 32 bytes inside a 64-dim K atom
                    const uint32_t ka = (uint32_t)(ks >> 2) * FA_K_ATOM + (uint32_t)(ks & 3) * 32;
                    const uint64_t dkh = sw128_kmajor_desc(kb + ka), dkl = sw128_kmajor_desc(kb + 2 * FA_K_ATOM + ka);
                    const uint32_t qc = 8u * (uint32_t)ks;
                    umma_ts(d, tmem + FA_T_QH + qc, dkh, idesc_s, ks > 0 ? 1u : 0u);
                    umma_ts(d, tmem + FA_T_QH + qc, dkl, idesc_s, 1u);
                    umma_ts(d, tmem + FA_T_QL + qc, dkh, idesc_s, 1u);
                }
                issued = true;
                umma_commit(&k_free[s]);  // the K stage may be refilled once these MMAs read it
                umma_commit(&s_full[b]);  // the scores are in TMEM
                return true;
            };
            if (mbar_wait(&q_full, 0, deadline, failed)) {
                if (nt > 0) issue_s(0);
                if (nt > 1) issue_s(1);
            }
            for (int j = 0; j < nt && !failed; ++j) {
                const int s = j % FA_VSTAGES, b = j & 1;
                if (!mbar_wait(&p_full[b], (uint32_t)(j >> 1) & 1u, deadline, failed)) break;
                if (!mbar_wait(&v_full[s], (uint32_t)(j / FA_VSTAGES) & 1u, deadline, failed)) break;
                tc_fence_after();
                const uint32_t vhi = smem_u32(smem + FA_OFF_V + s * FA_V_STAGE), vlo = vhi + FA_V_TILE;
                const uint32_t phi = smem_u32(smem + FA_OFF_P + 2 * b * FA_P_TILE), plo = phi + FA_P_TILE;
                const uint32_t o = tmem + FA_T_O + 128u * (uint32_t)b;
#pragma unroll
                for (int ks = 0; ks < FA_BN / 16; ++ks) {
                    const uint32_t off = (uint32_t)ks * 32;  // 16 keys = 32 bytes of a P row and a V^T row
                    const uint64_t dvh = sw128_kmajor_desc(vhi + off), dvl = sw128_kmajor_desc(vlo + off);
                    const uint64_t dph = sw128_kmajor_desc(phi + off), dpl = sw128_kmajor_desc(plo + off);
                    umma_bf16(o, dph, dvh, idesc_o, (j >= 2 || ks > 0) ? 1u : 0u);
                    umma_bf16(o, dph, dvl, idesc_o, 1u);
                    umma_bf16(o, dpl, dvh, idesc_o, 1u);
                }
                umma_commit(&v_free[s]);   // the V^T stage may be refilled once these MMAs read it
                umma_commit(&pv_done[b]);  // O_b holds its tiles <= j; P tile b may be rewritten
                if (j + 2 < nt && !issue_s(j + 2)) break;
            }
            if (failed && issued) {
                // the MMAs already issued finish before TMEM is freed
                umma_commit(&drain);
                bool f2 = false;
                mbar_wait(&drain, 0, globaltimer_ns() + p.timeout_ns, f2);
            }
        }
    } else {
        // softmax group gr = (warp - 2) / 4; warp w owns TMEM lanes [32*(w%4), 32*(w%4) + 32): row r
        const int gr = (warp - 2) >> 2;
        const int q4 = warp & 3;
        const int r = q4 * 32 + lane;
        const uint32_t trow = tmem + ((uint32_t)(q4 * 32) << 16);
        const int t = t0 + r / G, g = r % G;
        const int my_pos = p.pos0 + t;
        const int cta_pos = p.pos0 + t0;  // smallest position among the CTA's rows
        if (gr == 0) {
            // this row of Q as fp16 hi/lo into TMEM (rows past the prompt: zero)
            const float4* src = reinterpret_cast<const float4*>(p.q + ((size_t)t * p.n_heads + kvh * G + g) * ATT_D);
            bool bad = false;
#pragma unroll 1
            for (int half = 0; half < 2; ++half) {
                uint32_t hw[32], lw[32];
#pragma unroll
                for (int i = 0; i < 16; ++i) {
                    const float4 v = t < p.P ? src[16 * half + i] : make_float4(0.f, 0.f, 0.f, 0.f);
                    __half h0, h1, h2, h3, l0, l1, l2, l3;
                    split_f16(v.x, h0, l0, bad);
                    split_f16(v.y, h1, l1, bad);
                    split_f16(v.z, h2, l2, bad);
                    split_f16(v.w, h3, l3, bad);
                    hw[2 * i] = pack_half2(h0, h1);
                    hw[2 * i + 1] = pack_half2(h2, h3);
                    lw[2 * i] = pack_half2(l0, l1);
                    lw[2 * i + 1] = pack_half2(l2, l3);
                }
                tmem_st32(trow + FA_T_QH + 32 * half, hw);
                tmem_st32(trow + FA_T_QL + 32 * half, lw);
            }
            tmem_wait_st();
            if (bad) atomicOr(p.status, 4);
            tc_fence_before();
            mbar_arrive(&q_full);
        }
        // softmax in base 2: exp(x * scale) = 2^(x * scale * log2(e)); scale = 1/sqrt(128) (src/ops/kernels.cpp:88)
        const float c2 = (1.0f / sqrtf((float)ATT_D)) * 1.4426950408889634f;
        const uint32_t s_col = trow + FA_T_S + 64u * (uint32_t)gr;
        const uint32_t o_col = trow + FA_T_O + 128u * (uint32_t)gr;
        uint8_t* phi = smem + FA_OFF_P + 2 * gr * FA_P_TILE;
        uint8_t* plo = phi + FA_P_TILE;
        float m = -INFINITY, l = 0.f;
        for (int j = gr, i = 0; j < nt; j += 2, ++i) {
            mbar_wait(&s_full[gr], (uint32_t)i & 1u, deadline, failed);
            tc_fence_after();
            uint32_t sr[64];
            tmem_ld32_nowait(s_col, *reinterpret_cast<uint32_t(*)[32]>(sr));
            tmem_ld32_nowait(s_col + 32, *reinterpret_cast<uint32_t(*)[32]>(sr + 32));
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&s_free[gr]);
            // causal mask (tiles below the CTA's first position need none); max of the raw scores
            float sv[64];
            float mr = -INFINITY;
            if ((j + 1) * FA_BN - 1 <= cta_pos) {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sv[c] = __uint_as_float(sr[c]);
                    mr = fmaxf(mr, sv[c]);
                }
            } else {
#pragma unroll
                for (int c = 0; c < 64; ++c) {
                    sv[c] = (j * FA_BN + c <= my_pos) ? __uint_as_float(sr[c]) : -INFINITY;
                    mr = fmaxf(mr, sv[c]);
                }
            }
            // The running max m (scaled) moves only when the tile's max exceeds it by more than 8
            // (a factor 2^8): softmax is shift-invariant and O_g and l share m, so a stale m changes
            // rounding only (p <= 2^8) and O_g is rescaled rarely. A row may see no key in a
            // group's first tiles (m = -inf): its p are 0 and nothing accumulates.
            const float mx = mr * c2;
            const bool bump = mx > m + 8.f;
            const float mu = bump ? mx : m;
            const float mu_e = mu == -INFINITY ? 0.f : mu;
            const float alpha = bump ? ex2_approx(m - mu_e) : 1.f;
            float s4[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int c = 0; c < 64; ++c) {
                sv[c] = ex2_approx(fmaf(sv[c], c2, -mu_e));
                s4[c & 3] += sv[c];
            }
            l = fmaf(l, alpha, (s4[0] + s4[1]) + (s4[2] + s4[3]));
            m = mu;
            // P V of this group's previous tile is done: its P tile is free and O_g is stable
            if (i >= 1) mbar_wait(&pv_done[gr], (uint32_t)(i - 1) & 1u, deadline, failed);
            tc_fence_after();
            // P hi/lo of row r into the 128-byte-swizzled K-major tile (chunk c of 8 keys at c ^ (r % 8))
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
            // rescale this row of O_g when its running max moved (warp-collective TMEM access)
            if (i >= 1 && __any_sync(0xffffffffu, bump)) {
#pragma unroll 1
                for (int cc = 0; cc < ATT_D; cc += 32) {
                    uint32_t o[32];
                    tmem_ld32(o_col + cc, o);
#pragma unroll
                    for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    tmem_st32(o_col + cc, o);
                }
                tmem_wait_st();
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // P visible to the tensor core
            tc_fence_before();
            mbar_arrive(&p_full[gr]);
        }
        // merge: both groups' last P V done, then O = (O_0 a_0 + O_1 a_1) / (l_0 a_0 + l_1 a_1),
        // a_g = 2^(m_g - max(m_0, m_1)); group g writes dims [64 g, 64 g + 64)
        const int n_mine = (nt - gr + 1) >> 1;  // tiles this group processed
        if (n_mine > 0) mbar_wait(&pv_done[gr], (uint32_t)(n_mine - 1) & 1u, deadline, failed);
        // the P tiles are idle now (every P V is done): they hold the groups' (m, l) per row
        named_bar_sync(1, 256);
        float2* merge_s = reinterpret_cast<float2*>(smem + FA_OFF_P);  // [2][FA_BM]
        merge_s[gr * FA_BM + r] = make_float2(m, l);
        tc_fence_before();
        named_bar_sync(1, 256);
        tc_fence_after();
        const float2 ml0 = merge_s[r], ml1 = merge_s[FA_BM + r];
        const bool two = nt > 1;  // O_1 holds data only when group 1 had a tile
        const float mm = two ? fmaxf(ml0.x, ml1.x) : ml0.x;  // finite: key 0 is in group 0's tile 0
        const float a0 = ex2_approx(ml0.x - mm);
        const float a1 = two ? ex2_approx(ml1.x - mm) : 0.f;
        const float inv = 1.0f / (two ? fmaf(ml0.y, a0, ml1.y * a1) : ml0.y * a0);
        const float w0 = a0 * inv, w1 = a1 * inv;
#pragma unroll 1
        for (int cc = 64 * gr; cc < 64 * gr + 64; cc += 32) {
            uint32_t o0[32], o1[32];
            tmem_ld32_nowait(trow + FA_T_O + cc, o0);
            if (two) tmem_ld32_nowait(trow + FA_T_O + 128 + cc, o1);
            tmem_wait_ld();
            if (t < p.P && !failed) {
                const size_t base = ((size_t)t * p.n_heads + kvh * G + g) * ATT_D + cc;
#pragma unroll
                for (int e = 0; e < 32; e += 8) {
                    __align__(16) __nv_bfloat16 h[8], lo8[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) {
                        const float v = two ? fmaf(__uint_as_float(o0[e + u]), w0, __uint_as_float(o1[e + u]) * w1)
                                            : __uint_as_float(o0[e + u]) * w0;
                        split_bf16(v, h[u], lo8[u]);
                    }
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

// K cache rows [0, n_keys) of [Hkv][max_seq][128] (float or bf16) -> fp16 hi/lo
// [Hkv][ld][128], one warp per row. A value outside the fp16 range sets status bit 4.
template <typename KV>
__global__ void __launch_bounds__(256) fa_k_split_kernel(const KV* __restrict__ k_cache, int Hkv, int max_seq,
                                                         int n_keys, int ld, __half* kh, __half* kl, int* status) {
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    const long long rows = (long long)Hkv * n_keys;
    const long long warps = (long long)gridDim.x * (blockDim.x >> 5);
    bool bad = false;
    for (long long w = (long long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); w < rows; w += warps) {
        const int h = (int)(w / n_keys), key = (int)(w % n_keys);
        const float4 v = kv_ld4(k_cache + ((size_t)h * max_seq + key) * ATT_D + 4 * lane);
        const size_t dst = ((size_t)h * ld + key) * ATT_D + 4 * lane;
        __half h0, h1, h2, h3, l0, l1, l2, l3;
        split_f16(v.x, h0, l0, bad);
        split_f16(v.y, h1, l1, bad);
        split_f16(v.z, h2, l2, bad);
        split_f16(v.w, h3, l3, bad);
        *reinterpret_cast<uint2*>(kh + dst) = make_uint2(pack_half2(h0, h1), pack_half2(h2, h3));
        *reinterpret_cast<uint2*>(kl + dst) = make_uint2(pack_half2(l0, l1), pack_half2(l2, l3));
    }
    if (bad) atomicOr(status, 4);
}

// V cache rows [0, n_keys) of [Hkv][max_seq][128] (float or bf16) -> V^T bf16 hi/lo
// [Hkv][128][ld] (tiles of 64 keys x 128 dims through shared memory; grid
// (ceil(n_keys/64), Hkv)). A bf16 row splits into itself and zero.
template <typename KV>
__global__ void __launch_bounds__(256) fa_v_split_kernel(const KV* __restrict__ v_cache, int max_seq, int n_keys,
                                                         int ld, __nv_bfloat16* vh, __nv_bfloat16* vl) {
    __shared__ float tile[64][ATT_D + 1];
    pdl_launch_dependents();
    pdl_wait();
    const int k0 = blockIdx.x * 64, h = blockIdx.y;
    for (int i = threadIdx.x; i < 64 * ATT_D; i += blockDim.x) {
        const int kk = i / ATT_D, d = i % ATT_D;
        tile[kk][d] = (k0 + kk < n_keys) ? (float)v_cache[((size_t)h * max_seq + k0 + kk) * ATT_D + d] : 0.f;
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
