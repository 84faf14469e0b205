// Batched-prefill attention pieces.
//
// Reference semantics per prompt token t (src/models/qwen3/module.cpp:187-234,
// src/ops/kernels.cpp:31-110): Q/K RMSNorm per head, NeoX RoPE at position t,
// K/V row t appended to the cache, then for every query head softmax over
// positions [0, t] of (q.k) / sqrt(128) and the weighted sum of V rows. The
// batched form computes all P tokens of a layer at once; the per-token math
// (RMSNorm, the fused rotation, max-subtracted softmax) is the same, the
// softmax is evaluated online over 32-key tiles.
//
//  * prefill_qkv_post_kernel: one warp per (token, head), eight heads per
//    CTA: norm + RoPE of q
//    (-> Q buffer), of k (-> K cache row), v copied to the V cache row.
//  * prefill_attn_kernel: CTA = 64 query rows (QT tokens x G heads of one
//    KV head, QT = 64 / G) x one KV head; 256 threads. K/V tiles of 32 rows
//    (row stride padded to 132 floats) go through a double-buffered cp.async
//    ring; each thread owns a 4 x 2 block of scores (4 query rows, 2 keys)
//    and a 4 x 8 block of the output (4 rows, 8 dims). A half-warp shares
//    its 4 rows' running max/sum; probabilities go through shared memory.
//    The output is normalised and written as the O projection's bf16 hi/lo
//    operands. Tiles of the latest queries (most keys) are scheduled first.
#pragma once

#include <cuda_bf16.h>

#include "attention.cuh"
#include "mf_common.cuh"
#include "prefill_gemm.cuh"

namespace mf {

// qkv: [P][(Hq + 2 Hkv) * D] (projection output); Q out: [P][Hq * D];
// caches: this layer's [Hkv][max_seq][D] of KV (float, or bf16 rounded to
// nearest even). Positions are pos0 + token.
// One warp per (token, head): CTA (t, y) serves token t, heads 8y .. 8y + 7.
constexpr int QP_WARPS = 8;
template <typename KV>
__global__ void __launch_bounds__(QP_WARPS * 32) prefill_qkv_post_kernel(const float* __restrict__ qkv,
                                                                        const float* q_norm_w, const float* k_norm_w,
                                                                        float eps, const float2* rope, float* q_out,
                                                                        KV* k_cache, KV* v_cache, int max_seq,
                                                                        int n_heads, int n_kv_heads, int pos0) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x, h = blockIdx.y * QP_WARPS + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    const int Hq = n_heads, Hkv = n_kv_heads;
    const int pos = pos0 + t;
    if (pos >= max_seq) return;
    const size_t row = (size_t)t * (Hq + 2 * Hkv) * ATT_D;
    const float2* cs = rope + (size_t)pos * (ATT_D / 2);
    if (h < Hq) {
        const float4 v = reinterpret_cast<const float4*>(qkv + row + (size_t)h * ATT_D)[lane];
        reinterpret_cast<float4*>(q_out + ((size_t)t * Hq + h) * ATT_D)[lane] =
            norm_rope_head(v, q_norm_w, eps, cs, lane);
    } else if (h < Hq + Hkv) {
        const int kh = h - Hq;
        const float4 k = reinterpret_cast<const float4*>(qkv + row + (size_t)(Hq + kh) * ATT_D)[lane];
        const float4 v = reinterpret_cast<const float4*>(qkv + row + (size_t)(Hq + Hkv + kh) * ATT_D)[lane];
        const size_t c = ((size_t)kh * max_seq + pos) * ATT_D + 4 * lane;
        kv_st4(k_cache + c, norm_rope_head(k, k_norm_w, eps, cs, lane));
        kv_st4(v_cache + c, v);
    }
}

constexpr int PA_ROWS = 64;     // query rows per CTA
constexpr int PA_KT = 32;       // keys per tile
constexpr int PA_KS = 132;      // padded K/V row stride (floats)
constexpr int PA_THREADS = 256;
constexpr int PA_PS = PA_KT + 1;  // probability row stride

inline size_t pa_smem_bytes() {
    return ((size_t)PA_ROWS * ATT_D + 2 * 2 * PA_KT * PA_KS + PA_ROWS * PA_PS) * sizeof(float);
}

// Q: [P][Hq * D] (normed, rotated); caches [Hkv][max_seq][D] holding rows
// pos0 .. pos0 + P - 1 (and the history before pos0); out: bf16 hi/lo [P][Hq * D].
// bf16 cache rows are widened into the fp32 tiles with plain loads.
template <int G, typename KV>
__global__ void __launch_bounds__(PA_THREADS, 2)
    prefill_attn_kernel(const float* __restrict__ Q, const KV* __restrict__ k_cache,
                        const KV* __restrict__ v_cache, int max_seq, int P, int pos0, int n_heads,
                        __nv_bfloat16* out_hi, __nv_bfloat16* out_lo) {
    constexpr int QT = PA_ROWS / G;  // tokens per CTA
    extern __shared__ float4 pa_smem4[];
    float* q_s = reinterpret_cast<float*>(pa_smem4);  // [64][128]
    float* kv_s = q_s + PA_ROWS * ATT_D;              // [2 stages][K, V][32][132]
    float* p_s = kv_s + 2 * 2 * PA_KT * PA_KS;        // [64][33]

    const int tid = threadIdx.x, lane = tid & 31;
    const int n_qt = (P + QT - 1) / QT;
    const int qt = n_qt - 1 - (int)blockIdx.x;  // latest tokens (most keys) first
    const int kvh = blockIdx.y;
    const int Hq = n_heads;
    const int t0 = qt * QT;                      // first token of this tile
    const int t_last = min(t0 + QT, P) - 1;
    const KV* kc = k_cache + (size_t)kvh * max_seq * ATT_D;
    const KV* vc = v_cache + (size_t)kvh * max_seq * ATT_D;

    pdl_launch_dependents();
    pdl_wait();

    // query rows r = token_local * G + g
    for (int i = tid; i < PA_ROWS * ATT_D / 4; i += PA_THREADS) {
        const int r = i / (ATT_D / 4), c4 = i % (ATT_D / 4);
        const int t = t0 + r / G, g = r % G;
        float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
        if (t < P) v = reinterpret_cast<const float4*>(Q + ((size_t)t * Hq + kvh * G + g) * ATT_D)[c4];
        reinterpret_cast<float4*>(q_s + r * ATT_D)[c4] = v;
    }
    // keys [0, pos0 + t_last] (the history before pos0 and this prompt's rows)
    const int n_keys = pos0 + t_last + 1;
    const int n_tiles = (n_keys + PA_KT - 1) / PA_KT;
    auto issue = [&](int kt) {
        if (kt < n_tiles) {
            float* ks = kv_s + (kt & 1) * 2 * PA_KT * PA_KS;
            float* vs = ks + PA_KT * PA_KS;
            const int k0 = kt * PA_KT;
            for (int i = tid; i < PA_KT * ATT_D / 4; i += PA_THREADS) {
                const int r = i / (ATT_D / 4), c4 = i % (ATT_D / 4);
                if (k0 + r < n_keys) {
                    if constexpr (sizeof(KV) == sizeof(float)) {
                        cp_async16(ks + r * PA_KS + 4 * c4, kc + (size_t)(k0 + r) * ATT_D + 4 * c4);
                        cp_async16(vs + r * PA_KS + 4 * c4, vc + (size_t)(k0 + r) * ATT_D + 4 * c4);
                    } else {
                        *reinterpret_cast<float4*>(ks + r * PA_KS + 4 * c4) =
                            kv_ld4(kc + (size_t)(k0 + r) * ATT_D + 4 * c4);
                        *reinterpret_cast<float4*>(vs + r * PA_KS + 4 * c4) =
                            kv_ld4(vc + (size_t)(k0 + r) * ATT_D + 4 * c4);
                    }
                }
            }
        }
        cp_async_commit();
    };
    issue(0);

    // thread roles: rows rq..rq+3 (a half-warp shares them), keys 2*kq, 2*kq+1, dims 8*kq .. 8*kq+7
    const int rq = (tid >> 4) * 4, kq = tid & 15;
    int tok[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) tok[i] = pos0 + t0 + (rq + i) / G;  // absolute position of row rq+i
    const float scale = 1.0f / sqrtf((float)ATT_D);  // src/ops/kernels.cpp:88
    float m[4], l[4], o[4][8];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        m[i] = -INFINITY;
        l[i] = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j) o[i][j] = 0.f;
    }

    for (int kt = 0; kt < n_tiles; ++kt) {
        issue(kt + 1);
        cp_async_wait<1>();
        __syncthreads();
        const float* ks = kv_s + (kt & 1) * 2 * PA_KT * PA_KS;
        const float* vs = ks + PA_KT * PA_KS;
        const int k0 = kt * PA_KT;
        // scores of rows rq..rq+3 x keys 2kq, 2kq+1
        float s[4][2];
#pragma unroll
        for (int i = 0; i < 4; ++i) s[i][0] = s[i][1] = 0.f;
#pragma unroll 4
        for (int d4 = 0; d4 < ATT_D / 4; ++d4) {
            const float4 k0v = *reinterpret_cast<const float4*>(ks + (2 * kq) * PA_KS + 4 * d4);
            const float4 k1v = *reinterpret_cast<const float4*>(ks + (2 * kq + 1) * PA_KS + 4 * d4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float4 qv = *reinterpret_cast<const float4*>(q_s + (rq + i) * ATT_D + 4 * d4);
                s[i][0] = fmaf(qv.x, k0v.x, s[i][0]);
                s[i][0] = fmaf(qv.y, k0v.y, s[i][0]);
                s[i][0] = fmaf(qv.z, k0v.z, s[i][0]);
                s[i][0] = fmaf(qv.w, k0v.w, s[i][0]);
                s[i][1] = fmaf(qv.x, k1v.x, s[i][1]);
                s[i][1] = fmaf(qv.y, k1v.y, s[i][1]);
                s[i][1] = fmaf(qv.z, k1v.z, s[i][1]);
                s[i][1] = fmaf(qv.w, k1v.w, s[i][1]);
            }
        }
        // causal mask, online softmax over the half-warp's 32 keys
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            float p0 = (k0 + 2 * kq <= tok[i]) ? s[i][0] * scale : -INFINITY;
            float p1 = (k0 + 2 * kq + 1 <= tok[i]) ? s[i][1] * scale : -INFINITY;
            float mx = fmaxf(p0, p1);
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
            const float mn = fmaxf(m[i], mx);
            // mn is finite: key 0 is visible to every row
            const float a = (m[i] == -INFINITY) ? 0.f : expf(m[i] - mn);
            p0 = expf(p0 - mn);
            p1 = expf(p1 - mn);
            float sum = p0 + p1;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
            l[i] = fmaf(l[i], a, sum);
            m[i] = mn;
#pragma unroll
            for (int j = 0; j < 8; ++j) o[i][j] *= a;
            p_s[(rq + i) * PA_PS + 2 * kq] = p0;
            p_s[(rq + i) * PA_PS + 2 * kq + 1] = p1;
        }
        __syncwarp();
        // O[rows][8 dims] += P[rows][32 keys] . V[32 keys][8 dims]
        const int kmax = min(PA_KT, n_keys - k0);
        for (int kk = 0; kk < kmax; ++kk) {
            const float4 va = *reinterpret_cast<const float4*>(vs + kk * PA_KS + 8 * kq);
            const float4 vb = *reinterpret_cast<const float4*>(vs + kk * PA_KS + 8 * kq + 4);
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const float pr = p_s[(rq + i) * PA_PS + kk];
                o[i][0] = fmaf(pr, va.x, o[i][0]);
                o[i][1] = fmaf(pr, va.y, o[i][1]);
                o[i][2] = fmaf(pr, va.z, o[i][2]);
                o[i][3] = fmaf(pr, va.w, o[i][3]);
                o[i][4] = fmaf(pr, vb.x, o[i][4]);
                o[i][5] = fmaf(pr, vb.y, o[i][5]);
                o[i][6] = fmaf(pr, vb.z, o[i][6]);
                o[i][7] = fmaf(pr, vb.w, o[i][7]);
            }
        }
        __syncthreads();  // the stage and p_s are reused
    }
    cp_async_wait<0>();
    (void)lane;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const int r = rq + i, t = t0 + r / G, g = r % G;
        if (t >= P) continue;
        const float inv = 1.0f / l[i];
        const size_t base = ((size_t)t * Hq + kvh * G + g) * ATT_D + 8 * kq;
#pragma unroll
        for (int j = 0; j < 8; ++j) split_bf16(o[i][j] * inv, out_hi[base + j], out_lo[base + j]);
    }
}

}  // namespace mf
