// Decode attention for one token: per-head Q/K RMSNorm + NeoX RoPE + KV-cache
// append + GQA attention over the HBM-resident fp32 KV cache, as one kernel.
//
// Reference semantics (src/models/qwen3/module.cpp:187-234, src/ops/kernels.cpp:31-110):
//  * q_h <- rmsnorm(q_h, q_norm), k_h <- rmsnorm(k_h, k_norm) over d_head;
//  * NeoX RoPE on pairs (i, i + d_rot/2): x0' = cos*x0 - sin*x1,
//    x1' = sin*x0 + cos*x1 in float, first product fused; (cos, sin) of
//    each position come from a host-built table (same float libm as the
//    reference), so the rotation is bit-exact;
//  * K/V row `pos` appended to the cache, then for every query head h of KV
//    head h/kv_mul: scores = (q.k) * (1/sqrtf(d_head)) over positions [0, pos],
//    max-subtracted softmax, output = sum_p prob_p * v_p.
// Here the softmax is evaluated online (running max and sum) and the final
// division is done once; the result equals the reference's up to fp32
// rounding.
//
// B200 structure (split-K flash decode):
//  * grid = (n_split, n_kv_heads); each CTA serves ALL kv_mul query heads of
//    its KV head over one contiguous slice of positions, so every K/V row is
//    read from HBM exactly once per token.
//  * The cache layout is [kv_head][position][d_head] (fp32), so a slice is one
//    contiguous run of rows. Each warp streams 16-row K and V tiles into a
//    double-buffered shared-memory stage with cp.async (no register staging),
//    computes 16 scores per head with lanes owning positions (conflict-free
//    padded K rows), and accumulates P.V with lanes owning 4 dims each.
//  * Warps, then CTAs, are merged with the usual (max, sum, vector) rescaling;
//    the CTA that finishes last for a KV head merges the n_split partials in a
//    fixed order (deterministic; no spin-waits).
#pragma once

#include "mf_common.cuh"

namespace mf {

constexpr int ATT_D = 128;       // head dim (Qwen3)
constexpr int ATT_TILE = 16;     // positions per warp tile
constexpr int ATT_WARPS = 4;
constexpr int ATT_KSTRIDE = ATT_D + 4;  // padded K row (floats): conflict-free row-per-lane reads
constexpr int ATT_PF_ROWS = 256;        // L2 prefetch window per CTA (rows of K and of V)
constexpr int ATT_MIN_CHUNK = 128;      // fewest positions per split

struct AttnParams {
    const float* qkv;        // [Hq*D | Hkv*D | Hkv*D] (this rank's heads)
    const float* q_norm_w;   // [D]
    const float* k_norm_w;   // [D]
    float eps;
    const float2* rope;      // [max_seq][D/2] (cos, sin) per position and pair
    float* k_cache;          // this layer: [Hkv][max_seq][D]
    float* v_cache;
    int max_seq;
    const int* pos_ptr;      // current position (device)
    float* out;              // [Hq*D]
    float* part_o;           // [Hkv][n_split][G][D]
    float* part_ml;          // [Hkv][n_split][G][2]
    int* counters;           // [Hkv], zero-initialised, reset by the last CTA
    int n_heads;
    int n_kv_heads;
    int n_split;
};

struct AttnSmemLayout {
    static constexpr int K_STAGE = ATT_TILE * ATT_KSTRIDE;  // floats
    static constexpr int V_STAGE = ATT_TILE * ATT_D;
    static constexpr int WARP_FLOATS = 2 * (K_STAGE + V_STAGE);
};

MF_DEVICE void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
MF_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> MF_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

// RMSNorm + NeoX RoPE of one 128-dim head held by a warp (lane owns dims 4l..4l+3).
MF_DEVICE float4 norm_rope_head(float4 v, const float* nw, float eps, const float2* cs, int lane) {
    float ss = v.x * v.x;
    ss = fmaf(v.y, v.y, ss);
    ss = fmaf(v.z, v.z, ss);
    ss = fmaf(v.w, v.w, ss);
    ss = warp_sum(ss);
    const float inv = 1.0f / sqrtf(ss / (float)ATT_D + eps);
    const float4 w = *reinterpret_cast<const float4*>(nw + 4 * lane);
    float x[4] = {(inv * v.x) * w.x, (inv * v.y) * w.y, (inv * v.z) * w.z, (inv * v.w) * w.w};
    // partner lane (l ^ 16) holds the other half of each rotation pair
    float o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
        const float2 c = __ldg(cs + 4 * (lane & 15) + e);
        // x0' = cos*x0 - sin*x1, x1' = sin*x0 + cos*x1, with the first product
        // fused as the reference's compiler contracts it: fma(cos, x0, -(sin*x1))
        if (lane < 16) {
            o[e] = fmaf(c.x, x[e], -__fmul_rn(c.y, other));
        } else {
            o[e] = fmaf(c.y, other, __fmul_rn(c.x, x[e]));
        }
    }
    return make_float4(o[0], o[1], o[2], o[3]);
}

template <int G>
__global__ void __launch_bounds__(ATT_WARPS * 32) attn_decode_kernel(const AttnParams p) {
    extern __shared__ float4 att_smem4[];
    float* smem = reinterpret_cast<float*>(att_smem4);
    __shared__ __align__(16) float q_s[G][ATT_D];
    __shared__ float p_s[ATT_WARPS][G][ATT_TILE];
    __shared__ float wm[ATT_WARPS][G], wl[ATT_WARPS][G];
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int Hq = p.n_heads, Hkv = p.n_kv_heads;
    const size_t head_stride = (size_t)p.max_seq * ATT_D;
    float* kc = p.k_cache + (size_t)kvh * head_stride;
    float* vc = p.v_cache + (size_t)kvh * head_stride;

    pdl_launch_dependents();
    pdl_wait();

    const int pos = __ldcg(p.pos_ptr);
    const int len = pos + 1;
    const float2* cs = p.rope + (size_t)pos * (ATT_D / 2);
    // Effective split count for this context: slices of at least
    // ATT_MIN_CHUNK positions (short contexts use fewer CTAs and a cheaper
    // merge); CTAs past it only append K/V if they own `pos` (never: the
    // last effective slice ends at len).
    const int eff_split = min(p.n_split, max(1, (len + ATT_MIN_CHUNK - 1) / ATT_MIN_CHUNK));
    if (split >= eff_split) return;
    int chunk = (len + eff_split - 1) / eff_split;
    chunk = (chunk + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    const int start = split * chunk;
    const int end = min(start + chunk, len);

    // The CTA's K and V rows are contiguous: bulk-prefetch the first
    // ATT_PF_ROWS of each into L2 now; every tile issue below extends the
    // window by one tile, so the cp.async stream mostly hits L2.
    if (tid == 0 && end > start) {
        const uint32_t nb = (uint32_t)min(end - start, ATT_PF_ROWS) * ATT_D * sizeof(float);
        prefetch_l2(kc + (size_t)start * ATT_D, nb);
        prefetch_l2(vc + (size_t)start * ATT_D, nb);
    }
    float* ks = smem + warp * AttnSmemLayout::WARP_FLOATS;
    float* vs = ks + 2 * AttnSmemLayout::K_STAGE;
    const int ntiles = end > start ? (end - start + ATT_TILE - 1) / ATT_TILE : 0;
    auto issue = [&](int t, int stage) {
        const int p0 = start + t * ATT_TILE;
        const int nv = min(ATT_TILE, end - p0);
        float* kd = ks + stage * AttnSmemLayout::K_STAGE;
        float* vd = vs + stage * AttnSmemLayout::V_STAGE;
        const int pf = p0 + ATT_PF_ROWS;  // tile entering the prefetch window
        if (lane == 0 && pf < end) {
            const uint32_t nb = (uint32_t)min(ATT_TILE, end - pf) * ATT_D * sizeof(float);
            prefetch_l2(kc + (size_t)pf * ATT_D, nb);
            prefetch_l2(vc + (size_t)pf * ATT_D, nb);
        }
#pragma unroll 4
        for (int r = 0; r < nv; ++r) {
            cp_async16(kd + r * ATT_KSTRIDE + 4 * lane, kc + (size_t)(p0 + r) * ATT_D + 4 * lane);
            cp_async16(vd + r * ATT_D + 4 * lane, vc + (size_t)(p0 + r) * ATT_D + 4 * lane);
        }
        cp_async_commit();
    };
    // The warp's first tile does not depend on the queries: start its copy
    // now, unless it holds row `pos` (written by the append below).
    const bool early = warp < ntiles && (start + (warp + 1) * ATT_TILE <= pos);
    if (early) issue(warp, 0);

    // ---- prologue: normalised + rotated queries of this group
    for (int g = warp; g < G; g += ATT_WARPS) {
        const int h = kvh * G + g;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.qkv + (size_t)h * ATT_D) + lane);
        const float4 r = norm_rope_head(v, p.q_norm_w, p.eps, cs, lane);
        *reinterpret_cast<float4*>(&q_s[g][4 * lane]) = r;
    }
    // ---- KV append: the CTA whose slice holds `pos` writes row pos
    if (start <= pos && pos < end && warp == 0) {
        const float* kraw = p.qkv + (size_t)Hq * ATT_D + (size_t)kvh * ATT_D;
        const float* vraw = p.qkv + (size_t)(Hq + Hkv) * ATT_D + (size_t)kvh * ATT_D;
        const float4 k = norm_rope_head(__ldcg(reinterpret_cast<const float4*>(kraw) + lane), p.k_norm_w, p.eps,
                                        cs, lane);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(vraw) + lane);
        reinterpret_cast<float4*>(kc + (size_t)pos * ATT_D)[lane] = k;
        reinterpret_cast<float4*>(vc + (size_t)pos * ATT_D)[lane] = v;
    }
    __syncthreads();

    const float scale = 1.0f / sqrtf((float)ATT_D);  // src/ops/kernels.cpp:88

    float m[G], l[G];
    float4 o[G];
#pragma unroll
    for (int g = 0; g < G; ++g) {
        m[g] = -INFINITY;
        l[g] = 0.f;
        o[g] = make_float4(0.f, 0.f, 0.f, 0.f);
    }

    const int j = lane & 15, half = lane >> 4;
    int stage = 0;
    if (warp < ntiles && !early) issue(warp, 0);
    for (int t = warp; t < ntiles; t += ATT_WARPS) {
        const int tn = t + ATT_WARPS;
        if (tn < ntiles) {
            issue(tn, stage ^ 1);
            cp_async_wait<1>();
        } else {
            cp_async_wait<0>();
        }
        __syncwarp();
        const int p0 = start + t * ATT_TILE;
        const int nv = min(ATT_TILE, end - p0);
        const float* kt = ks + stage * AttnSmemLayout::K_STAGE;
        const float* vt = vs + stage * AttnSmemLayout::V_STAGE;
        // scores: lane (j, half) -> position j, dims [64*half, 64*half+64)
        float s[G];
#pragma unroll
        for (int g = 0; g < G; ++g) s[g] = 0.f;
        const float* krow = kt + j * ATT_KSTRIDE + 64 * half;
#pragma unroll 4
        for (int d4 = 0; d4 < 16; ++d4) {
            const float4 k4 = *reinterpret_cast<const float4*>(krow + 4 * d4);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float4 q4 = *reinterpret_cast<const float4*>(&q_s[g][64 * half + 4 * d4]);
                s[g] = fmaf(q4.x, k4.x, s[g]);
                s[g] = fmaf(q4.y, k4.y, s[g]);
                s[g] = fmaf(q4.z, k4.z, s[g]);
                s[g] = fmaf(q4.w, k4.w, s[g]);
            }
        }
#pragma unroll
        for (int g = 0; g < G; ++g) {
            float sc = (s[g] + __shfl_xor_sync(0xffffffffu, s[g], 16)) * scale;
            if (j >= nv) sc = -INFINITY;
            float mt = sc;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) mt = fmaxf(mt, __shfl_xor_sync(0xffffffffu, mt, off));
            const float mn = fmaxf(m[g], mt);
            const float alpha = expf(m[g] - mn);
            const float pj = expf(sc - mn);
            float ps = pj;
#pragma unroll
            for (int off = 8; off > 0; off >>= 1) ps += __shfl_xor_sync(0xffffffffu, ps, off);
            l[g] = l[g] * alpha + ps;
            m[g] = mn;
            o[g].x *= alpha; o[g].y *= alpha; o[g].z *= alpha; o[g].w *= alpha;
            if (half == 0) p_s[warp][g][j] = pj;
        }
        __syncwarp();
        for (int jj = 0; jj < nv; ++jj) {
            const float4 v4 = *reinterpret_cast<const float4*>(vt + jj * ATT_D + 4 * lane);
#pragma unroll
            for (int g = 0; g < G; ++g) {
                const float pg = p_s[warp][g][jj];
                o[g].x = fmaf(pg, v4.x, o[g].x);
                o[g].y = fmaf(pg, v4.y, o[g].y);
                o[g].z = fmaf(pg, v4.z, o[g].z);
                o[g].w = fmaf(pg, v4.w, o[g].w);
            }
        }
        __syncwarp();
        stage ^= 1;
    }

    // ---- merge the warps of this CTA (reuse the warp stages as scratch)
    __syncthreads();
    float* wo = smem;  // [ATT_WARPS][G][D]
#pragma unroll
    for (int g = 0; g < G; ++g) {
        reinterpret_cast<float4*>(wo + ((size_t)warp * G + g) * ATT_D)[lane] = o[g];
        if (lane == 0) {
            wm[warp][g] = m[g];
            wl[warp][g] = l[g];
        }
    }
    __syncthreads();
    if (eff_split == 1) {  // one slice: finish here, no partials
        for (int idx = tid; idx < G * ATT_D; idx += ATT_WARPS * 32) {
            const int g = idx / ATT_D, d = idx - g * ATT_D;
            float M = -INFINITY;
#pragma unroll
            for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, wm[w][g]);
            float acc = 0.f, L = 0.f;
#pragma unroll
            for (int w = 0; w < ATT_WARPS; ++w) {
                const float f = (wm[w][g] == -INFINITY) ? 0.f : expf(wm[w][g] - M);
                acc = fmaf(f, wo[((size_t)w * G + g) * ATT_D + d], acc);
                L = fmaf(f, wl[w][g], L);
            }
            p.out[((size_t)kvh * G + g) * ATT_D + d] = acc / L;
        }
        return;
    }
    const size_t pbase = ((size_t)kvh * p.n_split + split) * G;
    for (int idx = tid; idx < G * ATT_D; idx += ATT_WARPS * 32) {
        const int g = idx / ATT_D, d = idx - g * ATT_D;
        float M = -INFINITY;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; ++w) M = fmaxf(M, wm[w][g]);
        float acc = 0.f, L = 0.f;
        if (M != -INFINITY) {
#pragma unroll
            for (int w = 0; w < ATT_WARPS; ++w) {
                const float f = expf(wm[w][g] - M);
                acc = fmaf(f, wo[((size_t)w * G + g) * ATT_D + d], acc);
                L = fmaf(f, wl[w][g], L);
            }
        }
        p.part_o[(pbase + g) * ATT_D + d] = acc;
        if (d == 0) {
            p.part_ml[(pbase + g) * 2 + 0] = M;
            p.part_ml[(pbase + g) * 2 + 1] = L;
        }
    }

    // ---- the last CTA of this KV head merges the n_split partials
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const int ticket = atomicAdd(p.counters + kvh, 1);
        is_last = (ticket == eff_split - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // merge in three parallel passes through shared memory (the warp stages
    // are free now): (m, l) of every split, then the per-split scale factors,
    // then the weighted sum of the partial outputs with independent loads.
    const int ns = eff_split;
    float* ml = smem;                    // [ns][G][2]
    float* fs = smem + 2 * ns * G;       // [G][ns] scale factors
    float* Ls = fs + ns * G;             // [G] denominators
    const size_t hb = (size_t)kvh * p.n_split * G;
    for (int i = tid; i < ns * G * 2; i += ATT_WARPS * 32) ml[i] = __ldcg(p.part_ml + hb * 2 + i);
    __syncthreads();
    if (tid < G) {
        const int g = tid;
        float M = -INFINITY;
        for (int sidx = 0; sidx < ns; ++sidx) M = fmaxf(M, ml[(sidx * G + g) * 2]);
        float L = 0.f;
        for (int sidx = 0; sidx < ns; ++sidx) {
            const float ms = ml[(sidx * G + g) * 2];
            const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
            fs[g * ns + sidx] = f;
            L = fmaf(f, ml[(sidx * G + g) * 2 + 1], L);
        }
        Ls[g] = L;
    }
    __syncthreads();
    for (int idx = tid; idx < G * ATT_D; idx += ATT_WARPS * 32) {
        const int g = idx / ATT_D, d = idx - g * ATT_D;
        const float* po = p.part_o + (hb + g) * ATT_D + d;
        const float* f = fs + g * ns;
        float acc = 0.f;
        for (int s0 = 0; s0 < ns; s0 += 16) {
            float o[16];
#pragma unroll
            for (int u = 0; u < 16; ++u) o[u] = (s0 + u < ns) ? __ldcg(po + (size_t)(s0 + u) * G * ATT_D) : 0.f;
#pragma unroll
            for (int u = 0; u < 16; ++u)
                if (s0 + u < ns) acc = fmaf(f[s0 + u], o[u], acc);
        }
        p.out[((size_t)kvh * G + g) * ATT_D + d] = acc / Ls[g];
    }
    if (tid == 0) p.counters[kvh] = 0;
}

inline size_t attn_smem_bytes() { return (size_t)ATT_WARPS * AttnSmemLayout::WARP_FLOATS * sizeof(float); }

}  // namespace mf
