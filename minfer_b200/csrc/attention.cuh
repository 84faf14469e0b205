// Decode attention for one token: per-head Q/K RMSNorm + NeoX RoPE + KV-cache
// append + GQA attention over the HBM-resident KV cache, as one kernel. The
// cache holds fp32 rows (the reference's format) or, opt-in, bf16 rows
// (rounded to nearest even at the append; read back widened exactly, all
// arithmetic in fp32).
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
//  * grid = (n_split, n_kv_heads), 8 warps per CTA, two CTAs per SM; each CTA
//    serves ALL kv_mul query heads of its KV head over one contiguous slice of
//    positions, so every K/V row is read from HBM exactly once per token.
//  * The cache layout is [kv_head][position][d_head]: a slice is one
//    contiguous run of rows, streamed as 32-row tiles (16 KB fp32, 8 KB
//    bf16) through an 80 KB CTA-wide cp.async ring (5 or 10 stages) with one
//    barrier per tile.
//  * Two phases per 256-position super-chunk: (1) the K tiles -> scaled
//    scores of every query head into shared memory (8 lanes per position,
//    16 dims each, finished by a reduce-scatter over the 8 lanes); (2) one
//    CTA-wide softmax step (running max, rescale factor, exponentials in
//    place), then the V tiles -> P.V with the probabilities read as
//    broadcast float4s (each warp owns 4 rows of a tile, each lane 4 dims).
//    All warps share the CTA's running max, so warp partials just add.
//  * Slices are merged with the usual (max, sum, vector) rescaling by the CTA
//    that finishes last for its KV head, which pulls every partial in with one
//    burst of copies and merges in a fixed order (deterministic; no waits).
#pragma once

#include "mf_common.cuh"

namespace mf {

constexpr int ATT_D = 128;          // head dim (Qwen3)
constexpr int ATT_TILE = 32;        // positions per pipeline tile
constexpr int ATT_TILE_FLOATS = ATT_TILE * ATT_D;
constexpr int ATT_WARPS = 8;
constexpr int ATT_STAGES = 5;
constexpr int ATT_CTAS_PER_SM = 2;
constexpr int ATT_SC_TILES = 8;     // tiles per super-chunk
constexpr int ATT_SC = ATT_SC_TILES * ATT_TILE;
constexpr int ATT_SC_STRIDE = ATT_SC + 4;  // per-head score row (padded against bank conflicts)
constexpr int ATT_MIN_CHUNK = 64;   // fewest positions per split
constexpr int ATT_MAX_SPLIT = 128;  // merge tables live in the score area
// Per query head, the score area holds one super-chunk of scores and, in the
// merge, (m, l) and a scale factor per slice.
constexpr int ATT_HEAD_AREA = ATT_SC_STRIDE > 3 * ATT_MAX_SPLIT ? ATT_SC_STRIDE : 3 * ATT_MAX_SPLIT;
constexpr int ATT_PF_ROWS = 128;    // rows of K and of V prefetched into L2 before the dependency wait
// A merging CTA pulls partials through its ring in batches of NB = ring /
// (G * D) slices. More than two batches' worth of slices are merged in two
// levels instead: the last CTA of each group of min(NB, 16) slices merges the
// group, the last group merger merges the groups (a single CTA merging 128
// slices of 8 heads took longer than streaming them).
constexpr int ATT_MERGE_GROUP = 16;
constexpr int ATT_MAX_GROUPS = 16;  // ATT_MAX_SPLIT / (smallest group, 10 slices for 16 heads), rounded up

struct AttnParams {
    const float* qkv;        // [Hq*D | Hkv*D | Hkv*D] (this rank's heads)
    const float* q_norm_w;   // [D]
    const float* k_norm_w;   // [D]
    float eps;
    const float2* rope;      // [max_seq][D/2] (cos, sin) per position and pair
    void* k_cache;           // this layer: [Hkv][max_seq][D] of KV (float or bf16)
    void* v_cache;
    int max_seq;
    const int* pos_ptr;      // current position (device)
    float* out;              // [Hq*D]
    float* part_o;           // [Hkv][n_split][G][D]
    float* part_ml;          // [Hkv][n_split][G][2]
    int* counters;           // [Hkv] then [Hkv][ATT_MAX_GROUPS], zero-initialised, reset by the mergers
    float* group_o;          // [Hkv][ATT_MAX_GROUPS][G][D] merged groups (two-level merge)
    float* group_ml;         // [Hkv][ATT_MAX_GROUPS][G][2]
    int n_heads;
    int n_kv_heads;
    int n_split;
};

MF_DEVICE void cp_async16(void* smem, const void* gmem) {
    const unsigned s = (unsigned)__cvta_generic_to_shared(smem);
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
MF_DEVICE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N> MF_DEVICE void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

MF_DEVICE float f4_get(const float4& v, int i) { return i == 0 ? v.x : (i == 1 ? v.y : (i == 2 ? v.z : v.w)); }

// Four consecutive cache elements widened to fp32 (bf16 -> fp32 is exact: the
// 16 bits become the high half of the float), and their store.
MF_DEVICE float4 kv_ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
MF_DEVICE float4 kv_ld4(const __nv_bfloat16* p) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
}
MF_DEVICE void kv_ld16(const float* p, float4 (&o)[1]) { o[0] = *reinterpret_cast<const float4*>(p); }
MF_DEVICE void kv_ld16(const __nv_bfloat16* p, float4 (&o)[2]) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    o[0] = make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xffff0000u), __uint_as_float(u.y << 16),
                       __uint_as_float(u.y & 0xffff0000u));
    o[1] = make_float4(__uint_as_float(u.z << 16), __uint_as_float(u.z & 0xffff0000u), __uint_as_float(u.w << 16),
                       __uint_as_float(u.w & 0xffff0000u));
}
MF_DEVICE void kv_st4(float* p, float4 v) { *reinterpret_cast<float4*>(p) = v; }
MF_DEVICE void kv_st4(__nv_bfloat16* p, float4 v) {
    const __nv_bfloat162 a = __floats2bfloat162_rn(v.x, v.y), b = __floats2bfloat162_rn(v.z, v.w);
    uint2 u;
    u.x = *reinterpret_cast<const uint32_t*>(&a);
    u.y = *reinterpret_cast<const uint32_t*>(&b);
    *reinterpret_cast<uint2*>(p) = u;
}

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

// Split geometry for a context of `len` positions: effective slice count
// (slices of at least ATT_MIN_CHUNK positions, tile-aligned, none empty) and
// this slice's [start, end). The last slice ends at len and so owns len - 1.
struct AttnSlice {
    int eff, start, end;
};
MF_DEVICE AttnSlice attn_slice(int len, int n_split, int split) {
    int eff = min(n_split, max(1, (len + ATT_MIN_CHUNK - 1) / ATT_MIN_CHUNK));
    int chunk = (len + eff - 1) / eff;
    chunk = (chunk + ATT_TILE - 1) / ATT_TILE * ATT_TILE;
    eff = (len + chunk - 1) / chunk;
    const int start = split * chunk;
    return {eff, start, min(start + chunk, len)};
}

// Walks a slice's copy sequence: per super-chunk its K tiles, then its V
// tiles. Advanced once per tile by the producer and by the consumer alike.
struct AttnSeq {
    int sc_row0;  // first row of the current super-chunk
    int t;        // tile within the K or V run
    int n_sc;     // tiles in this super-chunk
    bool is_v;
    MF_DEVICE void init(int start, int end) {
        sc_row0 = start;
        t = 0;
        is_v = false;
        n_sc = min(ATT_SC_TILES, (end - start + ATT_TILE - 1) / ATT_TILE);
    }
    MF_DEVICE int row0() const { return sc_row0 + t * ATT_TILE; }
    MF_DEVICE void advance(int end) {
        if (++t < n_sc) return;
        t = 0;
        if (!is_v) {
            is_v = true;
        } else {
            is_v = false;
            sc_row0 += ATT_SC;
            n_sc = min(ATT_SC_TILES, (end - sc_row0 + ATT_TILE - 1) / ATT_TILE);
        }
    }
};

// Score lanes keep their query slices in registers when all heads' slices
// take at most MF_ATT_QREG_FLOATS floats; otherwise they read them from
// shared memory (broadcast within each quarter-warp, conflict-free across it).
#ifndef MF_ATT_QREG_FLOATS
#define MF_ATT_QREG_FLOATS 64
#endif

template <int G, typename KV>
__global__ void __launch_bounds__(ATT_WARPS * 32, (G <= 8 ? ATT_CTAS_PER_SM : 1)) attn_decode_kernel(const AttnParams p) {
    static_assert(G >= 1 && G <= 16 && (G & (G - 1)) == 0, "power-of-two query groups");
    constexpr int NT = ATT_WARPS * 32;
    constexpr int RB = ATT_D * (int)sizeof(KV);  // bytes per cache row
    constexpr int TB = ATT_TILE * RB;            // bytes per tile
    // the ring keeps the same bytes for either element type (5 fp32 or 10 bf16 tiles)
    constexpr int STAGES = ATT_STAGES * ATT_TILE_FLOATS * (int)sizeof(float) / TB;
    extern __shared__ float4 att_smem4[];
    float* ring = reinterpret_cast<float*>(att_smem4);      // [STAGES][TB bytes]; later merge staging
    float* sc_s = ring + ATT_STAGES * ATT_TILE_FLOATS;       // [G][ATT_SC_STRIDE] within [G][ATT_HEAD_AREA]
    __shared__ __align__(16) float q_s[G][ATT_D];
    __shared__ __align__(16) KV knew_s[ATT_D], vnew_s[ATT_D];  // row `pos` as stored, never re-read from HBM
    __shared__ float m_s[G], l_s[G], a_s[G];
    __shared__ int is_last;

    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int split = blockIdx.x, kvh = blockIdx.y;
    const int Hq = p.n_heads, Hkv = p.n_kv_heads;
    const size_t head_stride = (size_t)p.max_seq * ATT_D;
    const KV* kc = reinterpret_cast<const KV*>(p.k_cache) + (size_t)kvh * head_stride;
    const KV* vc = reinterpret_cast<const KV*>(p.v_cache) + (size_t)kvh * head_stride;

    // Before the dependency wait nothing produced by earlier kernels may be
    // used; a possibly stale position only steers an L2 prefetch of cache rows
    // (clamped into this head's cache, so always in bounds).
    if (tid == 0) {
        const int ps = min(max(__ldcg(p.pos_ptr), 0), p.max_seq - 1);
        const AttnSlice sl = attn_slice(ps + 1, p.n_split, split);
        if (split < sl.eff && sl.end > sl.start) {
            const uint32_t nb = (uint32_t)min(sl.end - sl.start, ATT_PF_ROWS) * RB;
            prefetch_l2(kc + (size_t)sl.start * ATT_D, nb);
            prefetch_l2(vc + (size_t)sl.start * ATT_D, nb);
        }
    }
    pdl_launch_dependents();
    pdl_wait();

    const int pos = __ldcg(p.pos_ptr);
    if (pos < 0 || pos >= p.max_seq) {  // no such cache row: write nothing but a zero output
        if (split == 0)
            for (int i = tid; i < G * ATT_D; i += NT) p.out[(size_t)kvh * G * ATT_D + i] = 0.f;
        return;
    }
    const int len = pos + 1;
    const AttnSlice sl = attn_slice(len, p.n_split, split);
    if (split >= sl.eff) return;
    const int start = sl.start, end = sl.end, nrows = end - start;
    const int nseq = 2 * ((nrows + ATT_TILE - 1) / ATT_TILE);
    const float2* cs = p.rope + (size_t)pos * (ATT_D / 2);
    // Row `pos` (the last row of the last slice) is appended by this kernel;
    // its values are taken from shared memory, so it is never copied.
    const int copy_end = (end == len) ? end - 1 : end;

    // Copy pieces: LPRC threads move one row (16 bytes each); thread tid moves
    // column chunk tid % LPRC of tile rows tid / LPRC + CP_ROWS * i.
    constexpr int LPRC = RB / 16;
    constexpr int CP_ROWS = NT / LPRC;  // rows per copy instruction
    const int crow = tid / LPRC;
    const int toff = crow * ATT_D + (tid % LPRC) * (16 / (int)sizeof(KV));
    AttnSeq ps;  // producer position
    ps.init(start, end);
    int pslot = 0;
    auto issue = [&](int q) {
        if (q < nseq) {
            const int row0 = ps.row0();
            KV* dst = reinterpret_cast<KV*>(ring) + pslot * (TB / (int)sizeof(KV)) + toff;
            const KV* src = (ps.is_v ? vc : kc) + (size_t)row0 * ATT_D + toff;
            const int ncopy = copy_end - row0;
            if (ncopy >= ATT_TILE) {
#pragma unroll
                for (int i = 0; i < ATT_TILE / CP_ROWS; ++i)
                    cp_async16(dst + i * CP_ROWS * ATT_D, src + (size_t)i * CP_ROWS * ATT_D);
            } else {
#pragma unroll
                for (int i = 0; i < ATT_TILE / CP_ROWS; ++i)
                    if (crow + i * CP_ROWS < ncopy) cp_async16(dst + i * CP_ROWS * ATT_D, src + (size_t)i * CP_ROWS * ATT_D);
            }
            ps.advance(end);
        }
        cp_async_commit();  // one group per sequence slot, empty groups included
        pslot = (pslot + 1 == STAGES) ? 0 : pslot + 1;
    };
#pragma unroll 1
    for (int q = 0; q < STAGES - 1; ++q) issue(q);

    // ---- prologue: normalised + rotated queries; the KV append
    for (int g = warp; g < G; g += ATT_WARPS) {
        const int h = kvh * G + g;
        const float4 v = __ldcg(reinterpret_cast<const float4*>(p.qkv + (size_t)h * ATT_D) + lane);
        *reinterpret_cast<float4*>(&q_s[g][4 * lane]) = norm_rope_head(v, p.q_norm_w, p.eps, cs, lane);
    }
    if (end == len && warp == ATT_WARPS - 1) {
        const float* kraw = p.qkv + (size_t)Hq * ATT_D + (size_t)kvh * ATT_D;
        const float* vraw = p.qkv + (size_t)(Hq + Hkv) * ATT_D + (size_t)kvh * ATT_D;
        const float4 k = norm_rope_head(__ldcg(reinterpret_cast<const float4*>(kraw) + lane), p.k_norm_w, p.eps,
                                        cs, lane);
        const float4 v = __ldcg(reinterpret_cast<const float4*>(vraw) + lane);
        const size_t row = (size_t)kvh * head_stride + (size_t)pos * ATT_D + 4 * lane;
        kv_st4(reinterpret_cast<KV*>(p.k_cache) + row, k);
        kv_st4(reinterpret_cast<KV*>(p.v_cache) + row, v);
        kv_st4(knew_s + 4 * lane, k);
        kv_st4(vnew_s + 4 * lane, v);
    }
    if (tid < G) {
        m_s[tid] = -INFINITY;
        l_s[tid] = 0.f;
    }
    __syncthreads();

    const float scale = 1.0f / sqrtf((float)ATT_D);  // src/ops/kernels.cpp:88
    // score mapping: LPR lanes per tile row, each summing DPL dims
    // {4*(c + LPR*j) + e}; a quarter-warp reads 128 contiguous bytes of one row
    // (each lane loads 16 bytes of a row at a time: EPL elements = NQ4 float4s)
    constexpr int LPR = G >= 8 ? 16 : 8;
    constexpr int EPL = 16 / (int)sizeof(KV);
    constexpr int NQ4 = EPL / 4;
    constexpr int NJ = ATT_D / EPL / LPR;  // 16-byte loads per lane and row
    constexpr int RPP = NT / LPR;          // rows per pass
    constexpr int NP = ATT_TILE / RPP;     // passes per tile
    const int r_k = tid / LPR, c = tid % LPR;
    constexpr bool QREG = G * NJ * EPL <= MF_ATT_QREG_FLOATS;
    constexpr int QG = QREG ? G : 1;
    float4 qreg[QG][NJ * NQ4];
    if constexpr (QREG) {
#pragma unroll
        for (int g = 0; g < G; ++g)
#pragma unroll
            for (int j = 0; j < NJ; ++j)
#pragma unroll
                for (int u = 0; u < NQ4; ++u)
                    qreg[g][j * NQ4 + u] = *reinterpret_cast<const float4*>(&q_s[g][EPL * (c + LPR * j) + 4 * u]);
    }
    // after the reduce-scatter a lane holds the sums of heads h_lane .. h_lane + HPL - 1
    constexpr int HPL = G >= LPR ? G / LPR : 1;
    constexpr int LPH = G >= LPR ? 1 : LPR / G;  // lanes holding each head
    int h_lane = 0;
    {
        int n = G;
#pragma unroll
        for (int m = LPR / 2; m >= 1; m >>= 1)
            if (n >= 2) {
                n >>= 1;
                if (c & m) h_lane += n;
            }
    }

    float4 o[G];
#pragma unroll
    for (int g = 0; g < G; ++g) o[g] = make_float4(0.f, 0.f, 0.f, 0.f);

    AttnSeq cq;  // consumer position
    cq.init(start, end);
    int cslot = 0;
#pragma unroll 1
    for (int q = 0; q < nseq; ++q) {
        cp_async_wait<STAGES - 2>();
        __syncthreads();  // tile q landed for every thread; slot (q - 1) is free
        issue(q + STAGES - 1);
        const KV* tile = reinterpret_cast<const KV*>(ring) + cslot * (TB / (int)sizeof(KV));
        const int row0 = cq.row0();
        const int nvalid = min(ATT_TILE, end - row0);  // rows of the slice in this tile
        const bool has_pos = pos < row0 + ATT_TILE && pos >= row0;
        if (!cq.is_v) {
            // ---- phase 1: scores of this tile's rows
#pragma unroll
            for (int pp = 0; pp < NP; ++pp) {
                const int r = r_k + pp * RPP;
                float sv[G];
#pragma unroll
                for (int g = 0; g < G; ++g) sv[g] = 0.f;
                if (r < nvalid) {
                    const KV* krow = tile + r * ATT_D + EPL * c;
                    if (has_pos && row0 + r == pos) krow = knew_s + EPL * c;
#pragma unroll
                    for (int j = 0; j < NJ; ++j) {
                        float4 k4[NQ4];
                        kv_ld16(krow + EPL * LPR * j, k4);
#pragma unroll
                        for (int u = 0; u < NQ4; ++u)
#pragma unroll
                            for (int g = 0; g < G; ++g) {
                                float4 q4;
                                if constexpr (QREG) q4 = qreg[g][j * NQ4 + u];
                                else q4 = *reinterpret_cast<const float4*>(&q_s[g][EPL * (c + LPR * j) + 4 * u]);
                                sv[g] = fmaf(q4.x, k4[u].x, sv[g]);
                                sv[g] = fmaf(q4.y, k4[u].y, sv[g]);
                                sv[g] = fmaf(q4.z, k4[u].z, sv[g]);
                                sv[g] = fmaf(q4.w, k4[u].w, sv[g]);
                            }
                    }
                }
                // reduce-scatter over the LPR lanes of the row (xor LPR/2 .. 1)
                int n = G;
#pragma unroll
                for (int m = LPR / 2; m >= 1; m >>= 1) {
                    if (n >= 2) {
                        const int hn = n >> 1;
                        const bool upper = (c & m) != 0;
#pragma unroll
                        for (int i = 0; i < hn; ++i) {
                            const float send = upper ? sv[i] : sv[i + hn];
                            const float keep = upper ? sv[i + hn] : sv[i];
                            sv[i] = keep + __shfl_xor_sync(0xffffffffu, send, m);
                        }
                        n = hn;
                    } else {
                        sv[0] += __shfl_xor_sync(0xffffffffu, sv[0], m);
                    }
                }
                if (c % LPH == 0) {
                    const int col = cq.t * ATT_TILE + r;
                    const bool valid = r < nvalid;
#pragma unroll
                    for (int i = 0; i < HPL; ++i)
                        sc_s[(h_lane + i) * ATT_SC_STRIDE + col] = valid ? sv[i] * scale : -INFINITY;
                }
            }
        } else {
            if (cq.t == 0) {
                // ---- softmax step over the super-chunk (every K tile done: barrier above)
                const int rows_sc = min(ATT_SC, end - cq.sc_row0);
                for (int g = warp; g < G; g += ATT_WARPS) {
                    float* srow = sc_s + g * ATT_SC_STRIDE;
                    float mx = -INFINITY;
                    for (int i = lane; i < rows_sc; i += 32) mx = fmaxf(mx, srow[i]);
                    mx = warp_max(mx);
                    const float m_old = m_s[g];
                    const float mn = fmaxf(m_old, mx);
                    float sum = 0.f;
                    for (int i = lane; i < rows_sc; i += 32) {
                        const float e = expf(srow[i] - mn);
                        srow[i] = e;
                        sum += e;
                    }
                    sum = warp_sum(sum);
                    if (lane == 0) {
                        const float a = (m_old == -INFINITY) ? 0.f : expf(m_old - mn);
                        a_s[g] = a;
                        l_s[g] = fmaf(l_s[g], a, sum);
                        m_s[g] = mn;
                    }
                }
                __syncthreads();
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float a = a_s[g];
                    o[g].x *= a; o[g].y *= a; o[g].z *= a; o[g].w *= a;
                }
            }
            // ---- phase 2: P.V, warp rows rb .. rb + 3, lane dims 4*lane .. 4*lane + 3
            const int rb = 4 * warp;
            const float* prow = sc_s + cq.t * ATT_TILE + rb;
            if (nvalid == ATT_TILE && !has_pos) {
                float4 v4[4];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) v4[rr] = kv_ld4(tile + (rb + rr) * ATT_D + 4 * lane);
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 pv = *reinterpret_cast<const float4*>(prow + g * ATT_SC_STRIDE);
                    const float pr[4] = {pv.x, pv.y, pv.z, pv.w};
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        o[g].x = fmaf(pr[rr], v4[rr].x, o[g].x);
                        o[g].y = fmaf(pr[rr], v4[rr].y, o[g].y);
                        o[g].z = fmaf(pr[rr], v4[rr].z, o[g].z);
                        o[g].w = fmaf(pr[rr], v4[rr].w, o[g].w);
                    }
                }
            } else if (rb < nvalid) {
                // partial tile or the tile holding `pos`: rows past the slice end
                // were never copied (weight 0, zeros), row `pos` comes from vnew_s
                float4 v4[4];
#pragma unroll
                for (int rr = 0; rr < 4; ++rr) {
                    const KV* vrow = (row0 + rb + rr == pos) ? vnew_s : tile + (rb + rr) * ATT_D;
                    v4[rr] = (rb + rr < nvalid) ? kv_ld4(vrow + 4 * lane) : make_float4(0.f, 0.f, 0.f, 0.f);
                }
#pragma unroll
                for (int g = 0; g < G; ++g) {
                    const float4 pv = *reinterpret_cast<const float4*>(prow + g * ATT_SC_STRIDE);
                    const float pr[4] = {pv.x, rb + 1 < nvalid ? pv.y : 0.f, rb + 2 < nvalid ? pv.z : 0.f,
                                         rb + 3 < nvalid ? pv.w : 0.f};
#pragma unroll
                    for (int rr = 0; rr < 4; ++rr) {
                        o[g].x = fmaf(pr[rr], v4[rr].x, o[g].x);
                        o[g].y = fmaf(pr[rr], v4[rr].y, o[g].y);
                        o[g].z = fmaf(pr[rr], v4[rr].z, o[g].z);
                        o[g].w = fmaf(pr[rr], v4[rr].w, o[g].w);
                    }
                }
            }
        }
        cq.advance(end);
        cslot = (cslot + 1 == STAGES) ? 0 : cslot + 1;
    }
    cp_async_wait<0>();

    // ---- sum the warps' accumulators (they share the CTA's running max)
    __syncthreads();
    float* wo = ring;  // [ATT_WARPS][G][D]
#pragma unroll
    for (int g = 0; g < G; ++g) reinterpret_cast<float4*>(wo + ((size_t)warp * G + g) * ATT_D)[lane] = o[g];
    __syncthreads();
    if (sl.eff == 1) {  // one slice: finish here, no partials
        for (int idx = tid; idx < G * ATT_D; idx += NT) {
            const int g = idx / ATT_D;
            float acc = 0.f;
#pragma unroll
            for (int w = 0; w < ATT_WARPS; ++w) acc += wo[(size_t)w * G * ATT_D + idx];
            p.out[(size_t)kvh * G * ATT_D + idx] = acc / l_s[g];
        }
        return;
    }
    const size_t pbase = ((size_t)kvh * p.n_split + split) * G;
    for (int idx = tid; idx < G * ATT_D; idx += NT) {
        float acc = 0.f;
#pragma unroll
        for (int w = 0; w < ATT_WARPS; ++w) acc += wo[(size_t)w * G * ATT_D + idx];
        p.part_o[pbase * ATT_D + idx] = acc;
    }
    if (tid < G) {
        p.part_ml[(pbase + tid) * 2 + 0] = m_s[tid];
        p.part_ml[(pbase + tid) * 2 + 1] = l_s[tid];
    }

    // ---- merge: the last CTA of this KV head (or, with more than
    // ATT_MERGE_GROUP slices, of this slice's group, then the last of the
    // group mergers) combines partials with the (max, sum, vector) rescaling
    constexpr int NB = (ATT_STAGES * ATT_TILE_FLOATS) / (G * ATT_D);
    constexpr int MG = NB < ATT_MERGE_GROUP ? NB : ATT_MERGE_GROUP;
    static_assert((ATT_MAX_SPLIT + MG - 1) / MG <= ATT_MAX_GROUPS, "merge groups");
    const int ns = sl.eff;
    const bool two = ns > 2 * NB;
    const int grp = split / MG;
    const int ngroups = (ns + MG - 1) / MG;
    int* gcnt = p.counters + Hkv + (size_t)kvh * ATT_MAX_GROUPS + grp;
    __syncthreads();
    if (tid == 0) {
        __threadfence();
        const int gsz = two ? min(MG, ns - grp * MG) : ns;
        const int ticket = atomicAdd(two ? gcnt : p.counters + kvh, 1);
        is_last = (ticket == gsz - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    float* ml = sc_s;    // [n][G][2], then the scale factors [n][G] (n <= ATT_MAX_SPLIT: both fit G * ATT_HEAD_AREA)
    float* fs = sc_s + 2 * ATT_MAX_SPLIT * G;
    float* po = ring;    // a batch of partial outputs [nb][G][D]
    constexpr int PER = (G * ATT_D / 4 + NT - 1) / NT;
    // Merges n partials (src_o [n][G][D], src_ml [n][G][2]); final: writes the
    // normalised output, else the merged partial (dst_o [G][D], dst_ml [G][2]).
    auto merge = [&](const float* src_o, const float* src_ml, int n, bool final, float* dst_o, float* dst_ml) {
        auto issue_batch = [&](int s0) {
            const int nb = min(NB, n - s0);
            const float* src = src_o + (size_t)s0 * G * ATT_D;
            for (int i = tid; i < nb * G * ATT_D / 4; i += NT) cp_async16(po + 4 * i, src + 4 * i);
            cp_async_commit();
        };
        issue_batch(0);
        for (int i = tid; i < n * G * 2; i += NT) ml[i] = __ldcg(src_ml + i);
        __syncthreads();
        // per head: max, per-partial factors, denominator (one warp per head)
        for (int g = warp; g < G; g += ATT_WARPS) {
            float M = -INFINITY;
            for (int s0 = lane; s0 < n; s0 += 32) M = fmaxf(M, ml[(s0 * G + g) * 2]);
            M = warp_max(M);
            float L = 0.f;
            for (int s0 = lane; s0 < n; s0 += 32) {
                const float ms = ml[(s0 * G + g) * 2];
                const float f = (ms == -INFINITY) ? 0.f : expf(ms - M);
                fs[s0 * G + g] = f;
                L = fmaf(f, ml[(s0 * G + g) * 2 + 1], L);
            }
            L = warp_sum(L);
            if (lane == 0) {
                a_s[g] = L;
                m_s[g] = M;
            }
        }
        // every thread owns float4 outputs idx4 = tid + k*NT of [G][D/4]
        float4 acc[PER];
#pragma unroll
        for (int k = 0; k < PER; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
        for (int s0 = 0; s0 < n; s0 += NB) {
            cp_async_wait<0>();
            __syncthreads();
            const int nb = min(NB, n - s0);
#pragma unroll
            for (int k = 0; k < PER; ++k) {
                const int idx4 = tid + k * NT;
                if (idx4 < G * ATT_D / 4) {
                    const int g = idx4 / (ATT_D / 4);
                    for (int b = 0; b < nb; ++b) {
                        const float f = fs[(s0 + b) * G + g];
                        const float4 v = reinterpret_cast<const float4*>(po + (size_t)b * G * ATT_D)[idx4];
                        acc[k].x = fmaf(f, v.x, acc[k].x);
                        acc[k].y = fmaf(f, v.y, acc[k].y);
                        acc[k].z = fmaf(f, v.z, acc[k].z);
                        acc[k].w = fmaf(f, v.w, acc[k].w);
                    }
                }
            }
            if (s0 + NB < n) {
                __syncthreads();  // the batch buffer is refilled
                issue_batch(s0 + NB);
            }
        }
#pragma unroll
        for (int k = 0; k < PER; ++k) {
            const int idx4 = tid + k * NT;
            if (idx4 < G * ATT_D / 4) {
                const float L = a_s[idx4 / (ATT_D / 4)];
                reinterpret_cast<float4*>(dst_o)[idx4] =
                    final ? make_float4(acc[k].x / L, acc[k].y / L, acc[k].z / L, acc[k].w / L) : acc[k];
            }
        }
        if (!final && tid < G) {
            dst_ml[tid * 2 + 0] = m_s[tid];
            dst_ml[tid * 2 + 1] = a_s[tid];
        }
        __syncthreads();  // smem staging is reused by a following merge
    };
    const size_t hb = (size_t)kvh * p.n_split * G;
    float* out = p.out + (size_t)kvh * G * ATT_D;
    if (!two) {
        merge(p.part_o + hb * ATT_D, p.part_ml + hb * 2, ns, true, out, nullptr);
        if (tid == 0) p.counters[kvh] = 0;
        return;
    }
    // level 1: this group's slices -> group partial
    const size_t gb = ((size_t)kvh * ATT_MAX_GROUPS + grp) * G;
    const int gs0 = grp * MG, gsz = min(MG, ns - gs0);
    merge(p.part_o + (hb + (size_t)gs0 * G) * ATT_D, p.part_ml + (hb + (size_t)gs0 * G) * 2, gsz, false,
          p.group_o + gb * ATT_D, p.group_ml + gb * 2);
    if (tid == 0) {
        *gcnt = 0;
        __threadfence();
        is_last = (atomicAdd(p.counters + kvh, 1) == ngroups - 1);
    }
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    // level 2: the groups -> output
    const size_t g0 = (size_t)kvh * ATT_MAX_GROUPS * G;
    merge(p.group_o + g0 * ATT_D, p.group_ml + g0 * 2, ngroups, true, out, nullptr);
    if (tid == 0) p.counters[kvh] = 0;
}

inline size_t attn_smem_bytes(int G) {
    return ((size_t)ATT_STAGES * ATT_TILE_FLOATS + (size_t)G * ATT_HEAD_AREA) * sizeof(float);
}
// Largest n_split the merge supports.
inline int attn_max_split(int G) { return ATT_MAX_SPLIT; }

// Workspace layout (byte offsets): counters | per-slice (m, l) | per-slice
// outputs | per-group (m, l) | per-group outputs. Every part 256-byte aligned.
struct AttnWsLayout {
    size_t cnt, ml, o, gml, go, total;
};
inline AttnWsLayout attn_ws_layout(int n_kv_heads, int n_split, int G) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    AttnWsLayout L;
    const size_t H = (size_t)n_kv_heads;
    L.cnt = 0;
    L.ml = al(H * (1 + ATT_MAX_GROUPS) * sizeof(int));
    L.o = L.ml + al(H * n_split * G * 2 * sizeof(float));
    L.gml = L.o + al(H * n_split * G * ATT_D * sizeof(float));
    const bool two = n_split > 2 * ((ATT_STAGES * ATT_TILE_FLOATS) / (G * ATT_D));
    L.go = L.gml + (two ? al(H * ATT_MAX_GROUPS * G * 2 * sizeof(float)) : 0);
    L.total = L.go + (two ? al(H * ATT_MAX_GROUPS * G * ATT_D * sizeof(float)) : 0);
    return L;
}

}  // namespace mf
