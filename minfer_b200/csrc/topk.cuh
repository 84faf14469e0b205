// The reference's router top-k as a warp-level device function (shared by the
// decode router kernels and the batched-prefill router).
#pragma once

#include <float.h>

#include "mf_common.cuh"

namespace mf {

// Router top-k + renormalisation for one token, one warp
// (src/ops/kernels.cpp:113-139): k passes of "first strictly greater" over
// unvisited experts starting from (index 0, -FLT_MAX), then a max-subtracted
// softmax over the k selected raw logits (src/ops/kernels.cpp:31-49).
// score(e) returns expert e's logit (e < n_experts <= 256); lane 0 writes.
template <typename F>
MF_DEVICE void topk_softmax_warp(F score, int n_experts, int k, int* __restrict__ ids, float* __restrict__ weights,
                                 float* sel_v, int* sel_i) {
    constexpr int MAXE = 8;  // experts per lane (n_experts <= 256)
    const int lane = threadIdx.x & 31;
    float v[MAXE];
    bool used[MAXE];
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < n_experts ? score(e) : -INFINITY;
        used[i] = e >= n_experts;
    }
    for (int r = 0; r < k; ++r) {
        float bv = -FLT_MAX;
        int bi = 0x7fffffff;  // "none" (loses every comparison against a real candidate)
#pragma unroll
        for (int i = 0; i < MAXE; ++i) {
            if (!used[i] && v[i] > bv) {  // strict: first index wins among equals in this lane
                bv = v[i];
                bi = lane + 32 * i;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
        }
        if (bi == 0x7fffffff) {  // nothing above -FLT_MAX: the reference keeps best = 0
            bi = 0;
            bv = -FLT_MAX;
        }
        if ((bi & 31) == lane) used[bi >> 5] = true;
        if (lane == 0) {
            sel_v[r] = bv;
            sel_i[r] = bi;
        }
    }
    __syncwarp();
    if (lane == 0) {
        float mx = -FLT_MAX;
        for (int r = 0; r < k; ++r) mx = sel_v[r] > mx ? sel_v[r] : mx;
        float out[32];
        float sum = 0.f;
        for (int r = 0; r < k; ++r) {
            out[r] = expf(sel_v[r] - mx);
            sum += out[r];
        }
        const float inv = 1.0f / sum;
        for (int r = 0; r < k; ++r) {
            ids[r] = sel_i[r];
            weights[r] = out[r] * inv;
        }
    }
}

}  // namespace mf
