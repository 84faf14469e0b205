// Small kernels of the token loop (embedding + per-token RoPE table, router
// top-k) and the op-level kernels that mirror the reference's CPU ops one to
// one (include/minfer/ops/kernels.hpp) for known-answer parity tests.
#pragma once

#include <float.h>

#include "comm.cuh"
#include "mf_common.cuh"

namespace mf {

// Per-token step state, device resident so a captured token graph can be
// replayed with new ids/positions.
struct StepState {
    int token;
    int pos;
    int next_token;  // greedy argmax of the last computed logits
    int chain;       // non-zero: the lm_head advances the record (token = next_token, pos += 1, frame += 1)
    int frame;       // frame sequence number (tags of the tensor-parallel exchange)
    int pad[3];
};
static_assert(sizeof(StepState) == MF_STEP_RECORD_BYTES, "step record layout");

// x = fp32(E[token]) (src/ops/kernels.cpp:153-187, src/base/types.cpp:14-38),
// token read from the device step record.
template <typename W>
__global__ void embed_kernel(float* __restrict__ x, const void* __restrict__ emb, int d_model, int vocab,
                             const StepState* __restrict__ st) {
    pdl_launch_dependents();
    pdl_wait();
    int token = __ldcg(&st->token);
    // the host rejects out-of-vocabulary ids; a device-produced id is in range
    // by construction, and the row read stays inside the table regardless
    if (token < 0 || token >= vocab) token = 0;
    const size_t row = (size_t)token * d_model;
    for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < d_model; i += blockDim.x * gridDim.x) {
        float v;
        if (W::CODE == MF_F32) v = reinterpret_cast<const float*>(emb)[row + i];
        else if (W::CODE == MF_BF16) v = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(emb)[row + i] << 16);
        else v = __half2float(reinterpret_cast<const __half*>(emb)[row + i]);
        x[i] = v;
    }
}

// Router top-k + renormalisation for one token, one warp
// (src/ops/kernels.cpp:113-139): k passes of "first strictly greater" over
// unvisited experts starting from (index 0, -FLT_MAX), then a max-subtracted
// softmax over the k selected raw logits (src/ops/kernels.cpp:31-49).
__global__ void topk_softmax_kernel(const float* __restrict__ scores, int n_experts, int k, int* __restrict__ ids,
                                    float* __restrict__ weights) {
    constexpr int MAXE = 8;  // experts per lane (n_experts <= 256)
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31;
    if (threadIdx.x >= 32) return;
    float v[MAXE];
    bool used[MAXE];
#pragma unroll
    for (int i = 0; i < MAXE; ++i) {
        const int e = lane + 32 * i;
        v[i] = e < n_experts ? __ldcg(scores + e) : -INFINITY;
        used[i] = e >= n_experts;
    }
    __shared__ float sel_v[32];
    __shared__ int sel_i[32];
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

// ------------------------------------------------------------------------
// Op-level kernels with the reference's exact signatures and semantics.
// They serve the known-answer tests and the single-op C-ABI entry points;
// the token loop uses the fused kernels instead.

// rmsnorm over `rows` independent vectors of length dim (src/ops/kernels.cpp:351-365)
__global__ void rmsnorm_rows_kernel(float* out, const float* in, const float* w, int dim, float eps) {
    __shared__ float scratch[32];
    const float* xi = in + (size_t)blockIdx.x * dim;
    float* xo = out + (size_t)blockIdx.x * dim;
    float ss = 0.f;
    for (int i = threadIdx.x; i < dim; i += blockDim.x) ss = fmaf(xi[i], xi[i], ss);
    ss = block_sum(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / (float)dim + eps);
    __syncthreads();
    for (int i = threadIdx.x; i < dim; i += blockDim.x) xo[i] = (inv * xi[i]) * w[i];
}

// softmax over `rows` vectors (src/ops/kernels.cpp:31-49)
__global__ void softmax_rows_kernel(float* out, const float* in, int n) {
    __shared__ float scratch[32];
    const float* xi = in + (size_t)blockIdx.x * n;
    float* xo = out + (size_t)blockIdx.x * n;
    float mx = -FLT_MAX;
    for (int i = threadIdx.x; i < n; i += blockDim.x) mx = fmaxf(mx, xi[i]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -FLT_MAX;
    for (int i = 0; i < (int)((blockDim.x + 31) >> 5); ++i) mx = fmaxf(mx, scratch[i]);
    __syncthreads();
    float s = 0.f;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float e = expf(xi[i] - mx);
        xo[i] = e;
        s += e;
    }
    s = block_sum(s, scratch);
    const float inv = 1.0f / s;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xo[i] *= inv;
}

__global__ void silu_kernel(float* out, const float* in, int n) {
    for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < n; i += blockDim.x * gridDim.x) out[i] = silu(in[i]);
}

// NeoX / interleaved RoPE of one head (src/ops/kernels.cpp:51-81); like the
// reference, dims at or past d_rot are not written.
__global__ void rope_head_kernel(float* out, const float* in, int head, int d_head, int d_rot, float base, int pos,
                                 int neox) {
    const float* hi = in + (size_t)head * d_head;
    float* ho = out + (size_t)head * d_head;
    const int half = d_rot / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        // float pow/cos/sin (the overloads the reference's unqualified calls
        // resolve to with <math.h> in scope)
        const float freq = 1.0f / powf(base, 2.0f * (float)i / (float)d_rot);
        const float angle = (float)pos * freq;
        const float c = cosf(angle), s = sinf(angle);
        const int a = neox ? i : 2 * i, b = neox ? i + half : 2 * i + 1;
        const float x0 = hi[a], x1 = hi[b];  // each thread owns its pair: in-place safe
        if (neox) {  // first product fused, as the reference's build evaluates it
            ho[a] = fmaf(c, x0, -__fmul_rn(s, x1));
            ho[b] = fmaf(s, x0, __fmul_rn(c, x1));
        } else {  // separate roundings
            ho[a] = __fsub_rn(__fmul_rn(c, x0), __fmul_rn(s, x1));
            ho[b] = __fadd_rn(__fmul_rn(s, x0), __fmul_rn(c, x1));
        }
    }
}

// Single-head attention with the reference's signature (src/ops/kernels.cpp:83-110):
// scores[pos] = softmax(q.k_pos * 1/sqrtf(d_head)), out = sum scores[pos] v_pos.
// One CTA; K/V rows are kv_dim floats apart.
__global__ void attn_head_kernel(float* scores, float* out, const float* q, const float* k, const float* v,
                                 int seq_len, int d_head, int kv_dim) {
    __shared__ float scratch[32];
    const float scale = 1.0f / sqrtf((float)d_head);
    for (int p = threadIdx.x; p < seq_len; p += blockDim.x) {
        float s = 0.f;
        for (int d = 0; d < d_head; ++d) s = fmaf(q[d], k[(size_t)p * kv_dim + d], s);
        scores[p] = s * scale;
    }
    __syncthreads();
    float mx = -FLT_MAX;
    for (int p = threadIdx.x; p < seq_len; p += blockDim.x) mx = fmaxf(mx, scores[p]);
    mx = warp_max(mx);
    if ((threadIdx.x & 31) == 0) scratch[threadIdx.x >> 5] = mx;
    __syncthreads();
    mx = -FLT_MAX;
    for (int i = 0; i < (int)((blockDim.x + 31) >> 5); ++i) mx = fmaxf(mx, scratch[i]);
    __syncthreads();
    float s = 0.f;
    for (int p = threadIdx.x; p < seq_len; p += blockDim.x) {
        const float e = expf(scores[p] - mx);
        scores[p] = e;
        s += e;
    }
    s = block_sum(s, scratch);
    const float inv = 1.0f / s;
    for (int p = threadIdx.x; p < seq_len; p += blockDim.x) scores[p] *= inv;
    __syncthreads();
    for (int d = threadIdx.x; d < d_head; d += blockDim.x) {
        float o = 0.f;
        for (int p = 0; p < seq_len; ++p) o = fmaf(scores[p], v[(size_t)p * kv_dim + d], o);
        out[d] = o;
    }
}

// One embedding row widened to fp32 (src/ops/kernels.cpp:174-187).
template <typename W>
__global__ void embed_row_kernel(float* x, const void* emb, uint32_t token, int d_model) {
    const size_t row = (size_t)token * d_model;
    for (int i = threadIdx.x + blockIdx.x * blockDim.x; i < d_model; i += blockDim.x * gridDim.x) {
        float v;
        if (W::CODE == MF_F32) v = reinterpret_cast<const float*>(emb)[row + i];
        else if (W::CODE == MF_BF16) v = __uint_as_float((uint32_t)reinterpret_cast<const uint16_t*>(emb)[row + i] << 16);
        else v = __half2float(reinterpret_cast<const __half*>(emb)[row + i]);
        x[i] = v;
    }
}

// Greedy argmax over n logits (first maximum), single CTA.
__global__ void argmax_kernel(const float* logits, int n, int* out) {
    __shared__ float sv[32];
    __shared__ int si[32];
    float bv = -INFINITY;
    int bi = 0x7fffffff;
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
        const float v = logits[i];
        if (better(v, i, bv, bi)) { bv = v; bi = i; }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
        if (better(ov, oi, bv, bi)) { bv = ov; bi = oi; }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = bv;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        bv = sv[0];
        bi = si[0];
        for (int w = 1; w < (int)(blockDim.x >> 5); ++w) {
            if (better(sv[w], si[w], bv, bi)) { bv = sv[w]; bi = si[w]; }
        }
        *out = bi;
    }
}

// Stand-alone all-reduce of an n-float vector in one CTA: push `partial` as
// tagged words into every rank's slot, then x_out = x_res + partial_0 +
// partial_1 + ... (rank order) as the words arrive (bounded waits).
__global__ void __launch_bounds__(1024) allreduce_kernel(const float* partial, const float* x_res, float* x_out, int n,
                                                         const CommDev c, int seq, const StepState* st) {
    const int tid = threadIdx.x;
    pdl_launch_dependents();
    pdl_wait();
    const uint32_t tag = comm_tag(__ldcg(&st->frame), seq);
    const int slot = seq & 1;
    for (int i = tid; i < n; i += blockDim.x) {
        const unsigned long long w = tagged(__ldcg(partial + i), tag);
        for (int r = 0; r < c.tp_size; ++r) st_tagged(c.recv(r, slot, c.tp_rank) + i, w);
    }
    int* status = &c.local()->status;
    const unsigned long long deadline = globaltimer_ns() + c.timeout_ns;
    bool late = false;
    recv_sum(c, slot, tag, x_res, tid, blockDim.x, n, deadline, &late, status, [&](int i, float v) { x_out[i] = v; });
}

}  // namespace mf
