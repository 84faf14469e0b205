// Small kernels of the token loop (embedding + per-token RoPE table, router
// top-k) and the op-level kernels that mirror the reference's CPU ops one to
// one (include/minfer/ops/kernels.hpp) for known-answer parity tests.
#pragma once

#include <float.h>

#include "comm.cuh"
#include "topk.cuh"
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

// One sampled token on the device, from the candidate list the top-k kernel
// left (ids / logits sorted by logit, largest first, ties: lower id first):
// the reference's Sampler::sample after its top-k (src/base/sampler.cpp:52-117):
// softmax over the top_k, top-p cut, min-p cut, temperature softmax over the
// kept prefix, then the first candidate whose cumulative probability reaches
// the draw r = draws[i], i = the record's sample index. The chosen id becomes
// the record's token (the next frame embeds it); position, frame number and
// sample index advance. Equal logits among the top_k + 1 candidates (an order
// the reference's nth_element + sort may not share) set bit 1 of *flags; a
// sample index outside the draws sets bit 2 and leaves the record as it is.
constexpr int SAMPLE_MAX_K = 64;
__global__ void sample_step_kernel(const int* __restrict__ cand_ids, const float* __restrict__ cand_vals, int top_k,
                                   float temp, float top_p, float min_p, const float* __restrict__ draws,
                                   int n_draws, StepState* st, int* __restrict__ out_ids, int* flags) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x != 0) return;
    const int idx = st->pad[2];
    if (idx < 0 || idx >= n_draws || top_k < 1 || top_k > SAMPLE_MAX_K) {
        atomicOr(flags, 2);
        return;
    }
    for (int i = 0; i < top_k; ++i)  // the list holds top_k + 1 candidates
        if (!(cand_vals[i] != cand_vals[i + 1])) atomicOr(flags, 1);
    float pr[SAMPLE_MAX_K];
    const float top = cand_vals[0];
    int cut = top_k;
    float acc = 0.f;
    for (int i = 0; i < cut; ++i) {
        pr[i] = expf(cand_vals[i] - top);
        acc += pr[i];
    }
    for (int i = 0; i < cut; ++i) pr[i] /= acc;
    acc = 0.f;
    for (int i = 0; i < cut; ++i) {
        acc += pr[i];
        if (acc >= top_p) {
            cut = i + 1;
            break;
        }
    }
    if (min_p > 0.f) {
        const float thr = top + logf(min_p);
        for (int i = 0; i < cut; ++i)
            if (cand_vals[i] < thr) {
                cut = i;
                break;
            }
    }
    int id = cand_ids[0];
    if (cut > 0) {
        acc = 0.f;
        for (int i = 0; i < cut; ++i) {
            pr[i] = expf((cand_vals[i] - top) / temp);
            acc += pr[i];
        }
        for (int i = 0; i < cut; ++i) pr[i] /= acc;
        const float r = draws[idx];
        id = cand_ids[cut - 1];
        acc = 0.f;
        for (int i = 0; i < cut; ++i) {
            acc += pr[i];
            if (acc >= r) {
                id = cand_ids[i];
                break;
            }
        }
    } else {
        atomicOr(flags, 4);  // the filters removed every candidate (the reference throws)
    }
    out_ids[idx] = id;
    st->token = id;
    st->next_token = id;
    st->pos += 1;
    st->frame += 1;
    st->pad[2] = idx + 1;
}

__global__ void topk_softmax_kernel(const float* __restrict__ scores, int n_experts, int k, int* __restrict__ ids,
                                    float* __restrict__ weights) {
    pdl_launch_dependents();
    pdl_wait();
    if (threadIdx.x >= 32) return;
    __shared__ float sel_v[32];
    __shared__ int sel_i[32];
    topk_softmax_warp([&](int e) { return __ldcg(scores + e); }, n_experts, k, ids, weights, sel_v, sel_i);
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

// Batched-prefill all-reduce of the [rows, d] partials in the ranks' bulk
// slots, as reduce-scatter + all-gather over NVLink (each rank reads
// 2 (T-1)/T of a partial instead of T-1 partials):
//  * bulk_reduce_kernel: rank r raises its flag to `flag` in every rank's
//    region (its partial is complete: the previous kernel wrote it), waits
//    for every rank's flag, then sums slice r of all ranks' partials in rank
//    order into slice r of its own slot;
//  * bulk_gather_kernel: raises its flag to `flag` again (its reduced slice is
//    complete), waits for every rank's, then x += the reduced slices, each
//    read from the rank that owns it. Every rank adds the same values.
// Waits are bounded (on timeout: status bit COMM_STATUS_AR_TIMEOUT, and the
// kernel leaves its output alone).
MF_DEVICE bool bulk_signal_wait(const CommDev& c, unsigned long long flag, int* ok_s) {
    int* status = &c.local()->status;
    if (blockIdx.x == 0 && threadIdx.x == 0) {
        __threadfence_system();
        for (int r = 0; r < c.tp_size; ++r)
            asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(c.flags(r) + c.tp_rank), "l"(flag) : "memory");
    }
    if (threadIdx.x == 0) {
        const unsigned long long deadline = globaltimer_ns() + c.timeout_ns;
        bool late = false;
        for (int r = 0; r < c.tp_size && !late; ++r) {
            for (long long i = 0;; ++i) {
                unsigned long long v;
                asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(c.flags(c.tp_rank) + r) : "memory");
                if (v >= flag) break;
                if (i >= COMM_MAX_POLLS || globaltimer_ns() > deadline) {
                    late = true;
                    atomicOr(status, COMM_STATUS_AR_TIMEOUT);
                    break;
                }
                __nanosleep(64);
            }
        }
        *ok_s = !late;
    }
    __syncthreads();
    return *ok_s != 0;
}

// float4 groups [lo, hi) of rank r's slice
MF_DEVICE void bulk_slice(size_t n4, int r, int T, size_t& lo, size_t& hi) {
    lo = n4 * (size_t)r / (size_t)T;
    hi = n4 * (size_t)(r + 1) / (size_t)T;
}

__global__ void __launch_bounds__(256) bulk_reduce_kernel(size_t n4, const CommDev c, int slot,
                                                          unsigned long long flag) {
    __shared__ int ok;
    pdl_launch_dependents();
    pdl_wait();
    if (!bulk_signal_wait(c, flag, &ok)) return;
    size_t lo, hi;
    bulk_slice(n4, c.tp_rank, c.tp_size, lo, hi);
    float4* own = reinterpret_cast<float4*>(c.bulk(c.tp_rank, slot));
    for (size_t i = lo + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < hi; i += (size_t)gridDim.x * blockDim.x) {
        float4 a = __ldcv(reinterpret_cast<const float4*>(c.bulk(0, slot)) + i);
        for (int r = 1; r < c.tp_size; ++r) {
            const float4 b = __ldcv(reinterpret_cast<const float4*>(c.bulk(r, slot)) + i);
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
        }
        own[i] = a;
    }
}

__global__ void __launch_bounds__(256) bulk_gather_kernel(float* __restrict__ x, size_t n4, const CommDev c, int slot,
                                                          unsigned long long flag) {
    __shared__ int ok;
    pdl_launch_dependents();
    pdl_wait();
    if (!bulk_signal_wait(c, flag, &ok)) return;
    float4* x4 = reinterpret_cast<float4*>(x);
    for (int r = 0; r < c.tp_size; ++r) {
        size_t lo, hi;
        bulk_slice(n4, r, c.tp_size, lo, hi);
        const float4* src = reinterpret_cast<const float4*>(c.bulk(r, slot));
        for (size_t i = lo + (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < hi;
             i += (size_t)gridDim.x * blockDim.x) {
            const float4 b = __ldcv(src + i);
            float4 a = x4[i];
            a.x += b.x;
            a.y += b.y;
            a.z += b.z;
            a.w += b.w;
            x4[i] = a;
        }
    }
}

// ---- top-k candidates for the host sampler -------------------------------
// The k largest of x[0, n) with their indices, sorted by value (largest
// first, equal values: lower index first; NaN counts as -inf), i.e. the list
// the reference's sampler builds with nth_element + sort before its top-p /
// min-p / temperature steps (src/base/sampler.cpp:40-50). Phase 1: CTA b
// takes x[b*TOPK_CHUNK, ...) into shared memory and extracts its k best by k
// block-wide arg-max rounds; the last CTA to finish (ticket) merges the
// grid's k-lists the same way.
constexpr int TOPK_MAX = 64;
constexpr int TOPK_CHUNK = 1024;
constexpr int TOPK_THREADS = 256;

// block-wide best (value, index) of this thread's candidate; all threads get it
MF_DEVICE void block_best(float& v, int& i, float* sv, int* si) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, v, o);
        const int oi = __shfl_xor_sync(0xffffffffu, i, o);
        if (better(ov, oi, v, i)) {
            v = ov;
            i = oi;
        }
    }
    __syncthreads();
    if (lane == 0) {
        sv[warp] = v;
        si[warp] = i;
    }
    __syncthreads();
    v = sv[0];
    i = si[0];
    for (int w = 1; w < TOPK_THREADS / 32; ++w)
        if (better(sv[w], si[w], v, i)) {
            v = sv[w];
            i = si[w];
        }
}

// k rounds over the m (value, index) pairs in shared memory
MF_DEVICE void extract_topk(float* vals, int* idx, int m, int k, float* out_v, int* out_i, float* sv, int* si) {
    for (int r = 0; r < k; ++r) {
        float v = -INFINITY;
        int i = 0x7fffffff, pos = -1;
        for (int e = threadIdx.x; e < m; e += TOPK_THREADS) {
            const int id = idx[e];
            if (better(vals[e], id, v, i)) {
                v = vals[e];
                i = id;
                pos = e;
            }
        }
        int mypos = pos;
        const int myid = i;
        block_best(v, i, sv, si);
        if (mypos >= 0 && myid == i) {  // the winner leaves the pool (a sentinel never wins)
            vals[mypos] = -INFINITY;
            idx[mypos] = 0x7fffffff;
        }
        if (threadIdx.x == 0) {
            out_v[r] = v;
            out_i[r] = i;
        }
        __syncthreads();
    }
}

__global__ void __launch_bounds__(TOPK_THREADS) topk_kernel(const float* __restrict__ x, int n, int k, int* out_ids,
                                                           float* out_vals, float* cand_v, int* cand_i,
                                                           unsigned int* counter) {
    extern __shared__ float tk_smem[];
    __shared__ float sv[TOPK_THREADS / 32];
    __shared__ int si[TOPK_THREADS / 32];
    __shared__ int is_last;
    pdl_launch_dependents();
    pdl_wait();
    const int c0 = blockIdx.x * TOPK_CHUNK, m = min(TOPK_CHUNK, n - c0);
    float* vals = tk_smem;  // [TOPK_CHUNK] in phase 1, [gridDim.x * k] in phase 2
    int* ids = reinterpret_cast<int*>(tk_smem + max(TOPK_CHUNK, (int)gridDim.x * k));
    for (int e = threadIdx.x; e < m; e += TOPK_THREADS) {
        const float v = __ldcg(x + c0 + e);
        vals[e] = v == v ? v : -INFINITY;
        ids[e] = c0 + e;
    }
    __syncthreads();
    extract_topk(vals, ids, m, k, cand_v + (size_t)blockIdx.x * k, cand_i + (size_t)blockIdx.x * k, sv, si);
    __threadfence();
    __syncthreads();
    if (threadIdx.x == 0) is_last = atomicAdd(counter, 1u) == gridDim.x - 1;
    __syncthreads();
    if (!is_last) return;
    __threadfence();
    const int mc = gridDim.x * k;
    for (int e = threadIdx.x; e < mc; e += TOPK_THREADS) {
        vals[e] = __ldcg(cand_v + e);
        ids[e] = __ldcg(cand_i + e);
    }
    __syncthreads();
    extract_topk(vals, ids, mc, k, out_vals, out_ids, sv, si);
    if (threadIdx.x == 0) *counter = 0;  // ready for the next launch
}

}  // namespace mf
