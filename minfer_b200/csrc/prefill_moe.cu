// Batched prefill of a MoE FFN layer (include/minfer_cuda.h, "Batched prefill").
//
// The reference runs each prompt token through Qwen3MoE::cpu_forward
// (src/models/qwen3/module.cpp:440-476): router scores over the normalised
// x, top-k with renormalised weights, then for each selected expert in slot
// order x += w_s * down_e(silu(gate_e(xn)) * up_e(xn)). Here all n prompt
// tokens of a layer go at once:
//   1. mf_prefill_moe_route   scores [n][E] = xn . W_router^T in fp32 (SIMT:
//                             the selection must see fp32 scores) and the
//                             reference's top-k + softmax per token;
//   2. mf_prefill_moe_group   a counting sort of the n*k (token, slot) pairs
//                             by expert (the experts stored here): per expert
//                             its rows [rows[e], rows[e+1]) of the grouped
//                             buffers and its GEMM tiles;
//   3. mf_prefill_moe_gather  each token's normalised row, split into bf16
//                             hi/lo, written to its k grouped rows;
//   4. mf_prefill_gemm_grouped (prefill.cu) gate/up with the SwiGLU epilogue
//                             and the down projection, one tcgen05 tile per
//                             (expert, 128 rows, 256 columns);
//   5. mf_prefill_moe_combine x[t] += w_s * y[row(t, s)] for s = 0..k-1 in
//                             slot order (the reference's order).
// Under expert parallelism every rank holds every token's row (attention is
// replicated), routes them all identically, runs only its experts, combines
// its slots into a partial from zero, and the ranks' partials are summed into
// the residual by the bulk all-reduce of the dense tensor-parallel prefill.
// Rows of one expert are independent in the GEMMs, so the order the counting
// sort assigns within an expert does not change any result.
#include <cuda_runtime.h>

#include <algorithm>

#include "minfer_cuda.h"
#include "prefill_gemm.cuh"
#include "topk.cuh"

namespace mf {
int record_error(int code, const char* msg);  // capi.cu
cudaStream_t resolve_stream(void* stream);    // capi.cu
}  // namespace mf

namespace mf {

constexpr int MR_TOK = 16;   // tokens per CTA
constexpr int MR_BK = 16;    // K per step
constexpr int MR_MAXE = 256;

// scores of MR_TOK tokens x E experts, then the top-k of each token.
// Thread t: tokens 2 (t / 32) and 2 (t / 32) + 1, experts 4 (t % 32) + 128 j.
__global__ void __launch_bounds__(256) moe_route_prefill_kernel(const float* __restrict__ xn,
                                                                const float* __restrict__ w, int n, int d,
                                                                int n_experts, int k, int* __restrict__ ids,
                                                                float* __restrict__ weights) {
    __shared__ __align__(16) float xs[MR_BK][MR_TOK];
    __shared__ __align__(16) float ws[MR_BK][MR_MAXE];
    __shared__ float sc[MR_TOK][MR_MAXE + 1];
    __shared__ float sel_v[8][32];
    __shared__ int sel_i[8][32];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int t0 = blockIdx.x * MR_TOK;
    const int tp = tid >> 5, eg = tid & 31;
    constexpr int EJ = MR_MAXE / 128;
    float acc[EJ][2][4] = {};
    for (int k0 = 0; k0 < d; k0 += MR_BK) {
        // x tile, transposed: xs[kk][token]
        for (int i = tid; i < MR_TOK * MR_BK; i += 256) {
            const int tk = i / MR_BK, kk = i % MR_BK;
            xs[kk][tk] = (t0 + tk < n && k0 + kk < d) ? xn[(size_t)(t0 + tk) * d + k0 + kk] : 0.f;
        }
        // router tile, transposed: ws[kk][expert]
        for (int i = tid; i < n_experts * MR_BK; i += 256) {
            const int e = i / MR_BK, kk = i % MR_BK;
            ws[kk][e] = (k0 + kk < d) ? __ldg(w + (size_t)e * d + k0 + kk) : 0.f;
        }
        __syncthreads();
#pragma unroll 4
        for (int kk = 0; kk < MR_BK; ++kk) {
            const float2 xv = *reinterpret_cast<const float2*>(&xs[kk][2 * tp]);
#pragma unroll
            for (int j = 0; j < EJ; ++j) {
                const int e0 = 4 * eg + 128 * j;
                if (e0 >= n_experts) continue;
                const float4 wv = *reinterpret_cast<const float4*>(&ws[kk][e0]);
                acc[j][0][0] = fmaf(xv.x, wv.x, acc[j][0][0]);
                acc[j][0][1] = fmaf(xv.x, wv.y, acc[j][0][1]);
                acc[j][0][2] = fmaf(xv.x, wv.z, acc[j][0][2]);
                acc[j][0][3] = fmaf(xv.x, wv.w, acc[j][0][3]);
                acc[j][1][0] = fmaf(xv.y, wv.x, acc[j][1][0]);
                acc[j][1][1] = fmaf(xv.y, wv.y, acc[j][1][1]);
                acc[j][1][2] = fmaf(xv.y, wv.z, acc[j][1][2]);
                acc[j][1][3] = fmaf(xv.y, wv.w, acc[j][1][3]);
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int j = 0; j < EJ; ++j)
#pragma unroll
        for (int u = 0; u < 4; ++u) {
            const int e = 4 * eg + 128 * j + u;
            if (e < n_experts) {
                sc[2 * tp][e] = acc[j][0][u];
                sc[2 * tp + 1][e] = acc[j][1][u];
            }
        }
    __syncthreads();
    // top-k + softmax per token: warp w takes tokens w and w + 8
    for (int tk = warp; tk < MR_TOK; tk += 8) {
        const int t = t0 + tk;
        if (t >= n) break;
        topk_softmax_warp([&](int e) { return sc[tk][e]; }, n_experts, k, ids + (size_t)t * k,
                          weights + (size_t)t * k, sel_v[warp], sel_i[warp]);
        __syncwarp();
    }
    (void)lane;
}

// Counting sort of the n*k (token, slot) pairs by expert, one CTA, over the
// experts stored here: [e_lo, e_lo + n_local) (all of them on one GPU; a
// rank's share under expert parallelism). rows[e]: first grouped row of local
// expert e (rows[n_local] = the pairs routed here); tiles[e]: its first
// 128-row GEMM tile; pos[t*k + s]: the grouped row of (t, s), -1 when its
// expert is stored elsewhere.
__global__ void __launch_bounds__(1024) moe_group_kernel(const int* __restrict__ ids, int nk, int e_lo, int n_local,
                                                         int* __restrict__ rows, int* __restrict__ tiles,
                                                         int* __restrict__ pos) {
    __shared__ int cnt[MR_MAXE], cur[MR_MAXE];
    pdl_launch_dependents();
    pdl_wait();
    const int tid = threadIdx.x;
    for (int e = tid; e < n_local; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < nk; i += blockDim.x) {
        const int e = ids[i] - e_lo;
        if (e >= 0 && e < n_local) atomicAdd(&cnt[e], 1);
    }
    __syncthreads();
    if (tid == 0) {
        int r = 0, tl = 0;
        for (int e = 0; e < n_local; ++e) {
            rows[e] = r;
            tiles[e] = tl;
            cur[e] = r;
            r += cnt[e];
            tl += (cnt[e] + PG_BM - 1) / PG_BM;
        }
        rows[n_local] = r;
        tiles[n_local] = tl;
    }
    __syncthreads();
    for (int i = tid; i < nk; i += blockDim.x) {
        const int e = ids[i] - e_lo;
        pos[i] = (e >= 0 && e < n_local) ? atomicAdd(&cur[e], 1) : -1;
    }
}

// Token t's normalised row -> bf16 hi/lo at each of its k grouped rows.
__global__ void __launch_bounds__(256) moe_gather_split_kernel(const float* __restrict__ xn,
                                                               const int* __restrict__ pos, int k, int d,
                                                               __nv_bfloat16* __restrict__ hi,
                                                               __nv_bfloat16* __restrict__ lo) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    const float* xr = xn + (size_t)t * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        __nv_bfloat16 h, l;
        split_bf16(xr[i], h, l);
        for (int s = 0; s < k; ++s) {
            const int r = pos[(size_t)t * k + s];
            if (r < 0) continue;  // expert stored on another rank
            hi[(size_t)r * d + i] = h;
            lo[(size_t)r * d + i] = l;
        }
    }
}

// x_out[t] = x_in[t] (or 0) + w[t][s] * y[pos(t, s)] for s = 0..k-1 in order,
// skipping slots whose expert is stored elsewhere
// (src/models/qwen3/module.cpp:471-474: x += expert_out * weight, one expert at a time).
__global__ void __launch_bounds__(256) moe_combine_kernel(float* x_out, const float* x_in,
                                                          const float* __restrict__ y, const int* __restrict__ pos,
                                                          const float* __restrict__ weights, int k, int d) {
    pdl_launch_dependents();
    pdl_wait();
    const int t = blockIdx.x;
    for (int j = threadIdx.x; j < d; j += blockDim.x) {
        float acc = x_in ? x_in[(size_t)t * d + j] : 0.f;
        for (int s = 0; s < k; ++s) {
            const int r = pos[(size_t)t * k + s];
            if (r >= 0) acc = fmaf(y[(size_t)r * d + j], weights[(size_t)t * k + s], acc);
        }
        x_out[(size_t)t * d + j] = acc;
    }
}

}  // namespace mf

namespace {

int fail(int code, const char* msg) { return mf::record_error(code, msg); }

cudaError_t launch(const void* fn, dim3 grid, dim3 block, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = st;
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    return cudaLaunchKernelExC(&cfg, fn, args);
}

int ck(cudaError_t e) { return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e)); }

}  // namespace

extern "C" {

int mf_prefill_moe_route(int* ids, float* weights, const float* xn, const float* w_router, int n_tokens, int d_model,
                         int n_experts, int k, void* stream) {
    if (!ids || !weights || !xn || !w_router || n_tokens <= 0 || d_model <= 0)
        return fail(MF_E_INVALID, "bad arguments");
    if (n_experts < 1 || n_experts > mf::MR_MAXE || n_experts % 4 != 0)
        return fail(MF_E_UNSUPPORTED, "n_experts must be a multiple of 4 up to 256");
    if (k < 1 || k > n_experts || k > 32) return fail(MF_E_INVALID, "bad k");
    void* args[] = {(void*)&xn, (void*)&w_router, &n_tokens, &d_model, &n_experts, &k, &ids, &weights};
    return ck(launch((const void*)&mf::moe_route_prefill_kernel, dim3((n_tokens + mf::MR_TOK - 1) / mf::MR_TOK),
                     dim3(256), mf::resolve_stream(stream), args));
}

int mf_prefill_moe_group(const int* ids, int n_tokens, int k, int expert_lo, int n_local, int* rows, int* tiles,
                         int* pos, void* stream) {
    if (!ids || !rows || !tiles || !pos || n_tokens <= 0 || k <= 0 || expert_lo < 0)
        return fail(MF_E_INVALID, "bad arguments");
    if (n_local < 1 || n_local > mf::MR_MAXE) return fail(MF_E_UNSUPPORTED, "local experts must be 1..256");
    int nk = n_tokens * k;
    void* args[] = {(void*)&ids, &nk, &expert_lo, &n_local, &rows, &tiles, &pos};
    return ck(launch((const void*)&mf::moe_group_kernel, dim3(1), dim3(1024), mf::resolve_stream(stream), args));
}

int mf_prefill_moe_gather(void* a_hi, void* a_lo, const float* xn, const int* pos, int n_tokens, int k, int d_model,
                          void* stream) {
    if (!a_hi || !a_lo || !xn || !pos || n_tokens <= 0 || k <= 0 || d_model <= 0)
        return fail(MF_E_INVALID, "bad arguments");
    __nv_bfloat16* h = (__nv_bfloat16*)a_hi;
    __nv_bfloat16* l = (__nv_bfloat16*)a_lo;
    void* args[] = {(void*)&xn, (void*)&pos, &k, &d_model, &h, &l};
    return ck(launch((const void*)&mf::moe_gather_split_kernel, dim3(n_tokens), dim3(256),
                     mf::resolve_stream(stream), args));
}

int mf_prefill_moe_combine(float* x_out, const float* x_in, const float* y, const int* pos, const float* weights,
                           int n_tokens, int k, int d_model, void* stream) {
    if (!x_out || !y || !pos || !weights || n_tokens <= 0 || k <= 0 || d_model <= 0)
        return fail(MF_E_INVALID, "bad arguments");
    void* args[] = {(void*)&x_out, (void*)&x_in, (void*)&y, (void*)&pos, (void*)&weights, &k, &d_model};
    return ck(launch((const void*)&mf::moe_combine_kernel, dim3(n_tokens), dim3(256), mf::resolve_stream(stream),
                     args));
}

}  // extern "C"
