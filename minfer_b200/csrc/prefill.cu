// Batched prefill entry points (include/minfer_cuda.h, "Batched prefill").
// The reference prefills token by token (src/base/model.cpp:120-129); these
// kernels process all prompt tokens of a layer at once: row-wise RMSNorm and
// fp32 -> bf16 hi/lo split, the tcgen05 GEMM (prefill_gemm.cuh), per-token
// Q/K RMSNorm + RoPE + KV-cache write, and causal attention.
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <mutex>

#include "minfer_cuda.h"
#include "prefill_attn.cuh"
#include "prefill_fa.cuh"
#include "prefill_gemm.cuh"

namespace mf {
int record_error(int code, const char* msg);  // capi.cu: message for mf_last_error
cudaStream_t resolve_stream(void* stream);    // capi.cu: NULL -> manager stream of the current device
}  // namespace mf

namespace {

__device__ int g_prefill_status;  // bit 1: a tcgen05 GEMM wait gave up

int fail(int code, const char* msg) { return mf::record_error(code, msg); }

bool pdl_on() {
    const char* e = std::getenv("MF_PDL");
    return !(e && e[0] == '0');
}

unsigned long long timeout_ns() {
    const char* e = std::getenv("MF_PREFILL_TIMEOUT_MS");
    const long v = (e && *e) ? std::atol(e) : 2000;
    return 1000000ull * (unsigned long long)(v > 0 ? v : 2000);
}

cudaError_t launch(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t st, void** args) {
    cudaLaunchConfig_t cfg = {};
    cudaLaunchAttribute at[1];
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    if (pdl_on()) {
        at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        at[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = at;
        cfg.numAttrs = 1;
    }
    return cudaLaunchKernelExC(&cfg, fn, args);
}

int set_smem(const void* fn, size_t smem) {
    static std::mutex mu;
    std::lock_guard<std::mutex> lk(mu);
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

using EncodeFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                              const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                              CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver entry point is looked up at run time, so the library loads (and
// its CPU-side checks run) on machines without a driver.
EncodeFn tmap_encoder() {
    static EncodeFn encode = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            encode = (EncodeFn)fn;
    });
    return encode;
}

// 16-bit (bf16 or fp16) tensor map of rank 2 or 3 (dims[0] innermost, strides in bytes of
// dims 1..rank-1), 128-byte swizzle, zero fill out of bounds. The box's inner
// extent is 64 elements (128 bytes).
int make_tmap_nd(CUtensorMap* tm, const void* base, int rank, const uint64_t* dims, const uint64_t* strides,
                 const uint32_t* box, CUtensorMapDataType dtype = CU_TENSOR_MAP_DATA_TYPE_BFLOAT16) {
    if (((uintptr_t)base & 15) != 0) return fail(MF_E_INVALID, "16-bit operand must be 16-byte aligned");
    for (int i = 0; i + 1 < rank; ++i)
        if (strides[i] % 16 != 0) return fail(MF_E_INVALID, "16-bit operand strides must be multiples of 16 bytes");
    EncodeFn encode = tmap_encoder();
    if (!encode) return fail(MF_E_CUDA, "cuTensorMapEncodeTiled is not available");
    cuuint64_t d[3], st[2];
    cuuint32_t bx[3], es[3] = {1, 1, 1};
    for (int i = 0; i < rank; ++i) {
        d[i] = dims[i];
        bx[i] = box[i];
    }
    for (int i = 0; i + 1 < rank; ++i) st[i] = strides[i];
    CUresult r = encode(tm, dtype, (cuuint32_t)rank, const_cast<void*>(base), d, st, bx,
                        es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? MF_OK : fail(MF_E_CUDA, "cuTensorMapEncodeTiled failed");
}

// 2-D bf16 tensor map over a row-major [rows, cols] matrix: 64-column
// (128-byte) x box_rows boxes.
int make_tmap(CUtensorMap* tm, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows) {
    if ((cols * 2) % 16 != 0) return fail(MF_E_INVALID, "bf16 operand row length must be a multiple of 8");
    const uint64_t dims[2] = {cols, rows}, strides[1] = {cols * 2};
    const uint32_t box[2] = {64, box_rows};
    return make_tmap_nd(tm, base, 2, dims, strides, box);
}

int* status_ptr() {
    static int* p[64] = {nullptr};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return nullptr;
    if (!p[dev]) cudaGetSymbolAddress((void**)&p[dev], g_prefill_status);
    return p[dev];
}

}  // namespace

// ---------------------------------------------------------------- row kernels
namespace mf {

// out = rmsnorm(x) * w split into bf16 hi/lo, one CTA per row
// (src/ops/kernels.cpp:351-365: inv = 1/sqrtf(sum(x^2)/n + eps); out = inv*x*w).
// Rows of a multiple of 4 elements go 16 bytes at a time (float4 loads,
// 8-byte stores of four bf16); other widths element by element.
__global__ void __launch_bounds__(256) norm_split_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                         float eps, int d, __nv_bfloat16* hi, __nv_bfloat16* lo,
                                                         float* xn) {
    __shared__ float scratch[32];
    pdl_launch_dependents();
    pdl_wait();
    const size_t r0 = (size_t)blockIdx.x * d;
    const float* xr = x + r0;
    const bool vec = (d & 3) == 0;
    float ss = 0.f;
    if (vec) {
        for (int i = 4 * threadIdx.x; i < d; i += 4 * blockDim.x) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            ss = fmaf(v.x, v.x, ss);
            ss = fmaf(v.y, v.y, ss);
            ss = fmaf(v.z, v.z, ss);
            ss = fmaf(v.w, v.w, ss);
        }
    } else {
        for (int i = threadIdx.x; i < d; i += blockDim.x) ss = fmaf(xr[i], xr[i], ss);
    }
    ss = block_sum(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / (float)d + eps);
    if (vec) {
        for (int i = 4 * threadIdx.x; i < d; i += 4 * blockDim.x) {
            const float4 v = *reinterpret_cast<const float4*>(xr + i);
            const float4 g = *reinterpret_cast<const float4*>(w + i);
            const float o[4] = {(inv * v.x) * g.x, (inv * v.y) * g.y, (inv * v.z) * g.z, (inv * v.w) * g.w};
            if (xn) *reinterpret_cast<float4*>(xn + r0 + i) = make_float4(o[0], o[1], o[2], o[3]);
            __nv_bfloat16 h[4], l[4];
#pragma unroll
            for (int e = 0; e < 4; ++e) split_bf16(o[e], h[e], l[e]);
            *reinterpret_cast<uint2*>(hi + r0 + i) =
                make_uint2((uint32_t)__bfloat16_as_ushort(h[0]) | ((uint32_t)__bfloat16_as_ushort(h[1]) << 16),
                           (uint32_t)__bfloat16_as_ushort(h[2]) | ((uint32_t)__bfloat16_as_ushort(h[3]) << 16));
            *reinterpret_cast<uint2*>(lo + r0 + i) =
                make_uint2((uint32_t)__bfloat16_as_ushort(l[0]) | ((uint32_t)__bfloat16_as_ushort(l[1]) << 16),
                           (uint32_t)__bfloat16_as_ushort(l[2]) | ((uint32_t)__bfloat16_as_ushort(l[3]) << 16));
        }
    } else {
        for (int i = threadIdx.x; i < d; i += blockDim.x) {
            const float v = (inv * xr[i]) * w[i];
            if (xn) xn[r0 + i] = v;
            split_bf16(v, hi[r0 + i], lo[r0 + i]);
        }
    }
}

// x[t] = embedding row tokens[t] (widened to fp32), one CTA per token; an id
// outside [0, vocab) reads row 0 (src/models/qwen3/module.cpp:13-44).
template <typename W>
__global__ void __launch_bounds__(256) prefill_embed_kernel(float* __restrict__ x, const void* __restrict__ emb,
                                                            const uint32_t* __restrict__ tokens, int vocab, int d) {
    pdl_launch_dependents();
    pdl_wait();
    uint32_t tok = tokens[blockIdx.x];
    if (tok >= (uint32_t)vocab) tok = 0;
    float* xr = x + (size_t)blockIdx.x * d;
    const typename W::T* row = reinterpret_cast<const typename W::T*>(emb) + (size_t)tok * d;
    for (int i = threadIdx.x; i < d; i += blockDim.x) {
        if constexpr (W::CODE == MF_F32) xr[i] = row[i];
        else if constexpr (W::CODE == MF_BF16) xr[i] = __uint_as_float((uint32_t)row[i] << 16);
        else xr[i] = __half2float(__ushort_as_half(row[i]));
    }
}

// plain fp32 -> bf16 hi/lo split of n elements
__global__ void split_kernel(const float* __restrict__ x, size_t n, __nv_bfloat16* hi, __nv_bfloat16* lo) {
    pdl_launch_dependents();
    pdl_wait();
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        split_bf16(x[i], hi[i], lo[i]);
}

// h = silu(g) * u of interleaved gate/up rows gu [n_rows][2 d_ff] (columns
// 2i, 2i+1 = g_i, u_i), written as the down GEMM's bf16 hi/lo operands [n_rows][d_ff]
__global__ void swiglu_split_kernel(const float* __restrict__ gu, size_t n_rows, int d_ff, __nv_bfloat16* hi,
                                    __nv_bfloat16* lo) {
    pdl_launch_dependents();
    pdl_wait();
    const size_t n = n_rows * (size_t)d_ff;
    for (size_t i = (size_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float2 g_u = reinterpret_cast<const float2*>(gu)[i];
        split_bf16(silu(g_u.x) * g_u.y, hi[i], lo[i]);  // src/models/qwen3/module.cpp:466-468
    }
}

}  // namespace mf

extern "C" {

int mf_prefill_swiglu_split(void* h_hi, void* h_lo, const float* gate_up, int n_rows, int d_ff, void* stream) {
    if (!h_hi || !h_lo || !gate_up || n_rows <= 0 || d_ff <= 0) return fail(MF_E_INVALID, "bad arguments");
    if (((uintptr_t)gate_up & 7) != 0) return fail(MF_E_INVALID, "gate_up must be 8-byte aligned");
    const float* g = gate_up;
    size_t rows = (size_t)n_rows;
    int F = d_ff;
    __nv_bfloat16* h = (__nv_bfloat16*)h_hi;
    __nv_bfloat16* l = (__nv_bfloat16*)h_lo;
    void* args[] = {(void*)&g, (void*)&rows, (void*)&F, (void*)&h, (void*)&l};
    const size_t n = rows * (size_t)d_ff;
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    cudaError_t e = launch((const void*)&mf::swiglu_split_kernel, dim3(blocks), dim3(256), 0,
                           mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_gemm(float* y, int ldy, const void* a_hi, const void* a_lo, const void* w, int M, int N, int K,
                    int mode, void* h_hi, void* h_lo, void* stream) {
    if (!a_hi || !a_lo || !w || M <= 0 || N <= 0 || K <= 0) return fail(MF_E_INVALID, "bad GEMM arguments");
    if (K % 8 != 0) return fail(MF_E_INVALID, "K must be a multiple of 8");
    if (mode == mf::PG_SWIGLU_SPLIT) {
        if (!h_hi || !h_lo || N % 2 != 0) return fail(MF_E_INVALID, "SwiGLU mode needs hi/lo outputs and even N");
    } else if (mode == mf::PG_STORE || mode == mf::PG_RESID) {
        if (!y || ldy < N || ((uintptr_t)y & 15) != 0 || ldy % 4 != 0)
            return fail(MF_E_INVALID, "output must be 16-byte aligned with ldy >= N, ldy % 4 == 0");
    } else {
        return fail(MF_E_INVALID, "unknown GEMM mode");
    }
    int* status = status_ptr();
    if (!status) return fail(MF_E_CUDA, "prefill status symbol");
    CUtensorMap ta_hi, ta_lo, tw;
    int rc = make_tmap(&ta_hi, a_hi, (uint64_t)M, (uint64_t)K, mf::PG_BM);
    if (!rc) rc = make_tmap(&ta_lo, a_lo, (uint64_t)M, (uint64_t)K, mf::PG_BM);
    if (!rc) rc = make_tmap(&tw, w, (uint64_t)N, (uint64_t)K, mf::PG_BN);
    if (rc) return rc;
    mf::PgParams p = {};
    p.M = M;
    p.N = N;
    p.K = K;
    p.y = y;
    p.ldy = ldy;
    p.h_hi = (__nv_bfloat16*)h_hi;
    p.h_lo = (__nv_bfloat16*)h_lo;
    p.status = status;
    p.timeout_ns = timeout_ns();
    const void* fn = mode == mf::PG_STORE  ? (const void*)&mf::prefill_gemm_kernel<mf::PG_STORE>
                     : mode == mf::PG_RESID ? (const void*)&mf::prefill_gemm_kernel<mf::PG_RESID>
                                            : (const void*)&mf::prefill_gemm_kernel<mf::PG_SWIGLU_SPLIT>;
    rc = set_smem(fn, mf::PG_SMEM_BYTES);
    if (rc) return rc;
    void* args[] = {&ta_hi, &ta_lo, &tw, &p};
    const dim3 grid((N + mf::PG_BN - 1) / mf::PG_BN, (M + mf::PG_BM - 1) / mf::PG_BM);
    cudaError_t e = launch(fn, grid, dim3(mf::PG_THREADS), mf::PG_SMEM_BYTES, mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_gemm_grouped(float* y, int ldy, const void* a_hi, const void* a_lo, const void* w, int n_groups,
                            int rows_cap, int N, int K, const int* grp_rows, const int* grp_tiles, int mode, void* h_hi,
                            void* h_lo, void* stream) {
    if (!a_hi || !a_lo || !w || !grp_rows || !grp_tiles || n_groups <= 0 || rows_cap <= 0 || N <= 0 || K <= 0)
        return fail(MF_E_INVALID, "bad grouped GEMM arguments");
    if (K % 8 != 0) return fail(MF_E_INVALID, "K must be a multiple of 8");
    if ((long long)n_groups * N > (1ll << 31) - 1) return fail(MF_E_INVALID, "n_groups * N too large");
    if (mode == mf::PG_SWIGLU_SPLIT) {
        if (!h_hi || !h_lo || N % 2 != 0) return fail(MF_E_INVALID, "SwiGLU mode needs hi/lo outputs and even N");
    } else if (mode == mf::PG_STORE || mode == mf::PG_RESID) {
        if (!y || ldy < N || ((uintptr_t)y & 15) != 0 || ldy % 4 != 0)
            return fail(MF_E_INVALID, "output must be 16-byte aligned with ldy >= N, ldy % 4 == 0");
    } else {
        return fail(MF_E_INVALID, "unknown GEMM mode");
    }
    int* status = status_ptr();
    if (!status) return fail(MF_E_CUDA, "prefill status symbol");
    CUtensorMap ta_hi, ta_lo, tw;
    int rc = make_tmap(&ta_hi, a_hi, (uint64_t)rows_cap, (uint64_t)K, mf::PG_BM);
    if (!rc) rc = make_tmap(&ta_lo, a_lo, (uint64_t)rows_cap, (uint64_t)K, mf::PG_BM);
    if (!rc) rc = make_tmap(&tw, w, (uint64_t)n_groups * (uint64_t)N, (uint64_t)K, mf::PG_BN);
    if (rc) return rc;
    mf::PgParams p = {};
    p.M = rows_cap;
    p.N = N;
    p.K = K;
    p.grp_rows = grp_rows;
    p.grp_tiles = grp_tiles;
    p.n_groups = n_groups;
    p.y = y;
    p.ldy = ldy;
    p.h_hi = (__nv_bfloat16*)h_hi;
    p.h_lo = (__nv_bfloat16*)h_lo;
    p.status = status;
    p.timeout_ns = timeout_ns();
    const void* fn = mode == mf::PG_STORE  ? (const void*)&mf::prefill_gemm_kernel<mf::PG_STORE>
                     : mode == mf::PG_RESID ? (const void*)&mf::prefill_gemm_kernel<mf::PG_RESID>
                                            : (const void*)&mf::prefill_gemm_kernel<mf::PG_SWIGLU_SPLIT>;
    rc = set_smem(fn, mf::PG_SMEM_BYTES);
    if (rc) return rc;
    void* args[] = {&ta_hi, &ta_lo, &tw, &p};
    // every group's tiles fit in ceil(rows / BM) + n_groups CTA rows; the
    // CTAs past the last tile leave at once
    const dim3 grid((N + mf::PG_BN - 1) / mf::PG_BN, (rows_cap + mf::PG_BM - 1) / mf::PG_BM + n_groups);
    cudaError_t e = launch(fn, grid, dim3(mf::PG_THREADS), mf::PG_SMEM_BYTES, mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_norm_split(void* hi, void* lo, float* xn, const float* x, const float* norm_w, float eps, int d,
                          int n_rows, void* stream) {
    if (!hi || !lo || !x || !norm_w || d <= 0 || n_rows <= 0) return fail(MF_E_INVALID, "bad arguments");
    if ((d & 3) == 0 && (((uintptr_t)hi | (uintptr_t)lo) & 7 || ((uintptr_t)x | (uintptr_t)norm_w | (uintptr_t)xn) & 15))
        return fail(MF_E_INVALID, "rows of a multiple of 4 need 16-byte aligned x/norm_w/xn and 8-byte aligned hi/lo");
    const float* xa = x;
    const float* wa = norm_w;
    __nv_bfloat16* h = (__nv_bfloat16*)hi;
    __nv_bfloat16* l = (__nv_bfloat16*)lo;
    void* args[] = {(void*)&xa, (void*)&wa, (void*)&eps, (void*)&d, (void*)&h, (void*)&l, (void*)&xn};
    cudaError_t e = launch((const void*)&mf::norm_split_kernel, dim3(n_rows), dim3(256), 0,
                           mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_split(void* hi, void* lo, const float* x, size_t n, void* stream) {
    if (!hi || !lo || !x || n == 0) return fail(MF_E_INVALID, "bad arguments");
    const float* xa = x;
    __nv_bfloat16* h = (__nv_bfloat16*)hi;
    __nv_bfloat16* l = (__nv_bfloat16*)lo;
    void* args[] = {(void*)&xa, (void*)&n, (void*)&h, (void*)&l};
    const unsigned blocks = (unsigned)std::min<size_t>((n + 255) / 256, 148 * 8);
    cudaError_t e = launch((const void*)&mf::split_kernel, dim3(blocks), dim3(256), 0, mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_embed(float* x, const void* emb, int dtype, int vocab, int d_model, const uint32_t* tokens, int n_tokens,
                     void* stream) {
    if (!x || !emb || !tokens || vocab <= 0 || d_model <= 0 || n_tokens <= 0) return fail(MF_E_INVALID, "bad arguments");
    const void* fn = dtype == MF_F32    ? (const void*)&mf::prefill_embed_kernel<mf::W_F32>
                     : dtype == MF_F16  ? (const void*)&mf::prefill_embed_kernel<mf::W_F16>
                     : dtype == MF_BF16 ? (const void*)&mf::prefill_embed_kernel<mf::W_BF16>
                                        : nullptr;
    if (!fn) return fail(MF_E_INVALID, "bad dtype");
    void* args[] = {(void*)&x, (void*)&emb, (void*)&tokens, (void*)&vocab, (void*)&d_model};
    cudaError_t e = launch(fn, dim3(n_tokens), dim3(256), 0, mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_qkv_post(float* q_out, void* k_cache, void* v_cache, const float* qkv, const float* q_norm_w,
                        const float* k_norm_w, float eps, const void* rope_table, int max_seq, int n_heads,
                        int n_kv_heads, int d_head, int n_tokens, int pos0, int kv_dtype, void* stream) {
    if (!q_out || !k_cache || !v_cache || !qkv || !q_norm_w || !k_norm_w || !rope_table || n_tokens <= 0 || pos0 < 0)
        return fail(MF_E_INVALID, "bad arguments");
    if (d_head != mf::ATT_D) return fail(MF_E_UNSUPPORTED, "d_head must be 128");
    if (kv_dtype != MF_F32 && kv_dtype != MF_BF16) return fail(MF_E_UNSUPPORTED, "KV cache dtype (f32 or bf16)");
    if (pos0 + n_tokens > max_seq) return fail(MF_E_INVALID, "prompt runs past max_seq");
    const float2* rope = (const float2*)rope_table;
    void* args[] = {(void*)&qkv, (void*)&q_norm_w, (void*)&k_norm_w, (void*)&eps, (void*)&rope, (void*)&q_out,
                    (void*)&k_cache, (void*)&v_cache, (void*)&max_seq, (void*)&n_heads, (void*)&n_kv_heads,
                    (void*)&pos0};
    const void* fn = kv_dtype == MF_F32 ? (const void*)&mf::prefill_qkv_post_kernel<float>
                                        : (const void*)&mf::prefill_qkv_post_kernel<__nv_bfloat16>;
    const unsigned hy = (unsigned)((n_heads + n_kv_heads + mf::QP_WARPS - 1) / mf::QP_WARPS);
    cudaError_t e = launch(fn, dim3(n_tokens, hy), dim3(mf::QP_WARPS * 32), 0, mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

extern "C++" {
template <typename KV>
static const void* prefill_attn_ptr(int G) {
    return G == 1    ? (const void*)&mf::prefill_attn_kernel<1, KV>
           : G == 2  ? (const void*)&mf::prefill_attn_kernel<2, KV>
           : G == 4  ? (const void*)&mf::prefill_attn_kernel<4, KV>
           : G == 8  ? (const void*)&mf::prefill_attn_kernel<8, KV>
           : G == 16 ? (const void*)&mf::prefill_attn_kernel<16, KV>
                     : nullptr;
}
}

int mf_prefill_attention(void* out_hi, void* out_lo, const float* q, const void* k_cache, const void* v_cache,
                         int max_seq, int n_tokens, int pos0, int n_heads, int n_kv_heads, int d_head, int kv_dtype,
                         void* stream) {
    if (!out_hi || !out_lo || !q || !k_cache || !v_cache || n_tokens <= 0 || pos0 < 0 || n_kv_heads <= 0 ||
        n_heads % n_kv_heads != 0)
        return fail(MF_E_INVALID, "bad arguments");
    if (d_head != mf::ATT_D) return fail(MF_E_UNSUPPORTED, "d_head must be 128");
    if (kv_dtype != MF_F32 && kv_dtype != MF_BF16) return fail(MF_E_UNSUPPORTED, "KV cache dtype (f32 or bf16)");
    if (pos0 + n_tokens > max_seq) return fail(MF_E_INVALID, "prompt runs past max_seq");
    const int G = n_heads / n_kv_heads;
    const void* fn = kv_dtype == MF_F32 ? prefill_attn_ptr<float>(G) : prefill_attn_ptr<__nv_bfloat16>(G);
    if (!fn) return fail(MF_E_UNSUPPORTED, "query heads per KV head must be 1, 2, 4, 8 or 16");
    const size_t smem = mf::pa_smem_bytes();
    int rc = set_smem(fn, smem);
    if (rc) return rc;
    const int QT = mf::PA_ROWS / G;
    __nv_bfloat16* hi = (__nv_bfloat16*)out_hi;
    __nv_bfloat16* lo = (__nv_bfloat16*)out_lo;
    void* args[] = {(void*)&q, (void*)&k_cache, (void*)&v_cache, (void*)&max_seq, (void*)&n_tokens, (void*)&pos0,
                    (void*)&n_heads, (void*)&hi, (void*)&lo};
    cudaError_t e = launch(fn, dim3((n_tokens + QT - 1) / QT, n_kv_heads), dim3(mf::PA_THREADS), smem,
                           mf::resolve_stream(stream), args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

// Scratch of mf_prefill_attention_tc: K fp16 hi/lo [Hkv][ld][128] and V^T
// bf16 hi/lo [Hkv][128][ld], ld = n_keys rounded up to 64, each section
// 256-byte aligned. (Q goes straight from the fp32 buffer into TMEM.)
static size_t fa_layout(int n_keys, int n_kv_heads, size_t off[4]) {
    const size_t ld = ((size_t)n_keys + 63) / 64 * 64;
    const size_t kv = (size_t)n_kv_heads * ld * mf::ATT_D * 2;
    size_t o = 0;
    for (int i = 0; i < 4; ++i) {
        off[i] = o;
        o += (kv + 255) / 256 * 256;
    }
    return o;
}

int mf_prefill_attention_scratch(int n_tokens, int n_keys, int n_heads, int n_kv_heads, size_t* bytes) {
    if (!bytes || n_tokens <= 0 || n_keys < n_tokens || n_heads <= 0 || n_kv_heads <= 0)
        return fail(MF_E_INVALID, "bad arguments");
    size_t off[4];
    *bytes = fa_layout(n_keys, n_kv_heads, off);
    return MF_OK;
}

int mf_prefill_attention_tc(void* out_hi, void* out_lo, const float* q, const void* k_cache, const void* v_cache,
                            int max_seq, int n_tokens, int pos0, int n_heads, int n_kv_heads, int d_head,
                            void* scratch, size_t scratch_bytes, int kv_dtype, void* stream) {
    if (!out_hi || !out_lo || !q || !k_cache || !v_cache || !scratch || n_tokens <= 0 || pos0 < 0 ||
        n_kv_heads <= 0 || n_heads % n_kv_heads != 0)
        return fail(MF_E_INVALID, "bad arguments");
    if (d_head != mf::ATT_D) return fail(MF_E_UNSUPPORTED, "d_head must be 128");
    if (kv_dtype != MF_F32 && kv_dtype != MF_BF16) return fail(MF_E_UNSUPPORTED, "KV cache dtype (f32 or bf16)");
    if (pos0 + n_tokens > max_seq) return fail(MF_E_INVALID, "prompt runs past max_seq");
    if (((uintptr_t)scratch & 255) != 0) return fail(MF_E_INVALID, "scratch must be 256-byte aligned");
    if (((uintptr_t)q & 15) != 0) return fail(MF_E_INVALID, "q must be 16-byte aligned");
    const int G = n_heads / n_kv_heads;
    const void* fn = G == 1    ? (const void*)&mf::prefill_fa_kernel<1>
                     : G == 2  ? (const void*)&mf::prefill_fa_kernel<2>
                     : G == 4  ? (const void*)&mf::prefill_fa_kernel<4>
                     : G == 8  ? (const void*)&mf::prefill_fa_kernel<8>
                     : G == 16 ? (const void*)&mf::prefill_fa_kernel<16>
                               : nullptr;
    if (!fn) return fail(MF_E_UNSUPPORTED, "query heads per KV head must be 1, 2, 4, 8 or 16");
    const int n_keys = pos0 + n_tokens;
    size_t off[4];
    if (fa_layout(n_keys, n_kv_heads, off) > scratch_bytes) return fail(MF_E_INVALID, "attention scratch too small");
    const size_t ld = ((size_t)n_keys + 63) / 64 * 64;
    uint8_t* base = (uint8_t*)scratch;
    __half *kh = (__half*)(base + off[0]), *kl = (__half*)(base + off[1]);
    __nv_bfloat16 *vh = (__nv_bfloat16*)(base + off[2]), *vl = (__nv_bfloat16*)(base + off[3]);
    CUtensorMap tk[2], tv[2];
    const uint64_t D = mf::ATT_D;
    {
        const uint64_t dims[3] = {D, (uint64_t)n_keys, (uint64_t)n_kv_heads}, strides[2] = {D * 2, ld * D * 2};
        const uint32_t box[3] = {64, mf::FA_BN, 1};
        int rc = make_tmap_nd(&tk[0], kh, 3, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
        if (!rc) rc = make_tmap_nd(&tk[1], kl, 3, dims, strides, box, CU_TENSOR_MAP_DATA_TYPE_FLOAT16);
        if (rc) return rc;
    }
    {
        const uint64_t dims[3] = {(uint64_t)n_keys, D, (uint64_t)n_kv_heads}, strides[2] = {ld * 2, D * ld * 2};
        const uint32_t box[3] = {64, (uint32_t)D, 1};
        int rc = make_tmap_nd(&tv[0], vh, 3, dims, strides, box);
        if (!rc) rc = make_tmap_nd(&tv[1], vl, 3, dims, strides, box);
        if (rc) return rc;
    }
    int rc = set_smem(fn, mf::FA_SMEM_BYTES);
    if (rc) return rc;
    int* status = status_ptr();
    if (!status) return fail(MF_E_CUDA, "prefill status symbol");
    cudaStream_t st = mf::resolve_stream(stream);
    // operands: K rows split (one warp per 128-float row), V transposed in 64-key tiles
    const int ldi = (int)ld;
    {
        const long long rows = (long long)n_kv_heads * n_keys;
        const int blocks = (int)std::min<long long>((rows + 7) / 8, 148LL * 16);
        void* args[] = {(void*)&k_cache, (void*)&n_kv_heads, (void*)&max_seq, (void*)&n_keys, (void*)&ldi,
                        (void*)&kh, (void*)&kl, (void*)&status};
        const void* kfn = kv_dtype == MF_F32 ? (const void*)&mf::fa_k_split_kernel<float>
                                             : (const void*)&mf::fa_k_split_kernel<__nv_bfloat16>;
        cudaError_t e = launch(kfn, dim3(blocks), dim3(256), 0, st, args);
        if (e != cudaSuccess) return fail(MF_E_CUDA, cudaGetErrorString(e));
    }
    {
        void* args[] = {(void*)&v_cache, (void*)&max_seq, (void*)&n_keys, (void*)&ldi, (void*)&vh, (void*)&vl};
        const void* vfn = kv_dtype == MF_F32 ? (const void*)&mf::fa_v_split_kernel<float>
                                             : (const void*)&mf::fa_v_split_kernel<__nv_bfloat16>;
        cudaError_t e = launch(vfn, dim3((n_keys + 63) / 64, n_kv_heads), dim3(256), 0, st, args);
        if (e != cudaSuccess) return fail(MF_E_CUDA, cudaGetErrorString(e));
    }
    mf::FaParams p;
    p.q = q;
    p.P = n_tokens;
    p.pos0 = pos0;
    p.n_heads = n_heads;
    p.out_hi = (__nv_bfloat16*)out_hi;
    p.out_lo = (__nv_bfloat16*)out_lo;
    p.status = status;
    p.timeout_ns = timeout_ns();
    const int QT = mf::FA_BM / G;
    void* args[] = {(void*)&tk[0], (void*)&tk[1], (void*)&tv[0], (void*)&tv[1], (void*)&p};
    cudaError_t e = launch(fn, dim3((n_tokens + QT - 1) / QT, n_kv_heads), dim3(mf::FA_THREADS),
                           mf::FA_SMEM_BYTES, st, args);
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

int mf_prefill_status(int* status, int clear) {
    if (!status) return fail(MF_E_INVALID, "null argument");
    int* p = status_ptr();
    if (!p) return fail(MF_E_CUDA, "prefill status symbol");
    cudaError_t e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(status, p, sizeof(int), cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && clear) e = cudaMemset(p, 0, sizeof(int));
    return e == cudaSuccess ? MF_OK : fail(MF_E_CUDA, cudaGetErrorString(e));
}

}  // extern "C"
