// mf_attn_decode_noalloc: the decode-attention op for callers that cannot
// allocate device memory.
//
// mf_attn_decode needs a caller-provided workspace (per-split partial results
// and completion counters). Some callers cannot obtain one: code that issues
// work while a stream is being captured in global mode (where cudaMalloc is
// not permitted), code running in stream callbacks or other contexts where
// CUDA allocation calls are forbidden, and hosts whose device memory is owned
// by another runtime's allocator or a fixed budget. This entry point takes
// only the inputs and outputs; its scratch is one file-scope device array of
// MF_ATTN_NOALLOC_SCRATCH_BYTES bytes that every GPU loading this library
// holds until the process exits.
//
// Properties a caller must know:
//  * The first call on a device looks up the array's device address
//    (cudaGetSymbolAddress, with that device current) and caches it; make that
//    first call before any stream capture on the device. The cache is tied to
//    the device's context: after the context is destroyed and re-created
//    (cudaDeviceReset), the next call looks the address up again, so make
//    that call, too, outside any stream capture.
//  * The array is shared by every call. It keeps the last call's contents;
//    the completion counters are cleared at the start of each call on the
//    caller's stream. Calls whose executions overlap on the GPU (different
//    streams, no ordering between them) race on the array and give wrong
//    results.
//  * A request whose scratch would exceed MF_ATTN_NOALLOC_SCRATCH_BYTES is
//    rejected with MF_E_UNSUPPORTED; nothing is launched.
//  * It calls no cudaMalloc, cudaFree or other allocating routine.
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <mutex>

#include "attention.cuh"
#include "minfer_cuda.h"

namespace mf {
const void* attn_kernel_ptr(int group, int kv_dtype);
int record_error(int code, const char* msg);  // capi.cu: message for mf_last_error
cudaStream_t resolve_stream(void* stream);    // capi.cu: NULL -> manager stream of the current device
}

namespace {

static __device__ __align__(256) unsigned char g_attn_scratch[MF_ATTN_NOALLOC_SCRATCH_BYTES];

int noalloc_fail(int code, const char* msg) { return mf::record_error(code, msg); }

// Device address of g_attn_scratch for the current device, looked up once per
// device and context: a context destroyed and re-created on the device (for
// example after cudaDeviceReset) gets the array at a new address, so the cached
// address is keyed on the context that was current when it was taken.
int scratch_address(void** out) {
    static std::mutex mu;
    static void* addr[64] = {nullptr};
    static CUcontext owner[64] = {nullptr};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64)
        return noalloc_fail(MF_E_CUDA, "no usable current device");
    // the driver's cuCtxGetCurrent, a query (resolved through the runtime, so the
    // library does not link the driver library directly)
    static CUresult (*ctx_current)(CUcontext*) = nullptr;
    std::lock_guard<std::mutex> lk(mu);
    if (!ctx_current) {
        void* fn = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &fn, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess || !fn)
            return noalloc_fail(MF_E_CUDA, "cuCtxGetCurrent is not available");
        ctx_current = (CUresult(*)(CUcontext*))fn;
    }
    // NULL before the runtime first touched the device on this thread
    CUcontext ctx = nullptr;
    if (ctx_current(&ctx) != CUDA_SUCCESS) ctx = nullptr;
    if (!addr[dev] || !ctx || owner[dev] != ctx) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_attn_scratch);  // makes the device's context current
        if (e != cudaSuccess) return noalloc_fail(MF_E_CUDA, cudaGetErrorString(e));
        if (ctx_current(&ctx) != CUDA_SUCCESS || !ctx) return noalloc_fail(MF_E_CUDA, "no current CUDA context");
        addr[dev] = p;
        owner[dev] = ctx;
    }
    *out = addr[dev];
    return MF_OK;
}

}  // namespace

extern "C" int mf_attn_decode_noalloc(const mf_attn_desc* d, void* stream) {
    if (!d) return noalloc_fail(MF_E_INVALID, "null descriptor");
    if (!(d->qkv && d->q_norm_w && d->k_norm_w && d->rope_table && d->k_cache && d->v_cache && d->step_state &&
          d->out))
        return noalloc_fail(MF_E_INVALID, "null pointer in attention descriptor");
    if (d->d_head != mf::ATT_D) return noalloc_fail(MF_E_UNSUPPORTED, "d_head must be 128");
    if (d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads != 0)
        return noalloc_fail(MF_E_INVALID, "n_heads must be a multiple of n_kv_heads");
    if (d->n_split < 1 || d->max_seq < 1) return noalloc_fail(MF_E_INVALID, "bad n_split/max_seq");
    const int G = d->n_heads / d->n_kv_heads;
    if (d->kv_dtype != MF_F32 && d->kv_dtype != MF_BF16) return noalloc_fail(MF_E_UNSUPPORTED, "KV cache dtype");
    const void* fn = mf::attn_kernel_ptr(G, d->kv_dtype);
    if (!fn) return noalloc_fail(MF_E_UNSUPPORTED, "query heads per KV head without a kernel");
    // scratch layout: counters | (m, l) per split and head | partial outputs | merged groups
    const mf::AttnWsLayout L = mf::attn_ws_layout(d->n_kv_heads, d->n_split, G);
    if (L.total > MF_ATTN_NOALLOC_SCRATCH_BYTES)
        return noalloc_fail(MF_E_UNSUPPORTED, "request needs more scratch than MF_ATTN_NOALLOC_SCRATCH_BYTES");
    if (d->n_split > mf::attn_max_split(G)) return noalloc_fail(MF_E_UNSUPPORTED, "n_split above the merge table size");
    void* base = nullptr;
    int rc = scratch_address(&base);
    if (rc) return rc;
    cudaStream_t st = mf::resolve_stream(stream);
    char* ws = (char*)base;
    // the counters must start at zero; a previous call may have been cut short
    cudaError_t e = cudaMemsetAsync(ws + L.cnt, 0, L.ml - L.cnt, st);
    if (e != cudaSuccess) return noalloc_fail(MF_E_CUDA, cudaGetErrorString(e));
    const size_t smem = mf::attn_smem_bytes(G);
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return noalloc_fail(MF_E_CUDA, cudaGetErrorString(e));
    mf::AttnParams p = {};
    p.qkv = d->qkv;
    p.q_norm_w = d->q_norm_w;
    p.k_norm_w = d->k_norm_w;
    p.eps = d->eps;
    p.rope = (const float2*)d->rope_table;
    p.k_cache = d->k_cache;
    p.v_cache = d->v_cache;
    p.max_seq = d->max_seq;
    p.pos_ptr = (const int*)d->step_state + 1;  // {token, pos, next_token, chain}
    p.out = d->out;
    p.counters = (int*)(ws + L.cnt);
    p.part_ml = (float*)(ws + L.ml);
    p.part_o = (float*)(ws + L.o);
    p.group_ml = (float*)(ws + L.gml);
    p.group_o = (float*)(ws + L.go);
    p.n_heads = d->n_heads;
    p.n_kv_heads = d->n_kv_heads;
    p.n_split = d->n_split;
    void* args[] = {&p};
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(d->n_split, d->n_kv_heads);
    cfg.blockDim = dim3(mf::ATT_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    e = cudaLaunchKernelExC(&cfg, fn, args);
    if (e != cudaSuccess) return noalloc_fail(MF_E_CUDA, cudaGetErrorString(e));
    return MF_OK;
}
