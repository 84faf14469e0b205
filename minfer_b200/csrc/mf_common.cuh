// Shared device helpers for the sm_100a decode/prefill kernels.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <cuda_bf16.h>
#include <stdint.h>

#include "minfer_cuda.h"

#define MF_DEVICE __device__ __forceinline__

namespace mf {

// ---------------------------------------------------------------- weights
// The reference widens every weight to fp32 before the FMA
// (src/ops/kernels.cpp:270-285,321-336); both widenings are exact.
MF_DEVICE float bf16_lo(uint32_t u) { return __uint_as_float(u << 16); }
MF_DEVICE float bf16_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }
MF_DEVICE float2 f16x2_to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2*>(&u);
    return __half22float2(h);
}

struct W_F32 { using T = float; static constexpr int VEC = 4; static constexpr int CODE = MF_F32; };
struct W_F16 { using T = uint16_t; static constexpr int VEC = 8; static constexpr int CODE = MF_F16; };
struct W_BF16 { using T = uint16_t; static constexpr int VEC = 8; static constexpr int CODE = MF_BF16; };

// Unpack one 16-byte weight vector into fp32 lanes.
template <typename W> MF_DEVICE void unpack16(const uint4& v, float* out);
template <> MF_DEVICE void unpack16<W_F32>(const uint4& v, float* o) {
    o[0] = __uint_as_float(v.x); o[1] = __uint_as_float(v.y);
    o[2] = __uint_as_float(v.z); o[3] = __uint_as_float(v.w);
}
template <> MF_DEVICE void unpack16<W_BF16>(const uint4& v, float* o) {
    o[0] = bf16_lo(v.x); o[1] = bf16_hi(v.x); o[2] = bf16_lo(v.y); o[3] = bf16_hi(v.y);
    o[4] = bf16_lo(v.z); o[5] = bf16_hi(v.z); o[6] = bf16_lo(v.w); o[7] = bf16_hi(v.w);
}
template <> MF_DEVICE void unpack16<W_F16>(const uint4& v, float* o) {
    float2 a = f16x2_to_f2(v.x), b = f16x2_to_f2(v.y), c = f16x2_to_f2(v.z), d = f16x2_to_f2(v.w);
    o[0] = a.x; o[1] = a.y; o[2] = b.x; o[3] = b.y; o[4] = c.x; o[5] = c.y; o[6] = d.x; o[7] = d.y;
}

// Streaming 16-byte load for data read once per token (weights): read-only
// path, no L1 allocation.
MF_DEVICE uint4 ld_stream(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}

// TMA bulk prefetch of [p, p+bytes) into L2 (p 16-byte aligned, bytes a
// multiple of 16). Issued by one thread; nothing waits on it.
MF_DEVICE void prefetch_l2(const void* p, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// L2-coherent loads (bypass L1) for data written by other CTAs of the same grid.
MF_DEVICE float ld_cg(const float* p) { return __ldcg(p); }
MF_DEVICE int ld_cg(const int* p) { return __ldcg(p); }

// Wall clock (ns) for bounded waits.
MF_DEVICE unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- PDL
// Programmatic dependent launch: the next kernel in the stream may start its
// weight prefetch while this one drains; `wait` blocks until every
// prerequisite grid has completed and flushed its writes.
// Thread-block clusters: this CTA's rank, a full-cluster barrier (every
// thread of every CTA arrives), and a float read from a peer CTA's shared
// memory at the address `local` has in this CTA.
MF_DEVICE uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
MF_DEVICE void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
MF_DEVICE float ld_cluster_f32(const float* local, uint32_t rank) {
    uint32_t remote;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;"
                 : "=r"(remote)
                 : "r"((uint32_t)__cvta_generic_to_shared(local)), "r"(rank));
    float v;
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(remote) : "memory");
    return v;
}

MF_DEVICE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
MF_DEVICE void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---------------------------------------------------------------- reductions
MF_DEVICE float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
MF_DEVICE float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Block-wide sum; `scratch` holds >= 32 floats. Result broadcast to all threads.
MF_DEVICE float block_sum(float v, float* scratch) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, nw = (blockDim.x + 31) >> 5;
    v = warp_sum(v);
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.f;
    for (int i = 0; i < nw; ++i) t += scratch[i];
    return t;
}

// (value, index) ordering shared by the greedy argmax and the router top-k:
// larger value wins; equal values go to the lower index (first maximum, as
// std::max_element in src/base/sampler.cpp:37 and the strict `>` scan in
// src/ops/kernels.cpp:126-131).
MF_DEVICE bool better(float va, int ia, float vb, int ib) {
    return va > vb || (va == vb && ia < ib);
}

// SiLU as in src/ops/kernels.cpp:27-29.
MF_DEVICE float silu(float x) { return x / (1.0f + expf(-x)); }

}  // namespace mf
