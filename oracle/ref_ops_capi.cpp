/*
 * extern "C" wrappers around the reference's own CPU ops
 * (include/minfer/ops/kernels.hpp:13-32, src/ops/kernels.cpp), so Python
 * tests can call them through ctypes with plain pointers. Each wrapper only
 * builds the reference's typed weight view (include/minfer/base/types.hpp)
 * over the caller's buffer and forwards the call. Test infrastructure only.
 */
#include "minfer/ops/kernels.hpp"
#include "minfer/base/types.hpp"

#include <cstddef>
#include <cstdint>

namespace {
std::byte* as_bytes(const void* p) { return reinterpret_cast<std::byte*>(const_cast<void*>(p)); }
}

extern "C" {

float ref_silu(float x) { return silu(x); }

void ref_softmax(float* out, const float* in, int n) { softmax(out, in, n); }

void ref_il_rope(float* out, const float* in, int head, int d_head, int d_rot, float base, int pos) {
    il_rope(out, in, head, d_head, d_rot, base, pos);
}

void ref_neox_rope(float* out, const float* in, int head, int d_head, int d_rot, float base, int pos) {
    neox_rope(out, in, head, d_head, d_rot, base, pos);
}

void ref_attn(float* scores, float* out, const float* q, const float* k, const float* v,
              int seq_len, int d_head, int kv_dim) {
    attn(scores, out, q, k, v, seq_len, d_head, kv_dim);
}

void ref_rmsnorm(float* out, const float* in, const float* w, int dim, float eps) {
    rmsnorm(out, in, fp32_t(as_bytes(w)), dim, eps);
}

void ref_route(const float* x, int* experts, float* weights, float* scores, const float* w_router,
               int d_model, int n_experts, int k) {
    route(x, experts, weights, scores, fp32_t(as_bytes(w_router)), d_model, n_experts, k);
}

void ref_matmul_f32(float* out, const float* x, const float* w, size_t off, int d_out, int d_in) {
    matmul_fp32(out, x, fp32_t(as_bytes(w)), off, d_out, d_in);
}

void ref_matmul_f16(float* out, const float* x, const uint16_t* w, size_t off, int d_out, int d_in) {
    matmul_fp16(out, x, fp16_t(as_bytes(w)), off, d_out, d_in);
}

void ref_matmul_bf16(float* out, const float* x, const uint16_t* w, size_t off, int d_out, int d_in) {
    matmul_bf16(out, x, bf16_t(as_bytes(w)), off, d_out, d_in);
}

void ref_embed_f32(float* out, const float* w, uint32_t tok, size_t d) { embed_fp32(out, fp32_t(as_bytes(w)), tok, d); }
void ref_embed_f16(float* out, const uint16_t* w, uint32_t tok, size_t d) { embed_fp16(out, fp16_t(as_bytes(w)), tok, d); }
void ref_embed_bf16(float* out, const uint16_t* w, uint32_t tok, size_t d) { embed_bf16(out, bf16_t(as_bytes(w)), tok, d); }

}  // extern "C"
