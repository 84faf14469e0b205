// Decode-attention kernel instantiations (one per query heads per KV head and
// cache element type).
#include "attention.cuh"

namespace mf {
template <typename KV>
static const void* attn_ptr(int group) {
    switch (group) {
        case 1: return (const void*)&attn_decode_kernel<1, KV>;
        case 2: return (const void*)&attn_decode_kernel<2, KV>;
        case 4: return (const void*)&attn_decode_kernel<4, KV>;
        case 8: return (const void*)&attn_decode_kernel<8, KV>;
        case 16: return (const void*)&attn_decode_kernel<16, KV>;
        default: return nullptr;
    }
}
const void* attn_kernel_ptr(int group, int kv_dtype) {
    if (kv_dtype == MF_F32) return attn_ptr<float>(group);
    if (kv_dtype == MF_BF16) return attn_ptr<__nv_bfloat16>(group);
    return nullptr;
}
}  // namespace mf
