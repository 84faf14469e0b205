// Decode-attention kernel instantiations (one per query heads per KV head).
#include "attention.cuh"

namespace mf {
const void* attn_kernel_ptr(int group) {
    switch (group) {
        case 1: return (const void*)&attn_decode_kernel<1>;
        case 2: return (const void*)&attn_decode_kernel<2>;
        case 4: return (const void*)&attn_decode_kernel<4>;
        case 8: return (const void*)&attn_decode_kernel<8>;
        case 16: return (const void*)&attn_decode_kernel<16>;
        default: return nullptr;
    }
}
}  // namespace mf
