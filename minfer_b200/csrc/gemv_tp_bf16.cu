// Tensor-parallel GEMV kernel instantiations for BF16 weights.
#include "gemv_inst.cuh"

namespace mf {
const void* gemv_tp_kernel_ptr_bf16(int xm, int ym, int T, int R) { return gemv_tp_kernel_ptr<W_BF16>(xm, ym, T, R); }
}  // namespace mf
