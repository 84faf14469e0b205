// Tensor-parallel GEMV kernel instantiations for F16 weights.
#include "gemv_inst.cuh"

namespace mf {
const void* gemv_tp_kernel_ptr_f16(int xm, int ym, int T, int R) { return gemv_tp_kernel_ptr<W_F16>(xm, ym, T, R); }
}  // namespace mf
