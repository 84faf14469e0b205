// Tensor-parallel GEMV kernel instantiations for F32 weights.
#include "gemv_inst.cuh"

namespace mf {
const void* gemv_tp_kernel_ptr_f32(int xm, int ym, int T, int R) { return gemv_tp_kernel_ptr<W_F32>(xm, ym, T, R); }
}  // namespace mf
