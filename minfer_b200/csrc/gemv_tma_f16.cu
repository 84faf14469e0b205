// TMA-fed dense and grouped-expert GEMV instantiations for F16 weights.
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace mf {
const void* gemv_tma_ptr_f16(int xm, int ym, int nwc, int j) { return gemv_tma_ptr<W_F16>(xm, ym, nwc, j); }
const void* moe_down_tma_ptr_f16(int j) { return moe_down_tma_ptr<W_F16>(j); }
}  // namespace mf
