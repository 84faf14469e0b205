// TMA-fed dense and grouped-expert GEMV instantiations for BF16 weights.
#include "gemv.cuh"
#include "gemv_tma.cuh"

namespace mf {
const void* gemv_tma_ptr_bf16(int xm, int ym, int nwc, int j) { return gemv_tma_ptr<W_BF16>(xm, ym, nwc, j); }
const void* moe_down_tma_ptr_bf16(int j) { return moe_down_tma_ptr<W_BF16>(j); }
}  // namespace mf
