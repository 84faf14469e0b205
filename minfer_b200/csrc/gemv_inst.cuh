// Kernel-pointer tables for the GEMV family, one translation unit per weight
// dtype (gemv_f32.cu, gemv_f16.cu, gemv_bf16.cu) so they compile in parallel.
#pragma once

#include "gemv.cuh"

namespace mf {

// Launch shapes offered per dtype/mode: T threads in {64, 128, 256};
// (R, PC) in {(8,1), (4,2), (2,4)}. Y_MOE_DOWN uses R = 8 (one row per slot).
template <typename W, int XM, int YM>
const void* gemv_ptr_rpc(int T, int R) {
#define MF_GEMV_T(TT)                                                                        \
    if (T == TT) {                                                                           \
        if (R == 8) return (const void*)&gemv_kernel<W, TT, 8, 1, XM, YM>;                  \
        if (YM != Y_MOE_DOWN && YM != Y_MOE_PUSH) {                                          \
            if (R == 4) return (const void*)&gemv_kernel<W, TT, 4, 2, XM, YM>;              \
            if (R == 2) return (const void*)&gemv_kernel<W, TT, 2, 4, XM, YM>;              \
        }                                                                                    \
        return nullptr;                                                                      \
    }
    MF_GEMV_T(64)
    MF_GEMV_T(128)
    MF_GEMV_T(256)
#undef MF_GEMV_T
    return nullptr;
}

template <typename W>
const void* gemv_kernel_ptr(int xm, int ym, int T, int R) {
    if (xm == X_NORM && ym == Y_STORE) return gemv_ptr_rpc<W, X_NORM, Y_STORE>(T, R);
    if (xm == X_PLAIN && ym == Y_STORE) return gemv_ptr_rpc<W, X_PLAIN, Y_STORE>(T, R);
    if (xm == X_PLAIN && ym == Y_RESID) return gemv_ptr_rpc<W, X_PLAIN, Y_RESID>(T, R);
    if (xm == X_NORM && ym == Y_SWIGLU) return gemv_ptr_rpc<W, X_NORM, Y_SWIGLU>(T, R);
    if (xm == X_PLAIN && ym == Y_MOE_DOWN) return gemv_ptr_rpc<W, X_PLAIN, Y_MOE_DOWN>(T, R);
    return nullptr;
}

// Tensor-parallel modes (all-reduce receive / send), compiled in gemv_tp_*.cu.
template <typename W>
const void* gemv_tp_kernel_ptr(int xm, int ym, int T, int R) {
    if (xm == X_AR_NORM && ym == Y_STORE) return gemv_ptr_rpc<W, X_AR_NORM, Y_STORE>(T, R);
    if (xm == X_AR_NORM && ym == Y_SWIGLU) return gemv_ptr_rpc<W, X_AR_NORM, Y_SWIGLU>(T, R);
    if (xm == X_PLAIN && ym == Y_PUSH) return gemv_ptr_rpc<W, X_PLAIN, Y_PUSH>(T, R);
    if (xm == X_PLAIN && ym == Y_MOE_PUSH) return gemv_ptr_rpc<W, X_PLAIN, Y_MOE_PUSH>(T, R);
    return nullptr;
}

const void* gemv_kernel_ptr_f32(int xm, int ym, int T, int R);
const void* gemv_kernel_ptr_f16(int xm, int ym, int T, int R);
const void* gemv_kernel_ptr_bf16(int xm, int ym, int T, int R);
const void* gemv_tp_kernel_ptr_f32(int xm, int ym, int T, int R);
const void* gemv_tp_kernel_ptr_f16(int xm, int ym, int T, int R);
const void* gemv_tp_kernel_ptr_bf16(int xm, int ym, int T, int R);

}  // namespace mf
