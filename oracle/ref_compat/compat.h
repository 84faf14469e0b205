/*
 * Force-included (g++ -include) into every reference source the oracle build
 * compiles. It papers over three portability gaps of the reference on
 * x86-64/libstdc++ without touching the reference's files:
 *  - include/minfer/ops/kernels.hpp and include/minfer/base/sampler.hpp use
 *    std::shared_ptr without including <memory>;
 *  - src/ops/kernels.cpp:28,41,88 and src/base/sampler.cpp:67,86,100 call
 *    std::expf / std::sqrtf / std::logf, which libstdc++ 13 does not declare;
 *    they name the same C functions, so they are re-exported into std;
 *  - __fp16 is an Arm-only spelling; on x86-64 the same IEEE binary16 type is
 *    _Float16.
 * Test infrastructure only.
 */
#pragma once
#ifdef __cplusplus
#include <memory>
#include <math.h>
namespace std {
using ::expf;
using ::sqrtf;
using ::logf;
}
#endif
#define __fp16 _Float16

/*
 * src/models/qwen3/module.cpp passes Metal buffer lists as compound literals
 * `(MTL::Buffer*[]){...}` (a clang extension g++ rejects). Those calls sit in
 * the metal_forward paths the CPU oracle never runs, so every dispatch call
 * (and the two declarations in include/minfer/interfaces/metal_interface.hpp)
 * is rewritten to one argument-less function that the oracle build defines
 * as an abort.
 */
#define dispatch1d(...) dispatch_unavailable()
#define dispatch2d(...) dispatch_unavailable()
