/*
 * Link-time definitions for the Metal manager symbols that the reference's
 * host sources reference (include/minfer/interfaces/metal_interface.hpp:9-37).
 * The CPU oracle never selects DeviceType::METAL, so every entry aborts if it
 * is ever reached. Test infrastructure only.
 */
#include <cstdio>
#include <cstdlib>
#include <cstddef>

namespace MTL { class Buffer; }

namespace MetalManager {
[[noreturn]] static void unavailable(const char* what) {
    std::fprintf(stderr, "oracle: Metal entry point %s reached on the CPU path\n", what);
    std::abort();
}
MTL::Buffer* upload(void*, size_t) { unavailable("upload"); }
void release(MTL::Buffer*) { unavailable("release"); }
void* cpu_ptr(MTL::Buffer*) { unavailable("cpu_ptr"); }
void init() { unavailable("init"); }
void begin_frame() { unavailable("begin_frame"); }
void end_frame() { unavailable("end_frame"); }
void dispatch_unavailable() { unavailable("dispatch"); }
}  // namespace MetalManager
