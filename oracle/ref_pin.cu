/*
 * ref_pin.cu -- TEST INFRASTRUCTURE ONLY.
 *
 * Compiles the reference GEMV source where it lies (the include paths come from oracle/Makefile;
 * nothing is copied) and exports its host-callable helpers with C linkage, so that the oracle's
 * restatements can be checked against the reference itself:
 *   mix32              applications/gemv/src/gemv_k1024_persistent_subwarp.cu:56-63
 *   predict_addr_side  applications/gemv/src/gemv_k1024_persistent_subwarp.cu:105-108
 *   predict_map_memory_attr_far  utility/latopt.cuh:255-263
 * Only host code runs: no kernel is launched and no CUDA runtime call is made, so the library
 * works on a machine without a GPU.  The reference's `main` is renamed out of the way.
 */
#define main l2d_ref_gemv_main
#include "gemv_k1024_persistent_subwarp.cu"
#undef main

#include <cstdint>
#include <vector>

extern "C" uint32_t ref_mix32(uint32_t x) { return mix32(x); }

extern "C" int ref_predict_far(int side, uint32_t mask, uint64_t addr, int attr) {
    return latopt::predict_map_memory_attr_far(side, mask, static_cast<uintptr_t>(addr), attr);
}

extern "C" int ref_predict_addr_side(uint64_t base, uint32_t mask, const int *attr, size_t n_attr, uint64_t addr) {
    std::vector<int> a(attr, attr + n_attr);
    return predict_addr_side(static_cast<uintptr_t>(base), mask, a, static_cast<uintptr_t>(addr));
}

extern "C" size_t ref_memory_alloc_gran(void) { return latopt::kMemoryAllocGran; }
