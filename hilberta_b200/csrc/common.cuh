// Shared helpers of the hilberta_b200 CUDA library (builder + attention).
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/hilberta_b200.h"

// On failure the runtime's last-error slot is cleared too, so a later launch
// check does not report this call's (non-sticky) error as its own.
#define HB_CUDA_TRY(expr)                                  \
    do {                                                   \
        cudaError_t _e = (expr);                           \
        if (_e != cudaSuccess) {                           \
            (void)cudaGetLastError();                      \
            return HB_ERR_CUDA;                            \
        }                                                  \
    } while (0)

#define HB_LAUNCH_CHECK() HB_CUDA_TRY(cudaGetLastError())

namespace hb {

__host__ __device__ inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Python-style modulo (result in [0, m) for m > 0).
__host__ __device__ inline int64_t pymod(int64_t a, int64_t m) {
    int64_t r = a % m;
    return r < 0 ? r + m : r;
}

inline bool is_pow2(int64_t x) { return x > 0 && (x & (x - 1)) == 0; }

}  // namespace hb
