// Shared helpers for the ancha_b200 CUDA library: status handling, bf16 conversion and
// small device utilities. Every kernel in this library targets sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <stdint.h>
#include <string>

#include "../../include/ancha_b200.h"

namespace ancha {

// Record `msg` as the calling thread's last error and return `code`.
int fail(int code, const std::string& msg);
// Record a CUDA failure (with the API name) and return ANCHA_E_CUDA.
int cuda_fail(cudaError_t err, const char* what);
// Check for a launch error right after a launch.
int check_launch(const char* what);

#define ANCHA_TRY(expr)                         \
    do {                                        \
        int _st = (expr);                       \
        if (_st != ANCHA_OK) return _st;        \
    } while (0)

#define ANCHA_CUDA(expr)                                    \
    do {                                                    \
        cudaError_t _e = (expr);                            \
        if (_e != cudaSuccess) return ::ancha::cuda_fail(_e, #expr); \
    } while (0)

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ void store_f(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

}  // namespace ancha
