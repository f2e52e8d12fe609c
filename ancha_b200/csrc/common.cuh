// Shared helpers for the ancha_b200 CUDA library: status handling, element types (f32,
// bf16, f16) and small device utilities. Every kernel in this library targets sm_100a only.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
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

// Element types of activations and GEMM / attention operands (the ANCHA_F32 / ANCHA_BF16 /
// ANCHA_F16 codes of the C ABI).
enum : int { ELT_F32 = 0, ELT_BF16 = 1, ELT_F16 = 2 };
inline size_t elt_size(int t) { return t == ELT_F32 ? 4 : 2; }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

inline int64_t ceil_div(int64_t a, int64_t b) { return (a + b - 1) / b; }

// Longest track a separation entry point accepts, per channel: 2^36 samples (about 18 days at
// 44.1 kHz), which keeps every byte count derived from it far from overflowing 64 bits.
constexpr int64_t kMaxTrackSamples = int64_t(1) << 36;
// The model schema's context limits (crates/ancha-models/src/config.rs:64): a chunk of at most
// 60 s at 44.1 kHz and an overlap divisor of at most 16. They also hold for a chunk or overlap
// given at call time, as the reference validates its config after command-line overrides.
constexpr int64_t kMaxChunkSamples = 44100 * 60;
constexpr int kMaxOverlap = 16;

__device__ __forceinline__ float load_f(const float* p) { return *p; }
__device__ __forceinline__ float load_f(const __nv_bfloat16* p) { return __bfloat162float(*p); }
__device__ __forceinline__ float load_f(const __half* p) { return __half2float(*p); }
__device__ __forceinline__ void store_f(float* p, float v) { *p = v; }
__device__ __forceinline__ void store_f(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
__device__ __forceinline__ void store_f(__half* p, float v) { *p = __float2half_rn(v); }

// Store v at element idx of a buffer of element type t.
__device__ __forceinline__ void store_elt(void* base, int64_t idx, float v, int t) {
    if (t == ELT_BF16) store_f(reinterpret_cast<__nv_bfloat16*>(base) + idx, v);
    else if (t == ELT_F16) store_f(reinterpret_cast<__half*>(base) + idx, v);
    else store_f(reinterpret_cast<float*>(base) + idx, v);
}

__device__ __forceinline__ float gelu_erf(float x) {
    return 0.5f * x * (1.0f + erff(x * 0.70710678118654752f));
}
__device__ __forceinline__ float sigmoidf_(float x) { return 1.0f / (1.0f + expf(-x)); }

}  // namespace ancha
