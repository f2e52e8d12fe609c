// Host side of the tensor-core kernels: the per-device error word that bounded waits report
// into, and TMA tensor-map encoding through the driver entry point (no libcuda link).
#include <cudaTypedefs.h>

#include <mutex>

#include "tc.cuh"

namespace ancha {
namespace {

__device__ int g_device_error;

std::mutex g_mu;
int* g_error_ptr[64];

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
    }();
    return fn;
}

}  // namespace

int* device_error_word() {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(g_mu);
    if (!g_error_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_device_error) != cudaSuccess) return nullptr;
        g_error_ptr[dev] = static_cast<int*>(p);
    }
    return g_error_ptr[dev];
}

int take_device_error(cudaStream_t s) {
    int* w = device_error_word();
    if (!w) return ANCHA_OK;
    int v = 0;
    ANCHA_CUDA(cudaMemcpyAsync(&v, w, sizeof(int), cudaMemcpyDeviceToHost, s));
    ANCHA_CUDA(cudaStreamSynchronize(s));
    if (v) {
        ANCHA_CUDA(cudaMemsetAsync(w, 0, sizeof(int), s));
        return fail(ANCHA_E_TIMEOUT, "a bounded device-side wait gave up (kernel aborted)");
    }
    return ANCHA_OK;
}

namespace {
// An mbarrier expecting one arrival that never comes: thread 0 waits for its first phase with
// the given budget, gives up, raises the abort flag and records the timeout in the error word;
// the other threads of the warp wait on the flag as the kernels' consumer warps do.
__global__ void wait_selftest_kernel(long long budget, int* err) {
    __shared__ uint64_t bar;
    __shared__ int abort_flag;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    __syncthreads();
    volatile int* abort = &abort_flag;
    if (threadIdx.x == 0) {
        mbar_wait(&bar, 0, abort, err, budget);
    } else {
        const long long t0 = clock64();
        while (!*abort && clock64() - t0 < 4 * budget + 1000000) {
        }
    }
}
}  // namespace

int wait_selftest(long long budget_cycles, cudaStream_t s) {
    if (budget_cycles < 0 || budget_cycles > kWaitCycles)
        return fail(ANCHA_E_INVALID, "wait_selftest: budget outside [0, the kernels' budget]");
    int* w = device_error_word();
    if (!w) return fail(ANCHA_E_CUDA, "device error word unavailable");
    wait_selftest_kernel<<<1, 32, 0, s>>>(budget_cycles, w);
    ANCHA_TRY(check_launch("wait_selftest"));
    return take_device_error(s);
}

int make_tma_3d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t rows,
                int64_t depth, int64_t ld, int64_t depth_stride, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * 2) % 16 || (depth_stride * 2) % 16 ||
        cols <= 0 || rows <= 0 || depth <= 0)
        return fail(ANCHA_E_UNSUPPORTED, "TMA operand not 16-byte aligned");
    const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)depth};
    const cuuint64_t strides[2] = {(cuuint64_t)(ld * 2), (cuuint64_t)(depth_stride * 2)};
    const cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    CUresult r = fn(map, elt == ELT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
    return ANCHA_OK;
}

int make_tma_store_3d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t rows,
                      int64_t depth, int64_t ld, int64_t depth_stride, int box_cols, int box_rows) {
    auto fn = encode_fn();
    if (!fn) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    const int es = (int)elt_size(elt);
    const int row_bytes = box_cols * es;
    if (reinterpret_cast<uintptr_t>(base) % 16 || (ld * es) % 16 || (depth_stride * es) % 16 || cols <= 0 ||
        rows <= 0 || depth <= 0 || (row_bytes != 64 && row_bytes != 128))
        return fail(ANCHA_E_UNSUPPORTED, "TMA store operand not 16-byte aligned");
    const cuuint64_t dims[3] = {(cuuint64_t)cols, (cuuint64_t)rows, (cuuint64_t)depth};
    const cuuint64_t strides[2] = {(cuuint64_t)(ld * es), (cuuint64_t)(depth_stride * es)};
    const cuuint32_t box[3] = {(cuuint32_t)box_cols, (cuuint32_t)box_rows, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    const CUtensorMapDataType dt = elt == ELT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32
                                   : elt == ELT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                                     : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
    CUresult r = fn(map, dt, 3, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    row_bytes == 128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_64B,
                    CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled (store) failed: " + std::to_string((int)r));
    return ANCHA_OK;
}

int make_tma_4d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t d1, int64_t d2,
                int64_t d3, int64_t s1, int64_t s2, int64_t s3, int b1, int b2) {
    auto fn = encode_fn();
    if (!fn) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled unavailable");
    if (reinterpret_cast<uintptr_t>(base) % 16 || (s1 * 2) % 16 || (s2 * 2) % 16 || (s3 * 2) % 16 ||
        cols <= 0 || d1 <= 0 || d2 <= 0 || d3 <= 0)
        return fail(ANCHA_E_UNSUPPORTED, "TMA operand not 16-byte aligned");
    const cuuint64_t dims[4] = {(cuuint64_t)cols, (cuuint64_t)d1, (cuuint64_t)d2, (cuuint64_t)d3};
    const cuuint64_t strides[3] = {(cuuint64_t)(s1 * 2), (cuuint64_t)(s2 * 2), (cuuint64_t)(s3 * 2)};
    const cuuint32_t box[4] = {64, (cuuint32_t)b1, (cuuint32_t)b2, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    CUresult r = fn(map, elt == ELT_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                    4, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(ANCHA_E_UNSUPPORTED, "cuTensorMapEncodeTiled (4-D) failed: " + std::to_string((int)r));
    return ANCHA_OK;
}

}  // namespace ancha
