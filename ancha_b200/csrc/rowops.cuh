// Row-wise and gather kernels of the RoFormer stack (see rowops.cu).
#pragma once
#include "common.cuh"

namespace ancha {

int norm_rows(float* x, int64_t ldx, const float* scale, void* xn, int xn_type, int64_t ldn,
              int64_t rows, int dim, cudaStream_t s);
int cast_rows(const float* x, int64_t ldx, void* y, int y_type, int64_t ldy, int64_t rows,
              int dim, cudaStream_t s);
// Three-way bf16 split of f32 rows for the tensor-core fp32 GEMM: hi = bf16(x), mid =
// bf16(x − hi), lo = bf16(x − hi − mid) (both differences exact in f32), so hi + mid + lo = x to
// within 2^-24 relative; written as planes y[p][r][c] (p = 0, 1, 2; plane stride rows·dim, row
// stride dim).
int split3_rows(const float* x, int64_t ldx, void* y, int64_t rows, int dim, cudaStream_t s);
// The same split of columns [0, dim) of each row into planes with row stride ldy, plane p at
// y + p · plane elements.
int split3_rows_strided(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t plane, int64_t rows, int dim,
                        cudaStream_t s);
int band_gather(const float* spec, int chunks, int frames, int columns, const int* cols,
                const int* offsets, int bands, int total, float* z, cudaStream_t s);
// band_gather in f16 with each band's row zero-padded to kp features, rows ordered
// (chunk, band, frame): the A operand of the grouped tensor-core band-split GEMM.
int band_gather_padded(const float* spec, int chunks, int frames, int columns, const int* cols,
                       const int* offsets, int bands, int kp, void* z, cudaStream_t s);
int mask_assemble(const float* glu, int64_t ldg, int bands, int frames, int rows,
                  const int* count, const int2* entries, int max_cover, int stems, int stem,
                  float* masks, int chunks, int* nonfinite, cudaStream_t s);

}  // namespace ancha
