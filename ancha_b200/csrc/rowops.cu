// Row-wise kernels of the RoFormer stack: L2 "RMSNorm" (unit_norm, roformer.rs:16-24) with
// the operand cast for the next GEMM, the Mel per-transformer SourceNorm (roformer.rs:51-54,
// 516-519), the band-split gather + norm (network.rs:316-324) and the overlapping-band mask
// assembly (network.rs:382-396). One warp per row; reductions in fp32 with a fixed order.
#include "rowops.cuh"

#include <algorithm>

namespace ancha {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

// x: [rows, dim] f32 (row stride ldx). If `scale` (f32 [dim]) is given the residual stream
// is first replaced by unit_norm(x)·scale (SourceNorm). Then xn = unit_norm(x) is written
// as TO (row stride ldn). dim <= 32·MAXV.
template <typename TO, int MAXV>
__global__ void norm_rows_kernel(float* __restrict__ x, int64_t ldx, const float* __restrict__ scale,
                                 TO* __restrict__ xn, int64_t ldn, int64_t rows, int dim) {
    const int64_t row = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (row >= rows) return;
    float* xr = x + row * ldx;
    float v[MAXV];
    float sq = 0.f;
#pragma unroll
    for (int i = 0; i < MAXV; ++i) {
        const int c = lane + 32 * i;
        v[i] = c < dim ? xr[c] : 0.f;
        sq = fmaf(v[i], v[i], sq);
    }
    float inv = 1.f / fmaxf(sqrtf(warp_sum(sq)), 1e-12f);
    if (scale) {
        sq = 0.f;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int c = lane + 32 * i;
            if (c < dim) {
                v[i] = v[i] * inv * scale[c];
                xr[c] = v[i];
            }
            sq = fmaf(v[i], v[i], sq);
        }
        inv = 1.f / fmaxf(sqrtf(warp_sum(sq)), 1e-12f);
    }
    if (xn) {
        TO* o = xn + row * ldn;
#pragma unroll
        for (int i = 0; i < MAXV; ++i) {
            const int c = lane + 32 * i;
            if (c < dim) store_f(o + c, v[i] * inv);
        }
    }
}

// Cast f32 rows to TO (the mask-estimator input copy of the residual stream).
template <typename TO>
__global__ void cast_rows_kernel(const float* __restrict__ x, int64_t ldx, TO* __restrict__ y,
                                 int64_t ldy, int64_t rows, int dim) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= rows * dim) return;
    const int64_t r = i / dim;
    const int c = (int)(i % dim);
    store_f(y + r * ldy + c, x[r * ldx + c]);
}

// Band split front end: for every (chunk, frame, band) gather the band's spectrum columns
// and write them L2-normalised into z[(c·frames + t)·total + offset[b] + j].
__global__ void band_gather_kernel(const float* __restrict__ spec, int frames, int columns,
                                   const int* __restrict__ cols, const int* __restrict__ offsets,
                                   int bands, int total, float* __restrict__ z, int64_t units) {
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (unit >= units) return;
    const int b = (int)(unit % bands);
    const int64_t ct = unit / bands;  // c·frames + t
    const float* s = spec + ct * columns;
    const int o0 = offsets[b], o1 = offsets[b + 1];
    float sq = 0.f;
    for (int j = o0 + lane; j < o1; j += 32) {
        const float v = s[cols[j]];
        sq = fmaf(v, v, sq);
    }
    const float inv = 1.f / fmaxf(sqrtf(warp_sum(sq)), 1e-12f);
    float* zr = z + ct * total;
    for (int j = o0 + lane; j < o1; j += 32) zr[j] = s[cols[j]] * inv;
}

// The same gather in the tensor-core GEMM's operand layout: one zero-padded f16 row of kp
// features per (chunk, band, frame), z[((c·bands + b)·frames + t)·kp + j] (bands of a chunk are
// consecutive groups of `frames` rows), so one grouped launch covers every (chunk, band).
__global__ void band_gather_padded_kernel(const float* __restrict__ spec, int frames, int columns,
                                          const int* __restrict__ cols, const int* __restrict__ offsets,
                                          int bands, int kp, __half* __restrict__ z, int64_t units) {
    const int64_t unit = (int64_t)blockIdx.x * (blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (unit >= units) return;
    const int b = (int)(unit % bands);
    const int64_t ct = unit / bands;  // c·frames + t
    const int64_t c = ct / frames, t = ct % frames;
    const float* s = spec + ct * columns;
    const int o0 = offsets[b], width = offsets[b + 1] - o0;
    float sq = 0.f;
    for (int j = lane; j < width; j += 32) {
        const float v = s[cols[o0 + j]];
        sq = fmaf(v, v, sq);
    }
    const float inv = 1.f / fmaxf(sqrtf(warp_sum(sq)), 1e-12f);
    __half* zr = z + ((c * bands + b) * frames + t) * kp;
    for (int j = lane; j < kp; j += 32) zr[j] = __float2half_rn(j < width ? s[cols[o0 + j]] * inv : 0.f);
}

// masks[c][stem][r][ri][t] = sum over the bands covering spectrum row r of the GLU output
// glu[(c·bands + band)·frames + t][feature + ri] / coverage. `entries` lists, per row r,
// `count[r]` (band, feature) pairs in band order.
__global__ void mask_assemble_kernel(const float* __restrict__ glu, int64_t ldg, int bands,
                                     int frames, int rows, const int* __restrict__ count,
                                     const int2* __restrict__ entries, int max_cover, int stems,
                                     int stem, float* __restrict__ masks, int chunks,
                                     int* __restrict__ nonfinite) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int64_t total = (int64_t)chunks * rows * 2 * frames;
    if (i >= total) return;
    const int t = (int)(i % frames);
    const int ri = (int)((i / frames) % 2);
    const int r = (int)((i / (2 * frames)) % rows);
    const int c = (int)(i / ((int64_t)2 * frames * rows));
    const int n = count[r];
    float acc = 0.f;
    for (int e = 0; e < n; ++e) {
        const int2 be = entries[r * max_cover + e];
        acc += glu[((int64_t)(c * bands + be.x) * frames + t) * ldg + be.y + ri];
    }
    const float m = acc / (float)n;
    if (!isfinite(m)) atomicOr(nonfinite, 1);
    masks[((((int64_t)c * stems + stem) * rows + r) * 2 + ri) * frames + t] = m;
}

}  // namespace

int norm_rows(float* x, int64_t ldx, const float* scale, void* xn, int xn_type, int64_t ldn,
              int64_t rows, int dim, cudaStream_t s) {
    if (rows == 0) return ANCHA_OK;
    if (dim > 32 * 16) return fail(ANCHA_E_UNSUPPORTED, "norm_rows: dim > 512");
    const int wpb = 8;
    dim3 grid((unsigned)ceil_div(rows, wpb));
    if (xn_type == ELT_BF16)
        norm_rows_kernel<__nv_bfloat16, 16><<<grid, 32 * wpb, 0, s>>>(
            x, ldx, scale, reinterpret_cast<__nv_bfloat16*>(xn), ldn, rows, dim);
    else if (xn_type == ELT_F16)
        norm_rows_kernel<__half, 16><<<grid, 32 * wpb, 0, s>>>(
            x, ldx, scale, reinterpret_cast<__half*>(xn), ldn, rows, dim);
    else
        norm_rows_kernel<float, 16><<<grid, 32 * wpb, 0, s>>>(
            x, ldx, scale, reinterpret_cast<float*>(xn), ldn, rows, dim);
    return check_launch("norm_rows");
}

int cast_rows(const float* x, int64_t ldx, void* y, int y_type, int64_t ldy, int64_t rows,
              int dim, cudaStream_t s) {
    const int64_t n = rows * dim;
    if (n == 0) return ANCHA_OK;
    dim3 grid((unsigned)ceil_div(n, 256));
    if (y_type == ELT_BF16)
        cast_rows_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(x, ldx, reinterpret_cast<__nv_bfloat16*>(y), ldy, rows, dim);
    else if (y_type == ELT_F16)
        cast_rows_kernel<__half><<<grid, 256, 0, s>>>(x, ldx, reinterpret_cast<__half*>(y), ldy, rows, dim);
    else
        cast_rows_kernel<float><<<grid, 256, 0, s>>>(x, ldx, reinterpret_cast<float*>(y), ldy, rows, dim);
    return check_launch("cast_rows");
}

namespace {
__global__ void split3_kernel(const float* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y, int64_t ldy,
                              int64_t plane, int64_t rows, int dim) {
    const int64_t n = rows * dim;
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= n) return;
    const int64_t r = i / dim, c = i % dim;
    const float v = x[r * ldx + c];
    const __nv_bfloat16 h = __float2bfloat16_rn(v);
    const float r1 = v - __bfloat162float(h);
    const __nv_bfloat16 m = __float2bfloat16_rn(r1);
    const float r2 = r1 - __bfloat162float(m);
    const int64_t o = r * ldy + c;
    y[o] = h;
    y[plane + o] = m;
    y[2 * plane + o] = __float2bfloat16_rn(r2);
}
// Eight consecutive columns per thread (threadIdx.x over 8-column groups of a row, the y
// dimension over rows, grid-striding when rows exceed the grid).
__global__ void split3_vec_kernel(const float* __restrict__ x, int64_t ldx, __nv_bfloat16* __restrict__ y, int64_t ldy,
                                  int64_t plane, int64_t rows, int groups) {
    const int gcol = blockIdx.x * blockDim.x + threadIdx.x;
    if (gcol >= groups) return;
    for (int64_t r = (int64_t)blockIdx.y * blockDim.y + threadIdx.y; r < rows; r += (int64_t)gridDim.y * blockDim.y) {
        const float4* src = reinterpret_cast<const float4*>(x + r * ldx + gcol * 8);
        const float4 a = src[0], b = src[1];
        const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        uint32_t h[4], m[4], l[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const __nv_bfloat162 hh = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
            const float r0 = v[2 * i] - __low2float(hh), r1 = v[2 * i + 1] - __high2float(hh);
            const __nv_bfloat162 mm = __floats2bfloat162_rn(r0, r1);
            const __nv_bfloat162 ll = __floats2bfloat162_rn(r0 - __low2float(mm), r1 - __high2float(mm));
            h[i] = *reinterpret_cast<const uint32_t*>(&hh);
            m[i] = *reinterpret_cast<const uint32_t*>(&mm);
            l[i] = *reinterpret_cast<const uint32_t*>(&ll);
        }
        __nv_bfloat16* o = y + r * ldy + gcol * 8;
        *reinterpret_cast<uint4*>(o) = make_uint4(h[0], h[1], h[2], h[3]);
        *reinterpret_cast<uint4*>(o + plane) = make_uint4(m[0], m[1], m[2], m[3]);
        *reinterpret_cast<uint4*>(o + 2 * plane) = make_uint4(l[0], l[1], l[2], l[3]);
    }
}
}  // namespace

int split3_rows_strided(const float* x, int64_t ldx, void* y, int64_t ldy, int64_t plane, int64_t rows, int dim,
                        cudaStream_t s) {
    const int64_t n = rows * dim;
    if (n == 0) return ANCHA_OK;
    const uintptr_t xa = reinterpret_cast<uintptr_t>(x), ya = reinterpret_cast<uintptr_t>(y);
    if (dim % 8 == 0 && ldx % 4 == 0 && ldy % 8 == 0 && plane % 8 == 0 && xa % 16 == 0 && ya % 16 == 0) {
        // Eight columns per thread: two 16-byte loads, three 16-byte stores.
        const int groups = dim / 8;
        const dim3 block(32, 8);
        const dim3 grid((unsigned)ceil_div(groups, 32), (unsigned)std::min<int64_t>(ceil_div(rows, 8), 65535));
        split3_vec_kernel<<<grid, block, 0, s>>>(x, ldx, reinterpret_cast<__nv_bfloat16*>(y), ldy, plane, rows,
                                                  groups);
        return check_launch("split3_rows");
    }
    split3_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(x, ldx, reinterpret_cast<__nv_bfloat16*>(y), ldy, plane,
                                                             rows, dim);
    return check_launch("split3_rows");
}

int split3_rows(const float* x, int64_t ldx, void* y, int64_t rows, int dim, cudaStream_t s) {
    return split3_rows_strided(x, ldx, y, dim, rows * dim, rows, dim, s);
}

int band_gather(const float* spec, int chunks, int frames, int columns, const int* cols,
                const int* offsets, int bands, int total, float* z, cudaStream_t s) {
    const int64_t units = (int64_t)chunks * frames * bands;
    if (units == 0) return ANCHA_OK;
    const int wpb = 8;
    band_gather_kernel<<<(unsigned)ceil_div(units, wpb), 32 * wpb, 0, s>>>(
        spec, frames, columns, cols, offsets, bands, total, z, units);
    return check_launch("band_gather");
}

int band_gather_padded(const float* spec, int chunks, int frames, int columns, const int* cols,
                       const int* offsets, int bands, int kp, void* z, cudaStream_t s) {
    const int64_t units = (int64_t)chunks * frames * bands;
    if (units == 0) return ANCHA_OK;
    const int wpb = 8;
    band_gather_padded_kernel<<<(unsigned)ceil_div(units, wpb), 32 * wpb, 0, s>>>(
        spec, frames, columns, cols, offsets, bands, kp, reinterpret_cast<__half*>(z), units);
    return check_launch("band_gather_padded");
}

int mask_assemble(const float* glu, int64_t ldg, int bands, int frames, int rows,
                  const int* count, const int2* entries, int max_cover, int stems, int stem,
                  float* masks, int chunks, int* nonfinite, cudaStream_t s) {
    const int64_t total = (int64_t)chunks * rows * 2 * frames;
    if (total == 0) return ANCHA_OK;
    mask_assemble_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(
        glu, ldg, bands, frames, rows, count, entries, max_cover, stems, stem, masks, chunks,
        nonfinite);
    return check_launch("mask_assemble");
}

}  // namespace ancha
