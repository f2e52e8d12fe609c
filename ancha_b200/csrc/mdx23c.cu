// MDX23C device kernels (declared in mdx23c.cuh). All of them are HBM-bound gathers and
// elementwise passes around the network's GEMMs:
//
// * mdx_norm_coef: f64 sum and sum of squares per NCHW plane, folded with gamma / beta into
//   one (scale, shift) per plane (the instance norms of mdx23c.rs:200-213 reduce over a whole
//   (batch, channel) plane, so the statistics must be complete before any element is
//   normalised);
// * mdx_pack: norm → GELU → zero-padded patch gather into the K-major patch matrix of a
//   convolution (the B operand of out[co][pos] = W[co][k]·P[pos][k]ᵀ), over a channel
//   concatenation of two sources so the decoder's cat(up, skip) and the final cat(mix, x)
//   are never materialised. One CTA stages the normalised input rows of 32 output columns ×
//   32 channels in shared memory and writes each patch row's 32·kh·kw columns contiguously;
// * mdx_norm_act, mdx_transpose, mdx_shuffle2x2: the TDF input, the time / frequency swaps
//   of mdx23c.rs:437 and 475, and the ConvTranspose2d(2, 2) scatter (spatial.rs:128-150).
#include "mdx23c.cuh"

#include <type_traits>

namespace ancha {
namespace {

constexpr int kPackCols = 32;   // output columns per CTA
constexpr int kPackChans = 32;  // channels per CTA
constexpr int kSplits = 32;     // partial sums per plane in mdx_norm_coef

__global__ void plane_sums_kernel(const float* __restrict__ x, int64_t n, double2* __restrict__ part) {
    const int64_t plane = blockIdx.x;
    const int64_t per = (n + kSplits - 1) / kSplits;
    const int64_t lo = per * blockIdx.y, hi = min(n, lo + per);
    const float* p = x + plane * n;
    double s = 0.0, q = 0.0;
    for (int64_t i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const double v = p[i];
        s += v;
        q += v * v;
    }
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    __shared__ double ws[2][32];
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    if (lane == 0) { ws[0][warp] = s; ws[1][warp] = q; }
    __syncthreads();
    if (warp == 0) {
        const int nw = blockDim.x / 32;
        s = lane < nw ? ws[0][lane] : 0.0;
        q = lane < nw ? ws[1][lane] : 0.0;
        for (int o = 16; o > 0; o >>= 1) {
            s += __shfl_xor_sync(0xffffffffu, s, o);
            q += __shfl_xor_sync(0xffffffffu, q, o);
        }
        if (lane == 0) part[plane * kSplits + blockIdx.y] = make_double2(s, q);
    }
}

// One warp per plane: add the partial sums, then scale = γ/√(var + eps), shift = β − mean·scale.
__global__ void plane_coef_kernel(const double2* __restrict__ part, int64_t planes, int64_t n, int channels,
                                  const float* __restrict__ gamma, const float* __restrict__ beta, float eps,
                                  float2* __restrict__ coef) {
    const int64_t plane = blockIdx.x * (int64_t)(blockDim.x / 32) + threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    if (plane >= planes) return;
    const double2 v = part[plane * kSplits + lane];  // kSplits == 32: one partial per lane
    double s = v.x, q = v.y;
    for (int o = 16; o > 0; o >>= 1) {
        s += __shfl_xor_sync(0xffffffffu, s, o);
        q += __shfl_xor_sync(0xffffffffu, q, o);
    }
    if (lane == 0) {
        const double mean = s / (double)n;
        const double var = fmax(q / (double)n - mean * mean, 0.0);
        const int c = (int)(plane % channels);
        const double scale = (double)gamma[c] / sqrt(var + (double)eps);
        coef[plane] = make_float2((float)scale, (float)((double)beta[c] - mean * scale));
    }
}

template <typename T> struct Pack8;
template <> struct Pack8<float> {
    static __device__ __forceinline__ void store(float* p, const float (&v)[8]) {
        reinterpret_cast<float4*>(p)[0] = make_float4(v[0], v[1], v[2], v[3]);
        reinterpret_cast<float4*>(p)[1] = make_float4(v[4], v[5], v[6], v[7]);
    }
};
template <> struct Pack8<__half> {
    static __device__ __forceinline__ void store(__half* p, const float (&v)[8]) {
        uint4 u;
        __half2 h[4] = {__floats2half2_rn(v[0], v[1]), __floats2half2_rn(v[2], v[3]), __floats2half2_rn(v[4], v[5]),
                        __floats2half2_rn(v[6], v[7])};
        memcpy(&u, h, 16);
        *reinterpret_cast<uint4*>(p) = u;
    }
};
template <> struct Pack8<__nv_bfloat16> {
    static __device__ __forceinline__ void store(__nv_bfloat16* p, const float (&v)[8]) {
        uint4 u;
        __nv_bfloat162 h[4] = {__floats2bfloat162_rn(v[0], v[1]), __floats2bfloat162_rn(v[2], v[3]),
                               __floats2bfloat162_rn(v[4], v[5]), __floats2bfloat162_rn(v[6], v[7])};
        memcpy(&u, h, 16);
        *reinterpret_cast<uint4*>(p) = u;
    }
};

// K × K taps, stride S (compile-time, so the patch-column arithmetic is shifts and
// multiplies). Every CTA's column range [k0, k0 + width) of a patch row starts and ends on
// a multiple of 8, so it is written in 8-element vectors.
template <int K, int S, typename OutT>
__global__ void __launch_bounds__(256) pack_kernel(const PackArgs a, int nchunks) {
    constexpr int NCOLS = (kPackCols - 1) * S + K;
    constexpr int TAPS = K * K;
    __shared__ float tile[kPackChans * K * NCOLS];
    const int ctot = a.a.channels + a.b.channels;
    const int chunk = blockIdx.z % nchunks, b = blockIdx.z / nchunks;
    const int ho = blockIdx.y, wo0 = blockIdx.x * kPackCols;
    const int c0 = chunk * kPackChans, cc = min(kPackChans, ctot - c0);
    const int hi0 = ho * S - a.ph, wi0 = wo0 * S - a.pw;
    const int64_t plane_n = (int64_t)a.h * a.w;
    for (int i = threadIdx.x; i < cc * K * NCOLS; i += blockDim.x) {
        const int col = i % NCOLS, r = (i / NCOLS) % K, c = c0 + i / (NCOLS * K);
        const int hi = hi0 + r, wi = wi0 + col;
        float v = 0.f;
        if (hi >= 0 && hi < a.h && wi >= 0 && wi < a.w) {
            const bool first = c < a.a.channels;
            const PackSource& src = first ? a.a : a.b;
            const int64_t plane = (int64_t)b * src.channels + (first ? c : c - a.a.channels);
            v = src.x[plane * plane_n + (int64_t)hi * a.w + wi];
            if (src.coef) {
                const float2 k = src.coef[plane];
                v = fmaf(v, k.x, k.y);
            }
            if (a.gelu) v = gelu_erf(v);
        }
        tile[i] = v;
    }
    __syncthreads();
    const int span = cc * TAPS;  // patch columns this CTA writes per output position
    const int k0 = c0 * TAPS;
    const int width8 = (c0 + cc == ctot ? (int)(a.kp - k0) : span) / 8;  // the last chunk zero-fills the pad
    const int nwo = min(kPackCols, a.wo_n - wo0);
    OutT* out = reinterpret_cast<OutT*>(a.out);
    const int64_t row0 = (int64_t)b * a.ho_n * a.wo_n + (int64_t)ho * a.wo_n + wo0;
    for (int i = threadIdx.x; i < nwo * width8; i += blockDim.x) {
        const int wl = i / width8, j0 = (i - wl * width8) * 8;
        float v[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            const int j = j0 + u;
            const int jc = min(j, span - 1);  // keeps the shared-memory index inside the tile
            const int c = jc / TAPS, t = jc - c * TAPS, ky = t / K, kx = t - ky * K;
            const float x = tile[(c * K + ky) * NCOLS + wl * S + kx];
            v[u] = j < span ? x : 0.f;
        }
        Pack8<OutT>::store(out + (row0 + wl) * a.kp + k0 + j0, v);
    }
}

// 32 positions × 64 channels per CTA through shared memory: coalesced reads along the planes,
// 128-byte writes along the channels.
template <typename OutT>
__global__ void __launch_bounds__(256) preact_nhwc_kernel(const PackSource a, const PackSource b, int64_t pos,
                                                          bool gelu, OutT* __restrict__ out) {
    __shared__ float t[64][33];
    const int ctot = a.channels + b.channels;
    const int64_t p0 = (int64_t)blockIdx.x * 32;
    const int c0 = blockIdx.y * 64, img = blockIdx.z;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    for (int r = ty; r < 64; r += 8) {
        const int c = c0 + r;
        const int64_t q = p0 + tx;
        float v = 0.f;
        if (q < pos) {
            const bool first = c < a.channels;
            const PackSource& src = first ? a : b;
            const int64_t plane = (int64_t)img * src.channels + (first ? c : c - a.channels);
            v = src.x[plane * pos + q];
            if (src.coef) {
                const float2 k = src.coef[plane];
                v = fmaf(v, k.x, k.y);
            }
            if (gelu) v = gelu_erf(v);
        }
        t[r][tx] = v;
    }
    __syncthreads();
    for (int r = ty; r < 32; r += 8) {
        const int64_t q = p0 + r;
        if (q >= pos) break;
        OutT* row = out + ((int64_t)img * pos + q) * ctot + c0;
        const float v0 = t[2 * tx][r], v1 = t[2 * tx + 1][r];
        if constexpr (sizeof(OutT) == 2) {
            if constexpr (std::is_same<OutT, __half>::value)
                reinterpret_cast<__half2*>(row)[tx] = __floats2half2_rn(v0, v1);
            else
                reinterpret_cast<__nv_bfloat162*>(row)[tx] = __floats2bfloat162_rn(v0, v1);
        }
    }
}

// Planes whose length is not a multiple of 8 (small bottlenecks): one element per thread.
__global__ void norm_act_scalar_kernel(const float* __restrict__ x, int64_t total, int64_t n,
                                       const float2* __restrict__ coef, bool gelu, void* out, int out_type) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const float2 k = coef ? coef[i / n] : make_float2(1.f, 0.f);
        float v = fmaf(x[i], k.x, k.y);
        if (gelu) v = gelu_erf(v);
        store_elt(out, i, v, out_type);
    }
}

template <typename OutT>
__global__ void norm_act_kernel(const float* __restrict__ x, int64_t total8, int64_t n,
                                const float2* __restrict__ coef, bool gelu, OutT* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total8;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int64_t e = i * 8;
        const float4 a = reinterpret_cast<const float4*>(x + e)[0];
        const float4 b = reinterpret_cast<const float4*>(x + e)[1];
        float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
        const float2 k = coef ? coef[e / n] : make_float2(1.f, 0.f);  // n % 8 == 0: one plane per vector
#pragma unroll
        for (int u = 0; u < 8; ++u) {
            v[u] = fmaf(v[u], k.x, k.y);
            if (gelu) v[u] = gelu_erf(v[u]);
        }
        Pack8<OutT>::store(out + e, v);
    }
}

__global__ void transpose_kernel(const float* __restrict__ x, const float* __restrict__ mul, int rows,
                                 int cols, float* __restrict__ out) {
    __shared__ float t[32][33];
    const int64_t plane = blockIdx.z;
    const float* src = x + plane * rows * (int64_t)cols;
    const int r0 = blockIdx.y * 32, c0 = blockIdx.x * 32;
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int r = r0 + j, c = c0 + threadIdx.x;
        if (r < rows && c < cols) t[j][threadIdx.x] = src[(int64_t)r * cols + c];
    }
    __syncthreads();
    for (int j = threadIdx.y; j < 32; j += blockDim.y) {
        const int c = c0 + j, r = r0 + threadIdx.x;
        if (r < rows && c < cols) {
            const int64_t o = plane * rows * (int64_t)cols + (int64_t)c * rows + r;
            out[o] = t[threadIdx.x][j] * (mul ? mul[o] : 1.f);
        }
    }
}

__global__ void shuffle2x2_kernel(const float* __restrict__ y, int channels, int h, int w,
                                  int64_t total, float* __restrict__ out, int c_total, int c_off) {
    const int ow = 2 * w, oh = 2 * h;
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total;
         i += (int64_t)gridDim.x * blockDim.x) {
        const int ox = (int)(i % ow);
        const int oy = (int)((i / ow) % oh);
        const int c = (int)((i / ((int64_t)ow * oh)) % channels);
        const int64_t b = i / ((int64_t)ow * oh * channels);
        const int row = (c * 2 + (oy & 1)) * 2 + (ox & 1);
        const float v = y[(b * channels * 4 + row) * (int64_t)h * w + (int64_t)(oy >> 1) * w + (ox >> 1)];
        out[((b * c_total + c_off + c) * oh + oy) * (int64_t)ow + ox] = v;
    }
}

int grid_for(int64_t total) {
    return (int)std::min<int64_t>(ceil_div(total, 256), 148 * 16);
}

}  // namespace

int mdx_norm_coef(const float* x, int64_t planes, int64_t n, int channels, const float* gamma,
                  const float* beta, float eps, double2* scratch, float2* coef, cudaStream_t s) {
    if (planes <= 0 || n <= 0 || channels <= 0) return fail(ANCHA_E_INVALID, "mdx_norm_coef: empty");
    if (planes > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "mdx_norm_coef: too many planes");
    plane_sums_kernel<<<dim3((unsigned)planes, kSplits), 256, 0, s>>>(x, n, scratch);
    ANCHA_TRY(check_launch("mdx_norm_coef"));
    plane_coef_kernel<<<(unsigned)ceil_div(planes, 8), 256, 0, s>>>(scratch, planes, n, channels, gamma, beta, eps,
                                                                      coef);
    return check_launch("mdx_norm_coef");
}

namespace {
template <int K, int S>
int launch_pack(const PackArgs& a, dim3 grid, int nchunks, cudaStream_t s) {
    if (a.out_type == ELT_F16) pack_kernel<K, S, __half><<<grid, 256, 0, s>>>(a, nchunks);
    else if (a.out_type == ELT_BF16) pack_kernel<K, S, __nv_bfloat16><<<grid, 256, 0, s>>>(a, nchunks);
    else pack_kernel<K, S, float><<<grid, 256, 0, s>>>(a, nchunks);
    return check_launch("mdx_pack");
}
}  // namespace

int mdx_pack(const PackArgs& a, cudaStream_t s) {
    const int ctot = a.a.channels + a.b.channels;
    if (a.batch <= 0 || ctot <= 0 || a.ho_n <= 0 || a.wo_n <= 0 || a.kp % 8 || a.kp < (int64_t)ctot * a.kh * a.kw)
        return fail(ANCHA_E_INVALID, "mdx_pack: shape");
    if (reinterpret_cast<uintptr_t>(a.out) % 32) return fail(ANCHA_E_INVALID, "mdx_pack: output alignment");
    const int nchunks = (ctot + kPackChans - 1) / kPackChans;
    if ((int64_t)a.batch * nchunks > 65535 || a.ho_n > 65535)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_pack: grid too large");
    const dim3 grid((unsigned)ceil_div(a.wo_n, kPackCols), (unsigned)a.ho_n, (unsigned)(a.batch * nchunks));
    const bool same = a.kh == a.kw && a.sh == a.sw;
    if (same && a.kh == 1 && a.sh == 1 && a.ph == 0 && a.pw == 0) return launch_pack<1, 1>(a, grid, nchunks, s);
    if (same && a.kh == 3 && a.sh == 1 && a.ph == 1 && a.pw == 1) return launch_pack<3, 1>(a, grid, nchunks, s);
    if (same && a.kh == 2 && a.sh == 2 && a.ph == 0 && a.pw == 0) return launch_pack<2, 2>(a, grid, nchunks, s);
    return fail(ANCHA_E_UNSUPPORTED, "mdx_pack: geometry");
}

int mdx_preact_nhwc(const PackSource& a, const PackSource& b, int batch, int64_t pos, bool gelu, void* out,
                    int out_type, cudaStream_t s) {
    const int ctot = a.channels + b.channels;
    if (batch <= 0 || pos <= 0 || ctot <= 0 || ctot % 64 || (out_type != ELT_F16 && out_type != ELT_BF16))
        return fail(ANCHA_E_INVALID, "mdx_preact_nhwc: shape");
    if (batch > 65535 || ctot / 64 > 65535 || ceil_div(pos, 32) > 0x7fffffff)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_preact_nhwc: grid too large");
    const dim3 grid((unsigned)ceil_div(pos, 32), (unsigned)(ctot / 64), (unsigned)batch);
    if (out_type == ELT_F16)
        preact_nhwc_kernel<__half><<<grid, 256, 0, s>>>(a, b, pos, gelu, reinterpret_cast<__half*>(out));
    else
        preact_nhwc_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(a, b, pos, gelu, reinterpret_cast<__nv_bfloat16*>(out));
    return check_launch("mdx_preact_nhwc");
}

int mdx_norm_act(const float* x, int64_t planes, int64_t n, const float2* coef, bool gelu, void* out, int out_type,
                 cudaStream_t s) {
    const int64_t total = planes * n;
    if (total <= 0) return ANCHA_OK;
    if (n % 8 || reinterpret_cast<uintptr_t>(x) % 32 || reinterpret_cast<uintptr_t>(out) % 32) {
        norm_act_scalar_kernel<<<grid_for(total), 256, 0, s>>>(x, total, n, coef, gelu, out, out_type);
        return check_launch("mdx_norm_act");
    }
    const int64_t total8 = total / 8;
    const int g = grid_for(total8);
    if (out_type == ELT_F16)
        norm_act_kernel<__half><<<g, 256, 0, s>>>(x, total8, n, coef, gelu, reinterpret_cast<__half*>(out));
    else if (out_type == ELT_BF16)
        norm_act_kernel<__nv_bfloat16><<<g, 256, 0, s>>>(x, total8, n, coef, gelu, reinterpret_cast<__nv_bfloat16*>(out));
    else
        norm_act_kernel<float><<<g, 256, 0, s>>>(x, total8, n, coef, gelu, reinterpret_cast<float*>(out));
    return check_launch("mdx_norm_act");
}

int mdx_transpose(const float* x, const float* mul, int64_t planes, int rows, int cols, float* out,
                  cudaStream_t s) {
    if (planes <= 0 || rows <= 0 || cols <= 0) return ANCHA_OK;
    if (planes > 65535) return fail(ANCHA_E_UNSUPPORTED, "mdx_transpose: too many planes");
    transpose_kernel<<<dim3((unsigned)ceil_div(cols, 32), (unsigned)ceil_div(rows, 32), (unsigned)planes),
                       dim3(32, 8), 0, s>>>(x, mul, rows, cols, out);
    return check_launch("mdx_transpose");
}

int mdx_shuffle2x2(const float* y, int batch, int channels, int h, int w, float* out, int c_total,
                   int c_off, cudaStream_t s) {
    const int64_t total = (int64_t)batch * channels * 4 * h * w;
    if (total <= 0) return ANCHA_OK;
    shuffle2x2_kernel<<<grid_for(total), 256, 0, s>>>(y, channels, h, w, total, out, c_total, c_off);
    return check_launch("mdx_shuffle2x2");
}

}  // namespace ancha
