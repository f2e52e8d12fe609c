// MDX23C device kernels (declared in mdx23c.cuh). All of them are HBM-bound gathers and
// elementwise passes around the network's GEMMs:
//
// * mdx_plane_sums: f64 sum and sum of squares per NCHW plane for tensors no GEMM produced
//   (the GEMM epilogues accumulate them for their own outputs); every consumer turns a plane's
//   sums into one (scale, shift) pair, so normalising is one FMA (the instance norms of
//   mdx23c.rs:200-213 reduce over a whole (batch, channel) plane, so the statistics must be
//   complete before any element is normalised);
// * mdx_pack: norm → GELU → zero-padded patch gather into the K-major patch matrix of a
//   convolution (the B operand of out[co][pos] = W[co][k]·P[pos][k]ᵀ), over a channel
//   concatenation of two sources so the decoder's cat(up, skip) and the final cat(mix, x)
//   are never materialised. One CTA stages the normalised input rows of 32 output columns ×
//   32 channels in shared memory and writes each patch row's 32·kh·kw columns contiguously;
// * mdx_norm_act, mdx_transpose, mdx_shuffle2x2: the TDF input, the time / frequency swaps
//   of mdx23c.rs:437 and 475, and the ConvTranspose2d(2, 2) scatter (spatial.rs:128-150).
#include "mdx23c.cuh"

#include <type_traits>

#include "tc.cuh"  // gelu_fast

namespace ancha {
namespace {

constexpr int kPackCols = 32;   // output columns per CTA
constexpr int kPackChans = 32;  // channels per CTA
constexpr int kSplits = 32;     // at most this many CTAs per plane in mdx_plane_sums

__global__ void plane_sums_kernel(const float* __restrict__ x, int64_t n, double2* __restrict__ sums) {
    const int64_t plane = blockIdx.x;
    const int64_t per = (n + gridDim.y - 1) / gridDim.y;
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
        if (lane == 0) {
            atomicAdd(&sums[plane].x, s);
            atomicAdd(&sums[plane].y, q);
        }
    }
}

// (scale, shift) of the instance norm of one plane: γ/√(var + eps) and β − mean·scale.
__device__ __forceinline__ float2 norm_coef(double2 sum, int64_t n, float gamma, float beta, float eps) {
    const double mean = sum.x / (double)n;
    const double var = fmax(sum.y / (double)n - mean * mean, 0.0);
    const double scale = (double)gamma / sqrt(var + (double)eps);
    return make_float2((float)scale, (float)((double)beta - mean * scale));
}


// GELU of a value that is stored in a 16-bit type (gelu_fast of tc.cuh: one MUFU ex2,
// |Δ| ≤ 7e-7, far below the storage rounding) or in f32 (the exact erf form).
template <typename OutT>
__device__ __forceinline__ float gelu_out(float x) {
    if constexpr (std::is_same<OutT, float>::value) return gelu_erf(x);
    else return gelu_fast(x);
}

// Norm coefficients for a 16-bit consumer: statistics in f64, the reciprocal square root in
// f32 (relative error ~1e-7, far below the 16-bit storage).
__device__ __forceinline__ float2 norm_coef_fast(double2 sum, int64_t n, float gamma, float beta, float eps) {
    const double mean = sum.x / (double)n;
    const double var = fmax(sum.y / (double)n - mean * mean, 0.0);
    const float scale = gamma * rsqrtf((float)var + eps);
    return make_float2(scale, beta - (float)mean * scale);
}

// Coefficients of channel c of the concatenation (a, b) for image `img`; (1, 0) without norm.
template <typename OutT>
__device__ __forceinline__ float2 source_coef(const PackArgs& a, int img, int c, int64_t n) {
    const bool first = c < a.a.channels;
    const PackSource& src = first ? a.a : a.b;
    const int cs = first ? c : c - a.a.channels;
    if (!src.sums) return make_float2(1.f, 0.f);
    const double2 sum = src.sums[(int64_t)img * src.channels + cs];
    return std::is_same<OutT, float>::value ? norm_coef(sum, n, src.gamma[cs], src.beta[cs], a.eps)
                                            : norm_coef_fast(sum, n, src.gamma[cs], src.beta[cs], a.eps);
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
    __shared__ float2 coef[kPackChans];
    const int ctot = a.a.channels + a.b.channels;
    const int chunk = blockIdx.z % nchunks, b = blockIdx.z / nchunks;
    const int ho = blockIdx.y, wo0 = blockIdx.x * kPackCols;
    const int c0 = chunk * kPackChans, cc = min(kPackChans, ctot - c0);
    const int hi0 = ho * S - a.ph, wi0 = wo0 * S - a.pw;
    const int64_t plane_n = (int64_t)a.h * a.w;
    if (threadIdx.x < cc) coef[threadIdx.x] = source_coef<OutT>(a, b, c0 + threadIdx.x, plane_n);
    __syncthreads();
    for (int i = threadIdx.x; i < cc * K * NCOLS; i += blockDim.x) {
        const int col = i % NCOLS, r = (i / NCOLS) % K, cl = i / (NCOLS * K), c = c0 + cl;
        const int hi = hi0 + r, wi = wi0 + col;
        float v = 0.f;
        if (hi >= 0 && hi < a.h && wi >= 0 && wi < a.w) {
            const bool first = c < a.a.channels;
            const PackSource& src = first ? a.a : a.b;
            const int64_t plane = (int64_t)b * src.channels + (first ? c : c - a.a.channels);
            v = fmaf(src.x[plane * plane_n + (int64_t)hi * a.w + wi], coef[cl].x, coef[cl].y);
            if (a.gelu) v = gelu_out<OutT>(v);
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

// 128 positions × 64 channels per CTA through shared memory: every thread issues its 32
// coalesced loads (8 channel rows × 4 runs of 32 positions) before any use, then each warp
// writes whole 128-byte channel runs of 16 positions. Row stride 129 keeps both phases free
// of shared-memory bank conflicts (2-way on the channel pairs).
constexpr int kPreactPos = 128;
template <typename OutT>
__global__ void __launch_bounds__(256) preact_nhwc_kernel(const PackArgs a, int64_t pos, OutT* __restrict__ out) {
    __shared__ float t[64][kPreactPos + 1];
    __shared__ float2 coef[64];
    const int ctot = a.a.channels + a.b.channels;
    const int64_t p0 = (int64_t)blockIdx.x * kPreactPos;
    const int c0 = blockIdx.y * 64, img = blockIdx.z;
    const int tx = threadIdx.x % 32, ty = threadIdx.x / 32;
    if (threadIdx.x < 64) {
        const int c = c0 + threadIdx.x;
        const bool first = c < a.a.channels;
        const PackSource& src = first ? a.a : a.b;
        const int cs = first ? c : c - a.a.channels;
        coef[threadIdx.x] = src.sums ? norm_coef_fast(src.sums[(int64_t)img * src.channels + cs], pos, src.gamma[cs],
                                                      src.beta[cs], a.eps)
                                     : make_float2(1.f, 0.f);
    }
    float v[8][4];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = ty + 8 * i, c = c0 + r;
        const bool first = c < a.a.channels;
        const PackSource& src = first ? a.a : a.b;
        const float* plane = src.x + ((int64_t)img * src.channels + (first ? c : c - a.a.channels)) * pos;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int64_t q = p0 + 32 * j + tx;
            v[i][j] = q < pos ? plane[q] : 0.f;
        }
    }
    __syncthreads();  // coef
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int r = ty + 8 * i;
        const float2 k = coef[r];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            float x = fmaf(v[i][j], k.x, k.y);
            if (a.gelu) x = gelu_out<OutT>(x);
            t[r][32 * j + tx] = x;
        }
    }
    __syncthreads();
    for (int q = ty; q < kPreactPos; q += 8) {
        if (p0 + q >= pos) break;
        OutT* row = out + ((int64_t)img * pos + p0 + q) * ctot + c0;
        const float v0 = t[2 * tx][q], v1 = t[2 * tx + 1][q];
        if constexpr (std::is_same<OutT, __half>::value)
            reinterpret_cast<__half2*>(row)[tx] = __floats2half2_rn(v0, v1);
        else
            reinterpret_cast<__nv_bfloat162*>(row)[tx] = __floats2bfloat162_rn(v0, v1);
    }
}

// grid (segments, planes): one plane's coefficients per CTA, 8 elements per thread when the
// plane length allows 16-byte vectors, else one.
template <typename OutT>
__global__ void __launch_bounds__(256) norm_act_kernel(const float* __restrict__ x, int64_t n, int channels,
                                                       const double2* __restrict__ sums,
                                                       const float* __restrict__ gamma,
                                                       const float* __restrict__ beta, float eps, bool gelu,
                                                       bool vec, OutT* __restrict__ out) {
    const int64_t plane = blockIdx.y;
    const int c = (int)(plane % channels);
    const float2 k = !sums ? make_float2(1.f, 0.f)
                     : std::is_same<OutT, float>::value ? norm_coef(sums[plane], n, gamma[c], beta[c], eps)
                                                        : norm_coef_fast(sums[plane], n, gamma[c], beta[c], eps);
    const float* xp = x + plane * n;
    OutT* op = out + plane * n;
    if (vec) {
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n / 8; i += (int64_t)gridDim.x * blockDim.x) {
            const float4 a = reinterpret_cast<const float4*>(xp + i * 8)[0];
            const float4 b = reinterpret_cast<const float4*>(xp + i * 8)[1];
            float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
            for (int u = 0; u < 8; ++u) {
                v[u] = fmaf(v[u], k.x, k.y);
                if (gelu) v[u] = gelu_out<OutT>(v[u]);
            }
            Pack8<OutT>::store(op + i * 8, v);
        }
    } else {
        for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
            float v = fmaf(xp[i], k.x, k.y);
            if (gelu) v = gelu_out<OutT>(v);
            store_f(op + i, v);
        }
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

// grid (⌈w / 256⌉, 2·h, batch · channels): thread x writes the pair of output columns
// (2x, 2x + 1) of output row oy, which come from the dx = 0 and dx = 1 GEMM rows at input
// position (oy / 2, x).
__global__ void shuffle2x2_kernel(const float* __restrict__ y, int channels, int h, int w, float* __restrict__ out,
                                  int c_total, int c_off) {
    const int x = blockIdx.x * blockDim.x + threadIdx.x;
    if (x >= w) return;
    const int oy = blockIdx.y;
    const int64_t bc = blockIdx.z;
    const int64_t b = bc / channels, c = bc % channels;
    const int64_t plane = (int64_t)h * w;
    const float* src = y + ((b * channels + c) * 4 + (oy & 1) * 2) * plane + (int64_t)(oy >> 1) * w + x;
    const float2 v = make_float2(src[0], src[plane]);
    reinterpret_cast<float2*>(out + ((b * c_total + c_off + c) * 2 * h + oy) * (int64_t)(2 * w))[x] = v;
}

}  // namespace

int mdx_plane_sums(const float* x, int64_t planes, int64_t n, double2* sums, cudaStream_t s) {
    if (planes <= 0 || n <= 0) return fail(ANCHA_E_INVALID, "mdx_plane_sums: empty");
    if (planes > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "mdx_plane_sums: too many planes");
    const int splits = (int)std::min<int64_t>(kSplits, ceil_div(n, 4096));
    plane_sums_kernel<<<dim3((unsigned)planes, splits), 256, 0, s>>>(x, n, sums);
    return check_launch("mdx_plane_sums");
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

int mdx_preact_nhwc(const PackSource& a, const PackSource& b, int batch, int64_t pos, bool gelu, float eps,
                    void* out, int out_type, cudaStream_t s) {
    const int ctot = a.channels + b.channels;
    if (batch <= 0 || pos <= 0 || ctot <= 0 || ctot % 64 || (out_type != ELT_F16 && out_type != ELT_BF16))
        return fail(ANCHA_E_INVALID, "mdx_preact_nhwc: shape");
    if (batch > 65535 || ctot / 64 > 65535 || ceil_div(pos, kPreactPos) > 0x7fffffff)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_preact_nhwc: grid too large");
    PackArgs p{};
    p.a = a; p.b = b; p.gelu = gelu; p.eps = eps;
    const dim3 grid((unsigned)ceil_div(pos, kPreactPos), (unsigned)(ctot / 64), (unsigned)batch);
    if (out_type == ELT_F16)
        preact_nhwc_kernel<__half><<<grid, 256, 0, s>>>(p, pos, reinterpret_cast<__half*>(out));
    else
        preact_nhwc_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(p, pos, reinterpret_cast<__nv_bfloat16*>(out));
    return check_launch("mdx_preact_nhwc");
}

int mdx_norm_act(const float* x, int64_t planes, int64_t n, int channels, const double2* sums, const float* gamma,
                 const float* beta, float eps, bool gelu, void* out, int out_type, cudaStream_t s) {
    if (planes <= 0 || n <= 0) return ANCHA_OK;
    if (planes > 65535) return fail(ANCHA_E_UNSUPPORTED, "mdx_norm_act: too many planes");
    const bool vec = n % 8 == 0 && reinterpret_cast<uintptr_t>(x) % 32 == 0 && reinterpret_cast<uintptr_t>(out) % 32 == 0;
    const int64_t per_plane = vec ? n / 8 : n;
    const int segs = (int)std::max<int64_t>(1, std::min<int64_t>(ceil_div(per_plane, 256), ceil_div(148 * 8, planes)));
    const dim3 grid((unsigned)segs, (unsigned)planes);
    if (out_type == ELT_F16)
        norm_act_kernel<__half><<<grid, 256, 0, s>>>(x, n, channels, sums, gamma, beta, eps, gelu, vec,
                                                     reinterpret_cast<__half*>(out));
    else if (out_type == ELT_BF16)
        norm_act_kernel<__nv_bfloat16><<<grid, 256, 0, s>>>(x, n, channels, sums, gamma, beta, eps, gelu, vec,
                                                            reinterpret_cast<__nv_bfloat16*>(out));
    else
        norm_act_kernel<float><<<grid, 256, 0, s>>>(x, n, channels, sums, gamma, beta, eps, gelu, vec,
                                                    reinterpret_cast<float*>(out));
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
    if (batch <= 0 || channels <= 0 || h <= 0 || w <= 0) return ANCHA_OK;
    if ((int64_t)batch * channels > 65535 || 2 * (int64_t)h > 65535)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_shuffle2x2: grid too large");
    const dim3 grid((unsigned)ceil_div(w, 256), (unsigned)(2 * h), (unsigned)(batch * channels));
    shuffle2x2_kernel<<<grid, 256, 0, s>>>(y, channels, h, w, out, c_total, c_off);
    return check_launch("mdx_shuffle2x2");
}

}  // namespace ancha
