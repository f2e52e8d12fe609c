// Classic MDX task kernels (declared in mdx_exec.hpp): the spectral front and back end and the
// Hann-weighted chunk overlap-add of src/mdx_runtime.rs, which the reference runs on the host.
//
// Its STFT sizes are not powers of two (n_fft 6144 = 3·2^11, 5120 = 5·2^10), so the n_fft-point
// real transform is an H = n_fft/2-point complex FFT of z[n] = x[2n] + i·x[2n+1] computed as R
// radix-2 FFTs of M = H/R points over the residues n mod R (decimation in time by R ∈ {1, 3, 5})
// followed by the radix-R combination X[k] = Σ_q W_H^{q·k}·F_q[k mod M], then the even/odd split.
// All twiddles come from one table exp(−2πij/n_fft), j ≤ n_fft/2, built in double precision.
#include "mdx_exec.hpp"

namespace ancha {
namespace {

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

// W_N^e for any integer e, from the half-circle table.
__device__ __forceinline__ float2 twiddle(const float2* __restrict__ tw, int n, int64_t e) {
    e %= n;
    if (e < 0) e += n;
    return e <= n / 2 ? tw[e] : conjf2(tw[n - e]);
}

__device__ __forceinline__ int64_t reflect(int64_t index, int64_t length) {
    if (length <= 1) return 0;
    const int64_t period = 2 * (length - 1);
    int64_t i = index % period;
    if (i < 0) i += period;
    return i < length ? i : period - i;
}

__global__ void task_tables_kernel(int n, float* __restrict__ window, float2* __restrict__ tw) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i <= n / 2) {
        double s, c;
        sincospi(-2.0 * i / n, &s, &c);
        tw[i] = make_float2((float)c, (float)s);
    }
    if (i < n) {
        const float arg = 6.28318548f * (float)i / (float)n;  // f32 TAU·i/n (dsp.rs:40-42)
        window[i] = 0.5f - 0.5f * cosf(arg);
    }
}

// Position of z[n] in the work buffer: residue block n mod R, bit-reversed index within it.
template <int R>
__device__ __forceinline__ int slot(int n, int m, int lm) {
    const int q = n % R, j = n / R;
    return q * m + (lm ? (int)(__brev((unsigned)j) >> (32 - lm)) : 0);
}

// buf: R blocks of m = 2^lm points, bit-reversed → out[k], k < R·m, the full complex FFT of the
// interleaved sequence. sign −1 forward, +1 inverse (unnormalised). All threads of the CTA.
template <int R>
__device__ void fft_mixed(float2* buf, float2* out, int m, const float2* __restrict__ tw, int n, float sign) {
    for (int len = 2; len <= m; len <<= 1) {
        const int half = len >> 1, stride = n / len;
        for (int i = threadIdx.x; i < R * (m / 2); i += blockDim.x) {
            const int blk = i / (m / 2), ii = i - blk * (m / 2);
            const int pos = ii & (half - 1);
            const int i0 = blk * m + 2 * (ii - pos) + pos, i1 = i0 + half;
            float2 w = tw[pos * stride];
            w.y *= -sign;
            const float2 a = buf[i0], b = cmul(buf[i1], w);
            buf[i0] = cadd(a, b);
            buf[i1] = csub(a, b);
        }
        __syncthreads();
    }
    const int h = R * m;
    for (int k = threadIdx.x; k < h; k += blockDim.x) {
        float2 acc = buf[k % m];
#pragma unroll
        for (int q = 1; q < R; ++q) {
            float2 w = twiddle(tw, n, 2 * (int64_t)q * k);  // W_H^{q·k} = W_N^{2·q·k}
            w.y *= -sign;
            acc = cadd(acc, cmul(w, buf[q * m + k % m]));
        }
        out[k] = acc;
    }
    __syncthreads();
}

// grid (frames, chunks · 2): one channel of one frame → packed[c][2·ch + re/im][f][t] for f <
// bins, the lowest `zero_low` bins zeroed (src/mdx_runtime.rs:79-83, src/spectral.rs:5-36).
template <int R>
__global__ void __launch_bounds__(256) task_stft_kernel(const float* __restrict__ audio, int samples, int hop,
                                                        int frames, int n, int m, int lm, int bins, int zero_low,
                                                        const float* __restrict__ win, const float2* __restrict__ tw,
                                                        float* __restrict__ packed) {
    extern __shared__ float2 sm[];
    const int h = n / 2;
    float2* buf = sm;
    float2* z = sm + h;
    const int t = blockIdx.x, cc = blockIdx.y;
    const float* x = audio + (int64_t)cc * samples;
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        const int64_t i0 = (int64_t)t * hop + 2 * i - h;
        buf[slot<R>(i, m, lm)] = make_float2(x[reflect(i0, samples)] * win[2 * i],
                                             x[reflect(i0 + 1, samples)] * win[2 * i + 1]);
    }
    __syncthreads();
    fft_mixed<R>(buf, z, m, tw, n, -1.f);
    const int c = cc / 2, ch = cc % 2;
    float* re = packed + ((int64_t)c * 4 + 2 * ch) * bins * frames + t;
    float* im = re + (int64_t)bins * frames;
    for (int k = threadIdx.x; k < bins; k += blockDim.x) {
        float2 X = make_float2(0.f, 0.f);
        if (k >= zero_low) {
            const float2 zk = z[k % h];
            const float2 zc = conjf2(z[(h - k % h) % h]);
            const float2 fe = make_float2(0.5f * (zk.x + zc.x), 0.5f * (zk.y + zc.y));
            const float2 d = csub(zk, zc);
            const float2 fo = make_float2(0.5f * d.y, -0.5f * d.x);  // d / (2i)
            X = cadd(fe, cmul(twiddle(tw, n, k), fo));
        }
        re[(int64_t)k * frames] = X.x;
        im[(int64_t)k * frames] = X.y;
    }
}

// grid (frames, chunks · 2): inverse of one channel's frame of spec[c][2·ch + re/im][f][t]
// (bins past `bins` zero, Im of DC and Nyquist dropped, 1/n) times the window, into
// scratch[c·2 + ch][t][n].
template <int R>
__global__ void __launch_bounds__(256) task_istft_kernel(const float* __restrict__ spec, int bins, int frames, int n,
                                                         int m, int lm, const float* __restrict__ win,
                                                         const float2* __restrict__ tw, float* __restrict__ scratch) {
    extern __shared__ float2 sm[];
    const int h = n / 2;
    float2* Y = sm;             // [h + 1]
    float2* buf = sm + h + 1;   // [h]
    float2* z = buf + h;        // [h]
    const int t = blockIdx.x, plane = blockIdx.y;
    const int c = plane / 2, ch = plane % 2;
    const float* re = spec + ((int64_t)c * 4 + 2 * ch) * bins * frames + t;
    const float* im = re + (int64_t)bins * frames;
    for (int k = threadIdx.x; k <= h; k += blockDim.x) {
        float2 y = k < bins ? make_float2(re[(int64_t)k * frames], im[(int64_t)k * frames]) : make_float2(0.f, 0.f);
        if (k == 0 || k == h) y.y = 0.f;
        Y[k] = y;
    }
    __syncthreads();
    for (int k = threadIdx.x; k < h; k += blockDim.x) {
        const float2 xk = Y[k];
        const float2 xc = conjf2(Y[h - k]);
        const float2 fe = make_float2(0.5f * (xk.x + xc.x), 0.5f * (xk.y + xc.y));
        const float2 d = make_float2(0.5f * (xk.x - xc.x), 0.5f * (xk.y - xc.y));
        const float2 fo = cmul(d, conjf2(twiddle(tw, n, k)));
        buf[slot<R>(k, m, lm)] = make_float2(fe.x - fo.y, fe.y + fo.x);  // fe + i·fo
    }
    __syncthreads();
    fft_mixed<R>(buf, z, m, tw, n, 1.f);
    float2* o = reinterpret_cast<float2*>(scratch + ((int64_t)plane * frames + t) * n);
    const float scale = 1.f / (float)h;
    for (int i = threadIdx.x; i < h; i += blockDim.x) {
        const float2 v = z[i];
        o[i] = make_float2(v.x * scale * win[2 * i], v.y * scale * win[2 * i + 1]);
    }
}

__global__ void task_gather_kernel(const float* __restrict__ planes, int64_t samples, MdxChunks4 ch, int chunk,
                                   int64_t trim, int64_t total, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int n = (int)(i % chunk);
    const int c2 = (int)((i / chunk) % 2);
    const int c = (int)(i / (2 * (int64_t)chunk));
    const int64_t pos = ch.start[c] + n;
    out[i] = n < ch.actual[c] && pos >= trim && pos < trim + samples ? planes[c2 * samples + pos - trim] : 0.f;
}

// One thread per output sample j in [lo, hi) of the trimmed track (chunks of the batch in order):
// weight = 1 (overlap 0) or the chunk's Hann weight in f64, rounded to f32 (mdx_runtime.rs:208-222).
__global__ void task_ola_kernel(const float* __restrict__ waves, MdxChunks4 ch, int chunks, int chunk, int64_t trim,
                                int64_t samples, int64_t lo, int64_t hi, int rectangular, float* __restrict__ result,
                                float* __restrict__ divisor) {
    const int64_t pos = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (pos >= hi) return;
    const int64_t o = pos - trim;
    float d = divisor[o], r0 = result[o], r1 = result[samples + o];
    for (int c = 0; c < chunks; ++c) {
        const int64_t s = ch.start[c];
        if (pos < s || pos >= s + ch.actual[c]) continue;
        const int64_t local = pos - s;
        const float w = rectangular ? 1.f
                                    : (float)(0.5 - 0.5 * cos(6.283185307179586 * (double)local /
                                                                (double)(ch.actual[c] - 1)));
        d += w;
        r0 += waves[((int64_t)c * 2) * chunk + local] * w;
        r1 += waves[((int64_t)c * 2 + 1) * chunk + local] * w;
    }
    divisor[o] = d;
    result[o] = r0;
    result[samples + o] = r1;
}

__global__ void task_finish_kernel(const float* __restrict__ result, const float* __restrict__ divisor,
                                   const float* __restrict__ input, int64_t samples, float compensate,
                                   float* __restrict__ predicted, float* __restrict__ residual, int* __restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= 2 * samples) return;
    const float d = divisor[i % samples];
    if (!(d > 0.f)) atomicOr(flag, 2);
    const float p = result[i] / d * compensate;
    if (!isfinite(p)) atomicOr(flag, 1);
    predicted[i] = p;
    residual[i] = input[i] - p;
}

__global__ void half_difference_kernel(const float* __restrict__ a, const float* __restrict__ b, int64_t n,
                                       float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = (a[i] - b[i]) * 0.5f;
}

__global__ void negate_kernel(const float* __restrict__ a, int64_t n, float* __restrict__ out) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        out[i] = -a[i];
}

unsigned grid_of(int64_t n) { return (unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 32); }

// (R, m, lm) of an n-point real transform, or false when n/2 is not R·2^lm with R ∈ {1, 3, 5}.
bool split(int n, int& r, int& m, int& lm) {
    if (n < 4 || n % 2) return false;
    const int h = n / 2;
    for (int cand : {1, 3, 5}) {
        if (h % cand) continue;
        const int mm = h / cand;
        if (mm & (mm - 1)) continue;
        r = cand;
        m = mm;
        lm = 0;
        while ((1 << lm) < mm) ++lm;
        return true;
    }
    return false;
}

template <typename K>
int set_smem(K kernel, size_t bytes) {
    if (bytes > 48 * 1024) ANCHA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
    return ANCHA_OK;
}

}  // namespace

bool mdx_task_fft_supported(int n_fft) {
    int r, m, lm;
    return n_fft <= 8192 && split(n_fft, r, m, lm);
}

int mdx_task_tables(int n_fft, float* window, float2* twiddle_table, cudaStream_t s) {
    if (!mdx_task_fft_supported(n_fft))
        return fail(ANCHA_E_UNSUPPORTED, "classic MDX STFT: n_fft/2 must be 2^k, 3·2^k or 5·2^k, n_fft <= 8192");
    task_tables_kernel<<<(unsigned)ceil_div(n_fft, 256), 256, 0, s>>>(n_fft, window, twiddle_table);
    return check_launch("mdx_task_tables");
}

int mdx_task_stft(const float* audio, int chunks, int samples, int hop, int n_fft, int bins, int zero_low,
                  const float* window, const float2* twiddle_table, float* packed, cudaStream_t s) {
    int r, m, lm;
    if (!split(n_fft, r, m, lm) || hop <= 0 || samples <= n_fft / 2 || bins <= 0 || bins > n_fft / 2 + 1)
        return fail(ANCHA_E_INVALID, "mdx_task_stft: shape");
    if (chunks <= 0) return ANCHA_OK;
    const int frames = samples / hop + 1;
    const size_t smem = (size_t)n_fft * sizeof(float2);  // buf + z: 2·(n/2)
    const dim3 grid(frames, chunks * 2);
    if (r == 1) {
        ANCHA_TRY(set_smem(task_stft_kernel<1>, smem));
        task_stft_kernel<1><<<grid, 256, smem, s>>>(audio, samples, hop, frames, n_fft, m, lm, bins, zero_low, window,
                                                    twiddle_table, packed);
    } else if (r == 3) {
        ANCHA_TRY(set_smem(task_stft_kernel<3>, smem));
        task_stft_kernel<3><<<grid, 256, smem, s>>>(audio, samples, hop, frames, n_fft, m, lm, bins, zero_low, window,
                                                    twiddle_table, packed);
    } else {
        ANCHA_TRY(set_smem(task_stft_kernel<5>, smem));
        task_stft_kernel<5><<<grid, 256, smem, s>>>(audio, samples, hop, frames, n_fft, m, lm, bins, zero_low, window,
                                                    twiddle_table, packed);
    }
    return check_launch("mdx_task_stft");
}

int mdx_task_istft(const float* spec, int chunks, int bins, int frames, int hop, int samples, int n_fft,
                   const float* window, const float2* twiddle_table, float* scratch, float* waves, int* flag,
                   cudaStream_t s) {
    int r, m, lm;
    if (!split(n_fft, r, m, lm) || hop <= 0 || frames <= 0 || bins <= 0 || bins > n_fft / 2 + 1 ||
        (int64_t)samples + n_fft / 2 > (int64_t)(frames - 1) * hop + n_fft)
        return fail(ANCHA_E_INVALID, "mdx_task_istft: shape");
    if (chunks <= 0) return ANCHA_OK;
    const size_t smem = (size_t)(3 * (n_fft / 2) + 1) * sizeof(float2);
    const dim3 grid(frames, chunks * 2);
    if (r == 1) {
        ANCHA_TRY(set_smem(task_istft_kernel<1>, smem));
        task_istft_kernel<1><<<grid, 256, smem, s>>>(spec, bins, frames, n_fft, m, lm, window, twiddle_table, scratch);
    } else if (r == 3) {
        ANCHA_TRY(set_smem(task_istft_kernel<3>, smem));
        task_istft_kernel<3><<<grid, 256, smem, s>>>(spec, bins, frames, n_fft, m, lm, window, twiddle_table, scratch);
    } else {
        ANCHA_TRY(set_smem(task_istft_kernel<5>, smem));
        task_istft_kernel<5><<<grid, 256, smem, s>>>(spec, bins, frames, n_fft, m, lm, window, twiddle_table, scratch);
    }
    ANCHA_TRY(check_launch("mdx_task_istft"));
    return mdx_istft_overlap(scratch, (int64_t)chunks * 2, frames, hop, samples, n_fft, window, waves, flag, s);
}

int mdx_task_gather(const float* planes, int64_t samples, const MdxChunks4& ch, int chunks, int chunk, int64_t trim,
                    float* out, cudaStream_t s) {
    if (chunks <= 0) return ANCHA_OK;
    const int64_t total = (int64_t)chunks * 2 * chunk;
    task_gather_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(planes, samples, ch, chunk, trim, total, out);
    return check_launch("mdx_task_gather");
}

int mdx_task_ola(const float* waves, const MdxChunks4& ch, int chunks, int chunk, int64_t trim, int64_t samples,
                 bool rectangular, float* result, float* divisor, cudaStream_t s) {
    if (chunks <= 0) return ANCHA_OK;
    int64_t lo = INT64_MAX, hi = INT64_MIN;
    for (int c = 0; c < chunks; ++c) {
        lo = std::min<int64_t>(lo, std::max<int64_t>(ch.start[c], trim));
        hi = std::max<int64_t>(hi, std::min<int64_t>(ch.start[c] + ch.actual[c], trim + samples));
    }
    if (hi <= lo) return ANCHA_OK;
    task_ola_kernel<<<(unsigned)ceil_div(hi - lo, 256), 256, 0, s>>>(waves, ch, chunks, chunk, trim, samples, lo, hi,
                                                                     rectangular ? 1 : 0, result, divisor);
    return check_launch("mdx_task_ola");
}

int mdx_task_finish(const float* result, const float* divisor, const float* input, int64_t samples, float compensate,
                    float* predicted, float* residual, int* flag, cudaStream_t s) {
    task_finish_kernel<<<(unsigned)ceil_div(2 * samples, 256), 256, 0, s>>>(result, divisor, input, samples,
                                                                           compensate, predicted, residual, flag);
    return check_launch("mdx_task_finish");
}

int mdx_negate(const float* a, int64_t n, float* out, cudaStream_t s) {
    negate_kernel<<<grid_of(n), 256, 0, s>>>(a, n, out);
    return check_launch("mdx_negate");
}

int mdx_half_difference(const float* a, const float* b, int64_t n, float* out, cudaStream_t s) {
    half_difference_kernel<<<grid_of(n), 256, 0, s>>>(a, b, n, out);
    return check_launch("mdx_half_difference");
}

}  // namespace ancha
