// Spectral runtime of the MDX23C task on the device (declared in mdx23c.cuh): UVR chunk
// windows, the centred n_fft-point STFT packed as [4][bins][frames], its inverse per stem and
// the rectangular chunk overlap-add of src/mdx23c_runtime.rs:135-248 and src/spectral.rs,
// which the reference runs on the host (realfft) between its device model calls.
//
// An n_fft-point real transform runs as an n_fft/2-point complex FFT of z[n] = x[2n] + i·x[2n+1]
// in shared memory (radix-2, decimation in time) plus the even/odd split, one CTA per
// (frame, chunk, channel). Twiddles come from one table exp(−2πik/8192), k ≤ 4096, built in
// double precision; a power-of-two size N reads it with stride 8192/N.
#include "mdx23c.cuh"

namespace ancha {
namespace {

constexpr int kMaxFft = 8192;

__global__ void dsp_tables_kernel(int n_fft, float* __restrict__ window, float2* __restrict__ twiddle) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i <= kMaxFft / 2) {
        double s, c;
        sincospi(-2.0 * i / kMaxFft, &s, &c);
        twiddle[i] = make_float2((float)c, (float)s);
    }
    if (i < n_fft) {
        const float arg = 6.28318548f * (float)i / (float)n_fft;  // f32 TAU·i/n (dsp.rs:40-42)
        window[i] = 0.5f - 0.5f * cosf(arg);
    }
}

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

__device__ __forceinline__ int64_t reflect(int64_t index, int64_t length) {
    if (length <= 1) return 0;
    const int64_t period = 2 * (length - 1);
    int64_t i = index % period;
    if (i < 0) i += period;
    return i < length ? i : period - i;
}

// In-place complex FFT of h = 2^lh points of `buf` (bit-reversed input), all threads of the
// CTA; sign −1 forward, +1 inverse (unnormalised).
__device__ void fft_pow2(float2* buf, int h, const float2* __restrict__ tw, float sign) {
    for (int len = 2; len <= h; len <<= 1) {
        const int half = len >> 1, stride = kMaxFft / len;
        for (int i = threadIdx.x; i < h / 2; i += blockDim.x) {
            const int pos = i & (half - 1);
            const int i0 = 2 * (i - pos) + pos, i1 = i0 + half;
            float2 w = tw[pos * stride];
            w.y *= -sign;
            const float2 a = buf[i0], b = cmul(buf[i1], w);
            buf[i0] = cadd(a, b);
            buf[i1] = csub(a, b);
        }
        __syncthreads();
    }
}

// grid (frames, chunks · 2): one channel of one frame.
__global__ void __launch_bounds__(256) stft_kernel(const float* __restrict__ audio, int samples, int hop, int frames,
                                                   int n_fft, int lh, int bins, const float* __restrict__ win,
                                                   const float2* __restrict__ tw, float* __restrict__ out) {
    extern __shared__ float2 buf[];  // [n_fft / 2]
    const int h = n_fft / 2;
    const int t = blockIdx.x, cc = blockIdx.y;
    const float* x = audio + (int64_t)cc * samples;
    for (int n = threadIdx.x; n < h; n += blockDim.x) {
        const int64_t i0 = (int64_t)t * hop + 2 * n - h;
        const float a = x[reflect(i0, samples)] * win[2 * n];
        const float b = x[reflect(i0 + 1, samples)] * win[2 * n + 1];
        buf[__brev(n) >> (32 - lh)] = make_float2(a, b);
    }
    __syncthreads();
    fft_pow2(buf, h, tw, -1.f);
    const int c = cc / 2, ch = cc % 2;
    float* re = out + ((int64_t)c * 4 + 2 * ch) * bins * frames + t;
    float* im = re + (int64_t)bins * frames;
    const int stride = kMaxFft / n_fft;
    for (int k = threadIdx.x; k < bins; k += blockDim.x) {
        const float2 zk = buf[k & (h - 1)];
        const float2 zc = conjf2(buf[(h - k) & (h - 1)]);
        const float2 fe = make_float2(0.5f * (zk.x + zc.x), 0.5f * (zk.y + zc.y));
        const float2 d = csub(zk, zc);
        const float2 fo = make_float2(0.5f * d.y, -0.5f * d.x);  // d / (2i)
        const float2 X = cadd(fe, cmul(tw[k * stride], fo));
        re[(int64_t)k * frames] = X.x;
        im[(int64_t)k * frames] = X.y;
    }
}

// grid (frames, chunks · stems · 2): one channel of one stem's frame → windowed time frame in
// scratch[plane][frame][n_fft], plane = (c · stems + stem) · 2 + ch.
__global__ void __launch_bounds__(256) istft_frames_kernel(const float* __restrict__ spec, int stems, int bins,
                                                           int frames, int n_fft, int lh,
                                                           const float* __restrict__ win,
                                                           const float2* __restrict__ tw,
                                                           float* __restrict__ scratch) {
    extern __shared__ float2 sm[];
    const int h = n_fft / 2;
    float2* Y = sm;           // [h + 1]
    float2* buf = sm + h + 1;  // [h]
    const int t = blockIdx.x, plane = blockIdx.y;
    const int ch = plane % 2, stem = (plane / 2) % stems, c = plane / (2 * stems);
    const float* re = spec + (((int64_t)c * stems + stem) * 4 + 2 * ch) * bins * frames + t;
    const float* im = re + (int64_t)bins * frames;
    for (int k = threadIdx.x; k <= h; k += blockDim.x) {
        float2 y = k < bins ? make_float2(re[(int64_t)k * frames], im[(int64_t)k * frames]) : make_float2(0.f, 0.f);
        if (k == 0 || k == h) y.y = 0.f;
        Y[k] = y;
    }
    __syncthreads();
    const int stride = kMaxFft / n_fft;
    for (int k = threadIdx.x; k < h; k += blockDim.x) {
        const float2 xk = Y[k];
        const float2 xc = conjf2(Y[h - k]);
        const float2 fe = make_float2(0.5f * (xk.x + xc.x), 0.5f * (xk.y + xc.y));
        const float2 d = make_float2(0.5f * (xk.x - xc.x), 0.5f * (xk.y - xc.y));
        const float2 fo = cmul(d, conjf2(tw[k * stride]));
        buf[__brev(k) >> (32 - lh)] = make_float2(fe.x - fo.y, fe.y + fo.x);  // fe + i·fo
    }
    __syncthreads();
    fft_pow2(buf, h, tw, 1.f);
    float2* o = reinterpret_cast<float2*>(scratch + ((int64_t)plane * frames + t) * n_fft);
    const float scale = 1.f / (float)h;  // the reference's 1/n_fft on its c2r output
    for (int n = threadIdx.x; n < h; n += blockDim.x) {
        const float2 z = buf[n];
        o[n] = make_float2(z.x * scale * win[2 * n], z.y * scale * win[2 * n + 1]);
    }
}

// waves[plane][i] = Σ_t frame_t[i + n_fft/2 − t·hop] / Σ_t w²[…], frames in ascending order.
__global__ void istft_overlap_kernel(const float* __restrict__ scratch, int64_t planes, int frames, int hop,
                                     int samples, int n_fft, const float* __restrict__ win, float* __restrict__ out,
                                     int* __restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= planes * samples) return;
    const int64_t p = i / samples;
    const int j = (int)(i % samples) + n_fft / 2;
    const int t0 = j - (n_fft - 1) <= 0 ? 0 : (j - (n_fft - 1) + hop - 1) / hop;
    const int t1 = min(frames - 1, j / hop);
    float num = 0.f, den = 0.f;
    const float* f = scratch + p * frames * n_fft;
    for (int t = t0; t <= t1; ++t) {
        const int n = j - t * hop;
        const float w = win[n];
        num += f[(int64_t)t * n_fft + n];
        den += w * w;
    }
    if (!(den > 1e-11f)) atomicOr(flag, 2);
    out[i] = num / den;
}

struct Starts4 {
    int64_t v[4];
};

__global__ void gather_kernel(const float* __restrict__ planes, int64_t samples, Starts4 starts, int chunk,
                              int64_t border, int64_t total, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int n = (int)(i % chunk);
    const int ch = (int)((i / chunk) % 2);
    const int c = (int)(i / (2 * (int64_t)chunk));
    const int64_t pos = starts.v[c] + n - border;
    out[i] = pos >= 0 && pos < samples ? planes[ch * samples + pos] : 0.f;
}

// One thread per (plane, sample j of the bordered track in [lo, hi)): chunks in order.
__global__ void overlap_add_kernel(const float* __restrict__ waves, Starts4 starts, int chunks, int planes, int chunk,
                                   int64_t border, int64_t samples, int64_t lo, int64_t hi, float* __restrict__ sums,
                                   int* __restrict__ flag) {
    const int64_t j = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    const int p = blockIdx.y;
    if (j >= hi) return;
    float acc = sums[(int64_t)p * samples + j - border];
    for (int c = 0; c < chunks; ++c) {
        const int64_t s = starts.v[c];
        if (j < s || j >= s + chunk) continue;
        const float v = waves[((int64_t)c * planes + p) * chunk + (j - s)];
        if (!isfinite(v)) atomicOr(flag, 1);
        acc += v;
    }
    sums[(int64_t)p * samples + j - border] = acc;
}

__global__ void scale_kernel(float* __restrict__ x, int64_t n, float k) {
    for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
        x[i] *= k;
}

int log2_exact(int n) {
    int l = 0;
    while ((1 << l) < n) ++l;
    return (1 << l) == n ? l : -1;
}

}  // namespace

int mdx_dsp_tables(int n_fft, float* window, float2* twiddle, cudaStream_t s) {
    if (n_fft < 32 || n_fft > kMaxFft || log2_exact(n_fft) < 0)
        return fail(ANCHA_E_UNSUPPORTED, "mdx_dsp: n_fft must be a power of two in 32..8192");
    dsp_tables_kernel<<<(unsigned)ceil_div(std::max(n_fft, kMaxFft / 2 + 1), 256), 256, 0, s>>>(n_fft, window, twiddle);
    return check_launch("mdx_dsp_tables");
}

int mdx_gather(const float* planes, int64_t samples, const int64_t* starts, int chunks, int chunk, int64_t border,
               float* out, cudaStream_t s) {
    if (chunks <= 0) return ANCHA_OK;
    if (chunks > 4) return fail(ANCHA_E_INVALID, "mdx_gather: at most 4 chunks per call");
    Starts4 st{};
    for (int c = 0; c < chunks; ++c) st.v[c] = starts[c];
    const int64_t total = (int64_t)chunks * 2 * chunk;
    gather_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(planes, samples, st, chunk, border, total, out);
    return check_launch("mdx_gather");
}

int mdx_stft(const MdxDsp& d, const float* audio, int chunks, int samples, int hop, int bins, float* out,
             cudaStream_t s) {
    const int lh = log2_exact(d.n_fft / 2);
    if (lh < 0 || hop <= 0 || hop > d.n_fft / 2 || samples <= d.n_fft / 2 || bins <= 0 || bins > d.n_fft / 2 + 1)
        return fail(ANCHA_E_INVALID, "mdx_stft: shape");
    if (chunks <= 0) return ANCHA_OK;
    const int frames = samples / hop + 1;
    const size_t smem = (size_t)(d.n_fft / 2) * sizeof(float2);
    if (smem > 48 * 1024) ANCHA_CUDA(cudaFuncSetAttribute(stft_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    stft_kernel<<<dim3(frames, chunks * 2), 256, smem, s>>>(audio, samples, hop, frames, d.n_fft, lh, bins, d.window,
                                                          d.twiddle, out);
    return check_launch("mdx_stft");
}

int mdx_istft(const MdxDsp& d, const float* spec, int chunks, int stems, int bins, int frames, int hop, int samples,
              float* scratch, float* waves, int* flag, cudaStream_t s) {
    const int lh = log2_exact(d.n_fft / 2);
    if (lh < 0 || hop <= 0 || frames <= 0 || bins <= 0 || bins > d.n_fft / 2 + 1 ||
        (int64_t)samples + d.n_fft / 2 > (int64_t)(frames - 1) * hop + d.n_fft)
        return fail(ANCHA_E_INVALID, "mdx_istft: shape");
    if (chunks <= 0 || stems <= 0) return ANCHA_OK;
    const int64_t planes = (int64_t)chunks * stems * 2;
    if (planes > 65535) return fail(ANCHA_E_UNSUPPORTED, "mdx_istft: too many planes");
    const size_t smem = (size_t)(d.n_fft + 1) * sizeof(float2);
    if (smem > 48 * 1024)
        ANCHA_CUDA(cudaFuncSetAttribute(istft_frames_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    istft_frames_kernel<<<dim3(frames, (unsigned)planes), 256, smem, s>>>(spec, stems, bins, frames, d.n_fft, lh,
                                                                         d.window, d.twiddle, scratch);
    ANCHA_TRY(check_launch("mdx_istft_frames"));
    istft_overlap_kernel<<<(unsigned)ceil_div(planes * samples, 256), 256, 0, s>>>(scratch, planes, frames, hop, samples,
                                                                                d.n_fft, d.window, waves, flag);
    return check_launch("mdx_istft_overlap");
}

int mdx_istft_overlap(const float* scratch, int64_t planes, int frames, int hop, int samples, int n_fft,
                      const float* window, float* out, int* flag, cudaStream_t s) {
    if (planes <= 0) return ANCHA_OK;
    istft_overlap_kernel<<<(unsigned)ceil_div(planes * samples, 256), 256, 0, s>>>(scratch, planes, frames, hop, samples,
                                                                                n_fft, window, out, flag);
    return check_launch("mdx_istft_overlap");
}

int mdx_overlap_add(const float* waves, const int64_t* starts, int chunks, int planes, int chunk, int64_t border,
                    int64_t samples, float* sums, int* flag, cudaStream_t s) {
    if (chunks <= 0) return ANCHA_OK;
    if (chunks > 4 || planes > 65535) return fail(ANCHA_E_INVALID, "mdx_overlap_add: shape");
    Starts4 st{};
    for (int c = 0; c < chunks; ++c) st.v[c] = starts[c];
    const int64_t lo = std::max<int64_t>(starts[0], border);
    const int64_t hi = std::min<int64_t>(starts[chunks - 1] + chunk, border + samples);
    if (hi <= lo) return ANCHA_OK;
    overlap_add_kernel<<<dim3((unsigned)ceil_div(hi - lo, 256), planes), 256, 0, s>>>(
        waves, st, chunks, planes, chunk, border, samples, lo, hi, sums, flag);
    return check_launch("mdx_overlap_add");
}

int mdx_scale(float* x, int64_t n, float k, cudaStream_t s) {
    if (n <= 0) return ANCHA_OK;
    scale_kernel<<<(unsigned)std::min<int64_t>(ceil_div(n, 256), 148 * 16), 256, 0, s>>>(x, n, k);
    return check_launch("mdx_scale");
}

}  // namespace ancha
