// Spectral front and back end on the device: chunk gather (runtime.rs:117-142), centered
// periodic-Hann STFT with the model packing (dsp.rs:52-79, runtime.rs:148-162), complex-mask
// multiply + inverse STFT with window-square normalised overlap-add (runtime.rs:181-201,
// dsp.rs:82-133), linear-fade chunk overlap-add (chunk.rs:26-88) and the border crop.
//
// The 2048-point real FFT runs as a 1024-point complex FFT of z[n] = x[2n] + i·x[2n+1] in
// shared memory (radix-2, decimation in time) plus the standard even/odd split; one CTA
// transforms both channels of a frame so the packed (bin, channel, re/im) output is written
// as contiguous float4s. Twiddles come from double-precision sincospi, rounded to f32.
#include "dsp.cuh"

#include <mutex>

namespace ancha {
namespace {

constexpr int NFFT = 2048, NH = 1024, BINS = 1025;

__device__ float2 g_tw1024[NH / 2];  // exp(-2πik/1024)
__device__ float2 g_tw2048[BINS];    // exp(-2πik/2048)
__device__ float g_hann[NFFT];       // periodic Hann, f32 as dsp.rs:40-42

__global__ void dsp_tables_kernel() {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < NH / 2) {
        double s, c;
        sincospi(-2.0 * i / NH, &s, &c);
        g_tw1024[i] = make_float2((float)c, (float)s);
    }
    if (i < BINS) {
        double s, c;
        sincospi(-2.0 * i / NFFT, &s, &c);
        g_tw2048[i] = make_float2((float)c, (float)s);
    }
    if (i < NFFT) {
        const float arg = 6.28318548f * (float)i / (float)NFFT;  // f32 TAU·i/n
        g_hann[i] = 0.5f - 0.5f * cosf(arg);
    }
}

std::once_flag g_table_once[64];
int g_table_status[64];

__device__ __forceinline__ float2 cadd(float2 a, float2 b) { return make_float2(a.x + b.x, a.y + b.y); }
__device__ __forceinline__ float2 csub(float2 a, float2 b) { return make_float2(a.x - b.x, a.y - b.y); }
__device__ __forceinline__ float2 cmul(float2 a, float2 b) {
    return make_float2(a.x * b.x - a.y * b.y, a.x * b.y + a.y * b.x);
}
__device__ __forceinline__ float2 conjf2(float2 a) { return make_float2(a.x, -a.y); }

__device__ __forceinline__ int64_t reflect_dev(int64_t index, int64_t length) {
    if (length <= 1) return 0;
    const int64_t period = 2 * (length - 1);
    int64_t i = index % period;
    if (i < 0) i += period;
    return i < length ? i : period - i;
}

__device__ __forceinline__ int bitrev10(int n) { return __brev(n) >> 22; }

// In-place 1024-point FFT of `buf` (already in bit-reversed order), all threads of the CTA.
// `sign` = -1 forward, +1 inverse (unnormalised).
__device__ void fft1024(float2* buf, float sign) {
    for (int len = 2; len <= NH; len <<= 1) {
        const int half = len >> 1, step = NH / len;
        for (int i = threadIdx.x; i < NH / 2; i += blockDim.x) {
            const int pos = i % half;
            const int i0 = (i / half) * len + pos, i1 = i0 + half;
            float2 w = g_tw1024[pos * step];
            w.y *= -sign;
            const float2 a = buf[i0], b = cmul(buf[i1], w);
            buf[i0] = cadd(a, b);
            buf[i1] = csub(a, b);
        }
        __syncthreads();
    }
}

// grid (frames, chunks), 256 threads: both channels of one frame.
__global__ void __launch_bounds__(256)
stft_kernel(const float* __restrict__ audio, int samples, int hop, int frames,
            float* __restrict__ packed) {
    __shared__ float2 buf[2][NH];
    const int t = blockIdx.x, c = blockIdx.y;
    for (int ch = 0; ch < 2; ++ch) {
        const float* x = audio + ((int64_t)c * 2 + ch) * samples;
        for (int n = threadIdx.x; n < NH; n += blockDim.x) {
            const int64_t i0 = (int64_t)t * hop + 2 * n - NH;
            const float a = x[reflect_dev(i0, samples)] * g_hann[2 * n];
            const float b = x[reflect_dev(i0 + 1, samples)] * g_hann[2 * n + 1];
            buf[ch][bitrev10(n)] = make_float2(a, b);
        }
    }
    __syncthreads();
    fft1024(buf[0], -1.f);
    fft1024(buf[1], -1.f);
    float4* out = reinterpret_cast<float4*>(packed + ((int64_t)c * frames + t) * (BINS * 4));
    for (int k = threadIdx.x; k < BINS; k += blockDim.x) {
        float2 X[2];
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            const float2 zk = buf[ch][k & (NH - 1)];
            const float2 zc = conjf2(buf[ch][(NH - k) & (NH - 1)]);
            const float2 fe = make_float2(0.5f * (zk.x + zc.x), 0.5f * (zk.y + zc.y));
            const float2 d = csub(zk, zc);
            const float2 fo = make_float2(0.5f * d.y, -0.5f * d.x);  // d / (2i)
            X[ch] = cadd(fe, cmul(g_tw2048[k], fo));
        }
        out[k] = make_float4(X[0].x, X[0].y, X[1].x, X[1].y);
    }
}

// grid (frames, stems, chunks): masked spectrum → windowed frames of both channels in
// scratch[((c·stems + s)·2 + ch)·frames + t][2048].
__global__ void __launch_bounds__(256)
istft_frames_kernel(const float* __restrict__ packed, const float* __restrict__ masks,
                    int stems, int frames, int zero_dc, float* __restrict__ scratch) {
    __shared__ float2 Y[2][BINS];
    __shared__ float2 buf[2][NH];
    const int t = blockIdx.x, s = blockIdx.y, c = blockIdx.z;
    const float4* spec = reinterpret_cast<const float4*>(packed + ((int64_t)c * frames + t) * (BINS * 4));
    const float* m = masks + ((int64_t)c * stems + s) * (int64_t)(2 * BINS) * 2 * frames + t;
    for (int k = threadIdx.x; k < BINS; k += blockDim.x) {
        const float4 sv = spec[k];
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            const int64_t r = (int64_t)(2 * k + ch) * 2 * frames;
            const float2 mk = make_float2(m[r], m[r + frames]);
            const float2 sk = ch ? make_float2(sv.z, sv.w) : make_float2(sv.x, sv.y);
            float2 y = cmul(sk, mk);
            if (k == 0 || k == BINS - 1) y.y = 0.f;
            if (k == 0 && zero_dc) y.x = 0.f;
            Y[ch][k] = y;
        }
    }
    __syncthreads();
    for (int k = threadIdx.x; k < NH; k += blockDim.x) {
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
            const float2 xk = Y[ch][k];
            const float2 xc = conjf2(Y[ch][NH - k]);
            const float2 fe = make_float2(0.5f * (xk.x + xc.x), 0.5f * (xk.y + xc.y));
            const float2 d = make_float2(0.5f * (xk.x - xc.x), 0.5f * (xk.y - xc.y));
            const float2 fo = cmul(d, conjf2(g_tw2048[k]));
            buf[ch][bitrev10(k)] = make_float2(fe.x - fo.y, fe.y + fo.x);  // fe + i·fo
        }
    }
    __syncthreads();
    fft1024(buf[0], 1.f);
    fft1024(buf[1], 1.f);
    for (int ch = 0; ch < 2; ++ch) {
        float2* o = reinterpret_cast<float2*>(scratch + ((((int64_t)c * stems + s) * 2 + ch) * frames + t) * NFFT);
        for (int n = threadIdx.x; n < NH; n += blockDim.x) {
            const float2 z = buf[ch][n];
            const float scale = 1.f / (float)NH;  // (c2r / 2048) of the reference
            o[n] = make_float2(z.x * scale * g_hann[2 * n], z.y * scale * g_hann[2 * n + 1]);
        }
    }
}

// out[c][s][ch][i] = Σ_t frame_t[i + 1024 − t·hop] / Σ_t w²[…], frames in ascending order.
__global__ void istft_overlap_kernel(const float* __restrict__ scratch, int64_t planes, int frames,
                                     int hop, int samples, float* __restrict__ out,
                                     int* __restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= planes * samples) return;
    const int64_t p = i / samples;
    const int j = (int)(i % samples) + NH;
    int t0 = j - (NFFT - 1) <= 0 ? 0 : (j - (NFFT - 1) + hop - 1) / hop;
    const int t1 = min(frames - 1, j / hop);
    float num = 0.f, den = 0.f;
    const float* f = scratch + p * frames * NFFT;
    for (int t = t0; t <= t1; ++t) {
        const int n = j - t * hop;
        const float w = g_hann[n];
        num += f[(int64_t)t * NFFT + n];
        den += w * w;
    }
    if (!(den > 1e-11f)) atomicOr(flag, 2);
    out[i] = num / den;
}

// Chunk input with reflect / zero tail (runtime.rs:117-142): grid over chunks·2·chunk.
// planes holds track samples [pcm_lo, pcm_lo + pcm_len) of each channel (row stride pcm_len).
__global__ void gather_chunks_kernel(const float* __restrict__ planes, int64_t samples, int64_t pcm_lo,
                                     int64_t pcm_len, ChunkStarts starts, int chunks, int chunk,
                                     int64_t border, int64_t length, float* __restrict__ out) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)chunks * 2 * chunk) return;
    const int n = (int)(i % chunk);
    const int ch = (int)((i / chunk) % 2);
    const int c = (int)(i / (2 * (int64_t)chunk));
    const int64_t start = starts.v[c];
    const int64_t remaining = min(length - start, (int64_t)chunk);
    float v = 0.f;
    if (!(n >= remaining && remaining <= chunk / 2)) {
        const int64_t local = n < remaining ? n : reflect_dev(n, remaining);
        v = planes[ch * pcm_len + reflect_dev(start + local - border, samples) - pcm_lo];
    }
    out[i] = v;
}

__device__ __forceinline__ float fade_weight(int i, int chunk, bool first, bool last) {
    const int fade = max(chunk / 10, 1);
    if (!first && i < fade) return (float)(i + 1) / (float)fade;
    if (!last && i >= chunk - fade) return (float)(chunk - i) / (float)fade;
    return 1.f;
}

// Overlap-add of `chunks` outputs y[c][planes][chunk] into sums / weights, chunk order.
// Absolute sample j of the padded track lives at index j − base of the span buffers
// (row stride `span`); fades use the true track `length` (chunk.rs:26-35, 52-75).
__global__ void ola_kernel(const float* __restrict__ y, int chunks, int planes, int chunk,
                           ChunkStarts starts, int64_t length, int64_t base, int64_t span,
                           int64_t lo, int64_t hi, float* __restrict__ sums,
                           float* __restrict__ weights) {
    const int64_t j = lo + (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (j >= hi) return;
    const int64_t o = j - base;
    float wsum = weights[o];
    for (int c = 0; c < chunks; ++c) {
        const int64_t s = starts.v[c];
        if (j < s || j >= s + chunk) continue;
        const int i = (int)(j - s);
        const float w = fade_weight(i, chunk, s == 0, s + chunk >= length);
        wsum += w;
        for (int p = 0; p < planes; ++p)
            sums[(int64_t)p * span + o] += w * y[((int64_t)c * planes + p) * chunk + i];
    }
    weights[o] = wsum;
}

// stems[p][i] = sums[p][border + i] / weights[border + i]; optional residual for one stem.
__global__ void finish_kernel(const float* __restrict__ sums, const float* __restrict__ weights,
                              int planes, int64_t length, int64_t border, int64_t samples,
                              const float* __restrict__ input, float* __restrict__ stems,
                              float* __restrict__ residual, int* __restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= planes * samples) return;
    const int64_t p = i / samples, n = i % samples;
    const float w = weights[border + n];
    if (!(w > 0.f)) atomicOr(flag, 4);
    const float v = sums[p * length + border + n] / w;
    if (!isfinite(v)) atomicOr(flag, 1);
    stems[i] = v;
    if (residual && p < 2) residual[i] = input[i] - v;
}

// sums[p][offset + j] += piece[p][j], weights[offset + j] += piece[planes][j] (a received halo:
// rows of `count` columns, the weights last).
__global__ void span_add_kernel(float* __restrict__ sums, float* __restrict__ weights, int planes, int64_t span,
                                int64_t offset, const float* __restrict__ piece, int64_t count) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= (int64_t)(planes + 1) * count) return;
    const int p = (int)(i / count);
    const int64_t j = i % count;
    if (p < planes) sums[p * span + offset + j] += piece[i];
    else weights[offset + j] += piece[i];
}

// out[p][n] = sums[p][offset + n] / weights[offset + n] for n < count (out row stride ld).
__global__ void span_finish_kernel(const float* __restrict__ sums, const float* __restrict__ weights, int planes,
                                   int64_t span, int64_t offset, int64_t count, float* __restrict__ out,
                                   int64_t ld, int* __restrict__ flag) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= planes * count) return;
    const int64_t p = i / count, n = i % count;
    const float w = weights[offset + n];
    if (!(w > 0.f)) atomicOr(flag, 4);
    const float v = sums[p * span + offset + n] / w;
    if (!isfinite(v)) atomicOr(flag, 1);
    out[p * ld + n] = v;
}

}  // namespace

int dsp_prepare(cudaStream_t s) {
    int dev = 0;
    ANCHA_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(ANCHA_E_INVALID, "device index out of range");
    std::call_once(g_table_once[dev], [&] {
        dsp_tables_kernel<<<(NFFT + 255) / 256, 256, 0, s>>>();
        g_table_status[dev] = check_launch("dsp_tables");
        if (g_table_status[dev] == ANCHA_OK) {
            cudaError_t e = cudaStreamSynchronize(s);
            if (e != cudaSuccess) g_table_status[dev] = cuda_fail(e, "dsp tables");
        }
    });
    return g_table_status[dev];
}

int stft_forward(const float* audio, int chunks, int samples, int hop, float* packed,
                 cudaStream_t s) {
    if (hop <= 0 || hop > NH || samples <= NH)
        return fail(ANCHA_E_INVALID, "stft: require hop in 1..=1024 and samples > 1024");
    if (chunks == 0) return ANCHA_OK;
    ANCHA_TRY(dsp_prepare(s));
    const int frames = samples / hop + 1;
    stft_kernel<<<dim3(frames, chunks), 256, 0, s>>>(audio, samples, hop, frames, packed);
    return check_launch("stft");
}

int istft_masked(const float* packed, const float* masks, int chunks, int stems, int samples,
                 int hop, int zero_dc, float* scratch, float* out, int* flag, cudaStream_t s) {
    if (hop <= 0 || hop > NH || samples <= NH)
        return fail(ANCHA_E_INVALID, "istft: require hop in 1..=1024 and samples > 1024");
    if (chunks == 0 || stems == 0) return ANCHA_OK;
    ANCHA_TRY(dsp_prepare(s));
    const int frames = samples / hop + 1;
    istft_frames_kernel<<<dim3(frames, stems, chunks), 256, 0, s>>>(packed, masks, stems, frames,
                                                                   zero_dc, scratch);
    ANCHA_TRY(check_launch("istft_frames"));
    const int64_t planes = (int64_t)chunks * stems * 2;
    istft_overlap_kernel<<<(unsigned)ceil_div(planes * samples, 256), 256, 0, s>>>(
        scratch, planes, frames, hop, samples, out, flag);
    return check_launch("istft_overlap");
}

int gather_chunks(const float* planes, int64_t samples, int64_t pcm_lo, int64_t pcm_len, const ChunkStarts& starts,
                  int chunks, int chunk, int64_t border, int64_t length, float* out, cudaStream_t s) {
    const int64_t n = (int64_t)chunks * 2 * chunk;
    if (n == 0) return ANCHA_OK;
    gather_chunks_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(planes, samples, pcm_lo, pcm_len, starts,
                                                                    chunks, chunk, border, length, out);
    return check_launch("gather_chunks");
}

int span_add(float* sums, float* weights, int planes, int64_t span, int64_t offset, const float* piece,
             int64_t count, cudaStream_t s) {
    if (count <= 0) return ANCHA_OK;
    if (offset < 0 || offset + count > span) return fail(ANCHA_E_INVALID, "span_add: piece outside the span");
    const int64_t n = (int64_t)(planes + 1) * count;
    span_add_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(sums, weights, planes, span, offset, piece, count);
    return check_launch("span_add");
}

int span_finish(const float* sums, const float* weights, int planes, int64_t span, int64_t offset, int64_t count,
                float* out, int64_t ld, int* flag, cudaStream_t s) {
    if (count <= 0) return ANCHA_OK;
    if (offset < 0 || offset + count > span || ld < count)
        return fail(ANCHA_E_INVALID, "span_finish: range outside the span");
    const int64_t n = planes * count;
    span_finish_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(sums, weights, planes, span, offset, count, out,
                                                                  ld, flag);
    return check_launch("span_finish");
}

int ola_add(const float* y, int chunks, int planes, int chunk, const ChunkStarts& starts,
            int64_t length, int64_t base, int64_t span, float* sums, float* weights,
            cudaStream_t s) {
    if (chunks == 0) return ANCHA_OK;
    const int64_t lo = starts.v[0];
    const int64_t hi = std::min<int64_t>(starts.v[chunks - 1] + chunk, length);
    if (hi <= lo) return ANCHA_OK;
    if (lo < base || hi > base + span) return fail(ANCHA_E_INVALID, "ola: chunks outside the span");
    ola_kernel<<<(unsigned)ceil_div(hi - lo, 256), 256, 0, s>>>(y, chunks, planes, chunk, starts,
                                                               length, base, span, lo, hi, sums,
                                                               weights);
    return check_launch("ola");
}

int ola_finish(const float* sums, const float* weights, int planes, int64_t length,
               int64_t border, int64_t samples, const float* input, float* stems,
               float* residual, int* flag, cudaStream_t s) {
    const int64_t n = planes * samples;
    if (n == 0) return ANCHA_OK;
    finish_kernel<<<(unsigned)ceil_div(n, 256), 256, 0, s>>>(sums, weights, planes, length, border,
                                                            samples, input, stems, residual, flag);
    return check_launch("ola_finish");
}

// ---- Masked iSTFT with library-owned scratch (ancha_istft_masked_static) -------------------
//
// The frame scratch lives in a fixed device array of this module instead of caller memory, so
// the call allocates nothing. Its contents need not start at zero: every element the overlap
// kernel reads was written by the frames kernel earlier in the same batch. The status word is
// zeroed by the call itself. The buffer is shared by every call on a device, so calls that may
// overlap in time (different streams, or different host threads without ordering) race on it.
// The array belongs to this module's device code: it is resident on every device where the
// module is loaded (any use of the DSP kernels), whether or not the static entry point is called.
namespace {

__device__ __align__(256) float g_static_scratch[kStaticIstftScratchFloats];
__device__ __align__(256) int g_static_status;

struct StaticScratch {
    float* frames = nullptr;
    int* status = nullptr;
    int rc = ANCHA_OK;
};
std::once_flag g_static_once[64];
StaticScratch g_static[64];

// Resolves the device addresses of the static scratch for the current device, once per device.
int static_scratch(StaticScratch** out) {
    int dev = 0;
    ANCHA_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(ANCHA_E_INVALID, "device index out of range");
    std::call_once(g_static_once[dev], [dev] {
        StaticScratch& st = g_static[dev];
        cudaError_t e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.frames), g_static_scratch);
        if (e == cudaSuccess)
            e = cudaGetSymbolAddress(reinterpret_cast<void**>(&st.status), g_static_status);
        st.rc = e == cudaSuccess ? ANCHA_OK : cuda_fail(e, "istft_static: scratch symbol lookup");
    });
    if (g_static[dev].rc != ANCHA_OK)
        return fail(g_static[dev].rc, "istft_static: scratch set-up failed on this device");
    *out = &g_static[dev];
    return ANCHA_OK;
}

}  // namespace

int istft_masked_static(const float* packed, const float* masks, int chunks, int stems,
                        int samples, int hop, int zero_dc, float* out, int* status,
                        cudaStream_t s) {
    if (hop <= 0 || hop > NH || samples <= NH)
        return fail(ANCHA_E_INVALID, "istft_static: require hop in 1..=1024 and samples > 1024");
    StaticScratch* st = nullptr;
    ANCHA_TRY(static_scratch(&st));
    ANCHA_TRY(dsp_prepare(s));
    const int frames = samples / hop + 1;
    // One (chunk, stem) pair needs both channels' windowed frames.
    const int64_t per_pair = 2LL * frames * NFFT;
    if (per_pair > kStaticIstftScratchFloats)
        return fail(ANCHA_E_INVALID,
                    "istft_static: one chunk-stem needs " + std::to_string(per_pair) +
                        " scratch floats (frames = " + std::to_string(frames) + ") but the static "
                        "scratch holds " + std::to_string(kStaticIstftScratchFloats) +
                        " (at most " + std::to_string(kStaticIstftScratchFloats / (2 * NFFT)) +
                        " frames); use ancha_istft_masked with caller scratch");
    ANCHA_CUDA(cudaMemsetAsync(st->status, 0, sizeof(int), s));
    if (chunks > 0 && stems > 0) {
        const int per_batch = (int)std::min<int64_t>(stems, kStaticIstftScratchFloats / per_pair);
        const int64_t spec = (int64_t)frames * BINS * 4;       // packed floats per chunk
        const int64_t mask = (int64_t)2 * BINS * 2 * frames;  // mask floats per (chunk, stem)
        // Batches run in stream order on the same scratch; within a batch the frames kernel
        // fills it and the overlap kernel consumes it.
        for (int c = 0; c < chunks; ++c)
            for (int s0 = 0; s0 < stems; s0 += per_batch) {
                const int n = std::min(per_batch, stems - s0);
                const int64_t q = (int64_t)c * stems + s0;
                ANCHA_TRY(istft_masked(packed + c * spec, masks + q * mask, 1, n, samples, hop,
                                       zero_dc, st->frames, out + q * 2 * samples, st->status, s));
            }
    }
    if (status)
        ANCHA_CUDA(cudaMemcpyAsync(status, st->status, sizeof(int), cudaMemcpyDeviceToDevice, s));
    return ANCHA_OK;
}

}  // namespace ancha
