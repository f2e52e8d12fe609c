// Spectral DSP kernels (see dsp.cu).
#pragma once
#include "common.cuh"

namespace ancha {

constexpr int kMaxChunksPerCall = 128;

// Chunk start samples passed by value to the gather / overlap-add kernels.
struct ChunkStarts {
    int64_t v[kMaxChunksPerCall];
};

int dsp_prepare(cudaStream_t s);
int stft_forward(const float* audio, int chunks, int samples, int hop, float* packed,
                 cudaStream_t s);
int istft_masked(const float* packed, const float* masks, int chunks, int stems, int samples,
                 int hop, int zero_dc, float* scratch, float* out, int* flag, cudaStream_t s);
// Reflect-padded chunks of a track whose samples [pcm_lo, pcm_lo + pcm_len) are held in
// planes[2][pcm_len] (pcm_lo = 0, pcm_len = samples for a whole track).
int gather_chunks(const float* planes, int64_t samples, int64_t pcm_lo, int64_t pcm_len, const ChunkStarts& starts,
                  int chunks, int chunk, int64_t border, int64_t length, float* out, cudaStream_t s);
// Add a received overlap-add piece [planes + 1][count] (sums rows, then weights) into the span
// buffers sums[planes][span] / weights[span] at column `offset`.
int span_add(float* sums, float* weights, int planes, int64_t span, int64_t offset, const float* piece,
             int64_t count, cudaStream_t s);
// out[p][n] = sums[p][offset + n] / weights[offset + n], n < count, out row stride `ld`; flag
// bit 4: a zero weight, bit 1: a non-finite result.
int span_finish(const float* sums, const float* weights, int planes, int64_t span, int64_t offset, int64_t count,
                float* out, int64_t ld, int* flag, cudaStream_t s);
int ola_add(const float* y, int chunks, int planes, int chunk, const ChunkStarts& starts,
            int64_t length, int64_t base, int64_t span, float* sums, float* weights,
            cudaStream_t s);
// Static scratch of ancha_istft_masked_static: 6 Mi floats (24 MiB) per device, enough for one
// chunk-stem of up to 1536 frames.
constexpr int64_t kStaticIstftScratchFloats = 6LL << 20;
int istft_masked_static(const float* packed, const float* masks, int chunks, int stems,
                        int samples, int hop, int zero_dc, float* out, int* status,
                        cudaStream_t s);
int ola_finish(const float* sums, const float* weights, int planes, int64_t length,
               int64_t border, int64_t samples, const float* input, float* stems,
               float* residual, int* flag, cudaStream_t s);

}  // namespace ancha
