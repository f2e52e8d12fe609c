// RoFormer model on one device: strict package loading with the reference's load-time
// folding, and the forward pass over this library's kernels.
#pragma once

#include <array>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "common.cuh"
#include "gemm.cuh"
#include "hostio.hpp"

namespace ancha {

// Owned device allocation (moved, never copied).
struct DevBuf {
    void* p = nullptr;
    size_t bytes = 0;
    DevBuf() = default;
    DevBuf(const DevBuf&) = delete;
    DevBuf& operator=(const DevBuf&) = delete;
    DevBuf(DevBuf&& o) noexcept : p(o.p), bytes(o.bytes) { o.p = nullptr; o.bytes = 0; }
    DevBuf& operator=(DevBuf&& o) noexcept {
        if (this != &o) { release(); p = o.p; bytes = o.bytes; o.p = nullptr; o.bytes = 0; }
        return *this;
    }
    ~DevBuf() { release(); }
    void release();
    void alloc(size_t n);  // throws std::runtime_error on failure
    template <typename T> T* as() const { return reinterpret_cast<T*>(p); }
};

// crates/ancha-models/src/config.rs::ModelConfig.
struct ModelConfig {
    std::string family;
    int dim = 0, depth = 0, heads = 0, head_dim = 0, ff_mult = 0, mask_depth = 0,
        mask_expansion = 0, sample_rate = 0, n_fft = 0, hop = 0, overlap = 0;
    int64_t chunk_samples = 0;
    bool zero_dc = false;
    std::vector<std::string> stems;
    std::vector<std::vector<int>> bands;
    bool mel() const { return family == "mel-band-roformer"; }
    void validate() const;  // throws std::runtime_error (config.rs:36-121)
    static ModelConfig from_json(const Json& j);
    Json to_json() const;
};

struct Manifest {
    int schema_version = 0;
    std::string model_id, weights_sha256, checkpoint_sha256, source_url, forward_revision,
        weight_license;
    ModelConfig config;
    static Manifest from_json(const Json& j);  // strict keys (deny_unknown_fields)
    void validate() const;
};

struct TransformerWeights {
    DevBuf wqkvg, bqkvg;  // [3·inner + heads, dim] (norm folded) + bias (0 for q/k/v)
    DevBuf wout;          // [dim, inner]
    DevBuf w1, b1;        // [hidden, dim] (norm folded) + bias
    DevBuf w2, b2;        // [dim, hidden] + bias
    DevBuf out_scale;     // f32 [dim], Mel SourceNorm sqrt(dim)·gamma
    int rope_set = 0;     // index into Model::rope_freqs
};

struct MaskWeights {
    std::vector<DevBuf> w, b;  // hidden layers: [bands, out, in], [bands, out]
    DevBuf glu_w, glu_b;       // [bands, 2·max_width, in] rows interleaved (value, gate)
};

struct Workspace {
    int chunks = 0, frames = 0;
    DevBuf x, xn, qkvg, att, hidden, h2, z, glu;
    DevBuf z16;  // f16 mode: the band-split input, zero-padded rows of split_kp features
    // Row-norm fusion (16-bit modes): per-row, per-32-column sums of squares [rows][dim / 32]
    // of x after the attention residual (ss_x), of the block output y (ss_y) and of y ⊙ the
    // SourceNorm scale (ss_yg).
    DevBuf ss_x, ss_y, ss_yg;
    DevBuf split_groups, mask_groups, glu_groups;
    DevBuf a3;  // fp32 mode: the three bf16 planes of a GEMM's A operand [3][rows][k]
    std::vector<DevBuf> rope;        // per rope set: [time table, band table], [4, tokens, hd]
    std::vector<DevBuf> rope_pairs;  // the same tables pair-major: [2, hd / 2, tokens] × float2
};

// Device buffers of the chunk pipeline (gather → STFT → model → iSTFT → overlap-add),
// allocated on first use and reused while the batch and chunk length fit.
struct PipelineBuffers {
    int batch = 0;
    int64_t chunk = 0;
    DevBuf audio, packed, masks, scratch, y, flag, acc;
    DevBuf pcm, span;  // host-PCM separations: the uploaded track samples and the span accumulators
    DevBuf halo;       // multi-GPU separations: overlap-add columns received from other GPUs
    DevBuf stems;      // single-device host-PCM separations: the finished stems before the copy
};

class Model {
public:
    static std::unique_ptr<Model> load(const std::string& package, int device, int precision);
    ~Model();
    // With check = false the non-finite status is left on the device (read_flag) and the
    // call does not synchronise.
    int forward(const float* spectrum, int chunks, int frames, float* masks,
                const volatile int* cancel, cudaStream_t stream, bool check = true);
    int reset_flag(cudaStream_t s);
    int read_flag(cudaStream_t s, int* flag);  // synchronises `s`

    PipelineBuffers pipe;

    Manifest manifest;
    int device = 0, precision = 0;
    size_t tensor_count = 0;
    int bands = 0, bins = 0, total_width = 0, max_width = 0, max_cover = 0;
    int ldq = 0;  // row stride of the packed q|k|v|gate projection
    std::string device_name;

    // Kernel choices actually used (run.json attention_kernel / gemm_kernel).
    bool tc_gemm() const;
    bool tc_attention() const;

private:
    Model() = default;
    int ensure_workspace(int chunks, int frames, cudaStream_t s);
    int linear(const void* x, int64_t ldx, const DevBuf& w, const float* bias,
               const float* residual, int64_t ldr, void* out, int64_t ldo, int out_type,
               int64_t m, int n, int k, int act, const float* rope, const float* rope_pairs,
               int rope_tokens, int rope_div, cudaStream_t s);
    int transformer(const TransformerWeights& t, bool time_axis, cudaStream_t s);

    // Operands of the row-norm fusion for one linear() call (null = not used); see GemmEpilogue.
    struct NormFusion {
        const float* row_ss = nullptr;
        const float* res_ss = nullptr;
        const float* res_col = nullptr;
        void* out16 = nullptr;
        const float* out16_col = nullptr;
        float* ss_out = nullptr;
        float* ss16_out = nullptr;
    };
    int linear_fused(const void* x, int64_t ldx, const DevBuf& w, const float* bias, const float* residual,
                     int64_t ldr, void* out, int64_t ldo, int out_type, int64_t m, int n, int k, int act,
                     const float* rope, const float* rope_pairs, int rope_tokens, int rope_div,
                     const NormFusion& nf, cudaStream_t s);
    // Whether the unit norms run fused into the GEMMs (16-bit modes, dim a multiple of 32),
    // and the state the fusion carries from one transformer block to the next: ws_.xn holds
    // the unnormalised next block input (row norms in block_ss_), and x still needs the
    // deferred SourceNorm (x · 1/‖x‖ · pending_scale_) before it is read as a residual.
    bool fuse_norms_ = false;
    const float* block_ss_ = nullptr;
    const float* pending_scale_ = nullptr;

    std::vector<int> width_, offset_;
    DevBuf zcols_, zoffsets_, wsplit_, bsplit_;
    // f16 mode: band-split weights [bands][dim][split_kp_] f16, K zero-padded to a multiple of 64,
    // for one grouped tensor-core launch over every (chunk, band); 0 = the fp32 FFMA split.
    DevBuf wsplit16_;
    int split_kp_ = 0;
    std::vector<int64_t> wsplit_off_;
    std::vector<std::array<TransformerWeights, 2>> layers_;
    DevBuf final_scale_;
    std::vector<MaskWeights> masks_;
    DevBuf cover_count_, cover_entries_;
    DevBuf glu_n_;  // [bands] GLU weight rows used per band (2·width)
    std::vector<std::vector<float>> rope_freqs_;
    Workspace ws_;
    DevBuf flag_;  // non-finite model output (sticky until reset_flag)
    int elt_ = ELT_F32;  // operand type of the GEMMs and attention (ELT_*)
    // fp32 mode on the tensor cores: the transformer weights' three-plane bf16 splits
    // ([3][n][k], keyed by the f32 weight's device pointer) for the split3 GEMM.
    bool split_ = false;
    std::map<const void*, DevBuf> split_w_;
    int cur_chunks_ = 0;  // chunks of the forward in progress
};

}  // namespace ancha

// The opaque handle of the C ABI.
struct ancha_model {
    std::unique_ptr<ancha::Model> impl;
};
