// MDX23C (TFC-TDF v3) network on the device: package loading and the forward pass of
// crates/ancha-models/src/mdx23c.rs behind ancha_mdx23c_* in the C ABI.
#pragma once
#include <memory>
#include <string>
#include <vector>

#include "hostio.hpp"
#include "mdx23c.cuh"
#include "model.hpp"

namespace ancha {

// crates/ancha-models/src/mdx23c.rs::Config (mdx23c.rs:37-52), checked like Config::validate
// (mdx23c.rs:76-122).
struct Mdx23cConfig {
    int sample_rate = 0, n_fft = 0, hop = 0, bins = 0, frames = 0, overlap = 0, subbands = 0,
        channels = 0, growth = 0, scales = 0, blocks_per_scale = 0, bottleneck_factor = 0;
    std::vector<int> scale;
    std::vector<std::string> stems;
    int64_t chunk_samples() const { return (int64_t)hop * (frames - 1); }
    void validate() const;  // throws std::runtime_error
    static Mdx23cConfig from_json(const Json& j);  // strict keys (deny_unknown_fields)
};

// OverlapPlan::new of mdx23c_runtime.rs:84-115 (UVR padding, Python modulo semantics):
// step = chunk / overlap, border = chunk − step, pad, padded length and chunk count; throws
// std::runtime_error on invalid arguments. `intersects` is OverlapPlan::intersects.
struct Mdx23cPlan {
    int64_t length = 0, chunk = 0, step = 0, border = 0, pad = 0, padded = 0, chunks = 0;
    static Mdx23cPlan make(int64_t length, int64_t chunk, int overlap);
    bool intersects(int64_t start) const { return start < border + length && start + chunk > border; }
};

struct Mdx23cManifest {
    int schema_version = 0;
    std::string model_id, weights_sha256, checkpoint_sha256, source_url, forward_revision,
        weight_license;
    Mdx23cConfig config;
    static Mdx23cManifest from_json(const Json& j);
    void validate() const;
};

class Mdx23c {
public:
    static std::unique_ptr<Mdx23c> load(const std::string& package, int device, int precision);
    // spectrum [batch][4][bins][frames] → out [batch][stems·4][bins][frames], both device f32
    // (mdx23c.rs:420-481). Checks *cancel (host, may be null) before every block.
    int forward(const float* spectrum, int batch, int frames, float* out, const volatile int* cancel,
                cudaStream_t s);
    // mdx23c_runtime::separate without file I/O (mdx23c_runtime.rs:135-248): host planes
    // [2][samples] → host stems [stems][2][samples]; chunks that lie entirely in the zero
    // borders are skipped as the reference does by default. overlap 0 = the manifest's;
    // batch = chunks per forward (1..4, 0 = 4). *seconds (may be null) = wall time.
    int separate_pcm(const float* planes, int64_t samples, int overlap, int batch, const volatile int* cancel,
                     float* stems, double* seconds);

    Mdx23cManifest manifest;
    int device = 0, precision = 0;
    size_t tensor_count = 0;

    struct Norm { DevBuf gamma, beta; };
    // w [co][kp] (elt): patch-column order (c, ky, kx) for the patch-matrix path, or
    // (ky, kx, c) when tap_major (3 × 3 layers that run as implicit GEMMs).
    struct Conv { DevBuf w; int co = 0, k = 0, kp = 0, kh = 1, kw = 1; bool tap_major = false; };
    struct Block {
        Norm n1, t0, t3, n2;
        Conv c1, c2, sc;
        DevBuf tdf1, tdf2;  // [f / bn][f], [f][f / bn] (NK), elt
        int ci = 0, co = 0, f = 0, fb = 0;
    };
    struct Down { std::vector<Block> blocks; Norm norm; Conv conv; };
    struct Up { Norm norm; Conv conv; std::vector<Block> blocks; int co = 0; };  // conv rows (co, dy, dx)

private:
    // An NCHW activation and the (Σ x, Σ x²) of its planes (null when it is never normalised).
    struct Act { float* x; int channels; double2* stats; };
    // Bias-free convolution of the channel concatenation (a, b) of NCHW [batch][·][h][wd]
    // planes: a gather (with the sources' norms and GELU) then one GEMM per batch item,
    // out[b][co][ho][wo] (+ residual of the same shape); `stats` (if set) receives the output's
    // plane statistics, a plane being `stats_div` consecutive output rows.
    int conv(const Conv& w, const PackSource& a, const PackSource& b, int batch, int h, int wd, int stride,
             int pad, bool gelu, float* out, const float* residual, double2* stats, int stats_div, cudaStream_t s);
    int gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int m, int n, int k, float* out,
             int64_t ldo, const float* residual, double2* stats, int stats_div, cudaStream_t s);
    int block(const Block& bk, const Act& a, const Act& b, int batch, int t, int f, const Act& out, cudaStream_t s);
    int ensure_workspace(int batch, int frames);
    double2* take_stats();  // the next zeroed statistics slot of this forward (null when exhausted)

    int elt_ = 0;
    DevBuf dsp_window_, dsp_twiddle_;  // MdxDsp tables for the manifest's n_fft
    Conv first_, final_first_, final_last_;
    std::vector<Down> down_;
    std::vector<Block> bottom_;
    std::vector<Up> up_;
    // Workspace for one (batch, frames) shape.
    int ws_batch_ = 0, ws_frames_ = 0;
    DevBuf first_f_, x0_, skip_sc_, h_, y1_, s_, blk_a_, blk_b_, up_raw_, up_out_, z_, ff_, in_, cur_, patch_,
        rows_, stats_;
    std::vector<DevBuf> skips_;
    std::vector<double2*> skip_stats_;
    int stat_slots_ = 0, next_slot_ = 0;
    int64_t stat_slot_len_ = 0;
};

}  // namespace ancha

struct ancha_mdx23c {
    std::unique_ptr<ancha::Mdx23c> impl;
};
