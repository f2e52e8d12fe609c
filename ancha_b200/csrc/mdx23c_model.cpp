// MDX23C (TFC-TDF v3) on the device (mdx23c_model.hpp).
//
// Layout: NCHW f32 planes, [batch][channels][time][frequency] inside the network (the
// reference's layout after swap_dims(2, 3), mdx23c.rs:437), so the TDF Linear over the
// frequency axis is one plain GEMM over rows (batch, channel, time), and its residual x + y
// (mdx23c.rs:271) is that GEMM's epilogue. Every convolution is a patch gather
// (mdx_pack: instance norm → GELU → zero padding → K-major patch rows, over a concatenation
// of two sources) and one GEMM per batch item, out[co][pos] = W[co][k]·P[pos][k]ᵀ, so the
// output lands in NCHW directly; the second convolution's `+ skip` (mdx23c.rs:272-273) is its
// epilogue. GEMMs run on the tcgen05 kernel with f16 / bf16 operands (the FFMA kernel when a
// shape breaks its 16-byte rules, and for f32); accumulation and activations stay f32.
#include "mdx23c_model.hpp"

#include <algorithm>
#include <chrono>
#include <climits>
#include <cstring>
#include <set>
#include <stdexcept>
#include <thread>

#include "gemm.cuh"

namespace ancha {

namespace {

[[noreturn]] void bad(const std::string& m) { throw std::runtime_error(m); }

void ensure(bool ok, const char* msg) {
    if (!ok) bad(msg);
}

void check_keys(const Json& j, const std::set<std::string>& keys, const char* what) {
    if (j.kind != Json::Object) bad(std::string(what) + " must be an object");
    std::set<std::string> seen;
    for (const auto& kv : j.obj) {
        if (!keys.count(kv.first)) bad(std::string("unknown field `") + kv.first + "` in " + what);
        seen.insert(kv.first);
    }
    for (const auto& k : keys)
        if (!seen.count(k)) bad(std::string("missing field `") + k + "` in " + what);
}

bool is_hex64(const std::string& s) {
    return s.size() == 64 && std::all_of(s.begin(), s.end(), [](char c) { return isxdigit((unsigned char)c) != 0; });
}

template <typename T>
void upload(DevBuf& d, const std::vector<T>& v) {
    d.alloc(v.size() * sizeof(T));
    cudaError_t e = cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) bad(std::string("cudaMemcpy: ") + cudaGetErrorString(e));
}

void upload_elt(DevBuf& d, const std::vector<float>& v, int elt) {
    if (elt == ELT_F32) return upload(d, v);
    if (elt == ELT_BF16) {
        std::vector<__nv_bfloat16> h(v.size());
        for (size_t i = 0; i < v.size(); ++i) h[i] = __float2bfloat16_rn(v[i]);
        return upload(d, h);
    }
    std::vector<__half> h(v.size());
    for (size_t i = 0; i < v.size(); ++i) h[i] = __float2half_rn(v[i]);
    upload(d, h);
}

int64_t round8(int64_t k) { return (k + 7) / 8 * 8; }

constexpr float kNormEps = 1e-5f;  // Preact's InstanceNorm epsilon (mdx23c.rs:204)

}  // namespace

Mdx23cPlan Mdx23cPlan::make(int64_t length, int64_t chunk, int overlap) {
    ensure(length > 0 && chunk > 0 && overlap >= 1 && overlap <= 16 && overlap <= chunk,
           "invalid MDX23C overlap plan");
    Mdx23cPlan p;
    p.length = length;
    p.chunk = chunk;
    p.step = chunk / overlap;
    const int64_t left = length % p.step, right = chunk % p.step;
    const int64_t remainder = left >= right ? left - right : p.step - (right - left);
    p.pad = p.step - remainder;
    p.border = chunk - p.step;
    if (length > INT64_MAX - p.pad - 2 * p.border) bad("MDX23C padded length overflow");
    p.padded = length + p.pad + 2 * p.border;
    ensure(p.padded >= chunk, "insufficient MDX23C padding");
    p.chunks = (p.padded - chunk) / p.step + 1;
    return p;
}

void Mdx23cConfig::validate() const {
    // mdx23c.rs:76-122.
    ensure(sample_rate == 44100 && n_fft >= 32 && n_fft <= 8192 && n_fft % 2 == 0 && hop > 0 && hop <= n_fft / 2,
           "MDX23C requires stereo 44100 Hz and a valid centered STFT");
    ensure(scales >= 1 && scales <= 6 && scale == std::vector<int>{2, 2},
           "MDX23C supports 1..=6 scales with 2x2 down/up sampling");
    const int factor = 1 << scales;
    ensure(subbands >= 1 && subbands <= 16 && bins > 0 && bins <= n_fft / 2 + 1 && bins % (subbands * factor) == 0 &&
               frames >= factor && frames <= 2048 && frames % factor == 0,
           "MDX23C frequency/time dimensions must survive all encoder scales");
    ensure(channels >= 1 && channels <= 1024 && growth >= 1 && growth <= 1024 && channels + scales * growth <= 2048 &&
               blocks_per_scale >= 1 && blocks_per_scale <= 4 && bottleneck_factor >= 1 && bottleneck_factor <= 16,
           "invalid MDX23C network size");
    const int bottom = bins / subbands / factor;
    ensure(bottom >= bottleneck_factor && (frames / factor) * bottom > 1,
           "MDX23C bottleneck is too small for Linear or InstanceNorm");
    ensure(chunk_samples() > n_fft / 2 && chunk_samples() <= 44100 * 60 && overlap >= 1 && overlap <= 16,
           "invalid MDX23C context");
    ensure(stems == std::vector<std::string>{"vocals", "instrumental"},
           "MDX23C schema 1 requires two native heads in vocals/instrumental order");
}

Mdx23cConfig Mdx23cConfig::from_json(const Json& j) {
    check_keys(j, {"family", "sample_rate", "n_fft", "hop", "bins", "frames", "overlap", "subbands", "channels",
                   "growth", "scales", "blocks_per_scale", "bottleneck_factor", "scale", "stems"},
               "MDX23C config");
    ensure(j.at("family").as_string() == "mdx23c", "not an MDX23C package");
    Mdx23cConfig c;
    auto i = [&](const char* k) { return j.at(k).as_int32(); };
    c.sample_rate = i("sample_rate"); c.n_fft = i("n_fft"); c.hop = i("hop"); c.bins = i("bins");
    c.frames = i("frames"); c.overlap = i("overlap"); c.subbands = i("subbands"); c.channels = i("channels");
    c.growth = i("growth"); c.scales = i("scales"); c.blocks_per_scale = i("blocks_per_scale");
    c.bottleneck_factor = i("bottleneck_factor");
    for (const Json& v : j.at("scale").arr) c.scale.push_back(v.as_int32());
    for (const Json& v : j.at("stems").arr) c.stems.push_back(v.as_string());
    return c;
}

Mdx23cManifest Mdx23cManifest::from_json(const Json& j) {
    check_keys(j, {"schema_version", "model_id", "weights_sha256", "checkpoint_sha256", "source_url",
                   "forward_revision", "weight_license", "config"},
               "manifest");
    Mdx23cManifest m;
    m.schema_version = j.at("schema_version").as_int32();
    m.model_id = j.at("model_id").as_string();
    m.weights_sha256 = j.at("weights_sha256").as_string();
    m.checkpoint_sha256 = j.at("checkpoint_sha256").as_string();
    m.source_url = j.at("source_url").as_string();
    m.forward_revision = j.at("forward_revision").as_string();
    m.weight_license = j.at("weight_license").as_string();
    m.config = Mdx23cConfig::from_json(j.at("config"));
    return m;
}

void Mdx23cManifest::validate() const {
    // config.rs:211-221 (validate_metadata), then the network config.
    ensure(schema_version == 1, "unsupported model package schema");
    ensure(!model_id.empty(), "model ID is empty");
    ensure(is_hex64(weights_sha256) && is_hex64(checkpoint_sha256), "invalid SHA256");
    config.validate();
}

std::unique_ptr<Mdx23c> Mdx23c::load(const std::string& package, int device, int precision) {
    if (precision != ANCHA_PRECISION_F32 && precision != ANCHA_PRECISION_BF16 && precision != ANCHA_PRECISION_F16)
        bad("unknown precision");
    std::unique_ptr<Mdx23c> m(new Mdx23c());
    // The manifest is checked before any device work, so a bad package fails the same way
    // with or without a GPU.
    m->manifest = Mdx23cManifest::from_json(Json::parse(read_file(package + "/manifest.json")));
    m->manifest.validate();
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) bad(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    m->device = device;
    m->precision = precision;
    m->elt_ = precision == ANCHA_PRECISION_BF16 ? ELT_BF16 : precision == ANCHA_PRECISION_F16 ? ELT_F16 : ELT_F32;
    const std::string bytes = read_file(package + "/model.safetensors");
    std::string digest;  // SHA-256 on another thread while the weights are converted (weights.rs:29-40)
    std::thread hasher([&] { digest = sha256_hex(reinterpret_cast<const uint8_t*>(bytes.data()), bytes.size()); });
    try {
        SafeTensors w(bytes);
        const Mdx23cConfig& c = m->manifest.config;
        const int elt = m->elt_;
        auto norm = [&](Norm& n, const std::string& p, int ch) {
            upload(n.gamma, w.take(p + ".weight", {ch}));
            upload(n.beta, w.take(p + ".bias", {ch}));
        };
        // [co][ci][kh][kw] → [co][kp]: PyTorch's flattening is the patch column order
        // k = (ci·kh + ky)·kw + kx of mdx_pack; columns k..kp−1 are zero. A 3 × 3 layer over
        // planes `width` wide that the implicit-GEMM kernel can run (16-bit operands, channels
        // in 64s, width a multiple or divisor of its 256-position tile) is stored tap-major.
        auto conv = [&](Conv& cv, const std::string& name, int co, int ci, int k, int width = 0) {
            const std::vector<float> src = w.take(name, {co, ci, k, k});
            cv.co = co; cv.kh = cv.kw = k; cv.k = ci * k * k; cv.kp = (int)round8(cv.k);
            cv.tap_major = k == 3 && elt != ELT_F32 && ci % 64 == 0 && width > 0 &&
                           (width % 256 == 0 || 256 % width == 0);
            std::vector<float> dst((size_t)co * cv.kp, 0.f);
            for (int o = 0; o < co; ++o) {
                if (cv.tap_major) {
                    for (int c = 0; c < ci; ++c)
                        for (int t = 0; t < k * k; ++t)
                            dst[(size_t)o * cv.kp + (size_t)t * ci + c] = src[((size_t)o * ci + c) * k * k + t];
                } else {
                    std::copy_n(&src[(size_t)o * cv.k], cv.k, &dst[(size_t)o * cv.kp]);
                }
            }
            upload_elt(cv.w, dst, elt);
        };
        auto blocks = [&](std::vector<Block>& out, const std::string& p, int ci, int co, int f) {
            const int bn = c.bottleneck_factor;
            for (int i = 0; i < c.blocks_per_scale; ++i) {
                // Block::load (mdx23c.rs:243-263).
                const std::string q = p + ".blocks." + std::to_string(i);
                Block b;
                b.ci = i == 0 ? ci : co; b.co = co; b.f = f; b.fb = f / bn;
                norm(b.n1, q + ".tfc1.0", b.ci);
                conv(b.c1, q + ".tfc1.2.weight", co, b.ci, 3, f);
                norm(b.t0, q + ".tdf.0", co);
                upload_elt(b.tdf1, w.take(q + ".tdf.2.weight", {b.fb, f}), elt);
                norm(b.t3, q + ".tdf.3", co);
                upload_elt(b.tdf2, w.take(q + ".tdf.5.weight", {f, b.fb}), elt);
                norm(b.n2, q + ".tfc2.0", co);
                conv(b.c2, q + ".tfc2.2.weight", co, co, 3, f);
                conv(b.sc, q + ".shortcut.weight", co, b.ci, 1);
                out.push_back(std::move(b));
            }
        };
        // Mdx23c::build (mdx23c.rs:379-418).
        const int input = 4 * c.subbands;
        conv(m->first_, "first_conv.weight", c.channels, input, 1);
        int ch = c.channels, f = c.bins / c.subbands;
        for (int i = 0; i < c.scales; ++i) {
            const std::string p = "encoder_blocks." + std::to_string(i);
            Down d;
            blocks(d.blocks, p + ".tfc_tdf", ch, ch, f);
            norm(d.norm, p + ".downscale.conv.0", ch);
            conv(d.conv, p + ".downscale.conv.2.weight", ch + c.growth, ch, 2);
            m->down_.push_back(std::move(d));
            f /= 2;
            ch += c.growth;
        }
        blocks(m->bottom_, "bottleneck_block", ch, ch, f);
        for (int i = 0; i < c.scales; ++i) {
            const std::string p = "decoder_blocks." + std::to_string(i);
            const int co = ch - c.growth;
            f *= 2;
            Up u;
            u.co = co;
            norm(u.norm, p + ".upscale.conv.0", ch);
            // ConvTranspose2d weight [ci][co][2][2] → GEMM rows (co, dy, dx) over K = ci.
            const std::vector<float> src = w.take(p + ".upscale.conv.2.weight", {ch, co, 2, 2});
            u.conv.co = 4 * co; u.conv.kh = u.conv.kw = 1; u.conv.k = ch; u.conv.kp = (int)round8(ch);
            std::vector<float> dst((size_t)4 * co * u.conv.kp, 0.f);
            for (int ci = 0; ci < ch; ++ci)
                for (int r = 0; r < 4 * co; ++r) dst[(size_t)r * u.conv.kp + ci] = src[(size_t)ci * 4 * co + r];
            upload_elt(u.conv.w, dst, elt);
            blocks(u.blocks, p + ".tfc_tdf", co * 2, co, f);
            m->up_.push_back(std::move(u));
            ch = co;
        }
        conv(m->final_first_, "final_conv.0.weight", ch, ch + input, 1);
        conv(m->final_last_, "final_conv.2.weight", (int)c.stems.size() * input, ch, 1);
        m->tensor_count = w.finish();
        // STFT tables for separate_pcm (power-of-two n_fft only; the network itself takes any
        // valid config).
        if ((c.n_fft & (c.n_fft - 1)) == 0) {
            m->dsp_window_.alloc((size_t)c.n_fft * sizeof(float));
            m->dsp_twiddle_.alloc((size_t)4097 * sizeof(float2));
            if (mdx_dsp_tables(c.n_fft, m->dsp_window_.as<float>(), m->dsp_twiddle_.as<float2>(), 0) != ANCHA_OK)
                bad(std::string("MDX23C DSP tables: ") + ancha_last_error());
            const cudaError_t te = cudaDeviceSynchronize();
            if (te != cudaSuccess) bad(std::string("MDX23C DSP tables: ") + cudaGetErrorString(te));
        }
    } catch (...) {
        hasher.join();
        throw;
    }
    hasher.join();
    if (digest != m->manifest.weights_sha256) bad("model checksum mismatch");
    return m;
}

int Mdx23c::ensure_workspace(int batch, int frames) {
    // Buffers sized for a larger batch serve a smaller one (the last call of a separation).
    if (frames == ws_frames_ && batch <= ws_batch_) return ANCHA_OK;
    const Mdx23cConfig& c = manifest.config;
    const int64_t b = batch, f0 = c.bins / c.subbands, t0 = frames;
    const size_t es = elt_size(elt_);
    int64_t act = 0, patch = 0, rows = 0;
    auto pos = [&](int l) { return (t0 >> l) * (f0 >> l); };
    for (int l = 0; l <= c.scales; ++l) {
        const int64_t cl = c.channels + (int64_t)l * c.growth;
        act = std::max(act, b * cl * pos(l));
        rows = std::max(rows, b * cl * pos(l));
        const int64_t cin = l < c.scales ? 2 * cl : cl;  // decoder blocks read cat(up, skip)
        patch = std::max(patch, b * pos(l) * round8(9 * std::max(cin, cl)));
        if (l < c.scales) {
            patch = std::max(patch, b * pos(l + 1) * round8(4 * cl));        // down
            patch = std::max(patch, b * pos(l + 1) * round8(cl + c.growth));  // up
        }
    }
    const int64_t input = 4 * c.subbands;
    patch = std::max(patch, b * pos(0) * round8(input + c.channels));  // final_first (and first)
    const size_t fb = sizeof(float);
    for (DevBuf* d : {&first_f_, &x0_, &z_, &ff_}) d->alloc((size_t)(b * c.channels * pos(0)) * fb);
    for (DevBuf* d : {&skip_sc_, &h_, &y1_, &s_, &blk_a_, &blk_b_, &up_raw_, &up_out_}) d->alloc((size_t)act * fb);
    in_.alloc((size_t)act * fb);
    cur_.alloc((size_t)act * fb);
    patch_.alloc((size_t)patch * es);
    rows_.alloc((size_t)rows * es);
    // One statistics slot per normalised tensor of a forward: block input, h, y1, s and output
    // per block, the level inputs, the up-convolution outputs.
    const int blocks = (2 * c.scales + 1) * c.blocks_per_scale;
    stat_slots_ = 4 * blocks + 2 * c.scales + 4;
    stat_slot_len_ = b * 2048;
    stats_.alloc((size_t)stat_slots_ * stat_slot_len_ * sizeof(double2));
    skips_.clear();
    skips_.resize(c.scales);
    skip_stats_.assign(c.scales, nullptr);
    for (int l = 0; l < c.scales; ++l)
        skips_[l].alloc((size_t)(b * (c.channels + (int64_t)l * c.growth) * pos(l)) * fb);
    ws_batch_ = batch;
    ws_frames_ = frames;
    return ANCHA_OK;
}

double2* Mdx23c::take_stats() {
    if (next_slot_ >= stat_slots_) return nullptr;
    return stats_.as<double2>() + (size_t)(next_slot_++) * stat_slot_len_;
}

int Mdx23c::gemm(const void* a, int64_t lda, const void* b, int64_t ldb, int m, int n, int k, float* out,
                 int64_t ldo, const float* residual, double2* stats, int stats_div, cudaStream_t s) {
    GemmGroup g{};
    g.a = a; g.b = b; g.bias = nullptr; g.residual = residual; g.out = out;
    g.m = m; g.n = n; g.k = k;
    g.lda = lda; g.ldb = ldb; g.ldr = ldo; g.ldo = ldo;
    GemmEpilogue e{};
    e.act = ANCHA_ACT_NONE;
    e.out_type = ELT_F32;
    e.rope_tokens = 1;
    e.rope_div = 1;
    e.rope_hd = 64;
    e.stats = stats;
    e.stats_div = stats_div;
    if (elt_ != ELT_F32) {
        const int st = gemm_tc(g, elt_, e, s);
        if (st != ANCHA_E_UNSUPPORTED) return st;
    }
    e.stats = nullptr;
    ANCHA_TRY(gemm_ffma(g, nullptr, 1, m, n, elt_, elt_, 1, e, s));
    // The FFMA kernel has no statistics epilogue: planes of stats_div rows are contiguous.
    if (stats) {
        if (ldo != n || m % stats_div) return fail(ANCHA_E_INVALID, "mdx23c: statistics of a strided output");
        return mdx_plane_sums(out, m / stats_div, (int64_t)stats_div * n, stats, s);
    }
    return ANCHA_OK;
}

int Mdx23c::conv(const Conv& w, const PackSource& a, const PackSource& b, int batch, int h, int wd, int stride,
                 int pad, bool gelu, float* out, const float* residual, double2* stats, int stats_div,
                 cudaStream_t s) {
    if (a.channels + b.channels != w.k / (w.kh * w.kw)) return fail(ANCHA_E_INVALID, "mdx23c: conv channels");
    const int ho = (h + 2 * pad - w.kh) / stride + 1, wo = (wd + 2 * pad - w.kw) / stride + 1;
    const int64_t npos = (int64_t)ho * wo;
    const size_t es = elt_size(elt_);
    const int cin = a.channels + b.channels;
    // Output statistics per image: planes co / stats_div of that image.
    auto image_stats = [&](int i) { return stats ? stats + (size_t)i * (w.co / stats_div) : nullptr; };
    const bool implicit = elt_ != ELT_F32 && stride == 1 && cin % 64 == 0 && (wd % 256 == 0 || 256 % wd == 0) &&
                          ((w.kh == 1 && pad == 0) || (w.kh == 3 && pad == 1 && w.tap_major));
    if (implicit) {
        // Channels-last act(norm(x)) once, then the GEMM reads each tap's shifted window
        // through TMA (zero fill at the borders is the padding).
        if ((size_t)(batch * npos * cin) * es > patch_.bytes) return fail(ANCHA_E_INVALID, "mdx23c: patch workspace");
        ANCHA_TRY(mdx_preact_nhwc(a, b, batch, npos, gelu, kNormEps, patch_.p, elt_, s));
        GemmEpilogue e{};
        e.act = ANCHA_ACT_NONE;
        e.out_type = ELT_F32;
        e.rope_tokens = 1;
        e.rope_div = 1;
        e.rope_hd = 64;
        e.stats_div = stats_div;
        for (int i = 0; i < batch; ++i) {
            ConvGemm q{};
            q.weight = w.w.p; q.ldw = w.kp; q.co = w.co;
            q.x = patch_.p; q.batch = batch; q.h = h; q.w = wd; q.channels = cin; q.image = i;
            q.taps = w.kh * w.kw;
            q.residual = residual ? residual + (size_t)i * w.co * npos : nullptr;
            q.out = out + (size_t)i * w.co * npos;
            q.ldo = npos;
            e.stats = image_stats(i);
            ANCHA_TRY(gemm_tc_conv(q, elt_, e, s));
        }
        return ANCHA_OK;
    }
    if (w.tap_major) return fail(ANCHA_E_INVALID, "mdx23c: tap-major weights need the implicit-GEMM path");
    if ((size_t)(batch * npos * w.kp) * es > patch_.bytes) return fail(ANCHA_E_INVALID, "mdx23c: patch workspace");
    PackArgs p{};
    p.a = a; p.b = b;
    p.batch = batch; p.h = h; p.w = wd; p.ho_n = ho; p.wo_n = wo;
    p.kh = w.kh; p.kw = w.kw; p.sh = p.sw = stride; p.ph = p.pw = pad;
    p.gelu = gelu; p.eps = kNormEps; p.kp = w.kp; p.out = patch_.p; p.out_type = elt_;
    ANCHA_TRY(mdx_pack(p, s));
    for (int i = 0; i < batch; ++i) {
        const uint8_t* pb = patch_.as<uint8_t>() + (size_t)(i * npos * w.kp) * es;
        ANCHA_TRY(gemm(w.w.p, w.kp, pb, w.kp, w.co, (int)npos, w.kp, out + (size_t)i * w.co * npos, npos,
                       residual ? residual + (size_t)i * w.co * npos : nullptr, image_stats(i), stats_div, s));
    }
    return ANCHA_OK;
}

int Mdx23c::block(const Block& bk, const Act& a, const Act& b, int batch, int t, int f, const Act& out,
                  cudaStream_t s) {
    // Block::forward (mdx23c.rs:264-274).
    const int64_t pos = (int64_t)t * f;
    const int co = bk.co;
    const PackSource none{nullptr, 0, nullptr, nullptr, nullptr};
    const PackSource ar{a.x, a.channels, nullptr, nullptr, nullptr}, br{b.x, b.channels, nullptr, nullptr, nullptr};
    ANCHA_TRY(conv(bk.sc, ar, b.channels ? br : none, batch, t, f, 1, 0, false, skip_sc_.as<float>(), nullptr,
                   nullptr, 1, s));
    // x = tfc1(x): the norm over the channels of the concatenation, per source.
    const float* g1 = bk.n1.gamma.as<float>();
    const float* b1 = bk.n1.beta.as<float>();
    const PackSource an{a.x, a.channels, a.stats, g1, b1};
    const PackSource bn{b.x, b.channels, b.stats, g1 + a.channels, b1 + a.channels};
    double2* sh = take_stats();
    double2* sy = take_stats();
    double2* ss = take_stats();
    if (!sh || !sy || !ss) return fail(ANCHA_E_INVALID, "mdx23c: statistics workspace");
    float* h = h_.as<float>();
    ANCHA_TRY(conv(bk.c1, an, b.channels ? bn : none, batch, t, f, 1, 1, true, h, nullptr, sh, 1, s));
    // y = tdf2(gelu(norm(tdf1(gelu(norm(x)))))); s = x + y. The TDF rows are (batch, channel,
    // time), so a plane is `t` consecutive rows.
    const int64_t rows = (int64_t)batch * co * t;
    ANCHA_TRY(mdx_norm_act(h, (int64_t)batch * co, pos, co, sh, bk.t0.gamma.as<float>(), bk.t0.beta.as<float>(),
                           kNormEps, true, rows_.p, elt_, s));
    float* y1 = y1_.as<float>();
    ANCHA_TRY(gemm(rows_.p, f, bk.tdf1.p, f, (int)rows, bk.fb, f, y1, bk.fb, nullptr, sy, t, s));
    ANCHA_TRY(mdx_norm_act(y1, (int64_t)batch * co, (int64_t)t * bk.fb, co, sy, bk.t3.gamma.as<float>(),
                           bk.t3.beta.as<float>(), kNormEps, true, rows_.p, elt_, s));
    float* sum = s_.as<float>();
    ANCHA_TRY(gemm(rows_.p, bk.fb, bk.tdf2.p, bk.fb, (int)rows, f, bk.fb, sum, f, h, ss, t, s));
    // out = tfc2(s) + shortcut(x).
    const PackSource sn{sum, co, ss, bk.n2.gamma.as<float>(), bk.n2.beta.as<float>()};
    return conv(bk.c2, sn, none, batch, t, f, 1, 1, true, out.x, skip_sc_.as<float>(), out.stats, 1, s);
}

int Mdx23c::forward(const float* spectrum, int batch, int frames, float* out, const volatile int* cancel,
                    cudaStream_t s) {
    const Mdx23cConfig& c = manifest.config;
    const int factor = 1 << c.scales;
    if (batch <= 0 || batch > 4 || frames < factor || frames % factor)
        return fail(ANCHA_E_INVALID, "invalid MDX23C spectrum shape");
    if ((int64_t)frames * c.bins > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "MDX23C spectrum too large");
    if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
    ANCHA_CUDA(cudaSetDevice(device));
    ANCHA_TRY(ensure_workspace(batch, frames));
    ANCHA_CUDA(cudaMemsetAsync(stats_.p, 0, stats_.bytes, s));
    next_slot_ = 0;
    const int input = 4 * c.subbands, f0 = c.bins / c.subbands, ch = c.channels;
    const PackSource none{nullptr, 0, nullptr, nullptr, nullptr};
    // mix = spectrum viewed as [batch][4·subbands][bins / subbands][frames] (mdx23c.rs:435).
    const PackSource mix{spectrum, input, nullptr, nullptr, nullptr};
    float* first = first_f_.as<float>();
    ANCHA_TRY(conv(first_, mix, none, batch, f0, frames, 1, 0, false, first, nullptr, nullptr, 1, s));
    ANCHA_TRY(mdx_transpose(first, nullptr, (int64_t)batch * ch, f0, frames, x0_.as<float>(), s));
    Act x{x0_.as<float>(), ch, take_stats()};
    ANCHA_TRY(mdx_plane_sums(x.x, (int64_t)batch * ch, (int64_t)frames * f0, x.stats, s));
    const Act none_act{nullptr, 0, nullptr};
    auto run_blocks = [&](const std::vector<Block>& blocks, Act a, Act b, int t, int f, const Act& dst) -> int {
        for (size_t i = 0; i < blocks.size(); ++i) {
            if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
            Act o = i + 1 == blocks.size()
                        ? dst
                        : Act{i % 2 ? blk_b_.as<float>() : blk_a_.as<float>(), blocks[i].co, take_stats()};
            if (!o.stats) return fail(ANCHA_E_INVALID, "mdx23c: statistics workspace");
            ANCHA_TRY(block(blocks[i], a, b, batch, t, f, o, s));
            a = o;
            b = none_act;
        }
        return ANCHA_OK;
    };
    // Encoder (mdx23c.rs:440-444): blocks, keep the skip, then norm → GELU → 2 × 2 / 2 conv.
    int t = frames, f = f0, cl = ch;
    for (int l = 0; l < c.scales; ++l) {
        const Act skip{skips_[l].as<float>(), cl, take_stats()};
        skip_stats_[l] = skip.stats;
        ANCHA_TRY(run_blocks(down_[l].blocks, x, none_act, t, f, skip));
        const PackSource sn{skip.x, cl, skip.stats, down_[l].norm.gamma.as<float>(), down_[l].norm.beta.as<float>()};
        x = Act{in_.as<float>(), cl + c.growth, take_stats()};
        if (!x.stats) return fail(ANCHA_E_INVALID, "mdx23c: statistics workspace");
        ANCHA_TRY(conv(down_[l].conv, sn, none, batch, t, f, 2, 0, true, in_.as<float>(), nullptr, x.stats, 1, s));
        t /= 2; f /= 2; cl += c.growth;
    }
    Act cur{cur_.as<float>(), cl, take_stats()};
    ANCHA_TRY(run_blocks(bottom_, x, none_act, t, f, cur));
    // Decoder (Up::forward, mdx23c.rs:330-355): norm → GELU → ConvTranspose2d(2, 2) as a GEMM
    // over the input positions (rows (co, dy, dx): a plane's statistics are 4 rows) plus a
    // scatter, then blocks over cat(up, skip).
    for (int i = 0; i < c.scales; ++i) {
        const Up& u = up_[i];
        const PackSource un{cur.x, cl, cur.stats, u.norm.gamma.as<float>(), u.norm.beta.as<float>()};
        const Act up{up_out_.as<float>(), u.co, take_stats()};
        if (!up.stats) return fail(ANCHA_E_INVALID, "mdx23c: statistics workspace");
        ANCHA_TRY(conv(u.conv, un, none, batch, t, f, 1, 0, true, up_raw_.as<float>(), nullptr, up.stats, 4, s));
        ANCHA_TRY(mdx_shuffle2x2(up_raw_.as<float>(), batch, u.co, t, f, up_out_.as<float>(), u.co, 0, s));
        t *= 2; f *= 2; cl = u.co;
        const int l = c.scales - 1 - i;
        const Act sk{skips_[l].as<float>(), u.co, skip_stats_[l]};
        cur = Act{cur_.as<float>(), u.co, take_stats()};
        if (!cur.stats) return fail(ANCHA_E_INVALID, "mdx23c: statistics workspace");
        ANCHA_TRY(run_blocks(u.blocks, up, sk, t, f, cur));
    }
    if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
    // x.swap_dims(2, 3) · first, then final_conv = 1×1 → GELU → 1×1 over cat(mix, x)
    // (mdx23c.rs:475-480).
    ANCHA_TRY(mdx_transpose(cur.x, first, (int64_t)batch * ch, frames, f0, z_.as<float>(), s));
    const PackSource z{z_.as<float>(), ch, nullptr, nullptr, nullptr};
    ANCHA_TRY(conv(final_first_, mix, z, batch, f0, frames, 1, 0, false, ff_.as<float>(), nullptr, nullptr, 1, s));
    const PackSource ffs{ff_.as<float>(), ch, nullptr, nullptr, nullptr};
    return conv(final_last_, ffs, none, batch, f0, frames, 1, 0, true, out, nullptr, nullptr, 1, s);
}

int Mdx23c::separate_pcm(const float* planes, int64_t samples, int overlap, int batch, const volatile int* cancel,
                         float* stems, double* seconds) {
    const auto t_start = std::chrono::steady_clock::now();
    const Mdx23cConfig& c = manifest.config;
    if (!planes || !stems || samples <= 0) return fail(ANCHA_E_INVALID, "mdx23c_separate: empty input");
    if (samples > kMaxTrackSamples) return fail(ANCHA_E_INVALID, "mdx23c_separate: track longer than 2^36 samples");
    const int ov = overlap > 0 ? overlap : c.overlap;
    const int64_t chunk = c.chunk_samples();
    Mdx23cPlan plan;
    try {
        plan = Mdx23cPlan::make(samples, chunk, ov);
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    const int64_t border = plan.border;
    std::vector<int64_t> starts;
    for (int64_t i = 0; i < plan.chunks; ++i)
        if (plan.intersects(i * plan.step)) starts.push_back(i * plan.step);
    const int b = batch > 0 ? std::min(batch, 4) : 4;
    if (batch < 0) return fail(ANCHA_E_INVALID, "mdx23c_separate: batch");
    const int stems_n = (int)c.stems.size(), frames = c.frames, bins = c.bins;
    if (chunk / c.hop + 1 != frames) return fail(ANCHA_E_INVALID, "MDX23C STFT frame count mismatch");
    if (!dsp_window_.p) return fail(ANCHA_E_UNSUPPORTED, "MDX23C separation: n_fft must be a power of two");
    ANCHA_CUDA(cudaSetDevice(device));
    try {
        DevBuf track, audio, spec, yout, scratch, waves, sums, flag;
        cudaStream_t s = nullptr;
        ANCHA_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
        // Declared after the buffers, so destroyed before them: no buffer is freed while work
        // queued on the stream (an early error return) may still use it, and the stream is
        // released on every path, an allocation failure included.
        struct StreamGuard {
            cudaStream_t s;
            ~StreamGuard() {
                cudaStreamSynchronize(s);
                cudaStreamDestroy(s);
            }
        } guard{s};
        track.alloc((size_t)2 * samples * sizeof(float));
        audio.alloc((size_t)b * 2 * chunk * sizeof(float));
        spec.alloc((size_t)b * 4 * bins * frames * sizeof(float));
        yout.alloc((size_t)b * stems_n * 4 * bins * frames * sizeof(float));
        scratch.alloc((size_t)b * stems_n * 2 * frames * c.n_fft * sizeof(float));
        waves.alloc((size_t)b * stems_n * 2 * chunk * sizeof(float));
        sums.alloc((size_t)stems_n * 2 * samples * sizeof(float));
        flag.alloc(sizeof(int));
        ANCHA_CUDA(cudaMemcpyAsync(track.p, planes, (size_t)2 * samples * sizeof(float), cudaMemcpyHostToDevice, s));
        ANCHA_CUDA(cudaMemsetAsync(sums.p, 0, sums.bytes, s));
        ANCHA_CUDA(cudaMemsetAsync(flag.p, 0, sizeof(int), s));
        MdxDsp d;
        d.n_fft = c.n_fft;
        d.window = dsp_window_.as<float>();
        d.twiddle = dsp_twiddle_.as<float2>();
        for (size_t i = 0; i < starts.size(); i += b) {
            if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
            const int n = (int)std::min<size_t>(b, starts.size() - i);
            const int64_t* st = starts.data() + i;
            ANCHA_TRY(mdx_gather(track.as<float>(), samples, st, n, (int)chunk, border, audio.as<float>(), s));
            ANCHA_TRY(mdx_stft(d, audio.as<float>(), n, (int)chunk, c.hop, bins, spec.as<float>(), s));
            ANCHA_TRY(forward(spec.as<float>(), n, frames, yout.as<float>(), cancel, s));
            ANCHA_TRY(mdx_istft(d, yout.as<float>(), n, stems_n, bins, frames, c.hop, (int)chunk, scratch.as<float>(),
                                waves.as<float>(), flag.as<int>(), s));
            ANCHA_TRY(mdx_overlap_add(waves.as<float>(), st, n, stems_n * 2, (int)chunk, border, samples,
                                      sums.as<float>(), flag.as<int>(), s));
        }
        ANCHA_TRY(mdx_scale(sums.as<float>(), (int64_t)stems_n * 2 * samples, 1.f / (float)ov, s));
        ANCHA_CUDA(cudaMemcpyAsync(stems, sums.p, sums.bytes, cudaMemcpyDeviceToHost, s));
        int status = 0;
        ANCHA_CUDA(cudaMemcpyAsync(&status, flag.p, sizeof(int), cudaMemcpyDeviceToHost, s));
        ANCHA_CUDA(cudaStreamSynchronize(s));
        if (status & 1) return fail(ANCHA_E_NONFINITE, "non-finite MDX23C output");
        if (status & 2) return fail(ANCHA_E_INVALID, "iSTFT has an uncovered sample");
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
    if (seconds)
        *seconds = std::chrono::duration<double>(std::chrono::steady_clock::now() - t_start).count();
    return ANCHA_OK;
}

}  // namespace ancha
