// RoFormer model: strict schema-1 loading with the reference's load-time folding
// (crates/ancha-models/src/network.rs:89-278, roformer.rs:205-256 and 381-409,
// weights.rs:29-176) and the forward pass (network.rs:301-400, roformer.rs:464-521) over
// this library's kernels.
//
// Device layout. The residual stream x is f32 [chunks, bands, frames, dim] for both axes:
// the time transformer sees groups = (chunk, band) with tokens = frames (token stride 1 row)
// and the band transformer sees groups = (chunk, frame) with tokens = bands (token stride =
// frames rows), so the axial swaps of network.rs:336-338 are strides, not copies. Every
// GEMM is row-wise, so it is indifferent to the grouping; RoPE finds its token as
// (row / div) % tokens. Projection weights are stored [out, in] (K-major).
#include "model.hpp"

#include <cmath>
#include <cstring>
#include <mutex>
#include <set>
#include <thread>

#include "attention.cuh"
#include "dsp.cuh"
#include "rowops.cuh"

#ifndef ANCHA_FP32_SPLIT
#define ANCHA_FP32_SPLIT 1
#endif

namespace ancha {

void DevBuf::release() {
    if (p) cudaFree(p);
    p = nullptr;
    bytes = 0;
}

void DevBuf::alloc(size_t n) {
    release();
    if (n == 0) n = 16;
    cudaError_t e = cudaMalloc(&p, n);
    if (e != cudaSuccess) {
        p = nullptr;
        throw std::runtime_error(std::string("cudaMalloc(") + std::to_string(n) + "): " +
                                 cudaGetErrorString(e));
    }
    bytes = n;
}

namespace {

[[noreturn]] void bad(const std::string& m) { throw std::runtime_error(m); }

void ensure(bool ok, const char* msg) {
    if (!ok) bad(msg);
}

template <typename T>
void upload(DevBuf& d, const std::vector<T>& v) {
    d.alloc(v.size() * sizeof(T));
    cudaError_t e = cudaMemcpy(d.p, v.data(), v.size() * sizeof(T), cudaMemcpyHostToDevice);
    if (e != cudaSuccess) bad(std::string("cudaMemcpy: ") + cudaGetErrorString(e));
}

// Upload f32 host weights as f32, bf16 or f16 (round to nearest even).
void upload_weights(DevBuf& d, const std::vector<float>& v, int elt) {
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

const std::set<std::string> kConfigKeys = {
    "family", "dim", "depth", "heads", "head_dim", "ff_mult", "mask_depth", "mask_expansion",
    "sample_rate", "n_fft", "hop", "chunk_samples", "overlap", "zero_dc", "stems", "bands"};
const std::set<std::string> kManifestKeys = {
    "schema_version", "model_id", "weights_sha256", "checkpoint_sha256", "source_url",
    "forward_revision", "weight_license", "config"};

void check_keys(const Json& j, const std::set<std::string>& keys, const char* what) {
    if (j.kind != Json::Object) bad(std::string(what) + " must be an object");
    for (auto& kv : j.obj)
        if (!keys.count(kv.first)) bad(std::string("unknown field `") + kv.first + "` in " + what);
    for (auto& k : keys)
        if (!j.find(k)) bad(std::string("missing field `") + k + "` in " + what);
}

bool is_hex64(const std::string& s) {
    if (s.size() != 64) return false;
    for (char c : s)
        if (!isxdigit((unsigned char)c)) return false;
    return true;
}

}  // namespace

// ------------------------------------------------------------------------ config (config.rs)
ModelConfig ModelConfig::from_json(const Json& j) {
    check_keys(j, kConfigKeys, "config");
    ModelConfig c;
    c.family = j.at("family").as_string();
    c.dim = j.at("dim").as_int32();
    c.depth = j.at("depth").as_int32();
    c.heads = j.at("heads").as_int32();
    c.head_dim = j.at("head_dim").as_int32();
    c.ff_mult = j.at("ff_mult").as_int32();
    c.mask_depth = j.at("mask_depth").as_int32();
    c.mask_expansion = j.at("mask_expansion").as_int32();
    c.sample_rate = j.at("sample_rate").as_int32();
    c.n_fft = j.at("n_fft").as_int32();
    c.hop = j.at("hop").as_int32();
    c.chunk_samples = j.at("chunk_samples").as_int();
    c.overlap = j.at("overlap").as_int32();
    c.zero_dc = j.at("zero_dc").as_bool();
    for (auto& s : j.at("stems").arr) c.stems.push_back(s.as_string());
    for (auto& b : j.at("bands").arr) {
        std::vector<int> band;
        for (auto& f : b.arr) band.push_back(f.as_int32());
        c.bands.push_back(band);
    }
    if (c.family != "bs-roformer" && c.family != "mel-band-roformer" && c.family != "hyperace-v2")
        bad("unknown family " + c.family);
    return c;
}

Json ModelConfig::to_json() const {
    Json j = Json::make_object();
    j.set("family", Json::of(family));
    j.set("dim", Json::of(dim));
    j.set("depth", Json::of(depth));
    j.set("heads", Json::of(heads));
    j.set("head_dim", Json::of(head_dim));
    j.set("ff_mult", Json::of(ff_mult));
    j.set("mask_depth", Json::of(mask_depth));
    j.set("mask_expansion", Json::of(mask_expansion));
    j.set("sample_rate", Json::of(sample_rate));
    j.set("n_fft", Json::of(n_fft));
    j.set("hop", Json::of(hop));
    j.set("chunk_samples", Json::of((double)chunk_samples));
    j.set("overlap", Json::of(overlap));
    j.set("zero_dc", Json::of_bool(zero_dc));
    Json st = Json::make_array();
    for (auto& s : stems) st.arr.push_back(Json::of(s));
    j.set("stems", st);
    Json bs = Json::make_array();
    for (auto& b : bands) {
        Json a = Json::make_array();
        for (int f : b) a.arr.push_back(Json::of(f));
        bs.arr.push_back(a);
    }
    j.set("bands", bs);
    return j;
}

void ModelConfig::validate() const {
    ensure(dim > 0 && depth > 0 && depth <= 64 && dim <= 4096, "invalid model dimensions");
    ensure(heads > 0 && heads <= 64 && head_dim > 0 && head_dim % 2 == 0 && head_dim <= 256,
           "invalid attention dimensions");
    ensure(ff_mult > 0 && ff_mult <= 16 && mask_depth > 0 && mask_depth <= 8 &&
               mask_expansion > 0 && mask_expansion <= 16,
           "invalid MLP dimensions");
    ensure(sample_rate == 44100 && n_fft == 2048 && hop >= 1 && hop <= 1024,
           "schema 1 requires 44100 Hz, FFT 2048 and hop <= 1024");
    ensure(chunk_samples > n_fft / 2 && chunk_samples <= 44100 * 60 && overlap > 0 && overlap <= 16,
           "invalid chunk settings");
    ensure(!stems.empty() && stems.size() <= 2, "invalid stem labels");
    for (auto& s : stems)
        ensure(s == "vocals" || s == "instrumental" || s == "lead_vocals", "invalid stem labels");
    ensure(stems.size() == 1 || stems[0] != stems[1], "duplicate stems");
    bool lead = false;
    for (auto& s : stems) lead |= s == "lead_vocals";
    ensure(!lead || (mel() && stems.size() == 1),
           "lead vocals require a single-head Mel karaoke model");
    ensure(bands.size() >= 2 && bands.size() <= 256, "invalid band count");
    const int nbins = n_fft / 2 + 1;
    std::vector<int> cov(nbins, 0);
    for (auto& b : bands) {
        ensure(!b.empty(), "bands must be nonempty and strictly ordered");
        for (size_t i = 1; i < b.size(); ++i)
            ensure(b[i - 1] < b[i], "bands must be nonempty and strictly ordered");
        for (int f : b) {
            ensure(f >= 0 && f < nbins, "band index out of range");
            cov[f]++;
        }
    }
    for (int n : cov) ensure(n > 0, "bands leave uncovered FFT bins");
    if (!mel()) {
        for (int n : cov) ensure(n == 1, "BS bands must partition the frequency axis");
        int expect = 0;
        for (auto& b : bands)
            for (int f : b) ensure(f == expect++, "BS bands must be contiguous and in frequency order");
    }
    if (family == "hyperace-v2")
        ensure(dim == 256 && bands.size() == 62 && stems.size() == 1,
               "HyperACE v2 requires dim=256, 62 bands and one stem");
}

Manifest Manifest::from_json(const Json& j) {
    check_keys(j, kManifestKeys, "manifest");
    Manifest m;
    m.schema_version = j.at("schema_version").as_int32();
    m.model_id = j.at("model_id").as_string();
    m.weights_sha256 = j.at("weights_sha256").as_string();
    m.checkpoint_sha256 = j.at("checkpoint_sha256").as_string();
    m.source_url = j.at("source_url").as_string();
    m.forward_revision = j.at("forward_revision").as_string();
    m.weight_license = j.at("weight_license").as_string();
    m.config = ModelConfig::from_json(j.at("config"));
    return m;
}

void Manifest::validate() const {
    ensure(schema_version == 1, "unsupported model package schema");
    ensure(!model_id.empty(), "model ID is empty");
    ensure(is_hex64(weights_sha256) && is_hex64(checkpoint_sha256), "invalid SHA256");
    config.validate();
}

// --------------------------------------------------------------------------- model loading
bool Model::tc_gemm() const { return elt_ != ELT_F32; }
bool Model::tc_attention() const { return elt_ != ELT_F32; }

Model::~Model() {
    if (device >= 0) cudaSetDevice(device);
}

std::unique_ptr<Model> Model::load(const std::string& package, int device, int precision) {
    if (precision != ANCHA_PRECISION_F32 && precision != ANCHA_PRECISION_BF16 &&
        precision != ANCHA_PRECISION_F16)
        bad("unknown precision");
    std::unique_ptr<Model> m(new Model());
    m->device = -1;  // no device yet: the destructor leaves the caller's current device alone
    // The manifest first: an invalid package is rejected before any device work, and the
    // configuration decides the norm fusion below.
    m->manifest = Manifest::from_json(Json::parse(read_file(package + "/manifest.json")));
    m->manifest.validate();
    cudaError_t e = cudaSetDevice(device);
    if (e != cudaSuccess) bad(std::string("cudaSetDevice: ") + cudaGetErrorString(e));
    m->device = device;
    m->precision = precision;
    m->elt_ = precision == ANCHA_PRECISION_BF16 ? ELT_BF16 : precision == ANCHA_PRECISION_F16 ? ELT_F16 : ELT_F32;
    m->fuse_norms_ = m->elt_ != ELT_F32 && m->manifest.config.dim % 32 == 0;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) m->device_name = prop.name;
    const std::string bytes = read_file(package + "/model.safetensors");
    // SHA-256 on another thread while the model is built (weights.rs:29-40).
    std::string digest;
    std::thread hasher([&] {
        digest = sha256_hex(reinterpret_cast<const uint8_t*>(bytes.data()), bytes.size());
    });
    try {
        SafeTensors w(bytes);
        const ModelConfig& c = m->manifest.config;
        const int bf = m->elt_;
        const int dim = c.dim, inner = c.heads * c.head_dim, hidden = c.dim * c.ff_mult;
        const int nb = (int)c.bands.size();
        m->bands = nb;
        m->bins = c.n_fft / 2 + 1;
        // Band split (network.rs:107-131): sqrt(width)·gamma folded into the input columns.
        std::vector<int> cols, offsets{0};
        std::vector<float> wsplit, bsplit;
        for (int b = 0; b < nb; ++b) {
            const int width = (int)c.bands[b].size() * 4;
            const std::string p = "band_split.to_features." + std::to_string(b);
            std::vector<float> gamma = w.take(p + ".0.gamma", {width});
            const float root = std::sqrt((float)width);
            std::vector<float> W = w.take(p + ".1.weight", {dim, width});
            m->wsplit_off_.push_back((int64_t)wsplit.size());
            for (int o = 0; o < dim; ++o)
                for (int i = 0; i < width; ++i) wsplit.push_back(W[(size_t)o * width + i] * (gamma[i] * root));
            std::vector<float> bias = w.take(p + ".1.bias", {dim});
            bsplit.insert(bsplit.end(), bias.begin(), bias.end());
            for (int f : c.bands[b])
                for (int k = 0; k < 4; ++k) cols.push_back(4 * f + k);
            m->width_.push_back(width);
            m->offset_.push_back(offsets.back());
            offsets.push_back(offsets.back() + width);
            m->max_width = std::max(m->max_width, width);
        }
        m->total_width = offsets.back();
        if (m->elt_ == ELT_F16) {
            // Tensor-core band split (f16 only: bf16's 8-bit mantissa on these inputs would eat
            // into the little margin bf16 has left; it keeps the fp32 split).
            const int kp = (m->max_width + 63) / 64 * 64;
            std::vector<float> w16((size_t)nb * dim * kp, 0.f);
            for (int b = 0; b < nb; ++b)
                for (int o = 0; o < dim; ++o)
                    for (int i = 0; i < m->width_[b]; ++i)
                        w16[((size_t)b * dim + o) * kp + i] = wsplit[m->wsplit_off_[b] + (size_t)o * m->width_[b] + i];
            upload_weights(m->wsplit16_, w16, ELT_F16);
            m->split_kp_ = kp;
        }
        upload(m->zcols_, cols);
        upload(m->zoffsets_, offsets);
        upload(m->wsplit_, wsplit);
        upload(m->bsplit_, bsplit);
        // Axial transformers (roformer.rs:205-256, 381-409; keys network.rs:133-152).
        const int ncols = 3 * inner + c.heads;
        m->ldq = (ncols + 7) / 8 * 8;
        const float root = std::sqrt((float)dim);
        for (int i = 0; i < c.depth; ++i) {
            std::array<TransformerWeights, 2> pair;
            for (int a = 0; a < 2; ++a) {
                TransformerWeights& t = pair[a];
                const std::string p = "layers." + std::to_string(i) + "." + std::to_string(a);
                const std::string at = p + ".layers.0.0";
                std::vector<float> g = w.take(at + ".norm.gamma", {dim});
                std::vector<float> norm(dim);
                for (int d = 0; d < dim; ++d) norm[d] = g[d] * root;
                std::vector<float> qkv = w.take(at + ".to_qkv.weight", {3 * inner, dim});
                std::vector<float> gw = w.take(at + ".to_gates.weight", {c.heads, dim});
                std::vector<float> gb = w.take(at + ".to_gates.bias", {c.heads});
                std::vector<float> packed((size_t)ncols * dim);
                for (int o = 0; o < 3 * inner; ++o)
                    for (int d = 0; d < dim; ++d) packed[(size_t)o * dim + d] = qkv[(size_t)o * dim + d] * norm[d];
                for (int h = 0; h < c.heads; ++h)
                    for (int d = 0; d < dim; ++d)
                        packed[(size_t)(3 * inner + h) * dim + d] = gw[(size_t)h * dim + d] * norm[d];
                std::vector<float> pbias(ncols, 0.f);
                for (int h = 0; h < c.heads; ++h) pbias[3 * inner + h] = gb[h];
                upload_weights(t.wqkvg, packed, bf);
                upload(t.bqkvg, pbias);
                upload_weights(t.wout, w.take(at + ".to_out.0.weight", {dim, inner}), bf);
                std::vector<float> freqs = w.take(at + ".rotary_embed.freqs", {c.head_dim / 2});
                int slot = -1;
                for (size_t s = 0; s < m->rope_freqs_.size(); ++s)
                    if (m->rope_freqs_[s] == freqs) slot = (int)s;
                if (slot < 0) {
                    slot = (int)m->rope_freqs_.size();
                    m->rope_freqs_.push_back(freqs);
                }
                t.rope_set = slot;
                const std::string ff = p + ".layers.0.1.net";
                std::vector<float> g2 = w.take(ff + ".0.gamma", {dim});
                std::vector<float> w1 = w.take(ff + ".1.weight", {hidden, dim});
                for (int o = 0; o < hidden; ++o)
                    for (int d = 0; d < dim; ++d) w1[(size_t)o * dim + d] *= g2[d] * root;
                upload_weights(t.w1, w1, bf);
                upload(t.b1, w.take(ff + ".1.bias", {hidden}));
                upload_weights(t.w2, w.take(ff + ".4.weight", {dim, hidden}), bf);
                upload(t.b2, w.take(ff + ".4.bias", {dim}));
                if (c.mel()) {
                    std::vector<float> s = w.take(p + ".norm.gamma", {dim});
                    for (float& v : s) v *= root;
                    upload(t.out_scale, s);
                }
            }
            m->layers_.push_back(std::move(pair));
        }
        if (!c.mel()) {
            std::vector<float> s = w.take("final_norm.gamma", {dim});
            for (float& v : s) v *= root;
            upload(m->final_scale_, s);
        }
        // Mask estimators (network.rs:158-205): hidden tanh layers, then the GLU layer with
        // value / gate rows interleaved so each output pair sits in one epilogue thread.
        const int hidden_layers = c.mel() ? c.mask_depth : c.mask_depth - 1;
        const int mh = c.dim * c.mask_expansion;
        for (size_t s = 0; s < c.stems.size(); ++s) {
            MaskWeights mw;
            int in = dim;
            auto key = [&](int b, int layer) {
                return "mask_estimators." + std::to_string(s) + ".to_freqs." + std::to_string(b) +
                       ".0." + std::to_string(layer * 2);
            };
            for (int l = 0; l < hidden_layers; ++l) {
                std::vector<float> W, B;
                for (int b = 0; b < nb; ++b) {
                    std::vector<float> wb = w.take(key(b, l) + ".weight", {mh, in});
                    std::vector<float> bb = w.take(key(b, l) + ".bias", {mh});
                    W.insert(W.end(), wb.begin(), wb.end());
                    B.insert(B.end(), bb.begin(), bb.end());
                }
                mw.w.emplace_back();
                mw.b.emplace_back();
                upload_weights(mw.w.back(), W, bf);
                upload(mw.b.back(), B);
                in = mh;
            }
            const int rows2 = 2 * m->max_width;
            std::vector<float> G((size_t)nb * rows2 * in, 0.f), GB((size_t)nb * rows2, 0.f);
            for (int b = 0; b < nb; ++b) {
                const int width = m->width_[b];
                std::vector<float> wb = w.take(key(b, hidden_layers) + ".weight", {2 * width, in});
                std::vector<float> bb = w.take(key(b, hidden_layers) + ".bias", {2 * width});
                for (int j = 0; j < width; ++j) {
                    for (int half = 0; half < 2; ++half) {
                        const size_t dst = (size_t)b * rows2 + 2 * j + half;
                        const size_t src = (size_t)(half * width + j);
                        std::memcpy(&G[dst * in], &wb[src * in], sizeof(float) * in);
                        GB[dst] = bb[src];
                    }
                }
            }
            upload_weights(mw.glu_w, G, bf);
            upload(mw.glu_b, GB);
            m->masks_.push_back(std::move(mw));
        }
        m->tensor_count = w.finish();
        // Overlapping-band coverage (network.rs:231-246): per spectrum row r = 2·bin + ch the
        // (band, feature) pairs that feed it, in band order.
        const int rows = 2 * m->bins;
        std::vector<std::vector<std::pair<int, int>>> cover(rows);
        for (int b = 0; b < nb; ++b)
            for (size_t i = 0; i < c.bands[b].size(); ++i)
                for (int ch = 0; ch < 2; ++ch)
                    cover[2 * c.bands[b][i] + ch].push_back({b, (int)(i * 2 + ch) * 2});
        for (auto& v : cover) m->max_cover = std::max(m->max_cover, (int)v.size());
        std::vector<int> count(rows);
        std::vector<int> ent((size_t)rows * m->max_cover * 2, 0);
        for (int r = 0; r < rows; ++r) {
            count[r] = (int)cover[r].size();
            for (size_t e = 0; e < cover[r].size(); ++e) {
                ent[((size_t)r * m->max_cover + e) * 2] = cover[r][e].first;
                ent[((size_t)r * m->max_cover + e) * 2 + 1] = cover[r][e].second;
            }
        }
        upload(m->cover_count_, count);
        upload(m->cover_entries_, ent);
        std::vector<int> glu_n(nb);
        for (int b = 0; b < nb; ++b) glu_n[b] = 2 * m->width_[b];
        upload(m->glu_n_, glu_n);
    } catch (...) {
        hasher.join();
        throw;
    }
    hasher.join();
    if (digest != m->manifest.weights_sha256) bad("model checksum mismatch");
    if (m->elt_ == ELT_F32 && ANCHA_FP32_SPLIT) {
        // fp32 on the tensor cores: three-plane bf16 splits of the transformer and mask-head
        // weights (the grouped band split, a small share of the FLOPs, stays on the FFMA kernel).
        const ModelConfig& c = m->manifest.config;
        const int dim = c.dim, inner = c.heads * c.head_dim, hidden = c.dim * c.ff_mult;
        const int ncols = 3 * inner + c.heads;
        auto split = [&](const DevBuf& w, int n, int k) {
            if (k % 8) return;  // the tensor-core GEMM needs 16-byte operand rows
            DevBuf d;
            d.alloc((size_t)3 * n * k * 2);
            if (split3_rows(w.as<float>(), k, d.p, n, k, nullptr) != ANCHA_OK) bad("weight split");
            m->split_w_[w.p] = std::move(d);
        };
        for (auto& pair : m->layers_)
            for (auto& t : pair) {
                split(t.wqkvg, ncols, dim);
                split(t.wout, dim, inner);
                split(t.w1, hidden, dim);
                split(t.w2, dim, hidden);
            }
        // Mask heads: [bands][rows][in] per layer, split as bands · rows rows (plane-major).
        const int mh = c.dim * c.mask_expansion;
        for (auto& mw : m->masks_) {
            for (size_t l = 0; l < mw.w.size(); ++l) split(mw.w[l], m->bands * mh, l == 0 ? dim : mh);
            split(mw.glu_w, m->bands * 2 * m->max_width, mh);
        }
        if (cudaDeviceSynchronize() != cudaSuccess) bad("weight split");
        m->split_ = true;
    }
    return m;
}

// --------------------------------------------------------------------------- forward pass
int Model::ensure_workspace(int chunks, int frames, cudaStream_t s) {
    if (ws_.chunks >= chunks && ws_.frames == frames) return ANCHA_OK;
    const ModelConfig& c = manifest.config;
    try {
        Workspace w;
        w.chunks = chunks;
        w.frames = frames;
        const int64_t R = (int64_t)chunks * bands * frames;
        const size_t e = elt_size(elt_);
        const int inner = c.heads * c.head_dim, hidden = c.dim * c.ff_mult;
        const int mh = c.dim * c.mask_expansion;
        w.x.alloc(R * c.dim * 4);
        w.xn.alloc(R * c.dim * e);
        w.qkvg.alloc(R * ldq * e);
        w.att.alloc(R * inner * e);
        w.hidden.alloc(R * std::max(hidden, mh) * e);
        w.h2.alloc(R * mh * e);
        w.z.alloc((int64_t)chunks * frames * total_width * 4);
        if (split_kp_) w.z16.alloc(R * split_kp_ * 2);
        w.glu.alloc(R * max_width * 4);
        // The three bf16 planes of a GEMM's A operand, or of the q | k | v rows for the time-axis
        // attention (3 · inner columns).
        if (split_) w.a3.alloc((size_t)3 * R * std::max(std::max(c.dim, 3 * inner), std::max(hidden, mh)) * 2);
        if (fuse_norms_) {
            w.ss_x.alloc(R * (c.dim / 32) * 4);
            w.ss_y.alloc(R * (c.dim / 32) * 4);
            w.ss_yg.alloc(R * (c.dim / 32) * 4);
        }
        if (!flag_.p) {
            flag_.alloc(16);
            if (cudaMemset(flag_.p, 0, 16) != cudaSuccess) bad("cudaMemset");
        }
        // Grouped GEMM descriptors: band split, then per stem the hidden layers and the GLU.
        const int G = chunks * bands;
        std::vector<GemmGroup> split(G);
        for (int cc = 0; cc < chunks; ++cc)
            for (int b = 0; b < bands; ++b) {
                GemmGroup& g = split[cc * bands + b];
                g.a = w.z.as<float>() + (int64_t)cc * frames * total_width + offset_[b];
                g.lda = total_width;
                g.b = wsplit_.as<float>() + wsplit_off_[b];
                g.ldb = width_[b];
                g.bias = bsplit_.as<float>() + (int64_t)b * c.dim;
                g.residual = nullptr;
                g.ldr = 0;
                g.out = w.x.as<float>() + ((int64_t)(cc * bands + b) * frames) * c.dim;
                g.ldo = c.dim;
                g.m = frames;
                g.n = c.dim;
                g.k = width_[b];
            }
        upload(w.split_groups, split);
        std::vector<GemmGroup> mg;
        const int hidden_layers = c.mel() ? c.mask_depth : c.mask_depth - 1;
        for (size_t st = 0; st < masks_.size(); ++st) {
            const MaskWeights& mw = masks_[st];
            int in = c.dim;
            const char* a_base = (const char*)(elt_ != ELT_F32 ? w.xn.p : w.x.p);
            for (int l = 0; l <= hidden_layers; ++l) {
                const bool glu = l == hidden_layers;
                const char* out_base = glu ? (const char*)w.glu.p
                                           : (const char*)(l % 2 == 0 ? w.hidden.p : w.h2.p);
                const int n = glu ? 0 : mh;
                for (int cc = 0; cc < chunks; ++cc)
                    for (int b = 0; b < bands; ++b) {
                        GemmGroup g{};
                        const int64_t row0 = (int64_t)(cc * bands + b) * frames;
                        g.a = a_base + row0 * in * e;
                        g.lda = in;
                        if (glu) {
                            g.b = (const char*)mw.glu_w.p + (size_t)b * 2 * max_width * in * e;
                            g.bias = mw.glu_b.as<float>() + (int64_t)b * 2 * max_width;
                            g.n = 2 * width_[b];
                            g.out = (char*)out_base + row0 * max_width * 4;
                            g.ldo = max_width;
                        } else {
                            g.b = (const char*)mw.w[l].p + (size_t)b * mh * in * e;
                            g.bias = mw.b[l].as<float>() + (int64_t)b * mh;
                            g.n = n;
                            g.out = (char*)out_base + row0 * mh * e;
                            g.ldo = mh;
                        }
                        g.ldb = in;
                        g.m = frames;
                        g.k = in;
                        mg.push_back(g);
                    }
                a_base = out_base;
                in = mh;
            }
        }
        upload(w.mask_groups, mg);
        // RoPE tables [4, tokens, head_dim] per frequency set and axis (roformer.rs:281-302):
        // angle t·f rounded to f32, sine / cosine in double, the query pair scaled by
        // 1/sqrt(head_dim).
        const int hd = c.head_dim;
        const float qscale = 1.f / std::sqrt((float)hd);
        for (auto& freqs : rope_freqs_) {
            for (int axis = 0; axis < 2; ++axis) {
                const int tokens = axis == 0 ? frames : bands;
                std::vector<float> tab((size_t)4 * tokens * hd), pairs((size_t)2 * tokens * hd);
                for (int q = 0; q < 2; ++q) {
                    const float sc = q == 0 ? qscale : 1.f;
                    for (int t = 0; t < tokens; ++t)
                        for (size_t j = 0; j < freqs.size(); ++j) {
                            const float ang = (float)t * freqs[j];
                            const double sn = std::sin((double)ang), cs = std::cos((double)ang);
                            const size_t base_c = ((size_t)(2 * q) * tokens + t) * hd + 2 * j;
                            const size_t base_s = ((size_t)(2 * q + 1) * tokens + t) * hd + 2 * j;
                            tab[base_c] = tab[base_c + 1] = (float)(cs * sc);
                            tab[base_s] = (float)(-sn * sc);
                            tab[base_s + 1] = (float)(sn * sc);
                            const size_t pr = (((size_t)q * (hd / 2) + j) * tokens + t) * 2;
                            pairs[pr] = (float)(cs * sc);
                            pairs[pr + 1] = (float)(sn * sc);
                        }
                }
                w.rope.emplace_back();
                upload(w.rope.back(), tab);
                w.rope_pairs.emplace_back();
                upload(w.rope_pairs.back(), pairs);
            }
        }
        ws_ = std::move(w);
    } catch (const std::exception& ex) {
        ws_ = Workspace();
        return fail(ANCHA_E_CUDA, std::string("workspace: ") + ex.what());
    }
    (void)s;
    return ANCHA_OK;
}

int Model::linear(const void* x, int64_t ldx, const DevBuf& w, const float* bias,
                  const float* residual, int64_t ldr, void* out, int64_t ldo, int out_type,
                  int64_t m, int n, int k, int act, const float* rope, const float* rope_pairs,
                  int rope_tokens, int rope_div, cudaStream_t s) {
    return linear_fused(x, ldx, w, bias, residual, ldr, out, ldo, out_type, m, n, k, act, rope, rope_pairs,
                        rope_tokens, rope_div, NormFusion{}, s);
}

int Model::linear_fused(const void* x, int64_t ldx, const DevBuf& w, const float* bias, const float* residual,
                        int64_t ldr, void* out, int64_t ldo, int out_type, int64_t m, int n, int k, int act,
                        const float* rope, const float* rope_pairs, int rope_tokens, int rope_div,
                        const NormFusion& nf, cudaStream_t s) {
    GemmGroup g{};
    g.a = x;
    g.lda = ldx;
    g.b = w.p;
    g.ldb = k;
    g.bias = bias;
    g.residual = residual;
    g.ldr = ldr;
    g.out = out;
    g.ldo = ldo;
    g.m = (int)m;
    g.n = n;
    g.k = k;
    GemmEpilogue e{};
    e.act = act;
    e.out_type = out_type;
    e.rope = rope;
    e.rope_pairs = rope_pairs;
    const ModelConfig& c = manifest.config;
    e.rope_width = rope ? c.heads * c.head_dim : 0;
    e.rope_tokens = rope_tokens;
    e.rope_div = rope_div;
    e.rope_hd = c.head_dim;
    const int slots = c.dim / 32;
    e.row_ss = nf.row_ss;
    e.row_ss_n = nf.row_ss ? slots : 0;
    e.res_ss = nf.res_ss;
    e.res_ss_n = nf.res_ss ? slots : 0;
    e.res_col = nf.res_col;
    e.out16 = nf.out16;
    e.out16_col = nf.out16_col;
    e.ss_out = nf.ss_out;
    e.ss16_out = nf.ss16_out;
    const bool fused = nf.row_ss || nf.res_ss || nf.out16 || nf.ss_out;
    if (elt_ == ELT_F32 && split_ && !fused) {
        // fp32 on the tensor cores: A split into three bf16 planes, the six significant plane
        // products in one K loop against the weight's planes, f32 accumulation and epilogue.
        const auto it = split_w_.find(w.p);
        if (it != split_w_.end()) {
            ANCHA_TRY(split3_rows(static_cast<const float*>(x), ldx, ws_.a3.p, m, k, s));
            GemmGroup g3 = g;
            g3.a = ws_.a3.p;
            g3.lda = k;
            g3.b = it->second.p;
            g3.ldb = k;
            g3.split3 = true;
            const int st = gemm_tc(g3, ELT_BF16, e, s);
            if (st != ANCHA_E_UNSUPPORTED) return st;
        }
    }
    if (elt_ != ELT_F32) {
        const int st = gemm_tc(g, elt_, e, s);
        if (st != ANCHA_E_UNSUPPORTED) return st;
        // The FFMA kernel has no row-norm fusion: a fused call must not fall back.
        if (fused) return fail(ANCHA_E_UNSUPPORTED, "linear: row-norm fusion needs the tensor-core GEMM");
    }
    return gemm_ffma(g, nullptr, 1, (int)m, n, elt_, elt_, 1, e, s);
}

int Model::transformer(const TransformerWeights& t, bool time_axis, cudaStream_t s) {
    const ModelConfig& c = manifest.config;
    const int T = ws_.frames, C = cur_chunks_;
    const int64_t R = (int64_t)C * bands * T;
    const int dim = c.dim, inner = c.heads * c.head_dim, hidden = c.dim * c.ff_mult;
    const int bf = elt_;
    float* x = ws_.x.as<float>();
    const size_t rope_slot = (size_t)t.rope_set * 2 + (time_axis ? 0 : 1);
    const DevBuf& rope = ws_.rope[rope_slot];
    // Packed q | k | v | gate projection of unit_norm(x), RoPE in the epilogue. With the
    // row-norm fusion the previous block left x's operand-type copy in xn and its row norms in
    // block_ss_, and the GEMM applies the unit norm to its output rows.
    NormFusion g1;
    if (fuse_norms_ && block_ss_) {
        g1.row_ss = block_ss_;
    } else {
        ANCHA_TRY(norm_rows(x, dim, nullptr, ws_.xn.p, bf, dim, R, dim, s));
    }
    ANCHA_TRY(linear_fused(ws_.xn.p, dim, t.wqkvg, t.bqkvg.as<float>(), nullptr, 0, ws_.qkvg.p, ldq, bf,
                           R, 3 * inner + c.heads, dim, ANCHA_ACT_NONE, rope.as<float>(),
                           ws_.rope_pairs[rope_slot].as<float>(), time_axis ? T : bands, time_axis ? 1 : T,
                           g1, s));
    // Gated attention within each group.
    AttnArgs a{};
    a.q = a.k = a.v = a.gate = ws_.qkvg.p;
    a.out = ws_.att.p;
    a.heads = c.heads;
    a.head_dim = c.head_dim;
    a.ld = ldq;
    a.out_ld = inner;
    a.q_col = 0;
    a.k_col = inner;
    a.v_col = 2 * inner;
    a.gate_col = 3 * inner;
    a.out_col = 0;
    a.elt = bf;
    if (time_axis) {
        a.groups = C * bands;
        a.tokens = T;
        a.group_inner = a.groups;
        a.group_inner_stride = T;
        a.group_outer_stride = 0;
        a.token_stride = 1;
    } else {
        a.groups = C * T;
        a.tokens = bands;
        a.group_inner = T;
        a.group_inner_stride = 1;
        a.group_outer_stride = (int64_t)bands * T;
        a.token_stride = T;
    }
    int ast = ANCHA_E_UNSUPPORTED;
    if (bf != ELT_F32) {
        ast = attention_tc(a, s);
    } else if (split_) {
        // fp32 on the tensor cores: the q | k | v rows split into three bf16 planes.
        ANCHA_TRY(split3_rows(ws_.qkvg.as<float>(), ldq, ws_.a3.p, R, 3 * inner, s));
        ast = attention_tc_split(a, ws_.a3.p, 3 * inner, R * 3 * inner, s);
    }
    if (ast == ANCHA_E_UNSUPPORTED) ast = attention_ffma(a, s);
    ANCHA_TRY(ast);
    // Output projection + residual (with the SourceNorm the previous block deferred), then the
    // GELU feed-forward + residual.
    if (fuse_norms_) {
        NormFusion g2;
        if (pending_scale_) {
            g2.res_ss = ws_.ss_y.as<float>();
            g2.res_col = pending_scale_;
        }
        g2.out16 = ws_.xn.p;
        g2.ss_out = ws_.ss_x.as<float>();
        ANCHA_TRY(linear_fused(ws_.att.p, inner, t.wout, nullptr, x, dim, x, dim, ELT_F32, R, dim, inner,
                               ANCHA_ACT_NONE, nullptr, nullptr, 1, 1, g2, s));
        pending_scale_ = nullptr;
        NormFusion g3;
        g3.row_ss = ws_.ss_x.as<float>();
        ANCHA_TRY(linear_fused(ws_.xn.p, dim, t.w1, t.b1.as<float>(), nullptr, 0, ws_.hidden.p, hidden, bf,
                               R, hidden, dim, ANCHA_ACT_GELU, nullptr, nullptr, 1, 1, g3, s));
        // Block output y: stored unnormalised; the next block's operand copy and row norms are
        // written here, and Mel's SourceNorm (y / ‖y‖ · scale, roformer.rs:516-519) is applied
        // when y is next read as a residual.
        NormFusion g4;
        g4.out16 = ws_.xn.p;
        g4.ss_out = ws_.ss_y.as<float>();
        if (t.out_scale.p) {
            g4.out16_col = t.out_scale.as<float>();
            g4.ss16_out = ws_.ss_yg.as<float>();
        }
        ANCHA_TRY(linear_fused(ws_.hidden.p, hidden, t.w2, t.b2.as<float>(), x, dim, x, dim, ELT_F32, R, dim,
                               hidden, ANCHA_ACT_NONE, nullptr, nullptr, 1, 1, g4, s));
        block_ss_ = t.out_scale.p ? ws_.ss_yg.as<float>() : ws_.ss_y.as<float>();
        pending_scale_ = t.out_scale.p ? t.out_scale.as<float>() : nullptr;
        return ANCHA_OK;
    }
    ANCHA_TRY(linear(ws_.att.p, inner, t.wout, nullptr, x, dim, x, dim, ELT_F32, R, dim, inner,
                     ANCHA_ACT_NONE, nullptr, nullptr, 1, 1, s));
    ANCHA_TRY(norm_rows(x, dim, nullptr, ws_.xn.p, bf, dim, R, dim, s));
    ANCHA_TRY(linear(ws_.xn.p, dim, t.w1, t.b1.as<float>(), nullptr, 0, ws_.hidden.p, hidden, bf,
                     R, hidden, dim, ANCHA_ACT_GELU, nullptr, nullptr, 1, 1, s));
    ANCHA_TRY(linear(ws_.hidden.p, hidden, t.w2, t.b2.as<float>(), x, dim, x, dim, ELT_F32, R, dim,
                     hidden, ANCHA_ACT_NONE, nullptr, nullptr, 1, 1, s));
    // Mel: SourceNorm of the block output (roformer.rs:516-519).
    if (t.out_scale.p) ANCHA_TRY(norm_rows(x, dim, t.out_scale.as<float>(), nullptr, 0, 0, R, dim, s));
    return ANCHA_OK;
}

int Model::reset_flag(cudaStream_t s) {
    if (!flag_.p) {
        try {
            flag_.alloc(16);
        } catch (const std::exception& e) {
            return fail(ANCHA_E_CUDA, e.what());
        }
    }
    ANCHA_CUDA(cudaMemsetAsync(flag_.p, 0, 16, s));
    return ANCHA_OK;
}

int Model::read_flag(cudaStream_t s, int* flag) {
    *flag = 0;
    if (!flag_.p) return ANCHA_OK;
    ANCHA_CUDA(cudaMemcpyAsync(flag, flag_.p, sizeof(int), cudaMemcpyDeviceToHost, s));
    ANCHA_CUDA(cudaStreamSynchronize(s));
    return ANCHA_OK;
}

int Model::forward(const float* spectrum, int chunks, int frames, float* masks,
                   const volatile int* cancel, cudaStream_t s, bool check) {
    const ModelConfig& c = manifest.config;
    if (chunks <= 0 || frames <= 0) return fail(ANCHA_E_INVALID, "invalid model spectrum shape");
    // The runtime's own calls: at most kMaxChunksPerCall chunks of at most 60 s, which keeps the
    // row counts in int and every workspace byte count far below 2^63.
    if (chunks > kMaxChunksPerCall || frames > kMaxChunkSamples / c.hop + 1)
        return fail(ANCHA_E_INVALID, "model_forward: at most 128 chunks of at most 60 s per call");
    ANCHA_CUDA(cudaSetDevice(device));
    ANCHA_TRY(ensure_workspace(chunks, frames, s));
    cur_chunks_ = chunks;
    const int64_t R = (int64_t)chunks * bands * frames;
    const int G = chunks * bands;
    auto cancelled = [&] { return cancel && *cancel; };
    if (cancelled()) return fail(ANCHA_E_CANCELLED, "task cancelled");
    if (check) ANCHA_TRY(reset_flag(s));
    // Band split (network.rs:316-330): gather + unit_norm per band, then one grouped affine
    // per (chunk, band) written straight into x [chunks, bands, frames, dim].
    if (split_kp_) {
        ANCHA_TRY(band_gather_padded(spectrum, chunks, frames, 4 * bins, zcols_.as<int>(), zoffsets_.as<int>(),
                                     bands, split_kp_, ws_.z16.p, s));
        GroupedGemm q{};
        q.a = ws_.z16.p;
        q.lda = split_kp_;
        q.a_group_stride = (int64_t)frames * split_kp_;
        q.m = frames;
        q.k = split_kp_;
        q.groups = G;
        q.b = wsplit16_.p;
        q.ldb = split_kp_;
        q.b_group_stride = (int64_t)c.dim * split_kp_;
        q.b_groups = bands;
        q.n = c.dim;
        q.group_n = nullptr;
        q.bias = bsplit_.as<float>();
        q.bias_group_stride = c.dim;
        q.out = ws_.x.p;
        q.ldo = c.dim;
        q.out_group_stride = (int64_t)frames * c.dim;
        GemmEpilogue e{};
        e.act = ANCHA_ACT_NONE;
        e.out_type = ELT_F32;
        ANCHA_TRY(gemm_tc_grouped(q, ELT_F16, e, s));
    } else {
        ANCHA_TRY(band_gather(spectrum, chunks, frames, 4 * bins, zcols_.as<int>(),
                              zoffsets_.as<int>(), bands, total_width, ws_.z.as<float>(), s));
        GemmEpilogue e{};
        e.act = ANCHA_ACT_NONE;
        ANCHA_TRY(gemm_ffma(GemmGroup{}, ws_.split_groups.as<GemmGroup>(), G, frames, c.dim, 0, 0, 1,
                            e, s));
    }
    // Axial stack (network.rs:333-339).
    block_ss_ = nullptr;
    pending_scale_ = nullptr;
    for (auto& layer : layers_) {
        if (cancelled()) return fail(ANCHA_E_CANCELLED, "task cancelled");
        ANCHA_TRY(transformer(layer[0], true, s));
        ANCHA_TRY(transformer(layer[1], false, s));
    }
    float* x = ws_.x.as<float>();
    if (pending_scale_)  // the last block's SourceNorm, deferred by the row-norm fusion
        ANCHA_TRY(norm_rows(x, c.dim, pending_scale_, nullptr, 0, 0, R, c.dim, s));
    block_ss_ = nullptr;
    pending_scale_ = nullptr;
    if (final_scale_.p)  // BS final norm (network.rs:340-342)
        ANCHA_TRY(norm_rows(x, c.dim, final_scale_.as<float>(), nullptr, 0, 0, R, c.dim, s));
    // Mask estimators (network.rs:364-398): the input is x itself (f32) or its bf16 / f16 copy.
    if (elt_ != ELT_F32) ANCHA_TRY(cast_rows(x, c.dim, ws_.xn.p, elt_, c.dim, R, c.dim, s));
    const int hidden_layers = c.mel() ? c.mask_depth : c.mask_depth - 1;
    const int mh = c.dim * c.mask_expansion;
    const GemmGroup* groups = ws_.mask_groups.as<GemmGroup>();
    for (size_t st = 0; st < masks_.size(); ++st) {
        if (cancelled()) return fail(ANCHA_E_CANCELLED, "task cancelled");
        for (int l = 0; l <= hidden_layers; ++l) {
            const bool glu = l == hidden_layers;
            GemmEpilogue e{};
            e.act = glu ? ANCHA_ACT_GLU : ANCHA_ACT_TANH;
            e.out_type = glu ? ELT_F32 : elt_;
            int gst = ANCHA_E_UNSUPPORTED;
            const MaskWeights& mw = masks_[st];
            const auto wsplit = split_ ? split_w_.find(glu ? mw.glu_w.p : mw.w[l].p) : split_w_.end();
            if (elt_ != ELT_F32 || wsplit != split_w_.end()) {
                // One tcgen05 launch over every (chunk, band) problem of this layer; in fp32 mode
                // on the three-plane splits of the f32 input rows and of the weights.
                const int in = l == 0 ? c.dim : mh;
                const void* a = l == 0 ? (elt_ != ELT_F32 ? ws_.xn.p : ws_.x.p) : (l % 2 == 1 ? ws_.hidden.p : ws_.h2.p);
                GroupedGemm q{};
                if (elt_ == ELT_F32) {
                    ANCHA_TRY(split3_rows(static_cast<const float*>(a), in, ws_.a3.p, R, in, s));
                    a = ws_.a3.p;
                    q.split3 = true;
                }
                q.a = a;
                q.lda = in;
                q.a_group_stride = (int64_t)frames * in;
                q.m = frames;
                q.k = in;
                q.groups = G;
                q.b_groups = bands;
                if (glu) {
                    q.b = mw.glu_w.p;
                    q.n = 2 * max_width;
                    q.group_n = glu_n_.as<int>();
                    q.bias = mw.glu_b.as<float>();
                    q.out = ws_.glu.p;
                    q.ldo = max_width;
                } else {
                    q.b = mw.w[l].p;
                    q.n = mh;
                    q.group_n = nullptr;
                    q.bias = mw.b[l].as<float>();
                    q.out = l % 2 == 0 ? ws_.hidden.p : ws_.h2.p;
                    q.ldo = mh;
                }
                q.ldb = in;
                q.b_group_stride = (int64_t)q.n * in;
                q.bias_group_stride = q.n;
                q.out_group_stride = (int64_t)frames * q.ldo;
                if (q.split3) q.b = wsplit->second.p;
                gst = gemm_tc_grouped(q, q.split3 ? ELT_BF16 : elt_, e, s);
            }
            if (gst == ANCHA_E_UNSUPPORTED) {
                const GemmGroup* gl = groups + ((size_t)st * (hidden_layers + 1) + l) * (size_t)ws_.chunks * bands;
                gst = gemm_ffma(GemmGroup{}, gl, G, frames, glu ? 2 * max_width : mh, elt_, elt_, 1, e, s);
            }
            ANCHA_TRY(gst);
        }
        ANCHA_TRY(mask_assemble(ws_.glu.as<float>(), max_width, bands, frames, 2 * bins,
                                cover_count_.as<int>(), cover_entries_.as<int2>(), max_cover,
                                (int)masks_.size(), (int)st, masks, chunks, flag_.as<int>(), s));
    }
    if (!check) return ANCHA_OK;
    int flag = 0;
    ANCHA_TRY(read_flag(s, &flag));
    if (flag) return fail(ANCHA_E_NONFINITE, "non-finite model output");
    return ANCHA_OK;
}

}  // namespace ancha
