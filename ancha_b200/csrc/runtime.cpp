// Separation task on one or more GPUs: the chunk plan of src/runtime.rs:103-116, the whole
// per-chunk pipeline on the device (gather → STFT → model → complex mask + iSTFT → weighted
// overlap-add, runtime.rs:117-209), the border crop and one-stem residual (210-238), and
// the outputs (float32 WAVs + run.json, atomically published, runtime.rs:240-397).
//
// Multi-GPU: the chunk starts are split into contiguous ranges, one host thread and model per
// GPU. Each GPU overlap-adds its own chunks into a partial sum over its sample span; the
// spans are added on the host in device order (only the chunk-overlap halos meet), then
// divided by the summed weights. No collective runs on the compute path.
#include <cuda_runtime.h>
#include <dirent.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <chrono>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <thread>
#include <vector>

#include "dsp.cuh"
#include "model.hpp"

namespace ancha {
namespace {

using Clock = std::chrono::steady_clock;
double since(Clock::time_point t) {
    return std::chrono::duration<double>(Clock::now() - t).count();
}

struct TrackPlan {
    int64_t samples = 0, chunk = 0, step = 0, border = 0, length = 0;
    int overlap = 1;
    std::vector<int64_t> starts;
};

// runtime.rs:103-111 and chunk.rs:10-23.
TrackPlan make_plan(int64_t samples, int64_t chunk, int overlap) {
    if (chunk <= 0 || overlap <= 0 || overlap > chunk) throw std::runtime_error("invalid chunk or overlap divisor");
    if (chunk > kMaxChunkSamples || overlap > kMaxOverlap)
        throw std::runtime_error("chunk longer than 60 s or overlap divisor above 16");
    if (samples > kMaxTrackSamples) throw std::runtime_error("track longer than 2^36 samples");
    TrackPlan p;
    p.samples = samples;
    p.chunk = chunk;
    p.overlap = overlap;
    p.step = chunk / overlap;
    int64_t border = chunk - p.step;
    p.border = samples > 2 * border ? border : 0;
    p.length = samples + 2 * p.border;
    for (int64_t s = 0; s < p.length; s += p.step) p.starts.push_back(s);
    return p;
}

// Chunks per model call when the caller passes 0: balanced batches of at most 8 (21 chunks run as
// 3 × 7, 47 as 6 × 8). Bigger batches mean fewer tail waves in the GEMMs and no near-empty last
// batch; 8 Mel chunks take ~6 GB of activations.
int default_batch(size_t chunks) {
    const size_t batches = std::max<size_t>(1, (chunks + 7) / 8);
    return (int)std::max<size_t>(1, (chunks + batches - 1) / batches);
}

struct Partial {
    int64_t lo = 0, hi = 0;         // sample span [lo, hi) of the padded track
    std::vector<float> sums;        // [planes][hi - lo]
    std::vector<float> weights;     // [hi - lo]
    int status = ANCHA_OK;
    std::string error;
    double model_seconds = 0.0;
};

// Chunks [i0, i1) of `plan` on the model's device: device PCM planes [2][samples] → the
// weighted overlap-add of those chunks into the device span buffers sums [planes][span] /
// weights [span] that start at padded-track sample `lo`. Buffers are cached on the model.
int run_chunks(Model& model, const float* planes, const TrackPlan& plan, size_t i0, size_t i1,
               int batch, int64_t lo, int64_t span, float* sums, float* weights,
               const volatile int* cancel, cudaStream_t s, double* model_seconds) {
    const ModelConfig& c = model.manifest.config;
    const int stems = (int)c.stems.size();
    const int planes_n = stems * 2;
    const int64_t chunk = plan.chunk;
    const int frames = (int)(chunk / c.hop + 1);
    const int bins = c.n_fft / 2 + 1;
    PipelineBuffers& p = model.pipe;
    if (p.batch < batch || p.chunk != chunk) {
        try {
            p.audio.alloc((size_t)batch * 2 * chunk * 4);
            p.packed.alloc((size_t)batch * frames * bins * 4 * 4);
            p.masks.alloc((size_t)batch * stems * 2 * bins * 2 * frames * 4);
            p.scratch.alloc((size_t)batch * stems * 2 * frames * 2048 * 4);
            p.y.alloc((size_t)batch * planes_n * chunk * 4);
            p.flag.alloc(16);
            p.batch = batch;
            p.chunk = chunk;
        } catch (const std::exception& e) {
            p.batch = 0;
            return fail(ANCHA_E_CUDA, std::string("pipeline buffers: ") + e.what());
        }
    }
    ANCHA_CUDA(cudaMemsetAsync(p.flag.p, 0, 16, s));
    ANCHA_TRY(model.reset_flag(s));
    for (size_t b0 = i0; b0 < i1; b0 += batch) {
        if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
        const int nb = (int)std::min<size_t>(batch, i1 - b0);
        ChunkStarts cs{};
        for (int k = 0; k < nb; ++k) cs.v[k] = plan.starts[b0 + k];
        ANCHA_TRY(gather_chunks(planes, plan.samples, cs, nb, (int)chunk, plan.border, plan.length,
                                p.audio.as<float>(), s));
        ANCHA_TRY(stft_forward(p.audio.as<float>(), nb, (int)chunk, c.hop, p.packed.as<float>(), s));
        auto t0 = Clock::now();
        ANCHA_TRY(model.forward(p.packed.as<float>(), nb, frames, p.masks.as<float>(), cancel, s, false));
        if (model_seconds) *model_seconds += since(t0);
        ANCHA_TRY(istft_masked(p.packed.as<float>(), p.masks.as<float>(), nb, stems, (int)chunk, c.hop,
                               c.zero_dc, p.scratch.as<float>(), p.y.as<float>(), p.flag.as<int>(), s));
        ANCHA_TRY(ola_add(p.y.as<float>(), nb, planes_n, (int)chunk, cs, plan.length, lo, span, sums,
                          weights, s));
    }
    return ANCHA_OK;
}

// Read the deferred status words of a pipeline run (synchronises the stream).
int pipeline_status(Model& model, cudaStream_t s) {
    int flag = 0, mflag = 0;
    ANCHA_CUDA(cudaMemcpyAsync(&flag, model.pipe.flag.p, 4, cudaMemcpyDeviceToHost, s));
    ANCHA_TRY(model.read_flag(s, &mflag));
    if (mflag) return fail(ANCHA_E_NONFINITE, "non-finite model output");
    if (flag) return fail(ANCHA_E_NONFINITE, "iSTFT has an uncovered sample");
    return ANCHA_OK;
}

// Run chunk starts [i0, i1) of `plan` on `model`'s device from host PCM; leaves the partial
// overlap-add of those chunks in `out` (host).
void run_device(Model& model, const float* planes, const TrackPlan& plan, size_t i0, size_t i1,
                int batch, const volatile int* cancel, Partial& out) {
    if (i0 >= i1) return;
    if (cudaSetDevice(model.device) != cudaSuccess) { out.status = ANCHA_E_CUDA; out.error = "cudaSetDevice"; return; }
    cudaStream_t s;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        out.status = ANCHA_E_CUDA; out.error = "cudaStreamCreate"; return;
    }
    const int planes_n = (int)model.manifest.config.stems.size() * 2;
    out.lo = plan.starts[i0];
    out.hi = std::min(plan.starts[i1 - 1] + plan.chunk, plan.length);
    const int64_t span = out.hi - out.lo;
    int st = ANCHA_OK;
    try {
        // Device copies of the track and the span accumulators are cached on the model (grown
        // as needed): a per-call cudaMalloc / cudaFree pair would synchronise the device.
        PipelineBuffers& pb = model.pipe;
        if (pb.pcm.bytes < (size_t)(2 * plan.samples * 4)) pb.pcm.alloc(2 * plan.samples * 4);
        if (pb.span.bytes < (size_t)(planes_n + 1) * span * 4) pb.span.alloc((size_t)(planes_n + 1) * span * 4);
        float* d_planes = pb.pcm.as<float>();
        float* d_sums = pb.span.as<float>();
        float* d_weights = d_sums + (size_t)planes_n * span;
        st = cudaMemcpyAsync(d_planes, planes, 2 * plan.samples * 4, cudaMemcpyHostToDevice, s) == cudaSuccess
                 ? ANCHA_OK : fail(ANCHA_E_CUDA, "upload PCM");
        if (!st) st = cudaMemsetAsync(d_sums, 0, (size_t)(planes_n + 1) * span * 4, s) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "memset");
        if (!st) st = run_chunks(model, d_planes, plan, i0, i1, batch, out.lo, span, d_sums, d_weights, cancel, s,
                                 &out.model_seconds);
        if (!st) {
            out.sums.resize((size_t)planes_n * span);
            out.weights.resize((size_t)span);
            cudaMemcpyAsync(out.sums.data(), d_sums, out.sums.size() * 4, cudaMemcpyDeviceToHost, s);
            cudaMemcpyAsync(out.weights.data(), d_weights, out.weights.size() * 4, cudaMemcpyDeviceToHost, s);
            st = pipeline_status(model, s);
        }
        cudaError_t e = cudaStreamSynchronize(s);
        if (!st && e != cudaSuccess) st = cuda_fail(e, "separate");
    } catch (const std::exception& ex) {
        st = fail(ANCHA_E_CUDA, ex.what());
    }
    if (st) { out.status = st; out.error = ancha_last_error(); }
    cudaStreamDestroy(s);
}

struct PcmResult {
    int status = ANCHA_OK;
    double model_seconds = 0.0;
    size_t chunks = 0;
};

// One device, the whole track: overlap-add, division and crop stay on the device and the
// stems are copied once into the caller's buffer (no host-side span merge).
PcmResult separate_single(Model& model, const float* planes, const TrackPlan& plan, int batch,
                          const volatile int* cancel, float* stems_out) {
    PcmResult r;
    r.chunks = plan.starts.size();
    const int64_t samples = plan.samples;
    const int planes_n = (int)model.manifest.config.stems.size() * 2;
    if (cudaSetDevice(model.device) != cudaSuccess) { r.status = fail(ANCHA_E_CUDA, "cudaSetDevice"); return r; }
    cudaStream_t s;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) {
        r.status = fail(ANCHA_E_CUDA, "cudaStreamCreate");
        return r;
    }
    int st = ANCHA_OK;
    try {
        PipelineBuffers& pb = model.pipe;
        const size_t acc = (size_t)(planes_n + 1) * plan.length;
        if (pb.pcm.bytes < (size_t)(2 * samples * 4)) pb.pcm.alloc(2 * samples * 4);
        if (pb.span.bytes < acc * 4) pb.span.alloc(acc * 4);
        if (pb.stems.bytes < (size_t)planes_n * samples * 4) pb.stems.alloc((size_t)planes_n * samples * 4);
        float* d_planes = pb.pcm.as<float>();
        float* d_sums = pb.span.as<float>();
        float* d_weights = d_sums + (size_t)planes_n * plan.length;
        st = cudaMemcpyAsync(d_planes, planes, 2 * samples * 4, cudaMemcpyHostToDevice, s) == cudaSuccess
                 ? ANCHA_OK : fail(ANCHA_E_CUDA, "upload PCM");
        if (!st) st = cudaMemsetAsync(d_sums, 0, acc * 4, s) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "memset");
        if (!st) st = run_chunks(model, d_planes, plan, 0, plan.starts.size(), batch, 0, plan.length, d_sums,
                                 d_weights, cancel, s, &r.model_seconds);
        if (!st) st = ola_finish(d_sums, d_weights, planes_n, plan.length, plan.border, samples, nullptr,
                                 pb.stems.as<float>(), nullptr, pb.flag.as<int>() + 1, s);
        if (!st) st = cudaMemcpyAsync(stems_out, pb.stems.p, (size_t)planes_n * samples * 4, cudaMemcpyDeviceToHost,
                                      s) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "download stems");
        int flags[2] = {0, 0};
        if (!st) st = cudaMemcpyAsync(flags, pb.flag.p, 8, cudaMemcpyDeviceToHost, s) == cudaSuccess
                          ? ANCHA_OK : fail(ANCHA_E_CUDA, "read status");
        int mflag = 0;
        if (!st) st = model.read_flag(s, &mflag);  // synchronises the stream
        if (!st && (mflag || (flags[1] & 1))) st = fail(ANCHA_E_NONFINITE, "non-finite chunk output");
        if (!st && (flags[0] || (flags[1] & 4))) st = fail(ANCHA_E_INVALID, "uncovered overlap-add sample");
        cudaError_t e = cudaStreamSynchronize(s);
        if (!st && e != cudaSuccess) st = cuda_fail(e, "separate");
    } catch (const std::exception& ex) {
        st = fail(ANCHA_E_CUDA, ex.what());
    }
    cudaStreamDestroy(s);
    r.status = st;
    return r;
}

// Stems [stems][2][samples] of host planes [2][samples] on the given models (one per GPU).
PcmResult separate_pcm(Model* const* models, int n, const float* planes, int64_t samples,
                       int64_t chunk, int overlap, int batch, const volatile int* cancel,
                       float* stems_out) {
    PcmResult r;
    if (n <= 0 || !models[0]) { r.status = fail(ANCHA_E_INVALID, "separate: no model"); return r; }
    if (samples <= 0) { r.status = fail(ANCHA_E_INVALID, "audio is empty"); return r; }
    const ModelConfig& c = models[0]->manifest.config;
    for (int d = 1; d < n; ++d)
        if (models[d]->manifest.weights_sha256 != models[0]->manifest.weights_sha256) {
            r.status = fail(ANCHA_E_INVALID, "separate: devices hold different models");
            return r;
        }
    if (chunk <= c.n_fft / 2) { r.status = fail(ANCHA_E_INVALID, "invalid chunk settings"); return r; }
    TrackPlan plan;
    try {
        plan = make_plan(samples, chunk, overlap);
    } catch (const std::exception& e) {
        r.status = fail(ANCHA_E_INVALID, e.what());
        return r;
    }
    r.chunks = plan.starts.size();
    if (batch <= 0) batch = default_batch((plan.starts.size() + n - 1) / n);
    batch = std::min(batch, kMaxChunksPerCall);
    if (n == 1) return separate_single(*models[0], planes, plan, batch, cancel, stems_out);
    const int stems = (int)c.stems.size();
    const int planes_n = stems * 2;
    // Contiguous ranges of chunk starts, ceil(chunks / n) per device.
    const size_t per = (plan.starts.size() + n - 1) / n;
    std::vector<Partial> parts(n);
    std::vector<std::thread> workers;
    for (int d = 0; d < n; ++d) {
        const size_t i0 = std::min(plan.starts.size(), d * per);
        const size_t i1 = std::min(plan.starts.size(), (d + 1) * per);
        workers.emplace_back([&, d, i0, i1] {
            run_device(*models[d], planes, plan, i0, i1, batch, cancel, parts[d]);
        });
    }
    for (auto& w : workers) w.join();
    for (auto& p : parts) {
        r.model_seconds = std::max(r.model_seconds, p.model_seconds);
        if (p.status != ANCHA_OK) {
            r.status = fail(p.status, p.error);
            return r;
        }
    }
    // Add the partial spans in device order, then divide and crop (chunk.rs:77-88,
    // runtime.rs:210-225).
    std::vector<float> sums((size_t)planes_n * plan.length, 0.f), weights((size_t)plan.length, 0.f);
    for (auto& p : parts) {
        const int64_t span = p.hi - p.lo;
        if (span <= 0) continue;
        for (int64_t j = 0; j < span; ++j) weights[p.lo + j] += p.weights[j];
        for (int q = 0; q < planes_n; ++q)
            for (int64_t j = 0; j < span; ++j)
                sums[(size_t)q * plan.length + p.lo + j] += p.sums[(size_t)q * span + j];
    }
    for (int64_t j = 0; j < plan.length; ++j)
        if (!(weights[j] > 0.f)) { r.status = fail(ANCHA_E_INVALID, "uncovered overlap-add sample"); return r; }
    for (int q = 0; q < planes_n; ++q)
        for (int64_t i = 0; i < samples; ++i) {
            const float v = sums[(size_t)q * plan.length + plan.border + i] / weights[plan.border + i];
            if (!std::isfinite(v)) { r.status = fail(ANCHA_E_NONFINITE, "non-finite chunk output"); return r; }
            stems_out[(size_t)q * samples + i] = v;
        }
    return r;
}

std::string output_stem(const std::string& name) {  // report.rs:24-30
    if (name == "vocals" || name == "lead_vocals" || name == "all_vocals") return "vocals";
    if (name == "instrumental" || name == "instrument" || name == "karaoke_mix") return "instrument";
    return name;
}

bool exists(const std::string& p) {
    struct stat st;
    return ::stat(p.c_str(), &st) == 0;
}

void remove_tree(const std::string& path) {
    DIR* d = opendir(path.c_str());
    if (d) {
        while (dirent* e = readdir(d)) {
            std::string n = e->d_name;
            if (n == "." || n == "..") continue;
            std::string full = path + "/" + n;
            struct stat st;
            if (lstat(full.c_str(), &st) == 0 && S_ISDIR(st.st_mode)) remove_tree(full);
            else ::unlink(full.c_str());
        }
        closedir(d);
    }
    ::rmdir(path.c_str());
}

std::string parent_of(const std::string& p) {
    std::string s = p;
    while (s.size() > 1 && s.back() == '/') s.pop_back();
    const size_t k = s.rfind('/');
    if (k == std::string::npos) return ".";
    return k == 0 ? "/" : s.substr(0, k);
}

std::string base_of(const std::string& p) {
    std::string s = p;
    while (s.size() > 1 && s.back() == '/') s.pop_back();
    const size_t k = s.rfind('/');
    return k == std::string::npos ? s : s.substr(k + 1);
}

void make_dirs(const std::string& p) {
    if (p.empty() || exists(p)) return;
    make_dirs(parent_of(p));
    ::mkdir(p.c_str(), 0755);
}

std::string make_temp_dir(const std::string& parent, const std::string& prefix) {
    std::string tmpl = parent + "/" + prefix + "XXXXXX";
    std::vector<char> buf(tmpl.begin(), tmpl.end());
    buf.push_back(0);
    if (!mkdtemp(buf.data())) throw std::runtime_error("create staging directory in " + parent);
    return std::string(buf.data());
}

// Move a finished staging directory onto `dest`, replacing a previous result and restoring
// it if the replacement fails (runtime.rs:367-397).
void publish_directory(const std::string& stage, const std::string& dest) {
    if (!exists(dest)) {
        if (::rename(stage.c_str(), dest.c_str()) != 0) throw std::runtime_error("publish separation outputs");
        return;
    }
    const std::string backup = make_temp_dir(parent_of(dest), "." + base_of(dest) + ".previous-");
    const std::string previous = backup + "/result";
    if (::rename(dest.c_str(), previous.c_str()) != 0) {
        remove_tree(backup);
        throw std::runtime_error("move previous output aside");
    }
    if (::rename(stage.c_str(), dest.c_str()) != 0) {
        if (::rename(previous.c_str(), dest.c_str()) != 0)
            throw std::runtime_error("publish separation outputs; restoring previous output failed; backup retained at " + backup);
        remove_tree(backup);
        throw std::runtime_error("publish separation outputs");
    }
    remove_tree(backup);
}

// The reference's AttentionPlan::worker_tiles with the CUDA defaults (roformer.rs:96-130,
// backend.rs:52-67), reported in run.json for schema compatibility.
std::pair<int64_t, int64_t> tiles(int64_t groups, int64_t tokens, int64_t heads) {
    const int64_t budget = 512ll << 20, row = heads * tokens * 4;
    const int64_t query = std::min(std::max<int64_t>(budget / row, 1), tokens);
    const int64_t group = std::min(std::max<int64_t>(budget / (row * query), 1), groups);
    return {group, query};
}

}  // namespace
}  // namespace ancha

using namespace ancha;

extern "C" int ancha_separate_pcm(ancha_model* const* models, int n_models, const float* planes,
                                  int64_t samples, int64_t chunk_samples, int overlap,
                                  int batch_chunks, const volatile int* cancel, float* stems_out,
                                  double* seconds_out) {
    if (!models || n_models <= 0 || !planes || !stems_out) return fail(ANCHA_E_INVALID, "separate_pcm: null argument");
    std::vector<Model*> ms;
    for (int i = 0; i < n_models; ++i) {
        if (!models[i]) return fail(ANCHA_E_INVALID, "separate_pcm: null model");
        ms.push_back(models[i]->impl.get());
    }
    const ModelConfig& c = ms[0]->manifest.config;
    const auto t0 = Clock::now();
    PcmResult r = separate_pcm(ms.data(), n_models, planes, samples,
                               chunk_samples > 0 ? chunk_samples : c.chunk_samples,
                               overlap > 0 ? overlap : c.overlap, batch_chunks, cancel, stems_out);
    if (seconds_out) *seconds_out = since(t0);
    return r.status;
}

extern "C" int ancha_chunk_plan(int64_t samples, int64_t chunk_samples, int overlap, int64_t* chunks,
                                int64_t* border, int64_t* length) {
    if (samples <= 0) return fail(ANCHA_E_INVALID, "audio is empty");
    try {
        const TrackPlan plan = make_plan(samples, chunk_samples, overlap);
        if (chunks) *chunks = (int64_t)plan.starts.size();
        if (border) *border = plan.border;
        if (length) *length = plan.length;
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    return ANCHA_OK;
}

extern "C" int ancha_chunk_span(int64_t samples, int64_t chunk_samples, int overlap, int64_t first,
                                int64_t last, int64_t* lo, int64_t* hi) {
    if (samples <= 0 || !lo || !hi) return fail(ANCHA_E_INVALID, "chunk_span: invalid arguments");
    try {
        const TrackPlan plan = make_plan(samples, chunk_samples, overlap);
        const int64_t n = (int64_t)plan.starts.size();
        if (first < 0 || last > n || first > last) return fail(ANCHA_E_INVALID, "chunk_span: chunk range outside the plan");
        if (first == last) {
            *lo = *hi = 0;
        } else {
            *lo = plan.starts[first];
            *hi = std::min(plan.starts[last - 1] + plan.chunk, plan.length);
        }
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    return ANCHA_OK;
}

extern "C" int ancha_separate_span(ancha_model* model, const float* planes, int64_t samples,
                                   int64_t chunk_samples, int overlap, int batch_chunks, int64_t first,
                                   int64_t last, const volatile int* cancel, float* sums, float* weights) {
    if (!model || !planes || !sums || !weights) return fail(ANCHA_E_INVALID, "separate_span: null argument");
    Model& m = *model->impl;
    const ModelConfig& c = m.manifest.config;
    TrackPlan plan;
    try {
        plan = make_plan(samples, chunk_samples > 0 ? chunk_samples : c.chunk_samples,
                         overlap > 0 ? overlap : c.overlap);
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    if (samples <= 0 || plan.chunk <= c.n_fft / 2) return fail(ANCHA_E_INVALID, "invalid chunk settings");
    if (first < 0 || last > (int64_t)plan.starts.size() || first > last)
        return fail(ANCHA_E_INVALID, "separate_span: chunk range outside the plan");
    if (first == last) return ANCHA_OK;
    int batch = batch_chunks > 0 ? std::min(batch_chunks, kMaxChunksPerCall) : default_batch((size_t)(last - first));
    Partial part;
    run_device(m, planes, plan, (size_t)first, (size_t)last, batch, cancel, part);
    if (part.status != ANCHA_OK) return fail(part.status, part.error);
    std::copy(part.sums.begin(), part.sums.end(), sums);
    std::copy(part.weights.begin(), part.weights.end(), weights);
    return ANCHA_OK;
}

extern "C" int ancha_separate_device(ancha_model* model, const float* planes, int64_t samples,
                                     int64_t chunk_samples, int overlap, int batch_chunks,
                                     float* stems, void* stream) {
    if (!model || !planes || !stems) return fail(ANCHA_E_INVALID, "separate_device: null argument");
    Model& m = *model->impl;
    const ModelConfig& c = m.manifest.config;
    TrackPlan plan;
    try {
        plan = make_plan(samples, chunk_samples > 0 ? chunk_samples : c.chunk_samples,
                         overlap > 0 ? overlap : c.overlap);
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    if (samples <= 0 || plan.chunk <= c.n_fft / 2) return fail(ANCHA_E_INVALID, "invalid chunk settings");
    int batch = batch_chunks > 0 ? std::min(batch_chunks, kMaxChunksPerCall) : default_batch(plan.starts.size());
    cudaStream_t s = as_stream(stream);
    ANCHA_CUDA(cudaSetDevice(m.device));
    const int planes_n = (int)c.stems.size() * 2;
    PipelineBuffers& p = m.pipe;
    if ((int64_t)(p.acc.bytes / 4) < (planes_n + 1) * plan.length) {
        try {
            p.acc.alloc((size_t)(planes_n + 1) * plan.length * 4);
        } catch (const std::exception& e) {
            return fail(ANCHA_E_CUDA, e.what());
        }
    }
    float* sums = p.acc.as<float>();
    float* weights = sums + (size_t)planes_n * plan.length;
    ANCHA_CUDA(cudaMemsetAsync(sums, 0, (size_t)(planes_n + 1) * plan.length * 4, s));
    ANCHA_TRY(run_chunks(m, planes, plan, 0, plan.starts.size(), batch, 0, plan.length, sums, weights,
                         nullptr, s, nullptr));
    ANCHA_TRY(ola_finish(sums, weights, planes_n, plan.length, plan.border, samples, nullptr, stems,
                         nullptr, p.flag.as<int>() + 1, s));
    return ANCHA_OK;
}

extern "C" int ancha_separate_status(ancha_model* model, void* stream) {
    if (!model) return fail(ANCHA_E_INVALID, "separate_status: null model");
    Model& m = *model->impl;
    ANCHA_CUDA(cudaSetDevice(m.device));
    cudaStream_t s = as_stream(stream);
    int flags[2] = {0, 0};
    ANCHA_CUDA(cudaMemcpyAsync(flags, m.pipe.flag.p, 8, cudaMemcpyDeviceToHost, s));
    int mflag = 0;
    ANCHA_TRY(m.read_flag(s, &mflag));
    if (mflag || (flags[1] & 1)) return fail(ANCHA_E_NONFINITE, "non-finite model output");
    if (flags[0] || (flags[1] & 4)) return fail(ANCHA_E_INVALID, "uncovered sample");
    return ANCHA_OK;
}

extern "C" int ancha_separate(const ancha_separate_opts* o, int n_devices, const int* devices,
                              void (*progress)(size_t, size_t, void*), void* user,
                              const volatile int* cancel, char** run_json) {
    if (!o || !o->input || !o->model || !o->output || n_devices <= 0 || !devices)
        return fail(ANCHA_E_INVALID, "separate: null argument");
    if (run_json) *run_json = nullptr;
    const auto total_start = Clock::now();
    if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
    try {
        Json timings = Json::make_object();
        // Decode (WAV only; the synthetic inputs are 44.1 kHz) and the decode window.
        auto t = Clock::now();
        Audio audio = read_wav(o->input);
        if (audio.planes.size() == 1) audio.planes.push_back(audio.planes[0]);
        const double decode_s = since(t);
        for (auto& p : audio.planes)
            for (float v : p)
                if (!std::isfinite(v)) return fail(ANCHA_E_INVALID, "non-finite PCM");
        const int64_t first = (int64_t)std::llround(std::max(0.0, o->start_seconds) * audio.sample_rate);
        if (first >= audio.samples()) return fail(ANCHA_E_INVALID, "start is past the end of the input");
        int64_t count = audio.samples() - first;
        if (o->duration_seconds > 0) count = std::min<int64_t>(count, (int64_t)std::llround(o->duration_seconds * audio.sample_rate));
        for (auto& p : audio.planes) p = std::vector<float>(p.begin() + first, p.begin() + first + count);
        // Models, one per device (weights verified and folded per device).
        t = Clock::now();
        std::vector<std::unique_ptr<Model>> models;
        for (int d = 0; d < n_devices; ++d) models.push_back(Model::load(o->model, devices[d], o->precision));
        Manifest& m = models[0]->manifest;
        const bool custom = o->chunk_samples > 0 || o->overlap > 0;
        ModelConfig& c = m.config;
        if (o->chunk_samples > 0) c.chunk_samples = o->chunk_samples;
        if (o->overlap > 0) c.overlap = o->overlap;
        m.validate();
        if (audio.sample_rate != c.sample_rate)
            return fail(ANCHA_E_UNSUPPORTED, "input sample rate " + std::to_string(audio.sample_rate) +
                                                 " Hz needs resampling to 44100 Hz, which this build does not do");
        for (auto& mm : models) mm->manifest.config = c;
        const double load_s = since(t);
        const int64_t samples = audio.samples();
        std::vector<float> planes(2 * samples);
        for (int ch = 0; ch < 2; ++ch) std::memcpy(&planes[ch * samples], audio.planes[ch].data(), samples * 4);
        const std::string pcm_sha = sha256_hex(reinterpret_cast<const uint8_t*>(planes.data()), planes.size() * 4);
        const int stems = (int)c.stems.size();
        std::vector<float> out((size_t)stems * 2 * samples);
        std::vector<Model*> ms;
        for (auto& mm : models) ms.push_back(mm.get());
        if (progress) progress(0, make_plan(samples, c.chunk_samples, c.overlap).starts.size(), user);
        t = Clock::now();
        PcmResult r = separate_pcm(ms.data(), n_devices, planes.data(), samples, c.chunk_samples,
                                   c.overlap, o->batch_chunks, cancel, out.data());
        const double sep_s = since(t);
        if (r.status != ANCHA_OK) return r.status;
        if (progress) progress(r.chunks, r.chunks, user);
        // Stems, then the one-stem residual (runtime.rs:226-238).
        struct Stem { std::string name, origin; Audio audio; };
        std::vector<Stem> outs;
        for (int s = 0; s < stems; ++s) {
            Stem st{c.stems[s], "predicted", Audio{}};
            st.audio.sample_rate = c.sample_rate;
            for (int ch = 0; ch < 2; ++ch)
                st.audio.planes.emplace_back(out.begin() + ((size_t)s * 2 + ch) * samples,
                                             out.begin() + ((size_t)s * 2 + ch + 1) * samples);
            outs.push_back(std::move(st));
        }
        Json recon;  // null unless one stem
        if (stems == 1) {
            const std::string n0 = c.stems[0];
            Stem res{n0 == "vocals" ? "instrumental" : n0 == "lead_vocals" ? "karaoke_mix" : "vocals",
                     "residual", Audio{}};
            res.audio.sample_rate = c.sample_rate;
            float err = 0.f;
            for (int ch = 0; ch < 2; ++ch) {
                std::vector<float> p(samples);
                for (int64_t i = 0; i < samples; ++i) {
                    p[i] = audio.planes[ch][i] - outs[0].audio.planes[ch][i];
                    err = std::max(err, std::fabs(audio.planes[ch][i] - (outs[0].audio.planes[ch][i] + p[i])));
                }
                res.audio.planes.push_back(std::move(p));
            }
            outs.push_back(std::move(res));
            recon = Json::of(err);
        }
        if (cancel && *cancel) return fail(ANCHA_E_CANCELLED, "task cancelled");
        const std::string dest = o->output;
        const std::string parent = parent_of(dest);
        make_dirs(parent);
        const std::string stage = make_temp_dir(parent, ".ancha-output-");
        t = Clock::now();
        Json stem_reports = Json::make_array();
        try {
            for (auto& st : outs) {
                const std::string name = output_stem(st.name);
                write_wav(stage + "/" + name + ".wav", st.audio);
                float peak = 0.f;
                double ss = 0.0;
                for (auto& p : st.audio.planes)
                    for (float v : p) { peak = std::max(peak, std::fabs(v)); ss += (double)v * v; }
                Json sr = Json::make_object();
                sr.set("name", Json::of(name));
                sr.set("origin", Json::of(st.origin));
                sr.set("peak", Json::of(peak));
                sr.set("rms", Json::of(std::sqrt(ss / (2.0 * samples))));
                stem_reports.arr.push_back(sr);
            }
        } catch (...) {
            remove_tree(stage);
            throw;
        }
        const double write_s = since(t);
        const double total_s = since(total_start);
        const double audio_s = (double)samples / c.sample_rate;
        const int frames = (int)(c.chunk_samples / c.hop + 1);
        auto tt = tiles((int64_t)c.bands.size(), frames, c.heads);
        auto ft = tiles(frames, (int64_t)c.bands.size(), c.heads);
        timings.set("model_load_seconds", Json::of(load_s));
        timings.set("decode_seconds", Json::of(decode_s));
        timings.set("resample_seconds", Json::of(0.0));
        timings.set("stft_seconds", Json::of(0.0));
        timings.set("model_seconds", Json::of(r.model_seconds));
        timings.set("istft_seconds", Json::of(0.0));
        timings.set("overlap_seconds", Json::of(0.0));
        timings.set("separate_seconds", Json::of(sep_s));
        timings.set("write_seconds", Json::of(write_s));
        timings.set("total_seconds", Json::of(total_s));
        timings.set("model_call_seconds", Json::make_array());
        Json rep = Json::make_object();
        rep.set("schema_version", Json::of(1));
        rep.set("ancha_version", Json::of(std::string(ancha_version())));
        rep.set("platform", Json::of(std::string("linux-x86_64")));
        rep.set("backend", Json::of(std::string("cuda")));
        rep.set("device", Json::of(models[0]->device_name));
        rep.set("gpus", Json::of(n_devices));
        rep.set("precision", Json::of(std::string(o->precision == ANCHA_PRECISION_BF16 ? "bf16"
                                                   : o->precision == ANCHA_PRECISION_F16 ? "f16" : "f32")));
        rep.set("dsp_backend", Json::of(std::string("cuda")));
        rep.set("model_id", Json::of(m.model_id));
        rep.set("weights_sha256", Json::of(m.weights_sha256));
        rep.set("input_path", Json::of(std::string(o->input)));
        rep.set("input_pcm_sha256", Json::of(pcm_sha));
        rep.set("start_seconds", Json::of(o->start_seconds));
        rep.set("duration_requested_seconds", o->duration_seconds > 0 ? Json::of(o->duration_seconds) : Json());
        rep.set("audio_seconds", Json::of(audio_s));
        rep.set("sample_rate", Json::of(c.sample_rate));
        rep.set("samples_per_channel", Json::of((double)samples));
        rep.set("channels", Json::of(2));
        rep.set("tensor_count", Json::of((double)models[0]->tensor_count));
        rep.set("chunks", Json::of((double)r.chunks));
        rep.set("profile", Json::of(std::string(custom ? "custom-context" : "native-context")));
        rep.set("effective_config", c.to_json());
        rep.set("query_tile", Json::of((double)tt.second));
        rep.set("group_tile", Json::of((double)tt.first));
        rep.set("frequency_query_tile", Json::of((double)ft.second));
        rep.set("frequency_group_tile", Json::of((double)ft.first));
        rep.set("attention_tiling", Json::of(std::string("auto")));
        rep.set("host_threads", Json::of(1));
        rep.set("linear_layout", Json::of(std::string("flattened")));
        rep.set("attention_kernel", Json::of(std::string("fused")));
        rep.set("gemm_kernel", Json::of(std::string("custom")));
        Json feats = Json::make_array();
        feats.arr.push_back(Json::of(std::string("cuda")));
        rep.set("build_features", feats);
        rep.set("cpu_thread_environment", Json::make_object());
        rep.set("estimated_time_attention_score_bytes", Json::of(0));
        rep.set("estimated_frequency_attention_score_bytes", Json::of(0));
        rep.set("residual_reconstruction_max_abs", recon);
        rep.set("stems", stem_reports);
        rep.set("timings", timings);
        rep.set("rtf", Json::of(total_s / audio_s));
        rep.set("xrealtime", Json::of(audio_s / sep_s));
        const std::string text = rep.dump(2);
        {
            FILE* f = std::fopen((stage + "/run.json").c_str(), "wb");
            if (!f) { remove_tree(stage); return fail(ANCHA_E_IO, "write run.json"); }
            std::fwrite(text.data(), 1, text.size(), f);
            std::fclose(f);
        }
        try {
            publish_directory(stage, dest);
        } catch (...) {
            remove_tree(stage);
            throw;
        }
        if (run_json) {
            *run_json = static_cast<char*>(std::malloc(text.size() + 1));
            std::memcpy(*run_json, text.c_str(), text.size() + 1);
        }
        return ANCHA_OK;
    } catch (const std::exception& e) {
        const std::string msg = e.what();
        return fail(msg.rfind("read ", 0) == 0 ? ANCHA_E_IO : ANCHA_E_INVALID, msg);
    }
}
