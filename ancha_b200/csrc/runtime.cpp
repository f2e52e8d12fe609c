// Separation task on one or more GPUs: the chunk plan of src/runtime.rs:103-116, the whole
// per-chunk pipeline on the device (gather → STFT → model → complex mask + iSTFT → weighted
// overlap-add, runtime.rs:117-209), the border crop and one-stem residual (210-238), and
// the outputs (float32 WAVs + run.json, atomically published, runtime.rs:240-397).
//
// Multi-GPU: the chunk starts are split into contiguous ranges, one host thread and model per
// GPU. Each GPU uploads only the track samples its chunks read and overlap-adds its chunks into
// a partial sum over its sample span, which stays on that GPU. GPU d owns the output samples
// from the start of its span to the start of the next GPU's span; the columns of its span past
// that point (the chunk-overlap halo, at most chunk − step samples) are peer-copied to the GPUs
// that own them and added there. Each GPU then divides and crops its owned range on the device
// and copies it into the caller's stems. No collective runs on the compute path.
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

// Track samples [*lo, *hi) read by the reflect-padded chunk gather for padded samples [p0, p1)
// (p0 < p1): the padded sample p reads track sample reflect(p − border), which is monotone on
// each fold interval [k·(samples − 1), (k + 1)·(samples − 1)].
void pcm_range(const TrackPlan& plan, int64_t p0, int64_t p1, int64_t* lo, int64_t* hi) {
    const int64_t n = plan.samples;
    if (n <= 1) {
        *lo = 0;
        *hi = n;
        return;
    }
    const int64_t n1 = n - 1, period = 2 * n1;
    auto reflect = [&](int64_t i) {
        int64_t r = i % period;
        if (r < 0) r += period;
        return r < n ? r : period - r;
    };
    const int64_t a = p0 - plan.border, b = p1 - plan.border - 1;  // inclusive
    int64_t mn = n, mx = -1;
    int64_t k = a >= 0 ? a / n1 : -((-a + n1 - 1) / n1);
    for (; k * n1 <= b; ++k) {
        const int64_t q0 = std::max(a, k * n1), q1 = std::min(b, (k + 1) * n1);
        if (q0 > q1) continue;
        const int64_t r0 = reflect(q0), r1 = reflect(q1);
        mn = std::min(mn, std::min(r0, r1));
        mx = std::max(mx, std::max(r0, r1));
        if (mn == 0 && mx == n - 1) break;
    }
    *lo = mn;
    *hi = mx + 1;
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

// Chunks [i0, i1) of `plan` on the model's device: device PCM planes [2][pcm_len] holding track
// samples [pcm_lo, pcm_lo + pcm_len) → the weighted overlap-add of those chunks into the device
// span buffers sums [planes][span] / weights [span] that start at padded-track sample `lo`.
// Buffers are cached on the model.
int run_chunks(Model& model, const float* planes, int64_t pcm_lo, int64_t pcm_len, const TrackPlan& plan,
               size_t i0, size_t i1, int batch, int64_t lo, int64_t span, float* sums, float* weights,
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
        ANCHA_TRY(gather_chunks(planes, plan.samples, pcm_lo, pcm_len, cs, nb, (int)chunk, plan.border, plan.length,
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
        int64_t pcm_lo = 0, pcm_hi = 0;
        pcm_range(plan, out.lo, out.hi, &pcm_lo, &pcm_hi);
        const int64_t pcm_len = pcm_hi - pcm_lo;
        if (pb.pcm.bytes < (size_t)(2 * pcm_len * 4)) pb.pcm.alloc(2 * pcm_len * 4);
        if (pb.span.bytes < (size_t)(planes_n + 1) * span * 4) pb.span.alloc((size_t)(planes_n + 1) * span * 4);
        float* d_planes = pb.pcm.as<float>();
        float* d_sums = pb.span.as<float>();
        float* d_weights = d_sums + (size_t)planes_n * span;
        for (int ch = 0; ch < 2 && !st; ++ch)
            st = cudaMemcpyAsync(d_planes + ch * pcm_len, planes + ch * plan.samples + pcm_lo, pcm_len * 4,
                                 cudaMemcpyHostToDevice, s) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "upload PCM");
        if (!st) st = cudaMemsetAsync(d_sums, 0, (size_t)(planes_n + 1) * span * 4, s) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "memset");
        if (!st) st = run_chunks(model, d_planes, pcm_lo, pcm_len, plan, i0, i1, batch, out.lo, span, d_sums,
                                 d_weights, cancel, s, &out.model_seconds);
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
        if (!st) st = run_chunks(model, d_planes, 0, samples, plan, 0, plan.starts.size(), batch, 0, plan.length,
                                 d_sums, d_weights, cancel, s, &r.model_seconds);
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

// One shard of a multi-GPU separation: chunks [i0, i1) on one GPU, the padded span [lo, hi) they
// cover, and the padded samples [own_lo, own_hi) whose output this GPU produces.
struct Shard {
    Model* model = nullptr;
    size_t i0 = 0, i1 = 0;
    int64_t lo = 0, hi = 0, own_lo = 0, own_hi = 0;
    cudaStream_t stream = nullptr;
    int status = ANCHA_OK;
    std::string error;
    double model_seconds = 0.0;
    float* sums() const { return model->pipe.span.as<float>(); }
};

// Chunks [i0, i1) of the shard from host PCM: upload the track samples they read, overlap-add
// into the device span buffers (enqueued on the shard's stream; no host synchronisation).
void run_shard(const float* planes, const TrackPlan& plan, int batch, const volatile int* cancel, Shard& sh) {
    Model& model = *sh.model;
    int st = cudaSetDevice(model.device) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "cudaSetDevice");
    const int planes_n = (int)model.manifest.config.stems.size() * 2;
    const int64_t span = sh.hi - sh.lo;
    try {
        PipelineBuffers& pb = model.pipe;
        int64_t pcm_lo = 0, pcm_hi = 0;
        pcm_range(plan, sh.lo, sh.hi, &pcm_lo, &pcm_hi);
        const int64_t pcm_len = pcm_hi - pcm_lo;
        if (!st && pb.pcm.bytes < (size_t)(2 * pcm_len * 4)) pb.pcm.alloc(2 * pcm_len * 4);
        if (!st && pb.span.bytes < (size_t)(planes_n + 1) * span * 4) pb.span.alloc((size_t)(planes_n + 1) * span * 4);
        float* d_planes = pb.pcm.as<float>();
        float* d_sums = pb.span.as<float>();
        for (int ch = 0; ch < 2 && !st; ++ch)
            st = cudaMemcpyAsync(d_planes + ch * pcm_len, planes + ch * plan.samples + pcm_lo, pcm_len * 4,
                                 cudaMemcpyHostToDevice, sh.stream) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "upload PCM");
        if (!st) st = cudaMemsetAsync(d_sums, 0, (size_t)(planes_n + 1) * span * 4, sh.stream) == cudaSuccess
                          ? ANCHA_OK : fail(ANCHA_E_CUDA, "memset");
        if (!st) st = run_chunks(model, d_planes, pcm_lo, pcm_len, plan, sh.i0, sh.i1, batch, sh.lo, span, d_sums,
                                 d_sums + (size_t)planes_n * span, cancel, sh.stream, &sh.model_seconds);
    } catch (const std::exception& ex) {
        st = fail(ANCHA_E_CUDA, ex.what());
    }
    if (st) { sh.status = st; sh.error = ancha_last_error(); }
}

// Several GPUs: shards of contiguous chunk ranges, then the halo exchange on the device
// (chunk.rs:77-88 rule: the output is the sum of every chunk's weighted samples over the sum of
// the weights, so partial spans can be added anywhere before the division).
PcmResult separate_multi(Model* const* models, int n, const float* planes, const TrackPlan& plan, int batch,
                         const volatile int* cancel, float* stems_out) {
    PcmResult r;
    r.chunks = plan.starts.size();
    const int64_t samples = plan.samples;
    const int planes_n = (int)models[0]->manifest.config.stems.size() * 2;
    const int rows = planes_n + 1;  // sums rows, then the weights row
    // Contiguous ranges of chunk starts, ceil(chunks / n) per device; empty trailing shards drop out.
    const size_t per = (plan.starts.size() + n - 1) / n;
    std::vector<Shard> sh;
    for (int d = 0; d < n; ++d) {
        Shard x;
        x.model = models[d];
        x.i0 = std::min(plan.starts.size(), d * per);
        x.i1 = std::min(plan.starts.size(), (d + 1) * per);
        if (x.i0 >= x.i1) continue;
        x.lo = plan.starts[x.i0];
        x.hi = std::min(plan.starts[x.i1 - 1] + plan.chunk, plan.length);
        sh.push_back(x);
    }
    for (size_t k = 0; k < sh.size(); ++k) {
        sh[k].own_lo = k == 0 ? 0 : sh[k].lo;
        sh[k].own_hi = k + 1 < sh.size() ? sh[k + 1].lo : plan.length;
    }
    std::vector<cudaEvent_t> events;
    auto cleanup = [&] {
        for (auto& x : sh)
            if (x.stream) {
                cudaSetDevice(x.model->device);
                cudaStreamSynchronize(x.stream);
                cudaStreamDestroy(x.stream);
                x.stream = nullptr;
            }
        for (cudaEvent_t e : events) cudaEventDestroy(e);
        events.clear();
    };
    for (auto& x : sh) {
        if (cudaSetDevice(x.model->device) != cudaSuccess ||
            cudaStreamCreateWithFlags(&x.stream, cudaStreamNonBlocking) != cudaSuccess) {
            r.status = fail(ANCHA_E_CUDA, "cudaStreamCreate");
            cleanup();
            return r;
        }
    }
    // Phase 1 (one host thread per GPU, so kernel launches overlap): spans on the devices.
    {
        std::vector<std::thread> workers;
        for (auto& x : sh) workers.emplace_back([&, px = &x] { run_shard(planes, plan, batch, cancel, *px); });
        for (auto& w : workers) w.join();
    }
    for (auto& x : sh) {
        r.model_seconds = std::max(r.model_seconds, x.model_seconds);
        if (x.status != ANCHA_OK) {
            r.status = fail(x.status, x.error);
            cleanup();
            return r;
        }
    }
    int st = ANCHA_OK;
    // Phase 2: each shard's span columns inside a later shard's owned range go to that shard's
    // halo buffer (one peer copy per row, on the sender's stream), which adds them into its own
    // span once the copies have landed (an event wait on the receiver's stream).
    for (size_t q = 1; q < sh.size() && !st; ++q) {
        Shard& rq = sh[q];
        int64_t total = 0;
        for (size_t p = 0; p < q; ++p)
            total += std::max<int64_t>(0, std::min(sh[p].hi, rq.own_hi) - std::max(sh[p].lo, rq.own_lo));
        if (total == 0) continue;
        try {
            cudaSetDevice(rq.model->device);
            DevBuf& halo = rq.model->pipe.halo;
            if (halo.bytes < (size_t)rows * total * 4) halo.alloc((size_t)rows * total * 4);
        } catch (const std::exception& ex) {
            st = fail(ANCHA_E_CUDA, ex.what());
            break;
        }
        int64_t off = 0;
        for (size_t p = 0; p < q && !st; ++p) {
            Shard& sp = sh[p];
            const int64_t a = std::max(sp.lo, rq.own_lo), b = std::min(sp.hi, rq.own_hi);
            if (b <= a) continue;
            const int64_t w = b - a, span_p = sp.hi - sp.lo;
            float* piece = rq.model->pipe.halo.as<float>() + (size_t)rows * off;
            cudaSetDevice(sp.model->device);
            for (int row = 0; row < rows && !st; ++row)
                st = cudaMemcpyPeerAsync(piece + (size_t)row * w, rq.model->device,
                                         sp.sums() + (size_t)row * span_p + (a - sp.lo), sp.model->device,
                                         (size_t)w * 4, sp.stream) == cudaSuccess
                         ? ANCHA_OK : fail(ANCHA_E_CUDA, "halo peer copy");
            cudaEvent_t e;
            if (!st && cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) st = fail(ANCHA_E_CUDA, "event");
            if (st) break;
            events.push_back(e);
            if (cudaEventRecord(e, sp.stream) != cudaSuccess) { st = fail(ANCHA_E_CUDA, "event record"); break; }
            cudaSetDevice(rq.model->device);
            if (cudaStreamWaitEvent(rq.stream, e, 0) != cudaSuccess) { st = fail(ANCHA_E_CUDA, "event wait"); break; }
            const int64_t span_q = rq.hi - rq.lo;
            st = span_add(rq.sums(), rq.sums() + (size_t)planes_n * span_q, planes_n, span_q, a - rq.lo, piece, w,
                          rq.stream);
            off += w;
        }
    }
    // Phase 3: each shard divides and crops its owned range and copies it into the caller's stems.
    for (size_t k = 0; k < sh.size() && !st; ++k) {
        Shard& x = sh[k];
        const int64_t o0 = std::max(x.own_lo, plan.border), o1 = std::min(x.own_hi, plan.border + samples);
        if (o1 <= o0) continue;
        const int64_t count = o1 - o0, span = x.hi - x.lo;
        cudaSetDevice(x.model->device);
        PipelineBuffers& pb = x.model->pipe;
        try {
            if (pb.stems.bytes < (size_t)planes_n * count * 4) pb.stems.alloc((size_t)planes_n * count * 4);
        } catch (const std::exception& ex) {
            st = fail(ANCHA_E_CUDA, ex.what());
            break;
        }
        st = span_finish(x.sums(), x.sums() + (size_t)planes_n * span, planes_n, span, o0 - x.lo, count,
                         pb.stems.as<float>(), count, pb.flag.as<int>() + 1, x.stream);
        for (int p = 0; p < planes_n && !st; ++p)
            st = cudaMemcpyAsync(stems_out + (size_t)p * samples + (o0 - plan.border),
                                 pb.stems.as<float>() + (size_t)p * count, (size_t)count * 4, cudaMemcpyDeviceToHost,
                                 x.stream) == cudaSuccess ? ANCHA_OK : fail(ANCHA_E_CUDA, "download stems");
    }
    // Phase 4: status words of every shard.
    for (auto& x : sh) {
        if (st) break;
        cudaSetDevice(x.model->device);
        int flags[2] = {0, 0};
        if (cudaMemcpyAsync(flags, x.model->pipe.flag.p, 8, cudaMemcpyDeviceToHost, x.stream) != cudaSuccess) {
            st = fail(ANCHA_E_CUDA, "read status");
            break;
        }
        int mflag = 0;
        st = x.model->read_flag(x.stream, &mflag);  // synchronises the stream
        if (!st && (mflag || (flags[1] & 1))) st = fail(ANCHA_E_NONFINITE, "non-finite chunk output");
        if (!st && flags[0]) st = fail(ANCHA_E_NONFINITE, "iSTFT has an uncovered sample");
        if (!st && (flags[1] & 4)) st = fail(ANCHA_E_INVALID, "uncovered overlap-add sample");
    }
    cleanup();
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
    return separate_multi(models, n, planes, plan, batch, cancel, stems_out);
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

extern "C" int ancha_chunk_pcm_range(int64_t samples, int64_t chunk_samples, int overlap, int64_t first,
                                     int64_t last, int64_t* lo, int64_t* hi) {
    if (samples <= 0 || !lo || !hi) return fail(ANCHA_E_INVALID, "chunk_pcm_range: invalid arguments");
    try {
        const TrackPlan plan = make_plan(samples, chunk_samples, overlap);
        const int64_t n = (int64_t)plan.starts.size();
        if (first < 0 || last > n || first > last)
            return fail(ANCHA_E_INVALID, "chunk_pcm_range: chunk range outside the plan");
        if (first == last) {
            *lo = *hi = 0;
        } else {
            pcm_range(plan, plan.starts[first], std::min(plan.starts[last - 1] + plan.chunk, plan.length), lo, hi);
        }
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
    return ANCHA_OK;
}

extern "C" int ancha_separate_span_device(ancha_model* model, const float* pcm, int64_t pcm_lo, int64_t pcm_len,
                                          int64_t samples, int64_t chunk_samples, int overlap, int batch_chunks,
                                          int64_t first, int64_t last, float* sums, float* weights, void* stream) {
    if (!model || !pcm || !sums || !weights) return fail(ANCHA_E_INVALID, "separate_span_device: null argument");
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
    if (first < 0 || last > (int64_t)plan.starts.size() || first >= last)
        return fail(ANCHA_E_INVALID, "separate_span_device: empty chunk range or outside the plan");
    const int64_t lo = plan.starts[first], hi = std::min(plan.starts[last - 1] + plan.chunk, plan.length);
    int64_t need_lo = 0, need_hi = 0;
    pcm_range(plan, lo, hi, &need_lo, &need_hi);
    if (pcm_lo < 0 || pcm_len <= 0 || pcm_lo > need_lo || pcm_lo + pcm_len < need_hi || pcm_lo + pcm_len > samples)
        return fail(ANCHA_E_INVALID, "separate_span_device: the PCM slice does not hold samples [" +
                                         std::to_string(need_lo) + ", " + std::to_string(need_hi) + ")");
    const int batch = batch_chunks > 0 ? std::min(batch_chunks, kMaxChunksPerCall) : default_batch((size_t)(last - first));
    cudaStream_t s = as_stream(stream);
    ANCHA_CUDA(cudaSetDevice(m.device));
    const int planes_n = (int)c.stems.size() * 2;
    ANCHA_CUDA(cudaMemsetAsync(sums, 0, (size_t)planes_n * (hi - lo) * 4, s));
    ANCHA_CUDA(cudaMemsetAsync(weights, 0, (size_t)(hi - lo) * 4, s));
    return run_chunks(m, pcm, pcm_lo, pcm_len, plan, (size_t)first, (size_t)last, batch, lo, hi - lo, sums, weights,
                      nullptr, s, nullptr);
}

extern "C" int ancha_span_add(float* sums, float* weights, int planes, int64_t span, int64_t offset,
                              const float* piece, int64_t count, void* stream) {
    if (!sums || !weights || !piece || planes <= 0 || span <= 0 || count < 0)
        return fail(ANCHA_E_INVALID, "span_add: invalid arguments");
    return span_add(sums, weights, planes, span, offset, piece, count, as_stream(stream));
}

extern "C" int ancha_span_finish(const float* sums, const float* weights, int planes, int64_t span, int64_t offset,
                                 int64_t count, float* out, int64_t ld, int* flag, void* stream) {
    if (!sums || !weights || !out || !flag || planes <= 0 || span <= 0 || count < 0)
        return fail(ANCHA_E_INVALID, "span_finish: invalid arguments");
    return span_finish(sums, weights, planes, span, offset, count, out, ld, flag, as_stream(stream));
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
    ANCHA_TRY(run_chunks(m, planes, 0, samples, plan, 0, plan.starts.size(), batch, 0, plan.length, sums, weights,
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
