// extern "C" entry points of include/ancha_b200.h: argument validation with the
// reference's rules (fused/mod.rs:20-176), status codes and the per-thread last error.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <string>

#ifndef ANCHA_FP32_SPLIT
#define ANCHA_FP32_SPLIT 1  // fp32 operands on the tensor cores as three-plane bf16 splits
#endif

#include "attention.cuh"
#include "rowops.cuh"
#include "dsp.cuh"
#include "gemm.cuh"
#include "mdx23c_model.hpp"
#include "mdx_exec.hpp"
#include "onnx.hpp"
#include "model.hpp"
#include "tc.cuh"

namespace ancha {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const std::string& msg) {
    g_last_error = msg;
    return code;
}

int cuda_fail(cudaError_t err, const char* what) {
    return fail(ANCHA_E_CUDA, std::string(what) + ": " + cudaGetErrorString(err));
}

int check_launch(const char* what) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return cuda_fail(e, what);
    return ANCHA_OK;
}

namespace {
// Rows up to the last one the attention's groups reach and the used q | k | v columns, rounded
// to 16-byte plane rows: the fp32 split's planes are 3 · rows · pld bf16.
void attention_plane_shape(const AttnArgs& a, int64_t* rows, int64_t* cols, int64_t* pld) {
    const int64_t outer = a.groups / a.group_inner;
    *rows = (outer - 1) * a.group_outer_stride + (a.group_inner - 1) * a.group_inner_stride +
            (int64_t)(a.tokens - 1) * a.token_stride + 1;
    *cols = std::max(std::max(a.q_col, a.k_col), a.v_col) + (int64_t)a.heads * 64;
    *pld = (*cols + 7) / 8 * 8;
}

bool attention_split_applies(const AttnArgs& a, const void* q, const void* k, const void* v) {
    return ANCHA_FP32_SPLIT && a.elt == ELT_F32 && q == k && q == v && a.tokens > 0 && a.groups > 0 &&
           a.groups % a.group_inner == 0;
}

int attention_args(const ancha_attn_desc* d, const void* q, const void* k, const void* v, const void* gate,
                   void* out, AttnArgs* a) {
    if (!d || !q || !k || !v || !out) return fail(ANCHA_E_INVALID, "attention: null argument");
    if (d->head_dim != 64) return fail(ANCHA_E_UNSUPPORTED, "attention: head_dim must be 64");
    if (d->groups < 0 || d->tokens < 0 || d->heads <= 0)
        return fail(ANCHA_E_INVALID, "attention: negative shape");
    if (d->dtype != ANCHA_F32 && d->dtype != ANCHA_BF16 && d->dtype != ANCHA_F16)
        return fail(ANCHA_E_INVALID, "attention: unknown dtype");
    if (d->group_inner <= 0 || d->token_stride < 0 || d->ld <= 0 || d->out_ld <= 0)
        return fail(ANCHA_E_INVALID, "attention: invalid strides");
    const int64_t span = (int64_t)d->heads * 64;
    if (d->q_col < 0 || d->k_col < 0 || d->v_col < 0 || d->out_col < 0 ||
        d->q_col + span > d->ld || d->k_col + span > d->ld || d->v_col + span > d->ld ||
        d->out_col + span > d->out_ld || (gate && (d->gate_col < 0 || d->gate_col + d->heads > d->ld)))
        return fail(ANCHA_E_INVALID, "attention: q / k / v column ranges do not fit the rows");
    *a = AttnArgs{};
    a->q = q; a->k = k; a->v = v; a->gate = gate; a->out = out;
    a->groups = d->groups; a->tokens = d->tokens; a->heads = d->heads; a->head_dim = 64;
    a->ld = d->ld; a->out_ld = d->out_ld;
    a->group_inner = d->group_inner; a->group_inner_stride = d->group_inner_stride;
    a->group_outer_stride = d->group_outer_stride; a->token_stride = d->token_stride;
    a->q_col = d->q_col; a->k_col = d->k_col; a->v_col = d->v_col;
    a->gate_col = gate ? d->gate_col : 0; a->out_col = d->out_col;
    a->elt = d->dtype;
    return ANCHA_OK;
}
}  // namespace

}  // namespace ancha

using namespace ancha;

extern "C" {

const char* ancha_last_error(void) { return g_last_error.c_str(); }

const char* ancha_version(void) { return "ancha-b200 0.1.0 (sm_100a)"; }

int ancha_wait_selftest(int64_t budget_cycles, void* stream) {
    return wait_selftest((long long)budget_cycles, as_stream(stream));
}

int ancha_available(int device) {
    int count = 0;
    cudaError_t e = cudaGetDeviceCount(&count);
    if (e != cudaSuccess) {
        cudaGetLastError();
        fail(ANCHA_E_CUDA, std::string("no CUDA device: ") + cudaGetErrorString(e));
        return 0;
    }
    if (device < 0 || device >= count) {
        fail(ANCHA_E_INVALID, "CUDA device " + std::to_string(device) + " not found");
        return 0;
    }
    cudaDeviceProp p;
    if (cudaGetDeviceProperties(&p, device) != cudaSuccess || p.major != 10) {
        fail(ANCHA_E_UNSUPPORTED, "device is not an sm_100 (B200-class) GPU");
        return 0;
    }
    return 1;
}


int ancha_attention_workspace(const ancha_attn_desc* d, size_t* bytes) {
    if (!d || !bytes) return fail(ANCHA_E_INVALID, "attention_workspace: null argument");
    *bytes = 0;
    if (d->dtype != ANCHA_F32 || d->groups <= 0 || d->tokens <= 0 || d->group_inner <= 0 ||
        d->groups % d->group_inner != 0)
        return ANCHA_OK;
    AttnArgs a{};
    a.groups = d->groups; a.tokens = d->tokens; a.heads = d->heads; a.group_inner = d->group_inner;
    a.group_inner_stride = d->group_inner_stride; a.group_outer_stride = d->group_outer_stride;
    a.token_stride = d->token_stride; a.q_col = d->q_col; a.k_col = d->k_col; a.v_col = d->v_col;
    int64_t rows, cols, pld;
    attention_plane_shape(a, &rows, &cols, &pld);
    *bytes = (size_t)(3 * rows * pld * 2);
    return ANCHA_OK;
}

int ancha_attention_fwd_ws(const ancha_attn_desc* d, const void* q, const void* k, const void* v,
                           const void* gate, void* out, void* workspace, size_t workspace_bytes, void* stream) {
    AttnArgs a{};
    ANCHA_TRY(attention_args(d, q, k, v, gate, out, &a));
    cudaStream_t s = as_stream(stream);
    if (a.elt != ELT_F32) {
        int st = attention_tc(a, s);
        if (st != ANCHA_E_UNSUPPORTED) return st;
    }
    // fp32 on the tensor cores: the used q | k | v columns of every row up to the last one the
    // groups reach, split into three bf16 planes in the caller's workspace.
    if (attention_split_applies(a, q, k, v) && workspace) {
        int64_t rows, cols, pld;
        attention_plane_shape(a, &rows, &cols, &pld);
        if (workspace_bytes >= (size_t)(3 * rows * pld * 2)) {
            int st = split3_rows_strided(static_cast<const float*>(q), a.ld, workspace, pld, rows * pld, rows,
                                         (int)cols, s);
            if (st == ANCHA_OK) st = attention_tc_split(a, workspace, pld, rows * pld, s);
            if (st != ANCHA_E_UNSUPPORTED) return st;
        }
    }
    return attention_ffma(a, s);
}

int ancha_attention_fwd(const ancha_attn_desc* d, const void* q, const void* k, const void* v,
                        const void* gate, void* out, void* stream) {
    return ancha_attention_fwd_ws(d, q, k, v, gate, out, nullptr, 0, stream);
}

int ancha_linear_workspace(const ancha_linear_desc* d, size_t* bytes) {
    if (!d || !bytes) return fail(ANCHA_E_INVALID, "linear_workspace: null argument");
    *bytes = d->rope_width && d->rope_tokens > 0 && d->dtype != ANCHA_F32 ? (size_t)2 * 32 * d->rope_tokens * 16 : 0;
    return ANCHA_OK;
}

int ancha_linear_fwd_ws(const ancha_linear_desc* d, const void* x, const void* w, const float* bias,
                        const float* residual, const float* rope, void* out, void* workspace,
                        size_t workspace_bytes, void* stream) {
    if (!d || !x || !w || !out) return fail(ANCHA_E_INVALID, "linear: null argument");
    if (d->m < 0 || d->n <= 0 || d->k <= 0) return fail(ANCHA_E_UNSUPPORTED, "linear: empty shape");
    if (d->dtype != ANCHA_F32 && d->dtype != ANCHA_BF16 && d->dtype != ANCHA_F16)
        return fail(ANCHA_E_INVALID, "linear: unknown dtype");
    if (d->out_dtype != ANCHA_F32 && d->out_dtype != ANCHA_BF16 && d->out_dtype != ANCHA_F16)
        return fail(ANCHA_E_INVALID, "linear: unknown output dtype");
    if (d->act < ANCHA_ACT_NONE || d->act > ANCHA_ACT_GLU) return fail(ANCHA_E_INVALID, "linear: unknown activation");
    if (d->act == ANCHA_ACT_GLU && (d->n % 2 || residual || d->rope_width))
        return fail(ANCHA_E_INVALID, "linear: GLU needs an even n and no residual / rotary");
    const int wl = d->weight_layout;
    if (wl != ANCHA_W_KN && wl != ANCHA_W_NK) return fail(ANCHA_E_INVALID, "linear: unknown weight layout");
    if (d->ldx < d->k || d->ldw < (wl == ANCHA_W_NK ? d->k : d->n))
        return fail(ANCHA_E_INVALID, "linear: leading dimension too small");
    const int n_out = d->act == ANCHA_ACT_GLU ? d->n / 2 : d->n;
    if (d->ldout < n_out || (residual && d->ldres < d->n))
        return fail(ANCHA_E_INVALID, "linear: output / residual leading dimension too small");
    if (d->rope_width) {
        // fused/mod.rs:114-124: [4, tokens, 64] table, whole token rows, width % 64, 2w <= n.
        if (!rope || d->rope_tokens <= 0 || d->rope_div <= 0 || d->rope_width % 64 ||
            2 * d->rope_width > d->n)
            return fail(ANCHA_E_UNSUPPORTED, "linear: rotary epilogue shape not supported");
    }
    GemmGroup g{};
    g.a = x; g.b = w; g.bias = bias; g.residual = residual; g.out = out;
    g.m = d->m; g.n = d->n; g.k = d->k;
    g.lda = d->ldx; g.ldb = d->ldw; g.ldr = d->ldres; g.ldo = d->ldout;
    GemmEpilogue e{};
    e.act = d->act;
    e.out_type = d->out_dtype;
    e.rope = d->rope_width ? rope : nullptr;
    e.rope_width = d->rope_width;
    e.rope_tokens = d->rope_tokens > 0 ? d->rope_tokens : 1;
    e.rope_div = d->rope_div > 0 ? d->rope_div : 1;
    e.rope_hd = 64;
    e.row_mul = d->row_scale;
    if (d->row_scale && reinterpret_cast<uintptr_t>(d->row_scale) % 4)
        return fail(ANCHA_E_INVALID, "linear: row_scale not 4-byte aligned");
    cudaStream_t s = as_stream(stream);
    if (d->dtype != ANCHA_F32 && wl == ANCHA_W_NK) {
        int st;
        const size_t qbytes = (size_t)2 * 32 * e.rope_tokens * 16;
        if (e.rope && workspace && workspace_bytes >= qbytes && reinterpret_cast<uintptr_t>(workspace) % 16 == 0) {
            // The tensor-core epilogue reads the table in its pair-major general form (same
            // arithmetic, coalesced loads), rewritten into the caller's workspace.
            GemmEpilogue eq = e;
            eq.rope = nullptr;
            eq.rope_quads = static_cast<const float*>(workspace);
            st = rope_quads_from_table(e.rope, e.rope_tokens, 64, workspace, s);
            if (st == ANCHA_OK) st = gemm_tc(g, d->dtype, eq, s);
        } else {
            st = gemm_tc(g, d->dtype, e, s);
        }
        if (st != ANCHA_E_UNSUPPORTED) return st;
    }
    return gemm_ffma(g, nullptr, 1, d->m, d->n, d->dtype, d->dtype, wl == ANCHA_W_NK, e, s);
}

int ancha_linear_fwd(const ancha_linear_desc* d, const void* x, const void* w, const float* bias,
                     const float* residual, const float* rope, void* out, void* stream) {
    return ancha_linear_fwd_ws(d, x, w, bias, residual, rope, out, nullptr, 0, stream);
}

int ancha_stft_fwd(const float* audio, int chunks, int samples, int hop, float* packed, void* stream) {
    if (!audio || !packed || chunks < 0) return fail(ANCHA_E_INVALID, "stft: invalid arguments");
    if (reinterpret_cast<uintptr_t>(packed) % 16)
        return fail(ANCHA_E_INVALID, "stft: packed spectrum must be 16-byte aligned");
    return stft_forward(audio, chunks, samples, hop, packed, as_stream(stream));
}

int ancha_istft_masked(const float* packed, const float* masks, int chunks, int stems, int samples,
                       int hop, int zero_dc, float* scratch, float* out, void* stream) {
    if (!packed || !masks || !scratch || !out || chunks < 0 || stems < 0 || hop <= 0)
        return fail(ANCHA_E_INVALID, "istft: invalid arguments");
    if (reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(scratch) % 8)
        return fail(ANCHA_E_INVALID, "istft: packed must be 16-byte and scratch 8-byte aligned");
    // Checked here as well as in istft_masked: the status word's address below derives from them.
    if (hop > 1024 || samples <= 1024)
        return fail(ANCHA_E_INVALID, "istft: require hop in 1..=1024 and samples > 1024");
    // The status word sits after the frame scratch; bit 2 = an uncovered sample.
    const int frames = samples / hop + 1;
    int* flag = reinterpret_cast<int*>(scratch + (int64_t)chunks * stems * 2 * frames * 2048);
    cudaStream_t s = as_stream(stream);
    ANCHA_CUDA(cudaMemsetAsync(flag, 0, sizeof(int), s));
    return istft_masked(packed, masks, chunks, stems, samples, hop, zero_dc, scratch, out, flag, s);
}

int ancha_istft_masked_static(const float* packed, const float* masks, int chunks, int stems,
                              int samples, int hop, int zero_dc, float* out, int* status,
                              void* stream) {
    if (!packed || !masks || !out || chunks < 0 || stems < 0 || hop <= 0)
        return fail(ANCHA_E_INVALID, "istft_static: invalid arguments");
    if (reinterpret_cast<uintptr_t>(packed) % 16 || reinterpret_cast<uintptr_t>(status) % 4)
        return fail(ANCHA_E_INVALID, "istft_static: packed must be 16-byte and status 4-byte aligned");
    return istft_masked_static(packed, masks, chunks, stems, samples, hop, zero_dc, out, status,
                               as_stream(stream));
}

int ancha_ola_add(const float* y, int chunks, int planes, int chunk, int overlap,
                  const int64_t* starts, int64_t length, float* sums, float* weights, void* stream) {
    if (!y || !starts || !sums || !weights || chunks < 0 || planes <= 0 || chunk <= 0 || overlap <= 0)
        return fail(ANCHA_E_INVALID, "ola: invalid arguments");
    if (chunks > kMaxChunksPerCall) return fail(ANCHA_E_INVALID, "ola: too many chunks per call");
    ChunkStarts cs{};
    for (int c = 0; c < chunks; ++c) {
        if (starts[c] < 0 || starts[c] >= length || (c && starts[c] < starts[c - 1]))
            return fail(ANCHA_E_INVALID, "ola: chunk starts must be ascending and inside the output");
        cs.v[c] = starts[c];
    }
    return ola_add(y, chunks, planes, chunk, cs, length, 0, length, sums, weights, as_stream(stream));
}

int ancha_model_load(const char* package_dir, int device, int precision, ancha_model** out) {
    if (!package_dir || !out) return fail(ANCHA_E_INVALID, "model_load: null argument");
    *out = nullptr;
    try {
        auto m = Model::load(package_dir, device, precision);
        *out = new ancha_model{std::move(m)};
        return ANCHA_OK;
    } catch (const std::exception& e) {
        const std::string msg = e.what();
        const bool io = msg.rfind("read ", 0) == 0;
        return fail(io ? ANCHA_E_IO : ANCHA_E_INVALID, msg);
    }
}

int ancha_model_info(const ancha_model* model, int* stems, int* bands, int* dim, int* bins,
                     int* chunk_samples, int* hop, int* overlap) {
    if (!model) return fail(ANCHA_E_INVALID, "model_info: null model");
    const ModelConfig& c = model->impl->manifest.config;
    if (stems) *stems = (int)c.stems.size();
    if (bands) *bands = (int)c.bands.size();
    if (dim) *dim = c.dim;
    if (bins) *bins = c.n_fft / 2 + 1;
    if (chunk_samples) *chunk_samples = (int)c.chunk_samples;
    if (hop) *hop = c.hop;
    if (overlap) *overlap = c.overlap;
    return ANCHA_OK;
}

int ancha_model_forward(ancha_model* model, const float* spectrum, int chunks, int frames,
                        float* masks, const volatile int* cancel, void* stream) {
    if (!model || !spectrum || !masks) return fail(ANCHA_E_INVALID, "model_forward: null argument");
    try {
        return model->impl->forward(spectrum, chunks, frames, masks, cancel, as_stream(stream));
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
}

void ancha_model_free(ancha_model* model) { delete model; }

int ancha_mdx23c_load(const char* package_dir, int device, int precision, ancha_mdx23c** out) {
    if (!package_dir || !out) return fail(ANCHA_E_INVALID, "mdx23c_load: null argument");
    *out = nullptr;
    try {
        auto m = Mdx23c::load(package_dir, device, precision);
        *out = new ancha_mdx23c{std::move(m)};
        return ANCHA_OK;
    } catch (const std::exception& e) {
        const std::string msg = e.what();
        const bool io = msg.rfind("read ", 0) == 0;
        return fail(io ? ANCHA_E_IO : ANCHA_E_INVALID, msg);
    }
}

int ancha_mdx23c_info(const ancha_mdx23c* model, int* bins, int* frames, int* n_fft, int* hop, int* overlap,
                      int* stems, int* tensor_count) {
    if (!model) return fail(ANCHA_E_INVALID, "mdx23c_info: null model");
    const Mdx23cConfig& c = model->impl->manifest.config;
    if (bins) *bins = c.bins;
    if (frames) *frames = c.frames;
    if (n_fft) *n_fft = c.n_fft;
    if (hop) *hop = c.hop;
    if (overlap) *overlap = c.overlap;
    if (stems) *stems = (int)c.stems.size();
    if (tensor_count) *tensor_count = (int)model->impl->tensor_count;
    return ANCHA_OK;
}

int ancha_mdx23c_forward(ancha_mdx23c* model, const float* spectrum, int batch, int frames, float* out,
                         const volatile int* cancel, void* stream) {
    if (!model || !spectrum || !out) return fail(ANCHA_E_INVALID, "mdx23c_forward: null argument");
    try {
        return model->impl->forward(spectrum, batch, frames, out, cancel, as_stream(stream));
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
}

int ancha_mdx23c_separate_pcm(ancha_mdx23c* model, const float* planes, int64_t samples, int overlap, int batch,
                              const volatile int* cancel, float* stems_out, double* seconds_out) {
    if (!model || !planes || !stems_out) return fail(ANCHA_E_INVALID, "mdx23c_separate_pcm: null argument");
    return model->impl->separate_pcm(planes, samples, overlap, batch, cancel, stems_out, seconds_out);
}

int ancha_mdx23c_plan(int64_t samples, int64_t chunk_samples, int overlap, int64_t* step, int64_t* border,
                      int64_t* pad, int64_t* padded, int64_t* chunks) {
    try {
        const Mdx23cPlan p = Mdx23cPlan::make(samples, chunk_samples, overlap);
        if (step) *step = p.step;
        if (border) *border = p.border;
        if (pad) *pad = p.pad;
        if (padded) *padded = p.padded;
        if (chunks) *chunks = p.chunks;
        return ANCHA_OK;
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
}

void ancha_mdx23c_free(ancha_mdx23c* model) { delete model; }

int ancha_mdx_graph_inspect(const void* onnx, size_t bytes, int optimized, int* nodes, int* instructions,
                            int* folded_bn, int* constants) {
    if (!onnx || bytes == 0) return fail(ANCHA_E_INVALID, "mdx_graph_inspect: empty model");
    try {
        const OnnxModel m = parse_onnx(static_cast<const uint8_t*>(onnx), bytes);
        const MdxGraph g = MdxGraph::build(m, optimized != 0);
        if (nodes) *nodes = g.nodes;
        if (instructions) *instructions = (int)g.instructions.size();
        if (folded_bn) *folded_bn = g.folded_bn;
        if (constants) *constants = (int)g.constants.size();
        return ANCHA_OK;
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
}

void ancha_free_string(char* s) { std::free(s); }

int ancha_mdx_load(const void* onnx, size_t bytes, int optimized, int device, ancha_mdx** out) {
    if (!onnx || bytes == 0 || !out) return fail(ANCHA_E_INVALID, "mdx_load: null argument");
    *out = nullptr;
    try {
        auto m = MdxModel::load(static_cast<const uint8_t*>(onnx), bytes, optimized != 0, device);
        *out = new ancha_mdx{std::move(m)};
        return ANCHA_OK;
    } catch (const std::exception& e) {
        return fail(ANCHA_E_INVALID, e.what());
    }
}

int ancha_mdx_output_shape(const ancha_mdx* graph, const int64_t input_shape[4], int64_t output_shape[4]) {
    if (!graph || !input_shape || !output_shape) return fail(ANCHA_E_INVALID, "mdx_output_shape: null argument");
    Shape4 in{input_shape[0], input_shape[1], input_shape[2], input_shape[3]}, out{};
    ANCHA_TRY(graph->impl->output_shape(in, out));
    for (int d = 0; d < 4; ++d) output_shape[d] = out[d];
    return ANCHA_OK;
}

int ancha_mdx_forward(ancha_mdx* graph, const float* x, const int64_t input_shape[4], float* out,
                      const volatile int* cancel, void* stream) {
    if (!graph || !x || !input_shape || !out) return fail(ANCHA_E_INVALID, "mdx_forward: null argument");
    Shape4 in{input_shape[0], input_shape[1], input_shape[2], input_shape[3]};
    try {
        return graph->impl->forward(x, in, out, cancel, as_stream(stream));
    } catch (const std::exception& e) {
        return fail(ANCHA_E_CUDA, e.what());
    }
}

int ancha_mdx_separate_pcm(ancha_mdx* graph, const ancha_mdx_task* task, const float* planes, int64_t samples,
                           const volatile int* cancel, float* predicted, float* residual, double* seconds_out) {
    if (!graph || !task || !planes || !predicted || !residual) return fail(ANCHA_E_INVALID, "mdx_separate_pcm: null argument");
    MdxTaskOpts o;
    o.n_fft = task->n_fft; o.hop = task->hop; o.bins = task->bins; o.frames = task->frames;
    o.compensate = (float)task->compensate; o.overlap = task->overlap; o.denoise = task->denoise != 0;
    o.batch = task->batch;
    return graph->impl->separate_pcm(o, planes, samples, cancel, predicted, residual, seconds_out);
}

int ancha_mdx_set_gemm(ancha_mdx* graph, int precision) {
    if (!graph) return fail(ANCHA_E_INVALID, "mdx_set_gemm: null graph");
    return graph->impl->set_gemm(precision);
}

void ancha_mdx_free(ancha_mdx* graph) { delete graph; }

}  // extern "C"
