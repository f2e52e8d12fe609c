/*
 * ancha_b200.h -- C ABI of the B200-native RoFormer separation engine.
 *
 * This is the drop-in boundary for the hot path of 3tic-project/Ancha: the kernel plug-in
 * API of crates/ancha-models/src/fused/mod.rs, the model API of
 * crates/ancha-models/src/network.rs and the task API of src/backend.rs / src/runtime.rs.
 * Every entry point takes plain pointers and sizes. Device pointers are CUDA device
 * addresses on the calling thread's current device; `stream` is a cudaStream_t passed as
 * void* (NULL = the legacy default stream). The caller owns every buffer: kernel entry
 * points never allocate.
 *
 * Status codes: ANCHA_OK, or a negative code. ANCHA_E_UNSUPPORTED is the reference's
 * `None` ("shape or backend not handled here, use your fallback"); the reference panics
 * inside `launch` on invalid operands, which maps to ANCHA_E_INVALID. After any non-zero
 * status, ancha_last_error() returns a message for the calling thread.
 */
#ifndef ANCHA_B200_H
#define ANCHA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define ANCHA_API __attribute__((visibility("default")))
#else
#define ANCHA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

enum {
    ANCHA_OK = 0,
    ANCHA_E_UNSUPPORTED = -1, /* the reference's `None`: caller falls back            */
    ANCHA_E_INVALID = -2,     /* invalid arguments (the reference asserts / errors)     */
    ANCHA_E_CUDA = -3,        /* a CUDA runtime or launch error                         */
    ANCHA_E_CANCELLED = -4,   /* the cancel flag was set (runtime.rs:44,118)           */
    ANCHA_E_IO = -5,          /* file or package error                                  */
    ANCHA_E_TIMEOUT = -6,     /* a bounded device-side wait gave up                     */
    ANCHA_E_NONFINITE = -7    /* non-finite model output (runtime.rs:173-176)           */
};

/* Element types of kernel operands. */
enum { ANCHA_F32 = 0, ANCHA_BF16 = 1, ANCHA_F16 = 2 };

/* Model arithmetic: F32 = fp32 operands, the transformer and mask-head GEMMs and the time-axis
 * attention on the tcgen05 tensor cores as three-plane bf16 splits (hi + mid + lo, 24 significant bits;
 * six plane products accumulated in fp32), the rest on fp32 FFMA kernels; BF16 / F16 = bf16 /
 * f16 operands on the tensor cores (GEMMs and attention) with fp32 accumulation; the residual
 * stream, norms, softmax statistics and DSP stay fp32 in every mode. */
enum { ANCHA_PRECISION_F32 = 0, ANCHA_PRECISION_BF16 = 1, ANCHA_PRECISION_F16 = 2 };

/* Message of the last failure on the calling thread ("" if none). */
ANCHA_API const char* ancha_last_error(void);

/* Library version string. */
ANCHA_API const char* ancha_version(void);

/* 1 when `device` is an sm_100 GPU this library can run on, else 0 (with a message).
 * Replaces fused::available::<B>() (fused/mod.rs:249-255) and src/cuda.rs::probe (19-46). */
ANCHA_API int ancha_available(int device);

/* Watchdog self-test of the current device: one kernel waits, with a budget of `budget_cycles`
 * SM clock cycles (0 to the kernels' own ~1 s budget), on an mbarrier that nothing arrives at,
 * through the same bounded wait every tensor-core kernel uses; the kernel gives up, records the
 * timeout in the library's device error word and returns. Returns ANCHA_E_TIMEOUT (with a
 * message) when the watchdog works; the device stays usable and the error word is cleared.
 * Diagnostics of the failure path that src/device.rs:11-41 and tests/cuda_device_failure.rs
 * cover in the reference; synchronises `stream`. */
ANCHA_API int ancha_wait_selftest(int64_t budget_cycles, void* stream);

/* ------------------------------------------------------------------------------------ *
 * Kernel plug-in API (replaces crates/ancha-models/src/fused/mod.rs)                   *
 * ------------------------------------------------------------------------------------ */

/* Attention operand layout. Token `i` of group `g` lives at row
 *     row(g, i) = (g / group_inner) * group_outer_stride + (g % group_inner) * group_inner_stride
 *                 + i * token_stride
 * of a row-major matrix whose rows are `ld` elements apart; head `h` of q / k / v starts at
 * column q_col / k_col / v_col + 64·h and the output head at out_col + 64·h of rows
 * `out_ld` apart. With gate_col >= 0 each output row of head h is scaled by
 * sigmoid(q[row, gate_col + h]) (the gated form). The reference's dense [groups, tokens,
 * heads, 64] layout is group_inner = groups, group_inner_stride = tokens, token_stride = 1,
 * ld = out_ld = heads·64. */
typedef struct {
    int groups, tokens, heads;
    int head_dim;                 /* must be 64 (ATTENTION_HEAD_DIM, fused/mod.rs:18) */
    int dtype;                    /* ANCHA_F32 / ANCHA_BF16 / ANCHA_F16: q/k/v/gate, out */
    int64_t ld, out_ld;           /* row strides in elements                           */
    int64_t group_inner, group_inner_stride, group_outer_stride, token_stride; /* rows */
    int q_col, k_col, v_col, gate_col, out_col;
} ancha_attn_desc;

/* softmax(q·kᵀ)·v per (group, head), non-causal, q pre-scaled by 1/sqrt(64); optionally
 * gated. Replaces fused::attention (fused/mod.rs:20-41) and fused::gated_attention
 * (fused/mod.rs:43-55), whose kernel is fused/attention.rs:24-298. No allocation: BF16 / F16
 * with q, k and v in one buffer (q == k == v) run on the tensor cores, everything else (F32
 * included) on the FFMA kernel. */
ANCHA_API int ancha_attention_fwd(const ancha_attn_desc* desc, const void* q, const void* k,
                        const void* v, const void* gate, void* out, void* stream);

/* Device workspace bytes ancha_attention_fwd_ws can use for `desc` (0: none helps): for F32,
 * the three-plane bf16 split of the used q / k / v columns of every row the groups reach. */
ANCHA_API int ancha_attention_workspace(const ancha_attn_desc* desc, size_t* bytes);

/* ancha_attention_fwd with a caller-owned device workspace (16-byte aligned, at least the
 * ancha_attention_workspace bytes; NULL or smaller = the ancha_attention_fwd paths). With it an
 * F32 call with q == k == v runs on the tensor cores: the used columns split into hi / mid / lo
 * bf16 planes in the workspace and six plane products per S = q·kᵀ and per P·v, with f32
 * accumulation (max abs error against float64 on par with the FFMA kernel's). */
ANCHA_API int ancha_attention_fwd_ws(const ancha_attn_desc* desc, const void* q, const void* k,
                           const void* v, const void* gate, void* out, void* workspace,
                           size_t workspace_bytes, void* stream);

/* Weight layouts accepted by ancha_linear_fwd. */
enum {
    ANCHA_W_KN = 0, /* weight[k][n]: Burn's Linear layout, the reference's fused::linear */
    ANCHA_W_NK = 1  /* weight[n][k]: PyTorch's [out, in]                                 */
};

/* Epilogue activations (applied after the bias, fused/gemm.rs:44-82 order). */
enum { ANCHA_ACT_NONE = 0, ANCHA_ACT_GELU = 1, ANCHA_ACT_TANH = 2, ANCHA_ACT_GLU = 3 };

/* out[m, n] = epilogue(sum_k x[m, k] · w(k, n)).
 * Epilogue, in order: + bias[n]; activation; interleaved RoPE on columns [0, 2·rope_width)
 * (queries then keys, token = (m / rope_div) % rope_tokens, table [4, rope_tokens, 64] =
 * query cos / signed sin (carrying 1/sqrt(64)), key cos / signed sin, as AxisRope::packed,
 * roformer.rs:281-302); + residual[m, n]. ANCHA_ACT_GLU pairs columns (2j, 2j+1) as
 * (value, gate) and writes value·sigmoid(gate) to column j (n_out = n / 2).
 * Replaces fused::linear + Epilogue (fused/mod.rs:57-176, kernel fused/gemm.rs:84-311).
 * x, w: `dtype` (F32 → fp32 FFMA kernel; BF16 / F16 → tcgen05 kernel with ANCHA_W_NK);
 * bias, residual, rope: f32; out: out_dtype. No allocation. */
typedef struct {
    int m, n, k;
    int dtype, out_dtype, weight_layout;
    int64_t ldx, ldw, ldout, ldres;
    int act;
    int rope_width, rope_tokens, rope_div;  /* rope_width = 0: no rotary epilogue */
    const float* row_scale;  /* optional device [m]: row r of x·w is multiplied by row_scale[r]
                                before the bias (the unit-norm of rows, applied after the GEMM
                                instead of to x); null = 1 */
} ancha_linear_desc;

ANCHA_API int ancha_linear_fwd(const ancha_linear_desc* desc, const void* x, const void* w,
                     const float* bias, const float* residual, const float* rope,
                     void* out, void* stream);

/* Device workspace bytes ancha_linear_fwd_ws can use for `desc`: with a rotary epilogue on the
 * tensor-core path (BF16 / F16), 1 KiB per table token; otherwise 0. */
ANCHA_API int ancha_linear_workspace(const ancha_linear_desc* desc, size_t* bytes);

/* ancha_linear_fwd with a caller-owned device workspace (16-byte aligned, at least the
 * ancha_linear_workspace bytes; NULL or smaller = the ancha_linear_fwd path). With it the
 * tensor-core rotary epilogue reads the table rewritten pair-major into the workspace
 * ([2][32][tokens] × the (cos, cos, sin, sin) entries of each column pair: the same arithmetic,
 * coalesced loads) instead of the [4, tokens, 64] rows. */
ANCHA_API int ancha_linear_fwd_ws(const ancha_linear_desc* desc, const void* x, const void* w,
                        const float* bias, const float* residual, const float* rope, void* out,
                        void* workspace, size_t workspace_bytes, void* stream);

/* ------------------------------------------------------------------------------------ *
 * Spectral DSP (replaces crates/ancha-audio/src/dsp.rs and chunk.rs on the device)     *
 * ------------------------------------------------------------------------------------ */

/* Centered periodic-Hann STFT (n_fft 2048, reflect padding, unnormalised FFT) of `chunks`
 * stereo chunks `audio[c][ch][samples]` into the model layout
 * `packed[c][frame][(bin·2 + ch)·2 + re/im]`, frames = samples / hop + 1 (dsp.rs:52-79,
 * runtime.rs:148-162). */
ANCHA_API int ancha_stft_fwd(const float* audio, int chunks, int samples, int hop, float* packed,
                   void* stream);

/* Complex-mask multiply + inverse STFT: for every chunk, stem and channel, multiply the
 * packed spectrum by masks[c][stem][bin·2+ch][re/im][frame] and invert (zero Im at DC and
 * Nyquist, zero Re at DC if zero_dc, 1/n scale, window-square normalised overlap-add,
 * dsp.rs:82-133, runtime.rs:181-201) into out[c][stem][ch][samples]. `scratch` holds
 * chunks·stems·2·frames·2048 floats followed by one int status word that the call sets to
 * a non-zero value if a sample had no window support ("iSTFT has an uncovered sample"). */
ANCHA_API int ancha_istft_masked(const float* packed, const float* masks, int chunks, int stems,
                       int samples, int hop, int zero_dc, float* scratch, float* out,
                       void* stream);

/* ancha_istft_masked without caller scratch, for callers that cannot allocate device memory:
 * a host whose allocator owns the whole device (a caching pool or fixed arenas that hand
 * out no extra buffers), or a real-time audio thread that must not block on cudaMalloc,
 * which can synchronise the device. No counterpart in the reference; same arguments and
 * results as ancha_istft_masked.
 *
 * The frames go through a fixed 24 MiB device array inside the library (6 Mi floats per
 * device), processed one chunk and as many stems as fit at a time; the call allocates
 * nothing. The array is part of the library's device code, so it is resident on every device
 * where the library's DSP kernels are loaded, whether or not this entry point is called. Limit: one chunk-stem needs 2·frames·2048 floats, so frames = samples / hop + 1
 * must be at most 1536; larger calls fail with ANCHA_E_INVALID and a message naming the
 * sizes. `status` is an optional DEVICE pointer to one int: the call sets it to 0, or to a
 * non-zero value if a sample had no window support; no other memory needs to start at zero.
 * The first call on each device (with that device current) looks up the scratch address and
 * builds the DSP tables, synchronising the stream once: make it before any stream capture.
 * The scratch is shared by all calls on a device, so calls that can overlap in time (other
 * streams, or host threads without ordering between them) race; serialise them on one
 * stream. */
ANCHA_API int ancha_istft_masked_static(const float* packed, const float* masks, int chunks,
                       int stems, int samples, int hop, int zero_dc, float* out, int* status,
                       void* stream);

/* Linear-fade overlap-add of `chunks` chunk outputs y[c][planes][chunk] starting at
 * starts[c] (host array, ascending) into sums[planes][length] and weights[length], in
 * chunk order (chunk.rs:26-75). */
ANCHA_API int ancha_ola_add(const float* y, int chunks, int planes, int chunk, int overlap,
                  const int64_t* starts, int64_t length, float* sums, float* weights,
                  void* stream);

/* ------------------------------------------------------------------------------------ *
 * Model API (replaces Roformer::load / forward, crates/ancha-models/src/network.rs)   *
 * ------------------------------------------------------------------------------------ */

typedef struct ancha_model ancha_model;

/* Load `package_dir/manifest.json` + `model.safetensors` (strict schema-1 checks, SHA-256
 * verification, load-time folding) onto `device` (network.rs:80-278, weights.rs:29-176). */
ANCHA_API int ancha_model_load(const char* package_dir, int device, int precision, ancha_model** out);

/* Model shape queries. */
ANCHA_API int ancha_model_info(const ancha_model* model, int* stems, int* bands, int* dim,
                     int* bins, int* chunk_samples, int* hop, int* overlap);

/* Masks for `chunks` spectra: spectrum[c][frames][bins·4] (device, packed as above) →
 * masks[c][stem][bins·2][2][frames] (device) (network.rs:301-400). Checks *cancel (host
 * memory, may be NULL) between layers (network.rs:334,367). The handle is bound to its
 * device and is not re-entrant. */
ANCHA_API int ancha_model_forward(ancha_model* model, const float* spectrum, int chunks, int frames,
                        float* masks, const volatile int* cancel, void* stream);

ANCHA_API void ancha_model_free(ancha_model* model);

/* ------------------------------------------------------------------------------------ *
 * MDX23C model API (replaces Mdx23c::load / forward, crates/ancha-models/src/mdx23c.rs) *
 * ------------------------------------------------------------------------------------ */

typedef struct ancha_mdx23c ancha_mdx23c;

/* Load an MDX23C (TFC-TDF v3) package: `package_dir/manifest.json` (strict schema-1
 * manifest whose config has family "mdx23c", checked like Config::validate,
 * mdx23c.rs:76-122) + `model.safetensors` (F32, SHA-256 verified, every tensor used) onto
 * `device` (Mdx23c::load / build, mdx23c.rs:372-418). */
ANCHA_API int ancha_mdx23c_load(const char* package_dir, int device, int precision, ancha_mdx23c** out);

/* Shape queries: bins, native frames, n_fft, hop, overlap, stems, and the number of
 * tensors the package held (Mdx23c::tensor_count). Any pointer may be NULL. */
ANCHA_API int ancha_mdx23c_info(const ancha_mdx23c* model, int* bins, int* frames, int* n_fft, int* hop,
                      int* overlap, int* stems, int* tensor_count);

/* spectrum[batch][4][bins][frames] (device f32: L.re, L.im, R.re, R.im) →
 * out[batch][stems·4][bins][frames] (device f32 spectra, not masks) (Mdx23c::forward,
 * mdx23c.rs:420-481). batch 1..4; frames a multiple of 2^scales (any such count, not only
 * the manifest's); ANCHA_E_INVALID otherwise. Checks *cancel (host memory, may be NULL)
 * before every block (mdx23c.rs:307). The handle is bound to its device and is not
 * re-entrant. */
ANCHA_API int ancha_mdx23c_forward(ancha_mdx23c* model, const float* spectrum, int batch, int frames,
                         float* out, const volatile int* cancel, void* stream);

/* mdx23c_runtime::separate without file I/O (src/mdx23c_runtime.rs:135-248) on the model's
 * GPU: host planes[2][samples] (f32, 44.1 kHz) → host stems_out[stems][2][samples]. UVR chunks
 * (zero borders, step = chunk / overlap), centred n_fft STFT packed as spectral::pack, the
 * network, each stem's inverse STFT, rectangular overlap-add divided by `overlap`, all on the
 * device; chunks entirely inside the zero borders are skipped (the reference's default).
 * overlap 0 = the manifest's; batch = chunks per forward (1..4, 0 = 4). *seconds_out (may be
 * NULL) = wall time. ANCHA_E_NONFINITE for a non-finite model output. */
ANCHA_API int ancha_mdx23c_separate_pcm(ancha_mdx23c* model, const float* planes, int64_t samples, int overlap,
                              int batch, const volatile int* cancel, float* stems_out, double* seconds_out);

/* The UVR chunk plan of a `samples`-long track (OverlapPlan::new, mdx23c_runtime.rs:84-115):
 * step = chunk / overlap, border = chunk − step, right pad, padded length and chunk count
 * (chunk i starts at i·step of the zero-bordered track). Any output pointer may be NULL.
 * Host-only. */
ANCHA_API int ancha_mdx23c_plan(int64_t samples, int64_t chunk_samples, int overlap, int64_t* step, int64_t* border,
                      int64_t* pad, int64_t* padded, int64_t* chunks);

ANCHA_API void ancha_mdx23c_free(ancha_mdx23c* model);

/* ------------------------------------------------------------------------------------ *
 * Classic MDX ONNX graphs (crates/ancha-models/src/mdx.rs)                             *
 * ------------------------------------------------------------------------------------ */

/* Read an ONNX model (`bytes` bytes at `onnx`, host memory) and build the classic MDX
 * executable graph as Graph::from_bytes does (mdx.rs:161-472): opset 13, one input and one
 * output, FLOAT initializers of at most four dims, the op set Conv / ConvTranspose / Relu /
 * Transpose / MatMul / Add / Mul / BatchNormalization with their attribute allow-list, and
 * with `optimized` the folding of a BatchNormalization into the ConvTranspose that is its
 * only producer. Reports the graph's node count, scheduled instructions, folded
 * BatchNormalizations and constants (any pointer may be NULL). Host-only, no device work;
 * ANCHA_E_INVALID with the reference's message for a graph it would reject. */
ANCHA_API int ancha_mdx_graph_inspect(const void* onnx, size_t bytes, int optimized, int* nodes, int* instructions,
                            int* folded_bn, int* constants);

typedef struct ancha_mdx ancha_mdx;

/* Build the graph as ancha_mdx_graph_inspect does and upload its constants to `device`
 * (Graph::from_bytes, mdx.rs:161-472). */
ANCHA_API int ancha_mdx_load(const void* onnx, size_t bytes, int optimized, int device, ancha_mdx** out);

/* Output shape of the graph for an NCHW input shape (host-only shape inference);
 * ANCHA_E_INVALID when an operation's shapes disagree. */
ANCHA_API int ancha_mdx_output_shape(const ancha_mdx* graph, const int64_t input_shape[4], int64_t output_shape[4]);

/* Graph::forward (mdx.rs:474-568) on the device: x (device f32, NCHW `input_shape`) → out
 * (device f32 of ancha_mdx_output_shape). Conv / ConvTranspose with any stride, padding,
 * dilation, groups and output padding, Relu, Transpose, MatMul and Add / Mul with NCHW
 * broadcasting, BatchNormalization as its per-channel affine form. Checks *cancel (host
 * memory, may be NULL) before every operation. Intermediate values use stream-ordered
 * allocations freed after their last consumer. Not re-entrant per handle. */
ANCHA_API int ancha_mdx_forward(ancha_mdx* graph, const float* x, const int64_t input_shape[4], float* out,
                      const volatile int* cancel, void* stream);

/* Options of the classic MDX task: the MdxConfig fields of a registered checkpoint
 * (mdx.rs:21-97), given explicitly, and the task options of MdxOptions (mdx_runtime.rs:22-34). */
typedef struct {
    int n_fft, hop, bins, frames;  /* n_fft/2 = 2^k, 3·2^k or 5·2^k, at most 8192 */
    double compensate;
    double overlap;                /* < 0: chunks every chunk − n_fft samples; else 0..0.95 */
    int denoise;                   /* (f(x) − f(−x)) / 2 */
    int batch;                     /* chunks per graph call, 1..4 */
} ancha_mdx_task;

/* separate_mdx without file I/O (src/mdx_runtime.rs:84-248) on the graph's GPU: host
 * planes[2][samples] → host predicted[2][samples] and residual[2][samples] (= input −
 * predicted). UVR trim / pad chunking, centred STFT packed [4][bins][frames] with the three
 * lowest bins zeroed, the graph, the inverse STFT and the Hann-weighted overlap-add divided by
 * the summed weights, times `compensate`, all on the device. *seconds_out may be NULL. */
ANCHA_API int ancha_mdx_separate_pcm(ancha_mdx* graph, const ancha_mdx_task* task, const float* planes, int64_t samples,
                           const volatile int* cancel, float* predicted, float* residual, double* seconds_out);

/* Graph::forward's conv_gemm option (mdx.rs:472-530, spatial.rs:21-67; the reference's CUDA
 * default, backend.rs:63): ungrouped, undilated convolutions with constant weights in the
 * patch-gather geometries (1x1, 3x3 with padding 1, 2x2 with stride 2) run as the weights
 * [co][ci*kh*kw] times a patch matrix, 2x2 / stride-2 ConvTranspose layers as one GEMM with
 * rows (co, dy, dx) plus a scatter, and a MatMul by a constant 2-D right operand as one GEMM,
 * for every later ancha_mdx_forward / ancha_mdx_separate_pcm on this handle.
 * precision < 0: off (the default; every operation on its direct kernel).
 * ANCHA_PRECISION_F32: those GEMMs in fp32 on FFMA. ANCHA_PRECISION_BF16 / _F16: on the
 * tensor cores with 16-bit weights and operands (patches; MatMul inputs cast once) and fp32
 * accumulation and output. Other convolutions keep their direct kernels. Uploads converted
 * weights; not to be called while a forward on this handle is in flight. */
ANCHA_API int ancha_mdx_set_gemm(ancha_mdx* graph, int precision);

ANCHA_API void ancha_mdx_free(ancha_mdx* graph);

/* ------------------------------------------------------------------------------------ *
 * Task API (replaces backend::separate / runtime::separate, src/backend.rs:145-199)    *
 * ------------------------------------------------------------------------------------ */

typedef struct {
    const char* input;         /* WAV path (PCM16/24/32 or float32, mono or stereo, 44.1 kHz) */
    const char* model;         /* package directory                                           */
    const char* output;        /* output directory (published atomically)                     */
    int64_t chunk_samples;     /* 0 = manifest value (runtime.rs:52-57)                       */
    int overlap;               /* 0 = manifest value                                          */
    int precision;             /* ANCHA_PRECISION_*                                           */
    int batch_chunks;          /* chunks per model call on each device (0 = automatic)        */
    double start_seconds;      /* decode window (DecodeOptions)                                */
    double duration_seconds;   /* <= 0: to the end                                             */
} ancha_separate_opts;

/* Separate a track on `n_devices` GPUs (chunks sharded in contiguous ranges, one host
 * thread per GPU). Writes <stem>.wav and run.json into opts->output and returns the run
 * report JSON in *run_json (free with ancha_free_string). `progress(done, total, user)` may
 * be NULL. */
ANCHA_API int ancha_separate(const ancha_separate_opts* opts, int n_devices, const int* devices,
                   void (*progress)(size_t done, size_t total, void* user), void* user,
                   const volatile int* cancel, char** run_json);

/* In-memory form of ancha_separate for host PCM: planes[2][samples] (host, f32) →
 * stems_out[stems][2][samples] (host, f32). Used by benchmarks and the SDK. */
ANCHA_API int ancha_separate_pcm(ancha_model* const* models, int n_models, const float* planes,
                       int64_t samples, int64_t chunk_samples, int overlap, int batch_chunks,
                       const volatile int* cancel, float* stems_out, double* seconds_out);

/* Chunk plan of a `samples`-long track (chunk.rs:1-23, runtime.rs:103-111): number of
 * chunks, reflect border and padded length. chunk_samples / overlap must be explicit here
 * (the model defaults come from ancha_model_info). Host-only. */
ANCHA_API int ancha_chunk_plan(int64_t samples, int64_t chunk_samples, int overlap, int64_t* chunks,
                     int64_t* border, int64_t* length);

/* Padded-track samples [*lo, *hi) covered by chunks [first, last) of that plan (both 0 for
 * an empty range). Host-only. */
ANCHA_API int ancha_chunk_span(int64_t samples, int64_t chunk_samples, int overlap, int64_t first,
                     int64_t last, int64_t* lo, int64_t* hi);

/* One shard of ancha_separate_pcm: chunks [first, last) of the plan of host planes[2][samples]
 * on `model`'s GPU, returning their weighted overlap-add over the span of
 * ancha_chunk_span (host sums[stems·2][hi − lo], weights[hi − lo]). Adding the spans of
 * disjoint chunk ranges at their offsets, dividing by the summed weights and cropping the
 * border gives the stems (chunk.rs:77-88, runtime.rs:210-225): this is how one track is
 * split over processes, one per GPU (ancha_b200.distributed). chunk_samples / overlap 0 take
 * the model defaults. */
ANCHA_API int ancha_separate_span(ancha_model* model, const float* planes, int64_t samples,
                        int64_t chunk_samples, int overlap, int batch_chunks, int64_t first,
                        int64_t last, const volatile int* cancel, float* sums, float* weights);

/* Track samples [*lo, *hi) that chunks [first, last) of the plan read (their reflect-padded
 * gather; both 0 for an empty range). A process separating that shard needs only this slice
 * of the PCM. Host-only; no reference counterpart beyond the padding rule of runtime.rs:103-116
 * and chunk.rs:1-23. */
ANCHA_API int ancha_chunk_pcm_range(int64_t samples, int64_t chunk_samples, int overlap, int64_t first,
                          int64_t last, int64_t* lo, int64_t* hi);

/* Device-resident shard of one track (one process per GPU): chunks [first, last) of the plan of a
 * track of `samples` samples per channel, read from `pcm` (device [2][pcm_len], holding track
 * samples [pcm_lo, pcm_lo + pcm_len), which must contain ancha_chunk_pcm_range's slice), overlap-
 * added into device sums[stems·2][hi − lo] and weights[hi − lo] over the span [lo, hi) of
 * ancha_chunk_span (the call zeroes them). Enqueued on `stream` without a host synchronisation;
 * ancha_separate_status reports the model's status words. Spans of different shards meet only in
 * their chunk-overlap columns: adding those (ancha_span_add), dividing and cropping
 * (ancha_span_finish) gives the stems (chunk.rs:77-88, runtime.rs:210-225). */
ANCHA_API int ancha_separate_span_device(ancha_model* model, const float* pcm, int64_t pcm_lo, int64_t pcm_len,
                               int64_t samples, int64_t chunk_samples, int overlap, int batch_chunks,
                               int64_t first, int64_t last, float* sums, float* weights, void* stream);

/* sums[p][offset + j] += piece[p][j] and weights[offset + j] += piece[planes][j] for j < count:
 * add overlap-add columns received from another shard (piece: device [planes + 1][count], the
 * sums rows then the weights row) into a span (device sums[planes][span], weights[span]). */
ANCHA_API int ancha_span_add(float* sums, float* weights, int planes, int64_t span, int64_t offset,
                   const float* piece, int64_t count, void* stream);

/* out[p][n] = sums[p][offset + n] / weights[offset + n] for n < count (out: device, row stride
 * ld): the stems of a span's owned, cropped range. `flag` (device int) gets bit 4 for a zero
 * weight and bit 1 for a non-finite value (runtime.rs:210-225). */
ANCHA_API int ancha_span_finish(const float* sums, const float* weights, int planes, int64_t span, int64_t offset,
                      int64_t count, float* out, int64_t ld, int* flag, void* stream);

/* Device-resident form for one model: planes[2][samples] (device) → stems[stems][2][samples]
 * (device), everything enqueued on `stream` without a host synchronisation (the model's
 * pipeline buffers are allocated on the first call and reused). Status words (non-finite
 * output, uncovered sample) stay on the device until ancha_separate_status. Replaces the
 * per-chunk loop of src/runtime.rs:117-225 for inputs already in HBM. */
ANCHA_API int ancha_separate_device(ancha_model* model, const float* planes, int64_t samples,
                                    int64_t chunk_samples, int overlap, int batch_chunks,
                                    float* stems, void* stream);

/* Synchronise `stream` and report the status words of the last ancha_separate_device. */
ANCHA_API int ancha_separate_status(ancha_model* model, void* stream);

ANCHA_API void ancha_free_string(char* s);

#ifdef __cplusplus
}
#endif

#endif /* ANCHA_B200_H */
