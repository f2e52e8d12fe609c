// GEMM problem descriptors shared by the FFMA and tcgen05 GEMM kernels.
#pragma once
#include "common.cuh"

namespace ancha {

// One GEMM problem: out[m, n'] = epilogue(sum_k a[m, k] · b(k, n)).
// b(k, n) = b[n·ldb + k] (NK, PyTorch [out, in]) or b[k·ldb + n] (KN, Burn [in, out]).
struct GemmGroup {
    const void* a;
    const void* b;
    const float* bias;      // [n] or null
    const float* residual;  // [m, n] f32 or null (row stride ldr)
    void* out;              // [m, n] (n/2 for GLU), row stride ldo
    int m, n, k;
    int64_t lda, ldb, ldr, ldo;
    // Tensor-core fp32 (gemm_tc, bf16 operands): a and b each hold three bf16 planes
    // [3][m][lda] / [3][n][ldb] of a three-way split (split3_rows), and the product is the sum
    // of the six significant plane products hi·hi, hi·mid, mid·hi, hi·lo, lo·hi, mid·mid, run
    // as one K loop of 6·k (the dropped terms are below 2^-24 of the product).
    bool split3;
};

// Epilogue shared by every group of one launch.
struct GemmEpilogue {
    int act;            // ANCHA_ACT_*
    int out_type;       // ELT_F32 / ELT_BF16 / ELT_F16
    const float* rope;  // [4, rope_tokens, 64] or null
    int rope_width;     // rotate columns [0, 2·rope_width)
    int rope_tokens;
    int rope_div;       // token = (row / rope_div) % rope_tokens
    int rope_hd;        // head width of the table (columns per head)
    // Optional pair-major copy of the same table for the tensor-core epilogue:
    // [2 (query, key)][rope_hd / 2 pairs][rope_tokens] × (cos, sin) float2, where a pair's two
    // columns share the cosine and carry ∓sin. Lanes of a warp hold consecutive rows, so a
    // token-fastest table makes their loads coalesce. Null: the tensor-core path reads `rope`.
    const float* rope_pairs;
    // Optional pair-major general form of a [4, tokens, hd] table for the tensor-core epilogue:
    // [2][rope_hd / 2][rope_tokens] × (C0, C1, S0, S1) float4, the cosine-row and sine-row entries
    // of a pair's two columns (rope_quads_from_table); the columns rotate as
    // (x0·C0 + x1·S0, x1·C1 + x0·S1), exactly the `rope` table's arithmetic, with coalesced loads.
    const float* rope_quads;
    // Row-norm fusion (tensor-core path only; null / 0 = off). Sums of squares are kept per
    // 32-column chunk, chunk-major: ss[c / 32][r] for an m-row output.
    //   row_ss / row_ss_n: scale row r of A·Bᵀ by 1 / max(√Σ row_ss[r][·], 1e-12) before the
    //     bias (A holds unnormalised rows; their unit norm is applied here instead);
    //   res_ss / res_ss_n, res_col: the residual is read as res[r][c] · res_scale[r] · res_col[c]
    //     with res_scale from res_ss like above (a row normalisation the producer deferred);
    //   out16 / out16_col: also write the output, times out16_col[c] when set, in the operand
    //     type (f16 / bf16) as a dense [m][n] copy, the next GEMM's A operand;
    //   ss_out / ss16_out: write the per-chunk sums of squares of the output / of that copy.
    const float* row_ss;
    int row_ss_n;
    const float* res_ss;
    int res_ss_n;
    const float* res_col;
    void* out16;
    const float* out16_col;
    float* ss_out;
    float* ss16_out;
    // Per-plane statistics of the output (tensor-core path, one group): Σ v and Σ v² of rows
    // r are added (f64 atomics) into stats[r / stats_div]; the caller zeroes them. Null = off.
    double2* stats;
    int stats_div;
    // Per-row multiplier of A·Bᵀ (row_mul[r], applied before the bias; null = 1), the plug-in
    // API's row_scale. Both paths; the row-norm fusion's row_ss takes precedence.
    const float* row_mul;
};

// FFMA GEMM (fp32 accumulation). `groups` is a device array of `count` problems when
// non-null, else `single` is the one problem. A and B are f32, or both bf16, or both f16.
int gemm_ffma(const GemmGroup& single, const GemmGroup* groups, int count, int max_m,
              int max_n, int a_type, int b_type, int b_nk, const GemmEpilogue& epi,
              cudaStream_t stream);

// tcgen05 / TMA GEMM (bf16 or f16 operands, fp32 accumulation in TMEM) for one problem
// with NK weights; `ab_type` is the operand type of both A and B. Returns ANCHA_E_UNSUPPORTED when the operands do not meet its alignment
// rules (16-byte rows, k % 8 == 0), so the caller can use gemm_ffma instead.
int gemm_tc(const GemmGroup& g, int ab_type, const GemmEpilogue& epi, cudaStream_t stream);

// A batch of same-shape problems for the tcgen05 GEMM: problem g multiplies depth g of
// A [groups, m, k] by depth g % b_groups of B [b_groups, n, k] (B group j uses only its
// first group_n[j] rows when group_n is non-null) into depth g of out [groups, m, ldo].
struct GroupedGemm {
    const void* a;
    int64_t lda, a_group_stride;
    const void* b;
    int64_t ldb, b_group_stride;
    int m, n, k, groups, b_groups;
    const int* group_n;
    const float* bias;
    int64_t bias_group_stride;
    void* out;
    int64_t ldo, out_group_stride;
    // Three-plane bf16 operands (see GemmGroup::split3), plane-major over the groups: A plane p
    // of group g at a + (p · groups + g) · a_group_stride, B plane p of group g at
    // b + (p · b_groups + g) · b_group_stride.
    bool split3 = false;
};

// The general pair-major (C0, C1, S0, S1) form of a [4, tokens, hd] rotary table (see
// GemmEpilogue::rope_quads): quads[key][pair][token], 2 · (hd / 2) · tokens float4.
int rope_quads_from_table(const float* table, int tokens, int hd, void* quads, cudaStream_t stream);

int gemm_tc_grouped(const GroupedGemm& q, int ab_type, const GemmEpilogue& epi, cudaStream_t stream);

// Implicit-GEMM convolution on the tcgen05 kernel, no patch matrix:
// out[co][y·w + x] = Σ_tap Σ_c weight[co][tap·channels + c] · act[image][y + dy][x + dx][c]
// (+ residual[co][y·w + x]) over a channels-last activation act[batch][h][w][channels]
// (operand type), taps 9 = the 3 × 3 stencil (dy, dx) ∈ {−1, 0, 1}² row-major with zero
// padding 1, taps 1 = a 1 × 1 convolution. channels % 64 == 0; w a multiple or a divisor of
// 256. Epilogue: no activation / rotary / row-norm fusion.
struct ConvGemm {
    const void* weight;  // [co][taps · channels] (row stride ldw)
    int64_t ldw;
    int co;
    const void* x;       // [batch][h][w][channels]
    int batch, h, w, channels, image, taps;
    const float* residual;  // [co][ldo] f32 or null
    void* out;           // [co][ldo] of the epilogue's out_type
    int64_t ldo;
};

int gemm_tc_conv(const ConvGemm& q, int ab_type, const GemmEpilogue& epi, cudaStream_t stream);

}  // namespace ancha
