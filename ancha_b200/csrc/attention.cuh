// Attention operand addressing shared by the attention kernels.
#pragma once
#include "common.cuh"

namespace ancha {

struct AttnArgs {
    const void* q;
    const void* k;
    const void* v;
    const void* gate;  // null: ungated
    void* out;
    int groups, tokens, heads, head_dim;  // head_dim <= 64 (FFMA) or == 64 (tcgen05)
    int64_t ld, out_ld;
    int64_t group_inner, group_inner_stride, group_outer_stride, token_stride;
    int q_col, k_col, v_col, gate_col, out_col;
    int elt;  // q/k/v/gate/out element type (ELT_*)
};

// First row of group g (see ancha_attn_desc).
__host__ __device__ __forceinline__ int64_t attn_group_row(const AttnArgs& a, int64_t g) {
    return (g / a.group_inner) * a.group_outer_stride + (g % a.group_inner) * a.group_inner_stride;
}

int attention_ffma(const AttnArgs& a, cudaStream_t stream);
int attention_tc(const AttnArgs& a, cudaStream_t stream);
// fp32 operands (a.elt == ELT_F32) on the tensor cores from their three-plane bf16
// split: `planes` holds hi, mid, lo of the q / k / v source rows (same row indexing and column
// offsets as the source, row stride plane_ld elements), plane p at planes + p · plane_stride
// elements (see split3_rows_strided); the gate logits (read from a.gate with a.ld) and out are f32.
int attention_tc_split(const AttnArgs& a, const void* planes, int64_t plane_ld, int64_t plane_stride,
                       cudaStream_t stream);

}  // namespace ancha
