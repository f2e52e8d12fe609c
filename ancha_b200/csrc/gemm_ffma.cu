// FFMA GEMM with the RoFormer epilogues (bias, GELU / tanh / GLU, interleaved RoPE,
// residual). This is the fp32 arithmetic path of the engine (precision F32) and the
// on-device cross-check of the tcgen05 kernels. 128×128 output tile per CTA, k-step 8,
// 256 threads as 16×16, each owning rows {4ty, 64+4ty}+0..3 and columns {4tx, 64+4tx}+0..3
// so that every RoPE / GLU column pair (2j, 2j+1) sits in one thread. The next k-slab is
// fetched into registers while the current one is multiplied.
#include "gemm.cuh"

namespace ancha {
namespace {

constexpr int BM = 128, BN = 128, BK = 8;

template <typename T>
__device__ __forceinline__ float ld_elem(const void* base, int64_t idx) {
    return load_f(reinterpret_cast<const T*>(base) + idx);
}

// Apply bias / activation / RoPE / residual to 4 consecutive columns (c0 % 4 == 0) of
// row `row` and store them.
__device__ __forceinline__ void finish4(const GemmGroup& g, const GemmEpilogue& e, int row,
                                        int c0, float v[4]) {
    if (row >= g.m) return;
    if (e.row_mul) {
        const float r = e.row_mul[row];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] *= r;
    }
    if (g.bias) {
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (c0 + j < g.n) v[j] += g.bias[c0 + j];
    }
    if (e.act == ANCHA_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = gelu_erf(v[j]);
    } else if (e.act == ANCHA_ACT_TANH) {
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = tanhf(v[j]);
    }
    if (e.rope && c0 < 2 * e.rope_width) {
        const int key = c0 >= e.rope_width;
        const int token = (row / e.rope_div) % e.rope_tokens;
        const int d = c0 % e.rope_hd;
        const float* cs = e.rope + ((size_t)(key * 2) * e.rope_tokens + token) * e.rope_hd + d;
        const float* sn = cs + (size_t)e.rope_tokens * e.rope_hd;
        float r[4];
        r[0] = v[0] * cs[0] + v[1] * sn[0];
        r[1] = v[1] * cs[1] + v[0] * sn[1];
        r[2] = v[2] * cs[2] + v[3] * sn[2];
        r[3] = v[3] * cs[3] + v[2] * sn[3];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = r[j];
    }
    if (e.act == ANCHA_ACT_GLU) {
        // (value, gate) pairs → value·sigmoid(gate) at column c/2.
#pragma unroll
        for (int j = 0; j < 4; j += 2) {
            const int c = c0 + j;
            if (c + 1 < g.n) {
                const float o = v[j] * sigmoidf_(v[j + 1]);
                store_elt(g.out, (int64_t)row * g.ldo + c / 2, o, e.out_type);
            }
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const int c = c0 + j;
        if (c >= g.n) break;
        float o = v[j];
        if (g.residual) o += g.residual[(int64_t)row * g.ldr + c];
        store_elt(g.out, (int64_t)row * g.ldo + c, o, e.out_type);
    }
}

template <typename TA, typename TB, bool NK>
__global__ void __launch_bounds__(256)
gemm_ffma_kernel(GemmGroup single, const GemmGroup* __restrict__ groups, GemmEpilogue e) {
    const GemmGroup g = groups ? groups[blockIdx.z] : single;
    const int m0 = blockIdx.y * BM, n0 = blockIdx.x * BN;
    if (m0 >= g.m || n0 >= g.n) return;
    __shared__ float As[BK][BM + 4];
    __shared__ float Bs[BK][BN + 4];
    const int t = threadIdx.x, tx = t % 16, ty = t / 16;

    // Loader mapping: A rows t/2, k (t%2)*4..+3. B: NK as A; KN k = t/32, n = (t%32)*4..+3.
    const int ar = t / 2, ak = (t % 2) * 4;
    float ra[4], rb[4];
    auto fetch = [&](int k0) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int k = k0 + ak + j, r = m0 + ar;
            ra[j] = (r < g.m && k < g.k) ? ld_elem<TA>(g.a, (int64_t)r * g.lda + k) : 0.f;
        }
        if (NK) {
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int k = k0 + ak + j, n = n0 + ar;
                rb[j] = (n < g.n && k < g.k) ? ld_elem<TB>(g.b, (int64_t)n * g.ldb + k) : 0.f;
            }
        } else {
            const int k = k0 + t / 32, nb = n0 + (t % 32) * 4;
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                const int n = nb + j;
                rb[j] = (n < g.n && k < g.k) ? ld_elem<TB>(g.b, (int64_t)k * g.ldb + n) : 0.f;
            }
        }
    };
    auto stash = [&]() {
#pragma unroll
        for (int j = 0; j < 4; ++j) As[ak + j][ar] = ra[j];
        if (NK) {
#pragma unroll
            for (int j = 0; j < 4; ++j) Bs[ak + j][ar] = rb[j];
        } else {
#pragma unroll
            for (int j = 0; j < 4; ++j) Bs[t / 32][(t % 32) * 4 + j] = rb[j];
        }
    };

    float acc[8][8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
#pragma unroll
        for (int j = 0; j < 8; ++j) acc[i][j] = 0.f;

    fetch(0);
    for (int k0 = 0; k0 < g.k; k0 += BK) {
        __syncthreads();
        stash();
        __syncthreads();
        if (k0 + BK < g.k) fetch(k0 + BK);
#pragma unroll
        for (int kk = 0; kk < BK; ++kk) {
            float a[8], b[8];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = As[kk][ty * 4 + i];
                a[4 + i] = As[kk][64 + ty * 4 + i];
                b[i] = Bs[kk][tx * 4 + i];
                b[4 + i] = Bs[kk][64 + tx * 4 + i];
            }
#pragma unroll
            for (int i = 0; i < 8; ++i)
#pragma unroll
                for (int j = 0; j < 8; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        const int row = m0 + (i < 4 ? ty * 4 + i : 64 + ty * 4 + (i - 4));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
            float v[4] = {acc[i][h * 4], acc[i][h * 4 + 1], acc[i][h * 4 + 2], acc[i][h * 4 + 3]};
            finish4(g, e, row, n0 + h * 64 + tx * 4, v);
        }
    }
}

template <typename TA, typename TB>
void launch_typed(dim3 grid, cudaStream_t s, int b_nk, const GemmGroup& single,
                  const GemmGroup* groups, const GemmEpilogue& e) {
    if (b_nk) gemm_ffma_kernel<TA, TB, true><<<grid, 256, 0, s>>>(single, groups, e);
    else gemm_ffma_kernel<TA, TB, false><<<grid, 256, 0, s>>>(single, groups, e);
}

}  // namespace

int gemm_ffma(const GemmGroup& single, const GemmGroup* groups, int count, int max_m,
              int max_n, int a_type, int b_type, int b_nk, const GemmEpilogue& epi,
              cudaStream_t stream) {
    if (count <= 0 || max_m <= 0 || max_n <= 0) return ANCHA_OK;
    if (count > 65535 || ceil_div(max_m, BM) > 65535)
        return fail(ANCHA_E_INVALID, "gemm: grid too large");
    dim3 grid((unsigned)ceil_div(max_n, BN), (unsigned)ceil_div(max_m, BM), (unsigned)count);
    using bf = __nv_bfloat16;
    if (a_type == ELT_F32 && b_type == ELT_F32) launch_typed<float, float>(grid, stream, b_nk, single, groups, epi);
    else if (a_type == ELT_BF16 && b_type == ELT_BF16) launch_typed<bf, bf>(grid, stream, b_nk, single, groups, epi);
    else if (a_type == ELT_F16 && b_type == ELT_F16) launch_typed<__half, __half>(grid, stream, b_nk, single, groups, epi);
    else return fail(ANCHA_E_UNSUPPORTED, "gemm: mixed operand types");
    return check_launch("gemm_ffma");
}

}  // namespace ancha
