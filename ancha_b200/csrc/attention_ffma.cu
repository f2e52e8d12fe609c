// Single-pass exact attention on the FFMA pipes (precision F32, and the on-device check of
// the tensor-core attention). One CTA per (64 queries, head, group); two threads per query,
// each owning 32 of the 64 channels. Key / value tiles of 64 tokens are staged in shared
// memory as f32; a tile's 64 scores stay in registers, so the online-softmax rescale runs
// once per tile (the order of ancha-kernels/src/attention.rs::tiled with a 64-key tile).
#include "attention.cuh"

namespace ancha {
namespace {

constexpr int TQ = 64, TK = 64, HALF = 32, PADH = HALF + 1;

template <typename T>
__global__ void __launch_bounds__(128) attention_ffma_kernel(AttnArgs a) {
    // [key][half][channel] with the halves 33 floats apart: the two halves of a warp read
    // different banks.
    __shared__ float ks[TK][2][PADH];
    __shared__ float vs[TK][2][PADH];
    const T* q = reinterpret_cast<const T*>(a.q);
    const T* k = reinterpret_cast<const T*>(a.k);
    const T* v = reinterpret_cast<const T*>(a.v);
    const int head = blockIdx.y;
    const int64_t group = blockIdx.z;
    const int64_t base = attn_group_row(a, group);
    const int t = threadIdx.x, qi = t / 2, half = t % 2;
    const int token = blockIdx.x * TQ + qi;
    const bool valid = token < a.tokens;

    float qr[HALF], acc[HALF];
    {
        const int64_t row = base + (int64_t)(valid ? token : 0) * a.token_stride;
        const T* qp = q + row * a.ld + a.q_col + head * a.head_dim + half * HALF;
#pragma unroll
        for (int d = 0; d < HALF; ++d) {
            qr[d] = (valid && half * HALF + d < a.head_dim) ? load_f(qp + d) : 0.f;
            acc[d] = 0.f;
        }
    }
    float m = -INFINITY, l = 0.f;
    for (int k0 = 0; k0 < a.tokens; k0 += TK) {
        __syncthreads();
        // 64 keys × 64 channels of k and v: thread t copies channels (t%16)*4..+3 of
        // keys t/16 + 8·i.
        for (int i = 0; i < 8; ++i) {
            const int key = t / 16 + 8 * i, c = (t % 16) * 4;
            const int tok = k0 + key;
            float kv[4] = {0.f, 0.f, 0.f, 0.f}, vv[4] = {0.f, 0.f, 0.f, 0.f};
            if (tok < a.tokens) {
                const int64_t row = base + (int64_t)tok * a.token_stride;
                const T* kp = k + row * a.ld + a.k_col + head * a.head_dim + c;
                const T* vp = v + row * a.ld + a.v_col + head * a.head_dim + c;
#pragma unroll
                for (int j = 0; j < 4; ++j) {
                    if (c + j < a.head_dim) {
                        kv[j] = load_f(kp + j);
                        vv[j] = load_f(vp + j);
                    }
                }
            }
#pragma unroll
            for (int j = 0; j < 4; ++j) {
                ks[key][(c + j) / HALF][(c + j) % HALF] = kv[j];
                vs[key][(c + j) / HALF][(c + j) % HALF] = vv[j];
            }
        }
        __syncthreads();
        const int nk = min(TK, a.tokens - k0);
        float s[TK];
        float tile_max = -INFINITY;
#pragma unroll
        for (int j = 0; j < TK; ++j) {
            float p = 0.f;
#pragma unroll
            for (int d = 0; d < HALF; ++d) p = fmaf(qr[d], ks[j][half][d], p);
            p += __shfl_xor_sync(0xffffffffu, p, 1);
            s[j] = j < nk ? p : -INFINITY;
            tile_max = fmaxf(tile_max, s[j]);
        }
        const float m_new = fmaxf(m, tile_max);
        const float corr = expf(m - m_new);
        l *= corr;
#pragma unroll
        for (int d = 0; d < HALF; ++d) acc[d] *= corr;
#pragma unroll
        for (int j = 0; j < TK; ++j) {
            const float p = expf(s[j] - m_new);
            l += p;
#pragma unroll
            for (int d = 0; d < HALF; ++d) acc[d] = fmaf(p, vs[j][half][d], acc[d]);
        }
        m = m_new;
    }
    if (!valid) return;
    const int64_t row = base + (int64_t)token * a.token_stride;
    float scale = 1.f / l;
    if (a.gate) {
        const float gl = load_f(reinterpret_cast<const T*>(a.gate) + row * a.ld + a.gate_col + head);
        scale /= 1.f + expf(-gl);
    }
    T* op = reinterpret_cast<T*>(a.out) + row * a.out_ld + a.out_col + head * a.head_dim + half * HALF;
#pragma unroll
    for (int d = 0; d < HALF; ++d)
        if (half * HALF + d < a.head_dim) store_f(op + d, acc[d] * scale);
}

}  // namespace

int attention_ffma(const AttnArgs& a, cudaStream_t stream) {
    if (a.groups == 0 || a.tokens == 0) return ANCHA_OK;
    if (a.groups > 65535 || a.heads > 65535)
        return fail(ANCHA_E_INVALID, "attention: grid too large");
    if (a.head_dim <= 0 || a.head_dim > 64 || a.head_dim % 4)
        return fail(ANCHA_E_UNSUPPORTED, "attention: head_dim must be a multiple of 4 up to 64");
    dim3 grid((unsigned)ceil_div(a.tokens, TQ), (unsigned)a.heads, (unsigned)a.groups);
    if (a.elt == ELT_BF16) attention_ffma_kernel<__nv_bfloat16><<<grid, 128, 0, stream>>>(a);
    else if (a.elt == ELT_F16) attention_ffma_kernel<__half><<<grid, 128, 0, stream>>>(a);
    else attention_ffma_kernel<float><<<grid, 128, 0, stream>>>(a);
    return check_launch("attention_ffma");
}

}  // namespace ancha
