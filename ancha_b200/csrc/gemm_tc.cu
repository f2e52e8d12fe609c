// tcgen05 GEMM with the RoFormer epilogues: out = epilogue(A · Bᵀ) for f16 / bf16 A [rows, K]
// and B [N, K] (both K-major, PyTorch [out, in] weights), fp32 accumulation in TMEM.
//
// One CTA computes a 128 × BN tile: warp 0 lane 0 streams 64-wide K slabs of A and B with TMA
// (128-byte swizzle) into a STAGES-deep shared-memory ring, warp 1 lane 0 issues
// tcgen05.mma (M = 128, N = BN, K = 16 per instruction) into a TMEM accumulator and releases
// each slab with tcgen05.commit, then all four warps drain TMEM (warp w owns rows
// 32w..32w+31), apply bias / GELU / tanh / GLU / RoPE / residual and store. Two CTAs fit per
// SM, so one CTA's epilogue overlaps the other's main loop.
//
// Groups (grid z) batch independent problems of the same shape — the per-band mask
// estimator layers: A group g is depth g of a [groups, rows, K] array, B is depth
// g % b_groups of [b_groups, N_pad, K], and each group may use fewer than N columns.
#include "gemm.cuh"
#include "tc.cuh"

namespace ancha {
namespace {

constexpr int BM = 128, BK = 64;
constexpr int A_BYTES = BM * BK * 2;

struct TcParams {
    int m, n, k;          // rows per group, columns (max over groups), depth
    int groups, b_groups;
    const int* group_n;   // [b_groups] columns used per B group, or null (all n)
    void* out;
    int64_t ldo, out_group_stride;
    const float* bias;
    int64_t bias_group_stride;
    const float* residual;
    int64_t ldr;
    int act, out_type;
    const float* rope;
    int rope_width, rope_tokens, rope_div, rope_hd;
    uint32_t idesc;
    int* err;
};

template <int BN, int STAGES>
struct Smem {
    static constexpr int B_BYTES = BN * BK * 2;
    static constexpr int TILES = STAGES * (A_BYTES + B_BYTES);
    static constexpr int BYTES = 1024 + TILES + 8 * (2 * STAGES + 1) + 16;
};

__device__ __forceinline__ void store_vec(void* out, int out_type, int64_t idx, const float* v, int n,
                                          bool vec) {
    if (out_type == ELT_F32) {
        float* o = reinterpret_cast<float*>(out) + idx;
        if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                if (j < n) *reinterpret_cast<float4*>(o + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
            }
        } else {
            for (int j = 0; j < n; ++j) o[j] = v[j];
        }
    } else if (out_type == ELT_BF16) {
        __nv_bfloat16* o = reinterpret_cast<__nv_bfloat16*>(out) + idx;
        if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                if (j < n) {
                    uint4 u;
                    __nv_bfloat162 h[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) h[q] = __floats2bfloat162_rn(v[j + 2 * q], v[j + 2 * q + 1]);
                    memcpy(&u, h, 16);
                    *reinterpret_cast<uint4*>(o + j) = u;
                }
            }
        } else {
            for (int j = 0; j < n; ++j) o[j] = __float2bfloat16_rn(v[j]);
        }
    } else {
        __half* o = reinterpret_cast<__half*>(out) + idx;
        if (vec) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
                if (j < n) {
                    uint4 u;
                    __half2 h[4];
#pragma unroll
                    for (int q = 0; q < 4; ++q) h[q] = __floats2half2_rn(v[j + 2 * q], v[j + 2 * q + 1]);
                    memcpy(&u, h, 16);
                    *reinterpret_cast<uint4*>(o + j) = u;
                }
            }
        } else {
            for (int j = 0; j < n; ++j) o[j] = __float2half_rn(v[j]);
        }
    }
}

// Epilogue for 32 consecutive accumulator columns c0.. of one row.
__device__ __forceinline__ void epilogue32(const TcParams& p, int g, int row, int c0, int n_g,
                                           const uint32_t (&r)[32]) {
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
    const int nv = min(32, n_g - c0);  // valid columns (> 0)
    if (p.bias) {
        const float* b = p.bias + (int64_t)(g % p.b_groups) * p.bias_group_stride + c0;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nv) v[j] += b[j];
    }
    if (p.act == ANCHA_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = gelu_erf(v[j]);
    } else if (p.act == ANCHA_ACT_TANH) {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = tanhf(v[j]);
    }
    if (p.rope && c0 < 2 * p.rope_width) {
        const int key = c0 >= p.rope_width;
        const int token = (row / p.rope_div) % p.rope_tokens;
        const int d = c0 % p.rope_hd;
        const float* cs = p.rope + ((int64_t)(key * 2) * p.rope_tokens + token) * p.rope_hd + d;
        const float* sn = cs + (int64_t)p.rope_tokens * p.rope_hd;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {
            const float x0 = v[j], x1 = v[j + 1];
            v[j] = x0 * cs[j] + x1 * sn[j];
            v[j + 1] = x1 * cs[j + 1] + x0 * sn[j + 1];
        }
    }
    const int64_t obase = (int64_t)g * p.out_group_stride;
    const bool vec_ok = (nv == 32);
    if (p.act == ANCHA_ACT_GLU) {
        float o[32];
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j] = v[2 * j] * sigmoidf_(v[2 * j + 1]);
        const int no = nv / 2;
        const int64_t idx = obase + (int64_t)row * p.ldo + c0 / 2;
        if (p.out_type == ELT_F32 && vec_ok) {
            float* op = reinterpret_cast<float*>(p.out) + idx;
#pragma unroll
            for (int j = 0; j < 16; j += 4) *reinterpret_cast<float4*>(op + j) = make_float4(o[j], o[j + 1], o[j + 2], o[j + 3]);
        } else {
            for (int j = 0; j < no; ++j) store_elt(p.out, idx + j, o[j], p.out_type);
        }
        return;
    }
    if (p.residual) {
        const float* rr = p.residual + (int64_t)row * p.ldr + c0;
        if (vec_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 q = *reinterpret_cast<const float4*>(rr + j);
                v[j] += q.x; v[j + 1] += q.y; v[j + 2] += q.z; v[j + 3] += q.w;
            }
        } else {
            for (int j = 0; j < nv; ++j) v[j] += rr[j];
        }
    }
    store_vec(p.out, p.out_type, obase + (int64_t)row * p.ldo + c0, v, nv, vec_ok);
}

template <int BN, int STAGES>
__global__ void __launch_bounds__(128, 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const TcParams p) {
    using S = Smem<BN, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + STAGES * A_BYTES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILES);
    uint64_t* empty = full + STAGES;
    uint64_t* done = empty + STAGES;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(done + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int g = blockIdx.z;
    const int bg = g % p.b_groups;
    const int n0 = blockIdx.x * BN, m0 = blockIdx.y * BM;
    const int n_g = p.group_n ? p.group_n[bg] : p.n;
    if (n0 >= n_g) return;  // uniform across the CTA, before any barrier or TMEM use
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        mbar_init(done, 1);
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tma_a);
        prefetch_tma(&tma_b);
    }
    if (warp == 0) {
        tmem_alloc(tmem_slot, BN);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int kblocks = (p.k + BK - 1) / BK;

    if (warp == 0 && lane == 0) {
        // TMA producer.
        int issued = 0;
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % STAGES;
            const uint32_t round = kb / STAGES;
            if (!mbar_wait(&empty[s], (round & 1) ^ 1, abort, p.err)) break;
            mbar_arrive_expect_tx(&full[s], A_BYTES + S::B_BYTES);
            tma_load_3d(a_tiles + s * A_BYTES, &tma_a, &full[s], kb * BK, m0, g);
            tma_load_3d(b_tiles + s * S::B_BYTES, &tma_b, &full[s], kb * BK, n0, bg);
            ++issued;
        }
        if (*abort) {
            // Let the copies already in flight land before the CTA exits (bounded).
            const long long t0 = clock64();
            for (int kb = max(0, issued - STAGES); kb < issued; ++kb)
                while (!mbar_try_wait(&full[kb % STAGES], (kb / STAGES) & 1) && clock64() - t0 < kWaitCycles) {
                }
        }
    } else if (warp == 1 && lane == 0) {
        // UMMA issuer.
        for (int kb = 0; kb < kblocks; ++kb) {
            const int s = kb % STAGES;
            if (!mbar_wait(&full[s], (kb / STAGES) & 1, abort, p.err)) break;
            tc_fence_after();
            const uint32_t a_addr = smem_u32(a_tiles + s * A_BYTES);
            const uint32_t b_addr = smem_u32(b_tiles + s * S::B_BYTES);
#pragma unroll
            for (int kk = 0; kk < BK / 16; ++kk)
                umma_f16(tmem, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32), p.idesc,
                         (kb | kk) != 0);
            umma_commit(&empty[s]);
        }
        umma_commit(done);
    }
    __syncwarp();
    // Epilogue: all four warps.
    const bool ok = __all_sync(0xffffffffu, mbar_wait(done, 0, abort, p.err));
    tc_fence_after();
    if (ok) {
        const int row = m0 + warp * 32 + lane;
        const bool live = row < p.m;
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
            uint32_t r[32];
            tmem_ld32(tmem + ((uint32_t)(warp * 32) << 16) + c, r);
            tmem_wait_ld();
            if (live && n0 + c < n_g) epilogue32(p, g, row, n0 + c, n_g, r);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, BN);
}

template <int BN, int STAGES>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const TcParams& p, cudaStream_t s) {
    using S = Smem<BN, STAGES>;
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(gemm_tc_kernel<BN, STAGES>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES));
        configured[dev & 63] = true;
    }
    dim3 grid((unsigned)ceil_div(p.n, BN), (unsigned)ceil_div(p.m, BM), (unsigned)p.groups);
    gemm_tc_kernel<BN, STAGES><<<grid, 128, S::BYTES, s>>>(ta, tb, p);
    return check_launch("gemm_tc");
}

int run(const CUtensorMap& ta, const CUtensorMap& tb, TcParams p, int ab_type, cudaStream_t s) {
    constexpr int BN = 128, STAGES = 3;
    p.idesc = umma_idesc_f16(ab_type == ELT_BF16, BM, BN);
    p.err = device_error_word();
    if (p.groups > 65535 || ceil_div(p.m, BM) > 65535) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: grid too large");
    return launch<BN, STAGES>(ta, tb, p, s);
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

int gemm_tc(const GemmGroup& g, int ab_type, const GemmEpilogue& e, cudaStream_t s) {
    if (ab_type != ELT_BF16 && ab_type != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: operand type");
    if (g.m <= 0 || g.n <= 0 || g.k <= 0) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: empty problem");
    const size_t oe = elt_size(e.out_type);
    if (!aligned16(g.out) || (g.ldo * oe) % 16 || (g.residual && (!aligned16(g.residual) || (g.ldr * 4) % 16)) ||
        (e.rope && (!aligned16(e.rope) || e.rope_hd % 32)))
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: epilogue operands not 16-byte aligned");
    CUtensorMap ta, tb;
    ANCHA_TRY(make_tma_3d(&ta, g.a, ab_type, g.k, g.m, 1, g.lda, (int64_t)g.m * g.lda, BM));
    ANCHA_TRY(make_tma_3d(&tb, g.b, ab_type, g.k, g.n, 1, g.ldb, (int64_t)g.n * g.ldb, 128));
    TcParams p{};
    p.m = g.m; p.n = g.n; p.k = g.k; p.groups = 1; p.b_groups = 1; p.group_n = nullptr;
    p.out = g.out; p.ldo = g.ldo; p.out_group_stride = 0;
    p.bias = g.bias; p.bias_group_stride = 0;
    p.residual = g.residual; p.ldr = g.ldr;
    p.act = e.act; p.out_type = e.out_type;
    p.rope = e.rope; p.rope_width = e.rope_width; p.rope_tokens = e.rope_tokens;
    p.rope_div = e.rope_div; p.rope_hd = e.rope_hd;
    return run(ta, tb, p, ab_type, s);
}

int gemm_tc_grouped(const GroupedGemm& q, int ab_type, const GemmEpilogue& e, cudaStream_t s) {
    if (ab_type != ELT_BF16 && ab_type != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: operand type");
    const size_t oe = elt_size(e.out_type);
    const int64_t ldo_out = q.ldo;
    if (!aligned16(q.out) || (ldo_out * oe) % 16 || (q.out_group_stride * oe) % 16)
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: output not 16-byte aligned");
    CUtensorMap ta, tb;
    ANCHA_TRY(make_tma_3d(&ta, q.a, ab_type, q.k, q.m, q.groups, q.lda, q.a_group_stride, BM));
    ANCHA_TRY(make_tma_3d(&tb, q.b, ab_type, q.k, q.n, q.b_groups, q.ldb, q.b_group_stride, 128));
    TcParams p{};
    p.m = q.m; p.n = q.n; p.k = q.k; p.groups = q.groups; p.b_groups = q.b_groups;
    p.group_n = q.group_n;
    p.out = q.out; p.ldo = q.ldo; p.out_group_stride = q.out_group_stride;
    p.bias = q.bias; p.bias_group_stride = q.bias_group_stride;
    p.residual = nullptr; p.ldr = 0;
    p.act = e.act; p.out_type = e.out_type;
    p.rope = nullptr; p.rope_width = 0; p.rope_tokens = 1; p.rope_div = 1; p.rope_hd = 64;
    return run(ta, tb, p, ab_type, s);
}

}  // namespace ancha
