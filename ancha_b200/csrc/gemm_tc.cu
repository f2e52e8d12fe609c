// tcgen05 GEMM with the RoFormer epilogues: out = epilogue(A · Bᵀ) for f16 / bf16 A [rows, K]
// and B [N, K] (both K-major, PyTorch [out, in] weights), fp32 accumulation in TMEM.
//
// Persistent and warp-specialised: each CTA (one per SM) walks the 128 × BN output tiles
// tile = blockIdx.x + i·gridDim.x (columns fastest, so co-resident CTAs share A rows in L2).
//   warp 0      TMA producer: 64-wide K slabs of A and B (128-byte swizzle) into a
//               STAGES-deep shared-memory ring;
//   warp 1      UMMA issuer: tcgen05.mma M 128 × N BN × K 16 into one of two TMEM
//               accumulators, tcgen05.commit releasing each slab and, per tile, the
//               accumulator;
//   warps 2..9  epilogue: warp w drains TMEM lanes 32·(w % 4).. and every other 32-column
//               chunk, applies bias / GELU / tanh / GLU / RoPE / residual, stages each
//               32 × 32 chunk in swizzled shared memory and writes it with a TMA tensor store
//               (coalesced, asynchronous, clipped at the matrix edges by the hardware).
// The two accumulators let the epilogue of tile i overlap the main loop of tile i + 1.
//
// Groups batch same-shape problems (the per-band mask-estimator layers): problem g takes A
// from depth g of [groups, rows, K] and B from depth g % b_groups of [b_groups, N_pad, K];
// B group j may use only its first group_n[j] columns (the others are skipped).
#include "gemm.cuh"
#include "tc.cuh"

namespace ancha {
namespace {

constexpr int BM = 128, BK = 64;
// split3: the six significant products of (hi, mid, lo) planes, smallest weight first (mm, lh, hl,
// mh, hm, hh) so that the small products accumulate before the large one sets the magnitude.
__constant__ int kSplitA[6] = {1, 2, 0, 1, 0, 0};
__constant__ int kSplitB[6] = {1, 0, 2, 0, 1, 0};
constexpr int A_BYTES = BM * BK * 2;
// Epilogue warps per CTA (a multiple of 4: EPI / 4 warps per TMEM lane quarter): 16 for the
// GELU / tanh epilogues, whose long dependent chains need the extra latency hiding, and for RoPE
// (its table loads wait on L2), 8 for the others, which need the registers (10 warps allow 168
// registers a thread, 18 warps 96).
constexpr int EPI_ACT = 16, EPI_PLAIN = 8;
constexpr int STAGE_BUFS = 1;       // staging buffers per epilogue warp
template <int EPI>
constexpr int threads_of() { return 64 + 32 * EPI; }

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
    const float2* rope_pairs;
    const float4* rope_quads;
    int rope_width, rope_tokens, rope_div, rope_hd;
    const float* row_mul;    // per-row multiplier (GemmEpilogue::row_mul)
    int split3;              // three-plane bf16 operands, six plane products (GemmGroup::split3)
    const float* row_ss;     // row-norm fusion, see GemmEpilogue
    int row_ss_n;
    const float* res_ss;
    int res_ss_n;
    const float* res_col;
    void* out16;
    const float* out16_col;
    float* ss_out;
    float* ss16_out;
    int ab16;                // operand type (ELT_BF16 / ELT_F16) of the out16 copy
    uint32_t idesc;
    int m_tiles, n_tiles, tiles;
    int* err;
    // Implicit-GEMM convolution (0 taps = off): B is read straight from a channels-last
    // activation [batch][h][w][channels] through a 4-D tensor map; k block kb is tap
    // kb / conv_cblocks (a 3 × 3 stencil with zero padding 1 for 9 taps, the centre for 1),
    // channels 64·(kb % conv_cblocks); output column n is position n = y·conv_w + x of image
    // conv_b.
    int conv_taps, conv_cblocks, conv_w, conv_b;
    // Per-plane output statistics (null = off): Σ v and Σ v² of the final output values of
    // rows r, r + 1, … are added into stats[r / stats_div] (f64), for the instance norm that
    // follows this GEMM. Single-group problems only.
    double2* stats;
    int stats_div;
};

// Adds a lane's accumulated (Σ v, Σ v²) into stats[plane]; lanes of a warp that share one
// plane are combined first, so a warp over consecutive rows of one plane issues one pair of
// atomics.
__device__ __forceinline__ void flush_stats(double2* stats, int plane, double& sum, double& sq, int lane) {
    const int first = __shfl_sync(0xffffffffu, plane, 0), last = __shfl_sync(0xffffffffu, plane, 31);
    if (first == last) {
        for (int o = 16; o > 0; o >>= 1) {
            sum += __shfl_xor_sync(0xffffffffu, sum, o);
            sq += __shfl_xor_sync(0xffffffffu, sq, o);
        }
        if (lane == 0 && plane >= 0) {
            atomicAdd(&stats[plane].x, sum);
            atomicAdd(&stats[plane].y, sq);
        }
    } else if (plane >= 0) {
        atomicAdd(&stats[plane].x, sum);
        atomicAdd(&stats[plane].y, sq);
    }
    sum = 0.0;
    sq = 0.0;
}

constexpr int STAGE_BYTES = 4096;    // one 32-row × 128-byte epilogue staging buffer
constexpr int STAGE16_BYTES = 2048;  // one 32-row × 64-byte buffer for the 16-bit copy
// One buffer per warp: a chunk waits for every store of the previous chunk (the output and the
// 16-bit copy) to have read its source before it overwrites either buffer. (Alternating two
// halves for 16-bit outputs measured within ±1 %.)
static_assert(STAGE_BUFS == 1, "the row-norm copy shares the single-buffer wait");

// PAIR: a CTA of a two-CTA pair holds half of the tile's B columns.
template <int BN, int STAGES, int EPI_WARPS, bool PAIR = false>
struct Smem {
    static constexpr int B_BYTES = (PAIR ? BN / 2 : BN) * BK * 2;
    static constexpr int TILES = STAGES * (A_BYTES + B_BYTES);
    static constexpr int STAGING = EPI_WARPS * STAGE_BUFS * STAGE_BYTES;
    // The row-norm fusion's 16-bit copy: only the plain (residual) epilogues write one.
    static constexpr int STAGING16 = EPI_WARPS == EPI_PLAIN ? EPI_WARPS * STAGE16_BYTES : 0;
    static constexpr int BYTES = 1024 + TILES + STAGING + STAGING16 + 8 * (2 * STAGES + 4) + 16;
};

// v[j], v[j + 1] = f2 result (the register pairs of the packed arithmetic below).
__device__ __forceinline__ void put2(float (&v)[32], int j, uint64_t x) { f2_split(x, v[j], v[j + 1]); }

// Bias, activation, RoPE and residual for 32 consecutive accumulator columns c0.. of one
// row, in registers. Returns the number of output values (32, or 16 for GLU). All indexing
// of the register arrays is static. The element-wise arithmetic runs on packed f32x2 pairs
// (one instruction issue per two values): these epilogues are issue-bound.
__device__ __forceinline__ int epilogue32(const TcParams& p, int g, int row, bool live, int c0, int n_g,
                                          const uint32_t (&r)[32], float (&v)[32], float row_scale,
                                          float res_scale) {
    const int nv = min(32, n_g - c0);  // valid columns (> 0)
    const uint64_t rs2 = f2(row_scale, row_scale);
    if (p.bias && nv == 32) {  // v = acc · row_scale + bias
        const float* b = p.bias + (int64_t)(g % p.b_groups) * p.bias_group_stride + c0;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 q = *reinterpret_cast<const float4*>(b + j);
            put2(v, j, ffma2(f2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), rs2, f2(q.x, q.y)));
            put2(v, j + 2, ffma2(f2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])), rs2, f2(q.z, q.w)));
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; j += 2)
            put2(v, j, fmul2(f2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])), rs2));
        if (p.bias) {
            const float* b = p.bias + (int64_t)(g % p.b_groups) * p.bias_group_stride + c0;
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) v[j] += b[j];
        }
    }
    if (p.act == ANCHA_ACT_GELU) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) gelu_fast2(v[j], v[j + 1]);
    } else if (p.act == ANCHA_ACT_TANH) {
#pragma unroll
        for (int j = 0; j < 32; j += 2) tanh_fast2(v[j], v[j + 1]);
    }
    if (p.rope_quads && c0 < 2 * p.rope_width) {
        const int key = c0 >= p.rope_width;
        const int token = (row / p.rope_div) % p.rope_tokens;
        const float4* t = p.rope_quads +
                          ((int64_t)key * (p.rope_hd / 2) + (c0 % p.rope_hd) / 2) * p.rope_tokens + token;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {  // (x0·C0 + x1·S0, x1·C1 + x0·S1), packed
            const float4 q = t[(int64_t)(j / 2) * p.rope_tokens];
            put2(v, j, ffma2(f2(v[j + 1], v[j]), f2(q.z, q.w), fmul2(f2(v[j], v[j + 1]), f2(q.x, q.y))));
        }
    } else if (p.rope_pairs && c0 < 2 * p.rope_width) {
        const int key = c0 >= p.rope_width;
        const int token = (row / p.rope_div) % p.rope_tokens;
        const float2* t = p.rope_pairs +
                          ((int64_t)key * (p.rope_hd / 2) + (c0 % p.rope_hd) / 2) * p.rope_tokens + token;
#pragma unroll
        for (int j = 0; j < 32; j += 2) {  // (x0·c − x1·s, x1·c + x0·s), packed
            const float2 cs = t[(int64_t)(j / 2) * p.rope_tokens];
            put2(v, j, ffma2(f2(v[j + 1], v[j]), f2(-cs.y, cs.y), fmul2(f2(v[j], v[j + 1]), f2(cs.x, cs.x))));
        }
    } else if (p.rope && c0 < 2 * p.rope_width) {
        const int key = c0 >= p.rope_width;
        const int token = (row / p.rope_div) % p.rope_tokens;
        const int d = c0 % p.rope_hd;
        const float* cs = p.rope + ((int64_t)(key * 2) * p.rope_tokens + token) * p.rope_hd + d;
        const float* sn = cs + (int64_t)p.rope_tokens * p.rope_hd;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 c4 = *reinterpret_cast<const float4*>(cs + j);
            const float4 s4 = *reinterpret_cast<const float4*>(sn + j);
            const float x0 = v[j], x1 = v[j + 1], x2 = v[j + 2], x3 = v[j + 3];
            v[j] = x0 * c4.x + x1 * s4.x;
            v[j + 1] = x1 * c4.y + x0 * s4.y;
            v[j + 2] = x2 * c4.z + x3 * s4.z;
            v[j + 3] = x3 * c4.w + x2 * s4.w;
        }
    }
    if (p.act == ANCHA_ACT_GLU) {
#pragma unroll
        for (int j = 0; j < 16; ++j) v[j] = v[2 * j] * sigmoid_fast(v[2 * j + 1]);
        return 16;
    }
    if (p.residual && live) {
        const float* rr = p.residual + (int64_t)row * p.ldr + c0;
        const uint64_t sc2 = f2(res_scale, res_scale);
        if (p.res_col && nv == 32) {
            const float* rc = p.res_col + c0;
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 q = *reinterpret_cast<const float4*>(rr + j);
                const float4 w = *reinterpret_cast<const float4*>(rc + j);
                put2(v, j, ffma2(fmul2(f2(q.x, q.y), sc2), f2(w.x, w.y), f2(v[j], v[j + 1])));
                put2(v, j + 2, ffma2(fmul2(f2(q.z, q.w), sc2), f2(w.z, w.w), f2(v[j + 2], v[j + 3])));
            }
        } else if (p.res_col) {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) v[j] = fmaf(rr[j] * res_scale, p.res_col[c0 + j], v[j]);
        } else if (nv == 32) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
                const float4 q = *reinterpret_cast<const float4*>(rr + j);
                put2(v, j, ffma2(f2(q.x, q.y), sc2, f2(v[j], v[j + 1])));
                put2(v, j + 2, ffma2(f2(q.z, q.w), sc2, f2(v[j + 2], v[j + 3])));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j)
                if (j < nv) v[j] = fmaf(rr[j], res_scale, v[j]);
        }
    }
    return 32;
}

// 1 / max(√(Σ_i ss[i·rows]), 1e-12): the unit-norm factor of a row from its per-chunk partial
// sums of squares, stored chunk-major so a warp's 32 rows read 128 contiguous bytes (the same
// epsilon as the row-norm kernel).
__device__ __forceinline__ float inv_norm(const float* ss, int n, int64_t rows) {
    float t = 0.f;
    for (int i = 0; i < n; ++i) t += ss[i * rows];
    return 1.f / fmaxf(sqrtf(t), 1e-12f);
}

// Row-norm fusion: the sum of squares of 32 values of a row (chunk-major slot, so the warp's
// 32 rows store 128 contiguous bytes); values past nv do not count.
__device__ __forceinline__ void store_ss(float* ss, const TcParams& p, int row, bool live, int c0, int nv,
                                         const float (&v)[32]) {
    float q = 0.f;
    if (nv == 32) {  // two packed accumulators
        uint64_t qa = 0, qb = 0;
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const uint64_t x = f2(v[j], v[j + 1]), y = f2(v[j + 2], v[j + 3]);
            qa = ffma2(x, x, qa);
            qb = ffma2(y, y, qb);
        }
        float a0, a1, b0, b1;
        f2_split(qa, a0, a1);
        f2_split(qb, b0, b1);
        q = (a0 + b0) + (a1 + b1);
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (j < nv) q = fmaf(v[j], v[j], q);
    }
    if (live) ss[(int64_t)(c0 / 32) * p.m + row] = q;
}

// v ⊙ out16_col[c0 ..] in place (the row-norm fusion's copy of the output).
__device__ __forceinline__ void scale_cols(const float* col, int c0, int nv, float (&v)[32]) {
    if (nv == 32) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
            const float4 c = *reinterpret_cast<const float4*>(col + c0 + j);
            f2_split(fmul2(f2(v[j], v[j + 1]), f2(c.x, c.y)), v[j], v[j + 1]);
            f2_split(fmul2(f2(v[j + 2], v[j + 3]), f2(c.z, c.w)), v[j + 2], v[j + 3]);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) v[j] = j < nv ? v[j] * col[c0 + j] : 0.f;
    }
}

// Write this lane's row of a 32-row staging buffer in the TMA swizzled layout: rows of
// 128 bytes (f32 × 32) use the 128-byte swizzle, rows of 64 bytes (16-bit × 32, or f32 × 16
// for GLU) the 64-byte swizzle.
__device__ __forceinline__ void stage_row(uint8_t* buf, int lane, int out_type, int count, const float (&v)[32]) {
    if (out_type == ELT_F32 && count == 32) {
        uint8_t* row = buf + lane * 128;
#pragma unroll
        for (int q = 0; q < 8; ++q)
            *reinterpret_cast<float4*>(row + ((q ^ (lane & 7)) * 16)) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        return;
    }
    uint8_t* row = buf + lane * 64;
    if (out_type == ELT_F32) {  // 16 f32 (GLU)
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<float4*>(row + ((q ^ ((lane >> 1) & 3)) * 16)) =
                make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        return;
    }
    uint32_t h[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
        if (out_type == ELT_BF16) {
            __nv_bfloat162 t = __floats2bfloat162_rn(v[2 * j], v[2 * j + 1]);
            h[j] = *reinterpret_cast<uint32_t*>(&t);
        } else {
            __half2 t = __floats2half2_rn(v[2 * j], v[2 * j + 1]);
            h[j] = *reinterpret_cast<uint32_t*>(&t);
        }
    }
    if (count == 32) {
#pragma unroll
        for (int q = 0; q < 4; ++q)
            *reinterpret_cast<uint4*>(row + ((q ^ ((lane >> 1) & 3)) * 16)) =
                make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
    } else {  // 16 values of 16 bits (GLU with a 16-bit output): 32-byte rows are not staged
#pragma unroll
        for (int q = 0; q < 2; ++q)
            *reinterpret_cast<uint4*>(row + ((q ^ ((lane >> 1) & 3)) * 16)) =
                make_uint4(h[4 * q], h[4 * q + 1], h[4 * q + 2], h[4 * q + 3]);
    }
}

struct TileCoord {
    int g, m0, n0, n_g;
};

__device__ __forceinline__ TileCoord tile_coord(const TcParams& p, int t, int bn, int bm = BM) {
    TileCoord c;
    const int per_group = p.m_tiles * p.n_tiles;
    c.g = t / per_group;
    const int r = t % per_group;
    c.m0 = (r / p.n_tiles) * bm;
    c.n0 = (r % p.n_tiles) * bn;
    c.n_g = p.group_n ? p.group_n[c.g % p.b_groups] : p.n;
    return c;
}

// PAIR: the kernel runs as clusters of two CTAs on two SMs. A tile is 256 × BN: CTA rank r
// loads A rows m0 + 128·r .. and B columns n0 + (BN / 2)·r .. of each K slab into its own
// shared memory (both completing on the even CTA's full barrier), the even CTA's issuer runs
// M = 256 UMMAs over both CTAs' operands (cta_group::2) into both CTAs' TMEM, and its commits
// arrive on both CTAs' barriers; each CTA's epilogue drains its own 128 rows and arrives on the
// even CTA's accumulator barrier. Per SM this halves the B slab loaded per tile (the GEMMs with
// K = 384 are limited by the operand traffic from L2).
template <int BN, int STAGES, int EPI_WARPS, bool PAIR>
__global__ void __launch_bounds__(threads_of<EPI_WARPS>(), 1)
gemm_tc_kernel(const __grid_constant__ CUtensorMap tma_a, const __grid_constant__ CUtensorMap tma_b,
               const __grid_constant__ CUtensorMap tma_out, const __grid_constant__ CUtensorMap tma_out16,
               const TcParams p) {
    using S = Smem<BN, STAGES, EPI_WARPS, PAIR>;
    constexpr int BMT = PAIR ? 2 * BM : BM;  // rows of a tile
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint8_t* a_tiles = smem;
    uint8_t* b_tiles = smem + STAGES * A_BYTES;
    uint8_t* staging = smem + S::TILES;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + S::TILES + S::STAGING + S::STAGING16);
    uint64_t* empty = full + STAGES;
    uint64_t* tfull = empty + STAGES;   // [2] accumulator ready
    uint64_t* tempty = tfull + 2;       // [2] accumulator drained
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(tempty + 2);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    constexpr uint32_t TMEM_COLS = 2 * BN <= 256 ? 256 : 512;

    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const uint32_t rank = PAIR ? cluster_ctarank() : 0;
    const int tile0 = PAIR ? (int)blockIdx.x / 2 : (int)blockIdx.x;
    const int tstep = PAIR ? (int)gridDim.x / 2 : (int)gridDim.x;
    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int b = 0; b < 2; ++b) {
            mbar_init(&tfull[b], 1);
            mbar_init(&tempty[b], PAIR ? 2 * EPI_WARPS : EPI_WARPS);
        }
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tma_a);
        prefetch_tma(&tma_b);
        prefetch_tma(&tma_out);
        if (p.out16) prefetch_tma(&tma_out16);
    }
    if (warp == 1) {
        if (PAIR) {
            tmem_alloc_pair(tmem_slot, TMEM_COLS);
            tmem_relinquish_pair();
        } else {
            tmem_alloc(tmem_slot, TMEM_COLS);
            tmem_relinquish();
        }
    }
    tc_fence_before();
    __syncthreads();
    if (PAIR) cluster_sync();  // the peer's barriers exist before anything arrives on them
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    const int kblocks = (p.k + BK - 1) / BK;
    const int kb_total = kblocks * (p.split3 ? 6 : 1);  // K steps per tile

    if (warp == 0) {
        if (lane == 0) {
            // TMA producer.
            uint32_t it = 0;
            for (int t = tile0; t < p.tiles && !*abort; t += tstep) {
                const TileCoord c = tile_coord(p, t, BN, BMT);
                if (c.n0 >= c.n_g) continue;
                const int bg = c.g % p.b_groups;
                for (int kt = 0; kt < kb_total; ++kt, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&empty[s], ((it / STAGES) & 1) ^ 1, abort, p.err)) break;
                    // split3: K step kt is slab kb of plane product `term` (A plane, B plane).
                    const int term = kt / kblocks, kb = kt - term * kblocks;
                    const int az = p.split3 ? kSplitA[term] * p.groups + c.g : c.g;
                    const int bz = p.split3 ? kSplitB[term] * p.b_groups + bg : bg;
                    if (PAIR) {
                        // Both CTAs' slabs complete on the even CTA's barrier, which expects both.
                        const uint32_t fb = mapa_shared(smem_u32(&full[s]), 0);
                        if (rank == 0) mbar_arrive_expect_tx(&full[s], 2 * (A_BYTES + S::B_BYTES));
                        tma_load_3d_pair(a_tiles + s * A_BYTES, &tma_a, fb, kb * BK, c.m0 + (int)rank * BM, az);
                        tma_load_3d_pair(b_tiles + s * S::B_BYTES, &tma_b, fb, kb * BK, c.n0 + (int)rank * (BN / 2),
                                         bz);
                        continue;
                    }
                    mbar_arrive_expect_tx(&full[s], A_BYTES + S::B_BYTES);
                    tma_load_3d(a_tiles + s * A_BYTES, &tma_a, &full[s], kb * BK, c.m0, az);
                    if (p.conv_taps) {
                        // The tap's shifted window; rows or columns outside the image load as
                        // zeros (the convolution's padding).
                        const int tap = kb / p.conv_cblocks, cb = kb - tap * p.conv_cblocks;
                        const int dy = p.conv_taps == 9 ? tap / 3 - 1 : 0, dx = p.conv_taps == 9 ? tap % 3 - 1 : 0;
                        const int y0 = c.n0 / p.conv_w, x0 = c.n0 - y0 * p.conv_w;
                        tma_load_4d(b_tiles + s * S::B_BYTES, &tma_b, &full[s], cb * BK, x0 + dx, y0 + dy, p.conv_b);
                    } else {
                        tma_load_3d(b_tiles + s * S::B_BYTES, &tma_b, &full[s], kb * BK, c.n0, bz);
                    }
                }
            }
            if (*abort && rank == 0) {  // let copies in flight land before the CTA exits (bounded;
                // with a pair the even CTA's barriers also count the peer's copies)
                const long long c0 = clock64();
                for (uint32_t j = it > (uint32_t)STAGES ? it - STAGES : 0; j < it; ++j)
                    while (!mbar_try_wait(&full[j % STAGES], (j / STAGES) & 1) && clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == 1) {
        if (lane == 0 && rank == 0) {
            // UMMA issuer (the even CTA of a pair issues for both).
            uint32_t it = 0, local = 0;
            for (int t = tile0; t < p.tiles && !*abort; t += tstep) {
                const TileCoord c = tile_coord(p, t, BN, BMT);
                if (c.n0 >= c.n_g) continue;
                const int b = local & 1;
                if (!mbar_wait(&tempty[b], ((local >> 1) & 1) ^ 1, abort, p.err)) break;
                tc_fence_after();
                const uint32_t acc = tmem + b * BN;
                for (int kb = 0; kb < kb_total; ++kb, ++it) {
                    const int s = it % STAGES;
                    if (!mbar_wait(&full[s], (it / STAGES) & 1, abort, p.err)) break;
                    tc_fence_after();
                    const uint32_t a_addr = smem_u32(a_tiles + s * A_BYTES);
                    const uint32_t b_addr = smem_u32(b_tiles + s * S::B_BYTES);
                    if (PAIR) {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            umma_f16_pair(acc, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32),
                                          p.idesc, (kb | kk) != 0);
                        umma_commit_pair(&empty[s], 0x3);
                    } else {
#pragma unroll
                        for (int kk = 0; kk < BK / 16; ++kk)
                            umma_f16(acc, umma_desc_sw128(a_addr + kk * 32), umma_desc_sw128(b_addr + kk * 32),
                                     p.idesc, (kb | kk) != 0);
                        umma_commit(&empty[s]);
                    }
                }
                if (PAIR)
                    umma_commit_pair(&tfull[b], 0x3);
                else
                    umma_commit(&tfull[b]);
                ++local;
            }
        }
    } else {
        // Epilogue warps: lane quarter (warp % 4); the quarter's warps take its 32-column
        // chunks in turn.
        constexpr int PER_QUARTER = EPI_WARPS / 4;
        const int quarter = warp % 4;
        const int first = (warp - 2) / 4;
        uint8_t* my_stage = staging + (warp - 2) * STAGE_BUFS * STAGE_BYTES;
        uint8_t* my_stage16 = staging + S::STAGING + (warp - 2) * STAGE16_BYTES;
        const bool glu = p.act == ANCHA_ACT_GLU;
        uint32_t local = 0, chunks = 0;
        // Output statistics, accumulated over every tile of the same rows (a persistent CTA
        // usually keeps its rows) and flushed when the plane changes.
        double st_sum = 0.0, st_sq = 0.0;
        int st_plane = -1;
        for (int t = tile0; t < p.tiles; t += tstep) {
            const TileCoord c = tile_coord(p, t, BN, BMT);
            if (c.n0 >= c.n_g) continue;
            const int b = local & 1;
            const bool ok = __all_sync(0xffffffffu, mbar_wait(&tfull[b], (local >> 1) & 1, abort, p.err));
            if (!ok) break;
            tc_fence_after();
            const int row0 = c.m0 + (int)rank * BM + quarter * 32;
            const int row = row0 + lane;
            const bool live = row < p.m;
            if (p.stats) {
                const int plane = live ? row / p.stats_div : -1;
                if (__any_sync(0xffffffffu, plane != st_plane)) {
                    flush_stats(p.stats, st_plane, st_sum, st_sq, lane);
                    st_plane = plane;
                }
            }
            const uint32_t base = tmem + b * BN + ((uint32_t)(quarter * 32) << 16);
            const float row_scale = !live ? 1.f
                                    : p.row_ss ? inv_norm(p.row_ss + row, p.row_ss_n, p.m)
                                    : p.row_mul ? p.row_mul[row] : 1.f;
            const float res_scale = p.res_ss && live ? inv_norm(p.res_ss + row, p.res_ss_n, p.m) : 1.f;
#pragma unroll 1
            for (int col = first * 32; col < BN; col += PER_QUARTER * 32) {
                uint32_t r[32];
                tmem_ld32(base + col, r);
                tmem_wait_ld();
                if (c.n0 + col >= c.n_g) continue;  // warp-uniform
                float v[32];
                const int count = epilogue32(p, c.g, row, live, c.n0 + col, c.n_g, r, v, row_scale, res_scale);
                const int nv = min(32, c.n_g - (c.n0 + col));
                if (p.stats && live) {
                    float s1 = 0.f, s2 = 0.f;
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (j < nv) {
                            s1 += v[j];
                            s2 = fmaf(v[j], v[j], s2);
                        }
                    st_sum += s1;
                    st_sq += s2;
                }
                if (p.ss_out && count == 32) store_ss(p.ss_out, p, row, live, c.n0 + col, nv, v);
                uint8_t* buf = my_stage + (chunks % STAGE_BUFS) * STAGE_BYTES;
                if (chunks >= STAGE_BUFS) {  // the store that last read this buffer is done with it
                    if (lane == 0) bulk_wait_read<STAGE_BUFS - 1>();
                    __syncwarp();
                }
                stage_row(buf, lane, p.out_type, count, v);
                fence_proxy_async();
                __syncwarp();
                if (lane == 0) {
                    tma_store_3d(&tma_out, buf, glu ? (c.n0 + col) / 2 : c.n0 + col, row0, c.g);
                    bulk_commit();
                }
                if (p.out16 && count == 32) {
                    if (p.out16_col) scale_cols(p.out16_col, c.n0 + col, nv, v);
                    if (p.ss16_out) store_ss(p.ss16_out, p, row, live, c.n0 + col, nv, v);
                    uint8_t* buf16 = my_stage16;
                    stage_row(buf16, lane, p.ab16, 32, v);
                    fence_proxy_async();
                    __syncwarp();
                    if (lane == 0) {
                        tma_store_3d(&tma_out16, buf16, c.n0 + col, row0, 0);
                        bulk_commit();
                    }
                }
                ++chunks;
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) {
                if (PAIR)
                    mbar_arrive_cluster(mapa_shared(smem_u32(&tempty[b]), 0));
                else
                    mbar_arrive(&tempty[b]);
            }
            ++local;
        }
        if (p.stats) flush_stats(p.stats, st_plane, st_sum, st_sq, lane);
        if (lane == 0) bulk_wait<0>();
        __syncwarp();
    }
    tc_fence_before();
    __syncthreads();
    // With a pair, neither CTA releases TMEM or exits while the other may still use its
    // shared memory (the even CTA's UMMAs read the peer's slabs) or its barriers.
    if (PAIR) cluster_sync();
    if (warp == 1) {
        __syncwarp();
        if (PAIR)
            tmem_dealloc_pair(tmem, TMEM_COLS);
        else
            tmem_dealloc(tmem, TMEM_COLS);
    }
}

template <int BN, int STAGES, int EPI_WARPS, bool PAIR = false>
int launch(const CUtensorMap& ta, const CUtensorMap& tb, const CUtensorMap& to, const CUtensorMap& to16,
           const TcParams& p, cudaStream_t s) {
    using S = Smem<BN, STAGES, EPI_WARPS, PAIR>;
    auto kernel = gemm_tc_kernel<BN, STAGES, EPI_WARPS, PAIR>;
    static bool configured[64] = {};
    static int slots[64] = {};  // co-resident CTAs (one CTA per SM) or CTA pairs
    int dev = 0;
    cudaGetDevice(&dev);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.blockDim = dim3(threads_of<EPI_WARPS>(), 1, 1);
    cfg.dynamicSmemBytes = S::BYTES;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, S::BYTES));
        if (PAIR) {
            cfg.gridDim = dim3(2, 1, 1);
            ANCHA_CUDA(cudaOccupancyMaxActiveClusters(&slots[dev & 63], (void*)kernel, &cfg));
            if (slots[dev & 63] < 1) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: no CTA pair fits an SM pair");
        } else {
            ANCHA_CUDA(cudaDeviceGetAttribute(&slots[dev & 63], cudaDevAttrMultiProcessorCount, dev));
        }
        configured[dev & 63] = true;
    }
    const int units = std::max(1, std::min(p.tiles, slots[dev & 63]));
    if (!PAIR) {
        kernel<<<units, threads_of<EPI_WARPS>(), S::BYTES, s>>>(ta, tb, to, to16, p);
        return check_launch("gemm_tc");
    }
    cfg.gridDim = dim3(2 * units, 1, 1);
    cfg.stream = s;
    ANCHA_CUDA(cudaLaunchKernelEx(&cfg, kernel, ta, tb, to, to16, p));
    return check_launch("gemm_tc (CTA pairs)");
}

// Output tile width: the widest of 256 / 192 / 128 whose padded N is within 1/6 of the least
// padded N. Wider tiles amortise the per-tile main-loop and epilogue overheads; a mostly empty
// last tile costs its main loop but almost no epilogue work (empty chunks are skipped).
int pick_bn(int n) {
    int64_t least = INT64_MAX;
    for (int bn : {128, 192, 256}) least = std::min<int64_t>(least, ceil_div(n, bn) * bn);
    for (int bn : {256, 192, 128})
        if (ceil_div(n, bn) * bn * 6 <= least * 7) return bn;
    return 128;
}

#ifndef ANCHA_GEMM_PAIRS
#define ANCHA_GEMM_PAIRS 1
#endif

int run(const void* a, int64_t lda, int64_t a_group_stride, const void* b, int64_t ldb,
        int64_t b_group_stride, TcParams p, int ab_type, cudaStream_t s) {
    const int bn = p.group_n ? 128 : pick_bn(p.n);
    // CTA pairs (256-row tiles over two SMs) for single problems with at least two 128-row tiles
    // and a long K loop: measured on the model's GEMMs, pairs take 12.5 % off the K = 1536
    // FFN-out and 7 % off the K = 1536 mask layer, where the operand traffic per SM limits the
    // main loop, but add 6-9 % at K = 384 / 512, where each SM's epilogue is the limit and a pair
    // must wait for both CTAs' epilogues before reusing an accumulator. Grouped problems and the
    // implicit-GEMM convolution keep one CTA per tile.
    const bool pair = ANCHA_GEMM_PAIRS && p.groups == 1 && !p.group_n && !p.conv_taps && p.m >= 2 * BM &&
                      p.k * (p.split3 ? 6 : 1) >= 1024;
    CUtensorMap ta, tb, to;
    // split3 operands are three planes along the depth coordinate of each map, plane-major over
    // the groups.
    ANCHA_TRY(make_tma_3d(&ta, a, ab_type, p.k, p.m, (p.split3 ? 3 : 1) * p.groups, lda, a_group_stride, BM));
    ANCHA_TRY(make_tma_3d(&tb, b, ab_type, p.k, p.n, (p.split3 ? 3 : 1) * p.b_groups, ldb, b_group_stride,
                          pair ? bn / 2 : bn));
    const bool glu = p.act == ANCHA_ACT_GLU;
    if (glu && p.out_type != ELT_F32) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: GLU output must be f32");
    const int64_t out_cols = glu ? p.n / 2 : p.n;
    const int64_t ogs = p.groups > 1 ? p.out_group_stride : (int64_t)p.m * p.ldo;
    ANCHA_TRY(make_tma_store_3d(&to, p.out, p.out_type, std::min<int64_t>(out_cols, p.ldo), p.m, p.groups, p.ldo,
                                ogs, glu ? 16 : 32, 32));
    CUtensorMap to16 = to;  // unused unless the row-norm fusion writes its copy
    if (p.out16) {
        if (p.groups != 1) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: row-norm fusion on grouped problems");
        ANCHA_TRY(make_tma_store_3d(&to16, p.out16, ab_type, p.n, p.m, 1, p.n, (int64_t)p.m * p.n, 32, 32));
    }
    p.idesc = umma_idesc_f16(ab_type == ELT_BF16, pair ? 2 * BM : BM, bn);
    p.err = device_error_word();
    p.m_tiles = (int)ceil_div(p.m, pair ? 2 * BM : BM);
    p.n_tiles = (int)ceil_div(p.n, bn);
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles * p.groups;
    if (tiles > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: too many tiles");
    p.tiles = (int)tiles;
    if ((p.act == ANCHA_ACT_GELU || p.act == ANCHA_ACT_TANH) && p.out16)
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: no 16-bit copy after an activation");
    // Sixteen epilogue warps for the activations and for RoPE (whose table loads wait on L2),
    // eight for the plain and residual epilogues.
    const bool act = p.act == ANCHA_ACT_GELU || p.act == ANCHA_ACT_TANH ||
                     ((p.rope || p.rope_pairs || p.rope_quads) && !p.out16);
    if (pair) {
        switch (bn) {
            case 256: return act ? launch<256, 4, EPI_ACT, true>(ta, tb, to, to16, p, s) : launch<256, 4, EPI_PLAIN, true>(ta, tb, to, to16, p, s);
            case 192: return act ? launch<192, 4, EPI_ACT, true>(ta, tb, to, to16, p, s) : launch<192, 5, EPI_PLAIN, true>(ta, tb, to, to16, p, s);
            default: return act ? launch<128, 6, EPI_ACT, true>(ta, tb, to, to16, p, s) : launch<128, 6, EPI_PLAIN, true>(ta, tb, to, to16, p, s);
        }
    }
    switch (bn) {
        case 256: return act ? launch<256, 3, EPI_ACT>(ta, tb, to, to16, p, s) : launch<256, 3, EPI_PLAIN>(ta, tb, to, to16, p, s);
        case 192: return act ? launch<192, 3, EPI_ACT>(ta, tb, to, to16, p, s) : launch<192, 3, EPI_PLAIN>(ta, tb, to, to16, p, s);
        default: return act ? launch<128, 4, EPI_ACT>(ta, tb, to, to16, p, s) : launch<128, 4, EPI_PLAIN>(ta, tb, to, to16, p, s);
    }
}

bool aligned16(const void* p) { return reinterpret_cast<uintptr_t>(p) % 16 == 0; }

}  // namespace

int gemm_tc(const GemmGroup& g, int ab_type, const GemmEpilogue& e, cudaStream_t s) {
    if (ab_type != ELT_BF16 && ab_type != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: operand type");
    if (g.m <= 0 || g.n <= 0 || g.k <= 0) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: empty problem");
    const size_t oe = elt_size(e.out_type);
    if (!aligned16(g.out) || (g.ldo * oe) % 16 || (g.residual && (!aligned16(g.residual) || (g.ldr * 4) % 16)) ||
        (g.bias && !aligned16(g.bias)) || (e.rope && (!aligned16(e.rope) || e.rope_hd % 32)) ||
        (e.rope_pairs && (!aligned16(e.rope_pairs) || e.rope_hd % 32)) ||
        (e.rope_quads && (!aligned16(e.rope_quads) || e.rope_hd % 32)) ||
        (e.out16 && (!aligned16(e.out16) || g.n % 8)) || (e.res_col && !aligned16(e.res_col)))
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: epilogue operands not 16-byte aligned");
    if ((e.res_ss && !g.residual) || e.act == ANCHA_ACT_GLU && (e.out16 || e.ss_out))
        return fail(ANCHA_E_INVALID, "gemm_tc: row-norm fusion operands without their epilogue");
    TcParams p{};
    p.m = g.m; p.n = g.n; p.k = g.k; p.groups = 1; p.b_groups = 1; p.group_n = nullptr;
    p.out = g.out; p.ldo = g.ldo; p.out_group_stride = 0;
    p.bias = g.bias; p.bias_group_stride = 0;
    p.residual = g.residual; p.ldr = g.ldr;
    p.act = e.act; p.out_type = e.out_type;
    p.rope = e.rope; p.rope_width = e.rope_width; p.rope_tokens = e.rope_tokens;
    p.rope_pairs = reinterpret_cast<const float2*>(e.rope_pairs);
    p.rope_quads = reinterpret_cast<const float4*>(e.rope_quads);
    p.rope_div = e.rope_div; p.rope_hd = e.rope_hd;
    p.row_ss = e.row_ss; p.row_ss_n = e.row_ss_n; p.res_ss = e.res_ss; p.res_ss_n = e.res_ss_n;
    p.row_mul = e.row_mul;
    p.split3 = g.split3 ? 1 : 0;
    if (g.split3 && ab_type != ELT_BF16) return fail(ANCHA_E_INVALID, "gemm_tc: split operands are bf16");
    p.res_col = e.res_col; p.out16 = e.out16; p.out16_col = e.out16_col;
    p.ss_out = e.ss_out; p.ss16_out = e.ss16_out; p.ab16 = ab_type;
    p.stats = e.stats; p.stats_div = e.stats_div > 0 ? e.stats_div : 1;
    if (e.stats && e.act == ANCHA_ACT_GLU) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: statistics of a GLU output");
    return run(g.a, g.lda, (int64_t)g.m * g.lda, g.b, g.ldb, (int64_t)g.n * g.ldb, p, ab_type, s);
}

int gemm_tc_conv(const ConvGemm& q, int ab_type, const GemmEpilogue& e, cudaStream_t s) {
    if (ab_type != ELT_BF16 && ab_type != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: operand type");
    if (q.taps != 1 && q.taps != 9) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: taps");
    if (q.channels <= 0 || q.channels % BK || q.co <= 0 || q.h <= 0 || q.w <= 0 || q.batch <= 0 ||
        q.image < 0 || q.image >= q.batch)
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: shape");
    constexpr int bn = 256;
    // A tile of 256 output positions is a box of whole rows (w ≤ 256) or a run inside one row.
    if (!(q.w % bn == 0 || bn % q.w == 0)) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: row width");
    const size_t oe = elt_size(e.out_type);
    if (!aligned16(q.out) || (q.ldo * oe) % 16 || (q.residual && (!aligned16(q.residual) || (q.ldo * 4) % 16)))
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: output not 16-byte aligned");
    if (e.act != ANCHA_ACT_NONE || e.rope || e.rope_pairs || e.rope_quads || e.row_ss || e.res_ss || e.out16 || e.ss_out)
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: epilogue");
    TcParams p{};
    p.m = q.co; p.n = q.h * q.w; p.k = q.taps * q.channels; p.groups = 1; p.b_groups = 1; p.group_n = nullptr;
    p.out = q.out; p.ldo = q.ldo; p.out_group_stride = 0;
    p.bias = nullptr; p.bias_group_stride = 0;
    p.residual = q.residual; p.ldr = q.ldo;
    p.act = ANCHA_ACT_NONE; p.out_type = e.out_type;
    p.rope_tokens = 1; p.rope_div = 1; p.rope_hd = 64; p.ab16 = ab_type;
    p.conv_taps = q.taps; p.conv_cblocks = q.channels / BK; p.conv_w = q.w; p.conv_b = q.image;
    p.stats = e.stats; p.stats_div = e.stats_div > 0 ? e.stats_div : 1;
    CUtensorMap ta, tb, to;
    ANCHA_TRY(make_tma_3d(&ta, q.weight, ab_type, p.k, p.m, 1, q.ldw, (int64_t)p.m * q.ldw, BM));
    const int bw = std::min(q.w, bn);
    ANCHA_TRY(make_tma_4d(&tb, q.x, ab_type, q.channels, q.w, q.h, q.batch, q.channels, (int64_t)q.w * q.channels,
                          (int64_t)q.h * q.w * q.channels, bw, bn / bw));
    ANCHA_TRY(make_tma_store_3d(&to, p.out, p.out_type, std::min<int64_t>(p.n, p.ldo), p.m, 1, p.ldo,
                                (int64_t)p.m * p.ldo, 32, 32));
    p.idesc = umma_idesc_f16(ab_type == ELT_BF16, BM, bn);
    p.err = device_error_word();
    p.m_tiles = (int)ceil_div(p.m, BM);
    p.n_tiles = (int)ceil_div(p.n, bn);
    const int64_t tiles = (int64_t)p.m_tiles * p.n_tiles;
    if (tiles > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc_conv: too many tiles");
    p.tiles = (int)tiles;
    return launch<bn, 3, EPI_PLAIN>(ta, tb, to, to, p, s);
}

int gemm_tc_grouped(const GroupedGemm& q, int ab_type, const GemmEpilogue& e, cudaStream_t s) {
    if (ab_type != ELT_BF16 && ab_type != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: operand type");
    const size_t oe = elt_size(e.out_type);
    if (!aligned16(q.out) || (q.ldo * oe) % 16 || (q.out_group_stride * oe) % 16 ||
        (q.bias && (!aligned16(q.bias) || (q.bias_group_stride * 4) % 16)))
        return fail(ANCHA_E_UNSUPPORTED, "gemm_tc: output not 16-byte aligned");
    TcParams p{};
    p.m = q.m; p.n = q.n; p.k = q.k; p.groups = q.groups; p.b_groups = q.b_groups;
    p.group_n = q.group_n;
    p.out = q.out; p.ldo = q.ldo; p.out_group_stride = q.out_group_stride;
    p.bias = q.bias; p.bias_group_stride = q.bias_group_stride;
    p.residual = nullptr; p.ldr = 0;
    p.act = e.act; p.out_type = e.out_type;
    p.rope = nullptr; p.rope_pairs = nullptr; p.rope_width = 0; p.rope_tokens = 1; p.rope_div = 1; p.rope_hd = 64;
    p.split3 = q.split3 ? 1 : 0;
    if (q.split3 && ab_type != ELT_BF16) return fail(ANCHA_E_INVALID, "gemm_tc: split operands are bf16");
    return run(q.a, q.lda, q.a_group_stride, q.b, q.ldb, q.b_group_stride, p, ab_type, s);
}


namespace {
__global__ void rope_quads_kernel(const float* __restrict__ tab, int tokens, int hd, float4* __restrict__ quads,
                                  int64_t total) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= total) return;
    const int64_t per_key = (int64_t)(hd / 2) * tokens;
    const int key = (int)(i / per_key);
    const int64_t rem = i - key * per_key;
    const int pair = (int)(rem / tokens), t = (int)(rem - (int64_t)pair * tokens);
    const float* c = tab + ((int64_t)(2 * key) * tokens + t) * hd + 2 * pair;
    const float* sn = tab + ((int64_t)(2 * key + 1) * tokens + t) * hd + 2 * pair;
    quads[i] = make_float4(c[0], c[1], sn[0], sn[1]);
}
}  // namespace

int rope_quads_from_table(const float* table, int tokens, int hd, void* quads, cudaStream_t s) {
    const int64_t total = (int64_t)2 * (hd / 2) * tokens;
    if (total == 0) return ANCHA_OK;
    rope_quads_kernel<<<(unsigned)ceil_div(total, 256), 256, 0, s>>>(table, tokens, hd,
                                                                      reinterpret_cast<float4*>(quads), total);
    return check_launch("rope_quads");
}

}  // namespace ancha
