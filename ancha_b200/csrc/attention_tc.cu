// Single-pass attention on the tcgen05 tensor cores for head width 64, f16 / bf16 operands:
// softmax(q·kᵀ)·v per (group, head), q pre-scaled, optionally gated by sigmoid(gate).
//
// Q, K and V tiles are TMA-loaded from the packed q|k|v|gate projection through one 4-D
// tensor map {columns, tokens, inner groups, outer groups}, so the time axis (tokens
// contiguous) and the band axis (tokens T rows apart) run on the model's one layout and
// nothing is transposed. Each tile is 128 query rows; S = Q·Kᵀ (M 128, N 128) accumulates in
// TMEM, the softmax warps (one query row per thread) read it with tcgen05.ld, take base-2
// exponentials on the MUFU pipe (log2 e folded into the row maximum), write P in f16 / bf16
// to shared memory in the UMMA K-major 128-byte-swizzled layout, and O = P·V (V as an
// MN-major operand) accumulates in TMEM.
//
// Two kernels: attention_pp_kernel for tokens > 64 (the time axis, online softmax over key
// blocks, one query tile per CTA, two CTAs per SM) and attention_band_kernel for tokens ≤ 64
// (the band axis, two problems per tile, persistent and pipelined across tiles).
#include <algorithm>

#include "attention.cuh"
#include "tc.cuh"

namespace ancha {
namespace {

constexpr int TILE = 128;           // query rows / keys per block
constexpr int HD = 64;              // head width
constexpr int QKV_BYTES = TILE * HD * 2;
constexpr float LOG2E = 1.4426950408889634f;

struct AttnTcParams {
    int tokens, group_inner, group_outer, tiles_per_group;
    int q_col, k_col, v_col, gate_col, out_col;
    const void* q;
    void* out;
    int64_t ld, out_ld, group_inner_stride, group_outer_stride, token_stride;
    uint32_t idesc_s, idesc_o;
    uint32_t idesc_s_half;  // S with N = 64 keys: a last key block with at most 64 valid keys
    int* err;
};

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float a, float b) {
    if (BF16) {
        __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    } else {
        __half2 h = __floats2half2_rn(a, b);
        return *reinterpret_cast<uint32_t*>(&h);
    }
}

// Softmax exponentials 2^(s·log2 e − m) of one row of scores, split between two pipes: the MUFU
// unit (ex2.approx, 16 results per SM per clock) and the FMA pipe. With head width 64 a score
// costs the tensor cores 256 flop, so MUFU alone delivers exponentials at half the rate the
// tensor cores consume scores; of every 8 column pairs POLY_PAIRS take the FMA-pipe form.
//
// FMA-pipe exp2 (Cody–Waite style range reduction, polynomial fitted here): for x =
// s·log2 e − m, t = x + 1.5·2^23 = 1.5·2^23 + j with j = round(x) (the sum's ulp is 1, so the
// addition rounds x to an integer held in the low mantissa bits), f = x − (t − 1.5·2^23) = x − j
// ∈ [−0.5, 0.5] exactly; 2^f ≈ P3(f), a degree-3 minimax fit of 2^f on [−0.5, 0.5] by Remez
// exchange on the relative error (max 7.5e-5 in f32 Horner evaluation, below the 16-bit
// rounding of P); and 2^j is added to the exponent field as bits(P) + (bits(t) << 23), the shift
// keeping j's low 9 bits in two's complement. Scores are clamped to x ≥ −124 first so the
// result stays a normal number; x ≤ 8 holds by the lazy rescale.
#ifndef ANCHA_ATTN_POLY_PAIRS
#define ANCHA_ATTN_POLY_PAIRS 2
#endif
constexpr int POLY_PAIRS = ANCHA_ATTN_POLY_PAIRS;
constexpr float EXP2_ROUND = 12582912.f;  // 1.5·2^23
constexpr float EXP2_C0 = 0.9999280571937561f, EXP2_C1 = 0.6932609677314758f, EXP2_C2 = 0.2426111251115799f,
                EXP2_C3 = 0.0551716685295105f;

__device__ __forceinline__ void exp2_fma_pair(uint64_t x, float& e0, float& e1) {
    const uint64_t t = fadd2(x, f2(EXP2_ROUND, EXP2_ROUND));
    const uint64_t f = fsub2(x, fsub2(t, f2(EXP2_ROUND, EXP2_ROUND)));
    uint64_t p = ffma2(f, f2(EXP2_C3, EXP2_C3), f2(EXP2_C2, EXP2_C2));
    p = ffma2(p, f, f2(EXP2_C1, EXP2_C1));
    p = ffma2(p, f, f2(EXP2_C0, EXP2_C0));
    float p0, p1, t0, t1;
    f2_split(p, p0, p1);
    f2_split(t, t0, t1);
    e0 = __int_as_float(__float_as_int(p0) + (__float_as_int(t0) << 23));
    e1 = __int_as_float(__float_as_int(p1) + (__float_as_int(t1) << 23));
}

// Columns [J0, J0 + 64) of one score row: P as 16-bit pairs into pk (one TMEM store of 32
// columns), row sums into the packed accumulators sa / sb. s_lo clamps the scores of the
// FMA-pipe columns to x ≥ −124.
template <bool BF16, int J0>
__device__ __forceinline__ void exp_columns(const uint32_t (&s)[4][32], uint32_t (&pk)[32], uint64_t& sa,
                                            uint64_t& sb, float m_used, float s_lo) {
    const uint64_t l2 = f2(LOG2E, LOG2E), nm2 = f2(-m_used, -m_used);
#pragma unroll
    for (int j = J0; j < J0 + 64; j += 2) {
        const float s0 = __uint_as_float(s[j / 32][j % 32]), s1 = __uint_as_float(s[j / 32][j % 32 + 1]);
        float e0, e1;
        if ((j / 2) % 8 < POLY_PAIRS) {
            exp2_fma_pair(ffma2(f2(fmaxf(s0, s_lo), fmaxf(s1, s_lo)), l2, nm2), e0, e1);
        } else {
            float x0, x1;
            f2_split(ffma2(f2(s0, s1), l2, nm2), x0, x1);
            e0 = ex2_approx(x0);
            e1 = ex2_approx(x1);
        }
        if ((j / 2) & 1)
            sb = fadd2(sb, f2(e0, e1));
        else
            sa = fadd2(sa, f2(e0, e1));
        pk[(j - J0) / 2] = pack2<BF16>(e0, e1);
    }
}

// Band-axis kernel (tokens ≤ 64). A persistent CTA walks tiles of two problems: inner groups
// gi0 and gi0 + 1 of one outer group and head, 128 query rows against one 128-key block
// whose cross-problem scores are ignored. Tiles stream through a 4-deep ring of Q | K | V
// stages so that the loads of later tiles are in flight while earlier ones compute: at 60
// tokens a tile moves 64 KB for 4 MFLOP and the axis is bound by HBM, not the tensor cores.
// Warps 0–3 and 4–7 are two softmax warpgroups that take alternate tiles (TMEM slot = tile
// parity: S at slot·128, O at 256 + slot·64); warp 8 issues TMA, warp 9 UMMA. A stage's Q | K
// bytes are reused for P once S = Q·Kᵀ has completed, and its V bytes for the output rows
// once P·V has completed; the output leaves through a TMA store that clips the padding rows
// (tokens ≥ `tokens`, a second group past the end).
constexpr int BD_STAGES = 4;
constexpr int BD_STAGE_BYTES = 3 * QKV_BYTES;
constexpr int BD_OFF_BAR = BD_STAGES * BD_STAGE_BYTES;
constexpr int BD_SMEM_BYTES = 1024 + BD_OFF_BAR + 20 * 8 + 16;
constexpr int BD_THREADS = 320;

template <bool BF16>
__global__ void __launch_bounds__(BD_THREADS, 1)
attention_band_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ CUtensorMap omap,
                      const AttnTcParams p, const int pairs, const int heads, const int total) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + BD_OFF_BAR);
    uint64_t* full = bars;          // [stage] Q | K | V landed
    uint64_t* empty = bars + 4;     // [stage] output stored, stage reusable
    uint64_t* s_full = bars + 8;    // [slot] S = Q·Kᵀ done
    uint64_t* p_ready = bars + 10;  // [slot] P written (128 arrivals)
    uint64_t* o_full = bars + 12;   // [slot] O = P·V done
    uint64_t* o_empty = bars + 14;  // [slot] O read (128 arrivals)
    uint64_t* staged = bars + 16;   // [slot] output rows written (128 arrivals)
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 18);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int my_tiles = (int)blockIdx.x < total ? (total - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    // Tile → (outer group, group pair, head); the head varies fastest, so CTAs running at the
    // same time read neighbouring column slices of the same rows.
    auto decode = [&](int i, int& go, int& gi0, int& head) {
        const int tile = (int)blockIdx.x + i * (int)gridDim.x;
        head = tile % heads;
        const int r = tile / heads;
        gi0 = 2 * (r % pairs);
        go = r / pairs;
    };

    if (threadIdx.x == 256) {
        for (int s = 0; s < BD_STAGES; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        for (int s = 0; s < 2; ++s) {
            mbar_init(&s_full[s], 1);
            mbar_init(&p_ready[s], 128);
            mbar_init(&o_full[s], 1);
            mbar_init(&o_empty[s], 128);
            mbar_init(&staged[s], 128);
        }
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tmap);
        prefetch_tma(&omap);
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 8) {
        if (lane == 0) {
            int issued = 0;
            for (int i = 0; i < my_tiles; ++i) {
                const int st = i % BD_STAGES;
                if (!mbar_wait(&empty[st], ((i / BD_STAGES) & 1) ^ 1, abort, p.err)) break;
                int go, gi0, head;
                decode(i, go, gi0, head);
                uint8_t* base = smem + st * BD_STAGE_BYTES;
                mbar_arrive_expect_tx(&full[st], 3 * QKV_BYTES);
                tma_load_4d(base, &tmap, &full[st], p.q_col + head * HD, 0, gi0, go);
                tma_load_4d(base + QKV_BYTES, &tmap, &full[st], p.k_col + head * HD, 0, gi0, go);
                tma_load_4d(base + 2 * QKV_BYTES, &tmap, &full[st], p.v_col + head * HD, 0, gi0, go);
                ++issued;
            }
            if (*abort) {  // let copies in flight land before the CTA exits (bounded)
                const long long c0 = clock64();
                for (int i = max(0, issued - BD_STAGES); i < issued; ++i)
                    while (!mbar_try_wait(&full[i % BD_STAGES], (i / BD_STAGES) & 1) &&
                           clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            auto issue_pv = [&](int j) -> bool {
                const int slot = j & 1;
                if (!mbar_wait(&p_ready[slot], (j >> 1) & 1, abort, p.err)) return false;
                if (j >= 2 && !mbar_wait(&o_empty[slot], ((j - 2) >> 1) & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint32_t p_addr = smem_u32(smem + (j % BD_STAGES) * BD_STAGE_BYTES);
                const uint32_t v_addr = p_addr + 2 * QKV_BYTES;
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk)
                    umma_f16(tmem + 256 + slot * HD,
                             umma_desc_sw128(p_addr + (kk >> 2) * (TILE * 128) + (kk & 3) * 32),
                             umma_desc_sw128(v_addr + kk * 16 * 128), p.idesc_o, kk != 0);
                umma_commit(&o_full[slot]);
                return true;
            };
            bool ok = true;
            for (int i = 0; i < my_tiles; ++i) {
                const int slot = i & 1, st = i % BD_STAGES;
                if (!mbar_wait(&full[st], (i / BD_STAGES) & 1, abort, p.err)) { ok = false; break; }
                // S(slot) is free once the softmax of tile i − 2 has read it (its P is ready).
                if (i >= 2 && !mbar_wait(&p_ready[slot], ((i - 2) >> 1) & 1, abort, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t q_addr = smem_u32(smem + st * BD_STAGE_BYTES);
                const uint32_t k_addr = q_addr + QKV_BYTES;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_f16(tmem + slot * TILE, umma_desc_sw128(q_addr + kk * 32),
                             umma_desc_sw128(k_addr + kk * 32), p.idesc_s, kk != 0);
                umma_commit(&s_full[slot]);
                if (i >= 1 && !issue_pv(i - 1)) { ok = false; break; }
            }
            if (ok && my_tiles > 0) issue_pv(my_tiles - 1);
        }
    } else {
        const int g = warp / 4, wq = warp % 4;
        const int row = threadIdx.x % 128;  // query row of the tile
        const int prob = wq / 2;            // rows 0–63: group gi0, rows 64–127: gi0 + 1
        const int tok = row % 64;
        const uint32_t lane_base = tmem + ((uint32_t)(wq * 32) << 16);
        for (int i = g; i < my_tiles; i += 2) {
            const int st = i % BD_STAGES, k = i >> 1;
            int go, gi0, head;
            decode(i, go, gi0, head);
            uint8_t* base = smem + st * BD_STAGE_BYTES;
            if (!__all_sync(0xffffffffu, mbar_wait(&s_full[g], k & 1, abort, p.err))) break;
            tc_fence_after();
            // Scores of this row against its own problem's keys (columns prob·64 ..).
            uint32_t ra[32], rb[32];
            tmem_ld32(lane_base + g * TILE + prob * 64, ra);
            tmem_ld32(lane_base + g * TILE + prob * 64 + 32, rb);
            tmem_wait_ld();
            float mx = -INFINITY;
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if (j < p.tokens) mx = fmaxf(mx, __uint_as_float(ra[j]));
                if (32 + j < p.tokens) mx = fmaxf(mx, __uint_as_float(rb[j]));
            }
            const float m = mx * LOG2E;
            float rowsum = 0.f;
            uint32_t pk[32];
#pragma unroll
            for (int j = 0; j < 64; j += 2) {
                const float s0 = __uint_as_float(j < 32 ? ra[j] : rb[j - 32]);
                const float s1 = __uint_as_float(j + 1 < 32 ? ra[j + 1] : rb[j + 1 - 32]);
                const float e0 = j < p.tokens ? ex2_approx(fmaf(s0, LOG2E, -m)) : 0.f;
                const float e1 = j + 1 < p.tokens ? ex2_approx(fmaf(s1, LOG2E, -m)) : 0.f;
                rowsum += e0 + e1;
                pk[j / 2] = pack2<BF16>(e0, e1);
            }
            // P row over the tile's 128 keys (K-major, 128-byte swizzle, over Q | K): this
            // problem's half holds the probabilities, the other half zeros.
            uint8_t* own = base + prob * (TILE * 128) + row * 128;
            uint8_t* other = base + (1 - prob) * (TILE * 128) + row * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int chunk = q ^ (row & 7);
                *reinterpret_cast<uint4*>(own + chunk * 16) = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                *reinterpret_cast<uint4*>(other + chunk * 16) = make_uint4(0u, 0u, 0u, 0u);
            }
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&p_ready[g]);

            if (!__all_sync(0xffffffffu, mbar_wait(&o_full[g], k & 1, abort, p.err))) break;
            tc_fence_after();
            tmem_ld32(lane_base + 256 + g * HD, ra);
            tmem_ld32(lane_base + 256 + g * HD + 32, rb);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(&o_empty[g]);
            const int gi = gi0 + prob;
            const bool valid = tok < p.tokens && gi < p.group_inner;
            float scale = valid ? 1.f / rowsum : 0.f;
            if (valid && p.gate_col >= 0) {
                const int64_t orow = (int64_t)go * p.group_outer_stride + (int64_t)gi * p.group_inner_stride +
                                     (int64_t)tok * p.token_stride;
                const float gl = BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[orow * p.ld + p.gate_col + head])
                                      : __half2float(reinterpret_cast<const __half*>(p.q)[orow * p.ld + p.gate_col + head]);
                scale /= 1.f + __expf(-gl);
            }
            // Output row into the stage's V bytes in the TMA layout (128-byte swizzle).
            uint8_t* orow_s = base + 2 * QKV_BYTES + row * 128;
#pragma unroll
            for (int q = 0; q < 8; ++q) {
                const int chunk = q ^ (row & 7);
                float v[8];
#pragma unroll
                for (int u = 0; u < 8; ++u)
                    v[u] = __uint_as_float(q < 4 ? ra[8 * q + u] : rb[8 * (q - 4) + u]) * scale;
                *reinterpret_cast<uint4*>(orow_s + chunk * 16) =
                    make_uint4(pack2<BF16>(v[0], v[1]), pack2<BF16>(v[2], v[3]), pack2<BF16>(v[4], v[5]),
                               pack2<BF16>(v[6], v[7]));
            }
            fence_proxy_async();
            mbar_arrive(&staged[g]);
            if (row == 0) {
                if (mbar_wait(&staged[g], k & 1, abort, p.err)) {
                    tma_store_4d(&omap, base + 2 * QKV_BYTES, p.out_col + head * HD, 0, gi0, go);
                    bulk_commit();
                    bulk_wait_read<0>();
                }
                mbar_arrive(&empty[st]);
            }
        }
        if (row == 0) bulk_wait<0>();
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tmem_dealloc(tmem, 512);
    }
}

// Time-axis kernel (tokens > 64): one 128-row query tile per CTA and two CTAs per SM. Warps
// 0–3 run the softmax (one query row per thread), warp 4 issues TMA (Q once, then K and V blocks
// through two 2-deep rings), warp 5 issues UMMA. A tcgen05.mma issue costs a fixed ~80 cycles
// whatever its N, so one issuing thread cannot keep the tensor cores busy with these small
// (N = 128 / 64, K = 16) instructions; two co-resident CTAs give each SM two independent issue
// streams, and the tensor cores interleave them (measured: 18–20 % faster than two query tiles
// sharing one CTA and one issuer).
//
// TMEM (256 columns per CTA): S at 0 (128), the output accumulator O at 128 (64) and P (16-bit
// pairs, the A operand of P·V) at 192 (64). The softmax copies its row of S(kb) into registers
// and releases the buffer at once, so S(kb+1) = Q·K(kb+1)ᵀ runs while the exponentials of kb
// are computed; P(kb) goes back to TMEM and the UMMA warp accumulates O += P(kb)·V(kb). The
// running maximum is updated lazily: it moves (and O, l are rescaled in TMEM) only when a row's
// block maximum exceeds it by more than 2^8, so P stays ≤ 256 and the rescale is rare.
// Interior key blocks skip masking.
constexpr int PP_K_STAGES = 2, PP_V_STAGES = 2;  // deeper rings measured no faster
constexpr int PP_OFF_Q = 0, PP_OFF_K = QKV_BYTES, PP_OFF_V = PP_OFF_K + PP_K_STAGES * QKV_BYTES;
constexpr int PP_OFF_BAR = PP_OFF_V + PP_V_STAGES * QKV_BYTES;
constexpr int PP_NBARS = 1 + 2 * PP_K_STAGES + 2 * PP_V_STAGES + 4;
constexpr int PP_SMEM_BYTES = 1024 + PP_OFF_BAR + PP_NBARS * 8 + 16;
constexpr int PP_THREADS = 192;
constexpr float PP_RESCALE_LOG2 = 8.f;
constexpr uint32_t PP_TMEM_COLS = 256, PP_O_COL = 128, PP_P_COL = 192;

template <bool BF16>
__global__ void __launch_bounds__(PP_THREADS, 2)
attention_pp_kernel(const __grid_constant__ CUtensorMap tmap, const AttnTcParams p) {
    constexpr int SOFT = 128;  // softmax threads
    constexpr int TMA_WARP = 4, MMA_WARP = 5;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PP_OFF_BAR);
    uint64_t* q_full = bars;
    // K and V run through separate rings: a K stage is free once S(kb) is done, a V stage once
    // P·V(kb) is, so the load of K(kb + 2) starts a block earlier than with shared K | V stages.
    uint64_t* k_full = bars + 1;                                  // [K stage]
    uint64_t* k_empty = k_full + PP_K_STAGES;                     // [K stage]
    uint64_t* v_full = k_empty + PP_K_STAGES;                     // [V stage]
    uint64_t* v_empty = v_full + PP_V_STAGES;                     // [V stage]
    uint64_t* s_full = v_empty + PP_V_STAGES;                     // S(kb) computed
    uint64_t* s_free = s_full + 1;                                // S(kb) copied to registers (128 arrivals)
    uint64_t* p_ready = s_full + 2;                               // P(kb) written (128 arrivals)
    uint64_t* pv_done = s_full + 3;                               // O += P(kb)·V(kb) completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + PP_NBARS);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tile = blockIdx.x % p.tiles_per_group;
    const int gi = blockIdx.x / p.tiles_per_group;
    const int go = blockIdx.z, head = blockIdx.y;
    const int nkb = p.tiles_per_group;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = tile * TILE;  // first query token of the tile

    if (threadIdx.x == SOFT) {
        mbar_init(q_full, 1);
        for (int s = 0; s < PP_K_STAGES; ++s) {
            mbar_init(&k_full[s], 1);
            mbar_init(&k_empty[s], 1);
        }
        for (int s = 0; s < PP_V_STAGES; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, SOFT);
        mbar_init(p_ready, SOFT);
        mbar_init(pv_done, 1);
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tmap);
    }
    if (warp == MMA_WARP) {
        tmem_alloc(tmem_slot, PP_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == TMA_WARP) {
        // Lane 0 loads Q and the K ring, lane 1 the V ring.
        if (lane < 2) {
            const bool is_k = lane == 0;
            uint64_t* full = is_k ? k_full : v_full;
            uint64_t* empty = is_k ? k_empty : v_empty;
            const int off = is_k ? PP_OFF_K : PP_OFF_V;
            const int col = (is_k ? p.k_col : p.v_col) + head * HD;
            const int stages = is_k ? PP_K_STAGES : PP_V_STAGES;
            if (is_k) {
                mbar_arrive_expect_tx(q_full, QKV_BYTES);
                tma_load_4d(smem + PP_OFF_Q, &tmap, q_full, p.q_col + head * HD, q0, gi, go);
            }
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb % stages;
                if (!mbar_wait(&empty[s], ((kb / stages) & 1) ^ 1, abort, p.err)) break;
                mbar_arrive_expect_tx(&full[s], QKV_BYTES);
                tma_load_4d(smem + off + s * QKV_BYTES, &tmap, &full[s], col, kb * TILE, gi, go);
                ++issued;
            }
            if (*abort) {  // let copies in flight land before the CTA exits (bounded)
                const long long c0 = clock64();
                if (is_k)
                    while (!mbar_try_wait(q_full, 0) && clock64() - c0 < kWaitCycles) {
                    }
                for (int kb = max(0, issued - stages); kb < issued; ++kb)
                    while (!mbar_try_wait(&full[kb % stages], (kb / stages) & 1) &&
                           clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == MMA_WARP) {
        if (lane == 0) {
            // Per key block j: S(j + 1) once the softmax has copied S(j) out, then P(j)·V(j) once
            // it has written P(j).
            const uint64_t q_desc = umma_desc_sw128(smem_u32(smem + PP_OFF_Q));
            auto issue_s = [&](int j) -> bool {
                if (j >= 1 && !mbar_wait(s_free, (j - 1) & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint64_t k_desc = umma_desc_sw128(smem_u32(smem + PP_OFF_K + (j % PP_K_STAGES) * QKV_BYTES));
                // A key block with at most 64 valid keys (the last one) computes only S[:, 0:64];
                // the softmax then reads only those columns.
                const uint32_t idesc = p.tokens - j * TILE <= TILE / 2 ? p.idesc_s_half : p.idesc_s;
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)  // K step of 16 = 32 bytes = 2 descriptor units
                    umma_f16(tmem, q_desc + 2 * kk, k_desc + 2 * kk, idesc, kk != 0);
                umma_commit(s_full);
                return true;
            };
            auto issue_pv = [&](int k) -> bool {
                if (!mbar_wait(p_ready, k & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint64_t v_desc = umma_desc_sw128(smem_u32(smem + PP_OFF_V + (k % PP_V_STAGES) * QKV_BYTES));
                // Steps of 16 keys up to the last valid key: P is 0 beyond it.
                const int steps = min(TILE / 16, (p.tokens - k * TILE + 15) / 16);
                // 16 keys = 16 rows of 128 bytes = 128 descriptor units; the full-block case is
                // unrolled (the issuing thread's loop overhead is comparable to an N = 64 UMMA).
                if (steps == TILE / 16) {
#pragma unroll
                    for (int kk = 0; kk < TILE / 16; ++kk)
                        umma_f16_ts(tmem + PP_O_COL, tmem + PP_P_COL + kk * 8, v_desc + 128 * kk, p.idesc_o,
                                    (k > 0 || kk > 0) ? 1u : 0u);
                } else {
                    for (int kk = 0; kk < steps; ++kk)
                        umma_f16_ts(tmem + PP_O_COL, tmem + PP_P_COL + kk * 8, v_desc + 128 * kk, p.idesc_o,
                                    (k > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(pv_done);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort, p.err) && mbar_wait(&k_full[0], 0, abort, p.err) && issue_s(0);
            if (ok) umma_commit(&k_empty[0]);  // fires once S(0) is done
            for (int j = 0; ok && j < nkb; ++j) {
                if (j + 1 < nkb) {
                    const int s1 = (j + 1) % PP_K_STAGES;
                    ok = mbar_wait(&k_full[s1], ((j + 1) / PP_K_STAGES) & 1, abort, p.err) && issue_s(j + 1);
                    if (ok) umma_commit(&k_empty[s1]);
                }
                if (ok) ok = mbar_wait(&v_full[j % PP_V_STAGES], (j / PP_V_STAGES) & 1, abort, p.err) && issue_pv(j);
                if (ok) umma_commit(&v_empty[j % PP_V_STAGES]);  // fires once P·V(j) is done
            }
        }
    } else {
        const int row = threadIdx.x;  // query row of the tile (warps 0–3)
        const int tok = q0 + row;
        const bool valid = tok < p.tokens;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const uint32_t s_addr = tmem + lane_off;
        const uint32_t o_addr = tmem + lane_off + PP_O_COL;
        const uint32_t p_addr = tmem + lane_off + PP_P_COL;
        // A warp whose 32 query rows all lie past the last token (in the last tile of a group)
        // has no output: it computes nothing and only keeps the barrier phases in step. Its
        // TMEM lanes of P and O hold stale values, which reach only its own (discarded) rows.
        const bool live = q0 + warp * 32 < p.tokens;
        float m_used = -INFINITY, l = 0.f;
        float s_lo = 0.f;  // score clamp of the FMA-pipe exp2 columns
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full, kb & 1, abort, p.err));
            if (!ok) break;
            if (!live) {
                mbar_arrive(s_free);
                // P(kb − 1) is complete (so the arrival below counts toward P(kb)) once its
                // product has finished.
                if (kb > 0) {
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (kb - 1) & 1, abort, p.err));
                    if (!ok) break;
                }
                mbar_arrive(p_ready);
                continue;
            }
            tc_fence_after();
            uint32_t s[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, s[c]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free);  // the tensor cores may compute S(kb + 1) now
            const int nvalid = min(TILE, p.tokens - kb * TILE);  // valid keys in this block
            // With at most 64 valid keys S holds keys 0..63 only (N = 64); the masking below
            // covers the stale columns 64..127 as well, and their exponentials are skipped.
            const bool half = nvalid <= TILE / 2;
            if (nvalid < TILE) {
#pragma unroll
                for (int c = 0; c < TILE; ++c)
                    if (c >= nvalid) s[c / 32][c % 32] = __float_as_uint(-INFINITY);
            }
            float mx0 = -INFINITY, mx1 = -INFINITY, mx2 = -INFINITY, mx3 = -INFINITY;
#pragma unroll
            for (int c = 0; c < TILE; c += 8) {
                mx0 = fmax3(mx0, __uint_as_float(s[c / 32][c % 32]), __uint_as_float(s[c / 32][c % 32 + 1]));
                mx1 = fmax3(mx1, __uint_as_float(s[c / 32][c % 32 + 2]), __uint_as_float(s[c / 32][c % 32 + 3]));
                mx2 = fmax3(mx2, __uint_as_float(s[c / 32][c % 32 + 4]), __uint_as_float(s[c / 32][c % 32 + 5]));
                mx3 = fmax3(mx3, __uint_as_float(s[c / 32][c % 32 + 6]), __uint_as_float(s[c / 32][c % 32 + 7]));
            }
            const float m_blk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * LOG2E;
            float corr = 1.f;
            if (m_blk > m_used + PP_RESCALE_LOG2) {  // also the first block (m_used = −∞)
                corr = m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_blk);
                m_used = m_blk;
                l *= corr;
                s_lo = (m_used - 124.f) * (1.f / LOG2E);
            }
            // P = 2^(s·log2 e − m_used) as 16-bit pairs: keys 0..63 are computed before the wait
            // for P(kb − 1)·V, which then has had that part of the exponential pass to finish,
            // and stored; keys 64..127 follow (skipped when the block has at most 64 valid keys:
            // P·V of such a block reads keys 0..63 only).
            uint64_t sa = 0, sb = 0;
            {
                uint32_t pk[32];
                exp_columns<BF16, 0>(s, pk, sa, sb, m_used, s_lo);
                if (kb > 0) {
                    // P(kb − 1)·V must have finished reading P before it is overwritten, and O
                    // must hold it before a rescale.
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (kb - 1) & 1, abort, p.err));
                    if (!ok) break;
                    tc_fence_after();
                }
                tmem_st32(p_addr, pk);
            }
            if (kb > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                uint32_t o[2][32];
                tmem_ld32(o_addr, o[0]);
                tmem_ld32(o_addr + 32, o[1]);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < 32; ++d) {
                    o[0][d] = __float_as_uint(__uint_as_float(o[0][d]) * corr);
                    o[1][d] = __float_as_uint(__uint_as_float(o[1][d]) * corr);
                }
                tmem_st32(o_addr, o[0]);
                tmem_st32(o_addr + 32, o[1]);
            }
            if (!half) {
                uint32_t pk[32];
                exp_columns<BF16, TILE / 2>(s, pk, sa, sb, m_used, s_lo);
                tmem_st32(p_addr + 32, pk);
            }
            float sum0, sum1, sum2, sum3;
            f2_split(sa, sum0, sum1);
            f2_split(sb, sum2, sum3);
            l += (sum0 + sum2) + (sum1 + sum3);
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_ready);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nkb - 1) & 1, abort, p.err));
        if (ok) {
            tc_fence_after();
            uint32_t o[2][32];
            tmem_ld32(o_addr, o[0]);
            tmem_ld32(o_addr + 32, o[1]);
            tmem_wait_ld();
            if (valid) {
                const int64_t orow = (int64_t)go * p.group_outer_stride + (int64_t)gi * p.group_inner_stride +
                                     (int64_t)tok * p.token_stride;
                float scale = 1.f / l;
                if (p.gate_col >= 0) {
                    const float gl = BF16 ? __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p.q)[orow * p.ld + p.gate_col + head])
                                          : __half2float(reinterpret_cast<const __half*>(p.q)[orow * p.ld + p.gate_col + head]);
                    scale /= 1.f + __expf(-gl);
                }
                uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(p.out) +
                                                      (orow * p.out_ld + p.out_col + head * HD) * 2);
#pragma unroll
                for (int q = 0; q < HD / 8; ++q) {
                    float v[8];
#pragma unroll
                    for (int u = 0; u < 8; ++u) v[u] = __uint_as_float(o[q / 4][(q % 4) * 8 + u]) * scale;
                    dst[q] = make_uint4(pack2<BF16>(v[0], v[1]), pack2<BF16>(v[2], v[3]),
                                        pack2<BF16>(v[4], v[5]), pack2<BF16>(v[6], v[7]));
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == MMA_WARP) {
        __syncwarp();
        tmem_dealloc(tmem, PP_TMEM_COLS);
    }
}

template <bool BF16>
int launch_pp(const CUtensorMap& map, const AttnTcParams& p, dim3 grid, cudaStream_t s) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(attention_pp_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        PP_SMEM_BYTES));
        configured[dev & 63] = true;
    }
    attention_pp_kernel<BF16><<<grid, PP_THREADS, PP_SMEM_BYTES, s>>>(map, p);
    return check_launch("attention_pp");
}

template <bool BF16>
int launch_band(const CUtensorMap& map, const CUtensorMap& omap, const AttnTcParams& p, int pairs, int heads,
                int total, cudaStream_t s) {
    static bool configured[64] = {};
    static int sms[64] = {};
    int dev = 0;
    ANCHA_CUDA(cudaGetDevice(&dev));
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(attention_band_kernel<BF16>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        BD_SMEM_BYTES));
        ANCHA_CUDA(cudaDeviceGetAttribute(&sms[dev & 63], cudaDevAttrMultiProcessorCount, dev));
        configured[dev & 63] = true;
    }
    const int grid = std::min(total, sms[dev & 63]);
    attention_band_kernel<BF16><<<grid, BD_THREADS, BD_SMEM_BYTES, s>>>(map, omap, p, pairs, heads, total);
    return check_launch("attention_band");
}

// fp32 mode on the tensor cores (both axes: a band-axis problem of ≤ 64 tokens is one tile with
// one key block). The f32 q / k / v arrive split into
// three bf16 planes, x = hi + mid + lo with hi = bf16(x), mid = bf16(x − hi), lo = bf16(x − hi −
// mid) (24 significant bits), and each product runs as the six plane products whose weight is at
// least 2^-24 of the leading one (mm, lh, hl, mh, hm, hh, in that order), accumulated in f32 in TMEM:
// S = Q·Kᵀ as 6 × 4 UMMAs per key block, O += P·V as 6 × 8, with P (f32 probabilities ≤ 2^8)
// split into three bf16 planes by the softmax and stored to TMEM as the A operand. The
// exponentials are MUFU ex2.approx only (no polynomial columns). One CTA per SM: TMEM holds S
// (128 columns), O (64) and the three P planes (3 × 64) in 512 columns. Shared memory holds the
// three Q planes, one K stage and two V stages (three planes each). Warp roles, barriers and
// the lazy rescale are those of attention_pp_kernel.
constexpr int SP_PLANE = QKV_BYTES;  // one 128 × 64 bf16 tile
constexpr int SP_V_STAGES = 2;
constexpr int SP_OFF_Q = 0, SP_OFF_K = 3 * SP_PLANE, SP_OFF_V = SP_OFF_K + 3 * SP_PLANE;
constexpr int SP_OFF_BAR = SP_OFF_V + SP_V_STAGES * 3 * SP_PLANE;
constexpr int SP_NBARS = 3 + 2 * SP_V_STAGES + 4;
constexpr int SP_SMEM_BYTES = 1024 + SP_OFF_BAR + SP_NBARS * 8 + 16;
constexpr uint32_t SP_TMEM_COLS = 512, SP_O_COL = 128, SP_P_COL = 256;

// Plane of the A and B operands in each of the six products, smallest weight first (mm, lh, hl,
// mh, hm, hh): each product is added to the f32 accumulator with one rounding at the
// accumulator's magnitude, so the small products are summed before the large one arrives.
__device__ __forceinline__ int split_a(int t) { return t == 0 || t == 3 ? 1 : t == 1 ? 2 : 0; }
__device__ __forceinline__ int split_b(int t) { return t == 0 || t == 4 ? 1 : t == 2 ? 2 : 0; }

struct PlaneMaps {
    CUtensorMap plane[3];  // {columns, tokens, inner groups, outer groups} over each bf16 plane
};

// Splits a pair of f32 probabilities into the hi / mid / lo bf16 pairs of the three P planes.
__device__ __forceinline__ void split_pair(float e0, float e1, uint32_t& h, uint32_t& m, uint32_t& l) {
    const __nv_bfloat162 hh = __floats2bfloat162_rn(e0, e1);
    const float r0 = e0 - __low2float(hh), r1 = e1 - __high2float(hh);
    const __nv_bfloat162 mm = __floats2bfloat162_rn(r0, r1);
    const __nv_bfloat162 ll = __floats2bfloat162_rn(r0 - __low2float(mm), r1 - __high2float(mm));
    h = *reinterpret_cast<const uint32_t*>(&hh);
    m = *reinterpret_cast<const uint32_t*>(&mm);
    l = *reinterpret_cast<const uint32_t*>(&ll);
}

// Exponentials of score columns [J0, J0 + 64) (MUFU), the three P planes of those columns
// (32 packed words each) and the row sum in f32.
template <int J0>
__device__ __forceinline__ void exp_planes(const uint32_t (&s)[4][32], uint32_t (&ph)[32], uint32_t (&pm)[32],
                                           uint32_t (&pl)[32], float& sum, float m_used) {
    float acc0 = 0.f, acc1 = 0.f;
#pragma unroll
    for (int j = J0; j < J0 + 64; j += 2) {
        const float e0 = ex2_approx(fmaf(__uint_as_float(s[j / 32][j % 32]), LOG2E, -m_used));
        const float e1 = ex2_approx(fmaf(__uint_as_float(s[j / 32][j % 32 + 1]), LOG2E, -m_used));
        acc0 += e0;
        acc1 += e1;
        split_pair(e0, e1, ph[(j - J0) / 2], pm[(j - J0) / 2], pl[(j - J0) / 2]);
    }
    sum += acc0 + acc1;
}

__global__ void __launch_bounds__(PP_THREADS, 1)
attention_split_kernel(const __grid_constant__ PlaneMaps maps, const AttnTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SP_OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* k_full = bars + 1;
    uint64_t* k_empty = bars + 2;
    uint64_t* v_full = bars + 3;                 // [V stage]
    uint64_t* v_empty = v_full + SP_V_STAGES;    // [V stage]
    uint64_t* s_full = v_empty + SP_V_STAGES;    // S(kb) computed
    uint64_t* s_free = s_full + 1;               // S(kb) copied to registers (128 arrivals)
    uint64_t* p_ready = s_full + 2;              // P(kb) planes written (128 arrivals)
    uint64_t* pv_done = s_full + 3;              // O += P(kb)·V(kb) completed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + SP_NBARS);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tile = blockIdx.x % p.tiles_per_group;
    const int gi = blockIdx.x / p.tiles_per_group;
    const int go = blockIdx.z, head = blockIdx.y;
    const int nkb = p.tiles_per_group;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = tile * TILE;

    if (threadIdx.x == 128) {
        mbar_init(q_full, 1);
        mbar_init(k_full, 1);
        mbar_init(k_empty, 1);
        for (int s = 0; s < SP_V_STAGES; ++s) {
            mbar_init(&v_full[s], 1);
            mbar_init(&v_empty[s], 1);
        }
        mbar_init(s_full, 1);
        mbar_init(s_free, 128);
        mbar_init(p_ready, 128);
        mbar_init(pv_done, 1);
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        for (int pl = 0; pl < 3; ++pl) prefetch_tma(&maps.plane[pl]);
    }
    if (warp == 5) {
        tmem_alloc(tmem_slot, SP_TMEM_COLS);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            // Q once; per key block K(kb) into the one K stage (free once S(kb − 1) is done),
            // then V(kb) into stage kb mod 2 (free once P·V(kb − 2) is done, which precedes
            // S(kb) in the UMMA stream, so the V wait never holds up the next K load).
            mbar_arrive_expect_tx(q_full, 3 * SP_PLANE);
            for (int pl = 0; pl < 3; ++pl)
                tma_load_4d(smem + SP_OFF_Q + pl * SP_PLANE, &maps.plane[pl], q_full, p.q_col + head * HD, q0, gi, go);
            int nk = 0, nv = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                if (!mbar_wait(k_empty, (kb & 1) ^ 1, abort, p.err)) break;
                mbar_arrive_expect_tx(k_full, 3 * SP_PLANE);
                for (int pl = 0; pl < 3; ++pl)
                    tma_load_4d(smem + SP_OFF_K + pl * SP_PLANE, &maps.plane[pl], k_full, p.k_col + head * HD,
                                kb * TILE, gi, go);
                ++nk;
                const int sv = kb % SP_V_STAGES;
                if (!mbar_wait(&v_empty[sv], ((kb / SP_V_STAGES) & 1) ^ 1, abort, p.err)) break;
                mbar_arrive_expect_tx(&v_full[sv], 3 * SP_PLANE);
                for (int pl = 0; pl < 3; ++pl)
                    tma_load_4d(smem + SP_OFF_V + (sv * 3 + pl) * SP_PLANE, &maps.plane[pl], &v_full[sv],
                                p.v_col + head * HD, kb * TILE, gi, go);
                ++nv;
            }
            if (*abort) {  // let copies in flight land before the CTA exits (bounded)
                const long long c0 = clock64();
                while (!mbar_try_wait(q_full, 0) && clock64() - c0 < kWaitCycles) {
                }
                if (nk > 0)
                    while (!mbar_try_wait(k_full, (nk - 1) & 1) && clock64() - c0 < kWaitCycles) {
                    }
                for (int kb = max(0, nv - SP_V_STAGES); kb < nv; ++kb)
                    while (!mbar_try_wait(&v_full[kb % SP_V_STAGES], (kb / SP_V_STAGES) & 1) &&
                           clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            const uint32_t q_base = smem_u32(smem + SP_OFF_Q), k_base = smem_u32(smem + SP_OFF_K);
            auto issue_s = [&](int j) -> bool {
                if (!mbar_wait(k_full, j & 1, abort, p.err)) return false;
                if (j >= 1 && !mbar_wait(s_free, (j - 1) & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint32_t idesc = p.tokens - j * TILE <= TILE / 2 ? p.idesc_s_half : p.idesc_s;
#pragma unroll
                for (int t = 0; t < 6; ++t) {
                    const uint64_t qd = umma_desc_sw128(q_base + split_a(t) * SP_PLANE);
                    const uint64_t kd = umma_desc_sw128(k_base + split_b(t) * SP_PLANE);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_f16(tmem, qd + 2 * kk, kd + 2 * kk, idesc, (t | kk) != 0);
                }
                umma_commit(s_full);
                umma_commit(k_empty);
                return true;
            };
            auto issue_pv = [&](int k) -> bool {
                const int sv = k % SP_V_STAGES;
                if (!mbar_wait(&v_full[sv], (k / SP_V_STAGES) & 1, abort, p.err)) return false;
                if (!mbar_wait(p_ready, k & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint32_t v_base = smem_u32(smem + SP_OFF_V + sv * 3 * SP_PLANE);
                const int steps = min(TILE / 16, (p.tokens - k * TILE + 15) / 16);
                for (int t = 0; t < 6; ++t) {
                    const uint64_t vd = umma_desc_sw128(v_base + split_b(t) * SP_PLANE);
                    const uint32_t pa = tmem + SP_P_COL + split_a(t) * (TILE / 2);
                    for (int kk = 0; kk < steps; ++kk)
                        umma_f16_ts(tmem + SP_O_COL, pa + kk * 8, vd + 128 * kk, p.idesc_o,
                                    (k > 0 || t > 0 || kk > 0) ? 1u : 0u);
                }
                umma_commit(pv_done);
                umma_commit(&v_empty[sv]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort, p.err) && issue_s(0);
            for (int j = 0; ok && j < nkb; ++j) {
                if (j + 1 < nkb) ok = issue_s(j + 1);
                if (ok) ok = issue_pv(j);
            }
        }
    } else {
        const int row = threadIdx.x;  // query row of the tile (warps 0–3)
        const int tok = q0 + row;
        const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
        const uint32_t s_addr = tmem + lane_off;
        const uint32_t o_addr = tmem + lane_off + SP_O_COL;
        const uint32_t p_addr = tmem + lane_off + SP_P_COL;
        const bool live = q0 + warp * 32 < p.tokens;
        float m_used = -INFINITY, l = 0.f;
        bool ok = true;
        for (int kb = 0; kb < nkb; ++kb) {
            ok = __all_sync(0xffffffffu, mbar_wait(s_full, kb & 1, abort, p.err));
            if (!ok) break;
            if (!live) {
                mbar_arrive(s_free);
                if (kb > 0) {
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (kb - 1) & 1, abort, p.err));
                    if (!ok) break;
                }
                mbar_arrive(p_ready);
                continue;
            }
            tc_fence_after();
            uint32_t s[4][32];
#pragma unroll
            for (int c = 0; c < 4; ++c) tmem_ld32(s_addr + c * 32, s[c]);
            tmem_wait_ld();
            tc_fence_before();
            mbar_arrive(s_free);
            const int nvalid = min(TILE, p.tokens - kb * TILE);
            const bool half = nvalid <= TILE / 2;
            if (nvalid < TILE) {
#pragma unroll
                for (int c = 0; c < TILE; ++c)
                    if (c >= nvalid) s[c / 32][c % 32] = __float_as_uint(-INFINITY);
            }
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int c = 0; c < TILE; c += 4) {
                mx0 = fmax3(mx0, __uint_as_float(s[c / 32][c % 32]), __uint_as_float(s[c / 32][c % 32 + 1]));
                mx1 = fmax3(mx1, __uint_as_float(s[c / 32][c % 32 + 2]), __uint_as_float(s[c / 32][c % 32 + 3]));
            }
            const float m_blk = fmaxf(mx0, mx1) * LOG2E;
            float corr = 1.f;
            if (m_blk > m_used + PP_RESCALE_LOG2) {
                corr = m_used == -INFINITY ? 0.f : ex2_approx(m_used - m_blk);
                m_used = m_blk;
                l *= corr;
            }
            {
                uint32_t ph[32], pm[32], pl[32];
                exp_planes<0>(s, ph, pm, pl, l, m_used);
                if (kb > 0) {
                    ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (kb - 1) & 1, abort, p.err));
                    if (!ok) break;
                    tc_fence_after();
                }
                tmem_st32(p_addr, ph);
                tmem_st32(p_addr + TILE / 2, pm);
                tmem_st32(p_addr + TILE, pl);
            }
            if (kb > 0 && __any_sync(0xffffffffu, corr != 1.f)) {
                uint32_t o[2][32];
                tmem_ld32(o_addr, o[0]);
                tmem_ld32(o_addr + 32, o[1]);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < 32; ++d) {
                    o[0][d] = __float_as_uint(__uint_as_float(o[0][d]) * corr);
                    o[1][d] = __float_as_uint(__uint_as_float(o[1][d]) * corr);
                }
                tmem_st32(o_addr, o[0]);
                tmem_st32(o_addr + 32, o[1]);
            }
            if (!half) {
                uint32_t ph[32], pm[32], pl[32];
                exp_planes<TILE / 2>(s, ph, pm, pl, l, m_used);
                tmem_st32(p_addr + 32, ph);
                tmem_st32(p_addr + TILE / 2 + 32, pm);
                tmem_st32(p_addr + TILE + 32, pl);
            }
            tmem_wait_st();
            tc_fence_before();
            mbar_arrive(p_ready);
        }
        if (ok) ok = __all_sync(0xffffffffu, mbar_wait(pv_done, (nkb - 1) & 1, abort, p.err));
        if (ok && live) {
            tc_fence_after();
            uint32_t o[2][32];
            tmem_ld32(o_addr, o[0]);
            tmem_ld32(o_addr + 32, o[1]);
            tmem_wait_ld();
            if (tok < p.tokens) {
                const int64_t orow = (int64_t)go * p.group_outer_stride + (int64_t)gi * p.group_inner_stride +
                                     (int64_t)tok * p.token_stride;
                float scale = 1.f / l;
                if (p.gate_col >= 0) {
                    const float gl = reinterpret_cast<const float*>(p.q)[orow * p.ld + p.gate_col + head];
                    scale /= 1.f + expf(-gl);
                }
                float4* dst = reinterpret_cast<float4*>(reinterpret_cast<float*>(p.out) + orow * p.out_ld + p.out_col +
                                                        head * HD);
#pragma unroll
                for (int q = 0; q < HD / 4; ++q)
                    dst[q] = make_float4(__uint_as_float(o[q / 8][(q % 8) * 4]) * scale,
                                         __uint_as_float(o[q / 8][(q % 8) * 4 + 1]) * scale,
                                         __uint_as_float(o[q / 8][(q % 8) * 4 + 2]) * scale,
                                         __uint_as_float(o[q / 8][(q % 8) * 4 + 3]) * scale);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 5) {
        __syncwarp();
        tmem_dealloc(tmem, SP_TMEM_COLS);
    }
}

int launch_split(const PlaneMaps& maps, const AttnTcParams& p, dim3 grid, cudaStream_t s) {
    static bool configured[64] = {};
    int dev = 0;
    ANCHA_CUDA(cudaGetDevice(&dev));
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(attention_split_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                        SP_SMEM_BYTES));
        configured[dev & 63] = true;
    }
    attention_split_kernel<<<grid, PP_THREADS, SP_SMEM_BYTES, s>>>(maps, p);
    return check_launch("attention_split");
}

}  // namespace

int attention_tc(const AttnArgs& a, cudaStream_t stream) {
    if (a.elt != ELT_BF16 && a.elt != ELT_F16) return fail(ANCHA_E_UNSUPPORTED, "attention_tc: operand type");
    if (a.head_dim != HD) return fail(ANCHA_E_UNSUPPORTED, "attention_tc: head_dim must be 64");
    if (a.groups == 0 || a.tokens == 0) return ANCHA_OK;
    // One tensor map over the q / k / v source needs them to share the buffer and row stride.
    if (a.q != a.k || a.q != a.v) return fail(ANCHA_E_UNSUPPORTED, "attention_tc: q, k, v must share one buffer");
    const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out);
    if (ob % 16 || (a.out_ld * 2) % 16 || (a.out_col * 2) % 16)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc: output not 16-byte aligned");
    if ((a.q_col * 2) % 16 || (a.k_col * 2) % 16 || (a.v_col * 2) % 16)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc: q / k / v columns not 16-byte aligned");
    const int BT = a.tokens <= 64 ? 64 : 128;
    const int BG = TILE / BT;
    AttnTcParams p{};
    p.tokens = a.tokens;
    p.group_inner = (int)a.group_inner;
    p.group_outer = (int)ceil_div(a.groups, a.group_inner);
    if ((int64_t)p.group_outer * a.group_inner != a.groups)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc: groups must be a multiple of group_inner");
    p.tiles_per_group = (int)ceil_div(a.tokens, BT);
    p.q_col = a.q_col; p.k_col = a.k_col; p.v_col = a.v_col;
    p.gate_col = a.gate ? a.gate_col : -1;
    p.out_col = a.out_col;
    p.q = a.gate ? a.gate : a.q;
    p.out = a.out;
    p.ld = a.ld; p.out_ld = a.out_ld;
    p.group_inner_stride = a.group_inner_stride;
    p.group_outer_stride = a.group_outer_stride;
    p.token_stride = a.token_stride;
    p.idesc_s = umma_idesc_f16(a.elt == ELT_BF16, TILE, TILE, 0);
    p.idesc_o = umma_idesc_f16(a.elt == ELT_BF16, TILE, HD, 1);
    p.idesc_s_half = umma_idesc_f16(a.elt == ELT_BF16, TILE, TILE / 2, 0);
    p.err = device_error_word();
    // Tensor map {columns, tokens, inner groups, outer groups}; unused strides still have to
    // be 16-byte multiples, so a one-long dimension reuses the row stride.
    const int64_t s1 = a.token_stride * a.ld;
    const int64_t s2 = a.group_inner_stride * a.ld;
    const int64_t s3 = p.group_outer > 1 ? a.group_outer_stride * a.ld : a.ld;
    CUtensorMap map;
    ANCHA_TRY(make_tma_4d(&map, a.q, a.elt, a.ld, a.tokens, a.group_inner, p.group_outer,
                          s1 > 0 ? s1 : a.ld, s2 > 0 ? s2 : a.ld, s3 > 0 ? s3 : a.ld, BT, BG));
    if (BT == 128) {
        // Time axis: one query tile of one (group, head) per CTA, two CTAs per SM.
        const int64_t gx = (int64_t)p.tiles_per_group * a.group_inner;
        if (gx > 0x7fffffff || a.heads > 65535 || p.group_outer > 65535)
            return fail(ANCHA_E_UNSUPPORTED, "attention_tc: grid too large");
        dim3 grid((unsigned)gx, (unsigned)a.heads, (unsigned)p.group_outer);
        return a.elt == ELT_BF16 ? launch_pp<true>(map, p, grid, stream) : launch_pp<false>(map, p, grid, stream);
    }
    // Band axis: persistent CTAs over (outer group, group pair, head) tiles; the output leaves
    // through a TMA store with the same {columns, tokens, inner groups, outer groups} shape.
    const int64_t pairs = ceil_div(a.group_inner, 2);
    const int64_t total = (int64_t)p.group_outer * pairs * a.heads;
    if (total > 0x7fffffff) return fail(ANCHA_E_UNSUPPORTED, "attention_tc: too many tiles");
    const int64_t o1 = a.token_stride * a.out_ld;
    const int64_t o2 = a.group_inner_stride * a.out_ld;
    const int64_t o3 = p.group_outer > 1 ? a.group_outer_stride * a.out_ld : a.out_ld;
    CUtensorMap omap;
    ANCHA_TRY(make_tma_4d(&omap, a.out, a.elt, a.out_col + (int64_t)a.heads * HD, a.tokens, a.group_inner,
                          p.group_outer, o1 > 0 ? o1 : a.out_ld, o2 > 0 ? o2 : a.out_ld, o3 > 0 ? o3 : a.out_ld,
                          BT, BG));
    return a.elt == ELT_BF16 ? launch_band<true>(map, omap, p, (int)pairs, a.heads, (int)total, stream)
                             : launch_band<false>(map, omap, p, (int)pairs, a.heads, (int)total, stream);
}


int attention_tc_split(const AttnArgs& a, const void* planes, int64_t plane_ld, int64_t plane_stride,
                       cudaStream_t stream) {
    if (a.elt != ELT_F32 || a.head_dim != HD)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: f32 with head_dim 64 only");
    if (a.groups == 0) return ANCHA_OK;
    if (a.q != a.k || a.q != a.v) return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: q, k, v must share one buffer");
    const uintptr_t pb = reinterpret_cast<uintptr_t>(planes);
    const int64_t span = (int64_t)a.heads * HD;
    if (plane_ld < std::max(std::max(a.q_col, a.k_col), a.v_col) + span)
        return fail(ANCHA_E_INVALID, "attention_tc_split: plane rows too short");
    if (pb % 16 || (plane_ld * 2) % 16 || (plane_stride * 2) % 16 || (a.q_col * 2) % 16 || (a.k_col * 2) % 16 ||
        (a.v_col * 2) % 16)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: planes not 16-byte aligned");
    const uintptr_t ob = reinterpret_cast<uintptr_t>(a.out);
    if (ob % 16 || (a.out_ld * 4) % 16 || (a.out_col * 4) % 16)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: output not 16-byte aligned");
    AttnTcParams p{};
    p.tokens = a.tokens;
    p.group_inner = (int)a.group_inner;
    p.group_outer = (int)ceil_div(a.groups, a.group_inner);
    if ((int64_t)p.group_outer * a.group_inner != a.groups)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: groups must be a multiple of group_inner");
    p.tiles_per_group = (int)ceil_div(a.tokens, TILE);
    p.q_col = a.q_col; p.k_col = a.k_col; p.v_col = a.v_col;
    p.gate_col = a.gate ? a.gate_col : -1;
    p.out_col = a.out_col;
    p.q = a.gate ? a.gate : a.q;  // f32 gate logits
    p.out = a.out;
    p.ld = a.ld; p.out_ld = a.out_ld;
    p.group_inner_stride = a.group_inner_stride;
    p.group_outer_stride = a.group_outer_stride;
    p.token_stride = a.token_stride;
    p.idesc_s = umma_idesc_f16(1, TILE, TILE, 0);
    p.idesc_o = umma_idesc_f16(1, TILE, HD, 1);
    p.idesc_s_half = umma_idesc_f16(1, TILE, TILE / 2, 0);
    p.err = device_error_word();
    // The planes keep the source's row indexing (row stride plane_ld elements), plane p at
    // planes + p · plane_stride elements.
    const int64_t s1 = a.token_stride * plane_ld;
    const int64_t s2 = a.group_inner_stride * plane_ld;
    const int64_t s3 = p.group_outer > 1 ? a.group_outer_stride * plane_ld : plane_ld;
    PlaneMaps maps;
    for (int pl = 0; pl < 3; ++pl)
        ANCHA_TRY(make_tma_4d(&maps.plane[pl], reinterpret_cast<const __nv_bfloat16*>(planes) + pl * plane_stride,
                              ELT_BF16, plane_ld, a.tokens, a.group_inner, p.group_outer, s1 > 0 ? s1 : plane_ld,
                              s2 > 0 ? s2 : plane_ld, s3 > 0 ? s3 : plane_ld, TILE, 1));
    const int64_t gx = (int64_t)p.tiles_per_group * a.group_inner;
    if (gx > 0x7fffffff || a.heads > 65535 || p.group_outer > 65535)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc_split: grid too large");
    dim3 grid((unsigned)gx, (unsigned)a.heads, (unsigned)p.group_outer);
    return launch_split(maps, p, grid, stream);
}

}  // namespace ancha
