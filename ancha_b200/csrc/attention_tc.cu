// Single-pass attention on the tcgen05 tensor cores for head width 64, f16 / bf16 operands:
// softmax(q·kᵀ)·v per (group, head), q pre-scaled, optionally gated by sigmoid(gate).
//
// One CTA owns a 128-row query tile. Q, K and V tiles are TMA-loaded from the packed q|k|v|gate
// projection through one 4-D tensor map {columns, tokens, inner groups, outer groups}, so
// the time axis (tokens contiguous) and the band axis (tokens T rows apart) share the code
// and nothing is transposed. A tile holds BG = 128 / BT problems of BT token rows: BT = 128
// for the time axis (T = 801 → 7 query tiles × 7 key blocks), BT = 64 for the band axis
// (two 60-token problems per tile, one key block, cross-problem scores masked).
//
// Warp roles (192 threads): warps 0–3 run the softmax, one query row per thread; warp 4
// issues TMA; warp 5 issues UMMA. Per key block kb: S(kb) = Q·K(kb)ᵀ into TMEM (M 128, N 128);
// the softmax warps read S twice (row max, then exponentials on the MUFU ex2 pipe), write
// P(kb) in f16 / bf16 into shared memory in the UMMA K-major 128-byte-swizzled layout, and the
// UMMA warp computes O(kb) = P(kb)·V(kb) into TMEM (V as an MN-major operand). S, P and O are
// double-buffered, so S(kb+1) and P(kb−1)·V run on the tensor cores while the softmax works on
// block kb; O(kb) is folded into a per-thread fp32 accumulator two blocks later with the
// online-softmax rescale. Scores use base 2 (log2 e folded into the running maximum).
#include "attention.cuh"
#include "tc.cuh"

namespace ancha {
namespace {

constexpr int TILE = 128;           // query rows / keys per block
constexpr int HD = 64;              // head width
constexpr int QKV_BYTES = TILE * HD * 2;
constexpr int P_BYTES = TILE * TILE * 2;
constexpr int OFF_Q = 0, OFF_K = QKV_BYTES, OFF_V = 3 * QKV_BYTES, OFF_P = 5 * QKV_BYTES;
constexpr int OFF_BAR = OFF_P + 2 * P_BYTES;
constexpr int SMEM_BYTES = 1024 + OFF_BAR + 16 * 8 + 16;
constexpr uint32_t S_COL = 0, O_COL = 256;  // TMEM columns: S[2] at 0 / 128, O[2] at 256 / 320
constexpr float LOG2E = 1.4426950408889634f;

struct AttnTcParams {
    int tokens, group_inner, group_outer, tiles_per_group;
    int q_col, k_col, v_col, gate_col, out_col;
    const void* q;
    void* out;
    int64_t ld, out_ld, group_inner_stride, group_outer_stride, token_stride;
    uint32_t idesc_s, idesc_o;
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

template <int BT, bool BF16>
__global__ void __launch_bounds__(192, 1)
attention_tc_kernel(const __grid_constant__ CUtensorMap tmap, const AttnTcParams p) {
    constexpr int BG = TILE / BT;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;   // [2]
    uint64_t* kv_empty = bars + 3;  // [2]
    uint64_t* s_full = bars + 5;    // [2]
    uint64_t* p_ready = bars + 7;   // [2]
    uint64_t* o_full = bars + 9;    // [2]
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int tile = blockIdx.x % p.tiles_per_group;
    const int gi0 = (blockIdx.x / p.tiles_per_group) * BG;
    const int go = blockIdx.z, head = blockIdx.y;
    const int t0 = tile * BT;
    const int nkb = p.tiles_per_group;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;

    if (threadIdx.x == 128) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_ready[s], 128);
            mbar_init(&o_full[s], 1);
        }
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tmap);
    }
    if (warp == 4) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;

    if (warp == 4) {
        if (lane == 0) {
            // TMA producer: Q once, then K / V blocks through a 2-deep ring.
            mbar_arrive_expect_tx(q_full, QKV_BYTES);
            tma_load_4d(smem + OFF_Q, &tmap, q_full, p.q_col + head * HD, t0, gi0, go);
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb & 1;
                if (!mbar_wait(&kv_empty[s], ((kb >> 1) & 1) ^ 1, abort, p.err)) break;
                mbar_arrive_expect_tx(&kv_full[s], 2 * QKV_BYTES);
                tma_load_4d(smem + OFF_K + s * QKV_BYTES, &tmap, &kv_full[s], p.k_col + head * HD, kb * BT, gi0, go);
                tma_load_4d(smem + OFF_V + s * QKV_BYTES, &tmap, &kv_full[s], p.v_col + head * HD, kb * BT, gi0, go);
                ++issued;
            }
            if (*abort) {  // let copies in flight land before the CTA exits (bounded)
                const long long c0 = clock64();
                while (!mbar_try_wait(q_full, 0) && clock64() - c0 < kWaitCycles) {
                }
                for (int kb = max(0, issued - 2); kb < issued; ++kb)
                    while (!mbar_try_wait(&kv_full[kb & 1], (kb >> 1) & 1) && clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == 5) {
        if (lane == 0) {
            // UMMA issuer.
            const uint32_t q_addr = smem_u32(smem + OFF_Q);
            auto issue_pv = [&](int j) -> bool {
                const int s = j & 1;
                if (!mbar_wait(&p_ready[s], (j >> 1) & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint32_t p_addr = smem_u32(smem + OFF_P + s * P_BYTES);
                const uint32_t v_addr = smem_u32(smem + OFF_V + s * QKV_BYTES);
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk)
                    umma_f16(tmem + O_COL + s * HD,
                             umma_desc_sw128(p_addr + (kk >> 2) * (TILE * 128) + (kk & 3) * 32),
                             umma_desc_sw128(v_addr + kk * 16 * 128), p.idesc_o, kk != 0);
                umma_commit(&o_full[s]);
                umma_commit(&kv_empty[s]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort, p.err);
            for (int kb = 0; ok && kb < nkb; ++kb) {
                const int s = kb & 1;
                if (!mbar_wait(&kv_full[s], (kb >> 1) & 1, abort, p.err)) break;
                if (kb >= 2 && !mbar_wait(&p_ready[s], ((kb - 2) >> 1) & 1, abort, p.err)) break;
                tc_fence_after();
                const uint32_t k_addr = smem_u32(smem + OFF_K + s * QKV_BYTES);
#pragma unroll
                for (int kk = 0; kk < HD / 16; ++kk)
                    umma_f16(tmem + S_COL + s * TILE, umma_desc_sw128(q_addr + kk * 32),
                             umma_desc_sw128(k_addr + kk * 32), p.idesc_s, kk != 0);
                umma_commit(&s_full[s]);
                if (kb >= 1 && !issue_pv(kb - 1)) { ok = false; break; }
            }
            if (ok && nkb > 0) issue_pv(nkb - 1);
        }
    } else {
        // Softmax warps: thread `row` owns query row `row` of the tile.
        const int row = threadIdx.x;
        const int prob = row / BT;
        const int tok = t0 + row % BT;
        const int gi = gi0 + prob;
        const bool valid = tok < p.tokens && gi < p.group_inner;
        const uint32_t lane_base = tmem + ((uint32_t)(warp * 32) << 16);
        float o[HD];
#pragma unroll
        for (int d = 0; d < HD; ++d) o[d] = 0.f;
        float m_run = -INFINITY, l = 0.f, m_acc = -INFINITY;
        float m_pend[2] = {0.f, 0.f};
        bool ok = true;

        auto fold = [&](int j) -> bool {  // o = o·2^(m_acc − m_j) + O(j); warp-uniform
            const int s = j & 1;
            if (!__all_sync(0xffffffffu, mbar_wait(&o_full[s], (j >> 1) & 1, abort, p.err))) return false;
            tc_fence_after();
            const float sc = m_acc == -INFINITY ? 0.f : ex2_approx(m_acc - m_pend[s]);
#pragma unroll
            for (int c = 0; c < HD; c += 32) {
                uint32_t r[32];
                tmem_ld32(lane_base + O_COL + s * HD + c, r);
                tmem_wait_ld();
#pragma unroll
                for (int d = 0; d < 32; ++d) o[c + d] = o[c + d] * sc + __uint_as_float(r[d]);
            }
            m_acc = m_pend[s];
            return true;
        };

        for (int kb = 0; kb < nkb; ++kb) {
            const int s = kb & 1;
            ok = __all_sync(0xffffffffu, mbar_wait(&s_full[s], (kb >> 1) & 1, abort, p.err));
            if (!ok) break;
            tc_fence_after();
            const uint32_t s_base = lane_base + S_COL + s * TILE;
            // Pass 1: row maximum over this block's valid keys.
            float mx = -INFINITY;
#pragma unroll
            for (int c = 0; c < TILE; c += 32) {
                uint32_t r[32];
                tmem_ld32(s_base + c, r);
                tmem_wait_ld();
#pragma unroll
                for (int j = 0; j < 32; ++j) {
                    const int col = c + j;
                    const bool kv = (col / BT == prob) && (kb * BT + col % BT < p.tokens);
                    if (kv) mx = fmaxf(mx, __uint_as_float(r[j]));
                }
            }
            const float m_new = fmaxf(m_run, mx * LOG2E);
            const float m_use = m_new == -INFINITY ? 0.f : m_new;
            // Fold O(kb−2) before its P buffer is overwritten.
            if (kb >= 2) {
                ok = fold(kb - 2);
                if (!ok) break;
            }
            // Pass 2: exponentials, row sum and P(kb) into shared memory (swizzled K-major).
            uint8_t* pbuf = smem + OFF_P + s * P_BYTES;
            float rowsum = 0.f;
#pragma unroll
            for (int c = 0; c < TILE; c += 32) {
                uint32_t r[32];
                tmem_ld32(s_base + c, r);
                tmem_wait_ld();
                uint32_t pk[16];
#pragma unroll
                for (int j = 0; j < 32; j += 2) {
                    float e[2];
#pragma unroll
                    for (int u = 0; u < 2; ++u) {
                        const int col = c + j + u;
                        const bool kv = (col / BT == prob) && (kb * BT + col % BT < p.tokens);
                        e[u] = kv ? ex2_approx(__uint_as_float(r[j + u]) * LOG2E - m_use) : 0.f;
                        rowsum += e[u];
                    }
                    pk[j / 2] = pack2<BF16>(e[0], e[1]);
                }
                uint8_t* half_base = pbuf + (c / 64) * (TILE * 128) + row * 128;
#pragma unroll
                for (int q = 0; q < 4; ++q) {
                    const int chunk = ((c % 64) / 8 + q) ^ (row & 7);
                    *reinterpret_cast<uint4*>(half_base + chunk * 16) =
                        make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                }
            }
            l = (m_run == -INFINITY ? 0.f : l * ex2_approx(m_run - m_use)) + rowsum;
            m_run = m_new == -INFINITY ? -INFINITY : m_use;
            m_pend[s] = m_use;
            fence_proxy_async();
            tc_fence_before();
            mbar_arrive(&p_ready[s]);
        }
        if (ok) {
            for (int j = max(0, nkb - 2); j < nkb && ok; ++j) ok = fold(j);
        }
        if (ok && valid) {
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
            for (int q = 0; q < HD / 8; ++q)
                dst[q] = make_uint4(pack2<BF16>(o[8 * q] * scale, o[8 * q + 1] * scale),
                                    pack2<BF16>(o[8 * q + 2] * scale, o[8 * q + 3] * scale),
                                    pack2<BF16>(o[8 * q + 4] * scale, o[8 * q + 5] * scale),
                                    pack2<BF16>(o[8 * q + 6] * scale, o[8 * q + 7] * scale));
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 4) {
        __syncwarp();
        tmem_dealloc(tmem, 512);
    }
}

// Time-axis kernel (tokens > 64): two 128-row query tiles of the same (group, head) per CTA
// share every K / V block. Warps 0–3 and 4–7 are the softmax warpgroups of tile 0 and 1
// (two warps per SM sub-partition), warp 8 issues TMA, warp 9 issues UMMA. Per tile S, O
// (TMEM) and P (shared memory) are single-buffered; the two tiles alternate on the tensor
// cores, so one warpgroup's softmax overlaps the other's S = Q·Kᵀ and P·V. Interior key
// blocks skip masking; only the last, partial block masks keys ≥ tokens.
constexpr int PP_OFF_Q = 0, PP_OFF_K = 2 * QKV_BYTES, PP_OFF_V = 4 * QKV_BYTES, PP_OFF_P = 6 * QKV_BYTES;
constexpr int PP_OFF_BAR = PP_OFF_P + 2 * P_BYTES;
constexpr int PP_SMEM_BYTES = 1024 + PP_OFF_BAR + 16 * 8 + 16;
constexpr int PP_THREADS = 320;

template <bool BF16>
__global__ void __launch_bounds__(PP_THREADS, 1)
attention_pp_kernel(const __grid_constant__ CUtensorMap tmap, const AttnTcParams p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + PP_OFF_BAR);
    uint64_t* q_full = bars;
    uint64_t* kv_full = bars + 1;   // [2] stages
    uint64_t* kv_empty = bars + 3;  // [2] stages
    uint64_t* s_full = bars + 5;    // [2] tiles
    uint64_t* p_ready = bars + 7;   // [2] tiles
    uint64_t* o_full = bars + 9;    // [2] tiles
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 11);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

    const int pairs = (p.tiles_per_group + 1) / 2;
    const int pair = blockIdx.x % pairs;
    const int gi = blockIdx.x / pairs;
    const int go = blockIdx.z, head = blockIdx.y;
    const int nkb = p.tiles_per_group;
    const int warp = threadIdx.x / 32, lane = threadIdx.x % 32;
    const int q0 = 2 * pair * TILE;                 // first query token of tile 0
    const bool active1 = q0 + TILE < p.tokens;      // tile 1 holds at least one query

    if (threadIdx.x == 256) {
        mbar_init(q_full, 1);
        for (int s = 0; s < 2; ++s) {
            mbar_init(&kv_full[s], 1);
            mbar_init(&kv_empty[s], 1);
            mbar_init(&s_full[s], 1);
            mbar_init(&p_ready[s], 128);
            mbar_init(&o_full[s], 1);
        }
        *abort = 0;
        fence_barrier_init();
        fence_proxy_async();
        prefetch_tma(&tmap);
    }
    if (warp == 9) {
        tmem_alloc(tmem_slot, 512);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = *tmem_slot;
    // TMEM columns: tile t uses S at t·256 + [0, 128) and O at t·256 + [128, 192).

    if (warp == 8) {
        if (lane == 0) {
            mbar_arrive_expect_tx(q_full, 2 * QKV_BYTES);
            tma_load_4d(smem + PP_OFF_Q, &tmap, q_full, p.q_col + head * HD, q0, gi, go);
            tma_load_4d(smem + PP_OFF_Q + QKV_BYTES, &tmap, q_full, p.q_col + head * HD, q0 + TILE, gi, go);
            int issued = 0;
            for (int kb = 0; kb < nkb; ++kb) {
                const int s = kb & 1;
                if (!mbar_wait(&kv_empty[s], ((kb >> 1) & 1) ^ 1, abort, p.err)) break;
                mbar_arrive_expect_tx(&kv_full[s], 2 * QKV_BYTES);
                tma_load_4d(smem + PP_OFF_K + s * QKV_BYTES, &tmap, &kv_full[s], p.k_col + head * HD, kb * TILE, gi, go);
                tma_load_4d(smem + PP_OFF_V + s * QKV_BYTES, &tmap, &kv_full[s], p.v_col + head * HD, kb * TILE, gi, go);
                ++issued;
            }
            if (*abort) {  // let copies in flight land before the CTA exits (bounded)
                const long long c0 = clock64();
                while (!mbar_try_wait(q_full, 0) && clock64() - c0 < kWaitCycles) {
                }
                for (int kb = max(0, issued - 2); kb < issued; ++kb)
                    while (!mbar_try_wait(&kv_full[kb & 1], (kb >> 1) & 1) && clock64() - c0 < kWaitCycles) {
                    }
            }
        }
    } else if (warp == 9) {
        if (lane == 0) {
            const int ntiles = active1 ? 2 : 1;
            auto issue_pv = [&](int t, int j) -> bool {
                if (!mbar_wait(&p_ready[t], j & 1, abort, p.err)) return false;
                tc_fence_after();
                const uint32_t p_addr = smem_u32(smem + PP_OFF_P + t * P_BYTES);
                const uint32_t v_addr = smem_u32(smem + PP_OFF_V + (j & 1) * QKV_BYTES);
#pragma unroll
                for (int kk = 0; kk < TILE / 16; ++kk)
                    umma_f16(tmem + t * 256 + 128,
                             umma_desc_sw128(p_addr + (kk >> 2) * (TILE * 128) + (kk & 3) * 32),
                             umma_desc_sw128(v_addr + kk * 16 * 128), p.idesc_o, kk != 0);
                umma_commit(&o_full[t]);
                return true;
            };
            bool ok = mbar_wait(q_full, 0, abort, p.err);
            for (int kb = 0; ok && kb < nkb; ++kb) {
                const int s = kb & 1;
                if (!mbar_wait(&kv_full[s], (kb >> 1) & 1, abort, p.err)) { ok = false; break; }
                tc_fence_after();
                const uint32_t k_addr = smem_u32(smem + PP_OFF_K + s * QKV_BYTES);
                for (int t = 0; t < ntiles && ok; ++t) {
                    if (kb >= 1 && !issue_pv(t, kb - 1)) { ok = false; break; }
                    const uint32_t q_addr = smem_u32(smem + PP_OFF_Q + t * QKV_BYTES);
#pragma unroll
                    for (int kk = 0; kk < HD / 16; ++kk)
                        umma_f16(tmem + t * 256, umma_desc_sw128(q_addr + kk * 32),
                                 umma_desc_sw128(k_addr + kk * 32), p.idesc_s, kk != 0);
                    umma_commit(&s_full[t]);
                }
                if (ok && kb >= 1) umma_commit(&kv_empty[(kb - 1) & 1]);
            }
            for (int t = 0; ok && t < ntiles; ++t) ok = issue_pv(t, nkb - 1);
            if (ok) umma_commit(&kv_empty[(nkb - 1) & 1]);
        }
    } else {
        const int t = warp / 4;  // tile of this softmax warpgroup
        const int row = threadIdx.x % 128;
        const int tok = q0 + t * TILE + row;
        const bool valid = tok < p.tokens;
        const uint32_t lane_base = tmem + t * 256 + ((uint32_t)((warp % 4) * 32) << 16);
        if (t == 0 || active1) {
            float o[HD];
#pragma unroll
            for (int d = 0; d < HD; ++d) o[d] = 0.f;
            float m_run = -INFINITY, l = 0.f, m_acc = -INFINITY, m_prev = 0.f;
            bool ok = true;
            uint8_t* pbuf = smem + PP_OFF_P + t * P_BYTES;
            auto fold = [&](int j) -> bool {
                if (!__all_sync(0xffffffffu, mbar_wait(&o_full[t], j & 1, abort, p.err))) return false;
                tc_fence_after();
                const float sc = m_acc == -INFINITY ? 0.f : ex2_approx(m_acc - m_prev);
#pragma unroll
                for (int c = 0; c < HD; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(lane_base + 128 + c, r);
                    tmem_wait_ld();
#pragma unroll
                    for (int d = 0; d < 32; ++d) o[c + d] = o[c + d] * sc + __uint_as_float(r[d]);
                }
                m_acc = m_prev;
                return true;
            };
            for (int kb = 0; kb < nkb; ++kb) {
                ok = __all_sync(0xffffffffu, mbar_wait(&s_full[t], kb & 1, abort, p.err));
                if (!ok) break;
                tc_fence_after();
                const int nvalid = min(TILE, p.tokens - kb * TILE);  // valid keys in this block
                float mx = -INFINITY;
                if (nvalid == TILE) {
#pragma unroll
                    for (int c = 0; c < TILE; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(lane_base + c, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j) mx = fmaxf(mx, __uint_as_float(r[j]));
                    }
                } else {
#pragma unroll
                    for (int c = 0; c < TILE; c += 32) {
                        uint32_t r[32];
                        tmem_ld32(lane_base + c, r);
                        tmem_wait_ld();
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (c + j < nvalid) mx = fmaxf(mx, __uint_as_float(r[j]));
                    }
                }
                const float m_new = fmaxf(m_run, mx * LOG2E);
                const float m_use = m_new == -INFINITY ? 0.f : m_new;
                if (kb >= 1) {
                    ok = fold(kb - 1);
                    if (!ok) break;
                }
                float rowsum = 0.f;
#pragma unroll
                for (int c = 0; c < TILE; c += 32) {
                    uint32_t r[32];
                    tmem_ld32(lane_base + c, r);
                    tmem_wait_ld();
                    uint32_t pk[16];
#pragma unroll
                    for (int j = 0; j < 32; j += 2) {
                        float e0 = ex2_approx(fmaf(__uint_as_float(r[j]), LOG2E, -m_use));
                        float e1 = ex2_approx(fmaf(__uint_as_float(r[j + 1]), LOG2E, -m_use));
                        if (nvalid < TILE) {
                            if (c + j >= nvalid) e0 = 0.f;
                            if (c + j + 1 >= nvalid) e1 = 0.f;
                        }
                        rowsum += e0 + e1;
                        pk[j / 2] = pack2<BF16>(e0, e1);
                    }
                    uint8_t* half_base = pbuf + (c / 64) * (TILE * 128) + row * 128;
#pragma unroll
                    for (int q = 0; q < 4; ++q) {
                        const int chunk = ((c % 64) / 8 + q) ^ (row & 7);
                        *reinterpret_cast<uint4*>(half_base + chunk * 16) =
                            make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
                    }
                }
                l = (m_run == -INFINITY ? 0.f : l * ex2_approx(m_run - m_use)) + rowsum;
                m_run = m_new == -INFINITY ? -INFINITY : m_use;
                m_prev = m_use;
                fence_proxy_async();
                tc_fence_before();
                mbar_arrive(&p_ready[t]);
            }
            if (ok) ok = fold(nkb - 1);
            if (ok && valid) {
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
                for (int q = 0; q < HD / 8; ++q)
                    dst[q] = make_uint4(pack2<BF16>(o[8 * q] * scale, o[8 * q + 1] * scale),
                                        pack2<BF16>(o[8 * q + 2] * scale, o[8 * q + 3] * scale),
                                        pack2<BF16>(o[8 * q + 4] * scale, o[8 * q + 5] * scale),
                                        pack2<BF16>(o[8 * q + 6] * scale, o[8 * q + 7] * scale));
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 9) {
        __syncwarp();
        tmem_dealloc(tmem, 512);
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

template <int BT, bool BF16>
int launch(const CUtensorMap& map, const AttnTcParams& p, dim3 grid, cudaStream_t s) {
    static bool configured[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (!configured[dev & 63]) {
        ANCHA_CUDA(cudaFuncSetAttribute(attention_tc_kernel<BT, BF16>,
                                        cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES));
        configured[dev & 63] = true;
    }
    attention_tc_kernel<BT, BF16><<<grid, 192, SMEM_BYTES, s>>>(map, p);
    return check_launch("attention_tc");
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
        // Time axis: two query tiles of one (group, head) per CTA.
        const int64_t gx = (int64_t)((p.tiles_per_group + 1) / 2) * a.group_inner;
        if (gx > 0x7fffffff || a.heads > 65535 || p.group_outer > 65535)
            return fail(ANCHA_E_UNSUPPORTED, "attention_tc: grid too large");
        dim3 grid((unsigned)gx, (unsigned)a.heads, (unsigned)p.group_outer);
        return a.elt == ELT_BF16 ? launch_pp<true>(map, p, grid, stream) : launch_pp<false>(map, p, grid, stream);
    }
    const int64_t gx = (int64_t)p.tiles_per_group * ceil_div(a.group_inner, BG);
    if (gx > 0x7fffffff || a.heads > 65535 || p.group_outer > 65535)
        return fail(ANCHA_E_UNSUPPORTED, "attention_tc: grid too large");
    dim3 grid((unsigned)gx, (unsigned)a.heads, (unsigned)p.group_outer);
    return a.elt == ELT_BF16 ? launch<64, true>(map, p, grid, stream) : launch<64, false>(map, p, grid, stream);
}

}  // namespace ancha
