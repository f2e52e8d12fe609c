// sm_100a building blocks shared by the tensor-core kernels: mbarriers with bounded waits,
// TMA tiled loads, TMEM allocation and loads, tcgen05 UMMA issue / commit, and the UMMA
// shared-memory and instruction descriptors (K-major operands, 128-byte swizzle).
//
// Every wait is bounded by a clock budget: on expiry the thread raises the CTA's abort flag
// and ORs ANCHA_DEVICE_TIMEOUT into the library's device error word, and every loop of the
// kernel unwinds, so a lost arrival ends the kernel with an error status instead of hanging.
#pragma once

#include <cuda.h>

#include "common.cuh"

namespace ancha {

constexpr int ANCHA_DEVICE_TIMEOUT = 1;
// ~1 s at the B200 boost clock.
constexpr long long kWaitCycles = 2000000000ll;

// Device error word of this device (allocated on first use, zero = no error).
int* device_error_word();
// Read and clear the device error word (synchronises `s`); ANCHA_E_TIMEOUT if it was set.
int take_device_error(cudaStream_t s);

// Watchdog self-test: one CTA waits, with a budget of `budget_cycles`, on an mbarrier that
// nothing arrives at, through the same bounded wait as the tensor-core kernels; returns the
// status the host reads back (ANCHA_E_TIMEOUT when the watchdog works).
int wait_selftest(long long budget_cycles, cudaStream_t s);

// Encode a 3-D tiled tensor map over a row-major [depth][rows][cols] array of 2-byte
// elements (row stride `ld`, depth stride `depth_stride`, in elements) with a
// {64, box_rows, 1} box and 128-byte swizzle; zero fill out of bounds.
int make_tma_3d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t rows,
                int64_t depth, int64_t ld, int64_t depth_stride, int box_rows);

// Encode a 4-D tiled tensor map over 2-byte elements: dims {cols, d1, d2, d3} with byte
// strides of d1..d3 given in elements (`s1..s3`), box {64, b1, b2, 1}, 128-byte swizzle,
// zero fill out of bounds.
int make_tma_4d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t d1, int64_t d2,
                int64_t d3, int64_t s1, int64_t s2, int64_t s3, int b1, int b2);

// Encode a 3-D tiled tensor map for TMA stores from a row-major [depth][rows][cols] array of
// `elt` (ELT_F32 / ELT_BF16 / ELT_F16) with box {box_cols, box_rows, 1}; `swizzle_bytes`
// (64 or 128) must equal the box row size in bytes.
int make_tma_store_3d(CUtensorMap* map, const void* base, int elt, int64_t cols, int64_t rows,
                      int64_t depth, int64_t ld, int64_t depth_stride, int box_cols, int box_rows);

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Non-blocking probe of a phase (mbarrier.test_wait), for issuers that poll several barriers.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Wait for the phase of `bar` with parity `parity`; false on timeout (after `budget` clock
// cycles) or when another thread of the CTA aborted (then `abort` is set and the device error
// word records the timeout).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* err, long long budget = kWaitCycles) {
    const long long t0 = clock64();
    while (!mbar_try_wait(bar, parity)) {
        if (*abort) return false;
        if (clock64() - t0 > budget) {
            *abort = 1;
            if (err) atomicOr(err, ANCHA_DEVICE_TIMEOUT);
            return false;
        }
    }
    return true;
}

// 3-D tiled TMA load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_3d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
        : "memory");
}

// 4-D tiled TMA load of one box into shared memory, completing on `bar`.
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x,
                                            int y, int z, int w) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5, %6}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
        : "memory");
}

// TMA store of one box from shared memory (bulk-group completion).
__device__ __forceinline__ void tma_store_3d(const CUtensorMap* map, const void* src, int x, int y, int z) {
    asm volatile("cp.async.bulk.tensor.3d.global.shared::cta.bulk_group [%0, {%2, %3, %4}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z)
                 : "memory");
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int x, int y, int z,
                                             int w) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%2, %3, %4, %5}], [%1];" ::"l"(
                     reinterpret_cast<uint64_t>(map)),
                 "r"(smem_u32(src)), "r"(x), "r"(y), "r"(z), "r"(w)
                 : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Wait until at most N committed bulk groups still read their shared-memory source.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
    asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N committed bulk groups are still in flight.
template <int N>
__device__ __forceinline__ void bulk_wait() {
    asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

__device__ __forceinline__ void prefetch_tma(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// TMEM allocation (whole warp).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t addr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(ncols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] · B[smem]ᵀ, kind::f16 (f16 / bf16 operands, fp32 accumulation).
__device__ __forceinline__ void umma_f16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// D (TMEM, f32) (+)= A·B with A read from TMEM (K-major: lane = row, 16-bit pairs along the
// columns, so a K step of 16 elements is 8 columns) and B from shared memory.
__device__ __forceinline__ void umma_f16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(tmem_d),
        "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// Arrive on `bar` once every previously issued tcgen05.mma of this thread has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                     smem_u32(bar))
                 : "memory");
}

// 32 consecutive 32-bit TMEM columns of this thread's lane (warp w reads lanes 32·(w%4)..).
__device__ __forceinline__ void tmem_ld32(uint32_t addr, uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
        "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
        "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
          "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
          "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
          "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(addr)
        : "memory");
}
__device__ __forceinline__ void tmem_wait_ld() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Store 32 consecutive 32-bit TMEM columns of this thread's lane (same lane rule as loads).
__device__ __forceinline__ void tmem_st32(uint32_t addr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, %16, "
        "%17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(addr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]),
        "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]),
        "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

__device__ __forceinline__ void tmem_wait_st() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// UMMA shared-memory descriptor of a K-major operand tile stored as rows of 128 bytes with
// the 128-byte swizzle (TMA SWIZZLE_128B): start address >> 4, leading byte offset unused
// (1), stride byte offset = 1024 B between 8-row groups, version 1 (sm_100), layout type 2.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t smem_addr) {
    uint64_t d = 0;
    d |= (uint64_t)((smem_addr >> 4) & 0x3FFF);
    d |= (uint64_t)1 << 16;
    d |= (uint64_t)(1024 >> 4) << 32;
    d |= (uint64_t)1 << 46;
    d |= (uint64_t)2 << 61;
    return d;
}

// Instruction descriptor of kind::f16: fp32 accumulator, A / B both f16 (0) or bf16 (1),
// A K-major, B K-major (b_mn = 0) or MN-major (b_mn = 1), shape M × N.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int ab_bf16, int m, int n, int b_mn = 0) {
    return (1u << 4) | ((uint32_t)ab_bf16 << 7) | ((uint32_t)ab_bf16 << 10) |
           ((uint32_t)b_mn << 16) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// exp2 on the MUFU pipe (PTX ex2.approx.ftz.f32: one instruction, subnormal results flush to
// zero; ex2(-inf) = +0).
__device__ __forceinline__ float ex2_approx(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// 1/x on the MUFU pipe (PTX rcp.approx.ftz.f32).
__device__ __forceinline__ float rcp_approx(float x) {
    float y;
    asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ---- CTA pairs (a cluster of two CTAs on two SMs sharing one tcgen05.mma, cta_group::2) ----

// This CTA's rank in its cluster.
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// All threads of both CTAs of the cluster (release / acquire).
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// The shared::cluster address of the same shared-memory offset in cluster CTA `rank`.
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
    return r;
}
// Arrive on an mbarrier of a cluster CTA (a shared::cluster address from mapa_shared).
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// 3-D tiled TMA load into this CTA's shared memory whose completion is counted on an mbarrier
// of either CTA of the pair (`bar`: a shared::cluster address). No multicast.
__device__ __forceinline__ void tma_load_3d_pair(void* dst, const CUtensorMap* map, uint32_t bar, int x, int y,
                                                 int z) {
    asm volatile(
        "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar), "r"(x), "r"(y), "r"(z)
        : "memory");
}
// TMEM allocation / release for the pair: one warp of each CTA, the same warp index in both.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t addr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(addr), "r"(ncols) : "memory");
}
// D (both CTAs' TMEM, 128 lanes each) (+)= A · Bᵀ over the pair: M = 256 rows, A rows 0..127
// from the issuing (even) CTA's shared memory and 128..255 from its peer's at the same offset,
// B's N columns split the same way. Issued by one thread of the even CTA.
__device__ __forceinline__ void umma_f16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                              uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on the mbarrier at `bar`'s offset in every CTA of `mask` once the issuing thread's
// previous pair UMMAs have completed.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
            smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Packed f32x2 arithmetic (sm_100: one instruction issue for two lanes of work).
__device__ __forceinline__ uint64_t f2(float a, float b) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(a), "f"(b));
    return r;
}
__device__ __forceinline__ void f2_split(uint64_t v, float& a, float& b) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(a), "=f"(b) : "l"(v));
}
__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}
__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fmul2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ uint64_t fsub2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Activations of the tensor-core epilogues (f16 / bf16 outputs), built from the MUFU ex2 and
// rcp instructions plus a few FMAs instead of the libm-accurate erff / tanhf, whose
// instruction count made the GEMM epilogues issue-bound.
//
// GELU(x) = x·Φ(x) = max(x, 0) − |x|·Φ(−|x|), with Φ(−u) = 2^R(u) for u = min(|x|, 5.5) and R
// a degree-7 polynomial in v = u·2/5.5 − 1: a Chebyshev least-squares fit of log2 Φ(−u) on
// [0, 5.5] made for this kernel (Φ(−5.5) = 1.9e-8, so the clamp costs < 2.5e-7 at |x| ≤ 12).
// One MUFU op per element (ex2) and 11 other instructions; emulated in f32 over [−12, 12] the
// error is ≤ 7e-7 absolute and ≤ 5e-6 relative where |GELU| > 1e-3, far below the 16-bit
// output rounding.
__device__ __forceinline__ float gelu_fast(float x) {
    const float v = fmaf(fminf(fabsf(x), 5.5f), 2.0f / 5.5f, -1.0f);
    float r = -0.0022850772365927696f;
    r = fmaf(r, v, 0.011377031914889812f);
    r = fmaf(r, v, -0.03212796524167061f);
    r = fmaf(r, v, 0.07807064056396484f);
    r = fmaf(r, v, -0.1830366849899292f);
    r = fmaf(r, v, -5.023968696594238f);
    r = fmaf(r, v, -12.107662200927734f);
    r = fmaf(r, v, -8.390584945678711f);
    return fmaf(-fabsf(x), ex2_approx(r), fmaxf(x, 0.f));
}
// tanh(x) = sign(x)·(1 − 2 / (e^(2|x|) + 1)); absolute error ~1e-7.
__device__ __forceinline__ float tanh_fast(float x) {
    const float e = ex2_approx(2.0f * 1.4426950408889634f * fabsf(x));
    return copysignf(fmaf(-2.0f, rcp_approx(e + 1.0f), 1.0f), x);
}
// gelu_fast on two values with the polynomial on packed f32x2 FMAs (same coefficients).
__device__ __forceinline__ void gelu_fast2(float& x0, float& x1) {
    const uint64_t v = ffma2(f2(fminf(fabsf(x0), 5.5f), fminf(fabsf(x1), 5.5f)), f2(2.0f / 5.5f, 2.0f / 5.5f),
                             f2(-1.0f, -1.0f));
    uint64_t r = ffma2(f2(-0.0022850772365927696f, -0.0022850772365927696f), v,
                       f2(0.011377031914889812f, 0.011377031914889812f));
    r = ffma2(r, v, f2(-0.03212796524167061f, -0.03212796524167061f));
    r = ffma2(r, v, f2(0.07807064056396484f, 0.07807064056396484f));
    r = ffma2(r, v, f2(-0.1830366849899292f, -0.1830366849899292f));
    r = ffma2(r, v, f2(-5.023968696594238f, -5.023968696594238f));
    r = ffma2(r, v, f2(-12.107662200927734f, -12.107662200927734f));
    r = ffma2(r, v, f2(-8.390584945678711f, -8.390584945678711f));
    float r0, r1;
    f2_split(r, r0, r1);
    x0 = fmaf(-fabsf(x0), ex2_approx(r0), fmaxf(x0, 0.f));
    x1 = fmaf(-fabsf(x1), ex2_approx(r1), fmaxf(x1, 0.f));
}
// tanh(x) = 1 − 2 / (e^(2x) + 1) on two values, packed: the form needs no sign handling (e^(2x)
// → 0 gives −1, → ∞ gives 1); absolute error ~2e-7, as tanh_fast.
__device__ __forceinline__ void tanh_fast2(float& x0, float& x1) {
    float t0, t1;
    f2_split(fmul2(f2(x0, x1), f2(2.0f * 1.4426950408889634f, 2.0f * 1.4426950408889634f)), t0, t1);
    float e0, e1;
    f2_split(fadd2(f2(ex2_approx(t0), ex2_approx(t1)), f2(1.0f, 1.0f)), e0, e1);
    f2_split(ffma2(f2(-2.0f, -2.0f), f2(rcp_approx(e0), rcp_approx(e1)), f2(1.0f, 1.0f)), x0, x1);
}
// σ(x) = 1 / (1 + e^(−x)).
__device__ __forceinline__ float sigmoid_fast(float x) {
    return rcp_approx(1.0f + ex2_approx(-1.4426950408889634f * x));
}

}  // namespace ancha
