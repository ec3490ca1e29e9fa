// common.cuh — device helpers shared by the Q4 kernels (sm_100a).
//
// Inline PTX wrappers for: mbarriers with bounded waits, 1-D TMA bulk copies (cp.async.bulk, no
// multicast), programmatic dependent launch (griddepcontrol), and the bf16 m16n8k16 mma used by
// the decode GEMV.  Every wait loop here is bounded: on timeout it records an error code in
// g_marlin_device_error and returns false so the kernel can exit; nothing traps.
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace marlin {

// Device-side error word: 0 = ok.  Written only on a wait timeout or an internal consistency
// failure.  Each translation unit that waits on device-side conditions has its own copy (the
// library is compiled without relocatable device code) and a host accessor that
// marlin_q4_device_error() combines.
static __device__ int g_marlin_device_error = 0;

enum DeviceError : int {
    kDevErrNone = 0,
    kDevErrMbarTimeout = 1,
    kDevErrTmemAlloc = 2,
    kDevErrBadIndex = 3,
};

__device__ __forceinline__ void record_device_error(int code) {
    atomicCAS(&g_marlin_device_error, 0, code);
}

// ---- bf16 helpers ------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint32_t h) { return __uint_as_float(h << 16); }

// round-to-nearest-even binary32 -> bf16 bits (finite inputs; NaN made quiet)
__device__ __forceinline__ uint32_t f32_to_bf16_bits(float f) {
    uint32_t u = __float_as_uint(f);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (u >> 16) | 0x40u;
    u += 0x7fffu + ((u >> 16) & 1u);
    return u >> 16;
}
__device__ __forceinline__ float bf16_round(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }

// ---- shared-memory address / mbarrier ----------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// The dynamic shared-memory base rounded up to a 1024-byte shared address (TMA swizzle atoms and
// UMMA descriptors need it).  Formed as the shared array plus an offset, never through an integer
// cast, so the pointer stays in the shared state space and accesses through it compile to
// shared-memory instructions rather than generic ones.
__device__ __forceinline__ uint8_t* align_smem_1024(uint8_t* base) {
    return base + ((1024u - (smem_u32(base) & 1023u)) & 1023u);
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cta.shared::cta.b64 _, [%0], %1;"
                 ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.release.cta.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// As mbar_try_wait, but a thread whose phase is not complete sleeps until it completes (or about
// 1 ms passes) instead of returning at once, so waiting warps leave the issue slots to the others.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.acquire.cta.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// Wait bound in SM clock cycles: about 2 s at 2 GHz (longer at lower clocks).  The cycle counter
// is cheap to read; the global timer is not, so it stays off the wait paths.
constexpr unsigned long long kWaitCycles = 4000000000ull;
__device__ __forceinline__ unsigned long long cycles_now() { return (unsigned long long)clock64(); }

// Bounded wait on an mbarrier phase.  try_wait suspends the thread for a hardware-defined time
// while the phase is pending; the loop gives up after kWaitCycles or 2^28 polls, records
// kDevErrMbarTimeout and returns false.  Returns true when the phase completed.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 1; it < (1u << 28); ++it) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((it & 255u) == 0 && cycles_now() - t0 > kWaitCycles) break;
    }
    record_device_error(kDevErrMbarTimeout);
    return false;
}

// ---- TMA 1-D bulk copy global -> shared (no multicast) -----------------------------------------
// dst and src 16-byte aligned, bytes a multiple of 16; completion counted on `bar` (complete_tx).
__device__ __forceinline__ void tma_bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
        ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}

// TMA tiled 2-D load (no multicast): box at element coordinates (x, y) of the tensor map into
// shared memory; x * element size must be a multiple of 16 bytes.  Out-of-range elements are
// zero-filled and still counted in the transaction bytes.
__device__ __forceinline__ void tma_load_2d(void* dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const void* tmap) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(tmap) : "memory");
}

// L2 prefetch of a contiguous range (16-byte aligned, multiple of 16 bytes).
__device__ __forceinline__ void tma_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- programmatic dependent launch ---------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- shared loads -------------------------------------------------------------------------------
__device__ __forceinline__ uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}
__device__ __forceinline__ uint2 lds64(const void* p) {
    uint2 v;
    asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(smem_u32(p)));
    return v;
}

// ---- mma.sync m16n8k16 bf16 x bf16 -> f32 ------------------------------------------------------
// A row-major 16x16 (a0: row g cols 2t..2t+1, a1: row g+8, a2: row g cols 2t+8.., a3: row g+8 ..),
// B col-major 16x8 (b0: k 2t..2t+1 col g, b1: k 2t+8..), D 16x8 (d0,d1: row g cols 2t,2t+1;
// d2,d3: row g+8), g = lane/4, t = lane%4.
__device__ __forceinline__ void mma_bf16_16816(float d[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                               uint32_t a3, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// Q4 nibble pairs -> bf16x2 holding 1 + q/16 (exact).  For a packed word w (nibble j = element j
// in bits [4j,4j+4)), pair j in {0..3} holds (element j, element j+4) in the (low, high) halves.
__device__ __forceinline__ uint32_t lop3_and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));  // (a & b) | c
    return r;
}

__device__ __forceinline__ uint32_t bf16x2_fma(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// Eight codes of one packed word -> eight bf16 weights s*q + b in natural K order (4 registers).
// LOP3 gives the pair (128 + q_i, 128 + q_i+4) as bf16 (exact), one FMA removes the 128 and one
// FMA forms q s + b with a single rounding; PRMTs regroup the pairs into K order 0..7.
__device__ __forceinline__ uint4 dequant_word(uint32_t w, uint32_t s2, uint32_t b2) {
    constexpr uint32_t kOne2 = 0x3F803F80u, kNeg128 = 0xC300C300u, kMagic = 0x43004300u;
    uint32_t p[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        const uint32_t v = lop3_and_or(w >> (4 * i), 0x000F000Fu, kMagic);
        p[i] = bf16x2_fma(bf16x2_fma(v, kOne2, kNeg128), s2, b2);  // (w_i, w_i+4)
    }
    uint4 o;
    o.x = __byte_perm(p[0], p[1], 0x5410);  // (w0, w1)
    o.y = __byte_perm(p[2], p[3], 0x5410);  // (w2, w3)
    o.z = __byte_perm(p[0], p[1], 0x7632);  // (w4, w5)
    o.w = __byte_perm(p[2], p[3], 0x7632);  // (w6, w7)
    return o;
}
__device__ __forceinline__ void q4_pairs(uint32_t w, uint32_t p[4]) {
    const uint32_t M = 0x00780078u, C = 0x3F803F80u;
    p[0] = lop3_and_or(w << 3, M, C);
    p[1] = lop3_and_or(w >> 1, M, C);
    p[2] = lop3_and_or(w >> 5, M, C);
    p[3] = lop3_and_or(w >> 9, M, C);
}

}  // namespace marlin

// ================================================================================================
// tcgen05 / TMEM (sm_100a) helpers
// ================================================================================================
namespace marlin {

// Allocate `ncols` TMEM columns (power of two >= 32) for this CTA; one full warp executes it and
// the base address is written to *dst (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst)), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// Warp-wide store of 32 consecutive 32-bit columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// Warp-wide load of 16 / 4 consecutive 32-bit columns of this warp's 32 TMEM lanes.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
          "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld4(uint32_t taddr, uint32_t (&r)[4]) {
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x4.b32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(taddr)
                 : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row atoms of 1024 B (SBO = 1024).
__device__ __forceinline__ uint64_t umma_desc_sw128(const void* smem_ptr) {
    const uint64_t addr = smem_u32(smem_ptr);
    return ((addr & 0x3FFFFull) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) | (2ull << 61);
}
// Instruction descriptor, kind::f16: D f32, A/B bf16, both K-major, M = 128, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// Instruction descriptor, kind::f16: D f32, A/B IEEE half, both K-major, M = m, N = n.
__host__ __device__ constexpr uint32_t umma_idesc_f16(int m, int n) {
    return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, single issuing thread.
__device__ __forceinline__ void umma_tmem_a(uint32_t d_taddr, uint32_t a_taddr, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
        ::"r"(d_taddr), "r"(a_taddr), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, single issuing thread.
__device__ __forceinline__ void umma_smem_a(uint32_t d_taddr, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                            bool accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.u32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
        ::"r"(d_taddr), "l"(a_desc), "l"(b_desc), "r"(idesc), "r"((uint32_t)accumulate)
        : "memory");
}
// y0 += c (d0 - 1.5 2^23) and y1 += c (d1 - 1.5 2^23), d0 / d1 integer accumulators that started at
// the bits of 1.5 2^23 read as binary32 (so d - 1.5 2^23 is the integer exactly): one packed add
// and one packed fma (sm_100 f32x2), each element rounded as the scalar FADD and FFMA would be.
__device__ __forceinline__ void fold_pair(float& y0, float& y1, uint32_t d0, uint32_t d1, float c) {
    unsigned long long dd, yy, cc;
    const unsigned long long mg = 0xCB400000CB400000ull;  // -1.5 2^23 twice
    asm("mov.b64 %0, {%1, %2};" : "=l"(dd) : "r"(d0), "r"(d1));
    asm("mov.b64 %0, {%1, %2};" : "=l"(yy) : "f"(y0), "f"(y1));
    asm("mov.b64 %0, {%1, %1};" : "=l"(cc) : "f"(c));
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(dd) : "l"(dd), "l"(mg));
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(yy) : "l"(cc), "l"(dd), "l"(yy));
    asm("mov.b64 {%0, %1}, %2;" : "=f"(y0), "=f"(y1) : "l"(yy));
}

// Arrive on `bar` once all tcgen05.mma issued so far by this thread have completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}


// D (16x8 s32) += A (16x32 s8, row-major) * B (32x8 s8, column-major); exact integer accumulation.
// Fragments (PTX ISA, mma.m16n8k32 with .s8): lane = 4 * g + t;
//   a0: row g, k 4t..4t+3;  a1: row g+8, k 4t..4t+3;  a2: row g, k 16+4t..;  a3: row g+8, k 16+4t..
//   b0: column g, k 4t..4t+3;  b1: column g, k 16+4t..
//   d0, d1: row g, columns 2t, 2t+1;  d2, d3: row g+8, columns 2t, 2t+1.
// As mma_s8_16832 with the A operand unsigned bytes (0..255).
__device__ __forceinline__ void mma_u8s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Orders the computation of `v` before whatever follows (an empty-slot release): a ring stage may be
// handed back to the producer only once every value loaded from it has been consumed, not merely
// once the loads were issued.
template <int N>
__device__ __forceinline__ void hold_regs(const float (&v)[N]) {
#pragma unroll
    for (int i = 0; i < N; ++i) asm volatile("" ::"f"(v[i]));
}

// ---- waits shared by the warp-specialised kernels ------------------------------------------------
// Bounded wait that also ends early once another role has aborted (timeout recorded on device).
// Every lane acquires the barrier; the exit is warp-uniform.  kSleep: wait with mbar_try_wait_sleep.
template <bool kSleep = false>
__device__ __forceinline__ bool warp_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (__all_sync(0xffffffffu, mbar_try_wait(bar, parity) ? 1 : 0)) return true;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0;; ++it) {
        const bool ok = kSleep ? mbar_try_wait_sleep(bar, parity) : mbar_try_wait(bar, parity);
        if (__all_sync(0xffffffffu, ok ? 1 : 0)) return true;
        if ((it & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0) {
                if (*abort) {
                    stop = 1;
                } else if (cycles_now() - t0 > kWaitCycles || it > (1u << 28)) {
                    record_device_error(kDevErrMbarTimeout);
                    *abort = 1;
                    stop = 1;
                }
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) return false;
        }
    }
}
// Single-thread bounded wait (producer / MMA issuer).
template <bool kSleep = false>
__device__ __forceinline__ bool thread_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0; it < (1u << 28); ++it) {
        if (kSleep ? mbar_try_wait_sleep(bar, parity) : mbar_try_wait(bar, parity)) return true;
        if ((it & 63u) == 63u) {
            if (*abort) return false;
            if (cycles_now() - t0 > kWaitCycles) {
                record_device_error(kDevErrMbarTimeout);
                *abort = 1;
                return false;
            }
        }
    }
    *abort = 1;
    return false;
}

// Bounded wait used on the exit path only (ignores the abort flag): returns when the phase is
// complete or after ~2 s.
__device__ __forceinline__ void drain_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0; it < (1u << 26); ++it) {
        if (mbar_try_wait(bar, parity)) return;
        if ((it & 63u) == 63u && cycles_now() - t0 > kWaitCycles) {
            record_device_error(kDevErrMbarTimeout);
            return;
        }
    }
}


// ---- thread-block clusters --------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_rank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
__device__ __forceinline__ void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
__device__ __forceinline__ void st_cluster_f32(const float* local_ptr, uint32_t rank, float v) {
    uint32_t raddr;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(raddr) : "r"(smem_u32(local_ptr)), "r"(rank));
    asm volatile("st.shared::cluster.f32 [%0], %1;" ::"r"(raddr), "f"(v) : "memory");
}


}  // namespace marlin
