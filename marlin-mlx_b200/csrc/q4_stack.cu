// q4_stack.cu — the decode step's layer stack as one persistent cooperative kernel (sm_100a).
//
// Replaces, for decode-sized batches, the per-layer sequence of marlin-mlx's text model restricted
// to its Q4 sublayers (src/model/marlin.cpp:103-146: h += mlp(rms_norm(h)) with mlp_forward
// :31-35): one launch for all layers instead of two dependent kernels per layer (each dependent
// kernel boundary costs about 3 us on B200).  The final norm, lm_head and argmax follow as the
// fused lm_head kernel.
//
// All CTAs are resident (cooperative launch, one per SM).  Per layer:
//   phase A  work item = 16 features: the 16 gate rows and 16 up rows over K = hidden.  Each CTA
//            stages RMSNorm(h) once as the exact s8 planes of the integer-MMA path (q4_i8.cu),
//            accumulates all of its items in registers, then reduces once and writes
//            act = SwiGLU(gate, up) (binary32) plus a per-row max |act| (atomicMax on the bits);
//   phase B  work item = 16 rows of down_proj over all of K = intermediate: each consumer warp
//            stages its own K slice of act against the global row maximum (no block barrier),
//            the eight K slices meet in shared memory in a fixed order, and the residual add
//            writes those 16 rows of the next h (deterministic, no partial sums in memory);
// separated by software grid barriers among the consumer warps (a monotonic arrival counter).
//
// Warp roles: warps 0-7 consume; warp 8 is the TMA producer, which walks the same schedule across
// items, phases and layers, so the next phase's weights stream while the consumers wait at a grid
// barrier or stage activations.
//
// Every wait is bounded: a grid barrier or mbarrier that does not complete within ~2 s records a
// device error and raises an abort flag that every CTA checks, so all CTAs leave.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_i8_common.cuh"
#include "q4_stack.cuh"

#include <algorithm>

// Optional instrumentation hooks, empty in the library build: STACK_MARK(layer, point) by consumer
// thread 0 of every CTA; STACK_ISSUE(n) by the producer when it issues ring stage n of this CTA's
// schedule, STACK_READY(n) by consumer thread 0 when that stage has landed.
#ifndef STACK_MARK
#define STACK_MARK(l, k)
#endif
#ifndef STACK_ISSUE
#define STACK_ISSUE(n)
#endif
#ifndef STACK_READY
#define STACK_READY(n)
#endif

namespace marlin {
namespace {

constexpr uint32_t kSPacked = 8192;                  // packed words per ring stage
constexpr uint32_t kSStage = kSPacked + 1024;        // + scales and biases: 9 KB
constexpr int kSCons = 8;                            // consumer warps
constexpr int kSThreads = (kSCons + 1) * 32;
constexpr int kSAGroups = 8;                         // phase A stage: 32 rows (16 gate + 16 up) x 8 groups
constexpr int kSBGroups = 16;                        // phase B stage: 16 rows x 16 groups
constexpr int kSAItems = 4;                          // phase A items per CTA at most
constexpr uint32_t kSSmemLimit = 225 * 1024;
constexpr int kSMinStages = 6;

// Words of the zero-invariant control block (StackLaunch::bar).
constexpr int kBarArrive = 0, kBarAbort = 1, kBarDone = 2, kBarAmax = 4;  // amax: [2][kStackMaxRows]

// Bounded barrier among `n` warps built on an mbarrier (arrival count n): every lane of the warp
// waits for the phase; after kWaitCycles (or once the CTA has aborted) it gives up, records `100 + where`
// and raises the CTA's abort flag, so no consumer can block forever.  `ph` is this warp's phase bit.
__device__ __forceinline__ void warp_group_bar(uint64_t* bar, uint32_t& ph, volatile int* abort, int where) {
    __syncwarp();
    if ((threadIdx.x & 31) == 0) mbar_arrive(bar);
    unsigned long long t0 = 0;
    for (uint32_t it = 0;; ++it) {
        if (__all_sync(0xffffffffu, mbar_try_wait(bar, ph) ? 1 : 0)) break;
        if (it == 0) t0 = cycles_now();
        if ((it & 63u) == 63u) {
            int stop = 0;
            if ((threadIdx.x & 31) == 0 && (*abort || cycles_now() - t0 > kWaitCycles)) {
                if (!*abort) record_device_error(100 + where);
                *abort = 1;
                stop = 1;
            }
            if (__shfl_sync(0xffffffffu, stop, 0)) break;
        }
    }
    ph ^= 1u;
}

// the consumer warps (threads 0..255)
struct ConsumerTeam {
    uint64_t* bar;
    volatile int* abort;
    uint32_t ph = 0;
    int where = 0;
    __device__ __forceinline__ int size() const { return kSCons * 32; }
    __device__ __forceinline__ int rank() const { return threadIdx.x; }
    __device__ __forceinline__ void sync() { warp_group_bar(bar, ph, abort, where); }
};

__device__ __forceinline__ unsigned ld_relaxed_gpu(const unsigned* p) {
    unsigned v;
    asm volatile("ld.relaxed.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void red_release_gpu_add(unsigned* p, unsigned v) {
    asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }

// Software grid barrier among the consumer warps of every CTA (all CTAs are co-resident by the
// cooperative launch): the team barrier orders this CTA's writes before thread 0's release-add on
// a counter that only grows during a call; thread 0 polls until the counter reaches `target`
// (= CTAs x barriers passed), then an acquire fence and the team barrier make every CTA's writes
// visible to the whole team.  Returns false once any CTA has aborted.
__device__ bool grid_sync(ConsumerTeam& team, unsigned* bar, unsigned target) {
    team.where = 1;
    team.sync();
    if (threadIdx.x == 0 && !*team.abort) {
        red_release_gpu_add(bar + kBarArrive, 1u);
        const volatile unsigned* gabort = bar + kBarAbort;
        const unsigned long long t0 = cycles_now();
        for (uint32_t it = 0;; ++it) {
            if (ld_relaxed_gpu(bar + kBarArrive) >= target) break;
            if ((it & 15u) == 15u) {
                if (*gabort) {
                    *team.abort = 1;
                    break;
                }
                if (cycles_now() - t0 > kWaitCycles) {
                    record_device_error(kDevErrMbarTimeout);
                    atomicExch(bar + kBarAbort, 1u);
                    *team.abort = 1;
                    break;
                }
            }
        }
        fence_acq_rel_gpu();
    }
    team.where = 2;
    team.sync();
    return !*team.abort;
}

struct StackLayerMaps {
    CUtensorMap g, gs, gb, u, us, ub, d, ds, db;  // every box is 16 rows high
};

struct StackArgs {
    StackLayerMaps layer[kStackMaxLayers];
    const uint16_t* norm_w[kStackMaxLayers];
    const void* h0;
    int h0_dtype;
    float eps;
    int nl, M, H, I, GA, nsb, ncols, S, items_a, items_b;
    float* hbuf;    // [2][M][H] residual stream between layers (binary32)
    float* h_last;  // [M][H] the last layer's output
    float* act;     // [M][I]
    unsigned* bar;  // control block (zero on entry, left zero)
    uint32_t off_bar, off_misc, off_scr, off_xs, off_cs, off_xq, off_red, off_ring, off_xe;
};

// Phase A, one 8-group stage, consumer warp (tile t = gate/up, groups 2kp and 2kp + 1): the same
// tensor-core step as the decode GEMV (codes x s8 planes, exact int32, binary32 fold).
// Stage layout: line c (groups 4c..4c+3) at c * 4 KB, gate rows 0-15 then up rows 16-31, 128 B
// per row with 128-byte swizzle; scales [32 rows][8] at 8 KB, biases [32 rows][8] at 8.5 KB.
template <int NTN>
__device__ __forceinline__ void stack_stage_a(const uint8_t* st, int gl0, const I8X& t, int ncols, int tile, int kp,
                                              int lane, float (&y)[NTN][4], float (&yb)[NTN][2]) {
    const int g = lane >> 2, tq = lane & 3;
    const int r0 = 16 * tile + g, r1 = r0 + 8;
#pragma unroll
    for (int qq = 0; qq < 2; ++qq) {
        const int q = 2 * kp + qq;
        const int c = q >> 2, gq = q & 3;
        const uint32_t off = (uint32_t)((((2 * gq + (tq >> 1)) ^ g) << 4) + 8 * (tq & 1));
        const uint2 wa = *reinterpret_cast<const uint2*>(st + c * 4096 + r0 * 128 + off);
        const uint2 wb = *reinterpret_cast<const uint2*>(st + c * 4096 + r1 * 128 + off);
        const float sr0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + r0 * 16 + 2 * q));
        const float sr1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + r1 * 16 + 2 * q));
        const float br0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + 512 + r0 * 16 + 2 * q));
        const float br1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + 512 + r1 * 16 + 2 * q));
        const int gl = gl0 + q;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4*>(t.xq + ((size_t)(gl * ncols + 8 * j + g) * 64 + 16 * tq));
            const int c0 = gl * ncols + 8 * j + 4 * (tq >> 1);
            i8_group(wa, wb, xv, sr0, sr1, br0, br1, t.xe[c0], t.xs[c0], y[j], yb[j]);
        }
    }
}

// Phase B, one 16-group stage, consumer warp w (groups 2w and 2w + 1 of the stage = its local
// groups 2s, 2s + 1).  Stage layout: line c (groups 4c..4c+3) at c * 2 KB, 16 rows x 128 B,
// 128-byte swizzle; scales [2 boxes][16 rows][8] at 8 KB, biases likewise at 8.5 KB.
template <int NTN>
__device__ __forceinline__ void stack_stage_b(const uint8_t* st, int s, const uint8_t* xqw, const float* xsw,
                                              const float (&pe)[NTN], int ncols, int warp, int lane,
                                              float (&y)[NTN][4], float (&yb)[NTN][2]) {
    const int g = lane >> 2, tq = lane & 3;
#pragma unroll
    for (int e = 0; e < 2; ++e) {
        const int q = 2 * warp + e;
        const int c = q >> 2, gq = q & 3;
        const uint32_t off = (uint32_t)((((2 * gq + (tq >> 1)) ^ g) << 4) + 8 * (tq & 1));
        const uint2 wa = *reinterpret_cast<const uint2*>(st + c * 2048 + g * 128 + off);
        const uint2 wb = *reinterpret_cast<const uint2*>(st + c * 2048 + (g + 8) * 128 + off);
        const uint32_t so = (uint32_t)((q >> 3) * 256 + 2 * (q & 7));
        const float sr0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + so + g * 16));
        const float sr1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + so + (g + 8) * 16));
        const float br0 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + 512 + so + g * 16));
        const float br1 = bf16_bits_to_f32(*reinterpret_cast<const uint16_t*>(st + kSPacked + 512 + so + (g + 8) * 16));
        const int lg = 2 * s + e;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const uint4 xv = *reinterpret_cast<const uint4*>(xqw + ((size_t)(lg * ncols + 8 * j + g) * 64 + 16 * tq));
            i8_group(wa, wb, xv, sr0, sr1, br0, br1, pe[j], xsw[lg * ncols + 8 * j + 4 * (tq >> 1)], y[j], yb[j]);
        }
    }
}

// Phase B staging by one warp: its 2 * nsb local groups (local group lg = K group
// 16 (lg >> 1) + 2 warp + (lg & 1)) of the M act rows as s8 planes against row exponents e[m]
// from the global maxima, with 64 x the plane-0 sums.  Same byte layout as stage_x_i8_team.
__device__ __forceinline__ void stage_b_warp(const float* act, int I, int M, int ncols, int nsb, int warp, int lane,
                                             const int (&e)[kStackMaxRows], uint8_t* xqw, float* xsw) {
    const int nlg = 2 * nsb;
    for (int i = lane; i < nlg * ncols; i += 32) xsw[i] = 0.f;
    const int pad = ncols - 4 * M;
    for (int i = lane; i < nlg * pad * 4; i += 32) {
        const int lg = i / (pad * 4), rem = i % (pad * 4);
        *reinterpret_cast<uint4*>(xqw + ((size_t)lg * ncols + 4 * M + rem / 4) * 64 + (rem % 4) * 16) =
            make_uint4(0, 0, 0, 0);
    }
    __syncwarp();
    constexpr int kU = 4;           // units per lane loaded together
    const int total = nlg * M * 8;  // a multiple of 32 (nlg is even, 8 units per group)
#pragma unroll 1
    for (int base = 0; base < total; base += 32 * kU) {
        float v[kU][8];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int idx = base + 32 * u + lane;
            if (idx < total) {
                const int un = idx & 7, rest = idx >> 3, lg = rest % nlg, m = rest / nlg;
                const int gk = 16 * (lg >> 1) + 2 * warp + (lg & 1);
                const float* p = act + (size_t)m * I + 64 * gk + 8 * un;
                const float4 x0 = *reinterpret_cast<const float4*>(p);
                const float4 x1 = *reinterpret_cast<const float4*>(p + 4);
                v[u][0] = x0.x; v[u][1] = x0.y; v[u][2] = x0.z; v[u][3] = x0.w;
                v[u][4] = x1.x; v[u][5] = x1.y; v[u][6] = x1.z; v[u][7] = x1.w;
            }
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
            const int idx = base + 32 * u + lane;
            if (base + 32 * u < total) {  // warp-uniform
                const int un = idx & 7, rest = idx >> 3, lg = rest % nlg, m = rest / nlg;
                int em = e[0];
#pragma unroll
                for (int r = 1; r < kStackMaxRows; ++r) em = m == r ? e[r] : em;
                uint32_t b[4][2];
                planes8(v[u], em, b);
#pragma unroll
                for (int p = 0; p < 4; ++p)
                    *reinterpret_cast<uint2*>(xqw + ((size_t)lg * ncols + 4 * m + p) * 64 + un * 8) =
                        make_uint2(b[p][0], b[p][1]);
                float s = 0.f;
#pragma unroll
                for (int j = 0; j < 8; ++j) s = __fadd_rn(s, v[u][j]);
                s += __shfl_xor_sync(0xffffffffu, s, 1);
                s += __shfl_xor_sync(0xffffffffu, s, 2);
                s += __shfl_xor_sync(0xffffffffu, s, 4);
                if (un == 0) xsw[lg * ncols + 4 * m] = __fmul_rn(s, 64.0f);
            }
        }
    }
    __syncwarp();
}

template <int NTN>
__global__ void __launch_bounds__(kSThreads, 1) q4_stack_kernel(const __grid_constant__ StackArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    constexpr int MS = 2 * NTN;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = a.M, S = a.S, ncols = a.ncols, H = a.H, I = a.I, nb = (int)gridDim.x, cta = (int)blockIdx.x;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    uint64_t* team_bar = reinterpret_cast<uint64_t*>(smem + a.off_misc + 16);
    float* red = reinterpret_cast<float*>(smem + a.off_red);
    uint8_t* ring = smem + a.off_ring;
    I8X tx{smem + a.off_xq, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_cs),
           reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
           reinterpret_cast<unsigned int*>(smem + a.off_misc + 64), reinterpret_cast<float*>(smem + a.off_xe)};
    const int spa = a.GA / kSAGroups;  // stages per phase-A item
    const int nsb = a.nsb;             // stages per phase-B item
    const int na = a.items_a > cta ? (a.items_a - 1 - cta) / nb + 1 : 0;
    const bool has_b = cta < a.items_b;
    unsigned* gbar = a.bar;
    unsigned* amax_g = a.bar + kBarAmax;

    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kSCons);
        }
        mbar_init(team_bar, kSCons);
        fence_mbar_init();
    }
    __syncthreads();

    if (warp == kSCons) {
        // ---------------------------------------------------------------- producer (one thread)
        if (lane == 0) {
            int slot = 0, round = 0, issued = 0;
            bool ok = true;
            auto acquire = [&]() -> uint8_t* {
                if (round > 0 && !thread_wait(&empty[slot], (uint32_t)((round - 1) & 1), abort)) {
                    ok = false;
                    return nullptr;
                }
                STACK_ISSUE(issued);
                mbar_arrive_expect_tx(&full[slot], kSStage);
                return ring + (size_t)slot * kSStage;
            };
            auto advance = [&]() {
                ++issued;
                if (++slot == S) {
                    slot = 0;
                    ++round;
                }
            };
            for (int l = 0; l < a.nl && ok; ++l) {
                const StackLayerMaps& mp = a.layer[l];
                if (l == 0) {
                    prefetch_tmap(&mp.g);
                    prefetch_tmap(&mp.u);
                    prefetch_tmap(&mp.d);
                }
                for (int i = 0; i < na && ok; ++i) {
                    const int f0 = 16 * (cta + i * nb);
                    for (int s = 0; s < spa && ok; ++s) {
                        uint8_t* st = acquire();
                        if (!st) break;
                        const int gs = kSAGroups * s;
                        for (int c = 0; c < 2; ++c) {
                            tma_load_2d(st + c * 4096, &mp.g, (gs + 4 * c) * 8, f0, &full[slot]);
                            tma_load_2d(st + c * 4096 + 2048, &mp.u, (gs + 4 * c) * 8, f0, &full[slot]);
                        }
                        tma_load_2d(st + kSPacked, &mp.gs, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + 256, &mp.us, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + 512, &mp.gb, gs, f0, &full[slot]);
                        tma_load_2d(st + kSPacked + 768, &mp.ub, gs, f0, &full[slot]);
                        advance();
                    }
                }
                if (has_b) {
                    const int r0 = 16 * cta;
                    for (int s = 0; s < nsb && ok; ++s) {
                        uint8_t* st = acquire();
                        if (!st) break;
                        const int gs = kSBGroups * s;
                        for (int c = 0; c < 4; ++c) tma_load_2d(st + c * 2048, &mp.d, (gs + 4 * c) * 8, r0, &full[slot]);
                        tma_load_2d(st + kSPacked, &mp.ds, gs, r0, &full[slot]);
                        tma_load_2d(st + kSPacked + 256, &mp.ds, gs + 8, r0, &full[slot]);
                        tma_load_2d(st + kSPacked + 512, &mp.db, gs, r0, &full[slot]);
                        tma_load_2d(st + kSPacked + 768, &mp.db, gs + 8, r0, &full[slot]);
                        advance();
                    }
                }
            }
            // exit only once every copy this thread started has landed
            for (int q = max(0, issued - S); q < issued; ++q) drain_wait(&full[q % S], (uint32_t)((q / S) & 1));
        }
    } else {
        // ---------------------------------------------------------------- consumers (warps 0-7)
        const int tile = warp & 1, kp = warp >> 1;
        const int g = lane >> 2, tq = lane & 3;
        ConsumerTeam team{team_bar, abort};
        int slot = 0, round = 0, consumed = 0;
        unsigned nbar = 0;
        bool ok = true;
        auto wait_stage = [&]() -> const uint8_t* {
            if (ok && !warp_wait(&full[slot], (uint32_t)(round & 1), abort)) ok = false;
            STACK_READY(consumed);
            return ok ? ring + (size_t)slot * kSStage : nullptr;
        };
        auto release_stage = [&]() {
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            ++consumed;
            if (++slot == S) {
                slot = 0;
                ++round;
            }
        };

        for (int l = 0; l < a.nl; ++l) {
            const void* hin = l == 0 ? a.h0 : a.hbuf + (size_t)((l - 1) & 1) * M * H;
            const int hin_dtype = l == 0 ? a.h0_dtype : kF32;
            float* hout = l == a.nl - 1 ? a.h_last : a.hbuf + (size_t)(l & 1) * M * H;
            STACK_MARK(l, 0);
            // the other amax slot was last read in phase B of layer l - 1 (before the barrier that
            // ended it) and is next written in phase A of layer l + 1
            if (cta == 0 && tid < M && l > 0) amax_g[((l - 1) & 1) * kStackMaxRows + tid] = 0u;

            // ---- phase A: x = RMSNorm(h) as s8 planes, then all of this CTA's 16-feature items
            stage_x_i8_team(team, hin, hin_dtype, H, a.norm_w[l], a.eps, 0, a.GA, M, ncols, tx);
            STACK_MARK(l, 1);
            float y[kSAItems][NTN][4], ya[kSAItems][NTN][2];
#pragma unroll
            for (int i = 0; i < kSAItems; ++i)
#pragma unroll
                for (int j = 0; j < NTN; ++j)
                    y[i][j][0] = y[i][j][1] = y[i][j][2] = y[i][j][3] = ya[i][j][0] = ya[i][j][1] = 0.f;
#pragma unroll
            for (int i = 0; i < kSAItems; ++i) {
                if (i < na) {
                    for (int s = 0; s < spa; ++s) {
                        const uint8_t* st = wait_stage();
                        if (st) stack_stage_a<NTN>(st, kSAGroups * s, tx, ncols, tile, kp, lane, y[i], ya[i]);
#pragma unroll
                        for (int j = 0; j < NTN; ++j) {  // consumed before release
                            hold_regs(y[i][j]);
                            hold_regs(ya[i][j]);
                        }
                        release_stage();
                    }
                }
            }
            STACK_MARK(l, 2);
            // planes -> one value per (K part, item, row, activation row)
#pragma unroll
            for (int i = 0; i < kSAItems; ++i) {
                if (i < na) {
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        const float2 cv = *reinterpret_cast<const float2*>(tx.cs + 8 * j + 2 * tq);
                        const float2 pp = i8_combine(y[i][j], ya[i][j], cv, tq);
                        const float p0 = pp.x, p1 = pp.y;
                        const int m = 2 * j + (tq >> 1);
                        if ((tq & 1) == 0 && m < M) {
                            float* r = red + ((size_t)(kp * kSAItems + i) * 32 + 16 * tile + g) * MS + m;
                            r[0] = p0;
                            r[8 * MS] = p1;
                        }
                    }
                }
            }
            team.where = 3;
            team.sync();
            {
                // SwiGLU per (item, feature, activation row), the 4 K parts summed in a fixed order
                const int per = 16 * M;
                unsigned bits = 0u;
                int mm = -1;
                if (tid < na * per) {
                    const int i = tid / per, f = (tid / M) % 16, m = tid % M;
                    float gsum = 0.f, usum = 0.f;
#pragma unroll
                    for (int k = 0; k < 4; ++k) {
                        gsum += red[((size_t)(k * kSAItems + i) * 32 + f) * MS + m];
                        usum += red[((size_t)(k * kSAItems + i) * 32 + 16 + f) * MS + m];
                    }
                    const float v = ((1.0f / (1.0f + expf(-gsum))) * gsum) * usum;
                    a.act[(size_t)m * I + 16 * (cta + i * nb) + f] = v;
                    bits = __float_as_uint(fabsf(v));
                    mm = m;
                }
                for (int m = 0; m < M; ++m) {
                    const unsigned r = __reduce_max_sync(0xffffffffu, mm == m ? bits : 0u);
                    if (lane == 0 && r) atomicMax(&amax_g[(l & 1) * kStackMaxRows + m], r);
                }
            }
            STACK_MARK(l, 3);
            if (!grid_sync(team, gbar, (++nbar) * (unsigned)nb)) ok = false;
            STACK_MARK(l, 4);

            // ---- phase B: 16 rows of down_proj over all of K, + residual
            if (has_b) {
                int e[kStackMaxRows];
#pragma unroll
                for (int m = 0; m < kStackMaxRows; ++m)
                    e[m] = m < M ? row_exp(*reinterpret_cast<volatile unsigned*>(&amax_g[(l & 1) * kStackMaxRows + m]))
                                 : 0;
                uint8_t* xqw = tx.xq + (size_t)warp * (2 * nsb) * ncols * 64;
                float* xsw = tx.xs + (size_t)warp * (2 * nsb) * ncols;
                stage_b_warp(a.act, I, M, ncols, nsb, warp, lane, e, xqw, xsw);
                STACK_MARK(l, 5);
                float yb[NTN][4], ybb[NTN][2], pe[NTN];
#pragma unroll
                for (int j = 0; j < NTN; ++j) {
                    yb[j][0] = yb[j][1] = yb[j][2] = yb[j][3] = ybb[j][0] = ybb[j][1] = 0.f;
                    const int m = 2 * j + (tq >> 1);
                    int em = e[0];
#pragma unroll
                    for (int r = 1; r < kStackMaxRows; ++r) em = m == r ? e[r] : em;
                    pe[j] = m < M ? pow2f(em) : 0.f;
                }
                for (int s = 0; s < nsb; ++s) {
                    const uint8_t* st = wait_stage();
                    if (st) stack_stage_b<NTN>(st, s, xqw, xsw, pe, ncols, warp, lane, yb, ybb);
#pragma unroll
                    for (int j = 0; j < NTN; ++j) {
                        hold_regs(yb[j]);
                        hold_regs(ybb[j]);
                    }
                    release_stage();
                }
                STACK_MARK(l, 6);
#pragma unroll
                for (int j = 0; j < NTN; ++j) {
                    const int m = 2 * j + (tq >> 1);
                    const int p = 2 * (tq & 1);
                    const float cx = m < M ? pow2f(-10 - 7 * p) : 0.f;
                    const float cy = m < M ? pow2f(-17 - 7 * p) : 0.f;
                    const float2 pp = i8_combine(yb[j], ybb[j], make_float2(cx, cy), tq);
                    const float p0 = pp.x, p1 = pp.y;
                    if ((tq & 1) == 0 && m < M) {
                        red[((size_t)warp * 16 + g) * MS + m] = p0;
                        red[((size_t)warp * 16 + g + 8) * MS + m] = p1;
                    }
                }
                team.where = 4;
                team.sync();
                if (tid < 16 * M) {
                    const int m = tid / 16, r = tid % 16;
                    float v = 0.f;
#pragma unroll
                    for (int w = 0; w < kSCons; ++w) v += red[((size_t)w * 16 + r) * MS + m];
                    const size_t o = (size_t)m * H + 16 * cta + r;
                    const float hv = hin_dtype == kBF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(hin)[o])
                                                         : static_cast<const float*>(hin)[o];
                    hout[o] = hv + v;
                }
            }
            STACK_MARK(l, 7);
            if (l < a.nl - 1 && !grid_sync(team, gbar, (++nbar) * (unsigned)nb)) ok = false;
        }
        (void)ok;
    }
    __syncthreads();
    __shared__ bool is_last;
    __threadfence();
    if (tid == 0) is_last = atomicAdd(gbar + kBarDone, 1u) == gridDim.x - 1;
    __syncthreads();
    if (is_last && tid == 0) {
        __threadfence();
        // the control block returns to zero for the next call (a timed-out call does not poison it)
        atomicExch(gbar + kBarArrive, 0u);
        atomicExch(gbar + kBarAbort, 0u);
        for (int r = 0; r < 2 * kStackMaxRows; ++r) atomicExch(amax_g + r, 0u);
        atomicExch(gbar + kBarDone, 0u);
    }
}

// Shared-memory plan of one launch; false when it does not fit.
struct StackPlan {
    int ntn, ncols, S;
    uint32_t off_bar, off_misc, off_scr, off_xs, off_cs, off_xq, off_red, off_ring, off_xe, smem;
};

bool stack_plan(int64_t m, int64_t hidden, int64_t inter, StackPlan& p) {
    p.ntn = m <= 2 ? 1 : 2;
    p.ncols = 8 * p.ntn;
    const int MS = 2 * p.ntn;
    const uint32_t GA = (uint32_t)(hidden / 64), nlg = (uint32_t)(2 * (inter / 64 / kSBGroups));
    uint32_t off = 0;
    auto take = [&](uint32_t bytes, uint32_t align) {
        off = (off + align - 1) / align * align;
        const uint32_t o = off;
        off += bytes;
        return o;
    };
    p.off_bar = take(2 * 32 * 8, 8);  // up to 32 stages
    p.off_misc = take(128, 16);
    p.off_scr = take((64 + (uint32_t)m * (uint32_t)(hidden / 8)) * 4, 16);
    p.off_cs = take(p.ncols * 4, 16);
    p.off_xs = take(std::max(GA, kSCons * nlg) * p.ncols * 4, 16);
    p.off_xe = take(GA * p.ncols * 4, 16);
    p.off_xq = take(std::max(GA, kSCons * nlg) * p.ncols * 64, 128);
    p.off_red = take(std::max<uint32_t>(4 * kSAItems * 32, kSCons * 16) * MS * 4, 16);
    off = (off + 1023) / 1024 * 1024;
    p.off_ring = off;
    const uint32_t avail = kSSmemLimit > off + 1024 ? kSSmemLimit - off - 1024 : 0;
    p.S = std::min<int>(32, (int)(avail / kSStage));
    p.smem = off + (uint32_t)p.S * kSStage + 1024;
    return p.S >= kSMinStages;
}

}  // namespace

size_t stack_scratch_size(int64_t m, int64_t hidden, int64_t inter) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    return al((size_t)3 * m * hidden * 4) + al((size_t)m * inter * 4);
}

bool stack_supported(int64_t m, int64_t hidden, int64_t inter, int n_layers) {
    if (!(m >= 1 && m <= kStackMaxRows && n_layers >= 1 && n_layers <= kStackMaxLayers && hidden % 512 == 0 &&
          inter % (64 * kSBGroups) == 0 && tmap_encode_fn() != nullptr))
        return false;
    const int sms = device_num_sms();
    if (hidden / 16 > sms || inter / 16 > (int64_t)kSAItems * sms) return false;
    StackPlan p;
    return stack_plan(m, hidden, inter, p);
}

cudaError_t launch_stack(const StackLaunch& L, cudaStream_t stream) {
    if (!stack_supported(L.m, L.hidden, L.inter, L.n_layers)) return cudaErrorInvalidValue;
    StackPlan p;
    stack_plan(L.m, L.hidden, L.inter, p);
    StackArgs a{};
    const int M = (int)L.m, H = (int)L.hidden, I = (int)L.inter;
    a.nl = L.n_layers;
    a.M = M;
    a.H = H;
    a.I = I;
    a.GA = H / 64;
    a.nsb = I / 64 / kSBGroups;
    a.ncols = p.ncols;
    a.S = p.S;
    a.items_a = I / 16;
    a.items_b = H / 16;
    a.h0 = L.h0;
    a.h0_dtype = L.h0_dtype;
    a.eps = L.eps;
    for (int l = 0; l < a.nl; ++l) {
        const StackLayer& s = L.layers[l];
        a.norm_w[l] = s.norm;
        StackLayerMaps& mp = a.layer[l];
        if (!encode_q4_maps(s.gate, 16, &mp.g, &mp.gs, &mp.gb) || !encode_q4_maps(s.up, 16, &mp.u, &mp.us, &mp.ub) ||
            !encode_q4_maps(s.down, 16, &mp.d, &mp.ds, &mp.db))
            return cudaErrorInvalidValue;
    }
    uint8_t* ws = static_cast<uint8_t*>(L.scratch);
    a.hbuf = reinterpret_cast<float*>(ws);
    a.act = reinterpret_cast<float*>(ws + (size_t)3 * M * H * 4);
    a.h_last = stack_output(L);
    a.bar = L.bar;
    a.off_bar = p.off_bar;
    a.off_misc = p.off_misc;
    a.off_scr = p.off_scr;
    a.off_xs = p.off_xs;
    a.off_cs = p.off_cs;
    a.off_xq = p.off_xq;
    a.off_red = p.off_red;
    a.off_ring = p.off_ring;
    a.off_xe = p.off_xe;
    const int grid = device_num_sms();

    auto go = [&](auto kernel) -> cudaError_t {
        cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)p.smem);
        if (e != cudaSuccess) return e;
        int per_sm = 0;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kSThreads, p.smem);
        if (e != cudaSuccess) return e;
        if (per_sm < 1) return cudaErrorInvalidConfiguration;
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kSThreads);
        cfg.dynamicSmemBytes = p.smem;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeCooperative;
        attr[0].val.cooperative = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        return cudaLaunchKernelEx(&cfg, kernel, a);
    };
    return p.ntn == 1 ? go(q4_stack_kernel<1>) : go(q4_stack_kernel<2>);
}

int stack_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
