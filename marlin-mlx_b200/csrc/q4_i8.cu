// q4_i8.cu — Q4 decode GEMV family and fused lm_head + argmax on integer tensor-core MMAs (sm_100a).
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) for decode-sized
// activations of marlin-mlx (src/model/marlin.cpp:18-25, :31-35, :161-169) and the greedy
// mx::argmax after the lm_head (src/sampling/sampler.cpp:14-16).
//
// Arithmetic.  Per 64-group, y = s * sum(x * q) + b * sum(x) (the reference's dequant w = s*q + b).
// The codes q (0..15) are the integer MMA's A operand as they are: one LOP3 turns a packed word
// into four code bytes, a shift and a LOP3 give the other four.  The activation row is written as
// four signed 8-bit planes with one power-of-two scale c_m per row and CTA:
//     x = c_m * (i0 + i1 / 128 + i2 / 128^2 + i3 / 128^3),   |i_p| <= 64,
// exact for every element within 2^-27 of the row's largest magnitude.  mma.m16n8k32 (s8 x s8 ->
// s32) then forms sum(q * i_p) exactly; the fold per group is y += s * D_p (binary32), the
// bias term b * sum(x) / c_m rides on plane 0, and the planes combine once per output
// (sum_p c_m 128^-p y_p).  No dequantized weight is ever materialised.
//
// Streaming.  A producer warp moves weights with 2-D TMA into a ring of stages: per stage one
// 128-byte line (4 groups) of 128 rows with 128-byte swizzle + the rows' scales and biases.  Eight
// consumer warps each own 16 rows.  The GEMV family splits K over a thread-block cluster and
// reduces partial sums through distributed shared memory; its weights are requested before
// griddepcontrol.wait so they stream while the previous kernel finishes.  The lm_head kernel is
// persistent over 128-row vocabulary blocks and keeps argmax keys (ordered logit << 32 | ~index).
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_i8.cuh"
#include "q4_i8_common.cuh"
#include "q4_stage.cuh"

#include <algorithm>

// Optional timeline hooks of the decode GEMV kernel, empty in the library build: I8_MARK_BEGIN()
// at entry, I8_MARK(point) at phase boundaries (evaluated by thread 0 of each CTA), I8_STAGE_MARK(q)
// when stage q of the ring is ready.
#ifndef I8_MARK_BEGIN
#define I8_MARK_BEGIN()
#endif
#ifndef I8_MARK
#define I8_MARK(k)
#endif
#ifndef I8_STAGE_MARK
#define I8_STAGE_MARK(q)
#endif

namespace marlin {
namespace {

constexpr int kI8Rows = 128;                          // weight rows per block: 8 warps x 16
constexpr int kI8Warps = 8;                           // consumer warps
constexpr int kI8Threads = (kI8Warps + 1) * 32;       // + the TMA producer warp
constexpr int kI8StageGroups = 4;                     // 64-groups per stage (one 128-byte line per row)
constexpr uint32_t kI8Packed = kI8Rows * 128;         // 16 KB of packed words per stage
constexpr uint32_t kI8Sb = kI8Rows * 16;              // scales (or biases) box: 8 groups x 128 rows
constexpr uint32_t kI8StageBytes = kI8Packed + 2 * kI8Sb;  // 20 KB
constexpr uint32_t kI8SmemLimit = 225 * 1024;
constexpr uint32_t kI8TwoPerSm = 110 * 1024;          // two CTAs per SM (PDL overlap of neighbours)

// Issue the TMA copies of one stage: groups [gs, gs + 4) of rows [row0, row0 + rows) of one matrix
// (rows = 128, or 64 per matrix for the gate/up pair with row offset ro).
__device__ __forceinline__ void i8_issue(uint8_t* st, const CUtensorMap* tw, const CUtensorMap* ts,
                                         const CUtensorMap* tb, int gs, int64_t row0, int ro, uint64_t* bar) {
    tma_load_2d(st + ro * 128, tw, gs * 8, (int32_t)row0, bar);
    tma_load_2d(st + kI8Packed + ro * 16, ts, gs & ~7, (int32_t)row0, bar);
    tma_load_2d(st + kI8Packed + kI8Sb + ro * 16, tb, gs & ~7, (int32_t)row0, bar);
}

// ------------------------------------------------------------------------------------------------
// activation planes handed between kernels (XPlanes)
// ------------------------------------------------------------------------------------------------
// Consumer side, one thread: bulk-copy groups [g0, g0 + ng) of the planes into shared memory.
__device__ __forceinline__ void copy_planes_in(const XPlanes& P, int g0, int ng, int ncols, const I8X& t,
                                               uint64_t* bar) {
    const uint32_t qb = (uint32_t)ng * ncols * 64, fb = (uint32_t)ng * ncols * 4;
    mbar_arrive_expect_tx(bar, qb + 2 * fb);
    tma_bulk_g2s(t.xq, P.q + (size_t)g0 * ncols * 64, qb, bar);
    tma_bulk_g2s(t.xs, P.xs + (size_t)g0 * ncols, fb, bar);
    tma_bulk_g2s(t.xe, P.xe + (size_t)g0 * ncols, fb, bar);
}

// Consumer side, whole block: the plane weights cs and, when an RMSNorm applies, the row factors
// r_m = 1/sqrt(sum(ssq blocks) / K + eps) (binary32, blocks summed in order).
__device__ __forceinline__ void planes_factors(const XPlanes& P, const uint16_t* norm_w, float eps, int M, int K,
                                               int ncols, const I8X& t) {
    for (int c = threadIdx.x; c < ncols; c += blockDim.x) t.cs[c] = (c >> 2) < M ? pow2f(-10 - 7 * (c & 3)) : 0.f;
    if (norm_w && (int)threadIdx.x < M) {
        float s = 0.f;
        for (int b = 0; b < P.nssq; ++b) s = __fadd_rn(s, P.ssq[(size_t)b * M + threadIdx.x]);
        const float var = __fmul_rn(s, (float)(1.0 / (double)K));
        t.rf[threadIdx.x] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
}

__device__ __forceinline__ void named_bar_sync(int id, int n) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(n) : "memory");
}

// Producer side, called by the `nthreads` epilogue threads (whole warps; two consecutive warps own
// one 64-group): thread holds element k of group gi, value v[m] (the operand) and raw[m] (whose
// squares feed P.ssq).  Per group: exponent from the group maximum, s8 digits as planes8, 64 x the
// group sum on plane 0, 2^e on every plane column; padding columns zeroed.  P.ssq[slot][m] gets the
// sum of squares over all `nthreads` rows (fixed order).  ep: shared scratch [nthreads/32][3][MS].
template <int MS>
__device__ __forceinline__ void write_planes(const XPlanes& P, int ncols, int M, int64_t gi, int k,
                                             const float (&v)[MS], const float (&raw)[MS], float* ep, int wig,
                                             int nthreads, int slot) {
    const int lane = threadIdx.x & 31;
    const bool with_ssq = P.ssq != nullptr;
#pragma unroll
    for (int m = 0; m < MS; ++m) {
        if (m < M) {  // warp-uniform
            const unsigned mx = __reduce_max_sync(0xffffffffu, __float_as_uint(fabsf(v[m])));
            float sm = v[m], sq = with_ssq ? __fmul_rn(raw[m], raw[m]) : 0.f;
#pragma unroll
            for (int o = 16; o; o >>= 1) sm += __shfl_xor_sync(0xffffffffu, sm, o);
            if (with_ssq) {
#pragma unroll
                for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
            }
            if (lane == 0) {
                ep[(wig * 3 + 0) * MS + m] = __uint_as_float(mx);
                ep[(wig * 3 + 1) * MS + m] = sm;
                ep[(wig * 3 + 2) * MS + m] = sq;
            }
        }
    }
    named_bar_sync(3, nthreads);
    const int w0 = wig & ~1;
    const size_t gbase = (size_t)gi * ncols;
    const int pos = plane_pos(k);
#pragma unroll
    for (int m = 0; m < MS; ++m) {
        if (m < M) {
            const float gmax = fmaxf(ep[(w0 * 3) * MS + m], ep[((w0 + 1) * 3) * MS + m]);
            const int e = row_exp(__float_as_uint(gmax));
            const float qa = rintf(__fmul_rn(v[m], pow2f(13 - e)));
            const int A = (int)qa;
            const int B = __float2int_rn(__fmul_rn(fmaf(-qa, pow2f(e - 13), v[m]), pow2f(27 - e)));
            const int i0 = (A + 64) >> 7, i2 = (B + 64) >> 7;
            const int d[4] = {i0, A - (i0 << 7), i2, B - (i2 << 7)};
#pragma unroll
            for (int p = 0; p < 4; ++p) P.q[(gbase + 4 * m + p) * 64 + pos] = (uint8_t)(d[p] & 0xff);
            if (k == 0) {
                const float sg = ep[(w0 * 3 + 1) * MS + m] + ep[((w0 + 1) * 3 + 1) * MS + m];
                const float pe = pow2f(e);
                *reinterpret_cast<float4*>(P.xs + gbase + 4 * m) = make_float4(__fmul_rn(sg, 64.0f), 0.f, 0.f, 0.f);
                *reinterpret_cast<float4*>(P.xe + gbase + 4 * m) = make_float4(pe, pe, pe, pe);
            }
        }
    }
    const int pad = ncols - 4 * M;  // padding columns: 16-byte stores spread over the group's 64 threads
    for (int i = k; i < 4 * pad; i += 64)
        *reinterpret_cast<uint4*>(P.q + (gbase + 4 * M + i / 4) * 64 + (i & 3) * 16) = make_uint4(0, 0, 0, 0);
    for (int i = k; i < pad; i += 64) {
        P.xs[gbase + 4 * M + i] = 0.f;
        P.xe[gbase + 4 * M + i] = 0.f;
    }
    if (with_ssq && threadIdx.x == 0) {
        for (int m = 0; m < M; ++m) {
            float sq = 0.f;
            for (int w = 0; w < nthreads / 32; ++w) sq = __fadd_rn(sq, ep[(w * 3 + 2) * MS + m]);
            P.ssq[(size_t)slot * M + m] = sq;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// tensor-parallel exchange (see TpExchange)
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ void st_word_sys(unsigned long long* p, unsigned long long v) {
    asm volatile("st.relaxed.sys.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_word_sys(const unsigned long long* p) {
    unsigned long long v;
    asm volatile("ld.relaxed.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool device_error_set() {
    return *reinterpret_cast<volatile int*>(&g_marlin_device_error) != 0;
}
// Bounded wait for the word at p to carry `tag`; returns its low 32 bits.  Returns 0 without
// spinning when the device error word is already set (an earlier wait ran out: the step's results
// are void and the host must look at the error anyway), and gives up after `limit` SM cycles,
// recording kDevErrMbarTimeout, which makes every later wait return at once.  So a step whose peer
// never writes ends after about one limit, whatever the number of words it waits for.
__device__ __forceinline__ uint32_t wait_word(const unsigned long long* p, uint32_t tag, unsigned long long limit) {
    unsigned long long w = ld_word_sys(p);
    if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
    if (device_error_set()) return 0u;
    const unsigned long long t0 = cycles_now();
    for (uint32_t it = 0;; ++it) {
        w = ld_word_sys(p);
        if ((uint32_t)(w >> 32) == tag) return (uint32_t)w;
        if ((it & 63u) == 63u) {
            if (device_error_set()) return 0u;
            if (cycles_now() - t0 > limit || it > (1u << 30)) {
                record_device_error(kDevErrMbarTimeout);
                return 0u;
            }
        }
    }
}
__device__ __forceinline__ uint32_t tp_tag(const TpExchange& X, int slot) {
    return (*reinterpret_cast<volatile unsigned*>(X.step) << 7) + (uint32_t)slot + 1u;
}

// One epilogue thread per output row: o[m] holds this rank's partial of the row; on return it holds
// the sum over all ranks in rank order (the same bits on every rank).  The thread stores its tagged
// partials into every rank's buffer, then reads each source's word for its row from its own buffer
// once the tag matches.  No barrier: each thread waits only for the words of its own row.
template <int MS>
__device__ __forceinline__ void tp_allreduce_rows(const TpExchange& X, int M, int64_t H, int64_t row, bool live,
                                                  float (&o)[MS]) {
    if (!live) return;
    const int tp = X.tp, P = X.parity;
    const uint32_t tag = tp_tag(X, X.layer);
    for (int p = 0; p < tp; ++p) {
        unsigned long long* dst = X.part[p] + ((size_t)(P * tp + X.rank) * M) * H + row;
#pragma unroll
        for (int m = 0; m < MS; ++m)
            if (m < M) st_word_sys(dst + (size_t)m * H, ((unsigned long long)tag << 32) | __float_as_uint(o[m]));
    }
    const unsigned long long* src = X.part[X.rank] + ((size_t)P * tp * M) * H + row;
#pragma unroll
    for (int m = 0; m < MS; ++m) {
        if (m < M) {
            float v = 0.f;
            for (int r = 0; r < tp; ++r) v += __uint_as_float(wait_word(src + ((size_t)r * M + m) * H, tag, X.wait_cycles));
            o[m] = v;
        }
    }
}

// ------------------------------------------------------------------------------------------------
// decode GEMV family: one 128-row block per thread-block cluster, K split over the cluster's CTAs
// ------------------------------------------------------------------------------------------------
struct I8UnitArgs {
    CUtensorMap tw0, ts0, tb0, tw1, ts1, tb1;  // w0 (gate / main) and w1 (up) maps
    GemvLaunch L;
    int G, CL, gpc, S, ncols;  // groups, cluster size, groups per CTA, ring stages, activation columns
    uint32_t off_bar, off_misc, off_scr, off_xs, off_cs, off_red, off_xq, off_ring, off_xe, off_ep;
};

// One instantiation per activation width serves all three epilogues (a run-time switch), so the
// gate/up and down launches of a decode step run the same, already cached, instructions.
template <int NTN>
__global__ void __launch_bounds__(kI8Threads, 2) i8_unit_kernel(const __grid_constant__ I8UnitArgs a) {
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    I8_MARK_BEGIN();
    constexpr int MS = 2 * NTN;  // activation rows per pass
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = (int)L.m, CL = a.CL, S = a.S;
    constexpr int ncols = 8 * NTN;  // == a.ncols
    const uint32_t rank = CL > 1 ? cluster_rank() : 0u;
    const int block = blockIdx.x / CL;
    const int g0 = (int)rank * a.gpc, ng = min(a.gpc, a.G - g0);
    const int nst = ng / kI8StageGroups;
    const int EPI = L.epi;
    const bool kSwiglu = EPI == kEpiSwiglu;
    const int kHalf = kSwiglu ? kI8Rows / 2 : kI8Rows;  // rows per matrix in the block
    const int64_t row0 = (int64_t)block * kHalf;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    float* red = reinterpret_cast<float*>(smem + a.off_red);  // [CL][128][MS], then the SwiGLU exchange
    uint8_t* ring = smem + a.off_ring;
    I8X tx{smem + a.off_xq, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_cs),
           reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
           reinterpret_cast<unsigned int*>(smem + a.off_misc + 64), reinterpret_cast<float*>(smem + a.off_xe)};

    auto issue = [&](int q) {
        uint8_t* st = ring + (size_t)(q % S) * kI8StageBytes;
        const int gs = g0 + q * kI8StageGroups;
        mbar_arrive_expect_tx(&full[q % S], kI8StageBytes);
        i8_issue(st, &a.tw0, &a.ts0, &a.tb0, gs, row0, 0, &full[q % S]);
        if (kSwiglu) i8_issue(st, &a.tw1, &a.ts1, &a.tb1, gs, row0, kHalf, &full[q % S]);
    };
    uint64_t* xbar = full + 2 * S;  // planes copied in (has_xin)
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kI8Warps);
        }
        mbar_init(xbar, 1);
        fence_mbar_init();
        prefetch_tmap(&a.tw0);
        // as much of this CTA's weight range as the ring holds, before the dependency wait
        for (int q = 0; q < min(S, nst); ++q) issue(q);
    }
    // epilogue operands that do not wait for the math, read early by the leader's epilogue threads
    // (small batches: held in registers through the main loop): the next RMSNorm weight (a weight,
    // read before the dependency wait) and the residual rows (read right after it)
    constexpr bool kEarly = MS <= 4;
    const bool early = kEarly && rank == 0 && tid < kI8Rows && EPI == kEpiResid && row0 + tid < L.w0.n;
    float wpre = 0.f, rpre[MS];
#pragma unroll
    for (int m = 0; m < MS; ++m) rpre[m] = 0.f;
    if (early && L.has_xout && L.out_norm) wpre = bf16_bits_to_f32(L.out_norm[row0 + tid]);
    __syncthreads();
    I8_MARK(1);
    pdl_wait();
    I8_MARK(2);
    pdl_launch_dependents();
    if (early) {
#pragma unroll
        for (int m = 0; m < MS; ++m)
            if (m < M)
                rpre[m] = L.resid_dtype == kBF16
                              ? bf16_bits_to_f32(static_cast<const uint16_t*>(L.resid)[(int64_t)m * L.ldr + row0 + tid])
                              : static_cast<const float*>(L.resid)[(int64_t)m * L.ldr + row0 + tid];
    }
    if (L.has_xin) {
        if (tid == kI8Warps * 32) copy_planes_in(L.xin, g0, ng, ncols, tx, xbar);
        planes_factors(L.xin, L.norm_w, L.eps, M, (int)L.w0.k, ncols, tx);
        __syncthreads();
    } else {
        stage_x_i8(L.x, L.x_dtype, (int)L.w0.k, L.norm_w, L.eps, g0, ng, M, ncols, tx);
    }
    I8_MARK(3);

    float y[NTN][4], yb[NTN][2];
#pragma unroll
    for (int j = 0; j < NTN; ++j) y[j][0] = y[j][1] = y[j][2] = y[j][3] = yb[j][0] = yb[j][1] = 0.f;
    if (warp == kI8Warps) {
        if (lane == 0) {
            int q = min(S, nst);
            for (; q < nst; ++q) {
                if (!thread_wait(&empty[q % S], (uint32_t)(((q / S) - 1) & 1), abort)) break;
                issue(q);
            }
            for (int r = max(0, q - S); r < q; ++r) drain_wait(&full[r % S], (uint32_t)((r / S) & 1));
            if (L.has_xin) drain_wait(xbar, 0u);
        }
    } else {
        const bool xin_ok = !L.has_xin || warp_wait(xbar, 0u, abort);
        I8_MARK(14);
        int slot = 0;  // ring position of stage q, kept as a counter (no division per stage)
        uint32_t ph = 0u;
        for (int q = 0; xin_ok && q < nst; ++q) {
            if (!warp_wait(&full[slot], ph, abort)) break;
            I8_STAGE_MARK(q);
            const int gs = g0 + q * kI8StageGroups;
            i8_stage<NTN>(ring + (size_t)slot * kI8StageBytes, (gs & 7) * 2, q * kI8StageGroups, tx, warp, lane, y, yb);
#pragma unroll
            for (int j = 0; j < NTN; ++j) {  // the stage's data is consumed before release
                hold_regs(y[j]);
                hold_regs(yb[j]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == S) {
                slot = 0;
                ph ^= 1u;
            }
        }
        // planes -> one partial per (row, activation row), into the leader's slot for this rank
        const int g = lane >> 2, tq = lane & 3;
        const int r0 = 16 * warp + g;
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            const float2 cv = *reinterpret_cast<const float2*>(tx.cs + 8 * j + 2 * tq);
            const float2 pp = i8_combine(y[j], yb[j], cv, tq);
            const float p0 = pp.x, p1 = pp.y;
            const int m = 2 * j + (tq >> 1);
            if ((tq & 1) == 0 && m < M) {
                float* s0 = red + ((size_t)rank * kI8Rows + r0) * MS + m;
                float* s1 = red + ((size_t)rank * kI8Rows + r0 + 8) * MS + m;
                if (rank == 0) {
                    *s0 = p0;
                    *s1 = p1;
                } else {
                    st_cluster_f32(s0, 0, p0);
                    st_cluster_f32(s1, 0, p1);
                }
            }
        }
        I8_MARK(4);
    }
    if (CL > 1) cluster_sync_all();
    else __syncthreads();
    I8_MARK(5);
    if (rank != 0 || tid >= kI8Rows) return;

    // leader epilogue: thread = block row lrow; out[m] = sum over the cluster's partials
    const int lrow = tid;
    const bool row_factor = L.has_xin && L.norm_w;  // RMSNorm as a row factor on planes copied in
    float* ep = reinterpret_cast<float*>(smem + a.off_ep);
    float o[MS];
#pragma unroll
    for (int m = 0; m < MS; ++m) {
        o[m] = 0.f;
        if (m < M) {
            for (int r = 0; r < CL; ++r) o[m] += red[((size_t)r * kI8Rows + lrow) * MS + m];
            if (row_factor) o[m] *= tx.rf[m];
        }
    }
    I8_MARK(16);
    if (kSwiglu) {
        // up rows (64..127) hand their outputs to the gate rows through shared memory
        float* xch = red + (size_t)CL * kI8Rows * MS;
        if (lrow >= kHalf) {
#pragma unroll
            for (int m = 0; m < MS; ++m) xch[(lrow - kHalf) * MS + m] = o[m];
        }
        asm volatile("bar.sync 2, 128;" ::: "memory");
        if (lrow < kHalf) {
            const int64_t f = row0 + lrow;
            float av[MS];
#pragma unroll
            for (int m = 0; m < MS; ++m) {
                av[m] = 0.f;
                if (m < M && f < L.w0.n) {
                    const float gsum = o[m], u = xch[lrow * MS + m];
                    if (L.y_dtype == kBF16) {
                        const float gq = bf16_round(gsum), uq = bf16_round(u);
                        const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
                        av[m] = bf16_round(bf16_round(sg * gq) * uq);
                        static_cast<uint16_t*>(L.y)[(int64_t)m * L.ldy + f] = (uint16_t)f32_to_bf16_bits(av[m]);
                    } else {
                        const float sg = 1.0f / (1.0f + expf(-gsum));
                        av[m] = (sg * gsum) * u;
                        static_cast<float*>(L.y)[(int64_t)m * L.ldy + f] = av[m];
                    }
                }
            }
            // one 64-group of the activation per block (kHalf = 64 rows per matrix)
            I8_MARK(15);
            if (L.has_xout) write_planes<MS>(L.xout, ncols, M, row0 / 64, lrow, av, av, ep, lrow >> 5, kHalf, block);
        }
        I8_MARK(6);
        return;
    }
    const int64_t row = row0 + lrow;
    const bool live = row < L.w0.n;
    if (L.tp.tp > 1) tp_allreduce_rows<MS>(L.tp, M, L.w0.n, row, live, o);
    float v[MS], u[MS];
    const float wn = early ? wpre : (L.has_xout && L.out_norm && live) ? bf16_bits_to_f32(L.out_norm[row]) : 0.f;
#pragma unroll
    for (int m = 0; m < MS; ++m) {
        v[m] = u[m] = 0.f;
        if (m < M && live) {
            v[m] = o[m];
            if (EPI == kEpiResid) {
                const float hv =
                    early ? rpre[m]
                    : L.resid_dtype == kBF16
                        ? bf16_bits_to_f32(static_cast<const uint16_t*>(L.resid)[(int64_t)m * L.ldr + row])
                        : static_cast<const float*>(L.resid)[(int64_t)m * L.ldr + row];
                v[m] = hv + v[m];
            }
            if (L.y_dtype == kBF16) {
                static_cast<uint16_t*>(L.y)[(int64_t)m * L.ldy + row] = (uint16_t)f32_to_bf16_bits(v[m]);
                v[m] = bf16_round(v[m]);
            } else {
                static_cast<float*>(L.y)[(int64_t)m * L.ldy + row] = v[m];
            }
            u[m] = L.out_norm ? __fmul_rn(v[m], __fadd_rn(1.0f, wn)) : v[m];
        }
    }
    // two 64-groups per 128-row block
    I8_MARK(15);
    if (L.has_xout) write_planes<MS>(L.xout, ncols, M, row / 64, lrow & 63, u, v, ep, lrow >> 5, kI8Rows, block);
    I8_MARK(6);
}

// ------------------------------------------------------------------------------------------------
// fused lm_head + argmax (persistent over 128-row vocabulary blocks)
// ------------------------------------------------------------------------------------------------
struct I8LmArgs {
    CUtensorMap tw, ts, tb;  // boxes of 128 rows
    LmHeadLaunch L;
    int G, S, nblocks, ncols;
    uint32_t off_bar, off_misc, off_keys, off_scr, off_xs, off_cs, off_xq, off_ring, off_xe;
};

// lm_head stage: 16 W rows x 4 groups, loaded as 16 W / 128 boxes of 128 rows per tensor
template <int W>
struct LmStage {
    static constexpr int kRows = 16 * W;
    static constexpr uint32_t kBytes = kRows * (128 + 2 * 16);
    static constexpr int kThreads = (W + 1) * 32;
};

__device__ __forceinline__ unsigned long long i8_logit_key(float v, int64_t idx) {
    const uint32_t u = __float_as_uint(v);
    const uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}

template <int NTN, int W>
__global__ void __launch_bounds__(LmStage<W>::kThreads, 1) i8_lm_head_kernel(const __grid_constant__ I8LmArgs a) {
    using ST = LmStage<W>;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const LmHeadLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.G, S = a.S, M = (int)L.m;
    constexpr int ncols = 8 * NTN;  // == a.ncols
    const int spb = G / kI8StageGroups;  // stages per block
    const int my_blocks =
        a.nblocks > (int)blockIdx.x ? (a.nblocks - 1 - (int)blockIdx.x) / (int)gridDim.x + 1 : 0;
    const int nst = my_blocks * spb;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint64_t* empty = full + S;
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_keys);  // [8][M]
    uint8_t* ring = smem + a.off_ring;
    I8X tx{smem + a.off_xq, reinterpret_cast<float*>(smem + a.off_xs), reinterpret_cast<float*>(smem + a.off_cs),
           reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
           reinterpret_cast<unsigned int*>(smem + a.off_misc + 64), reinterpret_cast<float*>(smem + a.off_xe)};

    // stage at ring slot `slot`: stage sp of this CTA's block bi
    auto issue_at = [&](int slot, int sp, int bi) {
        const int gs = sp * kI8StageGroups;
        const int64_t row0 = (int64_t)(blockIdx.x + (int64_t)bi * gridDim.x) * ST::kRows;
        uint8_t* st = ring + (size_t)slot * ST::kBytes;
        mbar_arrive_expect_tx(&full[slot], ST::kBytes);
#pragma unroll
        for (int h = 0; h < ST::kRows / kI8Rows; ++h) {
            const int32_t y = (int32_t)(row0 + h * kI8Rows);
            tma_load_2d(st + h * kI8Rows * 128, &a.tw, gs * 8, y, &full[slot]);
            tma_load_2d(st + ST::kRows * 128 + h * kI8Rows * 16, &a.ts, gs & ~7, y, &full[slot]);
            tma_load_2d(st + ST::kRows * 144 + h * kI8Rows * 16, &a.tb, gs & ~7, y, &full[slot]);
        }
    };
    auto issue = [&](int q) { issue_at(q % S, q % spb, q / spb); };
    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], W);
        }
        mbar_init(full + 2 * S, 1);
        fence_mbar_init();
        prefetch_tmap(&a.tw);
        prefetch_tmap(&a.ts);
        prefetch_tmap(&a.tb);
        for (int q = 0; q < min(S, nst); ++q) issue(q);
    }
    __syncthreads();
    pdl_wait();
    pdl_launch_dependents();
    if (blockIdx.x == 0) {
        if (L.reset && tid < L.n_reset) L.reset[tid] = 0u;
        if (L.x_out && L.x_dtype == kFix64) {
            const unsigned long long* xf = static_cast<const unsigned long long*>(L.x);
            for (int i = tid; i < M * (int)L.w.k; i += blockDim.x)
                L.x_out[i] = fix_value(__ldcg(xf + i));
        }
    }
    uint64_t* xbar = full + 2 * S;  // planes copied in (has_xin)
    if (L.has_xin) {
        if (tid == W * 32) copy_planes_in(L.xin, 0, G, ncols, tx, xbar);
        planes_factors(L.xin, L.norm_w, L.eps, M, (int)L.w.k, ncols, tx);
        __syncthreads();
    } else {
        stage_x_i8(L.x, L.x_dtype, (int)L.w.k, L.norm_w, L.eps, 0, G, M, ncols, tx);
    }

    if (warp == W) {
        if (lane == 0) {
            int q = min(S, nst);
            int slot = q % S, sp = q % spb, bi = q / spb;  // counters from here on
            uint32_t ph = (uint32_t)(((q / S) - 1) & 1);
            for (; q < nst; ++q) {
                if (!thread_wait(&empty[slot], ph, abort)) break;
                issue_at(slot, sp, bi);
                if (++slot == S) {
                    slot = 0;
                    ph ^= 1u;
                }
                if (++sp == spb) {
                    sp = 0;
                    ++bi;
                }
            }
            for (int r = max(0, q - S); r < q; ++r) drain_wait(&full[r % S], (uint32_t)((r / S) & 1));
            if (L.has_xin) drain_wait(xbar, 0u);
        }
    } else {
        const int g = lane >> 2, tq = lane & 3;
        const bool bf16_logits = L.x_dtype == kBF16 && !L.norm_w && !L.has_xin;
        const bool row_factor = L.has_xin && L.norm_w;
        const bool xin_ok = !L.has_xin || warp_wait(xbar, 0u, abort);
        float y[NTN][4], yb[NTN][2];
        unsigned long long best[NTN];
#pragma unroll
        for (int j = 0; j < NTN; ++j) {
            y[j][0] = y[j][1] = y[j][2] = y[j][3] = yb[j][0] = yb[j][1] = 0.f;
            best[j] = 0ull;
        }
        int slot = 0, sp = 0, bi = 0;  // ring position, stage within the block, block (counters)
        uint32_t ph = 0u;
        for (int q = 0; xin_ok && q < nst; ++q) {
            if (!warp_wait(&full[slot], ph, abort)) break;
            const int gs = sp * kI8StageGroups;
            i8_stage<NTN, ST::kRows>(ring + (size_t)slot * ST::kBytes, (gs & 7) * 2, gs, tx, warp, lane, y, yb);
#pragma unroll
            for (int j = 0; j < NTN; ++j) {  // the stage's data is consumed before release
                hold_regs(y[j]);
                hold_regs(yb[j]);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[slot]);
            if (++slot == S) {
                slot = 0;
                ph ^= 1u;
            }
            if (++sp == spb) {  // block finished: logits -> argmax keys (max over the warp's rows)
                sp = 0;
                const int64_t rowa = (int64_t)(blockIdx.x + (int64_t)bi * gridDim.x) * ST::kRows + 16 * warp + g;
                ++bi;
                const int64_t rowb = rowa + 8;
#pragma unroll
                for (int j = 0; j < NTN; ++j) {
                    const float2 cv = *reinterpret_cast<const float2*>(tx.cs + 8 * j + 2 * tq);
                    const float2 ll = i8_combine(y[j], yb[j], cv, tq);
                    float la = ll.x, lb = ll.y;
                    if (row_factor) {
                        const float rfm = tx.rf[min(2 * j + (tq >> 1), M - 1)];
                        la *= rfm;
                        lb *= rfm;
                    }
                    if (bf16_logits) {
                        la = bf16_round(la);
                        lb = bf16_round(lb);
                    }
                    const int m = 2 * j + (tq >> 1);
                    unsigned long long ka = (m < M && rowa < L.w.n) ? i8_logit_key(la, L.vocab_offset + rowa) : 0ull;
                    const unsigned long long kb =
                        (m < M && rowb < L.w.n) ? i8_logit_key(lb, L.vocab_offset + rowb) : 0ull;
                    ka = kb > ka ? kb : ka;
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        const unsigned long long other = __shfl_xor_sync(0xffffffffu, ka, o);
                        ka = other > ka ? other : ka;
                    }
                    best[j] = ka > best[j] ? ka : best[j];
                    y[j][0] = y[j][1] = y[j][2] = y[j][3] = yb[j][0] = yb[j][1] = 0.f;
                }
            }
        }
        if (g == 0 && (tq & 1) == 0) {
#pragma unroll
            for (int j = 0; j < NTN; ++j) {
                const int m = 2 * j + (tq >> 1);
                if (m < M) ckeys[warp * M + m] = best[j];
            }
        }
    }
    __syncthreads();
    __shared__ bool is_last;
    if (tid < M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < W; ++w) k = ckeys[w * M + tid] > k ? ckeys[w * M + tid] : k;
        if (k) atomicMax(&L.keys[tid], k);
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int prev = atomicAdd(L.counter, 1u);
        is_last = (prev == gridDim.x - 1);
    }
    __syncthreads();
    if (is_last) {
        __threadfence();
        unsigned long long k = 0ull;
        if (tid < M) k = atomicExch(&L.keys[tid], 0ull);
        if (L.tp.tp > 1) {
            // max-merge of the ranks' keys: tagged halves to every rank, then each rank's from the own buffer
            const TpExchange& X = L.tp;
            const uint32_t tag = tp_tag(X, 126);
            if (tid < M) {
                const unsigned long long th = (unsigned long long)tag << 32;
                for (int p = 0; p < X.tp; ++p) {
                    unsigned long long* d = X.keys[p] + ((size_t)X.rank * M + tid) * 2;
                    st_word_sys(d, th | (k & 0xffffffffull));
                    st_word_sys(d + 1, th | (k >> 32));
                }
                for (int r = 0; r < X.tp; ++r) {
                    const unsigned long long* sw = X.keys[X.rank] + ((size_t)r * M + tid) * 2;
                    const unsigned long long kr = (unsigned long long)wait_word(sw, tag, X.wait_cycles) |
                                                  ((unsigned long long)wait_word(sw + 1, tag, X.wait_cycles) << 32);
                    k = kr > k ? kr : k;
                }
            }
            __syncthreads();  // every thread of this CTA has read this step's words
            if (tid == 0) *reinterpret_cast<volatile unsigned*>(X.step) = *reinterpret_cast<volatile unsigned*>(X.step) + 1u;
        }
        if (tid < M) {
            if (L.keys_out) L.keys_out[tid] = k;
            const uint32_t o = (uint32_t)(k >> 32);
            const uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
            if (L.ids) L.ids[tid] = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
            if (L.best) L.best[tid] = __uint_as_float(u);
        }
        if (tid == 0) atomicExch(L.counter, 0u);
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
int ntn_for(int64_t m) { return m <= 2 ? 1 : (m <= 4 ? 2 : (m <= 8 ? 4 : 8)); }

size_t al256(size_t v) { return (v + 255) / 256 * 256; }

// Shared-memory layout common to both kernels; returns the byte offset after the activations.
uint32_t plan_common(int M, int K, bool normed, int ng, int ncols, uint32_t& off_bar, uint32_t& off_misc,
                     uint32_t& off_scr, uint32_t& off_xs, uint32_t& off_cs, uint32_t& off_xe, int S) {
    uint32_t off = 0;
    off_bar = off;
    off += align_up((2u * (uint32_t)S + 1u) * 8u, 128);  // full[S], empty[S], planes copy-in
    off_misc = off;
    off += 128;  // abort flag + amax[M <= 16]
    off_scr = off;
    off += align_up((64 + (normed ? (uint32_t)M * (K / 8) : 0u)) * 4, 128);
    off_xs = off;
    off += align_up((uint32_t)ng * ncols * 4, 128);
    off_cs = off;
    off += align_up((uint32_t)ncols * 4, 128);
    off_xe = off;
    off += align_up((uint32_t)ng * ncols * 4, 128);
    return off;
}

uint32_t plan_i8_unit(const GemvLaunch& L, I8UnitArgs& a) {
    a.L = L;
    const int K = (int)L.w0.k;
    a.G = K / kGroup;
    const int ntn = ntn_for(L.m);
    a.ncols = 8 * ntn;
    const bool swiglu = L.epi == kEpiSwiglu;
    const int half = swiglu ? kI8Rows / 2 : kI8Rows;
    const int blocks = (int)((L.w0.n + half - 1) / half);
    // cluster size: split K until the grid covers the SMs (groups per CTA stay a multiple of 4)
    int CL = 0;
    for (int c : {1, 2, 4, 8}) {
        if (a.G % c || (a.G / c) % kI8StageGroups) continue;
        CL = c;
        if ((int64_t)blocks * c >= device_num_sms()) break;
    }
    if (!CL) return 0;
    a.CL = CL;
    a.gpc = a.G / CL;
    const int nst = a.gpc / kI8StageGroups;
    const int ms = 2 * ntn;
    // two CTAs per SM (latency hiding, and the next launch's CTAs prefetching beside this one's) with
    // as deep a ring as fits them; else the whole weight range resident in one CTA per SM
    for (int S = nst; S >= 2; --S) {
        uint32_t off = plan_common((int)L.m, K, L.norm_w != nullptr, a.gpc, a.ncols, a.off_bar, a.off_misc, a.off_scr,
                                   a.off_xs, a.off_cs, a.off_xe, S);
        a.off_red = off;
        off += align_up((uint32_t)(CL + 1) * kI8Rows * ms * 4, 128);
        a.off_ep = off;
        off += align_up(4u * 3u * (uint32_t)ms * 4u, 128);
        a.off_xq = off;
        off += (uint32_t)a.gpc * a.ncols * 64;
        off = align_up(off, 1024);
        a.off_ring = off;
        off += (uint32_t)S * kI8StageBytes + 1024;
        if (off <= kI8TwoPerSm) {
            a.S = S;
            return off;
        }
    }
    for (int S = nst; S >= 2 || S == nst; --S) {
        uint32_t off = plan_common((int)L.m, K, L.norm_w != nullptr, a.gpc, a.ncols, a.off_bar, a.off_misc, a.off_scr,
                                   a.off_xs, a.off_cs, a.off_xe, S);
        a.off_red = off;
        off += align_up((uint32_t)(CL + 1) * kI8Rows * ms * 4, 128);  // partials + SwiGLU exchange
        a.off_ep = off;
        off += align_up(4u * 3u * (uint32_t)ms * 4u, 128);  // epilogue plane statistics
        a.off_xq = off;
        off += (uint32_t)a.gpc * a.ncols * 64;
        off = align_up(off, 1024);
        a.off_ring = off;
        off += (uint32_t)S * kI8StageBytes + 1024;
        const uint32_t limit = (S == nst && off <= kI8TwoPerSm) ? kI8TwoPerSm : kI8SmemLimit;
        if (off <= limit) {
            a.S = S;
            return off;
        }
        if (S <= 2) break;
    }
    return 0;
}

// consumer warps of the lm_head kernel: 16 (256-row blocks) while the activation planes leave
// room for at least three 40 KB stages, else 8
int lm_warps(int64_t m) { return ntn_for(m) <= 4 ? 16 : 8; }

uint32_t plan_i8_lm_head(const LmHeadLaunch& L, I8LmArgs& a, int W) {
    a.L = L;
    const int K = (int)L.w.k;
    a.G = K / kGroup;
    a.ncols = 8 * ntn_for(L.m);
    const int rows = 16 * W;
    const uint32_t stage = (uint32_t)rows * 160;
    a.nblocks = (int)((L.w.n + rows - 1) / rows);
    for (int S = 12; S >= 2; --S) {
        uint32_t off = plan_common((int)L.m, K, L.norm_w != nullptr, a.G, a.ncols, a.off_bar, a.off_misc, a.off_scr,
                                   a.off_xs, a.off_cs, a.off_xe, S);
        a.off_keys = off;
        off += align_up((uint32_t)W * (uint32_t)L.m * 8, 128);
        a.off_xq = off;
        off += (uint32_t)a.G * a.ncols * 64;
        off = align_up(off, 1024);
        a.off_ring = off;
        off += (uint32_t)S * stage + 1024;
        if (off <= kI8SmemLimit) {
            a.S = S;
            return off;
        }
    }
    return 0;
}

template <int NTN>
cudaError_t dispatch_i8_unit(const I8UnitArgs& a, int grid, uint32_t smem, cudaStream_t stream) {
    return launch_ex(i8_unit_kernel<NTN>, a, grid, kI8Threads, a.CL, smem, a.L.pdl, stream);
}

}  // namespace

bool i8_supported(int64_t k, int64_t m) {
    // k % 512: the scales/biases tensor maps need a row stride (k/64 * 2 bytes) that is a
    // multiple of 16 bytes
    return k % 512 == 0 && k <= 16384 && m >= 1 && m <= kI8MaxRows && tmap_encode_fn() != nullptr;
}

cudaError_t launch_i8_gemv(const GemvLaunch& L, cudaStream_t stream) {
    if (rows_gemv_applies(L)) return launch_rows_gemv(L, stream);
    I8UnitArgs a{};
    const uint32_t smem = plan_i8_unit(L, a);
    if (!smem) return cudaErrorInvalidConfiguration;
    const bool swiglu = L.epi == kEpiSwiglu;
    const int half = swiglu ? kI8Rows / 2 : kI8Rows;
    if (!encode_q4_maps(L.w0, half, &a.tw0, &a.ts0, &a.tb0)) return cudaErrorInvalidValue;
    if (swiglu && !encode_q4_maps(L.w1, half, &a.tw1, &a.ts1, &a.tb1)) return cudaErrorInvalidValue;
    const int blocks = (int)((L.w0.n + half - 1) / half);
    const int grid = blocks * a.CL;
    switch (a.ncols / 8) {
        case 1: return dispatch_i8_unit<1>(a, grid, smem, stream);
        case 2: return dispatch_i8_unit<2>(a, grid, smem, stream);
        case 4: return dispatch_i8_unit<4>(a, grid, smem, stream);
        default: return dispatch_i8_unit<8>(a, grid, smem, stream);
    }
}

cudaError_t launch_i8_lm_head(const LmHeadLaunch& L, cudaStream_t stream) {
    I8LmArgs a{};
    const int W = lm_warps(L.m);
    const uint32_t smem = plan_i8_lm_head(L, a, W);
    if (!smem) return cudaErrorInvalidConfiguration;
    if (!encode_q4_maps(L.w, kI8Rows, &a.tw, &a.ts, &a.tb)) return cudaErrorInvalidValue;
    const int grid = std::max(1, std::min(device_num_sms(), a.nblocks));
    if (W == 16) {
        constexpr int T = LmStage<16>::kThreads;
        switch (a.ncols / 8) {
            case 1: return launch_ex(i8_lm_head_kernel<1, 16>, a, grid, T, 1, smem, L.pdl, stream);
            case 2: return launch_ex(i8_lm_head_kernel<2, 16>, a, grid, T, 1, smem, L.pdl, stream);
            default: return launch_ex(i8_lm_head_kernel<4, 16>, a, grid, T, 1, smem, L.pdl, stream);
        }
    }
    return launch_ex(i8_lm_head_kernel<8, 8>, a, grid, LmStage<8>::kThreads, 1, smem, L.pdl, stream);
}

int i8_device_error(bool clear) { return tu_device_error(clear); }

int i8_ncols(int64_t m) { return 8 * ntn_for(m); }

size_t i8_planes_bytes(int64_t m, int64_t k) {
    const size_t g = (size_t)(k / kGroup), c = (size_t)i8_ncols(m);
    return al256(g * c * 64) + 2 * al256(g * c * 4);
}

XPlanes i8_planes_at(void* base, int64_t m, int64_t k, float* ssq, int nssq) {
    const size_t g = (size_t)(k / kGroup), c = (size_t)i8_ncols(m);
    uint8_t* p = static_cast<uint8_t*>(base);
    XPlanes P{};
    P.q = p;
    P.xs = reinterpret_cast<float*>(p + al256(g * c * 64));
    P.xe = reinterpret_cast<float*>(p + al256(g * c * 64) + al256(g * c * 4));
    P.ssq = ssq;
    P.nssq = nssq;
    return P;
}

}  // namespace marlin
