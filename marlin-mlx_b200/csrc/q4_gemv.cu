// q4_gemv.cu — Q4 (group-64 affine, MLX layout) decode GEMV / skinny GEMM for sm_100a.
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) on the decode path of
// marlin-mlx (src/model/marlin.cpp:18-25 qmatmul, :31-35 mlp_forward, :161-169 lm_head) and the
// greedy mx::argmax that follows the lm_head (src/sampling/sampler.cpp:14-16).
//
// Data path (per CTA):
//   * Weights stream HBM -> shared memory by 1-D TMA bulk copies (cp.async.bulk, one per packed row
//     into a padded row so the fragment loads are bank-conflict free, one for each tile's scales
//     and biases).  They are issued BEFORE griddepcontrol.wait: a kernel launched with
//     programmatic stream serialization fetches its weights while the previous kernel finishes.
//   * Activations (optionally RMSNorm'ed on the fly) are split into bf16 planes (1 plane for bf16
//     activations, 3 exact hi/mid/lo planes for binary32) and stored pre-permuted in shared memory
//     in mma.sync A-fragment order, together with per-(plane row, group) sums.
//   * Nibbles become bf16 (1 + q/16) with one LOP3 per pair (exact); mma.sync m16n8k16 (bf16 in,
//     fp32 accumulate) with the weights as the B operand (8 weight rows per n8 tile) produces, per
//     64-group, D = sum x*(1+q/16).  The group result is folded as
//        y += 16*s*D + (b - 16*s)*sum(x)  ==  s*sum(x*q) + b*sum(x)
//     so the per-group scale/bias stay in fp32 exactly as the reference's dequant formula says.
//   * K is split across the CTA's warps; partials meet in shared memory for the epilogue
//     (store / SwiGLU of gate+up rows / residual add).
//
// The lm_head kernel streams the vocabulary with a per-warp TMA ring and reduces the argmax on the
// fly: packed (ordered value << 32 | ~index) keys, one atomicMax per CTA and row, the last CTA
// decoding and re-zeroing the keys.  Logits are never written to memory.
#include "common.cuh"
#include "q4_gemv.cuh"

#include <algorithm>

namespace marlin {

namespace {

constexpr int kGroup = 64;
constexpr int kMaxThreads = 256;

// ------------------------------------------------------------------------------------------------
// shared-memory geometry
// ------------------------------------------------------------------------------------------------
// Packed row stride in shared memory: K/2 bytes padded so the row stride in 4-byte words is 8 mod
// 32 (rows g = 0..3 of a half-warp then hit disjoint banks in the fragment loads).
__host__ __device__ inline int packed_row_stride(int K) {
    int words = K / 8;
    int pad = ((8 - (words % 32)) % 32 + 32) % 32;
    return (words + pad) * 4;
}
__host__ __device__ inline uint32_t align_up(uint32_t v, uint32_t a) { return (v + a - 1) / a * a; }
// bytes of one 8-row weight tile in shared memory: packed rows, scales [8][G], biases [8][G]
__host__ __device__ inline uint32_t tile_bytes(int K) {
    int G = K / kGroup;
    return align_up(8u * packed_row_stride(K) + 2u * 8u * G * 2u, 128);
}

// ------------------------------------------------------------------------------------------------
// activation staging
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ float load_act(const void* x, int dtype, int64_t i) {
    if (dtype == kBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(x)[i]);
    return static_cast<const float*>(x)[i];
}

// position of element e (0..15) of a 16-element slot in mma A-fragment order
// (slot order: 0,4,1,5,2,6,3,7,8,12,9,13,10,14,11,15)
__device__ __forceinline__ int frag_pos(int e) { return (e & 8) | ((e & 3) << 1) | ((e >> 2) & 1); }

struct XGeom {
    uint8_t* xp;  // planes: row r = plane*M + m, stride XRS bytes, GC groups of 128 B
    float* xs;    // [M_eff][GC] plane sums per group
    float* rf;    // [M] RMSNorm factors
    float* scr;   // >= 32 floats reduction scratch
    int M, P, M_eff, XRS, GC;
};

// RMSNorm factors r_m = 1/sqrt(mean(x^2) + eps) as MLX's C++ API evaluates
// x * rsqrt(mean(square(x)) + eps) * (1.0f + w)  (src/model/marlin.cpp:12-16):
// bf16 x: square and mean in bf16 (binary32 accumulation, one bf16 rounding of the sum);
// binary32 x: all binary32.  The `+ eps` and everything after it is binary32.
__device__ void compute_norm_factors(const void* x, int dtype, int M, int K, float eps, const XGeom& g) {
    const int nt = blockDim.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    for (int m = 0; m < M; ++m) {
        float part = 0.f;
        for (int k = tid; k < K; k += nt) {
            float v = load_act(x, dtype, (int64_t)m * K + k);
            float sq = __fmul_rn(v, v);
            if (dtype == kBF16) sq = bf16_round(sq);
            part = __fadd_rn(part, sq);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
        if (lane == 0) g.scr[warp] = part;
        __syncthreads();
        if (tid == 0) {
            float sum = 0.f;
            for (int w = 0; w < nt / 32; ++w) sum = __fadd_rn(sum, g.scr[w]);
            float var;
            if (dtype == kBF16)
                var = bf16_round(__fmul_rn(bf16_round(sum), bf16_round((float)(1.0 / (double)K))));
            else
                var = __fmul_rn(sum, (float)(1.0 / (double)K));
            g.rf[m] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
        }
        __syncthreads();
    }
}

// Stage groups [gc0, gc0 + ngc) of the activations into planes + sums.  Ends with __syncthreads.
__device__ void stage_x_chunk(const void* x, int dtype, int K, const uint16_t* norm_w, int gc0, int ngc,
                              const XGeom& g) {
    const int nt = blockDim.x, tid = threadIdx.x;
    const int kc0 = gc0 * kGroup, kcn = ngc * kGroup;
    const int total = g.M * kcn;
    for (int idx = tid; idx < total; idx += nt) {
        const int m = idx / kcn, kl = idx - m * kcn, k = kc0 + kl;
        const int gl = kl >> 6, e = kl & 63, t = e >> 4, pos = frag_pos(e & 15);
        const uint32_t off = gl * 128 + t * 32 + pos * 2;
        float v = load_act(x, dtype, (int64_t)m * K + k);
        if (norm_w) v = __fmul_rn(__fmul_rn(v, g.rf[m]), __fadd_rn(1.0f, bf16_bits_to_f32(norm_w[k])));
        if (g.P == 1) {
            uint16_t h = (dtype == kBF16 && !norm_w) ? static_cast<const uint16_t*>(x)[(int64_t)m * K + k]
                                                      : (uint16_t)f32_to_bf16_bits(v);
            *reinterpret_cast<uint16_t*>(g.xp + (uint32_t)m * g.XRS + off) = h;
        } else {
            uint32_t h0 = f32_to_bf16_bits(v);
            float r1 = __fsub_rn(v, bf16_bits_to_f32(h0));
            uint32_t h1 = f32_to_bf16_bits(r1);
            float r2 = __fsub_rn(r1, bf16_bits_to_f32(h1));
            uint32_t h2 = f32_to_bf16_bits(r2);
            *reinterpret_cast<uint16_t*>(g.xp + (uint32_t)m * g.XRS + off) = (uint16_t)h0;
            *reinterpret_cast<uint16_t*>(g.xp + (uint32_t)(g.M + m) * g.XRS + off) = (uint16_t)h1;
            *reinterpret_cast<uint16_t*>(g.xp + (uint32_t)(2 * g.M + m) * g.XRS + off) = (uint16_t)h2;
        }
    }
    __syncthreads();
    for (int idx = tid; idx < g.M_eff * ngc; idx += nt) {
        const int r = idx / ngc, gl = idx - r * ngc;
        const uint32_t* p = reinterpret_cast<const uint32_t*>(g.xp + (uint32_t)r * g.XRS + gl * 128);
        float s = 0.f;
#pragma unroll 8
        for (int j = 0; j < 32; ++j) {
            uint32_t v = p[j];
            s += bf16_bits_to_f32(v & 0xffffu) + bf16_bits_to_f32(v >> 16);
        }
        g.xs[r * g.GC + gl] = s;
    }
    __syncthreads();
}

// ------------------------------------------------------------------------------------------------
// per-warp tensor-core group loop
// ------------------------------------------------------------------------------------------------
// Scale table entry (group, row): (16*s, b - 16*s), built once per tile and K range.
__device__ __forceinline__ void build_sb_table(const uint16_t* s_tile, const uint16_t* b_tile, int G,
                                               int g0, int g1, float2* table) {
    const int lane = threadIdx.x & 31;
    const int cnt = (g1 - g0) * 8;
    for (int e = lane; e < cnt; e += 32) {
        const int gg = g0 + (e >> 3), n = e & 7;
        const float s = bf16_bits_to_f32(s_tile[n * G + gg]);
        const float b = bf16_bits_to_f32(b_tile[n * G + gg]);
        const float s16 = s * 16.0f;
        table[gg * 8 + n] = make_float2(s16, b - s16);
    }
}

// acc[nb][mt][0..3]: rows (mt*16+g, mt*16+g+8) x weight rows (2t, 2t+1) of tile nb.
// Groups [g0, g1) of the weights; the staged activation chunk starts at group gx0.
template <int NB, int MT, bool HALF>
__device__ __forceinline__ void mma_groups(const uint8_t* const (&wt)[NB], int RS,
                                           const float2* const (&sbt)[NB], const uint8_t* xp, int XRS,
                                           const float* xs, int GC, int M_eff, int g0, int g1, int gx0,
                                           float (&acc)[NB][MT][4]) {
    const int lane = threadIdx.x & 31, g = lane >> 2, t = lane & 3;
#pragma unroll 1
    for (int gg = g0; gg < g1; ++gg) {
        const int gl = gg - gx0;
        uint32_t A[MT][2][8];
        float X[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int r = mt * 16 + h * 8 + g;
                if ((HALF && h == 1) || r >= M_eff) {
#pragma unroll
                    for (int j = 0; j < 8; ++j) A[mt][h][j] = 0u;
                    X[mt][h] = 0.f;
                } else {
                    const uint8_t* p = xp + (uint32_t)r * XRS + gl * 128 + t * 32;
                    const uint4 lo = lds128(p), hi = lds128(p + 16);
                    A[mt][h][0] = lo.x; A[mt][h][1] = lo.y; A[mt][h][2] = lo.z; A[mt][h][3] = lo.w;
                    A[mt][h][4] = hi.x; A[mt][h][5] = hi.y; A[mt][h][6] = hi.z; A[mt][h][7] = hi.w;
                    X[mt][h] = xs[r * GC + gl];
                }
            }
        }
#pragma unroll
        for (int nb = 0; nb < NB; ++nb) {
            const uint2 wv = lds64(wt[nb] + g * RS + gg * 32 + t * 8);
            uint32_t p0[4], p1[4];
            q4_pairs(wv.x, p0);
            q4_pairs(wv.y, p1);
            const float4 sb = *reinterpret_cast<const float4*>(sbt[nb] + gg * 8 + 2 * t);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                float d[4] = {0.f, 0.f, 0.f, 0.f};
                mma_bf16_16816(d, A[mt][0][0], A[mt][1][0], A[mt][0][1], A[mt][1][1], p0[0], p0[1]);
                mma_bf16_16816(d, A[mt][0][2], A[mt][1][2], A[mt][0][3], A[mt][1][3], p0[2], p0[3]);
                mma_bf16_16816(d, A[mt][0][4], A[mt][1][4], A[mt][0][5], A[mt][1][5], p1[0], p1[1]);
                mma_bf16_16816(d, A[mt][0][6], A[mt][1][6], A[mt][0][7], A[mt][1][7], p1[2], p1[3]);
                acc[nb][mt][0] = fmaf(sb.x, d[0], fmaf(sb.y, X[mt][0], acc[nb][mt][0]));
                acc[nb][mt][1] = fmaf(sb.z, d[1], fmaf(sb.w, X[mt][0], acc[nb][mt][1]));
                if (!HALF) {
                    acc[nb][mt][2] = fmaf(sb.x, d[2], fmaf(sb.y, X[mt][1], acc[nb][mt][2]));
                    acc[nb][mt][3] = fmaf(sb.z, d[3], fmaf(sb.w, X[mt][1], acc[nb][mt][3]));
                }
            }
        }
    }
}

// Issue the TMA copies of one 8-row weight tile (rows [row0, row0+8) of W) into `tile`.
// Returns the byte count (for expect_tx).  Scales/biases of a partial tile are not copied here.
__device__ __forceinline__ uint32_t tile_bytes_expected(const Q4Mat& W, int64_t row0) {
    const int64_t rows = (int64_t)min((long long)8, max((long long)0, (long long)(W.n - row0)));
    const int G = (int)(W.k / kGroup);
    uint32_t bytes = (uint32_t)(rows * (W.k / 2));
    if (rows == 8) bytes += 2u * 8u * G * 2u;
    return bytes;
}
__device__ __forceinline__ void issue_tile(const Q4Mat& W, int64_t row0, uint8_t* tile, int RS, uint64_t* bar) {
    const int64_t rows = (int64_t)min((long long)8, max((long long)0, (long long)(W.n - row0)));
    const int G = (int)(W.k / kGroup);
    const uint32_t rb = (uint32_t)(W.k / 2);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(W.w) + row0 * (int64_t)rb;
    for (int r = 0; r < rows; ++r) tma_bulk_g2s(tile + r * RS, src + (int64_t)r * rb, rb, bar);
    if (rows == 8) {
        uint8_t* sdst = tile + 8 * RS;
        tma_bulk_g2s(sdst, W.s + row0 * G, 8u * G * 2u, bar);
        tma_bulk_g2s(sdst + 8 * G * 2, W.b + row0 * G, 8u * G * 2u, bar);
    }
}
// Scales/biases of a partial tile, loaded by one warp with plain loads.
__device__ __forceinline__ void load_partial_scales(const Q4Mat& W, int64_t row0, uint8_t* tile, int RS) {
    const int64_t rows = (int64_t)min((long long)8, max((long long)0, (long long)(W.n - row0)));
    if (rows == 8) return;
    const int G = (int)(W.k / kGroup);
    uint16_t* sd = reinterpret_cast<uint16_t*>(tile + 8 * RS);
    uint16_t* bd = sd + 8 * G;
    for (int e = threadIdx.x & 31; e < 8 * G; e += 32) {
        const int r = e / G;
        const bool ok = r < rows;
        sd[e] = ok ? W.s[row0 * G + e] : (uint16_t)0;
        bd[e] = ok ? W.b[row0 * G + e] : (uint16_t)0;
    }
}

// ------------------------------------------------------------------------------------------------
// unit kernel: one CTA = NWR warp rows x NB tiles x 8 weight rows, K split over NWK warps
// ------------------------------------------------------------------------------------------------
struct UnitArgs {
    GemvLaunch L;
    int P, M_eff, G, NWR, NWK, GC, RS, XRS;
    uint32_t tbytes, off_tiles, off_sb, off_xp, off_xs, off_red, off_scr, off_bar;
};

__device__ __forceinline__ float swiglu_apply(float gv, float uv, int dtype) {
    if (dtype == kBF16) {
        const float gq = bf16_round(gv), uq = bf16_round(uv);
        const float sg = bf16_round(__fdividef(1.0f, 1.0f + expf(-gq)));
        const float tt = bf16_round(sg * gq);
        return bf16_round(tt * uq);
    }
    const float sg = 1.0f / (1.0f + expf(-gv));
    return (sg * gv) * uv;
}

template <int NB, int MT, bool HALF, int EPI>
__global__ void __launch_bounds__(kMaxThreads) q4_unit_kernel(const __grid_constant__ UnitArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int NWR = a.NWR, NWK = a.NWK, G = a.G;
    const int wr = warp % NWR, wk = warp / NWR;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    uint8_t* tiles = smem + a.off_tiles;
    float2* sbt_all = reinterpret_cast<float2*>(smem + a.off_sb);
    float* red = reinterpret_cast<float*>(smem + a.off_red);
    XGeom xg{smem + a.off_xp, reinterpret_cast<float*>(smem + a.off_xs),
             reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
             (int)L.m, a.P, a.M_eff, a.XRS, a.GC};

    // weight rows of tile (r, nb)
    const int64_t unit_rows = (int64_t)NWR * 8 * (EPI == kEpiSwiglu ? 1 : NB);
    const int64_t base = (int64_t)blockIdx.x * unit_rows;
    auto tile_row0 = [&](int r, int nb) -> int64_t {
        return EPI == kEpiSwiglu ? base + r * 8 : base + (int64_t)(r * NB + nb) * 8;
    };
    auto tile_mat = [&](int nb) -> const Q4Mat& { return (EPI == kEpiSwiglu && nb == 1) ? L.w1 : L.w0; };

    if (tid == 0) {
        mbar_init(bar, 1);
        fence_mbar_init();
        uint32_t bytes = 0;
        for (int r = 0; r < NWR; ++r)
            for (int nb = 0; nb < NB; ++nb) bytes += tile_bytes_expected(tile_mat(nb), tile_row0(r, nb));
        mbar_arrive_expect_tx(bar, bytes);
        for (int r = 0; r < NWR; ++r)
            for (int nb = 0; nb < NB; ++nb)
                issue_tile(tile_mat(nb), tile_row0(r, nb), tiles + (r * NB + nb) * a.tbytes, a.RS, bar);
    }
    // Everything above is independent of the previous kernel; activations below are not.
    pdl_wait();
    pdl_launch_dependents();

    if (L.norm_w) compute_norm_factors(L.x, L.x_dtype, (int)L.m, (int)L.w0.k, L.eps, xg);

    // this warp's tiles and group range
    const int g0 = wk * G / NWK, g1 = (wk + 1) * G / NWK;
    const uint8_t* wt[NB];
    const float2* sbt[NB];
    float2* sbt_w[NB];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb) {
        uint8_t* tb = tiles + (wr * NB + nb) * a.tbytes;
        wt[nb] = tb;
        sbt_w[nb] = sbt_all + (size_t)(wr * NB + nb) * G * 8;
        sbt[nb] = sbt_w[nb];
    }
    float acc[NB][MT][4];
#pragma unroll
    for (int nb = 0; nb < NB; ++nb)
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[nb][mt][j] = 0.f;

    bool weights_ready = false;
    for (int gc0 = 0; gc0 < G; gc0 += a.GC) {
        const int ngc = min(a.GC, G - gc0);
        stage_x_chunk(L.x, L.x_dtype, (int)L.w0.k, L.norm_w, gc0, ngc, xg);
        if (!weights_ready) {
            // uniform across the CTA: a timeout (recorded on the device) ends the whole CTA
            if (!__syncthreads_and(mbar_wait(bar, 0) ? 1 : 0)) return;
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                if (wk == 0) load_partial_scales(tile_mat(nb), tile_row0(wr, nb), const_cast<uint8_t*>(wt[nb]), a.RS);
            }
            __syncthreads();
#pragma unroll
            for (int nb = 0; nb < NB; ++nb) {
                const uint16_t* st = reinterpret_cast<const uint16_t*>(wt[nb] + 8 * a.RS);
                build_sb_table(st, st + 8 * G, G, g0, g1, sbt_w[nb]);
            }
            __syncwarp();
            weights_ready = true;
        }
        const int lo = max(g0, gc0), hi = min(g1, gc0 + ngc);
        if (lo < hi) mma_groups<NB, MT, HALF>(wt, a.RS, sbt, xg.xp, a.XRS, xg.xs, a.GC, a.M_eff, lo, hi, gc0, acc);
        __syncthreads();  // chunk buffer reuse
    }

    // partials -> shared memory: red[((wk*NWR + wr)*NB + nb)*M_eff*8 + r*8 + n]
    {
        const int g = lane >> 2, t = lane & 3;
#pragma unroll
        for (int nb = 0; nb < NB; ++nb)
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < (HALF ? 1 : 2); ++h) {
                    const int r = mt * 16 + h * 8 + g;
                    if (r < a.M_eff) {
                        float* dst = red + ((size_t)((wk * NWR + wr) * NB + nb) * a.M_eff + r) * 8 + 2 * t;
                        *reinterpret_cast<float2*>(dst) = make_float2(acc[nb][mt][2 * h], acc[nb][mt][2 * h + 1]);
                    }
                }
    }
    __syncthreads();

    // epilogue
    const int M = (int)L.m, P = a.P;
    const int NBO = EPI == kEpiSwiglu ? 1 : NB;
    const int total = NWR * NBO * M * 8;
    auto gather = [&](int r_, int nb, int m, int n) -> float {
        float v = 0.f;
        for (int w = 0; w < NWK; ++w)
            for (int p = 0; p < P; ++p)
                v += red[((size_t)((w * NWR + r_) * NB + nb) * a.M_eff + (p * M + m)) * 8 + n];
        return v;
    };
    for (int o = tid; o < total; o += blockDim.x) {
        const int n = o & 7;
        int rest = o >> 3;
        const int m = rest % M;
        rest /= M;
        const int nbo = rest % NBO, r_ = rest / NBO;
        const int64_t row = tile_row0(r_, nbo) + n;
        if (row >= L.w0.n) continue;
        const int64_t yi = (int64_t)m * L.ldy + row;
        float v;
        if (EPI == kEpiSwiglu) {
            v = swiglu_apply(gather(r_, 0, m, n), gather(r_, 1, m, n), L.y_dtype);
        } else {
            v = gather(r_, nbo, m, n);
            if (EPI == kEpiResid) v = load_act(L.resid, L.resid_dtype, (int64_t)m * L.ldr + row) + v;
        }
        if (L.y_dtype == kBF16)
            static_cast<uint16_t*>(L.y)[yi] = (uint16_t)f32_to_bf16_bits(v);
        else
            static_cast<float*>(L.y)[yi] = v;
    }
}

// ------------------------------------------------------------------------------------------------
// lm_head + argmax: persistent CTAs, per-warp TMA ring over 8-row vocabulary tiles
// ------------------------------------------------------------------------------------------------
struct LmArgs {
    LmHeadLaunch L;
    int P, M_eff, G, RS, XRS, D, nwarps;
    int64_t ntiles;
    uint32_t tbytes, off_ring, off_sb, off_xp, off_xs, off_scr, off_bar, off_out, off_keys;
};

__device__ __forceinline__ unsigned long long pack_key(float v, int64_t idx) {
    uint32_t u = __float_as_uint(v);
    uint32_t o = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
    return ((unsigned long long)o << 32) | (unsigned long long)(0xffffffffu - (uint32_t)idx);
}
__device__ __forceinline__ void unpack_key(unsigned long long k, int32_t* id, float* v) {
    uint32_t o = (uint32_t)(k >> 32);
    uint32_t u = (o & 0x80000000u) ? (o & 0x7fffffffu) : ~o;
    *v = __uint_as_float(u);
    *id = (int32_t)(0xffffffffu - (uint32_t)(k & 0xffffffffu));
}

template <int MT, bool HALF>
__global__ void __launch_bounds__(kMaxThreads) q4_lm_head_kernel(const __grid_constant__ LmArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    const LmHeadLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int D = a.D, G = a.G;
    const int64_t TW = (int64_t)gridDim.x * a.nwarps;
    const int64_t gw = (int64_t)blockIdx.x * a.nwarps + warp;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + a.off_bar) + warp * D;
    uint8_t* ring = smem + a.off_ring + (size_t)warp * D * a.tbytes;
    float2* table = reinterpret_cast<float2*>(smem + a.off_sb) + (size_t)warp * G * 8;
    float* wout = reinterpret_cast<float*>(smem + a.off_out) + (size_t)warp * a.M_eff * 8;
    unsigned long long* ckeys = reinterpret_cast<unsigned long long*>(smem + a.off_keys);
    XGeom xg{smem + a.off_xp, reinterpret_cast<float*>(smem + a.off_xs),
             reinterpret_cast<float*>(smem + a.off_scr), reinterpret_cast<float*>(smem + a.off_scr) + 64,
             (int)L.m, a.P, a.M_eff, a.XRS, G};

    if (lane == 0) {
        for (int s = 0; s < D; ++s) mbar_init(&bars[s], 1);
        fence_mbar_init();
        for (int s = 0; s < D; ++s) {
            const int64_t tile = gw + (int64_t)s * TW;
            if (tile < a.ntiles) {
                mbar_arrive_expect_tx(&bars[s], tile_bytes_expected(L.w, tile * 8));
                issue_tile(L.w, tile * 8, ring + (size_t)s * a.tbytes, a.RS, &bars[s]);
            }
        }
    }
    pdl_wait();
    pdl_launch_dependents();
    if (L.norm_w) compute_norm_factors(L.x, L.x_dtype, (int)L.m, (int)L.w.k, L.eps, xg);
    stage_x_chunk(L.x, L.x_dtype, (int)L.w.k, L.norm_w, 0, G, xg);

    const int M = (int)L.m, P = a.P;
    // lane owns output column n = lane & 7 and rows m = (lane >> 3) + 4j
    constexpr int kSlots = 8;  // M <= 32
    unsigned long long best[kSlots];
#pragma unroll
    for (int j = 0; j < kSlots; ++j) best[j] = 0ull;

    bool ok = true;
    for (int64_t i = 0;; ++i) {
        const int64_t tile = gw + i * TW;
        if (tile >= a.ntiles) break;
        const int s = (int)(i % D);
        const uint32_t parity = (uint32_t)((i / D) & 1);
        uint8_t* st = ring + (size_t)s * a.tbytes;
        // warp-uniform: on a (recorded) timeout the warp stops streaming
        if (!__all_sync(0xffffffffu, mbar_wait(&bars[s], parity) ? 1 : 0)) { ok = false; break; }
        load_partial_scales(L.w, tile * 8, st, a.RS);
        __syncwarp();
        {
            const uint16_t* sp = reinterpret_cast<const uint16_t*>(st + 8 * a.RS);
            build_sb_table(sp, sp + 8 * G, G, 0, G, table);
        }
        __syncwarp();
        float acc[1][MT][4];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt)
#pragma unroll
            for (int j = 0; j < 4; ++j) acc[0][mt][j] = 0.f;
        const uint8_t* wt[1] = {st};
        const float2* sbt[1] = {table};
        mma_groups<1, MT, HALF>(wt, a.RS, sbt, xg.xp, a.XRS, xg.xs, G, a.M_eff, 0, G, 0, acc);
        __syncwarp();
        if (lane == 0) {
            const int64_t nt = tile + (int64_t)D * TW;
            if (nt < a.ntiles) {
                mbar_arrive_expect_tx(&bars[s], tile_bytes_expected(L.w, nt * 8));
                issue_tile(L.w, nt * 8, st, a.RS, &bars[s]);
            }
        }
        {
            const int g = lane >> 2, t = lane & 3;
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int h = 0; h < (HALF ? 1 : 2); ++h) {
                    const int r = mt * 16 + h * 8 + g;
                    if (r < a.M_eff)
                        *reinterpret_cast<float2*>(wout + r * 8 + 2 * t) =
                            make_float2(acc[0][mt][2 * h], acc[0][mt][2 * h + 1]);
                }
        }
        __syncwarp();
        {
            const int n = lane & 7;
            const int64_t row = tile * 8 + n;
            if (row < L.w.n) {
#pragma unroll
                for (int j = 0; j < kSlots; ++j) {
                    const int m = (lane >> 3) + 4 * j;
                    if (m < M) {
                        float v = 0.f;
                        for (int p = 0; p < P; ++p) v += wout[(p * M + m) * 8 + n];
                        if (L.x_dtype == kBF16 && !L.norm_w) v = bf16_round(v);
                        const unsigned long long k = pack_key(v, L.vocab_offset + row);
                        best[j] = k > best[j] ? k : best[j];
                    }
                }
            }
        }
        __syncwarp();
    }
    (void)ok;
    // reduce over the 8 lanes sharing m, then over warps, then across CTAs
#pragma unroll
    for (int j = 0; j < kSlots; ++j) {
#pragma unroll
        for (int o = 1; o < 8; o <<= 1) {
            unsigned long long other = __shfl_xor_sync(0xffffffffu, best[j], o);
            best[j] = other > best[j] ? other : best[j];
        }
    }
    if ((lane & 7) == 0) {
#pragma unroll
        for (int j = 0; j < kSlots; ++j) {
            const int m = (lane >> 3) + 4 * j;
            if (m < M) ckeys[warp * M + m] = best[j];
        }
    }
    __syncthreads();
    __shared__ bool is_last;
    if (tid < M) {
        unsigned long long k = 0ull;
        for (int w = 0; w < a.nwarps; ++w) k = ckeys[w * M + tid] > k ? ckeys[w * M + tid] : k;
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
        if (tid < M) {
            const unsigned long long k = atomicExch(&L.keys[tid], 0ull);
            if (L.keys_out) L.keys_out[tid] = k;
            int32_t id;
            float v;
            unpack_key(k, &id, &v);
            if (L.ids) L.ids[tid] = id;
            if (L.best) L.best[tid] = v;
        }
        if (tid == 0) atomicExch(L.counter, 0u);
    }
}

__global__ void decode_keys_kernel(const unsigned long long* keys, int64_t m, int32_t* ids, float* best) {
    const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (i < m) {
        int32_t id;
        float v;
        unpack_key(keys[i], &id, &v);
        if (ids) ids[i] = id;
        if (best) best[i] = v;
    }
}

// ------------------------------------------------------------------------------------------------
// host side
// ------------------------------------------------------------------------------------------------
int num_sms() {
    static int n = 0;
    if (!n) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        if (n <= 0) n = 148;
    }
    return n;
}

constexpr uint32_t kSmemLimit = 226 * 1024;  // dynamic; leaves room for static shared memory

template <typename KernelT, typename ArgT>
cudaError_t launch_kernel(KernelT kernel, const ArgT& args, int grid, int threads, uint32_t smem, bool pdl,
                          cudaStream_t stream) {
    cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(threads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kernel, args);
}

template <int NB, int EPI>
cudaError_t dispatch_unit(const UnitArgs& a, int grid, int threads, uint32_t smem, bool pdl, cudaStream_t st) {
    if (a.M_eff <= 8) return launch_kernel(q4_unit_kernel<NB, 1, true, EPI>, a, grid, threads, smem, pdl, st);
    if (a.M_eff <= 16) return launch_kernel(q4_unit_kernel<NB, 1, false, EPI>, a, grid, threads, smem, pdl, st);
    return launch_kernel(q4_unit_kernel<NB, 2, false, EPI>, a, grid, threads, smem, pdl, st);
}

}  // namespace

int gemv_max_rows(int act_dtype) { return act_dtype == kBF16 ? 32 : 10; }

cudaError_t launch_q4_gemv(const GemvLaunch& L, cudaStream_t stream) {
    UnitArgs a{};
    a.L = L;
    const int K = (int)L.w0.k;
    a.G = K / kGroup;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.M_eff = (int)L.m * a.P;
    const int epi = L.epi;
    int NB, NWR;
    if (epi == kEpiSwiglu) {
        NB = 2;
        NWR = 2;
    } else {
        NB = (L.w0.n >= 2LL * 16 * num_sms()) ? 2 : 1;
        NWR = 1;
    }
    int NWK = std::max(1, std::min(epi == kEpiSwiglu ? 4 : 8, a.G / 8));
    a.NWR = NWR;
    a.NWK = NWK;
    a.RS = packed_row_stride(K);
    a.tbytes = tile_bytes(K);
    const uint32_t ntiles = NWR * NB;
    // shared-memory budget: weights + scale tables + reduction fixed, activation chunk takes the rest
    uint32_t off = 0;
    a.off_bar = off;
    off += 128;
    a.off_scr = off;
    off += align_up((64 + (uint32_t)L.m) * 4, 128);
    a.off_tiles = off;
    off += ntiles * a.tbytes;
    a.off_sb = off;
    off += align_up(ntiles * a.G * 8 * 8, 128);
    a.off_red = off;
    off += align_up((uint32_t)NWK * ntiles * a.M_eff * 8 * 4, 128);
    const uint32_t fixed = off;
    const uint32_t budget = std::min<uint32_t>(kSmemLimit, std::max<uint32_t>(fixed + 16384, 110 * 1024));
    const uint32_t per_group = (uint32_t)a.M_eff * (128 + 4);
    int GC = (int)((budget - fixed - (uint32_t)a.M_eff * 16 - 256) / per_group);
    GC = std::max(1, std::min(GC, a.G));
    a.GC = GC;
    a.XRS = GC * 128 + 16;
    a.off_xp = off;
    off += align_up((uint32_t)a.M_eff * a.XRS, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.M_eff * GC * 4, 128);
    const uint32_t smem = off;
    if (smem > kSmemLimit) return cudaErrorInvalidConfiguration;
    const int64_t unit_rows = (int64_t)NWR * 8 * (epi == kEpiSwiglu ? 1 : NB);
    const int grid = (int)((L.w0.n + unit_rows - 1) / unit_rows);
    if (grid <= 0) return cudaSuccess;
    const int threads = 32 * NWR * NWK;
    if (epi == kEpiSwiglu) return dispatch_unit<2, kEpiSwiglu>(a, grid, threads, smem, L.pdl, stream);
    if (epi == kEpiResid) {
        return NB == 2 ? dispatch_unit<2, kEpiResid>(a, grid, threads, smem, L.pdl, stream)
                       : dispatch_unit<1, kEpiResid>(a, grid, threads, smem, L.pdl, stream);
    }
    return NB == 2 ? dispatch_unit<2, kEpiStore>(a, grid, threads, smem, L.pdl, stream)
                   : dispatch_unit<1, kEpiStore>(a, grid, threads, smem, L.pdl, stream);
}

cudaError_t launch_q4_lm_head_argmax(const LmHeadLaunch& L, cudaStream_t stream) {
    LmArgs a{};
    a.L = L;
    const int K = (int)L.w.k;
    a.G = K / kGroup;
    a.P = (L.norm_w || L.x_dtype == kF32) ? 3 : 1;
    a.M_eff = (int)L.m * a.P;
    a.RS = packed_row_stride(K);
    a.tbytes = tile_bytes(K);
    a.XRS = a.G * 128 + 16;
    a.ntiles = (L.w.n + 7) / 8;
    const int nwarps = 8;
    a.nwarps = nwarps;
    uint32_t off = 0;
    a.off_bar = off;
    off += align_up(nwarps * 4 * 8, 128);
    a.off_scr = off;
    off += align_up((64 + (uint32_t)L.m) * 4, 128);
    a.off_keys = off;
    off += align_up(nwarps * (uint32_t)L.m * 8, 128);
    a.off_out = off;
    off += align_up(nwarps * (uint32_t)a.M_eff * 8 * 4, 128);
    a.off_sb = off;
    off += align_up(nwarps * (uint32_t)a.G * 8 * 8, 128);
    a.off_xp = off;
    off += align_up((uint32_t)a.M_eff * a.XRS, 128);
    a.off_xs = off;
    off += align_up((uint32_t)a.M_eff * a.G * 4, 128);
    a.off_ring = off;
    const uint32_t avail = kSmemLimit > off ? kSmemLimit - off : 0;
    int D = (int)(avail / (nwarps * a.tbytes));
    D = std::min(D, 4);
    if (D < 1) return cudaErrorInvalidConfiguration;
    a.D = D;
    off += (uint32_t)nwarps * D * a.tbytes;
    const uint32_t smem = off;
    const int64_t want = (a.ntiles + nwarps - 1) / nwarps;
    const int grid = (int)std::max<int64_t>(1, std::min<int64_t>(num_sms(), want));
    const int threads = 32 * nwarps;
    if (a.M_eff <= 8) return launch_kernel(q4_lm_head_kernel<1, true>, a, grid, threads, smem, L.pdl, stream);
    if (a.M_eff <= 16) return launch_kernel(q4_lm_head_kernel<1, false>, a, grid, threads, smem, L.pdl, stream);
    return launch_kernel(q4_lm_head_kernel<2, false>, a, grid, threads, smem, L.pdl, stream);
}

int gemv_device_error(bool clear) {
    int v = 0;
    if (cudaMemcpyFromSymbol(&v, g_marlin_device_error, sizeof(int)) != cudaSuccess) return -1;
    if (clear) {
        const int zero = 0;
        if (cudaMemcpyToSymbol(g_marlin_device_error, &zero, sizeof(int)) != cudaSuccess) return -1;
    }
    return v;
}

cudaError_t launch_decode_keys(const unsigned long long* keys, int64_t m, int32_t* ids, float* best,
                               cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    decode_keys_kernel<<<(unsigned)((m + 127) / 128), 128, 0, stream>>>(keys, m, ids, best);
    return cudaGetLastError();
}

}  // namespace marlin
