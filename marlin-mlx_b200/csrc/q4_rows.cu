// q4_rows.cu — whole-row Q4 GEMV for decode-sized activations (m <= 2), one launch (sm_100a).
//
// Replaces mx::quantized_matmul(x, w, scales, biases, transpose=true, 64, 4) for one or two
// activation rows (src/model/marlin.cpp:18-25), the single-op decode GEMV of config C1.
//
// Each CTA owns 16 T output rows over the whole K: every weight byte it needs (T x 16 rows x K/2
// bytes plus scales and biases, at most about 150 KB) is requested by TMA at kernel start, before the
// programmatic-dependent-launch wait, so it streams while the previous kernel finishes.  After the
// wait the activation row is split into exact s8 planes with one exponent per 64-group (8-lane
// shuffles, no block reduction), and 4 T consumer warps (tile t, K quarter k) run the integer-MMA
// group step of q4_i8_common.cuh over their quarter of the resident stages; the four quarters meet
// in shared memory in a fixed order.  No cluster, no cross-CTA reduction, no ring reuse.
#include "common.cuh"
#include "q4_gemv.cuh"
#include "q4_host.cuh"
#include "q4_i8.cuh"
#include "q4_i8_common.cuh"
#include "q4_stage.cuh"

#include <algorithm>

#ifndef ROWS_GEMV_MAX_K
#define ROWS_GEMV_MAX_K 16384
#endif

namespace marlin {
namespace {

constexpr int kRowsKParts = 4;  // consumer warps per 16-row tile (K quarters)
constexpr uint32_t kRowsSmemLimit = 225 * 1024;

struct RowsArgs {
    CUtensorMap tw, ts, tb;  // boxes of 16 T rows
    GemvLaunch L;
    int G, NS;               // 64-groups and 4-group stages of K
    uint32_t stage_stride;   // bytes per stage (packed [R][128], scales [R][16], biases [R][16]; 1024-aligned)
    uint32_t off_bar, off_misc, off_xq, off_xs, off_xe, off_cs, off_red, off_stages;
};

__host__ __device__ constexpr int rows_threads(int T) { return (kRowsKParts * T + 1) * 32; }

template <int T>
__global__ void __launch_bounds__(rows_threads(T), 1) rows_gemv_kernel(const __grid_constant__ RowsArgs a) {
    constexpr int R = 16 * T, W = kRowsKParts * T, ncols = 8;
    extern __shared__ __align__(1024) uint8_t smem_raw[];
    uint8_t* smem = align_smem_1024(smem_raw);
    const GemvLaunch& L = a.L;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int M = (int)L.m, K = (int)L.w0.k, G = a.G, NS = a.NS;
    const int64_t row0 = (int64_t)blockIdx.x * R;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + a.off_bar);
    volatile int* abort = reinterpret_cast<volatile int*>(smem + a.off_misc);
    uint8_t* xq = smem + a.off_xq;
    float* xs = reinterpret_cast<float*>(smem + a.off_xs);
    float* xe = reinterpret_cast<float*>(smem + a.off_xe);
    float* cs = reinterpret_cast<float*>(smem + a.off_cs);
    float* red = reinterpret_cast<float*>(smem + a.off_red);  // [4][R][2]
    uint8_t* stages = smem + a.off_stages;

    if (tid == 0) {
        *abort = 0;
        for (int s = 0; s < NS; ++s) mbar_init(&full[s], 1);
        fence_mbar_init();
    }
    __syncthreads();
    if (warp == W) {
        // every weight byte of this CTA, requested before the dependency wait
        pdl_launch_dependents();
        if (lane == 0) {
            prefetch_tmap(&a.tw);
            for (int s = 0; s < NS; ++s) {
                uint8_t* st = stages + (size_t)s * a.stage_stride;
                mbar_arrive_expect_tx(&full[s], (uint32_t)R * 160u);
                tma_load_2d(st, &a.tw, 4 * s * 8, (int32_t)row0, &full[s]);
                tma_load_2d(st + R * 128, &a.ts, (4 * s) & ~7, (int32_t)row0, &full[s]);
                tma_load_2d(st + R * 144, &a.tb, (4 * s) & ~7, (int32_t)row0, &full[s]);
            }
        }
        __syncwarp();
    } else {
        pdl_wait();
        pdl_launch_dependents();
        // operand: exact s8 planes of the rows, one exponent per 64-group
        for (int i = tid; i < G * ncols; i += W * 32) xs[i] = xe[i] = 0.f;
        for (int i = tid; i < G * ncols * 4; i += W * 32) reinterpret_cast<uint4*>(xq)[i] = make_uint4(0, 0, 0, 0);
        if (tid < ncols) cs[tid] = (tid >> 2) < M ? pow2f(-10 - 7 * (tid & 3)) : 0.f;
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        const int units = M * (K / 8);
        for (int base = 0; base < units; base += W * 32) {  // whole warps (units of a group in 8 lanes)
            const int u = base + tid;
            const bool live = u < units;
            float v[8];
            int m = 0, ku = 0;
            if (live) {
                m = u / (K / 8);
                ku = u - m * (K / 8);
                load8(L.x, L.x_dtype, (int64_t)m * K + 8 * ku, v);
            } else {
#pragma unroll
                for (int j = 0; j < 8; ++j) v[j] = 0.f;
            }
            float amx = 0.f, sm = 0.f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                amx = fmaxf(amx, fabsf(v[j]));
                sm = __fadd_rn(sm, v[j]);
            }
            unsigned bits = __float_as_uint(amx);
#pragma unroll
            for (int o = 1; o < 8; o <<= 1) {
                bits = max(bits, __shfl_xor_sync(0xffffffffu, bits, o));
                sm += __shfl_xor_sync(0xffffffffu, sm, o);
            }
            if (live) {
                const int e = row_exp(bits), grp = ku >> 3, u8 = ku & 7;
                uint32_t b[4][2];
                planes8(v, e, b);
#pragma unroll
                for (int p = 0; p < 4; ++p)
                    *reinterpret_cast<uint2*>(xq + ((size_t)(grp * ncols + 4 * m + p) * 64 + 8 * u8)) =
                        make_uint2(b[p][0], b[p][1]);
                if (u8 == 0) {
                    xs[grp * ncols + 4 * m] = __fmul_rn(sm, 64.0f);
                    xe[grp * ncols + 4 * m] = pow2f(e);
                }
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");

        // tile t, K quarter k: stages [k NS/4, (k+1) NS/4)
        const int t = warp % T, k = warp / T;
        const int g = lane >> 2, tq = lane & 3;
        const I8X tx{xq, xs, cs, nullptr, nullptr, nullptr, xe};
        float y[1][4] = {{0.f, 0.f, 0.f, 0.f}}, yb[1][2] = {{0.f, 0.f}};
        const int s0 = k * (NS / kRowsKParts), s1 = s0 + NS / kRowsKParts;
        for (int s = s0; s < s1; ++s) {
            if (!warp_wait(&full[s], 0u, abort)) break;
            i8_stage<1, R>(stages + (size_t)s * a.stage_stride, ((4 * s) & 7) * 2, 4 * s, tx, t, lane, y, yb);
        }
        {
            const float2 cv = *reinterpret_cast<const float2*>(cs + 2 * tq);
            const float2 pp = i8_combine(y[0], yb[0], cv, tq);
            const int m = tq >> 1, r0 = 16 * t + g;
            if ((tq & 1) == 0 && m < M) {
                red[(k * R + r0) * 2 + m] = pp.x;
                red[(k * R + r0 + 8) * 2 + m] = pp.y;
            }
        }
        asm volatile("bar.sync 1, %0;" ::"r"(W * 32) : "memory");
        for (int i = tid; i < R * M; i += W * 32) {
            const int r = i / M, m = i - r * M;
            const int64_t row = row0 + r;
            if (row < L.w0.n) {
                float o = 0.f;
                for (int kk = 0; kk < kRowsKParts; ++kk) o += red[(kk * R + r) * 2 + m];
                if (L.y_dtype == kBF16)
                    static_cast<uint16_t*>(L.y)[(int64_t)m * L.ldy + row] = (uint16_t)f32_to_bf16_bits(o);
                else
                    static_cast<float*>(L.y)[(int64_t)m * L.ldy + row] = o;
            }
        }
    }
    // every stage has landed before the CTA may leave (a consumer may have given up on one)
    __syncthreads();
    if (tid == 0)
        for (int s = 0; s < NS; ++s) drain_wait(&full[s], 0u);
}

// tiles per CTA: about one CTA per SM
int rows_tiles(int64_t n) {
    const int64_t per = (n + 16 * (int64_t)device_num_sms() - 1) / (16 * (int64_t)device_num_sms());
    return (int)std::max<int64_t>(1, std::min<int64_t>(6, per));
}

uint32_t plan_rows(RowsArgs& a, int T, int K) {
    const int R = 16 * T, ncols = 8;
    a.G = K / kGroup;
    a.NS = a.G / 4;
    a.stage_stride = align_up((uint32_t)R * 160u, 1024u);
    uint32_t off = 0;
    a.off_bar = off;
    off += align_up((uint32_t)a.NS * 8u, 128);
    a.off_misc = off;
    off += 128;
    a.off_xq = off;
    off += (uint32_t)a.G * ncols * 64;
    a.off_xs = off;
    off += align_up((uint32_t)a.G * ncols * 4, 128);
    a.off_xe = off;
    off += align_up((uint32_t)a.G * ncols * 4, 128);
    a.off_cs = off;
    off += 128;
    a.off_red = off;
    off += align_up((uint32_t)kRowsKParts * R * 2 * 4, 128);
    off = align_up(off, 1024);
    a.off_stages = off;
    off += (uint32_t)a.NS * a.stage_stride + 1024;
    return off <= kRowsSmemLimit ? off : 0;
}

}  // namespace

bool rows_gemv_applies(const GemvLaunch& L) {
    if (L.epi != kEpiStore || L.norm_w || L.has_xin || L.has_xout || L.tp.tp > 1) return false;
    if (L.m < 1 || L.m > 2 || L.w0.k % 1024 != 0 || L.w0.k > ROWS_GEMV_MAX_K) return false;
    if (L.x_dtype != kBF16 && L.x_dtype != kF32) return false;
    // two to six 16-row tiles per CTA in one wave: measured on B200 at one row, 6144x2048 takes
    // 5.0 us per back-to-back launch against 5.8 us on the cluster K-split kernel, but 2048x6144 (one
    // tile, four warps per CTA) 7.6 us against 6.1 us
    const int64_t sms = device_num_sms();
    if (L.w0.n <= 16 * sms || L.w0.n > 6 * 16 * sms) return false;
    RowsArgs a{};
    return plan_rows(a, rows_tiles(L.w0.n), (int)L.w0.k) != 0 && tmap_encode_fn() != nullptr;
}

cudaError_t launch_rows_gemv(const GemvLaunch& L, cudaStream_t stream) {
    RowsArgs a{};
    a.L = L;
    const int T = rows_tiles(L.w0.n);
    const uint32_t smem = plan_rows(a, T, (int)L.w0.k);
    if (!smem) return cudaErrorInvalidConfiguration;
    if (!encode_q4_maps(L.w0, 16 * T, &a.tw, &a.ts, &a.tb)) return cudaErrorInvalidValue;
    const int grid = (int)((L.w0.n + 16 * T - 1) / (16 * T));
    switch (T) {
        case 1: return launch_ex(rows_gemv_kernel<1>, a, grid, rows_threads(1), 1, smem, L.pdl, stream);
        case 2: return launch_ex(rows_gemv_kernel<2>, a, grid, rows_threads(2), 1, smem, L.pdl, stream);
        case 3: return launch_ex(rows_gemv_kernel<3>, a, grid, rows_threads(3), 1, smem, L.pdl, stream);
        case 4: return launch_ex(rows_gemv_kernel<4>, a, grid, rows_threads(4), 1, smem, L.pdl, stream);
        case 5: return launch_ex(rows_gemv_kernel<5>, a, grid, rows_threads(5), 1, smem, L.pdl, stream);
        default: return launch_ex(rows_gemv_kernel<6>, a, grid, rows_threads(6), 1, smem, L.pdl, stream);
    }
}

int rows_device_error(bool clear) { return tu_device_error(clear); }

}  // namespace marlin
