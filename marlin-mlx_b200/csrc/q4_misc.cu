// q4_misc.cu — Q4 quantize/pack, standalone RMSNorm, the Q4 embedding gather, and the seeded
// synthetic-input generator.
#include "common.cuh"
#include "q4_host.cuh"
#include "q4_misc.cuh"

#include <atomic>

namespace marlin {
namespace {

// ------------------------------------------------------------------------------------------------
// quantize: mx::quantize(w, group_size=64, bits=4) as called at src/model/weights.cpp:46 and :183.
// One warp covers 4 consecutive groups (groups are contiguous in row-major [n, k] since k % 64 == 0):
// 8 lanes per group, each lane loads 8 bf16 (16 B) and emits one packed u32 word.  Per group, in
// IEEE binary32 with no contraction:
//   max = max(0, w..), min = min(w..), s = max((max - min)/15, 1e-7)
//   side = |min| > |max|; s = side ? s : -s; edge = side ? min : max
//   q0 = round(edge/s); q0 != 0 ? (s = edge/q0, b = edge) : (b = 0)
//   q = min(max(round((w - b)/s), 0), 15);  round = ties away from zero
// scales/biases are stored as bf16 (round to nearest even).
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) quantize_kernel(const uint16_t* __restrict__ w, int64_t ngroups,
                                                       uint32_t* __restrict__ wq, uint16_t* __restrict__ scales,
                                                       uint16_t* __restrict__ biases) {
    const int lane = threadIdx.x & 31;
    const int64_t warp_global = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const int64_t gi = warp_global * 4 + (lane >> 3);
    const int j = lane & 7;
    const bool valid = gi < ngroups;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (valid) raw = __ldg(reinterpret_cast<const uint4*>(w + gi * 64 + j * 8));
    float v[8];
    const uint32_t rw[4] = {raw.x, raw.y, raw.z, raw.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
        v[2 * i] = bf16_bits_to_f32(rw[i] & 0xffffu);
        v[2 * i + 1] = bf16_bits_to_f32(rw[i] >> 16);
    }
    float wmin = INFINITY, wmax = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        wmin = fminf(wmin, v[i]);
        wmax = fmaxf(wmax, v[i]);
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) {
        wmin = fminf(wmin, __shfl_xor_sync(0xffffffffu, wmin, o));
        wmax = fmaxf(wmax, __shfl_xor_sync(0xffffffffu, wmax, o));
    }
    float scale = fmaxf(__fdiv_rn(__fsub_rn(wmax, wmin), 15.0f), 1e-7f);
    const bool side = fabsf(wmin) > fabsf(wmax);
    scale = side ? scale : -scale;
    const float edge = side ? wmin : wmax;
    const float q0 = roundf(__fdiv_rn(edge, scale));
    float bias = 0.0f;
    if (q0 != 0.0f) {
        scale = __fdiv_rn(edge, q0);
        bias = edge;
    }
    uint32_t word = 0;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        float c = roundf(__fdiv_rn(__fsub_rn(v[i], bias), scale));
        c = fminf(fmaxf(c, 0.0f), 15.0f);
        word |= (uint32_t)c << (4 * i);
    }
    if (valid) {
        wq[gi * 8 + j] = word;
        if (j == 0) {
            scales[gi] = (uint16_t)f32_to_bf16_bits(scale);
            biases[gi] = (uint16_t)f32_to_bf16_bits(bias);
        }
    }
}

// ------------------------------------------------------------------------------------------------
// RMSNorm (src/model/marlin.cpp:12-16) as MLX's C++ API evaluates it; one CTA per row.
// ------------------------------------------------------------------------------------------------
__global__ void __launch_bounds__(256) rms_norm_kernel(const void* __restrict__ x, int dtype,
                                                       const uint16_t* __restrict__ wn, int64_t H, float eps,
                                                       float* __restrict__ out) {
    __shared__ float scr[32];
    __shared__ float rf;
    const int64_t m = blockIdx.x;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    auto ld = [&](int64_t k) -> float {
        if (dtype == kDtypeBF16) return bf16_bits_to_f32(static_cast<const uint16_t*>(x)[m * H + k]);
        return static_cast<const float*>(x)[m * H + k];
    };
    float part = 0.f;
    for (int64_t k = tid; k < H; k += blockDim.x) {
        const float v = ld(k);
        float sq = __fmul_rn(v, v);
        if (dtype == kDtypeBF16) sq = bf16_round(sq);
        part = __fadd_rn(part, sq);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) part = __fadd_rn(part, __shfl_xor_sync(0xffffffffu, part, o));
    if (lane == 0) scr[warp] = part;
    __syncthreads();
    if (tid == 0) {
        float sum = 0.f;
        for (int w = 0; w < (int)(blockDim.x / 32); ++w) sum = __fadd_rn(sum, scr[w]);
        float var;
        if (dtype == kDtypeBF16)
            var = bf16_round(__fmul_rn(bf16_round(sum), bf16_round((float)(1.0 / (double)H))));
        else
            var = __fmul_rn(sum, (float)(1.0 / (double)H));
        rf = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(var, eps)));
    }
    __syncthreads();
    const float r = rf;
    for (int64_t k = tid; k < H; k += blockDim.x)
        out[m * H + k] = __fmul_rn(__fmul_rn(ld(k), r), __fadd_rn(1.0f, bf16_bits_to_f32(wn[k])));
}

// ------------------------------------------------------------------------------------------------
// Seeded generator: element i = bf16_rn(mean + sigma * (S - 393210)/65536), S = sum of twelve 16-bit
// lanes of three splitmix64 outputs.  Integer arithmetic plus one binary32 product and one sum
// (no contraction), so the host restatement reproduces it bit for bit.
// ------------------------------------------------------------------------------------------------
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z ^= z >> 30;
    z *= 0xbf58476d1ce4e5b9ull;
    z ^= z >> 27;
    z *= 0x94d049bb133111ebull;
    z ^= z >> 31;
    return z;
}

__global__ void synth_kernel(uint16_t* __restrict__ out, int64_t n, uint64_t seed, float mean, float sigma_scaled) {
    const uint64_t base = mix64(seed ^ 0x5851f42d4c957f2dull);
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        int64_t s = 0;
#pragma unroll
        for (uint64_t r = 0; r < 3; ++r) {
            const uint64_t h = mix64(base + (3ull * (uint64_t)i + r) * 0x9e3779b97f4a7c15ull);
            s += (int64_t)((h & 0xffffu) + ((h >> 16) & 0xffffu) + ((h >> 32) & 0xffffu) + (h >> 48));
        }
        const float z = (float)(s - 393210);
        const float v = __fadd_rn(__fmul_rn(z, sigma_scaled), mean);
        out[i] = (uint16_t)f32_to_bf16_bits(v);
    }
}

__global__ void residual_add_kernel(const void* __restrict__ h, int dtype, const float* __restrict__ y,
                                    int64_t n, float* __restrict__ out) {
    for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
        const float hv = dtype == kDtypeBF16 ? bf16_bits_to_f32(static_cast<const uint16_t*>(h)[i])
                                             : static_cast<const float*>(h)[i];
        out[i] = __fadd_rn(hv, y[i]);
    }
}

// out[i] = bf16(x[i]), round to nearest even: the activation dtype of a projection whose binary32
// partials were summed across GPUs (tensor-parallel down_proj of the prefill MLP).  Four elements
// per thread and step when both pointers allow 16 / 8-byte accesses.
__global__ void cast_bf16_kernel(const float* __restrict__ x, int64_t n, uint16_t* __restrict__ out, bool vec) {
    const int64_t stride = (int64_t)gridDim.x * blockDim.x;
    int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
    if (vec) {
        const int64_t n4 = n / 4;
        for (int64_t j = i; j < n4; j += stride) {
            const float4 v = reinterpret_cast<const float4*>(x)[j];
            reinterpret_cast<uint2*>(out)[j] = make_uint2(f32_to_bf16_bits(v.x) | (f32_to_bf16_bits(v.y) << 16),
                                                          f32_to_bf16_bits(v.z) | (f32_to_bf16_bits(v.w) << 16));
        }
        i += n4 * 4;  // the tail, one element per thread
    }
    for (; i < n; i += stride) out[i] = (uint16_t)f32_to_bf16_bits(x[i]);
}

// Rows `ids` of a Q4 table dequantized to bf16, out[i, :] = bf16(s q + b) per element with one
// rounding of the exact value (the operand the prefill GEMM builds): the embedding lookup
// MarlinModel::embed_tokens (src/model/marlin.cpp:63-65, mx::take of the embedding table) served
// from the tied, quantized lm_head instead of a separate bf16 table.  One CTA per row; each thread
// turns packed words into 16-byte row segments.  An id outside [0, n) writes a zero row and records
// kDevErrBadIndex.
__global__ void __launch_bounds__(256) embed_q4_kernel(const int32_t* __restrict__ ids, const uint32_t* __restrict__ wq,
                                                       const uint16_t* __restrict__ scales,
                                                       const uint16_t* __restrict__ biases, int64_t n, int64_t k,
                                                       uint16_t* __restrict__ out) {
    const int64_t i = blockIdx.x;
    const int32_t id = ids[i];
    const bool ok = id >= 0 && id < n;
    if (!ok && threadIdx.x == 0) record_device_error(kDevErrBadIndex);
    const int64_t words = k / 8, groups = k / 64;
    uint4* orow = reinterpret_cast<uint4*>(out + i * k);
    for (int64_t w = threadIdx.x; w < words; w += blockDim.x) {
        uint4 v = make_uint4(0u, 0u, 0u, 0u);
        if (ok) {
            const int64_t g = (int64_t)id * groups + w / 8;
            const uint32_t sb = scales[g], bb = biases[g];
            v = dequant_word(wq[(int64_t)id * words + w], sb | (sb << 16), bb | (bb << 16));
        }
        orow[w] = v;
    }
}

int sm_count() { return device_sm_count(); }

}  // namespace

int device_sm_count() {
    constexpr int kMaxDevices = 64;
    static std::atomic<int> cache[kMaxDevices];  // 0 = not yet queried
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return 148;
    }
    int n = cache[dev].load(std::memory_order_relaxed);
    if (n > 0) return n;
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
        cudaGetLastError();
        n = 148;
    }
    cache[dev].store(n, std::memory_order_relaxed);  // every thread that races here stores the same value
    return n;
}

cudaError_t launch_quantize(const uint16_t* w, int64_t n, int64_t k, uint32_t* wq, uint16_t* scales,
                            uint16_t* biases, cudaStream_t stream) {
    const int64_t ngroups = n * (k / 64);
    if (ngroups <= 0) return cudaSuccess;
    const int64_t warps = (ngroups + 3) / 4;
    const int64_t blocks = (warps * 32 + 255) / 256;
    quantize_kernel<<<(unsigned)blocks, 256, 0, stream>>>(w, ngroups, wq, scales, biases);
    return cudaGetLastError();
}

cudaError_t launch_rms_norm(const void* x, int dtype, const uint16_t* w, int64_t m, int64_t h, float eps,
                            float* out, cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    rms_norm_kernel<<<(unsigned)m, 256, 0, stream>>>(x, dtype, w, h, eps, out);
    return cudaGetLastError();
}

cudaError_t launch_residual_add(const void* h, int dtype, const float* y, int64_t n, float* out,
                                cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 8);
    residual_add_kernel<<<(unsigned)blocks, 256, 0, stream>>>(h, dtype, y, n, out);
    return cudaGetLastError();
}

cudaError_t launch_cast_bf16(const float* x, int64_t n, uint16_t* out, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const bool vec = (reinterpret_cast<uintptr_t>(x) & 15u) == 0 && (reinterpret_cast<uintptr_t>(out) & 7u) == 0;
    const int64_t blocks = std::min<int64_t>((n / (vec ? 4 : 1) + 255) / 256 + 1, (int64_t)sm_count() * 8);
    cast_bf16_kernel<<<(unsigned)blocks, 256, 0, stream>>>(x, n, out, vec);
    return cudaGetLastError();
}

cudaError_t launch_embed_q4(const int32_t* ids, int64_t m, const uint32_t* wq, const uint16_t* scales,
                            const uint16_t* biases, int64_t n, int64_t k, uint16_t* out, cudaStream_t stream) {
    if (m <= 0) return cudaSuccess;
    embed_q4_kernel<<<(unsigned)m, 256, 0, stream>>>(ids, wq, scales, biases, n, k, out);
    return cudaGetLastError();
}

int misc_device_error(bool clear) { return tu_device_error(clear); }

cudaError_t launch_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma, cudaStream_t stream) {
    if (n <= 0) return cudaSuccess;
    const int64_t blocks = std::min<int64_t>((n + 255) / 256, (int64_t)sm_count() * 16);
    synth_kernel<<<(unsigned)blocks, 256, 0, stream>>>(out, n, seed, mean, sigma * (1.0f / 65536.0f));
    return cudaGetLastError();
}

}  // namespace marlin
