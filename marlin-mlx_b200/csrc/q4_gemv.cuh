// q4_gemv.cuh — host-visible declarations of the Q4 decode kernels' launchers.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace marlin {

// kFix64 (internal): counted 64-bit fixed point (the one-kernel layer stack's h accumulator, see
// load_fix8).
enum ActDtype : int { kBF16 = 0, kF32 = 1, kFix64 = 2 };

// Device view of a QuantizedTensor (MLX layout).
struct Q4Mat {
    const uint32_t* w;  // [n, k/8]
    const uint16_t* s;  // bf16 [n, k/64]
    const uint16_t* b;  // bf16 [n, k/64]
    int64_t n;
    int64_t k;
};

enum Epilogue : int {
    kEpiStore = 0,   // y[m, row] = out                      (y dtype = out_dtype)
    kEpiSwiglu = 1,  // y[m, f] = (sigmoid(g)*g)*u of the gate (w0) and up (w1) rows f
    kEpiResid = 2,   // y[m, row] = resid[m, row] + out       (residual add, binary32)
};

// Activation rows handed from one integer-MMA decode kernel to the next in the operand form: the
// producing kernel's epilogue writes them, the consuming kernel copies its K range into shared
// memory instead of staging.  Per 64-group g of K and activation column c = 4 m + p (ncols =
// 8 * ceil(m / 2) rounded to a power of two, padding columns zero):
//   q[g][c][64]  s8 plane digits of the group, in the B-fragment byte order;
//   xs[g][c]     64 * (sum of the group's values) on plane-0 columns, 0 elsewhere;
//   xe[g][c]     2^e with e the group's exponent (|x| < 2^e), 0 on padding columns;
//   ssq[b][m]    sums of squares of the raw rows per 128-row block b < nssq (a following RMSNorm
//                takes its row factor from them); null when no RMSNorm follows.
struct XPlanes {
    uint8_t* q;
    float* xs;
    float* xe;
    float* ssq;
    int nssq;
};

// Cross-GPU exchange of the tensor-parallel decode step (plain peer loads/stores over NVLink, no
// multicast, no flags or fences): every value travels as one 8-byte word, (tag << 32) | bits, so a
// reader that sees the expected tag also sees the value (aligned 64-bit stores are single-copy
// atomic).  Tags are (step << 7) + slot + 1 with `step` a per-rank counter that every rank advances
// once per decode step (the lm_head's last CTA), so consecutive uses of a word carry different tags.
// Every rank owns one exchange buffer; part/keys hold the device addresses of all ranks' buffers in
// this process (the own one at [rank], the others IPC-mapped):
//   part[r]   [2 parities][tp sources][m][hidden] words: partial rows of down_proj (binary32 bits),
//   keys[r]   [tp sources][m][2] words: the low and high halves of the packed argmax keys,
//   step      this rank's step counter (in its own buffer).
// wait_cycles bounds each wait for a peer's word (SM clock cycles).  Once one wait has run out, the
// device error word is set and every later exchange wait returns at once, so a rank whose peer is
// gone finishes its step in about one wait limit instead of spinning once per word.
constexpr int kTpMax = 8;
constexpr unsigned long long kPeerWaitDefaultCycles = 4000000000ull;  // about 2 s at 2 GHz
struct TpExchange {
    int tp, rank, parity, layer;
    unsigned long long* part[kTpMax];
    unsigned long long* keys[kTpMax];
    unsigned* step;
    unsigned long long wait_cycles;
};

struct GemvLaunch {
    const void* x;  // [m, k] activations (x_dtype)
    int x_dtype;
    int64_t m;
    const uint16_t* norm_w;  // optional RMSNorm (1+w) applied to x first (k == hidden); null = none
    float eps;
    Q4Mat w0;  // main weight (gate for kEpiSwiglu)
    Q4Mat w1;  // up weight (kEpiSwiglu only)
    void* y;
    int y_dtype;
    int64_t ldy;         // row stride of y in elements
    const void* resid;   // kEpiResid input, [m, ldr]
    int resid_dtype;
    int64_t ldr;
    int epi;
    bool pdl;  // launch with programmatic stream serialization
    // integer-MMA family only: activations taken from planes (x unused; norm_w then applies as the
    // row factor from xin.ssq), and/or output rows also written as planes of y * (1 + out_norm)
    // (y when out_norm is null; xout.ssq, when set, receives the sums of squares of y)
    bool has_xin, has_xout;
    XPlanes xin, xout;
    const uint16_t* out_norm;
    // kEpiResid with tp.tp > 1: the partial rows are summed over the ranks (exchange) before the
    // residual add
    TpExchange tp;
};

// Decode kernel families (marlin_q4_set_decode_path): integer MMAs (default; the decode step's layers
// on the cluster K-split kernels with operand planes handed between them) and bf16 mma.sync.  Shapes
// the integer-MMA kernels do not cover (k % 512 != 0) use the bf16 mma.sync kernels.
enum DecodePath : int { kPathI8 = 0, kPathBf16 = 2 };
bool set_decode_path(int path);
int decode_path();
inline bool path_is_i8(int p) { return p == kPathI8; }

// Activation rows per launch of the selected family for this shape (the C ABI loops over passes).
int gemv_max_rows(int act_dtype, bool normed, int64_t k);
int lm_head_max_rows(int act_dtype, bool normed, int64_t k);

// Launches the decode GEMV family (one CTA per row block, weights fetched before the PDL wait).
// Returns cudaSuccess or the launch error.  Arguments are validated by the caller.
cudaError_t launch_q4_gemv(const GemvLaunch& L, cudaStream_t stream);

struct LmHeadLaunch {
    const void* x;  // [m, k] hidden state (x_dtype)
    int x_dtype;
    int64_t m;
    const uint16_t* norm_w;  // optional final RMSNorm
    float eps;
    Q4Mat w;                 // [vocab_shard, k]
    int64_t vocab_offset;    // global index of row 0 of this shard
    unsigned long long* keys;  // [m] packed (value, index) keys; must be zero on entry, left zero
    unsigned int* counter;     // completion counter; must be zero on entry, left zero
    unsigned long long* keys_out;  // optional [m]: final keys (for a cross-shard merge)
    int32_t* ids;            // optional [m]: argmax ids (vocab_offset applied)
    float* best;             // optional [m]: winning logit
    bool pdl;
    bool has_xin;            // integer-MMA family only: hidden state taken from planes (see XPlanes)
    XPlanes xin;
    // integer-MMA family, x_dtype kFix64 only: block 0 also writes x as binary32 [m, k] (optional)
    float* x_out;
    // words cleared by block 0 once the previous kernel in the stream has completed (the one-kernel
    // layer stack's barrier counter and abort word); null = none
    unsigned* reset;
    int n_reset;
    TpExchange tp;           // tp.tp > 1: the final keys are max-merged over the ranks (exchange)
};

cudaError_t launch_q4_lm_head_argmax(const LmHeadLaunch& L, cudaStream_t stream);

// Device error word of this translation unit (0 ok, >0 a DeviceError code, -1 CUDA failure).
int gemv_device_error(bool clear);

// SM count of the current device, cached per device index (thread-safe; 148 if the query fails).
int device_sm_count();

// Decode packed keys [m] into ids/best (used after a cross-GPU max-merge of keys).
cudaError_t launch_decode_keys(const unsigned long long* keys, int64_t m, int32_t* ids, float* best,
                               cudaStream_t stream);

}  // namespace marlin
