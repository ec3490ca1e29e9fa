// capi.cu — the extern "C" boundary declared in include/marlin_q4.h.
//
// Validates every argument before any launch, maps shapes onto the kernels' envelopes, and turns
// CUDA launch failures into MARLIN_Q4_ERR_CUDA.  Never synchronises the host (except
// marlin_q4_device_error, which is documented as synchronous) and never allocates.
#include "marlin_q4.h"

#include "q4_fused.cuh"
#include "q4_gemv.cuh"
#include "q4_i8.cuh"
#include "q4_prefill.cuh"
#include "q4_misc.cuh"

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>

namespace marlin {
namespace {

thread_local int t_last_cuda_error = 0;
// process-wide settings: set from any thread, read when a call is issued
std::atomic<bool> g_pdl{true};
std::atomic<int> g_step_kernels{MARLIN_Q4_STEP_FUSED};
std::atomic<unsigned long long> g_peer_wait_cycles{kPeerWaitDefaultCycles};

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return MARLIN_Q4_OK;
    t_last_cuda_error = (int)e;
    cudaGetLastError();  // clear the sticky-free launch error so later calls start clean
    return MARLIN_Q4_ERR_CUDA;
}

inline bool aligned(const void* p, uintptr_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
inline bool valid_dtype(int32_t d) { return d == MARLIN_Q4_BF16 || d == MARLIN_Q4_F32; }
inline size_t dtype_size(int32_t d) { return d == MARLIN_Q4_BF16 ? 2 : 4; }
inline size_t align16(size_t v) { return (v + 255) / 256 * 256; }

int check_tensor(const marlin_q4_tensor* t) {
    if (!t || !t->weight || !t->scales || !t->biases) return MARLIN_Q4_ERR_ARG;
    if (t->n <= 0 || t->k <= 0) return MARLIN_Q4_ERR_ARG;
    if (t->group_size != 64 || t->bits != 4 || t->k % 64 != 0) return MARLIN_Q4_ERR_SHAPE;
    if (t->k > (1 << 20) || t->n > (int64_t)1 << 31) return MARLIN_Q4_ERR_UNSUPPORTED;
    if (!aligned(t->weight, 16) || !aligned(t->scales, 16) || !aligned(t->biases, 16)) return MARLIN_Q4_ERR_ALIGN;
    return MARLIN_Q4_OK;
}

int check_act(const void* x, int32_t dtype) {
    if (!x) return MARLIN_Q4_ERR_ARG;
    if (!valid_dtype(dtype)) return MARLIN_Q4_ERR_ARG;
    if (!aligned(x, dtype_size(dtype))) return MARLIN_Q4_ERR_ALIGN;
    return MARLIN_Q4_OK;
}

// activations read by the GEMV kernels with 16-byte vector loads
int check_act16(const void* x, int32_t dtype) {
    int rc = check_act(x, dtype);
    if (rc) return rc;
    return aligned(x, 16) ? MARLIN_Q4_OK : MARLIN_Q4_ERR_ALIGN;
}

int check_norm(const uint16_t* w) { return (!w || aligned(w, 16)) ? MARLIN_Q4_OK : MARLIN_Q4_ERR_ALIGN; }

Q4Mat view(const marlin_q4_tensor* t) { return Q4Mat{t->weight, t->scales, t->biases, t->n, t->k}; }

// y[m, n] (y_dtype) for x[m, k]; rows processed in passes of at most rows_per_pass
int gemv_passes(const void* x, int32_t x_dtype, int64_t m, const uint16_t* norm_w, float eps, const Q4Mat& w0,
                const Q4Mat& w1, int epi, void* y, int32_t y_dtype, int64_t ldy, const void* resid,
                int32_t resid_dtype, int64_t ldr, cudaStream_t stream) {
    {
        // many bf16 rows (prefill): one tcgen05 GEMM launch over all of them
        GemvLaunch L{};
        L.x = x;
        L.x_dtype = x_dtype;
        L.m = m;
        L.norm_w = norm_w;
        L.eps = eps;
        L.w0 = w0;
        L.w1 = w1;
        L.y = y;
        L.y_dtype = y_dtype;
        L.ldy = ldy;
        L.resid = resid;
        L.resid_dtype = resid_dtype;
        L.ldr = ldr;
        L.epi = epi;
        L.pdl = g_pdl;
        if (prefill_applies(L)) return cuda_status(launch_prefill(L, stream));
    }
    const int64_t rp = gemv_max_rows(x_dtype, norm_w != nullptr, w0.k);
    for (int64_t r0 = 0; r0 < m; r0 += rp) {
        GemvLaunch L{};
        L.x = static_cast<const uint8_t*>(x) + r0 * w0.k * dtype_size(x_dtype);
        L.x_dtype = x_dtype;
        L.m = std::min(rp, m - r0);
        L.norm_w = norm_w;
        L.eps = eps;
        L.w0 = w0;
        L.w1 = w1;
        L.y = static_cast<uint8_t*>(y) + r0 * ldy * dtype_size(y_dtype);
        L.y_dtype = y_dtype;
        L.ldy = ldy;
        L.resid = resid ? static_cast<const uint8_t*>(resid) + r0 * ldr * dtype_size(resid_dtype) : nullptr;
        L.resid_dtype = resid_dtype;
        L.ldr = ldr;
        L.epi = epi;
        L.pdl = g_pdl;
        const int rc = cuda_status(launch_q4_gemv(L, stream));
        if (rc) return rc;
    }
    return MARLIN_Q4_OK;
}

}  // namespace
}  // namespace marlin

using namespace marlin;

extern "C" {

const char* marlin_q4_version(void) { return "marlin-q4-b200 0.1 (sm_100a)"; }

const char* marlin_q4_status_string(int status) {
    switch (status) {
        case MARLIN_Q4_OK: return "ok";
        case MARLIN_Q4_ERR_ARG: return "invalid argument";
        case MARLIN_Q4_ERR_SHAPE: return "invalid shape (k % 64, group_size 64, bits 4, matching dims)";
        case MARLIN_Q4_ERR_ALIGN: return "misaligned pointer";
        case MARLIN_Q4_ERR_UNSUPPORTED: return "unsupported size";
        case MARLIN_Q4_ERR_CUDA: return "CUDA launch failed";
        case MARLIN_Q4_ERR_WORKSPACE: return "workspace missing, too small or misaligned";
        default: return "unknown status";
    }
}

int marlin_q4_last_cuda_error(void) { return t_last_cuda_error; }

int marlin_q4_device_error(int clear) {
    int v = gemv_device_error(clear != 0);
    const int v_i8 = i8_device_error(clear != 0), v_pf = prefill_device_error(clear != 0),
              v_mi = misc_device_error(clear != 0), v_fu = fused_device_error(clear != 0),
              v_ro = rows_device_error(clear != 0);
    if (!v) v = v_fu;
    if (!v) v = v_ro;
    if (!v) v = v_i8;
    if (!v) v = v_pf;
    if (!v) v = v_mi;
    if (v < 0) return cuda_status(cudaGetLastError());
    return v;
}

void marlin_q4_set_pdl(int enable) { g_pdl = enable != 0; }

void marlin_q4_set_wait_limit_cycles(uint64_t cycles) {
    g_peer_wait_cycles = cycles ? (unsigned long long)cycles : kPeerWaitDefaultCycles;
}

int marlin_q4_set_step_kernels(int which) {
    if (which != MARLIN_Q4_STEP_FUSED && which != MARLIN_Q4_STEP_LAYERS) return MARLIN_Q4_ERR_ARG;
    g_step_kernels = which;
    return MARLIN_Q4_OK;
}

int marlin_q4_set_decode_path(int path) {
    return set_decode_path(path) ? MARLIN_Q4_OK : MARLIN_Q4_ERR_ARG;
}

int marlin_q4_quantize(const uint16_t* w, int64_t n, int64_t k, int32_t group_size, int32_t bits, uint32_t* wq,
                       uint16_t* scales, uint16_t* biases, void* stream) {
    if (!w || !wq || !scales || !biases || n <= 0 || k <= 0) return MARLIN_Q4_ERR_ARG;
    if (group_size != 64 || bits != 4 || k % 64 != 0) return MARLIN_Q4_ERR_SHAPE;
    if (!aligned(w, 16) || !aligned(wq, 4) || !aligned(scales, 2) || !aligned(biases, 2)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_quantize(w, n, k, wq, scales, biases, static_cast<cudaStream_t>(stream)));
}

int marlin_q4_matmul(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* w, void* y, void* stream) {
    int rc = check_tensor(w);
    if (rc) return rc;
    if ((rc = check_act16(x, x_dtype))) return rc;
    if ((rc = check_act(y, x_dtype))) return rc;
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    const Q4Mat v = view(w);
    return gemv_passes(x, x_dtype, m, nullptr, 0.f, v, v, kEpiStore, y, x_dtype, w->n, nullptr, 0, 0,
                       static_cast<cudaStream_t>(stream));
}

int marlin_q4_matmul_f32(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* w, float* y,
                         void* stream) {
    int rc = check_tensor(w);
    if (rc) return rc;
    if ((rc = check_act16(x, x_dtype))) return rc;
    if ((rc = check_act(y, MARLIN_Q4_F32))) return rc;
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    const Q4Mat v = view(w);
    return gemv_passes(x, x_dtype, m, nullptr, 0.f, v, v, kEpiStore, y, MARLIN_Q4_F32, w->n, nullptr, 0, 0,
                       static_cast<cudaStream_t>(stream));
}

int marlin_q4_cast_bf16(const float* x, int64_t count, uint16_t* out, void* stream) {
    if (!x || !out || count <= 0) return MARLIN_Q4_ERR_ARG;
    if (!aligned(x, 4) || !aligned(out, 2)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_cast_bf16(x, count, out, static_cast<cudaStream_t>(stream)));
}

int marlin_q4_embed(const int32_t* ids, int64_t m, const marlin_q4_tensor* table, uint16_t* out, void* stream) {
    int rc = check_tensor(table);
    if (rc) return rc;
    if (!ids || !out || m <= 0) return MARLIN_Q4_ERR_ARG;
    if (!aligned(ids, 4) || !aligned(out, 16)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_embed_q4(ids, m, table->weight, table->scales, table->biases, table->n, table->k, out,
                                       static_cast<cudaStream_t>(stream)));
}

int marlin_q4_rms_norm(const void* x, int32_t x_dtype, const uint16_t* weight, int64_t m, int64_t h, float eps,
                       float* out, void* stream) {
    int rc = check_act(x, x_dtype);
    if (rc) return rc;
    if (!weight || !out || m <= 0 || h <= 0) return MARLIN_Q4_ERR_ARG;
    if (!aligned(out, 4) || !aligned(weight, 2)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_rms_norm(x, x_dtype, weight, m, h, eps, out, static_cast<cudaStream_t>(stream)));
}

int marlin_q4_gate_up_swiglu(const void* x, int32_t x_dtype, int64_t m, const uint16_t* norm_weight, float eps,
                             const marlin_q4_tensor* gate, const marlin_q4_tensor* up, void* act, void* stream) {
    int rc;
    if ((rc = check_tensor(gate)) || (rc = check_tensor(up))) return rc;
    if ((rc = check_act16(x, x_dtype)) || (rc = check_norm(norm_weight))) return rc;
    if (gate->n != up->n || gate->k != up->k) return MARLIN_Q4_ERR_SHAPE;
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    const int32_t act_dtype = norm_weight ? MARLIN_Q4_F32 : x_dtype;
    if ((rc = check_act(act, act_dtype))) return rc;
    return gemv_passes(x, x_dtype, m, norm_weight, eps, view(gate), view(up), kEpiSwiglu, act, act_dtype, gate->n,
                       nullptr, 0, 0, static_cast<cudaStream_t>(stream));
}

int marlin_q4_matmul_residual(const void* act, int32_t act_dtype, int64_t m, const marlin_q4_tensor* w,
                              const void* resid, int32_t resid_dtype, float* y, void* stream) {
    int rc;
    if ((rc = check_tensor(w))) return rc;
    if ((rc = check_act16(act, act_dtype)) || (rc = check_act(resid, resid_dtype))) return rc;
    if ((rc = check_act(y, MARLIN_Q4_F32))) return rc;
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    const Q4Mat v = view(w);
    return gemv_passes(act, act_dtype, m, nullptr, 0.f, v, v, kEpiResid, y, MARLIN_Q4_F32, w->n, resid, resid_dtype,
                       w->n, static_cast<cudaStream_t>(stream));
}

size_t marlin_q4_mlp_workspace_size(int64_t m, int64_t intermediate, int32_t x_dtype) {
    if (m <= 0 || intermediate <= 0 || !valid_dtype(x_dtype)) return 0;
    return align16((size_t)m * intermediate * dtype_size(x_dtype));
}

int marlin_q4_mlp(const void* x, int32_t x_dtype, int64_t m, const marlin_q4_tensor* gate,
                  const marlin_q4_tensor* up, const marlin_q4_tensor* down, void* y, void* workspace,
                  size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_tensor(gate)) || (rc = check_tensor(up)) || (rc = check_tensor(down))) return rc;
    if ((rc = check_act16(x, x_dtype)) || (rc = check_act(y, x_dtype))) return rc;
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    if (gate->n != up->n || gate->k != up->k || down->k != gate->n || down->n != gate->k) return MARLIN_Q4_ERR_SHAPE;
    if (!workspace || !aligned(workspace, 16) || workspace_bytes < marlin_q4_mlp_workspace_size(m, gate->n, x_dtype))
        return MARLIN_Q4_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if ((rc = gemv_passes(x, x_dtype, m, nullptr, 0.f, view(gate), view(up), kEpiSwiglu, workspace, x_dtype,
                          gate->n, nullptr, 0, 0, st)))
        return rc;
    const Q4Mat d = view(down);
    return gemv_passes(workspace, x_dtype, m, nullptr, 0.f, d, d, kEpiStore, y, x_dtype, down->n, nullptr, 0, 0, st);
}

int marlin_q4_residual_add(const void* h, int32_t h_dtype, const float* y, int64_t count, float* out, void* stream) {
    int rc;
    if ((rc = check_act(h, h_dtype))) return rc;
    if (!y || !out || count <= 0) return MARLIN_Q4_ERR_ARG;
    if (!aligned(y, 4) || !aligned(out, 4)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_residual_add(h, h_dtype, y, count, out, static_cast<cudaStream_t>(stream)));
}

size_t marlin_q4_lm_head_workspace_size(int64_t m) {
    if (m <= 0) return 0;
    return align16((size_t)m * 8 + 16);
}

int marlin_q4_lm_head_argmax(const void* hidden, int32_t dtype, int64_t m, const uint16_t* norm_weight, float eps,
                             const marlin_q4_tensor* lm, int64_t vocab_offset, int32_t* ids, float* best,
                             uint64_t* keys_out, void* workspace, size_t workspace_bytes, void* stream) {
    int rc;
    if ((rc = check_tensor(lm))) return rc;
    if ((rc = check_act16(hidden, dtype)) || (rc = check_norm(norm_weight))) return rc;
    if (m <= 0 || vocab_offset < 0 || (!ids && !best && !keys_out)) return MARLIN_Q4_ERR_ARG;
    if (vocab_offset + lm->n > 0xffffffffLL || lm->k > 64 * 64) return MARLIN_Q4_ERR_UNSUPPORTED;
    if (!workspace || !aligned(workspace, 16) || workspace_bytes < marlin_q4_lm_head_workspace_size(m))
        return MARLIN_Q4_ERR_WORKSPACE;
    if ((ids && !aligned(ids, 4)) || (best && !aligned(best, 4)) || (keys_out && !aligned(keys_out, 8)))
        return MARLIN_Q4_ERR_ALIGN;
    unsigned long long* keys = static_cast<unsigned long long*>(workspace);
    unsigned int* counter = reinterpret_cast<unsigned int*>(keys + m);
    const int64_t rp = lm_head_max_rows(dtype, norm_weight != nullptr, lm->k);
    for (int64_t r0 = 0; r0 < m; r0 += rp) {
        LmHeadLaunch L{};
        L.x = static_cast<const uint8_t*>(hidden) + r0 * lm->k * dtype_size(dtype);
        L.x_dtype = dtype;
        L.m = std::min(rp, m - r0);
        L.norm_w = norm_weight;
        L.eps = eps;
        L.w = view(lm);
        L.vocab_offset = vocab_offset;
        L.keys = keys + r0;
        L.counter = counter;
        L.keys_out = keys_out ? reinterpret_cast<unsigned long long*>(keys_out) + r0 : nullptr;
        L.ids = ids ? ids + r0 : nullptr;
        L.best = best ? best + r0 : nullptr;
        L.pdl = g_pdl;
        if ((rc = cuda_status(launch_q4_lm_head_argmax(L, static_cast<cudaStream_t>(stream))))) return rc;
    }
    return MARLIN_Q4_OK;
}

int marlin_q4_decode_keys(const uint64_t* keys, int64_t m, int32_t* ids, float* best, void* stream) {
    if (!keys || m <= 0 || (!ids && !best)) return MARLIN_Q4_ERR_ARG;
    return cuda_status(launch_decode_keys(reinterpret_cast<const unsigned long long*>(keys), m, ids, best,
                                          static_cast<cudaStream_t>(stream)));
}

// Rows per pass of the decode step: more rows run as consecutive chunks of this many (every chunk a
// full step; the rows are independent).  Measured per row and step on B200: 112 us in passes of 8
// rows, 131 us in passes of 4 and 146 us in passes of 16 (the 16-row kernels run one CTA per SM).
constexpr int64_t kStepChunkRows = 8;

// Workspace of marlin_q4_decode_step: a zero-invariant head (the argmax keys and CTA counter, zero
// before the first call and left zero by every call) followed by the step's scratch.
namespace {
size_t step_zero_bytes(int64_t m) { return 256 + align16((size_t)m * 8 + 16); }
size_t step_ssq_bytes(int64_t m, int64_t hidden) { return align16((size_t)((hidden + 127) / 128) * m * 4); }
// h and act (binary32), then the activation planes handed between the integer-MMA kernels
size_t step_compose_bytes(int64_t m, int64_t hidden, int64_t inter) {
    size_t b = align16((size_t)m * hidden * 4) + align16((size_t)m * inter * 4);
    if (m <= kStepChunkRows)
        b = std::max((b + 255) / 256 * 256 + i8_planes_bytes(m, inter) + i8_planes_bytes(m, hidden) +
                         step_ssq_bytes(m, hidden),
                     fused_acc_bytes(m, hidden));  // or the one-kernel stack's accumulators
    else  // h for all rows, then the scratch of one chunk (the step runs in row chunks)
        b = std::max(b, align16((size_t)m * hidden * 4) + step_compose_bytes(kStepChunkRows, hidden, inter));
    return b;
}

// The decode step on the integer-MMA kernels with the activations handed over as planes: each
// kernel's epilogue writes the next kernel's operand (act planes; h * (1 + next norm weight) planes
// with per-block sums of squares), so only the first gate/up launch stages from h0.
// Exchange buffer of the tensor-parallel step (TpExchange), per rank.
struct TpLayout {
    size_t part, keys, step, total;
};
TpLayout tp_layout(int64_t m, int64_t hidden, int tp) {
    auto al = [](size_t v) { return (v + 255) / 256 * 256; };
    TpLayout t{};
    size_t off = 0;
    t.part = off;
    off += al((size_t)2 * tp * m * hidden * 8);
    t.keys = off;
    off += al((size_t)tp * m * 2 * 8);
    t.step = off;
    off += 256;
    t.total = off;
    return t;
}

int decode_step_planes(const uint16_t* h0, int64_t m, int64_t hidden, int64_t inter, int32_t n_layers,
                       const marlin_q4_layer* layers, const uint16_t* final_norm, float eps,
                       const marlin_q4_tensor* lm, int32_t* ids, float* best, float* h, uint8_t* scratch,
                       void* lmws, cudaStream_t st, const TpExchange* tpx = nullptr, int64_t vocab_offset = 0) {
    float* act = reinterpret_cast<float*>(scratch + align16((size_t)m * hidden * 4));
    uint8_t* pl = scratch + (align16((size_t)m * hidden * 4) + align16((size_t)m * inter * 4) + 255) / 256 * 256;
    const XPlanes ap = i8_planes_at(pl, m, inter, nullptr, 0);
    pl += i8_planes_bytes(m, inter);
    float* ssq = reinterpret_cast<float*>(pl + i8_planes_bytes(m, hidden));
    const XPlanes hp = i8_planes_at(pl, m, hidden, ssq, (int)((hidden + 127) / 128));
    int rc;
    const void* cur = h0;
    int32_t cur_dtype = MARLIN_Q4_BF16;
    for (int32_t l = 0; l < n_layers; ++l) {
        const marlin_q4_layer& Ly = layers[l];
        GemvLaunch G{};
        G.x = cur;
        G.x_dtype = cur_dtype;
        G.m = m;
        G.norm_w = Ly.post_attn_norm;
        G.eps = eps;
        G.w0 = view(&Ly.gate_proj);
        G.w1 = view(&Ly.up_proj);
        G.y = act;
        G.y_dtype = MARLIN_Q4_F32;
        G.ldy = inter;
        G.epi = kEpiSwiglu;
        G.pdl = g_pdl;
        G.has_xin = l > 0;
        G.xin = hp;
        G.has_xout = true;
        G.xout = ap;
        if ((rc = cuda_status(launch_i8_gemv(G, st)))) return rc;
        GemvLaunch D{};
        D.x = act;
        D.x_dtype = MARLIN_Q4_F32;
        D.m = m;
        D.w0 = view(&Ly.down_proj);
        D.y = h;
        D.y_dtype = MARLIN_Q4_F32;
        D.ldy = hidden;
        D.resid = cur;
        D.resid_dtype = cur_dtype;
        D.ldr = hidden;
        D.epi = kEpiResid;
        D.pdl = g_pdl;
        D.has_xin = true;
        D.xin = ap;
        D.has_xout = true;
        D.xout = hp;
        D.out_norm = l + 1 < n_layers ? layers[l + 1].post_attn_norm : final_norm;
        if (tpx) {
            D.tp = *tpx;
            D.tp.parity = l & 1;
            D.tp.layer = l;
        }
        if ((rc = cuda_status(launch_i8_gemv(D, st)))) return rc;
        cur = h;
        cur_dtype = MARLIN_Q4_F32;
    }
    LmHeadLaunch Lh{};
    Lh.x = h;
    Lh.x_dtype = MARLIN_Q4_F32;
    Lh.m = m;
    Lh.norm_w = final_norm;
    Lh.eps = eps;
    Lh.w = view(lm);
    Lh.keys = static_cast<unsigned long long*>(lmws);
    Lh.counter = reinterpret_cast<unsigned int*>(Lh.keys + m);
    Lh.ids = ids;
    Lh.best = best;
    Lh.pdl = g_pdl;
    Lh.has_xin = true;
    Lh.xin = hp;
    Lh.vocab_offset = vocab_offset;
    if (tpx) Lh.tp = *tpx;
    return cuda_status(launch_i8_lm_head(Lh, st));
}
// Whether marlin_q4_decode_step runs its MLP layers on the one-kernel layer stack (rows in chunks of
// kStepChunkRows), with the current settings on the current device.
bool step_uses_fused(int64_t m, int64_t hidden, int64_t inter, int32_t n_layers) {
    const int64_t mc = std::min<int64_t>(m, kStepChunkRows);
    return path_is_i8(decode_path()) && g_step_kernels == MARLIN_Q4_STEP_FUSED && i8_supported(hidden, mc) &&
           fused_supported(mc, hidden, inter, n_layers);
}

// The decode step with the MLP layers as one persistent kernel (q4_fused.cu) followed by the fused
// lm_head + argmax, which reads the final h from the kernel's fixed-point accumulator, writes h_out
// when asked, and clears the kernel's barrier words (sync, in the zero-invariant head of the
// workspace) for the next step.
int decode_step_fused(const uint16_t* h0, int64_t m, int64_t hidden, int64_t inter, int32_t n_layers,
                      const marlin_q4_layer* layers, const uint16_t* final_norm, float eps, const marlin_q4_tensor* lm,
                      int32_t* ids, float* best, float* h_out, uint8_t* scratch, unsigned* sync, void* lmws,
                      cudaStream_t st) {
    FusedLayer fl[kFusedMaxLayers];
    for (int32_t l = 0; l < n_layers; ++l)
        fl[l] = FusedLayer{layers[l].post_attn_norm, view(&layers[l].gate_proj), view(&layers[l].up_proj),
                           view(&layers[l].down_proj)};
    FusedLaunch F{};
    F.h0 = h0;
    F.m = m;
    F.hidden = hidden;
    F.inter = inter;
    F.n_layers = n_layers;
    F.layers = fl;
    F.eps = eps;
    F.acc = reinterpret_cast<unsigned long long*>(scratch);
    F.sync = sync;
    F.wait_cycles = g_peer_wait_cycles;
    F.pdl = g_pdl;
    int rc;
    if ((rc = cuda_status(launch_fused_layers(F, st)))) return rc;
    LmHeadLaunch Lh{};
    Lh.x = F.acc + (size_t)(n_layers % 3) * (size_t)m * (size_t)hidden;
    Lh.x_dtype = kFix64;
    Lh.m = m;
    Lh.norm_w = final_norm;
    Lh.eps = eps;
    Lh.w = view(lm);
    Lh.keys = static_cast<unsigned long long*>(lmws);
    Lh.counter = reinterpret_cast<unsigned int*>(Lh.keys + m);
    Lh.ids = ids;
    Lh.best = best;
    Lh.pdl = g_pdl;
    Lh.x_out = h_out;
    Lh.reset = sync;
    Lh.n_reset = 2;
    return cuda_status(launch_i8_lm_head(Lh, st));
}
}  // namespace

int marlin_q4_decode_step_kernels(int64_t m, int64_t hidden, int64_t intermediate, int32_t n_layers) {
    if (m < 1 || hidden < 1 || intermediate < 1 || n_layers < 1) return MARLIN_Q4_ERR_ARG;
    return step_uses_fused(m, hidden, intermediate, n_layers) ? MARLIN_Q4_STEP_FUSED : MARLIN_Q4_STEP_LAYERS;
}

size_t marlin_q4_decode_step_workspace_size(int64_t m, int64_t hidden, int64_t intermediate) {
    if (m <= 0 || hidden <= 0 || intermediate <= 0) return 0;
    return step_zero_bytes(m) + step_compose_bytes(m, hidden, intermediate);
}

int marlin_q4_decode_step(const uint16_t* h0, int64_t m, int64_t hidden, int32_t n_layers,
                          const marlin_q4_layer* layers, const uint16_t* final_norm, float eps,
                          const marlin_q4_tensor* lm, int32_t* ids, float* best, float* h_out, void* workspace,
                          size_t workspace_bytes, void* stream) {
    int rc;
    if (!h0 || m <= 0 || hidden <= 0 || n_layers < 1 || !layers || !final_norm || !ids)
        return MARLIN_Q4_ERR_ARG;
    if (!aligned(h0, 16) || !aligned(final_norm, 16) || (h_out && !aligned(h_out, 16))) return MARLIN_Q4_ERR_ALIGN;
    if ((rc = check_tensor(lm))) return rc;
    if (lm->k != hidden) return MARLIN_Q4_ERR_SHAPE;
    int64_t inter = layers[0].gate_proj.n;
    bool uniform = true;
    for (int32_t l = 0; l < n_layers; ++l) {
        const marlin_q4_layer& L = layers[l];
        if (!L.post_attn_norm) return MARLIN_Q4_ERR_ARG;
        if (!aligned(L.post_attn_norm, 16)) return MARLIN_Q4_ERR_ALIGN;
        if ((rc = check_tensor(&L.gate_proj)) || (rc = check_tensor(&L.up_proj)) || (rc = check_tensor(&L.down_proj)))
            return rc;
        if (L.gate_proj.k != hidden || L.up_proj.k != hidden || L.up_proj.n != L.gate_proj.n ||
            L.down_proj.k != L.gate_proj.n || L.down_proj.n != hidden)
            return MARLIN_Q4_ERR_SHAPE;
        uniform = uniform && L.gate_proj.n == inter;
        inter = std::max<int64_t>(inter, L.gate_proj.n);
    }
    if (!workspace || !aligned(workspace, 256) ||
        workspace_bytes < marlin_q4_decode_step_workspace_size(m, hidden, inter))
        return MARLIN_Q4_ERR_WORKSPACE;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* scratch = ws + step_zero_bytes(m);
    void* lmws = ws + 256;  // keys + counter, zero-invariant
    float* h = reinterpret_cast<float*>(scratch);
    float* act = reinterpret_cast<float*>(scratch + align16((size_t)m * hidden * 4));
    if (h_out) h = h_out;
    unsigned* sync = reinterpret_cast<unsigned*>(ws);  // barrier words of the one-kernel stack, zero-invariant
    const bool fused = uniform && step_uses_fused(m, hidden, inter, n_layers);
    if (fused && m <= kStepChunkRows)
        return decode_step_fused(h0, m, hidden, inter, n_layers, layers, final_norm, eps, lm, ids, best, h_out,
                                 scratch, sync, lmws, st);
    if (fused) {  // consecutive chunks of kStepChunkRows rows (the rows are independent)
        uint8_t* cs = scratch + align16((size_t)m * hidden * 4);
        for (int64_t r0 = 0; r0 < m; r0 += kStepChunkRows) {
            const int64_t mc = std::min<int64_t>(kStepChunkRows, m - r0);
            if ((rc = decode_step_fused(h0 + r0 * hidden, mc, hidden, inter, n_layers, layers, final_norm, eps, lm,
                                        ids + r0, best ? best + r0 : nullptr, h_out ? h_out + r0 * hidden : nullptr,
                                        cs, sync, lmws, st)))
                return rc;
        }
        return MARLIN_Q4_OK;
    }
    if (path_is_i8(decode_path()) && uniform && m <= kStepChunkRows && i8_supported(hidden, m) &&
        i8_supported(inter, m) && hidden % 128 == 0)
        return decode_step_planes(h0, m, hidden, inter, n_layers, layers, final_norm, eps, lm, ids, best, h, scratch,
                                  lmws, st);
    if (path_is_i8(decode_path()) && uniform && i8_supported(hidden, kStepChunkRows) &&
        i8_supported(inter, kStepChunkRows) && hidden % 128 == 0) {
        // more rows than one plane hand-off serves: the rows are independent (per-row norm, GEMV and
        // argmax), so the step runs on consecutive chunks of kStepChunkRows rows, stream-ordered, each
        // chunk in the scratch after h
        uint8_t* cs = scratch + align16((size_t)m * hidden * 4);
        for (int64_t r0 = 0; r0 < m; r0 += kStepChunkRows) {
            const int64_t mc = std::min<int64_t>(kStepChunkRows, m - r0);
            if ((rc = decode_step_planes(h0 + r0 * hidden, mc, hidden, inter, n_layers, layers, final_norm, eps, lm,
                                         ids + r0, best ? best + r0 : nullptr, h + r0 * hidden, cs, lmws, st)))
                return rc;
        }
        return MARLIN_Q4_OK;
    }
    const void* cur = h0;
    int32_t cur_dtype = MARLIN_Q4_BF16;
    for (int32_t l = 0; l < n_layers; ++l) {
        const marlin_q4_layer& L = layers[l];
        if ((rc = marlin_q4_gate_up_swiglu(cur, cur_dtype, m, L.post_attn_norm, eps, &L.gate_proj, &L.up_proj, act,
                                           stream)))
            return rc;
        if ((rc = marlin_q4_matmul_residual(act, MARLIN_Q4_F32, m, &L.down_proj, cur, cur_dtype, h, stream))) return rc;
        cur = h;
        cur_dtype = MARLIN_Q4_F32;
    }
    return marlin_q4_lm_head_argmax(cur, cur_dtype, m, final_norm, eps, lm, 0, ids, best, nullptr, lmws,
                                    marlin_q4_lm_head_workspace_size(m), st);
}

// ---- tensor-parallel decode step ------------------------------------------------------------------
size_t marlin_q4_tp_exchange_size(int64_t m, int64_t hidden, int32_t tp) {
    if (m <= 0 || hidden <= 0 || tp < 1) return 0;
    return tp_layout(std::min<int64_t>(m, kStepChunkRows), hidden, tp).total;
}

int marlin_q4_device_alloc(size_t bytes, void** ptr) {
    if (!ptr || !bytes) return MARLIN_Q4_ERR_ARG;
    *ptr = nullptr;
    if (cudaMalloc(ptr, bytes) != cudaSuccess) return cuda_status(cudaErrorMemoryAllocation);
    if (cudaMemset(*ptr, 0, bytes) != cudaSuccess || cudaDeviceSynchronize() != cudaSuccess) {
        cudaFree(*ptr);
        *ptr = nullptr;
        return MARLIN_Q4_ERR_CUDA;
    }
    return MARLIN_Q4_OK;
}

int marlin_q4_device_free(void* ptr) { return cuda_status(cudaFree(ptr)); }

int marlin_q4_ipc_get_handle(const void* ptr, void* handle) {
    if (!ptr || !handle) return MARLIN_Q4_ERR_ARG;
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, const_cast<void*>(ptr));
    if (e != cudaSuccess) return cuda_status(e);
    std::memcpy(handle, &h, sizeof(h));
    return MARLIN_Q4_OK;
}

int marlin_q4_ipc_open_handle(const void* handle, void** ptr) {
    if (!handle || !ptr) return MARLIN_Q4_ERR_ARG;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle, sizeof(h));
    return cuda_status(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
}

int marlin_q4_ipc_close_handle(void* ptr) { return cuda_status(cudaIpcCloseMemHandle(ptr)); }

int marlin_q4_tp_decode_step(const uint16_t* h0, int64_t m, int64_t hidden, int32_t n_layers,
                             const marlin_q4_layer* layers, const uint16_t* final_norm, float eps,
                             const marlin_q4_tensor* lm_shard, int64_t vocab_offset, int32_t* ids, float* best,
                             float* h_out, int32_t tp_rank, int32_t tp_size, void* const* exchange, void* workspace,
                             size_t workspace_bytes, void* stream) {
    int rc;
    if (!h0 || m <= 0 || hidden <= 0 || n_layers < 1 || !layers || !final_norm || !ids || !exchange)
        return MARLIN_Q4_ERR_ARG;
    if (tp_size < 1 || tp_size > kTpMax || tp_rank < 0 || tp_rank >= tp_size || vocab_offset < 0)
        return MARLIN_Q4_ERR_ARG;
    if (!aligned(h0, 16) || !aligned(final_norm, 16) || (h_out && !aligned(h_out, 16))) return MARLIN_Q4_ERR_ALIGN;
    if ((rc = check_tensor(lm_shard))) return rc;
    if (lm_shard->k != hidden || vocab_offset + lm_shard->n > 0xffffffffLL) return MARLIN_Q4_ERR_SHAPE;
    // the down shard may carry zero K padding beyond its gate/up rows (its K a multiple of 512)
    const int64_t inter = layers[0].down_proj.k;
    for (int32_t l = 0; l < n_layers; ++l) {
        const marlin_q4_layer& L = layers[l];
        if (!L.post_attn_norm) return MARLIN_Q4_ERR_ARG;
        if (!aligned(L.post_attn_norm, 16)) return MARLIN_Q4_ERR_ALIGN;
        if ((rc = check_tensor(&L.gate_proj)) || (rc = check_tensor(&L.up_proj)) || (rc = check_tensor(&L.down_proj)))
            return rc;
        if (L.gate_proj.k != hidden || L.up_proj.k != hidden || L.up_proj.n != L.gate_proj.n ||
            L.down_proj.n != hidden || L.down_proj.k != inter || L.gate_proj.n > inter || L.gate_proj.n % 64)
            return MARLIN_Q4_ERR_SHAPE;
    }
    // more than kStepChunkRows rows run as consecutive chunks of kStepChunkRows rows, each a full step with
    // its own exchanges (the step counter advances once per chunk on every rank, so the tags of one
    // chunk never match another's); the exchange layout is that of one chunk
    const int64_t mc = std::min<int64_t>(m, kStepChunkRows);
    if (hidden % 128 || !i8_supported(hidden, mc) || !i8_supported(inter, mc)) return MARLIN_Q4_ERR_UNSUPPORTED;
    if (!workspace || !aligned(workspace, 256) ||
        workspace_bytes < marlin_q4_decode_step_workspace_size(m, hidden, inter))
        return MARLIN_Q4_ERR_WORKSPACE;
    const TpLayout lay = tp_layout(mc, hidden, tp_size);
    if (n_layers > 120) return MARLIN_Q4_ERR_UNSUPPORTED;  // exchange tags hold the layer in 7 bits
    TpExchange X{};
    X.tp = tp_size;
    X.rank = tp_rank;
    X.wait_cycles = g_peer_wait_cycles;
    for (int r = 0; r < tp_size; ++r) {
        uint8_t* b = static_cast<uint8_t*>(exchange[r]);
        if (!b || !aligned(b, 256)) return MARLIN_Q4_ERR_ARG;
        X.part[r] = reinterpret_cast<unsigned long long*>(b + lay.part);
        X.keys[r] = reinterpret_cast<unsigned long long*>(b + lay.keys);
    }
    X.step = reinterpret_cast<unsigned*>(static_cast<uint8_t*>(exchange[tp_rank]) + lay.step);
    uint8_t* ws = static_cast<uint8_t*>(workspace);
    uint8_t* scratch = ws + step_zero_bytes(m);
    float* h = h_out ? h_out : reinterpret_cast<float*>(scratch);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (m <= kStepChunkRows)
        return decode_step_planes(h0, m, hidden, inter, n_layers, layers, final_norm, eps, lm_shard, ids, best, h,
                                  scratch, ws + 256, st, &X, vocab_offset);
    // chunk scratch after h (as in marlin_q4_decode_step)
    uint8_t* cs = scratch + align16((size_t)m * hidden * 4);
    for (int64_t r0 = 0; r0 < m; r0 += kStepChunkRows) {
        const int64_t n = std::min<int64_t>(kStepChunkRows, m - r0);
        if ((rc = decode_step_planes(h0 + r0 * hidden, n, hidden, inter, n_layers, layers, final_norm, eps, lm_shard,
                                     ids + r0, best ? best + r0 : nullptr, h + r0 * hidden, cs, ws + 256, st, &X,
                                     vocab_offset)))
            return rc;
    }
    return MARLIN_Q4_OK;
}

int marlin_q4_synth_bf16(uint16_t* out, int64_t n, uint64_t seed, float mean, float sigma, void* stream) {
    if (!out || n <= 0) return MARLIN_Q4_ERR_ARG;
    if (!aligned(out, 2)) return MARLIN_Q4_ERR_ALIGN;
    return cuda_status(launch_synth_bf16(out, n, seed, mean, sigma, static_cast<cudaStream_t>(stream)));
}

}  // extern "C"
