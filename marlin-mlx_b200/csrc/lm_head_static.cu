// lm_head_static.cu — marlin_q4_lm_head_argmax_static: the fused lm_head + argmax without a
// caller-provided workspace.
//
// Who needs it: callers that cannot allocate or own device scratch for this call.  A binding that
// replaces the lm_head + greedy sampling pair of a model's decode loop is one of them: that call
// shape passes only the hidden state and the weights, so there is no buffer to hand over, and a
// cudaMalloc there would synchronise the device inside the decode loop.  Bindings from runtimes
// that do not manage device memory themselves are in the same position.
//
// How: the argmax keys and the CTA-completion counter live in one file-scope device array
// (kStaticScratchBytes, room for kStaticMaxRows rows).  Its address is looked up with
// cudaGetSymbolAddress, with the device current, once per device and CUDA context (a context that
// was reset and created again gets a fresh lookup, since the module, and with it the array, may
// then sit at another address), and handed to the kernels as a plain pointer.  Every call first
// clears the keys and the counter it is about to use (cudaMemsetAsync on the caller's stream, no
// allocation), so it never depends on what an earlier call left there, even one that was cut short.
// Nothing is allocated: no cudaMalloc, no cudaFree, no allocating library routine.
//
// Limits: m <= kStaticMaxRows (larger m returns MARLIN_Q4_ERR_UNSUPPORTED before any CUDA call).
// All calls on a device share the one array, so two calls that may run at the same time on that
// device (different streams, or different host threads without ordering) race on the keys and give
// wrong ids; order them on one stream.  The lookup (the first call on each device and context) must
// happen outside stream capture.
#include "marlin_q4.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace {

constexpr int64_t kStaticMaxRows = MARLIN_Q4_LM_HEAD_STATIC_MAX_ROWS;
// keys [kStaticMaxRows] u64 + counter, rounded up to 256 bytes: 768 bytes
constexpr size_t kStaticScratchBytes = ((size_t)kStaticMaxRows * 8 + 16 + 255) / 256 * 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_lm_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
struct ScratchAddr {
    void* ptr;
    unsigned long long ctx_id;  // CUDA context the address belongs to
};
ScratchAddr g_scratch[kMaxDevices] = {};

// Unique id of the calling thread's current context (0 when there is none yet, or the driver is too
// old to give one).  The driver calls are resolved through the runtime, so the library still loads on
// machines without a CUDA driver.
unsigned long long current_ctx_id() {
    using GetCurrentFn = CUresult (*)(CUcontext*);
    using GetIdFn = CUresult (*)(CUcontext, unsigned long long*);
    static GetCurrentFn get_current = nullptr;
    static GetIdFn get_id = nullptr;
    static bool tried = false;
    if (!tried) {  // under g_scratch_mutex
        tried = true;
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_current = reinterpret_cast<GetCurrentFn>(p);
        p = nullptr;
        if (cudaGetDriverEntryPoint("cuCtxGetId", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            get_id = reinterpret_cast<GetIdFn>(p);
        cudaGetLastError();
    }
    CUcontext ctx = nullptr;
    unsigned long long id = 0;
    if (!get_current || !get_id || get_current(&ctx) != CUDA_SUCCESS || !ctx || get_id(ctx, &id) != CUDA_SUCCESS)
        return 0;
    return id;
}

// Device address of the scratch array in the current device's context (looked up once per device
// and context).
int scratch_for_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return MARLIN_Q4_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    const unsigned long long id = current_ctx_id();
    if (id && g_scratch[dev].ptr && g_scratch[dev].ctx_id == id) {
        *out = g_scratch[dev].ptr;
        return MARLIN_Q4_OK;
    }
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_lm_static_scratch) != cudaSuccess || !p) {  // creates the context if needed
        cudaGetLastError();
        return MARLIN_Q4_ERR_CUDA;
    }
    g_scratch[dev] = ScratchAddr{p, current_ctx_id()};
    *out = p;
    return MARLIN_Q4_OK;
}

}  // namespace

extern "C" {

int marlin_q4_lm_head_argmax_static(const void* hidden, int32_t dtype, int64_t m, const uint16_t* norm_weight,
                                    float eps, const marlin_q4_tensor* lm, int64_t vocab_offset, int32_t* ids,
                                    float* best, uint64_t* keys_out, void* stream) {
    if (m <= 0) return MARLIN_Q4_ERR_ARG;
    if (m > kStaticMaxRows) return MARLIN_Q4_ERR_UNSUPPORTED;
    static_assert(kStaticScratchBytes >= (size_t)kStaticMaxRows * 8 + 16, "scratch too small");
    void* scratch = nullptr;
    const int rc = scratch_for_current_device(&scratch);
    if (rc) return rc;
    // keys [m] then the counter, as marlin_q4_lm_head_argmax lays out its workspace
    if (cudaMemsetAsync(scratch, 0, (size_t)m * 8 + 16, static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        cudaGetLastError();
        return MARLIN_Q4_ERR_CUDA;
    }
    return marlin_q4_lm_head_argmax(hidden, dtype, m, norm_weight, eps, lm, vocab_offset, ids, best, keys_out,
                                    scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
