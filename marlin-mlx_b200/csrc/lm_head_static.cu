// lm_head_static.cu — marlin_q4_lm_head_argmax_static: the fused lm_head + argmax without a
// caller-provided workspace.
//
// Who needs it: callers that cannot allocate or own device scratch for this call.  The reference's
// own call shape is one of them: MarlinModel::lm_head followed by sample_token
// (src/model/marlin.cpp:161-169, src/sampling/sampler.cpp:14-16) passes only the hidden state and
// the weights, so a binding that replaces those two calls has no buffer to hand over, and adding a
// cudaMalloc there would synchronise the device inside the decode loop.  Bindings from runtimes
// that do not manage device memory themselves are in the same position.
//
// How: the argmax keys and the CTA-completion counter live in one file-scope device array
// (kStaticScratchBytes, room for kStaticMaxRows rows).  Its address is looked up once per device
// with cudaGetSymbolAddress, with that device current, and handed to the kernels as a plain
// pointer.  The array starts zeroed when the module loads, and every call leaves the keys and the
// counter zeroed again, which is what the next call needs.  Nothing is allocated: no cudaMalloc,
// no cudaFree, no allocating library routine.
//
// Limits: m <= kStaticMaxRows (larger m returns MARLIN_Q4_ERR_UNSUPPORTED before any CUDA call).
// All calls on a device share the one array, so two calls that may run at the same time on that
// device (different streams, or different host threads without ordering) race on the keys and give
// wrong ids; order them on one stream.  The first call on each device performs the symbol lookup
// and must happen outside stream capture.
#include "marlin_q4.h"

#include <cuda_runtime.h>

#include <mutex>

namespace {

constexpr int64_t kStaticMaxRows = MARLIN_Q4_LM_HEAD_STATIC_MAX_ROWS;
// keys [kStaticMaxRows] u64 + counter, rounded up to 256 bytes: 768 bytes
constexpr size_t kStaticScratchBytes = ((size_t)kStaticMaxRows * 8 + 16 + 255) / 256 * 256;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_lm_static_scratch[kStaticScratchBytes];

std::mutex g_scratch_mutex;
void* g_scratch_ptr[kMaxDevices] = {};

// Device address of the scratch array on the current device (looked up once per device).
int scratch_for_current_device(void** out) {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) {
        cudaGetLastError();
        return MARLIN_Q4_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_ptr[dev]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_lm_static_scratch) != cudaSuccess || !p) {
            cudaGetLastError();
            return MARLIN_Q4_ERR_CUDA;
        }
        g_scratch_ptr[dev] = p;
    }
    *out = g_scratch_ptr[dev];
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
    return marlin_q4_lm_head_argmax(hidden, dtype, m, norm_weight, eps, lm, vocab_offset, ids, best, keys_out,
                                    scratch, kStaticScratchBytes, stream);
}

}  // extern "C"
