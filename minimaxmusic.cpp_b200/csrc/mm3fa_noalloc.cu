// mm3fa_noalloc.cu - mm3fa_flash_attn_ext_noalloc: the attention call for callers that
// cannot allocate device memory, and mm3fa_noalloc_status, which reads its status word.
//
// Some hosts of this operator are not allowed to call cudaMalloc at the point where they
// run attention: a ggml backend whose buffers were all sized up front by ggml_gallocr, an
// engine that records its steps into a CUDA graph and forbids allocation while recording,
// or a plugin running under a strict memory budget that owns no allocator.  They can still
// pass inputs and outputs, but not the split-KV scratch workspace.  This entry point takes
// the scratch from a fixed buffer compiled into the library instead.
//
// The buffer is the file-scope device array below, MM3FA_NOALLOC_SCRATCH_BYTES in size.  Every
// GPU that loads the library holds one copy of it until the process exits.  Host code must not
// pass the array's name to a kernel (on the host it only names a stand-in); the device address
// is looked up with cudaGetSymbolAddress on the first call made while a device (more exactly:
// a CUDA context) is current, so that first call should happen before any stream capture.  The
// address is cached per device together with the context it was looked up in, and looked up
// again when the device's current context is a different one (after cudaDeviceReset).
//
// Layout (the workspace layout of mm3fa_flash_attn_ext): a 256-byte status word, then the
// decode kernels' per-unit arrival counters, then partial results.  Every call clears the
// counter region its operands use (cudaMemsetAsync on the caller's stream) and nothing else;
// the status word is left as it is so that a bounded wait that expired inside a call stays
// visible until mm3fa_noalloc_status reads and clears it.  All calls on a device share the one
// buffer and it keeps the last call's contents.  Two calls that can run at the same time on
// the GPU - different streams without ordering between them - race on the buffer and produce
// wrong results.
#include "../../include/mm3fa.h"
#include "fa_common.cuh"
#include "fa_decode.cuh"

#include <cuda.h>
#include <cuda_runtime.h>

#include <mutex>

namespace mm3fa {
// defined in mm3fa_abi.cu: bytes after the status word a call needs zeroed
size_t workspace_counter_bytes(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                               const mm3fa_tensor * mask, const mm3fa_tensor * dst);
}  // namespace mm3fa

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MM3FA_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;

using CtxGetCurrentFn = CUresult (*)(CUcontext *);

// The current CUDA context, or nullptr when it cannot be queried.
CUcontext current_context() {
    static CtxGetCurrentFn fn = [] {
        void *                          p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (CtxGetCurrentFn) nullptr;
        }
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    CUcontext c = nullptr;
    if (fn && fn(&c) != CUDA_SUCCESS) {
        c = nullptr;
    }
    return c;
}

// Device address of g_noalloc_scratch in the current device's context.  The first lookup in a
// context also clears the status word (on `stream`), so every context starts from "no error".
cudaError_t scratch_address(void ** out, cudaStream_t stream) {
    static std::mutex mu;
    static void *     addr[MAX_DEVICES] = {};
    static CUcontext  ctx[MAX_DEVICES]  = {};
    int               dev               = 0;
    cudaError_t       e                 = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return e;
    }
    if (dev < 0 || dev >= MAX_DEVICES) {
        return cudaErrorInvalidDevice;
    }
    std::lock_guard<std::mutex> lock(mu);
    CUcontext                   cur = current_context();  // nullptr before the device's first use
    if (!cur || !addr[dev] || ctx[dev] != cur) {
        // the lookup also creates the device's primary context when none is current yet
        void * p = nullptr;
        e        = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            return e;
        }
        cur = current_context();
        if (!addr[dev] || ctx[dev] != cur) {
            if ((e = cudaMemsetAsync(p, 0, mm3fa::WS_STATUS_BYTES, stream)) != cudaSuccess) {
                return e;
            }
            addr[dev] = p;
            ctx[dev]  = cur;
        }
    }
    *out = addr[dev];
    return cudaSuccess;
}

}  // namespace

extern "C" {

int mm3fa_flash_attn_ext_noalloc(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                 const mm3fa_tensor * mask, float scale, float max_bias, float logit_softcap,
                                 int prec, mm3fa_tensor * dst, void * stream) {
    // contract checks first: nothing is enqueued for operands the ABI would reject
    int st = mm3fa_supports(q, k, v, mask, max_bias, logit_softcap, dst);
    if (st != MM3FA_OK) {
        return st;
    }
    const size_t need = mm3fa_workspace_size(q, k, v, mask, dst);
    if (need > (size_t) MM3FA_NOALLOC_SCRATCH_BYTES) {
        return MM3FA_ERR_SCRATCH_LIMIT;
    }
    cudaStream_t cs      = static_cast<cudaStream_t>(stream);
    void *       scratch = nullptr;
    cudaError_t  e       = scratch_address(&scratch, cs);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_CUDA;
    }
    // the arrival counters of this call's decode geometry must start at zero (earlier calls
    // may have used the region for partial results); the status word is kept
    const size_t counters = mm3fa::workspace_counter_bytes(q, k, v, mask, dst);
    if (counters > 0) {
        e = cudaMemsetAsync(static_cast<char *>(scratch) + mm3fa::WS_STATUS_BYTES, 0, counters, cs);
        if (e != cudaSuccess) {
            cudaGetLastError();
            return MM3FA_ERR_CUDA;
        }
    }
    return mm3fa_flash_attn_ext(q, k, v, mask, scale, max_bias, logit_softcap, prec, dst, scratch,
                                (size_t) MM3FA_NOALLOC_SCRATCH_BYTES, stream);
}

int mm3fa_noalloc_status(void * stream, uint32_t * status_out) {
    if (!status_out) {
        return MM3FA_ERR_NULL;
    }
    void *      scratch = nullptr;
    cudaError_t e       = scratch_address(&scratch, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_CUDA;
    }
    return mm3fa_workspace_status(scratch, stream, status_out);
}

int mm3fa_noalloc_selftest_bounded_wait(uint32_t timeout_us, void * stream) {
    void *      scratch = nullptr;
    cudaError_t e       = scratch_address(&scratch, static_cast<cudaStream_t>(stream));
    if (e != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_CUDA;
    }
    return mm3fa_selftest_bounded_wait(scratch, timeout_us, stream);
}

}  // extern "C"
