// mm3fa_noalloc.cu - mm3fa_flash_attn_ext_noalloc: the attention call for callers that
// cannot allocate device memory.
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
// is looked up once per device with cudaGetSymbolAddress on the first call made while that
// device is current, so that first call should happen before any stream capture.
//
// All calls on a device share the one buffer and it keeps the last call's contents; the
// counters the kernel needs at zero are cleared (cudaMemsetAsync on the caller's stream) at the
// start of every call.  Two calls that can run at the same time on the GPU - different streams
// without ordering between them - race on the buffer and produce wrong results.
#include "../../include/mm3fa.h"
#include "fa_common.cuh"
#include "fa_decode.cuh"

#include <cuda_runtime.h>

#include <mutex>

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MM3FA_NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;

// Device address of g_noalloc_scratch on the current device (looked up once per device).
cudaError_t scratch_address(void ** out) {
    static std::mutex mu;
    static void *     addr[MAX_DEVICES] = {};
    int               dev               = 0;
    cudaError_t       e                 = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
        return e;
    }
    if (dev < 0 || dev >= MAX_DEVICES) {
        return cudaErrorInvalidDevice;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!addr[dev]) {
        void * p = nullptr;
        e        = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) {
            return e;
        }
        addr[dev] = p;
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
    void *      scratch = nullptr;
    cudaError_t e       = scratch_address(&scratch);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_CUDA;
    }
    // The status word and the per-unit arrival counters must start at zero.  They sit at the
    // front of the workspace and take at most 512 + need/4096 bytes (every unit also reserves
    // >= 16 KiB of partial results), so for need <= the scratch size the first 64 KiB hold them.
    const size_t zero_bytes = need < (size_t) 65536 ? need : (size_t) 65536;
    if (zero_bytes > 0) {
        e = cudaMemsetAsync(scratch, 0, zero_bytes, static_cast<cudaStream_t>(stream));
        if (e != cudaSuccess) {
            cudaGetLastError();
            return MM3FA_ERR_CUDA;
        }
    }
    return mm3fa_flash_attn_ext(q, k, v, mask, scale, max_bias, logit_softcap, prec, dst, scratch,
                                (size_t) MM3FA_NOALLOC_SCRATCH_BYTES, stream);
}

}  // extern "C"
