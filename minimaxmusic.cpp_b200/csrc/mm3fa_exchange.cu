// mm3fa_exchange.cu - the multi-GPU head exchange of include/mm3fa.h: mm3fa_allgather_heads
// (NCCL), the device-side wait of the fused peer-memory exchange (mm3fa_peer_wait) and the CUDA
// IPC helpers that map the ranks' buffers into each other's processes.
//
// NCCL is resolved at the first mm3fa_allgather_heads call with dlopen("libnccl.so.2"), taking
// the copy already loaded in the process when there is one (the one torch.distributed or the
// host's own NCCL set up, which owns the communicator passed in), so single-GPU users of the
// library need no NCCL at all.  Only nccl.h's types are used at compile time.
#include "../../include/mm3fa.h"
#include "fa_common.cuh"

#include <cuda.h>
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>

#include <algorithm>
#include <cstdlib>
#include <type_traits>
#include <cstring>
#include <mutex>

namespace {

// ---------------------------------------------------------------- NCCL entry points

struct NcclApi {
    ncclResult_t (*all_gather)(const void *, void *, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
    ncclResult_t (*comm_count)(const ncclComm_t, int *)                                               = nullptr;
    ncclResult_t (*user_rank)(const ncclComm_t, int *)                                                = nullptr;
    bool ok                                                                                           = false;
};

const NcclApi & nccl() {
    static NcclApi api = [] {
        NcclApi a;
        void *  h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
        if (!h) {
            h = dlopen("libnccl.so.2", RTLD_NOW);
        }
        if (!h) {
            return a;
        }
        a.all_gather = reinterpret_cast<decltype(a.all_gather)>(dlsym(h, "ncclAllGather"));
        a.comm_count = reinterpret_cast<decltype(a.comm_count)>(dlsym(h, "ncclCommCount"));
        a.user_rank  = reinterpret_cast<decltype(a.user_rank)>(dlsym(h, "ncclCommUserRank"));
        a.ok         = a.all_gather && a.comm_count && a.user_rank;
        return a;
    }();
    return api;
}

uint64_t wait_timeout_ns() {
    static uint64_t ns = [] {
        const char * e  = std::getenv("MM3FA_WAIT_TIMEOUT_MS");
        double       ms = e ? std::atof(e) : 2000.0;
        if (!(ms > 0.0)) {
            ms = 2000.0;
        }
        return (uint64_t) (ms * 1e6);
    }();
    return ns;
}

bool aligned(const void * p, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// gathered[r][s_l][i][h_l][d] (rank r = sequence group sg * HS + head group hg) -> the ggml result
// dst[s][i][h][d] with s = sg * SL + s_l, h = hg * HL + h_l.  One block row per (sequence, query
// row) of dst (grid y, strided past 65535), threads over its n_head * dv values as float4 (VEC) or
// floats, so the index arithmetic is a few 32-bit divisions per thread.
template <bool VEC>
__global__ void scatter_gathered_kernel(const float * __restrict__ gathered, float * __restrict__ dst, int dv, int n_head,
                                        int n_q, int64_t n_rows, int sl, int head_split) {
    using T         = typename std::conditional<VEC, float4, float>::type;
    constexpr int W = VEC ? 4 : 1;
    const int     dw = dv / W;               // vectors per head row
    const int     hl = n_head / head_split;
    const int     per_row = n_head * dw;
    const T *     src = reinterpret_cast<const T *>(gathered);
    T *           out = reinterpret_cast<T *>(dst);
    for (int64_t row = blockIdx.y; row < n_rows; row += gridDim.y) {
        const int64_t s = row / n_q;
        const int     i = (int) (row % n_q);
        const int64_t sg = s / sl, s_l = s % sl;
        for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < per_row; c += gridDim.x * blockDim.x) {
            const int     h = c / dw, d = c % dw;
            const int64_t r = sg * head_split + h / hl;
            out[row * per_row + c] = src[(((r * sl + s_l) * n_q + i) * hl + h % hl) * dw + d];
        }
    }
}

// ---------------------------------------------------------------- fused exchange: the consumer's wait

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t * a) {
    uint32_t v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(a) : "memory");
    return v;
}

// One thread: waits until *flag has passed *target + expect (wrap-safe), then moves *target
// there.  Launched with programmatic stream serialisation: griddepcontrol.wait first, so that this
// kernel completes only after the kernel before it (whose results the next kernel also reads).
__global__ void peer_wait_kernel(const uint32_t * flag, uint32_t * target, uint32_t expect, uint32_t * status,
                                 uint64_t timeout_ns) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (threadIdx.x != 0) {
        return;
    }
    const uint32_t t        = *target + expect;
    const uint64_t deadline = mm3fa::global_timer_ns() + timeout_ns;
    uint32_t       spins    = 0;
    while ((int32_t) (ld_acquire_sys(flag) - t) < 0) {
        if ((++spins & 63u) == 0 && mm3fa::global_timer_ns() > deadline) {
            atomicOr(&status[0], mm3fa::ST_TIMEOUT);
            atomicExch(&status[1], 0xfffffff0u);  // where: the peer-exchange wait
            break;
        }
        __nanosleep(64);
    }
    *target = t;
}

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) {
        return MM3FA_OK;
    }
    cudaGetLastError();
    return MM3FA_ERR_CUDA;
}

using MemGetAddressRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

MemGetAddressRangeFn address_range_fn() {
    static MemGetAddressRangeFn fn = [] {
        void *                          p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess) {
            cudaGetLastError();
            return (MemGetAddressRangeFn) nullptr;
        }
        return reinterpret_cast<MemGetAddressRangeFn>(p);
    }();
    return fn;
}

// Base of the allocation (or IPC mapping) that holds p.
bool allocation_base(const void * p, char ** base) {
    MemGetAddressRangeFn fn = address_range_fn();
    CUdeviceptr          b  = 0;
    size_t               sz = 0;
    if (!fn || fn(&b, &sz, reinterpret_cast<CUdeviceptr>(p)) != CUDA_SUCCESS) {
        return false;
    }
    *base = reinterpret_cast<char *>(b);
    return true;
}

}  // namespace

extern "C" {

int mm3fa_allgather_heads(const float * slice, float * gathered, float * dst, int64_t dv, int64_t n_head, int64_t n_q,
                          int64_t n_seq, int seq_split, void * nccl_comm, void * stream) {
    if (!slice || !dst || !nccl_comm) {
        return MM3FA_ERR_NULL;
    }
    if (dv <= 0 || n_head <= 0 || n_q <= 0 || n_seq <= 0 || seq_split <= 0 || n_seq % seq_split != 0) {
        return MM3FA_ERR_SHAPE;
    }
    if (!aligned(slice, 4) || !aligned(dst, 4) || (gathered && !aligned(gathered, 4))) {
        return MM3FA_ERR_ALIGN;
    }
    const NcclApi & api = nccl();
    if (!api.ok) {
        return MM3FA_ERR_COMM;
    }
    ncclComm_t comm = static_cast<ncclComm_t>(nccl_comm);
    int        G = 0, rank = 0;
    if (api.comm_count(comm, &G) != ncclSuccess || api.user_rank(comm, &rank) != ncclSuccess || G < 1) {
        return MM3FA_ERR_COMM;
    }
    if (G % seq_split != 0 || n_head % (G / seq_split) != 0) {
        return MM3FA_ERR_SHAPE;
    }
    const int     head_split = G / seq_split;
    const size_t  count      = (size_t) (dv * (n_head / head_split) * n_q * (n_seq / seq_split));
    const bool    direct     = head_split == 1 || (seq_split == 1 && n_q * n_seq == 1);
    cudaStream_t  cs         = static_cast<cudaStream_t>(stream);
    float *       out        = direct ? dst : gathered;
    if (!out) {
        return MM3FA_ERR_WORKSPACE;
    }
    // the all-gather may run in place (slice at its rank's position of the output); any other
    // overlap of the input with the gathered buffer is rejected
    const char * in_b = reinterpret_cast<const char *>(slice), *out_b = reinterpret_cast<const char *>(out);
    const size_t bytes = count * sizeof(float);
    const bool   in_place = in_b == out_b + (size_t) rank * bytes;
    if (!in_place && in_b < out_b + bytes * (size_t) G && out_b < in_b + bytes) {
        return MM3FA_ERR_SHAPE;
    }
    if (api.all_gather(slice, out, count, ncclFloat32, comm, cs) != ncclSuccess) {
        return MM3FA_ERR_COMM;
    }
    if (direct) {
        return MM3FA_OK;
    }
    if (dv * n_head > (int64_t) 1 << 30 || n_q > (int64_t) 1 << 30) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    const bool    vec     = dv % 4 == 0 && aligned(gathered, 16) && aligned(dst, 16);
    const int64_t per_row = dv * n_head / (vec ? 4 : 1);
    const dim3    grid((unsigned) std::min<int64_t>((per_row + 255) / 256, 64),
                       (unsigned) std::min<int64_t>(n_q * n_seq, 65535));
    const int     sl = (int) (n_seq / seq_split);
    if (vec) {
        scatter_gathered_kernel<true><<<grid, 256, 0, cs>>>(gathered, dst, (int) dv, (int) n_head, (int) n_q,
                                                             n_q * n_seq, sl, head_split);
    } else {
        scatter_gathered_kernel<false><<<grid, 256, 0, cs>>>(gathered, dst, (int) dv, (int) n_head, (int) n_q,
                                                              n_q * n_seq, sl, head_split);
    }
    return cuda_status(cudaGetLastError());
}

int mm3fa_peer_wait(const mm3fa_peers * peers, int slot, uint32_t * targets, void * workspace, void * stream) {
    if (!peers || !targets || !workspace) {
        return MM3FA_ERR_NULL;
    }
    if (peers->n_ranks < 2 || peers->n_ranks > MM3FA_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->n_ranks ||
        slot < 0 || !peers->flags[peers->rank]) {
        return MM3FA_ERR_SHAPE;
    }
    cudaLaunchConfig_t  cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim                                        = dim3(1);
    cfg.blockDim                                       = dim3(32);
    cfg.stream                                         = static_cast<cudaStream_t>(stream);
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_wait_kernel, (const uint32_t *) (peers->flags[peers->rank] + slot),
                                          targets + slot, (uint32_t) (peers->n_ranks - 1),
                                          static_cast<uint32_t *>(workspace), wait_timeout_ns()));
}

int mm3fa_ipc_export(const void * dev_ptr, mm3fa_ipc_handle * out) {
    if (!dev_ptr || !out) {
        return MM3FA_ERR_NULL;
    }
    char * base = nullptr;
    if (!allocation_base(dev_ptr, &base)) {
        return MM3FA_ERR_COMM;
    }
    cudaIpcMemHandle_t h;
    if (cudaIpcGetMemHandle(&h, base) != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_COMM;
    }
    static_assert(sizeof(h) <= sizeof(out->handle), "IPC handle size");
    std::memset(out->handle, 0, sizeof(out->handle));
    std::memcpy(out->handle, &h, sizeof(h));
    out->offset = (uint64_t) (static_cast<const char *>(dev_ptr) - base);
    return MM3FA_OK;
}

int mm3fa_ipc_open(const mm3fa_ipc_handle * h, void ** dev_ptr_out) {
    if (!h || !dev_ptr_out) {
        return MM3FA_ERR_NULL;
    }
    cudaIpcMemHandle_t mh;
    std::memcpy(&mh, h->handle, sizeof(mh));
    void * base = nullptr;
    if (cudaIpcOpenMemHandle(&base, mh, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_COMM;
    }
    *dev_ptr_out = static_cast<char *>(base) + h->offset;
    return MM3FA_OK;
}

int mm3fa_ipc_close(void * dev_ptr) {
    if (!dev_ptr) {
        return MM3FA_ERR_NULL;
    }
    char * base = nullptr;
    if (!allocation_base(dev_ptr, &base)) {
        return MM3FA_ERR_COMM;
    }
    if (cudaIpcCloseMemHandle(base) != cudaSuccess) {
        cudaGetLastError();
        return MM3FA_ERR_COMM;
    }
    return MM3FA_OK;
}

}  // extern "C"
