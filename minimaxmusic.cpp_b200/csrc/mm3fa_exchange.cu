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

// ---------------------------------------------------------------- fused exchange: the consumer's side

__device__ __forceinline__ uint4 ld_volatile_v4(const char * a) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(a)
                 : "memory");
    return v;
}

// Unpacks every other rank's slice of the latest call on a slot from this rank's receive buffer
// into the whole result.  Item t = (source s', value pair j): the 16-byte line {v0, epoch, v1,
// epoch} of values 2j, 2j+1 of source rank r (r != self), polled until both epochs match (bounded),
// then written to result at (d, r*hl + h_l, i, seq).  The last CTA to finish advances the slot's
// epoch.  Launched with programmatic stream serialisation: griddepcontrol.wait first, so the
// attention call before it (which read the epoch) has completed.  It lets the next kernel in the
// stream launch at once (that kernel's own griddepcontrol.wait still waits for this grid's
// completion), so the next layer's CTAs are resident and set up while this one polls.
struct UnpackParams {
    const char * recv;     // this rank's receive buffer, slot base
    char *       result;   // this rank's whole result [Dv, H, n_q, n_seq]
    int64_t      nb1, nb2, nb3;
    int64_t      parity;   // bytes of one parity half of the slot
    int64_t      region;   // bytes of one source region
    int64_t      vals;     // values of one slice (Dv * hl * n_q * n_seq)
    int          dv, hl, n_q, n_ranks, rank;
    uint32_t *   epoch;    // &epochs[slot]
    uint32_t *   status;   // workspace status word; status[WS_PEER_ARRIVE] counts finished CTAs
    uint64_t     timeout_ns;
};

__global__ void __launch_bounds__(256) peer_unpack_kernel(const UnpackParams p) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const uint32_t e      = *p.epoch + 1u;
    const int64_t  pairs  = p.vals / 2;
    const int64_t  items  = pairs * (p.n_ranks - 1);
    const char *   base   = p.recv + (int64_t) (e & 1u) * p.parity;
    const uint64_t dl     = mm3fa::global_timer_ns() + p.timeout_ns;
    bool           failed = false;
    for (int64_t t = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; t < items && !failed;
         t += (int64_t) gridDim.x * blockDim.x) {
        const int     sp = (int) (t / pairs);
        const int     r  = sp < p.rank ? sp : sp + 1;  // source rank (this rank skipped)
        const int64_t j  = t % pairs;
        const char *  line = base + r * p.region + 16 * j;
        uint4         w    = ld_volatile_v4(line);
        uint32_t      spins = 0;
        while (w.y != e || w.w != e) {
            if ((++spins & 63u) == 0 && mm3fa::global_timer_ns() > dl) {
                atomicOr(&p.status[0], mm3fa::ST_TIMEOUT);
                atomicExch(&p.status[1], 0xfffffff0u);  // where: the peer-exchange wait
                failed = true;
                break;
            }
            __nanosleep(32);
            w = ld_volatile_v4(line);
        }
        if (failed) {
            break;
        }
        const int64_t v0  = 2 * j;  // d, h_l, i, seq of the pair's first value (dv is even)
        const int     d   = (int) (v0 % p.dv);
        const int64_t rest = v0 / p.dv;
        const int     h_l = (int) (rest % p.hl);
        const int64_t rest2 = rest / p.hl;
        const int     i   = (int) (rest2 % p.n_q);
        const int64_t sq  = rest2 / p.n_q;
        float * dst = reinterpret_cast<float *>(p.result + (int64_t) (r * p.hl + h_l) * p.nb1 + (int64_t) i * p.nb2 +
                                                sq * p.nb3) + d;
        *reinterpret_cast<float2 *>(dst) = make_float2(__uint_as_float(w.x), __uint_as_float(w.z));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        const uint32_t old = atomicAdd(&p.status[mm3fa::WS_PEER_ARRIVE], 1u);
        if (old + 1u == gridDim.x) {
            p.status[mm3fa::WS_PEER_ARRIVE] = 0u;
            *p.epoch                        = e;
        }
    }
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

// Completion step of the fused dense exchange (mm3fa_flash_attn_ext_gather): launched after that
// rank's attention kernel in stream order, so the kernel's stores into the other ranks' results have
// been performed.  Lane 0 fences at system scope and stores the call's epoch into every other
// rank's flag word [slot][this rank] with release semantics; lane s (s != this rank) polls this
// rank's word [slot][s] with acquire loads, bounded by the global timer, until rank s's epoch of the
// call is there.  The epoch is the slot's call count + 1, advanced here.
struct SignalParams {
    uint32_t * flags[MM3FA_MAX_RANKS];  // every rank's flag array [n_slots][n_ranks]
    int        n_ranks, rank, slot;
    uint32_t * epoch;   // &epochs[slot]
    uint32_t * status;  // workspace status word
    uint64_t   timeout_ns;
};

__global__ void __launch_bounds__(32) gather_signal_wait_kernel(const SignalParams p) {
    const int      lane = threadIdx.x;
    const uint32_t e    = *p.epoch + 1u;
    if (lane == 0) {
        asm volatile("fence.sc.sys;" ::: "memory");
        for (int r = 0; r < p.n_ranks; r++) {
            if (r != p.rank) {
                uint32_t * f = p.flags[r] + (int64_t) p.slot * p.n_ranks + p.rank;
                asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(f), "r"(e) : "memory");
            }
        }
    }
    bool failed = false;
    if (lane < p.n_ranks && lane != p.rank) {
        const uint32_t * f  = p.flags[p.rank] + (int64_t) p.slot * p.n_ranks + lane;
        const uint64_t   dl = mm3fa::global_timer_ns() + p.timeout_ns;
        uint32_t         spins = 0;
        for (;;) {
            uint32_t v;
            asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(f) : "memory");
            if ((int32_t) (v - e) >= 0) {
                break;
            }
            if ((++spins & 63u) == 0 && mm3fa::global_timer_ns() > dl) {
                failed = true;
                break;
            }
            __nanosleep(64);
        }
    }
    if (failed) {
        atomicOr(&p.status[0], mm3fa::ST_TIMEOUT);
        atomicExch(&p.status[1], 0xfffffff1u);  // where: the dense exchange's wait
    }
    __syncwarp();
    if (lane == 0) {
        *p.epoch = e;
    }
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

int mm3fa_peer_wait(const mm3fa_peers * peers, int slot, uint32_t * epochs, mm3fa_tensor * result, void * workspace,
                    void * stream) {
    if (!peers || !epochs || !workspace || !result || !result->data) {
        return MM3FA_ERR_NULL;
    }
    if (peers->n_ranks < 2 || peers->n_ranks > MM3FA_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->n_ranks ||
        slot < 0 || !peers->recv[peers->rank]) {
        return MM3FA_ERR_SHAPE;
    }
    if (result->type != MM3FA_TYPE_F32) {
        return MM3FA_ERR_TYPE;
    }
    const int64_t dv = result->ne[0], H = result->ne[1], n_q = result->ne[2], n_seq = result->ne[3];
    if (dv <= 0 || dv % 2 || H <= 0 || H % peers->n_ranks || n_q <= 0 || n_seq <= 0 || dv > 4096 || H > 65535 ||
        n_q > 65535 || n_seq > 65535) {
        return MM3FA_ERR_SHAPE;
    }
    if (result->nb[0] != 4 || result->nb[1] % 8 || result->nb[2] % 8 || result->nb[3] % 8 ||
        !aligned(result->data, 8)) {
        return MM3FA_ERR_STRIDE;
    }
    UnpackParams p{};
    p.hl      = (int) (H / peers->n_ranks);
    p.vals    = dv * p.hl * n_q * n_seq;
    p.region  = 8 * p.vals;
    p.parity  = (int64_t) peers->n_ranks * p.region;
    if ((uint64_t) (2 * p.parity) > peers->recv_slot_bytes) {
        return MM3FA_ERR_WORKSPACE;
    }
    p.recv       = static_cast<const char *>(peers->recv[peers->rank]) + (uint64_t) slot * peers->recv_slot_bytes;
    p.result     = static_cast<char *>(result->data);
    p.nb1        = (int64_t) result->nb[1];
    p.nb2        = (int64_t) result->nb[2];
    p.nb3        = (int64_t) result->nb[3];
    p.dv         = (int) dv;
    p.n_q        = (int) n_q;
    p.n_ranks    = peers->n_ranks;
    p.rank       = peers->rank;
    p.epoch      = epochs + slot;
    p.status     = static_cast<uint32_t *>(workspace);
    p.timeout_ns = wait_timeout_ns();
    const int64_t items  = p.vals / 2 * (p.n_ranks - 1);
    const int     blocks = (int) std::max<int64_t>(1, std::min<int64_t>((items + 255) / 256, 148));
    cudaLaunchConfig_t  cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim                                        = dim3((unsigned) blocks);
    cfg.blockDim                                       = dim3(256);
    cfg.stream                                         = static_cast<cudaStream_t>(stream);
    attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs                                          = attr;
    cfg.numAttrs                                       = 1;
    // the next layer's attention CTAs become resident beside this kernel's (early trigger): the SMs
    // this kernel runs on keep the largest shared-memory carve-out, so two of those CTAs still fit
    static const cudaError_t carve = [] {
        const cudaError_t e = cudaFuncSetAttribute(peer_unpack_kernel, cudaFuncAttributePreferredSharedMemoryCarveout,
                                                   (int) cudaSharedmemCarveoutMaxShared);
        cudaGetLastError();
        return e;
    }();
    (void) carve;
    return cuda_status(cudaLaunchKernelEx(&cfg, peer_unpack_kernel, p));
}

int mm3fa_gather_signal_wait(const mm3fa_peers * flags, int slot, uint32_t * epochs, void * workspace, void * stream) {
    if (!flags || !epochs || !workspace) {
        return MM3FA_ERR_NULL;
    }
    if (flags->n_ranks < 2 || flags->n_ranks > MM3FA_MAX_RANKS || flags->rank < 0 ||
        flags->rank >= flags->n_ranks || slot < 0) {
        return MM3FA_ERR_SHAPE;
    }
    // recv_slot_bytes: the bytes of each rank's flag array, which holds [n_slots][n_ranks] words
    if ((uint64_t) (slot + 1) * (uint64_t) flags->n_ranks * 4u > flags->recv_slot_bytes) {
        return MM3FA_ERR_SHAPE;
    }
    SignalParams p{};
    for (int r = 0; r < flags->n_ranks; r++) {
        if (!flags->recv[r]) {
            return MM3FA_ERR_NULL;
        }
        if (!aligned(flags->recv[r], 4)) {
            return MM3FA_ERR_ALIGN;
        }
        p.flags[r] = static_cast<uint32_t *>(flags->recv[r]);
    }
    if (!aligned(epochs, 4)) {
        return MM3FA_ERR_ALIGN;
    }
    p.n_ranks    = flags->n_ranks;
    p.rank       = flags->rank;
    p.slot       = slot;
    p.epoch      = epochs + slot;
    p.status     = static_cast<uint32_t *>(workspace);
    p.timeout_ns = wait_timeout_ns();
    gather_signal_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
    return cuda_status(cudaGetLastError());
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
