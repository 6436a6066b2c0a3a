// mm3fa_abi.cu - the C ABI declared in include/mm3fa.h.
//
// Validates ggml tensor descriptors against the GGML_OP_FLASH_ATTN_EXT contract, sizes the
// caller-owned workspace, and enqueues the kernels on the caller's stream.  Nothing here
// allocates device memory or synchronises the host, except mm3fa_workspace_status, which
// reads the status word back by design.
#include "../../include/mm3fa.h"
#include "fa_common.cuh"
#include "fa_decode.cuh"
#include "fa_dense.cuh"
#include "fa_prologue.cuh"

#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>

using namespace mm3fa;

namespace {

thread_local char g_last_cuda_error[256] = "";

int record_cuda(cudaError_t e) {
    if (e == cudaSuccess) {
        return MM3FA_OK;
    }
    std::snprintf(g_last_cuda_error, sizeof(g_last_cuda_error), "%s: %s", cudaGetErrorName(e),
                  cudaGetErrorString(e));
    return MM3FA_ERR_CUDA;
}

int64_t type_unit_bytes(int t) {
    switch (t) {
        case MM3FA_TYPE_F32:
            return 4;
        case MM3FA_TYPE_F16:
        case MM3FA_TYPE_BF16:
            return 2;
        case MM3FA_TYPE_Q8_0:
            return Q8_0_BLOCK;
        default:
            return 0;
    }
}

int64_t row_bytes(int t, int64_t n) {
    if (t == MM3FA_TYPE_Q8_0) {
        return n / QK8_0 * Q8_0_BLOCK;
    }
    return type_unit_bytes(t) * n;
}

// Per-device facts cached once: SM count, compute capability.
struct DeviceInfo {
    int sms   = 0;
    int major = 0;
    int minor = 0;
};

DeviceInfo device_info() {
    static std::mutex mu;
    static DeviceInfo cache[64];
    int               dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) {
        cudaGetLastError();
        return DeviceInfo{};
    }
    std::lock_guard<std::mutex> lock(mu);
    if (cache[dev].sms == 0) {
        cudaDeviceGetAttribute(&cache[dev].sms, cudaDevAttrMultiProcessorCount, dev);
        cudaDeviceGetAttribute(&cache[dev].major, cudaDevAttrComputeCapabilityMajor, dev);
        cudaDeviceGetAttribute(&cache[dev].minor, cudaDevAttrComputeCapabilityMinor, dev);
        cudaGetLastError();
    }
    return cache[dev];
}

// Decode kernel variants: the CUDA-core kernel with bulk or element copies, and the
// tensor-core kernel with 8 or 16 rows per unit.
enum Variant { V_SIMT_BULK = 0, V_SIMT_COPY = 1, V_MMA_8 = 2, V_MMA_16 = 3 };

int ctas_per_sm_cached(int D, int kvt, Variant var) {
    static std::mutex mu;
    static int        cache[64][3][4][4];  // [dev][D 64/128/256][type idx][variant]
    int               dev = 0;
    cudaGetDevice(&dev);
    const int ti = kvt == MM3FA_TYPE_F16 ? 0 : (kvt == MM3FA_TYPE_BF16 ? 1 : (kvt == MM3FA_TYPE_Q8_0 ? 2 : 3));
    const int di = D == 64 ? 0 : (D == 128 ? 1 : 2);
    std::lock_guard<std::mutex> lock(mu);
    int & c = cache[dev & 63][di][ti][var];
    if (c == 0) {
        c = var >= V_MMA_8 ? decode_mma_ctas_per_sm(D, kvt, var == V_MMA_8 ? 8 : 16)
                           : decode_ctas_per_sm(D, kvt, var == V_SIMT_BULK);
    }
    return c;
}

// MM3FA_DECODE_SPLIT=streamk|auto (default auto): the tensor-core kernel's work split;
// auto uses thread-block clusters when there are enough units to fill the GPU.
int decode_mma_mode_preference() {
    const char * e = std::getenv("MM3FA_DECODE_SPLIT");
    return (e && std::strcmp(e, "streamk") == 0) ? 1 : 0;
}

// MM3FA_DECODE=simt|mma|auto (default auto) selects the decode kernel where both apply.
int decode_preference() {
    const char * e = std::getenv("MM3FA_DECODE");
    if (e && std::strcmp(e, "simt") == 0) {
        return 1;
    }
    if (e && std::strcmp(e, "mma") == 0) {
        return 2;
    }
    return 0;
}

// MM3FA_DENSE=0|1|auto (default auto): 0 never runs the tensor-core prefill kernel, 1 runs it
// whenever the operands allow, auto from DENSE_MIN_ROWS query rows on.
int dense_preference() {
    const char * e = std::getenv("MM3FA_DENSE");
    if (e && std::strcmp(e, "0") == 0) {
        return 0;
    }
    if (e && std::strcmp(e, "1") == 0) {
        return 1;
    }
    return 2;
}

constexpr int64_t DENSE_MIN_ROWS = 64;

uint64_t wait_timeout_ns() {
    static uint64_t ns = [] {
        const char * e = std::getenv("MM3FA_WAIT_TIMEOUT_MS");
        double       ms = e ? std::atof(e) : 2000.0;
        if (!(ms > 0.0)) {
            ms = 2000.0;
        }
        return (uint64_t) (ms * 1e6);
    }();
    return ns;
}

// Everything the dispatcher derives from the descriptors.
struct OpShape {
    int64_t D, DV, n_q, n_head, n_seq, n_kv, n_head_kv, n_seq_k;
    int     ratio, rk3;
    int     kvt;
    int     key_align;  // key granularity that keeps 1-D bulk copies 16-byte aligned
    bool    bulk;
    bool    tma;        // strides and base addresses a TMA tensor map can express
};

bool aligned(const void * p, uintptr_t a) {
    return (reinterpret_cast<uintptr_t>(p) % a) == 0;
}

// Host-side contract check.  check_data: also validate data pointers.
int check_op(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v, const mm3fa_tensor * mask,
             float max_bias, float softcap, const mm3fa_tensor * dst, bool check_data, OpShape & s) {
    if (!q || !k || !v || !dst) {
        return MM3FA_ERR_NULL;
    }
    if (check_data && (!q->data || !k->data || !v->data || !dst->data || (mask && !mask->data))) {
        return MM3FA_ERR_NULL;
    }
    // types
    if (q->type != MM3FA_TYPE_F32 && q->type != MM3FA_TYPE_F16 && q->type != MM3FA_TYPE_BF16) {
        return MM3FA_ERR_TYPE;
    }
    if (k->type != MM3FA_TYPE_F16 && k->type != MM3FA_TYPE_BF16 && k->type != MM3FA_TYPE_Q8_0 &&
        k->type != MM3FA_TYPE_F32) {
        return MM3FA_ERR_TYPE;
    }
    if (v->type != k->type || dst->type != MM3FA_TYPE_F32 || (mask && mask->type != MM3FA_TYPE_F16)) {
        return MM3FA_ERR_TYPE;
    }
    for (const mm3fa_tensor * t : { q, k, v, dst }) {
        for (int i = 0; i < 4; i++) {
            if (t->ne[i] < 0) {
                return MM3FA_ERR_SHAPE;
            }
        }
    }
    // shapes (ggml_flash_attn_ext's contract)
    s.D         = q->ne[0];
    s.n_q       = q->ne[1];
    s.n_head    = q->ne[2];
    s.n_seq     = q->ne[3];
    s.DV        = v->ne[0];
    s.n_kv      = k->ne[1];
    s.n_head_kv = k->ne[2];
    s.n_seq_k   = k->ne[3];
    s.kvt       = k->type;
    if (k->ne[0] != s.D || v->ne[1] != s.n_kv || v->ne[2] != s.n_head_kv || v->ne[3] != s.n_seq_k) {
        return MM3FA_ERR_SHAPE;
    }
    if (s.n_head_kv == 0 || s.n_seq_k == 0 || s.n_head % s.n_head_kv != 0 || s.n_seq % s.n_seq_k != 0) {
        return MM3FA_ERR_SHAPE;
    }
    if (dst->ne[0] != s.DV || dst->ne[1] != s.n_head || dst->ne[2] != s.n_q || dst->ne[3] != s.n_seq) {
        return MM3FA_ERR_SHAPE;
    }
    if (mask) {
        if (mask->ne[0] != s.n_kv || mask->ne[1] < s.n_q || mask->ne[2] < 1 || mask->ne[3] < 1 ||
            s.n_head % mask->ne[2] != 0 || s.n_seq % mask->ne[3] != 0) {
            return MM3FA_ERR_SHAPE;
        }
    }
    if (s.kvt == MM3FA_TYPE_Q8_0 && s.D % QK8_0 != 0) {
        return MM3FA_ERR_SHAPE;
    }
    if (!std::isfinite(max_bias) || !std::isfinite(softcap) || max_bias < 0.0f) {
        return MM3FA_ERR_SHAPE;
    }
    // strides: innermost dims packed, the rest multiples of the element (block) size
    const int64_t qe = type_unit_bytes(q->type), ke = type_unit_bytes(k->type);
    if ((int64_t) q->nb[0] != qe || (int64_t) k->nb[0] != ke || (int64_t) v->nb[0] != ke ||
        (int64_t) dst->nb[0] != 4 || (mask && mask->nb[0] != 2)) {
        return MM3FA_ERR_STRIDE;
    }
    const uint64_t kva = k->type == MM3FA_TYPE_F32 ? 4 : 2;  // K/V element alignment
    for (int i = 1; i < 4; i++) {
        if (q->nb[i] % (uint64_t) qe || k->nb[i] % kva || v->nb[i] % kva || dst->nb[i] % 4 ||
            (mask && mask->nb[i] % 2)) {
            return MM3FA_ERR_STRIDE;
        }
    }
    if ((int64_t) k->nb[1] < row_bytes(k->type, s.D) || (int64_t) v->nb[1] < row_bytes(v->type, s.DV) ||
        (int64_t) dst->nb[1] < 4 * s.DV) {
        return MM3FA_ERR_STRIDE;
    }
    if (check_data) {
        if (!aligned(q->data, (uintptr_t) qe) || !aligned(k->data, kva) || !aligned(v->data, kva) ||
            !aligned(dst->data, 4) || (mask && !aligned(mask->data, 2))) {
            return MM3FA_ERR_ALIGN;
        }
    }
    // what the kernels here implement
    // D = 256 (the depth decoder's heads) runs on the CUDA-core decode kernel
    if (s.DV != s.D || (s.D != 64 && s.D != 128 && s.D != 256)) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    // index math in the kernels uses 32-bit unit numbers and key counts
    if (s.n_kv > (int64_t) 0x7fffffff || s.n_q > 65535 || s.n_head > 65535 ||
        s.n_seq * s.n_head_kv * ((s.n_head / s.n_head_kv) * s.n_q / 32 + 1) > (int64_t) 0x7fffffff) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    s.ratio = (int) (s.n_head / s.n_head_kv);
    s.rk3   = (int) (s.n_seq / s.n_seq_k);
    // bulk (TMA engine) copies need 16-byte aligned starts and sizes for every chunk
    const int64_t rb = row_bytes(s.kvt, s.D);
    int           u  = 1;
    while ((rb * u) % 16 != 0) {
        u *= 2;
    }
    s.key_align = u;
    bool bulk   = (int64_t) k->nb[1] == rb && (int64_t) v->nb[1] == rb && s.n_kv % u == 0;
    for (const mm3fa_tensor * t : { k, v }) {
        if (t->ne[2] > 1 && t->nb[2] % 16) {
            bulk = false;
        }
        if (t->ne[3] > 1 && t->nb[3] % 16) {
            bulk = false;
        }
        if (check_data && !aligned(t->data, 16)) {
            bulk = false;
        }
    }
    s.bulk = bulk;
    // TMA tensor maps: 16-byte aligned base and strides (nb1 included), extents < 2^32
    bool tma = k->nb[1] % 16 == 0 && v->nb[1] % 16 == 0 && s.n_kv > 0;
    for (const mm3fa_tensor * t : { k, v }) {
        if ((t->ne[2] > 1 && t->nb[2] % 16) || (t->ne[3] > 1 && t->nb[3] % 16)) {
            tma = false;
        }
        if (check_data && !aligned(t->data, 16)) {
            tma = false;
        }
    }
    s.tma = tma;
    return MM3FA_OK;
}

// The decode kernel a call with these operands runs.
Variant variant_for(const OpShape & s) {
    const int  pref = decode_preference();
    const int  rows = s.ratio * (int) s.n_q;
    // F16/BF16 stages are TMA tensor tiles; Q8_0 rows (not 16-byte multiples) are bulk copies
    const bool tiles = s.kvt == MM3FA_TYPE_Q8_0 ? s.bulk : s.tma;
    const bool mma   = pref != 1 && tiles && decode_mma_eligible((int) s.D, s.kvt, rows);
    if (mma) {
        return rows <= 8 ? V_MMA_8 : V_MMA_16;
    }
    return s.bulk ? V_SIMT_BULK : V_SIMT_COPY;
}

DecodeGeometry geometry_for(const OpShape & s, Variant var) {
    const DeviceInfo di  = device_info();
    const int        cps = ctas_per_sm_cached((int) s.D, s.kvt, var);
    return decode_geometry((int) s.n_seq, (int) s.n_head_kv, s.ratio, (int) s.n_q, (int) s.n_kv, s.key_align,
                           di.sms, cps);
}

// The tensor-core prefill kernel can take these operands.
bool dense_applicable(const OpShape & s, const mm3fa_tensor * mask) {
    if (!s.tma || !dense_eligible((int) s.D, s.kvt) || s.n_seq > 65535) {
        return false;
    }
    return !mask || mask->ne[2] * mask->ne[3] <= 65535;
}

bool use_dense(const OpShape & s, const mm3fa_tensor * mask) {
    const int pref = dense_preference();
    if (pref == 0 || !dense_applicable(s, mask)) {
        return false;
    }
    return pref == 1 || s.n_q >= DENSE_MIN_ROWS;
}

bool rows_vec16(const mm3fa_tensor * t) {
    return aligned(t->data, 16) && t->nb[1] % 16 == 0 && t->nb[2] % 16 == 0 && t->nb[3] % 16 == 0;
}

int run_dense(const OpShape & s, const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
              const mm3fa_tensor * mask, float scale, float max_bias, float softcap, mm3fa_tensor * dst,
              void * workspace, size_t workspace_bytes, uint64_t timeout_ns, cudaStream_t cs,
              const int64_t * peer_off = nullptr, int n_peers = 0) {
    const int64_t planes = mask ? mask->ne[2] * mask->ne[3] : 1;
    if (!workspace || workspace_bytes < dense_workspace_bytes(s.n_q, s.n_kv, planes)) {
        return MM3FA_ERR_WORKSPACE;
    }
    DenseParams p{};
    p.q        = static_cast<const char *>(q->data);
    p.k        = static_cast<const char *>(k->data);
    p.v        = static_cast<const char *>(v->data);
    p.mask     = mask ? static_cast<const char *>(mask->data) : nullptr;
    p.dst      = static_cast<char *>(dst->data);
    p.q_nb1    = (int64_t) q->nb[1];
    p.q_nb2    = (int64_t) q->nb[2];
    p.q_nb3    = (int64_t) q->nb[3];
    p.k_nb1    = (int64_t) k->nb[1];
    p.k_nb2    = (int64_t) k->nb[2];
    p.k_nb3    = (int64_t) k->nb[3];
    p.v_nb1    = (int64_t) v->nb[1];
    p.v_nb2    = (int64_t) v->nb[2];
    p.v_nb3    = (int64_t) v->nb[3];
    p.m_nb1    = mask ? (int64_t) mask->nb[1] : 0;
    p.m_nb2    = mask ? (int64_t) mask->nb[2] : 0;
    p.m_nb3    = mask ? (int64_t) mask->nb[3] : 0;
    p.m_ne2    = mask ? (int) mask->ne[2] : 1;
    p.m_ne3    = mask ? (int) mask->ne[3] : 1;
    p.d_nb1    = (int64_t) dst->nb[1];
    p.d_nb2    = (int64_t) dst->nb[2];
    p.d_nb3    = (int64_t) dst->nb[3];
    p.q_type   = q->type;
    p.q_vec    = rows_vec16(q);
    p.dst_vec  = rows_vec16(dst);
    p.mask_vec = mask ? rows_vec16(mask) : 0;
    p.n_q      = (int) s.n_q;
    p.n_kv     = (int) s.n_kv;
    p.ratio    = s.ratio;
    p.rk3      = s.rk3;
    p.scale    = scale;
    p.softcap  = softcap;
    p.max_bias = max_bias;
    const int n_head_log2 = 1 << (int) std::floor(std::log2((double) s.n_head));
    p.n_head_log2 = n_head_log2;
    p.m0          = std::pow(2.0f, -max_bias / (float) n_head_log2);
    p.m1          = std::pow(2.0f, -max_bias / 2.0f / (float) n_head_log2);
    p.timeout_ns  = timeout_ns;
    p.n_peers     = n_peers;
    for (int i = 0; i < n_peers; i++) {
        p.peer_off[i] = peer_off[i];
    }
    const cudaError_t e = launch_dense(p, (int) s.D, s.kvt, s.n_head_kv, s.n_seq_k, s.n_head, s.n_seq, workspace, cs);
    if (e == cudaErrorNotSupported) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    return record_cuda(e);
}

__global__ void zero_rows_kernel(char * dst, int64_t dv, int64_t n1, int64_t n2, int64_t n3, int64_t nb1,
                                 int64_t nb2, int64_t nb3) {
    const int64_t total = dv * n1 * n2 * n3;
    for (int64_t i = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; i < total; i += (int64_t) gridDim.x * blockDim.x) {
        const int64_t d = i % dv, a = (i / dv) % n1, b = (i / (dv * n1)) % n2, c = i / (dv * n1 * n2);
        reinterpret_cast<float *>(dst + a * nb1 + b * nb2 + c * nb3)[d] = 0.0f;
    }
}

__global__ void assemble_heads_kernel(const float * __restrict__ gathered, float * __restrict__ dst, int64_t dv,
                                      int64_t n_head, int64_t n_q, int64_t n_seq, int n_ranks) {
    const int64_t hl    = n_head / n_ranks;
    const int64_t total = dv * n_head * n_q * n_seq;
    for (int64_t o = blockIdx.x * (int64_t) blockDim.x + threadIdx.x; o < total; o += (int64_t) gridDim.x * blockDim.x) {
        const int64_t d = o % dv;
        const int64_t h = (o / dv) % n_head;
        const int64_t i = (o / (dv * n_head)) % n_q;
        const int64_t s = o / (dv * n_head * n_q);
        const int64_t r = h / hl;
        dst[o]          = gathered[(((r * n_seq + s) * n_q + i) * hl + (h % hl)) * dv + d];
    }
}

// Status self-test: one CTA waits on an mbarrier that nothing ever arrives on, bounded by
// timeout_ns, then reports the expiry through the workspace status word.
__global__ void bounded_wait_selftest_kernel(uint32_t * status, uint64_t timeout_ns) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    const bool ok = mbar_wait_bounded(&bar, 0, global_timer_ns() + timeout_ns);
    if (!ok && threadIdx.x == 0) {
        atomicOr(&status[0], ST_TIMEOUT);
        atomicExch(&status[1], 0xffffffffu);
    }
}

}  // namespace

extern "C" {

int mm3fa_version(void) {
    return (1 << 16) | 0;
}

const char * mm3fa_status_string(int st) {
    switch (st) {
        case MM3FA_OK:
            return "ok";
        case MM3FA_ERR_NULL:
            return "null tensor or data pointer";
        case MM3FA_ERR_TYPE:
            return "unsupported tensor type";
        case MM3FA_ERR_SHAPE:
            return "inconsistent shapes";
        case MM3FA_ERR_STRIDE:
            return "unsupported strides";
        case MM3FA_ERR_ALIGN:
            return "misaligned data pointer";
        case MM3FA_ERR_WORKSPACE:
            return "workspace missing or too small";
        case MM3FA_ERR_CUDA:
            return "CUDA error";
        case MM3FA_ERR_UNSUPPORTED:
            return "shape not handled by these kernels";
        case MM3FA_ERR_TIMEOUT:
            return "a bounded device wait expired";
        case MM3FA_ERR_DEVICE:
            return "device is not sm_100";
        case MM3FA_ERR_SCRATCH_LIMIT:
            return "operands need more scratch than the built-in no-allocation buffer holds";
        case MM3FA_ERR_COMM:
            return "NCCL unavailable, or a collective or CUDA IPC call failed";
        default:
            return "unknown status";
    }
}

const char * mm3fa_last_cuda_error(void) {
    return g_last_cuda_error;
}

int mm3fa_supports(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                   const mm3fa_tensor * mask, float max_bias, float logit_softcap, const mm3fa_tensor * dst) {
    OpShape s{};
    return check_op(q, k, v, mask, max_bias, logit_softcap, dst, false, s);
}

size_t mm3fa_workspace_size(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                            const mm3fa_tensor * mask, const mm3fa_tensor * dst) {
    OpShape s{};
    if (check_op(q, k, v, mask, 0.0f, 0.0f, dst, false, s) != MM3FA_OK) {
        return 0;
    }
    if (s.n_kv == 0 || s.n_q == 0 || s.n_head == 0 || s.n_seq == 0) {
        return 0;
    }
    // data alignment is not known here: size for every variant these operands could take
    size_t    need = 0;
    const int rows = s.ratio * (int) s.n_q;
    for (Variant var : { V_SIMT_BULK, V_SIMT_COPY, V_MMA_8, V_MMA_16 }) {
        if (var == V_MMA_8 && !(rows <= 8 && decode_mma_eligible((int) s.D, s.kvt, rows))) {
            continue;
        }
        if (var == V_MMA_16 && !(rows > 8 && decode_mma_eligible((int) s.D, s.kvt, rows))) {
            continue;
        }
        need = std::max(need, decode_workspace_bytes(geometry_for(s, var), (int) s.DV));
    }
    if (dense_applicable(s, mask)) {
        const int64_t planes = mask ? mask->ne[2] * mask->ne[3] : 1;
        need                 = std::max(need, dense_workspace_bytes(s.n_q, s.n_kv, planes));
    }
    return need;
}

}  // extern "C"

namespace mm3fa {

// Bytes right after the status word that must be zero when a call with these operands starts:
// the decode kernels' per-unit arrival counters (one u32 per unit, the region rounded up to
// 256 bytes).  The dense kernel's mask-block flags need nothing here: launch_dense clears
// them on the stream itself.  Sized, like mm3fa_workspace_size, for every decode variant the
// operands could take.  Used by the no-allocation entry point.
size_t workspace_counter_bytes(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                               const mm3fa_tensor * mask, const mm3fa_tensor * dst) {
    OpShape s{};
    if (check_op(q, k, v, mask, 0.0f, 0.0f, dst, false, s) != MM3FA_OK || s.n_kv == 0 || s.n_q == 0 ||
        s.n_head == 0 || s.n_seq == 0) {
        return 0;
    }
    size_t    cnt  = 0;
    const int rows = s.ratio * (int) s.n_q;
    for (Variant var : { V_SIMT_BULK, V_SIMT_COPY, V_MMA_8, V_MMA_16 }) {
        if (var == V_MMA_8 && !(rows <= 8 && decode_mma_eligible((int) s.D, s.kvt, rows))) {
            continue;
        }
        if (var == V_MMA_16 && !(rows > 8 && decode_mma_eligible((int) s.D, s.kvt, rows))) {
            continue;
        }
        const DecodeGeometry g = geometry_for(s, var);
        cnt                    = std::max(cnt, ((size_t) g.n_units * 4 + 255) / 256 * 256);
    }
    return cnt;
}

}  // namespace mm3fa

namespace {

// The operator with an optional device array of per-sequence key counts (kv_len[s]: q sequence
// s sees keys [0, kv_len[s]) only, in addition to the mask).  With kv_len the decode kernels run
// whatever the row count: they skip (cluster split) or mask (stream-K split) the keys past it.
int flash_attn_impl(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v, const mm3fa_tensor * mask,
                    const int32_t * kv_len, float scale, float max_bias, float logit_softcap, int prec,
                    mm3fa_tensor * dst, void * workspace, size_t workspace_bytes, void * stream,
                    const mm3fa_peers * peers = nullptr, int slot = 0, const uint32_t * epochs = nullptr) {
    if (prec != MM3FA_PREC_DEFAULT && prec != MM3FA_PREC_F32) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    OpShape s{};
    int     st = check_op(q, k, v, mask, max_bias, logit_softcap, dst, true, s);
    if (st != MM3FA_OK) {
        return st;
    }
    const DeviceInfo di = device_info();
    if (di.major != 10) {
        return MM3FA_ERR_DEVICE;
    }
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    if (s.n_q == 0 || s.n_head == 0 || s.n_seq == 0 || s.DV == 0) {
        return MM3FA_OK;
    }
    if (s.n_kv == 0) {  // no keys: every row is empty
        zero_rows_kernel<<<148, 256, 0, cs>>>(static_cast<char *>(dst->data), s.DV, s.n_head, s.n_q, s.n_seq,
                                              (int64_t) dst->nb[1], (int64_t) dst->nb[2], (int64_t) dst->nb[3]);
        return record_cuda(cudaGetLastError());
    }
    if (!kv_len && !peers && use_dense(s, mask)) {
        return run_dense(s, q, k, v, mask, scale, max_bias, logit_softcap, dst, workspace, workspace_bytes,
                         wait_timeout_ns(), cs);
    }
    const Variant        var = variant_for(s);
    const DecodeGeometry g   = geometry_for(s, var);
    if (!workspace || workspace_bytes < decode_workspace_bytes(g, (int) s.DV)) {
        return MM3FA_ERR_WORKSPACE;
    }
    DecodeParams p{};
    p.q         = static_cast<const char *>(q->data);
    p.k         = static_cast<const char *>(k->data);
    p.v         = static_cast<const char *>(v->data);
    p.mask      = mask ? static_cast<const char *>(mask->data) : nullptr;
    p.dst       = static_cast<char *>(dst->data);
    p.q_nb1     = (int64_t) q->nb[1];
    p.q_nb2     = (int64_t) q->nb[2];
    p.q_nb3     = (int64_t) q->nb[3];
    p.k_nb1     = (int64_t) k->nb[1];
    p.k_nb2     = (int64_t) k->nb[2];
    p.k_nb3     = (int64_t) k->nb[3];
    p.v_nb1     = (int64_t) v->nb[1];
    p.v_nb2     = (int64_t) v->nb[2];
    p.v_nb3     = (int64_t) v->nb[3];
    p.m_nb1     = mask ? (int64_t) mask->nb[1] : 0;
    p.m_nb2     = mask ? (int64_t) mask->nb[2] : 0;
    p.m_nb3     = mask ? (int64_t) mask->nb[3] : 0;
    p.m_ne2     = mask ? (int) mask->ne[2] : 1;
    p.m_ne3     = mask ? (int) mask->ne[3] : 1;
    p.d_nb1     = (int64_t) dst->nb[1];
    p.d_nb2     = (int64_t) dst->nb[2];
    p.d_nb3     = (int64_t) dst->nb[3];
    p.q_type    = q->type;
    p.n_q       = (int) s.n_q;
    p.n_head    = (int) s.n_head;
    p.n_head_kv = (int) s.n_head_kv;
    p.n_seq     = (int) s.n_seq;
    p.ratio     = s.ratio;
    p.rk3       = s.rk3;
    p.n_kv      = (int) s.n_kv;
    p.rows_per_pair = s.ratio * (int) s.n_q;
    p.scale     = scale;
    p.softcap   = logit_softcap;
    p.max_bias  = max_bias;
    const int n_head_log2 = s.n_head > 0 ? 1 << (int) std::floor(std::log2((double) s.n_head)) : 1;
    p.n_head_log2 = n_head_log2;
    p.m0        = std::pow(2.0f, -max_bias / (float) n_head_log2);
    p.m1        = std::pow(2.0f, -max_bias / 2.0f / (float) n_head_log2);
    p.timeout_ns = wait_timeout_ns();
    p.dst_vec    = rows_vec16(dst);
    p.kv_vec     = rows_vec16(k) && rows_vec16(v);
    p.kv_len     = kv_len;
    if (var >= V_MMA_8) {
        const int pref    = decode_mma_mode_preference();
        MmaPlan   plan    = pref == 1 ? MmaPlan{ 0, 3 }
                                      : decode_mma_plan((int) s.D, s.kvt, p.rows_per_pair, g.n_units, device_info().sms);
        const int cluster = plan.cluster;
        if (peers) {
            // the exchange lives in the cluster merge's 16-byte result stores
            if (cluster == 0 || !p.dst_vec) {
                return MM3FA_ERR_UNSUPPORTED;
            }
            const int64_t vals   = s.DV * s.n_head * s.n_q * s.n_seq;  // this rank's slice
            const int64_t region = 8 * vals;
            if ((uint64_t) (2 * peers->n_ranks * region) > peers->recv_slot_bytes) {
                return MM3FA_ERR_WORKSPACE;
            }
            int n = 0;
            for (int r = 0; r < peers->n_ranks; r++) {
                if (r != peers->rank) {
                    p.peer_ll[n] = static_cast<char *>(peers->recv[r]) + (uint64_t) slot * peers->recv_slot_bytes +
                                   (uint64_t) peers->rank * region;
                    n++;
                }
            }
            p.n_peers   = n;
            p.ll_parity = (int64_t) peers->n_ranks * region;
            p.epoch_ptr = epochs + slot;
        }
        return record_cuda(
            launch_decode_mma(p, g, (int) s.D, s.kvt, s.n_head_kv, s.n_seq_k, plan, workspace, cs));
    }
    if (peers) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    return record_cuda(launch_decode(p, g, (int) s.D, s.kvt, s.bulk, workspace, cs));
}

}  // namespace

extern "C" {

int mm3fa_flash_attn_ext(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                         const mm3fa_tensor * mask, float scale, float max_bias, float logit_softcap, int prec,
                         mm3fa_tensor * dst, void * workspace, size_t workspace_bytes, void * stream) {
    return flash_attn_impl(q, k, v, mask, nullptr, scale, max_bias, logit_softcap, prec, dst, workspace,
                           workspace_bytes, stream);
}

int mm3fa_flash_attn_ext_peers(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                               const mm3fa_tensor * mask, const int32_t * kv_len, float scale, float max_bias,
                               float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                               size_t workspace_bytes, const mm3fa_peers * peers, int slot, const uint32_t * epochs,
                               void * stream) {
    if (!peers || !epochs) {
        return MM3FA_ERR_NULL;
    }
    if (peers->n_ranks < 2 || peers->n_ranks > MM3FA_MAX_RANKS || peers->rank < 0 || peers->rank >= peers->n_ranks ||
        slot < 0 || peers->recv_slot_bytes % 16 != 0) {
        return MM3FA_ERR_SHAPE;
    }
    for (int r = 0; r < peers->n_ranks; r++) {
        if (!peers->recv[r]) {
            return MM3FA_ERR_NULL;
        }
        if (!aligned(peers->recv[r], 16)) {
            return MM3FA_ERR_ALIGN;
        }
    }
    if (!aligned(epochs, 4)) {
        return MM3FA_ERR_ALIGN;
    }
    if (!dst || !dst->data) {
        return MM3FA_ERR_NULL;
    }
    // the receivers index values by their position in a contiguous [Dv, n_head, n_q, n_seq] slice
    if (dst->nb[0] != 4 || dst->nb[1] % 16 != 0) {
        return MM3FA_ERR_STRIDE;
    }
    if (!workspace) {
        return MM3FA_ERR_WORKSPACE;
    }
    // ALiBi slopes depend on the global head index, which a shard's descriptors do not carry
    if (max_bias != 0.0f) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    return flash_attn_impl(q, k, v, mask, kv_len, scale, max_bias, logit_softcap, prec, dst, workspace,
                           workspace_bytes, stream, peers, slot, epochs);
}

int mm3fa_flash_attn_ext_gather(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                const mm3fa_tensor * mask, float scale, float max_bias, float logit_softcap, int prec,
                                mm3fa_tensor * dst, void * workspace, size_t workspace_bytes,
                                const mm3fa_peers * results, void * stream) {
    if (!results || !dst || !dst->data) {
        return MM3FA_ERR_NULL;
    }
    const int G = results->n_ranks, me = results->rank;
    if (G < 2 || G > MM3FA_MAX_RANKS || me < 0 || me >= G) {
        return MM3FA_ERR_SHAPE;
    }
    for (int r = 0; r < G; r++) {
        if (!results->recv[r]) {
            return MM3FA_ERR_NULL;
        }
        if (!aligned(results->recv[r], 16)) {
            return MM3FA_ERR_ALIGN;
        }
    }
    // dst lies inside this rank's whole result [recv[me], recv[me] + recv_slot_bytes)
    const char * base = static_cast<const char *>(results->recv[me]);
    const char * d0   = static_cast<const char *>(dst->data);
    if (d0 < base) {
        return MM3FA_ERR_SHAPE;
    }
    const uint64_t last = (uint64_t) (d0 - base) + (uint64_t) ((dst->ne[1] - 1) * dst->nb[1] +
                                                               (dst->ne[2] - 1) * dst->nb[2] +
                                                               (dst->ne[3] - 1) * dst->nb[3]) +
                          (uint64_t) dst->ne[0] * 4;
    if (dst->ne[1] < 1 || dst->ne[2] < 1 || dst->ne[3] < 1 || last > results->recv_slot_bytes) {
        return MM3FA_ERR_SHAPE;
    }
    // ALiBi slopes depend on the global head index, which a shard's descriptors do not carry
    if (max_bias != 0.0f) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    if (prec != MM3FA_PREC_DEFAULT && prec != MM3FA_PREC_F32) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    OpShape s{};
    int     st = check_op(q, k, v, mask, max_bias, logit_softcap, dst, true, s);
    if (st != MM3FA_OK) {
        return st;
    }
    if (device_info().major != 10) {
        return MM3FA_ERR_DEVICE;
    }
    if (s.n_q == 0 || s.n_head == 0 || s.n_seq == 0 || s.DV == 0) {
        return MM3FA_OK;
    }
    // the exchange lives in the tensor-core kernel's TMA-store epilogue: many query rows, keys present
    if (s.n_kv == 0 || !use_dense(s, mask) || !rows_vec16(dst)) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    int64_t off[MM3FA_MAX_RANKS - 1];
    int     n = 0;
    for (int r = 0; r < G; r++) {
        if (r != me) {
            off[n++] = (int64_t) (static_cast<const char *>(results->recv[r]) - base);
        }
    }
    return run_dense(s, q, k, v, mask, scale, max_bias, logit_softcap, dst, workspace, workspace_bytes,
                     wait_timeout_ns(), static_cast<cudaStream_t>(stream), off, n);
}

int mm3fa_flash_attn_ext_kvlen(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                               const mm3fa_tensor * mask, const int32_t * kv_len, float scale, float max_bias,
                               float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                               size_t workspace_bytes, void * stream) {
    if (!kv_len) {
        return MM3FA_ERR_NULL;
    }
    return flash_attn_impl(q, k, v, mask, kv_len, scale, max_bias, logit_softcap, prec, dst, workspace,
                           workspace_bytes, stream);
}

}  // extern "C"

namespace {

// Checks the decode prologue's operands (mm3fa_decode_prologue) and fills its parameters.
int prepare_prologue(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                     const float * q_norm, const float * k_norm, float eps, const int32_t * pos, float rope_theta,
                     const int64_t * rows, mm3fa_tensor * k_cache, mm3fa_tensor * v_cache, mm3fa_tensor * q_out,
                     uint32_t flags, PrologueParams & p, int64_t & D_out) {
    if (flags & ~(uint32_t) MM3FA_PROLOGUE_CLAMP_FP16) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    if (!q_in || !k_in || !v_in || !k_cache || !v_cache || !q_out || !q_norm || !k_norm || !pos || !rows) {
        return MM3FA_ERR_NULL;
    }
    for (const mm3fa_tensor * t : { q_in, k_in, v_in, (const mm3fa_tensor *) k_cache, (const mm3fa_tensor *) v_cache,
                                    (const mm3fa_tensor *) q_out }) {
        if (!t->data) {
            return MM3FA_ERR_NULL;
        }
    }
    if (q_in->type != MM3FA_TYPE_F32 || k_in->type != MM3FA_TYPE_F32 || v_in->type != MM3FA_TYPE_F32 ||
        q_out->type != MM3FA_TYPE_F32) {
        return MM3FA_ERR_TYPE;
    }
    const int kvt = k_cache->type;
    if ((kvt != MM3FA_TYPE_F16 && kvt != MM3FA_TYPE_BF16 && kvt != MM3FA_TYPE_Q8_0) || v_cache->type != kvt) {
        return MM3FA_ERR_TYPE;
    }
    const int64_t D = q_in->ne[0], H = q_in->ne[1], N = q_in->ne[2], Hkv = k_in->ne[1];
    if (D != 64 && D != 128 && D != 256) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    if (H <= 0 || Hkv <= 0 || N <= 0 || q_in->ne[3] != 1 || k_in->ne[0] != D || k_in->ne[2] != N ||
        v_in->ne[0] != D || v_in->ne[1] != Hkv || v_in->ne[2] != N || q_out->ne[0] != D || q_out->ne[1] != H ||
        q_out->ne[2] != N) {
        return MM3FA_ERR_SHAPE;
    }
    for (const mm3fa_tensor * c : { (const mm3fa_tensor *) k_cache, (const mm3fa_tensor *) v_cache }) {
        if (c->ne[0] != D || c->ne[1] < 1 || c->ne[2] != Hkv || c->ne[3] != N) {
            return MM3FA_ERR_SHAPE;
        }
    }
    if (H > 65535 || Hkv > 65535 || N > 65535 || H % Hkv != 0) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    // rows packed, strides multiples of the element (block) size, F32 data 4-byte aligned
    const int64_t ce = type_unit_bytes(kvt);
    for (const mm3fa_tensor * t : { q_in, k_in, v_in, (const mm3fa_tensor *) q_out }) {
        if (t->nb[0] != 4 || t->nb[1] % 4 || t->nb[2] % 4 || (int64_t) t->nb[1] < 4 * D ||
            !aligned(t->data, 4)) {
            return MM3FA_ERR_STRIDE;
        }
    }
    for (const mm3fa_tensor * c : { (const mm3fa_tensor *) k_cache, (const mm3fa_tensor *) v_cache }) {
        if ((int64_t) c->nb[0] != ce || (int64_t) c->nb[1] < row_bytes(kvt, D) || c->nb[1] % 2 || c->nb[2] % 2 ||
            c->nb[3] % 2 || !aligned(c->data, 2)) {
            return MM3FA_ERR_STRIDE;
        }
    }
    if (!(eps >= 0.0f) || !std::isfinite(rope_theta) || !(rope_theta > 0.0f)) {
        return MM3FA_ERR_SHAPE;
    }
    if (device_info().major != 10) {
        return MM3FA_ERR_DEVICE;
    }
    p.q_in        = static_cast<const char *>(q_in->data);
    p.k_in        = static_cast<const char *>(k_in->data);
    p.v_in        = static_cast<const char *>(v_in->data);
    p.q_norm      = q_norm;
    p.k_norm      = k_norm;
    p.pos         = pos;
    p.rows        = rows;
    p.q_out       = static_cast<char *>(q_out->data);
    p.k_cache     = static_cast<char *>(k_cache->data);
    p.v_cache     = static_cast<char *>(v_cache->data);
    p.qi_nb1      = (int64_t) q_in->nb[1];
    p.qi_nb2      = (int64_t) q_in->nb[2];
    p.ki_nb1      = (int64_t) k_in->nb[1];
    p.ki_nb2      = (int64_t) k_in->nb[2];
    p.vi_nb1      = (int64_t) v_in->nb[1];
    p.vi_nb2      = (int64_t) v_in->nb[2];
    p.qo_nb1      = (int64_t) q_out->nb[1];
    p.qo_nb2      = (int64_t) q_out->nb[2];
    p.kc_nb1      = (int64_t) k_cache->nb[1];
    p.kc_nb2      = (int64_t) k_cache->nb[2];
    p.kc_nb3      = (int64_t) k_cache->nb[3];
    p.vc_nb1      = (int64_t) v_cache->nb[1];
    p.vc_nb2      = (int64_t) v_cache->nb[2];
    p.vc_nb3      = (int64_t) v_cache->nb[3];
    p.kvt         = kvt;
    p.n_head      = (int) H;
    p.n_head_kv   = (int) Hkv;
    p.n_set       = (int) N;
    p.k_rows      = k_cache->ne[1];
    p.v_rows      = v_cache->ne[1];
    p.eps         = eps;
    p.theta_scale = std::pow(rope_theta, -2.0f / (float) D);
    p.clamp_v     = (flags & MM3FA_PROLOGUE_CLAMP_FP16) ? 1 : 0;
    D_out         = D;
    return MM3FA_OK;
}

}  // namespace

extern "C" {

int mm3fa_decode_prologue_ex(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                             const float * q_norm, const float * k_norm, float eps, const int32_t * pos,
                             float rope_theta, const int64_t * rows, mm3fa_tensor * k_cache, mm3fa_tensor * v_cache,
                             mm3fa_tensor * q_out, uint32_t flags, void * stream) {
    PrologueParams p{};
    int64_t        D  = 0;
    const int      st = prepare_prologue(q_in, k_in, v_in, q_norm, k_norm, eps, pos, rope_theta, rows, k_cache, v_cache,
                                         q_out, flags, p, D);
    if (st != MM3FA_OK) {
        return st;
    }
    return record_cuda(launch_decode_prologue(p, (int) D, static_cast<cudaStream_t>(stream)));
}

int mm3fa_decode_prologue(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                          const float * q_norm, const float * k_norm, float eps, const int32_t * pos, float rope_theta,
                          const int64_t * rows, mm3fa_tensor * k_cache, mm3fa_tensor * v_cache, mm3fa_tensor * q_out,
                          void * stream) {
    return mm3fa_decode_prologue_ex(q_in, k_in, v_in, q_norm, k_norm, eps, pos, rope_theta, rows, k_cache, v_cache,
                                    q_out, 0u, stream);
}

int mm3fa_decode_step_ex(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                         const float * q_norm, const float * k_norm, float eps, const int32_t * pos, float rope_theta,
                         const int64_t * rows, mm3fa_tensor * k_cache, mm3fa_tensor * v_cache, mm3fa_tensor * q_out,
                         const mm3fa_tensor * k, const mm3fa_tensor * v, const mm3fa_tensor * mask, float scale,
                         float max_bias, float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                         size_t workspace_bytes, uint32_t flags, void * stream) {
    PrologueParams pp{};
    int64_t        D  = 0;
    int            st = prepare_prologue(q_in, k_in, v_in, q_norm, k_norm, eps, pos, rope_theta, rows, k_cache, v_cache,
                                         q_out, flags, pp, D);
    if (st != MM3FA_OK) {
        return st;
    }
    if (!k || !v) {
        return MM3FA_ERR_NULL;
    }
    // the attention reads q_out as [D, 1, n_head, N]; its operands are checked before the
    // prologue runs, so that a rejected call changes nothing
    mm3fa_tensor qa = *q_out;
    qa.ne[0] = D, qa.ne[1] = 1, qa.ne[2] = q_out->ne[1], qa.ne[3] = q_out->ne[2];
    qa.nb[0] = 4, qa.nb[1] = (size_t) (4 * D), qa.nb[2] = q_out->nb[1], qa.nb[3] = q_out->nb[2];
    {
        OpShape sh{};
        st = check_op(&qa, k, v, mask, max_bias, logit_softcap, dst, true, sh);
        if (st != MM3FA_OK) {
            return st;
        }
        const size_t need = mm3fa_workspace_size(&qa, k, v, mask, dst);
        if (need > 0 && (!workspace || workspace_bytes < need)) {
            return MM3FA_ERR_WORKSPACE;
        }
    }
    // the prologue kernel, then the attention (both launched with programmatic stream
    // serialisation, so the attention's CTAs start as the prologue's exit)
    st = record_cuda(launch_decode_prologue(pp, (int) D, static_cast<cudaStream_t>(stream)));
    if (st != MM3FA_OK) {
        return st;
    }
    return flash_attn_impl(&qa, k, v, mask, nullptr, scale, max_bias, logit_softcap, prec, dst, workspace,
                           workspace_bytes, stream);
}

int mm3fa_decode_step(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                      const float * q_norm, const float * k_norm, float eps, const int32_t * pos, float rope_theta,
                      const int64_t * rows, mm3fa_tensor * k_cache, mm3fa_tensor * v_cache, mm3fa_tensor * q_out,
                      const mm3fa_tensor * k, const mm3fa_tensor * v, const mm3fa_tensor * mask, float scale,
                      float max_bias, float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                      size_t workspace_bytes, void * stream) {
    return mm3fa_decode_step_ex(q_in, k_in, v_in, q_norm, k_norm, eps, pos, rope_theta, rows, k_cache, v_cache, q_out,
                                k, v, mask, scale, max_bias, logit_softcap, prec, dst, workspace, workspace_bytes, 0u,
                                stream);
}

int mm3fa_dit_prologue(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                       const int32_t * pos, int rot_dims, float rope_theta, mm3fa_tensor * q_out, mm3fa_tensor * k_out,
                       mm3fa_tensor * v_out, void * stream) {
    if (!q_in || !k_in || !v_in || !q_out || !k_out || !v_out || !pos) {
        return MM3FA_ERR_NULL;
    }
    for (const mm3fa_tensor * t : { q_in, k_in, v_in, (const mm3fa_tensor *) q_out, (const mm3fa_tensor *) k_out,
                                    (const mm3fa_tensor *) v_out }) {
        if (!t->data) {
            return MM3FA_ERR_NULL;
        }
    }
    if (q_in->type != MM3FA_TYPE_F32 || k_in->type != MM3FA_TYPE_F32 || v_in->type != MM3FA_TYPE_F32 ||
        q_out->type != MM3FA_TYPE_F32) {
        return MM3FA_ERR_TYPE;
    }
    const int ot = k_out->type;
    if ((ot != MM3FA_TYPE_F16 && ot != MM3FA_TYPE_BF16) || v_out->type != ot) {
        return MM3FA_ERR_TYPE;
    }
    const int64_t D = q_in->ne[0], H = q_in->ne[1], S = q_in->ne[2], B = q_in->ne[3];
    if (D != 64 && D != 128) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    for (const mm3fa_tensor * t : { k_in, v_in, (const mm3fa_tensor *) q_out }) {
        if (t->ne[0] != D || t->ne[1] != H || t->ne[2] != S || t->ne[3] != B) {
            return MM3FA_ERR_SHAPE;
        }
    }
    for (const mm3fa_tensor * t : { (const mm3fa_tensor *) k_out, (const mm3fa_tensor *) v_out }) {
        if (t->ne[0] != D || t->ne[1] != S || t->ne[2] != H || t->ne[3] != B) {
            return MM3FA_ERR_SHAPE;
        }
    }
    const int E = (int) D / 32;
    if (rot_dims <= 0 || rot_dims > D || rot_dims % (2 * E) != 0) {
        return MM3FA_ERR_SHAPE;
    }
    if (!std::isfinite(rope_theta) || !(rope_theta > 0.0f) || H <= 0 || S <= 0 || B <= 0) {
        return MM3FA_ERR_SHAPE;
    }
    for (const mm3fa_tensor * t : { q_in, k_in, v_in, (const mm3fa_tensor *) q_out }) {
        if (t->nb[0] != 4 || t->nb[1] % 4 || t->nb[2] % 4 || t->nb[3] % 4 || !aligned(t->data, 4)) {
            return MM3FA_ERR_STRIDE;
        }
    }
    for (const mm3fa_tensor * t : { (const mm3fa_tensor *) k_out, (const mm3fa_tensor *) v_out }) {
        if (t->nb[0] != 2 || t->nb[1] % 2 || t->nb[2] % 2 || t->nb[3] % 2 || !aligned(t->data, 2)) {
            return MM3FA_ERR_STRIDE;
        }
    }
    if (device_info().major != 10) {
        return MM3FA_ERR_DEVICE;
    }
    DitPrologueParams p{};
    p.q_in  = static_cast<const char *>(q_in->data);
    p.k_in  = static_cast<const char *>(k_in->data);
    p.v_in  = static_cast<const char *>(v_in->data);
    p.pos   = pos;
    p.q_out = static_cast<char *>(q_out->data);
    p.k_out = static_cast<char *>(k_out->data);
    p.v_out = static_cast<char *>(v_out->data);
    // (head, token, batch) strides: inputs and q_out are [D, H, S, B], k_out / v_out [D, S, H, B]
    auto hsb = [](const mm3fa_tensor * t, int64_t (&o)[3]) {
        o[0] = (int64_t) t->nb[1];
        o[1] = (int64_t) t->nb[2];
        o[2] = (int64_t) t->nb[3];
    };
    auto shb = [](const mm3fa_tensor * t, int64_t (&o)[3]) {
        o[0] = (int64_t) t->nb[2];
        o[1] = (int64_t) t->nb[1];
        o[2] = (int64_t) t->nb[3];
    };
    hsb(q_in, p.sq_in);
    hsb(k_in, p.sk_in);
    hsb(v_in, p.sv_in);
    hsb(q_out, p.sq_out);
    shb(k_out, p.sk_out);
    shb(v_out, p.sv_out);
    p.kvt         = ot;
    p.n_head      = (int) H;
    p.n_tok       = (int) S;
    p.n_batch     = (int) B;
    p.rot         = rot_dims;
    p.theta_scale = std::pow(rope_theta, -2.0f / (float) rot_dims);
    if (H > 65535 || S > 0x7fffffff / 4 || B > 65535) {
        return MM3FA_ERR_UNSUPPORTED;
    }
    return record_cuda(launch_dit_prologue(p, (int) D, static_cast<cudaStream_t>(stream)));
}

int mm3fa_assemble_heads(const float * gathered, float * dst, int64_t dv, int64_t n_head, int64_t n_q, int64_t n_seq,
                         int n_ranks, void * stream) {
    if (!gathered || !dst) {
        return MM3FA_ERR_NULL;
    }
    if (n_ranks < 1 || dv < 0 || n_head < 0 || n_q < 0 || n_seq < 0 || (n_head % n_ranks) != 0) {
        return MM3FA_ERR_SHAPE;
    }
    const int64_t total = dv * n_head * n_q * n_seq;
    if (total == 0) {
        return MM3FA_OK;
    }
    const int64_t blocks = std::min<int64_t>((total + 255) / 256, 148 * 8);
    assemble_heads_kernel<<<(unsigned) blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(gathered, dst, dv, n_head,
                                                                                            n_q, n_seq, n_ranks);
    return record_cuda(cudaGetLastError());
}

int mm3fa_workspace_status(void * workspace, void * stream, uint32_t * status_out) {
    if (!workspace || !status_out) {
        return MM3FA_ERR_NULL;
    }
    cudaStream_t cs = static_cast<cudaStream_t>(stream);
    uint32_t     st[2] = { 0, 0 };
    cudaError_t  e     = cudaMemcpyAsync(st, workspace, sizeof(st), cudaMemcpyDeviceToHost, cs);
    if (e == cudaSuccess) {
        e = cudaStreamSynchronize(cs);
    }
    if (e != cudaSuccess) {
        return record_cuda(e);
    }
    *status_out = st[0];
    if (st[0] != 0) {
        const uint32_t zero[2] = { 0, 0 };
        e                      = cudaMemcpyAsync(workspace, zero, sizeof(zero), cudaMemcpyHostToDevice, cs);
        if (e == cudaSuccess) {
            e = cudaStreamSynchronize(cs);
        }
        if (e != cudaSuccess) {
            return record_cuda(e);
        }
        return MM3FA_ERR_TIMEOUT;
    }
    return MM3FA_OK;
}

int mm3fa_selftest_bounded_wait(void * workspace, uint32_t timeout_us, void * stream) {
    if (!workspace) {
        return MM3FA_ERR_NULL;
    }
    bounded_wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint32_t *>(workspace), (uint64_t) timeout_us * 1000ull);
    return record_cuda(cudaGetLastError());
}

}  // extern "C"
