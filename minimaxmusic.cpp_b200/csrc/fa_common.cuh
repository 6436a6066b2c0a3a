// fa_common.cuh - shared device helpers for the mm3fa kernels (sm_100a).
//
// PTX wrappers for mbarriers, bulk (TMA engine) global->shared copies and the global
// timer, numeric conversions that follow ggml's conventions, and the launch-parameter
// structs shared by the C ABI and the kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace mm3fa {

// Storage types handled by the kernels (numbering of ggml.h's enum ggml_type).
enum KvType : int { KV_F32 = 0, KV_F16 = 1, KV_Q8_0 = 8, KV_BF16 = 30 };

constexpr int QK8_0          = 32;
constexpr int Q8_0_BLOCK     = 34;
constexpr float LOG2E        = 1.4426950408889634f;
constexpr uint32_t ST_TIMEOUT = 1u;  // status bit: a bounded wait expired

// Workspace layout shared by host and device (byte offsets from the workspace base).
constexpr size_t WS_STATUS_BYTES = 256;  // [0]: status bits, [1]: where the wait gave up
constexpr int    WS_PEER_ARRIVE  = 8;    // status[8]: CTAs of a peer-exchange wait done (reset by the last)
constexpr int    MAX_PEERS       = 7;    // other ranks a head exchange over peer memory can write to

// ------------------------------------------------------------------ PTX wrappers

__device__ __forceinline__ uint32_t smem_addr(const void * p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ void mbar_init(uint64_t * bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count) : "memory");
}

// Makes initialised mbarriers visible to the async (TMA) proxy.
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t * bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t * bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}

// Waits for phase `parity` of an mbarrier until the global timer passes deadline_ns.
// Returns false when the deadline expired first.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t * bar, uint32_t parity, uint64_t deadline_ns) {
    uint32_t spins = 0;
    while (!mbar_try_wait(bar, parity)) {
        if ((++spins & 255u) == 0 && global_timer_ns() > deadline_ns) {
            return mbar_try_wait(bar, parity);
        }
    }
    return true;
}

// 1-D bulk copy global -> this CTA's shared memory through the TMA engine; completion
// is signalled as transaction bytes on `bar`.  dst, src and bytes must be multiples of 16.
// No multicast: the destination is the issuing CTA only.
__device__ __forceinline__ void bulk_copy_g2s(void * dst, const void * src, uint32_t bytes, uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

// ------------------------------------------------------------------ conversions

__device__ __forceinline__ float round_to_f16(float x) {
    return __half2float(__float2half_rn(x));
}

__device__ __forceinline__ float round_to_bf16(float x) {
    return __bfloat162float(__float2bfloat16_rn(x));
}

__device__ __forceinline__ float2 h2_to_f2(uint32_t u) {
    __half2 h = *reinterpret_cast<__half2 *>(&u);
    return __half22float2(h);
}

__device__ __forceinline__ float2 bf2_to_f2(uint32_t u) {
    __nv_bfloat162 h = *reinterpret_cast<__nv_bfloat162 *>(&u);
    return __bfloat1622float2(h);
}

// Keys of q sequence s that are visible: kv_len[s] clamped to [0, n_kv], or n_kv without kv_len.
__device__ __forceinline__ int seq_kv_len(const int * kv_len, int s, int n_kv) {
    return kv_len ? min(max(kv_len[s], 0), n_kv) : n_kv;
}

// ALiBi slope of query head h; 1 when max_bias == 0.
__device__ __forceinline__ float alibi_slope(int h, float max_bias, int n_head_log2, float m0, float m1) {
    if (max_bias <= 0.0f) {
        return 1.0f;
    }
    return h < n_head_log2 ? powf(m0, (float) (h + 1)) : powf(m1, (float) (2 * (h - n_head_log2) + 1));
}

// ------------------------------------------------------------------ launch parameters

struct DecodeParams {
    // operands (device pointers + ggml byte strides)
    const char * q;
    const char * k;
    const char * v;
    const char * mask;  // F16, may be null
    char *       dst;
    int64_t      q_nb1, q_nb2, q_nb3;
    int64_t      k_nb1, k_nb2, k_nb3;
    int64_t      v_nb1, v_nb2, v_nb3;
    int64_t      m_nb1, m_nb2, m_nb3;
    int64_t      d_nb1, d_nb2, d_nb3;
    int          q_type;
    int          n_q, n_head, n_head_kv, n_seq;
    int          ratio;    // n_head / n_head_kv
    int          rk3;      // n_seq / n_seq_k
    int          m_ne2, m_ne3;
    int          n_kv;
    int          rows_per_pair;  // ratio * n_q
    int          rows_per_unit;  // <= 32
    int          groups;         // row groups per (seq, kv head)
    float        scale;          // softmax scale
    float        softcap;        // 0 = off
    float        max_bias, m0, m1;
    int          n_head_log2;
    // stream-K style split of the n_units * n_kv key positions
    int64_t      n_units;
    int64_t      keys_per_cta;   // W
    int          max_slots;      // partial slots per unit
    int          cluster;        // CTAs per thread-block cluster (tensor-core cluster mode)
    int          dst_vec;        // dst rows start 16-byte aligned: 16-byte stores
    int          kv_vec;         // every K and V row starts 16-byte aligned (element copies in 16 B)
    int          mask_tma;       // mask rows staged by TMA with K/V (cluster mode)
    const int *  kv_len;         // device [n_seq]: q sequence s sees keys [0, kv_len[s]) (null: all)
    // head exchange over peer memory (cluster mode only): every result value, at linear index e
    // of this rank's result view [Dv, n_head, n_q, n_seq], is also stored into each peer's
    // receive buffer as the 8-byte word {value, epoch} at peer_ll[i] + (epoch & 1) * ll_parity
    // + 8 * e (16-byte volatile stores, no fence), epoch = *epoch_ptr + 1 (the calls on this slot
    // so far, advanced by the receiver's wait kernel)
    int             n_peers;
    char *          peer_ll[MAX_PEERS];
    int64_t         ll_parity;
    const uint32_t *epoch_ptr;
    // workspace
    uint32_t *   status;
    uint32_t *   counters;
    float *      part_ml;        // [unit][slot][row][2] (m in log2 units, l)
    float *      part_o;         // [unit][slot][row][DV]
    uint64_t     timeout_ns;
};

}  // namespace mm3fa
