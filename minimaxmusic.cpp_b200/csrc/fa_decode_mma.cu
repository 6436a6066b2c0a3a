// fa_decode_mma.cu - split-KV decode attention on tensor cores, TMA tensor staging (sm_100a).
//
// Same operator and units as fa_decode.cu (<= 32 GQA rows sharing one K/V slab), for F16/BF16/
// Q8_0 K/V with <= 16 rows per unit (the CFG decode of src/qwen3-lm.h:784-824: 4 query heads per
// kv head, 1 query row).  Two work splits:
//   cluster mode (the default when the units fill the GPU): one thread-block cluster of CS <= 16
//     CTAs per unit, the CTAs taking interleaved chunks of the unit's keys, the partials merged by
//     pushing them over distributed shared memory to the rank that owns each (row, 4 dims) item;
//   stream-K: a cut of all unit keys over one wave of CTAs, partials merged through the
//     workspace by the last-arriving CTA in fixed order.
//
// Pipeline per CTA (160 threads, two CTAs per SM at D=128):
//   warp 4 (producer)  - one thread issues the loads of each stage into an NS-deep ring: 4-D
//                        tiled TMA boxes (cp.async.bulk.tensor, 128-byte swizzle, no multicast)
//                        of 64 keys x D of K and V, plus (cluster mode, one shared mask row)
//                        the stage's mask row; full/empty mbarriers, no block-wide barrier.
//   warps 0-3          - each owns 16 keys of every stage (Q8_0: 32, as two 16-key sub-tiles)
//                        and keeps its own online-softmax state; the four warp partials are
//                        combined once per unit.
// Math per warp and stage, with keys on the MMA's M dimension so the few GQA rows fill N:
//   S^T[16 keys x 8r rows] = K[16 x D] . Q^T        (mma.sync m16n8k16, A via ldmatrix)
//   P^T -> P fragments by movmatrix (register transpose, no shared-memory round trip)
//   O^T[D x 8r]           += V^T[D x 16] . P^T       (A via ldmatrix.trans)
// Q is rounded to K's type (ggml's convention for F16/BF16 K); P is rounded to that type for
// the PV product; accumulation, softmax and the running row sums are F32.
//
// Q8_0 K/V (Q8 = true; 34-byte blocks of an f16 scale d and 32 int8 values, rows of D/32
// blocks packed back to back, so a row is not 16-byte aligned and no tensor map applies):
//   * stages are 1-D bulk copies (cp.async.bulk, no multicast) of C whole rows, exact bytes;
//   * Q is quantized to Q8_0 per unit exactly as ggml's reference quantizer (d = amax/127
//     rounded to f16, q = round(x/d)), and S[key][row] = sum over blocks b of
//     int32 dot(qk_b, qq_b) * (dk_b * dq_b) - the integer block dots come from
//     mma.sync m16n8k32 s8 (one per block), exact like ggml's vec_dot_q8_0_q8_0;
//   * V is dequantized exactly: int8 values become f16 integers (magic-number conversion:
//     0x6400 | (v ^ 0x80) is the f16 value 1152 + v, minus 1152), and each key's block
//     scale is folded into P (P * dv_b rounded to f16 once, like P itself on the F16 path),
//     so O^T += V^T (P * dv)^T per 32-dim block with m16n8k16 f16 products and F32 sums.
#include "fa_decode.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

namespace mm3fa {

constexpr int MMA_CONSUMERS = 4;                         // consumer warps
constexpr int MMA_THREADS   = 32 * (MMA_CONSUMERS + 1);  // + producer warp
constexpr int MMA_C         = 16 * MMA_CONSUMERS;        // F16/BF16 keys per stage (16 per consumer warp)
constexpr int MMA_RMAX      = 32;                        // rows per unit in the partial layout
constexpr int MMA_MAX_CLUSTER = 16;                      // largest cluster (non-portable size)

template <int D, int NT, int NS, bool Q8 = false>
struct MmaSmem {
    static constexpr int HALVES     = D / 64;                 // 128-byte column blocks per row
    static constexpr int TILE       = MMA_C * 128;            // one TMA box: MMA_C keys x 128 B
    static constexpr int RB         = D / QK8_0 * Q8_0_BLOCK; // bytes of one Q8_0 row
    // keys per stage: Q8_0 with 8 rows per unit takes 32 per warp (two 16-key sub-tiles)
    static constexpr int CK         = (Q8 && NT == 1) ? 2 * MMA_C : MMA_C;
    static constexpr int MAT        = Q8 ? CK * RB : HALVES * TILE;  // K or V of one stage
    static constexpr int MASKB      = CK * 2;                 // the stage's mask row (TMA mask)
    // K, V, mask row; F16/BF16 stages keep the 1024-byte alignment of the 128-byte swizzle
    static constexpr int SALIGN     = Q8 ? 128 : 1024;
    static constexpr int STAGE      = (2 * MAT + MASKB + SALIGN - 1) / SALIGN * SALIGN;
    // [row][D] merged O of the 4 warps (stream-K); in cluster mode the receive buffer of this
    // CTA's share of the cluster merge: [source rank][item] float4, items <= rows * D/4 / CS + 1
    static constexpr int RED_O_B    = 8 * NT * D * 4 > (8 * NT * D / 4 + 16) * 16 ? 8 * NT * D * 4
                                                                                 : (8 * NT * D / 4 + 16) * 16;
    static constexpr int OFF_RED_O  = NS * STAGE;
    static constexpr int OFF_RECV_ML = OFF_RED_O + RED_O_B;           // [source rank][row][2] (m, l)
    static constexpr int OFF_RED_ML = OFF_RECV_ML + MMA_MAX_CLUSTER * 8 * NT * 2 * 4;  // [warp][row][2] (m, l)
    static constexpr int OFF_BAR    = OFF_RED_ML + MMA_CONSUMERS * 8 * NT * 2 * 4;
    static constexpr int OFF_FLAG   = OFF_BAR + (2 * NS + 1) * 8;  // full[NS], empty[NS], pushed
    // Q8_0: the quantized Q fragments, [nt][block][lane] x {2 int8x4 words, 2 row scales}
    static constexpr int OFF_QX     = (OFF_FLAG + 16 + 15) / 16 * 16;
    static constexpr int QX_B       = Q8 ? NT * (D / QK8_0) * 32 * 16 : 0;
    static constexpr int TOTAL      = OFF_QX + QX_B + 1024;   // + alignment slack for the ring
    // the cluster merge parks the 4 warps' O fragments ([warp][8 NT rows][D + 4] floats) in the ring
    static_assert(MMA_CONSUMERS * 8 * NT * (D + 4) * 4 <= NS * STAGE, "merge staging exceeds the ring");
};

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void tma_load_4d(void * dst, const CUtensorMap * tm, int c0, int c1, int c2, int c3,
                                            uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2, uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t & r0, uint32_t & r1, uint32_t & r2,
                                          uint32_t & r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}

// D = A.B + C on 16x32 int8 A (row) and 32x8 int8 B (col), int32 accumulators.
__device__ __forceinline__ void mma_s8_16832(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+r"(c[0]), "+r"(c[1]), "+r"(c[2]), "+r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// 4 bytes of shared memory at p, which lies MOD4 bytes past a 4-byte boundary (0 or 2).
template <int MOD4>
__device__ __forceinline__ uint32_t lds_word(const char * p) {
    if constexpr (MOD4 == 0) {
        return *reinterpret_cast<const uint32_t *>(p);
    } else {
        const uint32_t * w = reinterpret_cast<const uint32_t *>(p - 2);
        return __funnelshift_r(w[0], w[1], 16);
    }
}

__device__ __forceinline__ float lds_half(const char * p) {
    return __half2float(*reinterpret_cast<const __half *>(p));
}

// Two int8 values of one V dim for two keys, from a byte-interleaved word (x0 y0 x1 y1, each
// biased by 128 with ^0x80): SEL 0x4140 takes (x0, y0), 0x4342 takes (x1, y1).  Placing a
// byte u under the exponent bits 0x64 gives the f16 value 1024 + u, so subtracting 1152
// leaves u - 128, the signed value, exactly.
template <uint32_t SEL>
__device__ __forceinline__ uint32_t i8x2_to_h2(uint32_t il) {
    uint32_t h = __byte_perm(il, 0x64646464u, SEL), r;
    asm("sub.f16x2 %0, %1, %2;" : "=r"(r) : "r"(h), "r"(0x64806480u));
    return r;
}

__device__ __forceinline__ uint32_t movmatrix_t(uint32_t x) {
    uint32_t y;
    asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
    return y;
}

template <bool BF16>
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
    if (BF16) {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    } else {
        asm volatile(
            "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
            "{%0,%1,%2,%3};"
            : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
            : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
    }
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
    if (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    }
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

__device__ __forceinline__ void named_barrier_consumers() {
    asm volatile("bar.sync 1, %0;" ::"n"(32 * MMA_CONSUMERS) : "memory");
}

// Barrier over the consumer warps that also ORs a predicate: every consumer thread gets the
// same answer, so branches on it keep the warps' barrier sequences identical.
__device__ __forceinline__ bool consumers_any(bool v) {
    uint32_t r;
    asm volatile(
        "{\n\t.reg .pred pin, pout;\n\t"
        "setp.ne.u32 pin, %1, 0;\n\t"
        "bar.red.or.pred pout, 1, %2, pin;\n\t"
        "selp.u32 %0, 1, 0, pout;\n\t}"
        : "=r"(r)
        : "r"((uint32_t) v), "n"(32 * MMA_CONSUMERS)
        : "memory");
    return r != 0;
}

// ---- thread-block cluster / distributed shared memory
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}

// shared-memory address of the same variable in cluster CTA `rank`
__device__ __forceinline__ uint32_t dsmem_addr(const void * local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(local)), "r"(rank));
    return r;
}

// Split cluster barrier: every thread arrives once its CTA's mbarriers are initialised; a
// thread that will touch another CTA's shared memory waits first.  The arrive is relaxed: the
// only writes it has to publish are the mbarrier inits, which fence.mbarrier_init already
// released at cluster scope (a releasing arrive cost ~0.45 us at kernel start).
__device__ __forceinline__ void cluster_arrive() {
    asm volatile("barrier.cluster.arrive.relaxed.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
    asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Asynchronous store into another CTA's shared memory (addresses from mapa) that signals its
// bytes to the mbarrier `bar` of that CTA: the receiver's phase completes once every expected
// byte has landed, with no fence or separate arrive on the sending side.
__device__ __forceinline__ void st_async4(uint32_t addr, float4 v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v4.f32 [%0], {%1, %2, %3, %4}, [%5];" ::"r"(addr),
                 "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void st_async2(uint32_t addr, float2 v, uint32_t bar) {
    asm volatile("st.async.shared::cluster.mbarrier::complete_tx::bytes.v2.f32 [%0], {%1, %2}, [%3];" ::"r"(addr),
                 "f"(v.x), "f"(v.y), "r"(bar)
                 : "memory");
}

// Bounded wait on a local mbarrier phase whose arrivals come from other CTAs of the cluster.
__device__ __forceinline__ bool mbar_wait_cluster_bounded(uint64_t * bar, uint32_t parity, uint64_t deadline_ns) {
    uint32_t spins = 0;
    for (;;) {
        uint32_t ok;
        asm volatile(
            "{\n\t.reg .pred q;\n\t"
            "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 q, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, q;\n\t}"
            : "=r"(ok)
            : "r"(smem_addr(bar)), "r"(parity)
            : "memory");
        if (ok) {
            return true;
        }
        if ((++spins & 255u) == 0 && global_timer_ns() > deadline_ns) {
            return false;
        }
    }
}

// ---- programmatic dependent launch: this kernel is launched with programmatic stream
// serialisation, so its CTAs may start once every CTA of the previous kernel in the stream has
// exited; wait() returns when that kernel has completed and its memory writes are visible.
// This kernel never triggers its own dependents early (the trigger is implicit at CTA exit):
// a trigger after the main loop let the next layer's CTAs take SM slots during the merge and
// cost 1.3 us per layer, the implicit one saves 0.8 us of launch gap per layer.
__device__ __forceinline__ void pdl_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- head exchange over peer memory: 4 result values at linear index e (a multiple of 4) of this
// rank's result view go to each peer's receive buffer as 8-byte words {value, epoch}, two 16-byte
// volatile stores (each 8-byte half is single-copy atomic, so a word whose epoch matches carries
// its value: no fence and no flag are needed; the receiver polls the words themselves).
__device__ __forceinline__ void st_ll4(char * dst, float4 v, uint32_t epoch) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(__float_as_uint(v.x)),
                 "r"(epoch), "r"(__float_as_uint(v.y)), "r"(epoch)
                 : "memory");
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(dst + 16), "r"(__float_as_uint(v.z)),
                 "r"(epoch), "r"(__float_as_uint(v.w)), "r"(epoch)
                 : "memory");
}

// byte offset of (key row j, 16-byte chunk c) inside one 128-byte-swizzled TMA box
__device__ __forceinline__ uint32_t swz(int j, int c) {
    return (uint32_t) (j * 128 + ((c ^ (j & 7)) << 4));
}

// Visible keys of a unit (its q sequence's kv_len, or n_kv).
__device__ __forceinline__ int unit_kv_len(const DecodeParams & p, int64_t unit) {
    const int sq = (int) ((unit / p.groups) / p.n_head_kv);
    return seq_kv_len(p.kv_len, sq, p.n_kv);
}

// ------------------------------------------------------------------ kernel

// CLUSTER = false: the stream-K split of fa_decode.cu (partials merged through the workspace).
// CLUSTER = true : one unit per thread-block cluster of p.cluster CTAs; CTA rank r streams key
//                  slice [r*W, (r+1)*W) of the unit, and the CTAs merge their (m, l, O) over
//                  distributed shared memory behind a cluster barrier - no global partials,
//                  fences or atomics; the workspace only carries the status word.
template <int D, bool BF16, int NT, bool CLUSTER, int NS, bool Q8>
__global__ void __launch_bounds__(MMA_THREADS, 2)
    fa_decode_mma_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                         const __grid_constant__ CUtensorMap tmm, const DecodeParams p) {
    using L            = MmaSmem<D, NT, NS, Q8>;
    constexpr int KS   = D / 16;     // k-steps of QK, m-tiles of PV
    constexpr int NBLK = D / QK8_0;  // Q8_0 blocks per row (Q8)
    constexpr int SUB  = L::CK / MMA_C;  // 16-key sub-tiles per warp and stage
    constexpr int KPW  = 16 * SUB;    // keys per warp and stage
    constexpr int CK   = L::CK;       // keys per stage
    static_assert(!(Q8 && BF16), "Q8_0 V is multiplied in f16");
    extern __shared__ __align__(16) char smem_raw[];
    // 1024-byte aligned base, derived from smem_raw by pointer arithmetic (not through an
    // integer) so that the compiler keeps plain accesses in the shared address space
    char * smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);

    float *    redO  = reinterpret_cast<float *>(smem + L::OFF_RED_O);
    float *    redML = reinterpret_cast<float *>(smem + L::OFF_RED_ML);
    uint64_t * full  = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint64_t * empty = full + NS;
    uint64_t * pushed = full + 2 * NS;  // cluster mode: this CTA's share of the partials has arrived
    int *      flag  = reinterpret_cast<int *>(smem + L::OFF_FLAG);  // [0] abort, [1] last-arriver

    const int tid  = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    // the stages this CTA streams: in cluster mode the unit's C-key chunks rank, rank + CS,
    // rank + 2 CS, ... (interleaved, so the cluster sweeps the slab together and every CTA sees
    // the same mix of memory); otherwise a contiguous range of the stream-K cut
    int64_t g0, g1;
    if (CLUSTER) {
        g0 = g1 = 0;
    } else {
        const int64_t total = p.n_units * (int64_t) p.n_kv;
        g0                  = (int64_t) blockIdx.x * p.keys_per_cta;
        g1                  = min(total, g0 + p.keys_per_cta);
        if (g0 >= g1) {
            return;
        }
    }
    if (tid == 32 * MMA_CONSUMERS) {  // the producer thread: start the descriptor fetches first
        if (!Q8) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
        }
        if (p.mask_tma) {
            asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmm)) : "memory");
        }
        for (int s = 0; s < NS; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], MMA_CONSUMERS);
        }
        mbar_init(pushed, 1u);  // cluster mode: one local arrival plus the pushed bytes
        flag[0] = 0;
        flag[1] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    if (CLUSTER) {
        cluster_arrive();  // waited for before the first remote store (cluster merge)
    }
    pdl_wait();  // nothing global (inputs, dst, workspace) is touched before this point
    const uint64_t deadline = global_timer_ns() + p.timeout_ns;

    // ================================================================ producer warp
    if (warp == MMA_CONSUMERS) {
        if (lane == 0) {
            // cluster mode streams only the unit's visible keys (kv_len); stream-K masks them instead
            StageIter it = CLUSTER ? StageIter((int64_t) (blockIdx.x / p.cluster), (int) (blockIdx.x % p.cluster) * CK,
                                          p.cluster * CK, unit_kv_len(p, blockIdx.x / p.cluster), CK)
                                : StageIter(g0, g1, p.n_kv, CK);
            int        s = 0;
            bool       ok = true;
            while (it.has()) {
                int64_t unit;
                int     j0, n;
                it.next(unit, j0, n);
                const int slot = s % NS;
                if (s >= NS) {
                    ok = mbar_wait_bounded(&empty[slot], (uint32_t) (((s / NS) - 1) & 1), deadline);
                    if (!ok) {
                        atomicExch(&flag[0], 1);
                        break;
                    }
                }
                const int sg  = (int) unit / p.groups;  // unit < 2^31 (checked on the host)
                const int g   = sg % p.n_head_kv;
                const int sq  = sg / p.n_head_kv;
                const int ks3 = sq / p.rk3;
                char *        dk  = smem + slot * L::STAGE;
                char *        dv  = dk + L::MAT;
                // TMA mask (cluster mode, so j0 is a multiple of CK; one query row and a mask
                // shared by all heads, so every row of the unit reads the same mask row): one box
                // of CK keys, zero-filled past n_kv
                const uint32_t mbytes = p.mask_tma ? (uint32_t) L::MASKB : 0u;
                if constexpr (Q8) {
                    // whole rows of K and of V; j0 * RB is a multiple of 16, and the row count is
                    // rounded up to KA rows (n * RB a multiple of 16, as bulk copies need) - a
                    // kv_len can end a chunk anywhere, but the view's n_kv is a multiple of KA
                    // (checked on the host), so the rounded rows stay inside it
                    constexpr int  KA    = (L::RB % 16 == 0) ? 1 : ((L::RB % 8 == 0) ? 2 : ((L::RB % 4 == 0) ? 4 : 8));
                    const int      nc    = min((n + KA - 1) / KA * KA, p.n_kv - j0);
                    const uint32_t bytes = (uint32_t) (nc * L::RB);
                    const char *   sk = p.k + (int64_t) g * p.k_nb2 + (int64_t) ks3 * p.k_nb3 + (int64_t) j0 * L::RB;
                    const char *   sv = p.v + (int64_t) g * p.v_nb2 + (int64_t) ks3 * p.v_nb3 + (int64_t) j0 * L::RB;
                    mbar_arrive_expect_tx(&full[slot], 2 * bytes + mbytes);
                    bulk_copy_g2s(dk, sk, bytes, &full[slot]);
                    bulk_copy_g2s(dv, sv, bytes, &full[slot]);
                } else {
                    mbar_arrive_expect_tx(&full[slot], (uint32_t) (2 * L::MAT) + mbytes);
#pragma unroll
                    for (int h = 0; h < L::HALVES; h++) {
                        tma_load_4d(dk + h * L::TILE, &tmk, h * 64, j0, g, ks3, &full[slot]);
                        tma_load_4d(dv + h * L::TILE, &tmv, h * 64, j0, g, ks3, &full[slot]);
                    }
                }
                if (p.mask_tma) {
                    tma_load_4d(dk + 2 * L::MAT, &tmm, j0, 0, 0, sq % p.m_ne3, &full[slot]);
                }
                s++;
            }
            // the last loads issued must land before this CTA's shared memory is released
            // (consumers normally wait for them too; this matters when a wait expired)
            const uint64_t drain = global_timer_ns() + p.timeout_ns;
            for (int t = max(0, s - NS); t < s; t++) {
                mbar_wait_bounded(&full[t % NS], (uint32_t) ((t / NS) & 1), drain);
            }
        }
        if (!CLUSTER) {
            return;
        }
    } else {
    // ================================================================ consumer warps
    const int g4 = lane >> 2;  // fragment row group
    const int q4 = lane & 3;   // fragment column pair

    uint32_t qb[NT][Q8 ? 1 : KS][2];   // Q^T B fragments
    uint32_t q8b[NT][Q8 ? NBLK : 1][2];  // Q8: int8 Q^T B fragments per block (dims 4*q4.., 16+4*q4..)
    float    dq[NT][Q8 ? NBLK : 1][2];   // Q8: Q block scales of rows 8*nt + 2*q4 (+1)
    // O^T fragments: (dim = acc_dim(m, 0|1), row = 8*nt + 2*q4 (+1)); F16/BF16 tile m holds dims
    // 16*m + g4 (+8), Q8_0 tile m holds dims 32*(m/2) + 4*g4 + 2*(m%2) (+1), so that one thread's
    // V bytes of a block are 4 adjacent dims and every tile lies inside one 32-dim block
    float    acc[KS][NT][4];
    auto     acc_dim = [&](int m, int hi) -> int {
        return Q8 ? 32 * (m >> 1) + 4 * g4 + 2 * (m & 1) + hi : 16 * m + g4 + 8 * hi;
    };
    float    m_run[NT][2], l_run[NT][2];
    float    slope[NT][2];
    int64_t  moff[NT][2];
    bool     rvalid[NT][2];

    int64_t cur_unit = -1;
    int     nrow     = 0;
    int     seg_j0 = 0, seg_j1 = 0;
    int     u_rgrp = 0, u_g = 0, u_sq = 0;  // the current unit's row group, kv head, q sequence
    int     u_kvl  = p.n_kv;                // the current unit's visible keys
    bool    aborted  = false;

    // mask values [sub-tile][nt][row 2*q4 + e][key 16u + g4 + 8*kh]
    float mk_cur[SUB][NT][2][2], mk_nxt[SUB][NT][2][2];
    bool  mk_have = false;  // mk_cur already holds the coming stage's values
#pragma unroll
    for (int u = 0; u < SUB; u++) {
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                mk_cur[u][nt][e][0] = mk_cur[u][nt][e][1] = 0.0f;
                mk_nxt[u][nt][e][0] = mk_nxt[u][nt][e][1] = 0.0f;
            }
        }
    }
    auto load_mask = [&](float (&mk)[SUB][NT][2][2], int j0_, int n_) {
        const int kb_ = warp * KPW;
#pragma unroll
        for (int u = 0; u < SUB; u++) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
#pragma unroll
                    for (int kh = 0; kh < 2; kh++) {
                        const int j      = kb_ + 16 * u + g4 + 8 * kh;
                        mk[u][nt][e][kh] = 0.0f;
                        if (rvalid[nt][e] && j < n_) {
                            mk[u][nt][e][kh] = __half2float(
                                *reinterpret_cast<const __half *>(p.mask + moff[nt][e] + (int64_t) (j0_ + j) * 2));
                        }
                    }
                }
            }
        }
    };

    auto begin_unit = [&](int64_t unit) {
        const int64_t sg   = unit / p.groups;
        const int     rgrp = (int) (unit % p.groups);
        const int     g    = (int) (sg % p.n_head_kv);
        const int     sq   = (int) (sg / p.n_head_kv);
        u_rgrp             = rgrp;
        u_g                = g;
        u_sq               = sq;
        u_kvl              = seq_kv_len(p.kv_len, sq, p.n_kv);
        nrow               = min(p.rows_per_unit, p.rows_per_pair - rgrp * MMA_RMAX);
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
            // B fragment rows: n = g4 -> unit row 8*nt + g4
            const int  rb = nt * 8 + g4;
            const bool vb = rb < nrow;
            const int  rf = rgrp * MMA_RMAX + rb;
            const int  hb = g * p.ratio + rf / p.n_q;
            const int  ib = rf % p.n_q;
            const char * qrow = p.q + (int64_t) ib * p.q_nb1 + (int64_t) hb * p.q_nb2 + (int64_t) sq * p.q_nb3;
            if constexpr (Q8) {
                // the quad's 4 lanes hold the 32 values of one block of row rb: Q8_0-quantize them
                // as ggml's reference quantizer does (amax over the block, d = amax/127, stored
                // as f16, q = round(x / d) with the f32 reciprocal of d).  Warp w quantizes block
                // w (and w + 4, ...) for every lane and stages the fragments in shared memory; the
                // warps pick all blocks up after the barrier below (one block's dependency chain
                // per warp instead of NBLK).
                uint4 * qx = reinterpret_cast<uint4 *>(smem + L::OFF_QX);
                for (int b = warp; b < NBLK; b += MMA_CONSUMERS) {
                    float x[8];
                    ld_q_elems(x, qrow + 0, p.q_type, vb,
                               [&](int i) { return b * QK8_0 + (i >> 2) * 16 + 4 * q4 + (i & 3); });
                    float amax = 0.0f;
#pragma unroll
                    for (int i = 0; i < 8; i++) {
                        amax = fmaxf(amax, fabsf(x[i]));
                    }
                    amax           = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 1));
                    amax           = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, 2));
                    const float d  = amax / 127.0f;
                    const float id = d != 0.0f ? 1.0f / d : 0.0f;
                    uint32_t    w[2];
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        uint32_t v = 0;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            const int qv = (int) roundf(x[h * 4 + i] * id);
                            v |= ((uint32_t) qv & 0xffu) << (8 * i);
                        }
                        w[h] = v;
                    }
                    // C-fragment rows 8*nt + 2*q4 + e live on the quads g4 = 2*q4 + e
                    const float dh  = round_to_f16(d);
                    const float dq0 = __shfl_sync(0xffffffffu, dh, (2 * q4) << 2);
                    const float dq1 = __shfl_sync(0xffffffffu, dh, (2 * q4 + 1) << 2);
                    qx[(nt * NBLK + b) * 32 + lane] = make_uint4(w[0], w[1], __float_as_uint(dq0), __float_as_uint(dq1));
                }
            } else {
                // dims 16 ks + 2 q4 + {0, 1, 8, 9} of every k-step, all loads in flight together
                float x[KS * 4];
                ld_q_elems(x, qrow, p.q_type, vb,
                           [&](int i) { return (i >> 2) * 16 + 2 * q4 + (i & 1) + ((i & 2) << 2); });
#pragma unroll
                for (int ks = 0; ks < KS; ks++) {
                    qb[nt][ks][0] = pack2<BF16>(x[4 * ks + 0], x[4 * ks + 1]);
                    qb[nt][ks][1] = pack2<BF16>(x[4 * ks + 2], x[4 * ks + 3]);
                }
            }
            // softmax state rows: 8*nt + 2*q4 + {0,1}
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int r  = nt * 8 + 2 * q4 + e;
                const int rf2 = rgrp * MMA_RMAX + r;
                const int h  = g * p.ratio + rf2 / p.n_q;
                const int i  = rf2 % p.n_q;
                rvalid[nt][e] = r < nrow;
                m_run[nt][e]  = -INFINITY;
                l_run[nt][e]  = 0.0f;
                slope[nt][e]  = rvalid[nt][e] ? alibi_slope(h, p.max_bias, p.n_head_log2, p.m0, p.m1) : 1.0f;
                moff[nt][e]   = rvalid[nt][e] ? (int64_t) i * p.m_nb1 + (int64_t) (h % p.m_ne2) * p.m_nb2 +
                                                  (int64_t) (sq % p.m_ne3) * p.m_nb3
                                              : 0;
            }
        }
        if constexpr (Q8) {  // every warp's copy of the fragments the warps staged above
            named_barrier_consumers();
            const uint4 * qx = reinterpret_cast<const uint4 *>(smem + L::OFF_QX);
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                for (int b = 0; b < NBLK; b++) {
                    const uint4 v = qx[(nt * NBLK + b) * 32 + lane];
                    q8b[nt][b][0] = v.x;
                    q8b[nt][b][1] = v.y;
                    dq[nt][b][0]  = __uint_as_float(v.z);
                    dq[nt][b][1]  = __uint_as_float(v.w);
                }
            }
            named_barrier_consumers();  // the staging area is free for the next unit's
        }
#pragma unroll
        for (int m = 0; m < KS; m++) {
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    acc[m][nt][e] = 0.0f;
                }
            }
        }
    };

    auto end_unit = [&](int64_t unit) {
        if constexpr (CLUSTER) {
            // one unit per CTA, so the ring is free: each warp parks its raw O fragments there,
            // then all consumer threads combine the 4 warps per (row, 4 dims) in one pass
            // [warp][8 NT rows][OD]: rows padded by 4 floats so that the fragment stores of one
            // warp (rows 2 q4, dims g4 + 16 m) fall in 32 different banks
            constexpr int OD = D + 4;
            float *       o4 = reinterpret_cast<float *>(smem);
            named_barrier_consumers();  // every warp is done reading the ring
#pragma unroll
            for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                for (int e = 0; e < 2; e++) {
                    float l = l_run[nt][e];
                    l += __shfl_xor_sync(0xffffffffu, l, 4);
                    l += __shfl_xor_sync(0xffffffffu, l, 8);
                    l += __shfl_xor_sync(0xffffffffu, l, 16);
                    if (g4 == 0) {
                        const int r                        = nt * 8 + 2 * q4 + e;
                        redML[(warp * 8 * NT + r) * 2 + 0] = m_run[nt][e];
                        redML[(warp * 8 * NT + r) * 2 + 1] = l;
                    }
                }
#pragma unroll
                for (int m = 0; m < KS; m++) {
                    const int r  = nt * 8 + 2 * q4;
                    const int d  = acc_dim(m, 0), d1 = acc_dim(m, 1);
                    float *   ow = o4 + (size_t) warp * 8 * NT * OD;
                    ow[r * OD + d]        = acc[m][nt][0];
                    ow[(r + 1) * OD + d]  = acc[m][nt][1];
                    ow[r * OD + d1]       = acc[m][nt][2];
                    ow[(r + 1) * OD + d1] = acc[m][nt][3];
                }
            }
            named_barrier_consumers();
            // Cluster merge by pushing (reduce-scatter over DSMEM): item (row, 4 dims) number it
            // belongs to rank it / IPR, a contiguous range per rank, so that the owner's result
            // stores (and its peer-exchange words) of consecutive threads are consecutive in
            // memory (whole lines over NVLink; the interleaved it % CS split measured 4.6 us of
            // exchange per layer at 8 GPUs).  This CTA combines its 4 warps per item and stores the result
            // into the owner's receive buffer, and its (m, l) per row into every rank's, as
            // asynchronous stores that count their bytes on the receiver's `pushed` barrier.  Each
            // rank expects the bytes of its share from all CS ranks, waits for them and merges its
            // items from local memory, so no CTA ever reads another's memory and no fence or
            // cluster barrier follows.
            const int      CS    = p.cluster;
            const uint32_t rank  = cluster_ctarank();
            const int      total = nrow * (D / 4);
            const int      IPR   = (total + CS - 1) / CS;  // items per rank
            float4 *       rcv_o  = reinterpret_cast<float4 *>(redO);  // [source][IPR]
            float2 *       rcv_ml = reinterpret_cast<float2 *>(smem + L::OFF_RECV_ML);  // [source][8 NT]
            if (tid == 0) {
                const int mine = max(0, min(IPR, total - (int) rank * IPR));
                mbar_arrive_expect_tx(pushed, (uint32_t) (CS * (mine * 16 + nrow * 8)));
            }
            cluster_wait();  // every CTA of the cluster has initialised its barriers
            for (int it4 = tid; it4 < total; it4 += 32 * MMA_CONSUMERS) {
                const int r = it4 / (D / 4), d = (it4 % (D / 4)) * 4;
                float     mw[MMA_CONSUMERS], M = -INFINITY;
#pragma unroll
                for (int w = 0; w < MMA_CONSUMERS; w++) {
                    mw[w] = redML[(w * 8 * NT + r) * 2];
                    M     = fmaxf(M, mw[w]);
                }
                float4 O  = make_float4(0.f, 0.f, 0.f, 0.f);
                float  Ls = 0.0f;
#pragma unroll
                for (int w = 0; w < MMA_CONSUMERS; w++) {
                    const float  wt = mw[w] == -INFINITY ? 0.0f : exp2f(mw[w] - M);
                    const float4 v  = *reinterpret_cast<const float4 *>(o4 + ((size_t) w * 8 * NT + r) * OD + d);
                    O.x += wt * v.x;
                    O.y += wt * v.y;
                    O.z += wt * v.z;
                    O.w += wt * v.w;
                    Ls += wt * redML[(w * 8 * NT + r) * 2 + 1];
                }
                const uint32_t owner = (uint32_t) (it4 / IPR);
                st_async4(dsmem_addr(&rcv_o[(int) rank * IPR + (it4 - (int) owner * IPR)], owner), O,
                          dsmem_addr(pushed, owner));
                if (d == 0) {
                    for (int c = 0; c < CS; c++) {
                        st_async2(dsmem_addr(&rcv_ml[(int) rank * 8 * NT + r], (uint32_t) c), make_float2(M, Ls),
                                  dsmem_addr(pushed, (uint32_t) c));
                    }
                }
            }
            if (!mbar_wait_cluster_bounded(pushed, 0, global_timer_ns() + p.timeout_ns)) {
                if (tid == 0) {
                    atomicExch(&flag[0], 1);
                }
                return;
            }
            for (int li = tid; li < IPR; li += 32 * MMA_CONSUMERS) {
                const int it4 = (int) rank * IPR + li;
                if (it4 >= total) {
                    break;
                }
                const int r = it4 / (D / 4), d = (it4 % (D / 4)) * 4;
                // every source's (m, l) and partial O loaded before any is used: unrolled to the
                // largest cluster with the index clamped (always in bounds, no branches), so that
                // the loads are in flight together; sources from CS on are skipped in the sums
                float2 ml[MMA_MAX_CLUSTER];
                float4 po[MMA_MAX_CLUSTER];
                float  M = -INFINITY;
#pragma unroll
                for (int c = 0; c < MMA_MAX_CLUSTER; c++) {
                    const int cc = min(c, CS - 1);
                    ml[c]        = rcv_ml[cc * 8 * NT + r];
                    po[c]        = rcv_o[cc * IPR + li];
                }
#pragma unroll
                for (int c = 0; c < MMA_MAX_CLUSTER; c++) {
                    M = c < CS ? fmaxf(M, ml[c].x) : M;
                }
                float4 O  = make_float4(0.f, 0.f, 0.f, 0.f);
                float  Ls = 0.0f;
                if (M != -INFINITY) {
#pragma unroll
                    for (int c = 0; c < MMA_MAX_CLUSTER; c++) {
                        if (c < CS) {
                            const float  w = ml[c].x == -INFINITY ? 0.0f : exp2f(ml[c].x - M);
                            const float4 v = po[c];
                            O.x += w * v.x;
                            O.y += w * v.y;
                            O.z += w * v.z;
                            O.w += w * v.w;
                            Ls += w * ml[c].y;
                        }
                    }
                }
                const float inv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
                const int   rf  = u_rgrp * MMA_RMAX + r;
                const int   h   = u_g * p.ratio + rf / p.n_q;
                const int   i   = rf % p.n_q;
                float *     out = reinterpret_cast<float *>(p.dst + (int64_t) h * p.d_nb1 + (int64_t) i * p.d_nb2 +
                                                        (int64_t) u_sq * p.d_nb3) + d;
                if (p.dst_vec) {
                    const float4 r4                  = make_float4(O.x * inv, O.y * inv, O.z * inv, O.w * inv);
                    *reinterpret_cast<float4 *>(out) = r4;
                    if (p.n_peers > 0) {
                        // head exchange over peer memory: the 4 values into every peer's receive
                        // buffer as {value, epoch} words (the host guarantees dst_vec)
                        const uint32_t epoch = *p.epoch_ptr + 1u;
                        const int64_t  e = d + (int64_t) D * (h + (int64_t) p.n_head * (i + (int64_t) p.n_q * u_sq));
                        const int64_t  off = (int64_t) (epoch & 1u) * p.ll_parity + 8 * e;
#pragma unroll
                        for (int pp = 0; pp < MAX_PEERS; pp++) {
                            if (pp < p.n_peers) {
                                st_ll4(p.peer_ll[pp] + off, r4, epoch);
                            }
                        }
                    }
                } else {
                    out[0] = O.x * inv;
                    out[1] = O.y * inv;
                    out[2] = O.z * inv;
                    out[3] = O.w * inv;
                }
            }
            return;
        } else {
        // each warp's (m, l) per row to shared memory, l summed over the 8 key lanes
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                float l = l_run[nt][e];
                l += __shfl_xor_sync(0xffffffffu, l, 4);
                l += __shfl_xor_sync(0xffffffffu, l, 8);
                l += __shfl_xor_sync(0xffffffffu, l, 16);
                if (g4 == 0) {
                    const int r                        = nt * 8 + 2 * q4 + e;
                    redML[(warp * 8 * NT + r) * 2 + 0] = m_run[nt][e];
                    redML[(warp * 8 * NT + r) * 2 + 1] = l;
                }
            }
        }
        named_barrier_consumers();
        // the warps add their O, rescaled to the unit's row maximum, into one buffer in warp order
        float scl[NT][2];
#pragma unroll
        for (int nt = 0; nt < NT; nt++) {
#pragma unroll
            for (int e = 0; e < 2; e++) {
                const int r = nt * 8 + 2 * q4 + e;
                float     M = -INFINITY;
#pragma unroll
                for (int w = 0; w < MMA_CONSUMERS; w++) {
                    M = fmaxf(M, redML[(w * 8 * NT + r) * 2]);
                }
                scl[nt][e] = m_run[nt][e] == -INFINITY ? 0.0f : exp2f(m_run[nt][e] - M);
            }
        }
        for (int w = 0; w < MMA_CONSUMERS; w++) {
            if (warp == w) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                    for (int m = 0; m < KS; m++) {
                        const int r   = nt * 8 + 2 * q4;
                        const int d   = acc_dim(m, 0), d1 = acc_dim(m, 1);
                        float *   o00 = &redO[r * D + d];
                        float *   o10 = &redO[(r + 1) * D + d];
                        float *   o01 = &redO[r * D + d1];
                        float *   o11 = &redO[(r + 1) * D + d1];
                        const float v00 = scl[nt][0] * acc[m][nt][0], v10 = scl[nt][1] * acc[m][nt][1];
                        const float v01 = scl[nt][0] * acc[m][nt][2], v11 = scl[nt][1] * acc[m][nt][3];
                        *o00 = w == 0 ? v00 : *o00 + v00;
                        *o10 = w == 0 ? v10 : *o10 + v10;
                        *o01 = w == 0 ? v01 : *o01 + v01;
                        *o11 = w == 0 ? v11 : *o11 + v11;
                    }
                }
            }
            named_barrier_consumers();
        }
        // flag[0] can be raised by the producer at any time: decide once, for all warps alike
        if (!consumers_any(flag[0] != 0)) {
            const int     nthr    = 32 * MMA_CONSUMERS;
            const bool    whole   = seg_j0 == 0 && seg_j1 == p.n_kv;
            const int64_t u_first = unit * (int64_t) p.n_kv / p.keys_per_cta;
            for (int idx = tid; idx < nrow * D; idx += nthr) {
                const int r = idx / D, d = idx % D;
                float     M = -INFINITY;
#pragma unroll
                for (int w = 0; w < MMA_CONSUMERS; w++) {
                    M = fmaxf(M, redML[(w * 8 * NT + r) * 2]);
                }
                float O = 0.0f, Ls = 0.0f;
                if (M != -INFINITY) {
                    O = redO[r * D + d];
#pragma unroll
                    for (int w = 0; w < MMA_CONSUMERS; w++) {
                        const float mw = redML[(w * 8 * NT + r) * 2];
                        Ls += (mw == -INFINITY ? 0.0f : exp2f(mw - M)) * redML[(w * 8 * NT + r) * 2 + 1];
                    }
                }
                const int rf = u_rgrp * MMA_RMAX + r;
                const int h  = u_g * p.ratio + rf / p.n_q;
                const int i  = rf % p.n_q;
                if (whole) {
                    float * dst = reinterpret_cast<float *>(p.dst + (int64_t) h * p.d_nb1 + (int64_t) i * p.d_nb2 +
                                                            (int64_t) u_sq * p.d_nb3);
                    dst[d]      = Ls > 0.0f ? O / Ls : 0.0f;
                } else {
                    const int64_t pbase = unit * p.max_slots + ((int64_t) blockIdx.x - u_first);
                    p.part_o[pbase * MMA_RMAX * D + (int64_t) r * D + d] = O;
                    if (d == 0) {
                        p.part_ml[(pbase * MMA_RMAX + r) * 2 + 0] = M;
                        p.part_ml[(pbase * MMA_RMAX + r) * 2 + 1] = Ls;
                    }
                }
            }
            if (!whole) {
                __threadfence();
                named_barrier_consumers();
                if (tid == 0) {
                    const int64_t  first = unit * (int64_t) p.n_kv / p.keys_per_cta;
                    const int64_t  last  = (unit * (int64_t) p.n_kv + p.n_kv - 1) / p.keys_per_cta;
                    const uint32_t old   = atomicAdd(&p.counters[unit], 1u);
                    flag[1]              = (old == (uint32_t) (last - first)) ? 1 : 0;
                }
                named_barrier_consumers();
                if (flag[1]) {
                    __threadfence();
                    const int64_t first = unit * (int64_t) p.n_kv / p.keys_per_cta;
                    const int64_t last  = (unit * (int64_t) p.n_kv + p.n_kv - 1) / p.keys_per_cta;
                    const int     rgrp  = u_rgrp, g = u_g, sq = u_sq;
                    // redO / redML are free here: this CTA's own partial is already in the workspace
                    merge_unit_partials<D, MMA_RMAX, 8 * NT, 32 * MMA_CONSUMERS>(
                        p, unit, (int) (last - first + 1), nrow, tid, redO, redML, [] { named_barrier_consumers(); },
                        [&](int r) {
                            const int rf = rgrp * MMA_RMAX + r;
                            const int h  = g * p.ratio + rf / p.n_q;
                            const int i  = rf % p.n_q;
                            return reinterpret_cast<float *>(p.dst + (int64_t) h * p.d_nb1 + (int64_t) i * p.d_nb2 +
                                                             (int64_t) sq * p.d_nb3);
                        });
                    if (tid == 0) {
                        p.counters[unit] = 0u;
                    }
                }
            }
        }
        named_barrier_consumers();  // shared reduction buffers are free again
        }
    };

    if (CLUSTER) {  // the cluster's unit, even when this CTA's key slice is empty
        cur_unit = blockIdx.x / p.cluster;
        begin_unit(cur_unit);
    }
    StageIter it = CLUSTER ? StageIter((int64_t) (blockIdx.x / p.cluster), (int) (blockIdx.x % p.cluster) * CK,
                                          p.cluster * CK, unit_kv_len(p, blockIdx.x / p.cluster), CK)
                                : StageIter(g0, g1, p.n_kv, CK);
    int        s = 0;
    while (it.has()) {
        int64_t unit;
        int     j0, n;
        it.next(unit, j0, n);
        if (unit != cur_unit) {
            if (cur_unit >= 0) {
                end_unit(cur_unit);
            }
            begin_unit(unit);
            cur_unit = unit;
            seg_j0   = j0;
        }
        seg_j1 = j0 + n;

        const int slot = s % NS;
        const int kb   = warp * KPW;  // this warp's first key in the stage
        // mask values of this warp's keys: mk_cur for this stage (prefetched one stage ahead when
        // the next stage is in the same unit), mk_nxt requested now for the next stage
        if (p.mask && !p.mask_tma) {
            if (!mk_have) {
                load_mask(mk_cur, j0, n);
            }
            StageIter pk = it;
            mk_have      = false;
            if (pk.has()) {
                int64_t un;
                int     jn, nn;
                pk.next(un, jn, nn);
                if (un == unit) {
                    load_mask(mk_nxt, jn, nn);
                    mk_have = true;
                }
            }
        }
        if (!aborted) {
            aborted = !mbar_wait_bounded(&full[slot], (uint32_t) ((s / NS) & 1), deadline);
            if (aborted) {
                atomicExch(&flag[0], 1);
            }
        }
        if (!aborted && kb < n && p.mask_tma) {  // this stage's mask rows, staged with K and V
            const char * mrow = smem + slot * L::STAGE + 2 * L::MAT;
#pragma unroll
            for (int u = 0; u < SUB; u++) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                    for (int e = 0; e < 2; e++) {
#pragma unroll
                        for (int kh = 0; kh < 2; kh++) {
                            const int j          = kb + 16 * u + g4 + 8 * kh;
                            mk_cur[u][nt][e][kh] = rvalid[nt][e] ? lds_half(mrow + j * 2) : 0.0f;
                        }
                    }
                }
            }
        }
        if (!aborted && kb < n) {
            if constexpr (Q8) {
                // This warp's KPW keys as SUB independent 16-key sub-tiles (their loads, int8 dots
                // and conversions interleave), one online-softmax update for all of them.
                const char * kst = smem + slot * L::STAGE;
                const char * vst = kst + L::MAT;
                // ---- S^T = K Q^T: per block, int8 A fragments of key rows kb + 16u + g4 (+8)
                // (bytes 4*q4.. and 16 + 4*q4.. of the block's values; blocks at even indices
                // start 2 bytes past a word boundary), the exact int32 dot, then both f16 scales
                float sc[SUB][NT][4];
#pragma unroll
                for (int b = 0; b < NBLK; b++) {
#pragma unroll
                    for (int u = 0; u < SUB; u++) {
                        const char * r0 = kst + (kb + 16 * u + g4) * L::RB;
                        const char * r1 = r0 + 8 * L::RB;
                        const int    o  = b * Q8_0_BLOCK + 2 + 4 * q4;
                        uint32_t     a0, a1, a2, a3;
                        if (b & 1) {
                            a0 = lds_word<0>(r0 + o);
                            a1 = lds_word<0>(r1 + o);
                            a2 = lds_word<0>(r0 + o + 16);
                            a3 = lds_word<0>(r1 + o + 16);
                        } else {
                            a0 = lds_word<2>(r0 + o);
                            a1 = lds_word<2>(r1 + o);
                            a2 = lds_word<2>(r0 + o + 16);
                            a3 = lds_word<2>(r1 + o + 16);
                        }
                        const float dk0 = lds_half(r0 + b * Q8_0_BLOCK);
                        const float dk1 = lds_half(r1 + b * Q8_0_BLOCK);
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            int c[4] = { 0, 0, 0, 0 };
                            mma_s8_16832(c, a0, a1, a2, a3, q8b[nt][b][0], q8b[nt][b][1]);
                            const float f[4] = { dk0 * dq[nt][b][0], dk0 * dq[nt][b][1], dk1 * dq[nt][b][0],
                                                 dk1 * dq[nt][b][1] };
#pragma unroll
                            for (int e = 0; e < 4; e++) {
                                sc[u][nt][e] = b == 0 ? (float) c[e] * f[e] : sc[u][nt][e] + (float) c[e] * f[e];
                            }
                        }
                    }
                }
                // V block scales of keys kb + 16u + g4 (+8); zero past the stage's keys, where the
                // ring holds stale bytes (P is zero there, and 0 * NaN must not occur)
                float dv[SUB][2][NBLK];
#pragma unroll
                for (int u = 0; u < SUB; u++) {
#pragma unroll
                    for (int kh = 0; kh < 2; kh++) {
                        const int    j  = kb + 16 * u + g4 + 8 * kh;
                        const char * vr = vst + j * L::RB;
#pragma unroll
                        for (int b = 0; b < NBLK; b++) {
                            dv[u][kh][b] = j < n ? lds_half(vr + b * Q8_0_BLOCK) : 0.0f;
                        }
                    }
                }
                // ---- online softmax over the warp's keys; P scaled by each key's V block scale
                uint32_t pb8[SUB][NT][NBLK][2];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float x[SUB][4];
#pragma unroll
                    for (int u = 0; u < SUB; u++) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            const int re = e & 1;   // row 2*q4 + re
                            const int kh = e >> 1;  // key 16u + g4 + 8*kh
                            const int j  = kb + 16 * u + g4 + 8 * kh;
                            float     v  = sc[u][nt][e] * p.scale;
                            if (p.softcap != 0.0f) {
                                v = p.softcap * tanhf(v / p.softcap);
                            }
                            v += slope[nt][re] * mk_cur[u][nt][re][kh];
                            x[u][e] = (j < n && j0 + j < u_kvl) ? v * LOG2E : -INFINITY;
                        }
                    }
                    float mx0 = fmaxf(x[0][0], x[0][2]), mx1 = fmaxf(x[0][1], x[0][3]);
#pragma unroll
                    for (int u = 1; u < SUB; u++) {
                        mx0 = fmaxf(mx0, fmaxf(x[u][0], x[u][2]));
                        mx1 = fmaxf(mx1, fmaxf(x[u][1], x[u][3]));
                    }
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
                    }
                    const float mn0 = fmaxf(m_run[nt][0], mx0);
                    const float mn1 = fmaxf(m_run[nt][1], mx1);
                    const float al0 = mn0 == -INFINITY ? 1.0f : exp2f(m_run[nt][0] - mn0);
                    const float al1 = mn1 == -INFINITY ? 1.0f : exp2f(m_run[nt][1] - mn1);
                    m_run[nt][0]    = mn0;
                    m_run[nt][1]    = mn1;
                    float ls0 = 0.0f, ls1 = 0.0f;
#pragma unroll
                    for (int u = 0; u < SUB; u++) {
                        const float p0 = mn0 == -INFINITY ? 0.0f : exp2f(x[u][0] - mn0);
                        const float p1 = mn1 == -INFINITY ? 0.0f : exp2f(x[u][1] - mn1);
                        const float p2 = mn0 == -INFINITY ? 0.0f : exp2f(x[u][2] - mn0);
                        const float p3 = mn1 == -INFINITY ? 0.0f : exp2f(x[u][3] - mn1);
                        ls0 += p0 + p2;
                        ls1 += p1 + p3;
#pragma unroll
                        for (int b = 0; b < NBLK; b++) {
                            pb8[u][nt][b][0] = movmatrix_t(pack2<false>(p0 * dv[u][0][b], p1 * dv[u][0][b]));
                            pb8[u][nt][b][1] = movmatrix_t(pack2<false>(p2 * dv[u][1][b], p3 * dv[u][1][b]));
                        }
                    }
                    l_run[nt][0] = l_run[nt][0] * al0 + ls0;
                    l_run[nt][1] = l_run[nt][1] * al1 + ls1;
#pragma unroll
                    for (int m = 0; m < KS; m++) {
                        acc[m][nt][0] *= al0;
                        acc[m][nt][1] *= al1;
                        acc[m][nt][2] *= al0;
                        acc[m][nt][3] *= al1;
                    }
                }
                // ---- O^T += V^T (P dv)^T: per block, 4 adjacent dims 32*b + 4*g4.. of the
                // B-fragment keys kb + 16u + 2*q4 + {0, 1, 8, 9}, byte-interleaved per key pair
                // and widened to f16 (exact)
#pragma unroll
                for (int b = 0; b < NBLK; b++) {
#pragma unroll
                    for (int u = 0; u < SUB; u++) {
                        const char * v0 = vst + (kb + 16 * u + 2 * q4) * L::RB;
                        const int    o  = b * Q8_0_BLOCK + 2 + 4 * g4;
                        uint32_t     w0, w1, w8, w9;
                        if (b & 1) {
                            w0 = lds_word<0>(v0 + o);
                            w1 = lds_word<0>(v0 + L::RB + o);
                            w8 = lds_word<0>(v0 + 8 * L::RB + o);
                            w9 = lds_word<0>(v0 + 9 * L::RB + o);
                        } else {
                            w0 = lds_word<2>(v0 + o);
                            w1 = lds_word<2>(v0 + L::RB + o);
                            w8 = lds_word<2>(v0 + 8 * L::RB + o);
                            w9 = lds_word<2>(v0 + 9 * L::RB + o);
                        }
                        w0 ^= 0x80808080u;
                        w1 ^= 0x80808080u;
                        w8 ^= 0x80808080u;
                        w9 ^= 0x80808080u;
                        const uint32_t lo01 = __byte_perm(w0, w1, 0x5140), hi01 = __byte_perm(w0, w1, 0x7362);
                        const uint32_t lo89 = __byte_perm(w8, w9, 0x5140), hi89 = __byte_perm(w8, w9, 0x7362);
                        const uint32_t e0 = i8x2_to_h2<0x4140>(lo01), e1 = i8x2_to_h2<0x4342>(lo01);
                        const uint32_t e2 = i8x2_to_h2<0x4140>(lo89), e3 = i8x2_to_h2<0x4342>(lo89);
                        const uint32_t f0 = i8x2_to_h2<0x4140>(hi01), f1 = i8x2_to_h2<0x4342>(hi01);
                        const uint32_t f2 = i8x2_to_h2<0x4140>(hi89), f3 = i8x2_to_h2<0x4342>(hi89);
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            mma16816<false>(acc[2 * b][nt], e0, e1, e2, e3, pb8[u][nt][b][0], pb8[u][nt][b][1]);
                            mma16816<false>(acc[2 * b + 1][nt], f0, f1, f2, f3, pb8[u][nt][b][0], pb8[u][nt][b][1]);
                        }
                    }
                }
            } else {
                const uint32_t sk = smem_addr(smem + slot * L::STAGE);
                const uint32_t sv = sk + L::MAT;
                // ---- S^T = K Q^T for this warp's 16 keys
                float sc[NT][4];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        sc[nt][e] = 0.0f;
                    }
                }
                {
                    // all K fragments first (one shared-memory latency), then two independent
                    // accumulation chains over the even and odd k-steps
                    const int krow = kb + (lane & 7) + ((lane >> 3) & 1) * 8;  // A rows supplied by this lane
                    uint32_t  af[KS][4];
#pragma unroll
                    for (int ks = 0; ks < KS; ks++) {
                        const int dim0 = ks * 16 + (lane >> 4) * 8;
                        ldsm_x4(sk + (dim0 >> 6) * L::TILE + swz(krow, (dim0 & 63) >> 3), af[ks][0], af[ks][1],
                                af[ks][2], af[ks][3]);
                    }
                    float sc1[NT][4];
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            sc1[nt][e] = 0.0f;
                        }
                    }
#pragma unroll
                    for (int ks = 0; ks < KS; ks++) {
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            mma16816<BF16>((ks & 1) ? sc1[nt] : sc[nt], af[ks][0], af[ks][1], af[ks][2], af[ks][3],
                                           qb[nt][ks][0], qb[nt][ks][1]);
                        }
                    }
#pragma unroll
                    for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                        for (int e = 0; e < 4; e++) {
                            sc[nt][e] += sc1[nt][e];
                        }
                    }
                }
                // ---- online softmax (per warp), P^T -> P fragments
                uint32_t pb[NT][2];
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
                    float x[4];
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int re = e & 1;       // row 2*q4 + re
                        const int kh = e >> 1;      // key g4 + 8*kh
                        const int j  = kb + g4 + 8 * kh;
                        float     v  = sc[nt][e] * p.scale;
                        if (p.softcap != 0.0f) {
                            v = p.softcap * tanhf(v / p.softcap);
                        }
                        v += slope[nt][re] * mk_cur[0][nt][re][kh];
                        x[e] = (j < n && j0 + j < u_kvl) ? v * LOG2E : -INFINITY;
                    }
                    float mx0 = fmaxf(x[0], x[2]), mx1 = fmaxf(x[1], x[3]);
#pragma unroll
                    for (int o = 4; o < 32; o <<= 1) {
                        mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, o));
                        mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, o));
                    }
                    const float mn0 = fmaxf(m_run[nt][0], mx0);
                    const float mn1 = fmaxf(m_run[nt][1], mx1);
                    const float al0 = mn0 == -INFINITY ? 1.0f : exp2f(m_run[nt][0] - mn0);
                    const float al1 = mn1 == -INFINITY ? 1.0f : exp2f(m_run[nt][1] - mn1);
                    m_run[nt][0]    = mn0;
                    m_run[nt][1]    = mn1;
                    const float p0  = mn0 == -INFINITY ? 0.0f : exp2f(x[0] - mn0);
                    const float p1  = mn1 == -INFINITY ? 0.0f : exp2f(x[1] - mn1);
                    const float p2  = mn0 == -INFINITY ? 0.0f : exp2f(x[2] - mn0);
                    const float p3  = mn1 == -INFINITY ? 0.0f : exp2f(x[3] - mn1);
                    l_run[nt][0]    = l_run[nt][0] * al0 + p0 + p2;
                    l_run[nt][1]    = l_run[nt][1] * al1 + p1 + p3;
#pragma unroll
                    for (int m = 0; m < KS; m++) {
                        acc[m][nt][0] *= al0;
                        acc[m][nt][1] *= al1;
                        acc[m][nt][2] *= al0;
                        acc[m][nt][3] *= al1;
                    }
                    pb[nt][0] = movmatrix_t(pack2<BF16>(p0, p1));  // keys 0-7 of the warp's 16
                    pb[nt][1] = movmatrix_t(pack2<BF16>(p2, p3));  // keys 8-15
                }
                // ---- O^T += V^T P^T over this warp's 16 keys
                {
                    const int vkey = kb + (lane & 7) + ((lane >> 4) & 1) * 8;  // stored V row for ldmatrix.trans
                    uint32_t  vf[KS][4];
#pragma unroll
                    for (int m = 0; m < KS; m++) {
                        const int dim0 = m * 16 + ((lane >> 3) & 1) * 8;
                        ldsm_x4_t(sv + (dim0 >> 6) * L::TILE + swz(vkey, (dim0 & 63) >> 3), vf[m][0], vf[m][1],
                                  vf[m][2], vf[m][3]);
                    }
#pragma unroll
                    for (int m = 0; m < KS; m++) {
#pragma unroll
                        for (int nt = 0; nt < NT; nt++) {
                            mma16816<BF16>(acc[m][nt], vf[m][0], vf[m][1], vf[m][2], vf[m][3], pb[nt][0], pb[nt][1]);
                        }
                    }
                }
            }
        }
        __syncwarp();
        if (lane == 0) {
            mbar_arrive(&empty[slot]);  // this warp is done with the ring slot
        }
        if (p.mask && !p.mask_tma) {
#pragma unroll
            for (int u = 0; u < SUB; u++) {
#pragma unroll
                for (int nt = 0; nt < NT; nt++) {
#pragma unroll
                    for (int e = 0; e < 2; e++) {
#pragma unroll
                        for (int kh = 0; kh < 2; kh++) {
                            mk_cur[u][nt][e][kh] = mk_nxt[u][nt][e][kh];
                        }
                    }
                }
            }
        }
        s++;
    }
    if (cur_unit >= 0) {
        end_unit(cur_unit);
    }
    }  // consumer warps

    if (flag[0] && tid == 0) {
        atomicOr(&p.status[0], ST_TIMEOUT);
        atomicExch(&p.status[1], (uint32_t) blockIdx.x);
    }
}

// ------------------------------------------------------------------ host side

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    static std::once_flag                     once;
    std::call_once(once, [] {
        void *                          ptr = nullptr;
        cudaDriverEntryPointQueryResult q   = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
        }
        cudaGetLastError();
    });
    return fn;
}

// 4-D map of a [D, n_kv, Hkv, S_k] ggml view, box = 64 elements x box_rows keys, 128-byte swizzle.
bool encode_kv_tensor_map(CUtensorMap * tm, const void * data, bool bf16, int64_t D, int64_t n_kv, int64_t hkv,
                          int64_t sk, int64_t nb1, int64_t nb2, int64_t nb3, int box_rows) {
    auto enc = tensor_map_encoder();
    if (!enc) {
        return false;
    }
    // strides of size-1 dims are never stepped; give them the natural value
    if (hkv == 1) {
        nb2 = nb1 * n_kv;
    }
    if (sk == 1) {
        nb3 = nb2 * hkv;
    }
    cuuint64_t dims[4]    = { (cuuint64_t) D, (cuuint64_t) n_kv, (cuuint64_t) hkv, (cuuint64_t) sk };
    cuuint64_t strides[3] = { (cuuint64_t) nb1, (cuuint64_t) nb2, (cuuint64_t) nb3 };
    cuuint32_t box[4]     = { 64, (cuuint32_t) box_rows, 1, 1 };
    cuuint32_t estr[4]    = { 1, 1, 1, 1 };
    CUresult   r = enc(tm, bf16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                       const_cast<void *>(data), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                       CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

bool tensor_maps_available() {
    return tensor_map_encoder() != nullptr;
}

namespace {

// 4-D map of an F16 mask [n_kv, n_q, m_ne2, m_ne3] (rows n_q and up are never read), box = ck
// keys of one row, no swizzle, keys past n_kv read as zero.  False unless the base and the row
// strides are 16-byte multiples.  The kernel uses it for one query row and a mask shared by
// all heads, where all rows of a unit read the same mask row.
bool encode_mask_tensor_map(CUtensorMap * tm, const DecodeParams & p, int ck) {
    auto enc = tensor_map_encoder();
    if (!enc || !p.mask || reinterpret_cast<uintptr_t>(p.mask) % 16 != 0) {
        return false;
    }
    int64_t nb1 = p.m_nb1, nb2 = p.m_nb2, nb3 = p.m_nb3;
    if (p.n_q == 1) {
        nb1 = ((int64_t) p.n_kv * 2 + 15) / 16 * 16;  // never stepped
    }
    if (p.m_ne2 == 1) {
        nb2 = nb1 * p.n_q;
    }
    if (p.m_ne3 == 1) {
        nb3 = nb2 * p.m_ne2;
    }
    if (nb1 % 16 || nb2 % 16 || nb3 % 16) {
        return false;
    }
    cuuint64_t dims[4]    = { (cuuint64_t) p.n_kv, (cuuint64_t) p.n_q, (cuuint64_t) p.m_ne2, (cuuint64_t) p.m_ne3 };
    cuuint64_t strides[3] = { (cuuint64_t) nb1, (cuuint64_t) nb2, (cuuint64_t) nb3 };
    cuuint32_t box[4]     = { (cuuint32_t) ck, 1, 1, 1 };
    cuuint32_t estr[4]    = { 1, 1, 1, 1 };
    CUresult   r = enc(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<char *>(p.mask), dims, strides, box, estr,
                       CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_128B,
                       CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

namespace {

// Q8_0 ring depth: 3 stages of 128 keys (34 KiB each at D=128; 64 keys with 16 rows per unit).
constexpr int Q8_NSTAGE = 3;

template <int D, bool BF16, int NT, bool CL, bool Q8>
void * mma_kernel(int ns, int & smem) {
    if constexpr (Q8) {
        smem = MmaSmem<D, NT, Q8_NSTAGE, true>::TOTAL;
        return reinterpret_cast<void *>(&fa_decode_mma_kernel<D, false, NT, CL, Q8_NSTAGE, true>);
    } else {
        if (ns == 2) {
            smem = MmaSmem<D, NT, 2>::TOTAL;
            return reinterpret_cast<void *>(&fa_decode_mma_kernel<D, BF16, NT, CL, 2, false>);
        }
        smem = MmaSmem<D, NT, 3>::TOTAL;
        return reinterpret_cast<void *>(&fa_decode_mma_kernel<D, BF16, NT, CL, 3, false>);
    }
}

// F16/BF16 ring depth: 3 stages of 64 keys per CTA (two CTAs per SM, up to 192 KiB of K/V in
// flight per SM at D=128; measured 3% faster than 2 stages on the 36-layer decode graph) or 2
// with MM3FA_DECODE_NSTAGE=2.  A 4-stage ring at one CTA per SM (so that the headline's 16
// clusters of 9 CTAs sit one per SM instead of 13-CTA clusters two per SM) measured 19.9 against
// 14.6 us per layer: one CTA's 4 consumer warps do not keep an SM's share of HBM in flight.  A
// variant with 8 consumer warps, 128-key stages and one CTA per SM (clusters of 6: 96 CTAs, 192 KiB
// in flight per SM) measured 14.42 against 14.38 us per layer for F16 and 16.3 against 14.1 for
// Q8_0, so neither the CTA layout nor the SMs left idle limit the headline.
int mma_nstage_forced() {
    static const int ns = [] {
        const char * e = std::getenv("MM3FA_DECODE_NSTAGE");
        return (e && std::atoi(e) == 2) ? 2 : 0;
    }();
    return ns;
}

void * select_mma_kernel(int D, int kvt, int nt, bool cluster, int & smem, int ns = 3) {
    const bool bf16 = kvt == KV_BF16, q8 = kvt == KV_Q8_0;
#define MM3FA_SELM(DD, BB, QQ, NN)                                                                 \
    if (D == DD && bf16 == BB && q8 == QQ && nt == NN) {                                           \
        return cluster ? mma_kernel<DD, BB, NN, true, QQ>(ns, smem) : mma_kernel<DD, BB, NN, false, QQ>(ns, smem); \
    }
    MM3FA_SELM(128, false, false, 1)
    MM3FA_SELM(128, false, false, 2)
    MM3FA_SELM(128, true, false, 1)
    MM3FA_SELM(128, true, false, 2)
    MM3FA_SELM(128, false, true, 1)
    MM3FA_SELM(128, false, true, 2)
    MM3FA_SELM(64, false, false, 1)
    MM3FA_SELM(64, false, false, 2)
    MM3FA_SELM(64, true, false, 1)
    MM3FA_SELM(64, true, false, 2)
    MM3FA_SELM(64, false, true, 1)
    MM3FA_SELM(64, false, true, 2)
#undef MM3FA_SELM
    return nullptr;
}

// Clusters of `cs` CTAs the device can hold at once for this kernel (0 if it cannot).
int max_active_clusters(void * fn, int cs, int smem) {
    if (cs > 8) {
        if (cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1) != cudaSuccess) {
            cudaGetLastError();
            return 0;
        }
    }
    cudaLaunchConfig_t   cfg{};
    cudaLaunchAttribute  attr[1];
    cfg.gridDim          = dim3((unsigned) cs);
    cfg.blockDim         = dim3(MMA_THREADS);
    cfg.dynamicSmemBytes = (size_t) smem;
    attr[0].id               = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned) cs;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs                = attr;
    cfg.numAttrs             = 1;
    int n                    = 0;
    if (cudaOccupancyMaxActiveClusters(&n, fn, &cfg) != cudaSuccess) {
        cudaGetLastError();
        return 0;
    }
    return n;
}

}  // namespace

bool decode_mma_eligible(int D, int kvt, int rows_per_pair) {
    if (kvt == KV_Q8_0) {
        return (D == 64 || D == 128) && rows_per_pair <= 16;
    }
    return (kvt == KV_F16 || kvt == KV_BF16) && (D == 64 || D == 128) && rows_per_pair <= 16 &&
           tensor_map_encoder() != nullptr;
}

int decode_mma_ctas_per_sm(int D, int kvt, int rows_per_pair) {
    int    smem = 0;
    void * fn   = select_mma_kernel(D, kvt, rows_per_pair <= 8 ? 1 : 2, false, smem, mma_nstage_forced() == 2 ? 2 : 3);
    if (!fn) {
        return 0;
    }
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, MMA_THREADS, smem) != cudaSuccess || nb < 1) {
        cudaGetLastError();
        nb = 1;
    }
    return nb;
}

// Launch plan of the cluster split for `n_units` units on a device with n_sms SMs: the largest
// cluster size <= 16 (MM3FA_DECODE_CS caps it) with n_units * cs <= the cluster kernel's resident
// CTAs whose clusters all fit at once (0, the stream-K split, only when no cluster fits).  The
// cluster instance's own occupancy counts (it needs fewer registers than the stream-K one).
// Cached per (device, kernel, units).
MmaPlan decode_mma_plan(int D, int kvt, int rows_per_pair, int64_t n_units, int n_sms) {
    const int nt  = rows_per_pair <= 8 ? 1 : 2;
    const int ns  = kvt == KV_Q8_0 ? Q8_NSTAGE : (mma_nstage_forced() == 2 ? 2 : 3);
    int       dev = 0;
    cudaGetDevice(&dev);
    static std::mutex                                                   mu;
    static std::map<std::tuple<int, int, int, int, int, int64_t>, MmaPlan> cache;
    std::lock_guard<std::mutex>                                         lock(mu);
    const auto key = std::make_tuple(dev, D, kvt, nt, n_sms, n_units);
    auto       it  = cache.find(key);
    if (it != cache.end()) {
        return it->second;
    }
    static const int cs_cap = [] {
        const char * e = std::getenv("MM3FA_DECODE_CS");
        const int    v = e ? std::atoi(e) : 0;
        return (v >= 1 && v <= MMA_MAX_CLUSTER) ? v : MMA_MAX_CLUSTER;
    }();
    int    smem = 0;
    void * fn   = select_mma_kernel(D, kvt, nt, true, smem, ns);
    if (!fn || n_units <= 0) {
        return MmaPlan{ 0, ns };
    }
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int per_sm = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fn, MMA_THREADS, smem) != cudaSuccess || per_sm < 1) {
        cudaGetLastError();
        per_sm = 1;
    }
    const int slots = n_sms * per_sm;
    // Clusters for any number of units: with few units a cluster of up to 16 CTAs per unit
    // measured 2.3-2.5x faster than the stream-K split over all SMs (36-layer graphs at 2-8
    // units: 10.4-11.6 against 26-27 us per layer), whose last-arriver merge of many partials
    // dominates; stream-K stays available through MM3FA_DECODE_SPLIT=streamk.
    int cs = (int) std::min<int64_t>(cs_cap, std::max<int64_t>(1, slots / n_units));
    while (cs > 1) {
        const int n = max_active_clusters(fn, cs, smem);
        if ((int64_t) n >= std::min<int64_t>(n_units, (int64_t) slots / cs)) {
            break;
        }
        cs--;
    }
    const MmaPlan plan{ cs, ns };
    cache[key] = plan;
    return plan;
}

cudaError_t launch_decode_mma(DecodeParams p, const DecodeGeometry & g, int D, int kvt, int64_t n_head_kv,
                              int64_t n_seq_k, MmaPlan plan, void * workspace, cudaStream_t stream) {
    const bool bf16    = kvt == KV_BF16;
    const int  nt      = p.rows_per_pair <= 8 ? 1 : 2;
    const int  cluster = plan.cluster;
    int        smem    = 0;
    const int  ns      = cluster > 0 ? plan.nstage : (mma_nstage_forced() == 2 ? 2 : 3);
    void *     fn      = select_mma_kernel(D, kvt, nt, cluster > 0, smem, ns);
    if (!fn) {
        return cudaErrorInvalidValue;
    }
    alignas(64) CUtensorMap tmk, tmv, tmm;
    std::memset(&tmm, 0, sizeof(tmm));
    // cluster mode stages its mask rows by TMA (stage starts are multiples of the chunk size)
    const int ck = (kvt == KV_Q8_0 && nt == 1) ? 2 * MMA_C : MMA_C;
    static const int mask_tma_env = [] {
        const char * e = std::getenv("MM3FA_DECODE_MASK_TMA");
        return e ? std::atoi(e) : 1;
    }();
    p.mask_tma = (mask_tma_env && cluster > 0 && p.mask && p.n_q == 1 && p.m_ne2 == 1 &&
                  encode_mask_tensor_map(&tmm, p, ck))
                     ? 1
                     : 0;

    if (kvt == KV_Q8_0) {
        // bulk copies of packed rows: every slab start and chunk must be 16-byte aligned
        const int64_t rb = (int64_t) D / QK8_0 * Q8_0_BLOCK;
        if (p.k_nb1 != rb || p.v_nb1 != rb || (rb * (p.n_kv % 16)) % 16 != 0 ||
            (reinterpret_cast<uintptr_t>(p.k) | reinterpret_cast<uintptr_t>(p.v)) % 16 != 0 ||
            (n_head_kv > 1 && (p.k_nb2 % 16 || p.v_nb2 % 16)) || (n_seq_k > 1 && (p.k_nb3 % 16 || p.v_nb3 % 16))) {
            return cudaErrorInvalidValue;
        }
        std::memset(&tmk, 0, sizeof(tmk));  // unused by the Q8_0 instances
        std::memset(&tmv, 0, sizeof(tmv));
    } else if (!encode_kv_tensor_map(&tmk, p.k, bf16, D, p.n_kv, n_head_kv, n_seq_k, p.k_nb1, p.k_nb2, p.k_nb3,
                                     MMA_C) ||
               !encode_kv_tensor_map(&tmv, p.v, bf16, D, p.n_kv, n_head_kv, n_seq_k, p.v_nb1, p.v_nb2, p.v_nb3,
                                     MMA_C)) {
        return cudaErrorInvalidValue;
    }
    char *       ws   = static_cast<char *>(workspace);
    const size_t cnt  = ((size_t) g.n_units * 4 + 255) / 256 * 256;
    const size_t slot = (size_t) g.n_units * g.max_slots * MMA_RMAX;
    p.status          = reinterpret_cast<uint32_t *>(ws);
    p.counters        = reinterpret_cast<uint32_t *>(ws + WS_STATUS_BYTES);
    p.part_ml         = reinterpret_cast<float *>(ws + WS_STATUS_BYTES + cnt);
    p.part_o          = reinterpret_cast<float *>(ws + WS_STATUS_BYTES + cnt + slot * 2 * 4);
    p.n_units         = g.n_units;
    p.keys_per_cta    = g.keys_per_cta;
    p.max_slots       = g.max_slots;
    p.rows_per_unit   = g.rows_per_unit;
    p.groups          = g.groups;
    p.cluster         = cluster;
    unsigned grid     = (unsigned) g.n_ctas;
    if (cluster > 0) {
        grid = (unsigned) (g.n_units * cluster);  // one unit per cluster, chunks interleaved over its CTAs
    }
    cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        return e;
    }
    if (cluster > 8) {
        e = cudaFuncSetAttribute(fn, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
        if (e != cudaSuccess) {
            return e;
        }
    }
    cudaLaunchConfig_t  cfg{};
    cudaLaunchAttribute attr[2];
    cfg.gridDim          = dim3(grid);
    cfg.blockDim         = dim3(MMA_THREADS);
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream           = stream;
    cfg.attrs            = attr;
    cfg.numAttrs         = 0;
    // programmatic dependent launch (default on, MM3FA_PDL=0 turns it off): the CTAs launch as
    // soon as the previous kernel's CTAs have exited and wait on the device for its completion,
    // which hides the launch gap (0.8 us per layer on the 36-layer decode graph)
    static const bool pdl = [] {
        const char * e = std::getenv("MM3FA_PDL");
        return !(e && std::atoi(e) == 0);
    }();
    if (pdl) {
        attr[cfg.numAttrs].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs++;
    }
    if (cluster > 0) {
        attr[cfg.numAttrs].id               = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = (unsigned) cluster;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs++;
    }
    void * args[] = { &tmk, &tmv, &tmm, &p };
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace mm3fa
