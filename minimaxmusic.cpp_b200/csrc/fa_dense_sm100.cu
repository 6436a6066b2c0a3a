// fa_dense_sm100.cu - flash attention for many query rows on the 5th-generation tensor cores
// (tcgen05 + TMEM + TMA), sm_100a.
//
// Serves GGML_OP_FLASH_ATTN_EXT when every (sequence, query head) has many query rows: the causal
// LM prefill of src/qwen3-lm.h:395-436 (Q [128, S, 32] F32 permuted view, K/V F16 views of the
// cache, F16 causal mask [n_kv_pad, S]) and the bidirectional DiT attention of src/dit.h:201-222
// (Q [64, S, 32, B], K/V F16 contiguous, no mask).
//
// One CTA per (256 query rows = two 128-row Q tiles, query head, sequence); both Q tiles share
// every K/V tile.  384 threads in three warpgroups with fixed roles:
//   warpgroup 0   warp 0 lane 0: TMA producer - 128-key tiles of K and V (boxes of 64 elements x
//                 128 keys, 128-byte swizzle, no multicast) into NS-deep rings.
//                 warp 1: allocates all 512 TMEM columns; lane 0 issues every tcgen05.mma:
//                   S_t (TMEM cols [128t, 128t+128), f32) = Q_t . K_j^T   A, B K-major in smem
//                   O_t (TMEM cols [256+Dt, ...), f32)  += P_t . V_j     A = P_t in TMEM (16-bit,
//                                                                        aliasing S_t), B = V
//                                                                        MN-major in smem
//                 in the order QK0(j), PV1(j-1), QK1(j), PV0(j): while softmax warpgroup 0 works on
//                 S_0(j) the tensor core runs PV1(j-1) and QK1(j), and the other way round.
//                 tcgen05 operations of one thread execute in issue order, so QK_t(j+1) may
//                 overwrite S_t / P_t right after PV_t(j) was issued.
//   warpgroups 1, 2  softmax of Q tile 0 / 1: thread r owns query row r of its tile (TMEM lane r),
//                 so a row's maximum and sum never leave the thread.  Per K/V tile: tcgen05.ld
//                 S, scale / softcap / mask (log2 units), online softmax with a lazily updated
//                 maximum (O is rescaled in TMEM only when the row maximum grows by more than 2^8;
//                 otherwise the stale maximum is kept, which is exact), P rounded to K's type and
//                 stored into TMEM with tcgen05.st.  S_t(j) being complete implies PV_t(j-1) is
//                 complete (issue order), so the rescale needs no extra wait.  At the end O / l
//                 is written to dst.
// Registers are rebalanced with setmaxnreg: the softmax warpgroups hold a 128-score row.
// Q is converted from F32 (any ggml strides) to K's type by the softmax threads while the first
// tiles load - ggml's convention of rounding Q to K's vec-dot type.
//
// Masks: a pre-pass classifies every 256 x 128 (query, key) block of each mask plane as all -inf
// (the K/V tile is skipped - causal prefill skips about half the work), all zero (no mask
// arithmetic) or mixed (mask added element by element).  Keys past n_kv are masked explicitly.
//
// Every wait is bounded by the global timer; on expiry the CTA records the status word, waits
// (bounded) for its copies and tensor-core work in flight, frees its TMEM and returns.  Waits of
// the softmax warps are made warp-uniform so the .sync.aligned TMEM accesses never diverge.
#include "fa_dense.cuh"
#include "fa_decode.cuh"

#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

namespace mm3fa {

constexpr int DN_THREADS = 384;  // 3 warpgroups
constexpr int DN_M       = 128;  // query rows per Q tile (UMMA M)
constexpr int DN_QT      = 2;    // Q tiles per CTA
constexpr int DN_ROWS    = DN_M * DN_QT;
constexpr int DN_N       = 128;  // keys per K/V tile (UMMA N of QK, K of PV)
constexpr int DN_TMEM    = 512;  // S0 [0,128), S1 [128,256), O0 [256,256+D), O1 [256+D, 256+2D)
constexpr int DN_REGS_LAUNCH  = 168;  // 65536 / 384, rounded down to a multiple of 8
constexpr int DN_REGS_SOFTMAX = 216;  // 2 x 128 x 216 + 128 x 72 = 384 x 168
constexpr int DN_REGS_OTHER   = 72;
constexpr int DN_EMU          = 3;    // of every 8 exp2 pairs, those computed by polynomial
static_assert(2 * 128 * DN_REGS_SOFTMAX + 128 * DN_REGS_OTHER <= DN_THREADS * DN_REGS_LAUNCH,
              "register split exceeds the launch allocation");

template <int D>
struct DenseSmem {
    static constexpr int HALVES   = D / 64;               // 128-byte column blocks of a D-wide row
    static constexpr int NS       = D == 128 ? 2 : 4;     // K and V ring depth
    static constexpr int QT       = HALVES * DN_M * 128;  // one Q tile
    static constexpr int KT       = HALVES * DN_N * 128;  // one K or V tile
    static constexpr int OFF_Q    = 0;                    // [DN_QT]
    static constexpr int OFF_K    = OFF_Q + DN_QT * QT;   // [NS]
    static constexpr int OFF_V    = OFF_K + NS * KT;      // [NS]
    static constexpr int OFF_BAR  = OFF_V + NS * KT;      // 32 mbarriers
    static constexpr int OFF_MISC = OFF_BAR + 32 * 8;     // tmem base, abort flag
    static constexpr int TOTAL    = OFF_MISC + 32 + 1024; // + alignment slack
};

// mbarrier slots (NS <= 4)
enum : int {
    B_KFULL   = 0,   // [NS]
    B_KEMPTY  = 4,   // [NS]
    B_VFULL   = 8,   // [NS]
    B_VEMPTY  = 12,  // [NS]
    B_SFULL   = 16,  // [2] S_t complete (tcgen05.commit)
    B_PREADY  = 18,  // [2] P_t in TMEM, O_t rescaled (128 softmax threads)
    B_ODONE   = 20,  // [2] last PV_t complete
    B_QREADY  = 22,  // [2] Q_t staged in smem (128 softmax threads)
    B_MMADONE = 24,
    B_COUNT   = 25,
};

// ------------------------------------------------------------------ PTX helpers

__device__ __forceinline__ void dn_tma_load_4d(void * dst, const CUtensorMap * tm, int c0, int c1, int c2, int c3,
                                               uint64_t * bar) {
    asm volatile(
        "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
        "[%6];" ::"r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(tm)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(bar))
        : "memory");
}

// 4-D tiled TMA store shared -> global (bulk group); rows outside the tensor are not written
__device__ __forceinline__ void dn_tma_store_4d(const CUtensorMap * tm, const void * src, int c0, int c1, int c2,
                                                int c3) {
    asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.tile.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(
                     reinterpret_cast<uint64_t>(tm)),
                 "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_addr(src))
                 : "memory");
}

// distributed shared memory of the other CTA of a 2-CTA cluster
__device__ __forceinline__ uint32_t dn_mapa(const void * local, uint32_t rank) {
    uint32_t r;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(smem_addr(local)), "r"(rank));
    return r;
}

__device__ __forceinline__ float2 dn_ld_dsmem2(uint32_t addr) {
    float2 v;
    asm volatile("ld.shared::cluster.v2.f32 {%0, %1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr) : "memory");
    return v;
}

__device__ __forceinline__ float4 dn_ld_dsmem4(uint32_t addr) {
    float4 v;
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(addr)
                 : "memory");
    return v;
}

// all threads of both CTAs of the cluster; orders shared-memory writes before the peer's reads
__device__ __forceinline__ void dn_cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void dn_named_barrier(int id, int nthreads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

__device__ __forceinline__ void dn_mbar_arrive(uint64_t * bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// warp-uniform bounded wait: true only if every lane saw the phase complete
__device__ __forceinline__ bool dn_wait_warp(uint64_t * bar, uint32_t parity, uint64_t deadline) {
    return __all_sync(0xffffffffu, mbar_wait_bounded(bar, parity, deadline));
}

__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t * dst, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(dst)),
                 "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// The tcgen05.mma / tcgen05.commit wrappers below are executed by a whole converged warp: the
// operands are computed by every lane (so they stay in the uniform datapath) and elect.sync picks
// the one lane that issues the instruction.

// D (TMEM) = A (smem desc) * B (smem desc) [+ D]
__device__ __forceinline__ void umma_f16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// arrive on `bar` once every tcgen05 operation this thread issued before has completed
__device__ __forceinline__ void umma_commit(uint64_t * bar) {
    asm volatile(
        "{\n\t.reg .pred e;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "@e tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];\n\t}" ::"r"(smem_addr(bar))
        : "memory");
}

// 32 consecutive 32-bit columns of this thread's TMEM lane (r[0..31] must stay in registers)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t * r) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
        "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr)
        : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t * r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
        "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(
            taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
        "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
        "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
        "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}

// tcgen05.wait::ld that also names the 32 registers a tcgen05.ld wrote: the compiler cannot move
// any use of them above the wait (the load writes them asynchronously)
__device__ __forceinline__ void tmem_ld_wait_tie(uint32_t * r) {
    asm volatile("tcgen05.wait::ld.sync.aligned;"
                 : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                   "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                   "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                   "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                   "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
                 :
                 : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2^x on the special-function unit (PTX ex2.approx, flushes denormal results to zero); 2^-inf = 0
__device__ __forceinline__ float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// Shared-memory matrix descriptor of a 128-byte-swizzled operand (sm_100 format, version 1).
// K-major: sbo = 1024 (8-row groups), lbo unused (16).  MN-major: lbo = stride between 64-element
// column blocks, sbo = 1024 (8-row groups along K).
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
    uint64_t d = 0;
    d |= (uint64_t) ((saddr >> 4) & 0x3FFFu);
    d |= (uint64_t) ((lbo >> 4) & 0x3FFFu) << 16;
    d |= (uint64_t) ((sbo >> 4) & 0x3FFFu) << 32;
    d |= (uint64_t) 1 << 46;  // descriptor version of sm_100
    d |= (uint64_t) 2 << 61;  // SWIZZLE_128B
    return d;
}

// Instruction descriptor of kind::f16, F32 accumulator, M = 128, dense.
__host__ __device__ constexpr uint32_t umma_idesc(bool bf16, int n, bool b_mn_major) {
    return (1u << 4)                              // D format: F32
           | ((bf16 ? 1u : 0u) << 7)              // A format: F16 / BF16
           | ((bf16 ? 1u : 0u) << 10)             // B format
           | ((b_mn_major ? 1u : 0u) << 16)       // B major (A is K-major: bit 15 = 0)
           | ((uint32_t) (n >> 3) << 17)          // N / 8
           | ((uint32_t) (DN_M >> 4) << 24);      // M / 16
}

// byte offset of (row, 16-byte chunk) in a 128-byte-swizzled tile of 128-byte rows
__device__ __forceinline__ uint32_t sw128_off(int row, int chunk) {
    return (uint32_t) (row * 128 + ((chunk ^ (row & 7)) << 4));
}

template <bool BF16>
__device__ __forceinline__ uint32_t pack2_dn(float lo, float hi) {
    if (BF16) {
        __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
        return *reinterpret_cast<uint32_t *>(&v);
    }
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
}

// 8 consecutive Q elements (F32/F16/BF16) of a row from element e0; vec: the row and e0 allow
// 16-byte loads
__device__ __forceinline__ void ld_q8(const char * row, int type, int e0, bool vec, float (&x)[8]) {
    if (vec) {
        if (type == KV_F32) {
            const float4 a = *reinterpret_cast<const float4 *>(row + (int64_t) e0 * 4);
            const float4 b = *reinterpret_cast<const float4 *>(row + (int64_t) e0 * 4 + 16);
            x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
            return;
        }
        const uint4    u    = *reinterpret_cast<const uint4 *>(row + (int64_t) e0 * 2);
        const uint32_t w[4] = { u.x, u.y, u.z, u.w };
#pragma unroll
        for (int j = 0; j < 4; j++) {
            const float2 f = type == KV_F16 ? h2_to_f2(w[j]) : bf2_to_f2(w[j]);
            x[2 * j]       = f.x;
            x[2 * j + 1]   = f.y;
        }
        return;
    }
#pragma unroll
    for (int j = 0; j < 8; j++) {
        x[j] = ld_q_elem(row, type, e0 + j);
    }
}

__device__ __forceinline__ int tile_class(const DenseParams & p, int plane, int qt, int kt) {
    if (!p.blocks) {
        return BLK_NONE;
    }
    const uint32_t f = p.blocks[((int64_t) plane * p.n_qt + qt) * p.n_kt + kt];
    return !(f & BLKF_FINITE) ? BLK_SKIP : (!(f & BLKF_NONZERO) ? BLK_NONE : BLK_MIXED);
}

// D (TMEM) = A (TMEM, 16-bit, row m = lane m) * B (smem desc) [+ D]; whole warp, one lane issues
__device__ __forceinline__ void umma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred e, p;\n\t"
        "elect.sync _|e, 0xffffffff;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "@e tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

template <int N>
__device__ __forceinline__ void regs_inc() {
    asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N));
}

template <int N>
__device__ __forceinline__ void regs_dec() {
    asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N));
}

// max of three (PTX max.f32 with three sources, sm_100)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
    float d;
    asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
    return d;
}

// Packed pairs of f32 (PTX .f32x2 arithmetic, sm_100): lo in the low 32 bits.
__device__ __forceinline__ uint64_t f2pack(float lo, float hi) {
    uint64_t r;
    asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
    return r;
}

__device__ __forceinline__ void f2unpack(uint64_t v, float & lo, float & hi) {
    asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}

__device__ __forceinline__ uint64_t ffma2(uint64_t a, uint64_t b, uint64_t c) {
    uint64_t d;
    asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(d) : "l"(a), "l"(b), "l"(c));
    return d;
}

__device__ __forceinline__ uint64_t fadd2(uint64_t a, uint64_t b) {
    uint64_t d;
    asm("add.rn.f32x2 %0, %1, %2;" : "=l"(d) : "l"(a), "l"(b));
    return d;
}

// 2^x for a pair, on the FMA pipe: x = n + f with n = round(x) (added to the exponent field) and
// f in [-1/2, 1/2]; 2^f by a degree-3 polynomial fitted here for minimum relative error on that
// interval (max 7.5e-5, below half an f16 ulp).  x is clamped to >= -126 so n never underflows the
// exponent; 2^-126 instead of 0 for x = -inf is far below what a 16-bit P can hold.
__device__ __forceinline__ uint64_t exp2_poly2(uint64_t x2) {
    constexpr float C0 = 0.99992806f, C1 = 0.69326097f, C2 = 0.24261114f, C3 = 0.05517167f;
    constexpr float MAGIC = 12582912.0f;  // 1.5 * 2^23: adding it rounds to an integer
    float xl, xh;
    f2unpack(x2, xl, xh);
    x2                = f2pack(fmaxf(xl, -126.0f), fmaxf(xh, -126.0f));
    const uint64_t r2 = fadd2(x2, f2pack(MAGIC, MAGIC));
    const uint64_t n2 = fadd2(r2, f2pack(-MAGIC, -MAGIC));
    const uint64_t f2 = ffma2(n2, f2pack(-1.0f, -1.0f), x2);
    uint64_t       p2 = ffma2(f2pack(C3, C3), f2, f2pack(C2, C2));
    p2                = ffma2(p2, f2, f2pack(C1, C1));
    p2                = ffma2(p2, f2, f2pack(C0, C0));
    float rl, rh, pl, ph;
    f2unpack(r2, rl, rh);
    f2unpack(p2, pl, ph);
    // the low bits of r hold n; shifted by 23 they land in the exponent field (the magic's own bits
    // shift out)
    return f2pack(__int_as_float(__float_as_int(pl) + (__float_as_int(rl) << 23)),
                  __int_as_float(__float_as_int(ph) + (__float_as_int(rh) << 23)));
}

// ------------------------------------------------------------------ kernel

template <int D, bool BF16>
__global__ void __launch_bounds__(DN_THREADS, 1)
    fa_dense_kernel(const __grid_constant__ CUtensorMap tmk, const __grid_constant__ CUtensorMap tmv,
                    const __grid_constant__ CUtensorMap tmo, const DenseParams p) {
    using L          = DenseSmem<D>;
    constexpr int NS = L::NS;
    constexpr int KS = D / 16;  // k-steps of QK
    extern __shared__ __align__(16) char smem_raw[];
    // 1024-byte aligned base, derived from smem_raw by pointer arithmetic (not through an
    // integer) so that the compiler keeps plain accesses in the shared address space
    char * smem = smem_raw + ((1024u - (smem_addr(smem_raw) & 1023u)) & 1023u);
    uint64_t * bar       = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    uint32_t * tmem_slot = reinterpret_cast<uint32_t *>(smem + L::OFF_MISC);
    int *      abort_f   = reinterpret_cast<int *>(smem + L::OFF_MISC + 4);

    const int tid   = threadIdx.x;
    const int warp  = tid >> 5;
    const int lane  = tid & 31;
    const int wg    = warp >> 2;
    // Work item = (256-row query block, head, sequence).  With a mask, query blocks run last-first:
    // under a causal mask the last blocks see the most keys, so the longest CTAs start in the
    // first wave.  CTAs
    // from n_regular on come in 2-CTA clusters that share one item, each taking half of its K/V
    // tiles (the last, partial wave of a launch, or all items of a small launch), and merge their
    // (O, m, l) through distributed shared memory.
    int item = (int) blockIdx.x, half = -1;
    if (item >= p.n_regular) {
        const int rel = item - p.n_regular;
        item          = p.n_regular + rel / 2;
        half          = rel % 2;  // the CTA's rank in its cluster
    }
    // without a mask every item has the same length: query blocks vary fastest, so the CTAs in
    // flight share few (head, sequence) K/V slabs and those stay in L2
    const int hunits = p.pair ? p.n_head / 2 : p.n_head;  // heads, or head pairs
    const int hs    = hunits * p.n_seq;
    const int cq    = p.mask ? p.n_qt - 1 - item / hs : item % p.n_qt;  // query block
    const int hsi   = p.mask ? item % hs : item / p.n_qt;
    const int h     = (hsi % hunits) * (p.pair ? 2 : 1);  // the item's (first) query head
    const int sq    = hsi / hunits;
    const int g     = h / p.ratio;
    const int ks3   = sq / p.rk3;
    const int plane = (sq % p.m_ne3) * p.m_ne2 + (h % p.m_ne2);

    if (tid == 0) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmk)) : "memory");
        asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&tmv)) : "memory");
        for (int i = 0; i < B_COUNT; i++) {
            // the softmax warpgroups' 128 threads arrive on these; one thread (or a commit) on the others
            const bool grp = (i >= B_PREADY && i < B_PREADY + 2) || (i >= B_QREADY && i < B_QREADY + 2);
            mbar_init(&bar[i], grp ? 128u : 1u);
        }
        *abort_f = 0;
        fence_mbar_init();
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, DN_TMEM);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem     = *tmem_slot;
    const uint64_t deadline = global_timer_ns() + p.timeout_ns;

    // the K/V tiles this query block needs, in order (blocks whose mask is all -inf are skipped)
    auto next_tile = [&](int kt) {
        while (kt < p.n_kt && tile_class(p, plane, cq, kt) == BLK_SKIP) {
            kt++;
        }
        return kt;
    };
    // this CTA's share of them: positions [pos_lo, pos_lo + n_mine) of the list.  The block
    // classes and row summaries come from the mask pre-pass, which lets this kernel launch while
    // it runs (masked calls are launched with programmatic stream serialisation; everything
    // before the pre-pass has completed when it starts): each role reads them only after
    // griddepcontrol.wait, and the softmax warpgroups stage Q before that.
    int  n_mine = 0, kt_lo = 0;
    auto tile_share = [&]() {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        int n_all = 0;
        for (int kt = next_tile(0); kt < p.n_kt; kt = next_tile(kt + 1)) {
            n_all++;
        }
        const int pos_lo = half == 1 ? (n_all + 1) / 2 : 0;
        n_mine           = half == 0 ? (n_all + 1) / 2 : n_all - pos_lo;
        kt_lo            = next_tile(0);
        for (int k = 0; k < pos_lo; k++) {
            kt_lo = next_tile(kt_lo + 1);
        }
    };

    if (wg == 0) {
        regs_dec<DN_REGS_OTHER>();
        tile_share();
        if (warp == 0 && lane == 0) {
            // ======================================================= TMA producer
            int  nk_ld = 0, nv_ld = 0;  // K and V tile loads issued (stage = load index % NS)
            int  i     = 0;
            bool ok    = true;
            for (int kt = kt_lo; i < n_mine; kt = next_tile(kt + 1), i++) {
                const int      st  = i % NS;
                const uint32_t par = (uint32_t) ((i / NS - 1) & 1);
                if (i >= NS && !mbar_wait_bounded(&bar[B_KEMPTY + st], par, deadline)) {
                    ok = false;
                    break;
                }
                char * dk = smem + L::OFF_K + st * L::KT;
                mbar_arrive_expect_tx(&bar[B_KFULL + st], (uint32_t) L::KT);
#pragma unroll
                for (int hh = 0; hh < L::HALVES; hh++) {
                    dn_tma_load_4d(dk + hh * DN_N * 128, &tmk, hh * 64, kt * DN_N, g, ks3, &bar[B_KFULL + st]);
                }
                nk_ld++;
                if (i >= NS && !mbar_wait_bounded(&bar[B_VEMPTY + st], par, deadline)) {
                    ok = false;
                    break;
                }
                char * dv = smem + L::OFF_V + st * L::KT;
                mbar_arrive_expect_tx(&bar[B_VFULL + st], (uint32_t) L::KT);
#pragma unroll
                for (int hh = 0; hh < L::HALVES; hh++) {
                    dn_tma_load_4d(dv + hh * DN_N * 128, &tmv, hh * 64, kt * DN_N, g, ks3, &bar[B_VFULL + st]);
                }
                nv_ld++;
            }
            if (!ok) {
                atomicExch(abort_f, 1);
            }
            // a load into a stage is issued only after the previous one landed and was consumed, so
            // the last load of each stage is the only one that can still be in flight
            const uint64_t drain = global_timer_ns() + p.timeout_ns;
#pragma unroll
            for (int st = 0; st < NS; st++) {
                const int kc = (nk_ld - st + NS - 1) / NS, vc = (nv_ld - st + NS - 1) / NS;  // loads into st
                if (kc > 0) {
                    mbar_wait_bounded(&bar[B_KFULL + st], (uint32_t) ((kc - 1) & 1), drain);
                }
                if (vc > 0) {
                    mbar_wait_bounded(&bar[B_VFULL + st], (uint32_t) ((vc - 1) & 1), drain);
                }
            }
        } else if (warp == 1) {
            // ======================================================= MMA issuer (whole warp, elected lane)
            const uint32_t id_qk = umma_idesc(BF16, DN_N, false);
            const uint32_t id_pv = umma_idesc(BF16, D, true);
            const uint32_t q_a   = smem_addr(smem + L::OFF_Q);
            auto qk = [&](int t, int i) {  // S_t = Q_t . K_i^T
                const uint32_t sk = smem_addr(smem + L::OFF_K + (i % NS) * L::KT);
                const uint32_t sq_a = q_a + (uint32_t) (t * L::QT);
#pragma unroll
                for (int ks = 0; ks < KS; ks++) {
                    const uint32_t off = (uint32_t) ((ks >> 2) * DN_M * 128 + (ks & 3) * 32);
                    umma_f16(tmem + (uint32_t) (t * DN_N), sw128_desc(sq_a + off, 16, 1024),
                             sw128_desc(sk + off, 16, 1024), id_qk, ks > 0 ? 1u : 0u);
                }
            };
            auto pv = [&](int t, int i) {  // O_t += P_t . V_i
                const uint32_t sv = smem_addr(smem + L::OFF_V + (i % NS) * L::KT);
#pragma unroll
                for (int kk = 0; kk < DN_N / 16; kk++) {
                    umma_f16_ts(tmem + 256u + (uint32_t) (t * D), tmem + (uint32_t) (t * DN_N + kk * 8),
                                sw128_desc(sv + (uint32_t) (kk * 16 * 128), (uint32_t) (DN_N * 128), 1024), id_pv,
                                (i > 0 || kk > 0) ? 1u : 0u);
                }
            };
            auto wait = [&](int b, int i) { return dn_wait_warp(&bar[b], (uint32_t) (i & 1), deadline); };
            const int n = n_mine;
            bool ok = wait(B_QREADY, 0) && wait(B_QREADY + 1, 0);
            tc_fence_after();
            if (ok && n > 0) {
                // prologue: S0(0), S1(0), O0 += P0(0) V0
                ok = wait(B_KFULL + 0, 0);
                if (ok) {
                    tc_fence_after();
                    qk(0, 0);
                    umma_commit(&bar[B_SFULL + 0]);
                    qk(1, 0);
                    umma_commit(&bar[B_SFULL + 1]);
                    umma_commit(&bar[B_KEMPTY + 0]);
                    ok = wait(B_VFULL + 0, 0) && wait(B_PREADY + 0, 0);
                }
                if (ok) {
                    tc_fence_after();
                    pv(0, 0);
                }
                for (int i = 1; ok && i < n; i++) {
                    const int st = i % NS;
                    ok           = wait(B_KFULL + st, i / NS);
                    if (!ok) {
                        break;
                    }
                    tc_fence_after();
                    qk(0, i);  // S0/P0 are free: PV0(i-1) was issued before
                    umma_commit(&bar[B_SFULL + 0]);
                    ok = wait(B_PREADY + 1, i - 1);
                    if (!ok) {
                        break;
                    }
                    tc_fence_after();
                    pv(1, i - 1);
                    umma_commit(&bar[B_VEMPTY + (i - 1) % NS]);
                    qk(1, i);
                    umma_commit(&bar[B_SFULL + 1]);
                    umma_commit(&bar[B_KEMPTY + st]);
                    ok = wait(B_VFULL + st, i / NS) && wait(B_PREADY + 0, i);
                    if (!ok) {
                        break;
                    }
                    tc_fence_after();
                    pv(0, i);
                }
                if (ok) {
                    umma_commit(&bar[B_ODONE + 0]);
                    ok = wait(B_PREADY + 1, n - 1);
                }
                if (ok) {
                    tc_fence_after();
                    pv(1, n - 1);
                    umma_commit(&bar[B_VEMPTY + (n - 1) % NS]);
                    umma_commit(&bar[B_ODONE + 1]);
                }
            }
            if (!ok) {
                atomicExch(abort_f, 1);
            }
            // every MMA issued must have completed before TMEM and shared memory are released
            umma_commit(&bar[B_MMADONE]);
            dn_wait_warp(&bar[B_MMADONE], 0, global_timer_ns() + p.timeout_ns);
        }
        if (half >= 0) {  // the two cluster barriers of the split epilogue
            dn_cluster_sync();
            dn_cluster_sync();
        }
    } else {
        regs_inc<DN_REGS_SOFTMAX>();
        // ======================================================= softmax warpgroups 1, 2
        const int      t     = wg - 1;            // Q tile
        const int      ht    = p.pair ? h + t : h;                              // its query head
        const int      rbase = p.pair ? cq * DN_M : cq * DN_ROWS + t * DN_M;   // its first query row
        const int      quad  = warp & 3;          // TMEM lane quadrant this warp may access
        const int      r     = quad * 32 + lane;  // row in the tile (= TMEM lane)
        const uint32_t tl    = (uint32_t) (quad * 32) << 16;
        const uint32_t s_col = tmem + tl + (uint32_t) (t * DN_N);
        const uint32_t o_col = tmem + tl + 256u + (uint32_t) (t * D);
        const int      row   = rbase + r;
        const bool     valid = row < p.n_q;
        const int      qi    = valid ? row : 0;
        const float    slope = alibi_slope(ht, p.max_bias, p.n_head_log2, p.m0, p.m1);
        // ---- stage Q row r into the swizzled K-major tile t, rounded to K's type
        {
            const char * qrow = p.q + (int64_t) qi * p.q_nb1 + (int64_t) ht * p.q_nb2 + (int64_t) sq * p.q_nb3;
            char *       qs   = smem + L::OFF_Q + t * L::QT;
            if (p.q_type == KV_F32 && p.q_vec) {
                // coalesced: the lanes of a warp load whole rows (LPR lanes x 16 bytes per row) of this
                // warp's 32 rows, all loads in flight, then each lane writes its 4 rounded values
                // (8 bytes) into the row's swizzled 16-byte chunk
                constexpr int LPR = D / 4;       // lanes per row
                constexpr int RPI = 32 / LPR;    // rows per load instruction
                constexpr int NLD = 32 / RPI;    // loads per lane
                float4 x[NLD];
#pragma unroll
                for (int it = 0; it < NLD; it++) {
                    const int rr  = quad * 32 + it * RPI + lane / LPR;  // row in the tile
                    const int row = rbase + rr;
                    x[it]         = make_float4(0.f, 0.f, 0.f, 0.f);
                    if (row < p.n_q) {
                        x[it] = reinterpret_cast<const float4 *>(p.q + (int64_t) row * p.q_nb1 + (int64_t) ht * p.q_nb2 +
                                                                 (int64_t) sq * p.q_nb3)[lane % LPR];
                    }
                }
                const int e  = (lane % LPR) * 4;  // first element of this lane
                const int hb = e / 64, ch = (e % 64) / 8, sub = (e % 8) * 2;
#pragma unroll
                for (int it = 0; it < NLD; it++) {
                    const int rr = quad * 32 + it * RPI + lane / LPR;
                    uint2     v;
                    v.x = pack2_dn<BF16>(x[it].x, x[it].y);
                    v.y = pack2_dn<BF16>(x[it].z, x[it].w);
                    *reinterpret_cast<uint2 *>(qs + hb * (DN_M * 128) + sw128_off(rr, ch) + sub) = v;
                }
            } else {
#pragma unroll 4
                for (int c = 0; c < D / 8; c++) {
                    float x[8];
                    if (valid) {
                        ld_q8(qrow, p.q_type, c * 8, p.q_vec != 0, x);
                    } else {
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            x[e] = 0.0f;
                        }
                    }
                    uint4 v;
                    v.x = pack2_dn<BF16>(x[0], x[1]);
                    v.y = pack2_dn<BF16>(x[2], x[3]);
                    v.z = pack2_dn<BF16>(x[4], x[5]);
                    v.w = pack2_dn<BF16>(x[6], x[7]);
                    *reinterpret_cast<uint4 *>(qs + (c >> 3) * (DN_M * 128) + sw128_off(r, c & 7)) = v;
                }
            }
            fence_proxy_async_smem();  // generic-proxy stores -> visible to the tensor core
            dn_mbar_arrive(&bar[B_QREADY + t]);
        }
        tile_share();
        // step rows (the mask is 0 before column lim and -inf from it on, as in causal masks):
        // their mixed tiles take the fast path with a column bound instead of mask values
        int lim = p.n_kv, ri0 = 0, ri1 = 0, ri2 = 0;
        if (p.rowinfo && valid) {
            const int * ri = p.rowinfo + ((int64_t) plane * p.n_q + qi) * 3;
            ri0            = ri[0];
            ri1            = ri[1];
            ri2            = ri[2];
        }

        const __half * mrow = p.mask ? reinterpret_cast<const __half *>(
                                           p.mask + (int64_t) qi * p.m_nb1 + (int64_t) (ht % p.m_ne2) * p.m_nb2 +
                                           (int64_t) (sq % p.m_ne3) * p.m_nb3)
                                     : nullptr;
        const float sc    = p.softcap != 0.0f ? p.scale / p.softcap : p.scale;
        const float sl2   = sc * LOG2E;     // raw score -> log2 units (no softcap)
        const float ml2   = slope * LOG2E;  // mask -> log2 units
        const bool  plain = p.softcap == 0.0f && sl2 > 0.0f;
        const bool  is_step   = ri2 == 0 && ri0 + ri1 <= p.n_kv;
        const bool  step_warp = p.rowinfo != nullptr && __all_sync(0xffffffffu, is_step);
        lim                   = p.n_kv - ri0;
        float       m     = -INFINITY;      // running maximum (log2 units; may be stale by < 8)
        float       l     = 0.0f;
        bool        ok    = true;
        int         i     = 0;
        for (int kt = kt_lo; i < n_mine; kt = next_tile(kt + 1), i++) {
            const int  nk    = p.n_kv - kt * DN_N;  // keys of this tile that exist (may exceed DN_N)
            const int  cls   = tile_class(p, plane, cq, kt);
            // warp-uniform: every row of the warp is a step row, so the tile needs only a bound
            const bool use_lim = plain && step_warp && (cls == BLK_MIXED || nk < DN_N);
            const bool fast    = use_lim || (plain && nk >= DN_N && cls != BLK_MIXED);
            const bool mixed   = valid && cls == BLK_MIXED && !use_lim;
            const int  lt      = lim - kt * DN_N;  // columns of this tile the row sees (step rows)
            // this row's mask values of the tile: pulled into L1 before S is ready, so the loads of
            // the pass below hit
            const __half * mp = mixed ? mrow + (int64_t) kt * DN_N : nullptr;
            if (mixed) {
#pragma unroll
                for (int c = 0; c < DN_N * 2; c += 128) {
                    asm volatile("prefetch.global.L1 [%0];" ::"l"(reinterpret_cast<const char *>(mp) + c));
                }
            }
            if (!dn_wait_warp(&bar[B_SFULL + t], (uint32_t) (i & 1), deadline)) {
                ok = false;
                break;
            }
            tc_fence_after();
            if (!fast) {
                // general tile: rewrite S in TMEM in log2 units - softcap, mask, keys past n_kv -
                // 32 columns at a time, so the row pass below treats every tile alike
#pragma unroll 1
                for (int c = 0; c < DN_N / 32; c++) {
                    uint32_t v[32];
                    tmem_ld32(s_col + (uint32_t) (c * 32), v);
                    float mv[32];
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        mv[e] = 0.0f;
                    }
                    if (mixed) {
                        if (p.mask_vec && c * 32 + 32 <= nk) {
#pragma unroll
                            for (int q4 = 0; q4 < 4; q4++) {
                                const uint4    u    = *reinterpret_cast<const uint4 *>(mp + c * 32 + q4 * 8);
                                const uint32_t w[4] = { u.x, u.y, u.z, u.w };
#pragma unroll
                                for (int j = 0; j < 4; j++) {
                                    const float2 f      = h2_to_f2(w[j]);
                                    mv[q4 * 8 + 2 * j]     = f.x;
                                    mv[q4 * 8 + 2 * j + 1] = f.y;
                                }
                            }
                        } else {
#pragma unroll
                            for (int e = 0; e < 32; e++) {
                                mv[e] = c * 32 + e < nk ? __half2float(mp[c * 32 + e]) : 0.0f;
                            }
                        }
                    }
                    tmem_ld_wait_tie(v);
                    // the softcap branch stays outside the element loops (tanhf must not be if-converted)
                    if (p.softcap != 0.0f) {
                        const float cl2 = p.softcap * LOG2E;
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            v[e] = __float_as_uint(cl2 * tanhf(__uint_as_float(v[e]) * sc));
                        }
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            v[e] = __float_as_uint(__uint_as_float(v[e]) * sl2);
                        }
                    }
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        const float y = fmaf(ml2, mv[e], __uint_as_float(v[e]));
                        v[e]          = __float_as_uint(c * 32 + e < nk ? y : -INFINITY);
                    }
                    tmem_st32(s_col + (uint32_t) (c * 32), v);
                }
                tmem_st_wait();
            }
            // scores are raw (fast tiles, times sl2 > 0 gives log2 units) or already in log2 units
            const float    mult = fast ? sl2 : 1.0f;
            const uint64_t mul2 = f2pack(mult, mult);
            uint32_t       sr[DN_N];
            uint32_t       pk[DN_N / 2];
            uint64_t       acc[4];
            // p = 2^(s * mult - m) for pairs [j0, j1): packed f32x2 arithmetic; DN_EMU of every 8 pairs
            // take the FMA-pipe polynomial, the others the special-function unit
            auto exp_pairs = [&](int j0, int j1) {
                const uint64_t nm2 = f2pack(-m, -m);
#pragma unroll
                for (int j = 0; j < DN_N / 2; j++) {
                    if (j < j0 || j >= j1) {
                        continue;
                    }
                    const uint64_t x2 = ffma2(f2pack(__uint_as_float(sr[2 * j]), __uint_as_float(sr[2 * j + 1])), mul2, nm2);
                    uint64_t       p2;
                    if ((j & 7) < DN_EMU) {
                        p2 = exp2_poly2(x2);
                    } else {
                        float xl, xh;
                        f2unpack(x2, xl, xh);
                        p2 = f2pack(ex2(xl), ex2(xh));
                    }
                    acc[j & 3] = fadd2(acc[j & 3], p2);
                    float pl, ph;
                    f2unpack(p2, pl, ph);
                    pk[j] = pack2_dn<BF16>(pl, ph);
                }
            };
            auto acc_sum = [&]() {
                float s0, s1, s2, s3;
                f2unpack(fadd2(acc[0], acc[1]), s0, s1);
                f2unpack(fadd2(acc[2], acc[3]), s2, s3);
                return (s0 + s1) + (s2 + s3);
            };
            // step rows: columns from lt on are -inf (raw score bits, before the scale)
            auto apply_lim = [&](int j0, int j1) {
                if (use_lim) {
#pragma unroll
                    for (int j = 0; j < DN_N; j++) {
                        if (j >= j0 && j < j1) {
                            sr[j] = j < lt ? sr[j] : 0xFF800000u;
                        }
                    }
                }
            };
            auto load_all = [&]() {
#pragma unroll
                for (int c = 0; c < DN_N / 32; c++) {
                    tmem_ld32(s_col + (uint32_t) (c * 32), &sr[c * 32]);
                }
#pragma unroll
                for (int c = 0; c < DN_N / 32; c++) {
                    tmem_ld_wait_tie(&sr[c * 32]);
                }
            };
            float alpha = 1.0f, lsum = 0.0f;
            // The row maximum is needed while it is unknown (first tile of a row) or when the stale
            // maximum would let a p overflow 16 bits.  A tile sum <= 2^15 bounds every p below the
            // f16 limit, so the exp pass runs first with the stale maximum and the exact maximum is
            // computed (and the pass redone) only when some row's sum exceeds that.
            bool full = __any_sync(0xffffffffu, m == -INFINITY);
            if (!full) {
                // first half of the row in registers, second half loading while the first is used
                tmem_ld32(s_col + 0, &sr[0]);
                tmem_ld32(s_col + 32, &sr[32]);
                tmem_ld_wait_tie(&sr[0]);
                tmem_ld_wait_tie(&sr[32]);
                tmem_ld32(s_col + 64, &sr[64]);
                tmem_ld32(s_col + 96, &sr[96]);
                apply_lim(0, DN_N / 2);
                acc[0] = acc[1] = acc[2] = acc[3] = 0ull;
                exp_pairs(0, DN_N / 4);
                tmem_ld_wait_tie(&sr[64]);
                tmem_ld_wait_tie(&sr[96]);
                apply_lim(DN_N / 2, DN_N);
                exp_pairs(DN_N / 4, DN_N / 2);
                lsum = acc_sum();
                full = __any_sync(0xffffffffu, !(lsum <= 32768.0f));  // NaN included
            }
            if (full) {
                load_all();
                apply_lim(0, DN_N);
                float a0 = __uint_as_float(sr[0]), a1 = __uint_as_float(sr[1]), a2 = __uint_as_float(sr[2]),
                      a3 = __uint_as_float(sr[3]);
#pragma unroll
                for (int k = 4; k < DN_N - 4; k += 8) {
                    a0 = fmax3(a0, __uint_as_float(sr[k]), __uint_as_float(sr[k + 1]));
                    a1 = fmax3(a1, __uint_as_float(sr[k + 2]), __uint_as_float(sr[k + 3]));
                    a2 = fmax3(a2, __uint_as_float(sr[k + 4]), __uint_as_float(sr[k + 5]));
                    a3 = fmax3(a3, __uint_as_float(sr[k + 6]), __uint_as_float(sr[k + 7]));
                }
                a0 = fmax3(a0, __uint_as_float(sr[DN_N - 4]), __uint_as_float(sr[DN_N - 3]));
                a1 = fmax3(a1, __uint_as_float(sr[DN_N - 2]), __uint_as_float(sr[DN_N - 1]));
                const float mt = fmax3(a0, a1, fmaxf(a2, a3)) * mult;
                // lazy maximum: rescale only when the row maximum grows by more than 8 (a factor 2^8)
                if (mt > m + 8.0f) {
                    alpha = (m == -INFINITY) ? 0.0f : ex2(m - mt);
                    m     = mt;
                }
                if (m == -INFINITY) {
#pragma unroll
                    for (int k = 0; k < DN_N / 2; k++) {
                        pk[k] = 0u;
                    }
                    lsum = 0.0f;
                } else {
                    acc[0] = acc[1] = acc[2] = acc[3] = 0ull;
                    exp_pairs(0, DN_N / 2);
                    lsum = acc_sum();
                }
            }
            l = l * alpha + lsum;

            // P (16-bit, 2 per column) into the first 64 columns of S_t
            tmem_st32(s_col + 0, &pk[0]);
            tmem_st32(s_col + 32, &pk[32]);
            // O_t rescale: PV_t(i-1) is complete because QK_t(i) was issued after it
            if (i > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
#pragma unroll 1
                for (int c = 0; c < D / 32; c++) {
                    uint32_t o[32];
                    tmem_ld32(o_col + (uint32_t) (c * 32), o);
                    tmem_ld_wait_tie(o);
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
                    }
                    tmem_st32(o_col + (uint32_t) (c * 32), o);
                }
            }
            tmem_st_wait();
            tc_fence_before();
            dn_mbar_arrive(&bar[B_PREADY + t]);
        }
        if (!ok) {
            atomicExch(abort_f, 1);
        }

        // ---- epilogue: O / l -> dst row (rows without any key, or after an abort, are zero)
        bool have_o = ok && i > 0;
        if (have_o) {
            have_o = dn_wait_warp(&bar[B_ODONE + t], 0, deadline);
            if (!have_o) {
                atomicExch(abort_f, 1);
            }
            tc_fence_after();
        }
        const float inv = (have_o && l > 0.0f) ? 1.0f / l : 0.0f;
        if (half >= 0) {
            // split item: rank 1 publishes its raw O rows and (m, l) in its (now free) ring and Q
            // space; rank 0 combines them with its own and stores the result
            if (!dn_wait_warp(&bar[B_MMADONE], 0, deadline)) {
                atomicExch(abort_f, 1);
            }
            float2 * mls   = reinterpret_cast<float2 *>(smem + L::OFF_Q);  // [tile][row] (m, l)
            char *   stage = smem + L::OFF_K + t * (D / 32) * (DN_M * 128);
            if (half == 1) {
#pragma unroll
                for (int c = 0; c < D / 32; c++) {
                    uint32_t o[32];
                    if (have_o) {
                        tmem_ld32(o_col + (uint32_t) (c * 32), o);
                        tmem_ld_wait_tie(o);
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            o[e] = 0u;
                        }
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        *reinterpret_cast<uint4 *>(stage + c * (DN_M * 128) + sw128_off(r, j)) =
                            make_uint4(o[4 * j], o[4 * j + 1], o[4 * j + 2], o[4 * j + 3]);
                    }
                }
                mls[t * DN_M + r] = have_o ? make_float2(m, l) : make_float2(-INFINITY, 0.0f);
            }
            dn_cluster_sync();
            if (half == 0) {
                const float2 mb = dn_ld_dsmem2(dn_mapa(&mls[t * DN_M + r], 1));
                const float  ma = have_o ? m : -INFINITY, la = have_o ? l : 0.0f;
                const float  M  = fmaxf(ma, mb.x);
                const float  wa = ma == -INFINITY ? 0.0f : ex2(ma - M);
                const float  wb = mb.x == -INFINITY ? 0.0f : ex2(mb.x - M);
                const float  Ls = wa * la + wb * mb.y;
                const float  iv = Ls > 0.0f ? 1.0f / Ls : 0.0f;
                const float  ca = wa * iv, cb = wb * iv;
#pragma unroll
                for (int c = 0; c < D / 32; c++) {
                    uint32_t o[32];
                    if (have_o) {
                        tmem_ld32(o_col + (uint32_t) (c * 32), o);
                        tmem_ld_wait_tie(o);
                    } else {
#pragma unroll
                        for (int e = 0; e < 32; e++) {
                            o[e] = 0u;
                        }
                    }
                    char * tile = stage + c * (DN_M * 128);
                    float4 ob[8];
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        ob[j] = dn_ld_dsmem4(dn_mapa(tile + sw128_off(r, j), 1));
                    }
#pragma unroll
                    for (int j = 0; j < 8; j++) {
                        *reinterpret_cast<float4 *>(tile + sw128_off(r, j)) =
                            make_float4(ca * __uint_as_float(o[4 * j]) + cb * ob[j].x,
                                        ca * __uint_as_float(o[4 * j + 1]) + cb * ob[j].y,
                                        ca * __uint_as_float(o[4 * j + 2]) + cb * ob[j].z,
                                        ca * __uint_as_float(o[4 * j + 3]) + cb * ob[j].w);
                    }
                }
                if (p.tma_store) {
                    fence_proxy_async_smem();
                    dn_named_barrier(1 + t, 128);
                    if (quad == 0 && lane == 0) {
                        const int q0t = rbase;
#pragma unroll
                        for (int c = 0; c < D / 32; c++) {
                            dn_tma_store_4d(&tmo, stage + c * (DN_M * 128), c * 32, ht, q0t, sq);
                        }
                        asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
                    }
                } else if (valid) {
                    float * out = reinterpret_cast<float *>(p.dst + (int64_t) ht * p.d_nb1 + (int64_t) qi * p.d_nb2 +
                                                            (int64_t) sq * p.d_nb3);
#pragma unroll
                    for (int c = 0; c < D / 32; c++) {
#pragma unroll
                        for (int j = 0; j < 8; j++) {
                            const float4 v = *reinterpret_cast<const float4 *>(stage + c * (DN_M * 128) + sw128_off(r, j));
                            out[c * 32 + 4 * j]     = v.x;
                            out[c * 32 + 4 * j + 1] = v.y;
                            out[c * 32 + 4 * j + 2] = v.z;
                            out[c * 32 + 4 * j + 3] = v.w;
                        }
                    }
                }
            }
            dn_cluster_sync();  // rank 1's shared memory stays alive until rank 0 has read it
        } else if (p.tma_store) {
            // every MMA is done once MMADONE completes, so the K/V ring is free: each thread writes its
            // scaled O row into 128-byte-swizzled [128 rows][32 floats] tiles there, and one thread
            // of the warpgroup stores them with TMA (rows past n_q are clipped by the tensor map)
            if (!dn_wait_warp(&bar[B_MMADONE], 0, deadline)) {
                atomicExch(abort_f, 1);
            }
            char * stage = smem + L::OFF_K + t * (D / 32) * (DN_M * 128);
#pragma unroll
            for (int c = 0; c < D / 32; c++) {
                uint32_t o[32];
                if (have_o) {
                    tmem_ld32(o_col + (uint32_t) (c * 32), o);
                    tmem_ld_wait_tie(o);
                } else {
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        o[e] = 0u;
                    }
                }
                char * tile = stage + c * (DN_M * 128);
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    *reinterpret_cast<float4 *>(tile + sw128_off(r, j)) =
                        make_float4(__uint_as_float(o[4 * j]) * inv, __uint_as_float(o[4 * j + 1]) * inv,
                                    __uint_as_float(o[4 * j + 2]) * inv, __uint_as_float(o[4 * j + 3]) * inv);
                }
            }
            fence_proxy_async_smem();
            dn_named_barrier(1 + t, 128);
            if (p.n_peers > 0) {
                // fused exchange: the staged rows to the other ranks' results (the same place there,
                // at peer_off), a warp per 32 rows, each store instruction covering whole rows
                // (D / 4 lanes x 16 contiguous bytes per row), so that NVLink carries full lines
                constexpr int F4  = D / 4;    // 16-byte pieces of a row
                constexpr int RPW = 32 / F4;  // rows per warp instruction
                const int     c   = (lane % F4) / 8;
                const int     jj  = (lane % F4) % 8;
                for (int i = lane / F4; i < 32; i += RPW) {
                    const int rr = quad * 32 + i;
                    const int rw = rbase + rr;
                    if (rw < p.n_q) {
                        const float4 val = *reinterpret_cast<const float4 *>(stage + c * (DN_M * 128) + sw128_off(rr, jj));
                        char * prow = p.dst + (int64_t) ht * p.d_nb1 + (int64_t) rw * p.d_nb2 + (int64_t) sq * p.d_nb3 +
                                      c * 128 + jj * 16;
#pragma unroll
                        for (int pp = 0; pp < 7; pp++) {
                            if (pp < p.n_peers) {
                                *reinterpret_cast<float4 *>(prow + p.peer_off[pp]) = val;
                            }
                        }
                    }
                }
            }
            if (quad == 0 && lane == 0) {
                const int q0t = rbase;
#pragma unroll
                for (int c = 0; c < D / 32; c++) {
                    dn_tma_store_4d(&tmo, stage + c * (DN_M * 128), c * 32, ht, q0t, sq);
                }
                asm volatile("cp.async.bulk.commit_group;" ::: "memory");
                asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
            }
        } else {
        float * out =
            reinterpret_cast<float *>(p.dst + (int64_t) ht * p.d_nb1 + (int64_t) qi * p.d_nb2 + (int64_t) sq * p.d_nb3);
#pragma unroll
        for (int c = 0; c < D / 32; c++) {
            uint32_t o[32];
            if (have_o) {
                tmem_ld32(o_col + (uint32_t) (c * 32), o);
                tmem_ld_wait_tie(o);
            } else {
#pragma unroll
                for (int e = 0; e < 32; e++) {
                    o[e] = 0u;
                }
            }
            if (valid) {
                if (p.dst_vec) {
#pragma unroll
                    for (int e = 0; e < 32; e += 4) {
                        *reinterpret_cast<float4 *>(out + c * 32 + e) =
                            make_float4(__uint_as_float(o[e]) * inv, __uint_as_float(o[e + 1]) * inv,
                                        __uint_as_float(o[e + 2]) * inv, __uint_as_float(o[e + 3]) * inv);
                    }
                } else {
#pragma unroll
                    for (int e = 0; e < 32; e++) {
                        out[c * 32 + e] = __uint_as_float(o[e]) * inv;
                    }
                }
            }
        }
        }
    }

    // ---- teardown: all TMEM traffic is complete before the columns are released
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem, DN_TMEM);
    }
    if (tid == 0 && *abort_f) {
        atomicOr(&p.status[0], ST_TIMEOUT);
        atomicExch(&p.status[1], (uint32_t) (blockIdx.x | (blockIdx.y << 16)));
    }
}

// ------------------------------------------------------------------ mask block classes

// One CTA per (kv tile, 32 query rows, mask plane), 512 threads = 16 lanes per row: the flags of
// the 256 x 128 block the rows belong to (BLKF_FINITE: some entry is not -inf, BLKF_NONZERO: some
// entry is not zero; OR-ed into the block's word, zeroed before the launch) and, per row, the
// summary that identifies step rows (zeros, then -inf).  Only rows < n_q and columns < n_kv are
// examined.  With 16-byte aligned rows a lane tests 8 halves directly (-inf = 0xFC00, zero = +-0).
constexpr int MASK_CLASS_THREADS = 512;
constexpr int MASK_ROWS          = MASK_CLASS_THREADS / (DN_N / 8);  // 32

__global__ void __launch_bounds__(MASK_CLASS_THREADS)
    mask_block_class_kernel(const char * mask, int64_t nb1, int64_t nb2, int64_t nb3, int m_ne2, int n_q, int n_kv,
                            int n_qt, int n_kt, int qrows, int vec, uint32_t * bflags, int * rowinfo) {
    // the attention kernel may launch at once: it reads nothing this kernel writes before its
    // griddepcontrol.wait
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const int    kt = blockIdx.x, plane = blockIdx.z;
    const int    i2 = plane % m_ne2, i3 = plane / m_ne2;
    const int    r0 = blockIdx.y * MASK_ROWS, c0 = kt * DN_N;
    const int    nr = min(MASK_ROWS, n_q - r0), nc = min(DN_N, n_kv - c0);
    const char * base = mask + (int64_t) r0 * nb1 + (int64_t) i2 * nb2 + (int64_t) i3 * nb3 + (int64_t) c0 * 2;
    int          finite = 0, nonzero = 0;
    // per row of this tile: first -inf column, last zero column, any value that is neither; folded
    // into the row's summary (zeroed before the launch) with one set of atomics per row and tile
    auto summarize = [&](int rr, int ninf_first, int zero_last, int other) {
        int * ri = rowinfo + ((int64_t) plane * n_q + r0 + rr) * 3;
        if (ninf_first < DN_N) {
            atomicMax(&ri[0], n_kv - (c0 + ninf_first));
        }
        if (zero_last >= 0) {
            atomicMax(&ri[1], c0 + zero_last + 1);
        }
        if (other) {
            atomicOr(&ri[2], 1);
        }
    };
    if (vec && nc == DN_N) {
        constexpr int LPR = DN_N / 8;  // lanes per row: 16, half a warp
        const int     rr  = threadIdx.x / LPR, l = threadIdx.x % LPR;
        if (rr < nr) {  // uniform over the 16 lanes of the row
            const uint4    u    = *reinterpret_cast<const uint4 *>(base + (int64_t) rr * nb1 + l * 16);
            const uint32_t w[4] = { u.x, u.y, u.z, u.w };
            int            nf = DN_N, zl = -1, ot = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t lo = w[j] & 0xFFFFu, hi = w[j] >> 16;
                finite |= (lo != 0xFC00u) | (hi != 0xFC00u);
                nonzero |= ((lo & 0x7FFFu) != 0u) | ((hi & 0x7FFFu) != 0u);
                const int c = l * 8 + 2 * j;
                if (lo == 0xFC00u) { nf = min(nf, c); }
                if (hi == 0xFC00u) { nf = min(nf, c + 1); }
                if ((lo & 0x7FFFu) == 0u) { zl = c; }
                if ((hi & 0x7FFFu) == 0u) { zl = c + 1; }
                ot |= (lo != 0xFC00u && (lo & 0x7FFFu) != 0u) | (hi != 0xFC00u && (hi & 0x7FFFu) != 0u);
            }
            // the 16 lanes of a row are one half of the warp; the other half may have no row
            const unsigned hm = (threadIdx.x & 16u) ? 0xFFFF0000u : 0x0000FFFFu;
#pragma unroll
            for (int o = 1; o < LPR; o <<= 1) {
                nf = min(nf, __shfl_xor_sync(hm, nf, o));
                zl = max(zl, __shfl_xor_sync(hm, zl, o));
                ot |= __shfl_xor_sync(hm, ot, o);
            }
            if (l == 0) {
                summarize(rr, nf, zl, ot);
            }
        }
    } else if ((int) threadIdx.x < nr) {  // partial tile or unaligned rows: one thread per row
        const int rr = threadIdx.x;
        int       nf = DN_N, zl = -1, ot = 0;
        for (int c = 0; c < nc; c++) {
            const float v = __half2float(*reinterpret_cast<const __half *>(base + (int64_t) rr * nb1 + (int64_t) c * 2));
            finite |= v != -INFINITY;
            nonzero |= v != 0.0f;
            if (v == -INFINITY) {
                nf = min(nf, c);
            } else if (v == 0.0f) {
                zl = c;
            } else {
                ot = 1;
            }
        }
        summarize(rr, nf, zl, ot);
    }
    finite  = __syncthreads_or(finite);
    nonzero = __syncthreads_or(nonzero);
    if (threadIdx.x == 0) {
        const uint32_t f = (finite ? BLKF_FINITE : 0u) | (nonzero ? BLKF_NONZERO : 0u);
        if (f) {
            atomicOr(&bflags[((int64_t) plane * n_qt + r0 / qrows) * n_kt + kt], f);
        }
    }
}

// ------------------------------------------------------------------ host side

namespace {

template <int D, bool BF16>
void * dense_kernel_ptr(int & smem) {
    smem = DenseSmem<D>::TOTAL;
    return reinterpret_cast<void *>(&fa_dense_kernel<D, BF16>);
}

void * select_dense_kernel(int D, bool bf16, int & smem) {
    if (D == 128) {
        return bf16 ? dense_kernel_ptr<128, true>(smem) : dense_kernel_ptr<128, false>(smem);
    }
    if (D == 64) {
        return bf16 ? dense_kernel_ptr<64, true>(smem) : dense_kernel_ptr<64, false>(smem);
    }
    return nullptr;
}

// The register split of the warpgroups assumes the kernel launches with DN_REGS_LAUNCH registers
// per thread; a build that allocates fewer would make setmaxnreg.inc wait forever, so it is
// refused here instead of launched.
cudaError_t check_launch_registers(const void * fn) {
    cudaFuncAttributes a{};
    cudaError_t        e = cudaFuncGetAttributes(&a, fn);
    if (e != cudaSuccess) {
        return e;
    }
    return a.numRegs == DN_REGS_LAUNCH ? cudaSuccess : cudaErrorInvalidConfiguration;
}

}  // namespace

bool dense_eligible(int D, int kvt) {
    return (kvt == KV_F16 || kvt == KV_BF16) && (D == 64 || D == 128) && tensor_maps_available();
}

size_t dense_workspace_bytes(int64_t n_q, int64_t n_kv, int64_t planes) {
    const int64_t n_qt = (n_q + DN_M - 1) / DN_M, n_kt = (n_kv + DN_N - 1) / DN_N;  // 128-row blocks at most
    return WS_STATUS_BYTES + (size_t) ((planes * n_qt * n_kt * 4 + 255) / 256 * 256) +
           (size_t) ((planes * n_q * 12 + 255) / 256 * 256);
}

cudaError_t launch_dense(DenseParams p, int D, int kvt, int64_t n_head_kv, int64_t n_seq_k, int64_t n_head,
                         int64_t n_seq, void * workspace, cudaStream_t stream) {
    const bool bf16 = kvt == KV_BF16;
    int        smem = 0;
    void *     fn   = select_dense_kernel(D, bf16, smem);
    if (!fn) {
        return cudaErrorInvalidValue;
    }
    cudaError_t e = check_launch_registers(fn);
    if (e != cudaSuccess) {
        return e;
    }
    alignas(64) CUtensorMap tmk, tmv;
    if (!encode_kv_tensor_map(&tmk, p.k, bf16, D, p.n_kv, n_head_kv, n_seq_k, p.k_nb1, p.k_nb2, p.k_nb3, DN_N) ||
        !encode_kv_tensor_map(&tmv, p.v, bf16, D, p.n_kv, n_head_kv, n_seq_k, p.v_nb1, p.v_nb2, p.v_nb3, DN_N)) {
        return cudaErrorInvalidValue;
    }
    // result tensor map for the TMA-store epilogue: [D, n_head, n_q, n_seq] F32 (ggml's layout),
    // boxes of 32 floats x 128 rows, 128-byte swizzle; element stores are the fallback
    alignas(64) CUtensorMap tmo;
    p.tma_store = 0;
    if (p.dst_vec && p.d_nb1 % 16 == 0 && p.d_nb2 % 16 == 0 && p.d_nb3 % 16 == 0) {
        auto enc = tensor_map_encoder();
        if (enc) {
            const int64_t nb2 = p.n_q > 1 ? p.d_nb2 : p.d_nb1 * n_head, nb1 = n_head > 1 ? p.d_nb1 : 4 * D;
            const int64_t nb3 = n_seq > 1 ? p.d_nb3 : nb2 * p.n_q;
            cuuint64_t dims[4]    = { (cuuint64_t) D, (cuuint64_t) n_head, (cuuint64_t) p.n_q, (cuuint64_t) n_seq };
            cuuint64_t strides[3] = { (cuuint64_t) nb1, (cuuint64_t) nb2, (cuuint64_t) nb3 };
            cuuint32_t box[4]     = { 32, 1, (cuuint32_t) DN_M, 1 };
            cuuint32_t estr[4]    = { 1, 1, 1, 1 };
            p.tma_store = enc(&tmo, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, p.dst, dims, strides, box, estr,
                              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_NONE,
                              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
        }
    }
    if (p.n_peers > 0 && !p.tma_store) {
        return cudaErrorNotSupported;  // the fused exchange lives in the TMA-store epilogue
    }
    char * ws = static_cast<char *>(workspace);
    p.status  = reinterpret_cast<uint32_t *>(ws);
    // head pairs: GQA (an even number of query heads per kv head) with one mask plane for all heads
    p.pair          = (p.mask && p.ratio % 2 == 0 && p.m_ne2 == 1) ? 1 : 0;
    const int qrows = p.pair ? DN_M : DN_ROWS;
    p.n_qt    = (int) ((p.n_q + qrows - 1) / qrows);
    p.n_kt    = (int) ((p.n_kv + DN_N - 1) / DN_N);
    p.blocks  = nullptr;
    p.rowinfo = nullptr;
    if (p.mask) {
        uint32_t *   blocks = reinterpret_cast<uint32_t *>(ws + WS_STATUS_BYTES);
        const int    planes = p.m_ne2 * p.m_ne3;
        const size_t nblk   = (size_t) (((int64_t) planes * p.n_qt * p.n_kt * 4 + 255) / 256 * 256);
        int *        rinfo  = reinterpret_cast<int *>(ws + WS_STATUS_BYTES + nblk);
        e = cudaMemsetAsync(blocks, 0, nblk + (size_t) planes * p.n_q * 12, stream);  // flags and row summaries
        if (e != cudaSuccess) {
            return e;
        }
        const unsigned rgroups = (unsigned) ((p.n_q + MASK_ROWS - 1) / MASK_ROWS);
        // the attention's CTAs become resident beside this kernel's: its SMs keep the largest
        // shared-memory carve-out
        static const cudaError_t carve = [] {
            const cudaError_t c = cudaFuncSetAttribute(mask_block_class_kernel,
                                                       cudaFuncAttributePreferredSharedMemoryCarveout,
                                                       (int) cudaSharedmemCarveoutMaxShared);
            cudaGetLastError();
            return c;
        }();
        (void) carve;
        mask_block_class_kernel<<<dim3((unsigned) p.n_kt, rgroups, (unsigned) planes), MASK_CLASS_THREADS, 0,
                                  stream>>>(p.mask, p.m_nb1, p.m_nb2, p.m_nb3, p.m_ne2, p.n_q, p.n_kv, p.n_qt, p.n_kt,
                                            qrows, p.mask_vec, blocks, rinfo);
        e = cudaGetLastError();
        if (e != cudaSuccess) {
            return e;
        }
        p.blocks  = blocks;
        p.rowinfo = rinfo;
    }
    e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        return e;
    }
    // work items and the split of the last wave: one CTA per SM at a time, so a final wave that
    // would leave more than a quarter of the SMs idle is run as 2-CTA clusters that halve each
    // item's K/V range (all items, when there are at most half as many items as SMs)
    p.n_head          = (int) n_head;
    p.n_seq           = (int) n_seq;
    const int n_items = p.n_qt * (p.pair ? p.n_head / 2 : p.n_head) * p.n_seq;
    int       sms     = 148;
    int       dev     = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) {
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    }
    int         n_split = 0;
    const char * env    = std::getenv("MM3FA_DENSE_SPLIT");
    // a half item has its own Q staging, epilogue and merge: only items of at least 16 K/V tiles
    // gain from halving
    if (!(env && env[0] == '0') && p.n_kt >= 16 && p.n_peers == 0) {  // (split halves: no fused exchange)
        if (2 * n_items <= sms) {
            n_split = n_items;
        } else {
            const int tail = n_items % sms;
            n_split        = (tail > 0 && 4 * tail < 3 * sms) ? tail : 0;
        }
        if (n_split > 0 && (n_items - n_split) % 2) {
            n_split++;  // clusters tile the grid, so the whole items come in an even number
        }
    }
    p.n_regular   = n_items - n_split;
    void * args[] = { &tmk, &tmv, &tmo, &p };
    cudaLaunchConfig_t  cfg{};
    cudaLaunchAttribute attr[2];
    cfg.gridDim          = dim3((unsigned) (p.n_regular + 2 * n_split));
    cfg.blockDim         = dim3(DN_THREADS);
    cfg.dynamicSmemBytes = (size_t) smem;
    cfg.stream           = stream;
    cfg.attrs            = attr;
    cfg.numAttrs         = 0;
    if (n_split > 0) {
        attr[cfg.numAttrs].id               = cudaLaunchAttributeClusterDimension;
        attr[cfg.numAttrs].val.clusterDim.x = 2;
        attr[cfg.numAttrs].val.clusterDim.y = 1;
        attr[cfg.numAttrs].val.clusterDim.z = 1;
        cfg.numAttrs++;
    }
    // masked calls: programmatic launch after the pre-pass (MM3FA_PDL=0 turns it off)
    static const bool pdl = [] {
        const char * e = std::getenv("MM3FA_PDL");
        return !(e && std::atoi(e) == 0);
    }();
    if (p.mask && pdl) {
        attr[cfg.numAttrs].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[cfg.numAttrs].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs++;
    }
    return cudaLaunchKernelExC(&cfg, fn, args);
}

}  // namespace mm3fa
