// fa_decode.cu - split-KV flash-attention decode kernel for sm_100a.
//
// Serves GGML_OP_FLASH_ATTN_EXT when few query rows meet a long KV cache: the batched
// CFG decode of src/qwen3-lm.h:784-824 (1 row per KV set, 32 q heads over 8 kv heads,
// D=128, F16 cache viewed at [128, n_kv_pad, 8, N]) and, with the same kernel, up to
// 8 rows per sequence.  The op is HBM-bound: every K/V byte must be read once.
//
// Work decomposition.  A "unit" is (q sequence, kv head, row group): the <= 32 query rows
// (GQA heads x query positions) that share one K/V slab.  The n_units * n_kv key positions
// are cut into equal contiguous ranges, one per CTA, sized so that one wave of resident
// CTAs covers the whole job (a stream-K split: ranges may straddle unit boundaries, so the
// load is balanced for any n_units).  A CTA that covers a unit entirely writes dst
// directly; otherwise it writes an unnormalised partial (O, m, l) and the last CTA to finish
// a unit (arrival counter, no waiting) merges the partials into dst and re-zeroes the
// counter, so the kernel is one launch and replays in CUDA graphs.
//
// Data movement.  K and V rows of a slab are contiguous (nb1 == row bytes), so a stage of
// C keys is one 1-D bulk copy per tensor issued by a single thread through the TMA engine
// into a NSTAGE-deep shared-memory ring, completion tracked by mbarrier transaction
// counts.  Layouts whose strides break the 16-byte rule of bulk copies take a cooperative
// element-copy path instead (same math).
//
// Math (F32 accumulation): Q is rounded to K's vec-dot type first (F16, BF16, or quantized to
// Q8_0 blocks when K is Q8_0, whose dot is then an exact int8 dot per block times both fp16
// scales; F32 K keeps Q as it is).  F32 K/V (the depth decoder's manual attention,
// src/depth-decoder.h:210-219, is F32 throughout) use this kernel only.  Scores s = scale * q.k (then softcap), + slope_h * mask,
// kept in log2 units; one-pass online softmax per stage; V accumulated in F32 (Q8_0 V is
// dequantized exactly in registers as fp16(d) * int8).
#include "fa_decode.cuh"

#include <algorithm>
#include <cstdio>

namespace mm3fa {

constexpr int DEC_THREADS = 256;  // 8 warps
constexpr int DEC_RMAX    = 32;   // query rows per unit

template <int D, int KVT>
struct KvRow {
    static constexpr int BYTES = KVT == KV_Q8_0 ? D / QK8_0 * Q8_0_BLOCK : (KVT == KV_F32 ? 4 * D : 2 * D);
};

// 8 consecutive K or V elements of an F16, BF16 or F32 row in shared memory (16-byte aligned
// for 16-bit types, 32-byte for F32) as floats.
template <int KVT>
__device__ __forceinline__ void lds8(const char * p, float (&x)[8]) {
    if constexpr (KVT == KV_F32) {
        const float4 a = *reinterpret_cast<const float4 *>(p);
        const float4 b = *reinterpret_cast<const float4 *>(p + 16);
        x[0] = a.x, x[1] = a.y, x[2] = a.z, x[3] = a.w, x[4] = b.x, x[5] = b.y, x[6] = b.z, x[7] = b.w;
    } else {
        const uint4    raw   = *reinterpret_cast<const uint4 *>(p);
        const uint32_t rw[4] = { raw.x, raw.y, raw.z, raw.w };
#pragma unroll
        for (int w = 0; w < 4; w++) {
            const float2 f = KVT == KV_F16 ? h2_to_f2(rw[w]) : bf2_to_f2(rw[w]);
            x[2 * w]       = f.x;
            x[2 * w + 1]   = f.y;
        }
    }
}

template <int D, int KVT, int C, int NSTAGE>
struct DecodeSmem {
    static constexpr int ROW        = KvRow<D, KVT>::BYTES;
    static constexpr int MAT_BYTES  = ((C * ROW + 15) / 16) * 16;
    static constexpr int STAGE      = 2 * MAT_BYTES;
    static constexpr int OFF_STAGES = 0;
    static constexpr int OFF_S      = NSTAGE * STAGE + 16;               // scores / probabilities
    static constexpr int OFF_QO     = OFF_S + DEC_RMAX * C * 4;          // Q staging, O reduction
    static constexpr int OFF_Q8     = OFF_QO + DEC_RMAX * D * 4;         // int8 Q (Q8_0 K only)
    static constexpr int OFF_QD     = OFF_Q8 + DEC_RMAX * D;             // Q8_0 scales of Q
    static constexpr int OFF_ROW    = OFF_QD + DEC_RMAX * (D / QK8_0) * 4;
    // per-row: m, l, alpha, slope, mask offset (8 B), dst offset (8 B)
    static constexpr int OFF_BAR    = OFF_ROW + DEC_RMAX * 32;
    static constexpr int OFF_FLAG   = OFF_BAR + NSTAGE * 8;
    static constexpr int TOTAL      = OFF_FLAG + 16;
};

// Reads 4*NW bytes starting at a 2-byte aligned shared-memory offset (rows start 4-aligned).
template <int NW>
__device__ __forceinline__ void lds_bytes(const char * row, int off, uint32_t (&out)[NW]) {
    const uint32_t * p   = reinterpret_cast<const uint32_t *>(row + (off & ~3));
    const uint32_t   sel = (off & 2) ? 0x5432u : 0x3210u;
    uint32_t         w[NW + 1];
#pragma unroll
    for (int i = 0; i <= NW; i++) {
        w[i] = p[i];
    }
#pragma unroll
    for (int i = 0; i < NW; i++) {
        out[i] = __byte_perm(w[i], w[i + 1], sel);
    }
}

// Copies rows [j0, j0 + n) of a K and a V slab (row stride nbk / nbv) into the stage, W words of
// type T per row, every thread loading up to 4 words of each before it stores them.
template <typename T, int W>
__device__ __forceinline__ void copy_rows(const char * sk, const char * sv, const char * srck, const char * srcv,
                                          int j0, int n, int64_t nbk, int64_t nbv, int tid) {
    const int total = n * W;
    for (int base = tid; base < total; base += 4 * DEC_THREADS) {
        T a[4], b[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int idx = base + u * DEC_THREADS;
            if (idx < total) {
                const int j = idx / W, w = idx % W;
                a[u]        = reinterpret_cast<const T *>(srck + (int64_t) (j0 + j) * nbk)[w];
                b[u]        = reinterpret_cast<const T *>(srcv + (int64_t) (j0 + j) * nbv)[w];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int idx = base + u * DEC_THREADS;
            if (idx < total) {
                reinterpret_cast<T *>(const_cast<char *>(sk))[idx] = a[u];
                reinterpret_cast<T *>(const_cast<char *>(sv))[idx] = b[u];
            }
        }
    }
}

template <int D, int KVT, int C, int NSTAGE, bool BULK>
__global__ void __launch_bounds__(DEC_THREADS, 1) fa_decode_kernel(const DecodeParams p) {
    using L               = DecodeSmem<D, KVT, C, NSTAGE>;
    constexpr int ROW     = L::ROW;
    constexpr int EPL     = D / 8;          // K elements per lane in the QK phase (8 lanes per key)
    constexpr int NCH     = D / 64;         // 16-byte F16 chunks per lane
    constexpr int DG      = D / 8;          // dim groups of 8 in the PV phase
    constexpr int NBLK    = D / QK8_0;
    constexpr bool IS_Q8  = KVT == KV_Q8_0;
    constexpr int LPB     = QK8_0 / EPL;    // lanes per Q8_0 block (2 for D=128, 4 for D=64)
    static_assert(D == 64 || D == 128 || D == 256, "head dim");
    static_assert(C % 32 == 0, "stage keys");

    extern __shared__ __align__(128) char smem[];
    float *    sS    = reinterpret_cast<float *>(smem + L::OFF_S);
    float *    sQO   = reinterpret_cast<float *>(smem + L::OFF_QO);
    int8_t *   sQ8   = reinterpret_cast<int8_t *>(smem + L::OFF_Q8);
    float *    sQD   = reinterpret_cast<float *>(smem + L::OFF_QD);
    float *    sM    = reinterpret_cast<float *>(smem + L::OFF_ROW);
    float *    sL    = sM + DEC_RMAX;
    float *    sA    = sL + DEC_RMAX;
    float *    sSlp  = sA + DEC_RMAX;
    int64_t *  sMoff = reinterpret_cast<int64_t *>(sSlp + DEC_RMAX);
    int64_t *  sDoff = sMoff + DEC_RMAX;
    uint64_t * bars  = reinterpret_cast<uint64_t *>(smem + L::OFF_BAR);
    int *      sFlag = reinterpret_cast<int *>(smem + L::OFF_FLAG);

    const int tid  = threadIdx.x;
    const int warp = tid >> 5;
    const int lane = tid & 31;

    const int RU  = p.rows_per_unit;
    const int RG  = RU <= 4 ? 1 : (RU <= 8 ? 2 : (RU <= 16 ? 4 : 8));  // row groups of 4
    const int WK  = 8 / RG;                                            // warps along keys (QK)
    const int KG  = DEC_THREADS / (DG * RG);                           // key groups (PV)

    const int64_t total = p.n_units * (int64_t) p.n_kv;
    const int64_t g0    = (int64_t) blockIdx.x * p.keys_per_cta;
    const int64_t g1    = min(total, g0 + p.keys_per_cta);
    if (g0 >= g1) {
        return;
    }

    if (BULK && tid == 0) {
        for (int s = 0; s < NSTAGE; s++) {
            mbar_init(&bars[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    const uint64_t deadline = global_timer_ns() + p.timeout_ns;

    // slab base pointers of a unit
    auto kv_base = [&](int64_t unit, const char * base, int64_t nb2, int64_t nb3) -> const char * {
        const int64_t sg = unit / p.groups;  // s * n_head_kv + g
        const int     g  = (int) (sg % p.n_head_kv);
        const int     s  = (int) (sg / p.n_head_kv);
        return base + (int64_t) g * nb2 + (int64_t) (s / p.rk3) * nb3;
    };

    // producer (thread 0): issue stage `idx` (ring slot idx % NSTAGE)
    StageIter pit{ g0, g1, p.n_kv, C };
    int       issued = 0;
    auto      issue  = [&]() {
        int64_t unit;
        int     j0, n;
        pit.next(unit, j0, n);
        const int  slot = issued % NSTAGE;
        char *     dk   = smem + L::OFF_STAGES + slot * L::STAGE;
        char *     dv   = dk + L::MAT_BYTES;
        const char * srck = kv_base(unit, p.k, p.k_nb2, p.k_nb3) + (int64_t) j0 * p.k_nb1;
        const char * srcv = kv_base(unit, p.v, p.v_nb2, p.v_nb3) + (int64_t) j0 * p.v_nb1;
        const uint32_t bytes = (uint32_t) (n * ROW);
        mbar_arrive_expect_tx(&bars[slot], 2 * bytes);
        bulk_copy_g2s(dk, srck, bytes, &bars[slot]);
        bulk_copy_g2s(dv, srcv, bytes, &bars[slot]);
        issued++;
    };
    if (BULK && tid == 0) {
        for (int s = 0; s < NSTAGE && pit.has(); s++) {
            issue();
        }
    }

    // per-lane Q fragments for the QK phase (4 rows per warp)
    float    qf[4][IS_Q8 ? 1 : EPL];
    uint32_t qi[4][IS_Q8 ? EPL / 4 : 1];
    float    qd[4];
    // PV accumulators: 4 rows x 8 dims
    float acc[4][8];

    const int wr   = warp / WK;   // QK: row group of this warp
    const int wk   = warp % WK;   // QK: key slice of this warp
    const int ls   = lane & 7;    // QK: lane within a key's 8 lanes
    const int kk   = lane >> 3;   // QK: key within the warp-step
    const int dg   = tid % DG;    // PV: dim group
    const int prg  = (tid / DG) % RG;  // PV: row group
    const int pkg  = tid / (DG * RG);  // PV: key group

    StageIter cit{ g0, g1, p.n_kv, C };
    int       nrow      = RU;  // valid rows of the current unit (the last row group may be short)
    int64_t   cur_unit  = -1;
    int       seg_j0    = 0;
    int       seg_j1    = 0;
    int       stage_idx = 0;
    bool      aborted   = false;
    int       u_kvl     = p.n_kv;  // keys of the current unit's sequence that are visible

    // ---- unit begin: stage Q (rounded to K's convention), row metadata, reset state
    auto begin_unit = [&](int64_t unit) {
        const int64_t sg   = unit / p.groups;
        const int     rgrp = (int) (unit % p.groups);
        const int     g    = (int) (sg % p.n_head_kv);
        const int     s    = (int) (sg / p.n_head_kv);
        nrow               = min(RU, p.rows_per_pair - rgrp * DEC_RMAX);
        u_kvl              = seq_kv_len(p.kv_len, s, p.n_kv);
        for (int idx = tid; idx < nrow * D; idx += DEC_THREADS) {
            const int r  = idx / D;
            const int e  = idx % D;
            const int rf = rgrp * DEC_RMAX + r;
            const int h  = g * p.ratio + rf / p.n_q;
            const int i  = rf % p.n_q;
            const char * qrow = p.q + (int64_t) i * p.q_nb1 + (int64_t) h * p.q_nb2 + (int64_t) s * p.q_nb3;
            float x = ld_q_elem(qrow, p.q_type, e);
            if (KVT == KV_F16) {
                x = round_to_f16(x);
            } else if (KVT == KV_BF16) {
                x = round_to_bf16(x);
            }
            sQO[r * D + e] = x;
        }
        if (tid < nrow) {
            const int r  = tid;
            const int rf = rgrp * DEC_RMAX + r;
            const int h  = g * p.ratio + rf / p.n_q;
            const int i  = rf % p.n_q;
            sM[r]   = -INFINITY;
            sL[r]   = 0.0f;
            sSlp[r] = alibi_slope(h, p.max_bias, p.n_head_log2, p.m0, p.m1);
            sMoff[r] = (int64_t) i * p.m_nb1 + (int64_t) (h % p.m_ne2) * p.m_nb2 + (int64_t) (s % p.m_ne3) * p.m_nb3;
            sDoff[r] = (int64_t) h * p.d_nb1 + (int64_t) i * p.d_nb2 + (int64_t) s * p.d_nb3;
        }
        __syncthreads();
        if (IS_Q8) {
            // quantize each 32-element block of Q exactly as ggml's Q8_0 reference quantizer
            for (int b = warp; b < nrow * NBLK; b += DEC_THREADS / 32) {
                const int r    = b / NBLK;
                const int blk  = b % NBLK;
                const float x  = sQO[r * D + blk * QK8_0 + lane];
                float amax     = fabsf(x);
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
                }
                const float d  = amax / 127.0f;
                const float id = d != 0.0f ? 1.0f / d : 0.0f;
                sQ8[r * D + blk * QK8_0 + lane] = (int8_t) roundf(x * id);
                if (lane == 0) {
                    sQD[r * NBLK + blk] = __half2float(__float2half_rn(d));
                }
            }
            __syncthreads();
        }
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
            const int r = wr * 4 + rr;
            if (IS_Q8) {
                const int e0 = ls * EPL;
#pragma unroll
                for (int w = 0; w < EPL / 4; w++) {
                    qi[rr][w] = r < nrow ? *reinterpret_cast<const uint32_t *>(&sQ8[r * D + e0 + 4 * w]) : 0u;
                }
                qd[rr] = r < nrow ? sQD[r * NBLK + e0 / QK8_0] : 0.0f;
            } else {
#pragma unroll
                for (int c = 0; c < NCH; c++) {
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        qf[rr][c * 8 + e] = r < nrow ? sQO[r * D + 64 * c + 8 * ls + e] : 0.0f;
                    }
                }
            }
        }
#pragma unroll
        for (int rr = 0; rr < 4; rr++) {
#pragma unroll
            for (int e = 0; e < 8; e++) {
                acc[rr][e] = 0.0f;
            }
        }
        __syncthreads();
        for (int idx = tid; idx < DEC_RMAX * D; idx += DEC_THREADS) {
            sQO[idx] = 0.0f;
        }
        // (the next __syncthreads in the stage loop orders this before the O reduction)
    };

    // ---- unit end: reduce O over key groups, then write dst or a partial (+ merge if last)
    auto end_unit = [&](int64_t unit, int j0, int j1) {
        // key groups add their partial O in a fixed order: results are bit-reproducible
        for (int kg = 0; kg < KG; kg++) {
            if (pkg == kg) {
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    const int r = prg * 4 + rr;
                    if (r < nrow) {
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            sQO[r * D + dg * 8 + e] += acc[rr][e];
                        }
                    }
                }
            }
            __syncthreads();
        }
        if (j0 == 0 && j1 == p.n_kv) {  // whole unit in this CTA
            for (int idx = tid; idx < nrow * D; idx += DEC_THREADS) {
                const int   r = idx / D;
                const float l = sL[r];
                float *     o = reinterpret_cast<float *>(p.dst + sDoff[r]);
                o[idx % D]    = l > 0.0f ? sQO[idx] / l : 0.0f;
            }
            __syncthreads();
            return;
        }
        const int64_t first = unit * (int64_t) p.n_kv / p.keys_per_cta;
        const int64_t last  = (unit * (int64_t) p.n_kv + p.n_kv - 1) / p.keys_per_cta;
        const int     slot  = (int) ((int64_t) blockIdx.x - first);
        const int     nslot = (int) (last - first + 1);
        const int64_t pbase = unit * p.max_slots + slot;
        for (int idx = tid; idx < nrow * D; idx += DEC_THREADS) {
            p.part_o[pbase * DEC_RMAX * D + idx] = sQO[idx];
        }
        if (tid < nrow) {
            p.part_ml[(pbase * DEC_RMAX + tid) * 2 + 0] = sM[tid];
            p.part_ml[(pbase * DEC_RMAX + tid) * 2 + 1] = sL[tid];
        }
        __threadfence();
        __syncthreads();
        if (tid == 0) {
            const uint32_t old = atomicAdd(&p.counters[unit], 1u);
            *sFlag             = (old == (uint32_t) (nslot - 1)) ? 1 : 0;
        }
        __syncthreads();
        if (*sFlag) {  // uniform: written by thread 0 before the barrier above
            __threadfence();
            // sQO and sM/sL/sA are free here: this CTA's partial is already in the workspace
            merge_unit_partials<D, DEC_RMAX, DEC_RMAX, DEC_THREADS>(
                p, unit, nslot, nrow, tid, sQO, sM, [] { __syncthreads(); },
                [&](int r) { return reinterpret_cast<float *>(p.dst + sDoff[r]); });
            if (tid == 0) {
                p.counters[unit] = 0u;  // ready for the next launch on this workspace
            }
        }
        __syncthreads();
    };

    while (cit.has()) {
        int64_t unit;
        int     j0, n;
        cit.next(unit, j0, n);
        if (unit != cur_unit) {
            if (cur_unit >= 0) {
                end_unit(cur_unit, seg_j0, seg_j1);
            }
            begin_unit(unit);
            cur_unit = unit;
            seg_j0   = j0;
        }
        seg_j1 = j0 + n;

        const int  slot = stage_idx % NSTAGE;
        const char * sk = smem + L::OFF_STAGES + slot * L::STAGE;
        const char * sv = sk + L::MAT_BYTES;
        if (BULK) {
            const bool ok = mbar_wait_bounded(&bars[slot], (uint32_t) ((stage_idx / NSTAGE) & 1), deadline);
            if (__syncthreads_or(!ok)) {
                aborted = true;
                break;
            }
        } else {
            // cooperative element copy (strides that bulk copies cannot express): 16-byte words
            // when every row start is 16-byte aligned, else 2-byte words; each thread issues its
            // loads of a round together before storing them (one memory latency per round)
            const char * srck = kv_base(unit, p.k, p.k_nb2, p.k_nb3);
            const char * srcv = kv_base(unit, p.v, p.v_nb2, p.v_nb3);
            if (ROW % 16 == 0 && p.kv_vec) {
                copy_rows<uint4, ROW / 16>(sk, sv, srck, srcv, j0, n, p.k_nb1, p.v_nb1, tid);
            } else {
                copy_rows<uint16_t, ROW / 2>(sk, sv, srck, srcv, j0, n, p.k_nb1, p.v_nb1, tid);
            }
            __syncthreads();
        }

        // ---------------- QK: scores for rows [wr*4, wr*4+4) and this warp's keys
        for (int kb = wk * 4; kb < n; kb += 4 * WK) {
            const int  j     = kb + kk;
            const bool valid = j < n;
            const char * krow = sk + (valid ? j : 0) * ROW;
            float red0, red1;  // values kept after the first halving step
            float part[4];
            if (IS_Q8) {
                const int e0  = ls * EPL;
                const int blk = e0 / QK8_0;
                uint32_t  kw[EPL / 4];
                lds_bytes<EPL / 4>(krow, blk * Q8_0_BLOCK + 2 + (e0 % QK8_0), kw);
                const float dk = __half2float(*reinterpret_cast<const __half *>(krow + blk * Q8_0_BLOCK));
                int         si[4];
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    int a = 0;
#pragma unroll
                    for (int w = 0; w < EPL / 4; w++) {
                        a = __dp4a((int) qi[rr][w], (int) kw[w], a);
                    }
                    si[rr] = a;
                }
#pragma unroll
                for (int o = 1; o < LPB; o <<= 1) {
#pragma unroll
                    for (int rr = 0; rr < 4; rr++) {
                        si[rr] += __shfl_xor_sync(0xffffffffu, si[rr], o);
                    }
                }
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    part[rr] = (float) si[rr] * (qd[rr] * dk);
                }
            } else {
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    part[rr] = 0.0f;
                }
#pragma unroll
                for (int c = 0; c < NCH; c++) {
                    // elements [64c + 8ls, 64c + 8ls + 8) of the key row
                    float kf[8];
                    lds8<KVT>(krow + (KVT == KV_F32 ? 4 : 2) * (64 * c + 8 * ls), kf);
#pragma unroll
                    for (int rr = 0; rr < 4; rr++) {
#pragma unroll
                        for (int e = 0; e < 8; e++) {
                            part[rr] = fmaf(qf[rr][c * 8 + e], kf[e], part[rr]);
                        }
                    }
                }
            }
            // sum the 4 row partials over the key's 8 lanes; afterwards lanes {s, s^1}
            // hold row 2*bit2(s) + bit1(s)
            const bool b2 = (ls >> 2) & 1;
            const bool b1 = (ls >> 1) & 1;
            {
                const float s0 = b2 ? part[0] : part[2];
                const float s1 = b2 ? part[1] : part[3];
                const float r0 = __shfl_xor_sync(0xffffffffu, s0, 4);
                const float r1 = __shfl_xor_sync(0xffffffffu, s1, 4);
                red0           = (b2 ? part[2] : part[0]) + r0;
                red1           = (b2 ? part[3] : part[1]) + r1;
            }
            float val;
            if (IS_Q8 && LPB >= 4) {  // lanes s and s^2 already hold identical block sums
                val = b1 ? red1 : red0;
            } else {
                const float snd = b1 ? red0 : red1;
                const float rcv = __shfl_xor_sync(0xffffffffu, snd, 2);
                val             = (b1 ? red1 : red0) + rcv;
            }
            if (!(IS_Q8 && LPB >= 2)) {
                val += __shfl_xor_sync(0xffffffffu, val, 1);
            }
            const int r = wr * 4 + (b2 ? 2 : 0) + (b1 ? 1 : 0);
            if (valid && (ls & 1) == 0 && r < nrow) {
                float sc = val * p.scale;
                if (p.softcap != 0.0f) {
                    sc = p.softcap * tanhf(sc / p.softcap);
                }
                if (p.mask) {
                    const float mv = __half2float(
                        *reinterpret_cast<const __half *>(p.mask + sMoff[r] + (int64_t) (j0 + j) * 2));
                    sc += sSlp[r] * mv;
                }
                sS[r * C + j] = sc * LOG2E;
            }
        }
        __syncthreads();

        // ---------------- online softmax over the stage, one warp per row
        for (int r = warp; r < nrow; r += DEC_THREADS / 32) {
            float sv_[C / 32];
            float mx = -INFINITY;
#pragma unroll
            for (int t = 0; t < C / 32; t++) {
                const int j = lane + 32 * t;
                sv_[t]      = (j < n && j0 + j < u_kvl) ? sS[r * C + j] : -INFINITY;
                mx          = fmaxf(mx, sv_[t]);
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
            }
            const float m_old = sM[r];
            const float m_new = fmaxf(m_old, mx);
            float       alpha = 1.0f, sum = 0.0f;
            if (m_new != -INFINITY) {
                alpha = exp2f(m_old - m_new);
            }
#pragma unroll
            for (int t = 0; t < C / 32; t++) {
                const float pj = m_new != -INFINITY ? exp2f(sv_[t] - m_new) : 0.0f;
                sS[r * C + lane + 32 * t] = pj;
                sum += pj;
            }
#pragma unroll
            for (int o = 16; o > 0; o >>= 1) {
                sum += __shfl_xor_sync(0xffffffffu, sum, o);
            }
            if (lane == 0) {
                sL[r] = sL[r] * alpha + sum;
                sM[r] = m_new;
                sA[r] = alpha;
            }
        }
        __syncthreads();

        // ---------------- PV: acc[4 rows][8 dims] += p * v over this thread's keys
        {
            float al[4];
#pragma unroll
            for (int rr = 0; rr < 4; rr++) {
                const int r = prg * 4 + rr;
                al[rr]      = r < nrow ? sA[r] : 1.0f;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    acc[rr][e] *= al[rr];
                }
            }
            for (int j = pkg; j < n; j += KG) {
                const char * vrow = sv + j * ROW;
                float        vf[8];
                if (IS_Q8) {
                    const int blk = (dg * 8) / QK8_0;
                    uint32_t  vw[2];
                    lds_bytes<2>(vrow, blk * Q8_0_BLOCK + 2 + (dg * 8) % QK8_0, vw);
                    const float d = __half2float(*reinterpret_cast<const __half *>(vrow + blk * Q8_0_BLOCK));
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        const int8_t b = (int8_t) ((vw[e >> 2] >> (8 * (e & 3))) & 0xff);
                        vf[e]          = d * (float) b;
                    }
                } else {
                    lds8<KVT>(vrow + (KVT == KV_F32 ? 32 : 16) * dg, vf);
                }
#pragma unroll
                for (int rr = 0; rr < 4; rr++) {
                    const float pj = sS[(prg * 4 + rr) * C + j];
#pragma unroll
                    for (int e = 0; e < 8; e++) {
                        acc[rr][e] = fmaf(pj, vf[e], acc[rr][e]);
                    }
                }
            }
        }
        __syncthreads();  // the ring slot and sS are free again
        if (BULK && tid == 0 && pit.has()) {
            issue();
        }
        stage_idx++;
    }

    if (aborted) {
        if (tid == 0) {
            atomicOr(&p.status[0], ST_TIMEOUT);
            atomicExch(&p.status[1], (uint32_t) blockIdx.x);
            // let the copies this CTA still has in flight land before its shared memory is released
            const uint64_t drain = global_timer_ns() + p.timeout_ns;
            for (int s = stage_idx; s < issued; s++) {
                mbar_wait_bounded(&bars[s % NSTAGE], (uint32_t) ((s / NSTAGE) & 1), drain);
            }
        }
        __syncthreads();
        return;
    }
    if (cur_unit >= 0) {
        end_unit(cur_unit, seg_j0, seg_j1);
    }
}

// ------------------------------------------------------------------ host side

struct DecodeConfig {
    int C;
    int nstage;
    int smem;
};

template <int D, int KVT, bool BULK>
static void * decode_kernel_ptr(int & smem, int & C) {
    // D = 256 (the depth decoder's heads): 32-key stages, 2 deep, to stay within shared memory;
    // F32 K/V (rows twice as long) 2 deep as well
    constexpr int CC     = D == 256 ? 32 : ((D == 64 && KVT != KV_Q8_0) ? 128 : 64);
    constexpr int NSTAGE = (D == 256 || KVT == KV_F32) ? 2 : 4;
    smem                 = DecodeSmem<D, KVT, CC, NSTAGE>::TOTAL;
    C                    = CC;
    return reinterpret_cast<void *>(&fa_decode_kernel<D, KVT, CC, NSTAGE, BULK>);
}

static void * select_decode_kernel(int D, int kvt, bool bulk, int & smem, int & C) {
#define MM3FA_SEL(DD, TT)                                                                  \
    if (D == DD && kvt == TT) {                                                            \
        return bulk ? decode_kernel_ptr<DD, TT, true>(smem, C) : decode_kernel_ptr<DD, TT, false>(smem, C); \
    }
    MM3FA_SEL(128, KV_F16)
    MM3FA_SEL(128, KV_BF16)
    MM3FA_SEL(128, KV_Q8_0)
    MM3FA_SEL(64, KV_F16)
    MM3FA_SEL(64, KV_BF16)
    MM3FA_SEL(64, KV_Q8_0)
    MM3FA_SEL(256, KV_F16)
    MM3FA_SEL(256, KV_BF16)
    MM3FA_SEL(256, KV_Q8_0)
    MM3FA_SEL(64, KV_F32)
    MM3FA_SEL(128, KV_F32)
    MM3FA_SEL(256, KV_F32)
#undef MM3FA_SEL
    return nullptr;
}

int decode_ctas_per_sm(int D, int kvt, bool bulk) {
    int   smem = 0, C = 0;
    void *fn   = select_decode_kernel(D, kvt, bulk, smem, C);
    if (!fn) {
        return 0;
    }
    cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    int nb = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&nb, fn, DEC_THREADS, smem) != cudaSuccess || nb < 1) {
        cudaGetLastError();
        nb = 1;
    }
    return nb;
}

DecodeGeometry decode_geometry(int n_seq, int n_head_kv, int ratio, int n_q, int n_kv, int key_align, int n_sms,
                               int ctas_per_sm) {
    DecodeGeometry g{};
    const int rows  = ratio * n_q;
    g.groups        = (rows + DEC_RMAX - 1) / DEC_RMAX;
    g.rows_per_unit = rows < DEC_RMAX ? rows : DEC_RMAX;
    g.n_units       = (int64_t) n_seq * n_head_kv * g.groups;
    const int64_t total = g.n_units * (int64_t) n_kv;
    const int64_t slots = (int64_t) std::max(1, n_sms) * std::max(1, ctas_per_sm);
    int64_t W           = (total + slots - 1) / slots;
    if (n_kv < 64) {
        // short units (the depth decoder's S <= 8 steps, short prefixes): one CTA per whole unit,
        // so they all run at once and no partials are merged (a floor of 64 keys put several
        // units in sequence into one CTA)
        W = std::max(n_kv, 1);
    } else {
        W             = std::max<int64_t>(W, 64);
        const int64_t q = std::max(16, key_align);
        W             = (W + q - 1) / q * q;
    }
    g.keys_per_cta      = W;
    g.n_ctas            = total > 0 ? (total + W - 1) / W : 0;
    g.max_slots         = (int) ((n_kv + W - 1) / W + 1);
    return g;
}

size_t decode_workspace_bytes(const DecodeGeometry & g, int D) {
    const size_t cnt  = ((size_t) g.n_units * 4 + 255) / 256 * 256;
    const size_t slot = (size_t) g.n_units * g.max_slots * DEC_RMAX;
    return WS_STATUS_BYTES + cnt + slot * 2 * 4 + slot * (size_t) D * 4;
}

cudaError_t launch_decode(DecodeParams p, const DecodeGeometry & g, int D, int kvt, bool bulk, void * workspace,
                          cudaStream_t stream) {
    int   smem = 0, C = 0;
    void *fn   = select_decode_kernel(D, kvt, bulk, smem, C);
    if (!fn) {
        return cudaErrorInvalidValue;
    }
    char * ws          = static_cast<char *>(workspace);
    const size_t cnt   = ((size_t) g.n_units * 4 + 255) / 256 * 256;
    const size_t slot  = (size_t) g.n_units * g.max_slots * DEC_RMAX;
    p.status           = reinterpret_cast<uint32_t *>(ws);
    p.counters         = reinterpret_cast<uint32_t *>(ws + WS_STATUS_BYTES);
    p.part_ml          = reinterpret_cast<float *>(ws + WS_STATUS_BYTES + cnt);
    p.part_o           = reinterpret_cast<float *>(ws + WS_STATUS_BYTES + cnt + slot * 2 * 4);
    p.n_units          = g.n_units;
    p.keys_per_cta     = g.keys_per_cta;
    p.max_slots        = g.max_slots;
    p.rows_per_unit    = g.rows_per_unit;
    p.groups           = g.groups;
    cudaError_t e      = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) {
        return e;
    }
    void * args[] = { &p };
    return cudaLaunchKernel(fn, dim3((unsigned) g.n_ctas), dim3(DEC_THREADS), args, (size_t) smem, stream);
}

}  // namespace mm3fa
