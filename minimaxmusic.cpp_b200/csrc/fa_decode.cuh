// fa_decode.cuh - host interface of the split-KV decode kernel (fa_decode.cu).
#pragma once

#include "fa_common.cuh"

#include <cuda.h>
#include <cudaTypedefs.h>
#include <cuda_runtime.h>

namespace mm3fa {

// Iterates the stages of one CTA's key range [pos, end) of the n_units * n_kv key positions;
// a stage never crosses a unit boundary.  One division at construction, none per stage.
// Strided form (step > 0): the chunks j = first, first + step, ... of one unit.
struct StageIter {
    int64_t pos, end, unit;
    int     j, n_kv, C, step;

    __device__ StageIter(int64_t g0, int64_t g1, int n_kv_, int C_) : pos(g0), end(g1), n_kv(n_kv_), C(C_), step(0) {
        unit = g0 / n_kv_;
        j    = (int) (g0 - unit * n_kv_);
    }

    __device__ StageIter(int64_t unit_, int first, int step_, int n_kv_, int C_)
        : pos(0), end(0), unit(unit_), j(first), n_kv(n_kv_), C(C_), step(step_) {}

    __device__ bool has() const { return step ? j < n_kv : pos < end; }

    __device__ void next(int64_t & u, int & j0, int & n) {
        u  = unit;
        j0 = j;
        n  = min(C, n_kv - j);
        if (step) {
            j += step;
            return;
        }
        const int64_t left = end - pos;
        if ((int64_t) n > left) {
            n = (int) left;
        }
        pos += n;
        j += n;
        if (j == n_kv) {
            unit++;
            j = 0;
        }
    }
};

// Merges the split-KV partial slots of one unit into dst; run by the CTA that arrived last for
// the unit, with nthr threads (index t).  Partial slot s holds, per row r < RMAX, the running
// maximum m (log2 units), the row sum l and the unnormalised O[D].  Slots are folded in chunks
// of MERGE_SC with an online rescale: (m, l) of a chunk are fetched all at once into shared
// memory, and the O rows are read as float4 with 8 loads in flight, so no load waits on the
// one before it.  buf needs 2*nrow*MERGE_SC floats, rowst 3*nrow floats.  bar() synchronises
// the nthr threads; dst_row(r) returns the float* of unit row r in dst.
constexpr int MERGE_SC = 32;

template <int D, int RMAX, int RUSE, int NTHR, typename Bar, typename DstRow>
__device__ __forceinline__ void merge_unit_partials(const DecodeParams & p, int64_t unit, int nslot, int nrow, int t,
                                                    float * buf, float * rowst, Bar bar, DstRow dst_row) {
    // RMAX: rows reserved per partial slot; RUSE: upper bound of nrow for this caller
    constexpr int G4  = D / 4;                                // float4 groups per row
    constexpr int PER = (RUSE * G4 + NTHR - 1) / NTHR;        // groups per thread at most
    float *       sw  = buf;                                  // [nrow][MERGE_SC] m, then weights
    float *       sl  = buf + nrow * MERGE_SC;                // [nrow][MERGE_SC] l
    float *       Mr  = rowst;
    float *       Lr  = rowst + nrow;
    float *       So  = rowst + 2 * nrow;
    const int64_t b0  = unit * p.max_slots;
    const int     ngr = nrow * G4;
    float4        o[PER];
#pragma unroll
    for (int k = 0; k < PER; k++) {
        o[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (t < nrow) {
        Mr[t] = -INFINITY;
        Lr[t] = 0.0f;
    }
    bar();
    for (int c0 = 0; c0 < nslot; c0 += MERGE_SC) {
        const int cn = min(MERGE_SC, nslot - c0);
        for (int i = t; i < nrow * cn; i += NTHR) {
            const int     r  = i / cn, s = i % cn;
            const float * ml = &p.part_ml[((b0 + c0 + s) * RMAX + r) * 2];
            sw[r * MERGE_SC + s] = __ldcg(ml);
            sl[r * MERGE_SC + s] = __ldcg(ml + 1);
        }
        bar();
        if (t < nrow) {
            float Mc = Mr[t];
            for (int s = 0; s < cn; s++) {
                Mc = fmaxf(Mc, sw[t * MERGE_SC + s]);
            }
            const float so = (Mr[t] == -INFINITY || Mc == -INFINITY) ? 0.0f : exp2f(Mr[t] - Mc);
            float       L  = Lr[t] * so;
            for (int s = 0; s < cn; s++) {
                const float m = sw[t * MERGE_SC + s];
                const float w = (m == -INFINITY) ? 0.0f : exp2f(m - Mc);
                sw[t * MERGE_SC + s] = w;
                L += w * sl[t * MERGE_SC + s];
            }
            Mr[t] = Mc;
            Lr[t] = L;
            So[t] = so;
        }
        bar();
#pragma unroll
        for (int k = 0; k < PER; k++) {
            const int gi = t + k * NTHR;
            if (gi < ngr) {
                const int   r  = gi / G4, d4 = gi % G4;
                const float so = So[r];
                float4      a  = make_float4(o[k].x * so, o[k].y * so, o[k].z * so, o[k].w * so);
                const float4 * src = reinterpret_cast<const float4 *>(p.part_o + (b0 + c0) * RMAX * D + (int64_t) r * D) + d4;
#pragma unroll 8
                for (int s = 0; s < cn; s++) {
                    const float  w = sw[r * MERGE_SC + s];
                    const float4 v = __ldcg(src + (int64_t) s * RMAX * G4);
                    a.x += w * v.x;
                    a.y += w * v.y;
                    a.z += w * v.z;
                    a.w += w * v.w;
                }
                o[k] = a;
            }
        }
        bar();
    }
#pragma unroll
    for (int k = 0; k < PER; k++) {
        const int gi = t + k * NTHR;
        if (gi < ngr) {
            const int   r   = gi / G4, d4 = gi % G4;
            const float L   = Lr[r];
            const float inv = L > 0.0f ? 1.0f / L : 0.0f;
            float *     dst = dst_row(r) + 4 * d4;
            dst[0]          = o[k].x * inv;
            dst[1]          = o[k].y * inv;
            dst[2]          = o[k].z * inv;
            dst[3]          = o[k].w * inv;
        }
    }
}

// One element of a Q row of type F32, F16 or BF16.
__device__ __forceinline__ float ld_q_elem(const char * p, int type, int e) {
    if (type == KV_F32) {
        return reinterpret_cast<const float *>(p)[e];
    }
    if (type == KV_F16) {
        return __half2float(reinterpret_cast<const __half *>(p)[e]);
    }
    return __bfloat162float(reinterpret_cast<const __nv_bfloat16 *>(p)[e]);
}

// N elements idx(0..N-1) of one Q row as floats (zeros when !valid), the type decided once so
// that the N loads are independent and in flight together (a type test per element kept the
// compiler from batching them: one memory latency per element at kernel start).
template <int N, typename Idx>
__device__ __forceinline__ void ld_q_elems(float (&x)[N], const char * row, int type, bool valid, Idx idx) {
    if (!valid) {
#pragma unroll
        for (int i = 0; i < N; i++) {
            x[i] = 0.0f;
        }
    } else if (type == KV_F32) {
        const float * r = reinterpret_cast<const float *>(row);
#pragma unroll
        for (int i = 0; i < N; i++) {
            x[i] = r[idx(i)];
        }
    } else if (type == KV_F16) {
        const __half * r = reinterpret_cast<const __half *>(row);
#pragma unroll
        for (int i = 0; i < N; i++) {
            x[i] = __half2float(r[idx(i)]);
        }
    } else {
        const __nv_bfloat16 * r = reinterpret_cast<const __nv_bfloat16 *>(row);
#pragma unroll
        for (int i = 0; i < N; i++) {
            x[i] = __bfloat162float(r[idx(i)]);
        }
    }
}

// Launch geometry: the n_units * n_kv key positions cut into n_ctas ranges of keys_per_cta.
struct DecodeGeometry {
    int64_t n_units;        // (q sequence, kv head, row group) triples
    int64_t keys_per_cta;   // W
    int64_t n_ctas;
    int     max_slots;      // partial-result slots reserved per unit
    int     rows_per_unit;  // query rows per unit (<= 32)
    int     groups;         // row groups per (sequence, kv head)
};

// Resident CTAs per SM of the kernel instance for head dim D and K/V type kvt.
int decode_ctas_per_sm(int D, int kvt, bool bulk);

DecodeGeometry decode_geometry(int n_seq, int n_head_kv, int ratio, int n_q, int n_kv, int key_align, int n_sms,
                               int ctas_per_sm);

// Workspace bytes: status word, per-unit arrival counters, partial (m, l) and O.
size_t decode_workspace_bytes(const DecodeGeometry & g, int D);

cudaError_t launch_decode(DecodeParams p, const DecodeGeometry & g, int D, int kvt, bool bulk, void * workspace,
                          cudaStream_t stream);

// TMA tensor map of a [D, n_kv, Hkv, S_k] F16/BF16 ggml view: boxes of 64 elements x box_rows
// keys, 128-byte swizzle (fa_decode_mma.cu).  False when the driver entry point is missing or the
// strides cannot be expressed.
bool encode_kv_tensor_map(CUtensorMap * tm, const void * data, bool bf16, int64_t D, int64_t n_kv, int64_t hkv,
                          int64_t sk, int64_t nb1, int64_t nb2, int64_t nb3, int box_rows);
bool tensor_maps_available();
// cuTensorMapEncodeTiled from the driver (nullptr when unavailable)
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder();

// Tensor-core variant (fa_decode_mma.cu): F16/BF16 K/V, D 64 or 128, <= 16 rows per unit,
// strides that a TMA tensor map can express.
bool        decode_mma_eligible(int D, int kvt, int rows_per_pair);
int         decode_mma_ctas_per_sm(int D, int kvt, int rows_per_pair);
// Launch plan of the cluster mode: CTAs per thread-block cluster (0 = use the stream-K split) and
// the K/V ring depth of the instance.
struct MmaPlan {
    int cluster;
    int nstage;
};
MmaPlan     decode_mma_plan(int D, int kvt, int rows_per_pair, int64_t n_units, int n_sms);
cudaError_t launch_decode_mma(DecodeParams p, const DecodeGeometry & g, int D, int kvt, int64_t n_head_kv,
                              int64_t n_seq_k, MmaPlan plan, void * workspace, cudaStream_t stream);

}  // namespace mm3fa
