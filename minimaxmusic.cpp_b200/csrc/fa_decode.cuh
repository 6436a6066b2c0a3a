// fa_decode.cuh - host interface of the split-KV decode kernel (fa_decode.cu).
#pragma once

#include "fa_common.cuh"

#include <cuda_runtime.h>

namespace mm3fa {

// Iterates the stages of one CTA's key range [pos, end) of the n_units * n_kv key positions;
// a stage never crosses a unit boundary.
struct StageIter {
    int64_t pos, end;
    int     n_kv, C;

    __device__ bool has() const { return pos < end; }

    __device__ void next(int64_t & unit, int & j0, int & n) {
        unit               = pos / n_kv;
        j0                 = (int) (pos - unit * n_kv);
        const int64_t left = end - pos;
        n                  = min(C, n_kv - j0);
        if ((int64_t) n > left) {
            n = (int) left;
        }
        pos += n;
    }
};

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

// Tensor-core variant (fa_decode_mma.cu): F16/BF16 K/V, D 64 or 128, <= 16 rows per unit,
// strides that a TMA tensor map can express.
bool        decode_mma_eligible(int D, int kvt, int rows_per_pair);
int         decode_mma_ctas_per_sm(int D, int kvt, int rows_per_pair);
cudaError_t launch_decode_mma(DecodeParams p, const DecodeGeometry & g, int D, int kvt, int64_t n_head_kv,
                              int64_t n_seq_k, void * workspace, cudaStream_t stream);

}  // namespace mm3fa
