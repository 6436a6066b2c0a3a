// fa_decode.cuh - host interface of the split-KV decode kernel (fa_decode.cu).
#pragma once

#include "fa_common.cuh"

#include <cuda_runtime.h>

namespace mm3fa {

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

}  // namespace mm3fa
