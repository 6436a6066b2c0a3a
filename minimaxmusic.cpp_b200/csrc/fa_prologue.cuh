// fa_prologue.cuh - host interface of the fused decode prologue (fa_prologue.cu).
#pragma once

#include "fa_common.cuh"

#include <cuda_runtime.h>

namespace mm3fa {

struct PrologueParams {
    const char *    q_in;
    const char *    k_in;
    const char *    v_in;
    const float *   q_norm;
    const float *   k_norm;
    const int32_t * pos;
    const int64_t * rows;
    char *          q_out;
    char *          k_cache;
    char *          v_cache;
    int64_t         qi_nb1, qi_nb2, ki_nb1, ki_nb2, vi_nb1, vi_nb2;
    int64_t         qo_nb1, qo_nb2;
    int64_t         kc_nb1, kc_nb2, kc_nb3, vc_nb1, vc_nb2, vc_nb3;
    int             kvt;  // cache type (F16, BF16, Q8_0)
    int             n_head, n_head_kv, n_set;
    int64_t         k_rows, v_rows;  // rows of each cache slice: a row index outside is not written
    float           eps, theta_scale;
};

// D = 64, 128 or 256; one warp per q, k and v head vector of every set.
cudaError_t launch_decode_prologue(const PrologueParams & p, int D, cudaStream_t stream);

// DiT attention prologue: partial NeoX RoPE of q and k over the first rot dims, q to F32, k and
// v to F16/BF16, every tensor addressed by (head, token, batch) strides.
struct DitPrologueParams {
    const char *    q_in;
    const char *    k_in;
    const char *    v_in;
    const int32_t * pos;  // [S]
    char *          q_out;
    char *          k_out;
    char *          v_out;
    int64_t         sq_in[3], sk_in[3], sv_in[3];     // byte strides of (head, token, batch)
    int64_t         sq_out[3], sk_out[3], sv_out[3];
    int             kvt;  // F16 or BF16
    int             n_head, n_tok, n_batch, rot;
    float           theta_scale;
};

cudaError_t launch_dit_prologue(const DitPrologueParams & p, int D, cudaStream_t stream);

}  // namespace mm3fa
