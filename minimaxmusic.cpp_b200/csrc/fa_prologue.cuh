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

}  // namespace mm3fa
