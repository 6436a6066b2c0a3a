// fa_prologue.cuh - host interface of the fused decode prologue (fa_prologue.cu).
#pragma once

#include "fa_common.cuh"

#include <cuda_runtime.h>

namespace mm3fa {

// ---- per-vector steps of the prologue kernels.  Lane l of a warp holds elements [l*E, l*E + E)
// of a D = 32*E vector.

// RMSNorm of x over the D values in place: the row's mean square, scale = 1/sqrt(mean + eps),
// x*scale then times the weight (ggml's two roundings).
template <int E>
__device__ __forceinline__ void rms_norm_vec(float (&x)[E], const float * w, float eps, int lane) {
    constexpr int D  = 32 * E;
    float         ss = 0.0f;
#pragma unroll
    for (int e = 0; e < E; e++) {
        ss = fmaf(x[e], x[e], ss);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        ss += __shfl_xor_sync(0xffffffffu, ss, o);
    }
    const float scale = 1.0f / sqrtf(ss / (float) D + eps);
#pragma unroll
    for (int e = 0; e < E; e++) {
        x[e] = (x[e] * scale) * w[lane * E + e];
    }
}

// NeoX RoPE of x into y given cos/sin of this lane's pairs: the pair (i, i + D/2) of lanes
// l < 16 sits in lane l + 16 at the same offset; c[e], sn[e] belong to pair (l & 15)*E + e.
template <int E>
__device__ __forceinline__ void rope_vec(const float (&x)[E], float (&y)[E], const float (&c)[E], const float (&sn)[E],
                                         int lane) {
#pragma unroll
    for (int e = 0; e < E; e++) {
        const float xo = __shfl_xor_sync(0xffffffffu, x[e], 16);  // the pair's other value
        // lanes 0-15 hold x0 (first half), lanes 16-31 hold x1 (second half)
        y[e] = lane < 16 ? x[e] * c[e] - xo * sn[e] : xo * sn[e] + x[e] * c[e];
    }
}

// The angle of pair k is pos * theta_scale^k built by k successive products (ggml's rope cache).
__device__ __forceinline__ float rope_angle(float pos, float theta_scale, int k) {
    float th = pos;
    for (int i = 0; i < k; i++) {
        th *= theta_scale;
    }
    return th;
}

// RMSNorm, weight, then NeoX RoPE of one vector (lane layout above) into y.
template <int E>
__device__ __forceinline__ void rms_norm_rope_vec(float (&x)[E], float (&y)[E], const float * w, float eps, float pos,
                                                  float theta_scale, int lane) {
    rms_norm_vec<E>(x, w, eps, lane);
    float c[E], sn[E];
    float th = rope_angle(pos, theta_scale, (lane & 15) * E);
#pragma unroll
    for (int e = 0; e < E; e++) {
        c[e]  = cosf(th);
        sn[e] = sinf(th);
        th *= theta_scale;
    }
    rope_vec<E>(x, y, c, sn, lane);
}

// One cache row from the D values: F16/BF16 rounded to nearest even, or Q8_0 blocks (amax/127
// scale stored as f16, values round(x / d)).
template <int E>
__device__ __forceinline__ void store_cache_row(char * row, int kvt, const float (&y)[E], int lane) {
    if (kvt == KV_Q8_0) {
        // a 32-value block spans 32/E lanes
        constexpr int LPB  = QK8_0 / E;
        float         amax = 0.0f;
#pragma unroll
        for (int e = 0; e < E; e++) {
            amax = fmaxf(amax, fabsf(y[e]));
        }
#pragma unroll
        for (int o = 1; o < LPB; o <<= 1) {
            amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        }
        const float d    = amax / 127.0f;
        const float id   = d != 0.0f ? 1.0f / d : 0.0f;
        const int   blk  = lane / LPB;
        char *      bp   = row + blk * Q8_0_BLOCK;
        const int   off  = (lane % LPB) * E;
#pragma unroll
        for (int e = 0; e < E; e++) {
            bp[2 + off + e] = (char) (int8_t) roundf(y[e] * id);
        }
        if (lane % LPB == 0) {
            *reinterpret_cast<__half *>(bp) = __float2half_rn(d);
        }
        return;
    }
    if (kvt == KV_BF16) {
        __nv_bfloat16 * r = reinterpret_cast<__nv_bfloat16 *>(row) + lane * E;
#pragma unroll
        for (int e = 0; e < E; e++) {
            r[e] = __float2bfloat16_rn(y[e]);
        }
        return;
    }
    __half * r = reinterpret_cast<__half *>(row) + lane * E;
#pragma unroll
    for (int e = 0; e < E; e++) {
        r[e] = __float2half_rn(y[e]);
    }
}

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
    int             clamp_v;  // v clamped to [-65504, 65504] before the cache conversion (NaN kept)
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
