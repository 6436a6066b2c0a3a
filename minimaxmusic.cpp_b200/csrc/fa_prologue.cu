// fa_prologue.cu - fused decode prologue of one LM layer (sm_100a).
//
// The graph nodes the reference builds between the QKV projection and the attention call
// (src/qwen3-lm.h:764-800), one warp per head vector:
//   q -> ggml_rms_norm(eps) -> ggml_mul(q_norm) -> ggml_rope_ext(NEOX, all D dims) -> q_out
//   k -> ggml_rms_norm(eps) -> ggml_mul(k_norm) -> ggml_rope_ext(NEOX)     -> ggml_set_rows(k cache)
//   v                                                                       -> ggml_set_rows(v cache)
// Lane l holds elements [l*E, l*E + E) of a D = 32*E vector; the NeoX pair (i, i + D/2) of lanes
// l < 16 sits in lane l + 16 at the same offset, so the rotation is one shuffle.  Arithmetic
// follows ggml's CPU kernels: the row's mean square, then scale = 1/sqrt(mean + eps), x*scale
// and then times the weight (two roundings), the angle of pair i as the position times
// theta_scale^i built by repeated multiplication (theta_scale = theta^(-2/D)), cos/sin of it;
// the cache rows are rounded to F16/BF16 (nearest even) or quantized to Q8_0 blocks (amax/127
// scale stored as f16, values round(x / d)).
#include "fa_prologue.cuh"

#include <cstdlib>

namespace mm3fa {

constexpr int PRO_WARPS = 4;

// Both prologue kernels are launched with programmatic stream serialisation (MM3FA_PDL=0 turns
// it off, as for the attention kernels): their CTAs may start once the previous kernel's CTAs
// have exited, and wait on the device for its completion before reading anything.
__device__ __forceinline__ void prologue_dep_wait() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
}

template <typename Kern, typename Params>
cudaError_t launch_prologue(Kern kern, unsigned blocks, const Params & p, cudaStream_t stream) {
    static const bool pdl = [] {
        const char * e = std::getenv("MM3FA_PDL");
        return !(e && std::atoi(e) == 0);
    }();
    cudaLaunchConfig_t  cfg{};
    cudaLaunchAttribute attr[1];
    cfg.gridDim          = dim3(blocks);
    cfg.blockDim         = dim3(32 * PRO_WARPS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream           = stream;
    cfg.attrs            = attr;
    cfg.numAttrs         = 0;
    if (pdl) {
        attr[0].id                                         = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.numAttrs                                       = 1;
    }
    return cudaLaunchKernelEx(&cfg, kern, p);
}



template <int E>
__global__ void __launch_bounds__(32 * PRO_WARPS) decode_prologue_kernel(const PrologueParams p) {
    const int     lane = threadIdx.x & 31;
    const int     w    = (int) blockIdx.x * PRO_WARPS + (int) (threadIdx.x >> 5);
    const int     per  = p.n_head + 2 * p.n_head_kv;  // vectors per set: q heads, k heads, v heads
    prologue_dep_wait();
    if (w >= per * p.n_set) {
        return;
    }
    const int s = w / per, j = w % per;
    const int kind = j < p.n_head ? 0 : (j < p.n_head + p.n_head_kv ? 1 : 2);  // 0 q, 1 k, 2 v
    const int hh   = kind == 0 ? j : (kind == 1 ? j - p.n_head : j - p.n_head - p.n_head_kv);
    const char * src = kind == 0 ? p.q_in + (int64_t) hh * p.qi_nb1 + (int64_t) s * p.qi_nb2
                     : kind == 1 ? p.k_in + (int64_t) hh * p.ki_nb1 + (int64_t) s * p.ki_nb2
                                 : p.v_in + (int64_t) hh * p.vi_nb1 + (int64_t) s * p.vi_nb2;
    float x[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        x[e] = reinterpret_cast<const float *>(src)[lane * E + e];
    }
    const int64_t r_dst = p.rows[s];
    if (kind == 2) {  // v: conversion only (clamped first with --clamp-fp16, src/qwen3-lm.h:779-782)
        if (p.clamp_v) {
#pragma unroll
            for (int e = 0; e < E; e++) {
                x[e] = x[e] > 65504.0f ? 65504.0f : (x[e] < -65504.0f ? -65504.0f : x[e]);
            }
        }
        if (r_dst >= 0 && r_dst < p.v_rows) {
            char * row = p.v_cache + r_dst * p.vc_nb1 + (int64_t) hh * p.vc_nb2 + (int64_t) s * p.vc_nb3;
            store_cache_row<E>(row, p.kvt, x, lane);
        }
        return;
    }
    float y[E];
    rms_norm_rope_vec<E>(x, y, kind == 0 ? p.q_norm : p.k_norm, p.eps, (float) p.pos[s], p.theta_scale, lane);
    if (kind == 0) {
        float * dst = reinterpret_cast<float *>(p.q_out + (int64_t) hh * p.qo_nb1 + (int64_t) s * p.qo_nb2);
#pragma unroll
        for (int e = 0; e < E; e++) {
            dst[lane * E + e] = y[e];
        }
        return;
    }
    if (r_dst >= 0 && r_dst < p.k_rows) {
        char * row = p.k_cache + r_dst * p.kc_nb1 + (int64_t) hh * p.kc_nb2 + (int64_t) s * p.kc_nb3;
        store_cache_row<E>(row, p.kvt, y, lane);
    }
}

// ---- DiT attention prologue (src/dit.h:201-220): per (batch, token, head) the q and k vectors
// get ggml_rope_ext NEOX over their first `rot` dims (pair i with i + rot/2, angle pos[token] *
// theta_scale^i walked like ggml's rope cache, dims from rot on copied), q stays F32, k and v are
// cast (round to nearest even) into the [D, S, H, B] layout the attention reads.
template <int E>
__global__ void __launch_bounds__(32 * PRO_WARPS) dit_prologue_kernel(const DitPrologueParams p) {
    const int     lane = threadIdx.x & 31;
    const int64_t w    = (int64_t) blockIdx.x * PRO_WARPS + (threadIdx.x >> 5);
    const int64_t nv   = (int64_t) p.n_head * p.n_tok * p.n_batch;
    prologue_dep_wait();
    if (w >= 3 * nv) {
        return;
    }
    const int     kind = (int) (w / nv);  // 0 q, 1 k, 2 v
    const int64_t u    = w % nv;
    const int     hh   = (int) (u % p.n_head);
    const int     t    = (int) ((u / p.n_head) % p.n_tok);
    const int     b    = (int) (u / ((int64_t) p.n_head * p.n_tok));
    const int64_t * si = kind == 0 ? p.sq_in : (kind == 1 ? p.sk_in : p.sv_in);
    const int64_t * so = kind == 0 ? p.sq_out : (kind == 1 ? p.sk_out : p.sv_out);
    const char *  src  = (kind == 0 ? p.q_in : (kind == 1 ? p.k_in : p.v_in)) + hh * si[0] + t * si[1] + b * si[2];
    char *        dst  = (kind == 0 ? p.q_out : (kind == 1 ? p.k_out : p.v_out)) + hh * so[0] + t * so[1] + b * so[2];
    float         x[E];
#pragma unroll
    for (int e = 0; e < E; e++) {
        x[e] = reinterpret_cast<const float *>(src)[lane * E + e];
    }
    if (kind < 2) {
        // lanes [0, hl) hold the first halves of the rotated pairs, lanes [hl, 2 hl) the second
        const int hl      = p.rot / (2 * E);
        const int partner = lane < hl ? lane + hl : (lane < 2 * hl ? lane - hl : lane);
        const int pi0     = (lane < hl ? lane : lane - hl) * E;  // first pair index of this lane
        float     th      = (float) p.pos[t];
        for (int k = 0; k < pi0 && lane < 2 * hl; k++) {
            th *= p.theta_scale;
        }
#pragma unroll
        for (int e = 0; e < E; e++) {
            const float xo = __shfl_sync(0xffffffffu, x[e], partner);
            if (lane < 2 * hl) {
                const float c = cosf(th), sn = sinf(th);
                x[e]          = lane < hl ? x[e] * c - xo * sn : xo * sn + x[e] * c;
                th *= p.theta_scale;
            }
        }
    }
    if (kind == 0) {
#pragma unroll
        for (int e = 0; e < E; e++) {
            reinterpret_cast<float *>(dst)[lane * E + e] = x[e];
        }
        return;
    }
    store_cache_row<E>(dst, p.kvt, x, lane);
}

cudaError_t launch_dit_prologue(const DitPrologueParams & p, int D, cudaStream_t stream) {
    const int64_t warps  = 3 * (int64_t) p.n_head * p.n_tok * p.n_batch;
    const int64_t blocks = (warps + PRO_WARPS - 1) / PRO_WARPS;
    if (blocks <= 0) {
        return cudaSuccess;
    }
    if (blocks > 0x7fffffff) {
        return cudaErrorInvalidValue;
    }
    switch (D) {
        case 64:
            return launch_prologue(dit_prologue_kernel<2>, (unsigned) blocks, p, stream);
        case 128:
            return launch_prologue(dit_prologue_kernel<4>, (unsigned) blocks, p, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

cudaError_t launch_decode_prologue(const PrologueParams & p, int D, cudaStream_t stream) {
    const int64_t warps  = (int64_t) p.n_set * (p.n_head + 2 * p.n_head_kv);
    const int64_t blocks = (warps + PRO_WARPS - 1) / PRO_WARPS;
    if (blocks <= 0) {
        return cudaSuccess;
    }
    switch (D) {
        case 64:
            return launch_prologue(decode_prologue_kernel<2>, (unsigned) blocks, p, stream);
        case 128:
            return launch_prologue(decode_prologue_kernel<4>, (unsigned) blocks, p, stream);
        case 256:
            return launch_prologue(decode_prologue_kernel<8>, (unsigned) blocks, p, stream);
        default:
            return cudaErrorInvalidValue;
    }
}

}  // namespace mm3fa
