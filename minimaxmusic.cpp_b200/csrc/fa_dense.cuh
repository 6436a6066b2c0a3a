// fa_dense.cuh - host interface of the tensor-core (tcgen05) flash-attention kernel for many
// query rows (fa_dense_sm100.cu): LM prefill and DiT attention.
#pragma once

#include "fa_common.cuh"

#include <cuda_runtime.h>

namespace mm3fa {

// Class of one 128 x 128 (query, key) block of a mask plane.
enum : uint8_t { BLK_NONE = 0, BLK_MIXED = 1, BLK_SKIP = 2 };
// Flag bits of a block as the mask pre-pass records them: some entry is not -inf / not zero.
enum : uint32_t { BLKF_FINITE = 1u, BLKF_NONZERO = 2u };

struct DenseParams {
    const char * q;
    const char * k;
    const char * v;
    const char * mask;  // F16, may be null
    char *       dst;
    int64_t      q_nb1, q_nb2, q_nb3;
    int64_t      k_nb1, k_nb2, k_nb3;
    int64_t      v_nb1, v_nb2, v_nb3;
    int64_t      m_nb1, m_nb2, m_nb3;
    int64_t      d_nb1, d_nb2, d_nb3;
    int          q_type;
    int          q_vec;     // Q rows start 16-byte aligned: 16-byte loads
    int          dst_vec;   // dst rows start 16-byte aligned: 16-byte stores
    int          mask_vec;  // mask rows start 16-byte aligned: 16-byte loads
    int          tma_store; // the result is written by TMA (tensor map argument valid)
    int          n_q, n_kv;
    int          n_head, n_seq;
    int          n_regular;       // CTAs with a whole work item; the rest come in split pairs
    int          ratio;     // n_head / n_head_kv
    int          rk3;       // n_seq / n_seq_k
    int          m_ne2, m_ne3;
    float        scale, softcap, max_bias, m0, m1;
    int          n_head_log2;
    int          n_qt, n_kt;              // query blocks (256 rows, or 128 with pair), 128-key tiles
    // head pair mode (GQA with a mask shared by all heads): a work item is 128 query rows of two
    // query heads of one kv group, Q tile t holding head 2 hp + t - both tiles see the same
    // causal extent and share every K/V tile; otherwise 256 rows of one head (tile t = rows
    // 128 t ..)
    int          pair;
    // fused head exchange (TMA-store epilogue only): each finished result row is also stored at
    // the same byte offset from its dst address plus peer_off[i] - the same position in the other
    // ranks' whole results, mapped by CUDA IPC - with 16-byte stores (no fence: the exchange's
    // signal kernel, after this one in the stream, publishes the rows)
    int          n_peers;
    int64_t      peer_off[7];
    const uint32_t * blocks;              // [plane][n_qt][n_kt] block flags (BLKF_*), null without mask
    // [plane][row][3]: max(n_kv - first -inf column), max(last zero column + 1), any other value;
    // a row is a step row (zeros, then -inf from column lim = n_kv - [0] on) when [2] == 0 and
    // [0] + [1] <= n_kv.  Null without mask.
    const int *  rowinfo;
    uint32_t *   status;
    uint64_t     timeout_ns;
};

// F16/BF16 K and V, D = DV = 64 or 128, TMA-expressible strides.
bool        dense_eligible(int D, int kvt);
// Workspace bytes: status word, the mask block classes and the per-row mask summaries.
size_t      dense_workspace_bytes(int64_t n_q, int64_t n_kv, int64_t planes);
cudaError_t launch_dense(DenseParams p, int D, int kvt, int64_t n_head_kv, int64_t n_seq_k, int64_t n_head,
                         int64_t n_seq, void * workspace, cudaStream_t stream);

}  // namespace mm3fa
