/*
 * mm3fa.h - C ABI of the B200 (sm_100a) flash-attention operator for minimaxmusic.cpp.
 *
 * The operator is ggml's GGML_OP_FLASH_ATTN_EXT as the reference builds it with
 *     ggml_flash_attn_ext(ctx, q, k, v, mask, scale, max_bias, logit_softcap)
 *     ggml_flash_attn_ext_set_prec(result, GGML_PREC_F32)
 * at src/qwen3-lm.h:432-436 (prefill), src/qwen3-lm.h:816-820 (batched CFG decode) and
 * src/dit.h:218-222 (DiT).  Those three graph nodes are computed by whichever ggml backend
 * src/static-graph.h:54-57 dispatches to (ggml_backend_graph_compute or the scheduler);
 * this library replaces the device computation of that node.
 *
 * Tensor convention (ggml): ne[0] is the innermost (contiguous-element) dimension and nb[i]
 * is the byte stride of dimension i.  For Q8_0, ne[0] counts elements and nb[1] is the byte
 * size of one row of ne[0]/32 blocks of 34 bytes.
 *
 *   q    [D,  n_q,  n_head,    n_seq ]   F32 (F16/BF16 accepted)
 *   k    [D,  n_kv, n_head_kv, n_seq_k]  F16, BF16, Q8_0 or F32 (may be a strided view of a cache;
 *                                         F32 K/V - the depth decoder's F32 attention - run on
 *                                         the CUDA-core decode kernel)
 *   v    [Dv, n_kv, n_head_kv, n_seq_k]  same type family as k
 *   mask [n_kv, >=n_q, m2, m3] F16 or NULL; broadcast over heads (h % m2) and sequences (s % m3)
 *   dst  [Dv, n_head, n_q, n_seq] F32 -- heads BEFORE query rows, exactly as ggml's result
 *
 * GQA: query head h reads kv head h / (n_head / n_head_kv); query sequence s reads kv
 * sequence s / (n_seq / n_seq_k).
 *
 * All entry points are host functions.  None of them allocates device memory or
 * synchronises the host with the device; work is enqueued on the caller's stream,
 * so a call can be captured into a CUDA graph once its shape is fixed.
 */
#ifndef MM3FA_H
#define MM3FA_H

#include <stddef.h>
#include <stdint.h>

#if defined(_WIN32)
#    define MM3FA_API __declspec(dllexport)
#else
#    define MM3FA_API __attribute__((visibility("default")))
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ggml_type enum values used by the operator (ggml.h numbering). */
enum mm3fa_type {
    MM3FA_TYPE_F32  = 0,
    MM3FA_TYPE_F16  = 1,
    MM3FA_TYPE_Q8_0 = 8,
    MM3FA_TYPE_BF16 = 30,
};

/* ggml_prec values accepted by the prec argument (ggml_flash_attn_ext_set_prec). */
enum mm3fa_prec {
    MM3FA_PREC_DEFAULT = 0,
    MM3FA_PREC_F32     = 10,
};

/* Status codes.  The reference ignores ggml_status (src/qwen3-lm.h:620,921; src/dit.h:385);
 * this ABI reports every rejected input instead of asserting. */
enum mm3fa_status {
    MM3FA_OK              = 0,
    MM3FA_ERR_NULL        = 1,  /* a required tensor or data pointer is NULL           */
    MM3FA_ERR_TYPE        = 2,  /* unsupported tensor type                               */
    MM3FA_ERR_SHAPE       = 3,  /* shapes are inconsistent with the operator contract    */
    MM3FA_ERR_STRIDE      = 4,  /* a stride is not a multiple of the element/row size    */
    MM3FA_ERR_ALIGN       = 5,  /* data pointer not aligned to its element size          */
    MM3FA_ERR_WORKSPACE   = 6,  /* workspace missing or smaller than mm3fa_workspace_size */
    MM3FA_ERR_CUDA        = 7,  /* a CUDA launch failed (see mm3fa_last_cuda_error)       */
    MM3FA_ERR_UNSUPPORTED = 8,  /* valid op, but no kernel here handles this shape       */
    MM3FA_ERR_TIMEOUT     = 9,  /* a bounded device-side wait expired                     */
    MM3FA_ERR_DEVICE      = 10, /* current device is not an sm_100 part                   */
    MM3FA_ERR_SCRATCH_LIMIT = 11, /* needs more scratch than MM3FA_NOALLOC_SCRATCH_BYTES  */
    MM3FA_ERR_COMM        = 12, /* NCCL missing, or a collective / IPC call failed        */
};

/* Size of the fixed device scratch buffer behind mm3fa_flash_attn_ext_noalloc (8 MiB). */
#define MM3FA_NOALLOC_SCRATCH_BYTES (8u << 20)

/* One ggml tensor as the operator sees it (a plain view of struct ggml_tensor's
 * type / ne / nb / data fields). */
typedef struct mm3fa_tensor {
    int32_t  type;  /* enum mm3fa_type */
    int32_t  reserved;
    int64_t  ne[4];
    uint64_t nb[4]; /* bytes */
    void *   data;  /* device pointer */
} mm3fa_tensor;

/*
 * Computes dst = softmax(scale * q k^T [softcap] + slope_h * mask) v for every query row.
 *   scale          softmax scale (the reference passes 1/sqrt(D))
 *   max_bias       ALiBi maximum bias; 0 disables ALiBi (slope 1)
 *   logit_softcap  0 disables; otherwise s <- softcap * tanh(s / softcap) before the mask
 *   prec           MM3FA_PREC_DEFAULT or MM3FA_PREC_F32; accumulation is always F32
 *   workspace      device scratch of at least mm3fa_workspace_size(...) bytes, or NULL when
 *                  that size is 0.  Zero-fill it once after allocating it (cudaMemset); every
 *                  successful call leaves its status word and arrival counters zero again, so
 *                  the workspace can be reused and graph-replayed.  Calls that may run
 *                  concurrently (different streams) need different workspaces.
 *   stream         cudaStream_t (NULL = legacy default stream)
 * Rows whose every score is -inf produce zeros.
 * Replaces: the ggml-cuda compute of GGML_OP_FLASH_ATTN_EXT reached from
 *           src/static-graph.h:54-57 for the nodes built at src/qwen3-lm.h:432, :817 and
 *           src/dit.h:221.
 */
MM3FA_API int mm3fa_flash_attn_ext(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                         const mm3fa_tensor * mask, float scale, float max_bias, float logit_softcap, int prec,
                         mm3fa_tensor * dst, void * workspace, size_t workspace_bytes, void * stream);

/*
 * mm3fa_flash_attn_ext with the key range of each query sequence given on the device:
 * q sequence s sees keys [0, kv_len[s]) (clamped to [0, n_kv]); keys past it count as -inf, on
 * top of `mask` (which may be NULL).  kv_len: device int32 [n_seq].  Equal to passing the mask
 * the reference builds on the host every decode step (0 below kv_pos + 1, -inf from it on,
 * src/qwen3-lm.h:909-920), without building or copying it; with the cluster split (the CFG
 * decode shapes) the keys past kv_len are not read at all.  Uses the decode kernels for any
 * number of query rows; same workspace as mm3fa_flash_attn_ext.
 * Replaces: the host mask loop and its upload at src/qwen3-lm.h:909-920, and the attention node.
 */
MM3FA_API int mm3fa_flash_attn_ext_kvlen(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                         const mm3fa_tensor * mask, const int32_t * kv_len, float scale,
                                         float max_bias, float logit_softcap, int prec, mm3fa_tensor * dst,
                                         void * workspace, size_t workspace_bytes, void * stream);

/*
 * mm3fa_flash_attn_ext for callers that cannot allocate device memory: the same computation,
 * but the split-KV scratch comes from a buffer of MM3FA_NOALLOC_SCRATCH_BYTES built into the
 * library (one per GPU that loads it, held until the process exits) instead of a workspace
 * argument.  For hosts that may not call cudaMalloc where attention runs - a ggml backend whose
 * buffers were all planned ahead, a graph-recording engine, a plugin without an allocator.
 * Inputs and outputs are still the caller's.
 *   - Returns MM3FA_ERR_SCRATCH_LIMIT, enqueuing nothing, when the operands need more scratch
 *     than the buffer holds (mm3fa_workspace_size > MM3FA_NOALLOC_SCRATCH_BYTES).
 *   - The first call on a device looks up the buffer's device address (cudaGetSymbolAddress)
 *     with that device current; make that first call before any stream capture.  The address
 *     is cached per device and CUDA context; after cudaDeviceReset the next call looks it up
 *     again (so again outside capture).
 *   - Each call clears the arrival counters its operands use on `stream` and allocates
 *     nothing.  The status word is not cleared: a bounded device wait that expired inside a
 *     call stays recorded until mm3fa_noalloc_status reads it.  All calls on a device share the
 *     buffer: calls that can overlap on the GPU (unordered streams) race.
 * Replaces: nothing - it has no counterpart in the reference.
 */
MM3FA_API int mm3fa_flash_attn_ext_noalloc(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                           const mm3fa_tensor * mask, float scale, float max_bias,
                                           float logit_softcap, int prec, mm3fa_tensor * dst, void * stream);

/*
 * mm3fa_workspace_status for the built-in buffer of mm3fa_flash_attn_ext_noalloc on the current
 * device: MM3FA_OK, or MM3FA_ERR_TIMEOUT (status cleared) when a bounded wait of an earlier
 * no-allocation call expired; *status_out gets the raw bits.  Synchronises `stream`.
 * Replaces: nothing - it has no counterpart in the reference.
 */
MM3FA_API int mm3fa_noalloc_status(void * stream, uint32_t * status_out);

/*
 * mm3fa_selftest_bounded_wait on the built-in buffer of mm3fa_flash_attn_ext_noalloc: a wait that
 * nothing satisfies expires after timeout_us and is recorded in that buffer's status word, so
 * that tests can check mm3fa_noalloc_status without faulting or hanging the GPU.
 * Replaces: nothing - it has no counterpart in the reference.
 */
MM3FA_API int mm3fa_noalloc_selftest_bounded_wait(uint32_t timeout_us, void * stream);

/*
 * Bytes of device workspace mm3fa_flash_attn_ext needs for these operands on the current
 * device (0 if none).  Depends on shapes and types only, never on data pointers.
 * Replaces: the compute-buffer sizing ggml_gallocr / ggml_backend_sched do for the node
 *           (src/static-graph.h:31-52).
 */
MM3FA_API size_t mm3fa_workspace_size(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                            const mm3fa_tensor * mask, const mm3fa_tensor * dst);

/*
 * Returns MM3FA_OK when mm3fa_flash_attn_ext would accept these operands, otherwise the
 * status it would return.  Pure host check; data pointers are not dereferenced.
 * Replaces: ggml_backend_supports_op for the node (src/static-graph.h:12-19).
 */
MM3FA_API int mm3fa_supports(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                   const mm3fa_tensor * mask, float max_bias, float logit_softcap, const mm3fa_tensor * dst);

/*
 * Reads (and clears) the device status word of a workspace: MM3FA_OK, or MM3FA_ERR_TIMEOUT
 * when a bounded device-side wait of an earlier call on it expired (*status_out gets the raw
 * bits).  After a timeout the workspace must be zero-filled again before reuse.  This call
 * synchronises `stream`.
 * Replaces: the ggml_status the reference ignores (src/qwen3-lm.h:620,921; src/dit.h:385).
 */
MM3FA_API int mm3fa_workspace_status(void * workspace, void * stream, uint32_t * status_out);

/*
 * Diagnostics: launches one CTA that waits on an mbarrier nothing arrives on, bounded by
 * timeout_us, and records the expiry in the workspace status word exactly as the attention
 * kernels do.  Lets tests check the timeout path without faulting or hanging the GPU.
 * Replaces: nothing in the reference (it has no device-side failure detection).
 */
MM3FA_API int mm3fa_selftest_bounded_wait(void * workspace, uint32_t timeout_us, void * stream);

/* Human-readable name of a status code (static storage). */
MM3FA_API const char * mm3fa_status_string(int status);

/* Message of the last CUDA error seen by this thread's calls ("" if none). */
MM3FA_API const char * mm3fa_last_cuda_error(void);

/* ABI version: (major << 16) | minor. */
MM3FA_API int mm3fa_version(void);

/*
 * Fused decode prologue of one LM layer: the nodes the reference builds between the QKV
 * projection and the attention call, for N sets (CFG sequences) of one decode step:
 *   q_out        = rope_neox(rms_norm(q_in) * q_norm, pos[s])
 *   k_cache[s]   row rows[s] = rope_neox(rms_norm(k_in) * k_norm, pos[s])
 *   v_cache[s]   row rows[s] = v_in
 * rms_norm over dim 0 with eps; NeoX RoPE over all D dims with base rope_theta (freq_scale 1,
 * no YaRN); the cache rows are converted like ggml_set_rows (F32 -> F16/BF16 round to
 * nearest even, or Q8_0 blocks).  The attention call that follows reads q_out as
 * [D, 1, n_head, N] and the caches as its K/V views.
 *   q_in     F32 [D, n_head, N], k_in/v_in F32 [D, n_head_kv, N]   (nb[0] = 4)
 *   q_norm, k_norm   device F32 [D];  eps  the model's rms_norm_eps
 *   pos      device int32 [N]: RoPE position of set s
 *   rows     device int64 [N]: destination row of set s (rows outside [0, ne[1]) are not written)
 *   k_cache, v_cache [D, max_seq, n_head_kv, N] views of the cache slices of the N sets,
 *            F16, BF16 or Q8_0 (both the same type)
 *   q_out    F32 [D, n_head, N]
 * D = 64, 128 or 256.
 * Replaces: ggml_rms_norm, ggml_mul, ggml_rope_ext, ggml_cont and ggml_set_rows at
 *           src/qwen3-lm.h:764-800 (computed by the backend at src/static-graph.h:54-57).
 */
MM3FA_API int mm3fa_decode_prologue(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                                    const float * q_norm, const float * k_norm, float eps, const int32_t * pos,
                                    float rope_theta, const int64_t * rows, mm3fa_tensor * k_cache,
                                    mm3fa_tensor * v_cache, mm3fa_tensor * q_out, void * stream);

/*
 * Decode step of one LM layer as one call: mm3fa_decode_prologue followed by
 * mm3fa_flash_attn_ext with the query q_out viewed as [D, 1, n_head, N] (outputs: q_out, the
 * appended cache rows, dst).  The prologue arguments are those of mm3fa_decode_prologue; k, v,
 * mask, scale, max_bias, logit_softcap, prec, dst, workspace and stream those of
 * mm3fa_flash_attn_ext (k and v the attention's views of the caches; the workspace is sized by
 * mm3fa_workspace_size with q_out's view).  Every operand is checked before anything is
 * launched.  The two kernels are launched with programmatic stream serialisation, so the
 * attention's CTAs start as the prologue's exit.
 * No counterpart in the reference as one function: it replaces the nodes listed for
 * mm3fa_decode_prologue plus ggml_flash_attn_ext at src/qwen3-lm.h:816-820.
 */
MM3FA_API int mm3fa_decode_step(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                                const float * q_norm, const float * k_norm, float eps, const int32_t * pos,
                                float rope_theta, const int64_t * rows, mm3fa_tensor * k_cache,
                                mm3fa_tensor * v_cache, mm3fa_tensor * q_out, const mm3fa_tensor * k,
                                const mm3fa_tensor * v, const mm3fa_tensor * mask, float scale, float max_bias,
                                float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                                size_t workspace_bytes, void * stream);

/* Flags of mm3fa_decode_prologue_ex / mm3fa_decode_step_ex. */
enum mm3fa_prologue_flags {
    /* v is clamped to [-65504, 65504] before its conversion to the cache type (NaN passes
     * through): the ggml_clamp the reference inserts with --clamp-fp16 (src/qwen3-lm.h:779-782) */
    MM3FA_PROLOGUE_CLAMP_FP16 = 1,
};

/*
 * mm3fa_decode_prologue / mm3fa_decode_step with flags (enum mm3fa_prologue_flags; unknown bits
 * return MM3FA_ERR_UNSUPPORTED).  The plain entry points are these with flags = 0.
 * Replaces: as mm3fa_decode_prologue / mm3fa_decode_step, plus the ggml_clamp node of
 *           src/qwen3-lm.h:779-782 when MM3FA_PROLOGUE_CLAMP_FP16 is set.
 */
MM3FA_API int mm3fa_decode_prologue_ex(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in,
                                       const mm3fa_tensor * v_in, const float * q_norm, const float * k_norm,
                                       float eps, const int32_t * pos, float rope_theta, const int64_t * rows,
                                       mm3fa_tensor * k_cache, mm3fa_tensor * v_cache, mm3fa_tensor * q_out,
                                       uint32_t flags, void * stream);
MM3FA_API int mm3fa_decode_step_ex(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                                   const float * q_norm, const float * k_norm, float eps, const int32_t * pos,
                                   float rope_theta, const int64_t * rows, mm3fa_tensor * k_cache,
                                   mm3fa_tensor * v_cache, mm3fa_tensor * q_out, const mm3fa_tensor * k,
                                   const mm3fa_tensor * v, const mm3fa_tensor * mask, float scale, float max_bias,
                                   float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                                   size_t workspace_bytes, uint32_t flags, void * stream);

/*
 * DiT attention prologue: the nodes between the QKV projection and the attention call of a
 * DiT block, as one kernel (src/dit.h:201-220):
 *   q_out = rope_neox(q_in, pos, rot_dims)          (F32, same [D, n_head, S, B] layout)
 *   k_out = cast(rope_neox(k_in, pos, rot_dims))    ([D, S, n_head, B], F16 or BF16)
 *   v_out = cast(v_in)                              ([D, S, n_head, B], same type as k_out)
 * NeoX RoPE over the first rot_dims dims of each head (base rope_theta, freq_scale 1, no YaRN;
 * dims from rot_dims on unchanged), casts round to nearest even.  The attention then takes q_out
 * permuted to [D, S, n_head, B] (a view) and k_out / v_out.
 *   q_in, k_in, v_in  F32 [D, n_head, S, B]  (nb[0] = 4)
 *   pos      device int32 [S]: the position of each token
 *   rot_dims even, 0 < rot_dims <= D, a multiple of D/16
 * D = 64 or 128.
 * Replaces: ggml_rope_ext (x2), ggml_permute and ggml_cast (x2) at src/dit.h:206-220.
 */
MM3FA_API int mm3fa_dit_prologue(const mm3fa_tensor * q_in, const mm3fa_tensor * k_in, const mm3fa_tensor * v_in,
                                 const int32_t * pos, int rot_dims, float rope_theta, mm3fa_tensor * q_out,
                                 mm3fa_tensor * k_out, mm3fa_tensor * v_out, void * stream);

/*
 * Multi-GPU output assembly.  With the kv heads partitioned over G ranks, rank r computes
 * dst_r [Dv, n_head/G, n_q, n_seq] for query heads [r*n_head/G, (r+1)*n_head/G).  After an
 * all-gather (NCCL, by the caller) the blocks sit rank-major as gathered[G][n_seq][n_q]
 * [n_head/G][Dv]; this kernel permutes them into the ggml result [Dv, n_head, n_q, n_seq].
 * Both buffers are contiguous F32 device memory and must not overlap.
 * Replaces: nothing in the reference (single device); it is the exchange step of the
 *           head-sharded layout fed to the o_proj at src/qwen3-lm.h:823-827.
 */
MM3FA_API int mm3fa_assemble_heads(const float * gathered, float * dst, int64_t dv, int64_t n_head, int64_t n_q,
                         int64_t n_seq, int n_ranks, void * stream);

/* ------------------------------------------------------------------------------------------
 * Multi-GPU head exchange.  With the kv heads (decode, prefill) or the (sequence, head) units
 * (DiT) partitioned over G ranks, one process per GPU, each rank computes a slice of the ggml
 * result [Dv, n_head, n_q, n_seq]; the o_proj / to_out that follows the attention needs every
 * head of its rows, so the slices are exchanged after every attention call.  Two forms:
 *   - mm3fa_allgather_heads: one NCCL all-gather (the caller's communicator) + a permute;
 *   - mm3fa_flash_attn_ext_peers + mm3fa_peer_wait: the decode kernel stores its result rows
 *     straight into every rank's result buffer over NVLink (CUDA IPC mappings) and signals a
 *     counter, and the consumer waits for the counter on the device (bounded).
 * ------------------------------------------------------------------------------------------ */

/* Most ranks a head exchange spans (one node). */
#define MM3FA_MAX_RANKS 8

/*
 * All-gathers the result slices of G ranks over a NCCL communicator and writes the whole ggml
 * result on every rank.  The ranks split the sequences into seq_split groups and the heads into
 * G / seq_split groups; rank r = (sequence group) * (G / seq_split) + (head group) holds
 *   slice     F32 contiguous [Dv, n_head*seq_split/G, n_q, n_seq/seq_split]: its sequences'
 *             rows for its heads (the decode kernel's dst when it runs on the rank's shard)
 * and gets
 *   dst       F32 contiguous [Dv, n_head, n_q, n_seq] (may not overlap slice unless slice ==
 *             gathered + r * slice elements, the in-place form)
 *   gathered  F32 scratch of G slices, or NULL when the gathered order is already ggml's (each
 *             rank holds whole sequences: G / seq_split == 1; or a single row: n_q * n_seq /
 *             seq_split == 1 with seq_split == 1); then NCCL writes dst directly.
 * KV-head sharding of the LM is seq_split = 1; (batch x head) sharding of the DiT with G <= B is
 * seq_split = G, with G > B seq_split = B.  nccl_comm is an ncclComm_t of G ranks (e.g. from
 * ncclCommInitRank, or the one torch.distributed made); the library loads libnccl.so.2 at the
 * first call (the copy already in the process when there is one).
 * Replaces: nothing in the reference (one device): the exchange that turns the sharded attention
 *           into the [n_head*Dv, n_q, n_seq] input of the o_proj at src/qwen3-lm.h:823-827 (and
 *           of to_out after src/dit.h:221-226).
 */
MM3FA_API int mm3fa_allgather_heads(const float * slice, float * gathered, float * dst, int64_t dv, int64_t n_head,
                                    int64_t n_q, int64_t n_seq, int seq_split, void * nccl_comm, void * stream);

/* Every rank's receive buffer as mapped into this process (see mm3fa_ipc_open).  Slot s of a
 * receive buffer (recv_slot_bytes from s * recv_slot_bytes on) holds two halves, selected by the
 * parity of the call's epoch, of n_ranks source regions of 8 * V bytes each, V = the values of one
 * rank's result slice; a value is the 8-byte word {float bits, epoch}.  Zero-fill the buffers
 * once, before the first call. */
typedef struct mm3fa_peers {
    int32_t  n_ranks;                 /* G, 2 .. MM3FA_MAX_RANKS */
    int32_t  rank;                    /* this process's rank */
    void *   recv[MM3FA_MAX_RANKS];   /* rank i's receive buffer (16-byte aligned); recv[rank] is ours */
    uint64_t recv_slot_bytes;         /* >= 2 * n_ranks * 8 * V, a multiple of 16 */
} mm3fa_peers;

/*
 * mm3fa_flash_attn_ext on this rank's shard, with the head exchange fused into the kernel: dst is
 * this rank's slice of the result (e.g. heads [r*H/G, (r+1)*H/G) of [Dv, H, n_q, n_seq], as a view
 * of this rank's whole result buffer), and every result value is also stored, while other CTAs
 * still compute, into each other rank's receive buffer (slot `slot`, this rank's source region)
 * as {value, epoch} with epoch = epochs[slot] + 1 - plain volatile stores over NVLink, no fences,
 * no flags.  epochs: device u32 per slot, zeroed once, private to this rank, advanced only by
 * mm3fa_peer_wait.  kv_len may be NULL (as mm3fa_flash_attn_ext) or a device array (as _kvlen).
 * Only the tensor-core decode kernel's cluster split carries the exchange (<= 16 query rows per
 * (sequence, kv head), F16/BF16/Q8_0 caches it can stream, 16-byte aligned contiguous rows):
 * other shapes return MM3FA_ERR_UNSUPPORTED and enqueue nothing, as does max_bias != 0 (ALiBi
 * slopes follow the global head index, which a shard's descriptors do not carry; the reference
 * passes 0).  Peer memory is only ever written; nothing loads from it.
 * Replaces: the attention node of src/qwen3-lm.h:816-820 plus its exchange (see above).
 */
MM3FA_API int mm3fa_flash_attn_ext_peers(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                         const mm3fa_tensor * mask, const int32_t * kv_len, float scale,
                                         float max_bias, float logit_softcap, int prec, mm3fa_tensor * dst,
                                         void * workspace, size_t workspace_bytes, const mm3fa_peers * peers,
                                         int slot, const uint32_t * epochs, void * stream);

/*
 * The consumer's side of the fused exchange, enqueued on `stream` after this rank's
 * mm3fa_flash_attn_ext_peers call on `slot`: waits on the device until every other rank's values
 * of that call (epoch epochs[slot] + 1) are in this rank's receive buffer, writes them into
 * `result` - this rank's whole result [Dv, n_head, n_q, n_seq] F32, rank i's slice being heads
 * [i*n_head/G, (i+1)*n_head/G) - and advances epochs[slot].  Kernels enqueued after it read the
 * whole result.  It lets the next kernel in the stream launch as soon as it starts (programmatic
 * dependent launch): a kernel launched with programmatic stream serialisation reads the result
 * only after its own griddepcontrol.wait (cudaGridDependencySynchronize), as programmatic
 * launch requires; other kernels are ordered as usual.  Each wait is bounded
 * (MM3FA_WAIT_TIMEOUT_MS, 2 s by default); on expiry it sets
 * the workspace status word (mm3fa_workspace_status reports MM3FA_ERR_TIMEOUT) and returns.
 * Replaces: nothing in the reference (see above).
 */
MM3FA_API int mm3fa_peer_wait(const mm3fa_peers * peers, int slot, uint32_t * epochs, mm3fa_tensor * result,
                              void * workspace, void * stream);

/*
 * Dense attention (causal prefill, DiT) on this rank's shard with the exchange of the result fused
 * into the kernel: computes exactly what mm3fa_flash_attn_ext computes into dst, and stores every
 * finished result row, at the same byte offset, into each other rank's whole result as well (the
 * row leaves from the epilogue with plain 16-byte stores over NVLink while later tiles are still
 * computed; no permute, no collective library).
 *   results->recv[r]       base of rank r's whole result buffer for this call (the caller's own
 *                          at r = rank; the others mapped with mm3fa_ipc_open), each
 *                          results->recv_slot_bytes long
 *   dst                    this rank's slice: a view inside recv[rank] (e.g. its heads of the
 *                          [Dv, n_head, n_q, n_seq] result, or its sequences)
 * The other ranks' rows are complete only after mm3fa_gather_signal_wait on every rank.  A rank
 * may write into a buffer that another rank is still reading, so the caller alternates at least
 * two result buffers (slots) between calls, each followed by its mm3fa_gather_signal_wait.
 * Only for operands that take the tensor-core prefill/DiT kernel (many query rows, keys present,
 * dst rows 16-byte aligned, strides that its TMA store takes); other shapes and max_bias != 0
 * return MM3FA_ERR_UNSUPPORTED and enqueue nothing.
 * Replaces: the attention node of src/qwen3-lm.h:432-436 (prefill) or src/dit.h:218-222 (DiT) plus
 *           the all-gather of the head-concatenated result that a sharded run needs before the
 *           output projection (src/qwen3-lm.h:439, src/dit.h:226); the reference runs on one GPU.
 */
MM3FA_API int mm3fa_flash_attn_ext_gather(const mm3fa_tensor * q, const mm3fa_tensor * k, const mm3fa_tensor * v,
                                          const mm3fa_tensor * mask, float scale, float max_bias,
                                          float logit_softcap, int prec, mm3fa_tensor * dst, void * workspace,
                                          size_t workspace_bytes, const mm3fa_peers * results, void * stream);

/*
 * Completion of the exchange of mm3fa_flash_attn_ext_gather, enqueued on `stream` after this rank's
 * call: publishes this rank's rows to every other rank (a system-scope fence, then the call's
 * epoch - epochs[slot] + 1 - stored into each rank's flag word [slot][this rank]) and waits on the
 * device until every other rank's epoch is in this rank's words [slot][*]; then advances
 * epochs[slot].  Kernels enqueued after it read the whole result.
 *   flags->recv[r]          rank r's flag array: uint32 [n_slots][n_ranks], zero-filled before the
 *                           first call, mapped like the results; recv_slot_bytes = its size
 *   epochs                  this rank's device uint32 [n_slots], zero-filled before the first call
 * Every rank calls it with the same slot sequence.  The wait is bounded (MM3FA_WAIT_TIMEOUT_MS);
 * on expiry the workspace status word reports MM3FA_ERR_TIMEOUT.
 * Replaces: nothing in the reference (see above).
 */
MM3FA_API int mm3fa_gather_signal_wait(const mm3fa_peers * flags, int slot, uint32_t * epochs, void * workspace,
                                       void * stream);

/* CUDA IPC handle of a device buffer: the allocation's handle plus the buffer's offset in it. */
typedef struct mm3fa_ipc_handle {
    unsigned char handle[64];
    uint64_t      offset;
} mm3fa_ipc_handle;

/*
 * Host helpers for building mm3fa_peers across processes: mm3fa_ipc_export fills a handle for a
 * device buffer (cudaIpcGetMemHandle of the allocation that holds it); the caller moves the
 * handles between its processes by any means; mm3fa_ipc_open maps another process's buffer into
 * this one (cudaIpcOpenMemHandle, peer access enabled) and mm3fa_ipc_close unmaps it.
 * Replaces: nothing in the reference (see above).
 */
MM3FA_API int mm3fa_ipc_export(const void * dev_ptr, mm3fa_ipc_handle * out);
MM3FA_API int mm3fa_ipc_open(const mm3fa_ipc_handle * h, void ** dev_ptr_out);
MM3FA_API int mm3fa_ipc_close(void * dev_ptr);

#ifdef __cplusplus
}
#endif

#endif /* MM3FA_H */
