"""KV-head sharding of GGML_OP_FLASH_ATTN_EXT over G GPUs (one process per GPU).

The reference runs on one device (src/backend.h:123).  Across G GPUs the op shards
without any exchange inside it: rank r owns kv heads [r*Hkv/G, (r+1)*Hkv/G) of every KV
cache and the matching query heads [r*H/G, (r+1)*H/G) (query head h reads kv head
h // (H/Hkv), so both slices are contiguous).  Its result is the ggml tensor
[Dv, H/G, n_q, n_seq]; the o_proj that follows (src/qwen3-lm.h:823-827) needs all heads,
so the only exchange is an all-gather of the G slices (NCCL over NVLink through
torch.distributed) followed by mm3fa_assemble_heads, which permutes the rank-major
gather into [Dv, H, n_q, n_seq].  The DiT shards the same way over (batch x head) units.
"""
from __future__ import annotations

import numpy as np

from . import ggml


def head_slice(n_head: int, n_head_kv: int, rank: int, world: int) -> tuple[int, int, int, int]:
    """(h0, h1, g0, g1): query heads [h0, h1) and kv heads [g0, g1) owned by `rank`."""
    if n_head_kv % world or n_head % world:
        raise ValueError(f"{n_head} q heads / {n_head_kv} kv heads do not split over {world} ranks")
    gk = n_head_kv // world
    hq = n_head // world
    return rank * hq, (rank + 1) * hq, rank * gk, (rank + 1) * gk


def _slice_heads(t: ggml.Tensor, h0: int, h1: int) -> ggml.Tensor:
    ne = list(t.ne)
    ne[2] = h1 - h0
    return ggml.make(t.type, ne, (t.data or 0) + h0 * t.nb[2], list(t.nb))


def shard_operands(q: ggml.Tensor, k: ggml.Tensor, v: ggml.Tensor, mask: ggml.Tensor | None, rank: int,
                   world: int, max_bias: float = 0.0):
    """Per-rank views of the full-head operands (no copies).

    Each rank usually holds only its own heads' KV cache; then pass that cache's
    descriptors with rank=0, world=1 instead.  ALiBi (max_bias > 0) would need the
    global head index and is rejected, as is a mask that varies per head unless the
    per-rank head count is a multiple of its head dimension.
    """
    n_head, n_head_kv = q.ne[2], k.ne[2]
    h0, h1, g0, g1 = head_slice(n_head, n_head_kv, rank, world)
    if world > 1 and max_bias > 0.0:
        raise ValueError("head sharding with ALiBi slopes is not supported")
    if mask is not None and mask.ne[2] > 1 and (h1 - h0) % mask.ne[2]:
        raise ValueError("per-head mask does not split over the ranks")
    return _slice_heads(q, h0, h1), _slice_heads(k, g0, g1), _slice_heads(v, g0, g1), mask


def assemble_heads_np(gathered: np.ndarray, world: int) -> np.ndarray:
    """numpy statement of mm3fa_assemble_heads.

    gathered: (world, n_seq, n_q, H/world, Dv) -> (n_seq, n_q, H, Dv) (= ggml [Dv, H, n_q, n_seq]).
    """
    g = np.asarray(gathered)
    return np.ascontiguousarray(g.transpose(1, 2, 0, 3, 4).reshape(g.shape[1], g.shape[2], -1, g.shape[4]))


def unit_slice(n_seq: int, n_head: int, rank: int, world: int) -> tuple[int, int, int, int, int]:
    """(batch x head) sharding of the DiT (and of any call by sequence and head): the ranks split
    the sequences into seq_split = min(world, n_seq) groups and the heads into world / seq_split
    groups.  Returns (s0, s1, h0, h1, seq_split): rank r = sg * (world / seq_split) + hg owns
    sequences [s0, s1) and heads [h0, h1), in the rank order mm3fa_allgather_heads gathers."""
    seq_split = min(world, n_seq)
    if world % seq_split or n_seq % seq_split:
        raise ValueError(f"{n_seq} sequences do not split over {world} ranks")
    hs = world // seq_split
    if n_head % hs:
        raise ValueError(f"{n_head} heads do not split over {hs} head groups")
    sg, hg = rank // hs, rank % hs
    sl, hl = n_seq // seq_split, n_head // hs
    return sg * sl, (sg + 1) * sl, hg * hl, (hg + 1) * hl, seq_split


def allgather_scatter_np(gathered: np.ndarray, seq_split: int) -> np.ndarray:
    """numpy statement of mm3fa_allgather_heads' permute: gathered (G, n_seq/ss, n_q, H/hs, Dv) in
    rank order r = sg * hs + hg -> the ggml result (n_seq, n_q, H, Dv)."""
    g = np.asarray(gathered)
    G, sl, n_q, hl, dv = g.shape
    hs = G // seq_split
    x = g.reshape(seq_split, hs, sl, n_q, hl, dv).transpose(0, 2, 3, 1, 4, 5)
    return np.ascontiguousarray(x.reshape(seq_split * sl, n_q, hs * hl, dv))
