"""Seeded synthetic operands for GGML_OP_FLASH_ATTN_EXT at the shapes the reference uses.

No public dataset is involved: every tensor is generated from a seed with the value
distributions of the benchmark configurations, and laid out exactly as the reference
lays it out in device memory:

* LM decode (src/qwen3-lm.h:784-824): Q F32 [128, 1, 32, N] contiguous; K/V are
  [128, n_kv, 8, N] views of the [128, max_seq, 8, n_sets] F16 cache
  (nb = {2, 256, 256*max_seq, 256*max_seq*8}); mask F16 [n_kv, 1, 1, N].
* LM prefill (src/qwen3-lm.h:395-436): Q F32 is the permuted view [128, S, 32] of the
  [128, 32, S] projection (token stride 16 KiB, head stride 512 B); K/V [128, n_kv, 8]
  views of the cache; causal mask F16 [n_kv, S] with -inf above the diagonal.
* DiT (src/dit.h:201-222): Q F32 permuted view [D, S, H, B] of [D, H, S, B]; K/V F16
  contiguous [D, S, H, B] (ggml_cast output); no mask.
"""
from __future__ import annotations

import dataclasses
import math

import numpy as np

from . import ggml


@dataclasses.dataclass
class Operand:
    """One operand: its backing storage and the ggml view the operator sees."""

    storage: np.ndarray  # backing buffer (C-contiguous)
    gtype: int
    ne: list
    nb: list
    offset: int = 0  # byte offset of the view into storage

    def host_desc(self) -> ggml.Tensor:
        return ggml.make(self.gtype, self.ne, self.storage.ctypes.data + self.offset, self.nb)

    def device_desc(self, dev_storage) -> ggml.Tensor:
        return ggml.make(self.gtype, self.ne, dev_storage.data_ptr() + self.offset, self.nb)

    def view_bytes(self) -> int:
        """Bytes the operator reads through this view (rows actually addressed)."""
        rows = self.ne[1] * self.ne[2] * self.ne[3]
        return rows * ggml.row_bytes(self.gtype, self.ne[0])


@dataclasses.dataclass
class Case:
    name: str
    q: Operand
    k: Operand
    v: Operand
    mask: Operand | None
    scale: float
    max_bias: float = 0.0
    softcap: float = 0.0

    @property
    def dst_ne(self) -> list:
        return [self.v.ne[0], self.q.ne[2], self.q.ne[1], self.q.ne[3]]

    def dst_shape(self) -> tuple:
        dv, h, nq, ns = self.dst_ne
        return (ns, nq, h, dv)

    def algorithmic_bytes(self) -> int:
        """Bytes one call must move at minimum: K, V, Q and mask read once, dst written once."""
        b = self.k.view_bytes() + self.v.view_bytes() + self.q.view_bytes()
        b += 4 * int(np.prod(self.dst_ne))
        if self.mask is not None:
            m = self.mask
            b += m.ne[2] * m.ne[3] * self.q.ne[1] * ggml.row_bytes(m.gtype, m.ne[0])
        return b

    def algorithmic_flops(self, causal: bool = False) -> float:
        """2 matmuls x 2 flops per MAC over the (causally visible) score matrix."""
        D, n_q, H, B = self.q.ne
        n_kv = self.k.ne[1]
        if causal:
            pairs = n_q * (n_q + 1) / 2 + n_q * max(0, n_kv - n_q)
        else:
            pairs = n_q * n_kv
        return 2.0 * 2.0 * D * pairs * H * B


def _f16(x: np.ndarray) -> np.ndarray:
    return x.astype(np.float16)


def _rms_norm_heads(x: np.ndarray, eps: float = 1e-6) -> np.ndarray:
    return x / np.sqrt((x.astype(np.float64) ** 2).mean(axis=-1, keepdims=True) + eps).astype(np.float32)


def _rope_neox(x: np.ndarray, pos: np.ndarray, theta: float, n_rot: int | None = None) -> np.ndarray:
    """NeoX rotary embedding over the last axis (pairs (i, i + n_rot/2)), positions on axis -3."""
    D = x.shape[-1]
    n_rot = n_rot or D
    half = n_rot // 2
    inv = theta ** (-np.arange(half, dtype=np.float64) * 2.0 / n_rot)
    ang = pos.astype(np.float64)[:, None] * inv[None, :]  # [S, half]
    c = np.cos(ang).astype(np.float32)[:, None, :]
    s = np.sin(ang).astype(np.float32)[:, None, :]
    out = x.copy()
    a, b = x[..., :half], x[..., half:n_rot]
    out[..., :half] = a * c - b * s
    out[..., half:n_rot] = a * s + b * c
    return out


def kv_cache(rng, n_seq: int, n_head_kv: int, n_kv: int, D: int, std: float, max_seq: int | None = None,
             gtype: int = ggml.GGML_TYPE_F16) -> tuple[Operand, Operand]:
    """K and V as [D, n_kv, n_head_kv, n_seq] views of [D, max_seq, n_head_kv, n_seq] caches."""
    max_seq = max_seq or n_kv
    ops = []
    for _ in range(2):
        if gtype == ggml.GGML_TYPE_Q8_0:
            st = q8_0_random_blocks(rng, (n_seq, n_head_kv, max_seq), D)
        else:
            st = _f16(rng.standard_normal((n_seq, n_head_kv, max_seq, D), dtype=np.float32) * std)
        rb = ggml.row_bytes(gtype, D)
        nb = [ggml.elem_bytes(gtype), rb, rb * max_seq, rb * max_seq * n_head_kv]
        ops.append(Operand(st, gtype, [D, n_kv, n_head_kv, n_seq], nb))
    return ops[0], ops[1]


def q8_0_random_blocks(rng, lead: tuple, D: int) -> np.ndarray:
    """Q8_0 rows with int8 ~U[-127,127] and fp16 scales ~U[0.001,0.02] (benchmark config 3)."""
    nblk = D // ggml.QK8_0
    out = np.empty(lead + (nblk, ggml.Q8_0_BLOCK_BYTES), dtype=np.uint8)
    d = rng.uniform(0.001, 0.02, size=lead + (nblk,)).astype(np.float16)
    qs = rng.integers(-127, 128, size=lead + (nblk, ggml.QK8_0), dtype=np.int64).astype(np.int8)
    out[..., 0:2] = d.view(np.uint8).reshape(lead + (nblk, 2))
    out[..., 2:] = qs.view(np.uint8)
    return out.reshape(lead + (nblk * ggml.Q8_0_BLOCK_BYTES,))


def decode_case(n_seq: int = 2, n_kv: int = 2048, n_head: int = 32, n_head_kv: int = 8, D: int = 128,
                n_q: int = 1, kv_std: float = 0.5, seed: int = 1, max_seq: int | None = None,
                kv_type: int = ggml.GGML_TYPE_F16, kv_len: list | None = None, name: str = "decode") -> Case:
    """LM batched CFG decode (benchmark configs 1, 2, 3): 1..8 query rows per KV set.

    kv_len, when given, is the per-sequence visible length; the mask is 0 below it and
    -inf from it on (src/qwen3-lm.h:909-920).  Default: every position visible.
    """
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((n_seq, n_head, n_q, D), dtype=np.float32)
    qop = Operand(q, ggml.GGML_TYPE_F32, [D, n_q, n_head, n_seq], ggml.contiguous_nb(ggml.GGML_TYPE_F32,
                                                                                   [D, n_q, n_head, n_seq]))
    k, v = kv_cache(rng, n_seq, n_head_kv, n_kv, D, kv_std, max_seq, kv_type)
    mask = np.zeros((n_seq, 1, n_q, n_kv), dtype=np.float16)
    if kv_len is not None:
        for s in range(n_seq):
            for i in range(n_q):
                mask[s, 0, i, kv_len[s] - n_q + 1 + i:] = -np.inf
    mop = Operand(mask, ggml.GGML_TYPE_F16, [n_kv, n_q, 1, n_seq],
                  ggml.contiguous_nb(ggml.GGML_TYPE_F16, [n_kv, n_q, 1, n_seq]))
    return Case(name, qop, k, v, mop, 1.0 / math.sqrt(D))


def prefill_case(n_seq: int = 2, S: int = 1024, n_head: int = 32, n_head_kv: int = 8, D: int = 128,
                 seed: int = 4, kv_pos: int = 0, pad: int = 256, theta: float = 1e6) -> Case:
    """Causal LM prefill (benchmark config 4): RMS-normed (w=1), NeoX-RoPE'd Q/K.

    Q is the permuted F32 view [D, S, H, n_seq] of the [D, H, S, n_seq] projection; the
    causal mask [n_kv_pad, S] lets row i see columns <= kv_pos + i (src/qwen3-lm.h:604-617).
    """
    rng = np.random.default_rng(seed)
    n_kv = kv_pos + S
    n_kv_pad = -(-n_kv // pad) * pad
    pos = np.arange(kv_pos, kv_pos + S)
    q = rng.standard_normal((n_seq, S, n_head, D), dtype=np.float32)  # storage [D, H, S, B]
    q = _rope_neox(_rms_norm_heads(q), pos, theta)
    kf = rng.standard_normal((n_seq, n_kv, n_head_kv, D), dtype=np.float32)
    kf = _rope_neox(_rms_norm_heads(kf), np.arange(n_kv), theta)
    vf = rng.standard_normal((n_seq, n_kv, n_head_kv, D), dtype=np.float32)
    # cache layout [D, n_kv_pad, Hkv, n_seq]; the padded tail stays zero like the reference's cleared cache
    kc = np.zeros((n_seq, n_head_kv, n_kv_pad, D), dtype=np.float16)
    vc = np.zeros_like(kc)
    kc[:, :, :n_kv] = _f16(kf.transpose(0, 2, 1, 3))
    vc[:, :, :n_kv] = _f16(vf.transpose(0, 2, 1, 3))
    rb = 2 * D
    kv_nb = [2, rb, rb * n_kv_pad, rb * n_kv_pad * n_head_kv]
    qop = Operand(q, ggml.GGML_TYPE_F32, [D, S, n_head, n_seq], [4, 4 * D * n_head, 4 * D, 4 * D * n_head * S])
    kop = Operand(kc, ggml.GGML_TYPE_F16, [D, n_kv_pad, n_head_kv, n_seq], kv_nb)
    vop = Operand(vc, ggml.GGML_TYPE_F16, [D, n_kv_pad, n_head_kv, n_seq], list(kv_nb))
    mask = np.full((S, n_kv_pad), -np.inf, dtype=np.float16)
    for i in range(S):
        mask[i, :kv_pos + i + 1] = 0
    mop = Operand(mask, ggml.GGML_TYPE_F16, [n_kv_pad, S, 1, 1], ggml.contiguous_nb(ggml.GGML_TYPE_F16,
                                                                                   [n_kv_pad, S, 1, 1]))
    return Case("prefill", qop, kop, vop, mop, 1.0 / math.sqrt(D))


def dit_case(B: int = 2, S: int = 4096, H: int = 16, D: int = 128, seed: int = 5, name: str = "dit") -> Case:
    """Bidirectional DiT attention (benchmark config 5; real model: S=690, H=32, D=64).

    Q is the permuted F32 view [D, S, H, B] of the [D, H, S, B] projection; K/V are F16
    contiguous [D, S, H, B] (the ggml_cast nodes at src/dit.h:219-220); no mask.
    """
    rng = np.random.default_rng(seed)
    q = _rms_norm_heads(rng.standard_normal((B, S, H, D), dtype=np.float32))
    k = _rms_norm_heads(rng.standard_normal((B, H, S, D), dtype=np.float32))
    v = rng.standard_normal((B, H, S, D), dtype=np.float32)
    qop = Operand(q, ggml.GGML_TYPE_F32, [D, S, H, B], [4, 4 * D * H, 4 * D, 4 * D * H * S])
    kop = Operand(_f16(k), ggml.GGML_TYPE_F16, [D, S, H, B], ggml.contiguous_nb(ggml.GGML_TYPE_F16, [D, S, H, B]))
    vop = Operand(_f16(v), ggml.GGML_TYPE_F16, [D, S, H, B], ggml.contiguous_nb(ggml.GGML_TYPE_F16, [D, S, H, B]))
    return Case(name, qop, kop, vop, None, 1.0 / math.sqrt(D))
