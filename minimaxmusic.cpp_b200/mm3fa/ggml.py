"""ggml tensor descriptors for the mm3fa C ABI.

A ggml tensor is (type, ne[4], nb[4], data) with ne[0] the innermost dimension
(ggml.h's struct ggml_tensor).  The reference builds every operand of
GGML_OP_FLASH_ATTN_EXT as such a tensor or a strided view of one:
src/qwen3-lm.h:427-428 and :810-813 view the [D, max_seq, Nkv, n_sets] F16 KV
cache, src/qwen3-lm.h:401 and src/dit.h:212-214 pass permuted F32 Q views.

This module maps numpy arrays (host) and torch tensors (device) onto that
descriptor without copying.  A C-contiguous array of shape (ne3, ne2, ne1, ne0)
is the contiguous ggml tensor [ne0, ne1, ne2, ne3]; Q8_0 tensors are uint8
arrays whose last axis holds ne0/32 blocks of 34 bytes.
"""
from __future__ import annotations

import ctypes

GGML_TYPE_F32 = 0
GGML_TYPE_F16 = 1
GGML_TYPE_Q8_0 = 8
GGML_TYPE_BF16 = 30

GGML_PREC_DEFAULT = 0
GGML_PREC_F32 = 10

QK8_0 = 32
Q8_0_BLOCK_BYTES = 34

TYPE_NAMES = {GGML_TYPE_F32: "f32", GGML_TYPE_F16: "f16", GGML_TYPE_Q8_0: "q8_0", GGML_TYPE_BF16: "bf16"}


class Tensor(ctypes.Structure):
    """Mirror of mm3fa_tensor (include/mm3fa.h)."""

    _fields_ = [
        ("type", ctypes.c_int32),
        ("reserved", ctypes.c_int32),
        ("ne", ctypes.c_int64 * 4),
        ("nb", ctypes.c_uint64 * 4),
        ("data", ctypes.c_void_p),
    ]

    def __repr__(self) -> str:  # pragma: no cover - debugging aid
        return (f"Tensor({TYPE_NAMES.get(self.type, self.type)}, ne={list(self.ne)}, "
                f"nb={list(self.nb)}, data=0x{(self.data or 0):x})")


def row_bytes(gtype: int, n: int) -> int:
    """Bytes of one row of n elements (ggml_row_size)."""
    if gtype == GGML_TYPE_F32:
        return 4 * n
    if gtype in (GGML_TYPE_F16, GGML_TYPE_BF16):
        return 2 * n
    if gtype == GGML_TYPE_Q8_0:
        if n % QK8_0:
            raise ValueError("Q8_0 rows must hold a multiple of 32 elements")
        return n // QK8_0 * Q8_0_BLOCK_BYTES
    raise ValueError(f"unsupported ggml type {gtype}")


def elem_bytes(gtype: int) -> int:
    """Byte size of the addressable unit along ne[0] (a block for Q8_0)."""
    return {GGML_TYPE_F32: 4, GGML_TYPE_F16: 2, GGML_TYPE_BF16: 2, GGML_TYPE_Q8_0: Q8_0_BLOCK_BYTES}[gtype]


def contiguous_nb(gtype: int, ne) -> list[int]:
    """Byte strides of a contiguous tensor of shape ne (ggml_new_tensor)."""
    nb0 = elem_bytes(gtype)
    nb1 = row_bytes(gtype, ne[0])
    return [nb0, nb1, nb1 * ne[1], nb1 * ne[1] * ne[2]]


def make(gtype: int, ne, data_ptr: int, nb=None) -> Tensor:
    """Descriptor for a tensor at data_ptr; nb defaults to the contiguous strides."""
    ne = list(ne) + [1] * (4 - len(ne))
    nb = contiguous_nb(gtype, ne) if nb is None else list(nb)
    t = Tensor()
    t.type = gtype
    for i in range(4):
        t.ne[i] = int(ne[i])
        t.nb[i] = int(nb[i])
    t.data = ctypes.c_void_p(int(data_ptr)) if data_ptr else None
    return t


def view(base: Tensor, ne, nb, offset_bytes: int = 0) -> Tensor:
    """ggml_view_4d: a strided view of base starting offset_bytes into it."""
    return make(base.type, ne, (base.data or 0) + offset_bytes, nb)


def _fill_trailing_nb(gtype: int, ne, nb, ndim: int) -> None:
    """Strides of the size-1 dims an array of ndim < 4 dims leaves implicit."""
    for i in range(max(ndim, 1), 4):
        nb[i] = row_bytes(gtype, ne[0]) if i == 1 else nb[i - 1] * ne[i - 1]


def _numpy_gtype(arr) -> int:
    import numpy as np

    if arr.dtype == np.float32:
        return GGML_TYPE_F32
    if arr.dtype == np.float16:
        return GGML_TYPE_F16
    raise ValueError(f"cannot infer a ggml type from numpy dtype {arr.dtype}")


def from_numpy(arr, gtype: int | None = None, ne=None) -> Tensor:
    """Descriptor of a host numpy array (shape (ne3, ne2, ne1, ne0[-bytes for Q8_0])).

    The array's strides become nb; the array must outlive the descriptor.
    bf16 arrays are passed as uint16 with gtype=GGML_TYPE_BF16; Q8_0 as uint8.
    """
    if gtype is None:
        gtype = _numpy_gtype(arr)
    shape = list(arr.shape)[::-1] + [1] * (4 - arr.ndim)
    strides = list(arr.strides)[::-1] + [0] * (4 - arr.ndim)
    if ne is None:
        ne = list(shape)
        if gtype == GGML_TYPE_Q8_0:
            ne[0] = shape[0] // Q8_0_BLOCK_BYTES * QK8_0
    nb = [elem_bytes(gtype)] + strides[1:4]
    _fill_trailing_nb(gtype, ne, nb, arr.ndim)
    return make(gtype, ne, arr.ctypes.data, nb)


def _torch_gtype(t) -> int:
    import torch

    m = {torch.float32: GGML_TYPE_F32, torch.float16: GGML_TYPE_F16, torch.bfloat16: GGML_TYPE_BF16}
    if t.dtype in m:
        return m[t.dtype]
    raise ValueError(f"cannot infer a ggml type from torch dtype {t.dtype}")


def from_torch(t, gtype: int | None = None, ne=None) -> Tensor:
    """Descriptor of a torch tensor (any device) with ggml dims reversed from torch's.

    A torch tensor of shape (ne3, ne2, ne1, ne0) maps to ggml [ne0, ne1, ne2, ne3];
    strides may be arbitrary (views), as long as dim -1 is contiguous.
    Q8_0 tensors are uint8 with the last torch dim holding the block bytes.
    """
    if gtype is None:
        gtype = _torch_gtype(t)
    nd = t.dim()
    shape = list(t.shape)[::-1] + [1] * (4 - nd)
    esz = t.element_size()
    strides = [s * esz for s in list(t.stride())[::-1]] + [0] * (4 - nd)
    if ne is None:
        ne = list(shape)
        if gtype == GGML_TYPE_Q8_0:
            ne[0] = shape[0] // Q8_0_BLOCK_BYTES * QK8_0
    if nd and t.stride(-1) != 1:
        raise ValueError("innermost dimension must be contiguous")
    nb = [elem_bytes(gtype)] + strides[1:4]
    _fill_trailing_nb(gtype, ne, nb, nd)
    return make(gtype, ne, t.data_ptr(), nb)
