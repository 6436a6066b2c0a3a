"""Generates the golden fixtures under tests/golden/ (run from the repo root).

    python tests/golden/make_golden.py

The reference's implementation of GGML_OP_FLASH_ATTN_EXT (its ggml submodule) is absent
from the reference tree, so no reference-produced vectors exist.  Each fixture instead
stores seeded operands (in the exact ggml layouts the reference uses, see
mm3fa/workloads.py) with three independently computed results:

  out_exact     - the CPU oracle in exact mode (float64 accumulation)
  out_f32acc    - the CPU oracle in F32-accumulation mode (Q rounded to K's vec-dot type,
                  F32 softmax and V sums: the precision set_prec(F32) asks for)
  out_ggml_cpu  - the CPU oracle's restatement of ggml's CPU kernel (F16 V accumulator when
                  V is F16)
  out_torch     - torch.nn.functional.scaled_dot_product_attention in float64 on the
                  dequantized operands (only where no softcap/ALiBi is involved)

Tests check that the oracle still reproduces the three oracle outputs bit for bit and that
out_exact agrees with out_torch, and the GPU tests compare the CUDA path against them.
"""
from __future__ import annotations

import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "minimaxmusic.cpp_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

import oracle  # noqa: E402
from mm3fa import ggml, workloads  # noqa: E402


def cases():
    yield "decode_f16_ragged", workloads.decode_case(n_seq=2, n_kv=192, max_seq=224, n_head=8, n_head_kv=2,
                                                     kv_len=[100, 187], seed=11)
    yield "decode_q8_0", workloads.decode_case(n_seq=2, n_kv=256, n_head=8, n_head_kv=2, kv_type=ggml.GGML_TYPE_Q8_0,
                                               seed=12)
    yield "decode_multirow_gqa8", workloads.decode_case(n_seq=1, n_kv=160, n_q=3, n_head=16, n_head_kv=2,
                                                        kv_len=[150], seed=13)
    yield "prefill_causal", workloads.prefill_case(n_seq=1, S=40, n_head=8, n_head_kv=2, kv_pos=24, pad=64, seed=14)
    yield "dit_d64", workloads.dit_case(B=2, S=33, H=4, D=64, seed=15)
    c = workloads.decode_case(n_seq=1, n_kv=96, n_head=8, n_head_kv=4, seed=16, name="softcap_alibi")
    c.softcap = 30.0
    c.max_bias = 8.0
    yield "softcap_alibi", c


def torch_reference(c) -> np.ndarray:
    """SDPA in float64 on dequantized operands; returns (n_seq, n_q, n_head, Dv)."""
    import torch

    def dense(op):
        # gather the view into a dense (ne3, ne2, ne1, ne0) float64 array
        D, n1, n2, n3 = op.ne
        out = np.empty((n3, n2, n1, D), dtype=np.float64)
        raw = op.storage.view(np.uint8).reshape(-1)
        rb = ggml.row_bytes(op.gtype, D)
        for s in range(n3):
            for h in range(n2):
                for j in range(n1):
                    off = op.offset + j * op.nb[1] + h * op.nb[2] + s * op.nb[3]
                    row = raw[off:off + rb]
                    if op.gtype == ggml.GGML_TYPE_F32:
                        out[s, h, j] = row.view(np.float32)
                    elif op.gtype == ggml.GGML_TYPE_F16:
                        out[s, h, j] = row.view(np.float16)
                    elif op.gtype == ggml.GGML_TYPE_Q8_0:
                        out[s, h, j] = oracle.q8_0_dequantize(row[None])[0]
        return out

    q, k, v = dense(c.q), dense(c.k), dense(c.v)
    r = q.shape[1] // k.shape[1]
    k = np.repeat(k, r, axis=1)
    v = np.repeat(v, r, axis=1)
    bias = None
    if c.mask is not None:
        m = dense(c.mask)  # (m3, m2, n_q_pad, n_kv)
        bias = torch.from_numpy(m[:, :, :q.shape[2], :])
    o = torch.nn.functional.scaled_dot_product_attention(torch.from_numpy(q), torch.from_numpy(k),
                                                         torch.from_numpy(v), attn_mask=bias, scale=c.scale)
    return np.ascontiguousarray(o.numpy().transpose(0, 2, 1, 3)).astype(np.float32)


def save(name, c):
    qd, kd, vd = c.q.host_desc(), c.k.host_desc(), c.v.host_desc()
    md = c.mask.host_desc() if c.mask is not None else None
    ex = oracle.flash_attn_ext(qd, kd, vd, md, c.scale, c.max_bias, c.softcap, oracle.MODE_EXACT, threads=1)
    f32 = oracle.flash_attn_ext(qd, kd, vd, md, c.scale, c.max_bias, c.softcap, oracle.MODE_F32ACC, threads=1)
    cpu = oracle.flash_attn_ext(qd, kd, vd, md, c.scale, c.max_bias, c.softcap, oracle.MODE_GGML_CPU, threads=1)
    arrays = dict(out_exact=ex, out_f32acc=f32, out_ggml_cpu=cpu)
    if c.softcap == 0.0 and c.max_bias == 0.0:
        arrays["out_torch"] = torch_reference(c)
    for tag, op in (("q", c.q), ("k", c.k), ("v", c.v), ("mask", c.mask)):
        if op is None:
            continue
        arrays[f"{tag}_storage"] = op.storage
        arrays[f"{tag}_meta"] = np.array([op.gtype, *op.ne, *op.nb, op.offset], dtype=np.int64)
    arrays["params"] = np.array([c.scale, c.max_bias, c.softcap], dtype=np.float64)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **arrays)
    print(name, {k: v.shape for k, v in arrays.items()})


if __name__ == "__main__":
    for n, c in cases():
        save(n, c)
