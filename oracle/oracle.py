"""ctypes front end of the CPU oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, __graft_entry__.smoke() and bench.py's
CPU-baseline / reference arm, never by the product.  The algorithm and its citations are
in attn_oracle.cpp; parity at the op boundary is unpinned (the reference's ggml submodule
is absent), and the oracle is cross-checked against torch SDPA (float64) and gguf-py's
Q8_0 codec instead.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(ROOT, "minimaxmusic.cpp_b200"))

from mm3fa import ggml  # noqa: E402  (descriptor layout shared with the C ABI)

MODE_EXACT = 0
MODE_F32ACC = 1
MODE_GGML_CPU = 2

_lib = None


def build(force: bool = False) -> str:
    """Compiles liboracle.so with the Makefile beside this file."""
    path = os.path.join(HERE, "liboracle.so")
    if force or not os.path.exists(path) or os.path.getmtime(path) < os.path.getmtime(
            os.path.join(HERE, "attn_oracle.cpp")):
        subprocess.run(["make", "-s", "-C", HERE, "-B" if force else "liboracle.so"], check=True)
    return path


def lib():
    global _lib
    if _lib is None:
        _lib = ctypes.CDLL(build())
        P = ctypes.POINTER(ggml.Tensor)
        _lib.orc_flash_attn_ext.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                            ctypes.c_int, P, ctypes.c_int]
        _lib.orc_flash_attn_ext.restype = ctypes.c_int
        _lib.orc_q8_0_quantize_row.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _lib.orc_q8_0_dequantize_row.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _lib.orc_f32_to_f16_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _lib.orc_f16_to_f32_array.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64]
        _lib.orc_alibi_slope.argtypes = [ctypes.c_int, ctypes.c_int, ctypes.c_float]
        _lib.orc_alibi_slope.restype = ctypes.c_float
    return _lib


def f32_to_f16_bits(x: np.ndarray) -> np.ndarray:
    """IEEE binary16 round-to-nearest-even of x, as uint16 bit patterns."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    out = np.empty(x.shape, dtype=np.uint16)
    lib().orc_f32_to_f16_array(x.ctypes.data, out.ctypes.data, x.size)
    return out


def f16_bits_to_f32(h: np.ndarray) -> np.ndarray:
    h = np.ascontiguousarray(h, dtype=np.uint16)
    out = np.empty(h.shape, dtype=np.float32)
    lib().orc_f16_to_f32_array(h.ctypes.data, out.ctypes.data, h.size)
    return out


def q8_0_quantize(x: np.ndarray) -> np.ndarray:
    """Quantizes the last axis (multiple of 32) into Q8_0 block bytes."""
    x = np.ascontiguousarray(x, dtype=np.float32)
    n = x.shape[-1]
    out = np.empty(x.shape[:-1] + (n // 32 * 34,), dtype=np.uint8)
    rows = x.reshape(-1, n)
    orows = out.reshape(-1, n // 32 * 34)
    for r in range(rows.shape[0]):
        lib().orc_q8_0_quantize_row(rows[r].ctypes.data, orows[r].ctypes.data, n)
    return out


def q8_0_dequantize(b: np.ndarray) -> np.ndarray:
    b = np.ascontiguousarray(b, dtype=np.uint8)
    nbytes = b.shape[-1]
    n = nbytes // 34 * 32
    out = np.empty(b.shape[:-1] + (n,), dtype=np.float32)
    rows = b.reshape(-1, nbytes)
    orows = out.reshape(-1, n)
    for r in range(rows.shape[0]):
        lib().orc_q8_0_dequantize_row(rows[r].ctypes.data, orows[r].ctypes.data, n)
    return out


# ---------------------------------------------------------------- decode prologue
# The nodes src/qwen3-lm.h:764-800 builds before the attention call, restated from ggml's CPU
# kernels (ggml is an absent submodule of the reference; these follow ggml's published
# ggml-cpu ops: rms_norm_f32, mul, rope_f32 in NEOX mode with its rope cache, set_rows):
#   * rms_norm: sum of squares accumulated in double, mean = sum / D rounded to float,
#     scale = 1 / sqrtf(mean + eps), y = x * scale (float); ggml_mul then y * w (float).
#   * rope NEOX (freq_scale 1, ext_factor 0, attn_factor 1, all D dims): theta_scale =
#     powf(theta, -2/D); the cache walks pairs i = 0 .. D/2-1 with angle t (starting at the
#     position) and t *= theta_scale after each pair; out[i] = x[i] cos t - x[i + D/2] sin t,
#     out[i + D/2] = x[i] sin t + x[i + D/2] cos t.
#   * set_rows: F32 -> F16 / BF16 (round to nearest even) or Q8_0 (the block quantizer above).

def rms_norm_mul(x: np.ndarray, w: np.ndarray, eps: float) -> np.ndarray:
    """ggml_rms_norm over the last axis, then ggml_mul by w (float32 results)."""
    x = np.asarray(x, dtype=np.float32)
    mean = ((x.astype(np.float64) ** 2).sum(-1, keepdims=True) / x.shape[-1]).astype(np.float32)
    scale = (np.float32(1.0) / np.sqrt(mean + np.float32(eps))).astype(np.float32)
    return ((x * scale).astype(np.float32) * np.asarray(w, dtype=np.float32)).astype(np.float32)


def rope_neox(x: np.ndarray, pos: np.ndarray, theta: float, n_dims: int | None = None) -> np.ndarray:
    """ggml_rope_ext in NEOX mode over the first n_dims dims (all by default; the rest are copied);
    x [N, H, D], pos [N] (int)."""
    x = np.asarray(x, dtype=np.float32)
    n, _, d = x.shape
    nd = n_dims or d
    half = nd // 2
    ts = np.float32(np.power(np.float32(theta), np.float32(-2.0) / np.float32(nd)))
    out = x.copy()
    for s in range(n):
        t = np.float32(pos[s])
        cs = np.empty(half, dtype=np.float32)
        sn = np.empty(half, dtype=np.float32)
        for i in range(half):
            cs[i] = np.cos(t)
            sn[i] = np.sin(t)
            t = np.float32(t * ts)
        x0, x1 = x[s, :, :half], x[s, :, half:nd]
        out[s, :, :half] = (x0 * cs - x1 * sn).astype(np.float32)
        out[s, :, half:nd] = (x0 * sn + x1 * cs).astype(np.float32)
    return out


def clamp_fp16(x: np.ndarray) -> np.ndarray:
    """ggml_clamp(v, -65504, 65504) as the reference inserts it with --clamp-fp16
    (src/qwen3-lm.h:779-782): values beyond the F16 range saturate, NaN passes through."""
    x = np.asarray(x, dtype=np.float32)
    return np.where(x > np.float32(65504), np.float32(65504),
                    np.where(x < np.float32(-65504), np.float32(-65504), x)).astype(np.float32)


def decode_prologue(q_in: np.ndarray, k_in: np.ndarray, v_in: np.ndarray, q_norm: np.ndarray, k_norm: np.ndarray,
                    eps: float, pos: np.ndarray, theta: float,
                    clamp_v: bool = False) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(q_out, k_new, v_new) in F32: q_in [N, H, D], k_in/v_in [N, Hkv, D]; the caller converts
    k_new / v_new to the cache type (f32_to_f16_bits, q8_0_quantize) as set_rows does.  clamp_v:
    the --clamp-fp16 clamp of v before that conversion."""
    q = rope_neox(rms_norm_mul(q_in, q_norm, eps), pos, theta)
    k = rope_neox(rms_norm_mul(k_in, k_norm, eps), pos, theta)
    v = np.asarray(v_in, dtype=np.float32)
    return q, k, (clamp_fp16(v) if clamp_v else v)


def alibi_slope(h: int, n_head: int, max_bias: float) -> float:
    return float(lib().orc_alibi_slope(h, n_head, max_bias))


def flash_attn_ext(q: ggml.Tensor, k: ggml.Tensor, v: ggml.Tensor, mask: ggml.Tensor | None, scale: float,
                   max_bias: float = 0.0, logit_softcap: float = 0.0, mode: int = MODE_EXACT,
                   threads: int | None = None) -> np.ndarray:
    """Runs the oracle on host descriptors; returns dst as a numpy array of shape
    (n_seq, n_q, n_head, Dv), i.e. the contiguous ggml tensor [Dv, n_head, n_q, n_seq]."""
    dv, n_head, n_q, n_seq = v.ne[0], q.ne[2], q.ne[1], q.ne[3]
    out = np.zeros((n_seq, n_q, n_head, dv), dtype=np.float32)
    d = ggml.from_numpy(out)
    threads = threads or os.cpu_count() or 1
    rc = lib().orc_flash_attn_ext(ctypes.byref(q), ctypes.byref(k), ctypes.byref(v),
                                  ctypes.byref(mask) if mask is not None else None, scale, max_bias,
                                  logit_softcap, mode, ctypes.byref(d), threads)
    if rc != 0:
        raise ValueError(f"oracle rejected the operands (code {rc})")
    return out
