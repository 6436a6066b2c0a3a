"""The CPU oracle against independent implementations and the committed golden fixtures.

Parity at the op boundary is unpinned (the reference's ggml submodule is absent), so the
oracle is pinned here against: numpy's IEEE binary16 conversion, torch's bfloat16
rounding, gguf-py 0.19.0's Q8_0 codec (gguf/quants.py), torch SDPA in float64, and a
float64 numpy statement of softcap and ALiBi.
"""
import glob
import os

import numpy as np
import pytest
import torch

import oracle
from mm3fa import ggml, workloads

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden")


def test_f16_to_f32_all_patterns():
    bits = np.arange(65536, dtype=np.uint16)
    mine = oracle.f16_bits_to_f32(bits)
    ref = bits.view(np.float16).astype(np.float32)
    nan = np.isnan(ref)
    assert np.array_equal(np.isnan(mine), nan)
    assert np.array_equal(mine[~nan].view(np.uint32), ref[~nan].view(np.uint32))


def test_f32_to_f16_round_to_nearest_even():
    rng = np.random.default_rng(0)
    x = np.concatenate([
        rng.standard_normal(200000).astype(np.float32) * 10.0,
        (rng.standard_normal(50000) * 1e-5).astype(np.float32),  # subnormal halves
        np.array([65504, 65519.99, 65520, 65536, -65520, 1e-8, 2.0 ** -24, 2.0 ** -25, 3 * 2.0 ** -26,
                  np.inf, -np.inf, 0.0, -0.0], dtype=np.float32),
        # exact ties between neighbouring halves
        (np.arange(1, 2048, dtype=np.float32) + 0.5) * np.float32(2.0 ** -10),
    ])
    mine = oracle.f32_to_f16_bits(x)
    assert np.array_equal(mine, x.astype(np.float16).view(np.uint16))


def test_bf16_rounding_matches_torch():
    lib = oracle.lib()
    import ctypes

    lib.orc_f32_to_bf16.argtypes = [ctypes.c_float]
    lib.orc_f32_to_bf16.restype = ctypes.c_uint16
    x = torch.randn(4096, generator=torch.Generator().manual_seed(1)) * 37.0
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    mine = np.array([lib.orc_f32_to_bf16(float(v)) for v in x.numpy()], dtype=np.uint16)
    assert np.array_equal(mine, ref)


def test_q8_0_codec_matches_gguf_py():
    gguf = pytest.importorskip("gguf")
    from gguf import quants

    rng = np.random.default_rng(2)
    x = np.concatenate([rng.standard_normal((300, 128)).astype(np.float32) * 3,
                        np.zeros((2, 128), np.float32),  # all-zero block: d = 0
                        np.full((2, 128), -7.25, np.float32)])
    mine = oracle.q8_0_quantize(x)
    ref = quants.quantize(x, gguf.GGMLQuantizationType.Q8_0)
    assert mine.shape == (x.shape[0], 136)
    assert np.array_equal(mine, ref)
    assert np.array_equal(oracle.q8_0_dequantize(mine), quants.dequantize(ref, gguf.GGMLQuantizationType.Q8_0))


def test_q8_0_dequant_is_exact_product():
    rng = np.random.default_rng(3)
    blocks = workloads.q8_0_random_blocks(rng, (64,), 128)
    deq = oracle.q8_0_dequantize(blocks)
    b = blocks.reshape(64, 4, 34)
    d = b[:, :, 0:2].copy().view(np.float16).astype(np.float64)  # (64, 4, 1)
    qs = b[:, :, 2:].view(np.int8).astype(np.float64)
    ref = (d * qs).reshape(64, 128)
    assert np.array_equal(deq.astype(np.float64), ref)


def _np_reference(c) -> np.ndarray:
    """float64 numpy statement of the op incl. softcap and ALiBi (independent of the oracle)."""
    def dense(op):
        D, n1, n2, n3 = op.ne
        raw = op.storage.view(np.uint8).reshape(-1)
        rb = ggml.row_bytes(op.gtype, D)
        out = np.empty((n3, n2, n1, D))
        for s in range(n3):
            for h in range(n2):
                for j in range(n1):
                    off = op.offset + j * op.nb[1] + h * op.nb[2] + s * op.nb[3]
                    row = raw[off:off + rb]
                    out[s, h, j] = {ggml.GGML_TYPE_F32: lambda r: r.view(np.float32),
                                    ggml.GGML_TYPE_F16: lambda r: r.view(np.float16),
                                    ggml.GGML_TYPE_Q8_0: lambda r: oracle.q8_0_dequantize(r[None])[0]}[op.gtype](row)
        return out

    q, k, v = dense(c.q), dense(c.k), dense(c.v)
    n_seq, H, n_q, D = q.shape
    Hk = k.shape[1]
    out = np.zeros((n_seq, n_q, H, v.shape[3]))
    m = dense(c.mask) if c.mask is not None else None
    n_head_log2 = 2 ** int(np.floor(np.log2(H)))
    m0 = 2.0 ** (-c.max_bias / n_head_log2)
    m1 = 2.0 ** (-c.max_bias / 2.0 / n_head_log2)
    for s in range(n_seq):
        for h in range(H):
            slope = 1.0 if c.max_bias <= 0 else (m0 ** (h + 1) if h < n_head_log2 else
                                                 m1 ** (2 * (h - n_head_log2) + 1))
            kk = k[s // (n_seq // k.shape[0]), h // (H // Hk)]
            vv = v[s // (n_seq // v.shape[0]), h // (H // Hk)]
            sc = q[s, h] @ kk.T * c.scale
            if c.softcap:
                sc = c.softcap * np.tanh(sc / c.softcap)
            if m is not None:
                sc = sc + slope * m[s % m.shape[0], h % m.shape[1], :n_q, :]
            mx = sc.max(axis=1, keepdims=True)
            p = np.exp(sc - mx)
            out[s, :, h] = (p @ vv) / p.sum(axis=1, keepdims=True)
    return out.astype(np.float32)


@pytest.mark.parametrize("maker", [
    lambda: workloads.decode_case(n_seq=2, n_kv=100, n_head=8, n_head_kv=2, kv_len=[60, 99], seed=21),
    lambda: workloads.decode_case(n_seq=1, n_kv=64, n_head=4, n_head_kv=1, n_q=5, seed=22),
    lambda: workloads.decode_case(n_seq=2, n_kv=96, n_head=4, n_head_kv=4, kv_type=ggml.GGML_TYPE_Q8_0, seed=23),
    lambda: workloads.prefill_case(n_seq=2, S=17, n_head=4, n_head_kv=2, D=64, kv_pos=5, pad=32, seed=24),
    lambda: workloads.dit_case(B=1, S=29, H=2, D=64, seed=25),
])
@pytest.mark.parametrize("softcap,max_bias", [(0.0, 0.0), (20.0, 0.0), (0.0, 8.0)])
def test_exact_oracle_matches_float64_reference(maker, softcap, max_bias):
    c = maker()
    c.softcap, c.max_bias = softcap, max_bias
    md = c.mask.host_desc() if c.mask is not None else None
    got = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), md, c.scale, max_bias, softcap,
                                oracle.MODE_EXACT, threads=2)
    np.testing.assert_allclose(got, _np_reference(c), atol=2e-6, rtol=0)


def test_ggml_mode_within_tolerance_of_exact():
    c = workloads.decode_case(n_seq=2, n_kv=512, seed=26)
    args = (c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale)
    ex = oracle.flash_attn_ext(*args, mode=oracle.MODE_EXACT)
    gg = oracle.flash_attn_ext(*args, mode=oracle.MODE_F32ACC)
    assert np.abs(ex - gg).max() < 2e-3
    cos = (ex * gg).sum() / np.sqrt((ex * ex).sum() * (gg * gg).sum())
    assert cos > 0.99999


def test_fully_masked_rows_are_zero():
    c = workloads.decode_case(n_seq=2, n_kv=64, n_head=4, n_head_kv=1, seed=27)
    c.mask.storage[0, 0, 0, :] = -np.inf  # sequence 0 sees nothing
    for mode in (oracle.MODE_EXACT, oracle.MODE_F32ACC):
        out = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                                    mode=mode)
        assert np.all(out[0] == 0.0) and np.all(np.isfinite(out[1])) and np.abs(out[1]).sum() > 0


def _load_golden(path):
    z = np.load(path)
    ops = {}
    for tag in ("q", "k", "v", "mask"):
        if f"{tag}_meta" not in z:
            ops[tag] = None
            continue
        meta = z[f"{tag}_meta"]
        st = np.ascontiguousarray(z[f"{tag}_storage"])
        ops[tag] = workloads.Operand(st, int(meta[0]), [int(x) for x in meta[1:5]], [int(x) for x in meta[5:9]],
                                     int(meta[9]))
    scale, max_bias, softcap = [float(x) for x in z["params"]]
    c = workloads.Case(os.path.basename(path), ops["q"], ops["k"], ops["v"], ops["mask"], scale, max_bias, softcap)
    return c, z


GOLDEN_FILES = sorted(glob.glob(os.path.join(GOLDEN, "*.npz")))


def test_golden_fixtures_present():
    assert len(GOLDEN_FILES) >= 6


@pytest.mark.parametrize("path", GOLDEN_FILES, ids=[os.path.basename(p) for p in GOLDEN_FILES])
def test_oracle_reproduces_golden(path):
    c, z = _load_golden(path)
    md = c.mask.host_desc() if c.mask is not None else None
    args = (c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), md, c.scale, c.max_bias, c.softcap)
    assert np.array_equal(oracle.flash_attn_ext(*args, mode=oracle.MODE_EXACT, threads=1), z["out_exact"])
    assert np.array_equal(oracle.flash_attn_ext(*args, mode=oracle.MODE_F32ACC, threads=1), z["out_f32acc"])
    assert np.array_equal(oracle.flash_attn_ext(*args, mode=oracle.MODE_GGML_CPU, threads=1), z["out_ggml_cpu"])
    if "out_torch" in z:
        np.testing.assert_allclose(z["out_exact"], z["out_torch"], atol=1e-6, rtol=0)


def test_prologue_restatement_against_float64():
    """The decode-prologue restatement (rms_norm * w, NEOX rope) against float64 formulas; at small
    positions the float32 angle walk is exact to a few ulps."""
    rng = np.random.default_rng(5)
    x = rng.standard_normal((2, 3, 128)).astype(np.float32) * 2
    w = (1 + 0.1 * rng.standard_normal(128)).astype(np.float32)
    y = oracle.rms_norm_mul(x, w, 1e-6)
    ref = x / np.sqrt((x.astype(np.float64) ** 2).mean(-1, keepdims=True) + 1e-6) * w
    assert np.abs(y - ref).max() <= 2e-6
    pos = np.array([0, 37])
    r = oracle.rope_neox(y, pos, 1e6)
    ts = 1e6 ** (-2 / 128)
    th = pos[:, None] * ts ** np.arange(64)
    c, s = np.cos(th)[:, None], np.sin(th)[:, None]
    ref2 = np.concatenate([y[..., :64] * c - y[..., 64:] * s, y[..., :64] * s + y[..., 64:] * c], -1)
    assert np.abs(r - ref2).max() <= 2e-5
    # position 0 is the identity
    assert np.array_equal(r[0], y[0])


# ---------------------------------------------------------------- ggml's CPU kernel (F16 accumulator)

def _np_ggml_cpu_f16acc(c) -> np.ndarray:
    """numpy statement of ggml-cpu's one-row flash_attn_ext loop for F16 K/V (independent of the
    oracle's C code): Q rounded to f16, F32 dot, expf online softmax, V accumulated in f16 with
    one f32 FMA per key (y <- f16(fma(v, p, y))) and f16(y * ms) on a new maximum."""
    D, n_q, H, n_seq = c.q.ne
    Hk, n_kv = c.k.ne[2], c.k.ne[1]
    q = c.q.storage.reshape(n_seq, H, n_q, D)
    k = c.k.storage.reshape(n_seq, Hk, -1, D)[:, :, :n_kv]
    v = c.v.storage.reshape(n_seq, Hk, -1, D)[:, :, :n_kv]
    m = c.mask.storage.reshape(n_seq, -1, n_kv) if c.mask is not None else None
    out = np.zeros((n_seq, n_q, H, D), np.float32)
    for s in range(n_seq):
        for h in range(H):
            kh = h // (H // Hk)
            for i in range(n_q):
                qf = q[s, h, i].astype(np.float16).astype(np.float32)
                acc = np.zeros(D, np.float16)
                M, S = -np.inf, np.float32(0)
                for j in range(n_kv):
                    mv = np.float32(m[s, i, j]) if m is not None else np.float32(0)
                    if mv == -np.inf:
                        continue
                    sv = np.float32(np.float32(qf @ k[s, kh, j].astype(np.float32)) * np.float32(c.scale)) + mv
                    ms, vs = np.float32(1), np.float32(1)
                    if sv > M:
                        ms = np.float32(0) if M == -np.inf else np.float32(np.exp(np.float32(M - sv)))
                        M = sv
                        acc = (acc.astype(np.float32) * ms).astype(np.float16)
                    else:
                        vs = np.float32(np.exp(np.float32(sv - M)))
                    # f32 FMA emulated in float64 (the f16 x f32 product is exact there)
                    y = (v[s, kh, j].astype(np.float64) * np.float64(vs) + acc.astype(np.float64)).astype(np.float32)
                    acc = y.astype(np.float16)
                    S = np.float32(S * ms + vs)
                out[s, i, h] = acc.astype(np.float32) * (np.float32(1) / S if S > 0 else np.float32(0))
    return out


def test_ggml_cpu_mode_matches_numpy_restatement():
    c = workloads.decode_case(n_seq=2, n_kv=300, n_head=4, n_head_kv=2, n_q=2, kv_len=[300, 171], seed=91)
    got = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                                mode=oracle.MODE_GGML_CPU, threads=2)
    ref = _np_ggml_cpu_f16acc(c)
    # the float64 emulation of the f32 FMA can differ from fmaf by one f32 rounding, rarely
    # moving one f16 rounding of the accumulator; the outputs agree to a fraction of an f16 ulp
    assert np.abs(got - ref).max() <= 2e-4 * np.abs(ref).max()
    # and the F16 accumulator is measurably coarser than the F32 one
    f32 = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                                mode=oracle.MODE_F32ACC, threads=2)
    assert np.abs(got - f32).max() > 1e-6


def test_ggml_cpu_mode_equals_f32_mode_without_f16_v():
    """ggml's CPU kernel accumulates in F32 unless V is F16, so for Q8_0 (and BF16) V the two
    modes are the same computation."""
    c = workloads.decode_case(n_seq=2, n_kv=256, n_head=8, n_head_kv=2, kv_type=ggml.GGML_TYPE_Q8_0, seed=92)
    a = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                              mode=oracle.MODE_GGML_CPU, threads=2)
    b = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                              mode=oracle.MODE_F32ACC, threads=2)
    assert np.array_equal(a, b)


def test_exact_mode_threading_is_deterministic():
    """The exact mode's per-thread slab cache gives the same bits for any thread count."""
    c = workloads.prefill_case(n_seq=1, S=80, n_head=8, n_head_kv=2, kv_pos=30, seed=93)
    a = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                              mode=oracle.MODE_EXACT, threads=1)
    b = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                              mode=oracle.MODE_EXACT, threads=7)
    assert np.array_equal(a, b)


def test_oracle_rejects_unknown_mode():
    c = workloads.decode_case(n_seq=1, n_kv=8, n_head=2, n_head_kv=1, seed=94)
    with pytest.raises(ValueError):
        oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale, mode=9)
