"""Parity of the fused decode prologue (mm3fa_decode_prologue) against the oracle's restatement
of ggml's rms_norm, mul, rope_ext (NEOX) and set_rows as src/qwen3-lm.h:764-800 chains them,
and of the attention call that follows it on the updated caches.

Tolerances: q_out (F32) within 1e-4 absolute (float32 arithmetic on both sides; cos/sin may
differ in the last bit); k cache rows within one unit of the cache type's rounding (F16/BF16:
one ulp of the value; Q8_0: one quantum d of the block), because k is normed and rotated in
float32 on both sides first; v cache rows (a plain set_rows conversion of the same F32 input)
bit-identical, as is every other cache row; the
attention output at the north-star bound (max-abs 2e-3, cosine 0.99999) against the oracle run
on the oracle's own prologue results.
"""
import numpy as np
import pytest
import torch

import mm3fa
import oracle
from gpu_util import assert_close
from mm3fa import ggml

pytestmark = pytest.mark.gpu

F32, F16, BF16, Q8 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16, ggml.GGML_TYPE_BF16, ggml.GGML_TYPE_Q8_0


def bf16_bits(x: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(x, dtype=np.float32)).to(torch.bfloat16).view(torch.int16).numpy() \
        .view(np.uint16)


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return torch.from_numpy(np.ascontiguousarray(b).view(np.int16)).view(torch.bfloat16).float().numpy()


def to_cache_bytes(x: np.ndarray, kvt: int) -> np.ndarray:
    """F32 rows [..., D] in the cache type's storage (uint16 per value, or Q8_0 block bytes)."""
    if kvt == F16:
        return oracle.f32_to_f16_bits(x)
    if kvt == BF16:
        return bf16_bits(x)
    return oracle.q8_0_quantize(x)


def cache_to_f32(b: np.ndarray, kvt: int) -> np.ndarray:
    if kvt == F16:
        return oracle.f16_bits_to_f32(b)
    if kvt == BF16:
        return bf16_to_f32(b)
    return oracle.q8_0_dequantize(b)


def run_case(dev, kvt, D, N=2, H=8, Hkv=2, max_seq=300, pos=(123, 8191), rows=(123, 250), seed=0, v_in=None,
             flags=0):
    rng = np.random.default_rng(seed)
    eps, theta = 1e-6, 1e6
    q_in = (rng.standard_normal((N, H, D)) * 3).astype(np.float32)
    k_in = (rng.standard_normal((N, Hkv, D)) * 2).astype(np.float32)
    v_in = rng.standard_normal((N, Hkv, D)).astype(np.float32) if v_in is None else v_in
    q_norm = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    k_norm = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    pos = np.array(pos, dtype=np.int32)
    rows = np.array(rows, dtype=np.int64)
    # caches [N, Hkv, max_seq, D] (ggml [D, max_seq, Hkv, N]) with arbitrary existing rows
    kc0 = to_cache_bytes(rng.standard_normal((N, Hkv, max_seq, D)).astype(np.float32) * 0.5, kvt)
    vc0 = to_cache_bytes(rng.standard_normal((N, Hkv, max_seq, D)).astype(np.float32) * 0.5, kvt)

    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dk, dv = t(q_in), t(k_in), t(v_in)
    dqn, dkn, dpos, drows = t(q_norm), t(k_norm), t(pos), t(rows)
    dkc, dvc = t(kc0), t(vc0)
    dqo = torch.full((N, H, D), float("nan"), dtype=torch.float32, device=dev)
    rb = ggml.row_bytes(kvt, D)
    cnb = [ggml.elem_bytes(kvt), rb, rb * max_seq, rb * max_seq * Hkv]
    mk = lambda ty, ne, tt, nb=None: ggml.make(ty, ne, tt.data_ptr(), nb)
    qd, kd, vd = mk(F32, [D, H, N, 1], dq), mk(F32, [D, Hkv, N, 1], dk), mk(F32, [D, Hkv, N, 1], dv)
    kcd, vcd = mk(kvt, [D, max_seq, Hkv, N], dkc, cnb), mk(kvt, [D, max_seq, Hkv, N], dvc, list(cnb))
    qod = mk(F32, [D, H, N, 1], dqo)
    mm3fa.decode_prologue(qd, kd, vd, dqn.data_ptr(), dkn.data_ptr(), eps, dpos.data_ptr(), theta, drows.data_ptr(),
                          kcd, vcd, qod, torch.cuda.current_stream(dev).cuda_stream, flags=flags)
    torch.cuda.synchronize(dev)

    q_ref, k_ref, v_ref = oracle.decode_prologue(q_in, k_in, v_in, q_norm, k_norm, eps, pos, theta,
                                                 clamp_v=bool(flags & mm3fa.PROLOGUE_CLAMP_FP16))
    kc_ref, vc_ref = kc0.copy(), vc0.copy()
    for s in range(N):
        if 0 <= rows[s] < max_seq:
            kc_ref[s, :, rows[s]] = to_cache_bytes(k_ref[s], kvt)
            vc_ref[s, :, rows[s]] = to_cache_bytes(v_ref[s], kvt)
    return dict(q=dqo.cpu().numpy(), kc=dkc.cpu().numpy(), vc=dvc.cpu().numpy(), q_ref=q_ref, kc_ref=kc_ref,
                vc_ref=vc_ref, kc0=kc0, vc0=vc0, rows=rows, kvt=kvt, D=D, N=N, H=H, Hkv=Hkv, max_seq=max_seq)


def check_rows_close(got: np.ndarray, ref: np.ndarray, kvt: int, what: str):
    g, r = cache_to_f32(got, kvt), cache_to_f32(ref, kvt)
    if kvt == Q8:
        # one quantum of the block: d = max|x| / 127 of the reference block
        d = np.abs(r).reshape(r.shape[:-1] + (-1, 32)).max(-1, keepdims=True) / 127.0
        tol = np.repeat(d, 32, axis=-1).reshape(r.shape) * 1.0001 + 1e-12
    else:
        tol = np.maximum(np.abs(r) * (2.0 ** -10 if kvt == F16 else 2.0 ** -7), 1e-7)
    bad = np.abs(g - r) > tol
    assert not bad.any(), f"{what}: {bad.sum()} values beyond one rounding unit"


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
def test_prologue_matches_oracle(cuda_device, kvt, D):
    r = run_case(cuda_device, kvt, D, seed=D + kvt)
    err = float(np.abs(r["q"] - r["q_ref"]).max())
    assert err <= 1e-4, f"q_out max-abs {err:.3e}"
    for name in ("kc", "vc"):
        got, ref, before = r[name], r[name + "_ref"], r[name + "0"]
        touched = np.zeros(got.shape[:3], dtype=bool)
        for s in range(r["N"]):
            touched[s, :, r["rows"][s]] = True
        assert np.array_equal(got[~touched], before[~touched]), f"{name}: rows other than the new one changed"
        if name == "vc":
            # v goes into the cache with no arithmetic before set_rows: the F16/BF16 cast and the
            # Q8_0 quantization of identical F32 input must give identical bytes
            assert np.array_equal(got[touched], ref[touched]), "v rows: set_rows conversion not bit-exact"
        else:
            check_rows_close(got[touched], ref[touched], kvt, name)


def test_prologue_row_out_of_range_is_not_written(cuda_device):
    r = run_case(cuda_device, F16, 128, rows=(-1, 300), max_seq=300, seed=7)
    assert np.array_equal(r["kc"], r["kc0"]) and np.array_equal(r["vc"], r["vc0"])


@pytest.mark.parametrize("kvt", [F16, Q8])
def test_prologue_then_attention(cuda_device, kvt):
    """The decode step of src/qwen3-lm.h:764-820 at the LM's geometry (32q/8kv, D=128, CFG pair):
    prologue, then flash_attn_ext over rows [0, row] of each set's cache."""
    D, N, H, Hkv, max_seq = 128, 2, 32, 8, 640
    rows = (600, 600)
    r = run_case(cuda_device, kvt, D, N=N, H=H, Hkv=Hkv, max_seq=max_seq, pos=(600, 600), rows=rows, seed=11)
    n_kv = 608  # the padded view the reference attends over; keys past the new row are masked
    mask = np.full((N, 1, 1, n_kv), -np.inf, dtype=np.float16)
    for s in range(N):
        mask[s, 0, 0, :rows[s] + 1] = 0
    rb = ggml.row_bytes(kvt, D)
    cnb = [ggml.elem_bytes(kvt), rb, rb * max_seq, rb * max_seq * Hkv]

    def attend(q, kc, vc, on_gpu):
        if on_gpu:
            dev = cuda_device
            t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
            dq, dk, dv, dm = t(q), t(kc), t(vc), t(mask)
            out = torch.full((N, 1, H, D), float("nan"), dtype=torch.float32, device=dev)
            qd = ggml.make(F32, [D, 1, H, N], dq.data_ptr())
            kd = ggml.make(kvt, [D, n_kv, Hkv, N], dk.data_ptr(), cnb)
            vd = ggml.make(kvt, [D, n_kv, Hkv, N], dv.data_ptr(), list(cnb))
            md = ggml.make(F16, [n_kv, 1, 1, N], dm.data_ptr())
            dd = mm3fa.dst_desc(qd, vd, out.data_ptr())
            ws = mm3fa.Workspace(dev)
            mm3fa.run(qd, kd, vd, md, dd, 1.0 / np.sqrt(D), 0.0, 0.0, ws)
            torch.cuda.synchronize(dev)
            return out.cpu().numpy()
        q = np.ascontiguousarray(q, dtype=np.float32)
        kc, vc = np.ascontiguousarray(kc), np.ascontiguousarray(vc)
        qd = ggml.make(F32, [D, 1, H, N], q.ctypes.data)
        kd = ggml.make(kvt, [D, n_kv, Hkv, N], kc.ctypes.data, cnb)
        vd = ggml.make(kvt, [D, n_kv, Hkv, N], vc.ctypes.data, list(cnb))
        md = ggml.make(F16, [n_kv, 1, 1, N], mask.ctypes.data)
        return oracle.flash_attn_ext(qd, kd, vd, md, 1.0 / np.sqrt(D), 0.0, 0.0, oracle.MODE_F32ACC)

    got = attend(r["q"], r["kc"], r["vc"], True)
    ref = attend(r["q_ref"], r["kc_ref"], r["vc_ref"], False)
    assert_close(got.reshape(ref.shape), ref, what="prologue + attention vs oracle")


# ---------------------------------------------------------------- DiT attention prologue

@pytest.mark.parametrize("out_t", [F16, BF16])
def test_dit_prologue_real_dit_shapes(cuda_device, out_t):
    """The real DiT block (src/dit.h:201-222): 32 heads of 64, S = 690, partial NeoX RoPE over the
    first 32 dims (theta 1e4), k/v cast to F16 (or BF16), then flash_attn_ext over the permuted views."""
    dev = cuda_device
    B, S, H, D, rot, theta = 2, 690, 32, 64, 32, 1e4
    rng = np.random.default_rng(21 + out_t)
    q_in = rng.standard_normal((B, S, H, D)).astype(np.float32)   # ggml [D, H, S, B]
    k_in = rng.standard_normal((B, S, H, D)).astype(np.float32)
    v_in = rng.standard_normal((B, S, H, D)).astype(np.float32)
    pos = np.arange(S, dtype=np.int32)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dq, dk, dv, dpos = t(q_in), t(k_in), t(v_in), t(pos)
    dqo = torch.full((B, S, H, D), float("nan"), dtype=torch.float32, device=dev)
    ko_dtype = torch.float16 if out_t == F16 else torch.bfloat16
    dko = torch.zeros((B, H, S, D), dtype=ko_dtype, device=dev)  # ggml [D, S, H, B]
    dvo = torch.zeros((B, H, S, D), dtype=ko_dtype, device=dev)
    mk = lambda ty, ne, tt: ggml.make(ty, ne, tt.data_ptr())
    mm3fa.dit_prologue(mk(F32, [D, H, S, B], dq), mk(F32, [D, H, S, B], dk), mk(F32, [D, H, S, B], dv),
                       dpos.data_ptr(), rot, theta, mk(F32, [D, H, S, B], dqo), mk(out_t, [D, S, H, B], dko),
                       mk(out_t, [D, S, H, B], dvo), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    pos_bs = np.tile(pos, B)
    q_ref = oracle.rope_neox(q_in.reshape(B * S, H, D), pos_bs, theta, rot).reshape(B, S, H, D)
    k_ref = oracle.rope_neox(k_in.reshape(B * S, H, D), pos_bs, theta, rot).reshape(B, S, H, D)
    err = float(np.abs(dqo.cpu().numpy() - q_ref).max())
    assert err <= 1e-4, f"q_out max-abs {err:.3e}"
    # the dims past rot are copied unchanged
    assert np.array_equal(dqo.cpu().numpy()[..., rot:], q_in[..., rot:])
    k_bits = to_cache_bytes(k_ref.transpose(0, 2, 1, 3), out_t)
    v_bits = to_cache_bytes(v_in.transpose(0, 2, 1, 3), out_t)
    got_k = dko.cpu().view(torch.int16).numpy().view(np.uint16)
    got_v = dvo.cpu().view(torch.int16).numpy().view(np.uint16)
    check_rows_close(got_k, k_bits, out_t, "k_out")
    assert np.array_equal(got_v, v_bits), "v_out is a plain cast"
    # attention over the prologue's outputs vs the oracle over the oracle's
    qv = [4, 4 * D * H, 4 * D, 4 * D * H * S]   # q permuted to [D, S, H, B]
    kvnb = ggml.contiguous_nb(out_t, [D, S, H, B])
    out = torch.full((B, S, H, D), float("nan"), dtype=torch.float32, device=dev)
    qd = ggml.make(F32, [D, S, H, B], dqo.data_ptr(), qv)
    kd = ggml.make(out_t, [D, S, H, B], dko.data_ptr(), kvnb)
    vd = ggml.make(out_t, [D, S, H, B], dvo.data_ptr(), list(kvnb))
    dd = mm3fa.dst_desc(qd, vd, out.data_ptr())
    mm3fa.run(qd, kd, vd, None, dd, 1.0 / np.sqrt(D), 0.0, 0.0, mm3fa.Workspace(dev))
    torch.cuda.synchronize(dev)
    qh = np.ascontiguousarray(q_ref)
    kh, vh = np.ascontiguousarray(k_bits), np.ascontiguousarray(v_bits)
    ref = oracle.flash_attn_ext(ggml.make(F32, [D, S, H, B], qh.ctypes.data, qv),
                                ggml.make(out_t, [D, S, H, B], kh.ctypes.data, kvnb),
                                ggml.make(out_t, [D, S, H, B], vh.ctypes.data, list(kvnb)), None,
                                1.0 / np.sqrt(D), 0.0, 0.0, oracle.MODE_F32ACC)
    assert_close(out.cpu().numpy(), ref, what="DiT prologue + attention vs oracle")


def test_dit_prologue_full_rotation_d128(cuda_device):
    """rot_dims = D at D = 128 (every dim rotated), F16 outputs."""
    dev = cuda_device
    B, S, H, D = 1, 100, 4, 128
    rng = np.random.default_rng(33)
    x = [rng.standard_normal((B, S, H, D)).astype(np.float32) for _ in range(3)]
    pos = (np.arange(S, dtype=np.int32) * 7)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    dx = [t(a) for a in x]
    dpos = t(pos)
    dqo = torch.empty((B, S, H, D), dtype=torch.float32, device=dev)
    dko = torch.empty((B, H, S, D), dtype=torch.float16, device=dev)
    dvo = torch.empty((B, H, S, D), dtype=torch.float16, device=dev)
    mk = lambda ty, ne, tt: ggml.make(ty, ne, tt.data_ptr())
    mm3fa.dit_prologue(mk(F32, [D, H, S, B], dx[0]), mk(F32, [D, H, S, B], dx[1]), mk(F32, [D, H, S, B], dx[2]),
                       dpos.data_ptr(), D, 1e4, mk(F32, [D, H, S, B], dqo), mk(F16, [D, S, H, B], dko),
                       mk(F16, [D, S, H, B], dvo), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    q_ref = oracle.rope_neox(x[0].reshape(B * S, H, D), np.tile(pos, B), 1e4).reshape(B, S, H, D)
    assert float(np.abs(dqo.cpu().numpy() - q_ref).max()) <= 1e-4
    k_ref = oracle.rope_neox(x[1].reshape(B * S, H, D), np.tile(pos, B), 1e4).reshape(B, S, H, D)
    check_rows_close(dko.cpu().view(torch.int16).numpy().view(np.uint16),
                     to_cache_bytes(k_ref.transpose(0, 2, 1, 3), F16), F16, "k_out")


@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
def test_prologue_clamp_fp16(cuda_device, kvt):
    """--clamp-fp16 (src/qwen3-lm.h:779-782): v values beyond the F16 range saturate at +-65504 before
    the cache conversion (NaN passes through); without the flag they round to +-inf in an F16 cache.
    The v rows must equal the oracle's clamp-then-convert bit for bit."""
    N, Hkv, D = 2, 2, 128
    rng = np.random.default_rng(60 + kvt)
    v = rng.standard_normal((N, Hkv, D)).astype(np.float32)
    v[0, 0, :4] = [1e5, -7e4, 65519.0, -3e38]
    v[1, 1, 5] = np.nan if kvt != Q8 else 2e5  # a NaN would poison its whole Q8_0 block scale
    for flags in (mm3fa.PROLOGUE_CLAMP_FP16, 0):
        r = run_case(cuda_device, kvt, D, N=N, Hkv=Hkv, v_in=v.copy(), flags=flags, seed=61)
        got, ref = r["vc"], r["vc_ref"]
        for s_ in range(N):
            row = r["rows"][s_]
            g, w = got[s_, :, row], ref[s_, :, row]
            if kvt == Q8:
                assert np.array_equal(g, w), f"flags={flags} set {s_}: v rows differ"
            else:
                # bit-identical values; a NaN may carry a different payload on each side
                gf, wf = cache_to_f32(g, kvt), cache_to_f32(w, kvt)
                both_nan = np.isnan(gf) & np.isnan(wf)
                assert np.array_equal(g[~both_nan], w[~both_nan]), f"flags={flags} set {s_}: v rows differ"
                assert np.array_equal(np.isnan(gf), np.isnan(wf))
        if kvt == F16:
            vals = oracle.f16_bits_to_f32(got[0, 0, r["rows"][0], :4])
            if flags:
                assert list(vals) == [65504.0, -65504.0, 65504.0, -65504.0]
            else:
                assert np.isinf(vals[0]) and np.isinf(vals[1])
