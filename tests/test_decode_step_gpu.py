"""mm3fa_decode_step (the decode prologue and the attention in one call) against the same step
run as two calls (mm3fa_decode_prologue, then mm3fa_flash_attn_ext on q_out) and against the
oracle (its restatement of ggml's rms_norm / mul / rope_ext / set_rows, then the attention on the
updated caches), at the LM's decode geometry (32q/8kv, D=128, CFG pair).

Tolerances: caches bit-identical to the two-call path (rows other than the new one untouched);
q_out within 1e-4 absolute of it; the attention output at the north-star bound (max-abs 2e-3,
cosine 0.99999) against both references.
"""
import numpy as np
import pytest
import torch

import mm3fa
import oracle
from gpu_util import assert_close
from mm3fa import ggml
from test_prologue_gpu import to_cache_bytes

pytestmark = pytest.mark.gpu

F32, F16, BF16, Q8 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16, ggml.GGML_TYPE_BF16, ggml.GGML_TYPE_Q8_0


def step_case(dev, kvt, rows, n_kv=1024, max_seq=1100, seed=0):
    D, N, H, Hkv = 128, 2, 32, 8
    rng = np.random.default_rng(seed)
    eps, theta = 1e-6, 1e6
    q_in = (rng.standard_normal((N, H, D)) * 3).astype(np.float32)
    k_in = (rng.standard_normal((N, Hkv, D)) * 2).astype(np.float32)
    v_in = rng.standard_normal((N, Hkv, D)).astype(np.float32)
    q_norm = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    k_norm = (1 + 0.2 * rng.standard_normal(D)).astype(np.float32)
    pos = np.array([max(int(r), 0) for r in rows], dtype=np.int32)
    rows = np.array(rows, dtype=np.int64)
    kc0 = to_cache_bytes(rng.standard_normal((N, Hkv, max_seq, D)).astype(np.float32) * 0.5, kvt)
    vc0 = to_cache_bytes(rng.standard_normal((N, Hkv, max_seq, D)).astype(np.float32) * 0.5, kvt)
    mask = np.zeros((N, 1, 1, n_kv), dtype=np.float16)
    mask[:, :, :, n_kv - 7:] = -np.inf  # a padded tail, as the reference's decode mask has
    rb = ggml.row_bytes(kvt, D)
    cnb = [ggml.elem_bytes(kvt), rb, rb * max_seq, rb * max_seq * Hkv]
    scale = 1.0 / np.sqrt(D)
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    stream = torch.cuda.current_stream(dev).cuda_stream

    def run(fused: bool):
        dq, dk, dv = t(q_in), t(k_in), t(v_in)
        dqn, dkn, dpos, drows, dm = t(q_norm), t(k_norm), t(pos), t(rows), t(mask)
        dkc, dvc = t(kc0), t(vc0)
        dqo = torch.full((N, H, D), float("nan"), dtype=torch.float32, device=dev)
        out = torch.full((N, 1, H, D), float("nan"), dtype=torch.float32, device=dev)
        mk = lambda ty, ne, tt, nb=None: ggml.make(ty, ne, tt.data_ptr(), nb)
        qd, kd, vd = mk(F32, [D, H, N, 1], dq), mk(F32, [D, Hkv, N, 1], dk), mk(F32, [D, Hkv, N, 1], dv)
        kcd, vcd = mk(kvt, [D, max_seq, Hkv, N], dkc, cnb), mk(kvt, [D, max_seq, Hkv, N], dvc, list(cnb))
        qod = mk(F32, [D, H, N, 1], dqo)
        qa = mk(F32, [D, 1, H, N], dqo, [4, 4 * D, 4 * D, 4 * D * H])
        ka, va = mk(kvt, [D, n_kv, Hkv, N], dkc, cnb), mk(kvt, [D, n_kv, Hkv, N], dvc, list(cnb))
        md = mk(F16, [n_kv, 1, 1, N], dm)
        dd = mm3fa.dst_desc(qa, va, out.data_ptr())
        ws_bytes = max(mm3fa.workspace_size(qa, ka, va, md, dd), 256)
        ws = torch.zeros(ws_bytes, dtype=torch.uint8, device=dev)
        if fused:
            mm3fa.decode_step(qd, kd, vd, dqn.data_ptr(), dkn.data_ptr(), eps, dpos.data_ptr(), theta,
                              drows.data_ptr(), kcd, vcd, qod, ka, va, md, scale, 0.0, 0.0, dd, ws.data_ptr(),
                              ws_bytes, stream)
        else:
            mm3fa.decode_prologue(qd, kd, vd, dqn.data_ptr(), dkn.data_ptr(), eps, dpos.data_ptr(), theta,
                                  drows.data_ptr(), kcd, vcd, qod, stream)
            mm3fa.flash_attn_ext(qa, ka, va, md, scale, 0.0, 0.0, dd, ws.data_ptr(), ws_bytes, stream)
        torch.cuda.synchronize(dev)
        return dqo.cpu().numpy(), dkc.cpu().numpy(), dvc.cpu().numpy(), out.cpu().numpy()

    fused = run(True)
    split = run(False)
    # oracle: its prologue, then its attention over the view of the updated caches
    q_ref, k_ref, v_ref = oracle.decode_prologue(q_in, k_in, v_in, q_norm, k_norm, eps, pos, theta)
    kc_ref, vc_ref = kc0.copy(), vc0.copy()
    for s in range(N):
        if 0 <= rows[s] < max_seq:
            kc_ref[s, :, rows[s]] = to_cache_bytes(k_ref[s], kvt)
            vc_ref[s, :, rows[s]] = to_cache_bytes(v_ref[s], kvt)
    qh = np.ascontiguousarray(q_ref, dtype=np.float32)  # [N, H, D]: the [D, 1, H, N] view
    kh, vh, mh = np.ascontiguousarray(kc_ref), np.ascontiguousarray(vc_ref), np.ascontiguousarray(mask)
    qdh = ggml.make(F32, [D, 1, H, N], qh.ctypes.data, [4, 4 * D, 4 * D, 4 * D * H])
    kdh = ggml.make(kvt, [D, n_kv, Hkv, N], kh.ctypes.data, cnb)
    vdh = ggml.make(kvt, [D, n_kv, Hkv, N], vh.ctypes.data, list(cnb))
    mdh = ggml.make(F16, [n_kv, 1, 1, N], mh.ctypes.data)
    ref = oracle.flash_attn_ext(qdh, kdh, vdh, mdh, scale, 0.0, 0.0, oracle.MODE_F32ACC)
    return fused, split, ref


@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
@pytest.mark.parametrize("rows", [(1016, 1016), (5, 700), (1030, -1)],
                         ids=["last-visible", "first-chunk-and-middle", "outside-view-and-none"])
def test_decode_step_matches_two_calls_and_oracle(cuda_device, kvt, rows):
    (qf, kcf, vcf, of), (qs, kcs, vcs, os_), ref = step_case(cuda_device, kvt, rows, seed=3 + kvt)
    assert np.array_equal(kcf, kcs), "K cache differs from the two-call path"
    assert np.array_equal(vcf, vcs), "V cache differs from the two-call path"
    err = float(np.abs(qf - qs).max())
    assert err <= 1e-4, f"q_out max-abs {err:.3e} vs the two-call path"
    assert_close(of.reshape(ref.shape), os_.reshape(ref.shape), what="fused step vs two calls")
    assert_close(of.reshape(ref.shape), ref, what="fused step vs oracle")


def test_decode_step_repeat_is_bit_identical(cuda_device):
    a = step_case(cuda_device, F16, (1016, 1016), seed=5)[0]
    b = step_case(cuda_device, F16, (1016, 1016), seed=5)[0]
    for x, y in zip(a, b):
        assert np.array_equal(x, y)


def test_decode_step_rejects_before_launching(cuda_device):
    """A rejected attention operand (here: no workspace) leaves the caches and q_out untouched."""
    dev = cuda_device
    D, N, H, Hkv, max_seq, n_kv = 128, 2, 32, 8, 64, 64
    t = lambda a: torch.from_numpy(np.ascontiguousarray(a)).to(dev)
    z = lambda *shape: torch.zeros(*shape, dtype=torch.float32, device=dev)
    q_in, k_in, v_in, qn, kn = z(N, H, D), z(N, Hkv, D), z(N, Hkv, D), z(D) + 1, z(D) + 1
    pos, rows = t(np.zeros(N, np.int32)), t(np.zeros(N, np.int64))
    kc = torch.full((N, Hkv, max_seq, D), 7.0, device=dev).half()
    vc = kc.clone()
    qo = torch.full((N, H, D), 3.0, device=dev)
    out = z(N, 1, H, D)
    cnb = [2, 2 * D, 2 * D * max_seq, 2 * D * max_seq * Hkv]
    mk = lambda ty, ne, tt, nb=None: ggml.make(ty, ne, tt.data_ptr(), nb)
    qa = mk(F32, [D, 1, H, N], qo, [4, 4 * D, 4 * D, 4 * D * H])
    ka, va = mk(F16, [D, n_kv, Hkv, N], kc, cnb), mk(F16, [D, n_kv, Hkv, N], vc, list(cnb))
    dd = mm3fa.dst_desc(qa, va, out.data_ptr())
    with pytest.raises(mm3fa.MM3FAError):
        mm3fa.decode_step(mk(F32, [D, H, N, 1], q_in), mk(F32, [D, Hkv, N, 1], k_in), mk(F32, [D, Hkv, N, 1], v_in),
                          qn.data_ptr(), kn.data_ptr(), 1e-6, pos.data_ptr(), 1e6, rows.data_ptr(),
                          mk(F16, [D, max_seq, Hkv, N], kc, cnb), mk(F16, [D, max_seq, Hkv, N], vc, list(cnb)),
                          mk(F32, [D, H, N, 1], qo), ka, va, None, 1.0 / np.sqrt(D), 0.0, 0.0, dd, 0, 0,
                          torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    assert bool((kc == 7.0).all()) and bool((vc == 7.0).all()) and bool((qo == 3.0).all())
