"""Parity of the CUDA decode path (through the C ABI) against the CPU oracle.

Tolerance (north star, F32 output): max-abs <= 2e-3 and cosine >= 0.99999 against the
oracle's ggml-convention mode, i.e. ggml's own CPU arithmetic.  Against the exact (float64)
oracle the same bound holds for F16/BF16 K; for Q8_0 K the ggml convention itself quantizes
Q to 8 bits, so the exact comparison uses max-abs <= 5e-3, cosine >= 0.9999.
"""
import os

import numpy as np
import pytest
import torch

import mm3fa
import oracle
from gpu_util import assert_close, cosine, run_gpu, run_oracle
from mm3fa import ggml, workloads
from test_oracle import GOLDEN_FILES, _load_golden

pytestmark = pytest.mark.gpu

F16, BF16, Q8 = ggml.GGML_TYPE_F16, ggml.GGML_TYPE_BF16, ggml.GGML_TYPE_Q8_0


@pytest.fixture(params=["auto", "simt", "mma-streamk"])
def kernel(request, monkeypatch):
    """Runs a test on the default dispatch (the tensor-core kernel for F16/BF16 with <= 16 rows
    per unit, split over thread-block clusters when there are enough units), on the CUDA-core
    kernel (MM3FA_DECODE=simt), and on the tensor-core kernel forced onto the stream-K split."""
    if request.param == "mma-streamk":
        monkeypatch.setenv("MM3FA_DECODE", "mma")
        monkeypatch.setenv("MM3FA_DECODE_SPLIT", "streamk")
    else:
        monkeypatch.setenv("MM3FA_DECODE", request.param)
    return request.param


def check(c, dev, exact_abs=2e-3, exact_cos=0.99999):
    """GPU vs the ggml-convention oracle at the north-star tolerance; GPU vs the exact oracle
    at (exact_abs, exact_cos), widened to the ggml convention's own distance from exact math
    when that is larger (Q8_0 with a handful of keys: Q's 8-bit rounding moves the weights)."""
    got = run_gpu(c, dev)
    gg = run_oracle(c, oracle.MODE_GGML)
    ex = run_oracle(c, oracle.MODE_EXACT)
    assert_close(got, gg, what=f"{c.name} vs ggml-convention oracle")
    conv_abs = float(np.abs(gg - ex).max()) if ex.size else 0.0
    conv_cos = cosine(gg, ex)
    assert_close(got, ex, max(exact_abs, 1.25 * conv_abs), min(exact_cos, conv_cos - 1e-6),
                 what=f"{c.name} vs exact oracle")
    return got


def test_config1_decode(kernel, cuda_device):
    """benchmark config 1: CFG B=2, 32q/8kv, D=128, KV 2048, F16 cache view (max_seq 2560)."""
    check(workloads.decode_case(n_seq=2, n_kv=2048, max_seq=2560, seed=1), cuda_device)


def test_headline_decode_kv8192(kernel, cuda_device):
    check(workloads.decode_case(n_seq=2, n_kv=8192, max_seq=10240, seed=2), cuda_device)


def test_config3_q8_0_kv8192(kernel, cuda_device):
    c = workloads.decode_case(n_seq=2, n_kv=8192, kv_type=Q8, seed=3)
    check(c, cuda_device, exact_abs=5e-3, exact_cos=0.9999)


@pytest.mark.parametrize("n_seq,n_kv", [(4, 512), (8, 2048)])
def test_config2_sweep_points(kernel, cuda_device, n_seq, n_kv):
    check(workloads.decode_case(n_seq=n_seq, n_kv=n_kv, kv_std=0.5, seed=40 + n_seq), cuda_device)


def test_ragged_kv_lengths(kernel, cuda_device):
    """Per-sequence kv_len with the reference's -inf padded tail (src/qwen3-lm.h:909-920)."""
    check(workloads.decode_case(n_seq=4, n_kv=2304, kv_len=[1, 700, 2047, 2300], seed=5), cuda_device)


@pytest.mark.parametrize("n_q", [2, 4, 8])
def test_multirow_decode(kernel, cuda_device, n_q):
    check(workloads.decode_case(n_seq=2, n_kv=1024, n_q=n_q, kv_len=[900, 1024], seed=6 + n_q), cuda_device)


@pytest.mark.parametrize("n_kv", [1, 7, 255, 257, 1000])
def test_odd_kv_lengths(kernel, cuda_device, n_kv):
    check(workloads.decode_case(n_seq=2, n_kv=n_kv, seed=100 + n_kv), cuda_device)


@pytest.mark.parametrize("n_kv", [2, 62, 258])
def test_q8_0_small_and_odd(kernel, cuda_device, n_kv):
    check(workloads.decode_case(n_seq=2, n_kv=n_kv, kv_type=Q8, seed=200 + n_kv), cuda_device, 5e-3, 0.9999)


@pytest.mark.parametrize("n_q", [2, 4])
def test_q8_0_multirow_ragged(kernel, cuda_device, n_q):
    """Q8_0 cache with 8 and 16 GQA rows per unit and a -inf padded tail per sequence."""
    c = workloads.decode_case(n_seq=2, n_kv=1536, n_q=n_q, kv_len=[1000, 1536], kv_type=Q8, seed=300 + n_q)
    check(c, cuda_device, 5e-3, 0.9999)


def test_q8_0_softcap_alibi_kv_view(kernel, cuda_device):
    """Q8_0 view into a longer cache (nb2 = max_seq rows), softcap and ALiBi on."""
    c = workloads.decode_case(n_seq=2, n_kv=1280, max_seq=2048, n_head=8, n_head_kv=2, kv_type=Q8, seed=31)
    c.softcap, c.max_bias = 30.0, 4.0
    check(c, cuda_device, 5e-3, 0.9999)


def test_q8_0_odd_length_takes_element_copy_path(cuda_device):
    # 136-byte rows: an odd key count cannot be bulk-copied in 16-byte units
    check(workloads.decode_case(n_seq=2, n_kv=333, kv_type=Q8, seed=7), cuda_device, 5e-3, 0.9999)


def test_padded_rows_take_element_copy_path(cuda_device):
    c = workloads.decode_case(n_seq=2, n_kv=300, seed=8)
    # re-lay K/V with 8 bytes of padding after each 256-byte row (nb1 = 264)
    for name in ("k", "v"):
        op = getattr(c, name)
        st = op.storage  # (s, h, j, 128) f16
        padded = np.zeros(st.shape[:-1] + (132,), dtype=np.float16)
        padded[..., :128] = st
        setattr(c, name, workloads.Operand(padded, F16, op.ne, [2, 264, 264 * st.shape[2], 264 * st.shape[2] * 8]))
    check(c, cuda_device)


@pytest.mark.parametrize("D", [64, 128])
@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
def test_head_dims_and_types(kernel, cuda_device, D, kvt):
    c = workloads.decode_case(n_seq=2, n_kv=640, D=D, n_head=8, n_head_kv=2, seed=9, kv_type=kvt if kvt != BF16
                              else F16)
    if kvt == BF16:
        for name in ("k", "v"):
            op = getattr(c, name)
            bf = torch.from_numpy(op.storage.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
            setattr(c, name, workloads.Operand(bf.view(np.uint16), BF16, op.ne, op.nb))
    if kvt == Q8:
        check(c, cuda_device, 5e-3, 0.9999)
    else:
        check(c, cuda_device)


@pytest.mark.parametrize("ratio", [1, 2, 8, 32])
def test_gqa_ratios(kernel, cuda_device, ratio):
    check(workloads.decode_case(n_seq=2, n_kv=512, n_head=32, n_head_kv=32 // ratio, seed=10 + ratio), cuda_device)


def test_softcap_and_alibi(kernel, cuda_device):
    c = workloads.decode_case(n_seq=2, n_kv=777, n_head=8, n_head_kv=4, seed=11)
    c.softcap, c.max_bias = 25.0, 8.0
    check(c, cuda_device)


def test_f16_query_and_seq_broadcast(kernel, cuda_device):
    c = workloads.decode_case(n_seq=4, n_kv=512, seed=12)
    # Q as F16, and 4 query sequences over 2 kv sequences (ik3 = iq3 / 2)
    q16 = c.q.storage.astype(np.float16)
    c.q = workloads.Operand(q16, F16, c.q.ne, [2, 256, 256, 256 * 32])
    k = c.k
    c.k = workloads.Operand(k.storage, F16, [128, 512, 8, 2], k.nb)
    c.v = workloads.Operand(c.v.storage, F16, [128, 512, 8, 2], c.v.nb)
    check(c, cuda_device)


def test_fully_masked_sequence_gives_zeros(kernel, cuda_device):
    c = workloads.decode_case(n_seq=2, n_kv=1024, seed=13)
    c.mask.storage[1, 0, 0, :] = -np.inf
    got = check(c, cuda_device)
    assert np.all(got[1] == 0.0)


def test_zero_kv_gives_zeros(cuda_device):
    c = workloads.decode_case(n_seq=2, n_kv=64, seed=14)
    for name in ("k", "v"):
        op = getattr(c, name)
        setattr(c, name, workloads.Operand(op.storage, op.gtype, [128, 0, 8, 2], op.nb))
    c.mask = None
    got = run_gpu(c, cuda_device)
    assert np.all(got == 0.0)


def test_prefill_and_dit_shapes(cuda_device):
    check(workloads.prefill_case(n_seq=2, S=96, n_head=8, n_head_kv=2, kv_pos=40, pad=256, seed=15), cuda_device)
    check(workloads.dit_case(B=2, S=130, H=4, D=64, seed=16), cuda_device)


def test_workspace_reuse_is_stable(kernel, cuda_device):
    """Arrival counters reset themselves: repeated calls on one workspace agree exactly."""
    c = workloads.decode_case(n_seq=2, n_kv=4096, seed=17)
    ws = mm3fa.Workspace(cuda_device)
    a = run_gpu(c, cuda_device, ws)
    b = run_gpu(c, cuda_device, ws, repeat=3)
    assert np.array_equal(a, b)
    st, raw = mm3fa.workspace_status(ws.buf.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == mm3fa.OK and raw == 0


@pytest.mark.parametrize("path", GOLDEN_FILES, ids=[os.path.basename(p) for p in GOLDEN_FILES])
def test_golden_fixtures_on_gpu(kernel, cuda_device, path):
    c, z = _load_golden(path)
    got = run_gpu(c, cuda_device)
    assert_close(got, z["out_ggml"], what="vs golden ggml-convention")
    loose = c.k.gtype == Q8
    assert_close(got, z["out_exact"], 5e-3 if loose else 2e-3, 0.9999 if loose else 0.99999, what="vs golden exact")


def test_bounded_wait_reports_timeout(cuda_device):
    """A device wait that nothing satisfies expires after its limit and is reported through
    the workspace status word; the context stays usable."""
    ws = torch.zeros(4096, dtype=torch.uint8, device=cuda_device)
    s = torch.cuda.current_stream().cuda_stream
    assert mm3fa.lib().mm3fa_selftest_bounded_wait(ws.data_ptr(), 20000, s) == mm3fa.OK
    st, raw = mm3fa.workspace_status(ws.data_ptr(), s)
    assert st == mm3fa.ERR_TIMEOUT and raw & 1
    st, raw = mm3fa.workspace_status(ws.data_ptr(), s)
    assert st == mm3fa.OK and raw == 0
    check(workloads.decode_case(n_seq=1, n_kv=256, n_head=8, n_head_kv=2, seed=18), cuda_device)


def test_assemble_heads_matches_numpy(cuda_device):
    from mm3fa.sharding import assemble_heads_np

    G, n_seq, n_q, H, Dv = 4, 3, 2, 32, 128
    g = torch.randn(G, n_seq, n_q, H // G, Dv, device=cuda_device)
    out = torch.empty(n_seq, n_q, H, Dv, device=cuda_device)
    mm3fa.assemble_heads(g.data_ptr(), out.data_ptr(), Dv, H, n_q, n_seq, G, torch.cuda.current_stream().cuda_stream)
    torch.cuda.synchronize()
    assert np.array_equal(out.cpu().numpy(), assemble_heads_np(g.cpu().numpy(), G))


# ---------------------------------------------------------------- device kv_len (no host mask)

def run_gpu_kvlen(c, dev, kv_len, with_mask=False):
    """mm3fa_flash_attn_ext_kvlen on case c: keys past kv_len[s] are invisible to q sequence s."""
    from gpu_util import to_device
    tensors = {n: to_device(getattr(c, n), dev) for n in ("q", "k", "v", "mask") if getattr(c, n) is not None}
    descs = {n: getattr(c, n).device_desc(t) for n, t in tensors.items()}
    out = torch.full(c.dst_shape(), float("nan"), dtype=torch.float32, device=dev)
    dst = mm3fa.dst_desc(descs["q"], descs["v"], out.data_ptr())
    kl = torch.tensor(kv_len, dtype=torch.int32, device=dev)
    md = descs.get("mask") if with_mask else None
    need = mm3fa.workspace_size(descs["q"], descs["k"], descs["v"], md, dst)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    mm3fa.flash_attn_ext_kvlen(descs["q"], descs["k"], descs["v"], md, kl.data_ptr(), c.scale, c.max_bias, c.softcap,
                               dst, ws.data_ptr(), ws.numel(), torch.cuda.current_stream(dev).cuda_stream)
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


def length_mask_case(c, kv_len):
    """The same case with the reference's host-built length mask (src/qwen3-lm.h:909-920)."""
    n_kv, n_q, n_seq = c.k.ne[1], c.q.ne[1], c.q.ne[3]
    m = np.zeros((n_seq, 1, n_q, n_kv), dtype=np.float16)
    for s in range(n_seq):
        m[s, 0, :, max(0, min(kv_len[s], n_kv)):] = -np.inf
    c.mask = workloads.Operand(m, F16, [n_kv, n_q, 1, n_seq], ggml.contiguous_nb(F16, [n_kv, n_q, 1, n_seq]))
    return c


@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
def test_kv_len_equals_length_mask(kernel, cuda_device, kvt):
    """CFG decode over a padded view: the device kv_len gives the result of the reference's mask."""
    kv_len = [1537, 2044]
    c = workloads.decode_case(n_seq=2, n_kv=2048, max_seq=2560, kv_type=kvt if kvt != BF16 else F16, seed=61)
    if kvt == BF16:
        for name in ("k", "v"):
            op = getattr(c, name)
            bf = torch.from_numpy(op.storage.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
            setattr(c, name, workloads.Operand(bf.view(np.uint16), BF16, op.ne, op.nb))
    got = run_gpu_kvlen(c, cuda_device, kv_len)
    ref = run_oracle(length_mask_case(c, kv_len), oracle.MODE_GGML)
    assert_close(got, ref, what="kv_len vs length mask")


def test_kv_len_with_mask_multirow_and_edges(kernel, cuda_device):
    """kv_len combined with a mask, several query rows per sequence, a zero length (zeros) and a
    length past n_kv (clamped)."""
    kv_len = [0, 700, 5000, 333]
    c = workloads.decode_case(n_seq=4, n_kv=1024, n_q=2, kv_len=[1024, 1024, 900, 1024], seed=62)
    got = run_gpu_kvlen(c, cuda_device, kv_len, with_mask=True)
    m = c.mask.storage.copy()
    for s in range(4):
        m[s, :, :, max(0, min(kv_len[s], 1024)):] = -np.inf
    c.mask = workloads.Operand(m, F16, c.mask.ne, c.mask.nb)
    ref = run_oracle(c, oracle.MODE_GGML)
    assert_close(got, ref, what="kv_len + mask vs oracle")
    assert np.all(got[0] == 0)


# ---------------------------------------------------------------- D = 256 (depth decoder heads)

def depth_decoder_case(S: int, B: int, seed: int, kvt=F16):
    """The depth decoder's causal self-attention (src/depth-decoder.h:196-221: 16 heads of 256, no
    RoPE, S <= 8 steps, B = 2N sequences) as a flash_attn_ext call: Q F32 [256, S, 16, B], K/V cast to
    the cache type [256, S, 16, B], causal mask [S, S]."""
    D, H = 256, 16
    rng = np.random.default_rng(seed)
    q = rng.standard_normal((B, S, H, D), dtype=np.float32)
    qop = workloads.Operand(q, ggml.GGML_TYPE_F32, [D, S, H, B], [4, 4 * D * H, 4 * D, 4 * D * H * S])
    kf = rng.standard_normal((B, H, S, D), dtype=np.float32) * 0.5
    vf = rng.standard_normal((B, H, S, D), dtype=np.float32) * 0.5
    ops = []
    for x in (kf, vf):
        if kvt == Q8:
            st = oracle.q8_0_quantize(x)
        else:
            st = oracle.f32_to_f16_bits(x).view(np.float16)
        ops.append(workloads.Operand(st, kvt, [D, S, H, B], ggml.contiguous_nb(kvt, [D, S, H, B])))
    m = np.triu(np.full((S, S), -np.inf, dtype=np.float32), k=1).astype(np.float16)
    mop = workloads.Operand(m, F16, [S, S, 1, 1], ggml.contiguous_nb(F16, [S, S, 1, 1]))
    return workloads.Case("depth", qop, ops[0], ops[1], mop, 1.0 / np.sqrt(D))


@pytest.mark.parametrize("S,B", [(1, 2), (5, 4), (8, 2)])
def test_depth_decoder_d256(cuda_device, S, B):
    check(depth_decoder_case(S, B, seed=70 + S), cuda_device)


def test_depth_decoder_d256_q8_0(cuda_device):
    check(depth_decoder_case(8, 2, seed=79, kvt=Q8), cuda_device, 5e-3, 0.9999)


def test_decode_d256_long_kv(cuda_device):
    """D = 256 over several 32-key stages and the stream-K split (GQA 4, F16 cache view)."""
    check(workloads.decode_case(n_seq=2, n_kv=700, D=256, n_head=8, n_head_kv=2, seed=80), cuda_device)
