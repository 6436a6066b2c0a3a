"""Parity of the CUDA decode path (through the C ABI) against the CPU oracle.

Tolerance (north star, F32 output): max-abs <= 2e-3 and cosine >= 0.99999 against the
oracle's F32-accumulation mode (Q rounded to K's vec-dot type, F32 softmax and V sums: the
precision set_prec(F32) asks for).  Against the exact (float64) oracle the same bound holds for
F16/BF16 K; for Q8_0 K the convention itself quantizes Q to 8 bits, so the exact comparison
uses max-abs <= 5e-3, cosine >= 0.9999.  Against the restatement of ggml's CPU kernel, whose
F16 V accumulator is itself ~5e-4 / cos 0.9999 from exact math at KV 8192, the bound is
relative (gpu_util.check_three_ways).
"""
import os

import numpy as np
import pytest
import torch

import mm3fa
import oracle
from gpu_util import assert_close, check_three_ways, cosine, run_gpu, run_oracle
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
    """GPU vs the three oracle modes (gpu_util.check_three_ways): the F32-accumulation oracle at
    the north-star tolerance, the exact oracle at (exact_abs, exact_cos), and ggml's CPU kernel
    (F16 V accumulator) relative to the F32-accumulation mode's own distance from it."""
    got = run_gpu(c, dev)
    check_three_ways(got, c, exact_abs, exact_cos)
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
    assert_close(got, z["out_f32acc"], what="vs golden F32-accumulation")
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
    ref = run_oracle(length_mask_case(c, kv_len), oracle.MODE_F32ACC)
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
    ref = run_oracle(c, oracle.MODE_F32ACC)
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


# ---------------------------------------------------------------- bit-exact single-key rows

def single_key_case(kvt, n_kv: int, seed: int):
    """CFG decode where each row sees exactly one key (key 0; the others, if any, masked -inf).
    softmax over one score is exactly 1, so the result must be V's row 0 converted to F32 bit
    for bit: f16/bf16 -> f32, or the Q8_0 dequantization d * q (an exact product in F32)."""
    c = workloads.decode_case(n_seq=2, n_kv=n_kv, n_head=32, n_head_kv=8, seed=seed,
                              kv_type=Q8 if kvt == Q8 else F16)
    if kvt == BF16:
        for name in ("k", "v"):
            op = getattr(c, name)
            bf = torch.from_numpy(op.storage.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
            setattr(c, name, workloads.Operand(bf.view(np.uint16), BF16, op.ne, op.nb))
    c.mask.storage[..., 1:] = -np.inf
    return c


def v_row0_f32(c) -> np.ndarray:
    """V row 0 of every (sequence, kv head) as F32, broadcast to the result [n_seq, 1, H, D]."""
    st = c.v.storage  # [n_seq, Hkv, max_seq, row]
    if c.v.gtype == Q8:
        rows = oracle.q8_0_dequantize(st[:, :, 0])
    elif c.v.gtype == BF16:
        rows = (st[:, :, 0].astype(np.uint32) << 16).view(np.float32)
    else:
        rows = st[:, :, 0].astype(np.float32)
    ratio = c.q.ne[2] // c.v.ne[2]
    return np.repeat(rows, ratio, axis=1)[:, None]


@pytest.mark.parametrize("kvt", [F16, BF16, Q8])
@pytest.mark.parametrize("n_kv", [1, 2, 256])
def test_single_visible_key_is_bit_exact(kernel, cuda_device, kvt, n_kv):
    """One visible key: out == V row 0 exactly (for Q8_0 this pins the in-kernel dequantization
    d * q bit for bit).  n_kv = 1 runs the element-copy path for Q8_0 (136-byte rows are not
    16-byte multiples), n_kv = 2 and 256 the bulk-copied tensor-core path with masked keys."""
    c = single_key_case(kvt, n_kv, seed=500 + n_kv + kvt)
    got = run_gpu(c, cuda_device)
    want = v_row0_f32(c)
    assert got.shape == want.shape
    assert np.array_equal(got, want), f"max |diff| {np.abs(got - want).max():.3e}"


# ---------------------------------------------------------------- benchmark config 2, large end

@pytest.mark.parametrize("n_seq,n_kv", [(8, 8192), (8, 16384)])
def test_config2_large_end_full_output(kernel, cuda_device, n_seq, n_kv):
    """config 2 at batch 8 (4 CFG pairs) and KV 8192 / 16384 (K/V ~ N(0, 0.25)), every output row
    checked against the three oracle modes."""
    check(workloads.decode_case(n_seq=n_seq, n_kv=n_kv, max_seq=n_kv, kv_std=0.5, seed=45 + n_kv // 1024),
          cuda_device)


def test_config2_36_layer_graph_n8_kv8192(cuda_device):
    """The bench's step at config 2's batch 8: 36 independent layers (F16 caches [128, 10240, 8, 8]
    viewed at KV 8192) captured once in a CUDA graph and replayed twice.  Every layer's replayed
    output equals its eager call bit for bit, and three layers are checked against the oracle."""
    dev = cuda_device
    L, N, Hkv, H, D, n_kv, max_seq = 36, 8, 8, 32, 128, 8192, 10240
    g = torch.Generator(device=dev)
    g.manual_seed(4242)
    F32 = ggml.GGML_TYPE_F32
    rb = 2 * D
    nb = [2, rb, rb * max_seq, rb * max_seq * Hkv]
    mask = torch.zeros(N, 1, 1, n_kv, dtype=torch.float16, device=dev)
    layers = []
    for _ in range(L):
        kc = (torch.randn(N, Hkv, max_seq, D, generator=g, device=dev) * 0.5).half()
        vc = (torch.randn(N, Hkv, max_seq, D, generator=g, device=dev) * 0.5).half()
        q = torch.randn(N, H, 1, D, generator=g, device=dev)
        o = torch.full((N, 1, H, D), float("nan"), device=dev)
        descs = (ggml.make(F32, [D, 1, H, N], q.data_ptr()), ggml.make(F16, [D, n_kv, Hkv, N], kc.data_ptr(), nb),
                 ggml.make(F16, [D, n_kv, Hkv, N], vc.data_ptr(), list(nb)),
                 ggml.make(F16, [n_kv, 1, 1, N], mask.data_ptr()), ggml.make(F32, [D, H, 1, N], o.data_ptr()))
        layers.append(((kc, vc, q, o), descs))
    ws = mm3fa.Workspace(dev)
    s = torch.cuda.Stream(device=dev)

    def step():
        for _, (qd, kd, vd, md, dd) in layers:
            mm3fa.run(qd, kd, vd, md, dd, 1.0 / np.sqrt(D), 0.0, 0.0, ws, stream=s)

    with torch.cuda.stream(s):
        step()
    torch.cuda.synchronize(dev)
    eager = [t[3].cpu().numpy() for t, _ in layers]
    for t, _ in layers:
        t[3].fill_(float("nan"))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        step()
    for _ in range(2):
        with torch.cuda.stream(s):
            graph.replay()
    torch.cuda.synchronize(dev)
    for l, (t, _) in enumerate(layers):
        assert np.array_equal(t[3].cpu().numpy(), eager[l]), f"layer {l}: graph replay differs from the eager call"
    for l in (0, 17, 35):
        kc, vc, q, _ = layers[l][0]
        qn, kn, vn, mn = (x.cpu().numpy() for x in (q, kc, vc, mask))
        c = workloads.Case(f"cfg2-layer{l}", workloads.Operand(qn, F32, [D, 1, H, N], ggml.contiguous_nb(F32, [D, 1, H, N])),
                           workloads.Operand(kn, F16, [D, n_kv, Hkv, N], nb),
                           workloads.Operand(vn, F16, [D, n_kv, Hkv, N], list(nb)),
                           workloads.Operand(mn, F16, [n_kv, 1, 1, N], ggml.contiguous_nb(F16, [n_kv, 1, 1, N])),
                           1.0 / np.sqrt(D))
        check_three_ways(eager[l], c)
    del graph


# ---------------------------------------------------------------- F32 K/V (the depth decoder's attention)

def depth_decoder_f32_case(S: int, B: int, seed: int):
    """The depth decoder's attention exactly as src/depth-decoder.h:205-219 forms it: q, k and v are the
    F32 [D, Nh, S, B] projections viewed as [D, S, Nh, B] (ggml_permute 0,2,1,3: token stride D*Nh*4,
    head stride D*4), D = 256, 16 heads, causal; as a flash_attn_ext call with a causal F16 mask."""
    D, H = 256, 16
    rng = np.random.default_rng(seed)
    ops = []
    for sc in (1.0, 0.5, 0.5):
        x = (rng.standard_normal((B, S, H, D)) * sc).astype(np.float32)  # [D, Nh, S, B] storage
        ops.append(workloads.Operand(x, ggml.GGML_TYPE_F32, [D, S, H, B], [4, 4 * D * H, 4 * D, 4 * D * H * S]))
    m = np.triu(np.full((S, S), -np.inf, dtype=np.float32), k=1).astype(np.float16)
    mop = workloads.Operand(m, F16, [S, S, 1, 1], ggml.contiguous_nb(F16, [S, S, 1, 1]))
    return workloads.Case("depth-f32", ops[0], ops[1], ops[2], mop, 1.0 / np.sqrt(D))


@pytest.mark.parametrize("S,B", [(1, 2), (5, 4), (8, 2), (8, 16)])
def test_depth_decoder_f32_kv(cuda_device, S, B):
    """F32 K/V in the reference's permuted views (element-copy path): no numerics change against the
    F32 manual attention the reference runs."""
    check(depth_decoder_f32_case(S, B, seed=700 + S * B), cuda_device)


@pytest.mark.parametrize("D", [64, 128, 256])
def test_f32_kv_contiguous_long(kernel, cuda_device, D):
    """F32 caches with packed rows (bulk copies), several stages and the stream-K split, GQA 4."""
    c = workloads.decode_case(n_seq=2, n_kv=700, D=D, n_head=8, n_head_kv=2, seed=710 + D)
    for name in ("k", "v"):
        op = getattr(c, name)
        st = op.storage.astype(np.float32)
        setattr(c, name, workloads.Operand(st, ggml.GGML_TYPE_F32, op.ne,
                                           [4, 4 * D, 4 * D * st.shape[2], 4 * D * st.shape[2] * st.shape[1]]))
    check(c, cuda_device)
