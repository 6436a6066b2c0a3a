"""Parity of the tensor-core prefill / DiT kernel (tcgen05 + TMEM + TMA, fa_dense_sm100.cu),
through the C ABI, against the CPU oracle.

Same tolerance as the decode path (north star, F32 output): max-abs <= 2e-3 and cosine >= 0.99999
against the oracle's ggml-convention mode.  Shapes the oracle cannot finish in seconds are
checked on a seeded sample of query rows: every row of GGML_OP_FLASH_ATTN_EXT is independent,
so the oracle runs on a Q (and mask) holding just those rows.
"""
import numpy as np
import pytest
import torch

import mm3fa
import oracle
from gpu_util import assert_close, check_three_ways, run_gpu, run_oracle
from mm3fa import ggml, workloads
from test_decode_gpu import check

pytestmark = pytest.mark.gpu

F16, BF16, F32 = ggml.GGML_TYPE_F16, ggml.GGML_TYPE_BF16, ggml.GGML_TYPE_F32


@pytest.fixture(params=["dense", "dense-nosplit"])
def dense(request, monkeypatch):
    """Forces the tensor-core prefill kernel wherever the operands allow it; small launches then
    split every work item over a 2-CTA cluster (DSMEM merge), "dense-nosplit" runs each item in one
    CTA (MM3FA_DENSE_SPLIT=0)."""
    monkeypatch.setenv("MM3FA_DENSE", "1")
    if request.param == "dense-nosplit":
        monkeypatch.setenv("MM3FA_DENSE_SPLIT", "0")
    return request.param


def row_subset(c: workloads.Case, rows: np.ndarray) -> workloads.Case:
    """The same operation restricted to query rows `rows` (Q storage laid out [B, S, H, D])."""
    q = c.q
    assert q.gtype == F32 and q.storage.ndim == 4
    qs = np.ascontiguousarray(q.storage[:, rows])
    B, n, H, D = qs.shape
    qop = workloads.Operand(qs, F32, [D, n, H, B], [4, 4 * D * H, 4 * D, 4 * D * H * n])
    mop = None
    if c.mask is not None:
        ms = np.ascontiguousarray(c.mask.storage[rows])
        mop = workloads.Operand(ms, c.mask.gtype, [c.mask.ne[0], n, 1, 1],
                                ggml.contiguous_nb(c.mask.gtype, [c.mask.ne[0], n, 1, 1]))
    return workloads.Case(c.name + "-rows", qop, c.k, c.v, mop, c.scale, c.max_bias, c.softcap)


def check_rows(c: workloads.Case, dev, n_rows: int = 48, seed: int = 0):
    got = run_gpu(c, dev)
    S = c.q.ne[1]
    rng = np.random.default_rng(seed)
    rows = np.unique(np.concatenate([[0, S - 1], rng.choice(S, size=min(n_rows, S), replace=False)]))
    sub = row_subset(c, rows)
    ref = run_oracle(sub, oracle.MODE_F32ACC)
    assert_close(got[:, rows], ref, what=f"{c.name} rows vs F32-accumulation oracle")
    return got


_ORACLE_CACHE: dict = {}


def check_full(c: workloads.Case, dev, key: str):
    """Every output row against the three oracle modes; oracle results cached under `key`."""
    got = run_gpu(c, dev)
    _ORACLE_CACHE[key] = check_three_ways(got, c, refs=_ORACLE_CACHE.get(key))
    return got


def to_bf16(c: workloads.Case) -> workloads.Case:
    for name in ("k", "v"):
        op = getattr(c, name)
        bf = torch.from_numpy(op.storage.astype(np.float32)).to(torch.bfloat16).view(torch.int16).numpy()
        setattr(c, name, workloads.Operand(bf.view(np.uint16), BF16, op.ne, op.nb, op.offset))
    return c


# ---------------------------------------------------------------- LM prefill (causal mask)

@pytest.mark.parametrize("S,kv_pos", [(96, 40), (128, 0), (300, 0), (200, 1000)])
def test_prefill_causal(dense, cuda_device, S, kv_pos):
    """Causal prefill over the padded cache view: tiles past the diagonal are skipped, the
    diagonal tiles take the mask, a partial last query tile and the -inf padded tail."""
    check(workloads.prefill_case(n_seq=2, S=S, n_head=8, n_head_kv=2, kv_pos=kv_pos, seed=300 + S), cuda_device)


@pytest.mark.parametrize("H,HKV", [(4, 4), (6, 2), (4, 2), (16, 2)])
def test_prefill_head_layouts(dense, cuda_device, H, HKV):
    """GQA ratios that take the head-pair work items (2, 8: two query heads of one kv group per
    CTA, same rows) and those that do not (1: MHA, 3: odd), over several query blocks."""
    check(workloads.prefill_case(n_seq=2, S=300, n_head=H, n_head_kv=HKV, kv_pos=20, seed=340 + 10 * H + HKV),
          cuda_device)


def test_prefill_pair_alibi(dense, cuda_device):
    """ALiBi on head-pair items: each Q tile of a CTA takes its own head's slope."""
    c = workloads.prefill_case(n_seq=1, S=256, n_head=8, n_head_kv=2, kv_pos=8, seed=351)
    c.max_bias = 8.0
    check(c, cuda_device)


def test_prefill_per_head_mask(dense, cuda_device):
    """A mask plane per query head (m_ne2 = n_head) keeps one head per CTA: the causal mask with a
    finite per-head bias on the first column (so the diagonal and first tiles are general mixed
    tiles, not step rows)."""
    c = workloads.prefill_case(n_seq=1, S=260, n_head=8, n_head_kv=2, kv_pos=0, seed=352)
    m = c.mask.storage  # [S, n_kv_pad]
    S, nkv = m.shape
    H = 8
    mh = np.repeat(m[None], H, axis=0).copy()  # [H, S, n_kv_pad]
    for h in range(H):
        mh[h, :, 0] = np.float16(-0.5 * (h % 3))
    c.mask = workloads.Operand(mh, ggml.GGML_TYPE_F16, [nkv, S, H, 1],
                               ggml.contiguous_nb(ggml.GGML_TYPE_F16, [nkv, S, H, 1]))
    check(c, cuda_device)


def test_prefill_config4_full(dense, cuda_device):
    """benchmark config 4 at full size (2 x 1024 tokens, 32q/8kv, D=128, causal): 256 work items,
    more than one wave, every output row checked."""
    check_full(workloads.prefill_case(n_seq=2, S=1024, n_head=32, n_head_kv=8, seed=312), cuda_device, "cfg4")


def test_prefill_qwen3_heads(dense, cuda_device):
    """Qwen3-8B geometry (32 q heads over 8 kv heads, D=128), one 512-token prompt chunk."""
    check_full(workloads.prefill_case(n_seq=1, S=512, n_head=32, n_head_kv=8, seed=310), cuda_device, "qwen3-512")


def test_prefill_long_replay(dense, cuda_device):
    """A long teacher-forced prefill (the replay path runs the LM over thousands of frames): one
    sequence of 4096 tokens after 200 cached ones (a 4352-row padded view), sampled rows."""
    check_rows(workloads.prefill_case(n_seq=1, S=4096, n_head=32, n_head_kv=8, kv_pos=200, seed=313), cuda_device,
               n_rows=64)


def test_prefill_auto_dispatch(cuda_device, monkeypatch):
    """The default dispatch takes the tensor-core prefill kernel from 64 query rows on; the
    decode kernels (MM3FA_DENSE=0) agree with it."""
    c = workloads.prefill_case(n_seq=2, S=160, n_head=8, n_head_kv=2, kv_pos=16, seed=311)
    monkeypatch.delenv("MM3FA_DENSE", raising=False)
    a = check(c, cuda_device)
    monkeypatch.setenv("MM3FA_DENSE", "0")
    b = run_gpu(c, cuda_device)
    assert_close(a, b, what="dense vs decode kernels")


# ---------------------------------------------------------------- DiT (no mask)

@pytest.mark.parametrize("S,H,D", [(130, 4, 64), (256, 2, 128), (1, 2, 64), (127, 3, 128)])
def test_dit_shapes(dense, cuda_device, S, H, D):
    check(workloads.dit_case(B=2, S=S, H=H, D=D, seed=320 + S), cuda_device)


def test_dit_real_model(dense, cuda_device):
    """The real DiT attention: S=690 latent frames, 32 heads, D=64, CFG batch 2."""
    check_full(workloads.dit_case(B=2, S=690, H=32, D=64, seed=330), cuda_device, "dit-real")


def test_dit_config5_full(dense, cuda_device):
    """benchmark config 5 (S=4096, H=16, D=128, B=2), every output row checked."""
    check_full(workloads.dit_case(B=2, S=4096, H=16, D=128, seed=331), cuda_device, "cfg5")


# ---------------------------------------------------------------- operand variants

@pytest.mark.parametrize("D", [64, 128])
def test_bf16_kv(dense, cuda_device, D):
    """BF16 K/V: the tensor-core PV needs P in K/V's type, so P carries bf16 rounding (8-bit
    mantissa) that ggml's CPU path (P in F32) does not; against the ggml convention the north-star
    bound holds, against exact math the bound is that of the 8-bit Q8_0 case."""
    check(to_bf16(workloads.dit_case(B=1, S=200, H=4, D=D, seed=340 + D)), cuda_device, 5e-3, 0.9999)
    check(to_bf16(workloads.prefill_case(n_seq=1, S=150, n_head=4, n_head_kv=2, D=D, kv_pos=30, seed=342 + D)),
          cuda_device, 5e-3, 0.9999)


@pytest.mark.parametrize("ratio", [1, 4, 8])
def test_gqa_ratios(dense, cuda_device, ratio):
    check(workloads.prefill_case(n_seq=1, S=140, n_head=2 * ratio, n_head_kv=2, kv_pos=8, seed=350 + ratio),
          cuda_device)


def test_softcap_and_alibi(dense, cuda_device):
    c = workloads.prefill_case(n_seq=2, S=130, n_head=8, n_head_kv=4, kv_pos=5, seed=360)
    c.softcap, c.max_bias = 30.0, 8.0
    check(c, cuda_device)


def test_causal_mask_with_some_biased_rows(dense, cuda_device):
    """Step rows (zeros, then -inf) take a column bound on their mixed tiles; a warp with any other
    row (here: finite biases in a few rows) takes the general masked pass for the same tile."""
    c = workloads.prefill_case(n_seq=2, S=300, n_head=8, n_head_kv=2, kv_pos=37, seed=365)
    m = c.mask.storage  # [S, n_kv_pad] f16, shared by heads and sequences
    m[40, :20] = 0.5
    m[290, 5] = -1.25
    check(c, cuda_device)


def test_random_mask_per_head(dense, cuda_device):
    """A non-causal mask with a plane per (head, sequence): random -inf holes, finite biases,
    whole -inf blocks (skipped) and whole zero blocks (no mask arithmetic)."""
    rng = np.random.default_rng(370)
    c = workloads.dit_case(B=2, S=260, H=4, D=64, seed=371)
    n_kv, S = c.k.ne[1], c.q.ne[1]
    m = rng.standard_normal((2, 4, S, n_kv)).astype(np.float16)
    m[rng.random(m.shape) < 0.3] = -np.inf
    m[:, :, :128, 128:256] = -np.inf  # a skipped block
    m[:, :, 128:256, :128] = 0        # a block without mask arithmetic
    m[0, 1, 7, :] = -np.inf           # a row without any visible key -> zeros
    c.mask = workloads.Operand(m, F16, [n_kv, S, 4, 2], ggml.contiguous_nb(F16, [n_kv, S, 4, 2]))
    got = check(c, cuda_device)
    assert np.all(got[0, 7, 1] == 0)


def test_f16_query_and_unaligned_rows(dense, cuda_device):
    """F16 Q, and Q/dst rows whose starts are not 16-byte aligned (element loads/stores)."""
    c = workloads.dit_case(B=1, S=140, H=2, D=64, seed=380)
    qf = c.q.storage.astype(np.float16)  # [B, S, H, D]
    c.q = workloads.Operand(qf, F16, c.q.ne, [2, 2 * 64 * 2, 2 * 64, 2 * 64 * 2 * 140])
    check(c, cuda_device)
    # F32 Q with 4 bytes of padding after each row: nb1 = 260, rows 4-byte aligned only
    c = workloads.dit_case(B=1, S=140, H=2, D=64, seed=381)
    q = c.q.storage  # [1, 140, 2, 64]
    pad = np.zeros((1, 140, 2, 65), dtype=np.float32)
    pad[..., :64] = q
    c.q = workloads.Operand(pad, F32, [64, 140, 2, 1], [4, 4 * 65 * 2, 4 * 65, 4 * 65 * 2 * 140])
    check(c, cuda_device)


@pytest.mark.parametrize("n_kv", [1, 5, 127, 129])
def test_short_kv(dense, cuda_device, n_kv):
    """Fewer keys than one tile, or one more: keys past n_kv are masked inside the kernel."""
    rng = np.random.default_rng(390 + n_kv)
    S, H, D = 150, 2, 128
    c = workloads.dit_case(B=1, S=S, H=H, D=D, seed=391)
    k = rng.standard_normal((1, H, n_kv, D)).astype(np.float16)
    v = rng.standard_normal((1, H, n_kv, D)).astype(np.float16)
    nb = ggml.contiguous_nb(F16, [D, n_kv, H, 1])
    c.k = workloads.Operand(k, F16, [D, n_kv, H, 1], nb)
    c.v = workloads.Operand(v, F16, [D, n_kv, H, 1], list(nb))
    check(c, cuda_device)


def test_fully_masked_prefill_gives_zeros(dense, cuda_device):
    c = workloads.prefill_case(n_seq=1, S=130, n_head=4, n_head_kv=2, seed=395)
    c.mask.storage[:] = -np.inf
    got = run_gpu(c, cuda_device)
    assert np.all(got == 0)


def test_repeat_calls_bit_identical(dense, cuda_device):
    c = workloads.prefill_case(n_seq=2, S=200, n_head=8, n_head_kv=2, kv_pos=60, seed=396)
    ws = mm3fa.Workspace(cuda_device)
    a = run_gpu(c, cuda_device, ws)
    b = run_gpu(c, cuda_device, ws, repeat=3)
    assert np.array_equal(a, b)
    st, raw = mm3fa.workspace_status(ws.buf.data_ptr(), torch.cuda.current_stream().cuda_stream)
    assert st == mm3fa.OK and raw == 0


def test_padded_destination_rows(dense, cuda_device):
    """A result view whose rows are not 16-byte aligned takes the element-store epilogue instead
    of the TMA store; both write exactly ggml's [Dv, H, n_q, S] view."""
    c = workloads.dit_case(B=1, S=200, H=2, D=64, seed=397)
    dev = cuda_device
    q = torch.from_numpy(np.ascontiguousarray(c.q.storage)).to(dev)
    k = torch.from_numpy(np.ascontiguousarray(c.k.storage)).to(dev)
    v = torch.from_numpy(np.ascontiguousarray(c.v.storage)).to(dev)
    store = torch.full((1, 200, 2, 65), float("nan"), dtype=torch.float32, device=dev)  # one pad float per row
    dst = ggml.make(F32, [64, 2, 200, 1], store.data_ptr(), [4, 4 * 65, 4 * 65 * 2, 4 * 65 * 2 * 200])
    mm3fa.run(c.q.device_desc(q), c.k.device_desc(k), c.v.device_desc(v), None, dst, c.scale)
    torch.cuda.synchronize(dev)
    got = store[..., :64].cpu().numpy()
    assert np.all(np.isnan(store[..., 64].cpu().numpy())), "padding was written"
    assert_close(got, run_oracle(c, oracle.MODE_F32ACC), what="padded dst vs F32-accumulation oracle")
