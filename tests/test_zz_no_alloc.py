"""mm3fa_flash_attn_ext_noalloc, the entry point for callers that cannot allocate device
memory (a ggml backend whose buffers were all planned ahead, a graph-recording engine, a
plugin without an allocator): it takes its scratch from an 8 MiB buffer built into
libmm3fa.so instead of a workspace argument.

Checked through the C ABI against the workspace entry point on the same operands, on two
calls in a row (the second call reuses the buffer the first one left behind).  This file is
collected last on purpose, and passes alone in a fresh process as well.
"""
import ctypes
import math

import numpy as np
import pytest
import torch

import mm3fa
from gpu_util import assert_close
from mm3fa import ggml, workloads

pytestmark = pytest.mark.gpu


def _device_operands(c, dev):
    t = {n: torch.from_numpy(np.ascontiguousarray(getattr(c, n).storage)).to(dev)
         for n in ("q", "k", "v", "mask") if getattr(c, n) is not None}
    d = {n: getattr(c, n).device_desc(x) for n, x in t.items()}
    return t, d


@pytest.mark.parametrize("kv_type", [ggml.GGML_TYPE_F16, ggml.GGML_TYPE_Q8_0])
def test_noalloc_matches_workspace_entry_point_twice(cuda_device, kv_type):
    lib = mm3fa.lib()
    c = workloads.decode_case(n_seq=2, n_kv=8192, max_seq=8448, seed=31, kv_type=kv_type,
                              kv_len=[5000, 8190])
    t, d = _device_operands(c, cuda_device)
    need = mm3fa.workspace_size(d["q"], d["k"], d["v"], d["mask"], mm3fa.dst_desc(d["q"], d["v"], 1))
    assert 0 < need <= mm3fa.NOALLOC_SCRATCH_BYTES
    stream = torch.cuda.current_stream().cuda_stream

    ref = torch.empty(c.dst_shape(), device=cuda_device)
    ws = torch.zeros(need, dtype=torch.uint8, device=cuda_device)
    dref = mm3fa.dst_desc(d["q"], d["v"], ref.data_ptr())
    st = lib.mm3fa_flash_attn_ext(ctypes.byref(d["q"]), ctypes.byref(d["k"]), ctypes.byref(d["v"]),
                                  ctypes.byref(d["mask"]), c.scale, 0.0, 0.0, ggml.GGML_PREC_F32, ctypes.byref(dref),
                                  ctypes.c_void_p(ws.data_ptr()), need, ctypes.c_void_p(stream))
    assert st == mm3fa.OK

    outs = []
    for _ in range(2):
        out = torch.full(c.dst_shape(), float("nan"), device=cuda_device)
        dout = mm3fa.dst_desc(d["q"], d["v"], out.data_ptr())
        st = lib.mm3fa_flash_attn_ext_noalloc(ctypes.byref(d["q"]), ctypes.byref(d["k"]), ctypes.byref(d["v"]),
                                              ctypes.byref(d["mask"]), c.scale, 0.0, 0.0, ggml.GGML_PREC_F32,
                                              ctypes.byref(dout), ctypes.c_void_p(stream))
        assert st == mm3fa.OK, mm3fa.status_string(st)
        outs.append(out)
    torch.cuda.synchronize()
    r = ref.cpu().numpy()
    for out in outs:
        assert_close(out.cpu().numpy(), r, what="noalloc vs workspace entry point")


def test_noalloc_rejects_operands_beyond_its_scratch(cuda_device):
    # 32 CFG sequences x 8 kv heads at KV 8192 need more than 8 MiB of split-KV scratch;
    # the operands are real allocations of that size, so nothing could read out of bounds
    n_seq, n_kv, hkv, hq, D = 32, 8192, 8, 32, 128
    k = torch.zeros(n_seq, hkv, n_kv, D, dtype=torch.float16, device=cuda_device)
    v = torch.zeros_like(k)
    q = torch.zeros(n_seq, hq, 1, D, device=cuda_device)
    out = torch.zeros(n_seq, 1, hq, D, device=cuda_device)
    qd, kd, vd = ggml.from_torch(q), ggml.from_torch(k), ggml.from_torch(v)
    dd = mm3fa.dst_desc(qd, vd, out.data_ptr())
    assert mm3fa.workspace_size(qd, kd, vd, None, dd) > mm3fa.NOALLOC_SCRATCH_BYTES
    with pytest.raises(mm3fa.MM3FAError) as e:
        mm3fa.flash_attn_ext_noalloc(qd, kd, vd, None, 1.0 / math.sqrt(D), 0.0, 0.0, dd,
                                     torch.cuda.current_stream().cuda_stream)
    assert e.value.status == mm3fa.ERR_SCRATCH_LIMIT
    torch.cuda.synchronize()
    assert torch.all(out == 0)


def test_noalloc_dense_kernel_after_decode_calls(cuda_device):
    """A causal prefill (the tensor-core kernel, whose mask-block flags also live in the scratch)
    run twice through the built-in buffer right after the decode calls above left their partial
    results in it, compared with the workspace entry point."""
    from gpu_util import run_gpu

    c = workloads.prefill_case(n_seq=2, S=200, n_head=8, n_head_kv=2, kv_pos=37, seed=41)
    ref = run_gpu(c, cuda_device)
    t, d = _device_operands(c, cuda_device)
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):
        out = torch.full(c.dst_shape(), float("nan"), device=cuda_device)
        mm3fa.flash_attn_ext_noalloc(d["q"], d["k"], d["v"], d["mask"], c.scale, 0.0, 0.0,
                                     mm3fa.dst_desc(d["q"], d["v"], out.data_ptr()), stream)
        torch.cuda.synchronize()
        assert_close(out.cpu().numpy(), ref, what="noalloc dense vs workspace entry point")


def test_noalloc_status_reports_an_expired_wait(cuda_device):
    """A bounded wait that expires inside the built-in buffer's user is visible through
    mm3fa_noalloc_status (once), and later no-allocation calls are still correct."""
    stream = torch.cuda.current_stream().cuda_stream
    st, raw = mm3fa.noalloc_status(stream)
    assert st == mm3fa.OK and raw == 0
    assert mm3fa.lib().mm3fa_noalloc_selftest_bounded_wait(20000, ctypes.c_void_p(stream)) == mm3fa.OK
    st, raw = mm3fa.noalloc_status(stream)
    assert st == mm3fa.ERR_TIMEOUT and raw & 1
    st, raw = mm3fa.noalloc_status(stream)
    assert st == mm3fa.OK and raw == 0
    from gpu_util import run_gpu

    c = workloads.decode_case(n_seq=2, n_kv=1024, seed=42)
    t, d = _device_operands(c, cuda_device)
    out = torch.full(c.dst_shape(), float("nan"), device=cuda_device)
    mm3fa.flash_attn_ext_noalloc(d["q"], d["k"], d["v"], d["mask"], c.scale, 0.0, 0.0,
                                 mm3fa.dst_desc(d["q"], d["v"], out.data_ptr()), stream)
    torch.cuda.synchronize()
    assert_close(out.cpu().numpy(), run_gpu(c, cuda_device), what="noalloc after a reported timeout")
    assert mm3fa.noalloc_status(stream) == (mm3fa.OK, 0)
