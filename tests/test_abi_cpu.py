"""Host-only checks of the C ABI: the library loads, exports every declared entry point,
and its contract checks (mm3fa_supports) accept and reject descriptors as documented.
No kernel is launched here."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

import mm3fa
from mm3fa import ggml, workloads

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "mm3fa.h")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    return sorted(set(re.findall(r"\b(mm3fa_\w+)\s*\(", src)))


def test_header_declares_the_entry_points():
    names = declared_functions()
    for n in ("mm3fa_flash_attn_ext", "mm3fa_workspace_size", "mm3fa_supports", "mm3fa_assemble_heads",
              "mm3fa_status_string", "mm3fa_version"):
        assert n in names


def test_library_exports_every_declared_symbol():
    lib = mm3fa.lib()
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing
    out = subprocess.run(["nm", "-D", "--defined-only", mm3fa.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\b(mm3fa_\w+)\b", out))
    assert set(declared_functions()) <= exported
    # only the C ABI is visible
    assert all(n.startswith("mm3fa_") for n in exported)


def test_struct_layout_matches_header():
    assert ctypes.sizeof(ggml.Tensor) == 4 + 4 + 32 + 32 + 8
    assert ggml.Tensor.data.offset == 72


def test_version_and_status_strings():
    assert mm3fa.version()[0] == 1
    assert mm3fa.status_string(0) == "ok"
    assert "workspace" in mm3fa.status_string(mm3fa.ERR_WORKSPACE)
    assert mm3fa.status_string(12345) == "unknown status"


def _decode_descs(**kw):
    c = workloads.decode_case(**kw)
    q, k, v, m = c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc()
    d = mm3fa.dst_desc(q, v, 0x1000)
    return c, q, k, v, m, d


def test_supports_accepts_reference_layouts():
    _, q, k, v, m, d = _decode_descs(n_seq=2, n_kv=512, max_seq=1024)
    assert mm3fa.supports(q, k, v, m, d) == mm3fa.OK
    assert mm3fa.supports(q, k, v, None, d) == mm3fa.OK
    _, q, k, v, m, d = _decode_descs(n_seq=2, n_kv=256, kv_type=ggml.GGML_TYPE_Q8_0)
    assert mm3fa.supports(q, k, v, m, d) == mm3fa.OK
    c = workloads.prefill_case(n_seq=1, S=16, n_head=4, n_head_kv=2, pad=32)
    q, k, v, m = c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc()
    assert mm3fa.supports(q, k, v, m, mm3fa.dst_desc(q, v, 0x1000)) == mm3fa.OK
    c = workloads.dit_case(B=2, S=20, H=4, D=64)
    q, k, v = c.q.host_desc(), c.k.host_desc(), c.v.host_desc()
    assert mm3fa.supports(q, k, v, None, mm3fa.dst_desc(q, v, 0x1000)) == mm3fa.OK


def test_supports_rejections():
    _, q, k, v, m, d = _decode_descs(n_seq=2, n_kv=128)
    assert mm3fa.supports(None, k, v, m, d) == mm3fa.ERR_NULL
    bad = ggml.make(ggml.GGML_TYPE_F32, list(k.ne), k.data, [4, 512, 512 * 128, 512 * 128 * 8])
    assert mm3fa.supports(q, bad, v, m, d) == mm3fa.ERR_TYPE  # F32 K with F16 V
    assert mm3fa.supports(q, k, v, m, ggml.make(ggml.GGML_TYPE_F16, list(d.ne), 0x1000)) == mm3fa.ERR_TYPE
    wrong_dst = ggml.make(ggml.GGML_TYPE_F32, [128, 1, 32, 2], 0x1000)  # rows before heads
    assert mm3fa.supports(q, k, v, m, wrong_dst) == mm3fa.ERR_SHAPE
    short_mask = ggml.make(ggml.GGML_TYPE_F16, [64, 1, 1, 2], m.data)
    assert mm3fa.supports(q, k, v, short_mask, d) == mm3fa.ERR_SHAPE
    q7 = ggml.make(q.type, [128, 1, 28, 2], q.data)  # 28 heads over 8 kv heads
    assert mm3fa.supports(q7, k, v, m, mm3fa.dst_desc(q7, v, 0x1000)) == mm3fa.ERR_SHAPE
    transposed_k = ggml.make(k.type, list(k.ne), k.data, [256, 2, 256 * 128, 256 * 128 * 8])
    assert mm3fa.supports(q, transposed_k, v, m, d) == mm3fa.ERR_STRIDE
    q96 = ggml.make(q.type, [96, 1, 32, 2], q.data)
    k96 = ggml.make(k.type, [96, 128, 8, 2], k.data)
    v96 = ggml.make(v.type, [96, 128, 8, 2], v.data)
    assert mm3fa.supports(q96, k96, v96, m, mm3fa.dst_desc(q96, v96, 0x1000)) == mm3fa.ERR_UNSUPPORTED
    assert mm3fa.supports(q, k, v, m, d, max_bias=-1.0) == mm3fa.ERR_SHAPE
    assert mm3fa.supports(q, k, v, m, d, logit_softcap=float("nan")) == mm3fa.ERR_SHAPE


def test_flash_attn_ext_rejects_before_touching_the_device():
    _, q, k, v, m, d = _decode_descs(n_seq=2, n_kv=128)
    with pytest.raises(mm3fa.MM3FAError) as e:
        mm3fa.flash_attn_ext(q, k, v, m, 0.1, 0.0, 0.0, ggml.make(ggml.GGML_TYPE_F16, list(d.ne), 0x1000), 0, 0)
    assert e.value.status == mm3fa.ERR_TYPE
    with pytest.raises(mm3fa.MM3FAError) as e:
        mm3fa.flash_attn_ext(q, k, v, m, 0.1, 0.0, 0.0, d, 0, 0, prec=3)
    assert e.value.status == mm3fa.ERR_UNSUPPORTED
    with pytest.raises(mm3fa.MM3FAError) as e:
        mm3fa.assemble_heads(0, 0, 128, 32, 1, 2, 4)
    assert e.value.status == mm3fa.ERR_NULL


def test_descriptor_helpers_roundtrip():
    a = np.zeros((3, 5, 7, 64), dtype=np.float32)
    t = ggml.from_numpy(a)
    assert list(t.ne) == [64, 7, 5, 3] and list(t.nb) == [4, 256, 256 * 7, 256 * 35]
    b = np.zeros((2, 3, 136), dtype=np.uint8)
    t = ggml.from_numpy(b, ggml.GGML_TYPE_Q8_0)
    assert list(t.ne) == [128, 3, 2, 1] and list(t.nb) == [34, 136, 408, 816]


def _status(fn, *args, **kw):
    with pytest.raises(mm3fa.MM3FAError) as e:
        fn(*args, **kw)
    return e.value.status


def test_prologue_entry_points_reject_before_touching_the_device():
    F32, F16, Q8 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16, ggml.GGML_TYPE_Q8_0
    D, H, Hkv, N, S = 128, 32, 8, 2, 64
    q = ggml.make(F32, [D, H, N, 1], 0x1000)
    k = ggml.make(F32, [D, Hkv, N, 1], 0x2000)
    v = ggml.make(F32, [D, Hkv, N, 1], 0x3000)
    kc = ggml.make(F16, [D, 512, Hkv, N], 0x4000)
    vc = ggml.make(F16, [D, 512, Hkv, N], 0x5000)
    qo = ggml.make(F32, [D, H, N, 1], 0x6000)
    args = lambda **o: [o.get("q", q), o.get("k", k), v, 0x7000, 0x7100, 1e-6, 0x7200, 1e6, 0x7300,
                        o.get("kc", kc), vc, qo]
    assert _status(mm3fa.decode_prologue, q, k, v, 0, 0x7100, 1e-6, 0x7200, 1e6, 0x7300, kc, vc, qo) == mm3fa.ERR_NULL
    assert _status(mm3fa.decode_prologue, *args(kc=ggml.make(F32, [D, 512, Hkv, N], 0x4000))) == mm3fa.ERR_TYPE
    assert _status(mm3fa.decode_prologue, *args(kc=ggml.make(Q8, [D, 512, Hkv, N], 0x4000))) == mm3fa.ERR_TYPE  # v F16
    assert _status(mm3fa.decode_prologue, *args(q=ggml.make(F32, [96, H, N, 1], 0x1000))) == mm3fa.ERR_UNSUPPORTED
    assert _status(mm3fa.decode_prologue, *args(k=ggml.make(F32, [D, Hkv, N + 1, 1], 0x2000))) == mm3fa.ERR_SHAPE
    # DiT prologue: [D, H, S, B] in, [D, S, H, B] out
    qi = ggml.make(F32, [64, 32, S, 2], 0x1000)
    ko = ggml.make(F16, [64, S, 32, 2], 0x4000)
    vo = ggml.make(F16, [64, S, 32, 2], 0x5000)
    assert _status(mm3fa.dit_prologue, qi, qi, qi, 0x7000, 30, 1e4, qi, ko, vo) == mm3fa.ERR_SHAPE  # rot % 4
    v_heads_first = ggml.make(F16, [64, 32, S, 2], 0x5000)  # v_out not [D, S, H, B]
    assert _status(mm3fa.dit_prologue, qi, qi, qi, 0x7000, 32, 1e4, qi, ko, v_heads_first) == mm3fa.ERR_SHAPE
    assert _status(mm3fa.dit_prologue, qi, qi, qi, 0, 32, 1e4, qi, ko, vo) == mm3fa.ERR_NULL
    assert _status(mm3fa.dit_prologue, qi, qi, qi, 0x7000, 32, 1e4, qi, ko,
                   ggml.make(Q8, [64, S, 32, 2], 0x5000)) == mm3fa.ERR_TYPE
    # kv_len attention: the kv_len pointer is required; the operands are checked as usual
    _, q4, k4, v4, m4, d4 = _decode_descs(n_seq=2, n_kv=128)
    assert _status(mm3fa.flash_attn_ext_kvlen, q4, k4, v4, m4, 0, 0.1, 0.0, 0.0, d4, 0, 0) == mm3fa.ERR_NULL
    assert _status(mm3fa.flash_attn_ext_kvlen, q4, k4, v4, m4, 0x8000, 0.1, 0.0, 0.0,
                   ggml.make(F16, list(d4.ne), 0x1000), 0, 0) == mm3fa.ERR_TYPE


def test_exchange_entry_points_reject_before_touching_the_device():
    """mm3fa_allgather_heads / _flash_attn_ext_peers / _peer_wait / _flash_attn_ext_gather /
    _gather_signal_wait / IPC helpers: argument checks that need neither a GPU nor NCCL."""
    L = mm3fa.lib()
    vp = ctypes.c_void_p
    # allgather: null pointers, bad split, null communicator
    assert L.mm3fa_allgather_heads(None, None, vp(0x2000), 128, 32, 1, 2, 1, vp(0x9000), None) == mm3fa.ERR_NULL
    assert L.mm3fa_allgather_heads(vp(0x1000), None, vp(0x2000), 128, 32, 1, 2, 1, None, None) == mm3fa.ERR_NULL
    assert L.mm3fa_allgather_heads(vp(0x1000), None, vp(0x2000), 128, 32, 1, 3, 2, vp(0x9000), None) == \
        mm3fa.ERR_SHAPE
    assert L.mm3fa_allgather_heads(vp(0x1000), None, vp(0x2000), 128, 32, 1, 2, 0, vp(0x9000), None) == \
        mm3fa.ERR_SHAPE
    assert L.mm3fa_allgather_heads(vp(0x1002), None, vp(0x2000), 128, 32, 1, 2, 1, vp(0x9000), None) == \
        mm3fa.ERR_ALIGN
    # fused exchange: peers table checks
    _, q4, k4, v4, m4, d4 = _decode_descs(n_seq=2, n_kv=128)
    peers = mm3fa.Peers()
    peers.n_ranks, peers.rank = 1, 0
    st = lambda pr, **kw: _status(mm3fa.flash_attn_ext_peers, q4, k4, v4, m4, 0.1, kw.get("max_bias", 0.0), 0.0, d4,
                                  0x8000, 4096, pr, kw.get("slot", 0), kw.get("epochs", 0x7000))
    assert st(peers) == mm3fa.ERR_SHAPE  # one rank
    peers.n_ranks, peers.rank = 2, 2
    assert st(peers) == mm3fa.ERR_SHAPE  # rank out of range
    peers.rank = 1
    assert st(peers) == mm3fa.ERR_NULL  # buffers missing
    for r in range(2):
        peers.recv[r] = 0x100000 * (r + 1)
    peers.recv_slot_bytes = 1 << 20
    assert st(peers, slot=-1) == mm3fa.ERR_SHAPE
    assert st(peers, epochs=0) == mm3fa.ERR_NULL
    assert st(peers, epochs=0x7002) == mm3fa.ERR_ALIGN
    peers.recv[1] = 0x200008
    assert st(peers) == mm3fa.ERR_ALIGN
    peers.recv[1] = 0x200000
    peers.recv_slot_bytes = 1000
    assert st(peers) == mm3fa.ERR_SHAPE  # slot size not a multiple of 16
    peers.recv_slot_bytes = 1 << 20
    assert st(peers, max_bias=8.0) == mm3fa.ERR_UNSUPPORTED  # ALiBi needs the global head index
    assert L.mm3fa_flash_attn_ext_peers(ctypes.byref(q4), ctypes.byref(k4), ctypes.byref(v4), ctypes.byref(m4), None,
                                        0.1, 0.0, 0.0, 10, ctypes.byref(d4), vp(0x8000), 4096, None, 0, vp(0x7000),
                                        None) == mm3fa.ERR_NULL
    # wait: table, epochs, result
    res = ggml.make(ggml.GGML_TYPE_F32, [128, 32, 1, 2], 0x300000)
    assert L.mm3fa_peer_wait(ctypes.byref(peers), 0, None, ctypes.byref(res), vp(0x8000), None) == mm3fa.ERR_NULL
    bad = mm3fa.Peers()
    bad.n_ranks, bad.rank = 9, 0
    assert L.mm3fa_peer_wait(ctypes.byref(bad), 0, vp(0x7000), ctypes.byref(res), vp(0x8000), None) == mm3fa.ERR_SHAPE
    odd = ggml.make(ggml.GGML_TYPE_F32, [128, 31, 1, 2], 0x300000)  # heads do not split over 2 ranks
    assert L.mm3fa_peer_wait(ctypes.byref(peers), 0, vp(0x7000), ctypes.byref(odd), vp(0x8000), None) == \
        mm3fa.ERR_SHAPE
    peers.recv_slot_bytes = 1024  # smaller than 2 ranks x 2 parities x the slice's words
    assert L.mm3fa_peer_wait(ctypes.byref(peers), 0, vp(0x7000), ctypes.byref(res), vp(0x8000), None) == \
        mm3fa.ERR_WORKSPACE
    # fused dense exchange: results table, dst placement, ALiBi; the signal-wait's table and slot
    res = mm3fa.Peers()
    res.n_ranks, res.rank = 2, 0
    base = 0x400000
    dd = ggml.make(ggml.GGML_TYPE_F32, [128, 32, 1, 2], base + 4096)
    g = lambda pr, dst=dd, mb=0.0: L.mm3fa_flash_attn_ext_gather(ctypes.byref(q4), ctypes.byref(k4), ctypes.byref(v4),
                                                                  ctypes.byref(m4), 0.1, mb, 0.0, 10, ctypes.byref(dst),
                                                                  vp(0x8000), 4096, pr, None)
    assert g(None) == mm3fa.ERR_NULL
    assert g(ctypes.byref(res)) == mm3fa.ERR_NULL  # result buffers missing
    res.recv[0], res.recv[1] = base, base + 0x100000
    res.recv_slot_bytes = 0x10000
    res.n_ranks = 9
    assert g(ctypes.byref(res)) == mm3fa.ERR_SHAPE
    res.n_ranks = 2
    res.recv[1] = base + 0x100004
    assert g(ctypes.byref(res)) == mm3fa.ERR_ALIGN
    res.recv[1] = base + 0x100000
    below = ggml.make(ggml.GGML_TYPE_F32, [128, 32, 1, 2], base - 512)  # dst starts before the rank's result
    assert g(ctypes.byref(res), below) == mm3fa.ERR_SHAPE
    res.recv_slot_bytes = 4096 + 128 * 32 * 2 * 4 - 4  # dst's last row ends past the result
    assert g(ctypes.byref(res)) == mm3fa.ERR_SHAPE
    res.recv_slot_bytes = 0x10000
    assert g(ctypes.byref(res), mb=8.0) == mm3fa.ERR_UNSUPPORTED
    fl = mm3fa.Peers()
    fl.n_ranks, fl.rank = 2, 1
    fl.recv[0], fl.recv[1] = 0x500000, 0x600000
    fl.recv_slot_bytes = 2 * 2 * 4  # two slots of two ranks' words
    sw = lambda pr, slot=0, ep=0x7000, ws=0x8000: L.mm3fa_gather_signal_wait(pr, slot, vp(ep), vp(ws), None)
    assert sw(None) == mm3fa.ERR_NULL
    assert sw(ctypes.byref(fl), ep=0) == mm3fa.ERR_NULL
    assert sw(ctypes.byref(fl), slot=2) == mm3fa.ERR_SHAPE  # past the flag array
    assert sw(ctypes.byref(fl), slot=-1) == mm3fa.ERR_SHAPE
    assert sw(ctypes.byref(fl), ep=0x7002) == mm3fa.ERR_ALIGN
    fl.recv[0] = 0x500002
    assert sw(ctypes.byref(fl)) == mm3fa.ERR_ALIGN
    # IPC helpers
    h = mm3fa.IpcHandle()
    assert L.mm3fa_ipc_export(None, ctypes.byref(h)) == mm3fa.ERR_NULL
    assert L.mm3fa_ipc_open(None, ctypes.byref(ctypes.c_void_p())) == mm3fa.ERR_NULL
    assert L.mm3fa_ipc_close(None) == mm3fa.ERR_NULL
    assert ctypes.sizeof(mm3fa.Peers) == 8 + 8 * 8 + 8 and ctypes.sizeof(mm3fa.IpcHandle) == 72
