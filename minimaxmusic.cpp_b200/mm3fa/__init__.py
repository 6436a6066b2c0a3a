"""mm3fa: B200 (sm_100a) GGML_OP_FLASH_ATTN_EXT behind a C ABI (include/mm3fa.h).

Host-side mirror of the reference's operator interface.  The reference builds the op as

    attn = ggml_flash_attn_ext(ctx, q, k, v, mask, scale, max_bias, logit_softcap)
    ggml_flash_attn_ext_set_prec(attn, GGML_PREC_F32)

(src/qwen3-lm.h:432-436, :816-820; src/dit.h:221-222).  `flash_attn_ext` here takes the
same operands - ggml tensor descriptors of device memory, see `mm3fa.ggml` - plus the
caller-owned workspace and stream, and raises `MM3FAError` where ggml would assert.

The compute always runs in libmm3fa.so (CUDA); there is no CPU path.  If the library is
missing or fails to load, every call raises.
"""
from __future__ import annotations

import ctypes
import os

from . import ggml
from .ggml import (GGML_PREC_DEFAULT, GGML_PREC_F32, GGML_TYPE_BF16, GGML_TYPE_F16, GGML_TYPE_F32,  # noqa: F401
                   GGML_TYPE_Q8_0, Tensor)

_PKG = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB_PATH = os.path.join(_PKG, "lib", "libmm3fa.so")

OK = 0
ERR_NULL, ERR_TYPE, ERR_SHAPE, ERR_STRIDE, ERR_ALIGN = 1, 2, 3, 4, 5
ERR_WORKSPACE, ERR_CUDA, ERR_UNSUPPORTED, ERR_TIMEOUT, ERR_DEVICE = 6, 7, 8, 9, 10
ERR_SCRATCH_LIMIT = 11
ERR_COMM = 12

MAX_RANKS = 8


class Peers(ctypes.Structure):
    """struct mm3fa_peers: every rank's receive buffer mapped here, and the bytes of one slot."""
    _fields_ = [("n_ranks", ctypes.c_int32), ("rank", ctypes.c_int32), ("recv", ctypes.c_void_p * MAX_RANKS),
                ("recv_slot_bytes", ctypes.c_uint64)]


class IpcHandle(ctypes.Structure):
    """struct mm3fa_ipc_handle."""
    _fields_ = [("handle", ctypes.c_ubyte * 64), ("offset", ctypes.c_uint64)]

# size of the fixed scratch buffer behind flash_attn_ext_noalloc (MM3FA_NOALLOC_SCRATCH_BYTES)
NOALLOC_SCRATCH_BYTES = 8 << 20

_lib = None


class MM3FAError(RuntimeError):
    def __init__(self, status: int, what: str = ""):
        self.status = status
        msg = f"mm3fa status {status}: {status_string(status)}"
        if status == ERR_CUDA:
            msg += f" ({lib().mm3fa_last_cuda_error().decode()})"
        if what:
            msg = f"{what}: {msg}"
        super().__init__(msg)


def lib():
    """The loaded libmm3fa.so (raises if it has not been built)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"{LIB_PATH} is missing: run python minimaxmusic.cpp_b200/build.py")
        L = ctypes.CDLL(LIB_PATH)
        P = ctypes.POINTER(Tensor)
        L.mm3fa_flash_attn_ext.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_float, ctypes.c_float, ctypes.c_int,
                                           P, ctypes.c_void_p, ctypes.c_size_t, ctypes.c_void_p]
        L.mm3fa_flash_attn_ext.restype = ctypes.c_int
        L.mm3fa_workspace_size.argtypes = [P, P, P, P, P]
        L.mm3fa_workspace_size.restype = ctypes.c_size_t
        L.mm3fa_supports.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_float, P]
        L.mm3fa_supports.restype = ctypes.c_int
        L.mm3fa_status_string.argtypes = [ctypes.c_int]
        L.mm3fa_status_string.restype = ctypes.c_char_p
        L.mm3fa_last_cuda_error.argtypes = []
        L.mm3fa_last_cuda_error.restype = ctypes.c_char_p
        L.mm3fa_version.restype = ctypes.c_int
        L.mm3fa_assemble_heads.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.c_int64, ctypes.c_int64,
                                           ctypes.c_int64, ctypes.c_int64, ctypes.c_int, ctypes.c_void_p]
        L.mm3fa_assemble_heads.restype = ctypes.c_int
        L.mm3fa_workspace_status.argtypes = [ctypes.c_void_p, ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
        L.mm3fa_workspace_status.restype = ctypes.c_int
        L.mm3fa_selftest_bounded_wait.argtypes = [ctypes.c_void_p, ctypes.c_uint32, ctypes.c_void_p]
        L.mm3fa_selftest_bounded_wait.restype = ctypes.c_int
        L.mm3fa_flash_attn_ext_noalloc.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                   ctypes.c_int, P, ctypes.c_void_p]
        L.mm3fa_flash_attn_ext_noalloc.restype = ctypes.c_int
        L.mm3fa_noalloc_status.argtypes = [ctypes.c_void_p, ctypes.POINTER(ctypes.c_uint32)]
        L.mm3fa_noalloc_status.restype = ctypes.c_int
        L.mm3fa_noalloc_selftest_bounded_wait.argtypes = [ctypes.c_uint32, ctypes.c_void_p]
        L.mm3fa_noalloc_selftest_bounded_wait.restype = ctypes.c_int
        L.mm3fa_decode_prologue.argtypes = [P, P, P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float,
                                            ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p, P, P, P,
                                            ctypes.c_void_p]
        L.mm3fa_decode_prologue.restype = ctypes.c_int
        L.mm3fa_decode_prologue_ex.argtypes = L.mm3fa_decode_prologue.argtypes[:-1] + [ctypes.c_uint32,
                                                                                        ctypes.c_void_p]
        L.mm3fa_decode_prologue_ex.restype = ctypes.c_int
        L.mm3fa_decode_step.argtypes = [P, P, P, ctypes.c_void_p, ctypes.c_void_p, ctypes.c_float, ctypes.c_void_p,
                                        ctypes.c_float, ctypes.c_void_p, P, P, P, P, P, P, ctypes.c_float,
                                        ctypes.c_float, ctypes.c_float, ctypes.c_int, P, ctypes.c_void_p,
                                        ctypes.c_size_t, ctypes.c_void_p]
        L.mm3fa_decode_step.restype = ctypes.c_int
        L.mm3fa_decode_step_ex.argtypes = L.mm3fa_decode_step.argtypes[:-1] + [ctypes.c_uint32, ctypes.c_void_p]
        L.mm3fa_decode_step_ex.restype = ctypes.c_int
        L.mm3fa_flash_attn_ext_kvlen.argtypes = [P, P, P, P, ctypes.c_void_p, ctypes.c_float, ctypes.c_float,
                                                 ctypes.c_float, ctypes.c_int, P, ctypes.c_void_p, ctypes.c_size_t,
                                                 ctypes.c_void_p]
        L.mm3fa_flash_attn_ext_kvlen.restype = ctypes.c_int
        L.mm3fa_dit_prologue.argtypes = [P, P, P, ctypes.c_void_p, ctypes.c_int, ctypes.c_float, P, P, P,
                                         ctypes.c_void_p]
        L.mm3fa_dit_prologue.restype = ctypes.c_int
        vp, i64 = ctypes.c_void_p, ctypes.c_int64
        L.mm3fa_allgather_heads.argtypes = [vp, vp, vp, i64, i64, i64, i64, ctypes.c_int, vp, vp]
        L.mm3fa_allgather_heads.restype = ctypes.c_int
        L.mm3fa_flash_attn_ext_peers.argtypes = [P, P, P, P, vp, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                 ctypes.c_int, P, vp, ctypes.c_size_t, ctypes.POINTER(Peers),
                                                 ctypes.c_int, vp, vp]
        L.mm3fa_flash_attn_ext_peers.restype = ctypes.c_int
        L.mm3fa_peer_wait.argtypes = [ctypes.POINTER(Peers), ctypes.c_int, vp, P, vp, vp]
        L.mm3fa_peer_wait.restype = ctypes.c_int
        L.mm3fa_flash_attn_ext_gather.argtypes = [P, P, P, P, ctypes.c_float, ctypes.c_float, ctypes.c_float,
                                                  ctypes.c_int, P, vp, ctypes.c_size_t, ctypes.POINTER(Peers), vp]
        L.mm3fa_flash_attn_ext_gather.restype = ctypes.c_int
        L.mm3fa_gather_signal_wait.argtypes = [ctypes.POINTER(Peers), ctypes.c_int, vp, vp, vp]
        L.mm3fa_gather_signal_wait.restype = ctypes.c_int
        L.mm3fa_ipc_export.argtypes = [vp, ctypes.POINTER(IpcHandle)]
        L.mm3fa_ipc_export.restype = ctypes.c_int
        L.mm3fa_ipc_open.argtypes = [ctypes.POINTER(IpcHandle), ctypes.POINTER(ctypes.c_void_p)]
        L.mm3fa_ipc_open.restype = ctypes.c_int
        L.mm3fa_ipc_close.argtypes = [vp]
        L.mm3fa_ipc_close.restype = ctypes.c_int
        _lib = L
    return _lib


def status_string(status: int) -> str:
    return lib().mm3fa_status_string(status).decode()


def version() -> tuple[int, int]:
    v = lib().mm3fa_version()
    return v >> 16, v & 0xFFFF


def _ref(t):
    return ctypes.byref(t) if t is not None else None


def supports(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, dst: Tensor, max_bias: float = 0.0,
             logit_softcap: float = 0.0) -> int:
    """Status mm3fa_flash_attn_ext would return for these descriptors (0 = accepted)."""
    return lib().mm3fa_supports(_ref(q), _ref(k), _ref(v), _ref(mask), max_bias, logit_softcap, _ref(dst))


def workspace_size(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, dst: Tensor) -> int:
    return int(lib().mm3fa_workspace_size(_ref(q), _ref(k), _ref(v), _ref(mask), _ref(dst)))


def dst_desc(q: Tensor, v: Tensor, data_ptr: int) -> Tensor:
    """Contiguous F32 result descriptor [Dv, n_head, n_q, n_seq] (ggml_flash_attn_ext's)."""
    return ggml.make(GGML_TYPE_F32, [v.ne[0], q.ne[2], q.ne[1], q.ne[3]], data_ptr)


def flash_attn_ext(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, scale: float, max_bias: float,
                   logit_softcap: float, dst: Tensor, workspace: int, workspace_bytes: int, stream: int = 0,
                   prec: int = GGML_PREC_F32) -> None:
    """Enqueues the op on `stream` (a cudaStream_t as int).  Raises MM3FAError on rejection."""
    st = lib().mm3fa_flash_attn_ext(_ref(q), _ref(k), _ref(v), _ref(mask), scale, max_bias, logit_softcap, prec,
                                    _ref(dst), ctypes.c_void_p(workspace or None), workspace_bytes,
                                    ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_flash_attn_ext")


def flash_attn_ext_noalloc(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, scale: float, max_bias: float,
                           logit_softcap: float, dst: Tensor, stream: int = 0, prec: int = GGML_PREC_F32) -> None:
    """flash_attn_ext for callers that cannot allocate device memory.

    The scratch comes from a fixed 8 MiB buffer inside libmm3fa.so rather than a workspace
    argument, for hosts that may not call cudaMalloc where attention runs (a backend whose
    buffers were planned ahead, a graph-recording engine, a plugin without an allocator).
    Operands needing more scratch raise MM3FAError(ERR_SCRATCH_LIMIT).  The first call on a
    device looks the buffer up and should come before any stream capture; calls that can
    overlap on the GPU share the buffer and race.
    """
    st = lib().mm3fa_flash_attn_ext_noalloc(_ref(q), _ref(k), _ref(v), _ref(mask), scale, max_bias, logit_softcap,
                                            prec, _ref(dst), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_flash_attn_ext_noalloc")


def noalloc_status(stream: int = 0) -> tuple[int, int]:
    """(status, raw bits) of the built-in no-allocation buffer's status word, read and cleared
    (MM3FA_ERR_TIMEOUT when a bounded wait of an earlier no-allocation call expired)."""
    raw = ctypes.c_uint32(0)
    st = lib().mm3fa_noalloc_status(ctypes.c_void_p(stream or None), ctypes.byref(raw))
    return st, raw.value


def flash_attn_ext_kvlen(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, kv_len_ptr: int, scale: float,
                         max_bias: float, logit_softcap: float, dst: Tensor, workspace: int, workspace_bytes: int,
                         stream: int = 0, prec: int = GGML_PREC_F32) -> None:
    """flash_attn_ext where q sequence s sees keys [0, kv_len[s]) (kv_len: device int32 [n_seq])."""
    st = lib().mm3fa_flash_attn_ext_kvlen(_ref(q), _ref(k), _ref(v), _ref(mask), ctypes.c_void_p(kv_len_ptr), scale,
                                          max_bias, logit_softcap, prec, _ref(dst), ctypes.c_void_p(workspace or None),
                                          workspace_bytes, ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_flash_attn_ext_kvlen")


def dit_prologue(q_in: Tensor, k_in: Tensor, v_in: Tensor, pos_ptr: int, rot_dims: int, rope_theta: float,
                 q_out: Tensor, k_out: Tensor, v_out: Tensor, stream: int = 0) -> None:
    """DiT attention prologue: partial NeoX RoPE of q/k and the F16/BF16 cast of k/v ([D, S, H, B])."""
    st = lib().mm3fa_dit_prologue(_ref(q_in), _ref(k_in), _ref(v_in), ctypes.c_void_p(pos_ptr), rot_dims,
                                  rope_theta, _ref(q_out), _ref(k_out), _ref(v_out), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_dit_prologue")


PROLOGUE_CLAMP_FP16 = 1  # MM3FA_PROLOGUE_CLAMP_FP16: clamp v to +-65504 before the cache conversion


def decode_prologue(q_in: Tensor, k_in: Tensor, v_in: Tensor, q_norm_ptr: int, k_norm_ptr: int, eps: float,
                    pos_ptr: int, rope_theta: float, rows_ptr: int, k_cache: Tensor, v_cache: Tensor, q_out: Tensor,
                    stream: int = 0, flags: int = 0) -> None:
    """Fused decode prologue (RMSNorm + NeoX RoPE of q and k, append of the new k/v rows into the caches);
    pointers are device addresses (q_norm/k_norm F32 [D], pos int32 [N], rows int64 [N]).
    flags: PROLOGUE_CLAMP_FP16 adds the reference's --clamp-fp16 clamp of v."""
    st = lib().mm3fa_decode_prologue_ex(_ref(q_in), _ref(k_in), _ref(v_in), ctypes.c_void_p(q_norm_ptr),
                                        ctypes.c_void_p(k_norm_ptr), eps, ctypes.c_void_p(pos_ptr), rope_theta,
                                        ctypes.c_void_p(rows_ptr), _ref(k_cache), _ref(v_cache), _ref(q_out), flags,
                                        ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_decode_prologue")


def decode_step(q_in: Tensor, k_in: Tensor, v_in: Tensor, q_norm_ptr: int, k_norm_ptr: int, eps: float,
                pos_ptr: int, rope_theta: float, rows_ptr: int, k_cache: Tensor, v_cache: Tensor, q_out: Tensor,
                k: Tensor, v: Tensor, mask: Tensor | None, scale: float, max_bias: float, logit_softcap: float,
                dst: Tensor, workspace: int, workspace_bytes: int, stream: int = 0,
                prec: int = GGML_PREC_F32, flags: int = 0) -> None:
    """decode_prologue followed by flash_attn_ext on q_out viewed as [D, 1, n_head, N], as one call
    (two kernels on the stream, the attention's CTAs starting as the prologue's exit)."""
    st = lib().mm3fa_decode_step_ex(_ref(q_in), _ref(k_in), _ref(v_in), ctypes.c_void_p(q_norm_ptr),
                                    ctypes.c_void_p(k_norm_ptr), eps, ctypes.c_void_p(pos_ptr), rope_theta,
                                    ctypes.c_void_p(rows_ptr), _ref(k_cache), _ref(v_cache), _ref(q_out), _ref(k),
                                    _ref(v), _ref(mask), scale, max_bias, logit_softcap,
                                    prec, _ref(dst), ctypes.c_void_p(workspace or None), workspace_bytes, flags,
                                    ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_decode_step")


def assemble_heads(gathered_ptr: int, dst_ptr: int, dv: int, n_head: int, n_q: int, n_seq: int, n_ranks: int,
                   stream: int = 0) -> None:
    st = lib().mm3fa_assemble_heads(ctypes.c_void_p(gathered_ptr), ctypes.c_void_p(dst_ptr), dv, n_head, n_q, n_seq,
                                    n_ranks, ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_assemble_heads")


def workspace_status(workspace: int, stream: int = 0) -> tuple[int, int]:
    """(status code, raw bits) of a workspace's device status word; clears it."""
    raw = ctypes.c_uint32(0)
    st = lib().mm3fa_workspace_status(ctypes.c_void_p(workspace), ctypes.c_void_p(stream or None), ctypes.byref(raw))
    return st, raw.value


# ---------------------------------------------------------------------- torch conveniences

class Workspace:
    """A zero-filled device workspace that grows on demand (one per stream)."""

    def __init__(self, device=None):
        self.device = device
        self.buf = None

    def get(self, nbytes: int):
        import torch

        if nbytes == 0:
            return 0, 0
        if self.buf is None or self.buf.numel() < nbytes:
            self.buf = torch.zeros(max(nbytes, 1 << 16), dtype=torch.uint8, device=self.device)
        return self.buf.data_ptr(), self.buf.numel()


def run(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, dst: Tensor, scale: float, max_bias: float = 0.0,
        logit_softcap: float = 0.0, ws: Workspace | None = None, stream=None) -> None:
    """flash_attn_ext with a torch-allocated workspace on torch's current (or given) stream."""
    import torch

    ws = ws or Workspace(torch.device("cuda", torch.cuda.current_device()))
    nbytes = workspace_size(q, k, v, mask, dst)
    ptr, cap = ws.get(nbytes)
    s = stream if stream is not None else torch.cuda.current_stream()
    flash_attn_ext(q, k, v, mask, scale, max_bias, logit_softcap, dst, ptr, cap, s.cuda_stream)


# ---------------------------------------------------------------- multi-GPU head exchange

def allgather_heads(slice_ptr: int, gathered_ptr: int, dst_ptr: int, dv: int, n_head: int, n_q: int, n_seq: int,
                    seq_split: int, nccl_comm: int, stream: int = 0) -> None:
    """mm3fa_allgather_heads: every rank's result slice gathered over NCCL into the whole
    [Dv, n_head, n_q, n_seq] result (gathered_ptr: G-slice scratch, or 0 when not needed)."""
    st = lib().mm3fa_allgather_heads(ctypes.c_void_p(slice_ptr), ctypes.c_void_p(gathered_ptr or None),
                                     ctypes.c_void_p(dst_ptr), dv, n_head, n_q, n_seq, seq_split,
                                     ctypes.c_void_p(nccl_comm or None), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_allgather_heads")


def flash_attn_ext_peers(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, scale: float, max_bias: float,
                         logit_softcap: float, dst: Tensor, workspace: int, workspace_bytes: int, peers: Peers,
                         slot: int, epochs_ptr: int, stream: int = 0, kv_len_ptr: int = 0,
                         prec: int = GGML_PREC_F32) -> None:
    """Attention on this rank's shard with the head exchange fused into the kernel: the result values
    also go, as {value, epoch} words, into every other rank's receive buffer (slot `slot`)."""
    st = lib().mm3fa_flash_attn_ext_peers(_ref(q), _ref(k), _ref(v), _ref(mask), ctypes.c_void_p(kv_len_ptr or None),
                                          scale, max_bias, logit_softcap, prec, _ref(dst),
                                          ctypes.c_void_p(workspace or None), workspace_bytes, ctypes.byref(peers),
                                          slot, ctypes.c_void_p(epochs_ptr or None), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_flash_attn_ext_peers")


def peer_wait(peers: Peers, slot: int, epochs_ptr: int, result: Tensor, workspace: int, stream: int = 0) -> None:
    """Device-side bounded wait for every other rank's slice of the latest call on `slot`, unpacked
    into `result` (this rank's whole [Dv, n_head, n_q, n_seq] result); advances epochs[slot]."""
    st = lib().mm3fa_peer_wait(ctypes.byref(peers), slot, ctypes.c_void_p(epochs_ptr or None), _ref(result),
                               ctypes.c_void_p(workspace or None), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_peer_wait")


def flash_attn_ext_gather(q: Tensor, k: Tensor, v: Tensor, mask: Tensor | None, scale: float, dst: Tensor,
                          workspace: int, workspace_bytes: int, results: Peers, stream: int = 0,
                          max_bias: float = 0.0, logit_softcap: float = 0.0, prec: int = GGML_PREC_F32) -> None:
    """Dense attention on this rank's shard whose result rows also go straight into every other
    rank's whole result (results.recv[r]; dst is this rank's slice inside results.recv[rank])."""
    st = lib().mm3fa_flash_attn_ext_gather(_ref(q), _ref(k), _ref(v), _ref(mask), scale, max_bias, logit_softcap,
                                           prec, _ref(dst), ctypes.c_void_p(workspace or None), workspace_bytes,
                                           ctypes.byref(results), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_flash_attn_ext_gather")


def gather_signal_wait(flags: Peers, slot: int, epochs_ptr: int, workspace: int, stream: int = 0) -> None:
    """Publishes this rank's rows of the last mm3fa_flash_attn_ext_gather call on `slot` and waits
    (on the device, bounded) for every other rank's; advances epochs[slot]."""
    st = lib().mm3fa_gather_signal_wait(ctypes.byref(flags), slot, ctypes.c_void_p(epochs_ptr or None),
                                        ctypes.c_void_p(workspace or None), ctypes.c_void_p(stream or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_gather_signal_wait")


def ipc_export(ptr: int) -> bytes:
    h = IpcHandle()
    st = lib().mm3fa_ipc_export(ctypes.c_void_p(ptr or None), ctypes.byref(h))
    if st != OK:
        raise MM3FAError(st, "mm3fa_ipc_export")
    return bytes(ctypes.string_at(ctypes.addressof(h), ctypes.sizeof(h)))


def ipc_open(blob: bytes) -> int:
    h = IpcHandle.from_buffer_copy(blob)
    out = ctypes.c_void_p()
    st = lib().mm3fa_ipc_open(ctypes.byref(h), ctypes.byref(out))
    if st != OK:
        raise MM3FAError(st, "mm3fa_ipc_open")
    return int(out.value)


def ipc_close(ptr: int) -> None:
    st = lib().mm3fa_ipc_close(ctypes.c_void_p(ptr or None))
    if st != OK:
        raise MM3FAError(st, "mm3fa_ipc_close")
