"""Helpers shared by the GPU parity tests: move a workloads.Case to the device, run the
CUDA path through the C ABI, compare with the CPU oracle."""
from __future__ import annotations

import numpy as np
import torch

import mm3fa
import oracle
from mm3fa import workloads

# north-star tolerances (F32 output): max-abs error and cosine similarity
MAX_ABS = 2e-3
MIN_COS = 0.99999


def to_device(op: workloads.Operand, dev):
    return torch.from_numpy(np.ascontiguousarray(op.storage)).to(dev)


def run_gpu(c: workloads.Case, dev, ws: mm3fa.Workspace | None = None, repeat: int = 1) -> np.ndarray:
    tensors = {n: to_device(getattr(c, n), dev) for n in ("q", "k", "v", "mask") if getattr(c, n) is not None}
    descs = {n: getattr(c, n).device_desc(t) for n, t in tensors.items()}
    out = torch.full(c.dst_shape(), float("nan"), dtype=torch.float32, device=dev)
    dst = mm3fa.dst_desc(descs["q"], descs["v"], out.data_ptr())
    ws = ws or mm3fa.Workspace(dev)
    for _ in range(repeat):
        mm3fa.run(descs["q"], descs["k"], descs["v"], descs.get("mask"), dst, c.scale, c.max_bias, c.softcap, ws)
    torch.cuda.synchronize(dev)
    return out.cpu().numpy()


def run_oracle(c: workloads.Case, mode: int) -> np.ndarray:
    md = c.mask.host_desc() if c.mask is not None else None
    return oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), md, c.scale, c.max_bias,
                                 c.softcap, mode)


def cosine(a: np.ndarray, b: np.ndarray) -> float:
    a = a.astype(np.float64).ravel()
    b = b.astype(np.float64).ravel()
    na, nb = np.linalg.norm(a), np.linalg.norm(b)
    if na == 0 and nb == 0:
        return 1.0
    return float(a @ b / (na * nb))


def assert_close(got: np.ndarray, ref: np.ndarray, max_abs: float = MAX_ABS, min_cos: float = MIN_COS, what=""):
    assert got.shape == ref.shape, (got.shape, ref.shape)
    assert np.all(np.isfinite(got)), f"{what}: non-finite output"
    err = float(np.abs(got - ref).max()) if got.size else 0.0
    cs = cosine(got, ref)
    assert err <= max_abs and cs >= min_cos, f"{what}: max-abs {err:.3e} (<= {max_abs}), cos {cs:.7f} (>= {min_cos})"
    return err, cs
