"""Helpers shared by the GPU parity tests: move a workloads.Case to the device, run the
CUDA path through the C ABI, compare with the CPU oracle."""
from __future__ import annotations

import numpy as np
import torch

import mm3fa
import oracle  # the checker only (test infrastructure)
from mm3fa import ggml, workloads

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


def check_three_ways(got: np.ndarray, c: workloads.Case, exact_abs: float = MAX_ABS, exact_cos: float = MIN_COS,
                     refs: dict | None = None) -> dict:
    """Full-output parity of a GPU result against the three oracle modes.

    * F32 accumulation (the precision the callers request with set_prec(F32)): the north-star
      bound, max-abs <= 2e-3 and cosine >= 0.99999.
    * exact (float64): (exact_abs, exact_cos), widened to the F32-accumulation mode's own
      distance from exact math when that is larger (Q8_0 with few keys: Q's 8-bit rounding).
    * ggml's CPU kernel (F16 V accumulator when V is F16, otherwise F32 like the F32 mode):
      with F16 V that kernel is itself up to ~5e-3 / cos 0.9998 from exact math at these
      shapes, so the north-star bound is widened to the F32-accumulation mode's own distance
      from it; and with F16 V the GPU must be at least as close to exact math as it is.
    `refs` may carry precomputed oracle outputs keyed by mode."""
    refs = dict(refs or {})
    for mode in (oracle.MODE_F32ACC, oracle.MODE_EXACT, oracle.MODE_GGML_CPU):
        if mode not in refs:
            refs[mode] = run_oracle(c, mode)
    f32, ex, cpu = refs[oracle.MODE_F32ACC], refs[oracle.MODE_EXACT], refs[oracle.MODE_GGML_CPU]
    assert_close(got, f32, what=f"{c.name} vs F32-accumulation oracle")
    if not got.size:
        return refs
    conv_abs = float(np.abs(f32 - ex).max())
    assert_close(got, ex, max(exact_abs, 1.25 * conv_abs), min(exact_cos, cosine(f32, ex) - 1e-6),
                 what=f"{c.name} vs exact oracle")
    d_cpu = float(np.abs(f32 - cpu).max())
    assert_close(got, cpu, max(MAX_ABS, 1.25 * d_cpu), min(MIN_COS, cosine(f32, cpu) - 1e-6),
                 what=f"{c.name} vs ggml-cpu oracle")
    if c.v.gtype == ggml.GGML_TYPE_F16 and d_cpu > 0:
        assert cosine(got, ex) >= cosine(cpu, ex) - 1e-7, f"{c.name}: GPU less accurate than ggml's CPU kernel"
    return refs
