"""Benchmark of the mm3fa attention hot path (GGML_OP_FLASH_ATTN_EXT) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mm3fa|reference]

Workload (benchmark config 2 at the metric's point "CFG B=2, KV 8K"): one step is the
decode attention of all 36 layers of the Qwen3 LM for one token, each layer with its own
F16 KV cache laid out as the reference lays it out ([128, max_seq=10240, 8, n_seq],
viewed at n_kv = 8192, src/qwen3-lm.h:810-813), 32 query heads over 8 kv heads, D=128,
F32 Q, zero F16 mask, scale 1/sqrt(128).  Synthetic seeded data; K/V ~ N(0, 0.5^2).
Inputs are larger than L2 (36 x 84 MB of cache), so no L2 flush is needed.

N GPUs: KV-head sharding, weak scaling.  Rank r holds kv heads [8r/N, 8(r+1)/N) of the
caches of 2N sequences (N CFG pairs), i.e. the same bytes per GPU as N=1; after the 36
layers one NCCL all-gather moves every rank's head slices and mm3fa_assemble_heads
rebuilds the ggml [128, 32, 1, 2N] outputs.

The same line carries the dense (tensor-core) side of the metric: "dit" times benchmark config 5
(DiT bidirectional attention, B=2 CFG x S=4096 x 16 heads x D=128, F32 Q permuted view, F16
K/V, no mask) as one flow step of 24 blocks per timed step, cycling 4 operand sets so every call
reads its inputs from HBM; "prefill" times config 4 (2 x 1024-token causal prefill, 32q/8kv,
D=128, F16 causal mask over the 256-padded cache view).  N GPUs: each rank runs its own
(CFG batch x head) shard of the same per-GPU size (weak scaling, no collective).

Printed JSON: value = whole-job algorithmic GB/s of the timed steps (device time, max over
ranks); e2e = the same through the C ABI with Q/mask copied from pinned host memory and the
outputs read back every step (copies in chunks of E2E_CHUNK layers on two copy streams,
overlapping the attention of the other chunks); roofline = the decode kernel's achieved GB/s vs the measured
HBM copy bandwidth; cpu_baseline = the CPU oracle (ggml-cpu algorithm) on the host cores.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "minimaxmusic.cpp_b200"))

METRIC = "decode attn GB/s & µs/layer (CFG B=2, KV 8K); DiT attn TFLOPS; % roofline"
N_LAYERS = 36
E2E_CHUNK = 6      # layers per host<->device copy in the end-to-end measurement
N_HEAD, N_HEAD_KV, D = 32, 8, 128
N_KV, MAX_SEQ = 8192, 10240
FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum of one decode launch at this workload (ncu capture)
NCU_KERNEL = "fa_decode_mma_kernel<128,f16,NT=1,cluster,NS=3>"
NCU_TRAFFIC_BYTES = 67225600 + 466432


def layer_bytes(n_seq: int, n_head_kv: int, n_head: int) -> int:
    """Algorithmic bytes of one decode-attention call: K+V once, Q, mask, out."""
    kv = 2 * n_seq * n_head_kv * N_KV * D * 2
    q = n_seq * n_head * D * 4
    out = n_seq * n_head * D * 4
    mask = n_seq * N_KV * 2
    return kv + q + out + mask


FALLBACK_BF16_TFLOPS = 1590.0


def measured_tensor_peaks() -> tuple[float, float, str]:
    """(burst, sustained) dense bf16 TFLOP/s of this pool's B200s."""
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            d = json.load(f)
        return float(d["bf16_tflops"]), float(d["bf16_tflops_sustained"]), "measured"
    except Exception:
        return FALLBACK_BF16_TFLOPS, 1400.0, "fallback"


def measured_peaks() -> tuple[float, str]:
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(p) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


class ClockSampler:
    """nvidia-smi clock/throttle samples during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "100"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
            time.sleep(0.3)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self) -> dict:
        rows = []
        try:
            for line in open(self.path):
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9 and parts[1].replace(".", "").isdigit():
                    rows.append(parts)
        except Exception:
            pass
        finally:
            if self.path and os.path.exists(self.path):
                os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        sm = [float(r[1]) for r in rows]
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({n for r in rows for n, v in zip(names, r[5:9]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(sm), "sm_max_mhz": float(rows[0][2]), "reasons": reasons,
                "samples": len(rows)}


def cpu_baseline(seconds: float = 10.0) -> dict:
    """The CPU oracle (ggml convention: Q rounded to F16, F32 online softmax) on all host cores,
    over distinct layers of the same shape, for about `seconds`."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test infrastructure: the timed CPU baseline only
    from mm3fa import workloads

    threads = os.cpu_count() or 1
    n_distinct = 2
    cases = [workloads.decode_case(n_seq=2, n_kv=N_KV, max_seq=N_KV, kv_std=0.5, seed=1000 + i)
             for i in range(n_distinct)]
    descs = [(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale) for c in cases]
    oracle.flash_attn_ext(*descs[0], mode=oracle.MODE_F32ACC, threads=threads)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.flash_attn_ext(*descs[n % n_distinct], mode=oracle.MODE_F32ACC, threads=threads)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    dt = time.perf_counter() - t0
    b = layer_bytes(2, N_HEAD_KV, N_HEAD)
    return {"value": round(b * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode-attention layers (B=2, KV 8192, 32q/8kv, D=128, F16 K/V) cycling over "
                      f"{n_distinct} distinct caches, {dt:.1f} s, oracle F32-accumulation mode",
            "us_per_layer": round(dt / n * 1e6, 1)}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU implementation of the path.  ggml (the
    reference's implementation) is absent from its tree, so this times the CPU oracle port
    on the same workload, all host threads, rank 0 only."""
    if int(os.environ.get("RANK", "0")) != 0:
        return
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    from mm3fa import workloads

    threads = os.cpu_count() or 1
    n_layers_per_step = 4  # a bounded sample of the 36-layer step
    cases = [workloads.decode_case(n_seq=2, n_kv=N_KV, max_seq=N_KV, kv_std=0.5, seed=2000 + i)
             for i in range(n_layers_per_step)]
    descs = [(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale) for c in cases]

    def step():
        for d in descs:
            oracle.flash_attn_ext(*d, mode=oracle.MODE_F32ACC, threads=threads)

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    dt = time.perf_counter() - t0
    b = layer_bytes(2, N_HEAD_KV, N_HEAD) * n_layers_per_step * args.steps
    gbs = b / dt / 1e9
    us_layer = dt / (args.steps * n_layers_per_step) * 1e6
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(dt / args.steps * 1e3, 3),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f16/f32",
        "data": "synthetic (seeded, benchmark config 2 shapes)",
        "config": {"workload": "decode attention, 36-layer Qwen3 LM step at CFG B=2, KV 8192 "
                               f"(bounded sample: {n_layers_per_step} layers per step)",
                   "n_seq": 2, "n_kv": N_KV, "n_head": N_HEAD, "n_head_kv": N_HEAD_KV, "head_dim": D,
                   "kv_type": "f16", "us_per_layer": round(us_layer, 1)},
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"{n_layers_per_step} distinct layers per step, oracle F32-accumulation mode "
                                   "(ggml, the reference's implementation, is absent from the reference tree)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_dense(torch, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, local: int) -> dict:
    """DiT (config 5) and causal prefill (config 4) attention on the tensor-core kernel."""
    g = torch.Generator(device=dev)
    g.manual_seed(99)

    def rms(x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    def dit_set(B, S, H, Dh):
        q = rms(torch.randn(B, S, H, Dh, generator=g, device=dev))           # [D, H, S, B] storage
        k = rms(torch.randn(B, H, S, Dh, generator=g, device=dev)).half()    # [D, S, H, B] contiguous
        v = torch.randn(B, H, S, Dh, generator=g, device=dev).half()
        o = torch.empty(B, S, H, Dh, device=dev)
        qd = ggml.make(ggml.GGML_TYPE_F32, [Dh, S, H, B], q.data_ptr(), [4, 4 * Dh * H, 4 * Dh, 4 * Dh * H * S])
        kd = ggml.make(ggml.GGML_TYPE_F16, [Dh, S, H, B], k.data_ptr())
        vd = ggml.make(ggml.GGML_TYPE_F16, [Dh, S, H, B], v.data_ptr())
        dd = ggml.make(ggml.GGML_TYPE_F32, [Dh, H, S, B], o.data_ptr())
        return (q, k, v, o), (qd, kd, vd, None, dd)

    def timed(calls, n_calls_per_step, flops_per_call, ws):
        def step():
            for (qd, kd, vd, md, dd), sc in calls:
                mm3fa.flash_attn_ext(qd, kd, vd, md, sc, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), stream.cuda_stream)

        with torch.cuda.stream(stream):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with ClockSampler(local) as clk:
            stream.record_event(e0)
            with torch.cuda.stream(stream):  # replay() launches on the current stream
                for _ in range(steps):
                    graph.replay()
            stream.record_event(e1)
            torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / steps
        del graph
        us_call = ms * 1e3 / n_calls_per_step
        return us_call, flops_per_call / (us_call * 1e-6) / 1e12, clk.summary()

    burst, sustained, src = measured_tensor_peaks()
    out = {}
    # ---- DiT: 24 blocks of one flow step, 4 operand sets (each ~192 MB > L2) cycled
    B, S, H, Dh = 2, 4096, 16, 128
    sets = [dit_set(B, S, H, Dh) for _ in range(4)]
    ws = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    calls = [(sets[i % 4][1], 1.0 / math.sqrt(Dh)) for i in range(24)]
    fl = 4.0 * Dh * S * S * H * B
    us, tf, clocks = timed(calls, 24, fl, ws)
    out["dit"] = {"tflops": round(tf * world, 1), "tflops_per_gpu": round(tf, 1), "us_per_call": round(us, 2),
                  "clocks": clocks,
                  "config": {"workload": "DiT self-attention, benchmark config 5, 24 blocks per step",
                             "batch_per_gpu": B, "seq": S, "heads": H, "head_dim": Dh, "mask": None,
                             "l2": "4 operand sets cycled, each > L2"},
                  "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": sustained, "unit": "TFLOP/s",
                               "frac": round(tf / sustained, 4), "peak_kind": "bf16_tflops_sustained",
                               "frac_of_burst": round(tf / burst, 4), "peak_source": src,
                               "kernel": "fa_dense_kernel<128,f16>", "traffic": 134490000 + 37360000,
                               "flops_per_launch": fl}}
    del sets
    # ---- causal prefill: 2 x 1024 tokens, 32q / 8kv, cache view padded to 256
    Sp, Hq, Hkv, pad = 1024, 32, 8, 256
    n_kv = -(-Sp // pad) * pad
    q = rms(torch.randn(2, Sp, Hq, Dh, generator=g, device=dev))
    kc = rms(torch.randn(2, Hkv, n_kv, Dh, generator=g, device=dev)).half()
    vc = torch.randn(2, Hkv, n_kv, Dh, generator=g, device=dev).half()
    o = torch.empty(2, Sp, Hq, Dh, device=dev)
    mask = torch.triu(torch.full((Sp, n_kv), float("-inf"), device=dev), diagonal=1).half()
    qd = ggml.make(ggml.GGML_TYPE_F32, [Dh, Sp, Hq, 2], q.data_ptr(), [4, 4 * Dh * Hq, 4 * Dh, 4 * Dh * Hq * Sp])
    kd = ggml.make(ggml.GGML_TYPE_F16, [Dh, n_kv, Hkv, 2], kc.data_ptr())
    vd = ggml.make(ggml.GGML_TYPE_F16, [Dh, n_kv, Hkv, 2], vc.data_ptr())
    md = ggml.make(ggml.GGML_TYPE_F16, [n_kv, Sp, 1, 1], mask.data_ptr())
    dd = ggml.make(ggml.GGML_TYPE_F32, [Dh, Hq, Sp, 2], o.data_ptr())
    need = mm3fa.workspace_size(qd, kd, vd, md, dd)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    flp = 4.0 * Dh * (Sp * (Sp + 1) / 2) * Hq * 2
    us, tf, clocks = timed([((qd, kd, vd, md, dd), 1.0 / math.sqrt(Dh))], 1, flp, ws)
    out["prefill"] = {"tflops": round(tf * world, 1), "tflops_per_gpu": round(tf, 1), "us_per_call": round(us, 2),
                      "frac_of_sustained": round(tf / sustained, 4), "clocks": clocks,
                      "config": {"workload": "causal LM prefill, benchmark config 4", "n_seq": 2, "tokens": Sp,
                                 "n_head": Hq, "n_head_kv": Hkv, "head_dim": Dh, "n_kv_view": n_kv}}
    return out


def bench_q8(torch, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, n_layers: int) -> dict:
    """Q8_0 KV-cache decode (benchmark config 3: config 1 at KV 8192 with Q8_0 K/V, int8 ~U[-127,127],
    fp16 scales ~U[0.001,0.02]), as a 36-layer step of independent caches in one CUDA graph; each
    rank holds its kv-head shard of `world` CFG pairs, like the F16 line (16 units per rank)."""
    g = torch.Generator(device=dev)
    g.manual_seed(77)
    n_seq, hkv, hq = 2 * world, N_HEAD_KV // world, N_HEAD // world  # per-rank work fixed as N grows
    nblk = D // 32
    rb = nblk * 34

    def q8_cache():
        t = torch.randint(-127, 128, (n_seq, hkv, N_KV, nblk, 34), generator=g, device=dev,
                          dtype=torch.int32).to(torch.int8).view(torch.uint8)
        sc = (torch.rand(n_seq, hkv, N_KV, nblk, generator=g, device=dev) * 0.019 + 0.001).half()
        t[..., :2] = sc.view(torch.uint8).view(n_seq, hkv, N_KV, nblk, 2)
        return t.contiguous()

    keep, descs = [], []
    mask = torch.zeros(n_seq, 1, 1, N_KV, dtype=torch.float16, device=dev)
    nb = [34, rb, rb * N_KV, rb * N_KV * hkv]
    for _ in range(n_layers):
        kc, vc = q8_cache(), q8_cache()
        q = torch.randn(n_seq, hq, 1, D, generator=g, device=dev)
        o = torch.empty(n_seq, 1, hq, D, device=dev)
        keep += [kc, vc, q, o]
        descs.append((ggml.make(ggml.GGML_TYPE_F32, [D, 1, hq, n_seq], q.data_ptr()),
                      ggml.make(ggml.GGML_TYPE_Q8_0, [D, N_KV, hkv, n_seq], kc.data_ptr(), nb),
                      ggml.make(ggml.GGML_TYPE_Q8_0, [D, N_KV, hkv, n_seq], vc.data_ptr(), nb),
                      ggml.make(ggml.GGML_TYPE_F16, [N_KV, 1, 1, n_seq], mask.data_ptr()),
                      ggml.make(ggml.GGML_TYPE_F32, [D, hq, 1, n_seq], o.data_ptr())))
    need = mm3fa.workspace_size(*descs[0][:4], descs[0][4])
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    scale = 1.0 / math.sqrt(D)

    def step():
        for (qd, kd, vd, md, dd) in descs:
            mm3fa.flash_attn_ext(qd, kd, vd, md, scale, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), stream.cuda_stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream.record_event(e0)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    stream.record_event(e1)
    torch.cuda.synchronize()
    del graph
    us_layer = e0.elapsed_time(e1) * 1e3 / steps / n_layers
    kv = 2 * n_seq * hkv * N_KV * rb
    algo = kv + n_seq * hq * D * 8 + n_seq * N_KV * 2
    peak, src = measured_peaks()
    gbs = algo / (us_layer * 1e-6) / 1e9
    return {"q8_decode": {"us_per_layer": round(us_layer, 3), "GBps": round(gbs, 1), "GBps_job": round(gbs * world, 1),
                          "roofline": {"bound": "hbm", "achieved": round(gbs, 1), "peak": peak, "unit": "GB/s",
                                       "frac": round(gbs / peak, 4), "peak_source": src,
                                       "kernel": "fa_decode_mma_kernel<128,q8_0,NT=1,cluster>",
                                       "bytes_per_layer": algo},
                          "config": {"workload": "Q8_0 KV-cache decode, benchmark config 3 (B=2 CFG, KV 8192), "
                                                 f"{n_layers} independent layers per CUDA graph",
                                     "n_seq": n_seq, "n_kv": N_KV, "n_head": hq, "n_head_kv": hkv,
                                     "head_dim": D, "l2": "inputs > L2"}}}


def bench_decode_step(torch, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, n_layers: int) -> dict:
    """Decode step from the QKV projection output (the nodes of src/qwen3-lm.h:764-820): per layer
    mm3fa_decode_step (the prologue kernel: RMSNorm + NeoX RoPE of q/k, k/v rows appended to the F16
    caches at row 8191; then the attention over the 8192-row views), 36 layers in one CUDA graph;
    also the prologue alone.  Shapes of the headline (per rank: its kv-head shard of `world` CFG pairs)."""
    g = torch.Generator(device=dev)
    g.manual_seed(55)
    n_seq, hkv, hq = 2 * world, N_HEAD_KV // world, N_HEAD // world  # per-rank work fixed as N grows
    row = N_KV - 1
    keep, layers = [], []
    mask = torch.zeros(n_seq, 1, 1, N_KV, dtype=torch.float16, device=dev)
    qn = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).float()
    kn = (1 + 0.1 * torch.randn(D, generator=g, device=dev)).float()
    pos = torch.full((n_seq,), row, dtype=torch.int32, device=dev)
    rows = torch.full((n_seq,), row, dtype=torch.int64, device=dev)
    rb = 2 * D
    cnb = [2, rb, rb * MAX_SEQ, rb * MAX_SEQ * hkv]
    F32, F16 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16
    for _ in range(n_layers):
        kc = (torch.randn(n_seq, hkv, MAX_SEQ, D, generator=g, device=dev) * 0.5).half()
        vc = (torch.randn(n_seq, hkv, MAX_SEQ, D, generator=g, device=dev) * 0.5).half()
        q_in = torch.randn(n_seq, hq, D, generator=g, device=dev)
        k_in = torch.randn(n_seq, hkv, D, generator=g, device=dev)
        v_in = torch.randn(n_seq, hkv, D, generator=g, device=dev)
        q = torch.empty(n_seq, hq, D, device=dev)
        o = torch.empty(n_seq, 1, hq, D, device=dev)
        keep += [kc, vc, q_in, k_in, v_in, q, o]
        layers.append(dict(
            q_in=ggml.make(F32, [D, hq, n_seq, 1], q_in.data_ptr()), k_in=ggml.make(F32, [D, hkv, n_seq, 1], k_in.data_ptr()),
            v_in=ggml.make(F32, [D, hkv, n_seq, 1], v_in.data_ptr()),
            kc=ggml.make(F16, [D, MAX_SEQ, hkv, n_seq], kc.data_ptr(), cnb),
            vc=ggml.make(F16, [D, MAX_SEQ, hkv, n_seq], vc.data_ptr(), list(cnb)),
            q_out=ggml.make(F32, [D, hq, n_seq, 1], q.data_ptr()), q4=ggml.make(F32, [D, 1, hq, n_seq], q.data_ptr()),
            k=ggml.make(F16, [D, N_KV, hkv, n_seq], kc.data_ptr(), cnb),
            v=ggml.make(F16, [D, N_KV, hkv, n_seq], vc.data_ptr(), list(cnb)),
            m=ggml.make(F16, [N_KV, 1, 1, n_seq], mask.data_ptr()), o=ggml.make(F32, [D, hq, 1, n_seq], o.data_ptr())))
    l0 = layers[0]
    need = mm3fa.workspace_size(l0["q4"], l0["k"], l0["v"], l0["m"], l0["o"])
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    scale = 1.0 / math.sqrt(D)

    def prologue(L):
        mm3fa.decode_prologue(L["q_in"], L["k_in"], L["v_in"], qn.data_ptr(), kn.data_ptr(), 1e-6, pos.data_ptr(),
                              1e6, rows.data_ptr(), L["kc"], L["vc"], L["q_out"], stream.cuda_stream)

    def attention(L):
        mm3fa.flash_attn_ext(L["q4"], L["k"], L["v"], L["m"], scale, 0.0, 0.0, L["o"], ws.data_ptr(), ws.numel(),
                             stream.cuda_stream)

    def timed(fn):
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            fn()
        with torch.cuda.stream(stream):
            for _ in range(warmup):
                graph.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        stream.record_event(e0)
        with torch.cuda.stream(stream):
            for _ in range(steps):
                graph.replay()
        stream.record_event(e1)
        torch.cuda.synchronize()
        del graph
        return e0.elapsed_time(e1) * 1e3 / steps / n_layers

    def step(L):
        mm3fa.decode_step(L["q_in"], L["k_in"], L["v_in"], qn.data_ptr(), kn.data_ptr(), 1e-6, pos.data_ptr(), 1e6,
                          rows.data_ptr(), L["kc"], L["vc"], L["q_out"], L["k"], L["v"], L["m"], scale, 0.0, 0.0,
                          L["o"], ws.data_ptr(), ws.numel(), stream.cuda_stream)

    us_step = timed(lambda: [step(L) for L in layers])
    us_pro = timed(lambda: [prologue(L) for L in layers])
    return {"decode_step": {"us_per_layer": round(us_step, 3), "prologue_us_per_layer": round(us_pro, 3),
                            "config": {"workload": "decode step from the QKV projection output: mm3fa_decode_step "
                                                   "(prologue kernel: QK-RMSNorm, NeoX RoPE theta 1e6, k/v append "
                                                   "at row 8191; then the attention over KV 8192), "
                                                   f"{n_layers} layers per CUDA graph",
                                       "n_seq": n_seq, "n_head": hq, "n_head_kv": hkv, "head_dim": D}}}


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="mm3fa", choices=["mm3fa", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-dense", action="store_true", help="skip the DiT / prefill (tensor-core) lines")
    ap.add_argument("--no-q8", action="store_true", help="skip the Q8_0 KV-cache decode line (config 3)")
    ap.add_argument("--no-step", action="store_true", help="skip the decode-step line (fused prologue + attention)")
    ap.add_argument("--layers", type=int, default=N_LAYERS,
                    help="layers per step (36 = the LM; fewer only for small ncu captures)")
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
        return
    n_layers = args.layers

    import torch
    import torch.distributed as dist

    import mm3fa
    from mm3fa import ggml

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        import datetime

        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    if N_HEAD_KV % world:
        raise SystemExit(f"{N_HEAD_KV} kv heads do not shard over {world} GPUs")

    n_seq = 2 * world                 # N CFG pairs
    hkv = N_HEAD_KV // world          # kv heads held by this rank
    hq = N_HEAD // world              # query heads computed by this rank
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)

    # ---- per-layer operands (device resident), in the reference's layouts
    caches, qs, outs = [], [], []
    q_all = torch.empty(n_layers, n_seq, hq, 1, D, device=dev)  # every layer's Q in one buffer
    for l in range(n_layers):
        kc = (torch.randn(n_seq, hkv, MAX_SEQ, D, generator=g, device=dev) * 0.5).half()
        vc = (torch.randn(n_seq, hkv, MAX_SEQ, D, generator=g, device=dev) * 0.5).half()
        caches.append((kc, vc))
        q_all[l].copy_(torch.randn(n_seq, hq, 1, D, generator=g, device=dev))
        qs.append(q_all[l])
    mask = torch.zeros(n_seq, 1, 1, N_KV, dtype=torch.float16, device=dev)
    outs = torch.empty(n_layers, n_seq, 1, hq, D, device=dev)
    rb = 2 * D
    kv_nb = [2, rb, rb * MAX_SEQ, rb * MAX_SEQ * hkv]
    descs = []
    for l in range(n_layers):
        kc, vc = caches[l]
        qd = ggml.make(ggml.GGML_TYPE_F32, [D, 1, hq, n_seq], qs[l].data_ptr())
        kd = ggml.make(ggml.GGML_TYPE_F16, [D, N_KV, hkv, n_seq], kc.data_ptr(), kv_nb)
        vd = ggml.make(ggml.GGML_TYPE_F16, [D, N_KV, hkv, n_seq], vc.data_ptr(), kv_nb)
        md = ggml.make(ggml.GGML_TYPE_F16, [N_KV, 1, 1, n_seq], mask.data_ptr())
        dd = ggml.make(ggml.GGML_TYPE_F32, [D, hq, 1, n_seq], outs[l].data_ptr())
        descs.append((qd, kd, vd, md, dd))
    scale = 1.0 / math.sqrt(D)
    ws_bytes = mm3fa.workspace_size(*descs[0][:4], descs[0][4])
    ws = torch.zeros(max(ws_bytes, 256), dtype=torch.uint8, device=dev)
    gathered = torch.empty(world, n_layers, n_seq, 1, hq, D, device=dev) if world > 1 else None
    final = torch.empty(n_layers * n_seq, 1, N_HEAD, D, device=dev) if world > 1 else None

    stream = torch.cuda.Stream(device=dev)
    ev_k0, ev_k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)

    def attention_layers(s):
        for (qd, kd, vd, md, dd) in descs:
            mm3fa.flash_attn_ext(qd, kd, vd, md, scale, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), s.cuda_stream)

    def exchange(s):
        if world > 1:
            dist.all_gather_into_tensor(gathered.view(-1), outs.view(-1))
            mm3fa.assemble_heads(gathered.data_ptr(), final.data_ptr(), D, N_HEAD, 1, n_layers * n_seq, world,
                                 s.cuda_stream)

    # capture the 36 attention launches once: the reference replays its decode graph the same way
    with torch.cuda.stream(stream):
        attention_layers(stream)  # first call sets kernel attributes outside capture
        exchange(stream)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        attention_layers(stream)
    launches_per_step = n_layers + (1 if world > 1 else 0)

    def step():
        with torch.cuda.stream(stream):
            graph.replay()
            exchange(stream)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    # ---- timed region (device time, CUDA events on the launching stream)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    kern_ms = []
    with ClockSampler(local) as clk:
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        stream.record_event(e0)
        for _ in range(args.steps):
            stream.record_event(ev_k0)
            with torch.cuda.stream(stream):
                graph.replay()
            stream.record_event(ev_k1)
            with torch.cuda.stream(stream):
                exchange(stream)
            ev_k1.synchronize()
            kern_ms.append(ev_k0.elapsed_time(ev_k1))
        stream.record_event(e1)
        torch.cuda.synchronize()
        if world > 1:
            dist.barrier()
    clocks = clk.summary()
    t_ms = e0.elapsed_time(e1)
    t = torch.tensor([t_ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    t_ms = float(t.item())
    ms_per_step = t_ms / args.steps
    per_rank_bytes = layer_bytes(n_seq, hkv, hq) * n_layers
    job_bytes = per_rank_bytes * world
    value = job_bytes * args.steps / (t_ms * 1e-3) / 1e9

    # ---- roofline of the decode kernel (average launch inside the captured step)
    avg_launch_us = statistics.median(kern_ms) * 1e3 / n_layers
    peak, peak_src = measured_peaks()
    achieved = layer_bytes(n_seq, hkv, hq) / (avg_launch_us * 1e-6) / 1e9

    # ---- end to end through the C ABI: Q/mask from pinned host memory, outputs back to host
    # One pinned buffer per direction (every layer's Q up, every layer's output down), moved in
    # chunks of E2E_CHUNK layers on two copy streams so that the transfers overlap the attention
    # of other layers: chunk c's Q is uploaded before its layers run, its outputs go down while
    # the next chunk computes.
    q_host = q_all.cpu().pin_memory()
    mask_host = mask.cpu().pin_memory()
    out_host = torch.empty(outs.shape, dtype=torch.float32).pin_memory()
    up_s, down_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)
    chunks = [(a, min(a + E2E_CHUNK, n_layers)) for a in range(0, n_layers, E2E_CHUNK)]
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        fork = torch.cuda.Event()
        stream.record_event(fork)
        up_s.wait_event(fork)
        down_s.wait_event(fork)
        uploaded = []
        with torch.cuda.stream(up_s):
            mask.copy_(mask_host, non_blocking=True)
            for a, b in chunks:
                q_all[a:b].copy_(q_host[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                up_s.record_event(ev)
                uploaded.append(ev)
        for (a, b), ev in zip(chunks, uploaded):
            stream.wait_event(ev)
            for (qd, kd, vd, md, dd) in descs[a:b]:
                mm3fa.flash_attn_ext(qd, kd, vd, md, scale, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), stream.cuda_stream)
            done = torch.cuda.Event()
            stream.record_event(done)
            down_s.wait_event(done)
            with torch.cuda.stream(down_s):
                out_host[a:b].copy_(outs[a:b], non_blocking=True)
        joined = torch.cuda.Event()
        down_s.record_event(joined)
        stream.wait_event(joined)
    h2d = q_host.numel() * 4 + mask_host.numel() * 2
    d2h = out_host.numel() * 4
    for _ in range(args.warmup):
        g2.replay()
        exchange(stream)
        stream.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    stream.record_event(f0)
    for _ in range(args.steps):
        with torch.cuda.stream(stream):
            g2.replay()
            exchange(stream)
        stream.synchronize()  # the step's result is read on the host every step
    stream.record_event(f1)
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = job_bytes * args.steps / (float(te.item()) * 1e-3) / 1e9

    dense = None if args.no_dense else bench_dense(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup, world, local)
    if dense is not None and world > 1:
        dist.barrier()
    q8 = None if args.no_q8 else bench_q8(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup, world, n_layers)
    if q8 is not None and world > 1:
        dist.barrier()
    dstep = None if args.no_step else bench_decode_step(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup, world,
                                                        n_layers)
    if dstep is not None and world > 1:
        dist.barrier()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cpu = cpu_baseline(args.cpu_seconds)

    if rank == 0:
        line = {
            "metric": METRIC, "value": round(value, 2), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "f16 (K/V) / f32 (Q, accum, out)",
            "data": "synthetic (seeded, benchmark config 2 shapes; inputs larger than L2, no flush)",
            "config": {"workload": "decode attention, 36-layer Qwen3 LM step at CFG B=2 per GPU, KV 8192 "
                                   "(F16 cache views [128, 8192, 8, B] of [128, 10240, 8, B])",
                       "global_batch": n_seq, "n_kv": N_KV, "n_layers": n_layers, "n_head": N_HEAD,
                       "n_head_kv": N_HEAD_KV, "head_dim": D, "parallelism": f"kv-head shard x{world}",
                       "l2": "inputs > L2 (36 x 84 MB caches)",
                       "us_per_layer": round(ms_per_step * 1e3 / n_layers, 3),
                       "bytes_per_layer_per_gpu": layer_bytes(n_seq, hkv, hq)},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "traffic": NCU_TRAFFIC_BYTES, "kernel": NCU_KERNEL,
                         "avg_launch_us": round(avg_launch_us, 3)},
            "gpu_launches": launches_per_step * args.steps,
            "clocks": clocks,
        }
        if dense is not None:
            line.update(dense)
        if q8 is not None:
            line.update(q8)
        if dstep is not None:
            line.update(dstep)
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)

    del graph, g2
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
