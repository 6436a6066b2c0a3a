"""Benchmark of the mm3fa attention hot path (GGML_OP_FLASH_ATTN_EXT) on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl mm3fa|reference]

Workload (benchmark config 2 at the metric's point "CFG B=2, KV 8K"): one step is the
decode attention of all 36 layers of the Qwen3 LM for one token, each layer with its own
F16 KV cache laid out as the reference lays it out ([128, max_seq=10240, 8, n_seq],
viewed at n_kv = 8192, src/qwen3-lm.h:810-813), 32 query heads over 8 kv heads, D=128,
F32 Q, zero F16 mask, scale 1/sqrt(128).  Synthetic seeded data; K/V ~ N(0, 0.5^2).
Inputs are larger than L2 (36 x 84 MB of cache), so no L2 flush is needed.

N GPUs: KV-head sharding, weak scaling.  Rank r holds kv heads [8r/N, 8(r+1)/N) of the
caches of 2N sequences (N CFG pairs), i.e. the same bytes per GPU as N=1, and the heads are
exchanged after every layer, as the o_proj of each layer needs them (--exchange p2p: the fused
peer-store exchange in the decode kernel + the consumer's wait-and-unpack kernel; nccl: an
all-gather per layer; the other form is timed beside it).  "strong" splits fixed jobs over the
GPUs instead, "sweep" measures config 2 point by point.

The same line carries the dense (tensor-core) side of the metric: "dit" times benchmark config 5
(DiT bidirectional attention, B=2 CFG x S=4096 x 16 heads x D=128, F32 Q permuted view, F16
K/V, no mask) as one flow step of 24 blocks per timed step, cycling 4 operand sets so every call
reads its inputs from HBM; "dit_real" the same at the real model's shape (B=2 x S=690 x 32 heads x
D=64, 8 operand sets cycled); "prefill" times config 4 (2 x 1024-token causal prefill, 32q/8kv,
D=128, F16 causal mask over the 256-padded cache view).  At N GPUs the jobs grow with N: the DiT
by CFG pairs (every head of a pair on one rank: no exchange needed; "dit_strong" splits the B=2
job's heads over the ranks and exchanges the result after every call), the prefill by sequences
split by kv head, exchanged after every call - the kernel's epilogue stores each result row into
every rank's result (mm3fa_flash_attn_ext_gather), the NCCL all-gather is timed beside it.  "q8_decode" is config 3, "decode_step" the fused prologue +
attention, "depth" the depth decoder's F32 attention of one frame.

Printed JSON: value = whole-job algorithmic GB/s of the timed steps (device time, max over
ranks); e2e = the same through the C ABI with Q/mask copied from pinned host memory and the
outputs read back every step (copies on two copy streams in uneven chunks, E2E_UP / E2E_DOWN,
overlapping the attention of other layers); roofline = the decode kernel's achieved GB/s vs the
measured HBM copy bandwidth; cpu_baseline = the oracle's restatement of ggml's CPU kernel on the
host cores (all of them, and half).
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
# host<->device copies of the end-to-end measurement: Q uploads gate the layers they feed (each
# gate is an event wait in the graph, which also breaks the programmatic launch edge between two
# decode kernels, so there are few), results go down in chunks while later layers compute; the
# first upload and the last download are one layer each, so little copying is left exposed
E2E_UP = (1, 7)           # upload boundaries: Q[0:1], Q[1:8], Q[8:L]
E2E_DOWN = (8, 16, 24, 32, 35)  # download boundaries: out[0:8], ..., out[32:35], out[35:L]
N_HEAD, N_HEAD_KV, D = 32, 8, 128
N_KV, MAX_SEQ = 8192, 10240
FALLBACK_HBM_GBS = 6650.0

# dram__bytes_read.sum + dram__bytes_write.sum of one decode launch at this workload, from the ncu
# capture summarised in profiles/ (re-captured whenever the kernel changes)
NCU_KERNEL = "fa_decode_mma_kernel<128,f16,NT=1,cluster,NS=3>"
NCU_TRAFFIC_BYTES = 67227136 + 437760
NCU_TRAFFIC_SOURCE = "profiles/fa_decode_mma_kernel_cfg2_b2_kv8192.md (one ncu launch, 36-layer step)"


def layer_bytes(n_seq: int, n_head_kv: int, n_head: int, n_kv: int = N_KV) -> int:
    """Algorithmic bytes of one decode-attention call: K+V once, Q, mask, out (this rank's heads)."""
    kv = 2 * n_seq * n_head_kv * n_kv * D * 2
    q = n_seq * n_head * D * 4
    out = n_seq * n_head * D * 4
    mask = n_seq * n_kv * 2
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


def _cpu_layers_per_s(oracle, descs, threads: int, seconds: float) -> tuple[int, float]:
    """Runs the ggml-CPU restatement over `descs` in turn for about `seconds`."""
    oracle.flash_attn_ext(*descs[0], mode=oracle.MODE_GGML_CPU, threads=threads)  # warm
    t0 = time.perf_counter()
    n = 0
    while True:
        oracle.flash_attn_ext(*descs[n % len(descs)], mode=oracle.MODE_GGML_CPU, threads=threads)
        n += 1
        if time.perf_counter() - t0 >= seconds:
            break
    return n, time.perf_counter() - t0


def cpu_baseline(seconds: float = 10.0) -> dict:
    """The oracle's restatement of ggml's CPU flash_attn_ext kernel (Q rounded to F16, expf online
    softmax, F16 V accumulator) on all host cores and on half of them (the reference's own CPU
    thread count, hardware_concurrency / 2, src/backend.h:28-31), over distinct layers of the
    headline shape, about `seconds` each."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test infrastructure: the timed CPU baseline only
    from mm3fa import workloads

    threads = os.cpu_count() or 1
    n_distinct = 2
    cases = [workloads.decode_case(n_seq=2, n_kv=N_KV, max_seq=N_KV, kv_std=0.5, seed=1000 + i)
             for i in range(n_distinct)]
    descs = [(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale) for c in cases]
    b = layer_bytes(2, N_HEAD_KV, N_HEAD)
    n, dt = _cpu_layers_per_s(oracle, descs, threads, seconds)
    half = max(1, threads // 2)
    n2, dt2 = _cpu_layers_per_s(oracle, descs, half, seconds / 2)
    return {"value": round(b * n / dt / 1e9, 3), "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"{n} decode-attention layers (B=2, KV 8192, 32q/8kv, D=128, F16 K/V) cycling over "
                      f"{n_distinct} distinct caches, {dt:.1f} s, oracle restatement of ggml's CPU kernel "
                      "(F16 V accumulator)",
            "us_per_layer": round(dt / n * 1e6, 1),
            "half_cores": {"cores": half, "value": round(b * n2 / dt2 / 1e9, 3), "unit": "GB/s",
                           "us_per_layer": round(dt2 / n2 * 1e6, 1),
                           "note": "hardware_concurrency/2, the reference's CPU thread count (src/backend.h:28-31)"}}


def run_reference(args) -> None:
    """--impl reference: the reference's CPU implementation of the path.  ggml (the
    reference's implementation) is absent from its tree, so this times the CPU oracle's
    restatement of ggml's CPU flash_attn_ext kernel (F16 V accumulator) on the same workload,
    all host threads, rank 0 only."""
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
            oracle.flash_attn_ext(*d, mode=oracle.MODE_GGML_CPU, threads=threads)

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
                         "sample": f"{n_layers_per_step} distinct layers per step, oracle restatement of ggml's "
                                   "CPU kernel (ggml, the reference's implementation, is absent from the reference "
                                   "tree)"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def bench_dense(torch, dist, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, rank: int,
                local: int) -> dict:
    """DiT (config 5) and causal prefill (config 4) attention on the tensor-core kernel.

    N GPUs: the DiT job grows to N CFG pairs (B = 2N) and rank r computes pair r, all 16 heads
    (weak scaling, no exchange needed); a second line keeps the B = 2 job and splits its 32
    (batch x head) units over the ranks (strong scaling), each call followed by the exchange of the
    result, as to_out needs every head of its rows.  The prefill job grows to 2N sequences, split by
    kv head, with the same exchange after the call (o_proj).  The exchange the lines report is the
    fused one (the kernel stores its rows into every rank's result, then a signal-and-wait kernel);
    mm3fa_allgather_heads (NCCL + permute) is timed beside it."""
    from mm3fa import exchange as xch, sharding

    g = torch.Generator(device=dev)
    g.manual_seed(99 + rank)
    comm = xch.nccl_comm(dist, dev) if world > 1 else 0
    F32, F16 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16

    def rms(x):
        return x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6)

    def dit_set(B, S, H, Dh):
        q = rms(torch.randn(B, S, H, Dh, generator=g, device=dev))           # [D, H, S, B] storage
        k = rms(torch.randn(B, H, S, Dh, generator=g, device=dev)).half()    # [D, S, H, B] contiguous
        v = torch.randn(B, H, S, Dh, generator=g, device=dev).half()
        qd = ggml.make(F32, [Dh, S, H, B], q.data_ptr(), [4, 4 * Dh * H, 4 * Dh, 4 * Dh * H * S])
        kd = ggml.make(F16, [Dh, S, H, B], k.data_ptr())
        vd = ggml.make(F16, [Dh, S, H, B], v.data_ptr())
        return (q, k, v), (qd, kd, vd)

    def timed(calls, exchange_fn, n_calls_per_step, flops_per_call, ws):
        """calls: [(q, k, v, mask, dst descriptors, scale)]; exchange_fn(s) after each call or None."""
        def step(with_exchange=True):
            for (qd, kd, vd, md, dd), sc in calls:
                mm3fa.flash_attn_ext(qd, kd, vd, md, sc, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), stream.cuda_stream)
                if with_exchange and exchange_fn is not None:
                    exchange_fn(stream)

        res = {}
        for tag, ex in (("with_exchange", True), ("attention_only", False)):
            if tag == "attention_only" and exchange_fn is None:
                break
            with torch.cuda.stream(stream):
                step(ex)
            torch.cuda.synchronize()
            graph = torch.cuda.CUDAGraph()
            with torch.cuda.graph(graph, stream=stream):
                step(ex)
            with ClockSampler(local) as clk:
                ms = timed_replays(torch, dist, graph, stream, steps, warmup, world)
            del graph
            us_call = ms * 1e3 / n_calls_per_step
            res[tag] = (us_call, flops_per_call / (us_call * 1e-6) / 1e12, clk.summary())
        return res

    def timed_fused(calls, result_bytes, flops_per_call, ws):
        """The fused exchange: calls [(q, k, v, mask, scale, view_of)] where view_of(base) is this rank's
        dst slice inside a whole result at `base`; call i runs on result slot i % 2 through
        mm3fa_flash_attn_ext_gather (rows stored into every rank's result from the kernel) and is
        followed by mm3fa_gather_signal_wait.  Returns (us per call, TFLOP/s, clocks, status)."""
        gb = xch.GatherBuffers(torch, dist, dev, result_bytes, 2)

        def step():
            for i, (qd_, kd_, vd_, md_, sc_, view_of) in enumerate(calls):
                slot = i % 2
                mm3fa.flash_attn_ext_gather(qd_, kd_, vd_, md_, sc_, view_of(gb.result_ptr(slot)), ws.data_ptr(),
                                            ws.numel(), gb.results(slot), stream.cuda_stream)
                mm3fa.gather_signal_wait(gb.flags, slot, gb.epochs.data_ptr(), ws.data_ptr(), stream.cuda_stream)

        with torch.cuda.stream(stream):
            step()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=stream):
            step()
        with ClockSampler(local) as clk:
            ms = timed_replays(torch, dist, graph, stream, steps, warmup, world)
        del graph
        torch.cuda.synchronize()
        st, raw = mm3fa.workspace_status(ws.data_ptr(), stream.cuda_stream)
        dist.barrier()
        gb.close()
        us_call = ms * 1e3 / len(calls)
        return us_call, flops_per_call / (us_call * 1e-6) / 1e12, clk.summary(), int(st)

    burst, sustained, src = measured_tensor_peaks()
    out = {}
    def dit_line(B, S, H, Dh, n_sets, workload, l2):
        """24 blocks of one flow step over n_sets operand sets cycled (the sets together > L2).  At N GPUs
        the job is N CFG pairs and the (batch x head) units split by whole sequences (seq_split = N): rank
        r computes every head of pair r, so the head-concatenated output that to_out reads is local and
        no exchange is needed (the head-split exchange is the strong line's)."""
        fl = 4.0 * Dh * S * S * H * B
        sets = [dit_set(B, S, H, Dh) for _ in range(n_sets)]
        res = torch.empty(B, S, H, Dh, device=dev)  # this rank's pair ([D, H, S, B])
        dd = ggml.make(F32, [Dh, H, S, B], res.data_ptr())
        ws = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
        calls = [((*sets[i % n_sets][1], None, dd), 1.0 / math.sqrt(Dh)) for i in range(24)]
        us, tf, clocks = timed(calls, None, 24, fl, ws)["with_exchange"]
        line = {"tflops": round(tf * world, 1), "tflops_per_gpu": round(tf, 1), "us_per_call": round(us, 2),
                "clocks": clocks,
                "config": {"workload": workload, "batch_per_gpu": B, "global_batch": B * world, "seq": S, "heads": H,
                           "head_dim": Dh, "mask": None, "l2": l2,
                           "exchange": "none needed: every head of a rank's CFG pair is local" if world > 1
                                       else "none (1 GPU)"},
                "roofline": {"bound": "tensor", "achieved": round(tf, 1), "peak": burst, "unit": "TFLOP/s",
                             "frac": round(tf / burst, 4),
                             "peak_kind": "bf16_tflops (burst: the timed region is a fraction of a second)",
                             "frac_of_sustained": round(tf / sustained, 4), "peak_source": src,
                             "kernel": f"fa_dense_kernel<{Dh},f16>", "flops_per_launch": fl}}
        del res, calls
        return line, sets

    # ---- DiT, benchmark config 5: 4 operand sets (each ~192 MB > L2) cycled
    B, S, H, Dh = 2, 4096, 16, 128
    fl = 4.0 * Dh * S * S * H * B
    out["dit"], sets = dit_line(B, S, H, Dh, 4, "DiT self-attention, benchmark config 5, 24 blocks per step",
                                "4 operand sets cycled, each > L2")
    out["dit"]["roofline"]["traffic"] = 134490000 + 37360000
    if world > 1:
        # strong scaling: the B = 2 job's 32 (batch x head) units over the ranks
        s0, s1, h0, h1, ss = sharding.unit_slice(B, H, rank, world)
        sl, hl = s1 - s0, h1 - h0
        direct = world // ss == 1
        full2 = torch.empty(B, S, H, Dh, device=dev)
        gath = None if direct else torch.empty(world, sl, S, hl, Dh, device=dev)
        sptr = full2.data_ptr() + rank * sl * S * H * Dh * 4 if direct else gath[rank].data_ptr()
        dd2 = ggml.make(F32, [Dh, hl, S, sl], sptr)
        calls2 = []
        for i in range(24):
            qd, kd, vd = sets[i % 4][1]
            view = lambda t: ggml.make(t.type, [Dh, S, hl, sl], t.data + h0 * t.nb[2] + s0 * t.nb[3], list(t.nb))
            calls2.append(((view(qd), view(kd), view(vd), None, dd2), 1.0 / math.sqrt(Dh)))
        ex2 = lambda s_: mm3fa.allgather_heads(sptr, 0 if direct else gath.data_ptr(), full2.data_ptr(), Dh, H, S, B,
                                               ss, comm, s_.cuda_stream)
        ws2 = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
        r2 = timed(calls2, ex2, 24, fl, ws2)
        # the fused exchange: each rank's slice of the job's [Dh, H, S, B] result, stored by the kernel
        fcalls = [(c[0][0], c[0][1], c[0][2], None, c[1],
                   lambda base: ggml.make(F32, [Dh, hl, S, sl], base + (s0 * S * H + h0) * Dh * 4,
                                          [4, 4 * Dh, 4 * Dh * H, 4 * Dh * H * S])) for c in calls2]
        fu, ftf, fclk, fst = timed_fused(fcalls, B * S * H * Dh * 4, fl, ws2)
        out["dit_strong"] = {"tflops_job": round(ftf, 1), "us_per_call": round(fu, 2),
                             "exchange": "fused: rows stored into every rank's result from the kernel "
                                         "(mm3fa_flash_attn_ext_gather + mm3fa_gather_signal_wait)",
                             "exchange_status": fst,
                             "nccl_us_per_call": round(r2["with_exchange"][0], 2),
                             "nccl_tflops_job": round(r2["with_exchange"][1], 1),
                             "attention_only_us_per_call": round(r2["attention_only"][0], 2),
                             "attention_only_tflops_job": round(r2["attention_only"][1], 1),
                             "clocks": fclk,
                             "units_per_gpu": sl * hl, "config": {"global_batch": B, "heads": H, "seq": S,
                                                                  "seq_split": ss, "scaling": "strong"}}
        del full2, gath, calls2
    del sets
    torch.cuda.empty_cache()
    # ---- the real DiT's attention (src/dit.h:201-222: 32 heads x 64, 690 tokens per CFG pair member), 8
    # operand sets of 22.6 MB cycled so that the 24 calls read from HBM
    out["dit_real"], sets = dit_line(2, 690, 32, 64, 8, "DiT self-attention at the real model's shape, 24 blocks "
                                     "per step", "8 operand sets cycled, together > L2")
    del sets
    torch.cuda.empty_cache()
    # ---- causal prefill: 2 x 1024 tokens per GPU (the job: 2N sequences), 32q / 8kv, cache view padded to 256
    Sp, Hq, Hkv, pad = 1024, N_HEAD // world, N_HEAD_KV // world, 256
    nsp = 2 * world
    n_kv = -(-Sp // pad) * pad
    q = rms(torch.randn(nsp, Sp, Hq, Dh, generator=g, device=dev))
    kc = rms(torch.randn(nsp, Hkv, n_kv, Dh, generator=g, device=dev)).half()
    vc = torch.randn(nsp, Hkv, n_kv, Dh, generator=g, device=dev).half()
    mask = torch.triu(torch.full((Sp, n_kv), float("-inf"), device=dev), diagonal=1).half()
    gath = torch.empty(world, nsp, Sp, Hq, Dh, device=dev)
    fullp = torch.empty(nsp, Sp, N_HEAD, Dh, device=dev) if world > 1 else None
    qd = ggml.make(F32, [Dh, Sp, Hq, nsp], q.data_ptr(), [4, 4 * Dh * Hq, 4 * Dh, 4 * Dh * Hq * Sp])
    kd = ggml.make(F16, [Dh, n_kv, Hkv, nsp], kc.data_ptr())
    vd = ggml.make(F16, [Dh, n_kv, Hkv, nsp], vc.data_ptr())
    md = ggml.make(F16, [n_kv, Sp, 1, 1], mask.data_ptr())
    ddp = ggml.make(F32, [Dh, Hq, Sp, nsp], gath[rank].data_ptr())
    need = mm3fa.workspace_size(qd, kd, vd, md, ddp)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    flp = 4.0 * Dh * (Sp * (Sp + 1) / 2) * Hq * nsp
    exp_ = (lambda s_: mm3fa.allgather_heads(gath[rank].data_ptr(), gath.data_ptr(), fullp.data_ptr(), Dh, N_HEAD, Sp,
                                             nsp, 1, comm, s_.cuda_stream)) if world > 1 else None
    r = timed([((qd, kd, vd, md, ddp), 1.0 / math.sqrt(Dh))], exp_, 1, flp, ws)
    us, tf, clocks = r["with_exchange"]
    tf_k = r.get("attention_only", r["with_exchange"])[1]
    fused_info = None
    if world > 1:
        # the fused exchange (the line's figure): this rank's heads of the job's [Dh, 32, Sp, 2N] result,
        # stored by the kernel into every rank's result; two calls per step, one per result slot
        pview = lambda base: ggml.make(F32, [Dh, Hq, Sp, nsp], base + rank * Hq * Dh * 4,
                                       [4, 4 * Dh, 4 * Dh * N_HEAD, 4 * Dh * N_HEAD * Sp])
        nccl_us = us
        us, tf, clocks, fst = timed_fused([(qd, kd, vd, md, 1.0 / math.sqrt(Dh), pview)] * 2,
                                          nsp * Sp * N_HEAD * Dh * 4, flp, ws)
        fused_info = {"exchange": "fused: rows stored into every rank's result from the kernel "
                                  "(mm3fa_flash_attn_ext_gather + mm3fa_gather_signal_wait)",
                      "exchange_status": fst, "nccl_us_per_call": round(nccl_us, 2)}
    out["prefill"] = {"tflops": round(tf * world, 1), "tflops_per_gpu": round(tf, 1), "us_per_call": round(us, 2),
                      "frac_of_burst": round(tf_k / burst, 4), "frac_of_sustained": round(tf_k / sustained, 4),
                      "clocks": clocks,
                      "config": {"workload": "causal LM prefill, benchmark config 4", "n_seq": nsp, "tokens": Sp,
                                 "n_head": N_HEAD, "n_head_kv": N_HEAD_KV, "head_dim": Dh, "n_kv_view": n_kv,
                                 "parallelism": f"kv-head shard x{world}"
                                                + (", head exchange after the call" if world > 1 else "")}}
    if "attention_only" in r:
        out["prefill"]["attention_only_us_per_call"] = round(r["attention_only"][0], 2)
    if fused_info:
        out["prefill"].update(fused_info)
    return out


SWEEP_BATCH = (2, 4, 8)
SWEEP_KV = (512, 2048, 8192, 16384)


def bench_sweep(torch, dist, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, rank: int,
                n_layers: int) -> dict:
    """Benchmark config 2 as a sweep: batch 2/4/8 (CFG pairs) x KV 512/2048/8192/16384, 36 independent
    F16 layers (caches [128, max(10240, KV), 8, batch], K/V ~ N(0, 0.25)) per CUDA graph.  With N GPUs
    each point keeps its batch, rank r computes kv heads [8r/N, 8(r+1)/N) and the heads are exchanged
    after every layer (fused peer stores + device wait), so the per-layer time is the sharded time of
    the fixed job (strong scaling of the point)."""
    g = torch.Generator(device=dev)
    g.manual_seed(31 + rank)
    peak, src = measured_peaks()
    points = []
    for B in SWEEP_BATCH:
        for kv in SWEEP_KV:
            st = DecodeStack(torch, dist, mm3fa, ggml, dev, g, B, kv, n_layers, world, rank, "p2p")
            with torch.cuda.stream(stream):
                st.step(stream)
            torch.cuda.synchronize()
            graph = st.capture(stream)
            us_layer = timed_replays(torch, dist, graph, stream, steps, warmup, world) * 1e3 / n_layers
            del graph
            algo = st.layer_bytes()
            gbs = algo / (us_layer * 1e-6) / 1e9
            points.append({"n_seq": B, "n_kv": kv, "us_per_layer": round(us_layer, 3), "GBps": round(gbs, 1),
                           "GBps_job": round(gbs * world, 1), "frac": round(gbs / peak, 4),
                           "bytes_per_layer_per_gpu": algo})
            torch.cuda.synchronize()
            st.close()
            del st
            torch.cuda.empty_cache()
    return {"sweep": {"points": points, "peak": peak, "peak_source": src, "unit": "GB/s",
                      "config": {"workload": "benchmark config 2: 36-layer decode attention, batch x KV sweep",
                                 "n_layers": n_layers, "n_head": N_HEAD // world, "n_head_kv": N_HEAD_KV // world,
                                 "head_dim": D, "kv_type": "f16",
                                 "parallelism": f"kv-head shard x{world} of each point"
                                                + (", per-layer fused exchange" if world > 1 else ""),
                                 "l2": "inputs > L2 (36 layers of caches per point)"}}}


def bench_depth(torch, mm3fa, ggml, dev, stream, steps: int, warmup: int) -> dict:
    """The depth decoder's attention for one LM frame (src/depth-decoder.h:196-221, 249-253, 466): 7
    autoregressive steps over S = 2..8 codebook positions (no KV cache: each step attends over the
    whole prefix), 4 layers each, 16 heads x 256, CFG batch 2, F32 q/k/v as the reference's permuted
    [256, S, 16, 2] views of the [256, 16, S, 2] projections, causal F16 mask; 28 calls per frame in
    one CUDA graph on the CUDA-core decode kernel (F32 K/V).  Latency-bound: reported in us."""
    g = torch.Generator(device=dev)
    g.manual_seed(66)
    Dd, H, B, L = 256, 16, 2, 4
    F32, F16 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16
    keep, calls = [], []
    for S in range(2, 9):
        mask = torch.triu(torch.full((S, S), float("-inf"), device=dev), diagonal=1).half()
        keep.append(mask)
        for _ in range(L):
            q, k, v = (torch.randn(B, S, H, Dd, generator=g, device=dev) * sc for sc in (1.0, 0.5, 0.5))
            o = torch.empty(B, S, H, Dd, device=dev)
            keep += [q, k, v, o]
            nb = [4, 4 * Dd * H, 4 * Dd, 4 * Dd * H * S]
            calls.append((ggml.make(F32, [Dd, S, H, B], q.data_ptr(), nb), ggml.make(F32, [Dd, S, H, B], k.data_ptr(), nb),
                          ggml.make(F32, [Dd, S, H, B], v.data_ptr(), nb), ggml.make(F16, [S, S, 1, 1], mask.data_ptr()),
                          ggml.make(F32, [Dd, H, S, B], o.data_ptr())))
    need = max(mm3fa.workspace_size(*c[:4], c[4]) for c in calls)
    ws = torch.zeros(max(need, 256), dtype=torch.uint8, device=dev)
    scale = 1.0 / math.sqrt(Dd)

    def step():
        for (qd, kd, vd, md, dd) in calls:
            mm3fa.flash_attn_ext(qd, kd, vd, md, scale, 0.0, 0.0, dd, ws.data_ptr(), ws.numel(), stream.cuda_stream)

    with torch.cuda.stream(stream):
        step()
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    ms = timed_replays(torch, None, graph, stream, steps, warmup, 1)
    del graph
    return {"depth": {"us_per_frame": round(ms * 1e3, 2), "us_per_call": round(ms * 1e3 / len(calls), 3),
                      "calls_per_frame": len(calls),
                      "config": {"workload": "depth decoder attention of one frame: 7 steps (S = 2..8) x 4 layers, "
                                             "16 heads x 256, CFG batch 2, F32 K/V permuted views, causal",
                                 "kernel": "fa_decode_kernel<256,f32,C=32,NSTAGE=2,copy> (element copies: "
                                           "the views' rows are not contiguous)"}}}


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


class DecodeStack:
    """n_layers independent F16 decode-attention layers of one (batch, KV) point in the reference's
    cache layout ([128, max_seq, 8, batch] viewed at KV), this rank's kv-head shard of it, with the
    per-layer head exchange the model needs: layer l's o_proj consumes every head of layer l's
    result before layer l+1 starts (src/qwen3-lm.h:732, 823-827).

    world == 1: plain attention into [L, B, 1, 32, D].  world > 1, exchange "p2p": the attention
    kernel also stores its values into every other rank's receive buffer as {value, epoch} words
    (mm3fa_flash_attn_ext_peers) and the next layer starts after this rank's wait-and-unpack
    kernel (mm3fa_peer_wait); "nccl": mm3fa_allgather_heads after every layer."""

    def __init__(self, torch, dist, mm3fa, ggml, dev, gen, B: int, kv: int, n_layers: int, world: int, rank: int,
                 mode: str = "p2p", max_seq: int | None = None):
        from mm3fa import exchange as xch

        self.torch, self.mm3fa, self.world, self.rank, self.mode = torch, mm3fa, world, rank, mode
        self.B, self.kv, self.L = B, kv, n_layers
        self.hkv, self.hq = N_HEAD_KV // world, N_HEAD // world
        hkv, hq = self.hkv, self.hq
        max_seq = max_seq or max(MAX_SEQ, kv)
        rb = 2 * D
        nb = [2, rb, rb * max_seq, rb * max_seq * hkv]
        self.caches = []
        self.q_all = torch.empty(n_layers, B, hq, 1, D, device=dev)  # every layer's Q in one buffer
        for l in range(n_layers):
            kc = (torch.randn(B, hkv, max_seq, D, generator=gen, device=dev) * 0.5).half()
            vc = (torch.randn(B, hkv, max_seq, D, generator=gen, device=dev) * 0.5).half()
            self.caches.append((kc, vc))
            self.q_all[l].copy_(torch.randn(B, hq, 1, D, generator=gen, device=dev))
        self.mask = torch.zeros(B, 1, 1, kv, dtype=torch.float16, device=dev)
        self.pb = None
        F32, F16 = ggml.GGML_TYPE_F32, ggml.GGML_TYPE_F16
        layer_out = B * N_HEAD * D * 4
        if world == 1:
            self.full = torch.empty(n_layers, B, 1, N_HEAD, D, device=dev)
            dst_ptr = [self.full[l].data_ptr() for l in range(n_layers)]
        elif mode == "p2p":
            self.pb = xch.PeerBuffers(torch, dist, dev, B * hq * D, n_layers)
            self.full = torch.empty(n_layers, B, 1, N_HEAD, D, device=dev)
            dst_ptr = [self.full[l].data_ptr() + rank * hq * D * 4 for l in range(n_layers)]
            self.results = [ggml.make(F32, [D, N_HEAD, 1, B], self.full[l].data_ptr()) for l in range(n_layers)]
        else:
            self.comm = xch.nccl_comm(dist, dev)
            self.gathered = torch.empty(n_layers, world, B, 1, hq, D, device=dev)
            self.full = torch.empty(n_layers, B, 1, N_HEAD, D, device=dev)
            dst_ptr = [self.gathered[l, rank].data_ptr() for l in range(n_layers)]
        # this rank's heads of each layer's result: [D, hq, 1, B] with the strides of the whole
        # [D, 32, 1, B] result (world == 1, p2p) or the contiguous slice (nccl)
        dnb = [4, 4 * D, 4 * D * hq, 4 * D * hq] if (world > 1 and mode == "nccl") else \
            [4, 4 * D, 4 * D * N_HEAD, 4 * D * N_HEAD]
        self.descs = []
        for l in range(n_layers):
            kc, vc = self.caches[l]
            self.descs.append((ggml.make(F32, [D, 1, hq, B], self.q_all[l].data_ptr()),
                               ggml.make(F16, [D, kv, hkv, B], kc.data_ptr(), nb),
                               ggml.make(F16, [D, kv, hkv, B], vc.data_ptr(), list(nb)),
                               ggml.make(F16, [kv, 1, 1, B], self.mask.data_ptr()),
                               ggml.make(F32, [D, hq, 1, B], dst_ptr[l], dnb)))
        need = mm3fa.workspace_size(*self.descs[0][:4], self.descs[0][4])
        self.ws = torch.zeros(max(need, 4096), dtype=torch.uint8, device=dev)
        self.scale = 1.0 / math.sqrt(D)

    def layer(self, l: int, s, exchange: bool = True) -> int:
        """Enqueues layer l (attention, then the exchange when asked); returns its launches."""
        mm3fa, (qd, kd, vd, md, dd) = self.mm3fa, self.descs[l]
        ws = (self.ws.data_ptr(), self.ws.numel())
        if self.world > 1 and exchange and self.mode == "p2p":
            ep = self.pb.epochs.data_ptr()
            mm3fa.flash_attn_ext_peers(qd, kd, vd, md, self.scale, 0.0, 0.0, dd, *ws, self.pb.peers, l, ep,
                                       s.cuda_stream)
            mm3fa.peer_wait(self.pb.peers, l, ep, self.results[l], ws[0], s.cuda_stream)
            return 2
        mm3fa.flash_attn_ext(qd, kd, vd, md, self.scale, 0.0, 0.0, dd, *ws, s.cuda_stream)
        if self.world > 1 and exchange:
            g = self.gathered[l]
            mm3fa.allgather_heads(g[self.rank].data_ptr(), g.data_ptr(), self.full[l].data_ptr(), D, N_HEAD, 1, self.B,
                                  1, self.comm, s.cuda_stream)
            return 2
        return 1

    def step(self, s, exchange: bool = True, layers=None) -> int:
        return sum(self.layer(l, s, exchange) for l in (range(self.L) if layers is None else layers))

    def capture(self, s, exchange: bool = True):
        torch = self.torch
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=s):
            self.step(s, exchange)
        return graph

    def layer_bytes(self) -> int:
        return layer_bytes(self.B, self.hkv, self.hq, self.kv)

    def close(self):
        if self.pb is not None:
            self.pb.close()


def timed_replays(torch, dist, graph, stream, steps: int, warmup: int, world: int, clk=None) -> float:
    """ms per replay of `graph`, device time (CUDA events on `stream`), max over ranks, with a
    barrier and a synchronize on both sides of the timed replays."""
    with torch.cuda.stream(stream):
        for _ in range(warmup):
            graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize()
    stream.record_event(e0)
    with torch.cuda.stream(stream):
        for _ in range(steps):
            graph.replay()
    stream.record_event(e1)
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    t = torch.tensor([e0.elapsed_time(e1)], device=stream.device)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item()) / steps


def bench_strong(torch, dist, mm3fa, ggml, dev, stream, steps: int, warmup: int, world: int, rank: int,
                 n_layers: int) -> dict:
    """Strong scaling of fixed decode jobs over the GPUs: the headline point (B=2, KV 8192) and
    config 2's large end (B=8, KV 16384), each a 36-layer step whose 8 kv heads are split over the
    ranks, with the fused per-layer head exchange (world > 1)."""
    g = torch.Generator(device=dev)
    g.manual_seed(77 + rank)
    peak, src = measured_peaks()
    out = {}
    for name, B, kv in (("b2_kv8192", 2, 8192), ("b8_kv16384", 8, 16384)):
        st = DecodeStack(torch, dist, mm3fa, ggml, dev, g, B, kv, n_layers, world, rank, "p2p")
        with torch.cuda.stream(stream):
            st.step(stream)
        torch.cuda.synchronize()
        graph = st.capture(stream)
        ms = timed_replays(torch, dist, graph, stream, steps, warmup, world)
        del graph
        job = layer_bytes(B, N_HEAD_KV, N_HEAD, kv) * n_layers
        out[name] = {"n_seq": B, "n_kv": kv, "us_per_layer": round(ms * 1e3 / n_layers, 3),
                     "GBps_job": round(job / (ms * 1e-3) / 1e9, 1),
                     "frac_of_n_gpus_x_peak": round(job / (ms * 1e-3) / 1e9 / (peak * world), 4),
                     "exchange": "fused peer stores + device wait per layer" if world > 1 else "none (1 GPU)"}
        torch.cuda.synchronize()
        st.close()
        del st
        torch.cuda.empty_cache()
    return {"strong": {"points": out, "peak_per_gpu": peak, "peak_source": src, "n_layers": n_layers,
                       "scaling": "strong (fixed job, kv heads split over the ranks)"}}


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
    ap.add_argument("--no-sweep", action="store_true", help="skip the config 2 sweep (batch x KV)")
    ap.add_argument("--no-strong", action="store_true", help="skip the strong-scaling lines")
    ap.add_argument("--no-depth", action="store_true", help="skip the depth-decoder attention line")
    ap.add_argument("--exchange", default="p2p", choices=["p2p", "nccl"],
                    help="per-layer head exchange of the headline at N > 1 (the other is timed beside it)")
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

    n_seq = 2 * world                 # N CFG pairs: weak scaling, 16 (sequence, kv head) pairs per GPU
    g = torch.Generator(device=dev)
    g.manual_seed(1234 + rank)
    stream = torch.cuda.Stream(device=dev)
    st = DecodeStack(torch, dist, mm3fa, ggml, dev, g, n_seq, N_KV, n_layers, world, rank, args.exchange, MAX_SEQ)
    hkv, hq = st.hkv, st.hq

    # capture the step once: the reference replays its decode graph the same way
    with torch.cuda.stream(stream):
        st.step(stream)  # first calls set kernel attributes outside capture
    torch.cuda.synchronize()
    graph = st.capture(stream)
    launches_per_step = n_layers * (2 if world > 1 else 1)
    graph_attn = st.capture(stream, exchange=False) if world > 1 else graph

    # ---- timed region (device time, CUDA events on the launching stream, max over ranks)
    with ClockSampler(local) as clk:
        ms_per_step = timed_replays(torch, dist, graph, stream, args.steps, args.warmup, world)
    clocks = clk.summary()
    per_rank_bytes = st.layer_bytes() * n_layers
    job_bytes = per_rank_bytes * world
    value = job_bytes / (ms_per_step * 1e-3) / 1e9

    # ---- roofline of the decode kernel: its average launch in the attention-only graph
    ms_attn = timed_replays(torch, dist, graph_attn, stream, args.steps, args.warmup, world)
    avg_launch_us = ms_attn * 1e3 / n_layers
    peak, peak_src = measured_peaks()
    achieved = st.layer_bytes() / (avg_launch_us * 1e-6) / 1e9
    xinfo = None
    if world > 1:
        # the other exchange form, timed the same way (same shapes, its own buffers)
        other = "nccl" if args.exchange == "p2p" else "p2p"
        g_o = torch.Generator(device=dev)
        g_o.manual_seed(4321 + rank)
        st_o = DecodeStack(torch, dist, mm3fa, ggml, dev, g_o, n_seq, N_KV, n_layers, world, rank, other, MAX_SEQ)
        with torch.cuda.stream(stream):
            st_o.step(stream)
        torch.cuda.synchronize()
        graph_o = st_o.capture(stream)
        ms_o = timed_replays(torch, dist, graph_o, stream, args.steps, args.warmup, world)
        del graph_o
        torch.cuda.synchronize()
        st_o.close()
        del st_o
        torch.cuda.empty_cache()
        us = {args.exchange: ms_per_step * 1e3 / n_layers, other: ms_o * 1e3 / n_layers}
        xinfo = {"per_layer": True, "mode": args.exchange,
                 "us_per_layer": {"attention_only": round(avg_launch_us, 3), "p2p": round(us["p2p"], 3),
                                  "nccl": round(us["nccl"], 3)},
                 "exchange_us_per_layer": {"p2p": round(us["p2p"] - avg_launch_us, 3),
                                           "nccl": round(us["nccl"] - avg_launch_us, 3)},
                 "p2p": "mm3fa_flash_attn_ext_peers (values stored as {value, epoch} words into every rank's "
                        "receive buffer over NVLink from the decode kernel's merge, no fences) + mm3fa_peer_wait "
                        "(device-side bounded wait and unpack) per layer",
                 "nccl": "mm3fa_flash_attn_ext + mm3fa_allgather_heads (ncclAllGather + permute) per layer"}

    # ---- end to end through the C ABI: Q/mask from pinned host memory, outputs back to host
    # One pinned buffer per direction (every layer's Q up, every layer's whole result down), moved
    # in chunks (E2E_UP, E2E_DOWN) on two copy streams so that the transfers overlap the attention
    # of other layers: an upload chunk's Q arrives before its first layer runs, a download chunk's
    # results go down while later layers compute.
    q_all, mask, full = st.q_all, st.mask, st.full
    q_host = q_all.cpu().pin_memory()
    mask_host = mask.cpu().pin_memory()
    out_host = torch.empty(full.shape, dtype=torch.float32).pin_memory()
    up_s, down_s = torch.cuda.Stream(device=dev), torch.cuda.Stream(device=dev)

    def spans(bounds):
        cuts = [0] + [b for b in bounds if 0 < b < n_layers] + [n_layers]
        return [(a, b) for a, b in zip(cuts[:-1], cuts[1:]) if b > a]

    ups, downs = spans(E2E_UP), spans(E2E_DOWN)
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        fork = torch.cuda.Event()
        stream.record_event(fork)
        up_s.wait_event(fork)
        down_s.wait_event(fork)
        uploaded = {}
        with torch.cuda.stream(up_s):
            mask.copy_(mask_host, non_blocking=True)
            for a, b in ups:
                q_all[a:b].copy_(q_host[a:b], non_blocking=True)
                ev = torch.cuda.Event()
                up_s.record_event(ev)
                uploaded[a] = ev
        down_end = {b: a for a, b in downs}
        for l in range(n_layers):
            if l in uploaded:
                stream.wait_event(uploaded[l])
            st.step(stream, layers=[l])
            if l + 1 in down_end:
                a = down_end[l + 1]
                done = torch.cuda.Event()
                stream.record_event(done)
                down_s.wait_event(done)
                with torch.cuda.stream(down_s):
                    out_host[a:l + 1].copy_(full[a:l + 1], non_blocking=True)
        joined = torch.cuda.Event()
        down_s.record_event(joined)
        stream.wait_event(joined)
    h2d = (q_host.numel() * 4 + mask_host.numel() * 2) * world
    d2h = out_host.numel() * 4 * world
    for _ in range(args.warmup):
        with torch.cuda.stream(stream):
            g2.replay()
        stream.synchronize()
    if world > 1:
        dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        stream.record_event(f0)
        for _ in range(args.steps):
            g2.replay()
            stream.synchronize()  # the step's result is read on the host every step
        stream.record_event(f1)
    torch.cuda.synchronize()
    te = torch.tensor([f0.elapsed_time(f1)], device=dev)
    if world > 1:
        dist.all_reduce(te, op=dist.ReduceOp.MAX)
    e2e_value = job_bytes * args.steps / (float(te.item()) * 1e-3) / 1e9
    del g2
    if graph_attn is not graph:
        del graph_attn

    dense = None if args.no_dense else bench_dense(torch, dist, mm3fa, ggml, dev, stream, args.steps, args.warmup,
                                                   world, rank, local)
    if dense is not None and world > 1:
        dist.barrier()
    q8 = None if args.no_q8 else bench_q8(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup, world, n_layers)
    if q8 is not None and world > 1:
        dist.barrier()
    dstep = None if args.no_step else bench_decode_step(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup, world,
                                                        n_layers)
    if dstep is not None and world > 1:
        dist.barrier()

    depth = None if args.no_depth else bench_depth(torch, mm3fa, ggml, dev, stream, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
    sweep = None if args.no_sweep else bench_sweep(torch, dist, mm3fa, ggml, dev, stream, args.steps, args.warmup,
                                                   world, rank, n_layers)
    if sweep is not None and world > 1:
        dist.barrier()
    strong = None if args.no_strong else bench_strong(torch, dist, mm3fa, ggml, dev, stream, args.steps,
                                                      args.warmup, world, rank, n_layers)

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
                       "exchange": (f"per layer ({args.exchange})" if world > 1 else "none (1 GPU)"),
                       "l2": "inputs > L2 (36 x 84 MB caches)",
                       "us_per_layer": round(ms_per_step * 1e3 / n_layers, 3),
                       "bytes_per_layer_per_gpu": st.layer_bytes()},
            "e2e": {"value": round(e2e_value, 2), "unit": "GB/s", "h2d_bytes_per_step": h2d,
                    "d2h_bytes_per_step": d2h},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                         "frac": round(achieved / peak, 4), "peak_source": peak_src,
                         "traffic": NCU_TRAFFIC_BYTES, "traffic_source": NCU_TRAFFIC_SOURCE, "kernel": NCU_KERNEL,
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
        if sweep is not None:
            line.update(sweep)
        if strong is not None:
            line.update(strong)
        if depth is not None:
            line.update(depth)
        if xinfo is not None:
            line["exchange"] = xinfo
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)

    del graph
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    st.close()
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
