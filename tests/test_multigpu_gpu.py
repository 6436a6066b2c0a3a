"""The multi-GPU head exchange on 2 (or more) GPUs, one process per GPU over NCCL.

Each rank computes its shard of a CFG decode call (kv heads [8r/G, 8(r+1)/G)) and of a DiT call
((batch x head) units), and the slices are exchanged through the C ABI:
  * mm3fa_allgather_heads (NCCL all-gather of torch's communicator + the permute);
  * mm3fa_flash_attn_ext_peers + mm3fa_peer_wait (the decode kernel stores its values as
    {value, epoch} words into every other rank's receive buffer over NVLink, the consumer's
    kernel waits for them and unpacks them), over several slots and both epoch parities.
  * mm3fa_flash_attn_ext_gather + mm3fa_gather_signal_wait (DiT and causal prefill shards: the
    dense kernel's epilogue stores each result row into every rank's whole result, a signal
    kernel publishes them), over both result slots.
The exchanged result must equal, bit for bit, the slices computed one by one on rank 0's GPU
with the plain entry point (the exchange is a copy), and match the oracle at the north-star
bound.  Runs on MM3FA_TEST_GPUS ranks (2 by default; 4 and 8 split the heads further); skipped on
a box with fewer GPUs.
"""
import os
import socket

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

WORLD = int(os.environ.get("MM3FA_TEST_GPUS", "2"))


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _descs(torch, ggml, c, dev, keep):
    d = {}
    for n in ("q", "k", "v", "mask"):
        op = getattr(c, n)
        if op is None:
            d[n] = None
            continue
        t = torch.from_numpy(np.ascontiguousarray(op.storage)).to(dev)
        keep.append(t)
        d[n] = op.device_desc(t)
    return d


def _rank_main(rank, world, port, out_dir):
    import datetime
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "minimaxmusic.cpp_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import torch.distributed as dist

    import mm3fa
    from mm3fa import exchange, ggml, sharding, workloads

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    dev = torch.device("cuda", rank)
    torch.cuda.set_device(dev)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=dev)
    s = torch.cuda.current_stream(dev)
    comm = exchange.nccl_comm(dist, dev)
    keep = []
    F32 = ggml.GGML_TYPE_F32

    # ---------------- CFG decode, kv-head sharding (seq_split = 1)
    c = workloads.decode_case(n_seq=4, n_kv=2048, max_seq=2304, seed=900)  # the same operands on every rank
    d = _descs(torch, ggml, c, dev, keep)
    H, D, n_seq = c.q.ne[2], c.q.ne[0], c.q.ne[3]
    hl = H // world
    qs, ks, vs, ms = sharding.shard_operands(d["q"], d["k"], d["v"], d["mask"], rank, world)
    ws = mm3fa.Workspace(dev)
    # NCCL form: the slice is computed in place at its rank's position of the gather buffer
    gathered = torch.full((world, n_seq, 1, hl, D), float("nan"), device=dev)
    full_nccl = torch.full((n_seq, 1, H, D), float("nan"), device=dev)
    mm3fa.run(qs, ks, vs, ms, mm3fa.dst_desc(qs, vs, gathered[rank].data_ptr()), c.scale, ws=ws)
    mm3fa.allgather_heads(gathered[rank].data_ptr(), gathered.data_ptr(), full_nccl.data_ptr(), D, H, 1, n_seq, 1, comm,
                          s.cuda_stream)
    # fused form: 3 slots, then slots 0 and 1 again (both epoch parities of a slot), each call into
    # a NaN-filled result so that every value the exchange misses would show
    pb = exchange.PeerBuffers(torch, dist, dev, n_seq * hl * D, 3)
    wsz = mm3fa.workspace_size(qs, ks, vs, ms, mm3fa.dst_desc(qs, vs, 0))
    wsb = torch.zeros(max(wsz, 4096), dtype=torch.uint8, device=dev)
    peer_out = []
    for slot in (0, 1, 2, 0, 1):
        res = torch.full((n_seq, 1, H, D), float("nan"), device=dev)
        view = ggml.make(F32, [D, hl, 1, n_seq], res.data_ptr() + rank * hl * D * 4, [4, 4 * D, 4 * D * H, 4 * D * H])
        mm3fa.flash_attn_ext_peers(qs, ks, vs, ms, c.scale, 0.0, 0.0, view, wsb.data_ptr(), wsb.numel(),
                                   pb.peers, slot, pb.epochs.data_ptr(), s.cuda_stream)
        mm3fa.peer_wait(pb.peers, slot, pb.epochs.data_ptr(), ggml.make(F32, [D, H, 1, n_seq], res.data_ptr()),
                        wsb.data_ptr(), s.cuda_stream)
        peer_out.append(res)
    torch.cuda.synchronize(dev)
    st, raw = mm3fa.workspace_status(wsb.data_ptr(), s.cuda_stream)
    out = {"decode_nccl": full_nccl.cpu().numpy(), "decode_peer": np.stack([p.cpu().numpy() for p in peer_out]),
           "decode_status": np.array([st, raw])}
    if rank == 0:
        # every shard alone on this GPU with the plain entry point, assembled on the host
        parts = []
        for r in range(world):
            q_, k_, v_, m_ = sharding.shard_operands(d["q"], d["k"], d["v"], d["mask"], r, world)
            o = torch.full((n_seq, 1, hl, D), float("nan"), device=dev)
            mm3fa.run(q_, k_, v_, m_, mm3fa.dst_desc(q_, v_, o.data_ptr()), c.scale, ws=ws)
            parts.append(o.cpu().numpy())
        out["decode_ref"] = sharding.assemble_heads_np(np.stack(parts), world)

    # ---------------- DiT, (batch x head) sharding through mm3fa_allgather_heads
    cd = workloads.dit_case(B=2, S=300, H=8, D=64, seed=901)
    dd = _descs(torch, ggml, cd, dev, keep)
    B, S, Hd, Dd = 2, 300, 8, 64

    def shard(r):
        s0, s1, h0, h1, ss = sharding.unit_slice(B, Hd, r, world)
        q, k, v = dd["q"], dd["k"], dd["v"]
        qv = ggml.make(q.type, [Dd, S, h1 - h0, s1 - s0], q.data + h0 * q.nb[2] + s0 * q.nb[3], list(q.nb))
        kv = ggml.make(k.type, [Dd, S, h1 - h0, s1 - s0], k.data + h0 * k.nb[2] + s0 * k.nb[3], list(k.nb))
        vv = ggml.make(v.type, [Dd, S, h1 - h0, s1 - s0], v.data + h0 * v.nb[2] + s0 * v.nb[3], list(v.nb))
        return qv, kv, vv, (s1 - s0, h1 - h0, ss)

    qv, kv, vv, (sl, hd, ss) = shard(rank)
    g2 = torch.full((world, sl, S, hd, Dd), float("nan"), device=dev)
    full_dit = torch.full((B, S, Hd, Dd), float("nan"), device=dev)
    mm3fa.run(qv, kv, vv, None, mm3fa.dst_desc(qv, vv, g2[rank].data_ptr()), cd.scale, ws=ws)
    mm3fa.allgather_heads(g2[rank].data_ptr(), g2.data_ptr(), full_dit.data_ptr(), Dd, Hd, S, B, ss, comm,
                          s.cuda_stream)
    torch.cuda.synchronize(dev)
    out["dit_nccl"] = full_dit.cpu().numpy()
    if rank == 0:
        parts = []
        for r in range(world):
            q_, k_, v_, (sl_, hd_, ss_) = shard(r)
            o = torch.full((sl_, S, hd_, Dd), float("nan"), device=dev)
            mm3fa.run(q_, k_, v_, None, mm3fa.dst_desc(q_, v_, o.data_ptr()), cd.scale, ws=ws)
            parts.append(o.cpu().numpy())
        out["dit_ref"] = sharding.allgather_scatter_np(np.stack(parts), ss)
    # DiT through the fused dense exchange: the slice goes into every rank's whole result from the
    # kernel's epilogue; calls on slots 0, 1, 0, each into a NaN-filled result
    gb = exchange.GatherBuffers(torch, dist, dev, B * S * Hd * Dd * 4, 2)
    wsd = torch.zeros(1 << 20, dtype=torch.uint8, device=dev)
    s0, s1, h0, h1, _ = sharding.unit_slice(B, Hd, rank, world)

    def fused(case_q, case_k, case_v, case_m, scale, nbytes, view_of):
        res = []
        for slot in (0, 1, 0):
            gb.result(slot)[:nbytes].view(torch.float32).fill_(float("nan"))
            torch.cuda.synchronize(dev)
            dist.barrier()
            dv = view_of(gb.result_ptr(slot))
            mm3fa.flash_attn_ext_gather(case_q, case_k, case_v, case_m, scale, dv, wsd.data_ptr(), wsd.numel(),
                                        gb.results(slot), s.cuda_stream)
            mm3fa.gather_signal_wait(gb.flags, slot, gb.epochs.data_ptr(), wsd.data_ptr(), s.cuda_stream)
            torch.cuda.synchronize(dev)
            res.append(gb.result(slot)[:nbytes].view(torch.float32).cpu().numpy().copy())
        return np.stack(res)

    out["dit_fused"] = fused(qv, kv, vv, None, cd.scale, B * S * Hd * Dd * 4,
                             lambda base: ggml.make(F32, [Dd, h1 - h0, S, s1 - s0], base + (s0 * S * Hd + h0) * Dd * 4,
                                                    [4, 4 * Dd, 4 * Dd * Hd, 4 * Dd * Hd * S]))
    # causal prefill (32q / 8kv, head pairs) by kv-head shard, fused and through NCCL
    cp = workloads.prefill_case(n_seq=2, S=300, n_head=32, n_head_kv=8, kv_pos=20, seed=902)
    dp = _descs(torch, ggml, cp, dev, keep)
    Dp, Sp, Hp, nsp = 128, 300, 32, 2
    hlp = Hp // world
    pq, pk, pv, pm = sharding.shard_operands(dp["q"], dp["k"], dp["v"], dp["mask"], rank, world)
    pbytes = nsp * Sp * Hp * Dp * 4
    gb2 = gb if pbytes <= gb.slot_bytes else exchange.GatherBuffers(torch, dist, dev, pbytes, 2)
    gb_saved, gb = gb, gb2
    out["prefill_fused"] = fused(pq, pk, pv, pm, cp.scale, pbytes,
                                 lambda base: ggml.make(F32, [Dp, hlp, Sp, nsp], base + rank * hlp * Dp * 4,
                                                        [4, 4 * Dp, 4 * Dp * Hp, 4 * Dp * Hp * Sp]))
    gp = torch.full((world, nsp, Sp, hlp, Dp), float("nan"), device=dev)
    fullp = torch.full((nsp, Sp, Hp, Dp), float("nan"), device=dev)
    mm3fa.run(pq, pk, pv, pm, ggml.make(F32, [Dp, hlp, Sp, nsp], gp[rank].data_ptr()), cp.scale, ws=ws)
    mm3fa.allgather_heads(gp[rank].data_ptr(), gp.data_ptr(), fullp.data_ptr(), Dp, Hp, Sp, nsp, 1, comm, s.cuda_stream)
    torch.cuda.synchronize(dev)
    out["prefill_nccl"] = fullp.cpu().numpy()
    st2, raw2 = mm3fa.workspace_status(wsd.data_ptr(), s.cuda_stream)
    out["fused_status"] = np.array([st2, raw2])
    np.savez(os.path.join(out_dir, f"rank{rank}.npz"), **out)
    torch.cuda.synchronize(dev)
    dist.barrier()
    gb = gb_saved
    if gb2 is not gb:
        gb2.close()
    gb.close()
    torch.cuda.synchronize(dev)
    dist.barrier()
    pb.close()
    dist.barrier()
    dist.destroy_process_group()


@pytest.fixture(scope="module")
def exchange_results(tmp_path_factory):
    if torch.cuda.device_count() < WORLD:
        pytest.skip(f"needs {WORLD} GPUs")
    import torch.multiprocessing as mp

    out = str(tmp_path_factory.mktemp("exchange"))
    mp.start_processes(_rank_main, args=(WORLD, _free_port(), out), nprocs=WORLD, join=True, start_method="spawn")
    return [dict(np.load(os.path.join(out, f"rank{r}.npz"))) for r in range(WORLD)]


def test_nccl_exchange_is_the_shards_bit_for_bit(exchange_results):
    ref = exchange_results[0]["decode_ref"]
    for r, res in enumerate(exchange_results):
        assert np.array_equal(res["decode_nccl"], ref), f"rank {r}: decode all-gather differs"
        assert np.array_equal(res["dit_nccl"], exchange_results[0]["dit_ref"]), f"rank {r}: DiT all-gather differs"


def test_fused_peer_exchange_is_the_shards_bit_for_bit(exchange_results):
    import mm3fa

    ref = exchange_results[0]["decode_ref"]
    for r, res in enumerate(exchange_results):
        assert tuple(res["decode_status"]) == (mm3fa.OK, 0), f"rank {r}: a peer wait expired"
        for k in range(res["decode_peer"].shape[0]):
            assert np.array_equal(res["decode_peer"][k], ref), f"rank {r}: peer exchange call {k} differs"


def test_fused_dense_exchange_is_the_all_gather_bit_for_bit(exchange_results):
    import mm3fa

    for r, res in enumerate(exchange_results):
        assert tuple(res["fused_status"]) == (mm3fa.OK, 0), f"rank {r}: a dense exchange wait expired"
        for k in range(3):
            ref = exchange_results[0]["dit_ref"].reshape(res["dit_fused"][k].shape)
            assert np.array_equal(res["dit_fused"][k], ref), f"rank {r}: fused DiT exchange call {k} differs"
            got = res["prefill_fused"][k].reshape(res["prefill_nccl"].shape)
            assert np.array_equal(got, res["prefill_nccl"]), f"rank {r}: fused prefill exchange call {k} differs"


def test_exchanged_results_match_the_oracle(exchange_results):
    from gpu_util import check_three_ways
    from mm3fa import workloads

    check_three_ways(exchange_results[0]["decode_nccl"], workloads.decode_case(n_seq=4, n_kv=2048, max_seq=2304,
                                                                               seed=900))
    check_three_ways(exchange_results[1]["dit_nccl"], workloads.dit_case(B=2, S=300, H=8, D=64, seed=901))
    check_three_ways(exchange_results[-1]["prefill_nccl"],
                     workloads.prefill_case(n_seq=2, S=300, n_head=32, n_head_kv=8, kv_pos=20, seed=902))
