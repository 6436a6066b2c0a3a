"""Host logic of the KV-head-sharded multi-GPU path, run as world_size-2 gloo ranks on CPU.

Each rank computes its head slice of a CFG decode call with the CPU oracle (standing in for
its GPU), the slices are all-gathered over gloo exactly as bench.py gathers them over NCCL, and
the numpy statement of mm3fa_assemble_heads must rebuild the unsharded ggml result.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mm3fa import ggml, sharding


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank_main(rank, world, port, n_seq, n_q, result_path):
    import sys

    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    for p in (os.path.join(root, "minimaxmusic.cpp_b200"), os.path.join(root, "oracle")):
        sys.path.insert(0, p)
    import oracle
    from mm3fa import ggml as g, sharding as sh, workloads

    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    c = workloads.decode_case(n_seq=n_seq, n_kv=200, n_q=n_q, seed=77, kv_len=[150 + 20 * s for s in range(n_seq)])
    q, k, v, m = sh.shard_operands(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), rank,
                                   world)
    local = oracle.flash_attn_ext(q, k, v, m, c.scale, mode=oracle.MODE_EXACT, threads=1)  # (S, n_q, H/G, D)
    t = torch.from_numpy(np.ascontiguousarray(local))
    gathered = torch.empty((world,) + tuple(t.shape))
    dist.all_gather_into_tensor(gathered.view(-1), t.view(-1))  # flat, as bench.py gathers over NCCL
    full = sh.assemble_heads_np(gathered.numpy(), world)
    if rank == 0:
        ref = oracle.flash_attn_ext(c.q.host_desc(), c.k.host_desc(), c.v.host_desc(), c.mask.host_desc(), c.scale,
                                    mode=oracle.MODE_EXACT, threads=1)
        np.save(result_path, np.stack([full, ref]))
    dist.barrier()
    dist.destroy_process_group()
    del g


@pytest.mark.parametrize("n_seq,n_q", [(2, 1), (4, 3)])
def test_head_sharded_decode_matches_unsharded(tmp_path, n_seq, n_q):
    world = 2
    out = str(tmp_path / "res.npy")
    mp.start_processes(_rank_main, args=(world, _free_port(), n_seq, n_q, out), nprocs=world, join=True,
                       start_method="spawn")
    full, ref = np.load(out)
    assert np.array_equal(full, ref)  # each head row is computed by the same code either way


def test_head_slice_ranges():
    assert sharding.head_slice(32, 8, 0, 1) == (0, 32, 0, 8)
    assert sharding.head_slice(32, 8, 3, 4) == (24, 32, 6, 8)
    with pytest.raises(ValueError):
        sharding.head_slice(32, 8, 0, 3)


def test_shard_views_offsets():
    q = ggml.make(ggml.GGML_TYPE_F32, [128, 1, 32, 2], 0x10000)
    k = ggml.make(ggml.GGML_TYPE_F16, [128, 512, 8, 2], 0x20000, [2, 256, 256 * 1024, 256 * 1024 * 8])
    qs, ks, vs, _ = sharding.shard_operands(q, k, k, None, 1, 4)
    assert list(qs.ne) == [128, 1, 8, 2] and qs.data == 0x10000 + 8 * q.nb[2]
    assert list(ks.ne) == [128, 512, 2, 2] and ks.data == 0x20000 + 2 * k.nb[2]
    with pytest.raises(ValueError):
        sharding.shard_operands(q, k, k, None, 0, 2, max_bias=8.0)


def test_assemble_heads_np_layout():
    G, S, nq, H, D = 2, 3, 2, 8, 4
    x = np.arange(G * S * nq * (H // G) * D, dtype=np.float32).reshape(G, S, nq, H // G, D)
    full = sharding.assemble_heads_np(x, G)
    for r in range(G):
        np.testing.assert_array_equal(full[:, :, r * (H // G):(r + 1) * (H // G)], x[r])


@pytest.mark.parametrize("world,n_seq,n_head", [(2, 2, 16), (4, 2, 16), (8, 2, 16), (4, 8, 32), (8, 4, 32)])
def test_unit_slices_and_gather_permute_rebuild_the_result(world, n_seq, n_head):
    """(batch x head) sharding: the ranks' slices, gathered in rank order and permuted as
    mm3fa_allgather_heads does, are exactly the unsharded result."""
    rng = np.random.default_rng(world * 100 + n_seq)
    n_q, dv = 3, 4
    full = rng.standard_normal((n_seq, n_q, n_head, dv)).astype(np.float32)
    slices, ss = [], None
    for r in range(world):
        s0, s1, h0, h1, ss = sharding.unit_slice(n_seq, n_head, r, world)
        slices.append(full[s0:s1, :, h0:h1])
    got = sharding.allgather_scatter_np(np.stack(slices), ss)
    assert np.array_equal(got, full)
    if ss == 1:  # KV-head sharding is the special case seq_split = 1
        assert np.array_equal(got, sharding.assemble_heads_np(np.stack(slices), world))


def test_unit_slice_rejects_uneven_splits():
    with pytest.raises(ValueError):
        sharding.unit_slice(2, 15, 0, 4)
    with pytest.raises(ValueError):
        sharding.unit_slice(3, 16, 0, 2)
