"""Host side of the multi-GPU head exchange (one process per GPU, torch.distributed for the
plumbing).

Two forms, both behind the C ABI (include/mm3fa.h):

* NCCL: `nccl_comm` returns the ncclComm_t of torch's process group, which
  mm3fa_allgather_heads takes; the library calls ncclAllGather on it and permutes the
  rank-major gather into the ggml result.
* Peer memory: `PeerBuffers` gives every rank one zero-filled receive buffer (one slot per
  exchange site, e.g. per layer), exports it with CUDA IPC (mm3fa_ipc_export), swaps the handles
  with the other ranks and maps theirs (mm3fa_ipc_open).  mm3fa_flash_attn_ext_peers then
  stores each rank's result values as {value, epoch} words into the other ranks' receive
  buffers from inside the attention kernel (no fences: a matching epoch validates its value),
  and mm3fa_peer_wait is the consumer's kernel: it waits for the words of the current epoch and
  unpacks them into the local result.
* Dense form: `GatherBuffers` gives every rank n_slots whole-result buffers and a flag array, both
  mapped by the other ranks.  mm3fa_flash_attn_ext_gather stores each finished result row of the
  prefill/DiT kernel into every rank's whole result of the slot, and mm3fa_gather_signal_wait
  publishes the rows and waits for the other ranks' (epoch flags, system-scope release/acquire).

The reference runs on one device (src/backend.h:123); this is the exchange step of the
head-sharded layout the o_proj consumes (src/qwen3-lm.h:823-827).
"""
from __future__ import annotations

import mm3fa


def nccl_comm(dist, device) -> int:
    """ncclComm_t (as an int) of torch.distributed's default NCCL process group on `device`."""
    pg = dist.distributed_c10d._get_default_group()
    return int(pg._get_backend(device)._comm_ptr())


def _round_up(x: int, a: int) -> int:
    return (x + a - 1) // a * a


class PeerBuffers:
    """Receive buffers of the fused exchange: n_slots slots per rank, each holding two parity halves
    of `world` source regions of 8 * slice_values bytes ({value, epoch} words), in one zero-filled
    allocation per rank that every other rank maps; plus this rank's epoch counters (one u32 per
    slot, zero).  Collective: every rank constructs it at the same point, with the same arguments."""

    def __init__(self, torch, dist, device, slice_values: int, n_slots: int):
        self.torch = torch
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        if not 2 <= self.world <= mm3fa.MAX_RANKS:
            raise ValueError(f"peer exchange spans 2..{mm3fa.MAX_RANKS} ranks, not {self.world}")
        self.n_slots = n_slots
        self.slot_bytes = _round_up(2 * self.world * 8 * slice_values, 256)
        self.recv = torch.zeros(self.slot_bytes * n_slots, dtype=torch.uint8, device=device)
        self.epochs = torch.zeros(n_slots, dtype=torch.int32, device=device)
        handle = mm3fa.ipc_export(self.recv.data_ptr())
        handles = [None] * self.world
        dist.all_gather_object(handles, handle)
        self.bases = []
        for r in range(self.world):
            self.bases.append(self.recv.data_ptr() if r == self.rank else mm3fa.ipc_open(handles[r]))
        # every rank's zeroed buffer is in place before any rank's kernel writes into it
        torch.cuda.synchronize(device)
        dist.barrier()
        self.peers = mm3fa.Peers()
        self.peers.n_ranks, self.peers.rank = self.world, self.rank
        for r in range(self.world):
            self.peers.recv[r] = self.bases[r]
        self.peers.recv_slot_bytes = self.slot_bytes

    def close(self):
        """Unmaps the other ranks' buffers (collective: call on every rank, after all use)."""
        for r, b in enumerate(self.bases):
            if r != self.rank:
                mm3fa.ipc_close(b)
        self.bases = []


class _Mapped:
    """One device buffer per rank, every rank mapping all of them (collective)."""

    def __init__(self, torch, dist, buf):
        self.world, self.rank = dist.get_world_size(), dist.get_rank()
        self.buf = buf
        handles = [None] * self.world
        dist.all_gather_object(handles, mm3fa.ipc_export(buf.data_ptr()))
        self.bases = [buf.data_ptr() if r == self.rank else mm3fa.ipc_open(handles[r]) for r in range(self.world)]

    def peers(self, offset: int, nbytes: int):
        pr = mm3fa.Peers()
        pr.n_ranks, pr.rank = self.world, self.rank
        for r in range(self.world):
            pr.recv[r] = self.bases[r] + offset
        pr.recv_slot_bytes = nbytes
        return pr

    def close(self):
        for r, b in enumerate(self.bases):
            if r != self.rank:
                mm3fa.ipc_close(b)
        self.bases = []


class GatherBuffers:
    """Whole-result buffers of the fused dense exchange: n_slots F32 results of `result_bytes` per
    rank, a zero-filled flag array [n_slots][world] and this rank's epoch counters (zero).
    `results(slot)` is the mm3fa_peers for mm3fa_flash_attn_ext_gather, `flags` the one for
    mm3fa_gather_signal_wait, `result(slot)` this rank's own buffer of the slot (uint8 view).
    Collective: every rank constructs it at the same point with the same arguments."""

    def __init__(self, torch, dist, device, result_bytes: int, n_slots: int = 2):
        self.world = dist.get_world_size()
        if not 2 <= self.world <= mm3fa.MAX_RANKS:
            raise ValueError(f"the exchange spans 2..{mm3fa.MAX_RANKS} ranks, not {self.world}")
        self.n_slots = n_slots
        self.slot_bytes = _round_up(result_bytes, 256)
        self._res = _Mapped(torch, dist, torch.zeros(self.slot_bytes * n_slots, dtype=torch.uint8, device=device))
        self._flg = _Mapped(torch, dist, torch.zeros(_round_up(4 * n_slots * self.world, 256), dtype=torch.uint8,
                                                     device=device))
        self.epochs = torch.zeros(n_slots, dtype=torch.int32, device=device)
        self.flags = self._flg.peers(0, 4 * n_slots * self.world)
        # every rank's zeroed buffers are in place before any rank's kernel writes into them
        torch.cuda.synchronize(device)
        dist.barrier()

    def results(self, slot: int):
        return self._res.peers(slot * self.slot_bytes, self.slot_bytes)

    def result(self, slot: int):
        return self._res.buf[slot * self.slot_bytes:(slot + 1) * self.slot_bytes]

    def result_ptr(self, slot: int) -> int:
        return self._res.buf.data_ptr() + slot * self.slot_bytes

    def close(self):
        """Unmaps the other ranks' buffers (collective: call on every rank, after all use)."""
        self._res.close()
        self._flg.close()
