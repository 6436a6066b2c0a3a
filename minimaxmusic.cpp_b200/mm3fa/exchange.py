"""Host side of the multi-GPU head exchange (one process per GPU, torch.distributed for the
plumbing).

Two forms, both behind the C ABI (include/mm3fa.h):

* NCCL: `nccl_comm` returns the ncclComm_t of torch's process group, which
  mm3fa_allgather_heads takes; the library calls ncclAllGather on it and permutes the
  rank-major gather into the ggml result.
* Peer memory: `PeerBuffers` gives every rank one device allocation holding its whole result
  buffers (one per slot, e.g. per layer) and its arrival counters, exports it with CUDA IPC
  (mm3fa_ipc_export), swaps the handles with the other ranks and maps theirs
  (mm3fa_ipc_open).  mm3fa_flash_attn_ext_peers then stores each rank's result rows into all
  the buffers from inside the attention kernel and mm3fa_peer_wait is the consumer's wait.

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
    """n_slots result buffers of slot_bytes each plus n_slots u32 arrival counters per rank, in one
    allocation, mapped into every rank's process.

    Collective: every rank constructs it at the same point, with the same arguments."""

    def __init__(self, torch, dist, device, slot_bytes: int, n_slots: int):
        self.torch = torch
        self.world = dist.get_world_size()
        self.rank = dist.get_rank()
        if not 2 <= self.world <= mm3fa.MAX_RANKS:
            raise ValueError(f"peer exchange spans 2..{mm3fa.MAX_RANKS} ranks, not {self.world}")
        self.n_slots = n_slots
        self.slot_bytes = _round_up(slot_bytes, 256)
        self.flags_off = self.slot_bytes * n_slots
        total = self.flags_off + _round_up(4 * n_slots, 256)
        # zero-filled: the counters start at 0 (the result area need not)
        self.buf = torch.zeros(total, dtype=torch.uint8, device=device)
        self.targets = torch.zeros(n_slots, dtype=torch.int32, device=device)
        handle = mm3fa.ipc_export(self.buf.data_ptr())
        handles = [None] * self.world
        dist.all_gather_object(handles, handle)
        self.bases = []
        for r in range(self.world):
            self.bases.append(self.buf.data_ptr() if r == self.rank else mm3fa.ipc_open(handles[r]))
        # every rank's zeroed counters are in place before any rank's kernel writes to them
        torch.cuda.synchronize(device)
        dist.barrier()
        self.peers = []
        for s in range(n_slots):
            p = mm3fa.Peers()
            p.n_ranks, p.rank = self.world, self.rank
            for r in range(self.world):
                p.dst[r] = self.bases[r] + s * self.slot_bytes
                p.flags[r] = self.bases[r] + self.flags_off
            self.peers.append(p)

    def result_ptr(self, slot: int) -> int:
        """This rank's whole result buffer of `slot`."""
        return self.buf.data_ptr() + slot * self.slot_bytes

    def result(self, slot: int, shape, dtype=None):
        """This rank's result buffer of `slot` as a torch tensor view (F32 by default)."""
        torch = self.torch
        dtype = dtype or torch.float32
        n = 1
        for d in shape:
            n *= d
        esz = torch.tensor([], dtype=dtype).element_size()
        off = slot * self.slot_bytes
        return self.buf[off:off + n * esz].view(dtype).view(*shape)

    def close(self):
        """Unmaps the other ranks' buffers (collective: call on every rank, after all use)."""
        for r, b in enumerate(self.bases):
            if r != self.rank:
                mm3fa.ipc_close(b)
        self.bases = []
