"""ModelRunner.kv_connector_step for one tensor-parallel rank (lean_vllm/engine/model_runner.py:637-649), with the
per-step exchange of connector outputs through host shared memory instead of a gloo gather_object.

Every rank starts its step's loads and takes its finished transfers; rank 0 then needs every rank's output to tell
which requests are done on all ranks (KVOutputAggregator, kv_transfer/base.py:125-165). The reference gathers the
pickled outputs over gloo every step: a collective round trip per step, even when nothing finished anywhere. Here
each rank posts its output into its slot of a StepMailbox -- a file in /dev/shm that every rank of the instance
maps, whose ordering words are atomics of libkvx (kvx_mailbox_*) -- and rank 0 reads the slots in place. A rank with
nothing to report posts an empty slot, so a quiet step costs rank 0 one atomic load per rank: no pickling, no socket.
`exchange="gather"` keeps the reference's gather_object.
"""

from __future__ import annotations

import ctypes
import mmap
import os
import pickle
import tempfile
import uuid

from lean_vllm_b200._native import check, lib
from lean_vllm_b200.kv_transfer.base import KVConnectorOutput, KVOutputAggregator, KVTransferStats

SLOT_BYTES = 4 << 20  # one rank's output of one step: ~100k request ids
STEP_TIMEOUT = 300.0  # seconds rank 0 waits for a rank's step (and a rank for rank 0's read) before raising


def encode(output: KVConnectorOutput) -> bytes:
    """A rank's output as mailbox bytes; empty when it finished nothing."""
    if not output:
        return b""
    stats = {rid: (s.seconds, s.num_bytes) for rid, s in output.recv_stats.items()}
    return pickle.dumps((list(output.finished_sending), list(output.finished_recving), list(output.failed_recving),
                         list(output.expired_sending), stats), protocol=pickle.HIGHEST_PROTOCOL)


def decode(data: bytes) -> KVConnectorOutput:
    if not data:
        return KVConnectorOutput()
    sending, recving, failed, expired, stats = pickle.loads(data)
    return KVConnectorOutput(set(sending), set(recving), set(failed), set(expired),
                             {rid: KVTransferStats(s, b) for rid, (s, b) in stats.items()})


class StepMailbox:
    """One instance's mailbox as this rank maps it (layout and ordering: include/kvx.h, kvx_mailbox_*)."""

    def __init__(self, path: str, world: int, rank: int, slot_bytes: int = SLOT_BYTES, create: bool = False):
        self.path, self.world, self.rank, self.slot_bytes = path, world, rank, slot_bytes
        self.size = int(lib().kvx_mailbox_bytes(world, slot_bytes))
        self.stride = int(lib().kvx_mailbox_stride(slot_bytes))
        if create:
            fd = os.open(path, os.O_RDWR | os.O_CREAT | os.O_EXCL, 0o600)
            os.ftruncate(fd, self.size)  # zero-filled: every sequence word starts at 0
        else:
            fd = os.open(path, os.O_RDWR)
        try:
            self._map = mmap.mmap(fd, self.size)
        finally:
            os.close(fd)
        self._view = (ctypes.c_char * self.size).from_buffer(self._map)
        self.addr = ctypes.addressof(self._view)
        self._lens = (ctypes.c_uint64 * world)()

    def post(self, seq: int, payload: bytes, timeout: float = STEP_TIMEOUT):
        """Rank >= 1: step `seq`'s payload, once rank 0 has read step seq - 1."""
        check(lib().kvx_mailbox_post(self.addr, self.world, self.rank, self.slot_bytes, seq, payload or None,
                                     len(payload), timeout))

    def collect(self, seq: int, timeout: float = STEP_TIMEOUT) -> list[bytes]:
        """Rank 0: every other rank's payload of step `seq` (index 0 is this rank's, always empty)."""
        check(lib().kvx_mailbox_collect(self.addr, self.world, self.slot_bytes, seq, self._lens, timeout))
        out = [b""]
        for rank in range(1, self.world):
            n = self._lens[rank]
            at = 64 + rank * self.stride + 16
            out.append(self._map[at : at + n] if n else b"")
        return out

    def release(self, seq: int):
        check(lib().kvx_mailbox_release(self.addr, seq))

    def close(self):
        if self._map is not None:
            del self._view
            self._map.close()
            self._map = None


class KVConnectorStep:
    """kv_connector_step bound to one rank's connector worker half: call it with each step's metadata. Rank 0 gets
    the output aggregated over all ranks; other ranks get None (model_runner.py:637-649).

    `group` is the instance's host process group (the reference's call_group); the mailbox uses it once, to agree on
    the shared file. Ranks must share a node (the CUDA IPC connector requires it anyway)."""

    def __init__(self, connector, rank: int, world_size: int, group=None, exchange: str = "mailbox",
                 slot_bytes: int = SLOT_BYTES, timeout: float = STEP_TIMEOUT):
        if exchange not in ("mailbox", "gather"):
            raise ValueError(f"exchange is 'mailbox' or 'gather', not {exchange!r}")
        self.connector, self.rank, self.world_size, self.group = connector, rank, world_size, group
        self.exchange, self.timeout = exchange, timeout
        self.aggregator = KVOutputAggregator(world_size) if rank == 0 else None
        self.mailbox: StepMailbox | None = None
        self.seq = 0
        if world_size > 1 and exchange == "mailbox":
            import torch.distributed as dist

            # Host shared memory where the node has it (/dev/shm), else the temporary directory.
            folder = "/dev/shm" if os.path.isdir("/dev/shm") else tempfile.gettempdir()
            path = [os.path.join(folder, f"kvx-step-{os.getpid()}-{uuid.uuid4().hex[:12]}") if rank == 0 else None]
            if rank == 0:
                self.mailbox = StepMailbox(path[0], world_size, rank, slot_bytes, create=True)
            dist.broadcast_object_list(path, src=0, group=group)
            if rank != 0:
                self.mailbox = StepMailbox(path[0], world_size, rank, slot_bytes)
            dist.barrier(group=group)
            if rank == 0:
                os.unlink(path[0])  # every rank holds its mapping: nothing is left behind if a process dies

    def __call__(self, metadata) -> KVConnectorOutput | None:
        self.connector.start_load_kv(metadata)
        output = self.connector.get_finished()
        if self.world_size == 1:
            return output
        if self.exchange == "gather":
            import torch.distributed as dist

            outputs = [None] * self.world_size if self.rank == 0 else None
            dist.gather_object(output, outputs, dst=0, group=self.group)
            return self.aggregator.aggregate(outputs) if outputs is not None else None
        self.seq += 1
        if self.rank != 0:
            self.mailbox.post(self.seq, encode(output), self.timeout)
            return None
        payloads = self.mailbox.collect(self.seq, self.timeout)
        outputs = [output] + [decode(p) for p in payloads[1:]]
        self.mailbox.release(self.seq)
        if not any(outputs):
            return KVConnectorOutput()  # what aggregating empty outputs gives, without the walk
        return self.aggregator.aggregate(outputs)

    def close(self):
        if self.mailbox is not None:
            self.mailbox.close()
            self.mailbox = None


__all__ = ["KVConnectorStep", "StepMailbox", "encode", "decode", "SLOT_BYTES", "STEP_TIMEOUT"]
