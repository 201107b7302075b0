"""A host-memory stand-in for the NIXL agent under the reference's NixlConnectorWorker. TEST INFRASTRUCTURE ONLY.

NIXL (nixl==1.3.1, the reference's pinned transport, pyproject.toml:47-49) is not installed and has no source here.
The reference's own CPU tests replace it with a fake agent whose READ is one memmove per descriptor row
(tests/test_nixl_connector.py:33-115); this class restates that contract so the reference's worker runs unmodified
over host memory:

* register_memory / get_reg_descs      -- the (address, length) spans a READ may touch;
* initialize_xfer("READ", local, remote, peer, notification) -- checks both sides' rows lie in registered spans;
* transfer                             -- copies each remote row onto its local row (ctypes.memmove);
* check_xfer_state                     -- "DONE", delivering the notification to the peer, as NIXL does once the
                                          data has landed;
* send_notif / get_new_notifs          -- notifications between agents of this process.

Used by tests/golden/make_golden.py (the fixtures) and by bench.py's reference arm (the timed CPU path), never by the
product.
"""

from __future__ import annotations

import ctypes
import threading
from collections import defaultdict
from itertools import count

import numpy as np


class MemmoveAgent:
    """The NIXL agent surface NixlConnectorWorker calls, over host memory in this process."""

    registry: dict[str, "MemmoveAgent"] = {}

    def __init__(self, name: str):
        self.name = name
        self.memory: list[tuple[int, int]] = []
        self.peers: set[str] = set()
        self.pending: dict[int, tuple] = {}
        self.inbox: dict[str, list[bytes]] = defaultdict(list)
        self.mutex = threading.Lock()
        self.ids = count()
        MemmoveAgent.registry[name] = self

    def get_reg_descs(self, memory, mem_type):
        return [(addr, size) for addr, size, _, _ in memory]

    def register_memory(self, descs):
        self.memory.extend(descs)

    def deregister_memory(self, descs):
        self.memory = [d for d in self.memory if d not in descs]

    def get_agent_metadata(self) -> bytes:
        return self.name.encode()

    def add_remote_agent(self, metadata: bytes) -> str:
        self.peers.add(metadata.decode())
        return metadata.decode()

    def remove_remote_agent(self, name: str):
        self.peers.discard(name)

    def get_xfer_descs(self, rows, mem_type):
        return np.asarray(rows)

    @staticmethod
    def _inside(agent: "MemmoveAgent", rows) -> bool:
        """Every (address, length) row lies within one registered span. Vectorised, so the check costs the
        stand-in milliseconds per step and the timing stays the reference worker's."""
        rows = np.asarray(rows, dtype=np.uint64).reshape(-1, 3)
        if not len(rows):
            return True
        spans = np.asarray(sorted(agent.memory), dtype=np.uint64).reshape(-1, 2)
        if not len(spans):
            return False
        at = np.searchsorted(spans[:, 0], rows[:, 0], side="right").astype(np.int64) - 1
        if (at < 0).any():
            return False
        return bool((rows[:, 0] + rows[:, 1] <= spans[at, 0] + spans[at, 1]).all())

    def initialize_xfer(self, op, local, remote, peer_name, notification):
        peer = MemmoveAgent.registry[peer_name]
        if op != "READ" or len(local) != len(remote) or not (self._inside(self, local) and self._inside(peer, remote)):
            raise RuntimeError("bad transfer")
        handle = next(self.ids)
        self.pending[handle] = (local, remote, peer, notification)
        return handle

    def transfer(self, handle) -> str:
        local, remote, _, _ = self.pending[handle]
        for (dst, n, _), (src, _, _) in zip(local.tolist(), remote.tolist()):
            ctypes.memmove(dst, src, n)
        return "PROC"

    def check_xfer_state(self, handle) -> str:
        _, _, peer, notification = self.pending[handle]
        peer.deliver(self.name, notification)
        return "DONE"

    def release_xfer_handle(self, handle):
        self.pending.pop(handle, None)

    def send_notif(self, peer_name: str, message: bytes):
        MemmoveAgent.registry[peer_name].deliver(self.name, message)

    def deliver(self, sender: str, message: bytes):
        with self.mutex:
            self.inbox[sender].append(message)

    def get_new_notifs(self):
        with self.mutex:
            out, self.inbox = dict(self.inbox), defaultdict(list)
        return out
